// Low-latency exchange words of the tensor-parallel decode (tp.cu, and the GEMV epilogue
// that all-reduces inside the o and down projections): a value's f32 bits paired with the
// exchange's 32-bit tag in one aligned 64-bit store. A 64-bit store is single-copy atomic,
// so a receiver polls the data itself and needs no flag or system-scope fence.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace y2 {

constexpr long long kTpSpinCycles = 2000000000ll;  // about a second of SM clocks

Y2_DEV void st_ll(uint2* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
Y2_DEV uint2 ld_ll(const uint2* p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}
// Waits (bounded) until the word carries `tag` or a later one; its value then. After a wait
// that gave up (ok false, *error set) later calls return at once.
Y2_DEV float wait_ll(const uint2* p, uint32_t tag, int32_t* error, bool& ok) {
  uint2 v = ld_ll(p);
  if (v.y >= tag || !ok) return __uint_as_float(v.x);
  const long long t0 = clock64();
  while ((v = ld_ll(p)).y < tag)
    if (clock64() - t0 > kTpSpinCycles) {
      atomicExch(error, 1);
      ok = false;
      break;
    }
  return __uint_as_float(v.x);
}

}  // namespace y2
