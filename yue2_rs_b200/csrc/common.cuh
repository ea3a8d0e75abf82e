// Shared device helpers for the sm_100a decode kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "detmath.h"

#define Y2_DEV __device__ __forceinline__

namespace y2 {

constexpr int kWarp = 32;

// ---- bf16 helpers (activations and weights are raw bf16 bit patterns)
Y2_DEV float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
Y2_DEV float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
Y2_DEV float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
// bits of a value that is already bf16-exact
Y2_DEV uint16_t f2bf_exact(float f) { return (uint16_t)(__float_as_uint(f) >> 16); }
Y2_DEV uint16_t f2bf_round(float f) { return f2bf_exact(round_bf16(f)); }

// 16-byte streaming load that bypasses L1 (weights are read exactly once per step)
Y2_DEV uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// coherent 16-byte load of data produced by an earlier kernel
Y2_DEV uint4 ldg16(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Programmatic dependent launch: weights may be fetched before the wait; anything
// produced by the preceding kernel only after it. Both are no-ops without PDL.
Y2_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
Y2_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Fire-and-forget bulk prefetch of [p, p+bytes) into L2 (p and bytes 16-byte aligned).
Y2_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Ampere-style 16-byte async copy global -> shared (completion through wait_group).
Y2_DEV void cp_async16(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
Y2_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
Y2_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// D += A(16x16, row) * B(16x8, col), bf16 in, f32 accumulate
Y2_DEV void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

Y2_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
Y2_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// dot of 8 bf16 weights with 8 bf16 activations, accumulated into acc
Y2_DEV float dot8_bf(uint4 w, uint4 x, float acc) {
  acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
  acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
  acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
  acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
  acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
  acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
  acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
  acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
  return acc;
}

}  // namespace y2
