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

// 16-byte async copy that writes zeros instead when !valid (no global read then).
Y2_DEV void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0) : "memory");
}

// Four 8x8 b16 matrices from shared memory; lane i gives the address of row i % 8 of
// matrix i / 8, and register j receives this lane's fragment of matrix j.
Y2_DEV void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
// The same with each matrix transposed.
Y2_DEV void ldsm_x4_trans(uint32_t (&r)[4], const void* smem) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// Two f32 to a bf16x2 word (round to nearest even; lo in the low half).
Y2_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
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

// ---- activation staging for the GEMVs. Weight copies queued ahead of these loads make
// every round trip to memory long, so all loads of a batch are issued before any is used.

// Rows [0, R) of a bf16 [R, K] matrix into shared memory rows of `pitch` bytes (K % 8 == 0).
// CG: load through L2 only (data written earlier in the same kernel by other SMs).
template <int NT, bool CG = false>
Y2_DEV void stage_bf16_rows(const uint16_t* xb, int K, int R, unsigned char* xs, size_t pitch) {
  constexpr int kB = 8;
  const int K8 = K >> 3, total = R * K8, tid = threadIdx.x;
  for (int base = 0; base < total; base += NT * kB) {
    uint4 v[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int i = base + b * NT + tid;
      if (i < total) v[b] = CG ? __ldcg(reinterpret_cast<const uint4*>(xb) + i) : ldg16(xb + (size_t)i * 8);
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int i = base + b * NT + tid;
      if (i < total) {
        const int r = i / K8, c = i - r * K8;
        *reinterpret_cast<uint4*>(xs + (size_t)r * pitch + c * 16) = v[b];
      }
    }
  }
}

// Norm::apply (src/tensor.rs:1140-1157) of rows [0, R) of the f32 residual [R, K] with gains
// gamma, as bf16 into shared memory rows of `pitch` bytes: s = bf16(1/sqrt(sum x^2 / K + eps)),
// y = bf16(bf16(x * s) * gamma). K % 4 == 0. Up to RP <= 4 rows per pass: gains and the
// rows in one round trip, one block reduction for all of them (a caller that knows R <= RP
// passes it, so that no registers hold rows that do not exist). `red` holds 64 floats.
// Every thread of the block (NT threads, at most 8 warps for the one-pass form) takes part.
template <int NT, bool CG = false, int RP = 4>
Y2_DEV void stage_rmsnorm_rows(const float* xf, const float* gamma, int K, int R, float eps, unsigned char* xs,
                               size_t pitch, float* red) {
  auto ld = [](const float4* p) { return CG ? __ldcg(p) : *p; };
  static_assert(NT % 32 == 0 && NT <= 512, "block size");
  constexpr int NW = NT / 32;
  constexpr int kQ = 4;   // float4 columns per thread held in registers
  static_assert(RP >= 1 && RP <= 4, "rows per pass");
  constexpr int kRP = RP;  // rows per pass
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K4 = K >> 2;
  const float4* gm = reinterpret_cast<const float4*>(gamma);
  auto put = [&](int r, int i, const float4& v, const float4& gg, float scale) {
    const uint32_t a = f2bf_exact(round_bf16(round_bf16(v.x * scale) * gg.x));
    const uint32_t b = f2bf_exact(round_bf16(round_bf16(v.y * scale) * gg.y));
    const uint32_t c = f2bf_exact(round_bf16(round_bf16(v.z * scale) * gg.z));
    const uint32_t d = f2bf_exact(round_bf16(round_bf16(v.w * scale) * gg.w));
    reinterpret_cast<uint2*>(xs + (size_t)r * pitch)[i] = make_uint2(a | (b << 16), c | (d << 16));
  };
  auto sq = [](const float4& v, float s) {
    s = fmaf(v.x, v.x, s);
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    return fmaf(v.w, v.w, s);
  };
  if (NW <= 8 && K4 <= kQ * NT) {
    float4 gv[kQ];
#pragma unroll
    for (int q = 0; q < kQ; ++q)
      if (tid + q * NT < K4) gv[q] = gm[tid + q * NT];
    for (int r0 = 0, pass = 0; r0 < R; r0 += kRP, ++pass) {
      float4 v[kRP][kQ];
#pragma unroll
      for (int k = 0; k < kRP; ++k) {
        const float4* xr = reinterpret_cast<const float4*>(xf + (size_t)min(r0 + k, R - 1) * K);
#pragma unroll
        for (int q = 0; q < kQ; ++q)
          if (tid + q * NT < K4) v[k][q] = ld(xr + tid + q * NT);
      }
      float* rn = red + (pass & 1) * 32;  // double-buffered: no barrier after the read
#pragma unroll
      for (int k = 0; k < kRP; ++k) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < kQ; ++q)
          if (tid + q * NT < K4) s = sq(v[k][q], s);
        s = warp_sum(s);
        if (lane == 0) rn[k * 8 + warp] = s;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kRP; ++k) {
        if (r0 + k >= R) break;
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += rn[k * 8 + w];
        const float sc = round_bf16(1.0f / sqrtf(t / (float)K + eps));
#pragma unroll
        for (int q = 0; q < kQ; ++q)
          if (tid + q * NT < K4) put(r0 + k, tid + q * NT, v[k][q], gv[q], sc);
      }
    }
  } else {
    for (int r = 0; r < R; ++r) {
      const float4* xr = reinterpret_cast<const float4*>(xf + (size_t)r * K);
      float ss = 0.f;
      for (int i = tid; i < K4; i += NT) ss = sq(ld(xr + i), ss);
      ss = warp_sum(ss);
      __syncthreads();
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float t = 0.f;
      for (int w = 0; w < NW; ++w) t += red[w];
      __syncthreads();
      const float scale = round_bf16(1.0f / sqrtf(t / (float)K + eps));
      for (int i = tid; i < K4; i += NT) put(r, i, ld(xr + i), gm[i], scale);
    }
  }
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
