// Causal prefill attention on the tensor cores (the batched form of model::attention,
// src/model.rs:314-397: scores q.k * scale in f32, softmax in f32, P.V in f32, output
// rounded to bf16).
//
// One CTA per (tile of 64 chunk rows, q head); four warps of 16 rows each. The CTA walks
// the cache's pages (64 keys each, one page = one key tile of this kv head) from position
// 0 up to its last row, double-buffered with cp.async into XOR-swizzled shared memory.
// Per tile a warp computes S = Q K^T with mma.m16n8k16 (bf16 in, f32 accumulate), masks
// keys after each row's position, updates an online softmax in f32, and accumulates O +=
// P V where P is split into bf16 hi + lo parts (two MMAs), so P.V keeps f32 accuracy
// instead of rounding the probabilities to bf16. Keys past the CTA's last row are
// zero-filled, never read.
#include "common.cuh"
#include "kernels.h"

namespace y2 {

namespace {

constexpr int kRowsPerCta = 64;
constexpr int kKeys = kPageTokens;  // keys per tile = one page

// byte offset of 16-byte chunk c of row r in a [rows][D] bf16 tile, XOR-swizzled over
// groups of 8 chunks so that ldmatrix's 8 row addresses hit distinct banks
template <int D>
Y2_DEV uint32_t swz(int r, int c) {
  return (uint32_t)(r * D * 2 + ((c ^ (r & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(128, 2) prefill_attn_kernel(const PrefillAttnParams p) {
  constexpr int CH = D / 8;   // 16-byte chunks per row
  constexpr int KS = D / 16;  // k-steps over head dims
  constexpr int NT = D / 8;   // n-tiles over head dims
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* qs = smem;                          // [64][D]
  unsigned char* ks = qs + kRowsPerCta * D * 2;      // [2][64][D]
  unsigned char* vs = ks + 2 * kKeys * D * 2;        // [2][64][D]

  const Geometry& g = p.g;
  const int ntiles = (p.C + kRowsPerCta - 1) / kRowsPerCta;
  const int tile = ntiles - 1 - (int)blockIdx.x;  // longest rows first
  const int h = blockIdx.y, kvh = h / (g.heads / g.kvh);
  const int row0 = tile * kRowsPerCta;
  const int nrows = min(kRowsPerCta, p.C - row0);
  const int q0 = p.pos0 + row0;              // position of the tile's first row
  // causal: the tile's last row; otherwise (every row sees every row of the chunk) the
  // chunk's last row
  const int last_key = p.causal ? q0 + nrows - 1 : p.pos0 + p.C - 1;
  const int nkt = (last_key >> kPageLog2) + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = g.heads * D;
  const size_t koff = kv_offset(g, p.layer, 0, kvh), voff = kv_offset(g, p.layer, 1, kvh);

  // ---- Q tile (rows past the chunk zero-filled) and the first K/V tile
  for (int i = tid; i < kRowsPerCta * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < nrows;
    cp_async16_zfill(qs + swz<D>(r, c), p.q + (size_t)(row0 + (ok ? r : 0)) * qd + (size_t)h * D + c * 8, ok);
  }
  auto stage = [&](int kt) {
    const uint16_t* page = reinterpret_cast<const uint16_t*>(p.pages[kt]);
    unsigned char* kb = ks + (kt & 1) * kKeys * D * 2;
    unsigned char* vb = vs + (kt & 1) * kKeys * D * 2;
    for (int i = tid; i < kKeys * CH; i += 128) {
      const int r = i / CH, c = i % CH;
      const bool ok = (kt << kPageLog2) + r <= last_key;
      const size_t off = (size_t)(ok ? r : 0) * D + c * 8;
      cp_async16_zfill(kb + swz<D>(r, c), page + koff + off, ok);
      cp_async16_zfill(vb + swz<D>(r, c), page + voff + off, ok);
    }
  };
  stage(0);
  cp_async_commit();

  // per-thread rows of the warp's 16: g8 = lane / 4 and g8 + 8; columns 2 * (lane % 4) + {0, 1}
  const int g8 = lane >> 2, t4 = lane & 3;
  const int wrow = warp * 16;
  // the last key each of this thread's two rows may see (rows a = g8 and b = g8 + 8)
  const int pos_a = p.causal ? q0 + wrow + g8 : last_key, pos_b = p.causal ? pos_a + 8 : last_key;
  const int warp_first = p.causal ? q0 + wrow : last_key;  // the smallest such limit in the warp
  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[KS][4];

  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) stage(kt + 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int mi = lane >> 3, r = wrow + (mi & 1) * 8 + (lane & 7);
        ldsm_x4(qf[kk], qs + swz<D>(r, 2 * kk + (mi >> 1)));
      }
    }
    const int key0 = kt << kPageLog2;
    // a warp whose rows all precede this tile has nothing to add
    if (!p.causal || key0 <= q0 + wrow + 15) {
      const unsigned char* kb = ks + (kt & 1) * kKeys * D * 2;
      const unsigned char* vb = vs + (kt & 1) * kKeys * D * 2;
      // ---- S = Q K^T: 8 n-tiles of 8 keys
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; kk += 2) {
          uint32_t b[4];
          ldsm_x4(b, kb + swz<D>(8 * j + (lane & 7), 2 * kk + (lane >> 3)));
          mma_bf16_16816(s[j], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b[0], b[1]);
          mma_bf16_16816(s[j], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b[2], b[3]);
        }
      }
      // ---- scale, causal mask, online softmax (rows a = g8, b = g8 + 8)
      const bool diag = key0 + kKeys - 1 > warp_first;  // some key lies past some row's limit
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + 8 * j + 2 * t4 + e;
          float va = s[j][e] * p.scale, vb2 = s[j][2 + e] * p.scale;
          if (diag) {
            va = key <= pos_a ? va : -INFINITY;
            vb2 = key <= pos_b ? vb2 : -INFINITY;
          }
          s[j][e] = va;
          s[j][2 + e] = vb2;
          mx_a = fmaxf(mx_a, va);
          mx_b = fmaxf(mx_b, vb2);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      // key 0 is in tile 0 and precedes every row, so m is finite from the first tile on
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float al_a = m_a == -INFINITY ? 0.f : __expf(m_a - mn_a);
      const float al_b = m_b == -INFINITY ? 0.f : __expf(m_b - mn_b);
      m_a = mn_a;
      m_b = mn_b;
      float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pa = __expf(s[j][e] - mn_a), pb = __expf(s[j][2 + e] - mn_b);
          s[j][e] = pa;
          s[j][2 + e] = pb;
          sum_a += pa;
          sum_b += pb;
        }
      }
      sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 1);
      sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 2);
      sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 1);
      sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 2);
      l_a = l_a * al_a + sum_a;
      l_b = l_b * al_b + sum_b;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        o[j][0] *= al_a;
        o[j][1] *= al_a;
        o[j][2] *= al_b;
        o[j][3] *= al_b;
      }
      // ---- O += P V over 4 k-steps of 16 keys; P = hi + lo in bf16
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ah[4], alo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // a0: rows a, tile 2kk; a1: rows b, tile 2kk; a2: rows a, tile 2kk+1; a3: rows b, tile 2kk+1
          const int j = 2 * kk + (q >> 1), c = (q & 1) * 2;
          const float x0 = s[j][c], x1 = s[j][c + 1];
          ah[q] = pack_bf16x2(x0, x1);
          alo[q] = pack_bf16x2(x0 - bf_lo(ah[q]), x1 - bf_hi(ah[q]));
        }
#pragma unroll
        for (int jd = 0; jd < NT; jd += 2) {
          uint32_t b[4];
          const int mi = lane >> 3;
          ldsm_x4_trans(b, vb + swz<D>(16 * kk + (mi & 1) * 8 + (lane & 7), jd + (mi >> 1)));
          mma_bf16_16816(o[jd], ah[0], ah[1], ah[2], ah[3], b[0], b[1]);
          mma_bf16_16816(o[jd], alo[0], alo[1], alo[2], alo[3], b[0], b[1]);
          mma_bf16_16816(o[jd + 1], ah[0], ah[1], ah[2], ah[3], b[2], b[3]);
          mma_bf16_16816(o[jd + 1], alo[0], alo[1], alo[2], alo[3], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // buffer kt & 1 is refilled by the next iteration's stage
  }
  cp_async_wait<0>();

  // ---- normalise and store bf16
  const float inv_a = 1.0f / l_a, inv_b = 1.0f / l_b;
  const int ra = wrow + g8, rb = ra + 8;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int col = h * D + 8 * j + 2 * t4;
    if (ra < nrows) {
      const uint32_t w = (uint32_t)f2bf_round(o[j][0] * inv_a) | ((uint32_t)f2bf_round(o[j][1] * inv_a) << 16);
      *reinterpret_cast<uint32_t*>(p.out + (size_t)(row0 + ra) * qd + col) = w;
    }
    if (rb < nrows) {
      const uint32_t w = (uint32_t)f2bf_round(o[j][2] * inv_b) | ((uint32_t)f2bf_round(o[j][3] * inv_b) << 16);
      *reinterpret_cast<uint32_t*>(p.out + (size_t)(row0 + rb) * qd + col) = w;
    }
  }
}

template <int D>
constexpr int prefill_attn_smem() {
  return (kRowsPerCta + 4 * kKeys) * D * 2;
}

template <int D>
cudaError_t prefill_attn_go(cudaStream_t s, const PrefillAttnParams& p) {
  const void* fn = (const void*)prefill_attn_kernel<D>;
  static int set_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (set_dev != dev) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, prefill_attn_smem<D>());
    if (e != cudaSuccess) return e;
    set_dev = dev;
  }
  PrefillAttnParams copy = p;
  void* args[] = {&copy};
  const dim3 grid((p.C + kRowsPerCta - 1) / kRowsPerCta, p.g.heads);
  return launch_with(s, false, grid, dim3(128), prefill_attn_smem<D>(), fn, args);
}

}  // namespace

bool prefill_attention_supported(const Geometry& g) { return g.dim == 64 || g.dim == 128; }

cudaError_t launch_prefill_attention(cudaStream_t s, const PrefillAttnParams& p) {
  if (p.C < 1 || p.pos0 < 0) return cudaErrorInvalidValue;
  switch (p.g.dim) {
    case 64: return prefill_attn_go<64>(s, p);
    case 128: return prefill_attn_go<128>(s, p);
  }
  return cudaErrorInvalidValue;
}

}  // namespace y2
