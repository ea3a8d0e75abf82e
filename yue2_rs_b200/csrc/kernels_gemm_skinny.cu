// Skinny bf16 GEMM on the 5th-generation tensor cores (tcgen05) for the decode passes of
// 3..256 rows (several songs per GPU, two CFG rows each): Y[C, N] = X[C, K] . W[N, K]^T with
// f32 accumulation and Linear::finish's bf16 rounding (src/tensor.rs:1102-1118), or the
// SwiGLU form of Mlp::apply (src/model.rs:206-214) over W = [gate; up].
//
// Such a pass is bound by streaming W once (C is small next to N), so the layout is turned
// around against the prefill GEMM: 128 rows of W are the MMA's M side (A operand) and a
// chunk of CP <= 64 activation rows its N side (B operand; C > 64 rows take ceil(C / 64)
// chunks, which re-read the same W tile from L2). One 128 x CP accumulator in TMEM per
// CTA; the SwiGLU form issues a second MMA per K step with the matching up rows into
// columns CP.. of the same accumulator, so a thread's TMEM lane holds both the gate and the
// up sum of its output.
//
// A q|k|v or o matrix has only 24..40 tiles, too few for 148 SMs, so each (tile, chunk) is
// also split over S CTAs by K (S <= 8, chosen per shape to fill the SMs) that form one
// thread-block cluster. Each CTA streams its K range through a TMA ring; with S > 1 it
// leaves its partial accumulator in its own shared memory, and after a cluster barrier
// CTA s sums the S partials of rows [s * 128 / S, ...) through distributed shared memory,
// in rank order (the same bits every run), and applies the epilogue. A second barrier keeps
// every partial readable until all CTAs are done. No global workspace, fence or ticket.
//
// Programmatic dependent launch: the producer requests the first ring stages of W (which
// no earlier kernel writes) before griddepcontrol.wait; activations and outputs are touched
// only after it.
//
// Warps: 0 TMA producer (one lane), 1 TMEM allocation and MMA issue (one lane), 2-5 the
// epilogue (warp w reads TMEM lanes 32 (w % 4) ..). Every mbarrier wait is bounded and sets
// *error when it gives up; all threads still meet at both cluster barriers and the final
// one, where warp 1 frees its TMEM.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace y2 {
namespace {

constexpr int BM = 128;               // weight rows per tile: the MMA's M
constexpr int BK = 64;                // K block: one 128-byte swizzled row per operand row
constexpr int W_BYTES = BM * BK * 2;  // one weight block
constexpr int THREADS = 192;
constexpr int EPI_WARPS = 4;
constexpr int kMaxCP = 64;            // activation rows per chunk
constexpr int kMaxSplit = 8;          // CTAs per cluster (portable cluster size)
constexpr long kSpin = 1L << 24;

template <int CP, bool SW>
struct Shape {
  static constexpr int A_BYTES = (SW ? 2 : 1) * W_BYTES;
  static constexpr int X_BYTES = CP * BK * 2;
  static constexpr int STAGE = A_BYTES + X_BYTES;
  // two CTAs per SM (a ring of ~100 KB each), so that clusters of up to 8 always find room
  // in a GPC; the widest form (SwiGLU, 64 rows) keeps one CTA per SM and a deeper ring
  static constexpr int CTAS_PER_SM = (SW && CP == 64) ? 1 : 2;
  static constexpr int BUDGET = CTAS_PER_SM == 2 ? 110 * 1024 : 200 * 1024;
  static constexpr int STAGES = BUDGET / STAGE < 8 ? BUDGET / STAGE : 8;
  static constexpr int ACC = SW ? 2 * CP : CP;  // TMEM columns of the accumulator
  static constexpr int TMEM = ACC < 32 ? 32 : ACC;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int CW = CP < 32 ? CP : 32;  // columns per TMEM load
  static_assert(STAGE % 1024 == 0 && A_BYTES % 1024 == 0, "swizzled tiles start on 1024-byte boundaries");
  static_assert(STAGES >= 2 && (TMEM & (TMEM - 1)) == 0, "ring and TMEM");
  static_assert(ACC * BM * 4 <= STAGES * STAGE, "the partial fits in the ring");
};

struct SkinnyArgs {
  uint16_t* Y;
  int ldy, C, N, nk, nch, split;
  int32_t* error;
};

using tc::fence_after;
using tc::fence_before;
using tc::sdesc_sw128;
using tc::smem_u32;

Y2_DEV bool wait_bar(uint64_t* b, uint32_t parity, int32_t* error) {
  return tc::mbar_wait_bounded(b, parity, error, kSpin);
}

template <int CW>
Y2_DEV void tmem_load(uint32_t taddr, float (&v)[CW]) {
  uint32_t r[CW];
  if constexpr (CW == 32) tc::tmem_ld32(taddr, r);
  else tc::tmem_ld16(taddr, r);
#pragma unroll
  for (int j = 0; j < CW; ++j) v[j] = __uint_as_float(r[j]);
}

template <bool SW>
Y2_DEV uint16_t finish(float g, float u) {
  if constexpr (SW) {
    const float gv = round_bf16(g), uv = round_bf16(u);
    const float act = round_bf16(gv / (1.0f + det_expf(-gv)));
    return f2bf_round(act * uv);
  } else {
    return f2bf_round(g);
  }
}

template <int CP, bool SW>
__global__ void __launch_bounds__(THREADS, Shape<CP, SW>::CTAS_PER_SM)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                       const SkinnyArgs p) {
  using S = Shape<CP, SW>;
  constexpr int STAGES = S::STAGES, STAGE = S::STAGE, ACC = S::ACC, CW = S::CW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;  // the accumulator is complete (MMA -> epilogue)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(afull + 1);
  float* part = reinterpret_cast<float*>(ring);  // [ACC][BM] after the MMAs: this CTA's partial sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsp = p.split, sp = blockIdx.x % nsp, pr = blockIdx.x / nsp;  // split = cluster rank
  const int t = pr / p.nch, r0 = (pr - t * p.nch) * CP;                   // tile, first activation row
  const int ka = (int)(((long long)p.nk * sp) / nsp), kb_end = (int)(((long long)p.nk * (sp + 1)) / nsp);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, 1);
    }
    tc::mbar_init(afull, 1);
    tc::mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(S::TMEM)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_units = kb_end - ka;

  if (warp == 0) {
    if (lane == 0) {  // producer
      // W of the first stages before the dependency wait (weights are never written by an
      // earlier kernel); each stage's barrier completes only once its activations land too
      const int pre = min(n_units, STAGES);
      for (int i = 0; i < pre; ++i) {
        unsigned char* st = ring + i * STAGE;
        tc::mbar_arrive_expect_tx(full + i, STAGE);
        tc::tma_load_2d(st, &tmw, full + i, (ka + i) * BK, t * BM);
        if (SW) tc::tma_load_2d(st + W_BYTES, &tmw, full + i, (ka + i) * BK, p.N + t * BM);  // up rows
      }
      pdl_wait();
      pdl_trigger();
      for (int i = 0; i < n_units; ++i) {
        const int s = i % STAGES, kb = ka + i;
        unsigned char* st = ring + s * STAGE;
        if (i >= pre) {
          if (!wait_bar(empty + s, ((i / STAGES) - 1) & 1, p.error)) break;
          tc::mbar_arrive_expect_tx(full + s, STAGE);
          tc::tma_load_2d(st, &tmw, full + s, kb * BK, t * BM);
          if (SW) tc::tma_load_2d(st + W_BYTES, &tmw, full + s, kb * BK, p.N + t * BM);
        }
        tc::tma_load_2d(st + S::A_BYTES, &tmx, full + s, kb * BK, r0);
      }
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {  // MMA issue into the one accumulator
      constexpr uint32_t idesc = tc::idesc_bf16(BM, CP);
      for (int i = 0; i < n_units; ++i) {
        const int s = i % STAGES;
        if (!wait_bar(full + s, (i / STAGES) & 1, p.error)) break;
        fence_after();
        const uint32_t wa = smem_u32(ring + s * STAGE), xa = wa + S::A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {  // 16 columns = 32 bytes along the swizzled rows
          const uint32_t acc = (i != 0 || k != 0) ? 1u : 0u;
          tc::mma_bf16(tmem, sdesc_sw128(wa + 32 * k), sdesc_sw128(xa + 32 * k), idesc, acc);
          if (SW) tc::mma_bf16(tmem + CP, sdesc_sw128(wa + W_BYTES + 32 * k), sdesc_sw128(xa + 32 * k), idesc, acc);
        }
        tc::commit(empty + s);  // frees the stage once these MMAs have read it
      }
      tc::commit(afull);  // the MMAs are complete (also after a give-up)
    }
  } else {  // epilogue: TMEM lanes 32 q .. 32 q + 31 = weight rows of the tile
    pdl_wait();
    const int q = warp & 3, row = 32 * q + lane;
    const bool ok = wait_bar(afull, 0, p.error);
    fence_after();
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
    const int n = t * BM + row, rows = min(CP, p.C - r0);
    if (nsp == 1) {  // the whole K range is this CTA's: finish from TMEM
      if (ok) {
#pragma unroll 1
        for (int c0 = 0; c0 < CP; c0 += CW) {
          float g[CW], up[CW];
          tmem_load<CW>(tl + (uint32_t)c0, g);
          if (SW) tmem_load<CW>(tl + (uint32_t)(CP + c0), up);
#pragma unroll
          for (int j = 0; j < CW; ++j)
            if (c0 + j < rows && n < p.N)
              p.Y[(size_t)(r0 + c0 + j) * p.ldy + n] = finish<SW>(g[j], SW ? up[j] : 0.f);
        }
      }
    } else {  // the partial into shared memory ([col][row]: lanes write consecutive words)
#pragma unroll 1
      for (int c0 = 0; c0 < ACC; c0 += CW) {
        float v[CW];
        if (ok) tmem_load<CW>(tl + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < CW; ++j) part[(size_t)(c0 + j) * BM + row] = ok ? v[j] : 0.f;
      }
    }
  }
  if (nsp > 1) {
    cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
    // the producer and MMA lanes reach here apart from the rest of their warps: reconverge
    // every warp before the cluster barrier (its arrive is a warp-aligned operation)
    __syncwarp();
    cl.sync();  // every CTA's partial is in its shared memory
    if (warp >= 2) {
      // this CTA's rows [sp * BM / nsp, (sp + 1) * BM / nsp) of the tile, all CP columns
      const int rb = (sp * BM) / nsp, re = ((sp + 1) * BM) / nsp, nr = re - rb;
      const int rows = min(CP, p.C - r0);
      const float* src[kMaxSplit];  // every rank's partial, mapped once
#pragma unroll
      for (int k = 0; k < kMaxSplit; ++k) src[k] = k < nsp ? cl.map_shared_rank(part, k) : part;
      constexpr int OU = 2;  // outputs per thread and pass: their loads all in flight together
      const int total = nr * CP;
      for (int i0 = threadIdx.x - 64; i0 < total; i0 += 128 * OU) {
        // all ranks' values of OU outputs requested before any is added; each sum in rank
        // order (the same bits every run)
        float gv[OU][kMaxSplit], uv[OU][kMaxSplit];
#pragma unroll
        for (int o = 0; o < OU; ++o) {
          const int i = i0 + o * 128;
          const int c = i / nr, rr = rb + i % nr;  // consecutive threads: consecutive weight rows
#pragma unroll
          for (int k = 0; k < kMaxSplit; ++k) {
            const bool on = i < total && k < nsp;
            gv[o][k] = on ? src[k][(size_t)c * BM + rr] : 0.f;
            uv[o][k] = (SW && on) ? src[k][(size_t)(CP + c) * BM + rr] : 0.f;
          }
        }
#pragma unroll
        for (int o = 0; o < OU; ++o) {
          const int i = i0 + o * 128;
          if (i >= total) continue;
          const int c = i / nr, rr = rb + i % nr;
          float g = 0.f, up = 0.f;
#pragma unroll
          for (int k = 0; k < kMaxSplit; ++k)
            if (k < nsp) {
              g += gv[o][k];
              up += uv[o][k];
            }
          const int n = t * BM + rr;
          if (c < rows && n < p.N) p.Y[(size_t)(r0 + c) * p.ldy + n] = finish<SW>(g, up);
        }
      }
    }
    __syncwarp();
    cl.sync();  // the partials stay readable until every CTA of the cluster is done
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::TMEM) : "memory");
  }
}

template <int CP, bool SW>
cudaError_t go(cudaStream_t s, bool pdl, const CUtensorMap& mw, const CUtensorMap& mx, const SkinnyArgs& a,
               int grid) {
  using S = Shape<CP, SW>;
  const void* fn = (const void*)gemm_skinny_kernel<CP, SW>;
  static int set_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (set_dev != dev) {
    if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM)) != cudaSuccess)
      return e;
    set_dev = dev;
  }
  CUtensorMap w = mw, x = mx;
  SkinnyArgs args = a;
  void* argv[] = {&w, &x, &args};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;  // the splits of one tile
  attr[0].val.clusterDim.x = (unsigned)a.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelExC(&cfg, fn, argv);
}

template <bool SW>
cudaError_t go_rows(int CP, cudaStream_t s, bool pdl, const CUtensorMap& mw, const CUtensorMap& mx,
                    const SkinnyArgs& a, int grid) {
  switch (CP) {
    case 16: return go<16, SW>(s, pdl, mw, mx, a, grid);
    case 32: return go<32, SW>(s, pdl, mw, mx, a, grid);
    default: return go<64, SW>(s, pdl, mw, mx, a, grid);
  }
}

int padded_rows(int C) { return C <= 16 ? 16 : C <= 32 ? 32 : 64; }

// K splits per (tile, chunk): the largest count that still gives every CTA an SM of its own
// (two CTAs sharing an SM share its bandwidth, and clusters that do not fit at once start a
// wave late), with at least 4 K blocks per split and at most kMaxSplit.
int choose_split(int pairs, int nk, int sms) {
  int best = 1;
  for (int s = 2; s <= kMaxSplit && s * 4 <= nk; ++s)
    if ((long)pairs * s <= sms) best = s;
  return best;
}

}  // namespace

bool gemm_skinny_supported(int C, int N, int K, int ldx, int ldy, const void* X, const void* W, const void* Y,
                           bool swiglu) {
  return C >= 1 && C <= kSkinnyMaxRows && N >= 1 && K >= BK && K % BK == 0 && ldx % 8 == 0 && ldx >= K &&
         ldy >= N && (!swiglu || N % BM == 0) && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0 &&
         Y != nullptr;
}

cudaError_t launch_gemm_skinny(cudaStream_t s, bool pdl, const uint16_t* W, int N, int K, const uint16_t* X, int ldx,
                               uint16_t* Y, int ldy, int C, bool swiglu, int32_t* error) {
  if (!gemm_skinny_supported(C, N, K, ldx, ldy, X, W, Y, swiglu)) return cudaErrorInvalidValue;
  static int sms_dev = -1, sms = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (sms_dev != dev) {
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    sms_dev = dev;
  }
  const int CP = padded_rows(C), nch = (C + CP - 1) / CP;
  const int tiles = (N + BM - 1) / BM, nk = K / BK, pairs = tiles * nch;
  const int split = choose_split(pairs, nk, sms);
  const long long grid = (long long)pairs * split;
  if (grid > INT32_MAX) return cudaErrorInvalidValue;
  alignas(64) CUtensorMap mw, mx;
  if (!make_tma_map_bf16(&mw, W, swiglu ? 2 * N : N, K, K, BM) || !make_tma_map_bf16(&mx, X, C, K, ldx, CP))
    return cudaErrorInvalidValue;
  const SkinnyArgs a{Y, ldy, C, N, nk, nch, split, error};
  return swiglu ? go_rows<true>(CP, s, pdl, mw, mx, a, (int)grid) : go_rows<false>(CP, s, pdl, mw, mx, a, (int)grid);
}

}  // namespace y2
