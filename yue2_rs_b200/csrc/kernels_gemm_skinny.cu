// Skinny bf16 GEMM on the 5th-generation tensor cores (tcgen05) for the decode passes of
// 3..256 rows (several songs per GPU, two CFG rows each): Y[C, N] = X[C, K] . W[N, K]^T with
// f32 accumulation and Linear::finish's bf16 rounding (src/tensor.rs:1102-1118), or the
// SwiGLU form of Mlp::apply (src/model.rs:206-214) over W = [gate; up].
//
// Such a pass is bound by streaming W once (C is small next to N), so the layout is turned
// around against the prefill GEMM: 128 rows of W are the MMA's M side (A operand) and a
// chunk of CP <= 64 activation rows its N side (B operand; C > 64 rows take ceil(C / 64)
// chunks, which re-read the same W tile from L2 one after another). One 128 x CP
// accumulator in TMEM per (tile, chunk); the SwiGLU form issues a second MMA per K step with
// the matching up rows into columns CP.. of the same accumulator, so a thread's TMEM lane
// holds both the gate and the up sum of its output.
//
// A q|k|v or o matrix has only 24..40 tiles, too few for 148 SMs, so the work is cut by K
// blocks instead of by tiles: the (tile, chunk, K block) units are split into one contiguous
// equal range per CTA (one CTA per SM). A CTA streams its range through a TMA ring without
// pausing at tile boundaries. A (tile, chunk) that lies wholly inside one CTA's range is
// finished from TMEM. One cut by range boundaries (at most the first and the last of a
// CTA's range) leaves each of its CTAs a partial accumulator, written to a workspace; each
// epilogue warp then takes a ticket for its 32 rows, and the warp that completes the count
// adds the partials in CTA order (fixed, so results repeat bit for bit) and applies the
// epilogue. No CTA ever waits for another.
//
// Programmatic dependent launch: the producer requests the first ring stages of W (which
// no earlier kernel writes) before griddepcontrol.wait; activations, outputs, workspace and
// tickets are touched only after it.
//
// Warps: 0 TMA producer (one lane), 1 TMEM allocation and MMA issue (one lane), 2-5 the
// epilogue (warp w reads TMEM lanes 32 (w % 4) ..). Accumulators are double-buffered. Every
// mbarrier wait is bounded and sets *error when it gives up; all warps still meet at the
// final barrier, where warp 1 frees its TMEM.
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
constexpr int kMaxChunks = kSkinnyMaxRows / kMaxCP;
constexpr long kSpin = 1L << 24;
constexpr int kRingBudget = 200 * 1024;
constexpr int kMaxAcc = 2 * kMaxCP;   // TMEM columns of the widest accumulator (SwiGLU)
constexpr int RB = 8;                 // columns per reduction batch
constexpr int SB = 4;                 // partials per reduction batch

template <int CP, bool SW>
struct Shape {
  static constexpr int A_BYTES = (SW ? 2 : 1) * W_BYTES;
  static constexpr int X_BYTES = CP * BK * 2;
  static constexpr int STAGE = A_BYTES + X_BYTES;
  static constexpr int STAGES = kRingBudget / STAGE < 8 ? kRingBudget / STAGE : 8;
  static constexpr int ACC = SW ? 2 * CP : CP;  // TMEM columns of one accumulator
  static constexpr int TMEM = 2 * ACC < 32 ? 32 : 2 * ACC;  // two accumulators (a power of two)
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int CW = CP < 32 ? CP : 32;  // columns per TMEM load
  static_assert(STAGE % 1024 == 0 && A_BYTES % 1024 == 0, "swizzled tiles start on 1024-byte boundaries");
  static_assert(STAGES >= 2 && 2 * ACC <= 512 && (TMEM & (TMEM - 1)) == 0, "ring and TMEM");
};

struct SkinnyArgs {
  uint16_t* Y;
  int ldy, C, N, nk, nch;
  long long units;
  float* ws;
  uint32_t* tickets;
  int32_t* error;
};

using tc::fence_after;
using tc::fence_before;
using tc::sdesc_sw128;
using tc::smem_u32;

Y2_DEV bool wait_bar(uint64_t* b, uint32_t parity, int32_t* error) {
  return tc::mbar_wait_bounded(b, parity, error, kSpin);
}

// First unit of CTA b's range, and the CTA whose range holds unit u.
Y2_DEV long long unit0(int b, long long U, int G) { return (long long)b * U / G; }
Y2_DEV int cta_of(long long u, long long U, int G) { return (int)(((u + 1) * G + U - 1) / U - 1); }

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

// The segment of CTA range [.., u1) that starts at unit u: (tile, chunk) pair p, K blocks
// [ka, kend), and the unit after it.
struct Seg {
  int p, ka, kend;
  long long next;
};
Y2_DEV Seg segment(long long u, long long u1, int nk) {
  Seg s;
  s.p = (int)(u / nk);
  s.ka = (int)(u - (long long)s.p * nk);
  s.next = min(u1, (long long)(s.p + 1) * nk);
  s.kend = (int)(s.next - (long long)s.p * nk);
  return s;
}

template <int CP, bool SW>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                       const SkinnyArgs p) {
  using S = Shape<CP, SW>;
  constexpr int STAGES = S::STAGES, STAGE = S::STAGE, ACC = S::ACC, CW = S::CW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* ring = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;  // [2] accumulator complete (MMA -> epilogue)
  uint64_t* aempty = afull + 2;      // [2] accumulator drained (epilogue -> MMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, b = blockIdx.x, nk = p.nk, nch = p.nch;
  const long long U = p.units, u0 = unit0(b, U, G), u1 = unit0(b + 1, U, G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(afull + a, 1);
      tc::mbar_init(aempty + a, EPI_WARPS);
    }
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

  if (warp == 0) {
    if (lane == 0) {  // producer: every unit of the range, across tile boundaries
      // W of the first stages before the dependency wait (weights are never written by an
      // earlier kernel); each stage's barrier completes only once its activations land too
      const long long pre = min(u1 - u0, (long long)STAGES);
      for (long long i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const int pr = (int)(u / nk), kb = (int)(u - (long long)pr * nk), t = pr / nch;
        unsigned char* st = ring + (int)i * STAGE;
        tc::mbar_arrive_expect_tx(full + i, STAGE);
        tc::tma_load_2d(st, &tmw, full + i, kb * BK, t * BM);
        if (SW) tc::tma_load_2d(st + W_BYTES, &tmw, full + i, kb * BK, p.N + t * BM);  // up rows
      }
      pdl_wait();
      pdl_trigger();
      int it = 0;
      for (long long u = u0; u < u1; ++u, ++it) {
        const int pr = (int)(u / nk), kb = (int)(u - (long long)pr * nk), t = pr / nch, j = pr - t * nch;
        const int s = it % STAGES;
        unsigned char* st = ring + s * STAGE;
        if (it >= pre) {
          if (!wait_bar(empty + s, ((it / STAGES) - 1) & 1, p.error)) break;
          tc::mbar_arrive_expect_tx(full + s, STAGE);
          tc::tma_load_2d(st, &tmw, full + s, kb * BK, t * BM);
          if (SW) tc::tma_load_2d(st + W_BYTES, &tmw, full + s, kb * BK, p.N + t * BM);
        }
        tc::tma_load_2d(st + S::A_BYTES, &tmx, full + s, kb * BK, j * CP);
      }
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {  // MMA issue: one accumulator per segment
      constexpr uint32_t idesc = tc::idesc_bf16(BM, CP);
      bool ok = true;
      int it = 0, seg = 0;
      for (long long u = u0; u < u1 && ok; ++seg) {
        const Seg sg = segment(u, u1, nk);
        u = sg.next;
        const int a = seg & 1, use = seg >> 1;
        if (use > 0 && !(ok = wait_bar(aempty + a, (use - 1) & 1, p.error))) break;
        fence_after();
        const uint32_t d = tmem + (uint32_t)(a * ACC);
        for (int kb = sg.ka; kb < sg.kend; ++kb, ++it) {
          const int s = it % STAGES;
          if (!(ok = wait_bar(full + s, (it / STAGES) & 1, p.error))) break;
          fence_after();
          const uint32_t wa = smem_u32(ring + s * STAGE), xa = wa + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {  // 16 columns = 32 bytes along the swizzled rows
            const uint32_t acc = (kb != sg.ka || k != 0) ? 1u : 0u;
            tc::mma_bf16(d, sdesc_sw128(wa + 32 * k), sdesc_sw128(xa + 32 * k), idesc, acc);
            if (SW) tc::mma_bf16(d + CP, sdesc_sw128(wa + W_BYTES + 32 * k), sdesc_sw128(xa + 32 * k), idesc, acc);
          }
          tc::commit(empty + s);  // frees the stage once these MMAs have read it
        }
        tc::commit(afull + a);  // the segment's MMAs are complete (also after a give-up)
      }
    }
  } else {  // epilogue: TMEM lanes 32 q .. 32 q + 31 = weight rows of the tile
    pdl_wait();
    const int q = warp & 3, row = 32 * q + lane;
    const int first_pair = (int)(u0 / nk);
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const Seg sg = segment(u, u1, nk);
      u = sg.next;
      const int t = sg.p / nch, r0 = (sg.p - t * nch) * CP;  // tile, first activation row
      const int a = seg & 1, use = seg >> 1;
      if (!wait_bar(afull + a, use & 1, p.error)) break;
      fence_after();
      const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * ACC);
      const int n = t * BM + row;  // output column
      const int rows = min(CP, p.C - r0);
      uint16_t* yc = p.Y + (size_t)r0 * p.ldy + n;
      if (sg.ka == 0 && sg.kend == nk) {  // the whole K range is this CTA's: finish from TMEM
#pragma unroll 1
        for (int c0 = 0; c0 < CP; c0 += CW) {
          float g[CW], up[CW];
          tmem_load<CW>(tl + (uint32_t)c0, g);
          if (SW) tmem_load<CW>(tl + (uint32_t)(CP + c0), up);
#pragma unroll
          for (int j = 0; j < CW; ++j)
            if (c0 + j < rows && n < p.N) yc[(size_t)(c0 + j) * p.ldy] = finish<SW>(g[j], SW ? up[j] : 0.f);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(aempty + a);
        continue;
      }
      // a cut (tile, chunk): this CTA's partial sums to its workspace slot ([col][row])
      const int slot = sg.p == first_pair ? 0 : 1;
      float* wsp = p.ws + (size_t)(b * 2 + slot) * ACC * BM + row;
#pragma unroll 1
      for (int c0 = 0; c0 < ACC; c0 += CW) {
        float v[CW];
        tmem_load<CW>(tl + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < CW; ++j) wsp[(size_t)(c0 + j) * BM] = v[j];
      }
      fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(aempty + a);
      __threadfence();
      __syncwarp();
      const int c_first = cta_of((long long)sg.p * nk, U, G), c_last = cta_of((long long)sg.p * nk + nk - 1, U, G);
      uint32_t last = 0;
      if (lane == 0) {
        const uint32_t prev = atomicAdd(p.tickets + (size_t)sg.p * 4 + q, 1u);
        last = prev == (uint32_t)(c_last - c_first);
        if (last) atomicExch(p.tickets + (size_t)sg.p * 4 + q, 0u);  // ready for the next launch
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      // sum the partials in CTA order, SB partials x RB columns of loads in flight at a time
#pragma unroll 1
      for (int c0 = 0; c0 < CP; c0 += RB) {
        float g[RB], up[RB];
#pragma unroll
        for (int j = 0; j < RB; ++j) g[j] = up[j] = 0.f;
#pragma unroll 1
        for (int c = c_first; c <= c_last; c += SB) {
          float tg[SB][RB], tu[SB][RB];
#pragma unroll
          for (int k = 0; k < SB; ++k) {
            if (c + k > c_last) break;
            const int sc = sg.p == (int)(unit0(c + k, U, G) / nk) ? 0 : 1;
            const float* src = p.ws + (size_t)((c + k) * 2 + sc) * ACC * BM + row;
#pragma unroll
            for (int j = 0; j < RB; ++j) {
              tg[k][j] = __ldcg(src + (size_t)(c0 + j) * BM);
              if (SW) tu[k][j] = __ldcg(src + (size_t)(CP + c0 + j) * BM);
            }
          }
#pragma unroll
          for (int k = 0; k < SB; ++k) {
            if (c + k > c_last) break;
#pragma unroll
            for (int j = 0; j < RB; ++j) {
              g[j] += tg[k][j];
              if (SW) up[j] += tu[k][j];
            }
          }
        }
#pragma unroll
        for (int j = 0; j < RB; ++j)
          if (c0 + j < rows && n < p.N) yc[(size_t)(c0 + j) * p.ldy] = finish<SW>(g[j], up[j]);
      }
    }
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
  return launch_with(s, pdl, dim3(grid), dim3(THREADS), S::SMEM, fn, argv);
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

}  // namespace

bool gemm_skinny_supported(int C, int N, int K, int ldx, int ldy, const void* X, const void* W, const void* Y,
                           bool swiglu) {
  return C >= 1 && C <= kSkinnyMaxRows && N >= 1 && K >= BK && K % BK == 0 && ldx % 8 == 0 && ldx >= K &&
         ldy >= N && (!swiglu || N % BM == 0) && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0 &&
         Y != nullptr;
}

size_t gemm_skinny_ws_bytes(int sms) { return (size_t)sms * 2 * kMaxAcc * BM * sizeof(float); }
int gemm_skinny_tickets(int max_tiles) { return max_tiles * kMaxChunks * 4; }

cudaError_t launch_gemm_skinny(cudaStream_t s, bool pdl, const uint16_t* W, int N, int K, const uint16_t* X, int ldx,
                               uint16_t* Y, int ldy, int C, bool swiglu, const SkinnyWork& work, int32_t* error) {
  if (!gemm_skinny_supported(C, N, K, ldx, ldy, X, W, Y, swiglu) || !work.ws || !work.tickets)
    return cudaErrorInvalidValue;
  static int sms_dev = -1, sms = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (sms_dev != dev) {
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    sms_dev = dev;
  }
  const int CP = padded_rows(C), nch = (C + CP - 1) / CP;
  const int tiles = (N + BM - 1) / BM, nk = K / BK;
  const long long units = (long long)tiles * nch * nk;
  const int grid = (int)std::min<long long>(sms, units);
  const size_t acc = swiglu ? 2 * CP : CP;
  if (tiles > work.max_tiles || (size_t)grid * 2 * acc * BM * sizeof(float) > work.ws_bytes)
    return cudaErrorInvalidValue;
  alignas(64) CUtensorMap mw, mx;
  if (!make_tma_map_bf16(&mw, W, swiglu ? 2 * N : N, K, K, BM) || !make_tma_map_bf16(&mx, X, C, K, ldx, CP))
    return cudaErrorInvalidValue;
  const SkinnyArgs a{Y, ldy, C, N, nk, nch, units, work.ws, work.tickets, error};
  return swiglu ? go_rows<true>(CP, s, pdl, mw, mx, a, grid) : go_rows<false>(CP, s, pdl, mw, mx, a, grid);
}

}  // namespace y2
