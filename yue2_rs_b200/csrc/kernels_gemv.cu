// Tensor-core GEMV of the decode step (sm_100a).
//
// y[r, n] = sum_k W[n, k] * x[r, k] for R <= 16 activation rows, with the epilogues of
// Linear::finish (src/tensor.rs:1102-1118), the residual add (src/tensor.rs:632-640,
// src/model.rs:586-587), SwiGLU (src/model.rs:206-214) and the bf16 logits of
// Model::forward_phase (src/model.rs:465-507). The GPU realisation it replaces is
// weight_vector (src/attention.metal:179-203).
//
// One CTA per SM streams a contiguous share of the weight rows, in tiles of eight rows
// (four gate + four up rows for SwiGLU). The CTA's (tile, 128-column block) items are
// split into equal contiguous shares, one per warp. A warp copies an item (eight 256-byte
// row segments) with cp.async into its own slot of an eight-item shared-memory ring (four
// when the activations leave no room), seven items ahead of the one it multiplies; each copy instruction moves two whole segments,
// so every request is 256 contiguous bytes. cp.async.wait_group plus __syncwarp is the
// only wait: no block barrier, no spin, no cross-warp dependency while streaming.
//
// Each 16-byte piece is two mma.sync m16n8k16 steps with A = the R activation rows (the
// fragment's sixteen rows) and B = the eight weight rows: the lane's columns 8t..8t+3 act
// as k = {2t, 2t+1, 2t+8, 2t+9} of the first step and 8t+4..8t+7 of the second, and the
// activations use the same column order, so every dot product is unchanged. Four
// independent accumulator chains (one per piece) hide the mma latency. A tile that one
// warp covers completely is finished by that warp; the partial sums of a tile split
// between warps are added in warp order after the stream (deterministic).
//
// The first seven items are requested before griddepcontrol.wait, so they stream while
// the previous kernel drains and while the activations are staged.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace y2 {

constexpr int kTileRows = 8;           // weight rows per tile
constexpr int kTcMaxSmem = 227 * 1024 - 1024;

// Staged row of a BC-column block: 2*BC bytes + 64, so that rows start 64 bytes apart modulo
// 128 and the eight lanes of a quarter-warp (two rows x four 16-byte pieces) hit distinct banks.
__host__ __device__ constexpr int row_pitch(int bc) { return bc * 2 + 64; }
__host__ __device__ constexpr int slot_bytes(int bc) { return kTileRows * row_pitch(bc); }
__host__ __device__ constexpr int ring_bytes(int warps, int bc, int ring) { return warps * ring * slot_bytes(bc); }
__host__ __device__ constexpr int piece_bytes(int warps) { return warps * 2 * 32 * 16; }
// Activation row pitch: 64 mod 128 bytes, so that the eight lanes of a quarter-warp (two
// activation rows x four 16-byte pieces) hit distinct banks.
__host__ __device__ inline size_t x_pitch(int K) { return ((2 * (size_t)K + 127) / 128) * 128 + 64; }


template <int W, int BC, int kRing, bool PAIR, int XM, int EPI>
__global__ void __launch_bounds__(W * 32) gemv_tc_kernel(const GemvParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float red_norm[64];
  __shared__ int s_cut[W], s_ncut;
  constexpr int NT = W * 32;
  constexpr int kBlockCols = BC;
  constexpr int kCh = BC / 32;           // 32-column chunks per item = copies per lane per item
  constexpr int kPPR = BC / 8;           // 16-byte pieces per staged row
  constexpr int kRowPitch = row_pitch(BC), kSlot = slot_bytes(BC);
  constexpr int kLaneRows = BC == 128 ? 4 : 8;  // distinct rows one lane copies per item
  static_assert(BC == 128 || BC == 256 || BC == 512, "block width");
  constexpr int TU = PAIR ? kTileRows / 2 : kTileRows;  // output units per tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int K = p.K, R = p.R;
  const int u0 = (int)(((long long)p.N * blockIdx.x) / gridDim.x);
  const int u1 = (int)(((long long)p.N * (blockIdx.x + 1)) / gridDim.x);
  const int ntiles = (u1 - u0 + TU - 1) / TU;
  const int nkb = K / kBlockCols;
  const int items = ntiles * nkb;
  auto share = [&](int w) { return (int)(((long long)items * w) / W); };
  const int ia = share(warp), ib = share(warp + 1), T = ib - ia;
  const size_t xp = x_pitch(K);
  unsigned char* ring = smem + (size_t)warp * kRing * kSlot;  // [slot][row][kRowPitch]
  unsigned char* xs = smem + ring_bytes(W, BC, kRing);
  float4* pieces = reinterpret_cast<float4*>(xs + (size_t)R * xp);  // [W][2][32]

  auto wrow = [&](int n) -> const uint16_t* {
    const int s = (n >= p.seg_start[2]) ? 2 : (n >= p.seg_start[1]) ? 1 : 0;
    return p.w[s] + (size_t)(n - p.seg_start[s]) * K;
  };
  // weight row j of tile `tile` (nullptr past the CTA's share)
  auto tile_row = [&](int tile, int j) -> const uint16_t* {
    const int q = PAIR ? (j & 3) : j;
    const int n = u0 + tile * TU + q;
    if (n >= u1) return nullptr;
    if (PAIR) return j < 4 ? wrow(n) : p.wpair + (size_t)n * K;
    return wrow(n);
  };

  // ---- issue stream, advanced incrementally. Copy c of lane L moves the 16-byte piece
  // (32c + L) % kPPR of staged row (32c + L) / kPPR: each copy instruction covers whole
  // 256-byte (or longer) runs of a row.
  int i_cnt = 0, i_tile = ia / nkb, i_kb = ia % nkb;
  const uint16_t* i_src[kLaneRows];
  auto lane_row = [&](int c) { return (32 * c + lane) / kPPR; };        // staged row of copy c
  auto lane_slot = [&](int c) { return BC == 128 ? c : (BC == 256 ? c : c >> 1); };
  auto load_rows = [&]() {
#pragma unroll
    for (int c = 0; c < kCh; ++c)
      if (BC != 512 || (c & 1) == 0) i_src[lane_slot(c)] = tile_row(i_tile, lane_row(c));
  };
  if (T > 0) load_rows();
  auto issue = [&]() {
    if (i_cnt < T) {
      unsigned char* st = ring + (size_t)(i_cnt & (kRing - 1)) * kSlot;
#pragma unroll
      for (int c = 0; c < kCh; ++c) {
        const int row = lane_row(c), piece = (32 * c + lane) % kPPR;
        const uint16_t* src = i_src[lane_slot(c)];
        if (src) cp_async16(st + row * kRowPitch + piece * 16, src + (size_t)i_kb * kBlockCols + piece * 8);
      }
      if (++i_kb == nkb) {
        i_kb = 0;
        ++i_tile;
        if (i_cnt + 1 < T) load_rows();
      }
    }
    ++i_cnt;
    cp_async_commit();  // one group per item, empty past the end, so counts stay aligned
  };
  static_assert((kRing & (kRing - 1)) == 0, "ring index uses a mask");
#pragma unroll
  for (int i = 0; i < kRing - 1; ++i) issue();

  pdl_wait();
  pdl_trigger();
  if (p.skip && *p.skip) {
    cp_async_wait<0>();
    return;
  }

  // ---- activations
  if (XM == kXBf16) stage_bf16_rows<NT>(p.xb, K, R, xs, xp);
  else stage_rmsnorm_rows<NT>(p.xf, p.gamma, K, R, p.eps, xs, xp, red_norm);
  __syncthreads();

  // output of (activation row r, tile row j) of `tile` with value v (SwiGLU: gate v, up u)
  auto emit = [&](int tile, int r, int j, float v, float u) {
    const int n = u0 + tile * TU + j;
    if (r >= R || n >= u1) return;
    const int sg = (n >= p.seg_start[2]) ? 2 : (n >= p.seg_start[1]) ? 1 : 0;
    const int col = p.col0[sg] + (n - p.seg_start[sg]);
    if (EPI == kEpiSwiGLU) {
      const float gt = round_bf16(v);
      const float a = round_bf16(gt / (1.0f + det_expf(-gt)));
      p.ob[(size_t)r * p.ldo + col] = f2bf_round(a * round_bf16(u));
    } else if (EPI == kEpiBf16) {
      p.ob[(size_t)r * p.ldo + col] = f2bf_round(v);
    } else if (EPI == kEpiResidual) {
      float* xr = p.of + (size_t)r * p.ldo + col;
      *xr = round_bf16(*xr + round_bf16(v));
    } else if (EPI == kEpiLogits) {
      p.of[(size_t)r * p.ldo + col] = round_bf16(v);
    } else {
      p.of[(size_t)r * p.ldo + col] = v;
    }
  };

  // fragment rows g and g + 8 carry activation rows g and g + 8 (R <= 16)
  const bool has_x0 = g < R, has_x1 = g + 8 < R;
  const unsigned char* xrow = xs + (size_t)g * xp + t4 * 16;
  constexpr int kAcc = 4;
  float acc[kAcc][4];
#pragma unroll
  for (int a = 0; a < kAcc; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
  int c_tile = ia / nkb, c_kb = ia % nkb;
  const int first_tile = c_tile;
  int run_kb0 = c_kb;  // first block of the current tile covered by this warp
  for (int it = 0; it < T; ++it) {
    cp_async_wait<kRing - 2>();  // this lane's copies of item `it` have landed
    __syncwarp();                // ... and every other lane's (also: all reads of item it-1 are done)
    const unsigned char* st = ring + (size_t)(it & (kRing - 1)) * kSlot + g * kRowPitch + t4 * 16;
    const unsigned char* xk = xrow + (size_t)c_kb * kBlockCols * 2;
#pragma unroll
    for (int u = 0; u < kCh; ++u) {
      const uint4 w = *reinterpret_cast<const uint4*>(st + u * 64);
      uint4 x = make_uint4(0u, 0u, 0u, 0u), y = make_uint4(0u, 0u, 0u, 0u);
      if (has_x0) x = *reinterpret_cast<const uint4*>(xk + u * 64);
      if (has_x1) y = *reinterpret_cast<const uint4*>(xk + 8 * xp + u * 64);
      mma_bf16_16816(acc[u % kAcc], x.x, y.x, x.y, y.y, w.x, w.y);
      mma_bf16_16816(acc[u % kAcc], x.z, y.z, x.w, y.w, w.z, w.w);
    }
    issue();  // refills the slot item it-1 used
    const bool tile_end = c_kb == nkb - 1;
    if (tile_end || it == T - 1) {
      float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
      for (int a = 0; a < kAcc; ++a) {
        c0 += acc[a][0];
        c1 += acc[a][1];
        c2 += acc[a][2];
        c3 += acc[a][3];
        acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
      }
      if (run_kb0 == 0 && tile_end) {
        // the whole tile is this warp's: lane (g, t) holds tile rows 2t and 2t+1 of
        // activations g (c0, c1) and g + 8 (c2, c3)
        if (PAIR) {  // gate rows 0..3 sit in lanes t < 2, up rows 4..7 in lanes t + 2
          const float u0v = __shfl_down_sync(0xffffffffu, c0, 2);
          const float u1v = __shfl_down_sync(0xffffffffu, c1, 2);
          const float u2v = __shfl_down_sync(0xffffffffu, c2, 2);
          const float u3v = __shfl_down_sync(0xffffffffu, c3, 2);
          if (t4 < 2) {
            emit(c_tile, g, 2 * t4, c0, u0v);
            emit(c_tile, g, 2 * t4 + 1, c1, u1v);
            emit(c_tile, g + 8, 2 * t4, c2, u2v);
            emit(c_tile, g + 8, 2 * t4 + 1, c3, u3v);
          }
        } else {
          emit(c_tile, g, 2 * t4, c0, 0.f);
          emit(c_tile, g, 2 * t4 + 1, c1, 0.f);
          emit(c_tile, g + 8, 2 * t4, c2, 0.f);
          emit(c_tile, g + 8, 2 * t4 + 1, c3, 0.f);
        }
      } else {
        pieces[(warp * 2 + (c_tile == first_tile ? 0 : 1)) * 32 + lane] = make_float4(c0, c1, c2, c3);
      }
    }
    if (++c_kb == nkb) {
      c_kb = 0;
      ++c_tile;
      run_kb0 = 0;
    }
  }
  // ---- tiles split between warps (a warp boundary strictly inside): add the pieces in warp
  // order, one thread per output element of every such tile
  if (tid == 0) {
    int n = 0;
    for (int b = 1; b < W; ++b) {
      const int cut = share(b);
      if (cut >= items || cut % nkb == 0) continue;
      if (n == 0 || s_cut[n - 1] != cut / nkb) s_cut[n++] = cut / nkb;
    }
    s_ncut = n;
  }
  cp_async_wait<0>();
  __syncthreads();
  const int per = R * TU;
  for (int f = tid; f < s_ncut * per; f += NT) {
    const int tile = s_cut[f / per], e = f % per, r = e / TU, j = e % TU;
    const int lo = tile * nkb, hi = lo + nkb;
    float v = 0.f, u = 0.f;
    for (int w = 0; w < W; ++w) {
      const int a0 = share(w), a1 = share(w + 1);
      if (a0 >= a1 || a0 >= hi || a1 <= lo) continue;
      const float4* pw = pieces + (w * 2 + (a0 / nkb == tile ? 0 : 1)) * 32;
      // element (activation r, tile row q) sits in lane 4(r % 8) + q/2, component
      // (q & 1) of (x, y) for r < 8 and of (z, w) for r >= 8
      auto at = [&](int q) {
        const float4 el = pw[4 * (r & 7) + (q >> 1)];
        return r < 8 ? ((q & 1) ? el.y : el.x) : ((q & 1) ? el.w : el.z);
      };
      v += at(j);
      if (PAIR) u += at(j + 4);
    }
    emit(tile, r, j, v, u);
  }
}

// ------------------------------------------------------------------ launcher
static int sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

static cudaError_t set_smem_once(const void* fn) {
  static std::mutex mu;
  static unsigned long long done[64][64] = {{0}};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& f : done[dev])
    if (f == (unsigned long long)fn) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcMaxSmem);
  if (e != cudaSuccess) return e;
  for (auto& f : done[dev])
    if (!f) {
      f = (unsigned long long)fn;
      break;
    }
  return cudaSuccess;
}

// Path choice: the SIMT kernel for R <= 2 (one song with CFG: measured faster in the
// chained decode step, where its two CTAs per SM overlap the neighbouring launches), the
// tensor-core kernel for R > 2 (prefill chunks, batched songs), where the SIMT kernel is
// instruction bound. Within a path a row's result does not depend on the other rows.
// YUE2_CUDA_GEMV=tc or =simt forces one path for every shape (measurements).
static int gemv_tc_mode() {
  static const int mode = [] {
    const char* v = getenv("YUE2_CUDA_GEMV");
    if (v && strcmp(v, "simt") == 0) return 0;
    if (v && strcmp(v, "tc") == 0) return 2;
    return 1;
  }();
  return mode;
}

// Launch shapes (warps, block columns, ring depth, CTAs per SM), in order of preference.
struct TcShape {
  int warps, bc, ring, per_sm;
};
constexpr TcShape kShapes[] = {{8, 256, 4, 1}, {8, 128, 8, 1}, {8, 128, 4, 1}, {8, 128, 4, 2}, {4, 256, 4, 2},
                               {4, 128, 8, 2}};
constexpr int kNumShapes = sizeof(kShapes) / sizeof(kShapes[0]);

static size_t tc_smem(const TcShape& sh, const GemvParams& p) {
  return (size_t)ring_bytes(sh.warps, sh.bc, sh.ring) + (size_t)p.R * x_pitch(p.K) + piece_bytes(sh.warps);
}
static bool tc_fits(const TcShape& sh, const GemvParams& p) {
  return p.K % sh.bc == 0 && tc_smem(sh, p) <= (size_t)kTcMaxSmem;
}

// The preferred shape that fits (-1: none). YUE2_CUDA_GEMV_SHAPE=i moves shape i to the
// front, for measurements.
static int tc_shape(const GemvParams& p) {
  static const int first = [] {
    const char* v = getenv("YUE2_CUDA_GEMV_SHAPE");
    const int i = v ? atoi(v) : 0;
    return (i >= 0 && i < kNumShapes) ? i : 0;
  }();
  if (tc_fits(kShapes[first], p)) return first;
  for (int i = 0; i < kNumShapes; ++i)
    if (tc_fits(kShapes[i], p)) return i;
  return -1;
}

bool gemv_tc_eligible(int xmode, int epi, const GemvParams& p) {
  const int mode = gemv_tc_mode();
  if (mode == 0 || (mode == 1 && p.R <= 2)) return false;
  if (xmode != kXBf16 && xmode != kXNorm) return false;
  if (epi == kEpiRawF32) return false;
  if (p.R < 1 || p.R > 16 || p.K < 128 || (p.K % 128) || p.N < 1) return false;
  for (int s = 0; s < 3; ++s)
    if (((uintptr_t)p.w[s]) & 15) return false;
  if (((uintptr_t)p.wpair) & 15) return false;
  return tc_shape(p) >= 0;
}

template <int SH, bool PAIR, int XM, int EPI>
static cudaError_t tc_go(cudaStream_t s, bool pdl, const GemvParams& p, bool configure_only) {
  constexpr TcShape sh = kShapes[SH];
  const void* fn = (const void*)gemv_tc_kernel<sh.warps, sh.bc, sh.ring, PAIR, XM, EPI>;
  cudaError_t e = set_smem_once(fn);
  if (e != cudaSuccess || configure_only) return e;
  const int sms = sm_count();
  if (sms <= 0) return cudaErrorInvalidDevice;
  const int want = sms * sh.per_sm;
  const int grid = p.N < want ? p.N : want;
  GemvParams copy = p;
  void* args[] = {&copy};
  return launch_with(s, pdl, dim3(grid), dim3(sh.warps * 32), tc_smem(sh, p), fn, args);
}

template <bool PAIR, int XM, int EPI>
static cudaError_t tc_warps_go(cudaStream_t s, bool pdl, const GemvParams& p, bool configure_only) {
  const int sh = configure_only ? -2 : tc_shape(p);
  cudaError_t e = cudaSuccess;
  if (sh == 0 || sh == -2) e = tc_go<0, PAIR, XM, EPI>(s, pdl, p, configure_only);
  if (e == cudaSuccess && (sh == 1 || sh == -2)) e = tc_go<1, PAIR, XM, EPI>(s, pdl, p, configure_only);
  if (e == cudaSuccess && (sh == 2 || sh == -2)) e = tc_go<2, PAIR, XM, EPI>(s, pdl, p, configure_only);
  if (e == cudaSuccess && (sh == 3 || sh == -2)) e = tc_go<3, PAIR, XM, EPI>(s, pdl, p, configure_only);
  if (e == cudaSuccess && (sh == 4 || sh == -2)) e = tc_go<4, PAIR, XM, EPI>(s, pdl, p, configure_only);
  if (e == cudaSuccess && (sh == 5 || sh == -2)) e = tc_go<5, PAIR, XM, EPI>(s, pdl, p, configure_only);
  return sh == -1 ? cudaErrorInvalidValue : e;
}

cudaError_t launch_gemv_tc(cudaStream_t s, bool pdl, int xmode, int epi, const GemvParams& p,
                           bool configure_only) {
  switch (epi) {
    case kEpiBf16:
      if (xmode == kXNorm) return tc_warps_go<false, kXNorm, kEpiBf16>(s, pdl, p, configure_only);
      break;
    case kEpiResidual:
      if (xmode == kXBf16) return tc_warps_go<false, kXBf16, kEpiResidual>(s, pdl, p, configure_only);
      break;
    case kEpiSwiGLU:
      if (xmode == kXNorm) return tc_warps_go<true, kXNorm, kEpiSwiGLU>(s, pdl, p, configure_only);
      break;
    case kEpiLogits:
      if (xmode == kXNorm) return tc_warps_go<false, kXNorm, kEpiLogits>(s, pdl, p, configure_only);
      if (xmode == kXBf16) return tc_warps_go<false, kXBf16, kEpiLogits>(s, pdl, p, configure_only);
      break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace y2
