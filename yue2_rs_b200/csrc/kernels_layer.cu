// Per-layer decode kernels for sm_100a.
//
// Reference math (twally3/yue2_rs): Model::hidden decode branch (src/model.rs:523-591),
// Norm::apply/heads (src/tensor.rs:1140-1172), Rotary (src/model.rs:137-168),
// Linear::finish rounding (src/tensor.rs:1102-1118), Mlp::apply (src/model.rs:206-214),
// decode attention (src/model.rs:314-397, src/attention.metal:206-317).
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "attention.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tp.cuh"

namespace y2 {

// ------------------------------------------------------------------ embed
// x[r] = bf16(E[token_r]) (Model::embed, model.rs:452-464). The token of a row is the
// prompt id of its position inside [prompt_begin, prompt_end), else row.token.
__global__ void embed_kernel(DevRow* rows, int R, const uint16_t* __restrict__ embed, int hidden, int vocab,
                             float* __restrict__ x, int32_t* error) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  if (r >= R) return;
  DevRow& row = rows[r];
  int tok = (row.pos >= row.prompt_begin && row.pos < row.prompt_end) ? row.prompt[row.pos - row.prompt_begin]
                                                                      : row.token;
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicExch(error, 1);
    tok = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) row.token = tok;
  const uint16_t* src = embed + (size_t)tok * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) x[(size_t)r * hidden + i] = bf2f(src[i]);
}

// When set, the launchers below only configure their kernel (no launch).
static thread_local bool g_configure_only = false;

// Opt a kernel into more than 48 KB of dynamic shared memory, once per device.
static cudaError_t ensure_smem_attr(const void* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({fn, dev});
  return e;
}

cudaError_t launch_with(cudaStream_t s, bool pdl, dim3 grid, dim3 block, size_t smem, const void* fn,
                        void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_embed(cudaStream_t s, bool pdl, DevRow* rows, int R, const uint16_t* embed, int hidden,
                         int vocab, float* x, int32_t* error) {
  void* args[] = {&rows, &R, &embed, &hidden, &vocab, &x, &error};
  return launch_with(s, pdl, dim3(R), dim3(256), 0, (const void*)embed_kernel, args);
}

// ------------------------------------------------------------------ GEMV
template <int XM>
struct XTraits;
template <>
struct XTraits<kXBf16> {
  static constexpr int bytes = 2;
};
template <>
struct XTraits<kXNorm> {
  static constexpr int bytes = 2;
};
template <>
struct XTraits<kXF32> {
  static constexpr int bytes = 4;
};

Y2_DEV float dot8_f32(uint4 w, const float4& a, const float4& b, float acc) {
  acc = fmaf(bf_lo(w.x), a.x, acc);
  acc = fmaf(bf_hi(w.x), a.y, acc);
  acc = fmaf(bf_lo(w.y), a.z, acc);
  acc = fmaf(bf_hi(w.y), a.w, acc);
  acc = fmaf(bf_lo(w.z), b.x, acc);
  acc = fmaf(bf_hi(w.z), b.y, acc);
  acc = fmaf(bf_lo(w.w), b.z, acc);
  acc = fmaf(bf_hi(w.w), b.w, acc);
  return acc;
}


// Weight stream: every thread owns 16-byte chunks of its warp's current row and copies
// them with cp.async.cg (L2 only) into its own slots of a kStages-deep shared-memory
// ring, kStages-1 batches ahead of the batch it multiplies. A thread reads back only
// what it copied itself, so the hardware cp.async.wait_group is the only wait (no
// barrier, no spin). The first kStages-1 batches are requested before
// griddepcontrol.wait: they stream while the previous kernel drains.
constexpr int kGemvThreads = 256;
constexpr int kStages = 4;

template <int RM, bool PAIR, int XM, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  constexpr int NP = PAIR ? 2 : 1;
  constexpr int CH = PAIR ? 2 : 4;  // chunks per lane per batch and matrix
  constexpr int NT = kGemvThreads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = NT / 32;
  const int K = p.K, K8 = K >> 3;
  const int nb = (K8 + 32 * CH - 1) / (32 * CH);
  const int row_begin = (int)(((long long)p.N * blockIdx.x) / gridDim.x);
  const int row_end = (int)(((long long)p.N * (blockIdx.x + 1)) / gridDim.x);
  // The CTA's (row, batch) items are split into equal contiguous shares, one per warp, so
  // no warp idles while another finishes a row.
  const int items = (row_end - row_begin) * nb;
  const int ia = (int)(((long long)items * warp) / nwarps);
  const int T = (int)(((long long)items * (warp + 1)) / nwarps) - ia;
  uint4* ring = reinterpret_cast<uint4*>(smem_raw);  // [kStages][NP][CH][NT]
  unsigned char* xbase = smem_raw + (size_t)kStages * NP * CH * NT * 16;
  float* slots = reinterpret_cast<float*>(xbase + (size_t)RM * K * XTraits<XM>::bytes);  // [rows][nb][NP][RM]

  auto wrow = [&](int n) -> const uint16_t* {
    const int s = (n >= p.seg_start[2]) ? 2 : (n >= p.seg_start[1]) ? 1 : 0;
    return p.w[s] + (size_t)(n - p.seg_start[s]) * K;
  };
  // issue stream: (row, batch) of the next batch to request, advanced incrementally
  int i_cnt = 0, i_b = ia % nb, i_row = row_begin + ia / nb;
  const uint16_t* i_w0 = T > 0 ? wrow(i_row) : nullptr;
  const uint16_t* i_w1 = (PAIR && T > 0) ? p.wpair + (size_t)i_row * K : nullptr;
  auto issue = [&]() {
    if (i_cnt < T) {
      uint4* st = ring + (size_t)(i_cnt & (kStages - 1)) * NP * CH * NT + tid;
      const int base = i_b * CH * 32 + lane;
      if ((i_b + 1) * CH * 32 <= K8) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          cp_async16(st + c * NT, i_w0 + (size_t)(base + c * 32) * 8);
          if (PAIR) cp_async16(st + (CH + c) * NT, i_w1 + (size_t)(base + c * 32) * 8);
        }
      } else {
#pragma unroll
        for (int c = 0; c < CH; ++c)
          if (base + c * 32 < K8) {
            cp_async16(st + c * NT, i_w0 + (size_t)(base + c * 32) * 8);
            if (PAIR) cp_async16(st + (CH + c) * NT, i_w1 + (size_t)(base + c * 32) * 8);
          }
      }
      if (++i_b == nb) {
        i_b = 0;
        ++i_row;
        if (i_cnt + 1 < T) {
          i_w0 = wrow(i_row);
          if (PAIR) i_w1 = p.wpair + (size_t)i_row * K;
        }
      }
    }
    ++i_cnt;
    cp_async_commit();  // one group per batch, empty past the end, so counts stay aligned
  };
  static_assert((kStages & (kStages - 1)) == 0, "ring index uses a mask");

#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) issue();

  pdl_wait();
  pdl_trigger();
  if (p.skip && *p.skip) {
    cp_async_wait<0>();
    return;
  }
  // kEpiResidual, kEpiTpReduce: the residual values this thread's epilogue updates, requested
  // now so that their round trip overlaps the staging and the stream (only this CTA writes them)
  constexpr int kPreRes = 2;
  float res_pre[kPreRes];
  if (EPI == kEpiResidual || EPI == kEpiTpReduce) {
#pragma unroll
    for (int k = 0; k < kPreRes; ++k) {
      const int i = tid + k * NT;
      if (i < (row_end - row_begin) * RM && i % RM < p.R) {
        const int n = row_begin + i / RM;
        const int sg = (n >= p.seg_start[2]) ? 2 : (n >= p.seg_start[1]) ? 1 : 0;
        res_pre[k] = p.of[(size_t)(i % RM) * p.ldo + p.col0[sg] + (n - p.seg_start[sg])];
      }
    }
  }

  // ---- stage activations
  if (XM == kXF32) {
    float* xs = reinterpret_cast<float*>(xbase);
    for (int i = tid; i < RM * K; i += NT) {
      const int r = i / K;
      xs[i] = r < p.R ? p.xf[i] : 0.f;
    }
  } else {
    // rows past R are zero (the dot loops read all RM rows)
    uint4* xz = reinterpret_cast<uint4*>(xbase) + (size_t)p.R * K8;
    for (int i = tid; i < (RM - p.R) * K8; i += NT) xz[i] = make_uint4(0, 0, 0, 0);
    if (XM == kXBf16) stage_bf16_rows<NT>(p.xb, K, p.R, xbase, (size_t)K * 2);
    else  // kXNorm: RMSNorm of the f32 residual (Norm::apply)
      stage_rmsnorm_rows<NT, false, (RM < 4 ? RM : 4)>(p.xf, p.gamma, K, p.R, p.eps, xbase, (size_t)K * 2, red);
  }
  const int nrows = row_end - row_begin;
  for (int i = tid; i < nrows * nb * NP * RM; i += NT) slots[i] = 0.f;
  __syncthreads();

  float acc[NP][RM];
#pragma unroll
  for (int q = 0; q < NP; ++q)
#pragma unroll
    for (int r = 0; r < RM; ++r) acc[q][r] = 0.f;

  // Lane sums stay in registers while the warp's items stay on one row; at a row boundary
  // the warp reduces them and lane 0 stores the partial in the slot of the first batch of
  // that row it covered. Slots are summed in batch order at the end (deterministic).
  auto flush = [&](int row_local, int b_first) {
#pragma unroll
    for (int q = 0; q < NP; ++q)
#pragma unroll
      for (int r = 0; r < RM; ++r) acc[q][r] = warp_sum(acc[q][r]);
    if (lane == 0) {
#pragma unroll
      for (int q = 0; q < NP; ++q)
#pragma unroll
        for (int r = 0; r < RM; ++r) slots[((row_local * nb + b_first) * NP + q) * RM + r] = acc[q][r];
    }
#pragma unroll
    for (int q = 0; q < NP; ++q)
#pragma unroll
      for (int r = 0; r < RM; ++r) acc[q][r] = 0.f;
  };

  // compute stream: row and batch of item t, advanced incrementally
  int c_row = ia / nb, c_b = ia % nb, c_b0 = c_b;
  auto dots = [&](const uint4* st, int base, bool guard) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int idx = base + c * 32;
      if (guard && idx >= K8) continue;
      uint4 w[NP];
#pragma unroll
      for (int q = 0; q < NP; ++q) w[q] = st[(q * CH + c) * NT];
#pragma unroll
      for (int r = 0; r < RM; ++r) {
        if (XM == kXF32) {
          const float4* xs = reinterpret_cast<const float4*>(xbase) + ((size_t)r * K8 + idx) * 2;
          const float4 a = xs[0], bb = xs[1];
#pragma unroll
          for (int q = 0; q < NP; ++q) acc[q][r] = dot8_f32(w[q], a, bb, acc[q][r]);
        } else {
          const uint4 xv = reinterpret_cast<const uint4*>(xbase)[(size_t)r * K8 + idx];
#pragma unroll
          for (int q = 0; q < NP; ++q) acc[q][r] = dot8_bf(w[q], xv, acc[q][r]);
        }
      }
    }
  };
  for (int t = 0; t < T; ++t) {
    cp_async_wait<kStages - 2>();  // this thread's batch t has landed
    const uint4* st = ring + (size_t)(t & (kStages - 1)) * NP * CH * NT + tid;
    const int base = c_b * CH * 32 + lane;
    if ((c_b + 1) * CH * 32 <= K8) dots(st, base, false);
    else dots(st, base, true);
    issue();  // refills the slot batch t-1 used
    if (++c_b == nb) {  // the row ends inside this warp's share
      flush(c_row, c_b0);
      c_b = 0;
      c_b0 = 0;
      ++c_row;
    }
  }
  if (T > 0 && c_b != 0) flush(c_row, c_b0);  // share ended inside a row
  cp_async_wait<0>();
  __syncthreads();

  if (EPI == kEpiTpReduce) {  // tensor parallel: exchange, sum in rank order, residual
    const TpPeers& P = *p.tp_peers;
    const uint32_t tag = (*p.tp_epoch) * 256u + (uint32_t)p.tp_site + 1u;
    const size_t half = (size_t)(p.tp_site & 1) * kTpMaxWorld * kTpRows * p.N;  // parity half (words)
    const size_t slot = (size_t)kTpRows * p.N;                                   // one rank's words
    for (int i = tid; i < nrows * RM; i += NT) {  // this CTA's partial sums to every rank
      const int row_local = i / RM, r = i % RM;
      if (r >= p.R) continue;
      float sum = 0.f;
      for (int b = 0; b < nb; ++b) sum += slots[(row_local * nb + b) * RM + r];
      const size_t at = half + (size_t)p.tp_rank * slot + (size_t)r * p.N + row_begin + row_local;
      for (int t = 0; t < p.tp_world; ++t) st_ll(P.recv[t] + at, sum, tag);
    }
    // every rank's sums of the same outputs (their CTA with this index computes the same rows)
    bool ok = true;
    const uint2* mine = P.recv[p.tp_rank] + half;
    for (int i = tid; i < nrows * RM; i += NT) {
      const int row_local = i / RM, r = i % RM;
      if (r >= p.R) continue;
      const int n = row_begin + row_local;
      float s = 0.f;
      for (int q = 0; q < p.tp_world; ++q) s += wait_ll(mine + (size_t)q * slot + (size_t)r * p.N + n, tag, p.error, ok);
      float* xr = p.of + (size_t)r * p.ldo + n;
      const int k = (i - tid) / NT;  // which of this thread's items (kPreRes == 2)
      const float xv = k == 0 ? res_pre[0] : k == 1 ? res_pre[1] : *xr;
      *xr = round_bf16(xv + round_bf16(s));
    }
    return;
  }

  // ---- epilogue: one thread per (row, activation row), rounding where Linear::finish does
  for (int i = tid; i < nrows * RM; i += NT) {
    const int row_local = i / RM, r = i % RM;
    if (r >= p.R) continue;
    float v[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      float sum = 0.f;
      for (int b = 0; b < nb; ++b) sum += slots[((row_local * nb + b) * NP + q) * RM + r];
      v[q] = sum;
    }
    const int n = row_begin + row_local;
    const int sg = (n >= p.seg_start[2]) ? 2 : (n >= p.seg_start[1]) ? 1 : 0;
    const int col = p.col0[sg] + (n - p.seg_start[sg]);
    if (EPI == kEpiBf16) {
      p.ob[(size_t)r * p.ldo + col] = f2bf_round(v[0]);
    } else if (EPI == kEpiResidual) {
      float* xr = p.of + (size_t)r * p.ldo + col;
      const int k = (i - tid) / NT;  // which of this thread's items (kPreRes == 2)
      const float xv = k == 0 ? res_pre[0] : k == 1 ? res_pre[1] : *xr;
      *xr = round_bf16(xv + round_bf16(v[0]));
    } else if (EPI == kEpiSwiGLU) {
      const float g = round_bf16(v[0]);
      const float u = round_bf16(v[NP - 1]);
      const float a = round_bf16(g / (1.0f + det_expf(-g)));
      p.ob[(size_t)r * p.ldo + col] = f2bf_round(a * u);
    } else if (EPI == kEpiLogits) {
      p.of[(size_t)r * p.ldo + col] = round_bf16(v[0]);
    } else {
      p.of[(size_t)r * p.ldo + col] = v[0];
    }
  }
}

size_t gemv_smem_bytes(int xmode, int K, int R) {
  const int rm = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
  return (size_t)kStages * 4 * kGemvThreads * 16 + (size_t)rm * K * (xmode == kXF32 ? 4 : 2);
}

constexpr int kMaxSmem = 227 * 1024 - 1024;  // opt-in limit minus room for static shared memory

template <int RM, bool PAIR, int XM, int EPI>
static cudaError_t gemv_go(cudaStream_t s, bool pdl, const GemvParams& p, int grid) {
  const void* fn = (const void*)gemv_kernel<RM, PAIR, XM, EPI>;
  constexpr int NP = PAIR ? 2 : 1, CH = PAIR ? 2 : 4;
  const size_t nb = ((size_t)p.K / 8 + 32 * CH - 1) / (32 * CH);
  const size_t rows_max = ((size_t)p.N + grid - 1) / grid + 1;
  const size_t smem = (size_t)kStages * 4 * kGemvThreads * 16 + (size_t)RM * p.K * XTraits<XM>::bytes +
                      rows_max * nb * NP * RM * 4;
  if (smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_attr(fn, kMaxSmem);
  if (e != cudaSuccess || g_configure_only) return e;
  GemvParams copy = p;
  void* args[] = {&copy};
  return launch_with(s, pdl, dim3(grid), dim3(kGemvThreads), smem, fn, args);
}

template <bool PAIR, int XM, int EPI>
static cudaError_t gemv_rows(cudaStream_t s, bool pdl, const GemvParams& p, int grid) {
  if (p.R <= 1) return gemv_go<1, PAIR, XM, EPI>(s, pdl, p, grid);
  if (p.R <= 2) return gemv_go<2, PAIR, XM, EPI>(s, pdl, p, grid);
  if (p.R <= 4) return gemv_go<4, PAIR, XM, EPI>(s, pdl, p, grid);
  return gemv_go<8, PAIR, XM, EPI>(s, pdl, p, grid);
}

static cudaError_t launch_gemv_simt(cudaStream_t s, bool pdl, int xmode, int epi, const GemvParams& p, int grid) {
  if (p.R > 8) return cudaErrorInvalidValue;
  switch (epi) {
    case kEpiBf16:
      if (xmode == kXNorm) return gemv_rows<false, kXNorm, kEpiBf16>(s, pdl, p, grid);
      break;
    case kEpiResidual:
      if (xmode == kXBf16) return gemv_rows<false, kXBf16, kEpiResidual>(s, pdl, p, grid);
      break;
    case kEpiSwiGLU:
      if (xmode == kXNorm) return gemv_rows<true, kXNorm, kEpiSwiGLU>(s, pdl, p, grid);
      break;
    case kEpiLogits:
      if (xmode == kXNorm) return gemv_rows<false, kXNorm, kEpiLogits>(s, pdl, p, grid);
      if (xmode == kXBf16) return gemv_rows<false, kXBf16, kEpiLogits>(s, pdl, p, grid);
      break;
    case kEpiRawF32:
      if (xmode == kXF32 && p.R == 1) return gemv_go<1, false, kXF32, kEpiRawF32>(s, pdl, p, grid);
      if (xmode == kXBf16 && p.R <= 2) return gemv_rows<false, kXBf16, kEpiRawF32>(s, pdl, p, grid);
      break;
    case kEpiTpReduce:
      if (xmode == kXBf16 && p.R <= kTpRows &&
          (g_configure_only || (p.tp_peers && p.tp_epoch && p.tp_world >= 1 && p.tp_world <= kTpMaxWorld)))
        return gemv_rows<false, kXBf16, kEpiTpReduce>(s, pdl, p, grid);
      break;
  }
  return cudaErrorInvalidValue;
}

// gemv_tc_eligible decides the path (tensor-core kernel: bf16 activations, K % 128 == 0,
// R <= 16, chosen for R > 2; SIMT kernel: R <= 8, the f32 drop-in input, odd K).
// Configuration passes set up both, so either can be chosen at launch time.
cudaError_t launch_gemv(cudaStream_t s, bool pdl, int xmode, int epi, const GemvParams& p, int grid) {
  if (p.R < 1 || p.R > kMaxRows || (p.K & 7) || p.N < 1) return cudaErrorInvalidValue;
  const bool tc = gemv_tc_eligible(xmode, epi, p);
  if (p.R > 8 && !tc && !g_configure_only) {
    // more rows than one pass holds activations for (e.g. 16 rows of an 8,192-column
    // matrix): two passes over the weights, rows [0, 8) and [8, R)
    GemvParams a = p, b = p;
    a.R = 8;
    b.R = p.R - 8;
    if (xmode == kXF32 || xmode == kXNorm) b.xf = p.xf + (size_t)8 * p.K;
    else b.xb = p.xb + (size_t)8 * p.K;
    if (p.ob) b.ob = p.ob + (size_t)8 * p.ldo;
    if (p.of) b.of = p.of + (size_t)8 * p.ldo;
    cudaError_t e = launch_gemv(s, pdl, xmode, epi, a, grid);
    return e == cudaSuccess ? launch_gemv(s, pdl, xmode, epi, b, grid) : e;
  }
  if (g_configure_only) {
    cudaError_t e = launch_gemv_simt(s, pdl, xmode, epi, p, grid);
    if (e == cudaSuccess && tc) e = launch_gemv_tc(s, pdl, xmode, epi, p, true);
    return e;
  }
  if (tc) return launch_gemv_tc(s, pdl, xmode, epi, p, false);
  return launch_gemv_simt(s, pdl, xmode, epi, p, grid);
}

// ------------------------------------------------------------------ QK norm + RoPE + KV append
// One warp per (head, row), kRopeWarps heads of one row per CTA: q heads are normalised
// (Norm::heads) and rotated, k heads normalised, rotated and written to the row's page at
// its position, v heads copied. Each lane stores D / 32 consecutive elements.
constexpr int kRopeWarps = 8;

template <int D>
__global__ void __launch_bounds__(32 * kRopeWarps) rope_append_kernel(const RopeParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int DL = D / 32;  // elements per lane: 2, 4 or 8
  __shared__ float vbuf[kRopeWarps][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hix = blockIdx.x * kRopeWarps + warp, r = blockIdx.y;
  const Geometry& g = p.g;
  if (hix >= g.heads + 2 * g.kvh) return;
  const DevRow row = p.rows[r];
  if (!row.active) return;
  const int pos = row.pos;
  if (pos < 0 || pos >= p.max_pos) {
    if (lane == 0) atomicExch(p.error, 1);
    return;
  }
  const int width = (g.heads + 2 * g.kvh) * D;
  const uint16_t* src = p.qkv + (size_t)r * width + (size_t)hix * D;
  uint16_t* page = reinterpret_cast<uint16_t*>(row.pages[pos >> kPageLog2]);
  const int slot = pos & (kPageTokens - 1);
  if (hix >= g.heads + g.kvh) {  // value head: already bf16 (Linear::finish)
    const int head = hix - g.heads - g.kvh;
    uint16_t* dst = page + kv_offset(g, p.layer, 1, head) + (size_t)slot * D;
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src + lane * DL);
    uint32_t* d32 = reinterpret_cast<uint32_t*>(dst + lane * DL);
#pragma unroll
    for (int e = 0; e < DL / 2; ++e) d32[e] = __ldcg(s32 + e);
    return;
  }
  float* v = vbuf[warp];
  const bool is_q = hix < g.heads;
  norm_rope_head<D>(src, is_q ? p.q_norm : p.k_norm, g.eps, p.cos_tab + (size_t)pos * (D / 2),
                    p.sin_tab + (size_t)pos * (D / 2), v);
  uint16_t* dst = is_q ? p.q_out + (size_t)r * g.heads * D + (size_t)hix * D
                       : page + kv_offset(g, p.layer, 0, hix - g.heads) + (size_t)slot * D;
  uint32_t* d32 = reinterpret_cast<uint32_t*>(dst + lane * DL);
#pragma unroll
  for (int e = 0; e < DL / 2; ++e)
    d32[e] = (uint32_t)f2bf_exact(v[lane * DL + 2 * e]) | ((uint32_t)f2bf_exact(v[lane * DL + 2 * e + 1]) << 16);
}

cudaError_t launch_rope_append(cudaStream_t s, bool pdl, const RopeParams& p, int R) {
  RopeParams copy = p;
  void* args[] = {&copy};
  dim3 grid((p.g.heads + 2 * p.g.kvh + kRopeWarps - 1) / kRopeWarps, R);
  const dim3 block(32 * kRopeWarps);
  switch (p.g.dim) {
    case 64: return launch_with(s, pdl, grid, block, 0, (const void*)rope_append_kernel<64>, args);
    case 128: return launch_with(s, pdl, grid, block, 0, (const void*)rope_append_kernel<128>, args);
    case 256: return launch_with(s, pdl, grid, block, 0, (const void*)rope_append_kernel<256>, args);
  }
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ decode attention
// The standalone launch of attn_item (attention.cuh): one CTA per (split, kv head, row).
template <int D, int G>
__global__ void __launch_bounds__(128) attn_kernel(const AttnParams a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  attn_item<D, G>(a, blockIdx.x, blockIdx.y, blockIdx.z, smem_raw);
}

// Passes of more than kMaxRows rows: the pipelined tile loop.
template <int D, int G>
__global__ void __launch_bounds__(128) attn_pipe_kernel(const AttnParams a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  attn_item<D, G, true>(a, blockIdx.x, blockIdx.y, blockIdx.z, smem_raw);
}

// The pipelined loop with scores and P.V on the tensor cores (dim <= 128).
template <int D, int G>
__global__ void __launch_bounds__(128) attn_mma_kernel(const AttnParams a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  attn_item<D, G, true, true>(a, blockIdx.x, blockIdx.y, blockIdx.z, smem_raw);
}


static int attention_smem_need(int dim, int groups, bool pipe = false, bool mma = false) {
  const int tiles = (pipe ? 3 : 2) * 4 * 32 * dim * 2;
  const int extra = (groups * dim + 4 * groups * 32 + 8 * groups + 4 * dim + 3 * dim) * 4 + (mma ? 16 * dim * 2 : 0);
  const int merge = 4 * groups * dim * 4;
  return (tiles > merge ? tiles : merge) + extra;
}

// The reservation of a one-wave launch is at least 77 KB, so that no SM holds more than two
// attention CTAs: the block scheduler would otherwise stack three on the SMs that free up
// first and leave others idle.
int attention_smem_bytes(int dim, int groups) {
  const int need = attention_smem_need(dim, groups);
  return need > 77 * 1024 ? need : 77 * 1024;
}

// The pipelined tile loop (96 KB at dim 128, two CTAs per SM): always for passes of more
// than kMaxRows rows, which launch many waves of CTAs streaming many tiles per warp;
// for the others when the caller asks (p.pipe: long contexts). YUE2_CUDA_ATTN_PIPE=1 / 0
// forces it on / off everywhere.
static int env_mode(const char* name) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : -1;
}
static int attn_pipe_mode() {
  static int mode = env_mode("YUE2_CUDA_ATTN_PIPE");
  return mode;
}
// Tensor-core scores and P.V (dim <= 128) wherever the pipelined loop runs;
// YUE2_CUDA_ATTN_MMA=0 keeps the SIMT loop there, =1 uses the tensor cores everywhere.
static int attn_mma_mode() {
  static int mode = env_mode("YUE2_CUDA_ATTN_MMA");
  return mode;
}

template <int D, int G>
static cudaError_t attn_go(cudaStream_t s, bool pdl, const AttnParams& p, int R) {
  const int mode = attn_pipe_mode(), mm = attn_mma_mode();
  const bool pipe = mode == 1 || (mode != 0 && (R > kMaxRows || p.pipe));
  const bool mma = D <= 128 && (mm == 1 || (mm != 0 && pipe));
  const void* fn = pipe ? (const void*)attn_pipe_kernel<D, G> : (const void*)attn_kernel<D, G>;
  int smem = pipe ? attention_smem_need(D, G, true) : attention_smem_bytes(D, G);
  if constexpr (D <= 128) {
    if (mma) {
      fn = (const void*)attn_mma_kernel<D, G>;
      smem = attention_smem_need(D, G, true, true);
    }
  }
  cudaError_t e = ensure_smem_attr(fn, smem);
  if (e != cudaSuccess || g_configure_only) return e;
  AttnParams copy = p;
  void* args[] = {&copy};
  return launch_with(s, pdl, dim3(p.splits, p.g.kvh, R), dim3(128), smem, fn, args);
}

template <int D, int G>
__global__ void __launch_bounds__(32 * kClusterWarps, 1) attn_cluster_kernel(const AttnParams a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  attn_cluster_item<D, G>(a, smem_raw);
}

template <int D, int G>
static cudaError_t attn_cluster_go(cudaStream_t s, bool pdl, const AttnParams& p, int R) {
  const void* fn = (const void*)attn_cluster_kernel<D, G>;
  constexpr int smem = attn_cluster_smem<D, G>();
  cudaError_t e = ensure_smem_attr(fn, smem);
  if (e != cudaSuccess || g_configure_only) return e;
  if (!p.fused || p.cluster < 1 || p.cluster > kClusterMax) return cudaErrorInvalidValue;
  AttnParams copy = p;
  void* args[] = {&copy};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.cluster, p.g.kvh, R);
  cfg.blockDim = dim3(32 * kClusterWarps);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;  // the CTAs of one (kv head, row)
  attr[0].val.clusterDim.x = (unsigned)p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

template <int D, int G>
static cudaError_t attn_dim_go(cudaStream_t s, bool pdl, const AttnParams& p, int R) {
  if constexpr (D <= 128) {
    if (p.cluster > 0 || g_configure_only) {
      cudaError_t e = attn_cluster_go<D, G>(s, pdl, p, R);
      if (e != cudaSuccess || !g_configure_only) return e;
    }
  }
  return attn_go<D, G>(s, pdl, p, R);
}

template <int D>
static cudaError_t attn_dim(cudaStream_t s, bool pdl, const AttnParams& p, int R) {
  switch (p.g.heads / p.g.kvh) {
    case 1: return attn_dim_go<D, 1>(s, pdl, p, R);
    case 2: return attn_dim_go<D, 2>(s, pdl, p, R);
    case 3: return attn_dim_go<D, 3>(s, pdl, p, R);
    case 4: return attn_dim_go<D, 4>(s, pdl, p, R);
    case 8: return attn_dim_go<D, 8>(s, pdl, p, R);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_attention(cudaStream_t s, bool pdl, const AttnParams& p, int R) {
  switch (p.g.dim) {
    case 64: return attn_dim<64>(s, pdl, p, R);
    case 128: return attn_dim<128>(s, pdl, p, R);
    case 256: return attn_dim<256>(s, pdl, p, R);
  }
  return cudaErrorInvalidValue;
}

// Sets the shared-memory attribute of every GEMV and attention instantiation on the
// current device, so that no attribute call happens while a CUDA graph is captured.
cudaError_t prepare_kernels() {
  g_configure_only = true;
  cudaError_t e = cudaSuccess;
  const int pairs[][2] = {{kXNorm, kEpiBf16}, {kXBf16, kEpiResidual}, {kXNorm, kEpiSwiGLU},
                          {kXNorm, kEpiLogits}, {kXBf16, kEpiLogits}, {kXF32, kEpiRawF32},
                          {kXBf16, kEpiRawF32}, {kXBf16, kEpiTpReduce}};
  for (auto& pr : pairs)
    for (int K : {2048, 1536, 1024})
      for (int R : {1, 2, 4, 8}) {
        GemvParams p = {};
        p.K = K;
        p.N = 1;
        p.R = pr[0] == kXF32 ? 1 : (pr[1] == kEpiRawF32 || pr[1] == kEpiTpReduce) ? std::min(R, 2) : R;
        if (e == cudaSuccess) e = launch_gemv(nullptr, false, pr[0], pr[1], p, 1);
      }
  for (int D : {64, 128, 256})
    for (int G : {1, 2, 3, 4, 8}) {
      AttnParams a = {};
      a.g.dim = D;
      a.g.kvh = 1;
      a.g.heads = G;
      if (e == cudaSuccess) e = launch_attention(nullptr, false, a, 1);
      if (e == cudaSuccess) e = launch_attention(nullptr, false, a, kMaxRows + 1);  // pipelined form
    }
  g_configure_only = false;
  return e;
}

// ------------------------------------------------------------------ step bookkeeping
__global__ void step_end_kernel(DevRow* rows, int R) {
  pdl_wait();
  pdl_trigger();
  const int r = threadIdx.x;
  if (r < R && rows[r].active) rows[r].pos += rows[r].advance;
}

cudaError_t launch_step_end(cudaStream_t s, bool pdl, DevRow* rows, int R) {
  if (R < 1 || R > 1024) return cudaErrorInvalidValue;
  void* args[] = {&rows, &R};
  return launch_with(s, pdl, dim3(1), dim3((R + 31) / 32 * 32), 0, (const void*)step_end_kernel, args);
}

// ------------------------------------------------------------------ synthetic data
Y2_DEV uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
Y2_DEV float normal_at(uint64_t seed, uint64_t i) {
  const uint64_t z = mix64(seed + (i >> 1) * 0x9E3779B97F4A7C15ull);
  const float u1 = ((uint32_t)(z >> 40) + 1) * (1.0f / 16777217.0f);
  const float u2 = (uint32_t)(z & 0xffffff) * (1.0f / 16777216.0f);
  const float rad = sqrtf(-2.0f * logf(u1));
  return (i & 1) ? rad * sinf(6.2831853071795865f * u2) : rad * cosf(6.2831853071795865f * u2);
}

__global__ void fill_normal_kernel(uint16_t* dst, size_t count, uint64_t seed, float mean, float stddev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = f2bf_round(mean + stddev * normal_at(seed, i));
}

cudaError_t launch_fill_normal_bf16(cudaStream_t s, uint16_t* dst, size_t count, uint64_t seed, float mean,
                                    float stddev) {
  fill_normal_kernel<<<1184, 256, 0, s>>>(dst, count, seed, mean, stddev);
  return cudaGetLastError();
}

// The rows x cols block at (row0, col0) of a full [*, full_cols] tensor filled as
// fill_normal_kernel fills the whole tensor (a tensor-parallel shard of it).
__global__ void fill_normal_shard_kernel(uint16_t* dst, size_t rows, size_t cols, size_t full_cols, size_t row0,
                                         size_t col0, uint64_t seed, float stddev) {
  const size_t count = rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const size_t flat = (row0 + i / cols) * full_cols + col0 + i % cols;
    dst[i] = f2bf_round(stddev * normal_at(seed, flat));
  }
}

cudaError_t launch_fill_normal_shard(cudaStream_t s, uint16_t* dst, size_t rows, size_t cols, size_t full_cols,
                                     size_t row0, size_t col0, uint64_t seed, float stddev) {
  fill_normal_shard_kernel<<<1184, 256, 0, s>>>(dst, rows, cols, full_cols, row0, col0, seed, stddev);
  return cudaGetLastError();
}

__global__ void fill_f32_kernel(float* dst, size_t count, float value) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = value;
}

cudaError_t launch_fill_f32(cudaStream_t s, float* dst, size_t count, float value) {
  fill_f32_kernel<<<592, 256, 0, s>>>(dst, count, value);
  return cudaGetLastError();
}

// Seeded N(0,1) bf16 keys/values for positions [from, to) of every layer. The values depend
// on the KV head's index among all `full_kvh` heads (head0 + local head), so that a
// tensor-parallel rank holds exactly its heads' share of the unsharded fill.
__global__ void kv_fill_kernel(const uint64_t* pages, Geometry g, int from, int to, uint64_t seed, int head0,
                               int full_kvh) {
  const size_t per_tok = (size_t)g.layers * 2 * g.kvh * g.dim;
  const size_t total = per_tok * (size_t)(to - from);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int tok = from + (int)(i / per_tok);
    size_t rem = i % per_tok;
    const int d = (int)(rem % g.dim);
    rem /= g.dim;
    const int head = (int)(rem % g.kvh);
    rem /= g.kvh;
    const int kv = (int)(rem % 2);
    const int layer = (int)(rem / 2);
    uint16_t* page = reinterpret_cast<uint16_t*>(pages[tok >> kPageLog2]);
    const uint64_t flat =
        (((uint64_t)layer * 2 + kv) * full_kvh + head0 + head) * 1048576ull * 64 + (uint64_t)tok * g.dim + d;
    page[kv_offset(g, layer, kv, head) + (size_t)(tok & (kPageTokens - 1)) * g.dim + d] =
        f2bf_round(normal_at(seed, flat));
  }
}

cudaError_t launch_kv_fill(cudaStream_t s, const uint64_t* pages, const Geometry& g, int from, int to,
                           uint64_t seed, int head0, int full_kvh) {
  if (to <= from) return cudaSuccess;
  kv_fill_kernel<<<1184, 256, 0, s>>>(pages, g, from, to, seed, head0, full_kvh);
  return cudaGetLastError();
}

}  // namespace y2
