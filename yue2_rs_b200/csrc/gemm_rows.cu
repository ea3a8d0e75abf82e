// Forward passes over many rows as tensor-core GEMMs: prompt prefill chunks
// (Model::prefill_phase, src/model.rs:508-522) and decode steps of more than kMaxRows rows
// (many songs per GPU; Model::hidden's decode branch, src/model.rs:523-591, per row).
//
// A prompt of n >= kPrefillGemmMin ids is cut into equal chunks of at most
// m.prefill_chunk (<= kPrefillRows) consecutive positions of one cache. Each chunk goes
// through the layers with every projection as one bf16 GEMM over all of its rows
// (cuBLASLt, f32 accumulation, bf16 output: Linear::finish's rounding,
// src/tensor.rs:1102-1118), and small kernels for the rest:
//   residual_norm_kernel   x = bf16(x + y) (src/tensor.rs:632-640), then Norm::apply
//                          (src/tensor.rs:1140-1157) of the row into bf16
//   swiglu_kernel          Mlp::apply's pointwise part (src/model.rs:206-214)
//   rope_append_kernel     per-head QK norm + RoPE, K/V written to the cache pages
//   prefill_attn_kernel    causal attention of the chunk's rows over the paged cache on
//                          the tensor cores (kernels_prefill_attn.cu); head sizes it does
//                          not take (and YUE2_CUDA_PREFILL_ATTN=rows) use attn_kernel per row
// The last row's hidden state goes through the LM head GEMV when logits are wanted.
//
// A wide decode step runs the same layer sequence over R rows of distinct caches, with
// the decode attention kernel (QK norm, RoPE and the KV append fused in, one query per
// row), then the final norm and the LM head as one more GEMM (bf16 logits widened to f32).
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <array>
#include <map>
#include <new>
#include <string>

#include "common.cuh"
#include "engine.h"
#include "kernels.h"

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return y2::cuda_fail(e_, #expr); \
  } while (0)

namespace y2 {

// ------------------------------------------------------------------ kernels
__global__ void prefill_rows_kernel(DevRow* rows, int C, const uint64_t* pages, const int32_t* prompt,
                                    int32_t prompt_begin, int32_t prompt_end, int32_t pos0) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= C) return;
  DevRow r = {};
  r.pages = pages;
  r.prompt = prompt;
  r.prompt_begin = prompt_begin;
  r.prompt_end = prompt_end;
  r.pos = pos0 + i;
  r.active = 1;
  r.advance = 0;
  rows[i] = r;
}

// One row per CTA. y != nullptr: x = bf16(x + y) with y the bf16 output of the o or down
// projection. gamma != nullptr: out = bf16(bf16(x * s) * gamma), s = bf16(1/sqrt(sum x^2
// / H + eps)). H % 4 == 0.
template <int NT>
__global__ void __launch_bounds__(NT) residual_norm_kernel(float* __restrict__ x, const uint16_t* __restrict__ y,
                                                           const float* __restrict__ gamma, int H, float eps,
                                                           uint16_t* __restrict__ out) {
  __shared__ float red[NT / 32];
  pdl_wait();  // x and y come from the preceding kernels
  pdl_trigger();
  const int r = blockIdx.x, tid = threadIdx.x;
  float4* xr = reinterpret_cast<float4*>(x + (size_t)r * H);
  const uint2* yr = y ? reinterpret_cast<const uint2*>(y + (size_t)r * H) : nullptr;
  const int H4 = H >> 2;
  float ss = 0.f;
  for (int i = tid; i < H4; i += NT) {
    float4 v = xr[i];
    if (yr) {
      const uint2 w = yr[i];
      v.x = round_bf16(v.x + bf_lo(w.x));
      v.y = round_bf16(v.y + bf_hi(w.x));
      v.z = round_bf16(v.z + bf_lo(w.y));
      v.w = round_bf16(v.w + bf_hi(w.y));
      xr[i] = v;
    }
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  if (!gamma) return;
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += red[w];
  const float sc = round_bf16(1.0f / sqrtf(t / (float)H + eps));
  const float4* gm = reinterpret_cast<const float4*>(gamma);
  uint2* o = reinterpret_cast<uint2*>(out + (size_t)r * H);
  for (int i = tid; i < H4; i += NT) {
    const float4 v = xr[i], g = gm[i];
    const uint32_t a = f2bf_exact(round_bf16(round_bf16(v.x * sc) * g.x));
    const uint32_t b = f2bf_exact(round_bf16(round_bf16(v.y * sc) * g.y));
    const uint32_t c = f2bf_exact(round_bf16(round_bf16(v.z * sc) * g.z));
    const uint32_t d = f2bf_exact(round_bf16(round_bf16(v.w * sc) * g.w));
    o[i] = make_uint2(a | (b << 16), c | (d << 16));
  }
}

// h = bf16(bf16(silu(g)) * u) over rows of gu = [g (I columns) | u (I columns)], all bf16
// (the GEMV's SwiGLU epilogue on GEMM outputs). I % 8 == 0.
__global__ void swiglu_kernel(const uint16_t* __restrict__ gu, int I, int C, uint16_t* __restrict__ h) {
  pdl_wait();
  pdl_trigger();
  const int I8 = I >> 3;
  const size_t total = (size_t)C * I8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / I8, c = i - r * I8;
    const uint4 gv = ldg16(gu + r * 2 * I + c * 8);
    const uint4 uv = ldg16(gu + r * 2 * I + I + c * 8);
    const uint32_t* gw = &gv.x;
    const uint32_t* uw = &uv.x;
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float g0 = bf_lo(gw[k]), g1 = bf_hi(gw[k]);
      const float a0 = round_bf16(g0 / (1.0f + det_expf(-g0)));
      const float a1 = round_bf16(g1 / (1.0f + det_expf(-g1)));
      ow[k] = (uint32_t)f2bf_round(a0 * bf_lo(uw[k])) | ((uint32_t)f2bf_round(a1 * bf_hi(uw[k])) << 16);
    }
    *reinterpret_cast<uint4*>(h + r * I + c * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// ------------------------------------------------------------------ workspace
struct LtGemm {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, d = nullptr;
  cublasLtMatmulAlgo_t algo{};
};

struct PrefillBufs {
  int cap = 0;  // rows per chunk
  float* x = nullptr;                                     // [cap, H] f32 residual stream
  uint16_t *xb = nullptr, *qkv = nullptr, *q = nullptr;   // normed input, q|k|v, rotated q
  uint16_t *attn = nullptr, *y = nullptr;                 // attention output, o/down output
  uint16_t *gu = nullptr, *h = nullptr;                   // gate|up, SwiGLU output
  DevRow* rows = nullptr;
  float* part = nullptr;  // attention partials: cap rows x kvh x 1 split
  int32_t* counters = nullptr;
  cublasLtHandle_t lt = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  std::map<std::array<int, 6>, LtGemm> gemms;
};

void free_prefill(PrefillBufs* p) {
  if (!p) return;
  for (auto& kv : p->gemms) {
    cublasLtMatrixLayoutDestroy(kv.second.a);
    cublasLtMatrixLayoutDestroy(kv.second.b);
    cublasLtMatrixLayoutDestroy(kv.second.d);
    cublasLtMatmulDescDestroy(kv.second.op);
  }
  if (p->lt) cublasLtDestroy(p->lt);
  delete p;  // device buffers are the model's allocations
}

static int lt_fail(cublasStatus_t st, const char* what) {
  return fail(YUE2_ERR_CUDA, std::string(what) + " failed: cuBLASLt status " + std::to_string((int)st));
}

static int ensure_prefill(Yue2Model& m) {
  if (m.prefill) return 0;
  const Geometry& g = m.g;
  const int C = kPrefillRows, H = g.hidden, qd = g.heads * g.dim, kd = g.kvh * g.dim, I = g.inter;
  const int G = g.heads / g.kvh;
  PrefillBufs* P = new PrefillBufs();
  P->cap = C;
  void* p = nullptr;
  int rc;
  auto take = [&](size_t bytes) -> void* {
    if (rc) return nullptr;
    rc = m.alloc(&p, bytes);
    return rc ? nullptr : p;
  };
  rc = 0;
  P->x = (float*)take((size_t)C * H * 4);
  P->xb = (uint16_t*)take((size_t)C * H * 2);
  P->qkv = (uint16_t*)take((size_t)C * (qd + 2 * kd) * 2);
  P->q = (uint16_t*)take((size_t)C * qd * 2);
  P->attn = (uint16_t*)take((size_t)C * qd * 2);
  P->y = (uint16_t*)take((size_t)C * H * 2);
  P->gu = (uint16_t*)take((size_t)C * 2 * I * 2);
  P->h = (uint16_t*)take((size_t)C * I * 2);
  P->rows = (DevRow*)take((size_t)C * sizeof(DevRow));
  P->part = (float*)take((size_t)C * g.kvh * G * (g.dim + 2) * 4);
  P->counters = (int32_t*)take((size_t)C * g.kvh * 4);
  P->ws_bytes = 32u << 20;
  P->ws = take(P->ws_bytes);

  // buffers taken before a failure stay with the model's allocations until it closes
  if (rc) {
    delete P;
    return rc;
  }
  cudaError_t e = cudaMemset(P->counters, 0, (size_t)C * g.kvh * 4);

  if (e != cudaSuccess) {
    delete P;
    return cuda_fail(e, "prefill counters");
  }
  const cublasStatus_t st = cublasLtCreate(&P->lt);
  if (st != CUBLAS_STATUS_SUCCESS) {
    delete P;
    return lt_fail(st, "cublasLtCreate");
  }
  m.prefill = P;
  return 0;
}


// Y[C, N] (row stride ldy) = X[C, K] (row stride ldx) . W[N, K]^T, bf16 in and out, f32
// accumulation. Algorithms may split K only with an out-of-place f32 reduction in a
// separate pass (YUE2_CUDA_GEMM_SPLITK=1; default: no split), never with in-place or
// output-type partial sums, so a row's result depends only on the shapes and repeats
// bit for bit.
static int gemm_lt(Yue2Model& m, const uint16_t* W, int N, int K, const uint16_t* X, int ldx, void* Y, int ldy,
                   int C, bool f32out = false);

// The skinny kernel for the per-layer matrices of passes of up to m.skinny_rows rows; the LM
// head (more 128-row tiles than SMs, so several waves of CTAs each paying the kernel's
// start) stays on cuBLASLt.
static bool use_skinny(const Yue2Model& m, int C, int N, int K, int ldx, int ldy, const void* X, const void* W,
                       const void* Y, bool swiglu) {
  return C <= m.skinny_rows && (N + 127) / 128 <= m.sms && gemm_skinny_supported(C, N, K, ldx, ldy, X, W, Y, swiglu);
}

static int gemm_bf16(Yue2Model& m, const uint16_t* W, int N, int K, const uint16_t* X, int ldx, uint16_t* Y, int ldy,
                     int C) {
  if (use_skinny(m, C, N, K, ldx, ldy, X, W, Y, false)) {
    CK(launch_gemm_skinny(m.stream, m.wide_pdl, W, N, K, X, ldx, Y, ldy, C, false, m.flags + 2));
    return 0;
  }
  if (m.gemm_tc && C >= 128 && gemm_tc_supported(C, N, K, ldx, ldy, X, W, Y)) {
    CK(launch_gemm_tc(m.stream, W, N, K, X, ldx, Y, ldy, C, m.flags + 2));
    return 0;
  }
  return gemm_lt(m, W, N, K, X, ldx, Y, ldy, C);
}

// f32out: Y is f32 (the unrounded sums, for the biased linears of the NAR pathway).
static int gemm_lt(Yue2Model& m, const uint16_t* W, int N, int K, const uint16_t* X, int ldx, void* Y, int ldy,
                   int C, bool f32out) {
  PrefillBufs& P = *m.prefill;
  const std::array<int, 6> key = {N, K, ldx, ldy, C, f32out ? 1 : 0};
  auto it = P.gemms.find(key);
  if (it == P.gemms.end()) {
    LtGemm gm;
    cublasStatus_t st;
    const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    if ((st = cublasLtMatmulDescCreate(&gm.op, CUBLAS_COMPUTE_32F, CUDA_R_32F)) ||
        (st = cublasLtMatmulDescSetAttribute(gm.op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta))) ||
        (st = cublasLtMatmulDescSetAttribute(gm.op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb))) ||
        (st = cublasLtMatrixLayoutCreate(&gm.a, CUDA_R_16BF, K, N, K)) ||
        (st = cublasLtMatrixLayoutCreate(&gm.b, CUDA_R_16BF, K, C, ldx)) ||
        (st = cublasLtMatrixLayoutCreate(&gm.d, f32out ? CUDA_R_32F : CUDA_R_16BF, N, C, ldy)))
      return lt_fail(st, "cuBLASLt descriptor");
    cublasLtMatmulPreference_t pref = nullptr;
    const uint32_t no_split = m.gemm_split_k ? (uint32_t)CUBLASLT_REDUCTION_SCHEME_COMPUTE_TYPE
                                             : (uint32_t)CUBLASLT_REDUCTION_SCHEME_NONE;
    constexpr int kCand = 8;
    cublasLtMatmulHeuristicResult_t res[kCand] = {};
    int found = 0;
    if ((st = cublasLtMatmulPreferenceCreate(&pref)) ||
        (st = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &P.ws_bytes,
                                                   sizeof(P.ws_bytes))) ||
        (st = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_REDUCTION_SCHEME_MASK, &no_split,
                                                   sizeof(no_split))) ||
        (st = cublasLtMatmulAlgoGetHeuristic(P.lt, gm.op, gm.a, gm.b, gm.d, gm.d, pref, kCand, res, &found))) {
      if (pref) cublasLtMatmulPreferenceDestroy(pref);
      return lt_fail(st, "cuBLASLt heuristic");
    }
    cublasLtMatmulPreferenceDestroy(pref);
    if (found < 1) return fail(YUE2_ERR_CUDA, "cuBLASLt has no algorithm for a prefill GEMM");
    // Time the candidates once on the call's own operands (outside a stream capture; the
    // output is rewritten by the call itself) and keep the fastest; inside a capture the
    // heuristic's first choice stands.
    gm.algo = res[0].algo;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (found > 1 && cudaStreamIsCapturing(m.stream, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone) {
      cudaEvent_t e0 = nullptr, e1 = nullptr;
      float best = 1e30f;
      if (cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess) {
        const float alpha = 1.f, beta = 0.f;
        for (int i = 0; i < found; ++i) {
          bool ok = cublasLtMatmul(P.lt, gm.op, &alpha, W, gm.a, X, gm.b, &beta, Y, gm.d, Y, gm.d, &res[i].algo, P.ws,
                                   P.ws_bytes, m.stream) == CUBLAS_STATUS_SUCCESS;
          cudaEventRecord(e0, m.stream);
          for (int rep = 0; ok && rep < 3; ++rep)
            ok = cublasLtMatmul(P.lt, gm.op, &alpha, W, gm.a, X, gm.b, &beta, Y, gm.d, Y, gm.d, &res[i].algo, P.ws,
                                P.ws_bytes, m.stream) == CUBLAS_STATUS_SUCCESS;
          cudaEventRecord(e1, m.stream);
          float ms = 0.f;
          if (ok && cudaEventSynchronize(e1) == cudaSuccess && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess &&
              ms < best) {
            best = ms;
            gm.algo = res[i].algo;
          }
        }
      }
      if (e0) cudaEventDestroy(e0);
      if (e1) cudaEventDestroy(e1);
      CK(cudaGetLastError());
    }
    it = P.gemms.emplace(key, gm).first;
  }
  const LtGemm& gm = it->second;
  const float alpha = 1.f, beta = 0.f;
  const cublasStatus_t st = cublasLtMatmul(P.lt, gm.op, &alpha, W, gm.a, X, gm.b, &beta, Y, gm.d, Y, gm.d, &gm.algo,
                                           P.ws, P.ws_bytes, m.stream);
  if (st != CUBLAS_STATUS_SUCCESS) return lt_fail(st, "cublasLtMatmul");
  return 0;
}

// Several weight matrices [N_i, K] side by side in one output of row stride ldy: one GEMM
// when they are adjacent in memory (the model's arena places them so), else one each.
static int gemm_concat(Yue2Model& m, const uint16_t* const* W, const int* N, int parts, int K, const uint16_t* X,
                       int ldx, uint16_t* Y, int ldy, int C) {
  bool adjacent = true;
  int total = N[0];
  for (int i = 1; i < parts; ++i) {
    adjacent = adjacent && W[i] == W[i - 1] + (size_t)N[i - 1] * K;
    total += N[i];
  }
  if (adjacent) return gemm_bf16(m, W[0], total, K, X, ldx, Y, ldy, C);
  int col = 0;
  for (int i = 0; i < parts; ++i) {
    const int rc = gemm_bf16(m, W[i], N[i], K, X, ldx, Y + col, ldy, C);
    if (rc) return rc;
    col += N[i];
  }
  return 0;
}

static cudaError_t launch_residual_norm(cudaStream_t s, bool pdl, float* x, const uint16_t* y, const float* gamma,
                                        int H, float eps, uint16_t* out, int C) {
  void* args[] = {&x, &y, &gamma, &H, &eps, &out};
  return launch_with(s, pdl, dim3(C), dim3(256), 0, (const void*)residual_norm_kernel<256>, args);
}

// Split-K decode attention with one query per row: decode rows (fused: QK norm, RoPE and
// the row's K/V append in the kernel) or prefill chunk rows whose K/V rope_append wrote
// (head sizes the tensor-core prefill kernel does not take).
static int row_attention(Yue2Model& m, PrefillBufs& P, DevRow* rows, int l, int R, int splits, bool fused) {
  const LayerW& w = m.layers[l];
  const Geometry& g = m.g;
  AttnParams ap = {};
  ap.rows = rows;
  ap.q = P.q;
  ap.out = P.attn;
  ap.part = P.part;
  ap.counters = P.counters;
  ap.g = g;
  ap.layer = l;
  ap.splits = splits;
  ap.scale = 1.0f / sqrtf((float)g.dim);
  ap.fused = fused ? 1 : 0;
  ap.qkv = P.qkv;
  ap.q_norm = w.q_norm;
  ap.k_norm = w.k_norm;
  ap.cos_tab = m.cos_tab;
  ap.sin_tab = m.sin_tab;
  ap.max_pos = m.max_pos;
  ap.error = m.flags + 1;
  ap.pipe = fused ? 1 : 0;  // decode rows of the GEMM path: the pipelined tensor-core loop
  if (fused && R <= 8) {
    // the cluster form where the rows' contexts allow it (attn_cluster_for), with no more
    // CTAs per (kv head, row) than leave one wave of them on the SMs. Measured ms/step at a
    // ~1,040-position context, cluster form against split-K: 4 rows 2.260 / 2.374, 8 rows
    // 2.368 / 2.398, 16 rows 2.639 / 2.592 (so 16 rows keep the split-K loop)
    const int cs = attn_cluster_for(m, R);
    ap.cluster = m.attn_cluster > 0 ? cs : std::min(cs, std::max(1, m.sms / (g.kvh * R)));
  }
  CK(launch_attention(m.stream, m.wide_pdl, ap, R));
  return 0;
}

// h = SwiGLU(gate . x, up . x) of R rows (P.xb -> P.h): one GEMM with the epilogue fused
// (skinny tcgen05 for R <= 256, the prefill tcgen05 GEMM when opted in for R >= 128), else
// the gate|up GEMM into P.gu and swiglu_kernel.
static bool gate_up_fused(const Yue2Model& m, const PrefillBufs& P, const LayerW& w, int R) {
  const Geometry& g = m.g;
  const int H = g.hidden, I = g.inter;
  if (w.up != w.gate + (size_t)I * H || I % 128) return false;
  return use_skinny(m, R, I, H, H, I, P.xb, w.gate, P.h, true) ||
         (m.gemm_tc && R >= 128 && gemm_tc_supported(R, I, H, H, I, P.xb, w.gate, P.h));
}

static int gate_up_swiglu(Yue2Model& m, PrefillBufs& P, const LayerW& w, int R) {
  const Geometry& g = m.g;
  const int H = g.hidden, I = g.inter;
  cudaStream_t s = m.stream;
  if (gate_up_fused(m, P, w, R)) {
    if (use_skinny(m, R, I, H, H, I, P.xb, w.gate, P.h, true))
      CK(launch_gemm_skinny(s, m.wide_pdl, w.gate, I, H, P.xb, H, P.h, I, R, true, m.flags + 2));
    else
      CK(launch_gemm_tc_swiglu(s, w.gate, I, H, P.xb, H, P.h, I, R, m.flags + 2));
    return 0;
  }
  {
    const uint16_t* W[2] = {w.gate, w.up};
    const int N[2] = {I, I};
    const int rc = gemm_concat(m, W, N, 2, H, P.xb, H, P.gu, 2 * I, R);
    if (rc) return rc;
  }
  const uint16_t* gu = P.gu;
  uint16_t* h = P.h;
  int inter = I, nrows = R;
  void* args[] = {&gu, &inter, &nrows, &h};
  const int blocks = std::min(4 * m.sms, (int)(((size_t)R * (I / 8) + 255) / 256));
  CK(launch_with(s, m.wide_pdl, dim3(blocks), dim3(256), 0, (const void*)swiglu_kernel, args));
  return 0;
}

// ------------------------------------------------------------------ the layers over R rows
// Layers `lw` of R rows whose embeddings are in P.x (f32), ending with the last residual
// added (the final norm is the caller's). Prefill chunk rows (decode = false) belong to one
// cache at positions pos0 + r: rope_append writes all their K/V, then the causal prefill
// attention runs. Decode rows (decode = true) each have their own cache: the decode
// attention kernel applies the QK norm and RoPE and appends each row's K/V itself.
// causal = false (the NAR pathway's latent rows): every chunk row sees every key up to the
// chunk's last position.
static int encode_layers(Yue2Model& m, PrefillBufs& P, const std::vector<LayerW>& lw, DevRow* rows, int R,
                         bool decode, const uint64_t* pages, int pos0, bool causal = true) {
  if (!causal && (decode || !prefill_attention_supported(m.g)))
    return fail(YUE2_ERR_INVALID, "non-causal rows need the tensor-core prefill attention (head_dim 64 or 128)");
  const Geometry& g = m.g;
  const int H = g.hidden, qd = g.heads * g.dim, kd = g.kvh * g.dim, I = g.inter;
  cudaStream_t s = m.stream;
  int rc;
  // one wave of attention CTAs where R is small; the partials hold cap rows x kvh
  const int splits = std::max(1, std::min(std::min(m.max_splits, P.cap / R), 2 * m.sms / (g.kvh * R)));
  for (int l = 0; l < g.layers; ++l) {
    const LayerW& w = lw[l];
    CK(launch_residual_norm(s, m.wide_pdl, P.x, l ? P.y : nullptr, w.in_norm, H, g.eps, P.xb, R));
    {
      const uint16_t* W[3] = {w.q, w.k, w.v};
      const int N[3] = {qd, kd, kd};
      if ((rc = gemm_concat(m, W, N, 3, H, P.xb, H, P.qkv, qd + 2 * kd, R))) return rc;
    }
    if (decode) {
      if ((rc = row_attention(m, P, rows, l, R, splits, true))) return rc;
    } else {
      RopeParams rp = {};
      rp.rows = rows;
      rp.qkv = P.qkv;
      rp.q_out = P.q;
      rp.cos_tab = m.cos_tab;
      rp.sin_tab = m.sin_tab;
      rp.q_norm = w.q_norm;
      rp.k_norm = w.k_norm;
      rp.g = g;
      rp.layer = l;
      rp.max_pos = m.max_pos;
      rp.error = m.flags + 1;
      CK(launch_rope_append(s, false, rp, R));
      if ((m.prefill_tc_attn || !causal) && prefill_attention_supported(g)) {
        PrefillAttnParams fp = {};
        fp.pages = pages;
        fp.q = P.q;
        fp.out = P.attn;
        fp.g = g;
        fp.layer = l;
        fp.C = R;
        fp.pos0 = pos0;
        fp.scale = 1.0f / sqrtf((float)g.dim);
        fp.causal = causal ? 1 : 0;
        fp.error = m.flags + 2;
        const bool wide = (long)((R + 127) / 128) * g.heads >= 2L * m.sms;  // tcgen05 tiles: 128 rows
        if (prefill_attention_tc_supported(g) && (m.prefill_attn_tc5 == 1 || (m.prefill_attn_tc5 == 0 && wide))) {
          CK(launch_prefill_attention_tc(s, fp));
        } else {
          CK(launch_prefill_attention(s, fp));
        }
      } else if ((rc = row_attention(m, P, rows, l, R, splits, false))) {
        return rc;
      }
    }
    if ((rc = gemm_bf16(m, w.o, H, qd, P.attn, qd, P.y, H, R))) return rc;
    CK(launch_residual_norm(s, m.wide_pdl, P.x, P.y, w.post_norm, H, g.eps, P.xb, R));
    if ((rc = gate_up_swiglu(m, P, w, R))) return rc;
    if ((rc = gemm_bf16(m, w.down, H, I, P.h, I, P.y, H, R))) return rc;
  }
  return 0;
}

// ------------------------------------------------------------------ one prefill chunk
static int prefill_chunk(Yue2Model& m, Yue2Cache& c, const int32_t* d_ids, uint64_t L0, uint64_t n, uint64_t start,
                         int C) {
  PrefillBufs& P = *m.prefill;
  const Geometry& g = m.g;
  cudaStream_t s = m.stream;
  {
    DevRow* rows = P.rows;
    const uint64_t* pages = c.d_pages;
    int32_t pb = (int32_t)L0, pe = (int32_t)(L0 + n), p0 = (int32_t)(L0 + start);
    void* args[] = {&rows, &C, &pages, &d_ids, &pb, &pe, &p0};
    CK(launch_with(s, false, dim3((C + 127) / 128), dim3(128), 0, (const void*)prefill_rows_kernel, args));
  }
  CK(launch_embed(s, false, P.rows, C, m.embed, g.hidden, g.vocab, P.x, m.flags + 0));
  const int rc = encode_layers(m, P, m.layers, P.rows, C, false, c.d_pages, (int)(L0 + start));
  if (rc) return rc;
  // the last layer's residual (the LM head applies the final norm itself)
  CK(launch_residual_norm(s, m.wide_pdl, P.x, P.y, nullptr, g.hidden, g.eps, nullptr, C));
  return 0;
}

// ------------------------------------------------------------------ wide decode steps
// LM head rows [lo, hi) cover the phase's window and its stop row (project_phase,
// src/model.rs:478-507): the whole vocabulary, the codec window with MUSIC_END just below
// it, or the Abc window up to and including ABC_END (the 205 ids between are computed
// and dropped).
static void head_span(const Yue2Model& m, int phase, int& lo, int& hi, int& start, int& end, int& stop) {
  const int V = m.g.vocab;
  if (phase == kPhaseVocab) {
    lo = start = 0;
    hi = end = V;
    stop = -1;
    return;
  }
  start = phase == kPhaseAbc ? 0 : (int)kCodecOffset;
  end = phase == kPhaseAbc ? (int)kEOD : (int)(kCodecOffset + kCodecSize);
  stop = phase == kPhaseAbc ? (int)kAbcEnd : (int)kMusicEnd;
  lo = std::min(start, stop);
  hi = std::max(end, stop + 1);
}

// logits[r][id] = bf16 head output h[r][id - lo] for ids of the window and the stop row
// (the rest of the row is already -inf outside the full-vocabulary phase).
__global__ void head_scatter_kernel(const uint16_t* __restrict__ h, int ldh, int R, int lo, int n, int start, int end,
                                    int stop, float* __restrict__ logits, int V) {
  pdl_wait();
  pdl_trigger();
  const size_t total = (size_t)R * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / n), j = (int)(i - (size_t)r * n), id = lo + j;
    if ((id >= start && id < end) || id == stop) logits[(size_t)r * V + id] = bf2f(h[(size_t)r * ldh + j]);
  }
}

int ensure_wide(Yue2Model& m) {
  int rc = ensure_prefill(m);
  if (rc || m.wide_rows) return rc;
  const size_t V = m.g.vocab;
  void *a = nullptr, *b = nullptr, *c = nullptr;
  if ((rc = m.alloc(&a, kMaxWideRows * sizeof(DevRow))) || (rc = m.alloc(&b, kMaxWideRows * V * 4)) ||
      (rc = m.alloc(&c, kMaxWideRows * ((V + 7) & ~(size_t)7) * 2)))
    return rc;
  CK(cudaMemset(a, 0, kMaxWideRows * sizeof(DevRow)));
  m.wide_rows = (DevRow*)a;
  m.wide_logits = (float*)b;
  m.wide_head = (uint16_t*)c;
  return 0;
}

// Runs each GEMM shape of a wide step once, outside any stream capture, so that its
// algorithm is timed and chosen before a session graph captures the step. The operands are
// workspace buffers (their contents do not matter; the outputs are scratch).
int prepare_wide(Yue2Model& m, int R, int phase) {
  int rc = ensure_wide(m);
  if (rc) return rc;
  PrefillBufs& P = *m.prefill;
  const Geometry& g = m.g;
  const int H = g.hidden, qd = g.heads * g.dim, kd = g.kvh * g.dim, I = g.inter;
  const LayerW& w = m.layers[0];
  const uint16_t* Wqkv[3] = {w.q, w.k, w.v};
  const int Nqkv[3] = {qd, kd, kd};
  const uint16_t* Wgu[2] = {w.gate, w.up};
  const int Ngu[2] = {I, I};
  int lo, hi, start, end, stop;
  head_span(m, phase, lo, hi, start, end, stop);
  const int n = hi - lo, ldh = (n + 7) & ~7;
  if ((rc = gemm_concat(m, Wqkv, Nqkv, 3, H, P.xb, H, P.qkv, qd + 2 * kd, R)) ||
      (rc = gemm_bf16(m, w.o, H, qd, P.attn, qd, P.y, H, R)) ||
      (rc = gemm_concat(m, Wgu, Ngu, 2, H, P.xb, H, P.gu, 2 * I, R)) || (rc = gate_up_swiglu(m, P, w, R)) ||
      (rc = gemm_bf16(m, w.down, H, I, P.h, I, P.y, H, R)) ||
      (rc = gemm_bf16(m, m.lm_head + (size_t)lo * H, n, H, P.xb, H, m.wide_head, ldh, R)))
    return rc;
  CK(cudaStreamSynchronize(m.stream));
  return 0;
}

// One decode step of R (kMaxRows < R <= kMaxWideRows) rows in m.wide_rows: embed, layers,
// final norm, LM head into m.wide_logits, positions advanced.
int encode_forward_wide(Yue2Model& m, cudaStream_t s, int R, int phase) {
  if (s != m.stream) return fail(YUE2_ERR_INVALID, "wide decode steps run on the model's stream");
  int rc = ensure_wide(m);
  if (rc) return rc;
  PrefillBufs& P = *m.prefill;
  const Geometry& g = m.g;
  const int H = g.hidden, V = g.vocab;
  CK(launch_embed(s, m.wide_pdl, m.wide_rows, R, m.embed, H, V, P.x, m.flags + 0));
  if ((rc = encode_layers(m, *m.prefill, m.layers, m.wide_rows, R, true, nullptr, 0))) return rc;
  CK(launch_residual_norm(s, m.wide_pdl, P.x, P.y, m.final_norm, H, g.eps, P.xb, R));
  int lo, hi, start, end, stop;
  head_span(m, phase, lo, hi, start, end, stop);
  const int n = hi - lo, ldh = (n + 7) & ~7;
  if (phase != kPhaseVocab) CK(launch_fill_f32(s, m.wide_logits, (size_t)R * V, -INFINITY));
  if ((rc = gemm_bf16(m, m.lm_head + (size_t)lo * H, n, H, P.xb, H, m.wide_head, ldh, R))) return rc;
  {
    const uint16_t* h = m.wide_head;
    float* logits = m.wide_logits;
    int ld = ldh, rows = R, vocab = V;
    void* args[] = {&h, &ld, &rows, &lo, (void*)&n, &start, &end, &stop, &logits, &vocab};
    const int blocks = std::min(8 * m.sms, (int)(((size_t)R * n + 255) / 256));
    CK(launch_with(s, m.wide_pdl, dim3(blocks), dim3(256), 0, (const void*)head_scatter_kernel, args));
  }
  CK(launch_step_end(s, m.wide_pdl, m.wide_rows, R));
  return 0;
}

// Kernels of this library per wide step of R rows (cuBLASLt GEMMs not counted): embed, per
// layer two norms and attention, then either the four skinny GEMMs (q|k|v, o, gate|up with
// SwiGLU, down) or the SwiGLU kernel, the final norm, [the -inf fill], the head scatter and
// step_end (the LM head GEMM is cuBLASLt's).
int wide_kernels_per_step(const Yue2Model& m, int phase, int R) {
  const bool sk = R <= m.skinny_rows;
  return 1 + (3 + (sk ? 4 : 1)) * m.g.layers + 1 + (phase != kPhaseVocab) + 2;
}

int prefill_gemm(Yue2Model& m, Yue2Cache& c, const int32_t* d_ids, uint64_t n, int logits_row, int phase) {
  const Geometry& g = m.g;
  if (g.hidden % 8 || g.inter % 8 || (g.heads * g.dim) % 8 || g.dim % 8)
    return fail(YUE2_ERR_INVALID, "GEMM prefill needs hidden, intermediate and head sizes divisible by 8");
  int rc = ensure_prefill(m);
  if (rc) return rc;
  const uint64_t L0 = c.length;
  const uint64_t chunks = (n + m.prefill_chunk - 1) / m.prefill_chunk;
  const uint64_t per = (n + chunks - 1) / chunks;
  int lastC = 0;
  for (uint64_t start = 0; start < n; start += per) {
    const int C = (int)std::min<uint64_t>(per, n - start);
    if ((rc = prefill_chunk(m, c, d_ids, L0, n, start, C))) return rc;
    lastC = C;
  }
  if (logits_row >= 0)
    CK(encode_head_from(m, m.stream, false, m.prefill->x + (size_t)(lastC - 1) * g.hidden, 1, logits_row, phase,
                        nullptr));
  c.length = L0 + n;
  return 0;
}

}  // namespace y2

// ---------------------------------------------------------------- NAR velocity
namespace y2 {

// v = bf16(y + bias) (Linear::finish with a bf16 bias, src/tensor.rs:1102-1118), then with
// `silu` v = bf16(silu(v)) (the time embedder's activation, src/model.rs:635-638); into
// f32 and/or bf16 outputs.
__global__ void bias_round_kernel(const float* __restrict__ y, const float* __restrict__ bias, int rows, int N,
                                  int silu, float* __restrict__ outf, uint16_t* __restrict__ outb) {
  const size_t total = (size_t)rows * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float v = round_bf16(y[i] + bias[i % N]);
    if (silu) v = round_bf16(v / (1.0f + det_expf(-v)));
    if (outf) outf[i] = v;
    if (outb) outb[i] = f2bf_exact(v);
  }
}

// x[r] = bf16(bf16(bf16(vae2llm(padded)[r] + bias) + time) + pe[min(r, frames - 1)])
// (src/model.rs:623-649)
__global__ void nar_embed_kernel(const float* __restrict__ y, const float* __restrict__ bias,
                                 const float* __restrict__ time, const uint16_t* __restrict__ pe, int frames, int n,
                                 int H, float* __restrict__ x) {
  const size_t total = (size_t)n * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / H), c = (int)(i - (size_t)r * H);
    const float v = round_bf16(y[i] + bias[c]);
    x[i] = round_bf16(round_bf16(v + time[c]) + bf2f(pe[(size_t)min(r, frames - 1) * H + c]));
  }
}

// One device block for a velocity call of n rows: the layer activations (a PrefillBufs of
// capacity n; the attention partials and counters stay unused, as the non-causal rows take
// the tensor-core attention) and the NAR inputs and outputs. Taken from the model's scratch
// and given back when the call ends, so one song's repeated calls reuse it.
struct NarBufs {
  PrefillBufs act;
  uint16_t *lat_in = nullptr, *sinus = nullptr, *time_bf = nullptr;
  float *yf = nullptr, *time2 = nullptr, *lat_out = nullptr;
  void* block = nullptr;
};

static int take_nar(Yue2Model& m, int n, NarBufs& B) {
  const Geometry& g = m.g;
  const size_t C = n, H = g.hidden, qd = (size_t)g.heads * g.dim, kd = (size_t)g.kvh * g.dim, I = g.inter;
  const size_t L = m.nar.latent;
  size_t off = 0;
  std::vector<std::pair<void**, size_t>> plan;
  auto at = [&](void** p, size_t bytes) {
    plan.push_back({p, off});
    off += (bytes + 255) & ~(size_t)255;
  };
  PrefillBufs& P = B.act;
  at((void**)&P.x, C * H * 4);
  at((void**)&P.xb, C * H * 2);
  at((void**)&P.qkv, C * (qd + 2 * kd) * 2);
  at((void**)&P.q, C * qd * 2);
  at((void**)&P.attn, C * qd * 2);
  at((void**)&P.y, C * H * 2);
  at((void**)&P.gu, C * 2 * I * 2);
  at((void**)&P.h, C * I * 2);
  at((void**)&P.rows, C * sizeof(DevRow));
  at((void**)&B.lat_in, C * L * 2);
  at((void**)&B.yf, C * std::max(H, L) * 4);
  at((void**)&B.lat_out, C * L * 4);
  at((void**)&B.sinus, 256 * 2);
  at((void**)&B.time_bf, H * 2);
  at((void**)&B.time2, H * 4);
  const int rc = m.scratch_take(&B.block, off);
  if (rc) return rc;
  for (auto& p : plan) *p.first = (char*)B.block + p.second;
  P.cap = n;
  return 0;
}

static cudaError_t launch_bias_round(cudaStream_t s, const float* y, const float* bias, int rows, int N, int silu,
                                     float* outf, uint16_t* outb, int sms) {
  void* args[] = {&y, &bias, &rows, &N, &silu, &outf, &outb};
  const int blocks = std::max(1, std::min(4 * sms, (int)(((size_t)rows * N + 255) / 256)));
  return launch_with(s, false, dim3(blocks), dim3(256), 0, (const void*)bias_round_kernel, args);
}

// The body of yue2_velocity over the buffers B (rows + 2 rows).
static int velocity_rows(Yue2Model* m, Yue2Cache* c, NarBufs& B, const float* state, uint64_t rows, double raw_t,
                         float* out) {
  const Geometry& g = m->g;
  const uint64_t n = rows + 2;
  PrefillBufs& P = B.act;
  int rc;
  const auto& W = m->nar;
  const int H = g.hidden, L = W.latent, N = (int)n;
  cudaStream_t s = m->stream;
  // host: zero-padded latent rows and the timestep's sinusoidal features (f32 math in the
  // reference's order, src/model.rs:624-634)
  std::vector<uint16_t> padded((size_t)n * L, 0);
  for (size_t i = 0; i < rows * (size_t)L; ++i) padded[L + i] = (uint16_t)(det_f2u(round_bf16(state[i])) >> 16);
  const float raw = round_bf16((float)raw_t);
  const float sig = round_bf16(1.0f / (1.0f + expf(-raw)));
  const float top = round_bf16(W.shift * sig);
  const float bottom = round_bf16(1.f + round_bf16((W.shift - 1.f) * sig));
  const float t = round_bf16(top / bottom);
  std::vector<uint16_t> sinus(256);
  for (int i = 0; i < 128; ++i) {
    const float f = expf(-logf(10000.f) * (float)i / 128.f);
    sinus[i] = (uint16_t)(det_f2u(round_bf16(cosf(t * f))) >> 16);
    sinus[128 + i] = (uint16_t)(det_f2u(round_bf16(sinf(t * f))) >> 16);
  }
  CK(cudaMemcpyAsync(B.lat_in, padded.data(), padded.size() * 2, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(B.sinus, sinus.data(), 512, cudaMemcpyHostToDevice, s));
  // time embedder: time_out(bf16(silu(time_in(sinus))))
  if ((rc = gemm_lt(*m, W.time_in, H, 256, B.sinus, 256, B.yf, H, 1, true))) return rc;
  CK(launch_bias_round(s, B.yf, W.time_in_b, 1, H, 1, nullptr, B.time_bf, m->sms));
  if ((rc = gemm_lt(*m, W.time_out, H, H, B.time_bf, H, B.yf, H, 1, true))) return rc;
  CK(launch_bias_round(s, B.yf, W.time_out_b, 1, H, 0, B.time2, nullptr, m->sms));
  // latent rows into the hidden width, plus time and position
  if ((rc = gemm_lt(*m, W.vae2llm, H, L, B.lat_in, L, B.yf, H, N, true))) return rc;
  {
    const float *y = B.yf, *bias = W.vae2llm_b, *time = B.time2;
    const uint16_t* pe = W.pe;
    int frames = W.max_frames, nn = N, hh = H;
    float* x = P.x;
    void* args[] = {&y, &bias, &time, &pe, &frames, &nn, &hh, &x};
    const int blocks = std::min(4 * m->sms, (int)(((size_t)N * H + 255) / 256));
    CK(launch_with(s, false, dim3(blocks), dim3(256), 0, (const void*)nar_embed_kernel, args));
  }
  {
    DevRow* dr = P.rows;
    const uint64_t* pages = c->d_pages;
    const int32_t* none = nullptr;
    int32_t pb = 0, pe = 0, p0 = (int32_t)c->length;
    int nn = N;
    void* args[] = {&dr, &nn, &pages, &none, &pb, &pe, &p0};
    CK(launch_with(s, false, dim3((N + 127) / 128), dim3(128), 0, (const void*)prefill_rows_kernel, args));
  }
  if ((rc = encode_layers(*m, P, m->nar_layers, P.rows, N, false, c->d_pages, (int)c->length, false))) return rc;
  CK(launch_residual_norm(s, m->wide_pdl, P.x, P.y, m->final_norm, H, g.eps, P.xb, N));
  if ((rc = gemm_lt(*m, W.llm2vae, L, H, P.xb, H, B.yf, L, N, true))) return rc;
  CK(launch_bias_round(s, B.yf, W.llm2vae_b, N, L, 0, B.lat_out, nullptr, m->sms));
  CK(cudaMemcpyAsync(out, B.lat_out + L, rows * (size_t)L * 4, cudaMemcpyDeviceToHost, s));
  if ((rc = take_flags(*m))) return rc;
  CK(cudaStreamSynchronize(s));
  return 0;
}

}  // namespace y2

// Model::velocity (src/model.rs:611-697) with nar_cond_end = 0, on the device. The latent
// rows take positions cache.length .. + rows + 1: their K/V go into the cache's pages past
// its length (scratch; the length does not change), and every latent row attends to the
// whole prefix and to every latent row.
extern "C" int yue2_velocity(Yue2Model* m, Yue2Cache* c, const float* state, uint64_t rows, double raw_t,
                             float* out) {
  using namespace y2;
  if (!m || !c || !state || !out) return fail(YUE2_ERR_INVALID, "null argument");
  if (!m->finalized) return fail(YUE2_ERR_INVALID, "model not finalized");
  if (!m->nar_arena) return fail(YUE2_ERR_INVALID, "NAR tensors not enabled (yue2_model_enable_nar)");
  if (c->m != m) return fail(YUE2_ERR_INVALID, "cache belongs to another model");
  const Geometry& g = m->g;
  const uint64_t n = rows + 2;
  if (rows == 0) return fail(YUE2_ERR_INVALID, "velocity needs at least one latent row");
  if (rows >= c->capacity || c->length + n > c->capacity || c->length + n > (uint64_t)m->max_pos)
    return fail(YUE2_ERR_CAPACITY, "latent rows exceed the cache/model context");
  if (!prefill_attention_supported(g)) return fail(YUE2_ERR_INVALID, "NAR velocity needs head_dim 64 or 128");
  int rc = y2_set_device(m);
  if (rc) return rc;
  if ((rc = ensure_prefill(*m))) return rc;  // the cuBLASLt state the GEMMs share
  NarBufs B;
  if ((rc = take_nar(*m, (int)n, B))) return rc;
  try {  // the host copy of the padded frames: no exception crosses the C ABI
    rc = velocity_rows(m, c, B, state, rows, raw_t, out);
  } catch (const std::bad_alloc&) {
    rc = fail(YUE2_ERR_OOM, "host allocation failed");
  }
  if (rc) cudaStreamSynchronize(m->stream);  // nothing queued may still use the block
  m->scratch_give(B.block);
  return rc;
}

// ---------------------------------------------------------------- GEMM timing and parity hook
extern "C" int yue2_bench_gemm(Yue2Model* m, const void* X, const void* W, void* Y, int C, int N, int K, int impl,
                               int reps, double* avg_ms) {
  using namespace y2;
  if (!m || !X || !W || !Y || C < 1 || N < 1 || K < 1 || reps < 1 || impl < 0 || impl > 4)
    return fail(YUE2_ERR_INVALID, "bad GEMM benchmark arguments");
  int rc = y2_set_device(m);
  if (rc || (rc = ensure_prefill(*m))) return rc;
  const uint16_t *x = (const uint16_t*)X, *w = (const uint16_t*)W;
  uint16_t* y = (uint16_t*)Y;
  if ((impl == 1 || impl == 2) && (!gemm_tc_supported(C, N, K, K, N, X, W, Y) || (impl == 2 && N % 128)))
    return fail(YUE2_ERR_INVALID, "shape not supported by the tcgen05 GEMM");
  if (impl >= 3 && !gemm_skinny_supported(C, N, K, K, N, X, W, Y, impl == 4))
    return fail(YUE2_ERR_INVALID, "shape not supported by the skinny tcgen05 GEMM");
  cudaEvent_t a = nullptr, b = nullptr;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  for (int i = 0; i <= reps && !rc; ++i) {
    if (i == 1) cudaEventRecord(a, m->stream);
    if (impl == 1) {
      const cudaError_t e = launch_gemm_tc(m->stream, w, N, K, x, K, y, N, C, m->flags + 2);
      if (e != cudaSuccess) rc = cuda_fail(e, "launch_gemm_tc");
    } else if (impl == 2) {
      const cudaError_t e = launch_gemm_tc_swiglu(m->stream, w, N, K, x, K, y, N, C, m->flags + 2);
      if (e != cudaSuccess) rc = cuda_fail(e, "launch_gemm_tc_swiglu");
    } else if (impl >= 3) {
      const cudaError_t e =
          launch_gemm_skinny(m->stream, false, w, N, K, x, K, y, N, C, impl == 4, m->flags + 2);
      if (e != cudaSuccess) rc = cuda_fail(e, "launch_gemm_skinny");
    } else {
      rc = gemm_lt(*m, w, N, K, x, K, y, N, C);
    }
  }
  cudaEventRecord(b, m->stream);
  cudaEventSynchronize(b);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (rc) return rc;
  if (avg_ms) *avg_ms = ms / reps;
  return take_flags(*m);
}
