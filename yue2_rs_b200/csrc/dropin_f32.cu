// The reference's f32 Metal imports (src/tensor.rs:134-219, implemented by src/metal.m):
//   yue2_metal_gemm      (metal.m:164-181)  -> yue2_cuda_gemm
//   yue2_metal_linear    (metal.m:216-237)  -> yue2_cuda_linear
//   yue2_metal_attention (metal.m:330-362)  -> yue2_cuda_attention
//   yue2_metal_stack     (metal.m:429-538)  -> yue2_cuda_stack
// Same argument lists and 1 = done / 0 = not done; every 0 leaves yue2_last_error() (there
// is no CPU fallback). The reference computes these in f32 on Metal Performance Shaders
// matrices plus its own shaders (attention.metal), rounding to bf16 only where its shaders
// do; here the products are f32 cuBLASLt matmuls (compute type 32F, no TF32: the plain
// library GEMM the reference's MPS calls are) and the shaders' arithmetic is restated in
// CUDA kernels with the same roundings:
//   convert_weight (attention.metal:159-173): bf16 widened exactly; F32/F16 kept, rounded
//     to bf16 when the weight is marked bf16;
//   rms_norm (:80-97), normalize_rotary (:99-124), pointwise (:125-137),
//   merge_keys_values (:138-157), pack_queries / pack_keys_values / attention_softmax /
//   unpack_attention (:9-70).
// One process-wide context (its own lock, stream and caches) serves these four; the
// decode drop-ins of dropin.cu keep theirs. yue2_cuda_clear_weights / release_model /
// release_cache reach both.
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "common.cuh"
#include "detmath.h"
#include "engine.h"

using namespace y2;

namespace {

// ------------------------------------------------------------------ kernels
constexpr int kNT = 256;

// rms_norm: out = bf16(bf16(x * s) * gamma), s = bf16(1 / sqrt(sum(x^2) / cols + eps)).
__global__ void __launch_bounds__(kNT) f32_rms_norm_kernel(const float* __restrict__ in, const float* __restrict__ gamma,
                                                           float* __restrict__ out, int cols, float eps) {
  __shared__ float red[kNT / 32];
  const size_t base = (size_t)blockIdx.x * cols;
  float s = 0.f;
  for (int d = threadIdx.x; d < cols; d += kNT) {
    const float v = in[base + d];
    s = fmaf(v, v, s);
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNT / 32; ++w) t += red[w];
  const float scale = round_bf16(1.0f / sqrtf(t / (float)cols + eps));
  for (int d = threadIdx.x; d < cols; d += kNT) out[base + d] = round_bf16(round_bf16(in[base + d] * scale) * gamma[d]);
}

// normalize_rotary on one (row, head): the head (rounded to bf16 first) is RMS-normalised
// with gamma, then rotated by the row's cos/sin ([rows, dim/2]).
__global__ void __launch_bounds__(kNT) f32_rotary_kernel(float* __restrict__ x, const float* __restrict__ gamma,
                                                         const float* __restrict__ cs, const float* __restrict__ sn,
                                                         int heads, int dim, float eps) {
  __shared__ float red[kNT / 32];
  const int head = blockIdx.x, row = head / heads, half = dim / 2;
  float* v = x + (size_t)head * dim;
  float s = 0.f;
  for (int d = threadIdx.x; d < dim; d += kNT) {
    const float a = round_bf16(v[d]);
    s = fmaf(a, a, s);
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNT / 32; ++w) t += red[w];
  const float scale = round_bf16(1.0f / sqrtf(t / (float)dim + eps));
  for (int d = threadIdx.x; d < half; d += kNT) {
    const float a = round_bf16(round_bf16(round_bf16(v[d]) * scale) * gamma[d]);
    const float b = round_bf16(round_bf16(round_bf16(v[half + d]) * scale) * gamma[half + d]);
    const float c = cs[(size_t)row * half + d], sv = sn[(size_t)row * half + d];
    v[d] = round_bf16(round_bf16(a * c) - round_bf16(b * sv));
    v[half + d] = round_bf16(round_bf16(b * c) + round_bf16(a * sv));
  }
}

// pointwise: mode 0 a = bf16(a); mode 1 a = bf16(bf16(silu(bf16 a)) * bf16 b);
// mode 2 a = bf16(a + bf16 b).
__global__ void f32_pointwise_kernel(float* __restrict__ a, const float* __restrict__ b, size_t count, int mode) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    if (mode == 0) {
      a[i] = round_bf16(a[i]);
    } else if (mode == 1) {
      const float g = round_bf16(a[i]);
      const float act = round_bf16(g / (1.0f + det_expf(-g)));
      a[i] = round_bf16(act * round_bf16(b[i]));
    } else {
      a[i] = round_bf16(a[i] + round_bf16(b[i]));
    }
  }
}

// pack_keys_values / merge_keys_values: packed [kv][keys][dim] from rows [keys, kv*dim].
// Rows below `prefix` come from the bf16 prefix block ([prefix, kv*dim] keys, then values);
// the rest from the f32 key rows and the f32 value rows (values rounded when `round_v`).
__global__ void f32_pack_kv_kernel(const uint16_t* __restrict__ pre, int prefix, const float* __restrict__ key,
                                   const float* __restrict__ value, float* __restrict__ pk, float* __restrict__ pv,
                                   int keys, int kv, int dim, int round_v) {
  const size_t total = (size_t)kv * keys * dim;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % dim), r = (int)((i / dim) % keys), h = (int)(i / ((size_t)dim * keys));
    if (r < prefix) {
      const size_t src = (size_t)r * kv * dim + (size_t)h * dim + d;
      pk[i] = det_u2f((uint32_t)pre[src] << 16);
      pv[i] = det_u2f((uint32_t)pre[(size_t)prefix * kv * dim + src] << 16);
    } else {
      const size_t src = (size_t)(r - prefix) * kv * dim + (size_t)h * dim + d;
      pk[i] = key[src];
      pv[i] = round_v ? round_bf16(value[src]) : value[src];
    }
  }
}

// pack_queries: pq[head][r][d] = q[start + r][head*dim + d] for r < tile.
__global__ void f32_pack_q_kernel(const float* __restrict__ q, float* __restrict__ pq, int start, int tile, int heads,
                                  int dim) {
  const size_t total = (size_t)heads * tile * dim;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % dim), r = (int)((i / dim) % tile), h = (int)(i / ((size_t)dim * tile));
    pq[i] = q[(size_t)(start + r) * heads * dim + (size_t)h * dim + d];
  }
}

// attention_softmax on one score row (head-major rows of the tile): the visible keys are all
// of them (causal < 0) or min(keys, causal + query + 1); scores scaled, max-shifted,
// exponentiated, normalised; invisible entries become 0.
__global__ void __launch_bounds__(kNT) f32_softmax_kernel(float* __restrict__ scores, int stride, int keys, int tile,
                                                          int start, long long causal, float scale) {
  __shared__ float red[kNT / 32];
  __shared__ float bcast;
  float* data = scores + (size_t)blockIdx.x * stride;
  const int query = start + (int)(blockIdx.x % tile);
  const int visible = causal < 0 ? keys : (int)min((long long)keys, causal + query + 1);
  float m = -INFINITY;
  for (int i = threadIdx.x; i < visible; i += kNT) m = fmaxf(m, data[i] * scale);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = -INFINITY;
    for (int w = 0; w < kNT / 32; ++w) t = fmaxf(t, red[w]);
    bcast = t;
  }
  __syncthreads();
  const float mx = bcast;
  float s = 0.f;
  for (int i = threadIdx.x; i < keys; i += kNT) {
    const float e = i < visible ? det_expf(data[i] * scale - mx) : 0.f;
    data[i] = e;
    s += e;
  }
  s = warp_sum(s);
  __syncthreads();  // every thread has read bcast
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kNT / 32; ++w) t += red[w];
    bcast = t;
  }
  __syncthreads();
  const float total = bcast;
  for (int i = threadIdx.x; i < keys; i += kNT) data[i] /= total;
}

// unpack_attention: out[start + r][head*dim + d] = bf16(product[head][r][d]).
__global__ void f32_unpack_kernel(const float* __restrict__ prod, float* __restrict__ out, int start, int tile,
                                  int heads, int dim) {
  const size_t total = (size_t)heads * tile * dim;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % dim), r = (int)((i / dim) % tile), h = (int)(i / ((size_t)dim * tile));
    out[(size_t)(start + r) * heads * dim + (size_t)h * dim + d] = round_bf16(prod[i]);
  }
}

int grid_for(size_t n) { return (int)std::min<size_t>(4096, (n + 255) / 256 + 1); }

// ------------------------------------------------------------------ context
struct F32Ctx {
  std::mutex mu;
  bool init = false;
  int device = 0;
  cudaStream_t stream = nullptr;
  cublasLtHandle_t lt = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 32u << 20;
  // converted weights, keyed like metal.m's `converted` (metal.m:187-190)
  std::map<std::tuple<size_t, const void*, size_t, size_t, int, int>, float*> weights;
  // bf16 prefix K/V blocks of a stack call, keyed (cache, layer, prefix) (metal.m:411-427)
  std::map<std::tuple<size_t, size_t, size_t>, uint16_t*> prefixes;
  std::vector<void*> slot_ptr;
  std::vector<size_t> slot_bytes;
};

F32Ctx& fctx() {
  static F32Ctx c;
  return c;
}

int f_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 1;
  cudaGetLastError();
  fail(0, std::string(what) + ": " + cudaGetErrorString(e));
  return 0;
}

int f_init(F32Ctx& c) {
  if (c.init) return f_ok(cudaSetDevice(c.device), "cudaSetDevice");
  const char* env = getenv("YUE2_CUDA_DEVICE");
  c.device = env ? atoi(env) : 0;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || c.device >= n) {
    cudaGetLastError();
    return fail(0, "no CUDA device");
  }
  if (!f_ok(cudaSetDevice(c.device), "cudaSetDevice") ||
      !f_ok(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking), "stream") ||
      !f_ok(cudaMalloc(&c.ws, c.ws_bytes), "cuBLASLt workspace"))
    return 0;
  if (cublasLtCreate(&c.lt) != CUBLAS_STATUS_SUCCESS) return fail(0, "cublasLtCreate failed");
  c.init = true;
  return 1;
}

// Grow-only device scratch: slot i holds at least `bytes`.
void* slot(F32Ctx& c, size_t i, size_t bytes) {
  if (c.slot_ptr.size() <= i) {
    c.slot_ptr.resize(i + 1, nullptr);
    c.slot_bytes.resize(i + 1, 0);
  }
  if (c.slot_bytes[i] < bytes) {
    if (c.slot_ptr[i]) cudaFree(c.slot_ptr[i]);
    c.slot_ptr[i] = nullptr;
    c.slot_bytes[i] = 0;
    if (!f_ok(cudaMalloc(&c.slot_ptr[i], bytes ? bytes : 16), "scratch allocation")) return nullptr;
    c.slot_bytes[i] = bytes;
  }
  return c.slot_ptr[i];
}

// convert_weight on the host: [rows, cols] as f32.
float* weight_f32(F32Ctx& c, const uint8_t* raw, size_t mapping, size_t rows, size_t cols, int dtype, int rounded) {
  auto key = std::make_tuple(mapping, (const void*)raw, rows, cols, dtype, rounded);
  auto it = c.weights.find(key);
  if (it != c.weights.end()) return it->second;
  if (!raw || dtype < 0 || dtype > 2) {
    fail(0, "unknown weight dtype");
    return nullptr;
  }
  const size_t n = rows * cols;
  std::vector<float> h(n);
  for (size_t i = 0; i < n; ++i) {
    float f;
    if (dtype == YUE2_DTYPE_BF16) {
      uint16_t b;
      memcpy(&b, raw + i * 2, 2);
      f = det_u2f((uint32_t)b << 16);
    } else if (dtype == YUE2_DTYPE_F32) {
      memcpy(&f, raw + i * 4, 4);
    } else {
      uint16_t b;
      memcpy(&b, raw + i * 2, 2);
      const uint32_t sign = (uint32_t)(b >> 15) << 31, ex = (b >> 10) & 0x1f, man = b & 0x3ff;
      if (ex == 0) f = (sign ? -1.f : 1.f) * (float)man * (1.0f / 16777216.0f);
      else if (ex == 31) f = det_u2f(sign | 0x7f800000u | (man << 13));
      else f = det_u2f(sign | ((ex + 112) << 23) | (man << 13));
    }
    if (rounded && dtype != YUE2_DTYPE_BF16) f = round_bf16(f);
    h[i] = f;
  }
  float* dev = nullptr;
  if (!f_ok(cudaMalloc(&dev, n * 4), "weight upload")) return nullptr;
  if (!f_ok(cudaMemcpy(dev, h.data(), n * 4, cudaMemcpyHostToDevice), "weight upload")) {
    cudaFree(dev);
    return nullptr;
  }
  c.weights[key] = dev;
  return dev;
}

int lt_fail(cublasStatus_t st, const char* what) {
  return fail(0, std::string(what) + " failed: cuBLASLt status " + std::to_string((int)st));
}

// C[b] (row-major [m, n], ldc) = A[b] (row-major [m, k], lda) . op(B[b]) + beta C[b], with
// op(B) = B^T of a row-major [n, k] B (trans_b) or a row-major [k, n] B; batch strides in
// elements. f32 in, f32 out, f32 compute (no TF32). Column-major view: C^T = op(B)^T . A^T.
int sgemm(F32Ctx& c, int m, int n, int k, const float* A, long long lda, long long sa, const float* B,
          long long ldb, long long sb, bool trans_b, float* C, long long ldc, long long sc, int batch, float beta) {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasStatus_t st = cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
  int rc = 1;
  auto check = [&](cublasStatus_t s, const char* what) {
    if (rc && s != CUBLAS_STATUS_SUCCESS) rc = lt_fail(s, what);
  };
  check(st, "cublasLtMatmulDescCreate");
  const cublasOperation_t ta = trans_b ? CUBLAS_OP_T : CUBLAS_OP_N, tb = CUBLAS_OP_N;
  if (rc) {
    check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)), "set transa");
    check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)), "set transb");
    // the "A" of cuBLASLt is B's memory: [k, n] column-major (trans_b) or [n, k]
    check(cublasLtMatrixLayoutCreate(&la, CUDA_R_32F, trans_b ? k : n, trans_b ? n : k, ldb), "layout B");
    check(cublasLtMatrixLayoutCreate(&lb, CUDA_R_32F, k, m, lda), "layout A");
    check(cublasLtMatrixLayoutCreate(&lc, CUDA_R_32F, n, m, ldc), "layout C");
  }
  if (rc && batch > 1) {
    const int32_t bc = batch;
    check(cublasLtMatrixLayoutSetAttribute(la, CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT, &bc, sizeof(bc)), "batch");
    check(cublasLtMatrixLayoutSetAttribute(lb, CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT, &bc, sizeof(bc)), "batch");
    check(cublasLtMatrixLayoutSetAttribute(lc, CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT, &bc, sizeof(bc)), "batch");
    const int64_t s1 = sb, s2 = sa, s3 = sc;
    check(cublasLtMatrixLayoutSetAttribute(la, CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET, &s1, sizeof(s1)), "stride");
    check(cublasLtMatrixLayoutSetAttribute(lb, CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET, &s2, sizeof(s2)), "stride");
    check(cublasLtMatrixLayoutSetAttribute(lc, CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET, &s3, sizeof(s3)), "stride");
  }
  cublasLtMatmulHeuristicResult_t heur = {};
  if (rc) {
    cublasLtMatmulPreference_t pref = nullptr;
    check(cublasLtMatmulPreferenceCreate(&pref), "preference");
    if (rc)
      check(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &c.ws_bytes,
                                                 sizeof(c.ws_bytes)),
            "preference workspace");
    int found = 0;
    if (rc) check(cublasLtMatmulAlgoGetHeuristic(c.lt, op, la, lb, lc, lc, pref, 1, &heur, &found), "heuristic");
    if (rc && found == 0) rc = fail(0, "cuBLASLt found no f32 algorithm for the shape");
    if (pref) cublasLtMatmulPreferenceDestroy(pref);
  }
  const float alpha = 1.f;
  if (rc)
    check(cublasLtMatmul(c.lt, op, &alpha, B, la, A, lb, &beta, C, lc, C, lc, &heur.algo, c.ws, c.ws_bytes, c.stream),
          "cublasLtMatmul");
  if (lc) cublasLtMatrixLayoutDestroy(lc);
  if (lb) cublasLtMatrixLayoutDestroy(lb);
  if (la) cublasLtMatrixLayoutDestroy(la);
  if (op) cublasLtMatmulDescDestroy(op);
  return rc;
}

// The attention of metal.m's encodeAttention (metal.m:288-328) on device buffers: q rows
// [rows, heads*dim], packed pk/pv [kv][keys][dim], out [rows, heads*dim] bf16-rounded;
// tiles of at most 256 query rows. Scratch slots 10..12.
int attention_dev(F32Ctx& c, const float* q, const float* pk, const float* pv, float* out, int rows, int keys,
                  int heads, int kv, int dim, long long causal, float scale) {
  const int G = heads / kv, maxTile = std::min(rows, 256), stride = (keys + 15) & ~15;
  float* pq = (float*)slot(c, 10, (size_t)heads * maxTile * dim * 4);
  float* scores = (float*)slot(c, 11, (size_t)heads * maxTile * stride * 4);
  float* prod = (float*)slot(c, 12, (size_t)heads * maxTile * dim * 4);
  if (!pq || !scores || !prod) return 0;
  for (int start = 0; start < rows; start += maxTile) {
    const int tile = std::min(maxTile, rows - start);
    const size_t nq = (size_t)heads * tile * dim;
    f32_pack_q_kernel<<<grid_for(nq), 256, 0, c.stream>>>(q, pq, start, tile, heads, dim);
    if (!f_ok(cudaGetLastError(), "pack_queries")) return 0;
    // scores of kv group g: [G*tile, keys] = pq rows of heads g*G.. . pk[g]^T
    if (!sgemm(c, G * tile, keys, dim, pq, dim, (long long)G * tile * dim, pk, dim, (long long)keys * dim, true,
               scores, stride, (long long)G * tile * stride, kv, 0.f))
      return 0;
    f32_softmax_kernel<<<heads * tile, kNT, 0, c.stream>>>(scores, stride, keys, tile, start, causal, scale);
    if (!f_ok(cudaGetLastError(), "attention_softmax")) return 0;
    if (!sgemm(c, G * tile, dim, keys, scores, stride, (long long)G * tile * stride, pv, dim, (long long)keys * dim,
               false, prod, dim, (long long)G * tile * dim, kv, 0.f))
      return 0;
    f32_unpack_kernel<<<grid_for(nq), 256, 0, c.stream>>>(prod, out, start, tile, heads, dim);
    if (!f_ok(cudaGetLastError(), "unpack_attention")) return 0;
  }
  return 1;
}

int up(F32Ctx& c, void* dst, const void* src, size_t bytes, const char* what) {
  return f_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c.stream), what);
}

}  // namespace

// Called by the decode drop-ins' clear / release hooks (dropin.cu).
void y2_f32_clear(bool release) {
  F32Ctx& c = fctx();
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.init) return;
  cudaSetDevice(c.device);
  cudaStreamSynchronize(c.stream);
  for (auto& kv : c.weights) cudaFree(kv.second);
  c.weights.clear();
  for (auto& kv : c.prefixes) cudaFree(kv.second);
  c.prefixes.clear();
  if (release) {
    for (void* p : c.slot_ptr)
      if (p) cudaFree(p);
    c.slot_ptr.clear();
    c.slot_bytes.clear();
  }
}

void y2_f32_release_cache(size_t cache) {
  F32Ctx& c = fctx();
  std::lock_guard<std::mutex> lock(c.mu);
  if (!c.init) return;
  cudaSetDevice(c.device);
  cudaStreamSynchronize(c.stream);
  for (auto it = c.prefixes.begin(); it != c.prefixes.end();) {
    if (std::get<0>(it->first) == cache) {
      cudaFree(it->second);
      it = c.prefixes.erase(it);
    } else {
      ++it;
    }
  }
}

extern "C" {

int yue2_cuda_gemm(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int transpose_b,
                   size_t lda, size_t ldb, size_t ldc, float beta) {
  F32Ctx& x = fctx();
  std::lock_guard<std::mutex> lock(x.mu);
  if (m == 0 || n == 0) return 1;  // nothing to compute (tensor.rs:805-807)
  if (!a || !b || !c || k == 0 || lda < k || ldb < (transpose_b ? k : n) || ldc < n || m > INT32_MAX ||
      n > INT32_MAX || k > INT32_MAX || lda > INT32_MAX || ldb > INT32_MAX || ldc > INT32_MAX)
    return fail(0, "invalid GEMM shape");
  if (!f_init(x)) return 0;
  const size_t brows = transpose_b ? n : k, bcols = transpose_b ? k : n;
  float* dA = (float*)slot(x, 0, m * k * 4);
  float* dB = (float*)slot(x, 1, brows * bcols * 4);
  float* dC = (float*)slot(x, 2, m * n * 4);
  if (!dA || !dB || !dC) return 0;
  if (!f_ok(cudaMemcpy2DAsync(dA, k * 4, a, lda * 4, k * 4, m, cudaMemcpyHostToDevice, x.stream), "A upload") ||
      !f_ok(cudaMemcpy2DAsync(dB, bcols * 4, b, ldb * 4, bcols * 4, brows, cudaMemcpyHostToDevice, x.stream),
            "B upload"))
    return 0;
  if (beta != 0.f &&
      !f_ok(cudaMemcpy2DAsync(dC, n * 4, c, ldc * 4, n * 4, m, cudaMemcpyHostToDevice, x.stream), "C upload"))
    return 0;
  if (!sgemm(x, (int)m, (int)n, (int)k, dA, (long long)k, 0, dB, (long long)bcols, 0, transpose_b != 0, dC,
             (long long)n, 0, 1, beta))
    return 0;
  if (!f_ok(cudaMemcpy2DAsync(c, ldc * 4, dC, n * 4, n * 4, m, cudaMemcpyDeviceToHost, x.stream), "C download"))
    return 0;
  return f_ok(cudaStreamSynchronize(x.stream), "gemm");
}

int yue2_cuda_linear(const float* a, const uint8_t* weight, size_t mapping, int dtype, int round, float* c, size_t m,
                     size_t n, size_t k) {
  F32Ctx& x = fctx();
  std::lock_guard<std::mutex> lock(x.mu);
  if (!a || !weight || !c || m == 0 || n == 0 || k == 0 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return fail(0, "invalid linear shape");
  if (!f_init(x)) return 0;
  float* w = weight_f32(x, weight, mapping, n, k, dtype, round);
  if (!w) return 0;
  float* dA = (float*)slot(x, 0, m * k * 4);
  float* dC = (float*)slot(x, 2, m * n * 4);
  if (!dA || !dC || !up(x, dA, a, m * k * 4, "input upload")) return 0;
  if (!sgemm(x, (int)m, (int)n, (int)k, dA, (long long)k, 0, w, (long long)k, 0, true, dC, (long long)n, 0, 1, 0.f))
    return 0;
  if (!f_ok(cudaMemcpyAsync(c, dC, m * n * 4, cudaMemcpyDeviceToHost, x.stream), "output download")) return 0;
  return f_ok(cudaStreamSynchronize(x.stream), "linear");
}

int yue2_cuda_attention(const float* q, const float* k, const float* v, float* out, size_t rows, size_t keys,
                        size_t heads, size_t kv, size_t dim, int64_t causal, float scale) {
  F32Ctx& x = fctx();
  std::lock_guard<std::mutex> lock(x.mu);
  if (!q || !k || !v || !out || rows == 0 || keys == 0 || heads == 0 || kv == 0 || dim == 0 || heads % kv ||
      rows > INT32_MAX || keys > INT32_MAX || heads * dim > INT32_MAX || kv * dim > INT32_MAX)
    return fail(0, "invalid attention shape");
  if (!f_init(x)) return 0;
  const size_t qw = heads * dim, kw = kv * dim;
  float* dq = (float*)slot(x, 3, rows * qw * 4);
  float* dk = (float*)slot(x, 4, keys * kw * 4);
  float* dv = (float*)slot(x, 5, keys * kw * 4);
  float* pk = (float*)slot(x, 6, keys * kw * 4);
  float* pv = (float*)slot(x, 7, keys * kw * 4);
  float* dout = (float*)slot(x, 8, rows * qw * 4);
  if (!dq || !dk || !dv || !pk || !pv || !dout) return 0;
  if (!up(x, dq, q, rows * qw * 4, "q upload") || !up(x, dk, k, keys * kw * 4, "k upload") ||
      !up(x, dv, v, keys * kw * 4, "v upload"))
    return 0;
  const size_t nkv = keys * kw;
  f32_pack_kv_kernel<<<grid_for(nkv), 256, 0, x.stream>>>(nullptr, 0, dk, dv, pk, pv, (int)keys, (int)kv, (int)dim, 0);
  if (!f_ok(cudaGetLastError(), "pack_keys_values")) return 0;
  if (!attention_dev(x, dq, pk, pv, dout, (int)rows, (int)keys, (int)heads, (int)kv, (int)dim, causal, scale))
    return 0;
  if (!f_ok(cudaMemcpyAsync(out, dout, rows * qw * 4, cudaMemcpyDeviceToHost, x.stream), "output download")) return 0;
  return f_ok(cudaStreamSynchronize(x.stream), "attention");
}

int yue2_cuda_stack(const float* input, float* out, const Yue2GpuLayer* layers, size_t count, size_t rows,
                    size_t hidden, size_t heads, size_t kv, size_t dim, size_t intermediate, size_t prefix,
                    size_t cache, float eps, const float* cos, const float* sin) {
  F32Ctx& x = fctx();
  std::lock_guard<std::mutex> lock(x.mu);
  if (!input || !out || !layers || !cos || !sin || count == 0 || rows == 0 || hidden == 0 || heads == 0 ||
      kv == 0 || heads % kv || dim == 0 || dim % 2 || intermediate == 0 || rows > INT32_MAX ||
      prefix + rows > INT32_MAX || heads * dim > INT32_MAX || hidden > INT32_MAX || intermediate > INT32_MAX)
    return fail(0, "invalid stack shape");
  for (size_t l = 0; l < count; ++l) {
    const Yue2GpuLayer& L = layers[l];
    const size_t want[7][2] = {{heads * dim, hidden}, {kv * dim, hidden},         {kv * dim, hidden},
                               {hidden, heads * dim}, {intermediate, hidden},      {intermediate, hidden},
                               {hidden, intermediate}};
    for (int j = 0; j < 7; ++j)
      if (!L.weights[j].raw || L.weights[j].rows != want[j][0] || L.weights[j].cols != want[j][1])
        return fail(0, "stack layer " + std::to_string(l) + ": weight " + std::to_string(j) + " has the wrong shape");
    for (int j = 0; j < 4; ++j)
      if (!L.norms[j]) return fail(0, "stack layer " + std::to_string(l) + ": missing norm");
    if (prefix && (!L.key || !L.value)) return fail(0, "stack layer " + std::to_string(l) + ": missing prefix K/V");
  }
  if (!f_init(x)) return 0;
  const size_t qw = heads * dim, kw = kv * dim, keys = prefix + rows, H = hidden, I = intermediate;
  float* X = (float*)slot(x, 20, rows * H * 4);
  float* norm = (float*)slot(x, 21, rows * H * 4);
  float* q = (float*)slot(x, 22, rows * qw * 4);
  float* k = (float*)slot(x, 23, rows * kw * 4);
  float* v = (float*)slot(x, 24, rows * kw * 4);
  float* gate = (float*)slot(x, 25, rows * I * 4);
  float* upb = (float*)slot(x, 26, rows * I * 4);
  float* att = (float*)slot(x, 27, rows * qw * 4);
  float* proj = (float*)slot(x, 28, rows * H * 4);
  float* pk = (float*)slot(x, 6, keys * kw * 4);
  float* pv = (float*)slot(x, 7, keys * kw * 4);
  float* gm = (float*)slot(x, 29, (2 * H + 2 * dim) * 4);
  float* cs = (float*)slot(x, 30, rows * (dim / 2) * 4 * 2);
  if (!X || !norm || !q || !k || !v || !gate || !upb || !att || !proj || !pk || !pv || !gm || !cs) return 0;
  float* sn = cs + rows * (dim / 2);
  if (!up(x, X, input, rows * H * 4, "input upload") || !up(x, cs, cos, rows * (dim / 2) * 4, "cos upload") ||
      !up(x, sn, sin, rows * (dim / 2) * 4, "sin upload"))
    return 0;
  std::vector<uint16_t> pre;
  for (size_t l = 0; l < count; ++l) {
    const Yue2GpuLayer& L = layers[l];
    float* w[7];
    for (int j = 0; j < 7; ++j) {
      const Yue2GpuWeight& s = L.weights[j];
      if (!(w[j] = weight_f32(x, s.raw, s.mapping, s.rows, s.cols, s.dtype, s.rounded))) return 0;
    }
    // the prefix K/V of this layer as bf16 (the f32 rows' top halves, metal.m:417-420)
    uint16_t* pb = nullptr;
    if (prefix) {
      auto key = std::make_tuple(cache, l, prefix);
      auto it = x.prefixes.find(key);
      if (it != x.prefixes.end()) {
        pb = it->second;
      } else {
        pre.resize(2 * prefix * kw);
        for (size_t i = 0; i < prefix * kw; ++i) {
          pre[i] = (uint16_t)(det_f2u(L.key[i]) >> 16);
          pre[prefix * kw + i] = (uint16_t)(det_f2u(L.value[i]) >> 16);
        }
        if (!f_ok(cudaMalloc(&pb, pre.size() * 2), "prefix upload") ||
            !f_ok(cudaMemcpy(pb, pre.data(), pre.size() * 2, cudaMemcpyHostToDevice), "prefix upload"))
          return 0;
        x.prefixes[key] = pb;
      }
    }
    if (!up(x, gm, L.norms[0], H * 4, "norm upload") || !up(x, gm + H, L.norms[1], dim * 4, "norm upload") ||
        !up(x, gm + H + dim, L.norms[2], dim * 4, "norm upload") ||
        !up(x, gm + H + 2 * dim, L.norms[3], H * 4, "norm upload"))
      return 0;
    const int R = (int)rows;
    f32_rms_norm_kernel<<<R, kNT, 0, x.stream>>>(X, gm, norm, (int)H, eps);
    if (!sgemm(x, R, (int)qw, (int)H, norm, H, 0, w[0], H, 0, true, q, qw, 0, 1, 0.f) ||
        !sgemm(x, R, (int)kw, (int)H, norm, H, 0, w[1], H, 0, true, k, kw, 0, 1, 0.f) ||
        !sgemm(x, R, (int)kw, (int)H, norm, H, 0, w[2], H, 0, true, v, kw, 0, 1, 0.f))
      return 0;
    f32_rotary_kernel<<<R * (int)heads, kNT, 0, x.stream>>>(q, gm + H, cs, sn, (int)heads, (int)dim, eps);
    f32_rotary_kernel<<<R * (int)kv, kNT, 0, x.stream>>>(k, gm + H + dim, cs, sn, (int)kv, (int)dim, eps);
    const size_t nkv = keys * kw;
    f32_pack_kv_kernel<<<grid_for(nkv), 256, 0, x.stream>>>(pb, (int)prefix, k, v, pk, pv, (int)keys, (int)kv,
                                                            (int)dim, 1);
    if (!f_ok(cudaGetLastError(), "stack kernels")) return 0;
    if (!attention_dev(x, q, pk, pv, att, R, (int)keys, (int)heads, (int)kv, (int)dim, -1,
                       1.0f / sqrtf((float)dim)))
      return 0;
    if (!sgemm(x, R, (int)H, (int)qw, att, qw, 0, w[3], qw, 0, true, proj, H, 0, 1, 0.f)) return 0;
    f32_pointwise_kernel<<<grid_for(rows * H), 256, 0, x.stream>>>(X, proj, rows * H, 2);
    f32_rms_norm_kernel<<<R, kNT, 0, x.stream>>>(X, gm + H + 2 * dim, norm, (int)H, eps);
    if (!sgemm(x, R, (int)I, (int)H, norm, H, 0, w[4], H, 0, true, gate, I, 0, 1, 0.f) ||
        !sgemm(x, R, (int)I, (int)H, norm, H, 0, w[5], H, 0, true, upb, I, 0, 1, 0.f))
      return 0;
    f32_pointwise_kernel<<<grid_for(rows * I), 256, 0, x.stream>>>(gate, upb, rows * I, 1);
    if (!sgemm(x, R, (int)H, (int)I, gate, I, 0, w[6], I, 0, true, proj, H, 0, 1, 0.f)) return 0;
    f32_pointwise_kernel<<<grid_for(rows * H), 256, 0, x.stream>>>(X, proj, rows * H, 2);
    // every launch of the layer is queued: its host staging buffers must outlive them
    if (!f_ok(cudaGetLastError(), "stack kernels") || !f_ok(cudaStreamSynchronize(x.stream), "stack layer"))
      return 0;
  }
  if (!f_ok(cudaMemcpyAsync(out, X, rows * H * 4, cudaMemcpyDeviceToHost, x.stream), "output download")) return 0;
  return f_ok(cudaStreamSynchronize(x.stream), "stack");
}

}  // extern "C"
