// Drop-in replacements for the Metal imports of the reference's src/tensor.rs:118-219
// (implemented there by src/metal.m). Same argument lists, same 1 = done / 0 = not done
// convention; every 0 leaves a message in yue2_last_error() (the caller must raise it,
// there is no CPU fallback). One process-wide context serialises all calls, as the
// reference's NSLock does (metal.m:21), and keeps uploaded weights and per-(cache,
// layer) device KV contexts between calls.
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
#include "kernels.h"

using namespace y2;

// the f32 imports' context (dropin_f32.cu)
void y2_f32_clear(bool release);
void y2_f32_release_cache(size_t cache);

namespace {

// Gathers the f32 K and V rows of position `pos` of `count` single-layer contexts:
// shadow[l] = [K row (kv*dim), V row (kv*dim)] (metal.m:331-332).
__global__ void gather_shadow_kernel(const DevRow* rows, int count, Geometry g, float* shadow) {
  const int l = blockIdx.x;
  const DevRow r = rows[l];
  const int width = g.kvh * g.dim;
  const uint16_t* page = reinterpret_cast<const uint16_t*>(r.pages[r.pos >> kPageLog2]);
  const int slot = r.pos & (kPageTokens - 1);
  for (int i = threadIdx.x; i < 2 * width; i += blockDim.x) {
    const int kv = i / width, h = (i % width) / g.dim, d = i % g.dim;
    shadow[(size_t)l * 2 * width + i] = bf2f(page[kv_offset(g, 0, kv, h) + (size_t)slot * g.dim + d]);
  }
}

struct Context {  // one (cache, layer) KV mirror: single-layer pages
  std::vector<uint64_t> pages;
  uint64_t* d_pages = nullptr;
  size_t capacity = 0, length = 0;
  int kvh = 0, dim = 0;
};

struct DropIn {
  std::mutex mu;
  bool init = false;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::map<std::tuple<size_t, const void*, size_t, size_t, int>, uint16_t*> weights;
  std::map<std::pair<const float*, size_t>, float*> norms;
  std::map<std::pair<size_t, size_t>, Context> contexts;
  std::map<std::tuple<int, int>, PagePool> pools;  // by (kvh, dim)
  // scratch
  std::vector<void*> scratch;
  size_t cap_hidden = 0, cap_q = 0, cap_kv = 0, cap_inter = 0, cap_count = 0;
  int cap_groups = 0, cap_dim = 0;
  float *x = nullptr, *part = nullptr, *shadow = nullptr, *vec_in = nullptr, *vec_out = nullptr;
  uint16_t *qkv = nullptr, *qrot = nullptr, *attn = nullptr, *hbuf = nullptr;
  int32_t *counters = nullptr, *flags = nullptr;
  DevRow* rows = nullptr;
  float *cos_tab = nullptr, *sin_tab = nullptr;
  size_t vec_cap = 0;
  int sms = 148;
};

DropIn& ctx() {
  static DropIn d;
  return d;
}

int ensure_init(DropIn& d) {
  if (d.init) return 1;
  const char* env = getenv("YUE2_CUDA_DEVICE");
  d.device = env ? atoi(env) : 0;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || d.device >= n) {
    cudaGetLastError();
    return fail(0, "no CUDA device");
  }
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, d.device) != cudaSuccess || p.major != 10) {
    cudaGetLastError();
    return fail(0, "the drop-in path requires an sm_100 (B200) device");
  }
  d.sms = p.multiProcessorCount;
  if (cudaSetDevice(d.device) != cudaSuccess || cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking) != cudaSuccess ||
      prepare_kernels() != cudaSuccess) {
    cudaGetLastError();
    return fail(0, "CUDA initialisation failed");
  }
  d.init = true;
  return 1;
}

// returns 1 on success, 0 with a message otherwise
int ok_or(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 1;
  cudaGetLastError();
  fail(0, std::string(what) + ": " + cudaGetErrorString(e));
  return 0;
}

int dalloc(DropIn& d, void** p, size_t bytes) {
  if (!ok_or(cudaMalloc(p, bytes ? bytes : 16), "cudaMalloc")) return 0;
  d.scratch.push_back(*p);
  return 1;
}

void free_scratch(DropIn& d) {
  for (void* p : d.scratch) cudaFree(p);
  d.scratch.clear();
  d.cap_hidden = d.cap_q = d.cap_kv = d.cap_inter = d.cap_count = 0;
  d.cap_groups = d.cap_dim = 0;
  d.vec_cap = 0;
}

// Workspace for one row of a stack with the given shape.
int ensure_scratch(DropIn& d, size_t hidden, size_t heads, size_t kv, size_t dim, size_t inter, size_t count) {
  const size_t q = heads * dim, kd = kv * dim;
  const int groups = (int)(heads / kv);
  if (hidden <= d.cap_hidden && q <= d.cap_q && kd <= d.cap_kv && inter <= d.cap_inter && count <= d.cap_count &&
      groups <= d.cap_groups && (int)dim <= d.cap_dim)
    return 1;
  const size_t keep_vec = d.vec_cap;
  free_scratch(d);
  hidden = std::max(hidden, (size_t)1);
  count = std::max(count, (size_t)1);
  const int splits = 64;
  if (!dalloc(d, (void**)&d.x, hidden * 4) || !dalloc(d, (void**)&d.qkv, (q + 2 * kd) * 2) ||
      !dalloc(d, (void**)&d.qrot, q * 2) || !dalloc(d, (void**)&d.attn, q * 2) ||
      !dalloc(d, (void**)&d.hbuf, std::max(inter, (size_t)8) * 2) ||
      !dalloc(d, (void**)&d.part, kv * splits * groups * (dim + 2) * 4) || !dalloc(d, (void**)&d.counters, kv * 4) ||
      !dalloc(d, (void**)&d.flags, 64) || !dalloc(d, (void**)&d.rows, count * sizeof(DevRow)) ||
      !dalloc(d, (void**)&d.shadow, count * 2 * kd * 4) ||
      !dalloc(d, (void**)&d.cos_tab, (size_t)kContext * dim / 2 * 4) ||
      !dalloc(d, (void**)&d.sin_tab, (size_t)kContext * dim / 2 * 4))
    return 0;
  if (!ok_or(cudaMemset(d.counters, 0, kv * 4), "memset") || !ok_or(cudaMemset(d.flags, 0, 64), "memset")) return 0;
  d.cap_hidden = hidden;
  d.cap_q = q;
  d.cap_kv = kd;
  d.cap_inter = inter;
  d.cap_count = count;
  d.cap_groups = groups;
  d.cap_dim = (int)dim;
  (void)keep_vec;
  return 1;
}

// Uploads (once) a GpuWeight as bf16, keyed like metal.m's vector cache (metal.m:552).
uint16_t* weight(DropIn& d, const uint8_t* raw, size_t mapping, size_t rows, size_t cols, int dtype, int rounded) {
  auto key = std::make_tuple(mapping, (const void*)raw, rows, cols, dtype);
  auto it = d.weights.find(key);
  if (it != d.weights.end()) return it->second;
  if (dtype < 0 || dtype > 2) {
    fail(0, "unknown weight dtype");
    return nullptr;
  }
  if (dtype != YUE2_DTYPE_BF16 && !rounded) {
    fail(0, "unrounded F32/F16 weights are not supported on the bf16 decode path");
    return nullptr;
  }
  const size_t n = rows * cols;
  uint16_t* dev = nullptr;
  if (!ok_or(cudaMalloc(&dev, n * 2), "weight upload")) return nullptr;
  cudaError_t e;
  if (dtype == YUE2_DTYPE_BF16) {
    e = cudaMemcpy(dev, raw, n * 2, cudaMemcpyHostToDevice);
  } else {
    std::vector<uint16_t> h(n);
    for (size_t i = 0; i < n; ++i) {
      float f;
      if (dtype == YUE2_DTYPE_F32) {
        memcpy(&f, raw + i * 4, 4);
      } else {
        uint16_t b;
        memcpy(&b, raw + i * 2, 2);
        const uint32_t sign = (uint32_t)(b >> 15) << 31, ex = (b >> 10) & 0x1f, man = b & 0x3ff;
        if (ex == 0) f = (sign ? -1.f : 1.f) * (float)man * (1.0f / 16777216.0f);
        else if (ex == 31) f = det_u2f(sign | 0x7f800000u | (man << 13));
        else f = det_u2f(sign | ((ex + 112) << 23) | (man << 13));
      }
      h[i] = (uint16_t)(det_f2u(round_bf16(f)) >> 16);
    }
    e = cudaMemcpy(dev, h.data(), n * 2, cudaMemcpyHostToDevice);
  }
  if (!ok_or(e, "weight upload")) {
    cudaFree(dev);
    return nullptr;
  }
  d.weights[key] = dev;
  return dev;
}

float* norm(DropIn& d, const float* host, size_t len) {
  auto key = std::make_pair(host, len);
  auto it = d.norms.find(key);
  if (it != d.norms.end()) return it->second;
  float* dev = nullptr;
  if (!ok_or(cudaMalloc(&dev, len * 4), "norm upload")) return nullptr;
  if (!ok_or(cudaMemcpy(dev, host, len * 4, cudaMemcpyHostToDevice), "norm upload")) {
    cudaFree(dev);
    return nullptr;
  }
  d.norms[key] = dev;
  return dev;
}

void drop_context(DropIn& d, Context& c) {
  auto& pool = d.pools[std::make_tuple(c.kvh, c.dim)];
  pool.give(c.pages);
  if (c.d_pages) cudaFree(c.d_pages);
  c = Context{};
}

// Mirror of metal.m contextEntry (metal.m:633-668): the device context of (cache, layer)
// holds the host rows [0, keys) and has room for `extra` more.
Context* context(DropIn& d, const float* k, const float* v, size_t keys, size_t kv, size_t dim, size_t cache,
                 size_t layer, size_t extra) {
  Context& c = d.contexts[std::make_pair(cache, layer)];
  if (c.d_pages && (c.capacity < keys + extra || c.length > keys || c.kvh != (int)kv || c.dim != (int)dim))
    drop_context(d, c);
  if (!c.d_pages) {
    c.kvh = (int)kv;
    c.dim = (int)dim;
    c.capacity = (keys + extra + 127) & ~(size_t)127;
    const size_t npages = (c.capacity + kPageTokens - 1) / kPageTokens;
    Geometry g1{1, 1, (int)kv, (int)dim, 1, 1, 1, 0.f};
    auto& pool = d.pools[std::make_tuple(c.kvh, c.dim)];
    pool.page_bytes = page_bytes(g1);
    if (pool.take(npages, c.pages)) {
      c.pages.clear();
      fail(0, "KV context allocation failed");
      return nullptr;
    }
    if (!ok_or(cudaMalloc(&c.d_pages, npages * 8), "page table") ||
        !ok_or(cudaMemcpy(c.d_pages, c.pages.data(), npages * 8, cudaMemcpyHostToDevice), "page table")) {
      drop_context(d, c);
      return nullptr;
    }
    c.length = 0;
  }
  if (keys > c.length) {  // upload the new host rows (bf16 = top half of the bf16-valued f32)
    Geometry g1{1, 1, (int)kv, (int)dim, 1, 1, 1, 0.f};
    std::vector<uint16_t> kb(dim), vb(dim);
    for (size_t row = c.length; row < keys; ++row)
      for (size_t h = 0; h < kv; ++h) {
        for (size_t e = 0; e < dim; ++e) {
          kb[e] = (uint16_t)(det_f2u(k[row * kv * dim + h * dim + e]) >> 16);
          vb[e] = (uint16_t)(det_f2u(v[row * kv * dim + h * dim + e]) >> 16);
        }
        char* page = (char*)c.pages[row / kPageTokens];
        const size_t slot = row % kPageTokens;
        if (!ok_or(cudaMemcpyAsync(page + (kv_offset(g1, 0, 0, (int)h) + slot * dim) * 2, kb.data(), dim * 2,
                                   cudaMemcpyHostToDevice, d.stream),
                   "context upload") ||
            !ok_or(cudaMemcpyAsync(page + (kv_offset(g1, 0, 1, (int)h) + slot * dim) * 2, vb.data(), dim * 2,
                                   cudaMemcpyHostToDevice, d.stream),
                   "context upload") ||
            !ok_or(cudaStreamSynchronize(d.stream), "context upload"))
          return nullptr;
      }
    c.length = keys;
  }
  return &c;
}

void clear_all(DropIn& d) {
  for (auto& kv : d.weights) cudaFree(kv.second);
  d.weights.clear();
  for (auto& kv : d.norms) cudaFree(kv.second);
  d.norms.clear();
  for (auto& kv : d.contexts) drop_context(d, kv.second);
  d.contexts.clear();
  for (auto& kv : d.pools) kv.second.clear();
  d.pools.clear();
}

}  // namespace

extern "C" {

int yue2_cuda_available(void) {
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  return ensure_init(d) != 0 ? 1 : 0;
}

int yue2_cuda_vector_default(void) { return yue2_cuda_available(); }

const char* yue2_cuda_name(void) {
  static char name[256] = "CPU";
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (ensure_init(d)) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, d.device) == cudaSuccess) snprintf(name, sizeof(name), "%s", p.name);
  }
  return name;
}

void yue2_cuda_clear_weights(void) {
  y2_f32_clear(false);
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!d.init) return;
  cudaSetDevice(d.device);
  cudaStreamSynchronize(d.stream);
  clear_all(d);
}

void yue2_cuda_release_model(void) {
  y2_f32_clear(true);
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!d.init) return;
  cudaSetDevice(d.device);
  cudaStreamSynchronize(d.stream);
  clear_all(d);
  free_scratch(d);
}

void yue2_cuda_release_cache(size_t cache) {
  y2_f32_release_cache(cache);
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!d.init) return;
  cudaSetDevice(d.device);
  cudaStreamSynchronize(d.stream);
  for (auto it = d.contexts.begin(); it != d.contexts.end();) {
    if (it->first.first == cache) {
      drop_context(d, it->second);
      it = d.contexts.erase(it);
    } else {
      ++it;
    }
  }
}

int yue2_cuda_vector(const float* input, const uint8_t* raw, size_t mapping, int dtype, int rounded, int priority,
                     float* out, size_t rows, size_t cols) {
  (void)priority;
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!ensure_init(d)) return 0;
  if (!input || !raw || !out || rows == 0 || cols == 0) return fail(0, "null argument or empty shape");
  if (cols % 8 || rows > 0x7fffffff || cols > 32768) return fail(0, "cols must be a multiple of 8 (<= 32768)");
  if (!ok_or(cudaSetDevice(d.device), "cudaSetDevice")) return 0;
  uint16_t* w = weight(d, raw, mapping, rows, cols, dtype, rounded);
  if (!w) return 0;
  if (rows + cols > d.vec_cap) {
    float* p = nullptr;
    if (!dalloc(d, (void**)&p, (rows + cols) * 4)) return 0;
    d.vec_in = p;
    d.vec_out = p + cols;
    d.vec_cap = rows + cols;
  } else {
    d.vec_out = d.vec_in + cols;
  }
  if (!ok_or(cudaMemcpyAsync(d.vec_in, input, cols * 4, cudaMemcpyHostToDevice, d.stream), "input upload"))
    return 0;
  GemvParams p = {};
  p.w[0] = p.w[1] = p.w[2] = w;
  p.seg_start[1] = p.seg_start[2] = (int)rows;
  p.N = (int)rows;
  p.K = (int)cols;
  p.R = 1;
  p.xf = d.vec_in;
  p.of = d.vec_out;
  p.ldo = (int)rows;
  if (!ok_or(launch_gemv(d.stream, false, kXF32, kEpiRawF32, p, 2 * d.sms), "weight_vector launch")) return 0;
  if (!ok_or(cudaMemcpyAsync(out, d.vec_out, rows * 4, cudaMemcpyDeviceToHost, d.stream), "output copy")) return 0;
  return ok_or(cudaStreamSynchronize(d.stream), "weight_vector");
}

int yue2_cuda_cached_attention(const float* q, const float* k, const float* v, float* out, size_t keys,
                               size_t heads, size_t kv, size_t dim, size_t cache, size_t layer) {
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!ensure_init(d)) return 0;
  // metal.m:688 gate
  if (!q || !k || !v || !out || keys == 0 || keys > (size_t)kContext || dim == 0 || kv == 0 || heads == 0 ||
      heads % kv)
    return fail(0, "invalid cached attention shape");
  if (dim != 64 && dim != 128 && dim != 256) return fail(0, "head dim must be 64, 128 or 256");
  const size_t G = heads / kv;
  if (G != 1 && G != 2 && G != 3 && G != 4 && G != 8) return fail(0, "unsupported grouped-query factor");
  if (!ok_or(cudaSetDevice(d.device), "cudaSetDevice")) return 0;
  if (!ensure_scratch(d, 8, heads, kv, dim, 8, 1)) return 0;
  Context* c = context(d, k, v, keys, kv, dim, cache, layer, 0);
  if (!c) return 0;
  std::vector<uint16_t> qb(heads * dim);
  for (size_t i = 0; i < qb.size(); ++i) qb[i] = (uint16_t)(det_f2u(round_bf16(q[i])) >> 16);
  DevRow row = {};
  row.pages = c->d_pages;
  row.pos = (int32_t)(keys - 1);
  row.active = 1;
  if (!ok_or(cudaMemcpyAsync(d.qrot, qb.data(), qb.size() * 2, cudaMemcpyHostToDevice, d.stream), "q upload") ||
      !ok_or(cudaMemcpyAsync(d.rows, &row, sizeof(row), cudaMemcpyHostToDevice, d.stream), "row upload"))
    return 0;
  AttnParams ap = {};
  ap.rows = d.rows;
  ap.q = d.qrot;
  ap.out = d.attn;
  ap.part = d.part;
  ap.counters = d.counters;
  ap.g = Geometry{(int)(heads * dim), (int)heads, (int)kv, (int)dim, 1, 1, 1, 0.f};
  ap.layer = 0;
  ap.splits = std::max(1, std::min(64, (2 * d.sms + (int)kv - 1) / (int)kv));
  ap.scale = 1.0f / sqrtf((float)dim);
  ap.pipe = attn_pipe_for_keys((int)keys, ap.splits);  // the engine's choice of tile loop
  if (!ok_or(launch_attention(d.stream, false, ap, 1), "attention launch")) return 0;
  std::vector<uint16_t> ob(heads * dim);
  if (!ok_or(cudaMemcpyAsync(ob.data(), d.attn, ob.size() * 2, cudaMemcpyDeviceToHost, d.stream), "output") ||
      !ok_or(cudaStreamSynchronize(d.stream), "cached attention"))
    return 0;
  for (size_t i = 0; i < ob.size(); ++i) out[i] = det_u2f((uint32_t)ob[i] << 16);
  return 1;
}

int yue2_cuda_ar_stack(const float* input, float* out, float* shadow, const Yue2GpuLayer* layers, size_t count,
                       size_t hidden, size_t heads, size_t kv, size_t dim, size_t intermediate, size_t prefix,
                       size_t capacity, size_t cache, float eps, const float* cos, const float* sin) {
  DropIn& d = ctx();
  std::lock_guard<std::mutex> lock(d.mu);
  if (!ensure_init(d)) return 0;
  // metal.m:721 gate
  if (!input || !out || !shadow || !layers || !cos || !sin || !count || !kv || !dim || !heads ||
      prefix >= (size_t)kContext || capacity <= prefix || capacity > (size_t)kContext || heads % kv)
    return fail(0, "invalid AR stack arguments");
  if (dim != 64 && dim != 128 && dim != 256) return fail(0, "head dim must be 64, 128 or 256");
  const size_t G = heads / kv;
  if (G != 1 && G != 2 && G != 3 && G != 4 && G != 8) return fail(0, "unsupported grouped-query factor");
  if (hidden % 8 || intermediate % 8 || (heads * dim) % 8) return fail(0, "widths must be multiples of 8");
  const size_t qd = heads * dim, kd = kv * dim;
  const size_t shapes[7][2] = {{qd, hidden}, {kd, hidden}, {kd, hidden}, {hidden, qd},
                               {intermediate, hidden}, {intermediate, hidden}, {hidden, intermediate}};
  for (size_t l = 0; l < count; ++l)
    for (int j = 0; j < 7; ++j)
      if (layers[l].weights[j].rows != shapes[j][0] || layers[l].weights[j].cols != shapes[j][1] ||
          !layers[l].weights[j].raw)
        return fail(0, "AR stack weight shape mismatch");
  if (!ok_or(cudaSetDevice(d.device), "cudaSetDevice")) return 0;
  if (!ensure_scratch(d, hidden, heads, kv, dim, intermediate, count)) return 0;
  const Geometry g1{(int)hidden, (int)heads, (int)kv, (int)dim, (int)intermediate, 1, 1, eps};
  // weights, norms and KV contexts for every layer
  std::vector<LayerW> w(count);
  std::vector<DevRow> rows(count);
  for (size_t l = 0; l < count; ++l) {
    const Yue2GpuLayer& L = layers[l];
    const uint16_t* ws[7];
    for (int j = 0; j < 7; ++j) {
      const Yue2GpuWeight& gw = L.weights[j];
      ws[j] = weight(d, gw.raw, gw.mapping, gw.rows, gw.cols, gw.dtype, gw.rounded);
      if (!ws[j]) return 0;
    }
    w[l] = LayerW{ws[0], ws[1], ws[2], ws[3], ws[4], ws[5], ws[6], norm(d, L.norms[0], hidden),
                  norm(d, L.norms[1], dim), norm(d, L.norms[2], dim), norm(d, L.norms[3], hidden)};
    if (!w[l].in_norm || !w[l].q_norm || !w[l].k_norm || !w[l].post_norm) return 0;
    Context* c = context(d, L.key, L.value, prefix, kv, dim, cache, l, capacity - prefix);
    if (!c) return 0;
    rows[l] = DevRow{};
    rows[l].pages = c->d_pages;
    rows[l].pos = (int32_t)prefix;
    rows[l].active = 1;
  }
  // this position's rotary row (the caller's Rotary::new(prefix, 1))
  const size_t half = dim / 2;
  if (!ok_or(cudaMemcpyAsync(d.cos_tab + prefix * half, cos, half * 4, cudaMemcpyHostToDevice, d.stream), "cos") ||
      !ok_or(cudaMemcpyAsync(d.sin_tab + prefix * half, sin, half * 4, cudaMemcpyHostToDevice, d.stream), "sin") ||
      !ok_or(cudaMemcpyAsync(d.rows, rows.data(), count * sizeof(DevRow), cudaMemcpyHostToDevice, d.stream),
             "rows") ||
      !ok_or(cudaMemcpyAsync(d.x, input, hidden * 4, cudaMemcpyHostToDevice, d.stream), "input"))
    return 0;
  const int grid = 2 * d.sms;
  for (size_t l = 0; l < count; ++l) {
    GemvParams p = {};
    p.w[0] = w[l].q;
    p.w[1] = w[l].k;
    p.w[2] = w[l].v;
    p.seg_start[1] = (int)qd;
    p.seg_start[2] = (int)(qd + kd);
    p.col0[1] = (int)qd;
    p.col0[2] = (int)(qd + kd);
    p.N = (int)(qd + 2 * kd);
    p.K = (int)hidden;
    p.R = 1;
    p.xf = d.x;
    p.gamma = w[l].in_norm;
    p.eps = eps;
    p.ob = d.qkv;
    p.ldo = p.N;
    if (!ok_or(launch_gemv(d.stream, true, kXNorm, kEpiBf16, p, grid), "qkv")) return 0;
    RopeParams rp = {};
    rp.rows = d.rows + l;
    rp.qkv = d.qkv;
    rp.q_out = d.qrot;
    rp.cos_tab = d.cos_tab;
    rp.sin_tab = d.sin_tab;
    rp.q_norm = w[l].q_norm;
    rp.k_norm = w[l].k_norm;
    rp.g = g1;
    rp.layer = 0;
    rp.max_pos = (int)kContext;
    rp.error = d.flags;
    if (!ok_or(launch_rope_append(d.stream, true, rp, 1), "rope")) return 0;
    AttnParams ap = {};
    ap.rows = d.rows + l;
    ap.q = d.qrot;
    ap.out = d.attn;
    ap.part = d.part;
    ap.counters = d.counters;
    ap.g = g1;
    ap.layer = 0;
    ap.splits = std::max(1, std::min(64, (2 * d.sms + (int)kv - 1) / (int)kv));
    ap.scale = 1.0f / sqrtf((float)dim);
    if (!ok_or(launch_attention(d.stream, true, ap, 1), "attention")) return 0;
    p = GemvParams{};
    p.w[0] = p.w[1] = p.w[2] = w[l].o;
    p.seg_start[1] = p.seg_start[2] = (int)hidden;
    p.N = (int)hidden;
    p.K = (int)qd;
    p.R = 1;
    p.xb = d.attn;
    p.of = d.x;
    p.ldo = (int)hidden;
    if (!ok_or(launch_gemv(d.stream, true, kXBf16, kEpiResidual, p, grid), "o")) return 0;
    p = GemvParams{};
    p.w[0] = p.w[1] = p.w[2] = w[l].gate;
    p.wpair = w[l].up;
    p.seg_start[1] = p.seg_start[2] = (int)intermediate;
    p.N = (int)intermediate;
    p.K = (int)hidden;
    p.R = 1;
    p.xf = d.x;
    p.gamma = w[l].post_norm;
    p.eps = eps;
    p.ob = d.hbuf;
    p.ldo = (int)intermediate;
    if (!ok_or(launch_gemv(d.stream, true, kXNorm, kEpiSwiGLU, p, grid), "gate/up")) return 0;
    p = GemvParams{};
    p.w[0] = p.w[1] = p.w[2] = w[l].down;
    p.seg_start[1] = p.seg_start[2] = (int)hidden;
    p.N = (int)hidden;
    p.K = (int)intermediate;
    p.R = 1;
    p.xb = d.hbuf;
    p.of = d.x;
    p.ldo = (int)hidden;
    if (!ok_or(launch_gemv(d.stream, true, kXBf16, kEpiResidual, p, grid), "down")) return 0;
  }
  gather_shadow_kernel<<<(unsigned)count, 256, 0, d.stream>>>(d.rows, (int)count, g1, d.shadow);
  if (!ok_or(cudaGetLastError(), "shadow gather")) return 0;
  if (!ok_or(cudaMemcpyAsync(out, d.x, hidden * 4, cudaMemcpyDeviceToHost, d.stream), "output") ||
      !ok_or(cudaMemcpyAsync(shadow, d.shadow, count * 2 * kd * 4, cudaMemcpyDeviceToHost, d.stream), "shadow") ||
      !ok_or(cudaStreamSynchronize(d.stream), "AR stack"))
    return 0;
  for (size_t l = 0; l < count; ++l) d.contexts[std::make_pair(cache, l)].length = prefix + 1;
  return 1;
}

}  // extern "C"
