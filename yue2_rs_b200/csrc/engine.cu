// Host engine of libyue2cuda: device model, paged KV caches, step encoding (PDL chain),
// CUDA-graph capture and the decode loops that replace the reference's per-step host
// work (src/sampling.rs:222-294, src/model.rs:465-591).
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "detmath.h"
#include "engine.h"
#include "kernels.h"

using namespace y2;

namespace y2 {

thread_local std::string g_error;

int fail(int code, const std::string& msg) {
  g_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? YUE2_ERR_OOM : YUE2_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #expr);   \
  } while (0)

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  char* end = nullptr;
  long x = strtol(v, &end, 10);
  return (end && *end == '\0') ? (int)x : dflt;
}

// ---------------------------------------------------------------- page pool
int PagePool::take(size_t n, std::vector<uint64_t>& out) {
  if (free_pages.size() < n) {
    const size_t need = n - free_pages.size();
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, need * page_bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(YUE2_ERR_OOM, "KV page pool: cannot allocate " + std::to_string(need) + " pages of " +
                                    std::to_string(page_bytes) + " bytes");
    }
    chunks.push_back(p);
    for (size_t i = 0; i < need; ++i) free_pages.push_back((uint64_t)p + i * page_bytes);
  }
  for (size_t i = 0; i < n; ++i) {
    out.push_back(free_pages.back());
    free_pages.pop_back();
  }
  return 0;
}

void PagePool::give(const std::vector<uint64_t>& pages) {
  free_pages.insert(free_pages.end(), pages.begin(), pages.end());
}

void PagePool::clear() {
  for (void* p : chunks) cudaFree(p);
  chunks.clear();
  free_pages.clear();
}

}  // namespace y2

// ---------------------------------------------------------------- model
namespace {

inline uint16_t f32_to_bf16_bits(float f) { return (uint16_t)(det_f2u(round_bf16(f)) >> 16); }
inline float bf16_bits_to_f32(uint16_t b) { return det_u2f((uint32_t)b << 16); }

float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  if (exp == 0) {
    if (man == 0) return det_u2f(sign);
    float v = (float)man * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  if (exp == 31) return det_u2f(sign | 0x7f800000u | (man << 13));
  return det_u2f(sign | ((exp + 112) << 23) | (man << 13));
}

float host_value(int dtype, const void* data, size_t i) {
  if (dtype == YUE2_DTYPE_BF16) return bf16_bits_to_f32(((const uint16_t*)data)[i]);
  if (dtype == YUE2_DTYPE_F32) return ((const float*)data)[i];
  return half_to_float(((const uint16_t*)data)[i]);
}

}  // namespace

int y2_set_device(const Yue2Model* m) {
  CK(cudaSetDevice(m->device));
  return 0;
}

Yue2Model::~Yue2Model() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
  y2::free_prefill(prefill);
  for (auto& e : row_events)
    if (e) cudaEventDestroy(e);
  pool.clear();
  for (void* p : tp_opened) cudaIpcCloseMemHandle(p);
  for (void* p : allocations) cudaFree(p);
  if (pinned_rows) cudaFreeHost(pinned_rows);
  if (pinned_flags) cudaFreeHost(pinned_flags);
  if (stream) cudaStreamDestroy(stream);
  if (side) cudaStreamDestroy(side);
  if (ev_fork) cudaEventDestroy(ev_fork);
  if (ev_join) cudaEventDestroy(ev_join);
}

// The smallest cached buffer of at least `bytes` (and at most twice that), else a new one.
int Yue2Model::scratch_take(void** p, size_t bytes) {
  bytes = (bytes + 255) & ~(size_t)255;
  auto it = scratch_free.lower_bound(bytes);
  if (it != scratch_free.end() && it->first <= 2 * bytes) {
    *p = it->second;
    scratch_free.erase(it);
    return 0;
  }
  const int rc = alloc(p, bytes);
  if (!rc) scratch_cap[*p] = bytes;
  return rc;
}

void Yue2Model::scratch_give(void* p) {
  if (!p) return;
  auto it = scratch_cap.find(p);
  if (it != scratch_cap.end()) scratch_free.emplace(it->second, p);
}

int Yue2Model::alloc(void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(YUE2_ERR_OOM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  }
  allocations.push_back(*p);
  return 0;
}

extern "C" {

const char* yue2_last_error(void) { return y2::g_error.c_str(); }

static int create_model(int device, const Yue2Config* cfg, uint64_t tp_rank, uint64_t tp_world, Yue2Model** out);

int yue2_model_create(int device, const Yue2Config* cfg, Yue2Model** out) {
  return create_model(device, cfg, 0, 1, out);
}

int yue2_model_create_tp(int device, const Yue2Config* cfg, uint64_t tp_rank, uint64_t tp_world, Yue2Model** out) {
  if (!cfg || !out) return fail(YUE2_ERR_INVALID, "null argument");
  if (tp_world < 1 || tp_world > (uint64_t)kTpMaxWorld || tp_rank >= tp_world)
    return fail(YUE2_ERR_INVALID, "tensor-parallel rank/world out of range (world at most 8)");
  if (cfg->num_attention_heads % tp_world || cfg->num_key_value_heads % tp_world || cfg->intermediate_size % tp_world ||
      (cfg->intermediate_size / tp_world) % 8 || cfg->vocab_size < tp_world)
    return fail(YUE2_ERR_INVALID, "heads, KV heads and intermediate size must split evenly over the ranks");
  return create_model(device, cfg, tp_rank, tp_world, out);
}

static int create_model(int device, const Yue2Config* cfg, uint64_t tp_rank, uint64_t tp_world, Yue2Model** out) {
  if (!cfg || !out) return fail(YUE2_ERR_INVALID, "null argument");
  *out = nullptr;
  const Yue2Config& c = *cfg;
  // Config::read validation (src/model.rs:50-72)
  if (!c.hidden_size || !c.num_hidden_layers || !c.num_attention_heads || !c.num_key_value_heads || !c.head_dim ||
      !c.intermediate_size || !c.vocab_size || c.num_attention_heads % c.num_key_value_heads || c.head_dim % 2 ||
      !(c.rope_theta > 0.f) || !std::isfinite(c.rope_theta) || !(c.rms_norm_eps > 0.f) ||
      !std::isfinite(c.rms_norm_eps) || !c.max_position_embeddings)
    return fail(YUE2_ERR_INVALID, "Invalid transformer configuration");
  if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
    return fail(YUE2_ERR_INVALID, "head_dim must be 64, 128 or 256");
  const uint64_t G = c.num_attention_heads / c.num_key_value_heads;
  if (G != 1 && G != 2 && G != 3 && G != 4 && G != 8)
    return fail(YUE2_ERR_INVALID, "grouped-query factor must be 1, 2, 3, 4 or 8");
  if (c.hidden_size % 8 || c.intermediate_size % 8 || c.vocab_size > (1ull << 30) || c.hidden_size > 32768 ||
      c.intermediate_size > 65536)
    return fail(YUE2_ERR_INVALID, "hidden and intermediate sizes must be multiples of 8 (and bounded)");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return fail(YUE2_ERR_CUDA, "no CUDA device " + std::to_string(device));
  }
  Yue2Model* m = new Yue2Model();
  m->device = device;
  m->cfg = c;
  const uint64_t TP = tp_world;  // this rank's share of heads, KV heads, MLP rows and vocabulary
  m->tp_rank = (int)tp_rank;
  m->tp_world = (int)TP;
  m->head_row0 = (int)(c.vocab_size * tp_rank / TP);
  m->head_rows = (int)(c.vocab_size * (tp_rank + 1) / TP) - m->head_row0;
  m->g = Geometry{(int)c.hidden_size, (int)(c.num_attention_heads / TP), (int)(c.num_key_value_heads / TP),
                  (int)c.head_dim, (int)(c.intermediate_size / TP), (int)c.vocab_size, (int)c.num_hidden_layers,
                  c.rms_norm_eps};
  int rc = y2_set_device(m);
  if (rc) {
    delete m;
    return rc;
  }
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
    delete m;
    return cuda_fail(e, "cudaGetDeviceProperties");
  }
  m->sms = prop.multiProcessorCount;
  m->pool.page_bytes = page_bytes(m->g);
  // ---- weight arena: one allocation, 256-byte aligned sub-buffers
  const size_t H = c.hidden_size, V = c.vocab_size, D = c.head_dim;
  const size_t I = m->g.inter, qd = (size_t)m->g.heads * D, kd = (size_t)m->g.kvh * D;  // this rank's share
  const size_t r = tp_rank;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  size_t total = 0;
  std::vector<std::pair<std::string, TensorSlot>> plan;
  // rows x cols of the full [frows, fcols] tensor from (row0, col0)
  auto add = [&](const std::string& name, size_t rows, size_t cols, bool norm, size_t frows = 0, size_t fcols = 0,
                 size_t row0 = 0, size_t col0 = 0) {
    TensorSlot t;
    t.rows = rows;
    t.cols = cols;
    t.norm = norm;
    t.offset = total;
    t.full_rows = frows ? frows : rows;
    t.full_cols = fcols ? fcols : cols;
    t.row0 = row0;
    t.col0 = col0;
    total += al(rows * cols * (norm ? 4 : 2));
    plan.push_back({name, t});
  };
  add("model.embed_tokens.weight", V, H, false);
  if (!c.tie_word_embeddings) add("lm_head.weight", m->head_rows, H, false, V, H, m->head_row0, 0);
  add("model.norm.weight", 1, H, true);
  for (uint64_t l = 0; l < c.num_hidden_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    // column split (output rows) of q|k|v by heads and of gate|up; row split (input
    // columns) of o and down
    add(p + "self_attn.q_proj.weight", qd, H, false, qd * TP, H, r * qd, 0);
    add(p + "self_attn.k_proj.weight", kd, H, false, kd * TP, H, r * kd, 0);
    add(p + "self_attn.v_proj.weight", kd, H, false, kd * TP, H, r * kd, 0);
    add(p + "self_attn.o_proj.weight", H, qd, false, H, qd * TP, 0, r * qd);
    add(p + "mlp.gate_proj.weight", I, H, false, I * TP, H, r * I, 0);
    add(p + "mlp.up_proj.weight", I, H, false, I * TP, H, r * I, 0);
    add(p + "mlp.down_proj.weight", H, I, false, H, I * TP, 0, r * I);
    add(p + "input_layernorm.weight", 1, H, true);
    add(p + "self_attn.q_norm.weight", 1, D, true);
    add(p + "self_attn.k_norm.weight", 1, D, true);
    add(p + "post_attention_layernorm.weight", 1, H, true);
  }
  void* arena = nullptr;
  if ((rc = m->alloc(&arena, total))) {
    delete m;
    return rc;
  }
  m->arena = (char*)arena;
  for (auto& kv : plan) m->slots[kv.first] = kv.second;
  auto ptr = [&](const std::string& n) { return (void*)(m->arena + m->slots[n].offset); };
  m->embed = (uint16_t*)ptr("model.embed_tokens.weight");
  m->lm_head = c.tie_word_embeddings ? m->embed + (size_t)m->head_row0 * H : (uint16_t*)ptr("lm_head.weight");
  m->final_norm = (float*)ptr("model.norm.weight");
  m->layers.resize(c.num_hidden_layers);
  for (uint64_t l = 0; l < c.num_hidden_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    LayerW& w = m->layers[l];
    w.q = (uint16_t*)ptr(p + "self_attn.q_proj.weight");
    w.k = (uint16_t*)ptr(p + "self_attn.k_proj.weight");
    w.v = (uint16_t*)ptr(p + "self_attn.v_proj.weight");
    w.o = (uint16_t*)ptr(p + "self_attn.o_proj.weight");
    w.gate = (uint16_t*)ptr(p + "mlp.gate_proj.weight");
    w.up = (uint16_t*)ptr(p + "mlp.up_proj.weight");
    w.down = (uint16_t*)ptr(p + "mlp.down_proj.weight");
    w.in_norm = (float*)ptr(p + "input_layernorm.weight");
    w.q_norm = (float*)ptr(p + "self_attn.q_norm.weight");
    w.k_norm = (float*)ptr(p + "self_attn.k_norm.weight");
    w.post_norm = (float*)ptr(p + "post_attention_layernorm.weight");
  }
  if ((e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming)) != cudaSuccess) {
    delete m;
    return cuda_fail(e, "stream/event creation");
  }
  m->gemv_grid = m->sms * std::max(1, env_int("YUE2_CUDA_GEMV_CTAS_PER_SM", 2));
  m->use_pdl = env_int("YUE2_CUDA_PDL", 1) != 0;
  m->use_graphs = env_int("YUE2_CUDA_GRAPHS", 1) != 0;
  {
    const char* v = getenv("YUE2_CUDA_PREFILL");
    m->use_prefill_gemm = !(v && std::string(v) == "gemv");
    m->prefill_chunk = std::max(16, std::min(kPrefillRows, env_int("YUE2_CUDA_PREFILL_CHUNK", kPrefillRows)));
    const char* a = getenv("YUE2_CUDA_PREFILL_ATTN");
    m->prefill_tc_attn = !(a && std::string(a) == "rows");
    m->prefill_attn_tc5 = !a ? 0 : std::string(a) == "tc" ? 1 : std::string(a) == "sync" ? 2 : 0;
    m->gemm_split_k = env_int("YUE2_CUDA_GEMM_SPLITK", 0) != 0;
    m->wide_min = std::max(2, std::min(kMaxRows + 1, env_int("YUE2_CUDA_WIDE_MIN", 3)));
    const char* gm = getenv("YUE2_CUDA_GEMM");
    m->gemm_tc = gm && std::string(gm) == "tc";
    {
      const int sk = env_int("YUE2_CUDA_SKINNY", -1);
      m->skinny_rows = sk == 0 ? 0 : sk == 1 ? kSkinnyMaxRows : 16;
    }
    m->wide_pdl = m->use_pdl && env_int("YUE2_CUDA_WIDE_PDL", 1) != 0;
    m->attn_splits = std::max(0, env_int("YUE2_CUDA_ATTN_SPLITS", 0));
    m->attn_cluster = std::max(-1, std::min(kClusterMax, env_int("YUE2_CUDA_ATTN_CLUSTER", -1)));
  }
  *out = m;
  return 0;
}

// Model::open's NAR tensors (src/model.rs:246-270, 428-451), in an allocation of their own.
int yue2_model_enable_nar(Yue2Model* m, uint64_t latent_dim, uint64_t max_latent_frames, float timestep_shift) {
  if (!m) return fail(YUE2_ERR_INVALID, "null model");
  if (m->nar_arena) return fail(YUE2_ERR_INVALID, "NAR tensors already enabled");
  if (m->tp_world > 1) return fail(YUE2_ERR_INVALID, "the NAR tensors are not available on a tensor-parallel model");
  // Config::read validation (src/model.rs:50-72)
  if (!latent_dim || latent_dim % 8 || latent_dim > 4096 || !max_latent_frames || !(timestep_shift > 0.f) ||
      !std::isfinite(timestep_shift))
    return fail(YUE2_ERR_INVALID, "Invalid latent configuration (latent_dim a multiple of 8)");
  int rc = y2_set_device(m);
  if (rc) return rc;
  const Geometry& g = m->g;
  const size_t H = g.hidden, I = g.inter, D = g.dim, L = latent_dim, F = max_latent_frames;
  const size_t qd = (size_t)g.heads * D, kd = (size_t)g.kvh * D;
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  size_t total = 0;
  std::vector<std::pair<std::string, TensorSlot>> plan;
  auto add = [&](const std::string& name, size_t rows, size_t cols, bool norm) {
    TensorSlot t;
    t.rows = rows;
    t.cols = cols;
    t.norm = norm;
    t.offset = total;
    total += al(rows * cols * (norm ? 4 : 2));
    plan.push_back({name, t});
  };
  add("latent_pos_embed.pe", F, H, false);
  add("vae2llm.weight", H, L, false);
  add("vae2llm.bias", 1, H, true);
  add("llm2vae.weight", L, H, false);
  add("llm2vae.bias", 1, L, true);
  add("time_embedder.mlp.0.weight", H, 256, false);
  add("time_embedder.mlp.0.bias", 1, H, true);
  add("time_embedder.mlp.2.weight", H, H, false);
  add("time_embedder.mlp.2.bias", 1, H, true);
  for (int l = 0; l < g.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    add(p + "nar_self_attn.q_proj.weight", qd, H, false);
    add(p + "nar_self_attn.k_proj.weight", kd, H, false);
    add(p + "nar_self_attn.v_proj.weight", kd, H, false);
    add(p + "nar_self_attn.o_proj.weight", H, qd, false);
    add(p + "nar_mlp.gate_proj.weight", I, H, false);
    add(p + "nar_mlp.up_proj.weight", I, H, false);
    add(p + "nar_mlp.down_proj.weight", H, I, false);
    add(p + "nar_input_layernorm.weight", 1, H, true);
    add(p + "nar_self_attn.q_norm.weight", 1, D, true);
    add(p + "nar_self_attn.k_norm.weight", 1, D, true);
    add(p + "nar_pre_mlp_layernorm.weight", 1, H, true);
  }
  void* arena = nullptr;
  if ((rc = m->alloc(&arena, total))) return rc;
  m->nar_arena = (char*)arena;
  for (auto& kv : plan) {
    kv.second.base = m->nar_arena;
    m->slots[kv.first] = kv.second;
  }
  auto ptr = [&](const std::string& n) { return (void*)(m->nar_arena + m->slots[n].offset); };
  auto& W = m->nar;
  W.pe = (uint16_t*)ptr("latent_pos_embed.pe");
  W.vae2llm = (uint16_t*)ptr("vae2llm.weight");
  W.vae2llm_b = (float*)ptr("vae2llm.bias");
  W.llm2vae = (uint16_t*)ptr("llm2vae.weight");
  W.llm2vae_b = (float*)ptr("llm2vae.bias");
  W.time_in = (uint16_t*)ptr("time_embedder.mlp.0.weight");
  W.time_in_b = (float*)ptr("time_embedder.mlp.0.bias");
  W.time_out = (uint16_t*)ptr("time_embedder.mlp.2.weight");
  W.time_out_b = (float*)ptr("time_embedder.mlp.2.bias");
  W.latent = (int)L;
  W.max_frames = (int)F;
  W.shift = timestep_shift;
  m->nar_layers.resize(g.layers);
  for (int l = 0; l < g.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    LayerW& w = m->nar_layers[l];
    w.q = (uint16_t*)ptr(p + "nar_self_attn.q_proj.weight");
    w.k = (uint16_t*)ptr(p + "nar_self_attn.k_proj.weight");
    w.v = (uint16_t*)ptr(p + "nar_self_attn.v_proj.weight");
    w.o = (uint16_t*)ptr(p + "nar_self_attn.o_proj.weight");
    w.gate = (uint16_t*)ptr(p + "nar_mlp.gate_proj.weight");
    w.up = (uint16_t*)ptr(p + "nar_mlp.up_proj.weight");
    w.down = (uint16_t*)ptr(p + "nar_mlp.down_proj.weight");
    w.in_norm = (float*)ptr(p + "nar_input_layernorm.weight");
    w.q_norm = (float*)ptr(p + "nar_self_attn.q_norm.weight");
    w.k_norm = (float*)ptr(p + "nar_self_attn.k_norm.weight");
    w.post_norm = (float*)ptr(p + "nar_pre_mlp_layernorm.weight");
  }
  m->finalized = false;
  return 0;
}

int yue2_model_set_tensor(Yue2Model* m, const char* name, int dtype, const void* data, uint64_t rows,
                          uint64_t cols) {
  if (!m || !name || !data) return fail(YUE2_ERR_INVALID, "null argument");
  if (dtype < 0 || dtype > 2) return fail(YUE2_ERR_INVALID, "unknown dtype");
  auto it = m->slots.find(name);
  if (it == m->slots.end()) return 1;  // not on the AR decode path
  TensorSlot& t = it->second;
  const uint64_t count = rows * cols;
  if (count != t.rows * t.cols || (!t.norm && (rows != t.rows || cols != t.cols)))
    return fail(YUE2_ERR_INVALID, std::string("Tensor shape mismatch for ") + name);
  int rc = y2_set_device(m);
  if (rc) return rc;
  void* dst = m->slot_addr(t);
  if (t.norm) {  // Norm::new: values rounded to bf16 (tensor.rs:1126-1136)
    std::vector<float> v(count);
    for (size_t i = 0; i < count; ++i) v[i] = round_bf16(host_value(dtype, data, i));
    CK(cudaMemcpy(dst, v.data(), count * 4, cudaMemcpyHostToDevice));
  } else if (dtype == YUE2_DTYPE_BF16) {
    CK(cudaMemcpy(dst, data, count * 2, cudaMemcpyHostToDevice));
  } else {  // F32/F16 checkpoints are rounded to bf16 (tensor.rs:436-438)
    std::vector<uint16_t> v(count);
    for (size_t i = 0; i < count; ++i) v[i] = f32_to_bf16_bits(host_value(dtype, data, i));
    CK(cudaMemcpy(dst, v.data(), count * 2, cudaMemcpyHostToDevice));
  }
  m->loaded.insert(name);
  m->finalized = false;
  return 0;
}

int yue2_model_init_synthetic(Yue2Model* m, uint64_t seed, float stddev, float norm_mean) {
  if (!m) return fail(YUE2_ERR_INVALID, "null model");
  int rc = y2_set_device(m);
  if (rc) return rc;
  uint64_t idx = 0;
  for (auto& kv : m->slots) {
    TensorSlot& t = kv.second;
    const uint64_t tseed = seed * 0x9E3779B97F4A7C15ull + (++idx) * 0xD1B54A32D192ED03ull;
    if (t.norm) {
      std::vector<float> v(t.rows * t.cols);
      for (size_t i = 0; i < v.size(); i += 2) {
        uint64_t z = tseed + (i / 2 + 1) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        const double u1 = ((z >> 11) + 1) * (1.0 / 9007199254740992.0), u2 = (z & 0x1fffff) * (1.0 / 2097152.0);
        const double rad = sqrt(-2.0 * log(u1));
        v[i] = round_bf16(norm_mean + stddev * (float)(rad * cos(6.283185307179586 * u2)));
        if (i + 1 < v.size()) v[i + 1] = round_bf16(norm_mean + stddev * (float)(rad * sin(6.283185307179586 * u2)));
      }
      CK(cudaMemcpy(m->slot_addr(t), v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    } else if (t.rows == t.full_rows && t.cols == t.full_cols) {
      CK(launch_fill_normal_bf16(m->stream, (uint16_t*)m->slot_addr(t), t.rows * t.cols, tseed, 0.f,
                                 stddev));
    } else {  // a tensor-parallel shard: the values of the full tensor at the shard's positions
      CK(launch_fill_normal_shard(m->stream, (uint16_t*)m->slot_addr(t), t.rows, t.cols, t.full_cols, t.row0, t.col0,
                                  tseed, stddev));
    }
    m->loaded.insert(kv.first);
  }
  CK(cudaStreamSynchronize(m->stream));
  m->finalized = false;
  return 0;
}

int yue2_model_get_tensor(Yue2Model* m, const char* name, uint16_t* out, uint64_t count) {
  if (!m || !name || !out) return fail(YUE2_ERR_INVALID, "null argument");
  auto it = m->slots.find(name);
  if (it == m->slots.end()) return fail(YUE2_ERR_INVALID, std::string("unknown tensor ") + name);
  TensorSlot& t = it->second;
  if (count != t.rows * t.cols) return fail(YUE2_ERR_INVALID, "count mismatch");
  int rc = y2_set_device(m);
  if (rc) return rc;
  if (t.norm) {
    std::vector<float> v(count);
    CK(cudaMemcpy(v.data(), m->slot_addr(t), count * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < count; ++i) out[i] = f32_to_bf16_bits(v[i]);
  } else {
    CK(cudaMemcpy(out, m->slot_addr(t), count * 2, cudaMemcpyDeviceToHost));
  }
  return 0;
}

int yue2_model_finalize(Yue2Model* m) {
  if (!m) return fail(YUE2_ERR_INVALID, "null model");
  for (auto& kv : m->slots)
    if (!m->loaded.count(kv.first)) return fail(YUE2_ERR_INVALID, "Missing tensor " + kv.first);
  int rc = y2_set_device(m);
  if (rc) return rc;
  const Geometry& g = m->g;
  if (!m->workspace_ready) {
    CK(prepare_kernels());
    // RoPE tables, Rotary::new (src/model.rs:137-150) for every position
    const int half = g.dim / 2;
    m->max_pos = (int)std::min<uint64_t>(m->cfg.max_position_embeddings, 1u << 20);
    std::vector<float> ct((size_t)m->max_pos * half), st((size_t)m->max_pos * half);
    for (int i = 0; i < half; ++i) {
      const float freq = 1.0f / powf(m->cfg.rope_theta, (float)(2 * i) / (float)g.dim);
      for (int p = 0; p < m->max_pos; ++p) {
        const float angle = (float)p * freq;
        ct[(size_t)p * half + i] = round_bf16(cosf(angle));
        st[(size_t)p * half + i] = round_bf16(sinf(angle));
      }
    }
    void *cp, *sp;
    if ((rc = m->alloc(&cp, ct.size() * 4)) || (rc = m->alloc(&sp, st.size() * 4))) return rc;
    m->cos_tab = (float*)cp;
    m->sin_tab = (float*)sp;
    CK(cudaMemcpy(cp, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(sp, st.data(), st.size() * 4, cudaMemcpyHostToDevice));
    // workspaces for up to kMaxRows rows
    const size_t R = kMaxRows, H = g.hidden, qd = (size_t)g.heads * g.dim, kd = (size_t)g.kvh * g.dim;
    const int G = g.heads / g.kvh;
    m->max_splits = 64;
    void* p;
    if ((rc = m->alloc(&p, R * H * 4))) return rc;
    m->x = (float*)p;
    if ((rc = m->alloc(&p, R * (qd + 2 * kd) * 2))) return rc;
    m->qkv = (uint16_t*)p;
    if ((rc = m->alloc(&p, R * qd * 2))) return rc;
    m->qrot = (uint16_t*)p;
    if ((rc = m->alloc(&p, R * qd * 2))) return rc;
    m->attn = (uint16_t*)p;
    if ((rc = m->alloc(&p, R * (size_t)g.inter * 2))) return rc;
    m->hbuf = (uint16_t*)p;
    if ((rc = m->alloc(&p, R * (size_t)g.vocab * 4))) return rc;
    m->logits = (float*)p;
    if ((rc = m->alloc(&p, R * g.kvh * (size_t)m->max_splits * G * (g.dim + 2) * 4))) return rc;
    m->part = (float*)p;
    if ((rc = m->alloc(&p, R * g.kvh * 4))) return rc;
    m->counters = (int32_t*)p;
    CK(cudaMemset(p, 0, R * g.kvh * 4));
    if ((rc = m->alloc(&p, R * sizeof(DevRow)))) return rc;
    m->rows = (DevRow*)p;
    if ((rc = m->alloc(&p, 256))) return rc;
    m->flags = (int32_t*)p;
    CK(cudaMemset(p, 0, 256));
    if (m->tp_world > 1) {  // tensor-parallel exchange buffers (tp.cu)
      if ((rc = m->alloc(&p, tp_recv_bytes(g.hidden, g.vocab)))) return rc;
      m->tp_recv = (char*)p;
      CK(cudaMemset(p, 0, tp_recv_bytes(g.hidden, g.vocab)));
      if ((rc = m->alloc(&p, 256))) return rc;
      m->tp_epoch = (uint32_t*)p;
      CK(cudaMemset(p, 0, 256));
    }
    CK(cudaMallocHost(&m->pinned_rows, Yue2Model::kRowSlots * R * sizeof(DevRow)));
    CK(cudaMallocHost(&m->pinned_flags, 4096));
    m->workspace_ready = true;
  }
  m->finalized = true;
  return 0;
}

void yue2_model_free(Yue2Model* m) { delete m; }

// ---------------------------------------------------------------- caches
int yue2_cache_create(Yue2Model* m, uint64_t capacity, Yue2Cache** out) {
  if (!m || !out) return fail(YUE2_ERR_INVALID, "null argument");
  *out = nullptr;
  if (capacity == 0 || capacity > (uint64_t)m->max_pos_limit())
    return fail(YUE2_ERR_CAPACITY, "cache capacity must be in [1, max_position_embeddings]");
  int rc = y2_set_device(m);
  if (rc) return rc;
  Yue2Cache* c = new Yue2Cache();
  c->m = m;
  c->capacity = capacity;
  const size_t npages = (capacity + kPageTokens - 1) / kPageTokens;
  if ((rc = m->pool.take(npages, c->pages))) {
    delete c;
    return rc;
  }
  void* pt = nullptr;
  if ((rc = m->scratch_take(&pt, npages * 8))) {
    m->pool.give(c->pages);
    delete c;
    return rc;
  }
  c->d_pages = (uint64_t*)pt;
  cudaError_t e = cudaMemcpy(c->d_pages, c->pages.data(), npages * 8, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    yue2_cache_free(c);
    return cuda_fail(e, "page table upload");
  }
  *out = c;
  return 0;
}

void yue2_cache_free(Yue2Cache* c) {
  if (!c) return;
  cudaSetDevice(c->m->device);
  // work queued on the model's stream may still use the pages and the page table
  if (c->m->stream) cudaStreamSynchronize(c->m->stream);
  c->m->pool.give(c->pages);
  c->m->scratch_give(c->d_pages);
  delete c;
}

int yue2_cache_length(const Yue2Cache* c, uint64_t* length) {
  if (!c || !length) return fail(YUE2_ERR_INVALID, "null argument");
  *length = c->length;
  return 0;
}

int yue2_cache_fill_normal(Yue2Cache* c, uint64_t to, uint64_t seed) {
  if (!c) return fail(YUE2_ERR_INVALID, "null cache");
  if (to > c->capacity || to > (uint64_t)c->m->max_pos) return fail(YUE2_ERR_CAPACITY, "fill beyond capacity");
  if (to <= c->length) return 0;
  int rc = y2_set_device(c->m);
  if (rc) return rc;
  const Yue2Model& m = *c->m;
  CK(launch_kv_fill(m.stream, c->d_pages, m.g, (int)c->length, (int)to, seed, m.tp_rank * m.g.kvh,
                    m.g.kvh * m.tp_world));
  CK(cudaStreamSynchronize(c->m->stream));
  c->length = to;
  return 0;
}

int yue2_cache_read(const Yue2Cache* c, uint64_t layer, uint64_t begin, uint64_t count, uint16_t* k, uint16_t* v) {
  if (!c || !k || !v) return fail(YUE2_ERR_INVALID, "null argument");
  const Geometry& g = c->m->g;
  if (layer >= (uint64_t)g.layers || begin + count > c->length) return fail(YUE2_ERR_INVALID, "range");
  int rc = y2_set_device(c->m);
  if (rc) return rc;
  const size_t D = g.dim, kd = (size_t)g.kvh * D;
  // one copy per page: the layer's K and V blocks are adjacent ([K|V][kv head][64][dim])
  const size_t block = 2 * (size_t)g.kvh * kPageTokens * D;
  std::vector<uint16_t> tmp(block);
  for (uint64_t t = begin; t < begin + count;) {
    const uint64_t pg = t / kPageTokens, end = std::min<uint64_t>(begin + count, (pg + 1) * kPageTokens);
    const char* page = (const char*)c->pages[pg];
    CK(cudaMemcpy(tmp.data(), page + kv_offset(g, (int)layer, 0, 0) * 2, block * 2, cudaMemcpyDeviceToHost));
    for (; t < end; ++t)
      for (int h = 0; h < g.kvh; ++h)
        for (int kvsel = 0; kvsel < 2; ++kvsel)
          memcpy((kvsel ? v : k) + (t - begin) * kd + h * D,
                 tmp.data() + kv_offset(g, 0, kvsel, h) + (t % kPageTokens) * D, D * 2);
  }
  return 0;
}

}  // extern "C"

// ---------------------------------------------------------------- step encoding
namespace y2 {

// Splits per (row, kv head): as many as fill one wave of attention CTAs (two per SM).
int splits_for(const Yue2Model& m, int R) {
  if (m.attn_splits > 0) return std::min(m.max_splits, m.attn_splits);  // YUE2_CUDA_ATTN_SPLITS
  // kv heads x rows >= 8 (the 3B CFG pair): 8 splits per (kv head, row) up to 8,192
  // positions, 16 beyond (measured ms/step for the CFG pair, splits 8 / 12 / 16 / 24:
  // 1k 2.003 / 2.013 / 2.012 / 2.017; 4k 2.021 / 2.048 / 2.041 / 2.419;
  // 24k 2.962 / 2.804 / 2.790 / 3.117)
  if (R <= kMaxRows && m.g.kvh * R >= 8) return m.ctx_hint <= 8192 ? 8 : 16;
  const int want = (2 * m.sms) / (m.g.kvh * R);
  return std::max(1, std::min(m.max_splits, want));
}

// LM-head projection rows for a phase (model.rs:478-507): the window and the stop row,
// intersected with this rank's vocabulary rows [head_row0, head_row0 + head_rows) (all of
// them without tensor parallelism). p.N = 0 when the rank holds none of them.
static void head_params(const Yue2Model& m, int phase, GemvParams& p) {
  const size_t H = m.g.hidden;
  const int V = m.g.vocab;
  int ranges[2][2];
  int nr = 0;
  if (phase == kPhaseVocab) {
    ranges[nr][0] = 0;
    ranges[nr++][1] = V;
  } else {
    const int start = phase == kPhaseAbc ? 0 : (int)kCodecOffset;
    const int end = phase == kPhaseAbc ? (int)kEOD : (int)(kCodecOffset + kCodecSize);
    const int stop = phase == kPhaseAbc ? (int)kAbcEnd : (int)kMusicEnd;
    ranges[nr][0] = start;
    ranges[nr++][1] = end;
    ranges[nr][0] = stop;
    ranges[nr++][1] = stop + 1;
  }
  const int lo = m.head_row0, hi = m.head_row0 + m.head_rows;
  p.wpair = nullptr;
  int n = 0, seg = 0;
  for (int i = 0; i < nr; ++i) {
    const int a0 = std::max(ranges[i][0], lo), a1 = std::min(ranges[i][1], hi);
    if (a1 <= a0) continue;
    p.w[seg] = m.lm_head + (size_t)(a0 - lo) * H;
    p.seg_start[seg] = n;
    p.col0[seg] = a0;
    n += a1 - a0;
    ++seg;
  }
  for (int i = seg; i < 3; ++i) {
    p.w[i] = seg ? p.w[seg - 1] : m.lm_head;
    p.seg_start[i] = n;
    p.col0[i] = seg ? p.col0[seg - 1] : 0;
  }
  p.seg_start[0] = 0;
  p.N = n;
}

int check_phase_vocab(const Yue2Model& m, int phase) {
  const int64_t V = m.g.vocab;
  if (phase == kPhaseVocab) return 0;
  if (phase == kPhaseAbc && V > kAbcEnd) return 0;
  if (phase == kPhaseSemantic && V >= kCodecOffset + kCodecSize && V > kMusicEnd) return 0;
  if (phase < 0 || phase > 2) return fail(YUE2_ERR_INVALID, "unknown phase");
  return fail(YUE2_ERR_VOCAB, "Vocabulary does not support native music protocol");
}

// Final RMSNorm + LM head of `R` residual rows starting at x_row into logits rows [dst, dst+R).
cudaError_t encode_head(Yue2Model& m, cudaStream_t s, bool pdl, int x_row, int R, int dst_row, int phase,
                        const int32_t* skip) {
  return encode_head_from(m, s, pdl, m.x + (size_t)x_row * m.g.hidden, R, dst_row, phase, skip);
}

// Final norm + LM head of R rows of hidden states at x (f32 [R, hidden]) into logits rows
// [dst_row, dst_row + R).
cudaError_t encode_head_from(Yue2Model& m, cudaStream_t s, bool pdl, const float* x, int R, int dst_row, int phase,
                             const int32_t* skip) {
  const int V = m.g.vocab;
  if (phase != kPhaseVocab) {
    cudaError_t e = launch_fill_f32(s, m.logits + (size_t)dst_row * V, (size_t)R * V, -INFINITY);
    if (e != cudaSuccess) return e;
  }
  GemvParams p = {};
  p.error = m.flags + 2;
  head_params(m, phase, p);
  p.K = m.g.hidden;
  p.R = R;
  p.xf = x;
  p.gamma = m.final_norm;
  p.eps = m.g.eps;
  p.of = m.logits + (size_t)dst_row * V;
  p.ldo = V;
  p.skip = skip;
  if (p.N > 0) {
    cudaError_t e = launch_gemv(s, pdl, kXNorm, kEpiLogits, p, m.gemv_grid);
    if (e != cudaSuccess) return e;
  }
  if (m.tp_world == 1) return cudaSuccess;
  // every rank's vocabulary slice of the logits to every rank
  TpParams tp = tp_params(m);
  tp.R = R;
  tp.n = V;
  tp.col0 = m.head_row0;
  tp.cols = m.head_rows;
  tp.row_base = dst_row;
  tp.site = 255;
  return launch_tp_allgather(s, pdl, tp);
}

int tp_ready(const Yue2Model& m) {
  if (m.tp_world > 1 && !m.tp_connected)
    return fail(YUE2_ERR_INVALID, "tensor-parallel model: call yue2_tp_connect on every rank first");
  return 0;
}

TpParams tp_params(const Yue2Model& m) {
  TpParams p = {};
  p.peers = m.tp_peers;
  p.rank = m.tp_rank;
  p.world = m.tp_world;
  p.epoch = m.tp_epoch;
  p.error = m.flags + 2;
  return p;
}

// Parameters of layer l's kernels for R rows.
struct LayerOps {
  GemvParams qkv, o, gu, down;
  RopeParams rope;
  AttnParams attn;
};

static LayerOps layer_ops(const Yue2Model& m, int l, int R, bool fused, const int32_t* skip, int splits) {
  const Geometry& g = m.g;
  const int H = g.hidden, qd = g.heads * g.dim, kd = g.kvh * g.dim, I = g.inter;
  const LayerW& w = m.layers[l];
  LayerOps op;
  GemvParams p = {};
  p.error = m.flags + 2;
  // fused q|k|v projection with the input RMSNorm in the prologue
  p.w[0] = w.q;
  p.w[1] = w.k;
  p.w[2] = w.v;
  p.seg_start[0] = 0;
  p.seg_start[1] = qd;
  p.seg_start[2] = qd + kd;
  p.col0[0] = 0;
  p.col0[1] = qd;
  p.col0[2] = qd + kd;
  p.N = qd + 2 * kd;
  p.K = H;
  p.R = R;
  p.xf = m.x;
  p.gamma = w.in_norm;
  p.eps = g.eps;
  p.ob = m.qkv;
  p.ldo = qd + 2 * kd;
  p.skip = skip;
  op.qkv = p;
  RopeParams rp = {};
  rp.rows = m.rows;
  rp.qkv = m.qkv;
  rp.q_out = m.qrot;
  rp.cos_tab = m.cos_tab;
  rp.sin_tab = m.sin_tab;
  rp.q_norm = w.q_norm;
  rp.k_norm = w.k_norm;
  rp.g = g;
  rp.layer = l;
  rp.max_pos = m.max_pos;
  rp.error = m.flags + 1;
  op.rope = rp;
  AttnParams ap = {};
  ap.rows = m.rows;
  ap.q = m.qrot;
  ap.out = m.attn;
  ap.part = m.part;
  ap.counters = m.counters;
  ap.g = g;
  ap.layer = l;
  ap.splits = splits;
  ap.scale = 1.0f / sqrtf((float)g.dim);
  ap.fused = fused ? 1 : 0;
  ap.qkv = m.qkv;
  ap.q_norm = w.q_norm;
  ap.k_norm = w.k_norm;
  ap.cos_tab = m.cos_tab;
  ap.sin_tab = m.sin_tab;
  ap.max_pos = m.max_pos;
  ap.error = m.flags + 1;
  op.attn = ap;
  // o projection + residual
  p = GemvParams{};
  p.error = m.flags + 2;
  p.w[0] = p.w[1] = p.w[2] = w.o;
  p.seg_start[1] = p.seg_start[2] = H;
  p.N = H;
  p.K = qd;
  p.R = R;
  p.xb = m.attn;
  p.of = m.x;
  p.ldo = H;
  p.skip = skip;
  op.o = p;
  // gate|up with the post-attention RMSNorm, SwiGLU epilogue
  p = GemvParams{};
  p.error = m.flags + 2;
  p.w[0] = p.w[1] = p.w[2] = w.gate;
  p.wpair = w.up;
  p.seg_start[1] = p.seg_start[2] = I;
  p.N = I;
  p.K = H;
  p.R = R;
  p.xf = m.x;
  p.gamma = w.post_norm;
  p.eps = g.eps;
  p.ob = m.hbuf;
  p.ldo = I;
  p.skip = skip;
  op.gu = p;
  // down projection + residual
  p = GemvParams{};
  p.error = m.flags + 2;
  p.w[0] = p.w[1] = p.w[2] = w.down;
  p.seg_start[1] = p.seg_start[2] = H;
  p.N = H;
  p.K = I;
  p.R = R;
  p.xb = m.hbuf;
  p.of = m.x;
  p.ldo = H;
  p.skip = skip;
  op.down = p;
  return op;
}

// embed -> layers -> [final norm + LM head] -> position advance, as one PDL chain.
cudaError_t encode_forward(Yue2Model& m, cudaStream_t s, int R, bool head, int phase, const int32_t* skip) {
  const Geometry& g = m.g;
  const bool pdl = m.use_pdl;
  const bool tp = m.tp_world > 1;
  cudaError_t e;
  if (tp && (e = launch_tp_tick(s, pdl, m.tp_epoch)) != cudaSuccess) return e;
  if ((e = launch_embed(s, pdl, m.rows, R, m.embed, g.hidden, g.vocab, m.x, m.flags + 0)) != cudaSuccess) return e;
  const int splits = splits_for(m, R);
  // Decode steps (head = true) give every row its own cache, so attention itself applies
  // the QK norm and RoPE and appends the row's K/V; prefill chunks (rows of one cache,
  // consecutive positions) append all rows first with the separate kernel.
  const bool fused = head;
  const int pipe = attn_pipe_for(m, R);
  const int cluster = fused ? attn_cluster_for(m, R) : 0;
  for (int l = 0; l < g.layers; ++l) {
    LayerOps op = layer_ops(m, l, R, fused, skip, splits);
    op.attn.pipe = pipe;
    op.attn.cluster = cluster;
    if ((e = launch_gemv(s, pdl, kXNorm, kEpiBf16, op.qkv, m.gemv_grid)) != cudaSuccess) return e;
    if (!fused && (e = launch_rope_append(s, pdl, op.rope, R)) != cudaSuccess) return e;
    if ((e = launch_attention(s, pdl, op.attn, R)) != cudaSuccess) return e;
    if (!tp) {
      if ((e = launch_gemv(s, pdl, kXBf16, kEpiResidual, op.o, m.gemv_grid)) != cudaSuccess) return e;
      if ((e = launch_gemv(s, pdl, kXNorm, kEpiSwiGLU, op.gu, m.gemv_grid)) != cudaSuccess) return e;
      if ((e = launch_gemv(s, pdl, kXBf16, kEpiResidual, op.down, m.gemv_grid)) != cudaSuccess) return e;
      continue;
    }
    // tensor parallel: o and down leave partial sums over this rank's input columns, which
    // the same kernels exchange with every rank and add in rank order with the residual
    GemvParams o = op.o, down = op.down;
    for (GemvParams* p : {&o, &down}) {
      p->tp_peers = m.tp_peers;
      p->tp_epoch = m.tp_epoch;
      p->tp_rank = m.tp_rank;
      p->tp_world = m.tp_world;
    }
    o.tp_site = 2 * l;
    down.tp_site = 2 * l + 1;
    if ((e = launch_gemv(s, pdl, kXBf16, kEpiTpReduce, o, m.gemv_grid)) != cudaSuccess) return e;
    if ((e = launch_gemv(s, pdl, kXNorm, kEpiSwiGLU, op.gu, m.gemv_grid)) != cudaSuccess) return e;
    if ((e = launch_gemv(s, pdl, kXBf16, kEpiTpReduce, down, m.gemv_grid)) != cudaSuccess) return e;
  }
  if (head && (e = encode_head(m, s, pdl, 0, R, 0, phase, skip)) != cudaSuccess) return e;
  return launch_step_end(s, pdl, m.rows, R);
}

int attn_pipe_for(const Yue2Model& m, int R) { return attn_pipe_for_keys(m.ctx_hint, splits_for(m, R)); }

// Up to kClusterKeys keys over the life of a captured forward (its context plus the positions
// it will advance), decode passes of up to kMaxRows rows take the cluster form of attention:
// 8-warp CTAs with about six 32-key tiles each (one per warp, more CTAs for bandwidth),
// ceil(tiles / 6) CTAs per (kv head, row), at most kClusterCap (warps then stream further
// tiles, each K during the previous P.V). Larger clusters wait for room in one GPC.
// Measured decode step of the CFG pair (ms; split-K ticket kernel, then clusters of N CTAs):
//   1,040 positions: split 1.986, 3: 1.922, 4: 1.916, 5: 1.866, 6: 1.856 (1.840 pipelined)
//   1,500: split 1.935, 4: 1.840, 5: 1.850, 6: 1.813, 7: 2.023
//   2,600: split 1.925, 6: 1.851; 3,500: split 2.009, 6: 1.928
//   4,096: split 2.022, 6: 1.964; 6,000: split 2.124, 6: 2.065
//   8,192: split 2.169, 6: 2.199 (the split kernel keeps longer contexts)
constexpr int kClusterKeys = 7168;
constexpr int kClusterCap = 6;
int attn_cluster_for(const Yue2Model& m, int R) {
  if (m.attn_cluster == 0 || m.g.dim > 128 || R > kMaxRows || m.attn_splits > 0) return 0;
  if (m.attn_cluster > 0) return m.attn_cluster;
  const int keys = m.ctx_hint + m.ctx_growth;
  if (keys > kClusterKeys) return 0;
  const int tiles = (keys + 31) / 32;
  return std::max(1, std::min(kClusterCap, (tiles + 5) / 6));
}

int kernels_per_step(const Yue2Model& m, bool head, int phase, int R) {
  const int tp = m.tp_world > 1;  // the tick and the logits gather (o and down exchange in place)
  return 1 + (head ? 5 : 6) * m.g.layers + (head ? 1 + (phase != kPhaseVocab) : 0) + 1 + tp * (1 + (head ? 1 : 0));
}

// Runs (and caches as a CUDA graph) the forward step for R rows already in m.rows.
int run_forward(Yue2Model& m, int R, bool head, int phase) {
  const int key = R * 16 + (head ? 8 : 0) + phase + (attn_pipe_for(m, R) + 2 * attn_cluster_for(m, R)) * 8192;
  if (!m.use_graphs) {
    CK(encode_forward(m, m.stream, R, head, phase, nullptr));
    return 0;
  }
  auto it = m.graphs.find(key);
  if (it == m.graphs.end()) {
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = encode_forward(m, m.stream, R, head, phase, nullptr);
    cudaError_t e2 = cudaStreamEndCapture(m.stream, &graph);
    if (e != cudaSuccess) return cuda_fail(e, "encode_forward");
    if (e2 != cudaSuccess) return cuda_fail(e2, "cudaStreamEndCapture");
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    it = m.graphs.emplace(key, exec).first;
  }
  CK(cudaGraphLaunch(it->second, m.stream));
  return 0;
}

// Stages the row descriptors through a ring of pinned slots: an asynchronous copy reads
// its slot when the stream reaches it, so a slot is reused only after its copy is done.
int upload_rows(Yue2Model& m, const std::vector<DevRow>& rows) {
  const int slot = (int)(m.row_slot++ % Yue2Model::kRowSlots);
  if (m.row_events[slot]) CK(cudaEventSynchronize(m.row_events[slot]));
  else CK(cudaEventCreateWithFlags(&m.row_events[slot], cudaEventDisableTiming));
  DevRow* staging = m.pinned_rows + (size_t)slot * kMaxRows;
  memcpy(staging, rows.data(), rows.size() * sizeof(DevRow));
  CK(cudaMemcpyAsync(m.rows, staging, rows.size() * sizeof(DevRow), cudaMemcpyHostToDevice, m.stream));
  CK(cudaEventRecord(m.row_events[slot], m.stream));
  return 0;
}

// Reads and clears the device error flags (embed token range, RoPE range, stream stall).
int take_flags(Yue2Model& m) {
  CK(cudaMemcpyAsync(m.pinned_flags, m.flags, 12, cudaMemcpyDeviceToHost, m.stream));
  CK(cudaStreamSynchronize(m.stream));
  const int32_t tok = m.pinned_flags[0], pos = m.pinned_flags[1], stall = m.pinned_flags[2];
  if (tok || pos || stall) {
    CK(cudaMemsetAsync(m.flags, 0, 12, m.stream));
    CK(cudaStreamSynchronize(m.stream));
    if (stall) return fail(YUE2_ERR_TIMEOUT, "a bounded weight-stream wait gave up");
    if (tok) return fail(YUE2_ERR_TOKEN, "Token outside model vocabulary");
    return fail(YUE2_ERR_CAPACITY, "position outside the RoPE table");
  }
  return 0;
}

// Appends ids[0, n) to cache c in chunks of kMaxRows consecutive positions (prompts of at
// least kPrefillGemmMin ids: as GEMMs, gemm_rows.cu). The ids must already be on the
// device. When logits_row >= 0, the last id's final-normed hidden state goes through
// the LM head into logits row `logits_row`.
int prefill_device(Yue2Model& m, Yue2Cache& c, const int32_t* d_ids, uint64_t n, int logits_row, int phase) {
  // a tensor-parallel model runs prompts through the decode chain, kTpRows positions a pass
  const bool tp = m.tp_world > 1;
  if (!tp && m.use_prefill_gemm && n >= (uint64_t)kPrefillGemmMin)
    return prefill_gemm(m, c, d_ids, n, logits_row, phase);
  const uint64_t L0 = c.length;
  const uint64_t chunk = tp ? kTpRows : kMaxRows;
  int lastR = 0;
  for (uint64_t start = 0; start < n; start += chunk) {
    const int R = (int)std::min<uint64_t>(chunk, n - start);
    std::vector<DevRow> rows(R);
    for (int r = 0; r < R; ++r) {
      rows[r] = DevRow{};
      rows[r].pages = c.d_pages;
      rows[r].prompt = d_ids;
      rows[r].prompt_begin = (int32_t)L0;
      rows[r].prompt_end = (int32_t)(L0 + n);
      rows[r].pos = (int32_t)(L0 + start + r);
      rows[r].active = 1;
      rows[r].advance = 0;
    }
    int rc = upload_rows(m, rows);
    if (rc) return rc;
    m.ctx_hint = (int)(L0 + start + R);
    if ((rc = run_forward(m, R, false, phase))) return rc;
    lastR = R;
  }
  if (logits_row >= 0) CK(encode_head(m, m.stream, false, lastR - 1, 1, logits_row, phase, nullptr));
  c.length = L0 + n;
  return 0;
}

}  // namespace y2

// ---------------------------------------------------------------- forward / prefill API
extern "C" {

int yue2_forward(Yue2Model* m, Yue2Cache* const* caches, const int64_t* ids, uint64_t rows, int phase,
                 float* logits) {
  if (!m || !caches || !ids) return fail(YUE2_ERR_INVALID, "null argument");
  if (!m->finalized) return fail(YUE2_ERR_INVALID, "model not finalized");
  if (rows < 1 || rows > (uint64_t)kMaxWideRows) return fail(YUE2_ERR_INVALID, "rows must be in [1, 256]");
  if (m->tp_world > 1 && rows > (uint64_t)kTpRows)
    return fail(YUE2_ERR_INVALID, "a tensor-parallel forward takes at most 2 rows");
  int rc = check_phase_vocab(*m, phase);
  if (rc || (rc = tp_ready(*m))) return rc;
  std::set<const Yue2Cache*> seen;
  for (uint64_t r = 0; r < rows; ++r) {
    const Yue2Cache* c = caches[r];
    if (!c || c->m != m) return fail(YUE2_ERR_INVALID, "cache belongs to another model");
    if (!seen.insert(c).second) return fail(YUE2_ERR_INVALID, "a cache may appear once per forward");
    if (c->length + 1 > c->capacity || c->length + 1 > (uint64_t)m->max_pos)
      return fail(YUE2_ERR_CAPACITY, "AR input exceeds cache/model context");
    if (ids[r] < 0 || ids[r] >= (int64_t)m->g.vocab) return fail(YUE2_ERR_TOKEN, "Token outside model vocabulary");
  }
  if ((rc = y2_set_device(m))) return rc;
  std::vector<DevRow> dr(rows);
  for (uint64_t r = 0; r < rows; ++r) {
    dr[r] = DevRow{};
    dr[r].pages = caches[r]->d_pages;
    dr[r].pos = (int32_t)caches[r]->length;
    dr[r].token = (int32_t)ids[r];
    dr[r].active = 1;
    dr[r].advance = 1;
  }
  const float* out = m->logits;
  m->ctx_hint = 0;  // picks the attention form of this forward
  for (uint64_t r = 0; r < rows; ++r) m->ctx_hint = std::max(m->ctx_hint, (int)caches[r]->length + 1);
  if (rows >= (uint64_t)m->wide_min && m->tp_world == 1) {  // the GEMM path (gemm_rows.cu)
    if ((rc = ensure_wide(*m))) return rc;
    CK(cudaMemcpyAsync(m->wide_rows, dr.data(), rows * sizeof(DevRow), cudaMemcpyHostToDevice, m->stream));
    if ((rc = encode_forward_wide(*m, m->stream, (int)rows, phase))) return rc;
    out = m->wide_logits;
  } else {
    if ((rc = upload_rows(*m, dr))) return rc;
    if ((rc = run_forward(*m, (int)rows, true, phase))) return rc;
  }
  if (logits) CK(cudaMemcpyAsync(logits, out, rows * m->g.vocab * 4, cudaMemcpyDeviceToHost, m->stream));
  if ((rc = take_flags(*m))) return rc;
  for (uint64_t r = 0; r < rows; ++r) caches[r]->length += 1;
  return 0;
}

int yue2_prefill(Yue2Model* m, Yue2Cache* c, const int64_t* ids, uint64_t n, int phase, float* logits) {
  if (!m || !c || !ids) return fail(YUE2_ERR_INVALID, "null argument");
  if (!m->finalized) return fail(YUE2_ERR_INVALID, "model not finalized");
  if (n == 0) return fail(YUE2_ERR_INVALID, "Empty prefill");
  if (c->length + n > c->capacity || c->length + n > (uint64_t)m->max_pos)
    return fail(YUE2_ERR_CAPACITY, "AR input exceeds cache/model context");
  int rc = check_phase_vocab(*m, phase);
  if (rc || (rc = tp_ready(*m))) return rc;
  std::vector<int32_t> h(n);
  for (uint64_t i = 0; i < n; ++i) {
    if (ids[i] < 0 || ids[i] >= (int64_t)m->g.vocab) return fail(YUE2_ERR_TOKEN, "Token outside model vocabulary");
    h[i] = (int32_t)ids[i];
  }
  if ((rc = y2_set_device(m))) return rc;
  void* ids_mem = nullptr;
  if ((rc = m->scratch_take(&ids_mem, n * 4))) return rc;
  int32_t* d_ids = (int32_t*)ids_mem;
  cudaError_t e = cudaMemcpy(d_ids, h.data(), n * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    m->scratch_give(d_ids);
    return cuda_fail(e, "prefill ids");
  }
  const uint64_t before = c->length;
  rc = prefill_device(*m, *c, d_ids, n, logits ? 0 : -1, phase);
  if (!rc && logits) {
    e = cudaMemcpyAsync(logits, m->logits, m->g.vocab * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e != cudaSuccess) rc = cuda_fail(e, "logits copy");
  }
  if (!rc) rc = take_flags(*m);
  cudaStreamSynchronize(m->stream);
  m->scratch_give(d_ids);
  if (rc) c->length = before;
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------- kernel timing for bench.py
extern "C" int yue2_bench_gemv(Yue2Model* m, int kind, int rows, int launches, double* avg_ms, double* bytes) {
  if (!m || !avg_ms || !bytes || rows < 1 || rows > kMaxRows || launches < 1)
    return fail(YUE2_ERR_INVALID, "bad arguments");
  if (!m->finalized) return fail(YUE2_ERR_INVALID, "model not finalized");
  int rc = y2_set_device(m);
  if (rc) return rc;
  const Geometry& g = m->g;
  const int H = g.hidden, qd = g.heads * g.dim, kd = g.kvh * g.dim, I = g.inter;
  CK(launch_fill_f32(m->stream, m->x, (size_t)kMaxRows * H, 0.5f));
  CK(cudaMemsetAsync(m->attn, 0, (size_t)kMaxRows * qd * 2, m->stream));
  CK(cudaMemsetAsync(m->hbuf, 0, (size_t)kMaxRows * I * 2, m->stream));
  // launched as the decode chain launches them: programmatic dependents when the model uses
  // them, so one launch's ramp overlaps the previous launch's tail as it does in a step
  const bool pdl = m->use_pdl;
  auto one = [&](int layer) -> cudaError_t {
    const LayerW& w = m->layers[layer];
    GemvParams p = {};
    p.error = m->flags + 2;
    p.R = rows;
    p.eps = g.eps;
    switch (kind) {
      case 0:  // gate|up + SwiGLU (the largest per-layer matrix pair)
        p.w[0] = p.w[1] = p.w[2] = w.gate;
        p.wpair = w.up;
        p.seg_start[1] = p.seg_start[2] = p.N = I;
        p.K = H;
        p.xf = m->x;
        p.gamma = w.post_norm;
        p.ob = m->hbuf;
        p.ldo = I;
        return launch_gemv(m->stream, pdl, kXNorm, kEpiSwiGLU, p, m->gemv_grid);
      case 1:  // q|k|v
        p.w[0] = w.q;
        p.w[1] = w.k;
        p.w[2] = w.v;
        p.seg_start[1] = qd;
        p.seg_start[2] = qd + kd;
        p.col0[1] = qd;
        p.col0[2] = qd + kd;
        p.N = qd + 2 * kd;
        p.K = H;
        p.xf = m->x;
        p.gamma = w.in_norm;
        p.ob = m->qkv;
        p.ldo = p.N;
        return launch_gemv(m->stream, pdl, kXNorm, kEpiBf16, p, m->gemv_grid);
      case 2:  // down + residual
        p.w[0] = p.w[1] = p.w[2] = w.down;
        p.seg_start[1] = p.seg_start[2] = p.N = H;
        p.K = I;
        p.xb = m->hbuf;
        p.of = m->x;
        p.ldo = H;
        return launch_gemv(m->stream, pdl, kXBf16, kEpiResidual, p, m->gemv_grid);
      case 4:  // o + residual
        p.w[0] = p.w[1] = p.w[2] = w.o;
        p.seg_start[1] = p.seg_start[2] = p.N = H;
        p.K = qd;
        p.xb = m->attn;
        p.of = m->x;
        p.ldo = H;
        return launch_gemv(m->stream, pdl, kXBf16, kEpiResidual, p, m->gemv_grid);
      default:  // LM head
        return encode_head(*m, m->stream, pdl, 0, rows, 0, kPhaseVocab, nullptr);
    }
  };
  const double per_row_bytes = kind == 0 ? 2.0 * I * H * 2 : kind == 1 ? (double)(qd + 2 * kd) * H * 2
                               : kind == 2 ? (double)H * I * 2 : kind == 4 ? (double)H * qd * 2
                                                                           : (double)g.vocab * H * 2;
  for (int i = 0; i < 3; ++i) CK(one(i % g.layers));
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  CK(cudaEventRecord(a, m->stream));
  for (int i = 0; i < launches; ++i) CK(one(i % g.layers));
  CK(cudaEventRecord(b, m->stream));
  CK(cudaEventSynchronize(b));
  float ms = 0.f;
  CK(cudaEventElapsedTime(&ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  *avg_ms = ms / launches;
  *bytes = per_row_bytes;
  return 0;
}
