// yue2 decode oracle -- TEST INFRASTRUCTURE, NOT PART OF THE PRODUCT.
//
// A scalar host build of the reference's CPU decode math (twally3/yue2_rs):
//   * src/model.rs  : Attention/Rotary/Mlp (94-215), CPU attention (314-397),
//                     embed/forward/project_phase/prefill/hidden (452-610)
//   * src/tensor.rs : Tensor::add + round_bf16 (632-652), silu (658-686),
//                     softmax_row (706-724), Linear::finish (1102-1118), Norm (1120-1173)
//   * src/sampling.rs: Generator/MT19937 (10-62), choose (103-215), generate + CFG mix (222-294)
//   * src/protocol.rs: token constants (6-16), Sampling::validate (182-194)
// Apple Accelerate (cblas_sgemv/sgemm, vDSP, vvexpf) is replaced by plain loops.
// Label: "scalar host build of the reference's model.rs/sampling.rs decode math
// (Accelerate replaced by scalar loops)".
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
// this library, and only as the checker or the timed CPU baseline. The product
// path (yue2_rs_b200/libyue2cuda.so) never calls it.
//
// Pinning: the MT19937 stream is pinned against std::mt19937 known answers and the
// decode attention against the reference's own test (tensor.rs:7-83). The
// reference ships no vectors for GEMV, norms, RoPE, CFG mix, choose or end-to-end
// logits and cannot be built on Linux, so those parts are "parity unpinned"
// beyond this line-by-line restatement.
//
// The exp/log1p used by `choose` come from detmath.h (shared with the device
// sampler) so that token ids are bit-exact given identical logits; detmath is
// itself checked against libm in tests/test_oracle_detmath.py.
#include "../yue2_rs_b200/csrc/detmath.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

// src/protocol.rs:6-16
constexpr size_t EOD = 151643;
constexpr size_t ABC_END = 151848;
constexpr size_t MUSIC_END = 151852;
constexpr size_t CODEC_OFFSET = 151853;
constexpr size_t CODEC_SIZE = 32768;
constexpr size_t CONTEXT = 24576;

thread_local std::string g_error;
int fail(const std::string& m) {
  g_error = m;
  return -1;
}

struct Config {
  size_t hidden, layers, heads, kv, dim, inter, vocab, max_pos;
  float eps, theta;
  int tie;
};

struct Matrix {  // raw bf16 bits, row-major [rows, cols]
  std::vector<uint16_t> w;
  size_t rows = 0, cols = 0;
};

struct Layer {
  Matrix q, k, v, o, gate, up, down;
  std::vector<float> in_norm, q_norm, k_norm, post_norm;
};

struct Model {
  Config c;
  Matrix embed, lm_head;
  std::vector<float> final_norm;
  std::vector<Layer> layers;
  bool ready = false;
  // NAR pathway (model.rs:246-270, 401-451): per-layer nar_* weights (in_norm =
  // nar_input_layernorm, post_norm = nar_pre_mlp_layernorm), latent projections and the
  // time embedder; enabled by orc_model_nar
  bool nar_on = false;
  size_t latent = 0, max_frames = 0;
  float shift = 1.f;
  std::vector<Layer> nar;
  Matrix pe, vae2llm, llm2vae, time_in, time_out;
  std::vector<float> vae2llm_b, llm2vae_b, time_in_b, time_out_b;
};

struct Cache {
  std::vector<std::vector<float>> key, value;  // per layer [length, kv*dim], bf16-valued f32
  size_t length = 0, capacity = 0;
};

struct Rng {  // src/sampling.rs:10-62
  uint32_t s[624];
  size_t next;
};

inline float bf(uint16_t b) { return det_u2f((uint32_t)b << 16); }
inline uint16_t to_bf(float f) { return (uint16_t)(det_f2u(round_bf16(f)) >> 16); }

float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  if (exp == 0) {
    if (man == 0) return det_u2f(sign);
    float v = (float)man * (1.0f / 16777216.0f);  // man * 2^-24
    return sign ? -v : v;
  }
  if (exp == 31) return det_u2f(sign | 0x7f800000u | (man << 13));
  return det_u2f(sign | ((exp + 112) << 23) | (man << 13));
}

// Summation order of the dot products: Accelerate's cblas_sgemv order is unknown, so the
// checker offers two valid restatements -- 16 interleaved partial sums (default) and a
// strictly sequential sum. Their disagreement measures how far bf16 rounding after every
// op amplifies a change of f32 summation order (the parity noise floor).
int g_dot_order = 0;

// y[r, n] = round_bf16(sum_k W[n,k] x[r,k] [+ bias[n]]) -- Linear::apply + finish
// (tensor.rs:946-1118; the bias, already bf16-rounded, is added before the rounding)
void linear(const Matrix& W, const float* x, size_t rows, float* y, size_t begin = 0, size_t end = SIZE_MAX,
            const std::vector<float>* bias = nullptr) {
  if (end == SIZE_MAX) end = W.rows;
  const size_t K = W.cols, N = end - begin;
#pragma omp parallel
  {
    std::vector<float> wrow(K);
#pragma omp for schedule(static)
    for (long long n = 0; n < (long long)N; ++n) {
      const uint16_t* src = &W.w[(begin + n) * K];
      for (size_t k = 0; k < K; ++k) wrow[k] = bf(src[k]);
      for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * K;
        if (g_dot_order == 1) {
          float s = 0.f;
          for (size_t k = 0; k < K; ++k) s += wrow[k] * xr[k];
          if (bias) s += (*bias)[begin + n];
          y[r * N + n] = round_bf16(s);
          continue;
        }
        float acc[16] = {0};
        size_t k = 0;
        for (; k + 16 <= K; k += 16)
          for (int l = 0; l < 16; ++l) acc[l] += wrow[k + l] * xr[k + l];
        float s = 0.f;
        for (int l = 0; l < 16; ++l) s += acc[l];
        for (; k < K; ++k) s += wrow[k] * xr[k];
        if (bias) s += (*bias)[begin + n];
        y[r * N + n] = round_bf16(s);
      }
    }
  }
}

// Norm::apply (tensor.rs:1140-1157) on each row of width w.size()
void norm_rows(const std::vector<float>& g, float eps, float* x, size_t rows, size_t width, float* out) {
  for (size_t r = 0; r < rows; ++r) {
    const float* row = x + r * width;
    float sum = 0.f;
    for (size_t i = 0; i < width; ++i) sum += row[i] * row[i];
    float scale = 1.0f / sqrtf(sum / (float)width + eps);
    scale = round_bf16(scale);
    for (size_t i = 0; i < width; ++i) out[r * width + i] = round_bf16(round_bf16(row[i] * scale) * g[i]);
  }
}

// Rotary::new + Rotary::apply (model.rs:137-168)
struct Rotary {
  std::vector<float> cos, sin;
  size_t half, rows;
  Rotary(size_t start, size_t rows_, const Config& c) : half(c.dim / 2), rows(rows_) {
    cos.resize(rows * half);
    sin.resize(rows * half);
    for (size_t i = 0; i < half; ++i) {
      float freq = 1.0f / powf(c.theta, (float)(2 * i) / (float)c.dim);
      for (size_t r = 0; r < rows; ++r) {
        float angle = (float)(start + r) * freq;
        cos[r * half + i] = round_bf16(cosf(angle));
        sin[r * half + i] = round_bf16(sinf(angle));
      }
    }
  }
  void apply(float* x, size_t cols) const {
    for (size_t r = 0; r < rows; ++r)
      for (size_t i = 0; i < half; ++i) {
        float c = cos[r * half + i], s = sin[r * half + i];
        for (size_t h = 0; h < cols / (2 * half); ++h) {
          size_t a = r * cols + h * 2 * half + i, b = a + half;
          float left = x[a], right = x[b];
          x[a] = round_bf16(round_bf16(left * c) - round_bf16(right * s));
          x[b] = round_bf16(round_bf16(right * c) + round_bf16(left * s));
        }
      }
  }
};

// CPU attention (model.rs:314-397) for `rows` queries whose first row sits at
// position `causal_start`; keys = key rows of this layer's cache.
void attention(const Config& c, const float* q, size_t rows, const std::vector<float>& key,
               const std::vector<float>& value, size_t key_rows, size_t causal_start, float* out) {
  const size_t qcols = c.heads * c.dim, kcols = c.kv * c.dim, groups = c.heads / c.kv;
  const float scale = 1.0f / sqrtf((float)c.dim);
  for (size_t start = 0; start < rows; start += 256) {
    size_t nrows = std::min<size_t>(rows - start, 256);
    size_t keys = std::min(causal_start + start + nrows, key_rows);
#pragma omp parallel for schedule(static) collapse(2)
    for (long long head = 0; head < (long long)c.heads; ++head)
      for (long long r = 0; r < (long long)nrows; ++r) {
        std::vector<float> scores(keys);
        size_t kh = head / groups;
        const float* qr = q + (start + r) * qcols + head * c.dim;
        for (size_t j = 0; j < keys; ++j) {
          const float* kr = &key[j * kcols + kh * c.dim];
          float s = 0.f;
          for (size_t d = 0; d < c.dim; ++d) s += qr[d] * kr[d];
          scores[j] = s;
        }
        // softmax_row (tensor.rs:706-724); a causal start past the keys sees every key
        size_t visible = std::min<size_t>(causal_start + start + r + 1, keys);
        for (size_t j = visible; j < keys; ++j) scores[j] = 0.f;
        float mx = -INFINITY;
        for (size_t j = 0; j < visible; ++j) {
          scores[j] *= scale;
          mx = std::max(mx, scores[j]);
        }
        float sum = 0.f;
        for (size_t j = 0; j < visible; ++j) {
          scores[j] = expf(scores[j] - mx);
          sum += scores[j];
        }
        for (size_t j = 0; j < visible; ++j) scores[j] /= sum;
        float* o = out + (start + r) * qcols + head * c.dim;
        for (size_t d = 0; d < c.dim; ++d) {
          float acc = 0.f;
          for (size_t j = 0; j < keys; ++j) acc += scores[j] * value[j * kcols + kh * c.dim + d];
          o[d] = round_bf16(acc);  // out.rounded()
        }
      }
  }
}

// Model::hidden CPU branch (model.rs:523-591); returns final-normed rows.
int hidden(Model& m, Cache& cache, const int64_t* ids, size_t n, std::vector<float>& out) {
  const Config& c = m.c;
  if (n == 0 || cache.length + n > cache.capacity || cache.length + n > c.max_pos ||
      cache.key.size() != m.layers.size())
    return fail("AR input exceeds cache/model context");
  const size_t H = c.hidden, qd = c.heads * c.dim, kd = c.kv * c.dim;
  std::vector<float> x(n * H);
  for (size_t r = 0; r < n; ++r) {  // Model::embed (model.rs:452-464)
    if (ids[r] < 0 || (size_t)ids[r] >= c.vocab) return fail("Token outside model vocabulary");
    for (size_t i = 0; i < H; ++i) x[r * H + i] = bf(m.embed.w[(size_t)ids[r] * H + i]);
  }
  Rotary rot(cache.length, n, c);
  std::vector<float> h(n * H), q(n * qd), k(n * kd), v(n * kd), att(n * qd), proj(n * H);
  std::vector<float> gate(n * c.inter), up(n * c.inter);
  for (size_t li = 0; li < m.layers.size(); ++li) {
    Layer& L = m.layers[li];
    norm_rows(L.in_norm, c.eps, x.data(), n, H, h.data());
    linear(L.q, h.data(), n, q.data());
    linear(L.k, h.data(), n, k.data());
    linear(L.v, h.data(), n, v.data());
    // Norm::heads (tensor.rs:1158-1172)
    norm_rows(L.q_norm, c.eps, q.data(), n * c.heads, c.dim, q.data());
    norm_rows(L.k_norm, c.eps, k.data(), n * c.kv, c.dim, k.data());
    rot.apply(q.data(), qd);
    rot.apply(k.data(), kd);
    cache.key[li].insert(cache.key[li].end(), k.begin(), k.end());
    cache.value[li].insert(cache.value[li].end(), v.begin(), v.end());
    size_t key_rows = cache.key[li].size() / kd;
    attention(c, q.data(), n, cache.key[li], cache.value[li], key_rows, cache.length, att.data());
    linear(L.o, att.data(), n, proj.data());
    for (size_t i = 0; i < n * H; ++i) x[i] = round_bf16(x[i] + proj[i]);
    norm_rows(L.post_norm, c.eps, x.data(), n, H, h.data());
    // Mlp::apply (model.rs:206-214)
    linear(L.gate, h.data(), n, gate.data());
    linear(L.up, h.data(), n, up.data());
    for (size_t i = 0; i < n * c.inter; ++i) {
      float g = gate[i];
      g = round_bf16(g / (1.0f + expf(-g)));
      gate[i] = round_bf16(g * up[i]);
    }
    linear(L.down, gate.data(), n, proj.data());
    for (size_t i = 0; i < n * H; ++i) x[i] = round_bf16(x[i] + proj[i]);
  }
  cache.length += n;
  out.resize(n * H);
  norm_rows(m.final_norm, c.eps, x.data(), n, H, out.data());
  return 0;
}

const Matrix& head_matrix(const Model& m) { return m.c.tie ? m.embed : m.lm_head; }

// project_phase (model.rs:478-507); phase 0 = Abc, 1 = Semantic, 2 = full vocabulary.
int project(const Model& m, const float* x, int phase, float* logits) {
  const Matrix& W = head_matrix(m);
  const size_t V = m.c.vocab;
  if (phase == 2) {
    linear(W, x, 1, logits);
    return 0;
  }
  size_t start, end, stop;
  if (phase == 0) {
    start = 0; end = EOD; stop = ABC_END;
  } else if (phase == 1) {
    start = CODEC_OFFSET; end = CODEC_OFFSET + CODEC_SIZE; stop = MUSIC_END;
  } else {
    return fail("Unknown phase");
  }
  if (end > V || stop >= V) return fail("Vocabulary does not support native music protocol");
  for (size_t i = 0; i < V; ++i) logits[i] = -INFINITY;
  linear(W, x, 1, logits + start, start, end);
  linear(W, x, 1, logits + stop, stop, stop + 1);
  return 0;
}

void rng_init(Rng& g, uint64_t seed) {
  g.s[0] = (uint32_t)seed;
  for (uint32_t i = 1; i < 624; ++i) g.s[i] = 1812433253u * (g.s[i - 1] ^ (g.s[i - 1] >> 30)) + i;
  g.next = 624;
}
uint32_t rng_next(Rng& g) {
  if (g.next == 624) {
    for (size_t i = 0; i < 624; ++i) {
      uint32_t bits = (g.s[i] & 0x80000000u) | (g.s[(i + 1) % 624] & 0x7fffffffu);
      g.s[i] = g.s[(i + 397) % 624] ^ (bits >> 1) ^ ((bits & 1u) ? 0x9908b0dfu : 0u);
    }
    g.next = 0;
  }
  uint32_t y = g.s[g.next++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}
void rng_discard(Rng& g, size_t count) {
  while (count > 0) {
    if (g.next == 624) {
      rng_next(g);
      count -= 1;
    } else {
      size_t skip = std::min<size_t>(624 - g.next, count);
      g.next += skip;
      count -= skip;
    }
  }
}
double rng_uniform_f64(Rng& g) {
  uint64_t high = rng_next(g), low = rng_next(g);
  return (double)(((high << 32) | low) & ((1ull << 53) - 1)) / 9007199254740992.0;
}

}  // namespace

// ---------------------------------------------------------------- C ABI
struct OrcSampling {  // protocol.rs Sampling (142-151)
  float temperature, top_p;
  uint64_t top_k;
  float repetition_penalty;
  uint64_t penalty_window, min_tokens, max_tokens;
};

ORC_API const char* orc_last_error(void) { return g_error.c_str(); }
ORC_API void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
ORC_API void orc_set_dot_order(int order) { g_dot_order = order; }
ORC_API int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// cfg: [hidden, layers, heads, kv, dim, inter, vocab, max_pos, tie]; f: [eps, theta]
ORC_API void* orc_model_create(const uint64_t* cfg, const float* f) {
  Model* m = new Model();
  m->c = Config{cfg[0], cfg[1], cfg[2], cfg[3], cfg[4], cfg[5], cfg[6], cfg[7], f[0], f[1], (int)cfg[8]};
  const Config& c = m->c;
  if (!c.hidden || !c.layers || !c.heads || !c.kv || !c.dim || !c.inter || !c.vocab || c.heads % c.kv ||
      c.dim % 2 || !(c.theta > 0) || !(c.eps > 0)) {
    delete m;
    fail("Invalid transformer configuration");
    return nullptr;
  }
  m->layers.resize(c.layers);
  return m;
}
ORC_API void orc_model_free(void* p) { delete (Model*)p; }

// dtype: 0 bf16, 1 f32, 2 f16 (GpuWeight.dtype, tensor.rs:221-230)
ORC_API int orc_model_set(void* p, const char* name, int dtype, const void* data, uint64_t rows, uint64_t cols) {
  Model* m = (Model*)p;
  const Config& c = m->c;
  std::string n(name);
  size_t count = rows * cols;
  auto value = [&](size_t i) -> float {
    if (dtype == 0) return bf(((const uint16_t*)data)[i]);
    if (dtype == 1) return ((const float*)data)[i];
    return half_to_float(((const uint16_t*)data)[i]);
  };
  auto set_matrix = [&](Matrix& M, size_t r, size_t cc) -> int {
    if (rows != r || cols != cc) return fail("Tensor shape mismatch for " + n);
    M.rows = r;
    M.cols = cc;
    M.w.resize(count);
    for (size_t i = 0; i < count; ++i) M.w[i] = dtype == 0 ? ((const uint16_t*)data)[i] : to_bf(value(i));
    return 0;
  };
  auto set_norm = [&](std::vector<float>& g, size_t d) -> int {
    if (count != d) return fail("Tensor shape mismatch for " + n);
    g.resize(d);
    for (size_t i = 0; i < d; ++i) g[i] = round_bf16(value(i));  // Norm::new rounds (tensor.rs:1126-1136)
    return 0;
  };
  const size_t H = c.hidden, qd = c.heads * c.dim, kd = c.kv * c.dim;
  if (n == "model.embed_tokens.weight") return set_matrix(m->embed, c.vocab, H);
  if (n == "lm_head.weight") return set_matrix(m->lm_head, c.vocab, H);
  if (n == "model.norm.weight") return set_norm(m->final_norm, H);
  unsigned li;
  char rest[128];
  if (m->nar_on) {  // NAR tensors (model.rs:246-270, 428-451)
    const size_t D = m->latent, F = m->max_frames;
    if (n == "latent_pos_embed.pe") return set_matrix(m->pe, F, H);
    if (n == "vae2llm.weight") return set_matrix(m->vae2llm, H, D);
    if (n == "vae2llm.bias") return set_norm(m->vae2llm_b, H);
    if (n == "llm2vae.weight") return set_matrix(m->llm2vae, D, H);
    if (n == "llm2vae.bias") return set_norm(m->llm2vae_b, D);
    if (n == "time_embedder.mlp.0.weight") return set_matrix(m->time_in, H, 256);
    if (n == "time_embedder.mlp.0.bias") return set_norm(m->time_in_b, H);
    if (n == "time_embedder.mlp.2.weight") return set_matrix(m->time_out, H, H);
    if (n == "time_embedder.mlp.2.bias") return set_norm(m->time_out_b, H);
    if (sscanf(name, "model.layers.%u.%127s", &li, rest) == 2 && li < c.layers) {
      Layer& L = m->nar[li];
      std::string r(rest);
      if (r == "nar_input_layernorm.weight") return set_norm(L.in_norm, H);
      if (r == "nar_pre_mlp_layernorm.weight") return set_norm(L.post_norm, H);
      if (r == "nar_self_attn.q_norm.weight") return set_norm(L.q_norm, c.dim);
      if (r == "nar_self_attn.k_norm.weight") return set_norm(L.k_norm, c.dim);
      if (r == "nar_self_attn.q_proj.weight") return set_matrix(L.q, qd, H);
      if (r == "nar_self_attn.k_proj.weight") return set_matrix(L.k, kd, H);
      if (r == "nar_self_attn.v_proj.weight") return set_matrix(L.v, kd, H);
      if (r == "nar_self_attn.o_proj.weight") return set_matrix(L.o, H, qd);
      if (r == "nar_mlp.gate_proj.weight") return set_matrix(L.gate, c.inter, H);
      if (r == "nar_mlp.up_proj.weight") return set_matrix(L.up, c.inter, H);
      if (r == "nar_mlp.down_proj.weight") return set_matrix(L.down, H, c.inter);
    }
  }
  if (sscanf(name, "model.layers.%u.%127s", &li, rest) == 2 && li < c.layers) {
    Layer& L = m->layers[li];
    std::string r(rest);
    if (r == "input_layernorm.weight") return set_norm(L.in_norm, H);
    if (r == "post_attention_layernorm.weight") return set_norm(L.post_norm, H);
    if (r == "self_attn.q_norm.weight") return set_norm(L.q_norm, c.dim);
    if (r == "self_attn.k_norm.weight") return set_norm(L.k_norm, c.dim);
    if (r == "self_attn.q_proj.weight") return set_matrix(L.q, qd, H);
    if (r == "self_attn.k_proj.weight") return set_matrix(L.k, kd, H);
    if (r == "self_attn.v_proj.weight") return set_matrix(L.v, kd, H);
    if (r == "self_attn.o_proj.weight") return set_matrix(L.o, H, qd);
    if (r == "mlp.gate_proj.weight") return set_matrix(L.gate, c.inter, H);
    if (r == "mlp.up_proj.weight") return set_matrix(L.up, c.inter, H);
    if (r == "mlp.down_proj.weight") return set_matrix(L.down, H, c.inter);
  }
  return 1;  // not an AR-path tensor: ignored
}

ORC_API int orc_model_finalize(void* p) {
  Model* m = (Model*)p;
  if (m->embed.w.empty() || m->final_norm.empty() || (!m->c.tie && m->lm_head.w.empty()))
    return fail("Missing embedding, final norm or LM head");
  for (size_t i = 0; i < m->layers.size(); ++i) {
    Layer& L = m->layers[i];
    if (L.q.w.empty() || L.k.w.empty() || L.v.w.empty() || L.o.w.empty() || L.gate.w.empty() ||
        L.up.w.empty() || L.down.w.empty() || L.in_norm.empty() || L.post_norm.empty() ||
        L.q_norm.empty() || L.k_norm.empty())
      return fail("Missing tensor in layer " + std::to_string(i));
  }
  m->ready = true;
  return 0;
}

// Seeded synthetic weights for CPU timing runs: matrices N(0, std) and norm
// gains norm_mean + N(0, std), rounded to bf16 (splitmix64 + Box-Muller).
ORC_API int orc_model_init_synthetic(void* p, uint64_t seed, float std_, float norm_mean) {
  Model* m = (Model*)p;
  const Config& c = m->c;
  uint64_t tensor = 0;
  auto fill = [&](std::vector<uint16_t>& w, size_t count, float mean) {
    w.resize(count);
    uint64_t key = seed * 0x9E3779B97F4A7C15ull + (++tensor) * 0xD1B54A32D192ED03ull;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)(count + 1) / 2; ++i) {
      uint64_t z = key + (uint64_t)i * 0x9E3779B97F4A7C15ull;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      z ^= z >> 31;
      double u1 = ((z >> 11) + 1) * (1.0 / 9007199254740992.0);
      double u2 = (z & 0x1fffff) * (1.0 / 2097152.0);
      double rad = sqrt(-2.0 * log(u1));
      w[2 * i] = to_bf(mean + std_ * (float)(rad * cos(6.283185307179586 * u2)));
      if ((size_t)(2 * i + 1) < count) w[2 * i + 1] = to_bf(mean + std_ * (float)(rad * sin(6.283185307179586 * u2)));
    }
  };
  auto mat = [&](Matrix& M, size_t r, size_t cc) {
    M.rows = r;
    M.cols = cc;
    fill(M.w, r * cc, 0.f);
  };
  auto nrm = [&](std::vector<float>& g, size_t d) {
    std::vector<uint16_t> t;
    fill(t, d, norm_mean);
    g.resize(d);
    for (size_t i = 0; i < d; ++i) g[i] = bf(t[i]);
  };
  const size_t H = c.hidden, qd = c.heads * c.dim, kd = c.kv * c.dim;
  mat(m->embed, c.vocab, H);
  if (!c.tie) mat(m->lm_head, c.vocab, H);
  nrm(m->final_norm, H);
  for (auto& L : m->layers) {
    mat(L.q, qd, H); mat(L.k, kd, H); mat(L.v, kd, H); mat(L.o, H, qd);
    mat(L.gate, c.inter, H); mat(L.up, c.inter, H); mat(L.down, H, c.inter);
    nrm(L.in_norm, H); nrm(L.post_norm, H); nrm(L.q_norm, c.dim); nrm(L.k_norm, c.dim);
  }
  if (m->nar_on) {  // the NAR tensors too (biases N(0, std), gains norm_mean + N(0, std))
    auto bias = [&](std::vector<float>& b, size_t d) {
      std::vector<uint16_t> t;
      fill(t, d, 0.f);
      b.resize(d);
      for (size_t i = 0; i < d; ++i) b[i] = bf(t[i]);
    };
    const size_t D = m->latent;
    mat(m->pe, m->max_frames, H);
    mat(m->vae2llm, H, D); bias(m->vae2llm_b, H);
    mat(m->llm2vae, D, H); bias(m->llm2vae_b, D);
    mat(m->time_in, H, 256); bias(m->time_in_b, H);
    mat(m->time_out, H, H); bias(m->time_out_b, H);
    for (auto& L : m->nar) {
      mat(L.q, qd, H); mat(L.k, kd, H); mat(L.v, kd, H); mat(L.o, H, qd);
      mat(L.gate, c.inter, H); mat(L.up, c.inter, H); mat(L.down, H, c.inter);
      nrm(L.in_norm, H); nrm(L.post_norm, H); nrm(L.q_norm, c.dim); nrm(L.k_norm, c.dim);
    }
  }
  m->ready = true;
  return 0;
}

ORC_API void* orc_cache_create(void* p, uint64_t capacity) {
  Model* m = (Model*)p;
  Cache* c = new Cache();
  c->key.resize(m->c.layers);
  c->value.resize(m->c.layers);
  c->capacity = capacity;
  return c;
}
ORC_API void orc_cache_free(void* p) { delete (Cache*)p; }
ORC_API uint64_t orc_cache_length(void* p) { return ((Cache*)p)->length; }

// Read one layer's cached rows [0, length) as f32 K and V ([length, kv*dim] each).
ORC_API int orc_cache_read(void* p, uint64_t layer, float* k, float* v) {
  Cache* c = (Cache*)p;
  if (layer >= c->key.size()) return fail("layer out of range");
  memcpy(k, c->key[layer].data(), c->key[layer].size() * 4);
  memcpy(v, c->value[layer].data(), c->value[layer].size() * 4);
  return 0;
}

// Write rows [0, length) of every layer from bf16 bits laid out [layer][K|V][length][kv*dim].
ORC_API int orc_cache_write(void* p, void* mp, uint64_t length, const uint16_t* data) {
  Cache* c = (Cache*)p;
  Model* m = (Model*)mp;
  if (length > c->capacity) return fail("length exceeds capacity");
  const size_t kd = m->c.kv * m->c.dim, n = length * kd;
  for (size_t l = 0; l < c->key.size(); ++l) {
    c->key[l].resize(n);
    c->value[l].resize(n);
    const uint16_t* base = data + l * 2 * n;
    for (size_t i = 0; i < n; ++i) {
      c->key[l][i] = bf(base[i]);
      c->value[l][i] = bf(base[n + i]);
    }
  }
  c->length = length;
  return 0;
}

// Model::hidden: n ids through every layer; out = final-normed rows [n, H].
ORC_API int orc_hidden(void* mp, void* cp, const int64_t* ids, uint64_t n, float* out) {
  std::vector<float> x;
  int rc = hidden(*(Model*)mp, *(Cache*)cp, ids, n, x);
  if (rc == 0 && out) memcpy(out, x.data(), x.size() * 4);
  return rc;
}

// Model::forward (model.rs:465-468) with phase 2, forward_phase (469-477) with phase 0/1.
ORC_API int orc_forward(void* mp, void* cp, const int64_t* ids, uint64_t n, int phase, float* logits) {
  Model& m = *(Model*)mp;
  std::vector<float> x;
  int rc = hidden(m, *(Cache*)cp, ids, n, x);
  if (rc) return rc;
  return project(m, x.data() + (n - 1) * m.c.hidden, phase, logits);
}

// Model::prefill / prefill_phase (model.rs:508-522, 592-610): chunks of 256 ids.
ORC_API int orc_prefill(void* mp, void* cp, const int64_t* ids, uint64_t n, int phase, float* logits) {
  Model& m = *(Model*)mp;
  if (n == 0) return fail("Empty prefill");
  std::vector<float> x;
  for (uint64_t s = 0; s < n; s += 256) {
    uint64_t len = std::min<uint64_t>(256, n - s);
    int rc = hidden(m, *(Cache*)cp, ids + s, len, x);
    if (rc) return rc;
  }
  if (!logits) return 0;
  return project(m, x.data() + (x.size() / m.c.hidden - 1) * m.c.hidden, phase, logits);
}

ORC_API int orc_attention(const float* q, const float* k, const float* v, float* out, uint64_t keys,
                          uint64_t heads, uint64_t kv, uint64_t dim) {
  Config c{};
  c.heads = heads;
  c.kv = kv;
  c.dim = dim;
  std::vector<float> K(k, k + keys * kv * dim), V(v, v + keys * kv * dim);
  attention(c, q, 1, K, V, keys, keys - 1, out);
  return 0;
}

// Linear::apply + finish on host rows: y[rows, out] from x[rows, in] and bf16 W[out, in].
ORC_API int orc_linear(const uint16_t* w, uint64_t out, uint64_t in, const float* x, uint64_t rows, float* y) {
  Matrix M;
  M.rows = out;
  M.cols = in;
  M.w.assign(w, w + out * in);
  linear(M, x, rows, y);
  return 0;
}

ORC_API int orc_norm(const float* gamma, uint64_t width, float eps, const float* x, uint64_t rows, float* out) {
  std::vector<float> g(gamma, gamma + width), in(x, x + rows * width);
  norm_rows(g, eps, in.data(), rows, width, out);
  return 0;
}

// ---- sampling.rs
ORC_API void* orc_rng_create(uint64_t seed) {
  Rng* g = new Rng();
  rng_init(*g, seed);
  return g;
}
ORC_API void orc_rng_free(void* p) { delete (Rng*)p; }
ORC_API uint32_t orc_rng_next_u32(void* p) { return rng_next(*(Rng*)p); }
ORC_API double orc_rng_uniform_f64(void* p) { return rng_uniform_f64(*(Rng*)p); }
ORC_API float orc_rng_uniform_f32(void* p) { return (float)(rng_next(*(Rng*)p) & 0x00ffffffu) / 16777216.0f; }
ORC_API void orc_rng_discard(void* p, uint64_t n) { rng_discard(*(Rng*)p, n); }
ORC_API void orc_rng_state(void* p, uint32_t* state, uint64_t* next) {
  Rng* g = (Rng*)p;
  memcpy(state, g->s, sizeof(g->s));
  *next = g->next;
}

ORC_API int orc_sampling_validate(const OrcSampling* s) {  // protocol.rs:182-194
  if (!std::isfinite(s->temperature) || !(s->temperature >= 0.f && s->temperature <= 5.f) ||
      !std::isfinite(s->top_p) || s->top_p <= 0.f || s->top_p > 1.f || s->top_k < 1 ||
      !std::isfinite(s->repetition_penalty) || s->repetition_penalty <= 0.f || s->penalty_window < 1 ||
      s->penalty_window > 100 || s->min_tokens > s->max_tokens || s->max_tokens < 1)
    return fail("Invalid sampling configuration");
  return 0;
}

static inline float cast(float x, int legacy) { return legacy ? round_bf16(x) : x; }

// sampling::choose (sampling.rs:103-215). phase 0 Abc, 1 Semantic, 2 vocabulary-generic
// (no window, no stop row: the deviation used at vocab 84,000).
ORC_API int orc_choose(const float* logits, uint64_t V, const OrcSampling* sp, const int64_t* history,
                       uint64_t hlen, uint64_t step, int phase, int legacy, void* rp, int64_t* out) {
  Rng& rng = *(Rng*)rp;
  std::vector<float> scores(V, -INFINITY);
  size_t end = SIZE_MAX;
  if (phase == 0 || phase == 1) {
    end = phase == 0 ? ABC_END : MUSIC_END;
    if (V <= end) return fail("Vocabulary does not support native music protocol");
    if (phase == 0) {
      std::copy(logits, logits + EOD, scores.begin());
    } else {
      if (V < CODEC_OFFSET + CODEC_SIZE) return fail("Incomplete codec vocabulary");
      std::copy(logits + CODEC_OFFSET, logits + CODEC_OFFSET + CODEC_SIZE, scores.begin() + CODEC_OFFSET);
    }
    if (step >= sp->min_tokens) scores[end] = logits[end];
  } else {
    std::copy(logits, logits + V, scores.begin());
  }
  std::map<int64_t, int> freq;
  size_t from = hlen > sp->penalty_window ? hlen - sp->penalty_window : 0;
  for (size_t i = from; i < hlen; ++i) freq[history[i]] += 1;
  for (auto& kv : freq) {
    if (kv.first < 0 || (uint64_t)kv.first >= V) return fail("history id outside vocabulary");
    float alpha = cast(powi_f32(sp->repetition_penalty, kv.second), legacy);
    float& s = scores[kv.first];
    s = cast(s < 0.f ? s * alpha : s / alpha, legacy);
  }
  for (float s : scores)
    if (std::isnan(s) || s == INFINITY) return fail("Model produced invalid logits");
  if (sp->temperature == 0.f) {
    int64_t best = -1;
    for (size_t i = 0; i < V; ++i) {
      if (!std::isfinite(scores[i])) continue;
      if (best < 0 || total_key(scores[i]) > total_key(scores[best])) best = (int64_t)i;
    }
    if (best < 0) return fail("Empty sampling distribution");
    *out = best;
    return 0;
  }
  if (sp->temperature != 1.f)
    for (auto& s : scores) s = cast(s / sp->temperature, legacy);
  std::vector<uint32_t> sorted;
  for (size_t i = 0; i < V; ++i)
    if (std::isfinite(scores[i])) sorted.push_back((uint32_t)i);
  if (sorted.empty()) return fail("Empty sampling distribution");
  auto before = [&](uint32_t a, uint32_t b) {  // score desc (total order), id asc
    uint32_t ka = total_key(scores[a]), kb = total_key(scores[b]);
    return ka != kb ? ka > kb : a < b;
  };
  size_t rank = std::min<size_t>(sp->top_k - 1, sorted.size() - 1);
  std::nth_element(sorted.begin(), sorted.begin() + rank, sorted.end(), before);
  float threshold = scores[sorted[rank]];
  sorted.erase(std::remove_if(sorted.begin(), sorted.end(), [&](uint32_t i) { return !(scores[i] >= threshold); }),
               sorted.end());
  std::sort(sorted.begin(), sorted.end(), before);
  if (sp->top_p < 1.f) {
    float mx = scores[sorted[0]];
    float sum = 0.f;
    for (uint32_t i : sorted) sum += det_expf(scores[i] - mx);
    float cumulative = 0.f;
    size_t protect = legacy ? 3 : 1;
    std::vector<uint32_t> keep;
    for (size_t i = 0; i < sorted.size(); ++i) {
      float p = cast(det_expf(scores[sorted[i]] - mx) / sum, legacy);
      cumulative += p;
      float prior = cast(cast(cumulative, legacy) - p, legacy);
      if (prior <= sp->top_p || i < protect) keep.push_back(sorted[i]);
    }
    sorted.swap(keep);
  }
  float mx = scores[sorted[0]];
  float sum = 0.f;
  for (uint32_t i : sorted) sum += det_expf(scores[i] - mx);
  std::vector<std::pair<uint32_t, float>> probs;
  for (uint32_t i : sorted) probs.push_back({i, cast(det_expf(scores[i] - mx) / sum, legacy)});
  std::sort(probs.begin(), probs.end());
  float best = -INFINITY;
  int64_t selected = 0;
  size_t cursor = 0;
  for (auto& pr : probs) {
    rng_discard(rng, (pr.first - cursor) * 2);
    float noise = cast(det_d2f(-det_log1p(-rng_uniform_f64(rng))), legacy);
    cursor = pr.first + 1;
    float score = cast(pr.second / noise, legacy);
    if (score > best) {
      best = score;
      selected = pr.first;
    }
  }
  rng_discard(rng, (V - cursor) * 2);
  *out = selected;
  return 0;
}

// CFG mix (sampling.rs:261-266): l = bf16(u + bf16(s * bf16(c - u)))
ORC_API void orc_cfg_mix(const float* c, const float* u, float scale, float* out, uint64_t V) {
  for (size_t i = 0; i < V; ++i) out[i] = round_bf16(u[i] + round_bf16(scale * round_bf16(c[i] - u[i])));
}

// sampling::generate (sampling.rs:222-294). tokens holds max_tokens entries.
ORC_API int orc_generate(void* mp, const int64_t* prefix, uint64_t n, const int64_t* negative, uint64_t nn,
                         const OrcSampling* sp, uint64_t seed, int phase, float scale, int legacy,
                         int64_t* tokens, uint64_t* count, int* truncated) {
  Model& m = *(Model*)mp;
  if (orc_sampling_validate(sp)) return -1;
  if (n + sp->max_tokens > CONTEXT || (negative && nn + sp->max_tokens > CONTEXT))
    return fail("Prefix + requested generation budget exceeds 24576; no implicit truncation");
  if (scale != 1.f && !negative) return fail("Guidance requires negative prefix");
  const size_t V = m.c.vocab;
  Cache cond, uncond;
  cond.key.resize(m.c.layers); cond.value.resize(m.c.layers); cond.capacity = n + sp->max_tokens;
  std::vector<float> lc(V), lu(V), mix(V);
  int rc = orc_prefill(mp, &cond, prefix, n, phase, lc.data());
  if (rc) return rc;
  bool cfg = scale != 1.f;
  if (cfg) {
    uncond.key.resize(m.c.layers); uncond.value.resize(m.c.layers); uncond.capacity = nn + sp->max_tokens;
    rc = orc_prefill(mp, &uncond, negative, nn, phase, lu.data());
    if (rc) return rc;
  }
  Rng rng;
  rng_init(rng, seed);
  std::vector<int64_t> hist;
  *truncated = 1;
  int64_t stop = phase == 0 ? (int64_t)ABC_END : phase == 1 ? (int64_t)MUSIC_END : -1;
  for (uint64_t step = 0; step < sp->max_tokens; ++step) {
    if (cfg) orc_cfg_mix(lc.data(), lu.data(), scale, mix.data(), V);
    else mix = lc;
    int64_t id;
    rc = orc_choose(mix.data(), V, sp, hist.data(), hist.size(), step, phase, legacy, &rng, &id);
    if (rc) return rc;
    if (id == stop) {
      *truncated = 0;
      break;
    }
    hist.push_back(id);
    if (step + 1 < sp->max_tokens) {
      rc = orc_forward(mp, &cond, &id, 1, phase, lc.data());
      if (rc) return rc;
      if (cfg) {
        rc = orc_forward(mp, &uncond, &id, 1, phase, lu.data());
        if (rc) return rc;
      }
    }
  }
  memcpy(tokens, hist.data(), hist.size() * 8);
  *count = hist.size();
  return 0;
}

// ---- the shared deterministic functions, exported for their own tests
ORC_API float orc_det_expf(float x) { return det_expf(x); }
ORC_API double orc_det_log1p(double x) { return det_log1p(x); }
ORC_API float orc_round_bf16(float x) { return round_bf16(x); }
ORC_API float orc_powi(float a, int b) { return powi_f32(a, b); }

// ---------------------------------------------------------------- NAR velocity
// Enables the NAR tensors (Config latent_dim, max_latent_frames, timestep_shift).
ORC_API int orc_model_nar(void* p, uint64_t latent_dim, uint64_t max_frames, float shift) {
  Model* m = (Model*)p;
  if (!latent_dim || !max_frames || !(shift > 0.f)) return fail("Invalid latent configuration");
  m->nar_on = true;
  m->latent = latent_dim;
  m->max_frames = max_frames;
  m->shift = shift;
  m->nar.resize(m->c.layers);
  return 0;
}

// Model::velocity CPU branch (model.rs:611-697) with nar_cond_end = 0: the latent rows
// (state, zero-padded by one row on each side) at positions cache.length.. attend to the
// whole cache prefix and to each other; out = llm2vae(final_norm(x))[1 .. rows + 1].
ORC_API int orc_velocity(void* mp, void* cp, const float* state, uint64_t rows, double raw_t, float* out) {
  Model& m = *(Model*)mp;
  Cache& cache = *(Cache*)cp;
  const Config& c = m.c;
  if (!m.nar_on || m.vae2llm.w.empty() || m.llm2vae.w.empty() || m.time_in.w.empty() || m.time_out.w.empty() ||
      m.pe.w.empty())
    return fail("NAR tensors missing");
  for (auto& L : m.nar)
    if (L.q.w.empty() || L.down.w.empty() || L.in_norm.empty() || L.post_norm.empty() || L.q_norm.empty())
      return fail("NAR tensors missing");
  if (cache.key.size() != m.layers.size()) return fail("cache/model mismatch");
  const size_t n = rows + 2, H = c.hidden, D = m.latent, qd = c.heads * c.dim, kd = c.kv * c.dim;
  std::vector<float> padded(n * D, 0.f), x(n * H);
  for (size_t i = 0; i < rows * D; ++i) padded[D + i] = state[i];
  linear(m.vae2llm, padded.data(), n, x.data(), 0, SIZE_MAX, &m.vae2llm_b);
  // timestep embedding (f32 math in the reference's order)
  const float raw = round_bf16((float)raw_t);
  const float sig = round_bf16(1.0f / (1.0f + expf(-raw)));
  const float top = round_bf16(m.shift * sig);
  const float bottom = round_bf16(1.f + round_bf16((m.shift - 1.f) * sig));
  const float t = round_bf16(top / bottom);
  std::vector<float> sinus(256), time(H), time2(H);
  for (int i = 0; i < 128; ++i) {
    const float f = expf(-logf(10000.f) * (float)i / 128.f);
    sinus[i] = round_bf16(cosf(t * f));
    sinus[128 + i] = round_bf16(sinf(t * f));
  }
  linear(m.time_in, sinus.data(), 1, time.data(), 0, SIZE_MAX, &m.time_in_b);
  for (auto& v : time) v = round_bf16(v / (1.0f + expf(-v)));
  linear(m.time_out, time.data(), 1, time2.data(), 0, SIZE_MAX, &m.time_out_b);
  for (size_t r = 0; r < n; ++r)
    for (size_t i = 0; i < H; ++i) {
      const float pe = round_bf16(bf(m.pe.w[std::min(r, m.max_frames - 1) * H + i]));
      float& v = x[r * H + i];
      v = round_bf16(round_bf16(v + time2[i]) + pe);
    }
  const size_t visible = cache.length;
  Rotary rot(cache.length, n, c);
  std::vector<float> h(n * H), q(n * qd), k(n * kd), v(n * kd), att(n * qd), proj(n * H);
  std::vector<float> gate(n * c.inter), up(n * c.inter);
  for (size_t li = 0; li < m.nar.size(); ++li) {
    Layer& L = m.nar[li];
    norm_rows(L.in_norm, c.eps, x.data(), n, H, h.data());
    linear(L.q, h.data(), n, q.data());
    linear(L.k, h.data(), n, k.data());
    linear(L.v, h.data(), n, v.data());
    norm_rows(L.q_norm, c.eps, q.data(), n * c.heads, c.dim, q.data());
    norm_rows(L.k_norm, c.eps, k.data(), n * c.kv, c.dim, k.data());
    rot.apply(q.data(), qd);
    rot.apply(k.data(), kd);
    std::vector<float> key(cache.key[li].begin(), cache.key[li].begin() + visible * kd);
    std::vector<float> value(cache.value[li].begin(), cache.value[li].begin() + visible * kd);
    key.insert(key.end(), k.begin(), k.end());
    value.insert(value.end(), v.begin(), v.end());
    attention(c, q.data(), n, key, value, visible + n, visible + n, att.data());  // no causal mask
    linear(L.o, att.data(), n, proj.data());
    for (size_t i = 0; i < n * H; ++i) x[i] = round_bf16(x[i] + proj[i]);
    norm_rows(L.post_norm, c.eps, x.data(), n, H, h.data());
    linear(L.gate, h.data(), n, gate.data());
    linear(L.up, h.data(), n, up.data());
    for (size_t i = 0; i < n * c.inter; ++i) {
      float g = gate[i];
      g = round_bf16(g / (1.0f + expf(-g)));
      gate[i] = round_bf16(g * up[i]);
    }
    linear(L.down, gate.data(), n, proj.data());
    for (size_t i = 0; i < n * H; ++i) x[i] = round_bf16(x[i] + proj[i]);
  }
  std::vector<float> fin(n * H), lat(n * D);
  norm_rows(m.final_norm, c.eps, x.data(), n, H, fin.data());
  linear(m.llm2vae, fin.data(), n, lat.data(), 0, SIZE_MAX, &m.llm2vae_b);
  for (size_t i = 0; i < rows * D; ++i) out[i] = lat[D + i];
  return 0;
}

// Generator::normal_tensor (src/sampling.rs:63-78): every element first draws uniform_f32;
// then in each block of 16, elements i and i + 8 (i < 8) become a Box-Muller pair in f32
// (the angle is formed in f64 and cast).
static void normal_tensor(uint64_t seed, size_t count, float* out) {
  Rng g;
  rng_init(g, seed);
  for (size_t i = 0; i < count; ++i) out[i] = (float)(rng_next(g) & 0x00ffffffu) / 16777216.0f;
  for (size_t b = 0; b + 16 <= count; b += 16) {
    float* blk = out + b;
    for (int i = 0; i < 8; ++i) {
      const float radius = sqrtf(-2.f * logf(1.f - blk[i]));
      const float theta = (float)(2.0 * 3.14159265358979323846 * (double)blk[i + 8]);
      blk[i] = radius * cosf(theta);
      blk[i + 8] = radius * sinf(theta);
    }
  }
}

ORC_API int orc_normal_tensor(uint64_t seed, uint64_t rows, uint64_t cols, float* out) {
  const size_t n = rows * cols;
  if (n < 16 || n % 16) return fail("normal_tensor needs a multiple of 16 elements");
  normal_tensor(seed, n, out);
  return 0;
}

// logit (src/model.rs:778-780)
static double logit(double t) { return std::min(20.0, std::max(-20.0, std::log(t / (1.0 - t)))); }

// Model::synthesize (src/model.rs:699-776): chunks of `size` codec frames; each chunk
// prefills prefix + codec ids + MUSIC_END, then runs `steps` midpoint steps of the flow ODE
// from the chunk's slice of one song-wide noise tensor. out [codec_len, 64].
ORC_API int orc_synthesize(void* mp, const int64_t* prefix, uint64_t plen, const int64_t* codec, uint64_t clen,
                           uint64_t seed, uint64_t steps, float* out) {
  Model& m = *(Model*)mp;
  const uint64_t kContext = 24576, kMusicEnd = 151852, kCodecOffset = 151853, kCodecSize = 32768;
  if (!m.nar_on || m.latent != 64 || clen == 0 || steps == 0)
    return fail("Expected nonempty codec tokens and a 64-dimensional latent model");
  for (uint64_t i = 0; i < clen; ++i)
    if (codec[i] < 0 || (uint64_t)codec[i] >= kCodecSize)
      return fail("Expected nonempty codec tokens and a 64-dimensional latent model");
  const uint64_t capacity = std::min<uint64_t>(kContext, m.c.max_pos);
  if (capacity < plen + 3 || (capacity - (plen + 3)) / 2 == 0) return fail("Prefix leaves no acoustic context");
  const uint64_t size = (capacity - (plen + 3)) / 2;
  const size_t D = 64;
  std::vector<float> noise(clen * D);
  normal_tensor(seed, noise.size(), noise.data());
  const float dt = 1.f / (float)steps;
  for (uint64_t start = 0; start < clen; start += size) {
    const uint64_t end = std::min(start + size, clen), rows = end - start;
    std::vector<int64_t> ids(prefix, prefix + plen);
    for (uint64_t i = start; i < end; ++i) ids.push_back(codec[i] + (int64_t)kCodecOffset);
    ids.push_back((int64_t)kMusicEnd);
    Cache* cache = (Cache*)orc_cache_create(mp, ids.size());
    int rc = orc_prefill(mp, cache, ids.data(), ids.size(), 2, nullptr);
    std::vector<float> state(noise.begin() + start * D, noise.begin() + end * D), first(rows * D), mid(rows * D),
        vel(rows * D);
    for (auto& v : state) v = round_bf16(v);
    for (uint64_t step = 0; step < steps && !rc; ++step) {
      const double t = 1.0 - (double)step / (double)steps;
      if ((rc = orc_velocity(mp, cache, state.data(), rows, logit(t), first.data()))) break;
      for (size_t i = 0; i < state.size(); ++i) mid[i] = round_bf16(state[i] - round_bf16(first[i] * (dt / 2.f)));
      if ((rc = orc_velocity(mp, cache, mid.data(), rows, logit(t - 0.5 / (double)steps), vel.data()))) break;
      for (size_t i = 0; i < state.size(); ++i) state[i] = round_bf16(state[i] - round_bf16(vel[i] * dt));
    }
    delete cache;
    if (rc) return rc;
    for (float v : state)
      if (!std::isfinite(v)) return fail("Flow matching produced nonfinite latents");
    memcpy(out + start * D, state.data(), state.size() * 4);
  }
  return 0;
}
