// The acoustic stage's host driver: Model::synthesize (src/model.rs:699-776) over the device
// prefill and velocity.
//
// One song's codec frames are cut into chunks of (min(CONTEXT, max_position_embeddings) -
// prefix - 3) / 2 frames. Each chunk prefills prefix + codec ids + MUSIC_END into a fresh
// cache, then integrates the flow ODE from the chunk's slice of one song-wide noise tensor:
// `steps` midpoint steps, each two yue2_velocity calls, with the state updates rounded to
// bf16 as the reference rounds them. The noise is generated on the host, as the reference
// does: MT19937 uniform_f32 draws, then a 16-element-block Box-Muller with the host libm
// (src/sampling.rs:10-78).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "detmath.h"
#include "engine.h"
#include "kernels.h"

using namespace y2;

namespace {

constexpr uint64_t kLatent = 64;  // the latent width synthesize accepts

// Generator (src/sampling.rs:10-41): MT19937 seeded from the low 32 bits of the seed.
struct HostMt {
  uint32_t s[624];
  int next = 624;
  explicit HostMt(uint64_t seed) {
    s[0] = (uint32_t)seed;
    for (uint32_t i = 1; i < 624; ++i) s[i] = 1812433253u * (s[i - 1] ^ (s[i - 1] >> 30)) + i;
  }
  uint32_t u32() {
    if (next == 624) {
      for (int i = 0; i < 624; ++i) {
        const uint32_t y = (s[i] & 0x80000000u) | (s[(i + 1) % 624] & 0x7fffffffu);
        s[i] = s[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
      }
      next = 0;
    }
    uint32_t y = s[next++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    return y ^ (y >> 18);
  }
};

// Generator::normal_tensor (src/sampling.rs:63-78) over `count` elements (a multiple of 16).
void normal_tensor(uint64_t seed, size_t count, float* out) {
  HostMt g(seed);
  for (size_t i = 0; i < count; ++i) out[i] = (float)(g.u32() & 0x00ffffffu) / 16777216.0f;
  for (size_t b = 0; b + 16 <= count; b += 16) {
    float* blk = out + b;
    for (int i = 0; i < 8; ++i) {
      const float radius = sqrtf(-2.0f * logf(1.0f - blk[i]));
      const float theta = (float)(6.283185307179586 * (double)blk[i + 8]);
      blk[i] = radius * cosf(theta);
      blk[i + 8] = radius * sinf(theta);
    }
  }
}

// logit (src/model.rs:778-780)
double logit(double t) { return std::min(20.0, std::max(-20.0, std::log(t / (1.0 - t)))); }

}  // namespace

extern "C" int yue2_noise(uint64_t seed, uint64_t rows, uint64_t cols, float* out) {
  if (!out) return fail(YUE2_ERR_INVALID, "null argument");
  if (cols && rows > UINT64_MAX / cols) return fail(YUE2_ERR_INVALID, "noise tensor size overflows");
  const uint64_t n = rows * cols;
  if (n < 16 || n % 16) return fail(YUE2_ERR_INVALID, "normal_tensor needs a multiple of 16 elements");
  normal_tensor(seed, n, out);
  return 0;
}

static int synthesize(Yue2Model* m, const int64_t* prefix, uint64_t prefix_len, const int64_t* codec,
                      uint64_t codec_len, uint64_t seed, uint64_t steps, float* out) {
  const char* shape_msg = "Expected nonempty codec tokens and a 64-dimensional latent model";
  if (!m || !out || (prefix_len && !prefix) || (codec_len && !codec)) return fail(YUE2_ERR_INVALID, "null argument");
  if (!m->nar_arena) return fail(YUE2_ERR_INVALID, "NAR tensors not enabled (yue2_model_enable_nar)");
  if ((uint64_t)m->nar.latent != kLatent || codec_len == 0 || steps == 0) return fail(YUE2_ERR_INVALID, shape_msg);
  if (codec_len > SIZE_MAX / (kLatent * sizeof(float))) return fail(YUE2_ERR_INVALID, "codec length too large");
  for (uint64_t i = 0; i < codec_len; ++i)
    if (codec[i] < 0 || codec[i] >= kCodecSize) return fail(YUE2_ERR_INVALID, shape_msg);
  const uint64_t capacity = std::min<uint64_t>((uint64_t)kContext, m->cfg.max_position_embeddings);
  if (prefix_len >= capacity || capacity < prefix_len + 3 || (capacity - (prefix_len + 3)) / 2 == 0)
    return fail(YUE2_ERR_INVALID, "Prefix leaves no acoustic context");
  const uint64_t size = (capacity - (prefix_len + 3)) / 2;
  std::vector<float> noise(codec_len * kLatent);
  normal_tensor(seed, noise.size(), noise.data());
  const float dt = 1.0f / (float)steps;
  std::vector<int64_t> ids;
  for (uint64_t start = 0; start < codec_len; start += size) {
    const uint64_t end = std::min(start + size, codec_len), rows = end - start;
    ids.assign(prefix, prefix + prefix_len);
    for (uint64_t i = start; i < end; ++i) ids.push_back(codec[i] + kCodecOffset);
    ids.push_back(kMusicEnd);
    // the prefill's positions plus rows + 2 latent positions for the velocity passes
    struct Owned {
      Yue2Cache* c = nullptr;
      ~Owned() { yue2_cache_free(c); }
    } owned;
    int rc = yue2_cache_create(m, ids.size() + rows + 2, &owned.c);
    if (rc) return rc;
    Yue2Cache* cache = owned.c;
    rc = yue2_prefill(m, cache, ids.data(), ids.size(), YUE2_PHASE_VOCAB, nullptr);
    std::vector<float> state(noise.begin() + start * kLatent, noise.begin() + end * kLatent);
    std::vector<float> first(state.size()), mid(state.size()), vel(state.size());
    for (float& v : state) v = round_bf16(v);
    for (uint64_t step = 0; step < steps && !rc; ++step) {
      const double t = 1.0 - (double)step / (double)steps;
      if ((rc = yue2_velocity(m, cache, state.data(), rows, logit(t), first.data()))) break;
      for (size_t i = 0; i < state.size(); ++i) mid[i] = round_bf16(state[i] - round_bf16(first[i] * (dt / 2.0f)));
      if ((rc = yue2_velocity(m, cache, mid.data(), rows, logit(t - 0.5 / (double)steps), vel.data()))) break;
      for (size_t i = 0; i < state.size(); ++i) state[i] = round_bf16(state[i] - round_bf16(vel[i] * dt));
    }
    if (rc) return rc;
    for (float v : state)
      if (!std::isfinite(v)) return fail(YUE2_ERR_INVALID, "Flow matching produced nonfinite latents");
    memcpy(out + start * kLatent, state.data(), state.size() * sizeof(float));
  }
  return 0;
}

extern "C" int yue2_synthesize(Yue2Model* m, const int64_t* prefix, uint64_t prefix_len, const int64_t* codec,
                               uint64_t codec_len, uint64_t seed, uint64_t steps, float* out) {
  try {  // host vectors sized by the caller's song: no exception crosses the C ABI
    return synthesize(m, prefix, prefix_len, codec, codec_len, seed, steps, out);
  } catch (const std::bad_alloc&) {
    return fail(YUE2_ERR_OOM, "host allocation failed");
  } catch (const std::exception& e) {  // e.g. std::length_error from a vector size
    return fail(YUE2_ERR_INVALID, std::string("host error: ") + e.what());
  }
}
