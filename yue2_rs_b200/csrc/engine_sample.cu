// Sampling side of the host engine: request-local generators, sampling::choose on the
// device, and the decode session behind sampling::generate (src/sampling.rs:222-294):
// prefill every song, draw its first token, then one CUDA-graph launch per token
// (forward of every CFG row in one weight pass || the next MT19937 words, then the
// on-device CFG mix + choose that feeds the next forward).
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "engine.h"
#include "kernels.h"

using namespace y2;

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #expr);   \
  } while (0)

namespace {

// Generator::new (src/sampling.rs:15-24)
void mt_seed(MtState& s, uint64_t seed) {
  memset(&s, 0, sizeof(s));
  s.st[0] = (uint32_t)seed;
  for (uint32_t i = 1; i < 624; ++i) s.st[i] = 1812433253u * (s.st[i - 1] ^ (s.st[i - 1] >> 30)) + i;
  s.next = 624;
}

// Sampling::validate (src/protocol.rs:182-194)
int validate_sampling(const Yue2Sampling* s) {
  if (!s) return fail(YUE2_ERR_INVALID, "null sampling");
  if (!std::isfinite(s->temperature) || !(s->temperature >= 0.f && s->temperature <= 5.f) ||
      !std::isfinite(s->top_p) || s->top_p <= 0.f || s->top_p > 1.f || s->top_k < 1 ||
      !std::isfinite(s->repetition_penalty) || s->repetition_penalty <= 0.f || s->penalty_window < 1 ||
      s->penalty_window > 100 || s->min_tokens > s->max_tokens || s->max_tokens < 1)
    return fail(YUE2_ERR_INVALID, "Invalid sampling configuration");
  return 0;
}

SampleCfg make_cfg(const Yue2Sampling* s, int phase) {
  SampleCfg c;
  c.temperature = s->temperature;
  c.top_p = s->top_p;
  c.repetition_penalty = s->repetition_penalty;
  c.top_k = (int32_t)std::min<uint64_t>(s->top_k, 0x7fffffff);
  c.penalty_window = (int32_t)s->penalty_window;
  c.min_tokens = (int32_t)std::min<uint64_t>(s->min_tokens, 0x7fffffff);
  c.max_tokens = (int32_t)std::min<uint64_t>(s->max_tokens, 0x7fffffff);
  c.phase = phase;
  return c;
}

int choose_vocab_check(uint64_t V, int phase) {
  if (phase == kPhaseVocab) return 0;
  const uint64_t end = phase == kPhaseAbc ? kAbcEnd : kMusicEnd;
  if (phase < 0 || phase > 2) return fail(YUE2_ERR_INVALID, "unknown phase");
  if (V <= end) return fail(YUE2_ERR_VOCAB, "Vocabulary does not support native music protocol");
  if (phase == kPhaseSemantic && V < (uint64_t)(kCodecOffset + kCodecSize))
    return fail(YUE2_ERR_VOCAB, "Incomplete codec vocabulary");
  return 0;
}

int err_message(int status) {
  switch (status) {
    case YUE2_ERR_LOGITS: return fail(status, "Model produced invalid logits");
    case YUE2_ERR_EMPTY: return fail(status, "Empty sampling distribution");
    default: return fail(status, "sampler failed with status " + std::to_string(status));
  }
}

// Device scratch of the sampler for `n` requests over a vocabulary of V.
struct SamplerBufs {
  SampleReq* reqs = nullptr;
  int32_t* tokens = nullptr;
  MtState* mt = nullptr;
  uint32_t* words = nullptr;
  float *scores = nullptr, *expv = nullptr;
  unsigned long long* sortbuf = nullptr;
  int32_t* flags = nullptr;  // [0] live requests, [1] all done
  SampleAcc* acc = nullptr;
  int sort_cap = 0;
  Yue2Model* m = nullptr;
  std::vector<void*> owned;  // the model's scratch buffers, returned on destruction

  int get(void** p, size_t bytes) {
    const int rc = m->scratch_take(p, bytes);
    if (!rc) owned.push_back(*p);
    return rc;
  }

  int alloc(Yue2Model* model, size_t n, size_t V, size_t max_tokens, bool need_words) {
    m = model;
    sort_cap = 1;
    while ((size_t)sort_cap < V) sort_cap <<= 1;
    int rc;
    if ((rc = get((void**)&reqs, n * sizeof(SampleReq))) || (rc = get((void**)&tokens, n * max_tokens * 4 + 4)) ||
        (rc = get((void**)&mt, n * sizeof(MtState))) || (rc = get((void**)&scores, n * V * 4)) ||
        (rc = get((void**)&expv, n * V * 4)) || (rc = get((void**)&sortbuf, n * sort_cap * 8)) ||
        (rc = get((void**)&flags, 64)))
      return rc;
    if (need_words && (rc = get((void**)&words, n * 2 * V * 4))) return rc;
    if ((rc = get((void**)&acc, n * sizeof(SampleAcc)))) return rc;
    std::vector<SampleAcc> zero(n, SampleAcc{0, 0, ~0ull});
    if (cudaMemcpy(acc, zero.data(), n * sizeof(SampleAcc), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      return fail(YUE2_ERR_CUDA, "sampler accumulator initialisation failed");
    }
    return 0;
  }
  ~SamplerBufs() {
    for (void* p : owned) m->scratch_give(p);
  }
};

SampleParams make_params(Yue2Model& m, SamplerBufs& b, const SampleCfg& cfg, int V, const float* logits, int ldl) {
  SampleParams p = {};
  p.logits = logits;
  p.ldl = ldl;
  p.vocab = V;
  p.cfg = cfg;
  p.reqs = b.reqs;
  p.rows = m.rows;
  p.words = b.words;
  p.scores = b.scores;
  p.expv = b.expv;
  p.sortbuf = b.sortbuf;
  p.sort_cap = b.sort_cap;
  p.live = b.flags;
  p.all_done = b.flags + 1;
  p.acc = b.acc;
  return p;
}

}  // namespace

struct Yue2Session {
  Yue2Model* m = nullptr;
  Yue2Sampling s{};
  SampleCfg cfg{};
  int phase = 0;
  size_t n = 0;
  int R = 0;
  bool wide = false;  // more than kMaxRows rows: the GEMM forward
  std::vector<Yue2Cache*> caches;
  std::vector<int> cond_row, uncond_row;
  SamplerBufs bufs;
  SampleParams sp{};
  cudaGraphExec_t graph = nullptr;
  static constexpr int kWindow = 8;
  cudaEvent_t ring[kWindow] = {};
  int32_t* pinned = nullptr;  // done flag copies, one slot per ring entry
  uint64_t launched = 0;      // decode graph launches so far
  bool finished = false;
  double prefill_seconds = 0;

  ~Yue2Session() {
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    if (graph) cudaGraphExecDestroy(graph);
    for (auto& e : ring)
      if (e) cudaEventDestroy(e);
    if (pinned) cudaFreeHost(pinned);
    for (Yue2Cache* c : caches) yue2_cache_free(c);
  }
};

extern "C" {

// ---------------------------------------------------------------- generators
int yue2_rng_create(Yue2Model* m, uint64_t seed, Yue2Rng** out) {
  if (!m || !out) return fail(YUE2_ERR_INVALID, "null argument");
  *out = nullptr;
  int rc = y2_set_device(m);
  if (rc) return rc;
  MtState h;
  mt_seed(h, seed);
  Yue2Rng* r = new Yue2Rng();
  r->m = m;
  cudaError_t e = cudaMalloc(&r->state, sizeof(MtState));
  if (e != cudaSuccess) {
    delete r;
    return cuda_fail(e, "rng state");
  }
  if ((e = cudaMemcpy(r->state, &h, sizeof(h), cudaMemcpyHostToDevice)) != cudaSuccess) {
    yue2_rng_free(r);
    return cuda_fail(e, "rng state upload");
  }
  *out = r;
  return 0;
}

void yue2_rng_free(Yue2Rng* r) {
  if (!r) return;
  cudaSetDevice(r->m->device);
  cudaFree(r->state);
  delete r;
}

int yue2_rng_state(const Yue2Rng* r, uint32_t* state, uint64_t* next) {
  if (!r || !state || !next) return fail(YUE2_ERR_INVALID, "null argument");
  int rc = y2_set_device(r->m);
  if (rc) return rc;
  MtState h;
  CK(cudaMemcpy(&h, r->state, sizeof(h), cudaMemcpyDeviceToHost));
  memcpy(state, h.st, sizeof(h.st));
  *next = h.next;
  return 0;
}

// ---------------------------------------------------------------- choose
int yue2_choose(Yue2Model* m, const float* logits, uint64_t vocab, const Yue2Sampling* s, const int64_t* history,
                uint64_t hlen, uint64_t step, int phase, int legacy, Yue2Rng* rng, int64_t* out) {
  if (!m || !logits || !rng || !out || (hlen && !history)) return fail(YUE2_ERR_INVALID, "null argument");
  if (rng->m != m) return fail(YUE2_ERR_INVALID, "generator belongs to another model");
  if (vocab == 0 || vocab > (1u << 30)) return fail(YUE2_ERR_INVALID, "vocabulary size");
  int rc = validate_sampling(s);
  if (rc || (rc = choose_vocab_check(vocab, phase))) return rc;
  if (hlen > 0x7fffffff || step > 0x7fffffff) return fail(YUE2_ERR_INVALID, "history too long");
  std::vector<int32_t> hist(hlen + 1);
  for (uint64_t i = 0; i < hlen; ++i) {
    if (history[i] < 0 || (uint64_t)history[i] >= vocab) return fail(YUE2_ERR_INVALID, "history id outside vocabulary");
    hist[i] = (int32_t)history[i];
  }
  if ((rc = y2_set_device(m))) return rc;
  SamplerBufs b;
  const bool draw = s->temperature != 0.f;
  if ((rc = b.alloc(m, 1, vocab, hlen + 1, draw))) return rc;
  float* d_logits = nullptr;
  if ((rc = b.get((void**)&d_logits, vocab * 4))) return rc;
  CK(cudaMemcpy(d_logits, logits, vocab * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(b.tokens, hist.data(), hist.size() * 4, cudaMemcpyHostToDevice));
  SampleReq q = {};
  q.cond_row = 0;
  q.uncond_row = -1;
  q.scale = 1.f;
  q.legacy = legacy ? 1 : 0;
  q.step = (int32_t)step;
  q.hist_len = (int32_t)hlen;
  q.truncated = 1;
  q.last = -1;
  q.bookkeeping = 0;
  q.tokens = b.tokens;
  CK(cudaMemcpy(b.reqs, &q, sizeof(q), cudaMemcpyHostToDevice));
  const int32_t live[2] = {1, 0};
  CK(cudaMemcpy(b.flags, live, 8, cudaMemcpyHostToDevice));
  if (draw) {
    // the MT kernel advances rng->state by 2*vocab words (sampling.rs:198-213)
    CK(launch_mt_words(m->stream, rng->state, b.words, (int)(2 * vocab), b.reqs, 1));
  }
  SampleParams p = make_params(*m, b, make_cfg(s, phase), (int)vocab, d_logits, (int)vocab);
  p.rows = nullptr;
  CK(launch_sample(m->stream, false, p, 1));
  CK(cudaMemcpyAsync(&q, b.reqs, sizeof(q), cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if (q.status) return err_message(q.status);
  *out = q.last;
  return 0;
}

// ---------------------------------------------------------------- sessions
int yue2_session_create(Yue2Model* m, const Yue2Sampling* s, int phase, const Yue2Request* reqs, uint64_t n,
                        Yue2Session** out) {
  if (!m || !reqs || !out || n == 0) return fail(YUE2_ERR_INVALID, "null argument");
  *out = nullptr;
  if (!m->finalized) return fail(YUE2_ERR_INVALID, "model not finalized");
  int rc = validate_sampling(s);
  if (rc || (rc = check_phase_vocab(*m, phase))) return rc;
  const auto t0 = std::chrono::steady_clock::now();
  int R = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const Yue2Request& q = reqs[i];
    // sampling.rs:233-242
    if (q.context_fill + q.prefix_len + s->max_tokens > (uint64_t)kContext ||
        (q.negative && q.context_fill + q.negative_len + s->max_tokens > (uint64_t)kContext))
      return fail(YUE2_ERR_CAPACITY, "Prefix + requested generation budget exceeds 24576; no implicit truncation");
    if (q.scale != 1.f && !q.negative) return fail(YUE2_ERR_INVALID, "Guidance requires negative prefix");
    if (!q.prefix || q.prefix_len == 0 || (q.scale != 1.f && q.negative_len == 0))
      return fail(YUE2_ERR_INVALID, "Empty prefill");
    R += q.scale != 1.f ? 2 : 1;
  }
  if (R > kMaxWideRows)
    return fail(YUE2_ERR_INVALID, "at most 256 decode rows (CFG rows count twice) per session");
  if (m->tp_world > 1 && R > kTpRows)
    return fail(YUE2_ERR_INVALID, "a tensor-parallel session decodes one song (two rows with CFG)");
  if ((rc = tp_ready(*m))) return rc;
  if ((rc = y2_set_device(m))) return rc;
  const bool wide = R >= m->wide_min && m->tp_world == 1;  // the GEMM path (gemm_rows.cu)
  if (wide && (rc = ensure_wide(*m))) return rc;
  Yue2Session* ss = new Yue2Session();
  ss->m = m;
  ss->s = *s;
  ss->cfg = make_cfg(s, phase);
  ss->phase = phase;
  ss->n = n;
  ss->R = R;
  ss->wide = wide;
  auto bail = [&](int code) {
    delete ss;
    return code;
  };
  // ---- caches and prefills (model.rs:508-522 via sampling.rs:245-255)
  int row = 0;
  std::vector<int32_t*> d_prompts;
  auto free_prompts = [&]() {
    cudaStreamSynchronize(m->stream);  // queued prefills may still read them
    for (int32_t* p : d_prompts) m->scratch_give(p);
  };
  for (uint64_t i = 0; i < n; ++i) {
    const Yue2Request& q = reqs[i];
    const bool cfg = q.scale != 1.f;
    for (int side = 0; side < (cfg ? 2 : 1); ++side) {
      const int64_t* ids = side ? q.negative : q.prefix;
      const uint64_t len = side ? q.negative_len : q.prefix_len;
      Yue2Cache* c = nullptr;
      if ((rc = yue2_cache_create(m, q.context_fill + len + s->max_tokens, &c))) {
        free_prompts();
        return bail(rc);
      }
      ss->caches.push_back(c);
      if (q.context_fill && (rc = yue2_cache_fill_normal(c, q.context_fill, q.seed * 2 + side + 1))) {
        free_prompts();
        return bail(rc);
      }
      std::vector<int32_t> h(len);
      for (uint64_t j = 0; j < len; ++j) {
        if (ids[j] < 0 || ids[j] >= m->g.vocab) {
          free_prompts();
          return bail(fail(YUE2_ERR_TOKEN, "Token outside model vocabulary"));
        }
        h[j] = (int32_t)ids[j];
      }
      int32_t* d = nullptr;
      if ((rc = m->scratch_take((void**)&d, len * 4))) {
        free_prompts();
        return bail(rc);
      }
      d_prompts.push_back(d);
      cudaError_t e;
      if ((e = cudaMemcpy(d, h.data(), len * 4, cudaMemcpyHostToDevice)) != cudaSuccess) {
        free_prompts();
        return bail(cuda_fail(e, "prompt upload"));
      }
      // wide sessions: logits row 0 of the GEMV workspace, then into the wide logits
      if ((rc = prefill_device(*m, *c, d, len, wide ? 0 : row, phase))) {
        free_prompts();
        return bail(rc);
      }
      if (wide) {
        const size_t vb = (size_t)m->g.vocab * 4;
        cudaError_t ce = cudaMemcpyAsync(m->wide_logits + (size_t)row * m->g.vocab, m->logits, vb,
                                         cudaMemcpyDeviceToDevice, m->stream);
        if (ce != cudaSuccess) {
          free_prompts();
          return bail(cuda_fail(ce, "prefill logits"));
        }
      }
      (side ? ss->uncond_row : ss->cond_row).push_back(row);
      ++row;
    }
    if (!cfg) ss->uncond_row.push_back(-1);
  }
  cudaError_t e = cudaStreamSynchronize(m->stream);
  free_prompts();
  if (e != cudaSuccess) return bail(cuda_fail(e, "prefill"));
  if ((rc = take_flags(*m))) return bail(rc);
  ss->prefill_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

  // ---- sampler state
  const int V = m->g.vocab;
  const bool draw = s->temperature != 0.f;
  if ((rc = ss->bufs.alloc(m, n, V, s->max_tokens, draw))) return bail(rc);
  std::vector<SampleReq> hq(n);
  std::vector<MtState> hm(n);
  for (uint64_t i = 0; i < n; ++i) {
    SampleReq& q = hq[i];
    q = SampleReq{};
    q.cond_row = ss->cond_row[i];
    q.uncond_row = ss->uncond_row[i];
    q.scale = reqs[i].scale;
    q.legacy = reqs[i].legacy ? 1 : 0;
    q.truncated = 1;
    q.last = -1;
    q.bookkeeping = 1;
    q.tokens = ss->bufs.tokens + i * s->max_tokens;
    mt_seed(hm[i], reqs[i].seed);
  }
  CK(cudaMemcpy(ss->bufs.reqs, hq.data(), n * sizeof(SampleReq), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(ss->bufs.mt, hm.data(), n * sizeof(MtState), cudaMemcpyHostToDevice));
  const int32_t flags[2] = {(int32_t)n, 0};
  CK(cudaMemcpy(ss->bufs.flags, flags, 8, cudaMemcpyHostToDevice));
  // decode rows: one new token per cache per step
  std::vector<DevRow> rows(R);
  for (int r = 0; r < R; ++r) {
    rows[r] = DevRow{};
    rows[r].pages = ss->caches[r]->d_pages;
    rows[r].pos = (int32_t)ss->caches[r]->length;
    rows[r].active = 1;
    rows[r].advance = 1;
  }
  if (wide) {
    if ((e = cudaMemcpyAsync(m->wide_rows, rows.data(), R * sizeof(DevRow), cudaMemcpyHostToDevice, m->stream)) !=
        cudaSuccess)
      return bail(cuda_fail(e, "row descriptors"));
    ss->sp = make_params(*m, ss->bufs, ss->cfg, V, m->wide_logits, V);
    ss->sp.rows = m->wide_rows;
  } else {
    if ((rc = upload_rows(*m, rows))) return bail(rc);
    ss->sp = make_params(*m, ss->bufs, ss->cfg, V, m->logits, V);
  }

  // ---- step 0: the first token comes from the prefill logits (sampling.rs:260-267)
  if (draw && (e = launch_mt_words(m->stream, ss->bufs.mt, ss->bufs.words, 2 * V, ss->bufs.reqs, (int)n)))
    return bail(cuda_fail(e, "mt words"));
  if ((e = launch_sample(m->stream, false, ss->sp, (int)n)) != cudaSuccess) return bail(cuda_fail(e, "sample"));

  // ---- decode step graph: forward(R rows) || MT words, then sample
  if (s->max_tokens > 1) {
    if (wide && (rc = prepare_wide(*m, R, phase))) return bail(rc);
    m->ctx_hint = 0;
    for (int r = 0; r < R; ++r) m->ctx_hint = std::max(m->ctx_hint, (int)rows[r].pos + 1);
    // the graph is replayed for every later token: the attention form must suit the whole run
    m->ctx_growth = (int)std::min<uint64_t>(s->max_tokens, 1u << 20);
    cudaGraph_t graph;
    if ((e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
      return bail(cuda_fail(e, "capture"));
    cudaError_t ce = cudaSuccess;
    if (draw) {
      ce = cudaEventRecord(m->ev_fork, m->stream);
      if (ce == cudaSuccess) ce = cudaStreamWaitEvent(m->side, m->ev_fork, 0);
      if (ce == cudaSuccess) ce = launch_mt_words(m->side, ss->bufs.mt, ss->bufs.words, 2 * V, ss->bufs.reqs, (int)n);
      if (ce == cudaSuccess) ce = cudaEventRecord(m->ev_join, m->side);
    }
    int wrc = 0;
    if (ce == cudaSuccess) {
      if (wide) {
        if ((wrc = encode_forward_wide(*m, m->stream, R, phase))) ce = cudaErrorUnknown;
      } else {
        ce = encode_forward(*m, m->stream, R, true, phase, ss->bufs.flags + 1);
      }
    }
    if (ce == cudaSuccess && draw) ce = cudaStreamWaitEvent(m->stream, m->ev_join, 0);
    if (ce == cudaSuccess) ce = launch_sample(m->stream, false, ss->sp, (int)n);
    e = cudaStreamEndCapture(m->stream, &graph);
    m->ctx_growth = 0;
    if (wrc) {
      if (e == cudaSuccess) cudaGraphDestroy(graph);
      return bail(wrc);
    }
    if (ce != cudaSuccess) return bail(cuda_fail(ce, "decode step capture"));
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaStreamEndCapture"));
    e = cudaGraphInstantiate(&ss->graph, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaGraphInstantiate"));
    for (auto& ev : ss->ring)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess)
        return bail(cuda_fail(e, "events"));
    if ((e = cudaMallocHost(&ss->pinned, Yue2Session::kWindow * 4)) != cudaSuccess)
      return bail(cuda_fail(e, "pinned flags"));
    memset(ss->pinned, 0, Yue2Session::kWindow * 4);
  }
  *out = ss;
  return 0;
}

void* yue2_session_stream(Yue2Session* ss) { return ss ? (void*)ss->m->stream : nullptr; }

uint64_t yue2_session_kernels_per_step(const Yue2Session* ss) {
  if (!ss) return 0;
  const uint64_t forward = ss->wide ? (uint64_t)wide_kernels_per_step(*ss->m, ss->phase, ss->R)
                                    : (uint64_t)kernels_per_step(*ss->m, true, ss->phase, ss->R);
  return forward + (ss->s.temperature != 0.f ? 1 : 0) + 2;
}

int yue2_session_step(Yue2Session* ss, uint64_t steps, uint64_t* launched) {
  if (!ss) return fail(YUE2_ERR_INVALID, "null session");
  if (launched) *launched = 0;
  int rc = y2_set_device(ss->m);
  if (rc) return rc;
  const uint64_t limit = ss->s.max_tokens - 1;  // forwards of sampling.rs:281-286
  const int W = Yue2Session::kWindow;
  uint64_t done = 0;
  while (done < steps && !ss->finished && ss->launched < limit) {
    const uint64_t t = ss->launched;
    if (t >= (uint64_t)W) {  // bound the run-ahead; read the done flag of launch t-W
      CK(cudaEventSynchronize(ss->ring[t % W]));
      if (ss->pinned[t % W]) {
        ss->finished = true;
        break;
      }
    }
    CK(cudaGraphLaunch(ss->graph, ss->m->stream));
    CK(cudaMemcpyAsync(ss->pinned + t % W, ss->bufs.flags + 1, 4, cudaMemcpyDeviceToHost, ss->m->stream));
    CK(cudaEventRecord(ss->ring[t % W], ss->m->stream));
    ++ss->launched;
    ++done;
  }
  if (launched) *launched = done;
  return 0;
}

int yue2_session_sync(Yue2Session* ss) {
  if (!ss) return fail(YUE2_ERR_INVALID, "null session");
  int rc = y2_set_device(ss->m);
  if (rc) return rc;
  CK(cudaStreamSynchronize(ss->m->stream));
  return 0;
}

// Copies each song's tokens/count/truncated/status into reqs[i]; returns the first error.
int yue2_session_collect(Yue2Session* ss, Yue2Request* reqs) {
  if (!ss || !reqs) return fail(YUE2_ERR_INVALID, "null argument");
  int rc = y2_set_device(ss->m);
  if (rc) return rc;
  CK(cudaStreamSynchronize(ss->m->stream));
  std::vector<SampleReq> hq(ss->n);
  CK(cudaMemcpy(hq.data(), ss->bufs.reqs, ss->n * sizeof(SampleReq), cudaMemcpyDeviceToHost));
  std::vector<int32_t> tok(ss->n * ss->s.max_tokens);
  CK(cudaMemcpy(tok.data(), ss->bufs.tokens, tok.size() * 4, cudaMemcpyDeviceToHost));
  int first = 0;
  for (size_t i = 0; i < ss->n; ++i) {
    Yue2Request& q = reqs[i];
    q.count = (uint64_t)hq[i].step;
    q.truncated = hq[i].truncated;
    q.status = hq[i].status;
    if (q.tokens)
      for (uint64_t j = 0; j < q.count; ++j) q.tokens[j] = tok[i * ss->s.max_tokens + j];
    if (q.status && !first) first = q.status;
  }
  if (first) return err_message(first);
  return take_flags(*ss->m);
}

void yue2_session_free(Yue2Session* ss) { delete ss; }

int yue2_generate(Yue2Model* m, const Yue2Sampling* s, int phase, Yue2Request* reqs, uint64_t n, Yue2Timing* timing) {
  const auto t0 = std::chrono::steady_clock::now();
  Yue2Session* ss = nullptr;
  int rc = yue2_session_create(m, s, phase, reqs, n, &ss);
  if (rc) return rc;
  cudaEvent_t a = nullptr, b = nullptr;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, m->stream);
  uint64_t launched = 0;
  rc = yue2_session_step(ss, s->max_tokens, &launched);
  cudaEventRecord(b, m->stream);
  if (!rc) rc = yue2_session_collect(ss, reqs);
  float ms = 0.f;
  cudaEventSynchronize(b);
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (timing) {
    timing->prefill_seconds = ss->prefill_seconds;
    timing->decode_ms = ms;
    timing->decode_steps = ss->launched;
    timing->kernels_per_step = yue2_session_kernels_per_step(ss);
  }
  yue2_session_free(ss);
  if (timing) timing->seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return rc;
}

}  // extern "C"
