// On-device CFG mix, sampler and MT19937 stream for sm_100a.
//
// Reference: sampling::generate CFG mix (src/sampling.rs:261-266), sampling::choose
// (src/sampling.rs:103-215), Generator (src/sampling.rs:10-62). Token ids are bit-exact
// with the reference algorithm given identical logits: every float operation of
// `choose` is reproduced in the same order where the order matters (the sequential
// top-p and normalisation sums run on one lane), and exp/ln_1p come from detmath.h.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace y2 {

// ------------------------------------------------------------------ MT19937
// Twist in four dependency phases: [0,227) reads only old words, [227,454) reads
// words from the first phase, [454,623) from the second, and 623 reads the new
// words 0 and 396. Each phase reads everything before any thread writes.
Y2_DEV void mt_phase(uint32_t* st, int lo, int hi) {
  const int i = lo + (int)threadIdx.x;
  const bool act = i < hi;
  uint32_t v = 0;
  if (act) {
    const uint32_t y = (st[i] & 0x80000000u) | (st[(i + 1) % 624] & 0x7fffffffu);
    v = st[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
  }
  __syncthreads();
  if (act) st[i] = v;
  __syncthreads();
}

Y2_DEV uint32_t mt_temper(uint32_t y) {
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

// Emits the next `nwords` tempered outputs of each request's generator (one CTA per
// request) and advances its state; the stream depends only on the seed and on how
// many words were consumed, so it runs beside the forward pass.
__global__ void __launch_bounds__(256) mt_words_kernel(MtState* states, uint32_t* words, int nwords,
                                                        const SampleReq* reqs) {
  const int b = blockIdx.x;
  if (reqs && reqs[b].done) return;
  __shared__ uint32_t st[624];
  MtState* S = states + b;
  for (int i = threadIdx.x; i < 624; i += blockDim.x) st[i] = S->st[i];
  uint32_t next = S->next;
  __syncthreads();
  uint32_t* out = words + (size_t)b * nwords;
  int pos = 0;
  while (pos < nwords) {
    if (next == 624) {
      mt_phase(st, 0, 227);
      mt_phase(st, 227, 454);
      mt_phase(st, 454, 623);
      mt_phase(st, 623, 624);
      next = 0;
    }
    const int n = min(624 - (int)next, nwords - pos);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[pos + i] = mt_temper(st[next + i]);
    pos += n;
    next += n;
    __syncthreads();
  }
  for (int i = threadIdx.x; i < 624; i += blockDim.x) S->st[i] = st[i];
  if (threadIdx.x == 0) S->next = next;
}

cudaError_t launch_mt_words(cudaStream_t s, MtState* st, uint32_t* words, int nwords, const SampleReq* reqs,
                            int nreq) {
  mt_words_kernel<<<nreq, 256, 0, s>>>(st, words, nwords, reqs);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ sampler
Y2_DEV float cast(float x, bool legacy) { return legacy ? round_bf16(x) : x; }

// ascending order of this key == score descending (total order), id ascending
Y2_DEV unsigned long long composite(float s, int id) {
  return ((unsigned long long)(~total_key(s)) << 32) | (uint32_t)id;
}

template <typename T>
Y2_DEV void bitonic_sort(T* a, int m) {
  for (int k = 2; k <= m; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const T x = a[i], y = a[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
}

constexpr int kCand = 2048;  // samples, candidates and survivors sorted in shared memory
constexpr int kSampleThreads = 1024;
constexpr int kPrepChunks = 32;  // CTAs per request in sample_prep_kernel
constexpr int kPrepThreads = 256;

// Phase window [w0, w1) and stop id of choose (sampling.rs:112-129); stop = -1 for none.
Y2_DEV void phase_window(int phase, int V, int& w0, int& w1, int& stop) {
  w0 = 0;
  w1 = V;
  stop = -1;
  if (phase == kPhaseAbc) {
    w1 = (int)kEOD;
    stop = (int)kAbcEnd;
  } else if (phase == kPhaseSemantic) {
    w0 = (int)kCodecOffset;
    w1 = (int)(kCodecOffset + kCodecSize);
    stop = (int)kMusicEnd;
  }
}

// The first three passes of choose over one request's vocabulary, split over
// kPrepChunks CTAs (each a contiguous id range, staged in shared memory):
// A: CFG mix (sampling.rs:261-266) and phase window (sampling.rs:112-129);
// B: repetition penalty over the last penalty_window ids (sampling.rs:130-144);
// C: invalid-logit check, temperature, finite count (sampling.rs:145-167), and for T=0
//    the argmax key (highest total-order score, lowest id; sampling.rs:148-156).
// Every element goes through the same operations as in the single-CTA form. The scores
// go to p.scores; the flag, count and key are combined into p.acc[request] by atomics
// (order-independent: or, sum, min).
__global__ void __launch_bounds__(kPrepThreads) sample_prep_kernel(const SampleParams p) {
  extern __shared__ float sv[];  // this CTA's id range
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, ch = blockIdx.y, tid = threadIdx.x;
  const SampleReq& q = p.reqs[b];
  if (q.done) return;
  const int V = p.vocab;
  const SampleCfg c = p.cfg;
  const bool legacy = q.legacy != 0;
  const int V4 = V >> 2;
  const bool vec = (V & 3) == 0 && (p.ldl & 3) == 0;
  // ranges start on multiples of 4 ids when the rows allow 16-byte loads
  const int lo = vec ? 4 * (int)(((long long)V4 * ch) / kPrepChunks) : (int)(((long long)V * ch) / kPrepChunks);
  const int hi = vec ? 4 * (int)(((long long)V4 * (ch + 1)) / kPrepChunks)
                     : (int)(((long long)V * (ch + 1)) / kPrepChunks);
  const float* lc = p.logits + (size_t)q.cond_row * p.ldl;
  const float* lu = q.uncond_row >= 0 ? p.logits + (size_t)q.uncond_row * p.ldl : nullptr;
  const int step = q.step, hlen = q.hist_len;
  int w0, w1, stop;
  phase_window(c.phase, V, w0, w1, stop);
  const bool stop_on = stop >= 0 && step >= c.min_tokens;
  auto mix = [&](int i, float l, float u) -> float {
    if (lu) l = round_bf16(u + round_bf16(q.scale * round_bf16(l - u)));
    const bool in = (i >= w0 && i < w1) || (stop_on && i == stop);
    return in ? l : -INFINITY;
  };
  // ---- A
  if (vec) {
    const float4* c4 = reinterpret_cast<const float4*>(lc);
    const float4* u4 = reinterpret_cast<const float4*>(lu);
#pragma unroll 4
    for (int j = lo / 4 + tid; j < hi / 4; j += kPrepThreads) {
      const float4 a = c4[j];
      const float4 u = lu ? u4[j] : a;
      const int i = 4 * j;
      sv[i - lo] = mix(i, a.x, u.x);
      sv[i - lo + 1] = mix(i + 1, a.y, u.y);
      sv[i - lo + 2] = mix(i + 2, a.z, u.z);
      sv[i - lo + 3] = mix(i + 3, a.w, u.w);
    }
  } else {
    for (int i = lo + tid; i < hi; i += kPrepThreads) sv[i - lo] = mix(i, lc[i], lu ? lu[i] : 0.f);
  }
  __syncthreads();
  // ---- B: ids of this range among the last penalty_window generated ids
  {
    const int from = max(0, hlen - c.penalty_window);
    const int n = hlen - from;
    for (int k = tid; k < n; k += kPrepThreads) {
      const int id = q.tokens[from + k];
      if (id < lo || id >= hi) continue;
      bool first = true;
      int cnt = 0;
      for (int j = 0; j < n; ++j)
        if (q.tokens[from + j] == id) {
          if (j < k) first = false;
          ++cnt;
        }
      if (first) {
        const float alpha = cast(powi_f32(c.repetition_penalty, cnt), legacy);
        const float s = sv[id - lo];
        sv[id - lo] = cast(s < 0.f ? s * alpha : s / alpha, legacy);
      }
    }
  }
  __syncthreads();
  // ---- C
  const bool t0 = c.temperature == 0.f, t1 = c.temperature == 1.f;
  int bad = 0, nfin = 0;
  unsigned long long best = ~0ull;
  float* S = p.scores + (size_t)b * V;
  for (int i = lo + tid; i < hi; i += kPrepThreads) {
    float s = sv[i - lo];
    if (isnan(s) || s == INFINITY) bad = 1;
    if (t0) {
      if (isfinite(s)) best = min(best, composite(s, i));
    } else {
      if (!t1) s = cast(s / c.temperature, legacy);
      if (isfinite(s)) ++nfin;
    }
    S[i] = s;
  }
  bad = __syncthreads_or(bad);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nfin += __shfl_xor_sync(0xffffffffu, nfin, o);
    best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
  }
  if ((tid & 31) == 0) {
    SampleAcc& a = p.acc[b];
    if (nfin) atomicAdd(&a.nfin, nfin);
    if (best != ~0ull) atomicMin(&a.best, best);
    if (tid == 0 && bad) atomicOr(&a.bad, 1);
  }
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const SampleParams p) {
  __shared__ unsigned long long cand[kCand];
  __shared__ unsigned long long cand2[kCand];  // rank-sorted copy of cand; later per-survivor scratch
  __shared__ float es[kCand];
  __shared__ uint32_t hist[256];
  __shared__ int s_count, s_nkeep;
  __shared__ uint32_t s_prefix, s_target;
  __shared__ float s_sum;

  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nt = blockDim.x;
  SampleReq& q = p.reqs[b];
  if (q.done) return;
  const int V = p.vocab;
  const SampleCfg c = p.cfg;
  const bool legacy = q.legacy != 0;
  float* S = p.scores + (size_t)b * V;
  const int step = q.step, hlen = q.hist_len;

  auto finish = [&](int status, int id) {  // thread 0 only
    q.last = id;
    q.status = status;
    bool newly_done = false;
    if (status != 0) {
      newly_done = true;
    } else if (q.bookkeeping) {
      const int stop = c.phase == kPhaseAbc ? (int)kAbcEnd : c.phase == kPhaseSemantic ? (int)kMusicEnd : -1;
      if (id == stop) {
        q.truncated = 0;
        newly_done = true;
      } else {
        q.tokens[step] = id;
        q.step = step + 1;
        q.hist_len = hlen + 1;
        p.rows[q.cond_row].token = id;
        if (q.uncond_row >= 0) p.rows[q.uncond_row].token = id;
        if (step + 1 >= c.max_tokens) newly_done = true;
      }
    }
    if (newly_done && q.bookkeeping) {
      q.done = 1;
      p.rows[q.cond_row].active = 0;
      if (q.uncond_row >= 0) p.rows[q.uncond_row].active = 0;
      if (p.live && atomicSub(p.live, 1) == 1) *p.all_done = 1;
    }
  };

  // ---- A-C ran in sample_prep_kernel: scores in S, flag/count/argmax key in p.acc[b]
  const bool vec = (V & 3) == 0;  // 16-byte score loads (S rows are V floats apart)
  int w0, w1, stop;
  phase_window(c.phase, V, w0, w1, stop);
  const bool t0 = c.temperature == 0.f;
  __shared__ SampleAcc s_acc;
  if (tid == 0) {
    s_acc = p.acc[b];
    p.acc[b] = SampleAcc{0, 0, ~0ull};  // ready for the next step's prep
    s_count = 0;
  }
  __syncthreads();
  if (s_acc.bad) {
    if (tid == 0) finish(-5, -1);
    return;
  }
  if (t0) {  // greedy: highest total-order score, lowest id (sampling.rs:148-156)
    if (tid == 0) {
      if (s_acc.best == ~0ull) finish(-6, -1);
      else finish(0, (int)(s_acc.best & 0xffffffffu));
    }
    return;
  }
  const int n_finite = s_acc.nfin;
  if (n_finite == 0) {
    if (tid == 0) finish(-6, -1);
    return;
  }

  // ---- D: exact threshold = score at descending rank min(top_k-1, n-1) (select_nth, :168-172)
  const int rank = (int)min((long long)c.top_k - 1, (long long)n_finite - 1);
  const int iters = (V + nt - 1) / nt;
  unsigned long long* gbuf = p.sortbuf + (size_t)b * p.sort_cap;
  // Estimate: sort kCand strided samples of the phase window and take the one expected to
  // leave 3*(rank+1) + 64 elements at or above it; collect every finite element with a key
  // at least that large. The collection is exact whenever it holds rank+1 or more elements
  // (they are then exactly the top of the order); otherwise the general path runs.
  {
    constexpr int kSamples = 1024;
    const int span = w1 - w0;
    for (int j = tid; j < kSamples; j += nt) {
      const int i = w0 + (int)(((long long)j * span) / kSamples);
      const float s = S[i];
      cand[j] = isfinite(s) ? composite(s, i) : ~0ull;
    }
    if (tid == 0) {
      s_count = 0;
      s_nkeep = 0;
    }
    __syncthreads();
    bitonic_sort(cand, kSamples);
    const double want = 3.0 * (rank + 1) + 64.0;
    const int jj = (int)min((double)(kSamples - 1), max(0.0, ceil(want * kSamples / (double)span) - 1.0));
    const unsigned long long est = cand[jj];
    const uint32_t tau = est == ~0ull ? 0u : ~(uint32_t)(est >> 32);
    __syncthreads();  // every thread has read cand[jj] before it is overwritten
    auto take = [&](bool keep, float s, int i) {
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      if (bal == 0) return;  // warp-uniform: candidates are rare
      int base = 0;
      if (lane == 0 && bal) base = atomicAdd(&s_count, __popc(bal));
      base = __shfl_sync(0xffffffffu, base, 0);
      const int pos = base + __popc(bal & ((1u << lane) - 1));
      if (keep && pos < kCand) cand[pos] = composite(s, i);
    };
    if (vec) {  // four scores per thread per step, the next float4 requested before this one is used
      const float4* s4 = reinterpret_cast<const float4*>(S);
      const int V4 = V / 4, it4 = (V4 + nt - 1) / nt;
      const float4 none = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      float4 cur = tid < V4 ? s4[tid] : none;
      for (int it = 0; it < it4; ++it) {
        const int j = it * nt + tid, jn = j + nt;
        const float4 nxt = (it + 1 < it4 && jn < V4) ? s4[jn] : none;
        const float e[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) take(isfinite(e[u]) && total_key(e[u]) >= tau, e[u], 4 * j + u);
        cur = nxt;
      }
    } else {
      for (int it = 0; it < iters; ++it) {
        const int i = it * nt + tid;
        const float s = i < V ? S[i] : -INFINITY;
        take(isfinite(s) && total_key(s) >= tau, s, i);
      }
    }
    __syncthreads();
  }
  const int ncand = s_count;
  int n = -1;
  unsigned long long* srt = nullptr;
  if (ncand > rank && ncand <= kCand) {
    if (ncand <= kSampleThreads) {
      // rank sort: the keys are distinct (they hold the id), so an element's position is
      // the number of smaller keys; one pass instead of a bitonic network
      if (tid < ncand) {
        const unsigned long long key = cand[tid];
        int r = 0;
        for (int j = 0; j < ncand; ++j) r += cand[j] < key ? 1 : 0;
        cand2[r] = key;
      }
      __syncthreads();
      srt = cand2;
    } else {
      int m = 1;
      while (m < ncand) m <<= 1;
      for (int i = ncand + tid; i < m; i += nt) cand[i] = ~0ull;
      __syncthreads();
      bitonic_sort(cand, m);
      srt = cand;
    }
    const uint32_t thr_key = ~(uint32_t)(srt[rank] >> 32);
    // a +-0 threshold: IEEE `>=` (retain, :173) and key order differ there; general path
    if (thr_key != 0x80000000u && thr_key != 0x7fffffffu) {
      int mine = 0;
      for (int i = tid; i < ncand; i += nt) mine += (~(uint32_t)(srt[i] >> 32)) >= thr_key ? 1 : 0;
      atomicAdd(&s_nkeep, mine);
      __syncthreads();
      n = s_nkeep;
    } else {
      srt = nullptr;
    }
  }
  if (n < 0) {
  uint32_t prefix = 0, mask = 0;
  uint32_t target = (uint32_t)rank;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += nt) hist[i] = 0;
    __syncthreads();
    for (int it = 0; it < iters; ++it) {
      const int i = it * nt + tid;
      uint32_t d = 256;
      if (i < V) {
        const float s = S[i];
        if (isfinite(s)) {
          const uint32_t k = total_key(s);
          if ((k & mask) == prefix) d = (k >> shift) & 255u;
        }
      }
      const unsigned peers = __match_any_sync(0xffffffffu, d);
      if (d < 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[d], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t cum = 0;
      for (int d = 255; d >= 0; --d) {
        if (cum + hist[d] > target) {
          s_prefix = prefix | ((uint32_t)d << shift);
          s_target = target - cum;
          break;
        }
        cum += hist[d];
      }
    }
    __syncthreads();
    prefix = s_prefix;
    target = s_target;
    mask |= 255u << shift;
  }
  const float thr = total_key_to_float(prefix);

  // ---- E: survivors: finite and >= threshold (IEEE), as retain() keeps them (:173)
  if (tid == 0) s_count = 0;
  __syncthreads();
  for (int it = 0; it < iters; ++it) {
    const int i = it * nt + tid;
    bool keep = false;
    float s = 0.f;
    if (i < V) {
      s = S[i];
      keep = isfinite(s) && s >= thr;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    int base = 0;
    if (lane == 0 && bal) base = atomicAdd(&s_count, __popc(bal));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (keep) gbuf[base + __popc(bal & ((1u << lane) - 1))] = composite(s, i);
  }
  __syncthreads();
  n = s_count;

  // ---- F: sort by (score desc, id asc) (:174)
  int m = 1;
  while (m < n) m <<= 1;
  if (m <= kCand) {
    for (int i = tid; i < m; i += nt) cand[i] = i < n ? gbuf[i] : ~0ull;
    __syncthreads();
    bitonic_sort(cand, m);
    srt = cand;
  } else {
    for (int i = n + tid; i < m; i += nt) gbuf[i] = ~0ull;
    __syncthreads();
    bitonic_sort(gbuf, m);
    srt = gbuf;
  }
  }  // general path

  // ---- G: top-p, normalisation and the exponential race in warp 0 (:175-213)
  if (warp != 0) return;
  float* E = n <= kCand ? es : p.expv + (size_t)b * V;  // shared memory unless the support is huge
  auto idof = [&](int i) { return (int)(srt[i] & 0xffffffffu); };
  auto scoreof = [&](int i) { return total_key_to_float(~(uint32_t)(srt[i] >> 32)); };  // exact inverse
  const float mx = scoreof(0);
  for (int i = lane; i < n; i += 32) E[i] = det_expf(scoreof(i) - mx);
  __syncwarp();
  int nkeep = n;
  if (c.top_p < 1.f) {
    if (lane == 0) {
      float sum = 0.f;
      for (int i = 0; i < n; ++i) sum += E[i];  // the reference's order
      s_sum = sum;
    }
    __syncwarp();
    const float sum = s_sum;
    const int protect = legacy ? 3 : 1;
    if (n <= kCand && (srt == cand || srt == cand2)) {
      // the probabilities in parallel; only the cumulative sum runs in order on one lane.
      // Scratch: whichever candidate buffer does not hold the sorted survivors.
      unsigned long long* scratch = srt == cand2 ? cand : cand2;
      float* pr = reinterpret_cast<float*>(scratch);
      uint32_t* keep = reinterpret_cast<uint32_t*>(scratch) + kCand;  // bit i: survivor i kept
      for (int i = lane; i < n; i += 32) pr[i] = cast(E[i] / sum, legacy);
      __syncwarp();
      if (lane == 0) {
        float cumulative = 0.f;
        uint32_t bits = 0;
        for (int i = 0; i < n; ++i) {
          cumulative += pr[i];
          const float prior = cast(cast(cumulative, legacy) - pr[i], legacy);
          if (prior <= c.top_p || i < protect) bits |= 1u << (i & 31);
          if ((i & 31) == 31 || i == n - 1) {
            keep[i >> 5] = bits;
            bits = 0;
          }
        }
      }
      __syncwarp();
      // order-preserving compaction, 32 survivors at a time
      int w = 0;
      for (int i0 = 0; i0 < n; i0 += 32) {
        const uint32_t bits = keep[i0 >> 5];
        const int i = i0 + lane;
        const bool k = i < n && ((bits >> lane) & 1u);
        unsigned long long key = 0;
        float e = 0.f;
        if (k) {
          key = srt[i];
          e = E[i];
        }
        __syncwarp();  // every lane has read its element before any is overwritten
        if (k) {
          const int dst = w + __popc(bits & ((1u << lane) - 1));
          srt[dst] = key;
          E[dst] = e;
        }
        w += __popc(bits);
        __syncwarp();
      }
      nkeep = w;
    } else {
      if (lane == 0) {
        float cumulative = 0.f;
        int w = 0;
        for (int i = 0; i < n; ++i) {
          const float pr = cast(E[i] / sum, legacy);
          cumulative += pr;
          const float prior = cast(cast(cumulative, legacy) - pr, legacy);
          if (prior <= c.top_p || i < protect) {
            srt[w] = srt[i];
            E[w] = E[i];
            ++w;
          }
        }
        s_nkeep = w;
      }
      __syncwarp();
      nkeep = s_nkeep;
    }
  }
  if (lane == 0) {
    float sum = 0.f;
    for (int i = 0; i < nkeep; ++i) sum += E[i];
    s_sum = sum;
  }
  __syncwarp();
  const float sum2 = s_sum;
  const uint32_t* words = p.words + (size_t)b * 2 * V;
  bool any = false;
  float bv = 0.f;
  int bid = 0;
  for (int i = lane; i < nkeep; i += 32) {
    const int id = idof(i);
    const float pr = cast(E[i] / sum2, legacy);
    const unsigned long long hi = words[2 * id], lo = words[2 * id + 1];
    const double u = (double)(((hi << 32) | lo) & ((1ull << 53) - 1)) / 9007199254740992.0;
    const float noise = cast(det_d2f(-det_log1p(-u)), legacy);
    const float sc = cast(pr / noise, legacy);
    if (sc == sc && (!any || sc > bv || (sc == bv && id < bid))) {
      any = true;
      bv = sc;
      bid = id;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int oany = __shfl_xor_sync(0xffffffffu, (int)any, o);
    const float obv = __shfl_xor_sync(0xffffffffu, bv, o);
    const int obid = __shfl_xor_sync(0xffffffffu, bid, o);
    if (oany && (!any || obv > bv || (obv == bv && obid < bid))) {
      any = true;
      bv = obv;
      bid = obid;
    }
  }
  if (lane == 0) finish(0, any ? bid : 0);
}

// Launches the prep passes (kPrepChunks CTAs per request) and then the selection and
// draw (one CTA per request) as a programmatic-dependent pair.
cudaError_t launch_sample(cudaStream_t s, bool pdl, const SampleParams& p, int nreq) {
  SampleParams copy = p;
  void* args[] = {&copy};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nreq, kPrepChunks);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.dynamicSmemBytes = ((size_t)p.vocab / kPrepChunks + 8) * sizeof(float);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cfg.dynamicSmemBytes > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute((const void*)sample_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)sample_prep_kernel, args);
  if (e != cudaSuccess) return e;
  cfg = cudaLaunchConfig_t{};
  cfg.gridDim = dim3(nreq);
  cfg.blockDim = dim3(kSampleThreads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, (const void*)sample_kernel, args);
}

}  // namespace y2
