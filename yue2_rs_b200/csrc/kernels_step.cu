// Persistent decode-step kernel (sm_100a): embed, every layer and the LM head of one
// decode step in one cooperative launch, one CTA of eight warps per SM.
//
// Reference: Model::hidden decode branch (src/model.rs:523-591) and forward_phase
// (src/model.rs:465-507); the math of each phase is that of the standalone kernels
// (GEMV epilogues as in kernels_gemv.cu, attention as in attention.cuh).
//
// Why one kernel: a decode step at R <= 2 rows is a chain of ~140 dependent launches, and
// each launch boundary costs a few microseconds (the next grid's release, its activation
// staging, its tail). Here the phases of a layer (q|k|v, attention partials, attention
// merge, o, gate|up, down) are separated by grid-wide barriers instead, and the weight
// stream never stops: every warp keeps a ring of weight items in shared memory and runs
// ahead across phase boundaries, so while the grid waits at a barrier or computes
// attention, the next matrix is already streaming (the whole o projection fits in the
// rings). The ring uses the per-lane cp.async streaming and mma.sync tiles of the
// tensor-core GEMV.
//
// Barriers are a monotonically counted global arrival counter (zeroed before every
// launch), with bounded spins: a wait that gives up sets *stall, and every later wait of
// the launch returns at once, so the kernel always ends and the host reports
// YUE2_ERR_TIMEOUT. The cooperative launch guarantees that all CTAs are resident.
// Everything a phase reads that another SM wrote in this launch is read through L2
// (ld.global.cg / cp.async.cg), never through a possibly stale L1 line.
#include <cuda_runtime.h>

#include "attention.cuh"
#include "common.cuh"
#include "kernels.h"

namespace y2 {

constexpr int kSWarps = 8;
constexpr int kSThreads = kSWarps * 32;
constexpr int kSBC = 256;                       // weight block columns per item
constexpr int kSRing = 4;                       // items per warp in the ring
constexpr int kSPitch = kSBC * 2 + 64;          // staged row bytes (quarter-warp conflict-free)
constexpr int kSSlot = 8 * kSPitch;             // one item: 8 weight rows
constexpr int kSRingBytes = kSWarps * kSRing * kSSlot;
constexpr long long kSWait = 2000000000ll;      // ~1 s of SM clocks per barrier wait


size_t step_kernel_smem(int dim, int groups, int R, int max_k) {
  const size_t xp = ((2 * (size_t)max_k + 127) / 128) * 128 + 64;
  const size_t gemv = (size_t)R * xp + (size_t)kSWarps * 2 * 32 * 16;
  const size_t tiles = 2 * 4 * 32 * (size_t)dim * 2;
  const size_t attn = tiles + ((size_t)groups * dim + 4 * groups * 32 + 8 * groups + 4 * dim) * 4;
  return kSRingBytes + (gemv > attn ? gemv : attn);
}

Y2_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------------ the weight stream
// Phase p of the step's GEMV sequence (per layer q|k|v, o, gate|up, down; then the LM
// head): this CTA's units [u0, u1), this warp's contiguous share [ia, ib) of the
// CTA's (8-row tile, 256-column block) items.
struct PhaseShare {
  int tu, u0, u1, nkb, ia, ib;
};
Y2_DEV PhaseShare phase_share(const StepGemv& d, int warp) {
  PhaseShare s;
  s.tu = d.pair ? 4 : 8;
  s.u0 = (int)(((long long)d.p.N * blockIdx.x) / gridDim.x);
  s.u1 = (int)(((long long)d.p.N * (blockIdx.x + 1)) / gridDim.x);
  const int ntiles = (s.u1 - s.u0 + s.tu - 1) / s.tu;
  s.nkb = d.p.K / kSBC;
  const int items = ntiles * s.nkb;
  s.ia = (int)(((long long)items * warp) / kSWarps);
  s.ib = (int)(((long long)items * (warp + 1)) / kSWarps);
  return s;
}

// Issue side of one warp: walks the items of every phase in order and copies each into
// its ring slot (cp.async; staged row r of a slot holds row r of the tile, 512 bytes).
// The state is warp-uniform and lives in shared memory, so it holds no registers while
// the kernel is in other phases.
struct IssueState {
  int ph, cnt, tile, kb;
  PhaseShare sh;
  unsigned total;
  // the fields of the current phase's descriptor the copies need (read from global
  // memory once per phase, not once per item: L1 is small beside the ring)
  const uint16_t* w[3];
  const uint16_t* wpair;
  int seg1, seg2, K, pair;
};

Y2_DEV void issue_enter(IssueState& st, const StepGemv* phases, int nphase, int p, int warp) {
  for (st.ph = p; st.ph < nphase; ++st.ph) {
    st.sh = phase_share(phases[st.ph], warp);
    if (st.sh.ib > st.sh.ia) break;
  }
  if (st.ph < nphase) {
    const StepGemv& d = phases[st.ph];
    st.cnt = 0;
    st.tile = st.sh.ia / st.sh.nkb;
    st.kb = st.sh.ia % st.sh.nkb;
    st.w[0] = d.p.w[0];
    st.w[1] = d.p.w[1];
    st.w[2] = d.p.w[2];
    st.wpair = d.p.wpair;
    st.seg1 = d.p.seg_start[1];
    st.seg2 = d.p.seg_start[2];
    st.K = d.p.K;
    st.pair = d.pair;
  }
}

// The eight weight rows of the state's current tile, offset to this lane's 16-byte piece
// (nullptr past the CTA's share); refreshed once per tile, not once per item.
Y2_DEV void issue_rows(const IssueState& st, int nphase, int lane, const uint16_t* (&src)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int q = st.pair ? (c & 3) : c;
    const int n = st.sh.u0 + st.tile * st.sh.tu + q;
    const uint16_t* row = nullptr;
    if (st.ph < nphase && n < st.sh.u1) {
      if (st.pair && c >= 4) {
        row = st.wpair + (size_t)n * st.K;
      } else {
        row = n >= st.seg2 ? st.w[2] + (size_t)(n - st.seg2) * st.K
              : n >= st.seg1 ? st.w[1] + (size_t)(n - st.seg1) * st.K
                             : st.w[0] + (size_t)n * st.K;
      }
      row += lane * 8;
    }
    src[c] = row;
  }
}

// Copies this warp's next item (or commits an empty group past the last phase). `st` is
// the warp-uniform issue state and `src` its tile's rows, both in registers.
Y2_DEV void issue_item(IssueState& st, const uint16_t* (&src)[8], const StepGemv* phases, int nphase,
                       unsigned char* ring, int warp, int lane) {
  if (st.ph < nphase) {
    unsigned char* slot = ring + (size_t)(st.total & (kSRing - 1)) * kSSlot + lane * 16;
    const size_t off = (size_t)st.kb * kSBC;
    // copy c of lane L: staged row c, piece L (16 bytes) of the row's 512-byte segment
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (src[c]) cp_async16(slot + c * kSPitch, src[c] + off);
    bool new_rows = false;
    if (++st.kb == st.sh.nkb) {
      st.kb = 0;
      ++st.tile;
      new_rows = true;
    }
    if (++st.cnt == st.sh.ib - st.sh.ia) {
      issue_enter(st, phases, nphase, st.ph + 1, warp);
      new_rows = true;
    }
    if (new_rows) issue_rows(st, nphase, lane, src);
  }
  ++st.total;
  cp_async_commit();  // one group per item, empty past the end, so counts stay aligned
}

// ------------------------------------------------------------------ phases
// Shared state of one CTA, passed to the phase functions (each phase is a separate,
// non-inlined function so that the register budget of one phase does not add to another).
struct StepShared {
  StepGemv phase[2];  // GEMV phase descriptors: phase p in phase[p & 1], the next one prefetched
  AttnParams attn;    // the current layer's attention parameters
  IssueState issue[kSWarps];
  float red[64];
  int cut[kSWarps], ncut;
  unsigned bar_no;
  int stalled;
};

// Grid-wide barrier: arrival counted on sp.barrier; bounded wait (see the file comment).
Y2_DEV __noinline__ void grid_barrier(const StepParams& sp, StepShared& sh) {
  __syncthreads();
  if (threadIdx.x == 0) {
    // release: this CTA's writes (ordered before by the block barrier) precede the arrival
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(sp.barrier) : "memory");
    const unsigned target = (++sh.bar_no) * gridDim.x;
    if (!sh.stalled) {
      const long long t0 = clock64();
      unsigned polls = 0;
      while (ld_acquire(sp.barrier) < target) {
        if ((++polls & 255) == 0 && (clock64() - t0 > kSWait || *(volatile int*)sp.stall)) {
          sh.stalled = 1;
          atomicExch(sp.stall, 1);
          break;
        }
      }
    }
  }
  __syncthreads();
}

// One GEMV phase: stage the activations, consume this warp's items of phase p from the
// ring (refilling it from the stream), finish tiles. Returns the updated consumed count.
Y2_DEV __noinline__ unsigned gemv_phase(const StepParams& sp, StepShared& shs, int p, unsigned consumed,
                                        unsigned char* smem) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int R = sp.R;
  const int nphase = 4 * sp.layers + 1;
  unsigned char* my_ring = smem + (size_t)warp * kSRing * kSSlot;
  unsigned char* un = smem + kSRingBytes;
  const StepGemv& d = shs.phase[p & 1];  // loaded by the previous phase (or the kernel start)
  const GemvParams& gp = d.p;
  const int K = gp.K;
  const size_t xp = ((2 * (size_t)K + 127) / 128) * 128 + 64;
  unsigned char* xs = un;
  float4* pieces = reinterpret_cast<float4*>(un + (size_t)R * xp);  // [kSWarps][2][32]
  if (d.xmode == kXBf16) stage_bf16_rows<kSThreads, true>(gp.xb, K, R, xs, xp);
  else stage_rmsnorm_rows<kSThreads, true>(gp.xf, gp.gamma, K, R, gp.eps, xs, xp, shs.red);
  {  // the next phase's descriptor (and after q|k|v the layer's attention parameters) now,
     // so that no phase starts with a round trip for them
    if (p + 1 < nphase) {
      const int* src = reinterpret_cast<const int*>(&sp.phases[p + 1]);
      int* dst = reinterpret_cast<int*>(&shs.phase[(p + 1) & 1]);
      for (int i = tid; i < (int)(sizeof(StepGemv) / 4); i += kSThreads) dst[i] = src[i];
    }
    if ((p & 3) == 0 && p / 4 < sp.layers) {
      const int* src = reinterpret_cast<const int*>(&sp.attn[p / 4]);
      int* dst = reinterpret_cast<int*>(&shs.attn);
      for (int i = tid; i < (int)(sizeof(AttnParams) / 4); i += kSThreads) dst[i] = src[i];
    }
  }
  __syncthreads();
  const PhaseShare sh = phase_share(d, warp);
  const int T = sh.ib - sh.ia, TU = sh.tu, nkb = sh.nkb;
  const int pair = d.pair, epi = d.epi;
  auto emit = [&](int tile, int r, int j, float v, float u) {
    const int n = sh.u0 + tile * TU + j;
    if (r >= R || n >= sh.u1) return;
    const int sg = (n >= gp.seg_start[2]) ? 2 : (n >= gp.seg_start[1]) ? 1 : 0;
    const int col = gp.col0[sg] + (n - gp.seg_start[sg]);
    if (epi == kEpiSwiGLU) {
      const float gt = round_bf16(v);
      const float a = round_bf16(gt / (1.0f + det_expf(-gt)));
      gp.ob[(size_t)r * gp.ldo + col] = f2bf_round(a * round_bf16(u));
    } else if (epi == kEpiBf16) {
      gp.ob[(size_t)r * gp.ldo + col] = f2bf_round(v);
    } else if (epi == kEpiResidual) {
      float* xr = gp.of + (size_t)r * gp.ldo + col;
      *xr = round_bf16(__ldcg(xr) + round_bf16(v));
    } else {  // kEpiLogits
      gp.of[(size_t)r * gp.ldo + col] = round_bf16(v);
    }
  };
  const bool has_x = g8 < R;
  const unsigned char* xrow = xs + (size_t)g8 * xp + t4 * 16;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
  int c_tile = nkb ? sh.ia / nkb : 0, c_kb = nkb ? sh.ia % nkb : 0;
  const int first_tile = c_tile;
  int run_kb0 = c_kb;
  IssueState ist = shs.issue[warp];  // in registers for the whole phase
  const uint16_t* isrc[8];
  issue_rows(ist, nphase, lane, isrc);
  for (int it = 0; it < T; ++it) {
    cp_async_wait<kSRing - 2>();
    __syncwarp();
    const unsigned char* st = my_ring + (size_t)(consumed & (kSRing - 1)) * kSSlot + g8 * kSPitch + t4 * 16;
    const unsigned char* xk = xrow + (size_t)c_kb * kSBC * 2;
#pragma unroll
    for (int u = 0; u < kSBC / 32; ++u) {
      const uint4 w = *reinterpret_cast<const uint4*>(st + u * 64);
      uint4 x = make_uint4(0u, 0u, 0u, 0u);
      if (has_x) x = *reinterpret_cast<const uint4*>(xk + u * 64);
      mma_bf16_16816(acc[u & 3], x.x, 0u, x.y, 0u, w.x, w.y);
      mma_bf16_16816(acc[u & 3], x.z, 0u, x.w, 0u, w.z, w.w);
    }
    ++consumed;
    __syncwarp();  // every lane is done with the slot before it is refilled
    issue_item(ist, isrc, sp.phases, nphase, my_ring, warp, lane);
    const bool tile_end = c_kb == nkb - 1;
    if (tile_end || it == T - 1) {
      float c0 = 0.f, c1 = 0.f;
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        c0 += acc[a][0];
        c1 += acc[a][1];
        acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.f;
      }
      if (run_kb0 == 0 && tile_end) {
        if (pair) {  // gate rows 0..3 sit in lanes t < 2, up rows 4..7 in lanes t + 2
          const float u0v = __shfl_down_sync(0xffffffffu, c0, 2);
          const float u1v = __shfl_down_sync(0xffffffffu, c1, 2);
          if (t4 < 2) {
            emit(c_tile, g8, 2 * t4, c0, u0v);
            emit(c_tile, g8, 2 * t4 + 1, c1, u1v);
          }
        } else {
          emit(c_tile, g8, 2 * t4, c0, 0.f);
          emit(c_tile, g8, 2 * t4 + 1, c1, 0.f);
        }
      } else {
        pieces[(warp * 2 + (c_tile == first_tile ? 0 : 1)) * 32 + lane] = make_float4(c0, c1, 0.f, 0.f);
      }
    }
    if (++c_kb == nkb) {
      c_kb = 0;
      ++c_tile;
      run_kb0 = 0;
    }
  }
  __syncwarp();
  if (lane == 0) shs.issue[warp] = ist;
  // tiles split between warps: add the pieces in warp order
  const int ntiles = (sh.u1 - sh.u0 + TU - 1) / TU, items = ntiles * nkb;
  auto share = [&](int w) { return (int)(((long long)items * w) / kSWarps); };
  if (tid == 0) {
    int n = 0;
    for (int b = 1; b < kSWarps; ++b) {
      const int cut = share(b);
      if (cut >= items || cut % nkb == 0) continue;
      if (n == 0 || shs.cut[n - 1] != cut / nkb) shs.cut[n++] = cut / nkb;
    }
    shs.ncut = n;
  }
  __syncthreads();
  const int per = R * TU;
  for (int f = tid; f < shs.ncut * per; f += kSThreads) {
    const int tile = shs.cut[f / per], e = f % per, r = e / TU, j = e % TU;
    const int lo = tile * nkb, hi = lo + nkb;
    float v = 0.f, u = 0.f;
    for (int w = 0; w < kSWarps; ++w) {
      const int a0 = share(w), a1 = share(w + 1);
      if (a0 >= a1 || a0 >= hi || a1 <= lo) continue;
      const float4* pw = pieces + (w * 2 + (a0 / nkb == tile ? 0 : 1)) * 32;
      auto at = [&](int q) {
        const float4 el = pw[4 * r + (q >> 1)];
        return (q & 1) ? el.y : el.x;
      };
      v += at(j);
      if (pair) u += at(j + 4);
    }
    emit(tile, r, j, v, u);
  }
  return consumed;
}

// Attention of one layer: partials of item (split, kv head, row) = blockIdx.x on warps
// 0-3, a grid barrier, then the split merge with each CTA finishing a slice of outputs.
template <int D, int G>
Y2_DEV __noinline__ void attention_phase(const StepParams& sp, StepShared& shs, int layer, unsigned char* un) {
  const AttnParams& a = shs.attn;  // loaded during the q|k|v phase
  const int R = sp.R, S = a.splits, kvh = a.g.kvh;
  const int item = blockIdx.x;
  if ((threadIdx.x >> 5) < 4 && item < R * kvh * S)
    attn_item<D, G, false>(a, item % S, (item / S) % kvh, item / (S * kvh), un);
  grid_barrier(sp, shs);
  const int outw = a.g.heads * D, n = R * kvh * G * D;
  const int lo = (int)(((long long)n * blockIdx.x) / gridDim.x), hi = (int)(((long long)n * (blockIdx.x + 1)) / gridDim.x);
  for (int i = lo + (int)threadIdx.x; i < hi; i += kSThreads) {
    const int d = i % D, h = (i / D) % G, g = (i / (D * G)) % kvh, r = i / (D * G * kvh);
    const DevRow& row = sp.rows[r];
    if (!row.active) continue;
    const int ntiles = (row.pos + 1 + 31) >> 5;
    const int tps = max(4, (ntiles + S - 1) / S);
    const int nsplit = (ntiles + tps - 1) / tps;
    if (nsplit == 1) continue;  // attn_item wrote the output
    const float* part = a.part + ((size_t)(r * kvh + g) * S) * G * (D + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(part + ((size_t)s * G + h) * (D + 2)));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float* ph = part + ((size_t)s * G + h) * (D + 2);
      const float f = __expf(__ldcg(ph) - M);
      L = fmaf(__ldcg(ph + 1), f, L);
      O = fmaf(__ldcg(ph + 2 + d), f, O);
    }
    a.out[(size_t)r * outw + (size_t)(g * G + h) * D + d] = f2bf_round(O / L);
  }
  grid_barrier(sp, shs);
}

// Model::embed (model.rs:452-464): CTA c writes its column share of every row.
Y2_DEV __noinline__ void embed_phase(const StepParams& sp) {
  const int H = sp.hidden;
  const int c0 = (int)(((long long)H * blockIdx.x) / gridDim.x), c1 = (int)(((long long)H * (blockIdx.x + 1)) / gridDim.x);
  for (int r = 0; r < sp.R; ++r) {
    DevRow& row = sp.rows[r];
    int tok = (row.pos >= row.prompt_begin && row.pos < row.prompt_end) ? row.prompt[row.pos - row.prompt_begin]
                                                                        : row.token;
    if (tok < 0 || tok >= sp.vocab) {
      if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(sp.tok_error, 1);
      tok = 0;
    }
    const uint16_t* e = sp.embed + (size_t)tok * H;
    for (int i = c0 + (int)threadIdx.x; i < c1; i += kSThreads) sp.x[(size_t)r * H + i] = bf2f(e[i]);
    if (blockIdx.x == 0 && threadIdx.x == 0) row.token = tok;
  }
}

// ------------------------------------------------------------------ the kernel
template <int D, int G>
__global__ void __launch_bounds__(kSThreads, 1) step_kernel(const __grid_constant__ StepParams sp) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ StepShared shs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (sp.skip && *sp.skip) return;  // every CTA leaves before the first barrier
  const int nphase = 4 * sp.layers + 1;
  if (threadIdx.x == 0) {
    shs.bar_no = 0;
    shs.stalled = 0;
  }
  {
    const int* src = reinterpret_cast<const int*>(&sp.phases[0]);
    int* dst = reinterpret_cast<int*>(&shs.phase[0]);
    for (int i = threadIdx.x; i < (int)(sizeof(StepGemv) / 4); i += kSThreads) dst[i] = src[i];
  }
  if (lane == 0) {
    IssueState st;
    st.total = 0;
    issue_enter(st, sp.phases, nphase, 0, warp);
    shs.issue[warp] = st;
  }
  __syncthreads();
  unsigned char* my_ring = smem + (size_t)warp * kSRing * kSSlot;
  {
    IssueState ist = shs.issue[warp];
    const uint16_t* isrc[8];
    issue_rows(ist, nphase, lane, isrc);
    for (int i = 0; i < kSRing - 1; ++i) issue_item(ist, isrc, sp.phases, nphase, my_ring, warp, lane);
    __syncwarp();
    if (lane == 0) shs.issue[warp] = ist;
    __syncthreads();
  }
  unsigned consumed = 0;

  embed_phase(sp);
  grid_barrier(sp, shs);
  for (int l = 0; l < sp.layers; ++l) {
    consumed = gemv_phase(sp, shs, 4 * l, consumed, smem);  // q|k|v with the input RMSNorm
    grid_barrier(sp, shs);
    attention_phase<D, G>(sp, shs, l, smem + kSRingBytes);
    consumed = gemv_phase(sp, shs, 4 * l + 1, consumed, smem);  // o + residual
    grid_barrier(sp, shs);
    consumed = gemv_phase(sp, shs, 4 * l + 2, consumed, smem);  // gate|up + SwiGLU, post-attention norm
    grid_barrier(sp, shs);
    consumed = gemv_phase(sp, shs, 4 * l + 3, consumed, smem);  // down + residual
    grid_barrier(sp, shs);
  }
  gemv_phase(sp, shs, 4 * sp.layers, consumed, smem);  // final norm + LM head
  cp_async_wait<0>();
}

template <int G>
static const void* step_fn(int dim) {
  return dim == 128 ? (const void*)step_kernel<128, G> : nullptr;
}

cudaError_t launch_step(cudaStream_t s, const StepParams& p, int dim, int groups, int sms, bool configure_only) {
  const void* fn = nullptr;
  switch (groups) {
    case 1: fn = step_fn<1>(dim); break;
    case 2: fn = step_fn<2>(dim); break;
    case 3: fn = step_fn<3>(dim); break;
    case 4: fn = step_fn<4>(dim); break;
    case 8: fn = step_fn<8>(dim); break;
  }
  if (!fn) return cudaErrorInvalidValue;
  const size_t smem = p.smem;
  if (configure_only) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, fn);
    if (e != cudaSuccess) return e;
    const int dyn = 227 * 1024 - (int)fa.sharedSizeBytes;
    if ((int)smem > dyn) return cudaErrorInvalidValue;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
  }
  StepParams copy = p;
  void* args[] = {&copy};
  cudaLaunchConfig_t cfg = {};
  // one SM is left to the MT19937 kernel that runs beside the step on a forked branch
  cfg.gridDim = dim3(sms > 1 ? sms - 1 : 1);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace y2
