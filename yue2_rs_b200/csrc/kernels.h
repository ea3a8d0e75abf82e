// Device-side structures and kernel launchers of the decode step.
//
// One decode "row" is one new token of one KV cache. A step processes R rows in a
// single pass over every weight matrix (CFG cond + uncond rows, batched songs, or
// consecutive prompt positions of one cache during prefill).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace y2 {

// Token ids of the native protocol (src/protocol.rs:6-16 of the reference).
constexpr int64_t kEOD = 151643;
constexpr int64_t kAbcEnd = 151848;
constexpr int64_t kMusicEnd = 151852;
constexpr int64_t kCodecOffset = 151853;
constexpr int64_t kCodecSize = 32768;
constexpr int64_t kContext = 24576;

enum Phase { kPhaseAbc = 0, kPhaseSemantic = 1, kPhaseVocab = 2 };

constexpr int kMaxRows = 16;       // rows per decode step / prefill chunk (8 songs with CFG)
constexpr int kPageTokens = 64;    // KV page: 64 positions of every layer
constexpr int kPageLog2 = 6;
constexpr int kClusterWarps = 8;   // warps per CTA of the cluster form of decode attention
constexpr int kClusterMax = 8;     // CTAs per (kv head, row) cluster, at most (portable size)

struct DevRow {
  const uint64_t* pages;  // device array: base address of each page of this row's cache
  const int32_t* prompt;  // device ids of positions [prompt_begin, prompt_end)
  int32_t pos;            // position of this row's token
  int32_t token;          // token at `pos` outside the prompt range (sampler / host writes it)
  int32_t prompt_begin, prompt_end;
  int32_t active;         // 0: no KV write, no attention, no position advance
  int32_t advance;        // positions added after each step
};

struct LayerW {
  const uint16_t *q, *k, *v, *o, *gate, *up, *down;  // bf16 [out, in]
  const float *in_norm, *q_norm, *k_norm, *post_norm;  // bf16-valued gains
};

struct Geometry {
  int hidden, heads, kvh, dim, inter, vocab, layers;
  float eps;
};

// Page layout: [layer][K=0 / V=1][kv head][kPageTokens][dim] bf16.
__host__ __device__ inline size_t kv_offset(const Geometry& g, int layer, int kv, int head) {
  return ((size_t)(layer * 2 + kv) * g.kvh + head) * kPageTokens * g.dim;
}
inline size_t page_bytes(const Geometry& g) { return (size_t)g.layers * 2 * g.kvh * kPageTokens * g.dim * 2; }

// ---- GEMV (weight streaming; the SIMT kernel takes R <= 8, the tensor-core kernel R <= 16)
enum XMode { kXBf16 = 0, kXNorm = 1, kXF32 = 2 };
// kEpiTpReduce (tensor parallel, R <= 2): the o or down partial sums over this rank's input
// columns go to every rank as exchange words, and x = bf16(x + bf16(sum over ranks)) is
// formed in the same kernel (tp.cu describes the words).
enum EpiMode { kEpiBf16 = 0, kEpiResidual = 1, kEpiSwiGLU = 2, kEpiLogits = 3, kEpiRawF32 = 4, kEpiTpReduce = 5 };
struct TpPeers;

struct GemvParams {
  const uint16_t* w[3];  // row segments; logical row n lives in segment s with seg_start[s] <= n
  int seg_start[3];      // seg_start[0] = 0; unused segments start at N
  int col0[3];           // output column of each segment's first row
  const uint16_t* wpair;  // SwiGLU: up-projection rows paired with gate rows in w[0]
  int N, K, R;
  const uint16_t* xb;    // kXBf16: [R, K] bf16
  const float* xf;       // kXNorm: residual [R, K]; kXF32: input [R, K]
  const float* gamma;
  float eps;
  uint16_t* ob;          // bf16 outputs [R, ldo]
  float* of;             // f32 outputs [R, ldo] (logits / raw) or residual [R, N]
  int ldo;
  const int32_t* skip;   // optional: the whole launch is skipped when *skip != 0
  int32_t* error;        // optional: set to 1 when a bounded pipeline wait gives up
  int stages;            // set by the launcher: shared-memory ring depth of the streamed path
  // kEpiTpReduce: the peers' exchange buffers, this rank, the forward counter and the
  // exchange number (tags and parity halves as in tp.cu); `of` is the residual x [R, N]
  const TpPeers* tp_peers;
  const uint32_t* tp_epoch;
  int tp_rank, tp_world, tp_site;
};

struct AttnParams {
  const DevRow* rows;
  const uint16_t* q;     // rotated queries [R, heads*dim] bf16
  uint16_t* out;         // [R, heads*dim] bf16
  float* part;           // split partials [R][kvh][S][G][dim + 2]
  int32_t* counters;     // [R][kvh], zero between launches
  Geometry g;
  int layer, splits;
  float scale;
  // fused QK norm + RoPE + KV append (rows with distinct caches): q comes from qkv, and the
  // CTA whose split holds the row's position writes that position's K and V first
  int fused;
  const uint16_t* qkv;   // [R, (heads + 2 kvh) * dim]
  const float *q_norm, *k_norm, *cos_tab, *sin_tab;
  int max_pos;
  int32_t* error;
  int pipe;  // 1: the pipelined tile loop (long contexts); passes of > kMaxRows rows always use it
  // > 0 (fused decode rows, dim <= 128): that many CTAs per (kv head, row) as one thread-block
  // cluster that merges its partials through distributed shared memory (short contexts)
  int cluster;
};

// The pipelined attention loop pays off once a warp streams about 1.5 tiles of 32 keys or
// more (measured at two rows: +1.3% at 4k positions, +3.5% at 24k, -1.2% at 1k): 1 when
// `keys` keys over `splits` splits of four warps reach that.
inline int attn_pipe_for_keys(int keys, int splits) { return 2 * (long long)keys >= 3 * 32 * 4 * (long long)splits; }

// Causal attention of a prefill chunk: rows [0, C) at positions pos0 + row of one cache,
// whose K/V (those rows' included) are already in the pages.
struct PrefillAttnParams {
  const uint64_t* pages;  // the cache's page table
  const uint16_t* q;      // rotated queries [C, heads*dim] bf16
  uint16_t* out;          // [C, heads*dim] bf16
  Geometry g;
  int layer, C, pos0;
  float scale;
  int causal;  // 1: row r sees keys up to pos0 + r; 0: every row sees keys up to pos0 + C - 1
  int32_t* error;  // set when a bounded wait of the tcgen05 form gave up
};

struct RopeParams {
  const DevRow* rows;
  const uint16_t* qkv;   // [R, (heads + 2 kvh) * dim] bf16
  uint16_t* q_out;       // [R, heads*dim]
  const float* cos_tab;  // [max_pos, dim/2] bf16-valued
  const float* sin_tab;
  const float *q_norm, *k_norm;
  Geometry g;
  int layer, max_pos;
  int32_t* error;        // set to 1 when a position is outside the RoPE table
};

// ---- sampler
struct SampleCfg {  // protocol.rs Sampling
  float temperature, top_p, repetition_penalty;
  int32_t top_k, penalty_window, min_tokens, max_tokens;
  int32_t phase;
};

struct SampleReq {
  int32_t cond_row, uncond_row;  // logits rows; uncond_row < 0 without CFG
  float scale;
  int32_t legacy;
  int32_t step;        // index of the sampling step (min_tokens gate)
  int32_t hist_len;    // generated ids visible to the repetition penalty (tokens[0, hist_len))
  int32_t done;
  int32_t status;      // 0 or a negative YUE2_ERR_* code
  int32_t truncated;   // 1 until the phase's stop id is drawn
  int32_t last;        // id drawn by the latest step
  int32_t bookkeeping; // 1: append to tokens, stop on the phase end id (generate); 0: draw only (choose)
  int32_t pad;
  int32_t* tokens;     // generated ids (device): history in, appended out
};

struct MtState {
  uint32_t st[624];
  uint32_t next;
  uint32_t pad[3];
};

// Per-request results of the sampler's first passes (sample_prep_kernel), consumed and reset
// by sample_kernel: any NaN/+inf score, the finite count, the greedy (T=0) argmax key.
struct SampleAcc {
  int32_t bad, nfin;
  unsigned long long best;
};

struct SampleParams {
  const float* logits;
  int ldl, vocab;
  SampleCfg cfg;
  SampleReq* reqs;
  DevRow* rows;
  const uint32_t* words;   // [nreq][2*vocab] MT words of this step
  float* scores;           // scratch [nreq][vocab]
  float* expv;             // scratch [nreq][vocab]
  unsigned long long* sortbuf;  // scratch [nreq][sort_cap]
  int sort_cap;            // power of two >= vocab
  int32_t* live;           // requests not yet done; the last to finish sets *all_done
  int32_t* all_done;
  SampleAcc* acc;          // [nreq], {0, 0, ~0} between steps
};

// ---- tensor parallelism (tp.cu): the all-reduce and all-gather over peer memory
constexpr int kTpMaxWorld = 8;
constexpr int kTpRows = 2;    // rows of a tensor-parallel pass (one song with CFG)
constexpr int kTpCtas = 48;   // CTAs of the logits all-gather
struct TpPeers {
  uint2* recv[kTpMaxWorld];      // every rank's [2][kTpMaxWorld][kTpRows][hidden] exchange words (o, down)
  uint2* gather[kTpMaxWorld];    // every rank's [kMaxRows][vocab] logits words
  float* logits[kTpMaxWorld];    // every rank's [kMaxRows][vocab] logits
};
struct TpParams {
  const TpPeers* peers;
  int rank, world, R;
  int n;                  // vocab
  int col0, cols;         // this rank's logits columns
  int row_base;           // the first logits row (rows [row_base, row_base + R))
  const uint32_t* epoch;  // forwards run so far
  int site;               // exchange number within the forward
  int32_t* error;         // set when a bounded wait gives up
};
cudaError_t launch_tp_allgather(cudaStream_t s, bool pdl, const TpParams& p);
cudaError_t launch_tp_tick(cudaStream_t s, bool pdl, uint32_t* epoch);
size_t tp_recv_bytes(int hidden, int vocab);
cudaError_t launch_fill_normal_shard(cudaStream_t s, uint16_t* dst, size_t rows, size_t cols, size_t full_cols,
                                     size_t row0, size_t col0, uint64_t seed, float stddev);

// launchers (return cudaError_t of the launch)
cudaError_t launch_embed(cudaStream_t s, bool pdl, DevRow* rows, int R, const uint16_t* embed, int hidden,
                         int vocab, float* x, int32_t* error);
cudaError_t launch_gemv(cudaStream_t s, bool pdl, int xmode, int epi, const GemvParams& p, int grid);
// streamed tensor-core GEMV (one CTA per SM); used by launch_gemv where eligible
bool gemv_tc_eligible(int xmode, int epi, const GemvParams& p);
cudaError_t launch_gemv_tc(cudaStream_t s, bool pdl, int xmode, int epi, const GemvParams& p, bool configure_only);
cudaError_t launch_with(cudaStream_t s, bool pdl, dim3 grid, dim3 block, size_t smem, const void* fn, void** args);
cudaError_t launch_rope_append(cudaStream_t s, bool pdl, const RopeParams& p, int R);
cudaError_t launch_attention(cudaStream_t s, bool pdl, const AttnParams& p, int R);
bool prefill_attention_supported(const Geometry& g);
bool gemm_tc_supported(int C, int N, int K, int ldx, int ldy, const void* X, const void* W, const void* Y);
cudaError_t launch_gemm_tc(cudaStream_t s, const uint16_t* W, int N, int K, const uint16_t* X, int ldx, uint16_t* Y,
                           int ldy, int C, int32_t* error);
cudaError_t launch_gemm_tc_swiglu(cudaStream_t s, const uint16_t* Wgu, int I, int K, const uint16_t* X, int ldx,
                                  uint16_t* H, int ldh, int C, int32_t* error);
// 2D TMA descriptor (128 bytes at `map`, 64-byte aligned) of a row-major bf16 [rows, cols]
// matrix with row stride ld elements: boxes of 64 columns x box_rows rows, 128-byte swizzle,
// rows past the end read as zero.
bool make_tma_map_bf16(void* map, const void* base, int rows, int cols, int ld, int box_rows);

// Skinny tcgen05 GEMM for decode passes of 3..256 rows (kernels_gemm_skinny.cu):
// Y[C, N] = bf16(X[C, K] . W[N, K]^T), or with `swiglu` (W = [gate; up], up at row N)
// Y[C, N] = bf16(bf16(silu(bf16 g)) * bf16 u). The weight rows are the MMA's M side, the
// activation rows its N side; each tile's K range is split over the CTAs of one cluster,
// which sum their partials in rank order through distributed shared memory.
constexpr int kSkinnyMaxRows = 256;
bool gemm_skinny_supported(int C, int N, int K, int ldx, int ldy, const void* X, const void* W, const void* Y,
                           bool swiglu);
// pdl: launched as a programmatic dependent of the preceding kernel on the stream.
cudaError_t launch_gemm_skinny(cudaStream_t s, bool pdl, const uint16_t* W, int N, int K, const uint16_t* X, int ldx,
                               uint16_t* Y, int ldy, int C, bool swiglu, int32_t* error);

cudaError_t launch_prefill_attention(cudaStream_t s, const PrefillAttnParams& p);
// The same attention on tcgen05 (kernels_prefill_attn_tc.cu): head_dim 128.
bool prefill_attention_tc_supported(const Geometry& g);
cudaError_t launch_prefill_attention_tc(cudaStream_t s, const PrefillAttnParams& p);
cudaError_t launch_step_end(cudaStream_t s, bool pdl, DevRow* rows, int R);
cudaError_t launch_mt_words(cudaStream_t s, MtState* st, uint32_t* words, int nwords, const SampleReq* reqs,
                            int nreq);
cudaError_t launch_sample(cudaStream_t s, bool pdl, const SampleParams& p, int nreq);
cudaError_t launch_fill_normal_bf16(cudaStream_t s, uint16_t* dst, size_t count, uint64_t seed, float mean,
                                    float stddev);
cudaError_t launch_fill_f32(cudaStream_t s, float* dst, size_t count, float value);
cudaError_t launch_kv_fill(cudaStream_t s, const uint64_t* pages, const Geometry& g, int from, int to,
                           uint64_t seed, int head0, int full_kvh);

cudaError_t prepare_kernels();  // configure every kernel for this device (call outside capture)
size_t gemv_smem_bytes(int xmode, int K, int R);
int attention_smem_bytes(int dim, int groups);

}  // namespace y2
