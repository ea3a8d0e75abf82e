/* yue2_cuda.h -- C ABI of libyue2cuda, the sm_100a replacement for the reference's
 * Metal bridge (twally3/yue2_rs src/metal.m + src/attention.metal) on the
 * autoregressive single-token decode path.
 *
 * Two groups of entry points:
 *
 *  1. Drop-ins for the Metal imports that src/tensor.rs:118-219 declares. Same
 *     argument lists and the same convention: 1 = done, 0 = not done. The reference
 *     treats 0 as "fall back to the CPU"; a caller of this library must instead turn
 *     0 into an error carrying yue2_last_error() (no CPU fallback exists).
 *
 *  2. The resident fast path that replaces the per-step host work of
 *     sampling::generate (src/sampling.rs:222-294): weights, paged BF16 KV caches and
 *     the sampler state stay on the device and one decode step is one CUDA-graph
 *     launch. These return 0 on success or a negative YUE2_ERR_* code.
 *
 * All pointers are host pointers unless stated. Calls on one Yue2Model (and the
 * caches/generators made from it) must not run concurrently; distinct models may be
 * driven from distinct threads.
 */
#ifndef YUE2_CUDA_H
#define YUE2_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ error codes */
#define YUE2_OK 0
#define YUE2_ERR_INVALID (-1)   /* bad argument, shape or configuration (reference: invalid(..)) */
#define YUE2_ERR_CUDA (-2)      /* CUDA runtime failure */
#define YUE2_ERR_OOM (-3)       /* device allocation failed */
#define YUE2_ERR_CAPACITY (-4)  /* "AR input exceeds cache/model context" (model.rs:524-530) */
#define YUE2_ERR_LOGITS (-5)    /* "Model produced invalid logits" (sampling.rs:145-147) */
#define YUE2_ERR_EMPTY (-6)     /* "Empty sampling distribution" (sampling.rs:155,166) */
#define YUE2_ERR_TIMEOUT (-7)   /* a bounded device wait gave up */
#define YUE2_ERR_VOCAB (-8)     /* vocabulary does not support the phase (sampling.rs:113-122) */
#define YUE2_ERR_TOKEN (-9)     /* "Token outside model vocabulary" (model.rs:456-457) */

/* Phase (sampling.rs:81-99). YUE2_PHASE_VOCAB is this library's vocabulary-generic
 * variant: no phase window and no stop id, used for models whose vocabulary does not
 * contain the native protocol ids. */
#define YUE2_PHASE_ABC 0
#define YUE2_PHASE_SEMANTIC 1
#define YUE2_PHASE_VOCAB 2

/* Weight dtypes of GpuWeight.dtype (tensor.rs:221-230). */
#define YUE2_DTYPE_BF16 0
#define YUE2_DTYPE_F32 1
#define YUE2_DTYPE_F16 2

/* Last error message of the calling thread ("" when none). */
const char* yue2_last_error(void);

/* ================================================================== 1. drop-ins */

/* #[repr(C)] GpuWeight (src/tensor.rs:221-230). */
typedef struct {
  const uint8_t* raw;
  size_t mapping;
  size_t rows, cols;
  int32_t dtype, rounded;
} Yue2GpuWeight;

/* #[repr(C)] GpuLayer (src/tensor.rs:231-237): weights q,k,v,o,gate,up,down; norms
 * input, q_norm, k_norm, post_attention; the host F32 KV rows of this layer. */
typedef struct {
  Yue2GpuWeight weights[7];
  const float* norms[4];
  const float* key;
  const float* value;
} Yue2GpuLayer;

/* yue2_metal_available (tensor.rs:118, metal.m:71). 1 when a sm_100 device is usable. */
int yue2_cuda_available(void);
/* yue2_metal_vector_default (tensor.rs:119, metal.m:541-543). */
int yue2_cuda_vector_default(void);
/* yue2_metal_name (tensor.rs:193, metal.m:72). */
const char* yue2_cuda_name(void);
/* yue2_metal_vector (tensor.rs:120-130, metal.m:545-603): out[rows] = W[rows, cols] . input,
 * FP32 accumulation, no output rounding (Linear::finish rounds). The weight is uploaded
 * once and cached by (mapping, raw, rows, cols, dtype). dtype F32/F16 require rounded=1
 * (converted to bf16 on upload, as the reference's convert_weight does). */
int yue2_cuda_vector(const float* input, const uint8_t* raw, size_t mapping, int dtype, int rounded,
                     int priority, float* out, size_t rows, size_t cols);
/* yue2_metal_clear_weights (tensor.rs:132, metal.m:73-76). */
void yue2_cuda_clear_weights(void);
/* yue2_metal_release_model (tensor.rs:133, metal.m:77-83). */
void yue2_cuda_release_model(void);
/* yue2_metal_release_cache (tensor.rs:134, metal.m:84-103). */
void yue2_cuda_release_cache(size_t cache);
/* yue2_metal_ar_stack (tensor.rs:146-163, metal.m:718-874): one token through `count`
 * AR layers at position `prefix`; out = hidden state before the final norm; shadow =
 * [count][K row, V row] of the new token (f32, bf16-valued). The device KV context of
 * (cache, layer) mirrors the host rows layers[i].key/value[0, prefix). */
int yue2_cuda_ar_stack(const float* input, float* out, float* shadow, const Yue2GpuLayer* layers, size_t count,
                       size_t hidden, size_t heads, size_t kv, size_t dim, size_t intermediate, size_t prefix,
                       size_t capacity, size_t cache, float eps, const float* cos, const float* sin);
/* yue2_metal_stack (tensor.rs:164-180, metal.m:429-538): `rows` new rows ([rows, hidden]
 * f32) through `count` layers after `prefix` cached positions whose f32 K/V rows
 * ([prefix, kv*dim], bf16-valued) each layer carries; every row attends to every key (the
 * prefix and all new rows). cos/sin are the rows' RoPE tables ([rows, dim/2]). Products in
 * f32, bf16 roundings where the reference's shaders round; `out` gets the final residual
 * stream [rows, hidden]. The bf16 prefix blocks stay cached per (cache, layer, prefix) until
 * yue2_cuda_release_cache(cache). */
int yue2_cuda_stack(const float* input, float* out, const Yue2GpuLayer* layers, size_t count, size_t rows,
                    size_t hidden, size_t heads, size_t kv, size_t dim, size_t intermediate, size_t prefix,
                    size_t cache, float eps, const float* cos, const float* sin);
/* yue2_metal_linear (tensor.rs:135-145, metal.m:216-237): c[m, n] = a[m, k] . W[n, k]^T in
 * f32 with W the converted checkpoint matrix (bf16 widened exactly; F32/F16 kept, rounded
 * to bf16 when `round`), cached by (mapping, raw, n, k, dtype, round). */
int yue2_cuda_linear(const float* a, const uint8_t* weight, size_t mapping, int dtype, int round, float* c, size_t m,
                     size_t n, size_t k);
/* yue2_metal_gemm (tensor.rs:207-219, metal.m:164-181): c = a . op(b) + beta c in f32;
 * op(b) = b^T of a row-major [n, k] b when transpose_b, else b of [k, n]; row strides lda,
 * ldb, ldc. m or n of 0: nothing to do (returns 1). */
int yue2_cuda_gemm(const float* a, const float* b, float* c, size_t m, size_t n, size_t k, int transpose_b,
                   size_t lda, size_t ldb, size_t ldc, float beta);
/* yue2_metal_attention (tensor.rs:194-206, metal.m:330-362): GQA attention of q [rows,
 * heads*dim] over k/v [keys, kv*dim], all f32: scores in f32, softmax over the visible keys
 * (all of them when causal < 0, else the first min(keys, causal + row + 1)), f32 P.V,
 * output rounded to bf16 (attention.metal:29-70). */
int yue2_cuda_attention(const float* q, const float* k, const float* v, float* out, size_t rows, size_t keys,
                        size_t heads, size_t kv, size_t dim, int64_t causal, float scale);
/* yue2_metal_cached_attention (tensor.rs:181-192, metal.m:686-706): single-query GQA
 * attention over k/v rows [0, keys) ([keys, kv*dim] f32, bf16-valued), output bf16-rounded. */
int yue2_cuda_cached_attention(const float* q, const float* k, const float* v, float* out, size_t keys,
                               size_t heads, size_t kv, size_t dim, size_t cache, size_t layer);

/* No counterpart in the reference. The same single-query GQA decode attention for callers
 * that cannot allocate device memory -- code running inside a host framework that owns
 * every allocation (its own memory pool, or a rule against cudaMalloc/cudaFree after
 * start-up because they synchronise the device) or threads that may not block in the
 * allocator. The caller passes device buffers: q [heads*dim], k and v row-major
 * [keys, kv*dim], out [heads*dim], all bf16 bits, 16-byte aligned; `stream` is a
 * cudaStream_t (NULL for the default stream). No allocation happens: the split-K partials
 * and merge counters live in a 2 MiB static device array held on every GPU that loads the
 * library until exit. Sizes whose partials (heads * (dim + 2) * splits * 4 B, up to 32
 * splits) exceed it are rejected with YUE2_ERR_INVALID. The first call on a device, with
 * that device current, looks up the array's device address; make it before any stream
 * capture. All calls share the array: calls whose kernels overlap on the GPU race. Returns
 * 0 or a negative YUE2_ERR_* code; the work is asynchronous on `stream`. */
int yue2_attention_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, uint64_t keys,
                           uint64_t heads, uint64_t kv, uint64_t dim, void* stream);

/* ================================================================== 2. resident fast path */

typedef struct Yue2Model Yue2Model;
typedef struct Yue2Cache Yue2Cache;
typedef struct Yue2Rng Yue2Rng;

/* AR subset of model.rs Config (src/model.rs:11-27). */
typedef struct {
  uint64_t hidden_size, num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim,
      intermediate_size, vocab_size, max_position_embeddings;
  float rms_norm_eps, rope_theta;
  int32_t tie_word_embeddings;
} Yue2Config;

/* protocol.rs Sampling (src/protocol.rs:142-151). */
typedef struct {
  float temperature, top_p;
  uint64_t top_k;
  float repetition_penalty;
  uint64_t penalty_window, min_tokens, max_tokens;
} Yue2Sampling;

/* Model::open (src/model.rs:418-451) without file IO: allocate device storage for the
 * AR tensors of `cfg` on `device`. Tensors arrive through yue2_model_set_tensor. */
int yue2_model_create(int device, const Yue2Config* cfg, Yue2Model** out);
/* Tensor parallelism (no counterpart in the reference, which runs on one device; the
 * optional split of BASELINE's single-song latency configuration). Rank `tp_rank` of
 * `tp_world` (at most 8, one process per GPU) holds heads / world query and KV heads (its
 * own KV cache), intermediate / world MLP rows, the matching input columns of o_proj and
 * down_proj, and its share of the LM-head vocabulary rows; the embedding and the RMSNorm
 * gains are whole. yue2_model_init_synthetic fills a shard with exactly the values the
 * unsharded model holds at those positions; yue2_model_set_tensor takes the shard's own
 * slice (the checkpoint loader refuses a sharded model). After yue2_model_finalize every
 * rank calls yue2_tp_export, the ranks exchange the handles (any host channel), and every
 * rank calls yue2_tp_connect with all of them in rank order. Decode (forward, prefill,
 * sessions, generate) then runs one or two rows per pass, every rank the same calls in the
 * same order; o and down end in an exchange that sums the ranks' partials in rank order and
 * applies the residual, and the LM head ends in a gather of the vocabulary slices, so every
 * rank holds identical logits and samples identical tokens. */
int yue2_model_create_tp(int device, const Yue2Config* cfg, uint64_t tp_rank, uint64_t tp_world, Yue2Model** out);
/* 128 bytes: this rank's two CUDA IPC handles (exchange buffer, logits). */
int yue2_tp_export(Yue2Model* m, void* handles);
/* tp_world x 128 bytes of handles in rank order (this rank's own entry is not opened). */
int yue2_tp_connect(Yue2Model* m, const void* handles);
/* Upload one checkpoint tensor by its reference name (model.rs:76-93,103-114,176-200,
 * 250-270,418-451). Tensors outside the AR decode path are accepted and ignored (returns 1). */
int yue2_model_set_tensor(Yue2Model* m, const char* name, int dtype, const void* data, uint64_t rows,
                          uint64_t cols);
/* Seeded synthetic weights on the device: matrices and embeddings N(0, std), RMSNorm
 * gains norm_mean + N(0, std), all rounded to bf16. */
int yue2_model_init_synthetic(Yue2Model* m, uint64_t seed, float std, float norm_mean);
/* Checks that every AR tensor is present and prepares RoPE tables and workspaces. */
int yue2_model_finalize(Yue2Model* m);
/* Model::open's tensor reads (src/model.rs:418-451) over Weights::open
 * (src/checkpoint.rs:315-396): the checkpoint directory `dir` holds model.safetensors or
 * model.safetensors.index.json + shards. Headers are validated as the reference does
 * (header size, dtype F32/BF16/F16, extents, duplicates, overlaps, shard paths); every
 * tensor on the AR decode path is uploaded (BF16 matrices through pinned double-buffered
 * staging; gains and F32/F16 matrices converted as yue2_model_set_tensor does). Other
 * tensors (NAR, latent, VAE bridges) are skipped. `bytes_uploaded` (nullable) receives the
 * bytes copied to the device. Call yue2_model_finalize afterwards. */
int yue2_model_load_checkpoint(Yue2Model* m, const char* dir, uint64_t* bytes_uploaded);
/* Timing and parity hook for the prefill GEMMs: Y[C, N] = X[C, K] . W[N, K]^T on device
 * bf16 buffers (row-major, dense), `reps` timed runs after one untimed; impl 0 = cuBLASLt,
 * 1 = the tcgen05 kernel (K a multiple of 64), 2 = its gate|up form: W = [gate; up] of
 * [2N, K] and Y = bf16(bf16(silu(bf16 g)) * bf16 u) of [C, N] (N a multiple of 128);
 * 3 = the skinny tcgen05 kernel of the decode passes (C <= 256, K a multiple of 64),
 * 4 = its gate|up form. `avg_ms` (nullable) gets the mean. */
int yue2_bench_gemm(Yue2Model* m, const void* X, const void* W, void* Y, int C, int N, int K, int impl, int reps,
                    double* avg_ms);
/* Reserves device slots for the NAR (flow-matching) tensors of Model::open
 * (src/model.rs:418-451): latent_pos_embed.pe, vae2llm/llm2vae weight+bias,
 * time_embedder.mlp.{0,2} weight+bias and every layer's nar_self_attn / nar_mlp /
 * nar_*layernorm. Call before loading (yue2_model_load_checkpoint or set_tensor), then
 * yue2_model_finalize, which then also requires these tensors. */
int yue2_model_enable_nar(Yue2Model* m, uint64_t latent_dim, uint64_t max_latent_frames, float timestep_shift);
/* Header validation only (no device needed): the number of tensors in the checkpoint. */
int yue2_checkpoint_scan(const char* dir, uint64_t* tensors);
/* Copies a device tensor back as bf16 bits (count elements). */
int yue2_model_get_tensor(Yue2Model* m, const char* name, uint16_t* out, uint64_t count);
void yue2_model_free(Yue2Model* m);

/* Cache::new (src/model.rs:292-305): paged BF16 KV reserved for `capacity` positions. */
int yue2_cache_create(Yue2Model* m, uint64_t capacity, Yue2Cache** out);
/* Cache::drop (src/model.rs:286-290). */
void yue2_cache_free(Yue2Cache* c);
int yue2_cache_length(const Yue2Cache* c, uint64_t* length);
/* Fill positions [length, to) of every layer with seeded N(0,1) bf16 keys/values and set
 * the length to `to` (synthetic long-context state). */
int yue2_cache_fill_normal(Yue2Cache* c, uint64_t to, uint64_t seed);
/* Read positions [begin, begin+count) of one layer as bf16 bits [count, kv*dim] each. */
int yue2_cache_read(const Yue2Cache* c, uint64_t layer, uint64_t begin, uint64_t count, uint16_t* k,
                    uint16_t* v);

/* Model::forward / forward_phase (src/model.rs:465-477) for `rows` (<= 256) distinct caches
 * at once, one new id per cache; logits [rows, vocab] (nullable). One or two rows run as a
 * weight-streaming GEMV pass, more as tensor-core GEMMs. YUE2_PHASE_VOCAB returns
 * the full LM-head row; ABC/SEMANTIC return project_phase's window + stop row with -inf
 * elsewhere (model.rs:478-507). */
int yue2_forward(Yue2Model* m, Yue2Cache* const* caches, const int64_t* ids, uint64_t rows, int phase,
                 float* logits);
/* Model::prefill / prefill_phase (src/model.rs:508-522, 592-610): append `n` ids to the
 * cache; logits of the last id (nullable). */
int yue2_prefill(Yue2Model* m, Yue2Cache* c, const int64_t* ids, uint64_t n, int phase, float* logits);

/* Model::velocity (src/model.rs:611-697, nar_cond_end = 0): the flow-matching velocity of
 * `rows` latent frames `state` [rows, latent_dim] (host f32 holding bf16 values, as the
 * solver's states are) at logit time `raw_t`, attending to the whole cache prefix and to
 * every latent row (no causal mask); `out` [rows, latent_dim] (host). Cache length + rows + 2
 * within the cache capacity (the latent rows' K/V go to the pages past the length as
 * scratch); the cache's length does not change. Needs yue2_model_enable_nar and head_dim 64
 * or 128. */
int yue2_velocity(Yue2Model* m, Yue2Cache* c, const float* state, uint64_t rows, double raw_t, float* out);

/* Model::synthesize (src/model.rs:699-776): the acoustic latents [codec_len, 64] (host) of
 * one song. Chunks of (min(24576, max_position_embeddings) - prefix_len - 3) / 2 frames:
 * each prefills prefix + (codec + CODEC_OFFSET) + MUSIC_END into its own cache, then runs
 * `steps` midpoint steps (two yue2_velocity calls each) from the chunk's slice of the
 * song's noise (yue2_noise(seed, codec_len, 64)). Codec ids in [0, 32768); the reference's
 * errors: "Expected nonempty codec tokens and a 64-dimensional latent model", "Prefix leaves
 * no acoustic context", "Flow matching produced nonfinite latents". */
int yue2_synthesize(Yue2Model* m, const int64_t* prefix, uint64_t prefix_len, const int64_t* codec,
                    uint64_t codec_len, uint64_t seed, uint64_t steps, float* out);
/* Generator::new(seed).normal_tensor(rows, cols) (src/sampling.rs:63-78) on the host:
 * rows * cols a multiple of 16. Needs no device. */
int yue2_noise(uint64_t seed, uint64_t rows, uint64_t cols, float* out);

/* Request-local MT19937 (src/sampling.rs:10-62), state kept on the device of `m`. */
int yue2_rng_create(Yue2Model* m, uint64_t seed, Yue2Rng** out);
void yue2_rng_free(Yue2Rng* r);
/* state[624] and the next index (624 right after seeding). */
int yue2_rng_state(const Yue2Rng* r, uint32_t* state, uint64_t* next);

/* sampling::choose (src/sampling.rs:103-215) on the device: logits [vocab] (host), the
 * generated ids so far, the step index; draws from `rng` exactly as the reference
 * (2*vocab words per sampled step, none at temperature 0). */
int yue2_choose(Yue2Model* m, const float* logits, uint64_t vocab, const Yue2Sampling* s,
                const int64_t* history, uint64_t hlen, uint64_t step, int phase, int legacy, Yue2Rng* rng,
                int64_t* out);

/* One song of sampling::generate. */
typedef struct {
  const int64_t* prefix;
  uint64_t prefix_len;
  const int64_t* negative; /* NULL when scale == 1 */
  uint64_t negative_len;
  uint64_t seed;
  float scale;
  int32_t legacy;
  /* > 0: positions [0, context_fill) of the song's caches hold seeded N(0,1) bf16 keys
   * and values (synthetic long-context state) and the prefixes are appended after them. */
  uint64_t context_fill;
  int64_t* tokens;         /* out: room for sampling.max_tokens ids */
  uint64_t count;          /* out */
  int32_t truncated;       /* out */
  int32_t status;          /* out: 0 or YUE2_ERR_* */
} Yue2Request;

typedef struct {
  double seconds;          /* wall time of the whole call (reference `seconds`) */
  double prefill_seconds;  /* wall time of the prefills (reference `prefill_seconds`) */
  double decode_ms;        /* device time of the decode loop (CUDA events) */
  uint64_t decode_steps;   /* decode graph launches */
  uint64_t kernels_per_step;
} Yue2Timing;

/* sampling::generate (src/sampling.rs:222-294) for `n` independent songs sharing one
 * Sampling and phase (at most 256 rows per step: 128 songs with CFG; CFG rows count
 * twice): prefill (cond and, when scale != 1, uncond), then one graph launch per token:
 * both CFG rows of every song in one weight pass (GEMV for 1-2 rows, tensor-core GEMMs
 * from 3 rows), on-device CFG mix + choose. */
int yue2_generate(Yue2Model* m, const Yue2Sampling* s, int phase, Yue2Request* reqs, uint64_t n,
                  Yue2Timing* timing);

/* The same loop as a resumable session (sampling.rs:243-287 split at its step
 * boundary): create = validation, caches, prefills and the first draw; step = enqueue up
 * to `steps` decode steps (one graph launch each: forward of every row, then CFG mix +
 * choose) without waiting for them; collect = wait and copy each song's result into
 * reqs[i] (tokens, count, truncated, status). */
typedef struct Yue2Session Yue2Session;
int yue2_session_create(Yue2Model* m, const Yue2Sampling* s, int phase, const Yue2Request* reqs, uint64_t n,
                        Yue2Session** out);
int yue2_session_step(Yue2Session* ss, uint64_t steps, uint64_t* launched);
int yue2_session_sync(Yue2Session* ss);
int yue2_session_collect(Yue2Session* ss, Yue2Request* reqs);
/* cudaStream_t the session's kernels run on (for timing with events on that stream). */
void* yue2_session_stream(Yue2Session* ss);
uint64_t yue2_session_kernels_per_step(const Yue2Session* ss);
void yue2_session_free(Yue2Session* ss);

/* Measurement hook (no reference counterpart): `launches` back-to-back launches of one
 * weight-streaming GEMV kind over the layers in turn, `rows` activation rows, CUDA
 * events on the model's stream. kind 0 = gate|up + SwiGLU, 1 = q|k|v, 2 = down +
 * residual, 3 = final norm + LM head, 4 = o + residual. The launches are programmatic dependents
 * of each other when the model uses them, as in the decode chain. Returns the mean launch time and
 * the weight bytes one launch streams. */
int yue2_bench_gemv(Yue2Model* m, int kind, int rows, int launches, double* avg_ms, double* bytes);

#ifdef __cplusplus
}
#endif
#endif
