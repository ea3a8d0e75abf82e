// Host-side objects behind the opaque handles of include/yue2_cuda.h.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <set>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "kernels.h"

namespace y2 {

// Fixed-size KV pages (kPageTokens positions of every layer) carved from cudaMalloc
// chunks; a cache owns a page table of device addresses, so caches of any length
// share one pool without fragmentation.
struct PagePool {
  size_t page_bytes = 0;
  std::vector<void*> chunks;
  std::vector<uint64_t> free_pages;
  int take(size_t n, std::vector<uint64_t>& out);
  void give(const std::vector<uint64_t>& pages);
  void clear();
};

struct TensorSlot {
  size_t offset = 0, rows = 0, cols = 0;
  bool norm = false;      // f32 gain (or bias) vector; matrices are bf16
  char* base = nullptr;   // allocation holding the tensor (null: the model's weight arena)
  // a tensor-parallel shard holds rows [row0, row0 + rows) and columns [col0, col0 + cols)
  // of the full [full_rows, full_cols] tensor (the whole tensor without sharding)
  size_t full_rows = 0, full_cols = 0, row0 = 0, col0 = 0;
};

int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

struct PrefillBufs;  // GEMM workspace and cuBLASLt state (gemm_rows.cu)
void free_prefill(PrefillBufs* p);

}  // namespace y2

struct Yue2Model {
  int device = 0;
  Yue2Config cfg{};
  y2::Geometry g{};
  int sms = 148;
  int gemv_grid = 148;
  bool use_pdl = true, use_graphs = true;
  int ctx_hint = 0;       // longest row context of the next captured forward (picks the attention loop)
  bool use_prefill_gemm = true;  // prompts of >= kPrefillGemmMin ids as GEMMs (YUE2_CUDA_PREFILL=gemv: off)
  int prefill_chunk = 1024;      // rows per GEMM prefill chunk, <= kPrefillRows (YUE2_CUDA_PREFILL_CHUNK)
  bool prefill_tc_attn = true;   // tensor-core prefill attention (YUE2_CUDA_PREFILL_ATTN=rows: per-row kernel)
  // its tcgen05 form for head_dim 128: 0 when the grid fills two waves of the SMs (else the
  // mma.sync form), 1 always (YUE2_CUDA_PREFILL_ATTN=tc), 2 never (=sync)
  int prefill_attn_tc5 = 0;
  bool gemm_split_k = false;     // GEMMs may split K with an f32 out-of-place reduction (YUE2_CUDA_GEMM_SPLITK=1)
  int wide_min = 3;              // decode passes of at least this many rows use the GEMM path (YUE2_CUDA_WIDE_MIN)
  int attn_splits = 0;             // > 0: decode attention splits per (kv head, row), forced
  // decode attention as CTA clusters merged in distributed shared memory while a captured
  // forward's rows stay within kClusterKeys keys (YUE2_CUDA_ATTN_CLUSTER: -1 auto, 0 off,
  // 1..8 CTAs per (kv head, row) forced); ctx_growth = positions a captured graph advances
  int attn_cluster = -1;
  int ctx_growth = 0;
  bool wide_pdl = true;          // passes of > 2 rows launch their kernels as programmatic dependents
  // passes of up to this many rows run their per-layer GEMMs on the skinny tcgen05 kernel
  // (YUE2_CUDA_SKINNY: 0 off, 1 up to 256 rows; default 16, where it matches cuBLASLt)
  int skinny_rows = 16;
  bool gemm_tc = false;          // GEMMs of >= 128 rows on the tcgen05 kernel (YUE2_CUDA_GEMM=tc), else cuBLASLt
  y2::PrefillBufs* prefill = nullptr;
  // decode steps of more than kMaxRows rows (the GEMM path): row descriptors, logits
  // [kMaxWideRows, vocab] and the bf16 LM head output
  y2::DevRow* wide_rows = nullptr;
  float* wide_logits = nullptr;
  uint16_t* wide_head = nullptr;
  bool finalized = false, workspace_ready = false;

  char* arena = nullptr;
  std::map<std::string, y2::TensorSlot> slots;
  std::set<std::string> loaded;
  uint16_t *embed = nullptr, *lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<y2::LayerW> layers;
  // NAR pathway (Model::velocity, src/model.rs:611-697), after yue2_model_enable_nar: the
  // nar_* layer weights (in_norm = nar_input_layernorm, post_norm = nar_pre_mlp_layernorm),
  // the latent projections with their bf16-rounded biases and the time embedder
  struct NarW {
    const uint16_t *pe = nullptr, *vae2llm = nullptr, *llm2vae = nullptr, *time_in = nullptr, *time_out = nullptr;
    const float *vae2llm_b = nullptr, *llm2vae_b = nullptr, *time_in_b = nullptr, *time_out_b = nullptr;
    int latent = 0, max_frames = 0;
    float shift = 1.f;
  } nar;
  std::vector<y2::LayerW> nar_layers;
  char* nar_arena = nullptr;

  float *cos_tab = nullptr, *sin_tab = nullptr;
  int max_pos = 0;
  y2::PagePool pool;

  cudaStream_t stream = nullptr, side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;

  // step workspace (kMaxRows rows)
  float* x = nullptr;
  uint16_t *qkv = nullptr, *qrot = nullptr, *attn = nullptr, *hbuf = nullptr;
  float* logits = nullptr;
  float* part = nullptr;
  int32_t* counters = nullptr;
  y2::DevRow* rows = nullptr;
  int32_t* flags = nullptr;  // [0] token out of range, [1] position outside RoPE table, [2] GEMV stream stall
  int max_splits = 64;

  // ---- tensor parallelism (tp.cu): rank tp_rank of tp_world holds heads / tp_world query
  // and key-value heads, intermediate / tp_world MLP rows, the matching input columns of o
  // and down, and the LM-head rows [head_row0, head_row0 + head_rows) of the vocabulary
  int tp_rank = 0, tp_world = 1;
  int head_row0 = 0, head_rows = 0;
  char* tp_recv = nullptr;        // IPC-exported exchange words (tp.cu, tp_recv_bytes)
  uint32_t* tp_epoch = nullptr;   // forwards run so far (the same count on every rank)
  y2::TpPeers* tp_peers = nullptr;  // device copy of every rank's receive / logits addresses
  std::vector<void*> tp_opened;   // peer mappings to close
  bool tp_connected = false;
  static constexpr int kRowSlots = 32;  // pinned staging ring for row descriptors
  y2::DevRow* pinned_rows = nullptr;
  cudaEvent_t row_events[kRowSlots] = {};
  uint64_t row_slot = 0;
  int32_t* pinned_flags = nullptr;

  std::map<int, cudaGraphExec_t> graphs;
  std::vector<void*> allocations;
  // Device scratch reused across calls (sampler buffers, prompt uploads, page tables):
  // cudaFree can stall the host for hundreds of milliseconds, so finished calls return
  // their buffers here; they are freed with the model.
  std::multimap<size_t, void*> scratch_free;
  std::map<void*, size_t> scratch_cap;

  int alloc(void** p, size_t bytes);
  char* slot_addr(const y2::TensorSlot& t) const { return (t.base ? t.base : arena) + t.offset; }
  int scratch_take(void** p, size_t bytes);
  void scratch_give(void* p);
  int max_pos_limit() const {
    return (int)(cfg.max_position_embeddings < (1u << 20) ? cfg.max_position_embeddings : (1u << 20));
  }
  ~Yue2Model();
};

struct Yue2Cache {
  Yue2Model* m = nullptr;
  std::vector<uint64_t> pages;
  uint64_t* d_pages = nullptr;
  uint64_t capacity = 0, length = 0;
};

struct Yue2Rng {
  Yue2Model* m = nullptr;
  y2::MtState* state = nullptr;
};

int y2_set_device(const Yue2Model* m);

namespace y2 {
int splits_for(const Yue2Model& m, int R);
int check_phase_vocab(const Yue2Model& m, int phase);
cudaError_t encode_forward(Yue2Model& m, cudaStream_t s, int R, bool head, int phase, const int32_t* skip);
cudaError_t encode_head(Yue2Model& m, cudaStream_t s, bool pdl, int x_row, int R, int dst_row, int phase,
                        const int32_t* skip);
cudaError_t encode_head_from(Yue2Model& m, cudaStream_t s, bool pdl, const float* x, int R, int dst_row, int phase,
                             const int32_t* skip);
int kernels_per_step(const Yue2Model& m, bool head, int phase, int R);
TpParams tp_params(const Yue2Model& m);  // the rank, peers, epoch and error flag of m's exchanges
int tp_ready(const Yue2Model& m);        // 0, or an error when a TP model is not connected
int attn_pipe_for(const Yue2Model& m, int R);
// CTAs per (kv head, row) of the cluster form of decode attention, 0 for the split-K kernels
int attn_cluster_for(const Yue2Model& m, int R);
int run_forward(Yue2Model& m, int R, bool head, int phase);
int upload_rows(Yue2Model& m, const std::vector<DevRow>& rows);
int take_flags(Yue2Model& m);
int prefill_device(Yue2Model& m, Yue2Cache& c, const int32_t* d_ids, uint64_t n, int logits_row, int phase);
int prefill_gemm(Yue2Model& m, Yue2Cache& c, const int32_t* d_ids, uint64_t n, int logits_row, int phase);
int ensure_wide(Yue2Model& m);
int encode_forward_wide(Yue2Model& m, cudaStream_t s, int R, int phase);
int prepare_wide(Yue2Model& m, int R, int phase);
int wide_kernels_per_step(const Yue2Model& m, int phase, int R);
constexpr int kMaxWideRows = 256;    // rows of a wide decode step (128 songs with CFG)
constexpr int kPrefillGemmMin = 3;   // shorter prompts go through the GEMV chain
constexpr int kPrefillRows = 1024;   // capacity of the GEMM prefill buffers, in rows
}  // namespace y2
