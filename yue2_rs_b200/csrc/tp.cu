// Tensor parallelism of the decode step over NVLink peer memory (sm_100a).
//
// Rank r of W holds heads / W query heads and KV heads, intermediate / W MLP rows, the
// matching input columns of o and down, and W-th of the LM-head vocabulary rows. A layer's
// o and down projections then leave partial sums of the full hidden width on every rank.
// The GEMV that computes them also exchanges them (its kEpiTpReduce epilogue,
// kernels_layer.cu): every thread stores its outputs into every rank's receive buffer and
// then adds all ranks' values of the same outputs in rank order with the residual, the
// reference's x = bf16(x + bf16(Wo . h)) (src/model.rs:586, src/tensor.rs:632-640) with the
// f32 sum taken over the ranks' partial dot products. The LM head leaves each rank its
// vocabulary slice; `tp_allgather` copies every slice to every rank, so each rank holds
// identical logits and runs the same sampler on the same generator (no broadcast of the
// sampled id is needed).
//
// No exchange uses a library collective. Values travel as 8-byte words that pair the
// value with the exchange's tag (tp.cuh), stored into peers' buffers through CUDA IPC
// mappings; a reader polls the words it needs until they carry the tag: no flag, no
// system-scope fence, one pass over NVLink. Tags only grow (the forward count times 256
// plus the exchange's number), so nothing needs resetting, and a rank is at most one
// exchange ahead of another: the o/down buffers alternate by exchange parity. Every wait is
// bounded (about a second of SM clocks); a wait that gives up sets the error flag, and the
// host reports YUE2_ERR_TIMEOUT.
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/yue2_cuda.h"
#include "common.cuh"
#include "engine.h"
#include "kernels.h"
#include "tp.cuh"

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #expr);   \
  } while (0)

namespace y2 {

// Every rank's logits columns [col0_q, col0_q + cols_q) of rows [row_base, row_base + R) to
// every rank: this rank's slice to the others' word buffers, then theirs into its logits.
__global__ void __launch_bounds__(256) tp_allgather_kernel(const TpParams p) {
  pdl_wait();  // the logits come from the preceding LM-head GEMV
  pdl_trigger();
  const TpPeers& P = *p.peers;
  const uint32_t tag = (*p.epoch) * 256u + (uint32_t)p.site + 1u;
  const int stride = gridDim.x * blockDim.x;
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
  const float* mine = P.logits[p.rank];
  const int n = p.R * p.cols;
  for (int i = i0; i < n; i += stride) {
    const size_t at = (size_t)(p.row_base + i / p.cols) * p.n + p.col0 + i % p.cols;
    const float v = __ldcg(mine + at);
    for (int t = 0; t < p.world; ++t)
      if (t != p.rank) st_ll(P.gather[t] + at, v, tag);
  }
  bool ok = true;
  const uint2* words = P.gather[p.rank];
  float* out = P.logits[p.rank];
  for (int q = 0; q < p.world; ++q) {
    if (q == p.rank) continue;
    const int c0 = (int)((long long)p.n * q / p.world), cq = (int)((long long)p.n * (q + 1) / p.world) - c0;
    for (int i = i0; i < p.R * cq; i += stride) {
      const size_t at = (size_t)(p.row_base + i / cq) * p.n + c0 + i % cq;
      out[at] = wait_ll(words + at, tag, p.error, ok);
    }
  }
}

__global__ void tp_tick_kernel(uint32_t* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) *epoch += 1;
}

cudaError_t launch_tp_allgather(cudaStream_t s, bool pdl, const TpParams& p) {
  if (p.R < 1 || p.R > kTpRows || p.world < 1 || p.world > kTpMaxWorld) return cudaErrorInvalidValue;
  TpParams copy = p;
  void* args[] = {&copy};
  return launch_with(s, pdl, dim3(kTpCtas), dim3(256), 0, (const void*)tp_allgather_kernel, args);
}

cudaError_t launch_tp_tick(cudaStream_t s, bool pdl, uint32_t* epoch) {
  void* args[] = {&epoch};
  return launch_with(s, pdl, dim3(1), dim3(32), 0, (const void*)tp_tick_kernel, args);
}

// Bytes of a rank's receive allocation: two parity halves of [kTpMaxWorld][kTpRows][hidden]
// exchange words, then the logits words [kMaxRows][vocab].
size_t tp_recv_bytes(int hidden, int vocab) {
  return 2 * (size_t)kTpMaxWorld * kTpRows * hidden * 8 + (size_t)kMaxRows * vocab * 8;
}
static size_t tp_gather_offset(int hidden) { return 2 * (size_t)kTpMaxWorld * kTpRows * hidden * 8; }

}  // namespace y2

using namespace y2;

extern "C" {

int yue2_tp_export(Yue2Model* m, void* handles) {
  if (!m || !handles) return fail(YUE2_ERR_INVALID, "null argument");
  if (m->tp_world < 2) return fail(YUE2_ERR_INVALID, "not a tensor-parallel model");
  if (!m->tp_recv || !m->logits) return fail(YUE2_ERR_INVALID, "model not finalized");
  int rc = y2_set_device(m);
  if (rc) return rc;
  cudaIpcMemHandle_t h[2];
  CK(cudaIpcGetMemHandle(&h[0], m->tp_recv));
  CK(cudaIpcGetMemHandle(&h[1], m->logits));
  memcpy(handles, h, sizeof(h));
  return 0;
}

int yue2_tp_connect(Yue2Model* m, const void* handles) {
  if (!m || !handles) return fail(YUE2_ERR_INVALID, "null argument");
  if (m->tp_world < 2) return fail(YUE2_ERR_INVALID, "not a tensor-parallel model");
  if (!m->tp_recv || !m->logits) return fail(YUE2_ERR_INVALID, "model not finalized");
  if (m->tp_connected) return fail(YUE2_ERR_INVALID, "already connected");
  int rc = y2_set_device(m);
  if (rc) return rc;
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  TpPeers peers = {};
  for (int q = 0; q < m->tp_world; ++q) {
    char* recv = nullptr;
    float* logits = nullptr;
    if (q == m->tp_rank) {
      recv = m->tp_recv;
      logits = m->logits;
    } else {
      void* a = nullptr;
      void* b = nullptr;
      CK(cudaIpcOpenMemHandle(&a, h[2 * q], cudaIpcMemLazyEnablePeerAccess));
      m->tp_opened.push_back(a);
      CK(cudaIpcOpenMemHandle(&b, h[2 * q + 1], cudaIpcMemLazyEnablePeerAccess));
      m->tp_opened.push_back(b);
      recv = (char*)a;
      logits = (float*)b;
    }
    peers.recv[q] = (uint2*)recv;
    peers.gather[q] = (uint2*)(recv + tp_gather_offset(m->g.hidden));
    peers.logits[q] = logits;
  }
  void* d = nullptr;
  if ((rc = m->alloc(&d, sizeof(TpPeers)))) return rc;
  CK(cudaMemcpy(d, &peers, sizeof(TpPeers), cudaMemcpyHostToDevice));
  m->tp_peers = (TpPeers*)d;
  m->tp_connected = true;
  return 0;
}

}  // extern "C"
