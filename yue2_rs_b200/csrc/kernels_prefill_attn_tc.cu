// Chunk attention over the paged cache on the 5th-generation tensor cores (tcgen05), for
// head_dim 128: the same function as prefill_attn_kernel (attention, src/model.rs:314-397:
// scale 1/sqrt(dim), f32 softmax, P.V with f32 probabilities, bf16 output), causal for
// prefill chunks and non-causal for the NAR pathway's latent rows.
//
// One CTA of 4 warps takes 128 query rows of one head; thread t owns row t, which is TMEM
// lane t. Per 64-key tile (one cache page):
//   1. all threads copy the page's K rows into a 128-byte-swizzled K-major tile and its V
//      rows into a staging tile; the warps transpose V into V^T (dims as rows,
//      keys along the row: the K-major B operand of P.V) with ldmatrix.trans + stmatrix;
//   2. one thread issues S = Q.K^T (M 128, N 64, K 128: 8 MMAs) into TMEM columns 0..63;
//   3. each thread reads its row of S, masks, updates the running max, and writes its
//      probabilities as bf16 hi + lo parts (hi + lo carries the f32 value to 2^-16) into two
//      128-byte-swizzled tiles;
//   4. one thread issues O += P_hi.V + P_lo.V (M 128, N 128, K 64: 8 MMAs); O stays in
//      TMEM columns 128..255 across pages. Before that, a warp whose rows' running max moved
//      scales its rows of O by exp(m_old - m_new) (tcgen05.ld, multiply, tcgen05.st), so
//      O_t = alpha O_(t-1) + P_t V_t as before; the final O is read once.
// The next page's K copies (cp.async) and V loads (into registers) start as soon as S is
// computed, so they run under the softmax and P.V; two CTAs per SM overlap one's softmax
// with the other's MMAs. Every wait on an MMA is bounded: when one gives up, the CTA
// sets the model's error flag, stops, and still frees its TMEM.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace y2 {
namespace {

constexpr int D = 128;     // head dim
constexpr int QROWS = 128; // query rows per CTA (TMEM lanes)
constexpr int KT = 64;     // keys per tile: one page
constexpr int THREADS = 128;
constexpr int TMEM_COLS = 256;  // S: columns 0..63; O: columns 128..255
constexpr int O_COL = 128;
constexpr long kSpin = 1L << 22;

// shared memory, each tile 1024-byte aligned
constexpr int Q_BYTES = QROWS * D * 2;  // 2 slabs of [128 rows][128 B] (dims 0..63, 64..127)
constexpr int K_BYTES = KT * D * 2;     // 2 slabs of [64 rows][128 B]
constexpr int VT_BYTES = D * KT * 2;    // [128 dims][128 B = 64 keys]
constexpr int P_BYTES = QROWS * KT * 2; // [128 rows][128 B = 64 keys]
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + Q_BYTES;
constexpr int OFF_VT = OFF_K + K_BYTES;
constexpr int OFF_PH = OFF_VT + VT_BYTES;
constexpr int OFF_PL = OFF_PH + P_BYTES;  // also the V staging tile [64 keys][256 B] before P is written
constexpr int OFF_BAR = OFF_PL + P_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;  // + barrier, TMEM slot, alignment slack

__global__ void __launch_bounds__(THREADS, 2) prefill_attn_tc_kernel(const PrefillAttnParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* qs = smem + OFF_Q;
  unsigned char* ks = smem + OFF_K;
  unsigned char* vt = smem + OFF_VT;
  unsigned char* ph = smem + OFF_PH;
  unsigned char* pl = smem + OFF_PL;
  unsigned char* vstage = pl;
  uint64_t* bar = (uint64_t*)(smem + OFF_BAR);
  uint32_t* tmem_slot = (uint32_t*)(smem + OFF_BAR + 8);

  const Geometry& g = p.g;
  const int ntiles = (p.C + QROWS - 1) / QROWS;
  const int tile = ntiles - 1 - (int)blockIdx.x;  // longest rows first
  const int h = blockIdx.y, kvh = h / (g.heads / g.kvh);
  const int row0 = tile * QROWS;
  const int nrows = min(QROWS, p.C - row0);
  const int q0 = p.pos0 + row0;
  const int last_key = p.causal ? q0 + nrows - 1 : p.pos0 + p.C - 1;
  const int nkt = (last_key >> kPageLog2) + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = g.heads * D;
  const size_t koff = kv_offset(g, p.layer, 0, kvh), voff = kv_offset(g, p.layer, 1, kvh);
  const int pos_r = p.causal ? q0 + tid : last_key;  // the last key this thread's row sees

  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::mbar_init_fence();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // the Q tile: 128 rows x 16 chunks of 16 B, rows past the chunk zero-filled
  for (int i = tid; i < QROWS * 16; i += THREADS) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < nrows;
    cp_async16_zfill(qs + (c >> 3) * (QROWS * 128) + tc::sw128(r, c & 7),
                     p.q + (size_t)(row0 + (ok ? r : 0)) * qd + (size_t)h * D + c * 8, ok);
  }
  cp_async_commit();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  constexpr uint32_t ID_S = tc::idesc_bf16(QROWS, KT), ID_O = tc::idesc_bf16(QROWS, D);

  float m = -INFINITY, l = 0.f;
  uint32_t phase = 0;
  bool ok = true;

  // copies of one page: K into its swizzled K-major tile, V into the staging tile
  // ([key][256 B], chunk c at c ^ (key & 7)); keys past last_key are zero-filled
  auto load_k = [&](int kt) {
    const uint16_t* page = reinterpret_cast<const uint16_t*>(p.pages[kt]);
    for (int i = tid; i < KT * 16; i += THREADS) {
      const int r = i >> 4, c = i & 15;
      const bool valid = (kt << kPageLog2) + r <= last_key;
      cp_async16_zfill(ks + (c >> 3) * (KT * 128) + tc::sw128(r, c & 7),
                       page + koff + (size_t)(valid ? r : 0) * D + c * 8, valid);
    }
    cp_async_commit();
  };
  // the next page's V: each thread holds 8 chunks of 16 B in registers while the softmax and
  // P.V of this page run, then writes them to the staging tile ([key][256 B], chunk c at
  // c ^ (key & 7)) once P.V has released it
  uint4 vreg[8];
  auto fetch_v = [&](int kt) {
    const uint16_t* page = reinterpret_cast<const uint16_t*>(p.pages[kt]);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * THREADS, r = i >> 4, c = i & 15;
      const bool valid = (kt << kPageLog2) + r <= last_key;
      vreg[u] = valid ? ldg16(page + voff + (size_t)r * D + c * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  auto put_v = [&]() {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = tid + u * THREADS, r = i >> 4, c = i & 15;
      *reinterpret_cast<uint4*>(vstage + r * 256 + ((c ^ (r & 7)) << 4)) = vreg[u];
    }
  };
  // waits for the K copies, then V^T from the staging tile: 8 key blocks x 16 dim blocks of
  // 8 x 8, each warp moving 4 x 8 of them (ldmatrix.trans, stmatrix); ends with both tiles
  // ready for the tensor cores
  auto stage_v = [&]() {
    cp_async_wait<0>();
    tc::fence_before();
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = warp * 8 + u;          // 0..31
      const int kb = j >> 2, dbg = j & 3;  // key block, group of 4 dim blocks
      const int mi = lane >> 3, rr = lane & 7;
      const int db = dbg * 4 + mi;
      uint32_t f[4];
      const int key = kb * 8 + rr;
      ldsm_x4_trans(f, vstage + key * 256 + ((db ^ (key & 7)) << 4));
      tc::stsm_x4(vt + tc::sw128(db * 8 + rr, kb), f);
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
  };

  load_k(0);
  fetch_v(0);
  put_v();
  stage_v();
  for (int kt = 0; kt < nkt && ok; ++kt) {
    const bool more = kt + 1 < nkt;
    // ---- 2. S = Q . K^T
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t a = tc::sdesc_sw128(tc::smem_u32(qs + (kk >> 2) * (QROWS * 128) + (kk & 3) * 32));
        const uint64_t b = tc::sdesc_sw128(tc::smem_u32(ks + (kk >> 2) * (KT * 128) + (kk & 3) * 32));
        tc::mma_bf16(tmem, a, b, ID_S, kk > 0);
      }
      tc::commit(bar);
    }
    ok = tc::mbar_wait_bounded(bar, phase, p.error, kSpin);
    phase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc::fence_after();
    if (more) {  // the K tile is free: the next page's K and V load under the softmax and P.V
      load_k(kt + 1);
      fetch_v(kt + 1);
    }

    // ---- 3. softmax of this thread's row; P = hi + lo into shared memory
    float s[KT];
    {
      uint32_t v[32];
      tc::tmem_ld32(lane_base + 0, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(v[j]);
      tc::tmem_ld32(lane_base + 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) s[32 + j] = __uint_as_float(v[j]);
    }
    const int key0 = kt << kPageLog2;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      s[j] = key0 + j <= pos_r ? s[j] * p.scale : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    // key 0 is in tile 0 and precedes every row, so m is finite from the first tile on
    const float mn = fmaxf(m, mx);
    const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
    m = mn;
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float x0 = __expf(s[8 * c + 2 * q] - mn), x1 = __expf(s[8 * c + 2 * q + 1] - mn);
        sum += x0 + x1;
        hw[q] = pack_bf16x2(x0, x1);
        lw[q] = pack_bf16x2(x0 - bf_lo(hw[q]), x1 - bf_hi(hw[q]));
      }
      *reinterpret_cast<uint4*>(ph + tc::sw128(tid, c)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(pl + tc::sw128(tid, c)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    l = l * alpha + sum;
    // O (in TMEM since the last page) times exp(m_old - m_new), by the warps holding a row
    // whose max moved; page 0's P.V overwrites O instead
    if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(lane_base + O_COL + 32 * c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
        tc::tmem_st32(lane_base + O_COL + 32 * c, v);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();

    // ---- 4. O += P_hi . V + P_lo . V
    if (tid == 0) {
      tc::fence_after();
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        const uint64_t b = tc::sdesc_sw128(tc::smem_u32(vt + kk * 32));
        tc::mma_bf16(tmem + O_COL, tc::sdesc_sw128(tc::smem_u32(ph + kk * 32)), b, ID_O, kt > 0 || kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk) {
        const uint64_t b = tc::sdesc_sw128(tc::smem_u32(vt + kk * 32));
        tc::mma_bf16(tmem + O_COL, tc::sdesc_sw128(tc::smem_u32(pl + kk * 32)), b, ID_O, 1);
      }
      tc::commit(bar);
    }
    ok = tc::mbar_wait_bounded(bar, phase, p.error, kSpin);
    phase ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc::fence_after();
    if (more) {
      put_v();    // P_lo (the staging tile) and V^T are free
      stage_v();  // also orders this page's TMEM accesses before the next page's MMAs
    }
  }
  if (!ok) cp_async_wait<0>();


  // ---- normalise and store bf16 (rows of this chunk only); the TMEM loads are warp-wide
  if (ok) {
    const float inv = 1.0f / l;
    uint16_t* dst = p.out + (size_t)(row0 + tid) * qd + (size_t)h * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t v[32];
      tc::tmem_ld32(lane_base + O_COL + 32 * c, v);
      if (tid < nrows) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[8 * q + 0]) * inv, __uint_as_float(v[8 * q + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[8 * q + 2]) * inv, __uint_as_float(v[8 * q + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[8 * q + 4]) * inv, __uint_as_float(v[8 * q + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[8 * q + 6]) * inv, __uint_as_float(v[8 * q + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + 32 * c + 8 * q) = w;
        }
      }
    }
  }
  // after a wait that gave up, the MMAs it waited for get one more bounded wait before
  // their TMEM is freed
  if (!ok && tid == 0) tc::mbar_wait_bounded(bar, phase ^ 1, p.error, kSpin);
  tc::fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace

bool prefill_attention_tc_supported(const Geometry& g) { return g.dim == D; }

cudaError_t launch_prefill_attention_tc(cudaStream_t s, const PrefillAttnParams& p) {
  if (p.C < 1 || p.pos0 < 0 || p.g.dim != D || !p.error) return cudaErrorInvalidValue;
  const void* fn = (const void*)prefill_attn_tc_kernel;
  static int set_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (set_dev != dev) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    set_dev = dev;
  }
  PrefillAttnParams copy = p;
  void* args[] = {&copy};
  const dim3 grid((p.C + QROWS - 1) / QROWS, p.g.heads);
  return launch_with(s, false, grid, dim3(THREADS), SMEM_BYTES, fn, args);
}

}  // namespace y2
