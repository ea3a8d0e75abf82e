// bf16 GEMM on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for the
// prefill chunks: Y[C, N] = X[C, K] . W[N, K]^T, f32 accumulation, bf16 output rounded to
// nearest even (Linear::finish's rounding, src/tensor.rs:1102-1118).
//
// A persistent grid (one CTA per SM) walks 128 x 256 output tiles (128 rows of X, 256 rows
// of W), with two TMEM accumulators so that the epilogue of one tile overlaps the MMAs of
// the next: 10 warps.
//   warp 0       TMA producer: 64-column K blocks of X and W (128B-swizzled) into a
//                4-stage shared-memory ring, completion counted on the stage's mbarrier
//   warp 1       allocates all 512 TMEM columns (two accumulators); one lane issues
//                tcgen05.mma (M 128, N 256, K 16; four per K block), and tcgen05.commit
//                frees each stage and signals each finished accumulator
//   warps 2-9    epilogue, two warps per TMEM lane quarter (each half of the columns):
//                tcgen05.ld, bf16 rounding, stores; then each warp arrives on the
//                accumulator's "drained" barrier
// The SwiGLU form (gate|up of Mlp::apply, src/model.rs:206-214) takes the 256 B rows of a
// tile as 128 gate rows and the 128 up rows of the same outputs (W = [gate; up], up at row
// `inter`), and its epilogue writes h = bf16(bf16(silu(bf16 g)) * bf16 u) for 128 outputs,
// exactly the rounding of the unfused GEMM + swiglu kernel pair.
// Every mbarrier wait is bounded: after kSpin polls it sets *error and the CTA still
// reaches the final barrier, where warp 1 frees its TMEM.
#include <cuda.h>
#include <algorithm>
#include <cstdlib>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace y2 {
namespace {

constexpr int BM = 128, BK = 64, STAGES = 4, TMEM_COLS = 512;
constexpr int A_BYTES = BM * BK * 2;
// per tile width BN (rows of W): bytes of a W block and of a stage
template <int BN> __host__ __device__ constexpr int b_bytes() { return BN * BK * 2; }
template <int BN> __host__ __device__ constexpr int stage_bytes() { return A_BYTES + b_bytes<BN>(); }
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, each taking half of the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr long kSpin = 1L << 22;

struct TcGemmArgs {
  uint16_t* Y;
  int ldy, C, N, K;
  int inter;  // SwiGLU form: row of W where the up rows start; N = outputs (= inter)
  int32_t* error;
};

using tc::mbar_init;
using tc::mbar_try_wait;
using tc::sdesc_sw128;
using tc::smem_u32;
using tc::tmem_ld32;
using tc::mbar_arrive_expect_tx;
// Bounded wait for the phase of the given parity; false (and *error set) when it gave up.
Y2_DEV bool mbar_wait(uint64_t* b, uint32_t parity, int32_t* error) {
  return tc::mbar_wait_bounded(b, parity, error, kSpin);
}

using tc::tma_load_2d;

// Instruction descriptor: dense, D f32, A and B bf16, both K-major, N = BN, M = BM.
template <int BN>
__host__ __device__ constexpr uint32_t idesc() {
  return tc::idesc_bf16(BM, BN);
}

template <int BN>
Y2_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  tc::mma_bf16(tmem_d, adesc, bdesc, idesc<BN>(), accumulate);
}
Y2_DEV void umma_commit(uint64_t* bar) { tc::commit(bar); }
Y2_DEV void tc_fence_before() { tc::fence_before(); }
Y2_DEV void tc_fence_after() { tc::fence_after(); }

// 32 bf16 outputs (packed in pairs) of one row: four 16-byte stores, or element stores at
// the ragged right edge of the matrix.
Y2_DEV void store32(uint16_t* dst, const uint32_t (&w)[16], int valid) {
  if (valid >= 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
  }
}

template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const TcGemmArgs p) {
  constexpr int NOUT = SWIGLU ? BN / 2 : BN;  // output columns per tile
  constexpr int B_BYTES = b_bytes<BN>(), STAGE_BYTES = stage_bytes<BN>();
  static_assert(BN % 32 == 0 && (NOUT / 2) % 32 == 0 && 2 * BN <= TMEM_COLS, "tile width");
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte aligned ring (the swizzle pattern and the descriptors assume it)
  unsigned char* ring = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* afull = empty + STAGES;  // [2] accumulator b complete (MMA -> epilogue)
  uint64_t* aempty = afull + 2;      // [2] accumulator b drained (epilogue warps -> MMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (p.C + BM - 1) / BM, tiles = mt * ((p.N + NOUT - 1) / NOUT);
  const int nk = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(afull + b, 1);
      mbar_init(aempty + b, EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // two accumulators of BN columns in all of TMEM (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // tiles t = blockIdx.x, + gridDim.x, ...: rows of X vary fastest, so the CTAs working at
  // the same time share W tiles
  if (warp == 0) {
    if (lane == 0) {  // producer
      bool ok = true;
      for (int t = blockIdx.x, it = 0; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t % mt) * BM, n0 = (t / mt) * NOUT;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !(ok = mbar_wait(empty + s, ((it / STAGES) - 1) & 1, p.error))) break;
          unsigned char* a = ring + s * STAGE_BYTES;
          mbar_arrive_expect_tx(full + s, STAGE_BYTES);
          tma_load_2d(a, &tmx, full + s, kb * BK, m0);
          if (SWIGLU) {  // gate rows n0.., then up rows inter + n0..
            tma_load_2d(a + A_BYTES, &tmw, full + s, kb * BK, n0);
            tma_load_2d(a + A_BYTES + B_BYTES / 2, &tmw, full + s, kb * BK, p.inter + n0);
          } else {
            tma_load_2d(a + A_BYTES, &tmw, full + s, kb * BK, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: tile lt accumulates into TMEM columns (lt & 1) * BN ..
      bool ok = true;
      for (int t = blockIdx.x, it = 0, lt = 0; t < tiles && ok; t += gridDim.x, ++lt) {
        const int b = lt & 1, use = lt >> 1;
        if (use > 0 && !(ok = mbar_wait(aempty + b, (use - 1) & 1, p.error))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!(ok = mbar_wait(full + s, (it / STAGES) & 1, p.error))) break;
          tc_fence_after();
          const uint32_t a = smem_u32(ring + s * STAGE_BYTES), bb = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // 16 columns = 32 bytes along the swizzled row
            umma_bf16<BN>(d, sdesc_sw128(a + 32 * k), sdesc_sw128(bb + 32 * k), (kb | k) != 0);
          umma_commit(empty + s);  // frees the stage once these MMAs have read it
        }
        umma_commit(afull + b);  // the tile's MMAs are complete (also after a give-up)
      }
    }
  } else {  // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31, columns of half (w - 2) / 4
    const int q = warp & 3, half = (warp - 2) >> 2;
    constexpr int NH = NOUT / 2;
    for (int t = blockIdx.x, lt = 0; t < tiles; t += gridDim.x, ++lt) {
      const int b = lt & 1, use = lt >> 1;
      if (!mbar_wait(afull + b, use & 1, p.error)) break;
      tc_fence_after();
      const int row = (t % mt) * BM + 32 * q + lane, n0 = (t / mt) * NOUT;
      const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN);
      for (int c0 = half * NH; c0 < (half + 1) * NH; c0 += 32) {
        uint32_t w[16];
        if constexpr (SWIGLU) {
          uint32_t g[32], u[32];
          tmem_ld32(tl + (uint32_t)c0, g);
          tmem_ld32(tl + (uint32_t)(NOUT + c0), u);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float h2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float gv = round_bf16(__uint_as_float(g[2 * i + e]));
              const float uv = round_bf16(__uint_as_float(u[2 * i + e]));
              const float act = round_bf16(gv / (1.0f + det_expf(-gv)));
              h2[e] = act * uv;
            }
            w[i] = pack_bf16x2(h2[0], h2[1]);
          }
        } else {
          uint32_t v[32];
          tmem_ld32(tl + (uint32_t)c0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
        }
        if (row < p.C && n0 + c0 < p.N) store32(p.Y + (size_t)row * p.ldy + n0 + c0, w, p.N - n0 - c0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(aempty + b)) : "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// The driver's tensor-map encoder, looked up through the runtime (the library does not link
// the driver, so that it loads on machines without one).
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2D tensor map of a row-major bf16 matrix [rows, cols] with row stride ld elements, boxes of
// 64 columns (128 bytes, 128-byte swizzle) x box_rows rows; out-of-range rows read as zero.
bool make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
  const auto encode = encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
constexpr int smem_bytes() {
  return STAGES * stage_bytes<BN>() + 1024 + 256;
}

// Sets the kernel's shared-memory limit once per device; returns the device's SM count.
template <int BN, bool SWIGLU>
cudaError_t set_smem_once(int& sms) {
  static int set_dev = -1, set_sms = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (set_dev != dev) {
    if ((e = cudaFuncSetAttribute((const void*)gemm_tc_kernel<BN, SWIGLU>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<BN>())) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&set_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return e;
    set_dev = dev;
  }
  sms = set_sms;
  return cudaSuccess;
}

template <int BN, bool SWIGLU>
cudaError_t launch_tile(cudaStream_t s, const CUtensorMap& mx, const void* W, int wrows, int K, const TcGemmArgs& a,
                        int tiles) {
  int sms = 0;
  cudaError_t e = set_smem_once<BN, SWIGLU>(sms);
  if (e != cudaSuccess) return e;
  CUtensorMap mw;
  if (!make_map(&mw, W, wrows, K, K, SWIGLU ? BN / 2 : BN)) return cudaErrorInvalidValue;
  CUtensorMap mxc = mx;
  TcGemmArgs ac = a;
  void* args[] = {&mxc, &mw, &ac};
  return launch_with(s, false, dim3(std::min(tiles, sms)), dim3(THREADS), smem_bytes<BN>(),
                     (const void*)gemm_tc_kernel<BN, SWIGLU>, args);
}

// The persistent grid's time in units of W rows: tiles per CTA x (tile width + a fixed
// per-tile cost worth 64 rows, fitted to the measured q|k|v, o, gate|up and down shapes).
int tile_cost(int C, int N, int BN, int sms) {
  const int tiles = ((N + BN - 1) / BN) * ((C + BM - 1) / BM);
  return ((tiles + sms - 1) / sms) * (BN + 64);
}

}  // namespace

bool make_tma_map_bf16(void* map, const void* base, int rows, int cols, int ld, int box_rows) {
  return make_map(static_cast<CUtensorMap*>(map), base, rows, cols, ld, box_rows);
}

bool gemm_tc_supported(int C, int N, int K, int ldx, int ldy, const void* X, const void* W, const void* Y) {
  return C >= 1 && N >= 1 && K >= BK && K % BK == 0 && ldx % 8 == 0 && ldy % 8 == 0 && ldx >= K && ldy >= N &&
         ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0 && ((uintptr_t)Y & 15) == 0;
}

cudaError_t launch_gemm_tc(cudaStream_t s, const uint16_t* W, int N, int K, const uint16_t* X, int ldx, uint16_t* Y,
                           int ldy, int C, int32_t* error) {
  if (!gemm_tc_supported(C, N, K, ldx, ldy, X, W, Y)) return cudaErrorInvalidValue;
  int sms = 0;
  cudaError_t e = set_smem_once<256, false>(sms);
  if (e != cudaSuccess) return e;
  CUtensorMap mx;
  if (!make_map(&mx, X, C, K, ldx, BM)) return cudaErrorInvalidValue;
  const TcGemmArgs a{Y, ldy, C, N, K, 0, error};
  // 256- or 192-row tiles, whichever costs less (ties to the wider tile; 128-row tiles were
  // slower on every measured shape); YUE2_CUDA_GEMM_BN=128|192|256 forces one
  int best = tile_cost(C, N, 192, sms) < tile_cost(C, N, 256, sms) ? 192 : 256;
  static const int forced = [] {
    const char* v = getenv("YUE2_CUDA_GEMM_BN");
    return v ? atoi(v) : 0;
  }();
  if (forced == 128 || forced == 192 || forced == 256) best = forced;
  const int tiles = ((N + best - 1) / best) * ((C + BM - 1) / BM);
  if (best == 128) return launch_tile<128, false>(s, mx, W, N, K, a, tiles);
  if (best == 192) return launch_tile<192, false>(s, mx, W, N, K, a, tiles);
  return launch_tile<256, false>(s, mx, W, N, K, a, tiles);
}

// h[C, I] = bf16(bf16(silu(bf16(X . Wg^T))) * bf16(X . Wu^T)) with Wgu = [Wg; Wu] ([2I, K]).
cudaError_t launch_gemm_tc_swiglu(cudaStream_t s, const uint16_t* Wgu, int I, int K, const uint16_t* X, int ldx,
                                  uint16_t* H, int ldh, int C, int32_t* error) {
  if (I % 128 || !gemm_tc_supported(C, I, K, ldx, ldh, X, Wgu, H)) return cudaErrorInvalidValue;
  CUtensorMap mx;
  if (!make_map(&mx, X, C, K, ldx, BM)) return cudaErrorInvalidValue;
  const TcGemmArgs a{H, ldh, C, I, K, I, error};
  return launch_tile<256, true>(s, mx, Wgu, 2 * I, K, a, (I / 128) * ((C + BM - 1) / BM));
}

}  // namespace y2
