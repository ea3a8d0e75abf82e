// yue2_attention_noalloc: single-query GQA decode attention that allocates no device
// memory.
//
// Who needs it: callers that run inside a host framework which owns every device
// allocation (a serving runtime with its own memory pool, an engine that forbids
// cudaMalloc/cudaFree after start-up because they synchronise the device, or real-time
// threads that may not block in the allocator). They pass their own device buffers for
// the query, the key/value rows and the output; the split-K partial results and merge
// counters live in a fixed array of this library instead of in a workspace.
//
// The scratch is a file-scope __device__ array of kScratchBytes, present on every GPU that
// loads the library until the process exits. Host code never uses its name as an address:
// the first call on a device (with that device current) resolves the device address with
// cudaGetSymbolAddress and keeps it; make that first call before any stream capture. Every
// call shares the one array, so calls whose kernels overlap on the GPU race with each
// other; the merge counters are cleared at the start of every call.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "../../include/yue2_cuda.h"
#include "common.cuh"
#include "engine.h"
#include "kernels.h"

namespace {

using namespace y2;

constexpr size_t kScratchBytes = 2u << 20;  // 2 MiB: partials for heads * splits * (dim + 2) floats
constexpr int kMaxSplits = 32;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Same split-K flash decoding as the paged kernel, over row-major [keys, kv*dim] bf16
// keys and values that the caller owns.
template <int D, int G>
__global__ void __launch_bounds__(128) attn_rows_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                        const uint16_t* __restrict__ v, uint16_t* __restrict__ out,
                                                        int keys, int heads, int kvh, int splits, float scale,
                                                        float* part, int32_t* counters) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int CPR = D / 8;
  constexpr int DL = D / 32;
  constexpr int NW = 4;
  uint16_t* ktile = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* vtile = ktile + NW * 32 * D;
  float* qs = reinterpret_cast<float*>(vtile + NW * 32 * D);
  float* ps = qs + G * D;
  float* wm = ps + NW * G * 32;
  float* wl = wm + NW * G;
  __shared__ int s_ticket;

  const int split = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (keys + 31) >> 5;
  const int tps = (ntiles + splits - 1) / splits;
  const int nsplit = (ntiles + tps - 1) / tps;
  if (split >= nsplit) return;
  const int t0 = split * tps, t1 = min(ntiles, t0 + tps);
  const size_t stride = (size_t)kvh * D;

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) qs[i] = bf2f(q[(size_t)g * G * D + i]);
  __syncthreads();

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[h][e] = 0.f;
  }
  uint16_t* kt = ktile + warp * 32 * D;
  uint16_t* vt = vtile + warp * 32 * D;
  float* pw = ps + warp * G * 32;

  for (int t = t0 + warp; t < t1; t += NW) {
    const int key0 = t << 5;
    const int nk = min(32, keys - key0);
    const uint16_t* kb = k + (size_t)key0 * stride + (size_t)g * D;
    const uint16_t* vb = v + (size_t)key0 * stride + (size_t)g * D;
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int j = i / CPR, c = i % CPR;
      if (j < nk) {
        cp_async16(kt + (size_t)(j * CPR + (c ^ (j & 7))) * 8, kb + (size_t)j * stride + c * 8);
        cp_async16(vt + (size_t)i * 8, vb + (size_t)j * stride + c * 8);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.f;
    if (lane < nk) {
#pragma unroll 4
      for (int c = 0; c < CPR; ++c) {
        const uint4 kv = *reinterpret_cast<const uint4*>(kt + (size_t)(lane * CPR + (c ^ (lane & 7))) * 8);
        const float k0 = bf_lo(kv.x), k1 = bf_hi(kv.x), k2 = bf_lo(kv.y), k3 = bf_hi(kv.y);
        const float k4 = bf_lo(kv.z), k5 = bf_hi(kv.z), k6 = bf_lo(kv.w), k7 = bf_hi(kv.w);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + h * D + c * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qs + h * D + c * 8 + 4);
          float s = sc[h];
          s = fmaf(qa.x, k0, s);
          s = fmaf(qa.y, k1, s);
          s = fmaf(qa.z, k2, s);
          s = fmaf(qa.w, k3, s);
          s = fmaf(qb.x, k4, s);
          s = fmaf(qb.y, k5, s);
          s = fmaf(qb.z, k6, s);
          s = fmaf(qb.w, k7, s);
          sc[h] = s;
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float s = lane < nk ? sc[h] * scale : -INFINITY;
      const float mnew = fmaxf(m[h], warp_max(s));
      const float alpha = m[h] == -INFINITY ? 0.f : __expf(m[h] - mnew);
      const float pv = lane < nk ? __expf(s - mnew) : 0.f;
      l[h] = l[h] * alpha + warp_sum(pv);
      m[h] = mnew;
      pw[h * 32 + lane] = pv;
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[h][e] *= alpha;
    }
    __syncwarp();
    for (int j = 0; j < nk; ++j) {
      const uint16_t* vr = vt + (size_t)j * D + lane * DL;
      float vv[DL];
#pragma unroll
      for (int e = 0; e < DL; e += 2) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(vr + e);
        vv[e] = bf_lo(w);
        vv[e + 1] = bf_hi(w);
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pj = pw[h * 32 + j];
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[h][e] = fmaf(pj, vv[e], acc[h][e]);
      }
    }
    __syncwarp();
  }

  __syncthreads();
  float* wacc = reinterpret_cast<float*>(smem_raw);
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < G; ++h) {
      wm[warp * G + h] = m[h];
      wl[warp * G + h] = l[h];
    }
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int e = 0; e < DL; ++e) wacc[((size_t)warp * G + h) * D + lane * DL + e] = acc[h][e];
  __syncthreads();

  float* pg = part + (size_t)g * splits * G * (D + 2);
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w * G + h]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float mw = wm[w * G + h];
      if (mw == -INFINITY) continue;
      const float f = __expf(mw - M);
      L = fmaf(wl[w * G + h], f, L);
      O = fmaf(wacc[((size_t)w * G + h) * D + d], f, O);
    }
    if (nsplit == 1) {
      out[(size_t)(g * G + h) * D + d] = f2bf_round(O / L);
    } else {
      float* ph = pg + ((size_t)split * G + h) * (D + 2);
      if (d == 0) {
        ph[0] = M;
        ph[1] = L;
      }
      ph[2 + d] = O;
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_ticket = atomicAdd(counters + g, 1);
  __syncthreads();
  if (s_ticket != nsplit - 1) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(pg + ((size_t)s * G + h) * (D + 2)));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float* ph = pg + ((size_t)s * G + h) * (D + 2);
      const float f = __expf(__ldcg(ph) - M);
      L = fmaf(__ldcg(ph + 1), f, L);
      O = fmaf(__ldcg(ph + 2 + d), f, O);
    }
    out[(size_t)(g * G + h) * D + d] = f2bf_round(O / L);
  }
  if (threadIdx.x == 0) counters[g] = 0;
}

template <int D, int G>
const void* pick() {
  return (const void*)attn_rows_kernel<D, G>;
}

const void* kernel_for(int dim, int groups) {
#define Y2_PICK(DD)                    \
  switch (groups) {                    \
    case 1: return pick<DD, 1>();      \
    case 2: return pick<DD, 2>();      \
    case 3: return pick<DD, 3>();      \
    case 4: return pick<DD, 4>();      \
    case 8: return pick<DD, 8>();      \
  }                                    \
  return nullptr;
  switch (dim) {
    case 64: Y2_PICK(64)
    case 128: Y2_PICK(128)
    case 256: Y2_PICK(256)
  }
#undef Y2_PICK
  return nullptr;
}

struct DeviceSetup {
  bool done = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};

std::mutex g_mu;
DeviceSetup g_setup[kMaxDevices];

// Once per device, with that device current: resolve the scratch address and configure
// every kernel instantiation's shared-memory limit. Allocates nothing.
int setup_device(int dev, DeviceSetup*& out) {
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSetup& s = g_setup[dev];
  if (!s.done) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    for (int dim : {64, 128, 256})
      for (int grp : {1, 2, 3, 4, 8}) {
        e = cudaFuncSetAttribute(kernel_for(dim, grp), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attention_smem_bytes(dim, grp));
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
      }
    s.scratch = static_cast<unsigned char*>(ptr);
    s.sms = sms;
    s.done = true;
  }
  out = &s;
  return 0;
}

}  // namespace

extern "C" int yue2_attention_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                                      uint64_t keys, uint64_t heads, uint64_t kv, uint64_t dim, void* stream) {
  if (!q || !k || !v || !out) return fail(YUE2_ERR_INVALID, "null device pointer");
  if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15)
    return fail(YUE2_ERR_INVALID, "q, k, v and out must be 16-byte aligned device pointers");
  // bounds before any arithmetic on the caller's sizes: kv is the grid's y extent (at most
  // 65,535), and heads must fit the kernel's int arguments
  if (keys == 0 || keys > (1u << 30) || heads == 0 || kv == 0 || kv > 65535 || heads > (uint64_t)INT32_MAX ||
      heads % kv)
    return fail(YUE2_ERR_INVALID, "invalid attention shape");
  if (dim != 64 && dim != 128 && dim != 256) return fail(YUE2_ERR_INVALID, "head dim must be 64, 128 or 256");
  const uint64_t groups = heads / kv;
  if (groups != 1 && groups != 2 && groups != 3 && groups != 4 && groups != 8)
    return fail(YUE2_ERR_INVALID, "unsupported grouped-query factor");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(YUE2_ERR_INVALID, "device index out of range");
  DeviceSetup* s = nullptr;
  int rc = setup_device(dev, s);
  if (rc) return rc;
  const int splits = (int)std::max<uint64_t>(1, std::min<uint64_t>(kMaxSplits, (2 * (uint64_t)s->sms + kv - 1) / kv));
  const size_t counter_bytes = ((kv * 4 + 255) / 256) * 256;
  const size_t part_bytes = (size_t)heads * splits * (dim + 2) * 4;
  if (counter_bytes + part_bytes > kScratchBytes)
    return fail(YUE2_ERR_INVALID, "heads * (dim + 2) * " + std::to_string(splits) + " splits * 4 B of partials exceed the " +
                                      std::to_string(kScratchBytes) + "-byte static scratch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* counters = reinterpret_cast<int32_t*>(s->scratch);
  float* part = reinterpret_cast<float*>(s->scratch + counter_bytes);
  e = cudaMemsetAsync(counters, 0, kv * 4, st);
  if (e != cudaSuccess) return cuda_fail(e, "clearing the merge counters");
  const void* fn = kernel_for((int)dim, (int)groups);
  int keys_i = (int)keys, heads_i = (int)heads, kv_i = (int)kv, splits_i = splits;
  float scale = 1.0f / sqrtf((float)dim);
  void* args[] = {(void*)&q, (void*)&k, (void*)&v, (void*)&out, &keys_i, &heads_i, &kv_i,
                  &splits_i, &scale, &part, &counters};
  e = cudaLaunchKernel(fn, dim3(splits, (unsigned)kv), dim3(128), args, attention_smem_bytes((int)dim, (int)groups),
                       st);
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return 0;
}
