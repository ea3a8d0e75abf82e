// Decode attention and the QK norm + RoPE of one head, used by the decode attention kernels
// (kernels_layer.cu) and the no-alloc entry point (noalloc.cu).
#pragma once
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace y2 {

// Norm::heads (tensor.rs:1158-1172) then Rotary::apply (model.rs:151-168) of one head
// by one warp: src is the head's bf16 projection, v a warp-private [D] f32 buffer that
// receives the rotated, bf16-valued head.
template <int D>
Y2_DEV void norm_rope_head(const uint16_t* src, const float* gamma, float eps, const float* ct, const float* st,
                           float* v) {
  constexpr int DL = D / 32, HALF = D / 2;
  const int lane = threadIdx.x & 31;
  float x[DL];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < DL; ++e) {
    x[e] = bf2f(__ldcg(src + lane * DL + e));  // L2: src may come from another SM in this kernel
    ss = fmaf(x[e], x[e], ss);
  }
  ss = warp_sum(ss);
  const float scale = round_bf16(1.0f / sqrtf(ss / (float)D + eps));
#pragma unroll
  for (int e = 0; e < DL; ++e) v[lane * DL + e] = round_bf16(round_bf16(x[e] * scale) * gamma[lane * DL + e]);
  __syncwarp();
  for (int i = lane; i < HALF; i += 32) {
    const float a = v[i], b = v[i + HALF], c = ct[i], s = st[i];
    v[i] = round_bf16(round_bf16(a * c) - round_bf16(b * s));
    v[i + HALF] = round_bf16(round_bf16(b * c) + round_bf16(a * s));
  }
  __syncwarp();
}

// Split-K flash decoding. CTA (split, kv head, row) owns a contiguous range of 32-key
// tiles of the row's cache; each warp stages a tile of K (XOR-swizzled, conflict-free
// for lane-per-key reads) and V into shared memory with cp.async, computes the G
// grouped heads' scores with one key per lane, updates an online softmax, and
// accumulates P.V with lanes over head dims. Warps merge in shared memory; splits
// merge through f32 partials, and the last split CTA to finish (atomic ticket; no
// waiting) normalises and writes the bf16 output.
// 128-thread barrier of the attention CTA.
Y2_DEV void attn_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// One (split, kv head, row) item of split-K decode attention: one CTA of four warps, a
// programmatic dependent launch (the first tile requested before the wait), splits merged by
// the last CTA through an atomic ticket. PIPE (passes of many rows, each CTA streaming
// many tiles per warp): two K buffers per warp; the next tile's K is requested before the
// current tile's scores and its V right after the current P.V, so loads overlap compute.
// MMA (implies PIPE; G <= 8, D <= 128): scores and P.V on the tensor cores. The G query
// heads are the rows of one m16n8k16 A tile (bf16; q is already bf16-exact), a 32-key K
// tile gives four n-tiles, and P.V multiplies P split into bf16 hi + lo parts so that the
// probabilities keep f32 accuracy. V rows past the last key are zero-filled.
template <int D, int G, bool PIPE = false, bool MMA = false>
Y2_DEV void attn_item(const AttnParams& a, int split, int g, int r, unsigned char* smem_raw) {
  static_assert(!MMA || (PIPE && G <= 8 && D <= 128), "tensor-core attention shape");
  constexpr int CPR = D / 8;  // 16-byte chunks per key row
  constexpr int DL = D / 32;  // dims per lane
  constexpr int NW = 4;
  constexpr int KB = PIPE ? 2 : 1;  // K tile buffers per warp
  uint16_t* ktile = reinterpret_cast<uint16_t*>(smem_raw);           // [NW][KB][32][D]
  uint16_t* vtile = ktile + NW * KB * 32 * D;                          // [NW][32][D]
  float* qs = reinterpret_cast<float*>(vtile + NW * 32 * D);           // [G][D]
  float* ps = qs + G * D;                                              // [NW][G][32]
  float* wm = ps + NW * G * 32;                                        // [NW][G]
  float* wl = wm + NW * G;                                             // [NW][G]
  float* wbuf_all = wl + NW * G;                                       // [NW][D] norm/rope scratch
  float* gq = wbuf_all + NW * D;                                       // [D] q norm gains (fused)
  float* gk = gq + D;                                                  // [D] k norm gains
  float* cs = gk + D;                                                  // [D / 2] cos, [D / 2] sin at pos
  __shared__ int s_ticket;

  // Row descriptors are final once the preceding kernel has passed its own wait (it
  // triggers this launch only then), and cache rows below the new position were written
  // by earlier steps: read both, and start streaming the first tile, before the wait.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DevRow row = a.rows[r];
  if (!row.active) return;
  const Geometry& geo = a.g;
  const int keys = row.pos + 1;
  const int ntiles = (keys + 31) >> 5;
  // at least one tile per warp: short caches use fewer splits (the rest exit at once)
  const int tps = max(NW, (ntiles + a.splits - 1) / a.splits);
  const int nsplit = (ntiles + tps - 1) / tps;
  if (split >= nsplit) return;
  const int t0 = split * tps, t1 = min(ntiles, t0 + tps);
  uint16_t* kt = ktile + warp * KB * 32 * D;
  uint16_t* vt = vtile + warp * 32 * D;
  const size_t koff = kv_offset(geo, a.layer, 0, g), voff = kv_offset(geo, a.layer, 1, g);
  auto stage = [&](int t) {  // cp.async one 32-key tile of K (swizzled) and V
    const int key0 = t << 5;
    const int nk = min(32, keys - key0);
    const uint16_t* page = reinterpret_cast<const uint16_t*>(row.pages[key0 >> kPageLog2]);
    const uint16_t* kb = page + koff + (size_t)(key0 & (kPageTokens - 1)) * D;
    const uint16_t* vb = page + voff + (size_t)(key0 & (kPageTokens - 1)) * D;
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int j = i / CPR, c = i % CPR;
      if (j < nk) {
        cp_async16(kt + (size_t)(j * CPR + (c ^ (j & 7))) * 8, kb + (size_t)j * D + c * 8);
        cp_async16(vt + (size_t)i * 8, vb + (size_t)j * D + c * 8);
      }
    }
    cp_async_commit();
  };
  // the tile holding the new position is written in this launch (fused) or by the
  // preceding kernel (prefill rows): it is never fetched before the wait
  const int first_tile = t0 + warp;
  const bool early = a.fused && first_tile < t1 && first_tile != ntiles - 1;
  // PIPE: K (swizzled) of tile t into buffer buf, V of tile t; one commit group each. The
  // page base comes from the caller (fetched a tile ahead, off the issue path).
  auto page_of = [&](int t) { return reinterpret_cast<const uint16_t*>(row.pages[(t << 5) >> kPageLog2]); };
  auto stage_k = [&](int t, int buf, const uint16_t* page) {
    const int key0 = t << 5;
    const int nk = min(32, keys - key0);
    const uint16_t* kb = page + koff + (size_t)(key0 & (kPageTokens - 1)) * D;
    uint16_t* dst = kt + (size_t)buf * 32 * D;
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int j = i / CPR, c = i % CPR;
      if (j < nk) cp_async16(dst + (size_t)(j * CPR + (c ^ (j & 7))) * 8, kb + (size_t)j * D + c * 8);
    }
    cp_async_commit();
  };
  auto stage_v = [&](int t, const uint16_t* page) {
    const int key0 = t << 5;
    const int nk = min(32, keys - key0);
    const uint16_t* vb = page + voff + (size_t)(key0 & (kPageTokens - 1)) * D;
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int j = i / CPR, c = i % CPR;
      if constexpr (MMA) {  // swizzled for ldmatrix.trans; rows past the last key zeroed
        cp_async16_zfill(vt + (size_t)(j * CPR + (c ^ (j & 7))) * 8, vb + (size_t)(j < nk ? j : 0) * D + c * 8, j < nk);
      } else if (j < nk) {
        cp_async16(vt + (size_t)i * 8, vb + (size_t)j * D + c * 8);
      }
    }
    cp_async_commit();
  };
  if (early) {
    if constexpr (PIPE) {
      const uint16_t* p0 = page_of(first_tile);
      stage_k(first_tile, 0, p0);
      stage_v(first_tile, p0);
    } else {
      stage(first_tile);
    }
  }

  // fused rows: the norm gains and the RoPE row of the new position do not depend on the
  // preceding kernel, so they are staged now and the QK norm after the wait waits on q alone
  if (a.fused && row.pos >= 0 && row.pos < a.max_pos)
    for (int i = threadIdx.x; i < D; i += 128) {
      gq[i] = a.q_norm[i];
      gk[i] = a.k_norm[i];
      cs[i] = i < D / 2 ? a.cos_tab[(size_t)row.pos * (D / 2) + i] : a.sin_tab[(size_t)row.pos * (D / 2) + i - D / 2];
    }
  attn_sync();

  pdl_wait();
  pdl_trigger();

  if (a.fused) {
    const int pos = row.pos;
    if (pos < 0 || pos >= a.max_pos) {
      if (threadIdx.x == 0) atomicExch(a.error, 1);
      cp_async_wait<0>();
      return;
    }
    const int width = (geo.heads + 2 * geo.kvh) * D;
    const uint16_t* src = a.qkv + (size_t)r * width;
    const float* ct = cs;
    const float* st = cs + D / 2;
    float* wbuf = wbuf_all + warp * D;
    for (int h = warp; h < G; h += 4) {
      norm_rope_head<D>(src + (size_t)(g * G + h) * D, gq, geo.eps, ct, st, wbuf);
      for (int i = lane; i < D; i += 32) qs[h * D + i] = wbuf[i];
      __syncwarp();
    }
    if (split == nsplit - 1) {  // this CTA's last tile holds `pos`: write its K and V first
      uint16_t* page = reinterpret_cast<uint16_t*>(row.pages[pos >> kPageLog2]);
      const size_t slot = (size_t)(pos & (kPageTokens - 1)) * D;
      if (warp == 0) {
        norm_rope_head<D>(src + (size_t)(geo.heads + g) * D, gk, geo.eps, ct, st, wbuf);
        uint16_t* dst = page + kv_offset(geo, a.layer, 0, g) + slot;
        for (int i = lane; i < D; i += 32) dst[i] = f2bf_exact(wbuf[i]);
      } else if (warp == 1) {
        const uint16_t* vs = src + (size_t)(geo.heads + geo.kvh + g) * D;
        uint16_t* dst = page + kv_offset(geo, a.layer, 1, g) + slot;
        for (int i = lane; i < D; i += 32) dst[i] = __ldcg(vs + i);
      }
      __threadfence();
    }
  } else {
    const uint16_t* qsrc = a.q + (size_t)r * geo.heads * D + (size_t)g * G * D;
    for (int i = threadIdx.x; i < G * D; i += 128) qs[i] = bf2f(qsrc[i]);
  }
  attn_sync();

  float* wacc = reinterpret_cast<float*>(smem_raw);  // [NW][G][D] f32 after the loops
  if constexpr (MMA) {
    constexpr int KS = D / 16, NT = D / 8;
    auto sw = [](int rr, int c) { return (uint32_t)(rr * D * 2 + ((c ^ (rr & 7)) << 4)); };
    unsigned char* qsb = reinterpret_cast<unsigned char*>(cs + D);  // [16][D] bf16
    for (int i = threadIdx.x; i < 16 * CPR; i += 128) {
      const int rr = i / CPR, c = i % CPR;
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (rr < G) {
        const float* src = qs + rr * D + c * 8;
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = pack_bf16x2(src[2 * k], src[2 * k + 1]);
      }
      *reinterpret_cast<uint4*>(qsb + sw(rr, c)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    attn_sync();
    const int g8 = lane >> 2, t4 = lane & 3;
    uint32_t qf[KS][2];  // A fragments a0, a2 (head rows 0-7); rows 8-15 are zero
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t tq[4];
      const int mi = lane >> 3, rr = (mi & 1) * 8 + (lane & 7);
      ldsm_x4(tq, qsb + sw(rr, 2 * kk + (mi >> 1)));
      qf[kk][0] = tq[0];
      qf[kk][1] = tq[2];
    }
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float mrow = -INFINITY, lrow = 0.f;  // head g8
    if (first_tile < t1 && !early) {
      const uint16_t* p0 = page_of(first_tile);
      stage_k(first_tile, 0, p0);
      stage_v(first_tile, p0);
    }
    const uint16_t* pnext = first_tile + NW < t1 ? page_of(first_tile + NW) : nullptr;
    for (int t = first_tile, it = 0; t < t1; t += NW, ++it) {
      const int nk = min(32, keys - (t << 5));
      const unsigned char* kb = reinterpret_cast<const unsigned char*>(kt + (size_t)(it & 1) * 32 * D);
      const unsigned char* vb = reinterpret_cast<const unsigned char*>(vt);
      if (t + NW < t1) stage_k(t + NW, (it + 1) & 1, pnext);
      else cp_async_commit();
      const uint16_t* pafter = t + 2 * NW < t1 ? page_of(t + 2 * NW) : nullptr;  // in flight meanwhile
      cp_async_wait<2>();
      __syncwarp();
      float s[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; kk += 2) {
          uint32_t b[4];
          ldsm_x4(b, kb + sw(8 * j + (lane & 7), 2 * kk + (lane >> 3)));
          mma_bf16_16816(s[j], qf[kk][0], 0u, qf[kk][1], 0u, b[0], b[1]);
          mma_bf16_16816(s[j], qf[kk + 1][0], 0u, qf[kk + 1][1], 0u, b[2], b[3]);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = 8 * j + 2 * t4 + e < nk ? s[j][e] * a.scale : -INFINITY;
          s[j][e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(mrow, mx);  // key 0 of the tile is always valid: finite
      const float al = mrow == -INFINITY ? 0.f : __expf(mrow - mn);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = __expf(s[j][e] - mn);
          s[j][e] = p;
          sum += p;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow = lrow * al + sum;
      mrow = mn;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        o[j][0] *= al;
        o[j][1] *= al;
      }
      cp_async_wait<1>();  // V(t); K of the next tile may stay in flight
      __syncwarp();
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint32_t h0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        const uint32_t h2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        const uint32_t l0 = pack_bf16x2(s[2 * kk][0] - bf_lo(h0), s[2 * kk][1] - bf_hi(h0));
        const uint32_t l2 = pack_bf16x2(s[2 * kk + 1][0] - bf_lo(h2), s[2 * kk + 1][1] - bf_hi(h2));
#pragma unroll
        for (int jd = 0; jd < NT; jd += 2) {
          uint32_t b[4];
          const int mi = lane >> 3;
          ldsm_x4_trans(b, vb + sw(16 * kk + (mi & 1) * 8 + (lane & 7), jd + (mi >> 1)));
          mma_bf16_16816(o[jd], h0, 0u, h2, 0u, b[0], b[1]);
          mma_bf16_16816(o[jd], l0, 0u, l2, 0u, b[0], b[1]);
          mma_bf16_16816(o[jd + 1], h0, 0u, h2, 0u, b[2], b[3]);
          mma_bf16_16816(o[jd + 1], l0, 0u, l2, 0u, b[2], b[3]);
        }
      }
      __syncwarp();
      if (t + NW < t1) stage_v(t + NW, pnext);
      else cp_async_commit();
      pnext = pafter;
    }
    cp_async_wait<0>();
    // ---- merge the warps of this CTA (tiles reused as [NW][G][D] f32 accumulators)
    attn_sync();
    if (g8 < G) {
      if (t4 == 0) {
        wm[warp * G + g8] = mrow;
        wl[warp * G + g8] = lrow;
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        wacc[((size_t)warp * G + g8) * D + 8 * j + 2 * t4] = o[j][0];
        wacc[((size_t)warp * G + g8) * D + 8 * j + 2 * t4 + 1] = o[j][1];
      }
    }
  } else {
    float m[G], l[G], acc[G][DL];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m[h] = -INFINITY;
      l[h] = 0.f;
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[h][e] = 0.f;
    }
    float* pw = ps + warp * G * 32;

    const uint16_t* pnext = nullptr;
    if constexpr (PIPE) {
      if (first_tile < t1 && !early) {
        const uint16_t* p0 = page_of(first_tile);
        stage_k(first_tile, 0, p0);
        stage_v(first_tile, p0);
      }
      pnext = first_tile + NW < t1 ? page_of(first_tile + NW) : nullptr;
    }
    for (int t = t0 + warp, it = 0; t < t1; t += NW, ++it) {
      const int key0 = t << 5;
      const int nk = min(32, keys - key0);
      const uint16_t* kcur = kt + (PIPE ? (size_t)(it & 1) * 32 * D : 0);
      const uint16_t* pafter = nullptr;
      if constexpr (PIPE) {
        if (t + NW < t1) stage_k(t + NW, (it + 1) & 1, pnext);
        else cp_async_commit();  // keeps the group count: K(t) is third from the end
        pafter = t + 2 * NW < t1 ? page_of(t + 2 * NW) : nullptr;
        cp_async_wait<2>();
      } else {
        if (!(early && t == first_tile)) stage(t);
        cp_async_wait<0>();
      }
      __syncwarp();

      float sc[G];
#pragma unroll
      for (int h = 0; h < G; ++h) sc[h] = 0.f;
      if (lane < nk) {
#pragma unroll 4
        for (int c = 0; c < CPR; ++c) {
          const uint4 kv = *reinterpret_cast<const uint4*>(kcur + (size_t)(lane * CPR + (c ^ (lane & 7))) * 8);
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
        const float s = lane < nk ? sc[h] * a.scale : -INFINITY;
        const float mnew = fmaxf(m[h], warp_max(s));
        const float alpha = m[h] == -INFINITY ? 0.f : __expf(m[h] - mnew);
        const float pv = lane < nk ? __expf(s - mnew) : 0.f;
        l[h] = l[h] * alpha + warp_sum(pv);
        m[h] = mnew;
        pw[h * 32 + lane] = pv;
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[h][e] *= alpha;
      }
      if constexpr (PIPE) cp_async_wait<1>();  // V(t); K of the next tile may stay in flight
      __syncwarp();
      for (int j = 0; j < nk; ++j) {
        const uint16_t* vr = vt + (size_t)j * D + lane * DL;
        float vv[DL];
        if constexpr (DL == 2) {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(vr);
          vv[0] = bf_lo(w);
          vv[1] = bf_hi(w);
        } else if constexpr (DL == 4) {
          const uint2 w = *reinterpret_cast<const uint2*>(vr);
          vv[0] = bf_lo(w.x);
          vv[1] = bf_hi(w.x);
          vv[2] = bf_lo(w.y);
          vv[3] = bf_hi(w.y);
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(vr);
          vv[0] = bf_lo(w.x);
          vv[1] = bf_hi(w.x);
          vv[2] = bf_lo(w.y);
          vv[3] = bf_hi(w.y);
          vv[4] = bf_lo(w.z);
          vv[5] = bf_hi(w.z);
          vv[6] = bf_lo(w.w);
          vv[7] = bf_hi(w.w);
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pj = pw[h * 32 + j];
#pragma unroll
          for (int e = 0; e < DL; ++e) acc[h][e] = fmaf(pj, vv[e], acc[h][e]);
        }
      }
      __syncwarp();
      if constexpr (PIPE) {
        if (t + NW < t1) stage_v(t + NW, pnext);
        else cp_async_commit();
        pnext = pafter;
      }
    }
    if constexpr (PIPE) cp_async_wait<0>();

    // ---- merge the warps of this CTA (tiles reused as [NW][G][D] f32 accumulators)
    attn_sync();
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
  }
  attn_sync();

  const int outw = geo.heads * D;
  float* part = a.part + ((size_t)(r * geo.kvh + g) * a.splits) * G * (D + 2);
  for (int i = threadIdx.x; i < G * D; i += 128) {
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
      a.out[(size_t)r * outw + (size_t)(g * G + h) * D + d] = f2bf_round(O / L);
    } else {
      float* ph = part + ((size_t)split * G + h) * (D + 2);
      if (d == 0) {
        ph[0] = M;
        ph[1] = L;
      }
      ph[2 + d] = O;
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  attn_sync();
  if (threadIdx.x == 0) s_ticket = atomicAdd(a.counters + r * geo.kvh + g, 1);
  attn_sync();
  if (s_ticket != nsplit - 1) return;
  __threadfence();
  // split maxima and sums of every head in one round trip, then each thread's outputs
  float* sm_ml = wacc;  // [G][nsplit][2] (the warp accumulators are no longer needed)
  for (int i = threadIdx.x; i < G * nsplit; i += 128) {
    const int h = i / nsplit, sp = i % nsplit;
    const float* ph = part + ((size_t)sp * G + h) * (D + 2);
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(ph));
    sm_ml[2 * i] = ml.x;
    sm_ml[2 * i + 1] = ml.y;
  }
  attn_sync();
  for (int i = threadIdx.x; i < G * D; i += 128) {
    const int h = i / D, d = i % D;
    const float* mlh = sm_ml + 2 * h * nsplit;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, mlh[2 * sp]);
    float L = 0.f, O = 0.f;
    constexpr int kB = 8;  // partial outputs requested together
    for (int s0 = 0; s0 < nsplit; s0 += kB) {
      float o[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b)
        o[b] = s0 + b < nsplit ? __ldcg(part + ((size_t)(s0 + b) * G + h) * (D + 2) + 2 + d) : 0.f;
#pragma unroll
      for (int b = 0; b < kB; ++b)
        if (s0 + b < nsplit) {
          const float f = __expf(mlh[2 * (s0 + b)] - M);
          L = fmaf(mlh[2 * (s0 + b) + 1], f, L);
          O = fmaf(o[b], f, O);
        }
    }
    a.out[(size_t)r * outw + (size_t)(g * G + h) * D + d] = f2bf_round(O / L);
  }
  if (threadIdx.x == 0) a.counters[r * geo.kvh + g] = 0;
}

// ---- Cluster form for short decode contexts (fused decode rows, D <= 128). The CS CTAs of
// one (kv head, row) form a thread-block cluster; CTA rank c owns the 32-key tiles
// [c * TPC, min(ntiles, (c + 1) * TPC)), TPC = ceil(ntiles / CS), warp w the tiles w, w + 8,
// ... of them. Each warp's first tile is requested before griddepcontrol.wait; a later
// tile's K streams in during the previous tile's P.V and its V during its own scores. The
// tile holding the new position is fetched without that key: the CTA that computes the new K and V
// (QK norm, RoPE) appends them to the cache and also writes them into its shared-memory
// tile, so nothing in the launch reads them back from memory. Warps merge in shared memory,
// then, after a cluster barrier, CTA c merges outputs [c * G * D / CS, ...) of the CS
// partials through distributed shared memory, in rank order. No global partials, fence or
// ticket; a second cluster barrier keeps the partials readable until every CTA is done.
template <int D, int G>
__host__ __device__ constexpr int attn_cluster_smem() {
  return 2 * kClusterWarps * 32 * D * 2       // K and V tiles [NW][32][D] bf16
         + G * D * 4                          // rotated q heads
         + kClusterWarps * G * 32 * 4         // probabilities [NW][G][32]
         + 2 * kClusterWarps * G * 4          // warp maxima and sums
         + kClusterWarps * D * 4              // norm/rope scratch per warp
         + 2 * D * 4                          // the new position's K and V
         + G * (D + 2) * 4                    // this CTA's partial (read by the cluster)
         + 3 * D * 4;                         // q and k norm gains, the position's cos | sin
}

template <int D, int G>
Y2_DEV void attn_cluster_item(const AttnParams& a, unsigned char* smem_raw) {
  static_assert(D <= 128 && G <= kClusterWarps, "cluster attention shape");
  constexpr int NW = kClusterWarps, CPR = D / 8, DL = D / 32;
  uint16_t* ktile = reinterpret_cast<uint16_t*>(smem_raw);  // [NW][32][D] (XOR-swizzled rows)
  uint16_t* vtile = ktile + NW * 32 * D;                      // [NW][32][D]
  float* qs = reinterpret_cast<float*>(vtile + NW * 32 * D);  // [G][D]
  float* ps = qs + G * D;                                     // [NW][G][32]
  float* wm = ps + NW * G * 32;                               // [NW][G]
  float* wl = wm + NW * G;                                    // [NW][G]
  float* wbuf_all = wl + NW * G;                              // [NW][D]
  float* knew = wbuf_all + NW * D;                            // [D]
  float* vnew = knew + D;                                     // [D]
  float* cpart = vnew + D;                                    // [G][D + 2]: M, L, O[D]
  float* gq = cpart + G * (D + 2);                            // [D] q norm gains
  float* gk = gq + D;                                         // [D] k norm gains
  float* cs = gk + D;                                         // [D / 2] cos, [D / 2] sin at `pos`
  float* wacc = reinterpret_cast<float*>(smem_raw);           // [NW][G][D] once the tiles are used

  cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
  const int CS = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int g = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // every CTA of the cluster reads the same row: the returns below are taken by all of them
  const DevRow row = a.rows[r];
  if (!row.active) return;
  const Geometry& geo = a.g;
  const int pos = row.pos;
  if (pos < 0 || pos >= a.max_pos) {
    if (threadIdx.x == 0 && rank == 0) atomicExch(a.error, 1);
    return;
  }
  const int keys = pos + 1, ntiles = (keys + 31) >> 5;
  const int tpc = (ntiles + CS - 1) / CS;
  const int t0 = rank * tpc, t1 = min(ntiles, t0 + tpc);
  const size_t koff = kv_offset(geo, a.layer, 0, g), voff = kv_offset(geo, a.layer, 1, g);
  uint16_t* kt = ktile + warp * 32 * D;
  uint16_t* vt = vtile + warp * 32 * D;
  // the tile's keys below the new position (earlier steps wrote them): K (XOR-swizzled rows)
  // and V as one group (the first tile) or as two (later tiles, so that K can come early)
  auto stage_part = [&](int t, bool k, bool v) {
    const int key0 = t << 5;
    const int nk = min(32, pos - key0);
    const uint16_t* page = reinterpret_cast<const uint16_t*>(row.pages[key0 >> kPageLog2]);
    const uint16_t* kb = page + koff + (size_t)(key0 & (kPageTokens - 1)) * D;
    const uint16_t* vb = page + voff + (size_t)(key0 & (kPageTokens - 1)) * D;
    for (int i = lane; i < 32 * CPR; i += 32) {
      const int j = i / CPR, c = i % CPR;
      if (j < nk) {
        if (k) cp_async16(kt + (size_t)(j * CPR + (c ^ (j & 7))) * 8, kb + (size_t)j * D + c * 8);
        if (v) cp_async16(vt + (size_t)i * 8, vb + (size_t)j * D + c * 8);
      }
    }
    cp_async_commit();
  };
  auto stage = [&](int t) { stage_part(t, true, true); };
  if (t0 + warp < t1) stage(t0 + warp);
  // the norm gains and the RoPE row of `pos` do not depend on the preceding kernel: into
  // shared memory now, so that the QK norm + RoPE after the wait waits on q alone
  for (int i = threadIdx.x; i < D; i += NW * 32) {
    gq[i] = a.q_norm[i];
    gk[i] = a.k_norm[i];
    cs[i] = i < D / 2 ? a.cos_tab[(size_t)pos * (D / 2) + i] : a.sin_tab[(size_t)pos * (D / 2) + i - D / 2];
  }
  __syncthreads();

  pdl_wait();
  pdl_trigger();

  const int width = (geo.heads + 2 * geo.kvh) * D;
  const uint16_t* src = a.qkv + (size_t)r * width;
  const float* ct = cs;
  const float* st = cs + D / 2;
  float* wbuf = wbuf_all + warp * D;
  for (int h = warp; h < G; h += NW) {
    norm_rope_head<D>(src + (size_t)(g * G + h) * D, gq, geo.eps, ct, st, wbuf);
    for (int i = lane; i < D; i += 32) qs[h * D + i] = wbuf[i];
    __syncwarp();
  }
  if ((ntiles - 1) / tpc == rank) {  // this CTA's last tile holds `pos`: its K and V
    const int kw = G + 2 <= NW ? G : 0;  // warps without a q head when there are two
    uint16_t* page = reinterpret_cast<uint16_t*>(row.pages[pos >> kPageLog2]);
    const size_t slot = (size_t)(pos & (kPageTokens - 1)) * D;
    if (warp == kw) {
      norm_rope_head<D>(src + (size_t)(geo.heads + g) * D, gk, geo.eps, ct, st, wbuf);
      uint16_t* dst = page + koff + slot;
      for (int i = lane; i < D; i += 32) {
        dst[i] = f2bf_exact(wbuf[i]);
        knew[i] = wbuf[i];
      }
    } else if (warp == kw + 1) {
      const uint16_t* vs = src + (size_t)(geo.heads + geo.kvh + g) * D;
      uint16_t* dst = page + voff + slot;
      for (int i = lane; i < D; i += 32) {
        const uint16_t v = __ldcg(vs + i);
        dst[i] = v;
        vnew[i] = bf2f(v);
      }
    }
  }
  __syncthreads();

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[h][e] = 0.f;
  }
  float* pw = ps + warp * G * 32;
  // Warps with several tiles: K of the next tile is requested once the scores no longer need
  // the K buffer, and its V once P.V is done with the V buffer, so each load overlaps the
  // other half of the work. Commit groups in flight at the top of iteration it >= 1: K(t),
  // then V(t).
  for (int t = t0 + warp, it = 0; t < t1; t += NW, ++it) {
    const int key0 = t << 5;
    const int nk = min(32, keys - key0);
    const bool pos_tile = pos - key0 < 32, more = t + NW < t1;
    const int j_new = pos - key0;  // the new position's row in the pos tile
    if (it == 0) cp_async_wait<0>();
    else cp_async_wait<1>();  // K(t); V(t) may still be in flight
    __syncwarp();
    if (pos_tile) {  // the new position's K from shared memory
      for (int c = lane; c < CPR; c += 32) {
        uint32_t kw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) kw[e] = pack_bf16x2(knew[c * 8 + 2 * e], knew[c * 8 + 2 * e + 1]);
        *reinterpret_cast<uint4*>(kt + (size_t)(j_new * CPR + (c ^ (j_new & 7))) * 8) =
            make_uint4(kw[0], kw[1], kw[2], kw[3]);
      }
      __syncwarp();
    }
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
    __syncwarp();  // every lane is done with K(t)
    if (more) stage_part(t + NW, true, false);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float s = lane < nk ? sc[h] * a.scale : -INFINITY;
      const float mnew = fmaxf(m[h], warp_max(s));
      const float alpha = m[h] == -INFINITY ? 0.f : __expf(m[h] - mnew);
      const float pv = lane < nk ? __expf(s - mnew) : 0.f;
      l[h] = l[h] * alpha + warp_sum(pv);
      m[h] = mnew;
      pw[h * 32 + lane] = pv;
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[h][e] *= alpha;
    }
    if (it > 0) {  // V(t): the group before K(t + NW)
      if (more) cp_async_wait<1>();
      else cp_async_wait<0>();
    }
    __syncwarp();
    if (pos_tile) {  // the new position's V from shared memory
      for (int c = lane; c < CPR; c += 32) {
        uint32_t vw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) vw[e] = pack_bf16x2(vnew[c * 8 + 2 * e], vnew[c * 8 + 2 * e + 1]);
        *reinterpret_cast<uint4*>(vt + (size_t)j_new * D + c * 8) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
      }
      __syncwarp();
    }
    for (int j = 0; j < nk; ++j) {
      const uint16_t* vr = vt + (size_t)j * D + lane * DL;
      float vv[DL];
      if constexpr (DL == 2) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(vr);
        vv[0] = bf_lo(w);
        vv[1] = bf_hi(w);
      } else {
        const uint2 w = *reinterpret_cast<const uint2*>(vr);
        vv[0] = bf_lo(w.x);
        vv[1] = bf_hi(w.x);
        vv[2] = bf_lo(w.y);
        vv[3] = bf_hi(w.y);
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float pj = pw[h * 32 + j];
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[h][e] = fmaf(pj, vv[e], acc[h][e]);
      }
    }
    __syncwarp();  // every lane is done with V(t) and the probabilities
    if (more) stage_part(t + NW, false, true);
  }
  cp_async_wait<0>();

  // ---- this CTA's partial: warps merged in shared memory (tiles reused as accumulators)
  __syncthreads();
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
  for (int i = threadIdx.x; i < G * D; i += NW * 32) {
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
    float* ph = cpart + h * (D + 2);
    if (d == 0) {
      ph[0] = M;
      ph[1] = L;
    }
    ph[2 + d] = O;
  }
  __syncwarp();
  cl.sync();  // every CTA's partial is complete

  // ---- outputs [rank * G * D / CS, ...) from every CTA's partial, in rank order
  const float* parts[kClusterMax];
#pragma unroll
  for (int c = 0; c < kClusterMax; ++c) parts[c] = cl.map_shared_rank(cpart, c < CS ? c : 0);
  const int n = G * D, i0 = rank * n / CS, i1 = (rank + 1) * n / CS;
  const int outw = geo.heads * D;
  for (int i = i0 + threadIdx.x; i < i1; i += NW * 32) {
    const int h = i / D, d = i % D;
    float mv[kClusterMax], lv[kClusterMax], ov[kClusterMax];
#pragma unroll
    for (int c = 0; c < kClusterMax; ++c)
      if (c < CS) {
        const float* pc = parts[c] + h * (D + 2);
        mv[c] = pc[0];
        lv[c] = pc[1];
        ov[c] = pc[2 + d];
      }
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < kClusterMax; ++c)
      if (c < CS) M = fmaxf(M, mv[c]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int c = 0; c < kClusterMax; ++c)
      if (c < CS && mv[c] != -INFINITY) {
        const float f = __expf(mv[c] - M);
        L = fmaf(lv[c], f, L);
        O = fmaf(ov[c], f, O);
      }
    a.out[(size_t)r * outw + (size_t)(g * G + h) * D + d] = f2bf_round(O / L);
  }
  __syncwarp();
  cl.sync();  // the partials stay readable until every CTA of the cluster is done
}

}  // namespace y2
