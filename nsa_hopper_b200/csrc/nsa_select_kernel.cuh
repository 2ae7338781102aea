// NSA block selection for B200: the producer of the selected branch's index rows.
//
// What it computes (reference nsa_reference.py:27-44 with compress_kv :5-16 and the
// group-summed queries of :70-71): for every (batch b, KV head kvh, token t)
//     s(t, nb) = (sum_g q[b, kvh*G+g, t, :]) . kblk[b, kvh, nb, :]
//     kblk[nb]  = (1/sqrt(d)) * sum over the compressed keys i mapped to block nb of
//                 mean_{j < cmp_block} k[b, kvh, i*cmp_stride + j, :]
// (the reference sums the per-compressed-key scores into their block; the score is linear in
// the key, so summing the keys first gives the same value), visible iff nb * l_prime <= t,
// and writes the top-k blocks (k = min(n_sel, n_blk) <= 32) by score, highest first, -1 where
// fewer than k blocks are visible.
//
// Two kernels:
//  * kblk_kernel: one CTA per (block, b*Hkv), one thread per dimension, fp32 accumulation.
//  * select_kernel: one CTA per (64-token tile, b*Hkv), 256 threads.  The group-summed query
//    tile (fp32) stays in shared memory; block-key tiles of 64 blocks stream through shared
//    memory; each thread computes a 4 x 4 register tile of scores (fp32 FMA: the ranking must
//    agree with the reference's fp64 one except at near-ties, which bf16 or tf32 tensor-core
//    products would not).  Each warp keeps, for 8 tokens, the running top-k (score, block) in
//    registers, one entry per lane, in descending order; a candidate that beats the current
//    k-th entry is inserted at its rank (ballot + popcount) while the entries below it shift
//    down one lane, so after the first chunks only the few improving candidates cost work.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include "nsa_linspace.cuh"

namespace nsa {
namespace select {

constexpr int kTile = 64;       // tokens per CTA
constexpr int kChunk = 64;      // blocks per shared-memory chunk
constexpr int kThreads = 256;
constexpr int kMaxK = 32;       // top-k capacity (one list entry per lane)
constexpr int kMaxD = 256;

// Selection block of compressed key i: floor(linspace(0, T-1, n_cmp)[i] / l_prime), clamped to
// n_blk - 1 (nsa_reference.py:35-36); see nsa_linspace.cuh.
__device__ __forceinline__ int cmp_block_of(int i, int T, int n_cmp, int l_prime, int n_blk) {
  const int nb = (int)nsa::floor_div_f32(nsa::linspace_f32(i, T, n_cmp), (float)l_prime);
  return nb < n_blk - 1 ? nb : n_blk - 1;
}

// kblk[bh, nb, :] = scale * sum over compressed keys i of block nb of sum_j k[bh, i*stride + j, :]
// (scale = 1 / (cmp_block * sqrt(d))).  One CTA per (block, b*Hkv), one thread per dimension.
// SPLIT = false: an fp32 table [B*Hkv, n_blk, d].  SPLIT = true: the same bytes hold two bf16
// tables [2][B*Hkv, n_blk, d], hi = bf16(x) and lo = bf16(x - hi), the tensor-core operands of
// select_tc_kernel (nsa_select_tc_kernel.cuh).
template <bool SPLIT>
__global__ void kblk_kernel(const __nv_bfloat16* __restrict__ k, float* __restrict__ kblk, int T, int d, int n_blk,
                            int n_cmp, int l_prime, int cmp_block, int cmp_stride, float scale) {
  const int nb = blockIdx.x, bh = blockIdx.y, dd = threadIdx.x;
  if (dd >= d) return;
  // compressed keys whose linspace position falls in block nb: a window around the estimate,
  // each candidate checked exactly (the last block also takes everything clamped into it)
  int lo = 0, hi = 0;
  if (n_cmp > 0) {
    const double per = (n_cmp > 1) ? (double)(n_cmp - 1) / (double)(T - 1) : 0.0;
    lo = max(0, (int)floor((double)nb * l_prime * per) - 2);
    hi = (nb == n_blk - 1) ? n_cmp : min(n_cmp, (int)ceil((double)(nb + 1) * l_prime * per) + 3);
  }
  const __nv_bfloat16* kb = k + (size_t)bh * T * d + dd;
  float acc = 0.f;
  for (int i = lo; i < hi; ++i) {
    if (cmp_block_of(i, T, n_cmp, l_prime, n_blk) != nb) continue;
    const int r0 = i * cmp_stride;
    float w = 0.f;
    for (int j = 0; j < cmp_block; ++j) w += __bfloat162float(kb[(size_t)(r0 + j) * d]);
    acc += w;
  }
  const size_t at = ((size_t)bh * n_blk + nb) * d + dd;
  if constexpr (SPLIT) {
    const float x = acc * scale;
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    __nv_bfloat16* tab = reinterpret_cast<__nv_bfloat16*>(kblk);
    tab[at] = hi;
    tab[(size_t)gridDim.y * n_blk * d + at] = __float2bfloat16_rn(x - __bfloat162float(hi));
  } else {
    kblk[at] = acc * scale;
  }
}

// Ranking of (score, block) pairs: higher score first, ties by smaller block index.
__device__ __forceinline__ bool ranks_before(float a, int ai, float b, int bi) {
  return a > b || (a == b && ai < bi);
}
// Insert (v, vi) into a descending list held one entry per lane: entries ranked before it stay,
// the rest move down one lane (the last one drops out).
__device__ __forceinline__ void insert_sorted(float& lv, int& li, float v, int vi, int lane) {
  const int pos = __popc(__ballot_sync(0xffffffffu, ranks_before(lv, li, v, vi)));
  const float up = __shfl_up_sync(0xffffffffu, lv, 1);
  const int upi = __shfl_up_sync(0xffffffffu, li, 1);
  if (lane == pos) {
    lv = v;
    li = vi;
  } else if (lane > pos) {
    lv = up;
    li = upi;
  }
}

__global__ void __launch_bounds__(kThreads)
    select_kernel(const __nv_bfloat16* __restrict__ q, const float* __restrict__ kblk, int32_t* __restrict__ sel,
                  int Hq, int Hkv, int T, int d, int n_blk, int l_prime, int topk) {
  extern __shared__ __align__(16) float sm[];
  const int dp = d + 4;                      // padded row (floats)
  float* qg = sm;                            // [kTile][dp]
  float* kb = qg + kTile * dp;               // [kChunk][dp]
  float* sc = kb + kChunk * dp;              // [kTile][kChunk + 1]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / Hkv, kvh = bh - (bh / Hkv) * Hkv;
  const int G = Hq / Hkv;
  const int t0 = blockIdx.x * kTile;

  // group-summed queries of the tile (fp32), zero past the sequence end; 8 dimensions per item
  // (one 16-byte load per head)
  const int d8 = d / 8;
  for (int idx = tid; idx < kTile * d8; idx += kThreads) {
    const int tt = idx / d8, c8 = idx - (idx / d8) * d8, t = t0 + tt;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (t < T) {
      const uint4* qp = reinterpret_cast<const uint4*>(q + (((size_t)b * Hq + (size_t)kvh * G) * T + t) * d) + c8;
      const size_t head_stride = (size_t)T * d / 8;
      for (int g = 0; g < G; ++g) {
        const uint4 v = __ldg(qp + (size_t)g * head_stride);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          s[2 * e] += f.x;
          s[2 * e + 1] += f.y;
        }
      }
    }
    float* dst = qg + tt * dp + 8 * c8;
    *reinterpret_cast<float4*>(dst) = make_float4(s[0], s[1], s[2], s[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(s[4], s[5], s[6], s[7]);
  }

  float lv[8];
  int li[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    lv[r] = -INFINITY;
    li[r] = -1;
  }
  const int t_last = min(t0 + kTile, T) - 1;
  const int nb_end = min(n_blk, t_last / l_prime + 1);  // blocks any token of the tile may see
  const int ty = tid >> 4, tx = tid & 15;                // 4 tokens ty*4.., 4 blocks tx+16*j
  const float* kblk_bh = kblk + (size_t)bh * n_blk * d;

  for (int nb0 = 0; nb0 < nb_end; nb0 += kChunk) {
    __syncthreads();  // qg written / previous chunk's kb and sc consumed
    for (int idx = tid; idx < kChunk * (d / 4); idx += kThreads) {
      const int r = idx / (d / 4), c4 = idx - r * (d / 4);
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (nb0 + r < n_blk) x = *reinterpret_cast<const float4*>(kblk_bh + (size_t)(nb0 + r) * d + 4 * c4);
      *reinterpret_cast<float4*>(kb + r * dp + 4 * c4) = x;
    }
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
    for (int dd = 0; dd < d; dd += 4) {
      float4 qa[4], ka[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = *reinterpret_cast<const float4*>(qg + (ty * 4 + a) * dp + dd);
#pragma unroll
      for (int c = 0; c < 4; ++c) ka[c] = *reinterpret_cast<const float4*>(kb + (tx + 16 * c) * dp + dd);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[a][c] = fmaf(qa[a].x, ka[c].x, acc[a][c]);
          acc[a][c] = fmaf(qa[a].y, ka[c].y, acc[a][c]);
          acc[a][c] = fmaf(qa[a].z, ka[c].z, acc[a][c]);
          acc[a][c] = fmaf(qa[a].w, ka[c].w, acc[a][c]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int tt = ty * 4 + a, t = t0 + tt;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int nb = nb0 + tx + 16 * c;
        const bool vis = t < T && nb < n_blk && nb * l_prime <= t;
        sc[tt * (kChunk + 1) + tx + 16 * c] = vis ? acc[a][c] : -INFINITY;
      }
    }
    __syncthreads();
    // insert this chunk's candidates into the running top-k of the warp's 8 tokens (tokens
    // warp + 8 r): only candidates that beat the current k-th entry are inserted, one at a time
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int tt = warp + 8 * r;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float cv = sc[tt * (kChunk + 1) + lane + 32 * h];
        const int ci = nb0 + lane + 32 * h;
        float thr = __shfl_sync(0xffffffffu, lv[r], topk - 1);
        int thr_i = __shfl_sync(0xffffffffu, li[r], topk - 1);
        unsigned m = __ballot_sync(0xffffffffu, ranks_before(cv, ci, thr, thr_i));
        while (m != 0u) {
          const int src = __ffs(m) - 1;
          m &= m - 1u;
          const float v = __shfl_sync(0xffffffffu, cv, src);
          const int vi = __shfl_sync(0xffffffffu, ci, src);
          if (!ranks_before(v, vi, thr, thr_i)) continue;  // the k-th entry rose past it meanwhile
          insert_sorted(lv[r], li[r], v, vi, lane);
          thr = __shfl_sync(0xffffffffu, lv[r], topk - 1);
          thr_i = __shfl_sync(0xffffffffu, li[r], topk - 1);
        }
      }
    }
  }
  // write the top-k of each token, -1 for entries that are not visible blocks
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int t = t0 + warp + 8 * r;
    if (t < T && lane < topk)
      sel[((size_t)bh * T + t) * topk + lane] = (lv[r] == -INFINITY) ? -1 : li[r];
  }
}

}  // namespace select
}  // namespace nsa
