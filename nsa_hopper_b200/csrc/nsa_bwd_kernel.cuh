// NSA selected-branch attention backward for B200 (sm_100a): dQ, dK, dV of the forward in
// nsa_sel_kernel.cuh (per-token selection, d_qk = d_v = 128, G = Hq/Hkv in {8, 16}).
//
// Math (the gradient of reference ref_only.py:2-20 / nsa_reference.py:18-25, which the reference
// itself never implements: README (2).md:85), per query row i = (b, head, token t) and visible key
// j of t's selected blocks, with s = the softmax scale:
//     P_ij = exp(s q_i.k_j - LSE_i)          D_i = dO_i . O_i
//     dP_ij = dO_i . v_j                      dS_ij = P_ij (dP_ij - D_i)
//     dQ_i = s sum_j dS_ij k_j    dK_j = s sum_i dS_ij q_i    dV_j = sum_i P_ij dO_i
//
// Layout of the work (B200-first, not a restatement of any reference code): the scatter onto
// K/V is inverted.  An index lists, per (b*Hkv + kvh, token window, 64-key sub-block u), the tokens
// of the window whose selection row holds u (set semantics, visible keys only; built on the device
// with atomic counters, so in no fixed order within a bucket); a work item is one bucket's
// sub-block with up to kItemTokens of its tokens.  Items are ordered by window, so the CTAs sweep
// the tokens of one window at a time and its Q, dO and dQ rows stay in L2.  A CTA loads K_u, V_u
// once per item (TMA, 16 KB each) and walks the item's tokens in groups of 128 / G (128 query
// rows), each gathered by TMA (one box of G heads x 128 dims per token and tensor, issued by one
// lane per token), with five tcgen05 UMMAs per group:
//     S  [128 rows x 64 keys]  = Q_g  . K_u^T        (A K-major, B K-major)
//     dP [128 rows x 64 keys]  = dO_g . V_u^T        (A K-major, B K-major)
//     dV^T [128 d x 64 keys]  += dO_g^T . P          (A MN-major, B MN-major; TMEM accumulator)
//     dK^T [128 d x 64 keys]  += Q_g^T . dS          (A MN-major, B MN-major; TMEM accumulator)
//     dQ [128 rows x 128 d]    = dS . K_u            (A K-major, B MN-major; two TMEM buffers)
// A softmax-gradient warpgroup (one TMEM lane = one query row per thread) turns S and dP into
// P and dS (bf16, written into shared memory in the UMMA's SW128 layout).  While the UMMAs of
// group n run, it moves dQ of group n - 1 out of TMEM: scaled into SW128 staging tiles and added
// into the fp32 dQ by TMA reduce-adds (whole 128-byte rows at the L2, one instruction per token
// and 32 dimensions).  After an item's last group the same warpgroup adds dK^T and dV^T into
// the fp32 dK, dV (coalesced reductions: a sub-block's tokens span several items).  dQ, dK, dV
// must be zeroed by the caller.
//
// Roles: warp 0 TMA producer, warp 1 MMA issuer (owns TMEM), warps 2-5 softmax-gradient.
// Every mbarrier wait is bounded (nsa::Waiter); on a timeout all roles stop, in-flight TMA
// loads and UMMAs are drained and TMEM is freed.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include "ptx.cuh"
#include "nsa_sel_kernel.cuh"

namespace nsa {
namespace bwd {

constexpr int kD = 128;               // d_qk = d_v
constexpr int kKeys = 64;             // keys per sub-block (N of the S / dP UMMAs)
constexpr int kRows = 128;            // query rows per group (M)
constexpr int kItemTokens = 128;      // tokens per work item (upper bound)
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
// TMEM columns: S, dP, two dQ buffers (group n uses buffer n & 1), dK^T, dV^T
constexpr uint32_t kTmS = 0, kTmDP = 64, kTmDQ = 128, kTmDK = 384, kTmDV = 448;
// Shared-memory layout (bytes from a 1024-aligned base)
constexpr uint32_t kKVSlice = kKeys * 128;                 // one 64-dim slice of a 64-key tile: 8 KB
constexpr uint32_t kKVTile = 2 * kKVSlice;                 // K_u or V_u: 16 KB
constexpr uint32_t kRowSlice = kRows * 128;                // one 64-dim slice of a 128-row tile: 16 KB
constexpr uint32_t kRowTile = 2 * kRowSlice;               // Q_g or dO_g: 32 KB
// A Q / dO tile holds 8-row groups (rows 8i .. 8i+7 = 8 heads of one token) at 2 KB strides, the
// two 64-dim slices of a group 1 KB apart: one TMA box fills a token's G heads x 128 dims.
constexpr uint32_t kGrpStride = 2048, kSliceOff = 1024;
constexpr uint32_t kOffK = 0, kOffV = kKVTile;
constexpr uint32_t kOffQ = 2 * kKVTile;                    // [buf][Q, dO]
constexpr uint32_t kOffP = kOffQ + 4 * kRowTile;           // P [128 rows x 64 keys] bf16, SW128
constexpr uint32_t kOffDS = kOffP + kRows * 128;           // dS, same layout
// dQ staging: per softmax-gradient warp, its 32 rows x 64 fp32 dimensions (half of d): per token
// and 8-head octet, [2 x 32-dim chunks][8 heads][128 B] SW128, the source of one TMA reduce-add
// per token
constexpr uint32_t kStageWarp = 2 * 32 * 128;              // 8 KB
constexpr uint32_t kOffStage = kOffDS + kRows * 128;
constexpr uint32_t kOffBar = kOffStage + 4 * kStageWarp;

struct Bars {
  uint64_t kv_full, kv_empty, q_full[2], q_empty[2], s_full, s_empty, p_full, pd_empty, dq_full[2], dq_empty[2],
      acc_full, acc_empty, drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr uint32_t kSmemBytes = kOffBar + sizeof(Bars) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory of the backward kernel exceeds the per-block limit");

struct Params {
  const int32_t* tokens;  // inverse index: token ids, grouped by (bkv, token window, sub-block)
  const int32_t* items;   // [n_items][4]: bkv, sub-block u, first entry in `tokens`, count (<= kItemTokens)
  const float* lse;       // [B, Hq, T]
  const float* delta;     // [B, Hq, T]: rowsum(dO * O)
  float* dk;              // [B, Hkv, T, 128] fp32 (accumulated)
  float* dv;
  int32_t* err;
  const int* n_items_ptr;  // number of work items (written by the index kernels on the device)
  int B, Hq, Hkv, T, G;
  float scale, scale_log2;
  unsigned long long timeout_ns;
};

constexpr uint32_t kIdescS = ptx::idesc_bf16_f32(128, 64, false, false);
constexpr uint32_t kIdescAcc = ptx::idesc_bf16_f32(128, 64, true, true);
constexpr uint32_t kIdescDQ = ptx::idesc_bf16_f32(128, 128, false, true);

__device__ __forceinline__ int group_count(int count, int R) { return (count + R - 1) / R; }

// dQ of one group (TMEM buffer `tm_dq`, lane = query row of this warp) into the fp32 dQ: each half
// of d goes through this warp's staging tiles (scaled, SW128) and one TMA reduce-add per token.
// `t` is the token of this lane's row (-1: padding row); rows s*G .. s*G+G-1 of the warp are the
// G heads of one token.  Releases the TMEM buffer once it has been read.
__device__ __forceinline__ bool dq_flush(const Waiter& w, Bars* bars, uint32_t j, uint32_t tm_dq, uint8_t* stage,
                                         const CUtensorMap* tmDQ, int t, int hb0, int G, float scale, int lane) {
  if (!w.wait(&bars->dq_full[j & 1], (j >> 1) & 1)) return false;
  ptx::tc_fence_after();
  // this lane's 128-byte rows: token block (lane / G) * G * 256, octet (lane % G) / 8, head lane % 8
  const uint32_t row0 = ptx::smem_u32(stage) + (uint32_t)(lane / G) * G * 256 + (uint32_t)((lane % G) >> 3) * 2048 +
                        (uint32_t)(lane & 7) * 128;
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float a[32], c[32];
    ptx::tmem_ld32(tm_dq + half * 64, a);
    ptx::tmem_ld32(tm_dq + half * 64 + 32, c);
    ptx::tmem_wait_ld();
    if (half == 1) {
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->dq_empty[j & 1]);
    }
    // the previous reduce has finished reading the staging tiles
    if (lane == 0) ptx::bulk_wait_read<0>();
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // 16-byte chunk k of a row, at SW128 position k ^ (head & 7)
      const uint32_t off = row0 + (uint32_t)((k ^ (lane & 7)) << 4);
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(off), "f"(a[4 * k] * scale),
                   "f"(a[4 * k + 1] * scale), "f"(a[4 * k + 2] * scale), "f"(a[4 * k + 3] * scale)
                   : "memory");
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(off + 1024), "f"(c[4 * k] * scale),
                   "f"(c[4 * k + 1] * scale), "f"(c[4 * k + 2] * scale), "f"(c[4 * k + 3] * scale)
                   : "memory");
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    for (int s = 0; s < 32 / G; ++s) {
      const int ts = __shfl_sync(0xffffffffu, t, s * G);
      if (lane == 0 && ts >= 0) ptx::tma_reduce_add_5d(tmDQ, stage + s * G * 256, 0, 0, half * 2, ts, hb0);
    }
    if (lane == 0) ptx::bulk_commit();
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    nsa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ Params p) {
  uint8_t* smem = smem_base();
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = kRows / p.G;  // tokens per group
  const int n_items = *p.n_items_ptr;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars->kv_full, 1);
    ptx::mbar_init(&bars->kv_empty, 1);
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&bars->q_full[s], 1);
      ptx::mbar_init(&bars->q_empty[s], 1);
      ptx::mbar_init(&bars->dq_full[s], 1);
      ptx::mbar_init(&bars->dq_empty[s], 4);
    }
    ptx::mbar_init(&bars->s_full, 1);
    ptx::mbar_init(&bars->s_empty, 4);
    ptx::mbar_init(&bars->p_full, 4);
    ptx::mbar_init(&bars->pd_empty, 1);
    ptx::mbar_init(&bars->acc_full, 1);
    ptx::mbar_init(&bars->acc_empty, 4);
    ptx::mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  // Rows of a group without a token keep whatever the tile held; zero it once so that those rows
  // are finite (their P and dS are zero).
  for (uint32_t i = threadIdx.x; i < 4 * kRowTile / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kOffQ)[i] = make_uint4(0u, 0u, 0u, 0u);
  ptx::fence_proxy_async_smem();
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmDO);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmDQ);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&bars->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const Waiter w{&bars->abort_flag, p.err, p.timeout_ns};

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp:
    // lane 0 waits and arms the barriers, lane s loads token s of a group)
    const uint64_t pol_kv = ptx::policy_evict_last();
    const uint64_t pol_q = ptx::policy_evict_first();
    uint32_t kv_issued = 0, q_issued = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const int4 item = __ldg(reinterpret_cast<const int4*>(p.items) + it);
      const int bkv = item.x, u = item.y, first = item.z, count = item.w;
      const int b = bkv / p.Hkv, kvh = bkv - b * p.Hkv;
      if (lane == 0) {
        if (kv_issued > 0 && !w.wait(&bars->kv_empty, (kv_issued - 1) & 1)) {
          ok = false;
        } else {
          ptx::mbar_arrive_expect_tx(&bars->kv_full, 2 * kKVTile);
          ptx::tma_load_4d(smem + kOffK, &tmK, &bars->kv_full, 0, u * kKeys, 0, bkv, pol_kv);
          ptx::tma_load_4d(smem + kOffV, &tmV, &bars->kv_full, 0, u * kKeys, 0, bkv, pol_kv);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ++kv_issued;
      const int ng = group_count(count, R);
      for (int g = 0; g < ng; ++g) {
        const uint32_t n = q_issued, buf = n & 1;
        const int nt = min(R, count - g * R);
        // token ids of the group, one per lane, in flight while lane 0 waits for the buffer
        const int t = lane < nt ? __ldg(p.tokens + first + g * R + lane) : 0;
        if (lane == 0) {
          if (n >= 2 && !w.wait(&bars->q_empty[buf], ((n >> 1) - 1) & 1))
            ok = false;
          else
            ptx::mbar_arrive_expect_tx(&bars->q_full[buf], (uint32_t)(nt * 2 * p.G * kD * 2));
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++q_issued;
        if (lane < nt) {  // token `lane`: its G heads x 128 dims, one box per tensor
          uint8_t* qd = smem + kOffQ + buf * 2 * kRowTile + (uint32_t)(lane * p.G) * 256;
          const int hb0 = (b * p.Hq + kvh * p.G) >> 3;
          ptx::tma_load_5d(qd, &tmQ, &bars->q_full[buf], 0, 0, 0, t, hb0, pol_q);
          ptx::tma_load_5d(qd + kRowTile, &tmDO, &bars->q_full[buf], 0, 0, 0, t, hb0, pol_q);
        }
        __syncwarp();
      }
    }
    // Drain: the most recent load into each buffer has landed.
    if (lane == 0) {
      if (kv_issued > 0) w.wait_drain(&bars->kv_full, (kv_issued - 1) & 1);
      for (uint32_t back = 1; back <= 2 && back <= q_issued; ++back) {
        const uint32_t k = q_issued - back;
        w.wait_drain(&bars->q_full[k & 1], (k >> 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t k_base = ptx::smem_u32(smem + kOffK), v_base = ptx::smem_u32(smem + kOffV);
      const uint32_t p_base = ptx::smem_u32(smem + kOffP), ds_base = ptx::smem_u32(smem + kOffDS);
      uint32_t m = 0, n = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++m) {
        const int4 item = __ldg(reinterpret_cast<const int4*>(p.items) + it);
        const int ng = group_count(item.w, R);
        if (!w.wait(&bars->kv_full, m & 1)) { ok = false; break; }
        for (int g = 0; g < ng; ++g, ++n) {
          const uint32_t buf = n & 1, dqb = n & 1;
          const uint32_t q_base = ptx::smem_u32(smem + kOffQ + buf * 2 * kRowTile);
          const uint32_t do_base = q_base + kRowTile;
          if (!w.wait(&bars->q_full[buf], (n >> 1) & 1)) { ok = false; break; }
          // S and dP of the previous group have been read out of TMEM
          if (n >= 1 && !w.wait(&bars->s_empty, (n - 1) & 1)) { ok = false; break; }
          ptx::tc_fence_after();
#pragma unroll
          for (int j = 0; j < kD / 16; ++j) {
            const uint32_t oa = (j >> 2) * kSliceOff + (j & 3) * 32, ob = (j >> 2) * kKVSlice + (j & 3) * 32;
            ptx::umma_bf16(tmem + kTmS, ptx::sdesc_sw128(q_base + oa, 16, kGrpStride),
                           ptx::sdesc_sw128(k_base + ob, 16, 1024), kIdescS, j > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int j = 0; j < kD / 16; ++j) {
            const uint32_t oa = (j >> 2) * kSliceOff + (j & 3) * 32, ob = (j >> 2) * kKVSlice + (j & 3) * 32;
            ptx::umma_bf16(tmem + kTmDP, ptx::sdesc_sw128(do_base + oa, 16, kGrpStride),
                           ptx::sdesc_sw128(v_base + ob, 16, 1024), kIdescS, j > 0 ? 1u : 0u);
          }
          ptx::umma_commit(&bars->s_full);
          // P and dS of this group are in shared memory
          if (!w.wait(&bars->p_full, n & 1)) { ok = false; break; }
          // the accumulators of the previous item have been read out
          if (g == 0 && m >= 1 && !w.wait(&bars->acc_empty, (m - 1) & 1)) { ok = false; break; }
          // dQ buffer dqb was read out (group n - 2)
          if (n >= 2 && !w.wait(&bars->dq_empty[dqb], ((n >> 1) - 1) & 1)) { ok = false; break; }
          ptx::tc_fence_after();
#pragma unroll
          for (int j = 0; j < kRows / 16; ++j) {  // K = query rows, 16 per step
            const uint32_t o = (uint32_t)j * 2048, oq = (uint32_t)j * 2 * kGrpStride;
            const uint32_t acc = (g > 0 || j > 0) ? 1u : 0u;
            ptx::umma_bf16(tmem + kTmDV, ptx::sdesc_sw128(do_base + oq, kSliceOff, kGrpStride),
                           ptx::sdesc_sw128(p_base + o, kRowSlice, 1024), kIdescAcc, acc);
            ptx::umma_bf16(tmem + kTmDK, ptx::sdesc_sw128(q_base + oq, kSliceOff, kGrpStride),
                           ptx::sdesc_sw128(ds_base + o, kRowSlice, 1024), kIdescAcc, acc);
          }
#pragma unroll
          for (int j = 0; j < kKeys / 16; ++j) {  // K = keys, 16 per step
            ptx::umma_bf16(tmem + kTmDQ + dqb * 128, ptx::sdesc_sw128(ds_base + j * 32, 16, 1024),
                           ptx::sdesc_sw128(k_base + j * 2048, kKVSlice, 1024), kIdescDQ, j > 0 ? 1u : 0u);
          }
          ptx::umma_commit(&bars->pd_empty);
          ptx::umma_commit(&bars->q_empty[buf]);
          ptx::umma_commit(&bars->dq_full[dqb]);
        }
        if (!ok) break;
        ptx::umma_commit(&bars->kv_empty);
        ptx::umma_commit(&bars->acc_full);
      }
      ptx::umma_commit(&bars->drain);
      w.wait_drain(&bars->drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax-gradient warpgroup
    // Per group n: P and dS from S and dP; then dQ of group n - 1 (its UMMAs ran meanwhile) out of
    // TMEM into the fp32 dQ; after an item's last group, dK and dV of the item.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: query row of S / dP / dQ, dimension of dK^T / dV^T
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int slot = r / p.G, h = r - (r / p.G) * p.G;
    const float sl2 = p.scale_log2;
    uint8_t* stage = smem + kOffStage + (uint32_t)quarter * kStageWarp;
    uint32_t m = 0, n = 0;
    bool dead = false;
    int pend_t = -1, pend_hb = 0;  // the group whose dQ is still in TMEM: this row's token, first head octet
    uint8_t* prow = smem + kOffP + (uint32_t)r * 128;
    uint8_t* dsrow = smem + kOffDS + (uint32_t)r * 128;
    for (int it = blockIdx.x; it < n_items && !dead; it += gridDim.x, ++m) {
      const int4 item = __ldg(reinterpret_cast<const int4*>(p.items) + it);
      const int bkv = item.x, u = item.y, first = item.z, count = item.w;
      const int b = bkv / p.Hkv, kvh = bkv - b * p.Hkv;
      const int ng = group_count(count, R);
      const int key0 = u * kKeys;
      const size_t row0 = ((size_t)b * p.Hq + (size_t)kvh * p.G + h) * p.T;
      // the row data of group 0; later groups' are loaded one group ahead
      int t_next = slot < count ? __ldg(p.tokens + first + slot) : -1;
      float lse_next = t_next >= 0 ? __ldg(p.lse + row0 + t_next) * 1.4426950408889634f : 0.f;
      float dlt_next = t_next >= 0 ? __ldg(p.delta + row0 + t_next) : 0.f;
      for (int g = 0; g < ng && !dead; ++g, ++n) {
        const int t = t_next;
        const float lse2 = lse_next, dlt = dlt_next;
        const int ti1 = (g + 1) * R + slot;
        t_next = (g + 1 < ng && ti1 < count) ? __ldg(p.tokens + first + ti1) : -1;
        // keys of this sub-block visible to the row: key0 + j <= t
        const int nvis = t < 0 ? 0 : min(kKeys, t - key0 + 1);
        dead |= !w.wait(&bars->s_full, n & 1);
        if (dead) break;
        ptx::tc_fence_after();
        uint32_t pk[32], dk[32];  // bf16 pairs of P and dS, keys 2i, 2i+1
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float sv[32], dp[32];
          ptx::tmem_ld32(tmem + lane_addr + kTmS + half * 32, sv);
          ptx::tmem_ld32(tmem + lane_addr + kTmDP + half * 32, dp);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const int k0 = half * 32 + j;
            const float p0 = k0 < nvis ? ptx::ex2(fmaf(sv[j], sl2, -lse2)) : 0.f;
            const float p1 = k0 + 1 < nvis ? ptx::ex2(fmaf(sv[j + 1], sl2, -lse2)) : 0.f;
            const float d0 = p0 * (dp[j] - dlt), d1 = p1 * (dp[j + 1] - dlt);
            const __nv_bfloat162 pp = __floats2bfloat162_rn(p0, p1);
            const __nv_bfloat162 dd = __floats2bfloat162_rn(d0, d1);
            pk[half * 16 + j / 2] = *reinterpret_cast<const uint32_t*>(&pp);
            dk[half * 16 + j / 2] = *reinterpret_cast<const uint32_t*>(&dd);
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->s_empty);
        // P / dS tiles of the previous group have been read by its UMMAs
        if (n >= 1) dead |= !w.wait(&bars->pd_empty, (n - 1) & 1);
        if (dead) break;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = keys 8c..8c+7, SW128 position c ^ (r & 7)
          const uint32_t off = (uint32_t)((c ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          *reinterpret_cast<uint4*>(dsrow + off) = make_uint4(dk[4 * c], dk[4 * c + 1], dk[4 * c + 2], dk[4 * c + 3]);
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->p_full);
        if (t_next >= 0) {
          lse_next = __ldg(p.lse + row0 + t_next) * 1.4426950408889634f;
          dlt_next = __ldg(p.delta + row0 + t_next);
        }
        // dQ of the previous group
        if (n >= 1) {
          dead |= !dq_flush(w, bars, n - 1, tmem + lane_addr + kTmDQ + ((n - 1) & 1) * 128, stage, &tmDQ, pend_t,
                            pend_hb, p.G, p.scale, lane);
          if (dead) break;
        }
        pend_t = t;
        pend_hb = (b * p.Hq + kvh * p.G) >> 3;
      }
      if (dead) break;
      // dK^T, dV^T of the item: lane r = dimension, column j = key key0 + j
      dead |= !w.wait(&bars->acc_full, m & 1);
      if (dead) break;
      ptx::tc_fence_after();
      float* dkb = p.dk + ((size_t)bkv * p.T + key0) * kD + r;
      float* dvb = p.dv + ((size_t)bkv * p.T + key0) * kD + r;
      const int kmax = min(kKeys, p.T - key0);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float vk[32], vv[32];
        ptx::tmem_ld32(tmem + lane_addr + kTmDK + half * 32, vk);
        ptx::tmem_ld32(tmem + lane_addr + kTmDV + half * 32, vv);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = half * 32 + j;
          if (key < kmax) {
            atomicAdd(dkb + (size_t)key * kD, vk[j] * p.scale);
            atomicAdd(dvb + (size_t)key * kD, vv[j]);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->acc_empty);
    }
    // dQ of the last group
    if (!dead && n >= 1)
      dq_flush(w, bars, n - 1, tmem + lane_addr + kTmDQ + ((n - 1) & 1) * 128, stage, &tmDQ, pend_t, pend_hb, p.G,
               p.scale, lane);
    // every reduce has completed before the CTA (and its shared memory) goes away
    if (lane == 0) ptx::bulk_wait<0>();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------
// Preparation kernels (same stream, before nsa_bwd_kernel).
// ------------------------------------------------------------------------------------------

// delta[row] = sum_d dO[row, d] * O[row, d], one warp per (b, head, token) row of d = 128.
template <typename OT>
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ d_o, const OT* __restrict__ o, float* __restrict__ delta,
                             long long rows) {
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* g = d_o + row * kD + lane * 4;
  const OT* x = o + row * kD + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) acc = fmaf(__bfloat162float(g[i]), (float)x[i], acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[row] = acc;
}

// The 64-key sub-blocks that token t of row bkv attends to: entry e of its selection row names
// block e of l_prime keys (sub-blocks e*spb .. e*spb+spb-1); entries outside [0, n_blk), repeats
// of an earlier entry and sub-blocks that start after t select nothing (the forward's rules).
// Buckets are (bkv, token window, sub-block), windows of 2^win_shift tokens, so that the work
// items of one window (consecutive in the item list, run at the same time by the CTAs) touch the
// Q, dO and dQ rows of that window only: sized to stay in L2 while every sub-block the window's
// tokens select is visited.
struct IndexShape {
  int n_bkv, T, KSEL, spb, n_blk, nsub, item_tokens, win_shift, n_win;
};

template <bool kFill>
__global__ void index_rows_kernel(const int32_t* __restrict__ sel, IndexShape sh, int* __restrict__ counts,
                                  const int* __restrict__ tok_off, int* __restrict__ fill, int32_t* __restrict__ tokens) {
  const long long row = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= (long long)sh.n_bkv * sh.T) return;
  const int bkv = (int)(row / sh.T), t = (int)(row - (long long)bkv * sh.T);
  const int32_t* r = sel + row * sh.KSEL;
  for (int i = 0; i < sh.KSEL; ++i) {
    const int e = __ldg(r + i);
    if (e < 0 || e >= sh.n_blk) continue;
    bool rep = false;
    for (int j = 0; j < i; ++j) rep |= __ldg(r + j) == e;
    if (rep) continue;
    for (int s2 = 0; s2 < sh.spb; ++s2) {
      const int u = e * sh.spb + s2;
      if (u * kKeys > t) break;
      const int bucket = (bkv * sh.n_win + (t >> sh.win_shift)) * sh.nsub + u;
      if (kFill) {
        const int pos = atomicAdd(fill + bucket, 1);
        tokens[tok_off[bucket] + pos] = t;
      } else {
        atomicAdd(counts + bucket, 1);
      }
    }
  }
}

// One CTA: exclusive scans of the bucket sizes (token offsets) and of their item counts (item
// offsets); item_off[n] = the number of work items.
__global__ void index_scan_kernel(const int* __restrict__ counts, int n, int item_tokens, int* __restrict__ tok_off,
                                  int* __restrict__ item_off) {
  __shared__ int s_tok[1024], s_it[1024];
  __shared__ int carry_tok, carry_it;
  if (threadIdx.x == 0) carry_tok = carry_it = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int i = base + (int)threadIdx.x;
    const int c = i < n ? counts[i] : 0;
    const int it = (c + item_tokens - 1) / item_tokens;
    s_tok[threadIdx.x] = c;
    s_it[threadIdx.x] = it;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {  // inclusive Hillis-Steele scan
      const int a = threadIdx.x >= (unsigned)off ? s_tok[threadIdx.x - off] : 0;
      const int b = threadIdx.x >= (unsigned)off ? s_it[threadIdx.x - off] : 0;
      __syncthreads();
      s_tok[threadIdx.x] += a;
      s_it[threadIdx.x] += b;
      __syncthreads();
    }
    if (i < n) {
      tok_off[i] = carry_tok + s_tok[threadIdx.x] - c;
      item_off[i] = carry_it + s_it[threadIdx.x] - it;
    }
    __syncthreads();
    if (threadIdx.x == 1023) {
      carry_tok += s_tok[1023];
      carry_it += s_it[1023];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) item_off[n] = carry_it;
}

// Work items of each bucket: {bkv, sub-block, first token entry, token count <= item_tokens}.
__global__ void index_items_kernel(IndexShape sh, const int* __restrict__ counts, const int* __restrict__ tok_off,
                                   const int* __restrict__ item_off, int4* __restrict__ items) {
  const int bucket = blockIdx.x * blockDim.x + threadIdx.x;
  if (bucket >= sh.n_bkv * sh.n_win * sh.nsub) return;
  const int bkv = bucket / (sh.n_win * sh.nsub), u = bucket % sh.nsub;
  const int c = counts[bucket];
  int o = item_off[bucket];
  for (int k = 0; k * sh.item_tokens < c; ++k, ++o)
    items[o] = make_int4(bkv, u, tok_off[bucket] + k * sh.item_tokens, min(sh.item_tokens, c - k * sh.item_tokens));
}

}  // namespace bwd
}  // namespace nsa
