// Row-owner forward for 128-row query tiles (G heads x 128/G tokens sharing one selection row),
// and 64-row tiles (the reference's BQ * G = 64 mode) on M = 64 MMAs (softmax_role_ro_m64).
//
// Same operation, selection semantics, unit order and loaders as nsa_sel_fwd_kernel (the
// reference op's per-query-block mode, nsa_v2.cu:42-50, and the NSA window / compressed
// branches), but with the query rows on the UMMA's M instead of the keys:
//   S[128 rows x 128 keys] = Q_tile . K_chunk^T      (A = Q, B = K, both K-major SW128)
//   O[128 rows x d_v]     += P . V_chunk             (A = P in tensor memory, B = V MN-major)
// so TMEM lane r holds query row r of S, P and O.  The softmax thread that owns row r reads its
// 128 scores straight from TMEM (no shared-memory transpose, no cross-thread reductions),
// writes P back over the first 64 columns of the same score buffer as bf16 pairs, and rescales
// only its own O row when its running max grows.  A tile of 64 rows (the swap-AB kernel's
// widest) spends most of its time in that transpose; here shared memory carries only the
// TMA-written K/V/Q tiles, the tensor core's operand reads and the output staging.
//
// Warps: 0 K loader, 1 score MMA (owns TMEM), 2-5 epilogue, 6-13 softmax (two warpgroups: keys 0-63
// and 64-127 of every chunk), 14 V loader, 15 PV MMA, 16 scheduler.  TMEM: two score/P buffers of
// 128 columns, two O buffers of d_v columns.
// Every ring slot keeps a single in-order consumer per barrier lap, as in nsa_sel_kernel.cuh;
// the score buffer is released by the PV MMA that read its P (s_empty), which is also what a
// softmax rescale waits for.
#pragma once
#include "nsa_sel_kernel.cuh"

namespace nsa {

template <int DQK_, int DV_, typename OutT_, bool EXT_ = false>
struct CfgRO {
  static constexpr int DQK = DQK_, DV = DV_, NCOL = 128, NWG = 1;
  static constexpr bool kExt = EXT_;
  using OutT = OutT_;
  static_assert(DQK == 64 || DQK == 128, "d_qk must be 64 or 128");
  static_assert(DV == 64 || DV == 128, "d_v must be 64 or 128");
  static constexpr int kThreads = 17 * 32;
  static constexpr int kSoftWarp = 6, kVLoadWarp = 14, kPvWarp = 15, kSchedWarp = 16;
  static constexpr int kBox = kSub * 128;                 // 64 rows x 128 B TMA box (8 KB)
  static constexpr int kKChunkStride = 2 * kBox;          // one 64-wide d slice of a 128-key K tile
  static constexpr int kKStage = (DQK / 64) * kKChunkStride;
  static constexpr int kVSub = (DV / 64) * kBox;          // one 64-key sub-block of V
  static constexpr int kVStage = 2 * kVSub;
  static constexpr int kVGroups = 1;
  static constexpr int kQChunk = 128 * 128;               // one 64-wide d slice of the 128-row Q tile
  static constexpr int kQBytes = (DQK / 64) * kQChunk;
  static constexpr int kQS = 1;                           // Q tile ring depth
  static constexpr int kEPB = 128 / (int)sizeof(OutT);    // O elements per 128-byte box row
  static constexpr int kOutBoxes = DV / kEPB;             // 128-byte column boxes per O row
  static constexpr int kOutBox = 128 * 128;               // one staged box: 128 rows x 128 B
  static constexpr int kStgBoxes = 2;
  static constexpr int kTmemS = 0;                        // score / P buffers: 2 x 128 columns
  static constexpr int kTmemO = 256;                      // O accumulators: 2 x DV columns
  static constexpr int kTmemCols = 512;
  static constexpr uint32_t kIdescS = ptx::idesc_bf16_f32(128, 128, false, false);
  static constexpr uint32_t kIdescPV = ptx::idesc_bf16_f32(128, DV, false, true);
  // 64-row tiles (Params::ro_m64): M = 64, rows in TMEM lanes 0-15 of every 32-lane quarter
  static constexpr uint32_t kIdescS64 = ptx::idesc_bf16_f32(64, 128, false, false);
  static constexpr uint32_t kIdescPV64 = ptx::idesc_bf16_f32(64, DV, false, true);
};

template <class C>
__host__ __device__ inline SmemLayout smem_layout_ro(int KS, int VS, int maxsub, int /*out_bufs*/) {
  SmemLayout s{};
  uint32_t o = 0;
  s.off_k = o; o += (uint32_t)KS * C::kKStage;
  s.off_v = o; o += (uint32_t)VS * C::kVStage;
  s.off_q = o; o += (uint32_t)C::kQS * C::kQBytes;
  o = align_up(o, 1024);
  s.off_out = o; o += (uint32_t)C::kStgBoxes * C::kOutBox;
  s.off_ml = o; o += 8u * 2 * 128;  // [unit parity][row] x {m, l}
  s.off_alpha = o; o += 4u * 2 * 2 * 128;  // softmax exchange: [chunk parity][half][row] partial max
  s.off_fac = o; o += 4u * 128;            // softmax exchange: second half's row sum
  s.off_p = s.off_tr = 0;
  s.off_info = o; o += 4u * kInfoSlots * (kInfoHdr + maxsub);
  o = align_up(o, 16);
  s.off_bar = o; o += (uint32_t)sizeof(SmemBars);
  s.total = o + 1024;
  return s;
}

// ------------------------------------------------------------------------------------------
// Score MMA: S = Q_tile . K_chunk^T into score buffer kc % 2 once the PV MMA of chunk kc - 2
// has read that buffer's P.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void mma_s_role_ro(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem,
                              int lane) {
  if (lane == 0) {
    bool ok = true;
    if (p.debug_stall) ok = w.wait(&bars->stall, 0);
    uint32_t ui = 0, ne = 0, kc = 0;
    Ring k;
    const uint32_t k_base = ptx::smem_u32(smem + p.off_k), q_base = ptx::smem_u32(smem + p.off_q);
    const uint32_t idesc = p.ro_m64 ? C::kIdescS64 : C::kIdescS;
    for (; ok; ++ui) {
      const int slot = ui % kInfoSlots;
      if (!w.wait(&bars->info_full[slot], (ui / kInfoSlots) & 1)) break;
      const int* inf = info_slot(p, smem, slot);
      if (inf[kInfStop]) break;
      const int nsub = min(inf[kInfNsub], p.maxsub);
      const int ref = inf[kInfRef];
      const int nch = (nsub + 1) >> 1;
      if (nch > 0) {
        const int qs = ne % C::kQS;
        long long t_wait = 0;
        if (!w.wait(&bars->q_full[qs], (ne / C::kQS) & 1)) break;
        const uint64_t aq0 = ptx::sdesc_sw128(q_base + qs * C::kQBytes, 16, 1024);
        for (int c = 0; c < nch; ++c) {
          const int sl = (int)(kc & 1u);
          if (kc >= 2 && !w.wait(&bars->s_empty[sl], ((kc >> 1) - 1u) & 1u)) { ok = false; break; }
          const long long t0 = clock64();
          if (!w.wait(&bars->k_full[k.idx], k.phase)) { ok = false; break; }
          t_wait += clock64() - t0;
          ptx::tc_fence_after();
          const uint64_t bk0 = ptx::sdesc_sw128(k_base + k.idx * C::kKStage, 16, 1024);
          const uint32_t dS = tmem + C::kTmemS + sl * 128;
#pragma unroll
          for (int j = 0; j < C::DQK / 16; ++j) {
            const uint32_t ca = (j >> 2) * C::kQChunk + (j & 3) * 32;
            const uint32_t cb = (j >> 2) * C::kKChunkStride + (j & 3) * 32;
            ptx::umma_bf16(dS, desc_add(aq0, ca), desc_add(bk0, cb), idesc, j > 0 ? 1u : 0u);
          }
          ptx::umma_commit(&bars->k_empty[k.idx]);
          ptx::umma_commit(&bars->s_full[sl]);
          ++kc;
          k.next((uint32_t)p.KS);
        }
        if (!ok) break;
        ptx::umma_commit(&bars->q_empty[qs]);
        // the reference op's cycle counters (nsa_v2.cu:69-71): K-tile wait cycles of the unit
        if (p.cyc != nullptr) atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref),
                                        (unsigned long long)t_wait);
        ++ne;
      }
      ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    ptx::umma_commit(&bars->drain_s);
    w.wait_drain(&bars->drain_s, 0);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// PV MMA: O[unit parity] += P (TMEM) . V_chunk; the commit releases the V stage and the score
// buffer.  Only the sub-blocks that exist are multiplied (a half chunk leaves stale rows of the
// V stage untouched).
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void mma_pv_role_ro(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem,
                               int lane) {
  if (lane == 0) {
    bool ok = true;
    uint32_t ui = 0, ne = 0, kc = 0;
    Ring v;
    const uint32_t v_base = ptx::smem_u32(smem + p.off_v);
    const uint32_t idesc = p.ro_m64 ? C::kIdescPV64 : C::kIdescPV;
    for (; ok; ++ui) {
      const int slot = ui % kInfoSlots;
      if (!w.wait(&bars->info_full[slot], (ui / kInfoSlots) & 1)) break;
      const int* inf = info_slot(p, smem, slot);
      if (inf[kInfStop]) break;
      const int nsub = min(inf[kInfNsub], p.maxsub);
      const int ref = inf[kInfRef];
      const int nch = (nsub + 1) >> 1;
      if (nch > 0) {
        const long long t_unit0 = clock64();
        long long t_wait = 0;
        // this O buffer (and the unit's ml slot) was last read by the epilogue for unit ne - 2
        if (ne >= 2 && !w.wait(&bars->o_empty[ne & 1], ((ne >> 1) - 1) & 1)) break;
        const uint32_t dO = tmem + C::kTmemO + (ne & 1) * C::DV;
        for (int c = 0; c < nch; ++c) {
          const int sl = (int)(kc & 1u);
          const int nsc = min(2, nsub - 2 * c);
          if (!w.wait(&bars->p_full[sl], (kc >> 1) & 1u)) { ok = false; break; }
          const long long t0 = clock64();
          if (!w.wait(&bars->v_full[v.idx], v.phase)) { ok = false; break; }
          t_wait += clock64() - t0;
          ptx::tc_fence_after();
          const uint64_t b0 = ptx::sdesc_sw128(v_base + v.idx * C::kVStage, C::kBox, 1024);
          // P of keys 0-63 sits in columns 0-31 of the buffer, keys 64-127 in columns 64-95
          const uint32_t aP = tmem + C::kTmemS + sl * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j < nsc * 4) {
              const uint32_t cb = (j >> 2) * C::kVSub + (j & 3) * 2048;
              ptx::umma_bf16_ts(dO, aP + (j >> 2) * 64 + (j & 3) * 8, desc_add(b0, cb), idesc,
                                (c == 0 && j == 0) ? 0u : 1u);
            }
          }
          ptx::umma_commit(&bars->v_empty[v.idx]);
          ptx::umma_commit(&bars->s_empty[sl]);
          ++kc;
          v.next((uint32_t)p.VS);
        }
        if (!ok) break;
        ptx::umma_commit(&bars->o_full[ne & 1]);
        // cycle counters: V-tile wait cycles, and the unit's other cycles on this warp
        if (p.cyc != nullptr) {
          const long long tot = clock64() - t_unit0;
          atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref), (unsigned long long)t_wait);
          atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref + 1),
                    (unsigned long long)(tot > t_wait ? tot - t_wait : 0));
        }
        ++ne;
      }
      ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    ptx::umma_commit(&bars->drain_pv[0]);
    w.wait_drain(&bars->drain_pv[0], 0);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// Softmax: thread r owns query row r (TMEM lane r) of every chunk.
// ------------------------------------------------------------------------------------------
// Key visibility inside one 64-key sub-block that starts at key position s: the key at offset j
// is visible to a row iff the sub-block exists and lo <= s + j <= hi, s + j < kend (lo is
// INT_MIN / 2 without a window).  Those offsets form one interval [a, a + w) (w = 0: none), so
// masking an element is the single unsigned compare (j - a) < w.
__device__ __forceinline__ void ro_sub_interval(int s, bool exists, int hi, int lo, int kend, int& a, unsigned& w) {
  const int a0 = max(lo - s, 0);
  const int b0 = min(min(hi + 1, kend) - s, kSub);
  a = a0;
  w = (exists && b0 > a0) ? (unsigned)(b0 - a0) : 0u;
}

template <class C>
__device__ void softmax_role_ro(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem,
                                int h) {
  // Warpgroup h handles keys [64h, 64h + 64) of every chunk for all 128 rows: the row max is
  // combined through shared memory once per chunk (one 256-thread barrier), both groups apply
  // the same running max, group 0 rescales O, and the row sums meet at the end of the unit.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = threadIdx.x - (C::kSoftWarp + 4 * h) * 32;  // 0..127 inside the warpgroup
  const int quarter = warp & 3;
  const int r = quarter * 32 + lane;                         // the row (TMEM lane) this thread owns
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  float2* ml = reinterpret_cast<float2*>(smem + p.off_ml);
  float* xmax = reinterpret_cast<float*>(smem + p.off_alpha);  // [chunk parity][half][row]
  float* lsum1 = reinterpret_cast<float*>(smem + p.off_fac);   // [row]
  const float sl2 = p.scale_log2;
  const int ci = r - (r / p.BQs) * p.BQs;                   // token of the row inside the unit
  // A 64-row tile (G * BQs = 64) leaves rows 64-127 as zero query padding: their scores are exactly
  // 0 and the PV MMA reads those unrewritten score columns as P = 0, so the two warps of each group
  // that own only padding rows skip the exp pass and the P stores (half the exp work of the mode).
  const bool pad = quarter * 32 >= p.G * p.BQs;
  uint32_t ui = 0, ne = 0, kc = 0;
  bool dead = false;

  for (;; ++ui) {
    const int slot = ui % kInfoSlots;
    dead |= !w.wait_inline(&bars->info_full[slot], (ui / kInfoSlots) & 1);
    if (ptx::named_bar_or(kWgBar0, 256, dead)) break;
    const int* inf = info_slot(p, smem, slot);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int t0 = inf[kInfT0], kend = inf[kInfKend];
    const int nch = (nsub + 1) >> 1;
    if (nch == 0) {
      if (h == 0 && i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
      continue;
    }
    const int t = t0 + ci;
    int hi = t, lo = INT_MIN / 2, hi_all = t0, lo_all = INT_MIN / 2;
    if constexpr (C::kExt) {
      hi = key_hi(p, t);
      lo = key_lo(p, t);
      hi_all = key_hi(p, t0);
      lo_all = key_lo(p, t0 + p.BQs - 1);
    }
    const uint32_t obase = tmem + lane_addr + C::kTmemO + (ne & 1) * C::DV;
    float m_run = -INFINITY, l_run = 0.f;
    bool first = true;

    for (int c = 0; c < nch; ++c, ++kc) {
      const int sl = (int)(kc & 1u);
      if (pad) {  // only the row-max barrier and the P-ready arrival
        ptx::named_bar_sync(kWgBar0, 256);
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->p_full[sl]);
        continue;
      }
      dead |= !w.wait_inline(&bars->s_full[sl], (kc >> 1) & 1u);
      ptx::tc_fence_after();
      const uint32_t sbase = tmem + lane_addr + C::kTmemS + sl * 128 + 64 * h;
      // This group's keys are exactly sub-block h of the chunk.  It needs a mask only when some
      // row does not see all of that sub-block; each row's visible part is one interval.
      const bool has = h == 0 || (2 * c + 1) < nsub;
      const int sh = has ? inf[kInfoHdr + 2 * c + h] : 0;
      bool full = has && (sh + kSub - 1 <= hi_all) && (sh + kSub <= kend);
      if constexpr (C::kExt) full = full && (sh >= lo_all);
      int ma = 0;
      unsigned mw = kSub;
      if (!full) ro_sub_interval(sh, has, hi, lo, kend, ma, mw);

      // pass 1: the row's max over this group's 64 keys, combined with the other group's
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        float v[32];
        ptx::tmem_ld32(sbase + 32 * b, v);
        ptx::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if ((unsigned)(32 * b + j - ma) >= mw) v[j] = -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], v[j]);
      }
      float* xm = xmax + (kc & 1u) * 256;
      xm[h * 128 + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      ptx::named_bar_sync(kWgBar0, 256);
      const float cmax_x = fmaxf(xm[r], xm[128 + r]) * sl2;
      float m_use = m_run, alpha = 1.f;
      bool need = false;
      if (first) {
        m_use = cmax_x;
      } else {
        const float m_cand = fmaxf(m_run, cmax_x);
        if (m_cand > m_run + kRescaleLog2) {
          alpha = (m_run == -INFINITY) ? 0.f : ptx::ex2(m_run - m_cand);
          m_use = m_cand;
          need = true;
        }
      }
      // Rescale O in group 0.  The decision is per row, but tcgen05.ld / tcgen05.st are
      // .sync.aligned (the whole warp executes them together), so a warp with any row to rescale
      // runs the pass for all its lanes, the others with alpha = 1.  (A lane-divergent pass here
      // stalled the warp: rows whose running max jumped by more than 2^8 next to rows whose did not.)
      if (h == 0 && __any_sync(0xffffffffu, need)) {
        // the rows' O, once the PV of the previous chunk (which released its buffer) is done
        dead |= !w.wait_inline(&bars->s_empty[(kc - 1) & 1u], ((kc - 1) >> 1) & 1u);
        ptx::tc_fence_after();
#pragma unroll
        for (int h0 = 0; h0 < C::DV; h0 += 16) {
          float o[16];
          ptx::tmem_ld16(obase + h0, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= alpha;
          ptx::tmem_st16(obase + h0, o);
        }
        ptx::tmem_wait_st();
      }

      // pass 2: exp2, the partial row sum, and P as bf16 pairs in columns [64h, 64h + 32) of the
      // buffer (this group's own score columns, already read).  Both loads come before the P
      // stores: a tcgen05.ld issued after a tcgen05.st of the same thread waits for the store.
      // (mref is finite, so a masked score of -inf gives ex2(-inf) = 0 without a select.)
      const float mref = (m_use == -INFINITY) ? 0.f : m_use;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[2][16];
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        float v[32];
        ptx::tmem_ld32(sbase + 32 * b, v);
        ptx::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if ((unsigned)(32 * b + j - ma) >= mw) v[j] = -INFINITY;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = ptx::ex2(fmaf(v[j], sl2, -mref));
#pragma unroll
        for (int j = 0; j < 32; ++j) ls[j & 3] += v[j];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * jj], v[2 * jj + 1]);
          pk[b][jj] = *reinterpret_cast<const uint32_t*>(&hh);
        }
      }
#pragma unroll
      for (int b = 0; b < 2; ++b) ptx::tmem_st16u(sbase + 16 * b, pk[b]);
      ptx::tmem_wait_st();
      l_run = l_run * alpha + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
      m_run = m_use;
      first = false;
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[sl]);
    }

    // Row sums meet in group 0, which publishes (m, l) for the epilogue; the ml slot of unit ne
    // was last read by the epilogue for unit ne - 2.
    if (h == 1) lsum1[r] = l_run;
    ptx::named_bar_sync(kWgBar0, 256);
    if (h == 0) {
      const float l_tot = l_run + lsum1[r];
      if (ne >= 2) dead |= !w.wait_inline(&bars->o_empty[ne & 1], ((ne >> 1) - 1) & 1);
      ml[(ne & 1) * 128 + r] = make_float2(m_run, l_tot);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->wg_done[ne & 1]);
      if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    ++ne;
  }
}

// ------------------------------------------------------------------------------------------
// Softmax of a 64-row tile computed by M = 64 MMAs (Params::ro_m64).  Tile row 16q + j sits in
// TMEM lane 32q + j (j < 16) of S, P and O.  The warp of quarter q in group h owns rows
// 16q .. 16q + 15 through the 16-lane access shapes.  Thread t holds rows 16q + t/4 ("A") and
// 16q + t/4 + 8 ("B"), at columns 8g + 2(t%4) and 8g + 2(t%4) + 1 of the group's 64 keys,
// g = 0..7.  So each thread exps 32 scores per chunk, where the 128-row form of a 64-row tile
// gives 64 to each thread of half the warps, and all eight softmax warps share the work.  The
// four threads of a row combine their maxima and sums with two shuffles.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void softmax_role_ro_m64(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w,
                                    uint32_t tmem, int h) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = threadIdx.x - (C::kSoftWarp + 4 * h) * 32;
  const int quarter = warp & 3;
  const int cp = lane & 3;                          // column pair inside every 8-column group
  const int rA = quarter * 16 + (lane >> 2), rB = rA + 8;
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  float2* ml = reinterpret_cast<float2*>(smem + p.off_ml);
  float* xmax = reinterpret_cast<float*>(smem + p.off_alpha);  // [chunk parity][half][row]
  float* lsum1 = reinterpret_cast<float*>(smem + p.off_fac);   // [row]
  const float sl2 = p.scale_log2;
  const int ciA = rA % p.BQs, ciB = rB % p.BQs;
  uint32_t ui = 0, ne = 0, kc = 0;
  bool dead = false;

  for (;; ++ui) {
    const int slot = ui % kInfoSlots;
    dead |= !w.wait_inline(&bars->info_full[slot], (ui / kInfoSlots) & 1);
    if (ptx::named_bar_or(kWgBar0, 256, dead)) break;
    const int* inf = info_slot(p, smem, slot);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int t0 = inf[kInfT0], kend = inf[kInfKend];
    const int nch = (nsub + 1) >> 1;
    if (nch == 0) {
      if (h == 0 && i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
      continue;
    }
    const int tA = t0 + ciA, tB = t0 + ciB;
    int hiA = tA, loA = INT_MIN / 2, hiB = tB, loB = INT_MIN / 2, hi_all = t0, lo_all = INT_MIN / 2;
    if constexpr (C::kExt) {
      hiA = key_hi(p, tA);
      loA = key_lo(p, tA);
      hiB = key_hi(p, tB);
      loB = key_lo(p, tB);
      hi_all = key_hi(p, t0);
      lo_all = key_lo(p, t0 + p.BQs - 1);
    }
    const uint32_t obase = tmem + lane_addr + C::kTmemO + (ne & 1) * C::DV;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    bool first = true;

    for (int c = 0; c < nch; ++c, ++kc) {
      const int sl = (int)(kc & 1u);
      dead |= !w.wait_inline(&bars->s_full[sl], (kc >> 1) & 1u);
      ptx::tc_fence_after();
      const uint32_t sbase = tmem + lane_addr + C::kTmemS + sl * 128 + 64 * h;
      // as in the 128-row form: this group's keys are sub-block h, masked by one interval per row
      const bool has = h == 0 || (2 * c + 1) < nsub;
      const int sh = has ? inf[kInfoHdr + 2 * c + h] : 0;
      bool full = has && (sh + kSub - 1 <= hi_all) && (sh + kSub <= kend);
      if constexpr (C::kExt) full = full && (sh >= lo_all);

      float v[32];
      ptx::tmem_ld16x256b_x8(sbase, v);
      ptx::tmem_wait_ld();
      if (!full) {
        int aA, aB;
        unsigned wA, wB;
        ro_sub_interval(sh, has, hiA, loA, kend, aA, wA);
        ro_sub_interval(sh, has, hiB, loB, kend, aB, wB);
        const int oA = 2 * cp - aA, oB = 2 * cp - aB;  // element (g, e) sits at offset 8g + 2cp + e
#pragma unroll
        for (int g = 0; g < 8; ++g)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            if ((unsigned)(8 * g + e + oA) >= wA) v[4 * g + e] = -INFINITY;
            if ((unsigned)(8 * g + e + oB) >= wB) v[4 * g + 2 + e] = -INFINITY;
          }
      }
      float xa = -INFINITY, xb = -INFINITY;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        xa = fmaxf(xa, fmaxf(v[4 * g], v[4 * g + 1]));
        xb = fmaxf(xb, fmaxf(v[4 * g + 2], v[4 * g + 3]));
      }
      xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 1));
      xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 1));
      xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 2));
      xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 2));
      float* xm = xmax + (kc & 1u) * 256;
      if (cp == 0) {
        xm[h * 128 + rA] = xa;
        xm[h * 128 + rB] = xb;
      }
      ptx::named_bar_sync(kWgBar0, 256);
      const float cA = fmaxf(xm[rA], xm[128 + rA]) * sl2, cB = fmaxf(xm[rB], xm[128 + rB]) * sl2;
      float muA = mA, muB = mB, alA = 1.f, alB = 1.f;
      bool need = false;
      if (first) {
        muA = cA;
        muB = cB;
      } else {
        const float ca = fmaxf(mA, cA), cb = fmaxf(mB, cB);
        if (ca > mA + kRescaleLog2) {
          alA = (mA == -INFINITY) ? 0.f : ptx::ex2(mA - ca);
          muA = ca;
          need = true;
        }
        if (cb > mB + kRescaleLog2) {
          alB = (mB == -INFINITY) ? 0.f : ptx::ex2(mB - cb);
          muB = cb;
          need = true;
        }
      }
      // Group 0 rescales O (warp-uniform: the 16-lane accesses are .sync.aligned as well).
      if (h == 0 && __any_sync(0xffffffffu, need)) {
        dead |= !w.wait_inline(&bars->s_empty[(kc - 1) & 1u], ((kc - 1) >> 1) & 1u);
        ptx::tc_fence_after();
#pragma unroll
        for (int h0 = 0; h0 < C::DV; h0 += 16) {
          float o[8];
          ptx::tmem_ld16x256b_x2(obase + h0, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            o[4 * g] *= alA;
            o[4 * g + 1] *= alA;
            o[4 * g + 2] *= alB;
            o[4 * g + 3] *= alB;
          }
          ptx::tmem_st16x256b_x2(obase + h0, o);
        }
        ptx::tmem_wait_st();
      }

      // exp2, the partial row sums, and P as bf16 pairs: keys 8g + 2cp, 8g + 2cp + 1 of the
      // group form pair 4g + cp, stored in column 64h + 4g + cp (the group's own score columns,
      // already read).  mref is finite, so a masked score of -inf gives ex2(-inf) = 0.
      const float mrA = (muA == -INFINITY) ? 0.f : muA, mrB = (muB == -INFINITY) ? 0.f : muB;
      float sA = 0.f, sB = 0.f;
      uint32_t pk[16];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const float a0 = ptx::ex2(fmaf(v[4 * g], sl2, -mrA)), a1 = ptx::ex2(fmaf(v[4 * g + 1], sl2, -mrA));
        const float b0 = ptx::ex2(fmaf(v[4 * g + 2], sl2, -mrB)), b1 = ptx::ex2(fmaf(v[4 * g + 3], sl2, -mrB));
        sA += a0 + a1;
        sB += b0 + b1;
        const __nv_bfloat162 ha = __floats2bfloat162_rn(a0, a1), hb = __floats2bfloat162_rn(b0, b1);
        pk[2 * g] = *reinterpret_cast<const uint32_t*>(&ha);
        pk[2 * g + 1] = *reinterpret_cast<const uint32_t*>(&hb);
      }
      ptx::tmem_st16x128b_x8(sbase, pk);
      ptx::tmem_wait_st();
      lA = lA * alA + sA;
      lB = lB * alB + sB;
      mA = muA;
      mB = muB;
      first = false;
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[sl]);
    }

    // Row sums: the four threads of a row, then the two groups in group 0, which publishes
    // (m, l) for the epilogue; the ml slot of unit ne was last read by the epilogue for unit ne - 2.
    lA += __shfl_xor_sync(0xffffffffu, lA, 1);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1);
    lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 2);
    if (h == 1 && cp == 0) {
      lsum1[rA] = lA;
      lsum1[rB] = lB;
    }
    ptx::named_bar_sync(kWgBar0, 256);
    if (h == 0) {
      if (ne >= 2) dead |= !w.wait_inline(&bars->o_empty[ne & 1], ((ne >> 1) - 1) & 1);
      if (cp == 0) {
        ml[(ne & 1) * 128 + rA] = make_float2(mA, lA + lsum1[rA]);
        ml[(ne & 1) * 128 + rB] = make_float2(mB, lB + lsum1[rB]);
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->wg_done[ne & 1]);
      if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    ++ne;
  }
}

// ------------------------------------------------------------------------------------------
// Epilogue: thread r scales O row r by w / l, writes the LSE, and stages the row into 128-byte
// boxes (SW128 layout: 16-byte chunk j of row r at j ^ (r & 7)) that TMA stores, or adds with a
// TMA reduce when the descriptor asks to accumulate.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void epilogue_role_ro(const CUtensorMap* tmO, const Params& p, uint8_t* smem, SmemBars* bars,
                                 const Waiter& w, uint32_t tmem) {
  using OutT = typename C::OutT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = threadIdx.x - kEpiWarp0 * 32;
  const int quarter = warp & 3;
  // The tile row held by this thread's TMEM lane; -1 for lanes 16-31 of a quarter, which the
  // M = 64 layout leaves unused.
  const int r = p.ro_m64 ? (lane < 16 ? quarter * 16 + lane : -1) : quarter * 32 + lane;
  const int rr = r < 0 ? 0 : r;
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  const float2* ml = reinterpret_cast<const float2*>(smem + p.off_ml);
  uint8_t* stg = smem + p.off_out;
  const float wgt = p.o_weight != nullptr ? __ldg(p.o_weight) : 1.f;
  const int cg = rr / p.BQs, ci = rr - (rr / p.BQs) * p.BQs;
  uint32_t ui = 0, ne = 0, nbox = 0;
  bool dead = false;

  for (;; ++ui) {
    const int slot = ui % kInfoSlots;
    dead |= !w.wait(&bars->info_full[slot], (ui / kInfoSlots) & 1);
    if (ptx::named_bar_or(kEpiBar, 128, dead)) break;
    const int* inf = info_slot(p, smem, slot);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int t0 = inf[kInfT0], ntok = inf[kInfNtok], b = inf[kInfB], kvh = inf[kInfKvh];
    const int nch = (nsub + 1) >> 1;
    if (nch > 0) {
      dead |= !w.wait(&bars->wg_done[ne & 1], (ne >> 1) & 1);
      dead |= !w.wait(&bars->o_full[ne & 1], (ne >> 1) & 1);
      ptx::tc_fence_after();
    }
    const float2 v_ml = nch > 0 ? ml[(ne & 1) * 128 + rr] : make_float2(-INFINITY, 0.f);
    const float scale = v_ml.y > 0.f ? wgt / v_ml.y : 0.f;
    if (r >= 0 && r < p.G * p.BQs && ci < ntok && p.lse != nullptr) {
      const float lse = v_ml.y > 0.f ? (v_ml.x + log2f(v_ml.y)) * 0.69314718055994530942f : -INFINITY;
      p.lse[((size_t)b * p.Hq + (size_t)kvh * p.G + cg) * p.T + t0 + ci] = lse;
    }
    if (ntok > 0) {
      const uint32_t obase = tmem + lane_addr + C::kTmemO + (ne & 1) * C::DV;
      for (int bx = 0; bx < C::kOutBoxes; ++bx, ++nbox) {
        uint8_t* box = stg + (nbox % C::kStgBoxes) * C::kOutBox;
        if (i == 0) ptx::bulk_wait_read<C::kStgBoxes - 1>();  // the box's previous store has read it
        ptx::named_bar_sync(kEpiBar, 128);
        float v[C::kEPB];
#pragma unroll
        for (int h0 = 0; h0 < C::kEPB; h0 += 16) {
          if (nch > 0) {
            ptx::tmem_ld16(obase + bx * C::kEPB + h0, *reinterpret_cast<float(*)[16]>(&v[h0]));
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[h0 + j] = 0.f;
          }
        }
        if (nch > 0) ptx::tmem_wait_ld();
        uint8_t* row = box + rr * 128;
#pragma unroll
        for (int j = 0; j < 8 && r >= 0; ++j) {
          uint4 q;
          if constexpr (sizeof(OutT) == 4) {
            q.x = __float_as_uint(v[4 * j + 0] * scale);
            q.y = __float_as_uint(v[4 * j + 1] * scale);
            q.z = __float_as_uint(v[4 * j + 2] * scale);
            q.w = __float_as_uint(v[4 * j + 3] * scale);
          } else {
            __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * j + 0] * scale, v[8 * j + 1] * scale);
            __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * j + 2] * scale, v[8 * j + 3] * scale);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * j + 4] * scale, v[8 * j + 5] * scale);
            __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * j + 6] * scale, v[8 * j + 7] * scale);
            q.x = *reinterpret_cast<const uint32_t*>(&h0);
            q.y = *reinterpret_cast<const uint32_t*>(&h1);
            q.z = *reinterpret_cast<const uint32_t*>(&h2);
            q.w = *reinterpret_cast<const uint32_t*>(&h3);
          }
          *reinterpret_cast<uint4*>(row + ((j ^ (rr & 7)) << 4)) = q;
        }
        ptx::fence_proxy_async_smem();
        ptx::named_bar_sync(kEpiBar, 128);
        if (i == 0) {
          if (p.o_accum)
            ptx::tma_reduce_add_4d(tmO, box, bx * C::kEPB, t0, kvh * p.G, b);
          else
            ptx::tma_store_4d(tmO, box, bx * C::kEPB, t0, kvh * p.G, b);
          ptx::bulk_commit();
        }
      }
    }
    if (nch > 0) {
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->o_empty[ne & 1]);  // O buffer and ml slot are free
      ++ne;
    }
    if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
  }
  if (i == 0) ptx::bulk_wait<0>();
}

// ------------------------------------------------------------------------------------------
template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    nsa_ro_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                      const __grid_constant__ Params p) {
  uint8_t* smem = smem_base();
  SmemBars* bars = reinterpret_cast<SmemBars*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kInfoSlots; ++s) {
      ptx::mbar_init(&bars->info_full[s], 1);
      // consumers: K and V loaders, score MMA, PV MMA, softmax, epilogue
      ptx::mbar_init(&bars->info_empty[s], 6);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&bars->s_full[s], 1);   // score MMA commit
      ptx::mbar_init(&bars->s_empty[s], 1);  // PV MMA commit: P read, buffer free
      ptx::mbar_init(&bars->p_full[s], 8);   // softmax warps
      ptx::mbar_init(&bars->o_full[s], 1);
      ptx::mbar_init(&bars->wg_done[s], 4);
      ptx::mbar_init(&bars->o_empty[s], 4);
    }
    for (int s = 0; s < kQSlots; ++s) {
      ptx::mbar_init(&bars->q_full[s], 1);
      ptx::mbar_init(&bars->q_empty[s], 1);
    }
    for (int s = 0; s < kMaxStages; ++s) {
      ptx::mbar_init(&bars->k_full[s], 1);
      ptx::mbar_init(&bars->k_empty[s], 1);
      ptx::mbar_init(&bars->v_full[s], 1);
      ptx::mbar_init(&bars->v_empty[s], 1);
    }
    ptx::mbar_init(&bars->drain_s, 1);
    ptx::mbar_init(&bars->drain_pv[0], 1);
    ptx::mbar_init(&bars->drain_pv[1], 1);
    ptx::mbar_init(&bars->stall, 1);
    bars->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  // Rows of the Q tile beyond G*BQs (a 64-row tile) are never written by TMA and must read as
  // zero, so their score rows stay finite.
  if (p.G * p.BQs < 128)
    for (int idx = threadIdx.x; idx < C::kQS * C::kQBytes / 16; idx += C::kThreads)
      reinterpret_cast<uint4*>(smem + p.off_q)[idx] = make_uint4(0u, 0u, 0u, 0u);
  ptx::fence_proxy_async_smem();
  if (warp == kLoaderWarp && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmO);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(&bars->tmem_base, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const Waiter w{&bars->abort_flag, p.err, p.timeout_ns};

  if (warp == kLoaderWarp) {
    kloader_role<C>(&tmK, p, smem, bars, w, lane);
  } else if (warp == kMmaWarp) {
    mma_s_role_ro<C>(p, smem, bars, w, tmem, lane);
  } else if (warp < C::kSoftWarp) {
    epilogue_role_ro<C>(&tmO, p, smem, bars, w, tmem);
  } else if (warp < C::kVLoadWarp) {
    if (p.ro_m64)
      softmax_role_ro_m64<C>(p, smem, bars, w, tmem, (warp - C::kSoftWarp) >> 2);
    else
      softmax_role_ro<C>(p, smem, bars, w, tmem, (warp - C::kSoftWarp) >> 2);
  } else if (warp == C::kVLoadWarp) {
    vloader_role<C>(&tmV, p, smem, bars, w, lane);
  } else if (warp == C::kPvWarp) {
    mma_pv_role_ro<C>(p, smem, bars, w, tmem, lane);
  } else {
    scheduler_role<C>(&tmQ, p, smem, bars, w, lane);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace nsa
