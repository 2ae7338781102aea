// NSA selected-branch attention forward for B200 (sm_100a).
//
// What it computes (reference semantics: ref_only.py:2-20, nsa_reference.py:18-25 and
// 66-77, kernels nsa_v0.cu:10-116 / nsa_v2.cu:24-145): for every (batch b, KV head kvh,
// query block qb) the selection row sel[b, kvh, qb, :] names up to KSEL key blocks of
// l_prime keys.  Each of the G = Hq/Hkv query heads of kvh and each of the BQ query tokens
// of the block attends, with scale 1/sqrt(d_qk) and a causal mask (key <= query), to the
// union of those blocks; O = softmax(S) V and LSE = log(sum exp S) per (head, token).
//
// How (B200-first design, not a translation of the Hopper kernels):
//  * Persistent CTAs (one per SM) walk work units u = (b*Hkv+kvh, qb, part) in
//    KV-head-major order, so all SMs sweep the tokens of one KV head together and the
//    gathered K/V blocks of that head are re-read from L2 rather than HBM.  K/V loads carry
//    an L2 evict_last hint, the streaming Q loads evict_first.
//  * Scheduler warp: turns each unit's selection row into a list of 64-key sub-blocks (set
//    semantics, padding, causal and range clipping) in a shared-memory "info" ring and loads
//    the unit's Q tile, running several units ahead.  The K-loader warp and the V-loader warp
//    only wait for free ring stages and issue the K and V boxes of each 128-key chunk (two
//    sub-blocks), one box per lane.
//  * MMA warps, one issuing thread each, use tcgen05 UMMAs in swap-AB form, so the 128 keys of
//    a chunk are the M=128 dimension and the G*BQ query rows of the unit are N (16..64):
//        S^T[keys x rows]  = K_chunk[keys x d_qk] . Q^T          (A K-major, B K-major)
//        O^T[d_v x rows]  += V_chunk^T[d_v x keys] . P^T          (A MN-major, B K-major)
//    The score warp runs ahead of the softmax into TMEM score buffers; there is one PV warp
//    per softmax group, so the two groups' PV streams never queue behind each other.
//  * NWG softmax warpgroups (1 or 2): chunk c of a unit belongs to group c % NWG, which keeps
//    its own online-softmax state and its own O^T accumulator in TMEM (a split over the
//    unit's keys, merged by the epilogue).  Per chunk a group reads S^T from TMEM, transposes
//    it through shared memory so each thread owns NCOL keys of one query row, masks, runs an
//    exp2 online softmax with a warp-shuffle row max and lazy O rescaling (only when the
//    running max grows by more than 2^8), and writes P^T as bf16 in the UMMA K-major SW128
//    layout (two P buffers per group when they fit, so it runs a chunk ahead of its PVs).
//  * Epilogue warpgroup: merges the groups' partial results (O, running max, sum), writes
//    the fp32 log-sum-exp and stores O (bf16 or fp32) with TMA tensor stores, overlapping
//    the softmax of the next unit.
//
// Every ring slot (score buffers, V stages, P tiles) has exactly one consumer that waits on
// its laps in order: an mbarrier parity wait for lap L returns at once while lap L-1 is still
// incomplete, so slots shared by two consumers in alternation would let one of them read a
// stale tile.
// Every mbarrier wait is bounded by %globaltimer; a wait that runs out sets an error bit,
// all roles stop, in-flight TMA loads/stores and UMMAs are drained and TMEM is freed.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include <limits.h>
#include "ptx.cuh"
#include "nsa_linspace.cuh"

namespace nsa {

constexpr int kSub = 64;          // keys per sub-block (one TMA box of rows)
constexpr int kChunk = 128;       // keys per chunk = M of the UMMAs
constexpr int kInfoSlots = 4;     // depth of the unit-info ring
constexpr int kInfoHdr = 16;      // ints of header per info slot
constexpr int kMaxStages = 8;     // upper bound on K and V ring depth
#ifndef NSA_SSLOTS
#define NSA_SSLOTS 4
#endif
constexpr int kMaxSSlots = 8;     // TMEM score buffers (MMA look-ahead), split between softmax groups
constexpr int kQSlots = 3;        // Q tile ring (the loader stages one unit ahead)
constexpr int kLoaderWarp = 0;    // K tiles
constexpr int kMmaWarp = 1;       // score MMAs; owns the TMEM allocation
constexpr int kEpiWarp0 = 2;      // warps 2..5: epilogue
constexpr int kSoftWarp0 = 6;     // warps 6..6+4*NWG-1: softmax warpgroups; then the V loader, one
                                  // PV MMA warp per softmax group and the scheduler (unit info, Q)
constexpr uint32_t kEpiBar = 1;   // named barrier of the epilogue warpgroup
constexpr uint32_t kWgBar0 = 2;   // named barrier of softmax warpgroup w = kWgBar0 + w
constexpr float kRescaleLog2 = 8.0f;
constexpr int kDevErrTimeout = 1;

#ifndef NSA_SPLIT_PV
#define NSA_SPLIT_PV 1
#endif
// PV MMA warps: one per softmax group when split, else one for all chunks.
__host__ __device__ constexpr int pv_warps(int nwg) { return NSA_SPLIT_PV ? nwg : 1; }
__host__ __device__ constexpr int vloader_warp(int nwg) { return kSoftWarp0 + 4 * nwg; }
__host__ __device__ constexpr int pv_warp(int nwg) { return kSoftWarp0 + 4 * nwg + 1; }
__host__ __device__ constexpr int sched_warp(int nwg) { return kSoftWarp0 + 4 * nwg + 1 + pv_warps(nwg); }
__host__ __device__ constexpr int threads_for(int nwg) { return 32 * (sched_warp(nwg) + 1); }

// Position in a ring of `n` slots: slot index and the parity of the lap (the mbarrier phase of
// a "full" wait; an "empty" wait of a later lap uses the opposite parity).
struct Ring {
  uint32_t idx = 0, phase = 0;
  bool lapped = false;  // true once every slot has been used at least once
  __device__ __forceinline__ void next(uint32_t n) {
    if (++idx == n) {
      idx = 0;
      phase ^= 1u;
      lapped = true;
    }
  }
};

// Info-slot header fields.
enum : int { kInfNsub = 0, kInfT0, kInfNtok, kInfKend, kInfB, kInfKvh, kInfBkv, kInfSeq0, kInfRef, kInfStop };

struct Params {
  const int32_t* sel;
  const int32_t* cu_seqlens;
  float* lse;
  int64_t* cyc;
  int32_t* err;
  int B, Hq, Hkv, T, G, LP, BQ, BQs, parts, NQB, KSEL, n_seq;
  int bkv_begin, bkv_end, qb_begin, qb_end;
  int n_units, maxsub, KS, VS;
  float scale_log2;
  unsigned long long timeout_ns;
  uint32_t off_k, off_v, off_q, off_p, off_out, off_tr, off_alpha, off_fac, off_ml, off_info, off_bar;
  // Key visibility: key position p (0..kv_len) is visible to query token t iff p <= hi(t) and
  // p >= t - window + 1 (window > 0 only); hi(t) = t, or with key_map = 1 (compressed keys) the
  // last key whose float32 linspace(0, T-1, kv_len) position is <= t.
  int kv_len, window, key_map;
  int debug_stall;  // 1: the MMA warp first waits on a barrier nothing arrives on (error-path test)
  int out_bufs;     // output staging tiles (2: double buffer; 1 when shared memory is tight)
  // Work distribution: after the first wave (unit = blockIdx.x), each CTA takes the next unit
  // from this global counter, zeroed on the stream just before the launch, so SMs that run
  // faster take more units; nullptr = fixed strides of gridDim.x.
  unsigned int* work_counter;
  int o_accum;             // 1: O += w * result through TMA reduce-add (fp32 O); 0: O = w * result
  const float* o_weight;   // device float w, or nullptr for 1
  // Row-owner kernel, 64-row tiles: 1 = M = 64 MMAs (rows in TMEM lanes 0-15 of each 32-lane
  // quarter, every softmax warp owns 16 rows); 0 = 128-row MMAs with 64 rows of zero padding.
  int ro_m64;
};

// P tiles: NP buffers (4 for N <= 32 and d_qk <= 128, else 2), NP / NWG per softmax group; the k-th chunk of
// group w uses buffer w * (NP / NWG) + k % (NP / NWG), and k / (NP / NWG) is the phase index of
// that use.  More than one buffer per group lets the softmax run a chunk ahead of the PV MMAs.
constexpr int kMaxPSlots = 4;
template <int NP, int NWG>
__device__ __forceinline__ int pslot_of(int wg, uint32_t k) {
  return wg * (NP / NWG) + (int)(k % (uint32_t)(NP / NWG));
}
template <int NP, int NWG>
__device__ __forceinline__ uint32_t pphase_of(uint32_t k) { return k / (uint32_t)(NP / NWG); }

struct SmemBars {
  uint64_t info_full[kInfoSlots], info_empty[kInfoSlots];
  uint64_t q_full[kQSlots], q_empty[kQSlots];
  uint64_t k_full[kMaxStages], k_empty[kMaxStages];
  uint64_t v_full[kMaxStages], v_empty[kMaxStages];
  uint64_t s_full[kMaxSSlots], s_empty[kMaxSSlots];
  uint64_t p_full[kMaxPSlots], pv_done[kMaxPSlots];
  uint64_t o_full[2], wg_done[2], o_empty[2];
  uint64_t drain_s, drain_pv[2];
  uint64_t stall;  // never arrived on; only the debug_stall path waits on it
  uint32_t tmem_base;
  int abort_flag;
};

__host__ __device__ constexpr int ceil_pow2_32(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}
__host__ __device__ constexpr uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// EXT_: key visibility beyond the causal default (window bound, compressed key map; the
// Params fields window / key_map / kv_len).  The causal instantiations keep the plain mask.
template <int DQK_, int DV_, int NCOL_, typename OutT_, int NWG_, bool EXT_ = false>
struct Cfg {
  static constexpr int DQK = DQK_, DV = DV_, NCOL = NCOL_, NWG = NWG_;
  static constexpr bool kExt = EXT_;
  using OutT = OutT_;
  static_assert(DQK % 64 == 0 && DQK >= 64 && DQK <= 256, "d_qk must be 64..256 in steps of 64");
  static_assert(DV == 64 || DV == 128, "d_v must be 64 or 128");
  static_assert(NCOL == 16 || NCOL == 32 || NCOL == 64, "N must be 16/32/64");
  static_assert(NWG == 1 || NWG == 2, "one or two softmax warpgroups");
  static constexpr int kThreads = threads_for(NWG);
  static constexpr int kDvPad = DV < 128 ? 128 : DV;       // PV runs M=128; pad V tiles to 128 rows of d
  static constexpr int kBox = kSub * 128;                   // 64 rows x 128 B = 8 KB TMA box
  static constexpr int kKChunkStride = 2 * kBox;            // one 64-wide d slice of a 128-key K tile
  static constexpr int kKStage = (DQK / 64) * kKChunkStride;
  static constexpr int kVSub = (kDvPad / 64) * kBox;        // one 64-key sub-block of the V tile
  static constexpr int kVStage = 2 * kVSub;
  static constexpr int kQChunk = NCOL * 128;                // one 64-wide d slice of the Q tile
  static constexpr int kQBytes = (DQK / 64) * kQChunk;
  static constexpr int kPSub = NCOL * 128;                  // P^T for one 64-key sub-block
  static constexpr int kPBytes = 2 * kPSub;
  static constexpr int kPSlots = (NCOL <= 32 && DQK <= 128) ? 4 : 2;  // P tiles (see pslot_of); measured best
  static constexpr int kTPC = 128 / NCOL;                   // softmax threads per query row
  static constexpr int kKPT = NCOL;                         // keys per softmax thread per chunk
  static constexpr int kTRS = kChunk + 4;                   // transpose row stride (floats)
  static constexpr int kTrBytes = NCOL * kTRS * 4;
  static constexpr int kOutChunkElems = NCOL * 64;
  static constexpr int kOutBytes = (DV / 64) * kOutChunkElems * (int)sizeof(OutT);
  static constexpr int kSSlots = NCOL >= 64 ? 4 : NSA_SSLOTS;  // score buffers (TMEM: 512 columns)
  static constexpr int kSPer = kSSlots / NWG;               // score buffers per softmax group
  static constexpr int kPvWarps = pv_warps(NWG);
  static constexpr int kVGroups = kPvWarps;                 // V stages are split between PV warps
  static constexpr int kTmemS = 0;                          // score buffers: kSSlots x NCOL columns
  static constexpr int kTmemO = kSSlots * NCOL;             // O^T accumulators: [wg][unit parity] x NCOL
  static constexpr int kTmemCols = ceil_pow2_32((kSSlots + 2 * NWG) * NCOL);
  static_assert(kTmemCols <= 512, "TMEM holds 512 columns");
  static_assert(kSSlots <= kMaxSSlots && kSSlots % NWG == 0, "score buffers");
  static constexpr uint32_t kIdescS = ptx::idesc_bf16_f32(128, NCOL, false, false);
  static constexpr uint32_t kIdescPV = ptx::idesc_bf16_f32(128, NCOL, true, false);
  static constexpr int kQS = kQSlots;  // Q tile ring depth
};

// Shared-memory layout (byte offsets from a 1024-aligned base); identical on host and device.
struct SmemLayout {
  uint32_t off_k, off_v, off_q, off_p, off_out, off_tr, off_alpha, off_fac, off_ml, off_info, off_bar, total;
};
template <class C>
__host__ __device__ inline SmemLayout smem_layout(int KS, int VS, int maxsub, int out_bufs) {
  SmemLayout s{};
  uint32_t o = 0;
  s.off_k = o; o += (uint32_t)KS * C::kKStage;
  s.off_v = o; o += (uint32_t)VS * C::kVStage;
  s.off_q = o; o += (uint32_t)C::kQS * C::kQBytes;
  o = align_up(o, 1024);
  s.off_p = o; o += (uint32_t)C::kPSlots * C::kPBytes;
  o = align_up(o, 128);
  s.off_out = o; o += (uint32_t)out_bufs * C::kOutBytes;
  o = align_up(o, 16);
  s.off_tr = o; o += (uint32_t)C::NWG * C::kTrBytes;
  s.off_alpha = o; o += 4u * C::NWG * C::NCOL;
  s.off_fac = o; o += 4u * C::NWG * C::NCOL;
  s.off_ml = o; o += 8u * C::NWG * 2 * C::NCOL;  // [wg][unit parity][col] x {m, l}
  s.off_info = o; o += 4u * kInfoSlots * (kInfoHdr + maxsub);
  o = align_up(o, 16);
  s.off_bar = o; o += (uint32_t)sizeof(SmemBars);
  s.total = o + 1024;  // slack to align the dynamic shared-memory base to 1024 B
  return s;
}

// The bounded part of a wait, out of line: inlined at the ~30 wait sites it made the warp roles'
// hot loops large enough that instruction fetch stalled them (one copy: north star 11.1 -> 9.8 ms).
__device__ __noinline__ bool wait_slow(uint64_t* bar, uint32_t parity, int* abort_flag, int32_t* err,
                                       unsigned long long timeout_ns) {
  const uint64_t t0 = ptx::globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*(volatile int*)abort_flag != 0) return false;
    if (ptx::globaltimer() - t0 > timeout_ns) {
      *(volatile int*)abort_flag = 1;
      if (err != nullptr) atomicOr(err, kDevErrTimeout);
      return false;
    }
  }
}

// A bounded mbarrier wait.  Returns false if the CTA is aborting or the wait ran out of time
// (then it raises the abort flag and the device error bit).
struct Waiter {
  int* abort_flag;
  int32_t* err;
  unsigned long long timeout_ns;

  __device__ __forceinline__ void raise() const {
    *(volatile int*)abort_flag = 1;
    if (err != nullptr) atomicOr(err, kDevErrTimeout);
  }
  __device__ __forceinline__ bool aborted() const { return *(volatile int*)abort_flag != 0; }
  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) const {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    return wait_slow(bar, parity, abort_flag, err, timeout_ns);
  }
  // Fully inlined variant, for code whose live registers a call would spill (the wide-tile
  // softmax holds KPT = 64 scores).
  __device__ __forceinline__ bool wait_inline(uint64_t* bar, uint32_t parity) const {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 32; ++i)
        if (ptx::mbar_try_wait(bar, parity)) return true;
      if (aborted()) return false;
      if (ptx::globaltimer() - t0 > timeout_ns) {
        raise();
        return false;
      }
    }
  }
  // Used while draining: ignores the abort flag, bounded by its own limit.
  __device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity) const {
    const uint64_t t0 = ptx::globaltimer();
    while (!ptx::mbar_try_wait(bar, parity)) {
      if (ptx::globaltimer() - t0 > 200000000ull) {  // 200 ms
        if (err != nullptr) atomicOr(err, kDevErrTimeout);
        return false;
      }
    }
    return true;
  }
};

__device__ __forceinline__ int key_hi(const Params& p, int t) {
  return p.key_map ? compressed_limit(t, p.T, p.kv_len) : t;
}
__device__ __forceinline__ int key_lo(const Params& p, int t) { return p.window > 0 ? t - p.window + 1 : INT_MIN / 2; }

__device__ __forceinline__ uint8_t* smem_base() {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t a = ptx::smem_u32(smem_raw);
  return smem_raw + ((1024u - (a & 1023u)) & 1023u);
}

__device__ __forceinline__ int* info_slot(const Params& p, uint8_t* smem, int slot) {
  return reinterpret_cast<int*>(smem + p.off_info) + slot * (kInfoHdr + p.maxsub);
}

// ------------------------------------------------------------------------------------------
// Unit decode + selection-row compaction (whole loader warp).  Produces the list of 64-key
// sub-block starts the unit attends to, in selection-row order:
//   * entries < 0 or >= the number of blocks of the (sub)sequence select nothing
//     (ref_only.py:9-12 routes them to a discarded column);
//   * a repeated entry selects nothing new (the reference builds a set, ref_only.py:11);
//   * sub-blocks that start after the last query token of the unit, or at/after the end of
//     the sequence, are dropped (every key in them is masked, nsa_v0.cu:73).
// ------------------------------------------------------------------------------------------
// Selection-row entry `lane` of unit u (-1 past KSEL).  The loader issues this load two units
// ahead so its latency overlaps the K-tile traffic of the current unit.
__device__ __forceinline__ const int32_t* unit_row(const Params& p, int u) {
  const int per_bkv = (p.qb_end - p.qb_begin) * p.parts;
  const int bkv_off = u / per_bkv;
  const int qb = p.qb_begin + (u - bkv_off * per_bkv) / p.parts;
  return p.sel + ((size_t)(p.bkv_begin + bkv_off) * p.NQB + qb) * p.KSEL;
}
__device__ __forceinline__ int fetch_row_entry(const Params& p, int u, int lane) {
  return (u < p.n_units && lane < p.KSEL) ? __ldg(unit_row(p, u) + lane) : -1;
}

// `idx0` is entry `lane` of the unit's selection row (fetch_row_entry).
template <bool EXT>
__device__ int build_unit_info(const Params& p, int u, int* inf, int lane, int idx0) {
  const int per_bkv = (p.qb_end - p.qb_begin) * p.parts;
  const int bkv_off = u / per_bkv;
  const int bkv = p.bkv_begin + bkv_off;
  const int rem = u - bkv_off * per_bkv;
  const int qb_off = rem / p.parts;
  const int qb = p.qb_begin + qb_off;
  const int part = rem - qb_off * p.parts;
  const int b = bkv / p.Hkv, kvh = bkv - b * p.Hkv;
  const int t0 = qb * p.BQ + part * p.BQs;
  const int ntok = max(0, min(p.BQs, p.T - t0));
  int seq0 = 0, kend = p.kv_len;
  if (p.cu_seqlens != nullptr && ntok > 0) {
    int lo = 0, hi = p.n_seq;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(p.cu_seqlens + mid) <= t0) lo = mid; else hi = mid;
    }
    seq0 = __ldg(p.cu_seqlens + lo);
    kend = __ldg(p.cu_seqlens + lo + 1);
  }
  // last key position any row of the unit may see; first key position any row may see
  const int lim = min(EXT ? key_hi(p, t0 + ntok - 1) : t0 + ntok - 1, kend - 1);
  const int low = EXT ? key_lo(p, t0) : 0;
  const int nblk = (kend - seq0 + p.LP - 1) / p.LP;
  const int spb = p.LP / kSub;
  const int32_t* row = p.sel + ((size_t)bkv * p.NQB + qb) * p.KSEL;
  int count = 0;
  if (ntok > 0) {
    for (int base = 0; base < p.KSEL; base += 32) {
      const int j = base + lane;
      const int idx = base == 0 ? idx0 : ((j < p.KSEL) ? __ldg(row + j) : -1);
      bool valid = idx >= 0 && idx < nblk && (seq0 + idx * p.LP) <= lim;
      if (EXT) valid = valid && (seq0 + idx * p.LP + p.LP - 1) >= low;
      // set semantics: drop repeats of an earlier entry (same 32-entry group)
      if ((__match_any_sync(0xffffffffu, idx) & ((1u << lane) - 1u)) != 0u) valid = false;
      if (valid && base > 0) {  // earlier groups (KSEL > 32 only)
        for (int k2 = 0; k2 < base; ++k2)
          if (__ldg(row + k2) == idx) { valid = false; break; }
      }
      const int bstart = valid ? seq0 + idx * p.LP : 0;
      const int cnt = valid ? min(spb, (lim - bstart) / kSub + 1) : 0;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int tot = __shfl_sync(0xffffffffu, incl, 31);
      const int excl = incl - cnt;
      for (int s = 0; s < cnt; ++s) {
        const int pos = count + excl + s;
        if (pos < p.maxsub) inf[kInfoHdr + pos] = bstart + s * kSub;
      }
      count += tot;
    }
  }
  count = min(count, p.maxsub);
  if (lane == 0) {
    inf[kInfNsub] = count;
    inf[kInfT0] = t0;
    inf[kInfNtok] = ntok;
    inf[kInfKend] = kend;
    inf[kInfB] = b;
    inf[kInfKvh] = kvh;
    inf[kInfBkv] = bkv;
    inf[kInfSeq0] = seq0;
    inf[kInfRef] = bkv * p.NQB + qb;
    inf[kInfStop] = 0;
  }
  return count;
}

// ------------------------------------------------------------------------------------------
// Scheduler warp: decodes each unit into the info ring and loads its Q tile (three-deep Q
// ring), running ahead of the consumers; the selection row of the unit after next is already in
// flight while a unit is decoded.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void scheduler_role(const CUtensorMap* tmQ, const Params& p, uint8_t* smem, SmemBars* bars,
                               const Waiter& w, int lane) {
  const uint64_t pol_q = ptx::policy_evict_first();
  Ring info, q;
  bool ok = true;
  // The unit after the current one is claimed (and its selection row fetched) one step ahead.
  auto next_unit = [&](int cur) -> int {
    if (p.work_counter == nullptr) return cur + (int)gridDim.x;
    unsigned v = 0;
    if (lane == 0) v = atomicAdd(p.work_counter, 1u);
    return (int)gridDim.x + (int)__shfl_sync(0xffffffffu, v, 0);
  };
  int u = blockIdx.x;
  int idx = fetch_row_entry(p, u, lane);
  int u_next = u < p.n_units ? next_unit(u) : p.n_units;
  while (u < p.n_units && ok) {
    const int uc = u;
    const int idx_next = fetch_row_entry(p, u_next, lane);  // next row, in flight
    u = u_next;
    if (u < p.n_units) u_next = next_unit(u);
    if (info.lapped) {
      int r = 1;
      if (lane == 0) r = w.wait(&bars->info_empty[info.idx], info.phase ^ 1u) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, r, 0)) break;
    }
    int* inf = info_slot(p, smem, info.idx);
    const int nsub = build_unit_info<C::kExt>(p, uc, inf, lane, idx);
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&bars->info_full[info.idx]);
    info.next(kInfoSlots);
    idx = idx_next;
    if (nsub == 0) continue;
    int r = 1;
    if (lane == 0) {
      const int t0 = inf[kInfT0], b = inf[kInfB], kvh = inf[kInfKvh];
      if (q.lapped && !w.wait(&bars->q_empty[q.idx], q.phase ^ 1u)) {
        r = 0;
      } else {
        uint8_t* qdst = smem + p.off_q + q.idx * C::kQBytes;
        ptx::mbar_arrive_expect_tx(&bars->q_full[q.idx], (uint32_t)(C::DQK * p.BQs * p.G * 2));
        for (int cc = 0; cc < C::DQK / 64; ++cc)
          ptx::tma_load_4d(qdst + cc * C::kQChunk, tmQ, &bars->q_full[q.idx], cc * 64, t0, kvh * p.G, b, pol_q);
      }
    }
    ok = __shfl_sync(0xffffffffu, r, 0) != 0;
    if (ok) q.next(C::kQS);
  }
  // Every consumer leaves its loop at the stop entry that follows the last unit.
  if (ok) {
    int r = 1;
    if (info.lapped && lane == 0) r = w.wait(&bars->info_empty[info.idx], info.phase ^ 1u) ? 1 : 0;
    if (__shfl_sync(0xffffffffu, r, 0)) {
      int* inf = info_slot(p, smem, info.idx);
      if (lane == 0) inf[kInfStop] = 1;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->info_full[info.idx]);
    }
  }
  // Drain: the most recent Q load of every slot has landed.
  if (lane == 0) {
    Ring d = q;
    for (int s2 = 0; s2 < C::kQS; ++s2) {
      // slot d.idx - 1 - s2 (mod kQS), lap parity adjusted when it wraps
      const uint32_t back = (uint32_t)s2 + 1u;
      const uint32_t slot = (d.idx + C::kQS - back % C::kQS) % C::kQS;
      const uint32_t ph = (d.idx >= back) ? d.phase : (d.phase ^ 1u);
      if (d.lapped || d.idx >= back) w.wait_drain(&bars->q_full[slot], ph);
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// K loader warp: the K chunk tiles of each unit into their ring, in chunk order.  A K tile is
// nsc x (DQK/64) boxes of 64 rows x 128 B; box b is issued by lane b, since the TMA throughput of
// one issuing thread is well below what the SM can absorb.  Everything but the issue itself is
// computed before the wait for a free slot.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void kloader_role(const CUtensorMap* tmK, const Params& p, uint8_t* smem, SmemBars* bars,
                             const Waiter& w, int lane) {
  const uint64_t pol_kv = ptx::policy_evict_last();
  constexpr int kNdc = C::DQK / 64;
  const int j = lane / kNdc, cc = lane - (lane / kNdc) * kNdc;  // this lane's (sub-block, d slice)
  uint8_t* kdst0 = smem + p.off_k + cc * C::kKChunkStride + j * C::kBox;
  Ring info, k;
  bool ok = true;
  while (ok) {
    int got = 1;
    if (lane == 0) got = w.wait(&bars->info_full[info.idx], info.phase) ? 1 : 0;
    if (!__shfl_sync(0xffffffffu, got, 0)) break;
    const int* inf = info_slot(p, smem, info.idx);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int bkv = inf[kInfBkv];
    const int nch = (nsub + 1) >> 1;
    for (int c = 0; c < nch; ++c) {
      const int nsc = min(2, nsub - 2 * c);
      const bool mine = lane < nsc * kNdc;
      const int row = mine ? inf[kInfoHdr + 2 * c + j] : 0;
      uint8_t* dst = kdst0 + k.idx * C::kKStage;
      int go = 1;
      if (lane == 0) {
        go = (!k.lapped || w.wait(&bars->k_empty[k.idx], k.phase ^ 1u)) ? 1 : 0;
        if (go) ptx::mbar_arrive_expect_tx(&bars->k_full[k.idx], (uint32_t)(nsc * kSub * C::DQK * 2));
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) { ok = false; break; }
      if (mine) ptx::tma_load_3d(dst, tmK, &bars->k_full[k.idx], cc * 64, row, bkv, pol_kv);
      k.next((uint32_t)p.KS);
    }
    if (ok && lane == 0) ptx::mbar_arrive(&bars->info_empty[info.idx]);
    info.next(kInfoSlots);
  }
  // Drain: wait until the most recent load issued into every ring stage has landed, so no
  // TMA write can reach this CTA's shared memory after it exits.
  if (lane == 0) {
    for (int s2 = 0; s2 < p.KS; ++s2) {
      const uint32_t back = (uint32_t)s2 + 1u;
      const uint32_t slot = (k.idx + (uint32_t)p.KS - back % (uint32_t)p.KS) % (uint32_t)p.KS;
      const uint32_t ph = (k.idx >= back) ? k.phase : (k.phase ^ 1u);
      if (k.lapped || k.idx >= back) w.wait_drain(&bars->k_full[slot], ph);
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// V loader warp: V chunk tiles into their ring, in the same chunk order.  Each 64-key
// sub-block of V is one box (64 rows x DV/64 slices of 128 B) issued by its own lane.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void vloader_role(const CUtensorMap* tmV, const Params& p, uint8_t* smem, SmemBars* bars,
                             const Waiter& w, int lane) {
  const uint64_t pol_kv = ptx::policy_evict_last();
  uint8_t* vdst0 = smem + p.off_v + lane * C::kVSub;
  const uint32_t vper = (uint32_t)(p.VS / C::kVGroups);  // V stages per PV warp
  Ring info, v0, v1;  // V stage ring of PV warp 0 / 1
  bool ok = true;
  while (ok) {
    int got = 1;
    if (lane == 0) got = w.wait(&bars->info_full[info.idx], info.phase) ? 1 : 0;
    if (!__shfl_sync(0xffffffffu, got, 0)) break;
    const int* inf = info_slot(p, smem, info.idx);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int bkv = inf[kInfBkv];
    const int nch = (nsub + 1) >> 1;
    for (int c = 0; c < nch; ++c) {
      const int nsc = min(2, nsub - 2 * c);
      const bool mine = lane < nsc;
      const int row = mine ? inf[kInfoHdr + 2 * c + lane] : 0;
      const bool g1 = C::kVGroups > 1 && (c & 1);
      const Ring v = g1 ? v1 : v0;
      const uint32_t vs = (g1 ? vper : 0u) + v.idx;
      uint8_t* dst = vdst0 + vs * C::kVStage;
      int go = 1;
      if (lane == 0) {
        go = (!v.lapped || w.wait(&bars->v_empty[vs], v.phase ^ 1u)) ? 1 : 0;
        if (go) ptx::mbar_arrive_expect_tx(&bars->v_full[vs], (uint32_t)(nsc * kSub * C::DV * 2));
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) { ok = false; break; }
      if (mine) ptx::tma_load_4d(dst, tmV, &bars->v_full[vs], 0, row, 0, bkv, pol_kv);
      if (g1) v1.next(vper); else v0.next(vper);
    }
    if (ok && lane == 0) ptx::mbar_arrive(&bars->info_empty[info.idx]);
    info.next(kInfoSlots);
  }
  // Drain: the most recent load of every stage has landed.
  if (lane == 0) {
    for (int wg = 0; wg < C::kVGroups; ++wg) {
      const Ring v = wg ? v1 : v0;
      for (uint32_t back = 1; back <= vper; ++back) {
        const uint32_t slot = (v.idx + vper - back % vper) % vper;
        const uint32_t ph = (v.idx >= back) ? v.phase : (v.phase ^ 1u);
        if (v.lapped || v.idx >= back) w.wait_drain(&bars->v_full[wg * vper + slot], ph);
      }
    }
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// MMA issue.  Each MMA warp issues one stream from one thread, in ring order, with blocking
// (bounded) waits:
//   score warp: S = K_chunk . Q^T into the next score buffer of the chunk's softmax group as
//               soon as the K tile has landed and the group has read that buffer's previous
//               chunk (so it runs ahead of the softmax);
//   PV warp w:  O^T += V_chunk^T . P^T into group w's accumulator as soon as the group's P tile
//               and its V stage are ready.
// Shared-memory descriptors are built once per tile; each 16-wide K step adds a constant.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t byte_off) { return d + (uint64_t)(byte_off >> 4); }

template <class C>
__device__ void mma_s_role(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem, int lane) {
  if (lane == 0) {
    bool ok = true;
    // Error-path test hook: a bounded wait that can only end by running out of time.
    if (p.debug_stall) ok = w.wait(&bars->stall, 0);
    uint32_t ui = 0, ne = 0;
    Ring k;
    uint32_t sc0 = 0, sc1 = 0;  // chunks issued so far for softmax group 0 / 1 (their score buffers)
    const uint32_t k_base = ptx::smem_u32(smem + p.off_k);
    const uint32_t q_base = ptx::smem_u32(smem + p.off_q);
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
        const uint64_t bq0 = ptx::sdesc_sw128(q_base + qs * C::kQBytes, 16, 1024);
        for (int c = 0; c < nch; ++c, k.next((uint32_t)p.KS)) {
          const bool g1 = C::NWG == 2 && (c & 1);
          const uint32_t scnt = g1 ? sc1 : sc0;  // the group's score buffers: its own ring
          const int sslot = (g1 ? C::kSPer : 0) + (int)(scnt % (uint32_t)C::kSPer);
          const uint32_t ks = k.idx;
          const uint64_t a0 = ptx::sdesc_sw128(k_base + ks * C::kKStage, 16, 1024);
          if (scnt >= (uint32_t)C::kSPer &&
              !w.wait(&bars->s_empty[sslot], ((scnt / (uint32_t)C::kSPer) - 1u) & 1u)) { ok = false; break; }
          const long long t0 = clock64();
          if (!w.wait(&bars->k_full[ks], k.phase)) { ok = false; break; }
          t_wait += clock64() - t0;
          ptx::tc_fence_after();
          const uint32_t dS = tmem + C::kTmemS + sslot * C::NCOL;
#pragma unroll
          for (int j = 0; j < C::DQK / 16; ++j) {
            const uint32_t ca = (j >> 2) * C::kKChunkStride + (j & 3) * 32;
            const uint32_t cb = (j >> 2) * C::kQChunk + (j & 3) * 32;
            ptx::umma_bf16(dS, desc_add(a0, ca), desc_add(bq0, cb), C::kIdescS, j > 0 ? 1u : 0u);
          }
          ptx::umma_commit(&bars->k_empty[ks]);
          ptx::umma_commit(&bars->s_full[sslot]);
          if (g1) ++sc1; else ++sc0;
        }
        if (!ok) break;
        ptx::umma_commit(&bars->q_empty[qs]);
        if (p.cyc != nullptr) atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref),
                                        (unsigned long long)t_wait);
        ++ne;
      }
      ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    // Drain: every UMMA issued by this thread completes before TMEM is released.
    ptx::umma_commit(&bars->drain_s);
    w.wait_drain(&bars->drain_s, 0);
  }
  __syncwarp();
}

// PV warp `mine` issues the PV MMAs of softmax group `mine`'s chunks (all chunks with one group),
// so the two groups' PV streams do not queue behind each other.
template <class C>
__device__ void mma_pv_role(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem,
                            int lane, int mine) {
  if (lane == 0) {
    bool ok = true;
    uint32_t ui = 0, ne = 0;
    Ring v;                    // this warp's V stages
    uint32_t kw0 = 0, kw1 = 0;  // chunks so far of softmax group 0 / 1
    const uint32_t vper = (uint32_t)(p.VS / C::kVGroups);
    const uint32_t v_base = ptx::smem_u32(smem + p.off_v);
    const uint32_t p_base = ptx::smem_u32(smem + p.off_p);
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
        // The unit's O^T buffers were last read by the epilogue for unit ne-2.  Every PV warp
        // waits, even one without chunks in this unit: its o_full commit below must not complete
        // the phase of an earlier unit that the other PV warp is still accumulating.
        if (ne >= 2 && !w.wait(&bars->o_empty[ne & 1], ((ne >> 1) - 1) & 1)) break;
        for (int c = mine; c < nch; c += C::kPvWarps) {
          const int wg = c % C::NWG;
          const uint32_t k = wg ? kw1 : kw0;
          const int ps = pslot_of<C::kPSlots, C::NWG>(wg, k);
          const int nsc = min(2, nsub - 2 * c);
          const uint32_t vs = (uint32_t)mine * vper + v.idx;
          const bool first = c < C::NWG;
          const uint64_t a0 = ptx::sdesc_sw128(v_base + vs * C::kVStage, C::kBox, 1024);
          const uint64_t b0 = ptx::sdesc_sw128(p_base + ps * C::kPBytes, 16, 1024);
          const uint32_t dO = tmem + C::kTmemO + (wg * 2 + (ne & 1)) * C::NCOL;
          if (!w.wait(&bars->p_full[ps], pphase_of<C::kPSlots, C::NWG>(k) & 1)) { ok = false; break; }
          const long long t0 = clock64();
          if (!w.wait(&bars->v_full[vs], v.phase)) { ok = false; break; }
          t_wait += clock64() - t0;
          ptx::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j < nsc * 4) {
              const uint32_t ca = (j >> 2) * C::kVSub + (j & 3) * 2048;
              const uint32_t cb = (j >> 2) * C::kPSub + (j & 3) * 32;
              ptx::umma_bf16(dO, desc_add(a0, ca), desc_add(b0, cb), C::kIdescPV, (first && j == 0) ? 0u : 1u);
            }
          }
          ptx::umma_commit(&bars->v_empty[vs]);
          ptx::umma_commit(&bars->pv_done[ps]);
          if (wg) ++kw1; else ++kw0;
          v.next(vper);
        }
        if (!ok) break;
        ptx::umma_commit(&bars->o_full[ne & 1]);
        if (p.cyc != nullptr && mine == 0) {
          const long long tot = clock64() - t_unit0;
          atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref), (unsigned long long)t_wait);
          atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref + 1),
                    (unsigned long long)(tot > t_wait ? tot - t_wait : 0));
        }
        ++ne;
      }
      ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    ptx::umma_commit(&bars->drain_pv[mine]);
    w.wait_drain(&bars->drain_pv[mine], 0);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// Softmax warpgroup `wg` (128 threads): chunk c of every unit with c % NWG == wg.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void softmax_role(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem,
                             int wg) {
  constexpr int NCOL = C::NCOL, TPC = C::kTPC, KPT = C::kKPT, NWG = C::NWG;
  const uint32_t bar_id = kWgBar0 + wg;
  const int i = threadIdx.x - (kSoftWarp0 + 4 * wg) * 32;  // 0..127 inside the warpgroup
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
  const int L = quarter * 32 + lane;               // TMEM lane (key of a chunk / d of O^T)
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  const int col = i / TPC, kg = i - (i / TPC) * TPC;
  float* tr = reinterpret_cast<float*>(smem + p.off_tr + wg * C::kTrBytes);
  float* alpha_s = reinterpret_cast<float*>(smem + p.off_alpha) + wg * NCOL;
  float2* ml = reinterpret_cast<float2*>(smem + p.off_ml) + wg * 2 * NCOL;
  const float sl2 = p.scale_log2;
  const int nrows = p.G * p.BQs;
  const bool col_real = col < nrows;
  const int col_i = col - (col / p.BQs) * p.BQs;
  uint32_t ui = 0, ne = 0, k = 0;  // k: chunks this group has processed (also its score-buffer ring)
  bool dead = false;
  auto wt = [&](uint64_t* bar, uint32_t parity) -> bool {
    if constexpr (NCOL >= 32) return w.wait_inline(bar, parity);
    else return w.wait(bar, parity);
  };

  for (;; ++ui) {
    const int slot = ui % kInfoSlots;
    dead |= !wt(&bars->info_full[slot], (ui / kInfoSlots) & 1);
    if (ptx::named_bar_or(bar_id, 128, dead)) break;
    const int* inf = info_slot(p, smem, slot);
    if (inf[kInfStop]) break;
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int t0 = inf[kInfT0], kend = inf[kInfKend];
    const int nch = (nsub + 1) >> 1;
    if (nch == 0) {
      if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
      continue;
    }
    const int tcol = t0 + col_i;
    // extended visibility only: this row's visible keys, and the keys every row of the unit sees
    int hi_col = tcol, lo_col = 0, hi_all = t0, lo_all = 0;
    if constexpr (C::kExt) {
      hi_col = key_hi(p, tcol);
      lo_col = key_lo(p, tcol);
      hi_all = key_hi(p, t0);
      lo_all = key_lo(p, t0 + p.BQs - 1);
    }
    const uint32_t obase = tmem + lane_addr + C::kTmemO + (wg * 2 + (ne & 1)) * NCOL;
    float m_run = -INFINITY, l_run = 0.f;
    bool first = true, quit = false;

    for (int c = wg; c < nch; c += NWG) {
      const int sslot = wg * C::kSPer + (int)(k % (uint32_t)C::kSPer);
      dead |= !wt(&bars->s_full[sslot], (k / (uint32_t)C::kSPer) & 1u);
      ptx::tc_fence_after();
      {
        const uint32_t saddr = tmem + lane_addr + C::kTmemS + sslot * NCOL;
        float v[NCOL];
#pragma unroll
        for (int h0 = 0; h0 < NCOL; h0 += 16) ptx::tmem_ld16(saddr + h0, *reinterpret_cast<float(*)[16]>(&v[h0]));
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->s_empty[sslot]);  // score buffer may be rewritten
#pragma unroll
        for (int j = 0; j < NCOL; ++j) tr[j * C::kTRS + L] = v[j];
      }
      if (ptx::named_bar_or(bar_id, 128, dead)) { quit = true; break; }

      // This thread's keys of row `col`: key = 4*TPC*q4 + 4*kg + j.
      const int s0 = inf[kInfoHdr + 2 * c];
      const bool has1 = (2 * c + 1) < nsub;
      const int s1 = has1 ? inf[kInfoHdr + 2 * c + 1] : 0;
      bool full;
      if constexpr (C::kExt)
        full = has1 && (max(s0, s1) + kSub - 1 <= hi_all) && (max(s0, s1) + kSub <= kend) && (min(s0, s1) >= lo_all);
      else
        full = has1 && (max(s0, s1) + kSub - 1 <= t0) && (max(s0, s1) + kSub <= kend);
      float sc[KPT];
#pragma unroll
      for (int q4 = 0; q4 < KPT / 4; ++q4) {
        const float4 x = *reinterpret_cast<const float4*>(&tr[col * C::kTRS + 4 * TPC * q4 + 4 * kg]);
        sc[4 * q4 + 0] = x.x;
        sc[4 * q4 + 1] = x.y;
        sc[4 * q4 + 2] = x.z;
        sc[4 * q4 + 3] = x.w;
      }
      if (!full) {
#pragma unroll
        for (int q4 = 0; q4 < KPT / 4; ++q4) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int key = 4 * TPC * q4 + 4 * kg + j;
            const int sb = key >> 6;
            const int kpos = (sb ? s1 : s0) + (key & 63);
            bool valid;
            if constexpr (C::kExt)
              valid = (sb == 0 || has1) && kpos <= hi_col && kpos >= lo_col && kpos < kend;
            else
              valid = (sb == 0 || has1) && kpos <= tcol && kpos < kend;
            if (!valid) sc[4 * q4 + j] = -INFINITY;
          }
        }
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int q = 0; q < KPT; ++q) mx[q & 3] = fmaxf(mx[q & 3], sc[q]);
      float cmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
#pragma unroll
      for (int o = 1; o < TPC; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      const float cmax_x = cmax * sl2;
      float m_use = m_run, alpha = 1.f;
      bool need = false;
      if (first) {
        m_use = cmax_x;
      } else {
        const float m_cand = fmaxf(m_run, cmax_x);
        if (col_real && m_cand > m_run + kRescaleLog2) {
          need = true;
          alpha = (m_run == -INFINITY) ? 0.f : ptx::ex2(m_run - m_cand);
          m_use = m_cand;
        }
      }
      if (kg == 0) alpha_s[col] = alpha;
      const bool any = ptx::named_bar_or(bar_id, 128, need);
      if (any) {
        // Rescale this group's O^T (lane L = d) once its previous PV (chunk k-1) has landed.
        dead |= !wt(&bars->pv_done[pslot_of<C::kPSlots, NWG>(wg, k - 1)], pphase_of<C::kPSlots, NWG>(k - 1) & 1);
        ptx::tc_fence_after();
#pragma unroll
        for (int h0 = 0; h0 < NCOL; h0 += 16) {
          float o[16];
          ptx::tmem_ld16(obase + h0, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= alpha_s[h0 + j];
          ptx::tmem_st16(obase + h0, o);
        }
        ptx::tmem_wait_st();
      }
      // The P buffer was last read by this group's PV of chunk k - NP/NWG.
      const int ps = pslot_of<C::kPSlots, NWG>(wg, k);
      const uint32_t pph = pphase_of<C::kPSlots, NWG>(k);
      if (pph >= 1) dead |= !wt(&bars->pv_done[ps], (pph - 1) & 1);

      const float mref = (m_use == -INFINITY) ? 0.f : m_use;
      float lsum = 0.f;
      uint8_t* pbuf = smem + p.off_p + ps * C::kPBytes;
#pragma unroll
      for (int q4 = 0; q4 < KPT / 4; ++q4) {
        float pr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float s = sc[4 * q4 + j];
          pr[j] = (s == -INFINITY) ? 0.f : ptx::ex2(fmaf(s, sl2, -mref));
          lsum += pr[j];
        }
        const int key0 = 4 * TPC * q4 + 4 * kg;
        const int sb = key0 >> 6, kin = key0 & 63;
        const uint32_t off = (uint32_t)(sb * C::kPSub + (col >> 3) * 1024 + (col & 7) * 128 +
                                        ((((kin >> 3) ^ (col & 7)) << 4) | ((kin & 4) << 1)));
        const __nv_bfloat162 lo = __floats2bfloat162_rn(pr[0], pr[1]);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(pr[2], pr[3]);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&lo);
        pk.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(pbuf + off) = pk;
      }
      l_run = l_run * alpha + lsum;
      m_run = m_use;
      first = false;
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[ps]);
      ++k;
    }
    if (quit) break;

    // Publish this group's running max and sum for the epilogue's merge.  The slot of unit
    // ne was last read by the epilogue for unit ne-2 (it arrives on o_empty after that).
    if (ne >= 2) dead |= !wt(&bars->o_empty[ne & 1], ((ne >> 1) - 1) & 1);
    float lt = l_run;
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o);
    if (kg == 0) ml[(ne & 1) * NCOL + col] = make_float2(m_run, lt);
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&bars->wg_done[ne & 1]);
    if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
    ++ne;
  }
}

// ------------------------------------------------------------------------------------------
// Epilogue warpgroup: merge the softmax groups' partial results, write LSE, store O.
// ------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T to_out(float x);
template <>
__device__ __forceinline__ float to_out<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <class C>
__device__ void epilogue_role(const CUtensorMap* tmO, const Params& p, uint8_t* smem, SmemBars* bars,
                              const Waiter& w, uint32_t tmem) {
  constexpr int NCOL = C::NCOL, NWG = C::NWG;
  using OutT = typename C::OutT;
  const int i = threadIdx.x - kEpiWarp0 * 32;  // 0..127
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int L = quarter * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  float* fac = reinterpret_cast<float*>(smem + p.off_fac);  // [wg][col]: merge weight / sum
  const float2* ml = reinterpret_cast<const float2*>(smem + p.off_ml);
  const int nrows = p.G * p.BQs;
  const float wgt = p.o_weight != nullptr ? __ldg(p.o_weight) : 1.f;  // output weight (NSA gate)
  uint32_t ui = 0, ne = 0, st = 0;
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
    // group q took part iff the unit has a chunk c with c % NWG == q
    bool part[NWG];
#pragma unroll
    for (int q = 0; q < NWG; ++q) part[q] = nch > q;
    if (nch > 0) {
      dead |= !w.wait(&bars->wg_done[ne & 1], (ne >> 1) & 1);
      dead |= !w.wait(&bars->o_full[ne & 1], (ne >> 1) & 1);
      ptx::tc_fence_after();
    }
    if (i < NCOL) {
      // merge: O = sum_w O_w 2^(m_w - M) / sum_w l_w 2^(m_w - M)
      float mw[NWG], lw[NWG], M = -INFINITY;
#pragma unroll
      for (int q = 0; q < NWG; ++q) {
        const float2 v = (nch > 0 && part[q]) ? ml[(q * 2 + (ne & 1)) * NCOL + i] : make_float2(-INFINITY, 0.f);
        mw[q] = v.x;
        lw[q] = v.y;
        M = fmaxf(M, v.x);
      }
      float a[NWG], Ls = 0.f;
#pragma unroll
      for (int q = 0; q < NWG; ++q) {
        a[q] = (mw[q] == -INFINITY || lw[q] == 0.f) ? 0.f : ptx::ex2(mw[q] - M);
        Ls += lw[q] * a[q];
      }
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
      for (int q = 0; q < NWG; ++q) fac[q * NCOL + i] = a[q] * (inv * wgt);
      const int cg = i / p.BQs, ci = i - (i / p.BQs) * p.BQs;
      if (i < nrows && ci < ntok && p.lse != nullptr) {
        const float lse = Ls > 0.f ? (M + log2f(Ls)) * 0.69314718055994530942f : -INFINITY;
        p.lse[((size_t)b * p.Hq + (size_t)kvh * p.G + cg) * p.T + t0 + ci] = lse;
      }
    }
    if (ntok > 0 && i == 0) {  // the store that last read this staging buffer is done
      if (p.out_bufs == 2) ptx::bulk_wait_read<1>(); else ptx::bulk_wait_read<0>();
    }
    ptx::named_bar_sync(kEpiBar, 128);
    if (ntok > 0) {
      OutT* stg = reinterpret_cast<OutT*>(smem + p.off_out + (p.out_bufs == 2 ? (st & 1) : 0u) * C::kOutBytes);
      OutT* dst = stg + (L >> 6) * C::kOutChunkElems + (L & 63);
#pragma unroll
      for (int h0 = 0; h0 < NCOL; h0 += 16) {
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll
        for (int q = 0; q < NWG; ++q) {
          if (part[q]) {
            float t16[16];
            ptx::tmem_ld16(tmem + lane_addr + C::kTmemO + (q * 2 + (ne & 1)) * NCOL + h0, t16);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = fmaf(t16[j], fac[q * NCOL + h0 + j], acc[j]);
          }
        }
        if (L < C::DV) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (h0 + j < nrows) dst[(h0 + j) * 64] = to_out<OutT>(acc[j]);
        }
      }
    }
    if (nch > 0) {
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->o_empty[ne & 1]);  // O^T buffers and ml slot are free
    }
    ptx::fence_proxy_async_smem();
    ptx::named_bar_sync(kEpiBar, 128);
    if (i == 0) {
      if (ntok > 0) {
        OutT* stg = reinterpret_cast<OutT*>(smem + p.off_out + (p.out_bufs == 2 ? (st & 1) : 0u) * C::kOutBytes);
        if (p.o_accum) {
          for (int dc = 0; dc < C::DV / 64; ++dc)
            ptx::tma_reduce_add_4d(tmO, stg + dc * C::kOutChunkElems, dc * 64, t0, kvh * p.G, b);
        } else {
          for (int dc = 0; dc < C::DV / 64; ++dc)
            ptx::tma_store_4d(tmO, stg + dc * C::kOutChunkElems, dc * 64, t0, kvh * p.G, b);
        }
        ptx::bulk_commit();
      }
      ptx::mbar_arrive(&bars->info_empty[slot]);
    }
    if (ntok > 0) ++st;
    if (nch > 0) ++ne;
  }
  if (i == 0) ptx::bulk_wait<0>();
}

// ------------------------------------------------------------------------------------------
template <class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    nsa_sel_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                       const __grid_constant__ Params p) {
  uint8_t* smem = smem_base();
  SmemBars* bars = reinterpret_cast<SmemBars*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kInfoSlots; ++s) {
      ptx::mbar_init(&bars->info_full[s], 1);
      // consumers: score MMA, K and V loaders, epilogue, the softmax groups and the PV warps
      ptx::mbar_init(&bars->info_empty[s], 4 + C::NWG + C::kPvWarps);
    }
    for (int s = 0; s < C::kSSlots; ++s) {
      ptx::mbar_init(&bars->s_full[s], 1);
      ptx::mbar_init(&bars->s_empty[s], 4);
    }
    for (int s = 0; s < kQSlots; ++s) {
      ptx::mbar_init(&bars->q_full[s], 1);
      ptx::mbar_init(&bars->q_empty[s], 1);
    }
    for (int s = 0; s < kMaxPSlots; ++s) {
      ptx::mbar_init(&bars->p_full[s], 4);
      ptx::mbar_init(&bars->pv_done[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&bars->o_full[s], C::kPvWarps);  // each PV warp commits once per unit
      ptx::mbar_init(&bars->wg_done[s], 4 * C::NWG);
      ptx::mbar_init(&bars->o_empty[s], 4);
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
  // Rows of the Q tiles beyond G*BQs are never written by TMA and must read as zero.
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
    mma_s_role<C>(p, smem, bars, w, tmem, lane);
  } else if (warp < kSoftWarp0) {
    epilogue_role<C>(&tmO, p, smem, bars, w, tmem);
  } else if (warp < vloader_warp(C::NWG)) {
    softmax_role<C>(p, smem, bars, w, tmem, (warp - kSoftWarp0) >> 2);
  } else if (warp == vloader_warp(C::NWG)) {
    vloader_role<C>(&tmV, p, smem, bars, w, lane);
  } else if (warp < sched_warp(C::NWG)) {
    mma_pv_role<C>(p, smem, bars, w, tmem, lane, warp - pv_warp(C::NWG));
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
