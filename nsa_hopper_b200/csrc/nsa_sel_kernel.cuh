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
//    gathered K/V blocks of that head are re-read from L2 rather than HBM.  K/V loads
//    carry an L2 evict_last hint, the streaming Q loads evict_first.
//  * Warp 0 (loader) turns a unit's selection row into a list of 64-key sub-blocks
//    (dedupe, padding, causal and range clipping) in a shared-memory "info" ring and issues
//    TMA tensor loads: the unit's Q tile and, per chunk of two sub-blocks (128 keys), a K
//    tile and a V tile into two mbarrier-driven rings.
//  * Warp 1 (MMA) issues tcgen05 UMMAs from one thread in swap-AB form so the 128 keys of
//    a chunk are the M=128 dimension and the G*BQ query rows are N (16..128):
//        S^T[keys x rows]  = K_chunk[keys x d_qk] . Q^T          (A K-major, B K-major)
//        O^T[d_v x rows]  += V_chunk^T[d_v x keys] . P^T          (A MN-major, B K-major)
//    S^T and O^T accumulate in TMEM (S double-buffered, O double-buffered per unit).
//  * Warps 2-5 (softmax warpgroup) read S^T from TMEM, transpose it through shared memory
//    so each thread owns 16 keys of one query row, mask, do an exp2 online softmax with a
//    warp-shuffle row max/sum and lazy O rescaling (only when the running max grows by
//    more than 2^8), write P^T as bf16 in the UMMA K-major SW128 layout, and finally
//    normalise O^T, write LSE and store O with a TMA tensor store.
//
// Every mbarrier wait is bounded by %globaltimer; a wait that runs out sets an error bit,
// all roles stop, in-flight TMA loads/stores and UMMAs are drained and TMEM is freed.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include "ptx.cuh"

namespace nsa {

constexpr int kSub = 64;         // keys per sub-block (one TMA box of rows)
constexpr int kChunk = 128;      // keys per chunk = M of the UMMAs
constexpr int kInfoSlots = 4;    // depth of the unit-info ring
constexpr int kInfoHdr = 16;     // ints of header per info slot
constexpr int kMaxStages = 8;    // upper bound on K and V ring depth
constexpr int kThreads = 192;    // loader warp + MMA warp + 4 softmax warps
constexpr int kLoaderWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kSoftmaxWarp0 = 2;
constexpr uint32_t kWgBar = 1;   // named barrier of the softmax warpgroup
constexpr float kRescaleLog2 = 8.0f;
constexpr int kDevErrTimeout = 1;

// Info-slot header fields.
enum : int { kInfNsub = 0, kInfT0, kInfNtok, kInfKend, kInfB, kInfKvh, kInfBkv, kInfSeq0, kInfRef };

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
  uint32_t off_k, off_v, off_q, off_p, off_out, off_tr, off_alpha, off_inv, off_info, off_bar;
  int stage_alias;  // 1: the output staging tile lives in the transpose buffer (single buffer)
  int debug_stall;  // 1: the MMA warp first waits on a barrier nothing arrives on (error-path test)
};

struct SmemBars {
  uint64_t info_full[kInfoSlots], info_empty[kInfoSlots];
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kMaxStages], k_empty[kMaxStages];
  uint64_t v_full[kMaxStages], v_empty[kMaxStages];
  uint64_t s_full[2], p_full[2], pv_done[2], o_empty[2];
  uint64_t drain;
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

template <int DQK_, int DV_, int NCOL_, typename OutT_>
struct Cfg {
  static constexpr int DQK = DQK_, DV = DV_, NCOL = NCOL_;
  using OutT = OutT_;
  static_assert(DQK % 64 == 0 && DQK >= 64 && DQK <= 256, "d_qk must be 64..256 in steps of 64");
  static_assert(DV == 64 || DV == 128, "d_v must be 64 or 128");
  static_assert(NCOL == 16 || NCOL == 32 || NCOL == 64, "N must be 16/32/64");
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
  static constexpr int kTPC = 128 / NCOL;                   // softmax threads per query row
  static constexpr int kKPT = NCOL;                         // keys per softmax thread per chunk
  static constexpr int kTRS = kChunk + 4;                   // transpose row stride (floats)
  static constexpr int kTrBytes = NCOL * kTRS * 4;
  static constexpr int kOutChunkElems = NCOL * 64;
  static constexpr int kOutBytes = (DV / 64) * kOutChunkElems * (int)sizeof(OutT);
  static constexpr int kTmemCols = ceil_pow2_32(4 * NCOL);
  static constexpr uint32_t kIdescS = ptx::idesc_bf16_f32(128, NCOL, false, false);
  static constexpr uint32_t kIdescPV = ptx::idesc_bf16_f32(128, NCOL, true, false);
};

// Shared-memory layout (byte offsets from a 1024-aligned base); identical on host and device.
struct SmemLayout {
  uint32_t off_k, off_v, off_q, off_p, off_out, off_tr, off_alpha, off_inv, off_info, off_bar, total;
};
// With `alias`, the (single) output staging tile reuses the transpose buffer, which is idle
// between a unit's last chunk and the next unit's first chunk.
template <class C>
__host__ __device__ inline SmemLayout smem_layout(int KS, int VS, int maxsub, int alias) {
  static_assert(C::kOutBytes <= C::kTrBytes, "staging tile must fit in the transpose buffer");
  SmemLayout s{};
  uint32_t o = 0;
  s.off_k = o; o += (uint32_t)KS * C::kKStage;
  s.off_v = o; o += (uint32_t)VS * C::kVStage;
  s.off_q = o; o += 2u * C::kQBytes;
  o = align_up(o, 1024);
  s.off_p = o; o += 2u * C::kPBytes;
  o = align_up(o, 1024);
  s.off_tr = o; o += C::kTrBytes;
  o = align_up(o, 128);
  if (alias) {
    s.off_out = s.off_tr;
  } else {
    s.off_out = o; o += 2u * C::kOutBytes;
  }
  s.off_alpha = o; o += 4u * C::NCOL;
  s.off_inv = o; o += 4u * C::NCOL;
  s.off_info = o; o += 4u * kInfoSlots * (kInfoHdr + maxsub);
  o = align_up(o, 16);
  s.off_bar = o; o += (uint32_t)sizeof(SmemBars);
  s.total = o + 1024;  // slack to align the dynamic shared-memory base to 1024 B
  return s;
}

// A bounded mbarrier wait.  Returns false if the CTA is aborting or the wait ran out of time
// (then it raises the abort flag and the device error bit).
struct Waiter {
  int* abort_flag;
  int32_t* err;
  unsigned long long timeout_ns;

  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity) const {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 32; ++i)
        if (ptx::mbar_try_wait(bar, parity)) return true;
      if (*(volatile int*)abort_flag) return false;
      if (ptx::globaltimer() - t0 > timeout_ns) {
        *(volatile int*)abort_flag = 1;
        if (err != nullptr) atomicOr(err, kDevErrTimeout);
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
__device__ int build_unit_info(const Params& p, int u, int* inf, int lane) {
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
  int seq0 = 0, kend = p.T;
  if (p.cu_seqlens != nullptr && ntok > 0) {
    int lo = 0, hi = p.n_seq;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(p.cu_seqlens + mid) <= t0) lo = mid; else hi = mid;
    }
    seq0 = __ldg(p.cu_seqlens + lo);
    kend = __ldg(p.cu_seqlens + lo + 1);
  }
  const int lim = min(t0 + ntok - 1, kend - 1);  // last key position any row of the unit may see
  const int nblk = (kend - seq0 + p.LP - 1) / p.LP;
  const int spb = p.LP / kSub;
  const int32_t* row = p.sel + ((size_t)bkv * p.NQB + qb) * p.KSEL;
  int count = 0;
  if (ntok > 0) {
    for (int base = 0; base < p.KSEL; base += 32) {
      const int j = base + lane;
      const int idx = (j < p.KSEL) ? __ldg(row + j) : -1;
      bool valid = idx >= 0 && idx < nblk && (seq0 + idx * p.LP) <= lim;
      if (valid) {
        for (int k2 = 0; k2 < j; ++k2)
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
  }
  return count;
}

// ------------------------------------------------------------------------------------------
// Loader warp: info ring + TMA loads of Q tiles and K/V chunk tiles.
// ------------------------------------------------------------------------------------------
template <class C>
__device__ void loader_role(const CUtensorMap* tmQ, const CUtensorMap* tmK, const CUtensorMap* tmV,
                            const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, int lane) {
  const uint64_t pol_kv = ptx::policy_evict_last();
  const uint64_t pol_q = ptx::policy_evict_first();
  uint32_t ui = 0, qc = 0, kc = 0, vc = 0;  // units seen; Q, K and V tile loads issued
  bool ok = true;
  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ui) {
    const int slot = ui % kInfoSlots;
    if (ui >= (uint32_t)kInfoSlots) {
      int r = 1;
      if (lane == 0) r = w.wait(&bars->info_empty[slot], ((ui / kInfoSlots) - 1) & 1) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, r, 0) != 0;
      if (!ok) break;
    }
    int* inf = info_slot(p, smem, slot);
    const int nsub = build_unit_info(p, u, inf, lane);
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&bars->info_full[slot]);
    if (nsub == 0) continue;
    int r = 1;
    if (lane == 0) {
      const int t0 = inf[kInfT0], b = inf[kInfB], kvh = inf[kInfKvh], bkv = inf[kInfBkv];
      const int qbuf = qc & 1;
      if (qc >= 2 && !w.wait(&bars->q_empty[qbuf], ((qc >> 1) - 1) & 1)) {
        r = 0;
      } else {
        uint8_t* qdst = smem + p.off_q + qbuf * C::kQBytes;
        ptx::mbar_arrive_expect_tx(&bars->q_full[qbuf], (uint32_t)(C::DQK * p.BQs * p.G * 2));
        for (int cc = 0; cc < C::DQK / 64; ++cc)
          ptx::tma_load_4d(qdst + cc * C::kQChunk, tmQ, &bars->q_full[qbuf], cc * 64, t0, kvh * p.G, b, pol_q);
        ++qc;
      }
      const int nch = (nsub + 1) >> 1;
      for (int c = 0; c < nch && r; ++c) {
        const int nsc = min(2, nsub - 2 * c);
        const int ks = (int)(kc % (uint32_t)p.KS);
        if (kc >= (uint32_t)p.KS && !w.wait(&bars->k_empty[ks], ((kc / p.KS) - 1) & 1)) { r = 0; break; }
        uint8_t* kdst = smem + p.off_k + ks * C::kKStage;
        ptx::mbar_arrive_expect_tx(&bars->k_full[ks], (uint32_t)(nsc * kSub * C::DQK * 2));
        for (int j = 0; j < nsc; ++j) {
          const int row = inf[kInfoHdr + 2 * c + j];
          for (int cc = 0; cc < C::DQK / 64; ++cc)
            ptx::tma_load_3d(kdst + cc * C::kKChunkStride + j * C::kBox, tmK, &bars->k_full[ks], cc * 64, row, bkv,
                             pol_kv);
        }
        ++kc;
        const int vs = (int)(vc % (uint32_t)p.VS);
        if (vc >= (uint32_t)p.VS && !w.wait(&bars->v_empty[vs], ((vc / p.VS) - 1) & 1)) { r = 0; break; }
        uint8_t* vdst = smem + p.off_v + vs * C::kVStage;
        ptx::mbar_arrive_expect_tx(&bars->v_full[vs], (uint32_t)(nsc * kSub * C::DV * 2));
        for (int j = 0; j < nsc; ++j) {
          const int row = inf[kInfoHdr + 2 * c + j];
          for (int cc = 0; cc < C::DV / 64; ++cc)
            ptx::tma_load_3d(vdst + j * C::kVSub + cc * C::kBox, tmV, &bars->v_full[vs], cc * 64, row, bkv, pol_kv);
        }
        ++vc;
      }
    }
    ok = __shfl_sync(0xffffffffu, r, 0) != 0;
    qc = __shfl_sync(0xffffffffu, qc, 0);
    kc = __shfl_sync(0xffffffffu, kc, 0);
    vc = __shfl_sync(0xffffffffu, vc, 0);
    if (!ok) break;
  }
  // Drain: wait until the most recent load issued into every ring stage has landed, so no
  // TMA write can reach this CTA's shared memory after it exits.
  if (lane == 0) {
    for (uint32_t s = 0; s < (uint32_t)p.KS; ++s)
      if (kc > s) w.wait_drain(&bars->k_full[s], ((s + ((kc - 1 - s) / p.KS) * p.KS) / p.KS) & 1);
    for (uint32_t s = 0; s < (uint32_t)p.VS; ++s)
      if (vc > s) w.wait_drain(&bars->v_full[s], ((s + ((vc - 1 - s) / p.VS) * p.VS) / p.VS) & 1);
    for (uint32_t s = 0; s < 2; ++s)
      if (qc > s) w.wait_drain(&bars->q_full[s], ((s + ((qc - 1 - s) / 2) * 2) / 2) & 1);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// MMA warp (lane 0 issues): S_g = K_g . Q^T, then PV_{g-1}, keeping one chunk of slack so
// the softmax of chunk g-1 overlaps the score MMA of chunk g.
// ------------------------------------------------------------------------------------------
struct PendPV {
  int valid, g, obuf, ne, first, nsc, vc;
};

template <class C>
__device__ bool issue_pv(const PendPV& pd, const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w,
                         uint32_t tmem, long long& t_wait) {
  if (!w.wait(&bars->p_full[pd.g & 1], (pd.g >> 1) & 1)) return false;
  if (pd.first && pd.ne >= 2 && !w.wait(&bars->o_empty[pd.obuf], ((pd.ne >> 1) - 1) & 1)) return false;
  const int vs = pd.vc % p.VS;
  const long long t0 = clock64();
  if (!w.wait(&bars->v_full[vs], (pd.vc / p.VS) & 1)) return false;
  t_wait += clock64() - t0;
  ptx::tc_fence_after();
  const uint32_t vaddr = ptx::smem_u32(smem + p.off_v + vs * C::kVStage);
  const uint32_t paddr = ptx::smem_u32(smem + p.off_p + (pd.g & 1) * C::kPBytes);
  const uint32_t dO = tmem + 2 * C::NCOL + pd.obuf * C::NCOL;
  for (int j = 0; j < pd.nsc * 4; ++j) {
    const int sb = j >> 2, kk = j & 3;
    const uint64_t a = ptx::sdesc_sw128(vaddr + sb * C::kVSub + kk * 2048, C::kBox, 1024);
    const uint64_t bp = ptx::sdesc_sw128(paddr + sb * C::kPSub + kk * 32, 16, 1024);
    ptx::umma_bf16(dO, a, bp, C::kIdescPV, (pd.first && j == 0) ? 0u : 1u);
  }
  ptx::umma_commit(&bars->v_empty[vs]);
  ptx::umma_commit(&bars->pv_done[pd.g & 1]);
  return true;
}

template <class C>
__device__ void mma_role(const Params& p, uint8_t* smem, SmemBars* bars, const Waiter& w, uint32_t tmem, int lane) {
  if (lane == 0) {
    uint32_t ui = 0, ne = 0, kc = 0, vc = 0, g = 0;
    PendPV pend{0, 0, 0, 0, 0, 0, 0};
    bool ok = true;
    long long t_wait = 0;
    // Error-path test hook: a bounded wait that can only end by running out of time.
    if (p.debug_stall) ok = w.wait(&bars->stall, 0);
    for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x, ++ui) {
      const int slot = ui % kInfoSlots;
      if (!w.wait(&bars->info_full[slot], (ui / kInfoSlots) & 1)) { ok = false; break; }
      const int* inf = info_slot(p, smem, slot);
      const int nsub = min(inf[kInfNsub], p.maxsub);
      const int ref = inf[kInfRef];
      const int nch = (nsub + 1) >> 1;
      if (nch == 0) {
        // Nothing to overlap with: retire the previous unit's last PV now, so its epilogue
        // (and the info slot it holds) never waits on units further ahead.
        if (pend.valid) {
          if (!issue_pv<C>(pend, p, smem, bars, w, tmem, t_wait)) { ok = false; break; }
          pend.valid = 0;
        }
        ptx::mbar_arrive(&bars->info_empty[slot]);
        continue;
      }
      const long long t_unit0 = clock64();
      t_wait = 0;
      const int qbuf = ne & 1;
      if (!w.wait(&bars->q_full[qbuf], (ne >> 1) & 1)) { ok = false; break; }
      const uint32_t qaddr = ptx::smem_u32(smem + p.off_q + qbuf * C::kQBytes);
      for (int c = 0; c < nch; ++c) {
        const int nsc = min(2, nsub - 2 * c);
        const int ks = kc % p.KS;
        const long long tw = clock64();
        if (!w.wait(&bars->k_full[ks], (kc / p.KS) & 1)) { ok = false; break; }
        t_wait += clock64() - tw;
        ptx::tc_fence_after();
        const uint32_t kaddr = ptx::smem_u32(smem + p.off_k + ks * C::kKStage);
        const uint32_t dS = tmem + (g & 1) * C::NCOL;
#pragma unroll
        for (int j = 0; j < C::DQK / 16; ++j) {
          const int cc = j >> 2, kk = j & 3;
          const uint64_t a = ptx::sdesc_sw128(kaddr + cc * C::kKChunkStride + kk * 32, 16, 1024);
          const uint64_t bq = ptx::sdesc_sw128(qaddr + cc * C::kQChunk + kk * 32, 16, 1024);
          ptx::umma_bf16(dS, a, bq, C::kIdescS, j > 0 ? 1u : 0u);
        }
        ptx::umma_commit(&bars->k_empty[ks]);
        ptx::umma_commit(&bars->s_full[g & 1]);
        if (c == nch - 1) ptx::umma_commit(&bars->q_empty[qbuf]);
        ++kc;
        if (pend.valid && !issue_pv<C>(pend, p, smem, bars, w, tmem, t_wait)) { ok = false; break; }
        pend = PendPV{1, (int)g, (int)(ne & 1), (int)ne, c == 0 ? 1 : 0, nsc, (int)vc};
        ++vc;
        ++g;
      }
      if (!ok) break;
      ptx::mbar_arrive(&bars->info_empty[slot]);
      ++ne;
      if (p.cyc != nullptr) {
        const long long tot = clock64() - t_unit0;
        atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref), (unsigned long long)t_wait);
        atomicAdd(reinterpret_cast<unsigned long long*>(p.cyc + 2 * (size_t)ref + 1),
                  (unsigned long long)(tot > t_wait ? tot - t_wait : 0));
      }
    }
    if (ok && pend.valid) issue_pv<C>(pend, p, smem, bars, w, tmem, t_wait);
    // Drain: every UMMA issued by this thread completes before TMEM is released.
    ptx::umma_commit(&bars->drain);
    w.wait_drain(&bars->drain, 0);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------------------
// Softmax warpgroup.
// ------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T to_out(float x);
template <>
__device__ __forceinline__ float to_out<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <class C>
__device__ void softmax_role(const CUtensorMap* tmO, const Params& p, uint8_t* smem, SmemBars* bars,
                             const Waiter& w, uint32_t tmem) {
  constexpr int NCOL = C::NCOL, TPC = C::kTPC, KPT = C::kKPT;
  using OutT = typename C::OutT;
  const int i = threadIdx.x - kSoftmaxWarp0 * 32;  // 0..127 inside the warpgroup
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;                    // TMEM lane quarter this warp may access
  const int L = quarter * 32 + lane;               // TMEM lane (key of a chunk / d of O^T)
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  const int col = i / TPC, kg = i - (i / TPC) * TPC;
  float* tr = reinterpret_cast<float*>(smem + p.off_tr);
  float* alpha_s = reinterpret_cast<float*>(smem + p.off_alpha);
  float* inv_s = reinterpret_cast<float*>(smem + p.off_inv);
  const float sl2 = p.scale_log2;
  const int nrows = p.G * p.BQs;
  const bool col_real = col < nrows;
  const int col_g = col / p.BQs, col_i = col - (col / p.BQs) * p.BQs;
  uint32_t ui = 0, ne = 0, g = 0, st = 0;
  bool dead = false, quit = false;

  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ui) {
    const int slot = ui % kInfoSlots;
    dead |= !w.wait(&bars->info_full[slot], (ui / kInfoSlots) & 1);
    if (p.stage_alias && i == 0) ptx::bulk_wait_read<0>();  // staging (= transpose buffer) is free
    if (ptx::named_bar_or(kWgBar, 128, dead)) break;
    const int* inf = info_slot(p, smem, slot);
    const int nsub = min(inf[kInfNsub], p.maxsub);
    const int t0 = inf[kInfT0], ntok = inf[kInfNtok], kend = inf[kInfKend];
    const int b = inf[kInfB], kvh = inf[kInfKvh];
    const int nch = (nsub + 1) >> 1;
    const int tcol = t0 + col_i;
    const bool col_live = col_real && col_i < ntok;
    const uint32_t obase = tmem + lane_addr + 2 * NCOL + (ne & 1) * NCOL;
    float m_run = -INFINITY, l_run = 0.f;

    for (int c = 0; c < nch; ++c) {
      dead |= !w.wait(&bars->s_full[g & 1], (g >> 1) & 1);
      ptx::tc_fence_after();
      {
        const uint32_t saddr = tmem + lane_addr + (g & 1) * NCOL;
#pragma unroll
        for (int h0 = 0; h0 < NCOL; h0 += 16) {
          float v[16];
          ptx::tmem_ld16(saddr + h0, v);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) tr[(h0 + j) * C::kTRS + L] = v[j];
        }
      }
      if (ptx::named_bar_or(kWgBar, 128, dead)) { quit = true; break; }

      // This thread's keys of row `col`: key = 4*TPC*q4 + 4*kg + j.
      const int s0 = inf[kInfoHdr + 2 * c];
      const bool has1 = (2 * c + 1) < nsub;
      const int s1 = has1 ? inf[kInfoHdr + 2 * c + 1] : 0;
      const bool full = has1 && (max(s0, s1) + kSub - 1 <= t0) && (max(s0, s1) + kSub <= kend);
      float sc[KPT];
#pragma unroll
      for (int q4 = 0; q4 < KPT / 4; ++q4) {
        const float4 x = *reinterpret_cast<const float4*>(&tr[col * C::kTRS + 4 * TPC * q4 + 4 * kg]);
        sc[4 * q4 + 0] = x.x;
        sc[4 * q4 + 1] = x.y;
        sc[4 * q4 + 2] = x.z;
        sc[4 * q4 + 3] = x.w;
      }
      float cmax = -INFINITY;
#pragma unroll
      for (int q4 = 0; q4 < KPT / 4; ++q4) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int key = 4 * TPC * q4 + 4 * kg + j;
          if (!full) {
            const int sb = key >> 6;
            const int kpos = (sb ? s1 : s0) + (key & 63);
            const bool valid = (sb == 0 || has1) && kpos <= tcol && kpos < kend;
            if (!valid) sc[4 * q4 + j] = -INFINITY;
          }
          cmax = fmaxf(cmax, sc[4 * q4 + j]);
        }
      }
#pragma unroll
      for (int o = 1; o < TPC; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      const float cmax_x = cmax * sl2;
      float m_use = m_run, alpha = 1.f;
      bool need = false;
      if (c == 0) {
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
      const bool any = ptx::named_bar_or(kWgBar, 128, need);
      if (any) {
        // Rescale O^T (lane L = d) by the per-row factors once the previous PV has landed.
        dead |= !w.wait(&bars->pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1);
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
      // P buffer (g & 1) was read by PV_{g-2}.
      if (g >= 2) dead |= !w.wait(&bars->pv_done[g & 1], ((g - 2) >> 1) & 1);

      const float mref = (m_use == -INFINITY) ? 0.f : m_use;
      float lsum = 0.f;
      uint8_t* pbuf = smem + p.off_p + (g & 1) * C::kPBytes;
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
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[g & 1]);
      ++g;
    }
    if (quit) break;

    // ---- epilogue: normalise, LSE, O store
    if (nch > 0) {
      dead |= !w.wait(&bars->pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1);
      ptx::tc_fence_after();
    }
    float lt = l_run;
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o);
    if (kg == 0) {
      inv_s[col] = lt > 0.f ? 1.f / lt : 0.f;
      if (col_live && p.lse != nullptr) {
        const float lse = lt > 0.f ? (m_run + log2f(lt)) * 0.69314718055994530942f : -INFINITY;
        p.lse[((size_t)b * p.Hq + (size_t)kvh * p.G + col_g) * p.T + tcol] = lse;
      }
    }
    if (ntok > 0) {
      if (i == 0) ptx::bulk_wait_read<1>();  // the TMA store that last read this staging buffer is done
      ptx::named_bar_sync(kWgBar, 128);
      OutT* stg = reinterpret_cast<OutT*>(smem + p.off_out + (p.stage_alias ? 0u : (st & 1) * C::kOutBytes));
      OutT* dst = stg + (L >> 6) * C::kOutChunkElems + (L & 63);
#pragma unroll
      for (int h0 = 0; h0 < NCOL; h0 += 16) {
        float t16[16];
        if (nch > 0) {
          ptx::tmem_ld16(obase + h0, t16);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) t16[j] = 0.f;
        }
        if (L < C::DV) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (h0 + j < nrows) dst[(h0 + j) * 64] = to_out<OutT>(t16[j] * inv_s[h0 + j]);
        }
      }
      if (nch > 0) {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->o_empty[ne & 1]);
      }
      ptx::fence_proxy_async_smem();
      ptx::named_bar_sync(kWgBar, 128);
      if (i == 0) {
        for (int dc = 0; dc < C::DV / 64; ++dc)
          ptx::tma_store_4d(tmO, stg + dc * C::kOutChunkElems, dc * 64, t0, kvh * p.G, b);
        ptx::bulk_commit();
      }
      ++st;
    }
    if (i == 0) ptx::mbar_arrive(&bars->info_empty[slot]);
    if (nch > 0) ++ne;
  }
  if (i == 0) ptx::bulk_wait<0>();
}

// ------------------------------------------------------------------------------------------
template <class C>
__global__ void __launch_bounds__(kThreads, 1)
    nsa_sel_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                       const __grid_constant__ Params p) {
  uint8_t* smem = smem_base();
  SmemBars* bars = reinterpret_cast<SmemBars*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kInfoSlots; ++s) {
      ptx::mbar_init(&bars->info_full[s], 1);
      ptx::mbar_init(&bars->info_empty[s], 2);
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&bars->q_full[s], 1);
      ptx::mbar_init(&bars->q_empty[s], 1);
      ptx::mbar_init(&bars->s_full[s], 1);
      ptx::mbar_init(&bars->p_full[s], 4);
      ptx::mbar_init(&bars->pv_done[s], 1);
      ptx::mbar_init(&bars->o_empty[s], 4);
    }
    for (int s = 0; s < kMaxStages; ++s) {
      ptx::mbar_init(&bars->k_full[s], 1);
      ptx::mbar_init(&bars->k_empty[s], 1);
      ptx::mbar_init(&bars->v_full[s], 1);
      ptx::mbar_init(&bars->v_empty[s], 1);
    }
    ptx::mbar_init(&bars->drain, 1);
    ptx::mbar_init(&bars->stall, 1);
    bars->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  // Rows of the Q tiles beyond G*BQs are never written by TMA and must read as zero.
  for (int idx = threadIdx.x; idx < 2 * C::kQBytes / 16; idx += kThreads)
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
    loader_role<C>(&tmQ, &tmK, &tmV, p, smem, bars, w, lane);
  } else if (warp == kMmaWarp) {
    mma_role<C>(p, smem, bars, w, tmem, lane);
  } else {
    softmax_role<C>(&tmO, p, smem, bars, w, tmem);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace nsa
