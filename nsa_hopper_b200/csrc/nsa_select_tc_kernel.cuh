// NSA block selection with the scores on the tensor cores (d = 64 or 128).
//
// Same result as select_kernel (nsa_select_kernel.cuh; reference nsa_reference.py:27-44 with
// compress_kv :5-16 and the group-summed queries :70-71): for every (b, kvh, token t) the top-k
// visible blocks by s(t, nb) = qsum(t) . kblk(nb), highest first, ties to the smaller block, -1
// where fewer than k blocks are visible.
//
// The scores of a unit (128 consecutive tokens of one (b, kvh), all their visible blocks) are
// one tcgen05 GEMM per 128-block N tile: D[128 tokens x 128 blocks] in tensor memory, with
//   A = the group-summed query tile, computed in fp32 by four producer warps and stored into
//       tensor memory as two bf16 parts, hi = bf16(x) and lo = bf16(x - hi);
//   B = the block-key table, written by kblk_kernel<true> as the same two bf16 parts and
//       streamed into shared memory by TMA (128 blocks x 64 dims per 16 KB box, SW128);
//   D = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi, accumulated in fp32 (three UMMAs per K = 16 step).
// The split keeps about 16 bits of both operands, so a score's error is ~2^-16 of the products'
// magnitudes: well inside the ranking tolerance of the reference's fp64 scores (near-ties
// excepted, as for the fp32 FMA kernel), where a single bf16 or tf32 product would not be.
// The top-k runs one token per thread, on the row its tensor-memory lane holds: each thread keeps
// its token's best KCAP (score, block) pairs sorted in registers, and a visible candidate that
// ranks before the last entry is inserted without branches (its rank by KCAP independent
// comparisons, then a select-shift), so no shuffle or ballot sits on the dependency chain.  Two
// warps share every lane quarter: one takes the first 64 blocks of each N tile, the other the
// last 64, and the second hands its list to the first through shared memory at the end of the unit.
//
// Warps: 0-3 producers (query tiles, two tensor-memory buffers so the next unit's tile is built
// while this one is scored), 4-11 top-k (4-7 first halves, 8-11 second halves), 12 TMA loader,
// 13 MMA issuer (owns the 512 TMEM columns).
// Every mbarrier wait is bounded by %globaltimer; one that runs out sets the library's selection
// error word and every role stops (the rows of the launch are then undefined).
#pragma once
#include "nsa_sel_kernel.cuh"
#include "nsa_select_kernel.cuh"

namespace nsa {
namespace seltc {

constexpr int kRows = 128;       // tokens per unit: TMEM lanes, the UMMA's M
constexpr int kNT = 128;         // selection blocks per N tile: the UMMA's N
constexpr int kBStages = 2;      // block-key tile ring
constexpr int kTop0 = 4;         // warps 4-11: top-k
constexpr int kLoadWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kThreads = 448;
constexpr int kMaxCap = 32;      // list capacity (k <= 32)
constexpr uint32_t kPairBar0 = 1;  // named barrier of the two top-k warps of lane quarter q: 1 + q
constexpr int kStageRow = 144;     // bytes per staged query row: 32 dims hi (64 B), lo (64 B), pad

template <int D>
struct Cfg {
  static_assert(D == 64 || D == 128, "tensor-core selection covers d = 64 and 128");
  static constexpr int kSlices = D / 64;           // 64-dim (128-byte) slices of a row
  static constexpr int kBox = kNT * 128;           // one TMA box: 128 blocks x 64 dims bf16 (16 KB)
  static constexpr int kSplit = kSlices * kBox;    // the hi (or lo) part of one N tile
  static constexpr int kStage = 2 * kSplit;        // hi + lo
  static constexpr int kACols = D / 2;             // TMEM columns of one bf16 part of the A tile
  static constexpr int kTmemA = 0;                 // A buffers: [2][hi, lo] x kACols columns
  static constexpr int kTmemD = 4 * kACols;        // D buffers: [2] x kNT fp32 columns
  static constexpr int kTmemCols = 512;
  static_assert(kTmemD + 2 * kNT <= kTmemCols, "tensor memory");
  static constexpr uint32_t kIdesc = ptx::idesc_bf16_f32(128, kNT, false, false);
  // shared memory: B ring | the second-half lists handed to the first halves | barriers
  static constexpr uint32_t kOffB = 0;
  static constexpr uint32_t kOffMerge = kOffB + kBStages * kStage;
  static constexpr uint32_t kMergeBytes = (uint32_t)kRows * kMaxCap * 8;  // [row][entry] x {score, block}
  static constexpr uint32_t kOffStage = kOffMerge + kMergeBytes;             // per producer warp: 32 rows
  static constexpr uint32_t kStageBytes = 4u * 32 * kStageRow;
  static constexpr uint32_t kOffBar = kOffStage + kStageBytes;
};

struct Bars {
  uint64_t a_full[2], a_empty[2], b_full[kBStages], b_empty[kBStages], d_full[2], d_empty[2], drain;
  uint32_t tmem_base;
  int abort_flag;
};

template <int D>
__host__ __device__ constexpr uint32_t smem_bytes() {
  return Cfg<D>::kOffBar + (uint32_t)sizeof(Bars) + 1024;
}

struct Params {
  const __nv_bfloat16* q;
  int32_t* sel;
  int32_t* err;
  int Hq, Hkv, T, G, n_blk, l_prime, topk, n_tiles, n_units;
  unsigned long long timeout_ns;
};

// The unit's visible-block bound: blocks nb < nb_end are visible to some token of the tile.
__device__ __forceinline__ int unit_nb_end(const Params& p, int t0) {
  const int t_last = min(t0 + kRows, p.T) - 1;
  return min(p.n_blk, t_last / p.l_prime + 1);
}

// ---------------------------------------------------------------------------------------------
// Producers (warps 0-3; warp w owns token rows 32w..32w+31 = its TMEM lane quarter): the
// group-summed query rows in fp32, split into bf16 hi / lo and stored as bf16 pairs (dims 2j,
// 2j + 1 in column j).  The loads are coalesced (four lanes per row) and a per-warp staging area
// turns them around so that each thread stores its own row into tensor memory.
// ---------------------------------------------------------------------------------------------
template <int D>
__device__ void producer_role(const Params& p, uint8_t* smem, Bars* bars, const Waiter& w, uint32_t tmem) {
  using C = Cfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
  uint8_t* stage = smem + C::kOffStage + warp * 32 * kStageRow;  // this warp's 32 rows
  // loads: 4 lanes per row (16 bytes = 8 dims each), 8 rows per instruction, so every warp-wide
  // load reads eight whole 64-byte row segments
  const int lrow = lane >> 2, lpart = lane & 3;
  int li = 0;
  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++li) {
    const int bkv = u / p.n_tiles, t0 = (u - bkv * p.n_tiles) * kRows;
    const int b = bkv / p.Hkv, kvh = bkv - b * p.Hkv;
    const int ab = li & 1;
    if (li >= 2 && !w.wait(&bars->a_empty[ab], ((li >> 1) - 1) & 1)) break;
    ptx::tc_fence_after();
    const uint32_t abase = tmem + lane_addr + C::kTmemA + (uint32_t)ab * 2 * C::kACols;
    const size_t head = (size_t)p.T * D / 8;  // uint4 per head
    const uint4* qbase = reinterpret_cast<const uint4*>(p.q + ((size_t)b * p.Hq + (size_t)kvh * p.G) * p.T * D);
#pragma unroll 1
    for (int ch = 0; ch < D / 32; ++ch) {
      // this lane's 8 dims of rows warp*32 + 8*g4 + lrow, g4 = 0..3, summed over the G heads
      float acc[4][8];
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g4][e] = 0.f;
      int rmax = 0;  // row groups inside the sequence
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) rmax += (t0 + warp * 32 + 8 * g4 + lrow < p.T) ? 1 : 0;
#pragma unroll 4
      for (int g = 0; g < p.G; ++g) {  // 16 independent loads in flight per lane
        uint4 x[4];
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          const int t = t0 + warp * 32 + 8 * g4 + lrow;
          x[g4] = g4 < rmax ? __ldg(qbase + (size_t)g * head + ((size_t)t * D + ch * 32) / 8 + lpart)
                            : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&x[g4]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h2[e]);
            acc[g4][2 * e] += f.x;
            acc[g4][2 * e + 1] += f.y;
          }
        }
      }
      // split into bf16 hi / lo and stage the rows (row: 64 B hi | 64 B lo)
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        uint32_t hp[4], lp[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat16 h0 = __float2bfloat16_rn(acc[g4][2 * e]), h1 = __float2bfloat16_rn(acc[g4][2 * e + 1]);
          const __nv_bfloat16 l0 = __float2bfloat16_rn(acc[g4][2 * e] - __bfloat162float(h0));
          const __nv_bfloat16 l1 = __float2bfloat16_rn(acc[g4][2 * e + 1] - __bfloat162float(h1));
          hp[e] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
          lp[e] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        uint8_t* rowp = stage + (8 * g4 + lrow) * kStageRow + lpart * 16;
        *reinterpret_cast<uint4*>(rowp) = make_uint4(hp[0], hp[1], hp[2], hp[3]);
        *reinterpret_cast<uint4*>(rowp + 64) = make_uint4(lp[0], lp[1], lp[2], lp[3]);
      }
      __syncwarp();
      // each thread stores its own row (TMEM lane) into the A buffer's columns of this chunk
      uint32_t hrow[16], lrow16[16];
      const uint8_t* mine = stage + lane * kStageRow;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 hv = *reinterpret_cast<const uint4*>(mine + 16 * c);
        const uint4 lv = *reinterpret_cast<const uint4*>(mine + 64 + 16 * c);
        hrow[4 * c] = hv.x; hrow[4 * c + 1] = hv.y; hrow[4 * c + 2] = hv.z; hrow[4 * c + 3] = hv.w;
        lrow16[4 * c] = lv.x; lrow16[4 * c + 1] = lv.y; lrow16[4 * c + 2] = lv.z; lrow16[4 * c + 3] = lv.w;
      }
      __syncwarp();  // the staging rows are rewritten by the next chunk
      ptx::tmem_st16u(abase + ch * 16, hrow);
      ptx::tmem_st16u(abase + C::kACols + ch * 16, lrow16);
    }
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&bars->a_full[ab]);
  }
}

// ---------------------------------------------------------------------------------------------
// TMA loader (warp 8): the block-key N tiles of every unit, hi and lo parts, into the B ring.
// Lane 2 * part + slice issues that box; rows past the table's end read as zero.
// ---------------------------------------------------------------------------------------------
template <int D>
__device__ void loader_role(const CUtensorMap* tmB, const Params& p, uint8_t* smem, Bars* bars, const Waiter& w) {
  using C = Cfg<D>;
  const int lane = threadIdx.x & 31;
  const uint64_t pol = ptx::policy_evict_last();
  const int part = lane / C::kSlices, sl = lane - part * C::kSlices;
  Ring s;
  bool ok = true;
  for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x) {
    const int bkv = u / p.n_tiles, t0 = (u - bkv * p.n_tiles) * kRows;
    const int n_nt = (unit_nb_end(p, t0) + kNT - 1) / kNT;
    for (int j = 0; j < n_nt; ++j) {
      int go = 1;
      if (lane == 0) {
        go = (!s.lapped || w.wait(&bars->b_empty[s.idx], s.phase ^ 1u)) ? 1 : 0;
        if (go) ptx::mbar_arrive_expect_tx(&bars->b_full[s.idx], (uint32_t)C::kStage);
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) { ok = false; break; }
      if (lane < 2 * C::kSlices)
        ptx::tma_load_4d(smem + C::kOffB + s.idx * C::kStage + part * C::kSplit + sl * C::kBox, tmB,
                         &bars->b_full[s.idx], sl * 64, j * kNT, bkv, part, pol);
      s.next(kBStages);
    }
  }
  if (lane == 0) {  // the most recent load of every stage has landed
    for (int s2 = 0; s2 < kBStages; ++s2) {
      const uint32_t back = (uint32_t)s2 + 1u;
      const uint32_t slot = (s.idx + kBStages - back % kBStages) % kBStages;
      const uint32_t ph = (s.idx >= back) ? s.phase : (s.phase ^ 1u);
      if (s.lapped || s.idx >= back) w.wait_drain(&bars->b_full[slot], ph);
    }
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------------
// MMA issuer (warp 9, one thread): per N tile, D = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi.
// ---------------------------------------------------------------------------------------------
template <int D>
__device__ void mma_role(const Params& p, uint8_t* smem, Bars* bars, const Waiter& w, uint32_t tmem) {
  using C = Cfg<D>;
  if ((threadIdx.x & 31) == 0) {
    Ring s;
    uint32_t dc = 0;
    int li = 0;
    bool ok = true;
    const uint32_t b_base = ptx::smem_u32(smem + C::kOffB);
    for (int u = blockIdx.x; u < p.n_units && ok; u += gridDim.x, ++li) {
      const int bkv = u / p.n_tiles, t0 = (u - bkv * p.n_tiles) * kRows;
      const int n_nt = (unit_nb_end(p, t0) + kNT - 1) / kNT;
      const int ab = li & 1;
      if (!w.wait(&bars->a_full[ab], (li >> 1) & 1)) break;
      ptx::tc_fence_after();
      const uint32_t aH = tmem + C::kTmemA + (uint32_t)ab * 2 * C::kACols, aL = aH + C::kACols;
      for (int j = 0; j < n_nt; ++j, ++dc) {
        const uint32_t db = dc & 1u;
        if (dc >= 2 && !w.wait(&bars->d_empty[db], ((dc >> 1) - 1u) & 1u)) { ok = false; break; }
        if (!w.wait(&bars->b_full[s.idx], s.phase)) { ok = false; break; }
        ptx::tc_fence_after();
        const uint32_t dD = tmem + C::kTmemD + db * kNT;
        const uint64_t bH = ptx::sdesc_sw128(b_base + s.idx * C::kStage, 16, 1024);
        const uint64_t bL = ptx::sdesc_sw128(b_base + s.idx * C::kStage + C::kSplit, 16, 1024);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * C::kBox + (ks & 3) * 32;  // 64-dim slice, 16-dim step
          ptx::umma_bf16_ts(dD, aH + ks * 8, desc_add(bH, off), C::kIdesc, ks > 0 ? 1u : 0u);
          ptx::umma_bf16_ts(dD, aH + ks * 8, desc_add(bL, off), C::kIdesc, 1u);
          ptx::umma_bf16_ts(dD, aL + ks * 8, desc_add(bH, off), C::kIdesc, 1u);
        }
        ptx::umma_commit(&bars->b_empty[s.idx]);
        ptx::umma_commit(&bars->d_full[db]);
        s.next(kBStages);
      }
      if (!ok) break;
      ptx::umma_commit(&bars->a_empty[ab]);
    }
    ptx::umma_commit(&bars->drain);
    w.wait_drain(&bars->drain, 0);
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------------
// Top-k (warps 4-11): thread = token row.  The list is sorted best first; rank order is
// select::ranks_before (higher score, then the smaller block).
// ---------------------------------------------------------------------------------------------
template <int K>
__device__ __forceinline__ void row_insert(float (&lv)[K], int (&li)[K], float v, int vi) {
  // (v, vi) ranks before lv[K-1]: its position is the number of entries that rank before it
  int pos = 0;
#pragma unroll
  for (int i = 0; i < K; ++i) pos += select::ranks_before(lv[i], li[i], v, vi) ? 1 : 0;
#pragma unroll
  for (int i = K - 1; i > 0; --i) {  // downwards, so lv[i - 1] is still the old entry
    lv[i] = i > pos ? lv[i - 1] : (i == pos ? v : lv[i]);
    li[i] = i > pos ? li[i - 1] : (i == pos ? vi : li[i]);
  }
  if (pos == 0) {
    lv[0] = v;
    li[0] = vi;
  }
}

// v[c] for a per-lane index c: a select tree on c's five bits (31 selects, registers only), so a
// lane can visit its own candidates without staging them in shared memory.
__device__ __forceinline__ float pick32(const float (&v)[32], int c) {
  float a[16], b[8], d[4], e[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (c & 1) ? v[2 * i + 1] : v[2 * i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = (c & 2) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = (c & 4) ? b[2 * i + 1] : b[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) e[i] = (c & 8) ? d[2 * i + 1] : d[2 * i];
  return (c & 16) ? e[1] : e[0];
}

template <int D, int K>
__device__ void topk_role(const Params& p, uint8_t* smem, Bars* bars, const Waiter& w, uint32_t tmem) {
  using C = Cfg<D>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3;
  const int half = (warp - kTop0) >> 2;  // 0: blocks 0-63 of each N tile; 1: blocks 64-127
  const int row = quarter * 32 + lane;
  const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
  float2* merge = reinterpret_cast<float2*>(smem + C::kOffMerge) + row * kMaxCap;
  uint32_t dc = 0;
  bool dead = false;
  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x) {
    const int bkv = u / p.n_tiles, t0 = (u - bkv * p.n_tiles) * kRows;
    const int n_nt = (unit_nb_end(p, t0) + kNT - 1) / kNT;
    const int t = t0 + row;
    const int vis = t < p.T ? min(p.n_blk, t / p.l_prime + 1) : 0;  // blocks nb < vis are visible
    float lv[K];
    int li[K];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      lv[i] = -INFINITY;
      li[i] = -1;
    }
    for (int j = 0; j < n_nt; ++j, ++dc) {
      const uint32_t db = dc & 1u;
      dead |= !w.wait(&bars->d_full[db], (dc >> 1) & 1u);
      ptx::tc_fence_after();
#pragma unroll 1
      for (int q2 = 0; q2 < 2; ++q2) {
        float v[32];
        ptx::tmem_ld32(tmem + lane_addr + C::kTmemD + db * kNT + half * 64 + q2 * 32, v);
        ptx::tmem_wait_ld();
        if (q2 == 1) {  // the last load of this N tile by this warp: release the D buffer
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->d_empty[db]);
        }
        // candidates that rank before this row's current k-th entry: a bit mask, then only those
        // are visited, each fetched with pick32 (so the insert code appears once and the hot loop
        // touches no shared memory)
        const int nb0 = j * kNT + half * 64 + q2 * 32;
        const float thr_v = lv[K - 1];
        const int thr_i = li[K - 1];
        uint32_t m = 0;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          v[c] = nb0 + c < vis ? v[c] : -INFINITY;
          m |= select::ranks_before(v[c], nb0 + c, thr_v, thr_i) ? (1u << c) : 0u;
        }
        while (m != 0u) {
          const int c = __ffs(m) - 1;
          m &= m - 1u;
          const float x = pick32(v, c);
          if (select::ranks_before(x, nb0 + c, lv[K - 1], li[K - 1])) row_insert<K>(lv, li, x, nb0 + c);
        }
      }
    }
    // the second half's list joins the first half's, then the first half writes the row
    if (half == 1) {
#pragma unroll
      for (int i = 0; i < K; ++i) merge[i] = make_float2(lv[i], __int_as_float(li[i]));
    }
    ptx::named_bar_sync(kPairBar0 + quarter, 64);
    if (half == 0) {
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const float2 e = merge[i];
        const int ei = __float_as_int(e.y);
        if (select::ranks_before(e.x, ei, lv[K - 1], li[K - 1])) row_insert<K>(lv, li, e.x, ei);
      }
      if (!dead && t < p.T) {
        int32_t* out = p.sel + ((size_t)bkv * p.T + t) * p.topk;
#pragma unroll
        for (int i = 0; i < K; ++i)
          if (i < p.topk) out[i] = lv[i] == -INFINITY ? -1 : li[i];
      }
    }
    // the merge slots are rewritten next unit; both warps of the pair leave together
    if (ptx::named_bar_or(kPairBar0 + quarter, 64, dead)) break;
  }
}

template <int D, int K>
__global__ void __launch_bounds__(kThreads, 1)
    select_tc_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ Params p) {
  using C = Cfg<D>;
  uint8_t* smem = smem_base();
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(&bars->a_full[s], 4);
      ptx::mbar_init(&bars->a_empty[s], 1);
      ptx::mbar_init(&bars->d_full[s], 1);
      ptx::mbar_init(&bars->d_empty[s], 8);  // both top-k warps of every lane quarter
    }
    for (int s = 0; s < kBStages; ++s) {
      ptx::mbar_init(&bars->b_full[s], 1);
      ptx::mbar_init(&bars->b_empty[s], 1);
    }
    ptx::mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kLoadWarp && (threadIdx.x & 31) == 0) ptx::prefetch_tmap(&tmB);
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(&bars->tmem_base, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const Waiter w{&bars->abort_flag, p.err, p.timeout_ns};
  if (warp < kTop0) producer_role<D>(p, smem, bars, w, tmem);
  else if (warp < kLoadWarp) topk_role<D, K>(p, smem, bars, w, tmem);
  else if (warp == kLoadWarp) loader_role<D>(&tmB, p, smem, bars, w);
  else mma_role<D>(p, smem, bars, w, tmem);
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace seltc
}  // namespace nsa
