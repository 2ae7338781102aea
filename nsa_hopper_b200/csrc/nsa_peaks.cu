// Microbenchmarks of the on-chip ceilings that bound the selected-branch forward's dataflow
// (bench.py --stage peaks, and the denominators of the bench line's roofline).  Measurement
// code only: libnsa_peaks.so holds these kernels and nothing on the product path calls them.
//
// The dataflow being bounded (nsa_sel_kernel.cuh, per-token selection, d_qk = d_v = 128): every
// 128-key chunk is gathered from L2 into shared memory by TMA as four 8 KB K boxes (64 keys x 64
// dims, SW128) and two 16 KB V boxes (64 keys x 128 dims), then read by the tensor core as the A
// operand of 8 score UMMAs (M = 128 keys, N = 16 query rows, K = 16) and 8 PV UMMAs.  The kernels
// here keep exactly that traffic and drop everything else:
//   mode 0 (gather): the K and V loader warps run the same rings (3 K stages; 2 V stages, one per
//                    PV issuer) and consumers release each stage as soon as it lands: the
//                    L2 -> SMEM ceiling of this gather;
//   mode 1 (gather + UMMA): the consumers are the product kernel's three MMA issuers: one thread
//                    issues every chunk's 8 score UMMAs on the landed K tile, and one thread per
//                    softmax group (even / odd chunks) issues the chunk's 8 PV UMMAs on its landed V
//                    stage, each releasing its stage with tcgen05.commit: the ceiling of the whole
//                    data path without the softmax and epilogue;
//   mode 2 (UMMA only): the same three issuers and UMMAs on resident tiles: the tensor-pipe cost
//                    of one chunk at N = 16;
//   mode 3 / 4:      modes 1 / 2 with the score UMMAs' A operand (the K tile) first copied into
//                    tensor memory by tcgen05.cp (one 128 x 32 B copy per K = 16 step) and read from
//                    there by the UMMA: the same bytes leave shared memory once, by the copy engine.
// Block positions are pseudo-random per (CTA, chunk, sub-block), and all CTAs walk the KV heads
// in the same order (head = chunk * heads / chunks), as the product kernel's KV-head-major unit
// order does, so one head's K/V (32 MB) is L2-resident while it is gathered.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdio.h>

#include "nsa_sel_kernel.cuh"

namespace peaks {

using C = nsa::Cfg<128, 128, 16, __nv_bfloat16, 2>;
constexpr int kKS = 3, kVS = 2;        // ring depths of the product kernel at this shape
constexpr int kThreads = 160;  // warp 0 K loader, 1 V loader, 2 score MMA, 3 / 4 PV MMA of even / odd chunks
constexpr int kTmemCols = 256;  // S, one O per PV issuer (16 columns each); modes 3-4: two 64-column K tiles at 64

struct Bars {
  uint64_t k_full[kKS], k_empty[kKS], v_full[kVS], v_empty[kVS], done_s, done_pv[2];
  uint32_t tmem_base;
  int abort_flag;
};

struct Params {
  int n_chunks, n_blk, n_heads, mode;
  uint32_t seed;
  unsigned long long timeout_ns;
  int32_t* err;
};

constexpr uint32_t kOffK = 0;
constexpr uint32_t kOffV = kOffK + kKS * C::kKStage;
constexpr uint32_t kOffQ = kOffV + kVS * C::kVStage;
constexpr uint32_t kOffP = kOffQ + C::kQBytes;
constexpr uint32_t kOffBar = kOffP + C::kPBytes;
constexpr uint32_t kSmemBytes = kOffBar + sizeof(Bars) + 1024;

__device__ __forceinline__ uint32_t mix(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
__device__ __forceinline__ int block_row(const Params& p, int c, int s) {
  const uint32_t h = mix(p.seed ^ mix(blockIdx.x * 0x9E3779B9u + (uint32_t)c * 2u + (uint32_t)s));
  return (int)(h % (uint32_t)p.n_blk) * nsa::kSub;
}
__device__ __forceinline__ int head_of(const Params& p, int c) {
  return (int)((long long)c * p.n_heads / p.n_chunks);
}

// Wait until the most recent load issued into each of the `n` stages of ring `r` has landed.
__device__ void drain_ring(const nsa::Ring& r, uint64_t* full, int n, const nsa::Waiter& w) {
  for (int s = 0; s < n; ++s) {
    const uint32_t back = (uint32_t)s + 1u;
    const uint32_t slot = (r.idx + (uint32_t)n - back % (uint32_t)n) % (uint32_t)n;
    const uint32_t ph = (r.idx >= back) ? r.phase : (r.phase ^ 1u);
    if (r.lapped || r.idx >= back) w.wait_drain(&full[slot], ph);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    peaks_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                 const __grid_constant__ Params p) {
  uint8_t* smem = nsa::smem_base();
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kKS; ++s) {
      nsa::ptx::mbar_init(&bars->k_full[s], 1);
      nsa::ptx::mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < kVS; ++s) {
      nsa::ptx::mbar_init(&bars->v_full[s], 1);
      nsa::ptx::mbar_init(&bars->v_empty[s], 1);
    }
    nsa::ptx::mbar_init(&bars->done_s, 1);
    nsa::ptx::mbar_init(&bars->done_pv[0], 1);
    nsa::ptx::mbar_init(&bars->done_pv[1], 1);
    bars->abort_flag = 0;
    nsa::ptx::fence_mbar_init();
  }
  // Q and P operand tiles are zero: the UMMAs read defined data.
  for (uint32_t i = threadIdx.x; i < (C::kQBytes + C::kPBytes) / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kOffQ)[i] = make_uint4(0u, 0u, 0u, 0u);
  nsa::ptx::fence_proxy_async_smem();
  if (warp == 2) {
    nsa::ptx::tmem_alloc(&bars->tmem_base, kTmemCols);
    nsa::ptx::tmem_relinquish();
  }
  nsa::ptx::tc_fence_before();
  __syncthreads();
  nsa::ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const nsa::Waiter w{&bars->abort_flag, p.err, p.timeout_ns};
  const uint64_t pol = nsa::ptx::policy_evict_last();
  const bool loads = p.mode != 2 && p.mode != 4;
  const bool tmem_a = p.mode >= 3;

  if (warp == 0 && loads) {
    // K loader: lane j issues the box of sub-block j / 2, d slice j % 2
    nsa::Ring k;
    const int s = lane >> 1, cc = lane & 1;
    for (int c = 0; c < p.n_chunks; ++c) {
      int go = 1;
      if (lane == 0) {
        go = (!k.lapped || w.wait(&bars->k_empty[k.idx], k.phase ^ 1u)) ? 1 : 0;
        if (go) nsa::ptx::mbar_arrive_expect_tx(&bars->k_full[k.idx], (uint32_t)C::kKStage);
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (lane < 4)
        nsa::ptx::tma_load_3d(smem + kOffK + k.idx * C::kKStage + cc * C::kKChunkStride + s * C::kBox, &tmK,
                              &bars->k_full[k.idx], cc * 64, block_row(p, c, s), head_of(p, c), pol);
      k.next(kKS);
    }
    if (lane == 0) drain_ring(k, bars->k_full, kKS, w);
    __syncwarp();
  } else if (warp == 1 && loads) {
    // V loader: chunk c goes to stage c % 2, the stage of the PV issuer of c's softmax group
    for (int c = 0; c < p.n_chunks; ++c) {
      const int vs = c & 1;
      const uint32_t use = (uint32_t)c >> 1;
      int go = 1;
      if (lane == 0) {
        go = (use == 0 || w.wait(&bars->v_empty[vs], (use - 1u) & 1u)) ? 1 : 0;
        if (go) nsa::ptx::mbar_arrive_expect_tx(&bars->v_full[vs], (uint32_t)C::kVStage);
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (lane < 2)
        nsa::ptx::tma_load_4d(smem + kOffV + vs * C::kVStage + lane * C::kVSub, &tmV, &bars->v_full[vs], 0,
                              block_row(p, c, lane), 0, head_of(p, c), pol);
    }
    if (lane == 0) {  // the most recent load of each stage has landed
      for (int vs = 0; vs < 2; ++vs) {
        const int last = p.n_chunks - 1 - ((p.n_chunks - 1 - vs) & 1);  // last chunk with parity vs
        if (last >= 0 && (last & 1) == vs) w.wait_drain(&bars->v_full[vs], ((uint32_t)last >> 1) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 2 && lane == 0) {
    // score issuer: S^T[128 keys x 16] = K_chunk . Q^T into TMEM columns 0-15
    const uint32_t k_base = nsa::ptx::smem_u32(smem + kOffK);
    const uint64_t bq0 = nsa::ptx::sdesc_sw128(nsa::ptx::smem_u32(smem + kOffQ), 16, 1024);
    nsa::Ring k;
    for (int c = 0; c < p.n_chunks; ++c) {
      if (loads && !w.wait(&bars->k_full[k.idx], k.phase)) break;
      if (p.mode == 0) {
        nsa::ptx::mbar_arrive(&bars->k_empty[k.idx]);
      } else {
        nsa::ptx::tc_fence_after();
        const uint64_t a0 = nsa::ptx::sdesc_sw128(k_base + k.idx * C::kKStage, 16, 1024);
        if (tmem_a) {
          const uint32_t ta = tmem + 64 + 64 * (uint32_t)(c & 1);
#pragma unroll
          for (int j = 0; j < C::DQK / 16; ++j)
            nsa::ptx::tmem_cp_128x256b(ta + 8 * j, nsa::desc_add(a0, (j >> 2) * C::kKChunkStride + (j & 3) * 32));
#pragma unroll
          for (int j = 0; j < C::DQK / 16; ++j)
            nsa::ptx::umma_bf16_ts(tmem, ta + 8 * j, nsa::desc_add(bq0, (j >> 2) * C::kQChunk + (j & 3) * 32),
                                   C::kIdescS, j > 0 ? 1u : 0u);
        } else {
#pragma unroll
          for (int j = 0; j < C::DQK / 16; ++j)
            nsa::ptx::umma_bf16(tmem, nsa::desc_add(a0, (j >> 2) * C::kKChunkStride + (j & 3) * 32),
                                nsa::desc_add(bq0, (j >> 2) * C::kQChunk + (j & 3) * 32), C::kIdescS, j > 0 ? 1u : 0u);
        }
        if (loads) nsa::ptx::umma_commit(&bars->k_empty[k.idx]);
      }
      k.next(kKS);
    }
    // every UMMA issued by this thread completes before TMEM is released
    nsa::ptx::umma_commit(&bars->done_s);
    w.wait_drain(&bars->done_s, 0);
  } else if ((warp == 3 || warp == 4) && lane == 0) {
    // PV issuer of softmax group g (chunks c % 2 == g): O^T[128 dims x 16] += V_chunk^T . P^T
    const int g = warp - 3;
    const uint32_t v_base = nsa::ptx::smem_u32(smem + kOffV + g * C::kVStage);
    const uint64_t bp0 = nsa::ptx::sdesc_sw128(nsa::ptx::smem_u32(smem + kOffP), 16, 1024);
    for (int c = g; c < p.n_chunks; c += 2) {
      const uint32_t use = (uint32_t)c >> 1;
      if (loads && !w.wait(&bars->v_full[g], use & 1u)) break;
      if (p.mode == 0) {
        nsa::ptx::mbar_arrive(&bars->v_empty[g]);
      } else {
        nsa::ptx::tc_fence_after();
        const uint64_t a0 = nsa::ptx::sdesc_sw128(v_base, C::kBox, 1024);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          nsa::ptx::umma_bf16(tmem + 16 + 16 * g, nsa::desc_add(a0, (j >> 2) * C::kVSub + (j & 3) * 2048),
                              nsa::desc_add(bp0, (j >> 2) * C::kPSub + (j & 3) * 32), C::kIdescPV, 1u);
        if (loads) nsa::ptx::umma_commit(&bars->v_empty[g]);
      }
    }
    nsa::ptx::umma_commit(&bars->done_pv[g]);
    w.wait_drain(&bars->done_pv[g], 0);
  }
  nsa::ptx::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    nsa::ptx::tc_fence_after();
    nsa::ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 f = nullptr;
  if (f == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return f;
}

}  // namespace peaks

extern "C" {

// Launch one microbenchmark (mode 0 to 4, see above) on `stream` over K, V bf16
// [n_heads, T, 128] with `ctas` CTAs (one per SM) of `n_chunks` 128-key chunks each.  Returns 0,
// or a negative code with a message on stderr.  `err` (device int32, optional) receives the
// bounded-wait timeout bit.  Bytes gathered per launch (modes 0, 1, 3): ctas * n_chunks * 64 KB.
int nsa_peaks_run(const void* k, const void* v, int n_heads, int T, int n_chunks, int mode, int ctas, int32_t* err,
                  cudaStream_t stream) {
  if (k == nullptr || v == nullptr || n_heads <= 0 || T < 128 || T % 64 != 0 || n_chunks <= 0 || ctas <= 0 ||
      mode < 0 || mode > 4) {
    fprintf(stderr, "nsa_peaks_run: bad arguments\n");
    return -1;
  }
  PFN_cuTensorMapEncodeTiled_v12000 f = peaks::encode_fn();
  if (f == nullptr) return -4;
  CUtensorMap tmK, tmV;
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  {
    cuuint64_t dims[3] = {128, (cuuint64_t)T, (cuuint64_t)n_heads};
    cuuint64_t str[2] = {256, 256ull * T};
    cuuint32_t box[3] = {64, 64, 1};
    if (f(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(k), dims, str, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return -1;
  }
  {
    cuuint64_t dims[4] = {64, (cuuint64_t)T, 2, (cuuint64_t)n_heads};
    cuuint64_t str[3] = {256, 128, 256ull * T};
    cuuint32_t box[4] = {64, 64, 2, 1};
    if (f(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v), dims, str, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return -1;
  }
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(peaks::peaks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)peaks::kSmemBytes) != cudaSuccess)
      return -3;
    attr = true;
  }
  peaks::Params p{n_chunks, T / 64, n_heads, mode, 0x1234567u, 2000000000ull, err};
  peaks::peaks_kernel<<<ctas, peaks::kThreads, peaks::kSmemBytes, stream>>>(tmK, tmV, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    fprintf(stderr, "nsa_peaks_run: %s\n", cudaGetErrorString(e));
    return -3;
  }
  return 0;
}

}  // extern "C"
