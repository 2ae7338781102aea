// Host side of the C ABI declared in include/nsa_sel.h: argument validation, launch
// planning (work-unit split, tensor-core N, ring depths within the 227 KB shared-memory
// budget), TMA tensor-map encoding and dispatch over the compiled kernel family.
//
// Boundary being replaced: the reference's libtorch op `forward(Q,K,V,sel,l_prime,BQ,cyc)`
// (nsa_v2.cu:147-170; same op in nsa_v1.cu:125-147 and nsa_v0.cu:118-146), which reads shapes
// from tensors, allocates a zeroed fp32 O, sets scale = 1/sqrt(D) and launches one CTA per
// (query block, b*Hkv) on the legacy stream.  This launcher takes caller-owned buffers, runs
// on the stream it is given and launches one persistent CTA per SM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <algorithm>
#include <mutex>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "nsa_sel.h"
#include "nsa_sel_kernel.cuh"
#include "nsa_ro_kernel.cuh"
#include "nsa_select_kernel.cuh"
#include "nsa_select_tc_kernel.cuh"
#include "nsa_bwd_kernel.cuh"

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(NSA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per block on sm_100
constexpr int kMaxCols = 64;        // widest N of the tensor-core tiles (G * tokens per unit)
constexpr int kMaxSub = 128;        // widest per-unit list of 64-key sub-blocks
constexpr int kMaxDevices = 64;

// ------------------------------------------------------------------ driver entry point
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// ------------------------------------------------------------------ per-device cache
struct DeviceCache {
  std::mutex mu;
  int sm_count[kMaxDevices] = {};
  uint64_t attr_done[kMaxDevices] = {};  // one bit per kernel instantiation
};
DeviceCache g_dev;

}  // namespace

// Unit counters of the dynamic work distribution (Params::work_counter): 4-byte slots in static
// device memory (nothing is allocated), each zeroed on the launch's stream just before the
// launch that uses it (a graph captures the reset with the launch).  Launches that are not being
// captured take the eager slots round-robin, so launches in flight on different streams use
// different slots.  A launch captured into a CUDA graph keeps its slot for every replay, so each
// capture takes a slot of its own that is never handed out again; when those run out, further
// captured launches use the fixed-stride schedule (no counter).  A zeroing kernel-side reset
// (the last CTA clearing the slot) was measured 3-5 % slower on the north-star shape.
constexpr int kEagerCounterSlots = 2048;
constexpr int kCaptureCounterSlots = 2048;
__device__ unsigned int g_work_counters[kEagerCounterSlots + kCaptureCounterSlots];

namespace {
unsigned int* g_work_counter_base[kMaxDevices] = {};
unsigned int g_work_counter_next[kMaxDevices] = {};
unsigned int g_capture_counter_next[kMaxDevices] = {};

// *out = the slot for a launch on `stream`, or nullptr for the fixed-stride schedule.
int next_work_counter(int dev, cudaStream_t stream, unsigned int** out) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  std::lock_guard<std::mutex> lk(g_dev.mu);
  if (g_work_counter_base[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_work_counters);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(work counters)");
    g_work_counter_base[dev] = static_cast<unsigned int*>(ptr);
  }
  unsigned int slot;
  if (cs == cudaStreamCaptureStatusActive) {
    if (g_capture_counter_next[dev] >= (unsigned)kCaptureCounterSlots) {
      *out = nullptr;
      return NSA_OK;
    }
    slot = kEagerCounterSlots + g_capture_counter_next[dev]++;
  } else {
    slot = g_work_counter_next[dev]++ % (unsigned)kEagerCounterSlots;
  }
  *out = g_work_counter_base[dev] + slot;
  return NSA_OK;
}

int current_sm_count(int* sm_count, int* device) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(NSA_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev.mu);
  if (g_dev.sm_count[dev] == 0) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(NSA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, major,
                  minor);
    g_dev.sm_count[dev] = n;
  }
  *sm_count = g_dev.sm_count[dev];
  *device = dev;
  return NSA_OK;
}

// ------------------------------------------------------------------ kernel family
using bf16 = __nv_bfloat16;

typedef void (*KernelFn)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                         const nsa::Params);
typedef nsa::SmemLayout (*LayoutFn)(int, int, int, int);

struct Variant {
  int dqk, dv, ncol, out_f32, nwg, ext, vgroups, threads;
  KernelFn kernel;
  LayoutFn layout;
  int k_stage, v_stage, tmem_cols;
  int ro;  // row-owner kernel (128-row query tiles, nsa_ro_kernel.cuh)
};

template <int DQK, int DV, int NCOL, typename OutT, int NWG, bool EXT = false>
Variant make_variant() {
  using C = nsa::Cfg<DQK, DV, NCOL, OutT, NWG, EXT>;
  return Variant{DQK,
                 DV,
                 NCOL,
                 sizeof(OutT) == 4 ? 1 : 0,
                 NWG,
                 EXT ? 1 : 0,
                 C::kVGroups,
                 C::kThreads,
                 reinterpret_cast<KernelFn>(&nsa::nsa_sel_fwd_kernel<C>),
                 &nsa::smem_layout<C>,
                 C::kKStage,
                 C::kVStage,
                 C::kTmemCols,
                 0};
}

template <int DQK, int DV, typename OutT, bool EXT = false>
Variant make_variant_ro() {
  using C = nsa::CfgRO<DQK, DV, OutT, EXT>;
  return Variant{DQK,
                 DV,
                 128,
                 sizeof(OutT) == 4 ? 1 : 0,
                 1,
                 EXT ? 1 : 0,
                 1,
                 C::kThreads,
                 reinterpret_cast<KernelFn>(&nsa::nsa_ro_fwd_kernel<C>),
                 &nsa::smem_layout_ro<C>,
                 C::kKStage,
                 C::kVStage,
                 C::kTmemCols,
                 1};
}

// Narrow tiles (N = 16: per-token selection with G <= 16) split every unit's chunks over two
// softmax warpgroups; wider tiles (per-query-block selection) use one.
#define NSA_VARIANTS_FOR(DQK, DV)                                                                      \
  make_variant<DQK, DV, 16, bf16, 2>(), make_variant<DQK, DV, 32, bf16, 1>(),                           \
      make_variant<DQK, DV, 64, bf16, 1>(), make_variant<DQK, DV, 16, float, 2>(),                      \
      make_variant<DQK, DV, 32, float, 1>(), make_variant<DQK, DV, 64, float, 1>()

// Extended key visibility (window, compressed key map): the NSA window and compressed branches,
// fp32 output, d_qk == d_v in {64, 128}.
#define NSA_EXT_VARIANTS_FOR(D)                                                                      \
  make_variant<D, D, 16, float, 2, true>(), make_variant<D, D, 32, float, 1, true>(),                 \
      make_variant<D, D, 64, float, 1, true>()

const Variant* variants(int* n) {
  static const Variant v[] = {NSA_VARIANTS_FOR(64, 64),  NSA_VARIANTS_FOR(128, 128), NSA_VARIANTS_FOR(192, 128),
                              NSA_VARIANTS_FOR(128, 64), NSA_EXT_VARIANTS_FOR(64),   NSA_EXT_VARIANTS_FOR(128),
                              // 128-row query tiles (G * tokens per unit = 128): row-owner kernel
                              make_variant_ro<64, 64, bf16>(), make_variant_ro<64, 64, float>(),
                              make_variant_ro<128, 128, bf16>(), make_variant_ro<128, 128, float>(),
                              make_variant_ro<64, 64, float, true>(), make_variant_ro<128, 128, float, true>()};
  *n = (int)(sizeof(v) / sizeof(v[0]));
  return v;
}

int find_variant(int dqk, int dv, int ncol, int out_f32, int ext) {
  int n = 0;
  const Variant* v = variants(&n);
  for (int i = 0; i < n; ++i)
    if (v[i].dqk == dqk && v[i].dv == dv && v[i].ncol == ncol && v[i].out_f32 == out_f32 && v[i].ext == ext)
      return i;
  return -1;
}

// ------------------------------------------------------------------ planning
struct Plan {
  int G, BQs, parts, ncol, maxsub, n_units, KS, VS, out_bufs, grid, variant;
  int bkv_begin, bkv_end, qb_begin, qb_end;
  nsa::SmemLayout layout;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int make_plan(const nsa_sel_desc* d, int sm_count, Plan* pl) {
  if (d == nullptr) return fail(NSA_ERR_INVALID_ARG, "desc is NULL");
  if (d->q == nullptr || d->k == nullptr || d->v == nullptr || d->sel == nullptr || d->o == nullptr)
    return fail(NSA_ERR_INVALID_ARG, "q, k, v, sel and o must be non-NULL");
  if (!aligned16(d->q) || !aligned16(d->k) || !aligned16(d->v) || !aligned16(d->o))
    return fail(NSA_ERR_INVALID_ARG, "q, k, v and o must be 16-byte aligned (TMA requirement)");
  if ((reinterpret_cast<uintptr_t>(d->sel) & 3u) != 0) return fail(NSA_ERR_INVALID_ARG, "sel must be 4-byte aligned");
  const int B = d->batch, Hq = d->heads_q, Hkv = d->heads_kv, T = d->seq_len;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0) return fail(NSA_ERR_INVALID_ARG, "B, Hq, Hkv, T must be positive");
  if (Hq % Hkv != 0) return fail(NSA_ERR_INVALID_ARG, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  const int G = Hq / Hkv;
  if (G > 128 || (G > kMaxCols && 128 % G != 0))
    return fail(NSA_ERR_UNSUPPORTED, "group size G=%d exceeds %d", G, kMaxCols);
  if (d->d_qk <= 0 || d->d_v <= 0) return fail(NSA_ERR_INVALID_ARG, "d_qk and d_v must be positive");
  if (d->block_size <= 0) return fail(NSA_ERR_INVALID_ARG, "l_prime must be positive");
  if (d->block_size % 64 != 0 || d->block_size > 256)
    return fail(NSA_ERR_UNSUPPORTED, "l_prime=%d: the kernel family supports 64, 128 and 256", d->block_size);
  if (d->q_block <= 0) return fail(NSA_ERR_INVALID_ARG, "BQ must be positive");
  const int NQB = (T + d->q_block - 1) / d->q_block;
  if (d->n_qblocks != NQB)
    return fail(NSA_ERR_INVALID_ARG, "sel has NQB=%d query blocks, expected ceil(T/BQ)=%d", d->n_qblocks, NQB);
  if (d->n_sel <= 0) return fail(NSA_ERR_INVALID_ARG, "KSEL must be positive");
  const int spb = d->block_size / 64;
  if ((long long)d->n_sel * spb > kMaxSub)
    return fail(NSA_ERR_UNSUPPORTED, "KSEL*l_prime/64 = %lld exceeds %d sub-blocks", (long long)d->n_sel * spb,
                kMaxSub);
  if (d->o_dtype != NSA_DTYPE_BF16 && d->o_dtype != NSA_DTYPE_F32)
    return fail(NSA_ERR_INVALID_ARG, "o_dtype must be NSA_DTYPE_BF16 or NSA_DTYPE_F32");
  const int kv_len = d->kv_len > 0 ? d->kv_len : T;
  if (d->kv_len < 0) return fail(NSA_ERR_INVALID_ARG, "kv_len must be >= 0 (0 = seq_len)");
  if (d->window < 0) return fail(NSA_ERR_INVALID_ARG, "window must be >= 0 (0 = none)");
  if (d->key_map != NSA_KEYMAP_CAUSAL && d->key_map != NSA_KEYMAP_COMPRESSED)
    return fail(NSA_ERR_INVALID_ARG, "key_map must be NSA_KEYMAP_CAUSAL or NSA_KEYMAP_COMPRESSED");
  if (d->key_map == NSA_KEYMAP_CAUSAL && kv_len != T)
    return fail(NSA_ERR_INVALID_ARG, "kv_len (%d) != seq_len (%d) needs key_map = NSA_KEYMAP_COMPRESSED", kv_len, T);
  if (d->key_map == NSA_KEYMAP_COMPRESSED && d->window > 0)
    return fail(NSA_ERR_UNSUPPORTED, "window and key_map = NSA_KEYMAP_COMPRESSED cannot be combined");
  if (d->o_accumulate != 0 && d->o_accumulate != 1) return fail(NSA_ERR_INVALID_ARG, "o_accumulate must be 0 or 1");
  if (d->o_accumulate && d->o_dtype != NSA_DTYPE_F32)
    return fail(NSA_ERR_UNSUPPORTED, "o_accumulate needs fp32 O (o_dtype = NSA_DTYPE_F32)");
  if ((reinterpret_cast<uintptr_t>(d->o_weight) & 3u) != 0) return fail(NSA_ERR_INVALID_ARG, "o_weight must be 4-byte aligned");
  if (d->cu_seqlens != nullptr && (d->window > 0 || d->key_map != NSA_KEYMAP_CAUSAL))
    return fail(NSA_ERR_UNSUPPORTED, "a varlen batch supports neither window nor key_map");
  if (d->cu_seqlens != nullptr) {
    if (B != 1) return fail(NSA_ERR_INVALID_ARG, "a varlen batch (cu_seqlens) needs B == 1");
    if (d->q_block != 1) return fail(NSA_ERR_UNSUPPORTED, "a varlen batch needs per-token selection (BQ == 1)");
    if (d->n_seqs <= 0) return fail(NSA_ERR_INVALID_ARG, "n_seqs must be positive with cu_seqlens");
  }
  // 32-bit coordinates and index arithmetic inside the kernel.
  if ((long long)kv_len * d->d_qk >= (1ll << 31) || (long long)T >= (1ll << 24) ||
      (long long)T * d->d_qk >= (1ll << 31) || (long long)B * Hkv * NQB * d->n_sel >= (1ll << 31))
    return fail(NSA_ERR_UNSUPPORTED, "problem too large for 32-bit coordinates");

  // Tokens per work unit.  When 128 query rows (G heads x 128/G tokens) fit one selection row,
  // the row-owner kernel takes the unit (queries on the MMA's M); otherwise the largest divisor
  // of BQ with G * tokens <= 64 goes to the swap-AB kernel (keys on M).
  const int ext = (d->window > 0 || d->key_map != NSA_KEYMAP_CAUSAL) ? 1 : 0;
  const int of32 = d->o_dtype == NSA_DTYPE_F32 ? 1 : 0;
  int bqs = 1, ncol = 16, vi = -1;
  if (!(d->debug_flags & NSA_DEBUG_NO_ROW_OWNER)) {
    // 128 query rows per tile, or 64 (the reference's BQ * G = 64 mode, on M = 64 MMAs unless
    // NSA_DEBUG_RO_PAD128 asks for the padded 128-row form)
    for (int rows = 128; rows >= 64 && vi < 0; rows -= 64) {
      if (rows % G != 0 || d->q_block % (rows / G) != 0) continue;
      vi = find_variant(d->d_qk, d->d_v, 128, of32, ext);
      if (vi >= 0) {
        bqs = rows / G;
        ncol = 128;
      }
    }
  }
  if (vi < 0 && G > kMaxCols) return fail(NSA_ERR_UNSUPPORTED, "group size G=%d exceeds %d", G, kMaxCols);
  if (vi < 0) {
    for (int c = d->q_block; c >= 1; --c)
      if (d->q_block % c == 0 && G * c <= kMaxCols) { bqs = c; break; }
    const int rows = G * bqs;
    while (ncol < rows) ncol <<= 1;
    vi = find_variant(d->d_qk, d->d_v, ncol, of32, ext);
  }
  if (vi < 0)
    return fail(NSA_ERR_UNSUPPORTED,
                ext ? "no kernel with window / key map for (d_qk=%d, d_v=%d, %s O); built: d_qk == d_v in {64, 128}, fp32 O"
                    : "no kernel for (d_qk=%d, d_v=%d, %s O); built: (64,64), (128,128), (192,128), (128,64)",
                d->d_qk, d->d_v, d->o_dtype == NSA_DTYPE_F32 ? "fp32" : "bf16");
  int nv = 0;
  const Variant& V = variants(&nv)[vi];

  pl->G = G;
  pl->BQs = bqs;
  pl->parts = d->q_block / bqs;
  pl->ncol = ncol;
  pl->maxsub = d->n_sel * spb;
  pl->variant = vi;
  pl->bkv_begin = d->bkv_begin;
  pl->bkv_end = d->bkv_end > 0 ? d->bkv_end : B * Hkv;
  pl->qb_begin = d->qb_begin;
  pl->qb_end = d->qb_end > 0 ? d->qb_end : NQB;
  if (pl->bkv_begin < 0 || pl->bkv_begin >= pl->bkv_end || pl->bkv_end > B * Hkv)
    return fail(NSA_ERR_INVALID_ARG, "shard bkv range [%d,%d) invalid for B*Hkv=%d", pl->bkv_begin, pl->bkv_end,
                B * Hkv);
  if (pl->qb_begin < 0 || pl->qb_begin >= pl->qb_end || pl->qb_end > NQB)
    return fail(NSA_ERR_INVALID_ARG, "shard query-block range [%d,%d) invalid for NQB=%d", pl->qb_begin,
                pl->qb_end, NQB);
  const long long units = (long long)(pl->bkv_end - pl->bkv_begin) * (pl->qb_end - pl->qb_begin) * pl->parts;
  if (units >= (1ll << 31)) return fail(NSA_ERR_UNSUPPORTED, "too many work units");
  pl->n_units = (int)units;

  // Ring depths: the deepest equal K/V rings that fit, then one more K stage if it fits (the
  // score MMAs run ahead of the softmax, so K tiles are consumed earlier than V tiles).  The
  // output staging tile is double-buffered unless a single buffer is what makes it fit.
  int ob = 2;
  auto fits = [&](int k, int v) { return (int)V.layout(k, v, pl->maxsub, ob).total <= kSmemLimit; };
  int ks = 0, vs = 0;
  for (int c = nsa::kMaxStages; c >= 1; --c)
    if (fits(c, c)) { ks = vs = c; break; }
  if (ks < 2) {
    ob = 1;
    for (int c = nsa::kMaxStages; c >= 1; --c)
      if (fits(c, c)) { ks = vs = c; break; }
  }
  if (ks == 0) return fail(NSA_ERR_UNSUPPORTED, "tile does not fit in shared memory");
  if (ks < nsa::kMaxStages && fits(ks + 1, vs)) ++ks;
  // With one PV warp per softmax group the V stages are split between them: keep a multiple.
  const int vmult = V.vgroups;
  if (vmult > 1) vs -= vs % vmult;
  if (vs < vmult) return fail(NSA_ERR_UNSUPPORTED, "tile does not fit in shared memory");
  pl->KS = ks;
  pl->VS = vs;
  pl->out_bufs = ob;
  pl->layout = V.layout(ks, vs, pl->maxsub, ob);
  int grid = sm_count > 0 ? sm_count : 148;
  if (d->max_ctas > 0 && d->max_ctas < grid) grid = d->max_ctas;
  if (grid > pl->n_units) grid = pl->n_units;
  pl->grid = grid;
  return NSA_OK;
}

int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* ptr, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw, CUtensorMapL2promotion prom,
           const char* what) {
  PFN_cuTensorMapEncodeTiled_v12000 f = encode_fn();
  if (f == nullptr) return fail(NSA_ERR_DRIVER, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = f(m, dt, (cuuint32_t)rank, const_cast<void*>(ptr), dims, strides, box, es,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, sw, prom, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NSA_ERR_INVALID_ARG, "cuTensorMapEncodeTiled(%s) failed with %d", what, (int)r);
  return NSA_OK;
}

int launch(const nsa_sel_desc* d, nsa_stream_t stream) {
  int sm = 0, dev = 0;
  int rc = current_sm_count(&sm, &dev);
  if (rc != NSA_OK) return rc;
  Plan pl;
  rc = make_plan(d, sm, &pl);
  if (rc != NSA_OK) return rc;
  int nv = 0;
  const Variant& V = variants(&nv)[pl.variant];

  const int B = d->batch, Hq = d->heads_q, Hkv = d->heads_kv, T = d->seq_len;
  const cuuint64_t dqk = (cuuint64_t)d->d_qk, dv = (cuuint64_t)d->d_v;
  const cuuint64_t KVL = (cuuint64_t)(d->kv_len > 0 ? d->kv_len : T);  // K/V rows per (b, kvh)
  CUtensorMap tmQ, tmK, tmV, tmO;
  {
    cuuint64_t dims[4] = {dqk, (cuuint64_t)T, (cuuint64_t)Hq, (cuuint64_t)B};
    cuuint64_t str[3] = {dqk * 2, dqk * 2 * T, dqk * 2 * T * Hq};
    cuuint32_t box[4] = {64, (cuuint32_t)pl.BQs, (cuuint32_t)pl.G, 1};
    rc = encode(&tmQ, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, d->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, "Q");
    if (rc != NSA_OK) return rc;
  }
  {
    cuuint64_t dims[3] = {dqk, KVL, (cuuint64_t)B * Hkv};
    cuuint64_t str[2] = {dqk * 2, dqk * 2 * KVL};
    cuuint32_t box[3] = {64, 64, 1};
    rc = encode(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d->k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "K");
    if (rc != NSA_OK) return rc;
  }
  {
    // V viewed as (64 d, T, d_v/64 slices, B*Hkv): one box = a 64-key sub-block, slice-major in
    // shared memory ([slice][row][64]), the MN-major layout the PV UMMA reads.
    cuuint64_t dims[4] = {64, KVL, dv / 64, (cuuint64_t)B * Hkv};
    cuuint64_t str[3] = {dv * 2, 128, dv * 2 * KVL};
    cuuint32_t box[4] = {64, 64, (cuuint32_t)(dv / 64), 1};
    rc = encode(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, d->v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "V");
    if (rc != NSA_OK) return rc;
  }
  {
    const bool f32 = d->o_dtype == NSA_DTYPE_F32;
    const cuuint64_t es = f32 ? 4 : 2;
    cuuint64_t dims[4] = {dv, (cuuint64_t)T, (cuuint64_t)Hq, (cuuint64_t)B};
    cuuint64_t str[3] = {dv * es, dv * es * T, dv * es * T * Hq};
    // row-owner kernel: 128-byte-wide boxes staged in the SW128 layout; swap-AB kernel: 64-column
    // unswizzled boxes
    cuuint32_t box[4] = {V.ro ? (cuuint32_t)(128 / es) : 64u, (cuuint32_t)pl.BQs, (cuuint32_t)pl.G, 1};
    rc = encode(&tmO, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, d->o, dims, str,
                box, V.ro ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, "O");
    if (rc != NSA_OK) return rc;
  }

  nsa::Params p{};
  p.sel = d->sel;
  p.cu_seqlens = d->cu_seqlens;
  p.lse = d->lse;
  p.cyc = d->cyc;
  p.err = d->err;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.G = pl.G;
  p.LP = d->block_size;
  p.BQ = d->q_block;
  p.BQs = pl.BQs;
  p.parts = pl.parts;
  p.NQB = d->n_qblocks;
  p.KSEL = d->n_sel;
  p.n_seq = d->cu_seqlens ? d->n_seqs : 1;
  p.bkv_begin = pl.bkv_begin;
  p.bkv_end = pl.bkv_end;
  p.qb_begin = pl.qb_begin;
  p.qb_end = pl.qb_end;
  p.n_units = pl.n_units;
  p.maxsub = pl.maxsub;
  p.KS = pl.KS;
  p.VS = pl.VS;
  const double scale = d->scale > 0.f ? (double)d->scale : 1.0 / sqrt((double)d->d_qk);
  p.scale_log2 = (float)(scale * 1.4426950408889634074);
  int tmo = d->timeout_ms;
  if (tmo <= 0) {
    const char* e = getenv("NSA_SEL_TIMEOUT_MS");
    tmo = e ? atoi(e) : 0;
    if (tmo <= 0) tmo = 2000;
  }
  p.timeout_ns = (unsigned long long)tmo * 1000000ull;
  p.off_k = pl.layout.off_k;
  p.off_v = pl.layout.off_v;
  p.off_q = pl.layout.off_q;
  p.off_p = pl.layout.off_p;
  p.off_out = pl.layout.off_out;
  p.off_tr = pl.layout.off_tr;
  p.off_alpha = pl.layout.off_alpha;
  p.off_fac = pl.layout.off_fac;
  p.off_ml = pl.layout.off_ml;
  p.off_info = pl.layout.off_info;
  p.off_bar = pl.layout.off_bar;
  p.kv_len = (int)KVL;
  p.window = d->window;
  p.key_map = d->key_map;
  p.debug_stall = (d->debug_flags & NSA_DEBUG_STALL) ? 1 : 0;
  p.out_bufs = pl.out_bufs;
  p.o_accum = d->o_accumulate;
  p.o_weight = d->o_weight;
  p.ro_m64 = (V.ro && pl.G * pl.BQs == 64 && !(d->debug_flags & NSA_DEBUG_RO_PAD128)) ? 1 : 0;

  {
    std::lock_guard<std::mutex> lk(g_dev.mu);
    const uint64_t bit = 1ull << pl.variant;
    if ((g_dev.attr_done[dev] & bit) == 0) {
      cudaFuncAttributes fa;
      cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(V.kernel));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(V.kernel), cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kSmemLimit - (int)fa.sharedSizeBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
      g_dev.attr_done[dev] |= bit;
    }
  }
  p.work_counter = nullptr;
  if (pl.n_units > pl.grid && !(d->debug_flags & NSA_DEBUG_STATIC_UNITS)) {
    rc = next_work_counter(dev, reinterpret_cast<cudaStream_t>(stream), &p.work_counter);
    if (rc != NSA_OK) return rc;
    if (p.work_counter != nullptr) {
      cudaError_t me = cudaMemsetAsync(p.work_counter, 0, sizeof(unsigned int), reinterpret_cast<cudaStream_t>(stream));
      if (me != cudaSuccess) return cuda_fail(me, "cudaMemsetAsync(work counter)");
    }
  }
  void* args[] = {&tmQ, &tmK, &tmV, &tmO, &p};
  cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(V.kernel), dim3(pl.grid), dim3(V.threads), args,
                                   pl.layout.total, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  g_last_error[0] = '\0';
  return NSA_OK;
}

}  // namespace

// Static scratch of the allocation-free selection entry point (nsa_sel_select_noalloc): the
// block-key table lives in this module-scope device array, so the call never allocates.
constexpr size_t kStaticSelectScratchFloats = (size_t)4 << 20;  // 16 MB
__device__ __align__(256) float g_select_scratch[kStaticSelectScratchFloats];
// Device error word of the tensor-core selection kernel (NSA_DEVERR_* bits; read and cleared by
// nsa_sel_select_status).  Static device memory, resolved per device like the others.
__device__ int32_t g_select_err;

namespace {
float* g_select_scratch_ptr[kMaxDevices] = {};

// Resolve the static scratch's device address once per device (this also loads the module, so
// no later call allocates).
int static_select_scratch(int dev, float** out) {
  std::lock_guard<std::mutex> lk(g_dev.mu);
  if (g_select_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_select_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(select scratch)");
    g_select_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_select_scratch_ptr[dev];
  return NSA_OK;
}

int32_t* g_select_err_ptr[kMaxDevices] = {};

int select_err_word(int dev, int32_t** out) {
  std::lock_guard<std::mutex> lk(g_dev.mu);
  if (g_select_err_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_select_err);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(selection error word)");
    g_select_err_ptr[dev] = static_cast<int32_t*>(ptr);
  }
  *out = g_select_err_ptr[dev];
  return NSA_OK;
}

// ------------------------------------------------------------------ block selection
int select_shape(int32_t B, int32_t Hq, int32_t Hkv, int32_t T, int32_t d, int32_t l_prime, int32_t n_sel,
                 int32_t cmp_block, int32_t cmp_stride, int* n_blk, int* topk, int* n_cmp) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0 || d <= 0 || l_prime <= 0 || n_sel <= 0 || cmp_block <= 0 ||
      cmp_stride <= 0)
    return fail(NSA_ERR_INVALID_ARG, "B, Hq, Hkv, T, d, l_prime, n_sel, cmp_block and cmp_stride must be positive");
  if (Hq % Hkv != 0) return fail(NSA_ERR_INVALID_ARG, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  if (d % 8 != 0 || d > nsa::select::kMaxD)
    return fail(NSA_ERR_UNSUPPORTED, "d=%d: selection supports d %% 8 == 0, d <= %d", d, nsa::select::kMaxD);
  if ((long long)B * Hkv > 65535) return fail(NSA_ERR_UNSUPPORTED, "B*Hkv exceeds 65535");
  if ((long long)B * Hq * T * d >= (1ll << 40)) return fail(NSA_ERR_UNSUPPORTED, "problem too large");
  *n_blk = (T + l_prime - 1) / l_prime;
  *topk = n_sel < *n_blk ? n_sel : *n_blk;
  if (*topk > nsa::select::kMaxK) return fail(NSA_ERR_UNSUPPORTED, "top-k of %d exceeds %d", *topk, nsa::select::kMaxK);
  *n_cmp = T >= cmp_block ? (T - cmp_block) / cmp_stride + 1 : 0;
  return NSA_OK;
}

// The tensor-core selection (d = 64 or 128): the split block-key table, then select_tc_kernel.
template <int D, int K>
int select_tc_launch(const void* q, float* ws, int32_t* sel, int B, int Hq, int Hkv, int T, int l_prime, int topk,
                     int n_blk, int sm, int dev, cudaStream_t st) {
  CUtensorMap tmB;
  {
    // [part (hi, lo)][b*Hkv][n_blk][D] bf16; one box = 64 dims x 128 blocks (SW128)
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)n_blk, (cuuint64_t)B * Hkv, 2};
    const cuuint64_t str[3] = {(cuuint64_t)D * 2, (cuuint64_t)D * 2 * n_blk, (cuuint64_t)D * 2 * n_blk * B * Hkv};
    const cuuint32_t box[4] = {64, (cuuint32_t)nsa::seltc::kNT, 1, 1};
    int rc = encode(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ws, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "block keys");
    if (rc != NSA_OK) return rc;
  }
  int32_t* err = nullptr;
  int rc = select_err_word(dev, &err);
  if (rc != NSA_OK) return rc;
  nsa::seltc::Params p{};
  p.q = static_cast<const bf16*>(q);
  p.sel = sel;
  p.err = err;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.G = Hq / Hkv;
  p.n_blk = n_blk;
  p.l_prime = l_prime;
  p.topk = topk;
  p.n_tiles = (T + nsa::seltc::kRows - 1) / nsa::seltc::kRows;
  p.n_units = B * Hkv * p.n_tiles;
  const char* e = getenv("NSA_SEL_TIMEOUT_MS");
  const int tmo = e ? atoi(e) : 0;
  p.timeout_ns = (unsigned long long)(tmo > 0 ? tmo : 2000) * 1000000ull;
  const uint32_t smem = nsa::seltc::smem_bytes<D>();
  {
    std::lock_guard<std::mutex> lk(g_dev.mu);
    const uint64_t bit = 1ull << (59 + (D == 64 ? 0 : 2) + (K == 16 ? 0 : 1));
    if ((g_dev.attr_done[dev] & bit) == 0) {
      cudaError_t ae = cudaFuncSetAttribute(reinterpret_cast<const void*>(&nsa::seltc::select_tc_kernel<D, K>),
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (ae != cudaSuccess) return cuda_fail(ae, "cudaFuncSetAttribute(tensor-core selection smem)");
      g_dev.attr_done[dev] |= bit;
    }
  }
  const int grid = p.n_units < sm ? p.n_units : sm;
  void* args[] = {&tmB, &p};
  cudaError_t le = cudaLaunchKernel(reinterpret_cast<const void*>(&nsa::seltc::select_tc_kernel<D, K>), dim3(grid),
                                    dim3(nsa::seltc::kThreads), args, smem, st);
  if (le != cudaSuccess) return cuda_fail(le, "tensor-core selection kernel launch");
  return NSA_OK;
}

int select_tc(const void* q, const void* k, float* ws, int32_t* sel, int B, int Hq, int Hkv, int T, int d,
              int l_prime, int topk, int n_blk, int n_cmp, int cmp_block, int cmp_stride, float scale, int sm, int dev,
              cudaStream_t st) {
  nsa::select::kblk_kernel<true><<<dim3(n_blk, B * Hkv), d, 0, st>>>(static_cast<const bf16*>(k), ws, T, d, n_blk,
                                                                      n_cmp, l_prime, cmp_block, cmp_stride, scale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "block-key kernel launch");
  // list capacity: 16 when k <= 16 (the BASELINE top-16), else 32
  int rc;
  if (d == 64)
    rc = topk <= 16 ? select_tc_launch<64, 16>(q, ws, sel, B, Hq, Hkv, T, l_prime, topk, n_blk, sm, dev, st)
                    : select_tc_launch<64, 32>(q, ws, sel, B, Hq, Hkv, T, l_prime, topk, n_blk, sm, dev, st);
  else
    rc = topk <= 16 ? select_tc_launch<128, 16>(q, ws, sel, B, Hq, Hkv, T, l_prime, topk, n_blk, sm, dev, st)
                    : select_tc_launch<128, 32>(q, ws, sel, B, Hq, Hkv, T, l_prime, topk, n_blk, sm, dev, st);
  if (rc == NSA_OK) g_last_error[0] = '\0';
  return rc;
}

// ------------------------------------------------------------------ host-buffer pipeline
constexpr int kMaxSlices = 64;
struct HostPipe {
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t entry = nullptr, done = nullptr;
  cudaEvent_t in[kMaxSlices] = {}, out[kMaxSlices] = {};
};
std::mutex g_pipe_mu;
HostPipe g_pipe[kMaxDevices];

int pipe_for(int dev, HostPipe** out) {
  HostPipe& hp = g_pipe[dev];
  if (!hp.ready) {
    cudaError_t e = cudaStreamCreateWithFlags(&hp.h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&hp.d2h, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.entry, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.done, cudaEventDisableTiming);
    for (int i = 0; i < kMaxSlices && e == cudaSuccess; ++i) {
      e = cudaEventCreateWithFlags(&hp.in[i], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&hp.out[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return cuda_fail(e, "creating the host pipeline's streams and events");
    hp.ready = true;
  }
  *out = &hp;
  return NSA_OK;
}

// G rows of `width` bytes, `pitch` apart, at the same offset in both buffers.
cudaError_t copy_rows(void* dst, const void* src, size_t off, size_t width, size_t pitch, int rows,
                      cudaMemcpyKind kind, cudaStream_t s) {
  return cudaMemcpy2DAsync(static_cast<char*>(dst) + off, pitch, static_cast<const char*>(src) + off, pitch, width,
                           (size_t)rows, kind, s);
}

int run_host(const nsa_sel_desc* d, const nsa_sel_host_io* io, nsa_stream_t stream) {
  if (io == nullptr) return fail(NSA_ERR_INVALID_ARG, "io is NULL");
  if (io->q == nullptr || io->k == nullptr || io->v == nullptr || io->sel == nullptr || io->o == nullptr)
    return fail(NSA_ERR_INVALID_ARG, "io->q, k, v, sel and o must be non-NULL");
  if (io->token_slices < 0) return fail(NSA_ERR_INVALID_ARG, "token_slices must be >= 0");
  if (d != nullptr && d->o_accumulate != 0)
    return fail(NSA_ERR_UNSUPPORTED, "o_accumulate is not supported with host buffers");
  int sm = 0, dev = 0;
  int rc = current_sm_count(&sm, &dev);
  if (rc != NSA_OK) return rc;
  Plan pl;
  rc = make_plan(d, sm, &pl);
  if (rc != NSA_OK) return rc;

  const int Hq = d->heads_q, Hkv = d->heads_kv, T = d->seq_len, G = pl.G, BQ = d->q_block, NQB = d->n_qblocks;
  const size_t KVL = (size_t)(d->kv_len > 0 ? d->kv_len : T);
  const size_t qrow = (size_t)d->d_qk * 2, orow = (size_t)d->d_v * (d->o_dtype == NSA_DTYPE_F32 ? 4 : 2);
  const size_t krow = (size_t)d->d_qk * 2, vrow = (size_t)d->d_v * 2, srow = (size_t)d->n_sel * 4;
  const int rows = pl.bkv_end - pl.bkv_begin, nqb = pl.qb_end - pl.qb_begin;
  int per_row = io->token_slices > 0 ? io->token_slices : (16 + rows - 1) / rows;
  per_row = per_row < nqb ? per_row : nqb;
  while (per_row > 1 && rows * per_row > kMaxSlices) --per_row;
  if (rows * per_row > kMaxSlices) per_row = 1;
  const bool lse = d->lse != nullptr && io->lse != nullptr;

  std::lock_guard<std::mutex> lk(g_pipe_mu);
  HostPipe* hp = nullptr;
  rc = pipe_for(dev, &hp);
  if (rc != NSA_OK) return rc;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaEventRecord(hp->entry, cs);  // the copies follow earlier work on `stream`
  if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->h2d, hp->entry, 0);
  if (e != cudaSuccess) return cuda_fail(e, "ordering the host pipeline after the stream");
  int slice = 0;
  const int nslices = rows * per_row;
  for (int r = pl.bkv_begin; r < pl.bkv_end; ++r) {
    const int b = r / Hkv, kvh = r - (r / Hkv) * Hkv;
    for (int j = 0; j < per_row; ++j, ++slice) {
      const int qa = pl.qb_begin + (int)((long long)nqb * j / per_row);
      const int qe = pl.qb_begin + (int)((long long)nqb * (j + 1) / per_row);
      const int ta = qa * BQ, te = qe * BQ < T ? qe * BQ : T;
      const size_t head0 = ((size_t)b * Hq + (size_t)kvh * G) * T + ta;  // first (head, token) row
      if (j == 0) {  // the whole K/V row before the row's first kernel
        e = cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(d->k)) + (size_t)r * KVL * krow,
                            static_cast<const char*>(io->k) + (size_t)r * KVL * krow, KVL * krow,
                            cudaMemcpyHostToDevice, hp->h2d);
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(d->v)) + (size_t)r * KVL * vrow,
                              static_cast<const char*>(io->v) + (size_t)r * KVL * vrow, KVL * vrow,
                              cudaMemcpyHostToDevice, hp->h2d);
        if (e != cudaSuccess) return cuda_fail(e, "copying K/V to the device");
      }
      e = copy_rows(const_cast<void*>(d->q), io->q, head0 * qrow, (size_t)(te - ta) * qrow, (size_t)T * qrow, G,
                    cudaMemcpyHostToDevice, hp->h2d);
      if (e == cudaSuccess) {
        const size_t so = ((size_t)r * NQB + qa) * srow;
        e = cudaMemcpyAsync(reinterpret_cast<char*>(const_cast<int32_t*>(d->sel)) + so,
                            reinterpret_cast<const char*>(io->sel) + so, (size_t)(qe - qa) * srow,
                            cudaMemcpyHostToDevice, hp->h2d);
      }
      if (e == cudaSuccess) e = cudaEventRecord(hp->in[slice], hp->h2d);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, hp->in[slice], 0);
      if (e != cudaSuccess) return cuda_fail(e, "copying Q/sel to the device");
      nsa_sel_desc ds = *d;
      ds.bkv_begin = r;
      ds.bkv_end = r + 1;
      ds.qb_begin = qa;
      ds.qb_end = qe;
      rc = launch(&ds, stream);
      if (rc != NSA_OK) return rc;
      e = cudaEventRecord(hp->out[slice], cs);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(hp->d2h, hp->out[slice], 0);
      if (e == cudaSuccess)
        e = copy_rows(io->o, d->o, head0 * orow, (size_t)(te - ta) * orow, (size_t)T * orow, G,
                      cudaMemcpyDeviceToHost, hp->d2h);
      if (e == cudaSuccess && lse)
        e = copy_rows(io->lse, d->lse, head0 * 4, (size_t)(te - ta) * 4, (size_t)T * 4, G, cudaMemcpyDeviceToHost,
                      hp->d2h);
      if (e != cudaSuccess) return cuda_fail(e, "copying O/LSE to the host");
    }
  }
  (void)nslices;
  e = cudaEventRecord(hp->done, hp->d2h);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, hp->done, 0);
  if (e != cudaSuccess) return cuda_fail(e, "ordering the stream after the host pipeline");
  g_last_error[0] = '\0';
  return NSA_OK;
}

// ------------------------------------------------------------------ backward
struct BwdLayout {
  size_t off_delta, off_counts, off_fill, off_tok_off, off_item_off, off_tokens, off_items, total;
  int n_buckets, nsub, spb, n_blk, G, win_shift, n_win;
  long long max_pairs;
};

size_t align16(size_t x) { return (x + 15) / 16 * 16; }

int bwd_layout(const nsa_sel_bwd_desc* d, BwdLayout* L) {
  if (d == nullptr) return fail(NSA_ERR_INVALID_ARG, "desc is NULL");
  const int B = d->batch, Hq = d->heads_q, Hkv = d->heads_kv, T = d->seq_len;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || T <= 0) return fail(NSA_ERR_INVALID_ARG, "B, Hq, Hkv, T must be positive");
  if (Hq % Hkv != 0) return fail(NSA_ERR_INVALID_ARG, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  const int G = Hq / Hkv;
  if (G != 8 && G != 16) return fail(NSA_ERR_UNSUPPORTED, "backward: group size G=%d; built for G = 8 and 16", G);
  if (d->d != nsa::bwd::kD) return fail(NSA_ERR_UNSUPPORTED, "backward: d=%d; built for d = 128", d->d);
  if (d->block_size != 64 && d->block_size != 128 && d->block_size != 256)
    return fail(NSA_ERR_UNSUPPORTED, "l_prime=%d: the kernel family supports 64, 128 and 256", d->block_size);
  if (d->n_sel <= 0 || d->n_sel > 64) return fail(NSA_ERR_INVALID_ARG, "KSEL must be in 1..64");
  if (d->o_dtype != NSA_DTYPE_BF16 && d->o_dtype != NSA_DTYPE_F32)
    return fail(NSA_ERR_INVALID_ARG, "o_dtype must be NSA_DTYPE_BF16 or NSA_DTYPE_F32");
  if ((long long)T >= (1ll << 24) || (long long)B * Hq * T >= (1ll << 31))
    return fail(NSA_ERR_UNSUPPORTED, "problem too large for 32-bit token indices");
  L->G = G;
  L->spb = d->block_size / 64;
  L->n_blk = (T + d->block_size - 1) / d->block_size;
  L->nsub = (T + 63) / 64;
  // Token windows of the inverse index: the Q, dO (bf16) and dQ (fp32) rows of one window, G KB
  // per token, take 64 MB (half the L2); at most 32 windows per (b, kvh).
  int ws = G == 16 ? 12 : 13;
  while (ws < 24 && ((T + (1 << ws) - 1) >> ws) > 32) ++ws;
  L->win_shift = ws;
  L->n_win = (T + (1 << ws) - 1) >> ws;
  const long long n_bkv = (long long)B * Hkv;
  const long long nb = n_bkv * L->n_win * L->nsub;
  if (nb >= (1ll << 30)) return fail(NSA_ERR_UNSUPPORTED, "too many (b, kvh, window, sub-block) buckets");
  L->n_buckets = (int)nb;
  const long long per_row = std::min<long long>((long long)d->n_sel * L->spb, L->nsub);
  L->max_pairs = n_bkv * T * per_row;
  if (L->max_pairs >= (1ll << 31)) return fail(NSA_ERR_UNSUPPORTED, "selection index exceeds 2^31 entries");
  const long long max_items = L->max_pairs / nsa::bwd::kItemTokens + L->n_buckets;  // ceil per bucket
  size_t o = 0;
  L->off_delta = o; o = align16(o + (size_t)B * Hq * T * 4);
  L->off_counts = o; o = align16(o + (size_t)L->n_buckets * 4);
  L->off_fill = o; o = align16(o + (size_t)L->n_buckets * 4);
  L->off_tok_off = o; o = align16(o + (size_t)L->n_buckets * 4);
  L->off_item_off = o; o = align16(o + (size_t)(L->n_buckets + 1) * 4);
  L->off_tokens = o; o = align16(o + (size_t)L->max_pairs * 4);
  L->off_items = o; o = align16(o + (size_t)max_items * 16);
  L->total = o;
  return NSA_OK;
}

bool g_bwd_attr[kMaxDevices] = {};

int backward(const nsa_sel_bwd_desc* d, nsa_stream_t stream) {
  BwdLayout L;
  int rc = bwd_layout(d, &L);
  if (rc != NSA_OK) return rc;
  if (d->q == nullptr || d->k == nullptr || d->v == nullptr || d->sel == nullptr || d->o == nullptr ||
      d->lse == nullptr || d->d_o == nullptr || d->dq == nullptr || d->dk == nullptr || d->dv == nullptr ||
      d->workspace == nullptr)
    return fail(NSA_ERR_INVALID_ARG, "q, k, v, sel, o, lse, d_o, dq, dk, dv and workspace must be non-NULL");
  if (!aligned16(d->q) || !aligned16(d->k) || !aligned16(d->v) || !aligned16(d->o) || !aligned16(d->d_o) ||
      !aligned16(d->dq) || !aligned16(d->dk) || !aligned16(d->dv) || !aligned16(d->workspace))
    return fail(NSA_ERR_INVALID_ARG, "q, k, v, o, d_o, dq, dk, dv and workspace must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(d->sel) & 3u) != 0 || (reinterpret_cast<uintptr_t>(d->lse) & 3u) != 0)
    return fail(NSA_ERR_INVALID_ARG, "sel and lse must be 4-byte aligned");
  int sm = 0, dev = 0;
  rc = current_sm_count(&sm, &dev);
  if (rc != NSA_OK) return rc;
  const int B = d->batch, Hq = d->heads_q, Hkv = d->heads_kv, T = d->seq_len, G = L.G;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(d->workspace);
  float* delta = reinterpret_cast<float*>(ws + L.off_delta);
  int* counts = reinterpret_cast<int*>(ws + L.off_counts);
  int* fillc = reinterpret_cast<int*>(ws + L.off_fill);
  int* tok_off = reinterpret_cast<int*>(ws + L.off_tok_off);
  int* item_off = reinterpret_cast<int*>(ws + L.off_item_off);
  int32_t* tokens = reinterpret_cast<int32_t*>(ws + L.off_tokens);
  int4* items = reinterpret_cast<int4*>(ws + L.off_items);

  // Tensor maps.  Q, dO (bf16) and dQ (fp32) are [B, Hq, T, 128]; they are described as 5D views
  // (dims in element order: dimension-in-chunk, head-in-octet, dimension chunk, token, head octet
  // of the whole batch) so that one box holds a token's G heads x 128 dims laid out as 8-head
  // groups, each group's dimension chunks 1 KB apart -- the UMMA operand layout of the kernel.
  // The strides are not increasing (head before dimension chunk); the hardware only sums
  // coordinate x stride.  K and V per 64-key sub-block.
  CUtensorMap tmQ, tmDO, tmK, tmV, tmDQ;
  {
    const cuuint64_t dims[5] = {64, 8, 2, (cuuint64_t)T, (cuuint64_t)(Hq / 8) * B};
    const cuuint64_t str[4] = {256ull * T, 128, 256, 8ull * 256 * T};
    const cuuint32_t box[5] = {64, 8, 2, 1, (cuuint32_t)(G / 8)};
    rc = encode(&tmQ, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, d->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "Q");
    if (rc == NSA_OK)
      rc = encode(&tmDO, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, d->d_o, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "dO");
    if (rc != NSA_OK) return rc;
    const cuuint64_t dims32[5] = {32, 8, 4, (cuuint64_t)T, (cuuint64_t)(Hq / 8) * B};
    const cuuint64_t str32[4] = {512ull * T, 128, 512, 8ull * 512 * T};
    const cuuint32_t box32[5] = {32, 8, 2, 1, (cuuint32_t)(G / 8)};  // half of the dimensions
    rc = encode(&tmDQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, d->dq, dims32, str32, box32, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "dQ");
    if (rc != NSA_OK) return rc;
  }
  {
    const cuuint64_t dims[4] = {64, (cuuint64_t)T, 2, (cuuint64_t)B * Hkv};
    const cuuint64_t str[3] = {256, 128, 256ull * T};
    const cuuint32_t box[4] = {64, 64, 2, 1};
    rc = encode(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, d->k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "K");
    if (rc == NSA_OK)
      rc = encode(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, d->v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, "V");
    if (rc != NSA_OK) return rc;
  }
  {
    std::lock_guard<std::mutex> lk(g_dev.mu);
    if (!g_bwd_attr[dev]) {
      cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&nsa::bwd::nsa_bwd_kernel),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nsa::bwd::kSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(backward smem)");
      g_bwd_attr[dev] = true;
    }
  }

  // 1. row sums dO . O
  const long long rows = (long long)B * Hq * T;
  if (d->o_dtype == NSA_DTYPE_BF16)
    nsa::bwd::delta_kernel<__nv_bfloat16><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(d->d_o), static_cast<const __nv_bfloat16*>(d->o), delta, rows);
  else
    nsa::bwd::delta_kernel<float><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(d->d_o), static_cast<const float*>(d->o), delta, rows);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "backward row-sum kernel launch");
  // 2. inverse index: counts, offsets, token lists, work items
  e = cudaMemsetAsync(counts, 0, L.off_tok_off - L.off_counts, st);  // counts and fill counters
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(backward index counters)");
  nsa::bwd::IndexShape sh{B * Hkv, T, d->n_sel, L.spb, L.n_blk, L.nsub, nsa::bwd::kItemTokens, L.win_shift, L.n_win};
  const unsigned row_blocks = (unsigned)(((long long)B * Hkv * T + 255) / 256);
  nsa::bwd::index_rows_kernel<false><<<row_blocks, 256, 0, st>>>(d->sel, sh, counts, nullptr, nullptr, nullptr);
  nsa::bwd::index_scan_kernel<<<1, 1024, 0, st>>>(counts, L.n_buckets, nsa::bwd::kItemTokens, tok_off, item_off);
  nsa::bwd::index_rows_kernel<true><<<row_blocks, 256, 0, st>>>(d->sel, sh, nullptr, tok_off, fillc, tokens);
  nsa::bwd::index_items_kernel<<<(unsigned)((L.n_buckets + 255) / 256), 256, 0, st>>>(sh, counts, tok_off, item_off,
                                                                                      items);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "backward index kernel launch");
  // 3. gradients
  nsa::bwd::Params p{};
  p.tokens = tokens;
  p.items = reinterpret_cast<const int32_t*>(items);
  p.lse = d->lse;
  p.delta = delta;
  p.dk = d->dk;
  p.dv = d->dv;
  p.err = d->err;
  p.n_items_ptr = item_off + L.n_buckets;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.T = T;
  p.G = G;
  const double scale = d->scale > 0.f ? (double)d->scale : 1.0 / sqrt((double)d->d);
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634074);
  int tmo = d->timeout_ms;
  if (tmo <= 0) {
    const char* env = getenv("NSA_SEL_TIMEOUT_MS");
    tmo = env ? atoi(env) : 0;
    if (tmo <= 0) tmo = 2000;
  }
  p.timeout_ns = (unsigned long long)tmo * 1000000ull;
  int grid = sm;
  if (d->max_ctas > 0 && d->max_ctas < grid) grid = d->max_ctas;
  void* args[] = {&tmQ, &tmDO, &tmK, &tmV, &tmDQ, &p};
  e = cudaLaunchKernel(reinterpret_cast<const void*>(&nsa::bwd::nsa_bwd_kernel), dim3(grid),
                       dim3(nsa::bwd::kThreads), args, nsa::bwd::kSmemBytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "backward kernel launch");
  g_last_error[0] = '\0';
  return NSA_OK;
}

}  // namespace

extern "C" {

int64_t nsa_sel_backward_workspace_bytes(const nsa_sel_bwd_desc* desc) {
  BwdLayout L;
  if (bwd_layout(desc, &L) != NSA_OK) return -1;
  return (int64_t)L.total;
}

int nsa_sel_backward(const nsa_sel_bwd_desc* desc, nsa_stream_t stream) { return backward(desc, stream); }

int nsa_sel_run_host(const nsa_sel_desc* desc, const nsa_sel_host_io* io, nsa_stream_t stream) {
  return run_host(desc, io, stream);
}

int64_t nsa_sel_select_workspace_bytes(int32_t B, int32_t Hkv, int32_t T, int32_t d, int32_t l_prime) {
  if (B <= 0 || Hkv <= 0 || T <= 0 || d <= 0 || l_prime <= 0) return -1;
  const int64_t n_blk = (T + l_prime - 1) / l_prime;
  return (int64_t)B * Hkv * n_blk * d * (int64_t)sizeof(float);
}

int nsa_sel_select(const void* q, const void* k, float* kblk_workspace, int32_t* sel_out, int32_t B, int32_t Hq,
                   int32_t Hkv, int32_t T, int32_t d, int32_t l_prime, int32_t n_sel, int32_t cmp_block,
                   int32_t cmp_stride, nsa_stream_t stream) {
  if (q == nullptr || k == nullptr || kblk_workspace == nullptr || sel_out == nullptr)
    return fail(NSA_ERR_INVALID_ARG, "q, k, kblk_workspace and sel_out must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(kblk_workspace) & 15u) != 0)
    return fail(NSA_ERR_INVALID_ARG, "kblk_workspace must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0 || (reinterpret_cast<uintptr_t>(k) & 1u) != 0 ||
      (reinterpret_cast<uintptr_t>(sel_out) & 3u) != 0)
    return fail(NSA_ERR_INVALID_ARG, "q must be 16-byte aligned, k and sel_out aligned to their element size");
  int n_blk = 0, topk = 0, n_cmp = 0;
  int rc = select_shape(B, Hq, Hkv, T, d, l_prime, n_sel, cmp_block, cmp_stride, &n_blk, &topk, &n_cmp);
  if (rc != NSA_OK) return rc;
  int sm = 0, dev = 0;
  rc = current_sm_count(&sm, &dev);
  if (rc != NSA_OK) return rc;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float scale = (float)(1.0 / ((double)cmp_block * sqrt((double)d)));
  if (d == 64 || d == 128) return select_tc(q, k, kblk_workspace, sel_out, B, Hq, Hkv, T, d, l_prime, topk, n_blk,
                                            n_cmp, cmp_block, cmp_stride, scale, sm, dev, st);
  const int smem = (2 * nsa::select::kTile * (d + 4) + nsa::select::kTile * (nsa::select::kChunk + 1)) * 4;
  {
    std::lock_guard<std::mutex> lk(g_dev.mu);
    const uint64_t bit = 1ull << 63;
    if ((g_dev.attr_done[dev] & bit) == 0) {
      cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&nsa::select::select_kernel),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (2 * nsa::select::kTile * (nsa::select::kMaxD + 4) +
                                            nsa::select::kTile * (nsa::select::kChunk + 1)) * 4);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(select max dynamic smem)");
      g_dev.attr_done[dev] |= bit;
    }
  }
  nsa::select::kblk_kernel<false><<<dim3(n_blk, B * Hkv), d, 0, st>>>(static_cast<const bf16*>(k), kblk_workspace, T, d,
                                                               n_blk, n_cmp, l_prime, cmp_block, cmp_stride, scale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "block-key kernel launch");
  nsa::select::select_kernel<<<dim3((T + nsa::select::kTile - 1) / nsa::select::kTile, B * Hkv),
                               nsa::select::kThreads, smem, st>>>(static_cast<const bf16*>(q), kblk_workspace, sel_out,
                                                                  Hq, Hkv, T, d, n_blk, l_prime, topk);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selection kernel launch");
  g_last_error[0] = '\0';
  return NSA_OK;
}

int nsa_sel_select_noalloc(const void* q, const void* k, int32_t* sel_out, int32_t B, int32_t Hq, int32_t Hkv,
                           int32_t T, int32_t d, int32_t l_prime, int32_t n_sel, int32_t cmp_block,
                           int32_t cmp_stride, nsa_stream_t stream) {
  int n_blk = 0, topk = 0, n_cmp = 0;
  int rc = select_shape(B, Hq, Hkv, T, d, l_prime, n_sel, cmp_block, cmp_stride, &n_blk, &topk, &n_cmp);
  if (rc != NSA_OK) return rc;
  const int64_t need = nsa_sel_select_workspace_bytes(B, Hkv, T, d, l_prime);
  if (need < 0 || (uint64_t)need > kStaticSelectScratchFloats * sizeof(float))
    return fail(NSA_ERR_UNSUPPORTED, "selection needs %lld bytes of scratch; the static scratch holds %zu",
                (long long)need, kStaticSelectScratchFloats * sizeof(float));
  int sm = 0, dev = 0;
  rc = current_sm_count(&sm, &dev);
  if (rc != NSA_OK) return rc;
  float* scratch = nullptr;
  rc = static_select_scratch(dev, &scratch);
  if (rc != NSA_OK) return rc;
  return nsa_sel_select(q, k, scratch, sel_out, B, Hq, Hkv, T, d, l_prime, n_sel, cmp_block, cmp_stride, stream);
}

int64_t nsa_sel_select_static_scratch_bytes(void) { return (int64_t)(kStaticSelectScratchFloats * sizeof(float)); }

int32_t nsa_sel_select_status(void) {
  int sm = 0, dev = 0;
  if (current_sm_count(&sm, &dev) != NSA_OK) return -1;
  int32_t* w = nullptr;
  if (select_err_word(dev, &w) != NSA_OK) return -1;
  int32_t v = 0;
  if (cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  const int32_t zero = 0;
  if (cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess) return -1;
  return v;
}

int nsa_sel_run(const nsa_sel_desc* desc, nsa_stream_t stream) { return launch(desc, stream); }

int nsa_sel_plan(const nsa_sel_desc* desc, int32_t sm_count, nsa_sel_plan_info* out) {
  if (out == nullptr) return fail(NSA_ERR_INVALID_ARG, "out is NULL");
  int sm = sm_count;
  if (sm <= 0) {
    int dev = 0;
    int rc = current_sm_count(&sm, &dev);
    if (rc != NSA_OK) return rc;
  }
  Plan pl;
  int rc = make_plan(desc, sm, &pl);
  if (rc != NSA_OK) return rc;
  int nv = 0;
  const Variant& V = variants(&nv)[pl.variant];
  memset(out, 0, sizeof(*out));
  out->n_cols = pl.ncol;
  out->q_per_unit = pl.BQs;
  out->parts = pl.parts;
  out->n_units = pl.n_units;
  out->k_stages = pl.KS;
  out->v_stages = pl.VS;
  out->smem_bytes = (int32_t)pl.layout.total;
  out->grid = pl.grid;
  out->tmem_cols = V.tmem_cols;
  g_last_error[0] = '\0';
  return NSA_OK;
}

int nsa_sel_forward(const void* q, const void* k, const void* v, const int32_t* sel, float* o, int64_t* cyc,
                    int32_t B, int32_t Hq, int32_t Hkv, int32_t S, int32_t D, int32_t NQB, int32_t KSEL,
                    int32_t l_prime, int32_t BQ, nsa_stream_t stream) {
  nsa_sel_desc d;
  memset(&d, 0, sizeof(d));
  d.q = q;
  d.k = k;
  d.v = v;
  d.sel = sel;
  d.o = o;
  d.cyc = cyc;
  d.batch = B;
  d.heads_q = Hq;
  d.heads_kv = Hkv;
  d.seq_len = S;
  d.d_qk = D;
  d.d_v = D;
  d.n_qblocks = NQB;
  d.n_sel = KSEL;
  d.block_size = l_prime;
  d.q_block = BQ;
  d.o_dtype = NSA_DTYPE_F32;
  return launch(&d, stream);
}

int nsa_sel_forward_lse(const void* q, const void* k, const void* v, const int32_t* sel,
                        const int32_t* cu_seqlens, int32_t n_seqs, void* o, float* lse, int32_t o_dtype, int32_t B,
                        int32_t Hq, int32_t Hkv, int32_t T, int32_t d_qk, int32_t d_v, int32_t NQB, int32_t KSEL,
                        int32_t l_prime, int32_t BQ, float scale, nsa_stream_t stream) {
  nsa_sel_desc d;
  memset(&d, 0, sizeof(d));
  d.q = q;
  d.k = k;
  d.v = v;
  d.sel = sel;
  d.cu_seqlens = cu_seqlens;
  d.n_seqs = n_seqs;
  d.o = o;
  d.lse = lse;
  d.batch = B;
  d.heads_q = Hq;
  d.heads_kv = Hkv;
  d.seq_len = T;
  d.d_qk = d_qk;
  d.d_v = d_v;
  d.n_qblocks = NQB;
  d.n_sel = KSEL;
  d.block_size = l_prime;
  d.q_block = BQ;
  d.o_dtype = o_dtype;
  d.scale = scale;
  return launch(&d, stream);
}

const char* nsa_sel_last_error(void) { return g_last_error; }

int32_t nsa_sel_version(void) { return NSA_SEL_VERSION; }

}  // extern "C"
