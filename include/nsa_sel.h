/*
 * nsa_sel.h -- C ABI of the B200 (sm_100a) NSA selected-branch attention forward, with the
 * block selection that produces its index rows and the backward that the reference lacks.
 *
 * This is the drop-in boundary for the one hot path of the nsa-hopper reference: the
 * selected-branch forward that its kernels expose through pybind as
 *
 *     torch::Tensor forward(Tensor Q, Tensor K, Tensor V, Tensor sel,
 *                           int64 l_prime, int64 BQ, Tensor cyc)
 *
 * (reference nsa_v0.cu:118-146, nsa_v1.cu:125-147, nsa_v2.cu:147-170).  Every entry point
 * takes plain pointers and sizes; no torch type crosses this boundary.  The library never
 * calls cudaMalloc: all buffers belong to the caller, except one static device array inside the
 * library (16 MB) that only nsa_sel_select_noalloc uses.  All launches go to the stream
 * passed in; a call returns as soon as the work is queued (like the reference op, which is
 * asynchronous on the legacy stream).  The library is reentrant: concurrent calls from
 * several host threads are safe, and the error text is kept per host thread.  Two exceptions
 * share device state between calls: nsa_sel_select_noalloc (one static scratch per device:
 * calls on one device must be serialised, e.g. on one stream), and replays of one captured CUDA
 * graph (each captured forward launch owns one work-counter slot: replays of the same graph
 * must not overlap each other).
 *
 * Layouts (all contiguous, row-major, as in the reference):
 *   Q   bf16 [B, Hq,  T, d_qk]        K bf16 [B, Hkv, T, d_qk]      V bf16 [B, Hkv, T, d_v]
 *   sel int32 [B, Hkv, NQB, KSEL]    NQB = ceil(T / BQ); entry = block index (block = l_prime
 *                                     keys); negative entries are padding and are skipped
 *   O   [B, Hq, T, d_v]  bf16 or fp32 (every element is written; rows with no visible key = 0)
 *   LSE fp32 [B, Hq, T]  natural log of sum_j exp(scale * q.k_j) over the visible keys
 *                        (-inf for a row with no visible key)
 *   cyc int64 [NQB * B * Hkv * 2]  optional; slot (b*Hkv+kvh)*NQB+qb holds
 *                        {cycles the MMA issuer waited for K/V tiles, other cycles}
 *
 * Semantics (pinned against the reference's PyTorch oracle ref_only.py:2-20 and
 * nsa_reference.py:18-25,66-77): query token t of KV head kvh attends to every key position
 * p with p <= t inside the selected blocks of its query block; selection is a set
 * (duplicates count once); entries < 0 or >= ceil(T / l_prime) select nothing; the softmax
 * scale defaults to 1/sqrt(d_qk); a row with no visible key gives O = 0.
 */
#ifndef NSA_SEL_H_
#define NSA_SEL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* nsa_stream_t;

#define NSA_SEL_VERSION 10000 /* 1.0.0 */

/* Return codes (0 = success). */
#define NSA_OK 0
#define NSA_ERR_INVALID_ARG (-1) /* bad pointer, shape, stride or alignment */
#define NSA_ERR_UNSUPPORTED (-2) /* valid request outside the built kernel family */
#define NSA_ERR_CUDA (-3)        /* a CUDA runtime call failed; see nsa_sel_last_error() */
#define NSA_ERR_DRIVER (-4)      /* the driver entry point for tensor maps is unavailable */

/* Bits a kernel ORs into the optional device error word (nsa_sel_desc.err). */
#define NSA_DEVERR_TIMEOUT 1 /* a bounded wait inside the kernel ran out; outputs invalid */

/* Test hook: the MMA warp starts with a wait that nothing completes, so the launch ends through
   the bounded-wait error path (NSA_DEVERR_TIMEOUT after timeout_ms) without any fault. */
#define NSA_DEBUG_STALL 1
/* Comparison switches (same results, different schedule): hand out work units in fixed strides
   instead of from the dynamic counter; never use the row-owner kernel for 64/128-row tiles; run a
   64-row tile of the row-owner kernel as 128-row MMAs with 64 rows of zero padding instead of
   M = 64 MMAs. */
#define NSA_DEBUG_STATIC_UNITS 2
#define NSA_DEBUG_NO_ROW_OWNER 4
#define NSA_DEBUG_RO_PAD128 8

#define NSA_DTYPE_BF16 0
#define NSA_DTYPE_F32 1

#define NSA_KEYMAP_CAUSAL 0     /* key position p is visible to query t iff p <= t */
#define NSA_KEYMAP_COMPRESSED 1 /* compressed key i is visible iff linspace(0, T-1, kv_len)[i] <= t */

/* Full description of one call.  Zero-initialise, then fill the fields you need. */
typedef struct nsa_sel_desc {
  const void* q;              /* bf16 [B, Hq, T, d_qk] */
  const void* k;              /* bf16 [B, Hkv, T, d_qk] */
  const void* v;              /* bf16 [B, Hkv, T, d_v] */
  const int32_t* sel;         /* int32 [B, Hkv, NQB, KSEL] */
  const int32_t* cu_seqlens;  /* optional int32 [n_seqs + 1]: packed varlen batch (B == 1, BQ == 1);
                                 block ids are relative to each sequence's first token */
  void* o;                    /* [B, Hq, T, d_v], dtype o_dtype */
  float* lse;                 /* optional fp32 [B, Hq, T] */
  int64_t* cyc;               /* optional int64 [NQB * B * Hkv * 2], accumulated into */
  int32_t* err;               /* optional device int32; NSA_DEVERR_* bits are ORed into it */
  int32_t batch, heads_q, heads_kv, seq_len, d_qk, d_v;
  int32_t n_qblocks;          /* NQB, must equal ceil(seq_len / q_block) */
  int32_t n_sel;              /* KSEL */
  int32_t block_size;         /* l_prime: 64, 128 or 256 */
  int32_t q_block;            /* BQ: query tokens sharing one selection row (1 = per token) */
  int32_t n_seqs;             /* number of sequences when cu_seqlens is set */
  int32_t o_dtype;            /* NSA_DTYPE_BF16 or NSA_DTYPE_F32 */
  float scale;                /* softmax scale; <= 0 selects 1/sqrt(d_qk) */
  /* Shard: process only (b*Hkv+kvh) in [bkv_begin, bkv_end) and query blocks in
     [qb_begin, qb_end); an end of 0 means "to the end".  Outputs outside the shard are
     left untouched. */
  int32_t bkv_begin, bkv_end, qb_begin, qb_end;
  int32_t timeout_ms;         /* bound on every in-kernel wait; 0 = default (2000 ms) */
  int32_t max_ctas;           /* 0 = one CTA per SM */
  int32_t debug_flags;        /* NSA_DEBUG_* bits; 0 in normal use */
  /* Key visibility beyond the causal default (the sliding-window and compressed branches of NSA,
     reference nsa_reference.py:59-64 and 79-82, run on the same kernel): */
  int32_t kv_len;             /* K/V rows per (b, kvh); 0 = seq_len.  Other values need
                                 key_map = NSA_KEYMAP_COMPRESSED (then K, V are [B, Hkv, kv_len, d]) */
  int32_t window;             /* > 0: key p is visible to query t only if t - p < window (causal
                                 key map only; not with cu_seqlens) */
  int32_t key_map;            /* NSA_KEYMAP_CAUSAL: key p visible to query t iff p <= t;
                                 NSA_KEYMAP_COMPRESSED: key i visible iff the float32
                                 linspace(0, seq_len-1, kv_len)[i] <= t (not with cu_seqlens) */
  /* Fused output combination (the NSA gate, reference nsa_reference.py:86-88): */
  int32_t o_accumulate;       /* 0: O is overwritten; 1: O += w * result (fp32 O only; TMA reduce-add) */
  int32_t reserved;
  const float* o_weight;      /* optional device float w multiplying the result; NULL = 1 */
} nsa_sel_desc;

/* Launch plan chosen for a description (filled by nsa_sel_plan, used by the launcher). */
typedef struct nsa_sel_plan_info {
  int32_t n_cols;       /* N of the tensor-core tiles: G * q_tokens_per_unit rounded up */
  int32_t q_per_unit;   /* query tokens per work unit */
  int32_t parts;        /* work units per query block */
  int32_t n_units;      /* work units in the shard */
  int32_t k_stages, v_stages;
  int32_t smem_bytes;
  int32_t grid;
  int32_t tmem_cols;
  int32_t reserved[7];
} nsa_sel_plan_info;

/* Replaces the reference's forward(Q,K,V,sel,l_prime,BQ,cyc) (nsa_v2.cu:147-170,
   nsa_v1.cu:125-147, nsa_v0.cu:118-146): fp32 O, d_qk == d_v == D, scale 1/sqrt(D).
   cyc may be NULL (the reference passes an empty tensor for "none", nsa_v2.cu:159). */
int nsa_sel_forward(const void* q, const void* k, const void* v, const int32_t* sel, float* o, int64_t* cyc,
                    int32_t B, int32_t Hq, int32_t Hkv, int32_t S, int32_t D, int32_t NQB, int32_t KSEL,
                    int32_t l_prime, int32_t BQ, nsa_stream_t stream);

/* The BASELINE path: bf16 O plus fp32 LSE, d_qk may differ from d_v, optional varlen.
   Extends the same reference op (nsa_v2.cu:147) with the outputs the reference lacks. */
int nsa_sel_forward_lse(const void* q, const void* k, const void* v, const int32_t* sel,
                        const int32_t* cu_seqlens, int32_t n_seqs, void* o, float* lse, int32_t o_dtype,
                        int32_t B, int32_t Hq, int32_t Hkv, int32_t T, int32_t d_qk, int32_t d_v, int32_t NQB,
                        int32_t KSEL, int32_t l_prime, int32_t BQ, float scale, nsa_stream_t stream);

/* General entry point: everything above plus shards, cycle counters, a device error word
   and the wait bound.  Same reference op (nsa_v2.cu:147-170). */
int nsa_sel_run(const nsa_sel_desc* desc, nsa_stream_t stream);

/* Host buffers for nsa_sel_run_host (same layouts as the device buffers of the descriptor;
   pinned host memory lets the copies overlap the kernel). */
typedef struct nsa_sel_host_io {
  const void* q;              /* [B, Hq, T, d_qk] bf16 */
  const void* k;              /* [B, Hkv, kv_len, d_qk] bf16 */
  const void* v;              /* [B, Hkv, kv_len, d_v] bf16 */
  const int32_t* sel;         /* [B, Hkv, NQB, KSEL] */
  void* o;                    /* [B, Hq, T, d_v], dtype o_dtype; receives O */
  float* lse;                 /* optional [B, Hq, T]; receives the LSE when desc->lse is set */
  int32_t token_slices;       /* query-block ranges per (b, kvh) row; 0 = automatic */
  int32_t reserved[7];
} nsa_sel_host_io;

/* The same forward for a caller whose tensors live in host memory (the reference op takes
   whatever tensors it is given, nsa_v2.cu:147-170): copies the inputs of the descriptor's shard
   into its device buffers, runs the kernel and copies O (and LSE) back, pipelined over (b, kvh)
   rows x token slices so that the host-to-device copy of slice i+1, the kernel on slice i and the
   device-to-host copy of slice i-1 overlap (two library-owned copy streams, ordered against
   `stream` with events; no device memory is allocated).  Asynchronous: the host outputs are
   complete when `stream` reaches the point after this call.  o_accumulate must be 0;
   cu_seqlens, when set, must already be in device memory. */
int nsa_sel_run_host(const nsa_sel_desc* desc, const nsa_sel_host_io* io, nsa_stream_t stream);

/* Validate a description and report the launch plan without touching the GPU.
   sm_count <= 0 means "query the current device". */
int nsa_sel_plan(const nsa_sel_desc* desc, int32_t sm_count, nsa_sel_plan_info* out);

/* Block selection: the producer of the selected branch's index rows (replaces the PyTorch
   select_blocks of reference nsa_reference.py:27-44, with compress_kv :5-16 and the group-summed
   queries of :70-71).  For every (b, kvh, token t) it scores selection block nb as
       s(t, nb) = (sum_g q[b, kvh*G + g, t, :]) . kblk[b, kvh, nb, :],
       kblk[nb] = 1/sqrt(d) * sum over compressed keys i of block nb of
                  mean_{j < cmp_block} k[b, kvh, i*cmp_stride + j, :],
   where compressed key i belongs to block floor(linspace(0, T-1, n_cmp)[i] / l_prime) (float32,
   clamped to the last block; n_cmp = (T - cmp_block) / cmp_stride + 1), and writes
       sel_out int32 [B, Hkv, T, k],  k = min(n_sel, ceil(T / l_prime)) <= 32,
   the k best visible blocks (nb * l_prime <= t) by score, highest first; -1 where fewer than k
   blocks are visible (the reference's topk returns masked future blocks there, which the
   selected branch ignores in the same way).  q, k bf16 as in nsa_sel_forward (d_qk = d,
   d % 8 == 0, d <= 256; q 16-byte aligned); kblk_workspace: caller-owned buffer of
   nsa_sel_select_workspace_bytes() bytes, 16-byte aligned.  Two kernel launches on `stream`.
   For d = 64 and 128 the scores run on the tensor cores with each operand split into two bf16
   parts (hi + lo, three products accumulated in fp32: about 16 bits of each operand, ranking
   equal to fp32 scores except at near-ties); other d use fp32 FMA.  The tensor-core kernel's
   in-kernel waits are bounded; nsa_sel_select_status() reports one that ran out. */
int nsa_sel_select(const void* q, const void* k, float* kblk_workspace, int32_t* sel_out, int32_t B, int32_t Hq,
                   int32_t Hkv, int32_t T, int32_t d, int32_t l_prime, int32_t n_sel, int32_t cmp_block,
                   int32_t cmp_stride, nsa_stream_t stream);

/* Bytes of the workspace nsa_sel_select needs (B * Hkv * ceil(T / l_prime) * d * 4), -1 if
   an argument is not positive. */
int64_t nsa_sel_select_workspace_bytes(int32_t B, int32_t Hkv, int32_t T, int32_t d, int32_t l_prime);

/* nsa_sel_select without a caller workspace and without any allocation: the block-key table is
   kept in a static device array of nsa_sel_select_static_scratch_bytes() bytes inside the
   library (its address is resolved once per device with cudaGetSymbolAddress; the library
   never calls cudaMalloc).  Requests whose workspace would exceed it return
   NSA_ERR_UNSUPPORTED without launching.  The scratch is shared per device: calls on one device
   must not run concurrently on different streams. */
int nsa_sel_select_noalloc(const void* q, const void* k, int32_t* sel_out, int32_t B, int32_t Hq, int32_t Hkv,
                           int32_t T, int32_t d, int32_t l_prime, int32_t n_sel, int32_t cmp_block,
                           int32_t cmp_stride, nsa_stream_t stream);

/* Backward of the selected-branch forward.  The reference has no backward pass (its README
   (2).md:85 lists it as missing); these entry points give the gradients of the same attention
   (ref_only.py:2-20, nsa_reference.py:18-25) with respect to Q, K and V:
       P = exp(scale * q.k - LSE),  dP = dO . v,  dS = P * (dP - sum_d dO * O),
       dQ = scale * dS K,  dK = scale * dS^T Q,  dV = P^T dO
   over the keys each query token sees in the forward (per-token selection, BQ == 1; same
   duplicate, padding and causal rules).  Supported: d_qk == d_v == 128, G = Hq / Hkv in {8, 16},
   l_prime in {64, 128, 256}, no cu_seqlens.  Zero-initialise, then fill the fields. */
typedef struct nsa_sel_bwd_desc {
  const void* q;              /* bf16 [B, Hq, T, 128] */
  const void* k;              /* bf16 [B, Hkv, T, 128] */
  const void* v;              /* bf16 [B, Hkv, T, 128] */
  const int32_t* sel;         /* int32 [B, Hkv, T, KSEL] */
  const void* o;              /* the forward's O [B, Hq, T, 128], dtype o_dtype */
  const float* lse;           /* the forward's LSE, fp32 [B, Hq, T] */
  const void* d_o;            /* bf16 [B, Hq, T, 128]: gradient of the loss with respect to O */
  float* dq;                  /* fp32 [B, Hq, T, 128]  } accumulated into (atomic adds): */
  float* dk;                  /* fp32 [B, Hkv, T, 128] } zero them first for plain gradients */
  float* dv;                  /* fp32 [B, Hkv, T, 128] } */
  void* workspace;            /* nsa_sel_backward_workspace_bytes() bytes, 16-byte aligned */
  int32_t* err;               /* optional device int32; NSA_DEVERR_* bits are ORed into it */
  int32_t batch, heads_q, heads_kv, seq_len, d;
  int32_t n_sel;              /* KSEL */
  int32_t block_size;         /* l_prime: 64, 128 or 256 */
  int32_t o_dtype;            /* NSA_DTYPE_BF16 or NSA_DTYPE_F32 */
  float scale;                /* softmax scale of the forward; <= 0 selects 1/sqrt(d) */
  int32_t timeout_ms;         /* bound on every in-kernel wait; 0 = default (2000 ms) */
  int32_t max_ctas;           /* 0 = one CTA per SM */
  int32_t reserved[5];
} nsa_sel_bwd_desc;

/* Bytes of the workspace nsa_sel_backward needs for a description, or -1 if the description is
   invalid (see nsa_sel_last_error()): the row sums dO . O (4 * B*Hq*T bytes) and the inverse
   selection index, i.e. about 4.2 bytes per (token, selected 64-key sub-block) pair (at most
   B*Hkv*T*KSEL*l_prime/64 of them) plus 32 bytes per bucket, a bucket being one (b, kvh, token
   window, sub-block): B*Hkv * ceil(T/64) * (number of windows, at most 32). */
int64_t nsa_sel_backward_workspace_bytes(const nsa_sel_bwd_desc* desc);

/* Adds dQ, dK, dV for the description on `stream` (six kernel launches and one memset, no
   allocation, asynchronous): the row sums dO . O, the inverse index (per (b, kvh, 64-key
   sub-block) the tokens that attend to it) and the tcgen05 gradient kernel.  The sums are
   accumulated with atomic adds, so the last bits may differ between runs. */
int nsa_sel_backward(const nsa_sel_bwd_desc* desc, nsa_stream_t stream);

/* Size in bytes of the static scratch used by nsa_sel_select_noalloc. */
int64_t nsa_sel_select_static_scratch_bytes(void);

/* NSA_DEVERR_* bits that selection launches on the current device set since the last call (0 =
   none), cleared on return; -1 if the device cannot be queried.  Synchronous: it waits for the
   device's pending work through a blocking copy. */
int32_t nsa_sel_select_status(void);

/* Text of the last error on this host thread ("" if none). */
const char* nsa_sel_last_error(void);

/* NSA_SEL_VERSION of the loaded library. */
int32_t nsa_sel_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NSA_SEL_H_ */
