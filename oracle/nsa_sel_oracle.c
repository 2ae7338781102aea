/*
 * nsa_sel_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the nsa-hopper reference's selected-branch forward.  It is the checker
 * used by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg; the product
 * (the sm_100a kernel behind include/nsa_sel.h) never calls it.
 *
 * Algorithm, per (batch b, KV head kvh, query token t) -- ref_only.py:2-20:
 *   qb   = t / BQ                                   (ref_only.py:14, repeat_interleave(BQ))
 *   keep = set of block ids in sel[b, kvh, qb, :]   (ref_only.py:8-12: scatter_ into a bool row;
 *          negative ids and id == n_blk go to a discarded scratch column; an id > n_blk makes
 *          the reference raise, which strict mode reports as NSA_ORACLE_ERR_INDEX)
 *   keys = { p : p / l_prime in keep, p < S, p <= t }   (ref_only.py:13-16, causal tril)
 *   for each query head h = kvh*G + g (ref_only.py:16, repeat_interleave(G, 1)):
 *     s_p = (q_h . k_p) * scale, scale = 1/sqrt(d_qk)   (ref_only.py:17)
 *     O   = softmax(s) @ V, a row with no key gives 0   (ref_only.py:18-20, nan_to_num)
 *     LSE = log(sum_p exp(s_p)) (-inf with no key)      (not in the reference; same convention
 *                                                        as nsa_reference.py:22-23's softmax)
 * Varlen (cu_seqlens): token t of sequence [c0, c1) uses block ids relative to c0, keys in
 * [c0, c1), n_blk = ceil((c1 - c0) / l_prime).  The reference has no varlen; this is the
 * natural restatement of the same rule per sequence.
 *
 * Inputs are bf16 bit patterns (uint16); the arithmetic is double (nsa_oracle_forward) or
 * float (nsa_oracle_forward_f32, the "reference math in fp32" used as the timed CPU baseline).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define NSA_ORACLE_OK 0
#define NSA_ORACLE_ERR_ARG (-1)
#define NSA_ORACLE_ERR_INDEX (-2)
#define NSA_ORACLE_ERR_NOMEM (-3)

static inline float bf16_to_f32(uint16_t h) {
  union {
    uint32_t u;
    float f;
  } c;
  c.u = ((uint32_t)h) << 16;
  return c.f;
}

typedef struct {
  const uint16_t *q, *k, *v;
  const int32_t* sel;
  const int32_t* cu;
  int n_seqs, B, Hq, Hkv, T, dqk, dv, NQB, KSEL, LP, BQ, strict;
  double scale;
  /* q, o and lse hold tokens [tq0, tq0 + Tq) of every (b, head): the full sequence (tq0 = 0,
     Tq = T) or only the computed row window (the *_window entry points). */
  int tq0, Tq;
} oracle_args;

/* Locate the sequence [c0, c1) holding token t (whole range when not varlen). */
static void seq_bounds(const oracle_args* a, int t, int* c0, int* c1) {
  if (a->cu == NULL) {
    *c0 = 0;
    *c1 = a->T;
    return;
  }
  int lo = 0, hi = a->n_seqs;
  while (hi - lo > 1) {
    int mid = (lo + hi) / 2;
    if (a->cu[mid] <= t) lo = mid; else hi = mid;
  }
  *c0 = a->cu[lo];
  *c1 = a->cu[lo + 1];
}

/* Fills `keys` (ascending key positions visible to token t) and returns their count, or a
   negative error.  `keep` has room for n_blk + 1 flags. */
static int visible_keys(const oracle_args* a, int b, int kvh, int t, unsigned char* keep, int* keys) {
  int c0, c1;
  seq_bounds(a, t, &c0, &c1);
  const int n_blk = (c1 - c0 + a->LP - 1) / a->LP;
  memset(keep, 0, (size_t)n_blk + 1);
  const int qb = t / a->BQ;
  const int32_t* row = a->sel + ((size_t)(b * a->Hkv + kvh) * a->NQB + qb) * a->KSEL;
  for (int j = 0; j < a->KSEL; ++j) {
    const int idx = row[j];
    if (idx < 0 || idx == n_blk) continue; /* scratch column */
    if (idx > n_blk) {
      if (a->strict) return NSA_ORACLE_ERR_INDEX;
      continue;
    }
    keep[idx] = 1;
  }
  int n = 0;
  for (int blk = 0; blk < n_blk; ++blk) {
    if (!keep[blk]) continue;
    for (int r = 0; r < a->LP; ++r) {
      const int p = c0 + blk * a->LP + r;
      if (p >= c1 || p > t) break;
      keys[n++] = p;
    }
  }
  return n;
}

#define ORACLE_BODY(REAL, EXPF, LOGF)                                                                         \
  const int G = a->Hq / a->Hkv;                                                                               \
  const long long rows = (long long)(bkv_end - bkv_begin) * (t_end - t_begin);                               \
  int status = NSA_ORACLE_OK;                                                                                 \
  _Pragma("omp parallel num_threads(nthreads)") {                                                            \
    unsigned char* keep = (unsigned char*)malloc((size_t)a->T + 2);                                           \
    int* keys = (int*)malloc(sizeof(int) * ((size_t)a->KSEL * a->LP + 1));                                    \
    REAL* kf = (REAL*)malloc(sizeof(REAL) * (size_t)a->KSEL * a->LP * a->dqk + sizeof(REAL));                 \
    REAL* sc = (REAL*)malloc(sizeof(REAL) * (size_t)a->KSEL * a->LP + sizeof(REAL));                          \
    REAL* qf = (REAL*)malloc(sizeof(REAL) * (size_t)a->dqk);                                                  \
    REAL* acc = (REAL*)malloc(sizeof(REAL) * (size_t)a->dv);                                                  \
    if (!keep || !keys || !kf || !sc || !qf || !acc) {                                                        \
      _Pragma("omp atomic write") status = NSA_ORACLE_ERR_NOMEM;                                              \
    } else {                                                                                                  \
      _Pragma("omp for schedule(dynamic, 8)") for (long long rr = 0; rr < rows; ++rr) {                       \
        const int bkv = bkv_begin + (int)(rr / (t_end - t_begin));                                            \
        const int t = t_begin + (int)(rr % (t_end - t_begin));                                                \
        const int b = bkv / a->Hkv, kvh = bkv % a->Hkv;                                                       \
        const int n = visible_keys(a, b, kvh, t, keep, keys);                                                 \
        if (n < 0) {                                                                                          \
          _Pragma("omp atomic write") status = n;                                                             \
          continue;                                                                                           \
        }                                                                                                     \
        const uint16_t* kbase = a->k + (size_t)bkv * a->T * a->dqk;                                           \
        const uint16_t* vbase = a->v + (size_t)bkv * a->T * a->dv;                                            \
        for (int j = 0; j < n; ++j)                                                                           \
          for (int d = 0; d < a->dqk; ++d) kf[(size_t)j * a->dqk + d] = bf16_to_f32(kbase[(size_t)keys[j] * a->dqk + d]); \
        for (int g = 0; g < G; ++g) {                                                                         \
          const int h = kvh * G + g;                                                                          \
          const size_t qrow = ((size_t)(b * a->Hq + h) * a->Tq + (t - a->tq0));                               \
          for (int d = 0; d < a->dqk; ++d) qf[d] = bf16_to_f32(a->q[qrow * a->dqk + d]);                      \
          REAL mx = -INFINITY;                                                                                \
          for (int j = 0; j < n; ++j) {                                                                       \
            const REAL* kr = kf + (size_t)j * a->dqk;                                                         \
            REAL s0 = 0, s1 = 0, s2 = 0, s3 = 0;                                                              \
            int d = 0;                                                                                        \
            for (; d + 4 <= a->dqk; d += 4) {                                                                 \
              s0 += qf[d] * kr[d];                                                                            \
              s1 += qf[d + 1] * kr[d + 1];                                                                    \
              s2 += qf[d + 2] * kr[d + 2];                                                                    \
              s3 += qf[d + 3] * kr[d + 3];                                                                    \
            }                                                                                                 \
            for (; d < a->dqk; ++d) s0 += qf[d] * kr[d];                                                      \
            sc[j] = ((s0 + s1) + (s2 + s3)) * (REAL)a->scale;                                                 \
            if (sc[j] > mx) mx = sc[j];                                                                       \
          }                                                                                                   \
          REAL sum = 0;                                                                                       \
          for (int d = 0; d < a->dv; ++d) acc[d] = 0;                                                         \
          for (int j = 0; j < n; ++j) {                                                                       \
            const REAL pj = EXPF(sc[j] - mx);                                                                 \
            sum += pj;                                                                                        \
            const uint16_t* vr = vbase + (size_t)keys[j] * a->dv;                                             \
            for (int d = 0; d < a->dv; ++d) acc[d] += pj * (REAL)bf16_to_f32(vr[d]);                          \
          }                                                                                                   \
          REAL* orow = o + qrow * a->dv;                                                                      \
          if (n == 0) {                                                                                       \
            for (int d = 0; d < a->dv; ++d) orow[d] = 0;                                                      \
            if (lse) lse[qrow] = -INFINITY;                                                                   \
          } else {                                                                                            \
            const REAL inv = (REAL)1 / sum;                                                                   \
            for (int d = 0; d < a->dv; ++d) orow[d] = acc[d] * inv;                                           \
            if (lse) lse[qrow] = mx + LOGF(sum);                                                              \
          }                                                                                                   \
        }                                                                                                     \
      }                                                                                                       \
    }                                                                                                         \
    free(keep);                                                                                               \
    free(keys);                                                                                               \
    free(kf);                                                                                                 \
    free(sc);                                                                                                 \
    free(qf);                                                                                                 \
    free(acc);                                                                                                \
  }                                                                                                           \
  return status;

static int check_args(const oracle_args* a, int bkv_begin, int bkv_end, int t_begin, int t_end, const void* o) {
  if (!a->q || !a->k || !a->v || !a->sel || !o) return NSA_ORACLE_ERR_ARG;
  if (a->B <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->T <= 0 || a->Hq % a->Hkv) return NSA_ORACLE_ERR_ARG;
  if (a->dqk <= 0 || a->dv <= 0 || a->KSEL <= 0 || a->LP <= 0 || a->BQ <= 0) return NSA_ORACLE_ERR_ARG;
  if (a->NQB != (a->T + a->BQ - 1) / a->BQ) return NSA_ORACLE_ERR_ARG;
  if (a->cu && (a->B != 1 || a->BQ != 1 || a->n_seqs <= 0)) return NSA_ORACLE_ERR_ARG;
  if (bkv_begin < 0 || bkv_end > a->B * a->Hkv || bkv_begin >= bkv_end) return NSA_ORACLE_ERR_ARG;
  if (t_begin < 0 || t_end > a->T || t_begin >= t_end) return NSA_ORACLE_ERR_ARG;
  return NSA_ORACLE_OK;
}

#define ORACLE_SETUP(WINDOW)                                                                                  \
  oracle_args A = {q, k, v, sel, cu_seqlens, n_seqs, B, Hq, Hkv, T, dqk, dv, NQB, KSEL, LP, BQ, strict,      \
                   scale > 0 ? scale : 1.0 / sqrt((double)dqk), 0, T};                                        \
  oracle_args* a = &A;                                                                                        \
  if (bkv_end <= 0) bkv_end = B * Hkv;                                                                        \
  if (t_end <= 0) t_end = T;                                                                                  \
  if (nthreads <= 0) nthreads = 1;                                                                            \
  {                                                                                                           \
    int rc = check_args(a, bkv_begin, bkv_end, t_begin, t_end, o);                                            \
    if (rc) return rc;                                                                                        \
  }                                                                                                           \
  if (WINDOW) {                                                                                               \
    a->tq0 = t_begin;                                                                                         \
    a->Tq = t_end - t_begin;                                                                                  \
  }

/* Rows (b*Hkv+kvh in [bkv_begin, bkv_end), t in [t_begin, t_end)) are computed; others are
   left untouched.  bkv_end/t_end <= 0 mean "to the end". */
int nsa_oracle_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* sel,
                       const int32_t* cu_seqlens, int n_seqs, int B, int Hq, int Hkv, int T, int dqk, int dv,
                       int NQB, int KSEL, int LP, int BQ, double scale, int bkv_begin, int bkv_end, int t_begin,
                       int t_end, int strict, double* o, double* lse, int nthreads) {
  ORACLE_SETUP(0);
  ORACLE_BODY(double, exp, log)
}

int nsa_oracle_forward_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* sel,
                           const int32_t* cu_seqlens, int n_seqs, int B, int Hq, int Hkv, int T, int dqk, int dv,
                           int NQB, int KSEL, int LP, int BQ, double scale, int bkv_begin, int bkv_end,
                           int t_begin, int t_end, int strict, float* o, float* lse, int nthreads) {
  ORACLE_SETUP(0);
  ORACLE_BODY(float, expf, logf)
}

/* The same rows, with q, o and lse holding only tokens [t_begin, t_end) of every (b, head):
   q [B, Hq, t_end - t_begin, dqk], o [B, Hq, t_end - t_begin, dv], lse [B, Hq, t_end - t_begin]
   (k, v and sel stay whole: the gather reaches any earlier key).  For parity checks of long
   sequences without a host copy of the whole Q and O. */
int nsa_oracle_forward_window(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* sel,
                              const int32_t* cu_seqlens, int n_seqs, int B, int Hq, int Hkv, int T, int dqk, int dv,
                              int NQB, int KSEL, int LP, int BQ, double scale, int bkv_begin, int bkv_end,
                              int t_begin, int t_end, int strict, double* o, double* lse, int nthreads) {
  ORACLE_SETUP(1);
  ORACLE_BODY(double, exp, log)
}

int nsa_oracle_forward_window_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int32_t* sel,
                                  const int32_t* cu_seqlens, int n_seqs, int B, int Hq, int Hkv, int T, int dqk,
                                  int dv, int NQB, int KSEL, int LP, int BQ, double scale, int bkv_begin, int bkv_end,
                                  int t_begin, int t_end, int strict, float* o, float* lse, int nthreads) {
  ORACLE_SETUP(1);
  ORACLE_BODY(float, expf, logf)
}

/* Number of visible keys per (b*Hkv+kvh, t) row -- the mask alone, for bit-exact mask checks
   and for the FLOP count of the roofline. */
int nsa_oracle_count_keys(const int32_t* sel, const int32_t* cu_seqlens, int n_seqs, int B, int Hkv, int T,
                          int NQB, int KSEL, int LP, int BQ, int32_t* counts, int nthreads) {
  if (!sel || !counts || B <= 0 || Hkv <= 0 || T <= 0 || KSEL <= 0 || LP <= 0 || BQ <= 0) return NSA_ORACLE_ERR_ARG;
  if (NQB != (T + BQ - 1) / BQ) return NSA_ORACLE_ERR_ARG;
  oracle_args A;
  memset(&A, 0, sizeof(A));
  A.sel = sel;
  A.cu = cu_seqlens;
  A.n_seqs = n_seqs;
  A.B = B;
  A.Hkv = Hkv;
  A.T = T;
  A.NQB = NQB;
  A.KSEL = KSEL;
  A.LP = LP;
  A.BQ = BQ;
  const oracle_args* a = &A;
  if (nthreads <= 0) nthreads = 1;
  const long long rows = (long long)B * Hkv * T;
  int status = NSA_ORACLE_OK;
#pragma omp parallel num_threads(nthreads)
  {
    unsigned char* keep = (unsigned char*)malloc((size_t)T + 2);
    int* keys = (int*)malloc(sizeof(int) * ((size_t)KSEL * LP + 1));
    if (!keep || !keys) {
#pragma omp atomic write
      status = NSA_ORACLE_ERR_NOMEM;
    } else {
#pragma omp for schedule(static)
      for (long long rr = 0; rr < rows; ++rr) {
        const int bkv = (int)(rr / T), t = (int)(rr % T);
        counts[rr] = visible_keys(a, bkv / Hkv, bkv % Hkv, t, keep, keys);
      }
    }
    free(keep);
    free(keys);
  }
  return status;
}
