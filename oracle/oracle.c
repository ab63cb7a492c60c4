/*
 * oracle.c — CPU restatement of gollama's training hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker for libgollama_cuda; never part of the
 * product path).  Parity status: UNPINNED — the reference has no tests or
 * golden vectors and cannot be run here (no Go toolchain); see oracle.h.
 *
 * Compiled twice: with real = float and prefix orc_ (the Go float32
 * semantics), and with -DORC_DOUBLE (real = double, prefix orcd_).  Build with
 * -ffp-contract=off: Go on amd64 does not fuse multiply-add.
 *
 * Threading.  set_threads(n, literal):
 *   literal = 1 follows the reference's loop nests and threading exactly
 *     (row-parallel MatMulTransposeB, single-threaded dA loop, N-parallel dB
 *     loop, everything else on one thread) — this is the timed CPU baseline;
 *   literal = 0 runs the same per-element arithmetic in the same order but
 *     with cache-friendly loop nests and every loop parallel over its outer
 *     index — used by the tests.  Both produce bit-identical results.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

#ifdef ORC_DOUBLE
typedef double real;
#define FN(n) orcd_##n
#else
typedef float real;
#define FN(n) orc_##n
#endif

#define NOVEC __attribute__((optimize("no-tree-vectorize")))

static int g_threads = 1;
static int g_literal = 0;

void FN(set_threads)(int nthreads, int literal) {
  g_threads = nthreads < 1 ? 1 : (nthreads > 256 ? 256 : nthreads);
  g_literal = literal;
}

/* ------------------------------------------------------------------ threads */
typedef void (*range_fn)(void* arg, int start, int end);
typedef struct {
  range_fn fn;
  void* arg;
  int start, end;
} job_t;

static void* job_main(void* p) {
  job_t* j = (job_t*)p;
  j->fn(j->arg, j->start, j->end);
  return NULL;
}

/* Splits [0,n) into nthreads contiguous chunks of ceil(n/nthreads), the way the
 * reference splits rows over GOMAXPROCS workers (pkg/tensor/matmul.go:198-221). */
static void parallel_for(int n, int nthreads, range_fn fn, void* arg) {
  if (nthreads <= 1 || n < 2) {
    fn(arg, 0, n);
    return;
  }
  if (nthreads > n) nthreads = n;
  int per = (n + nthreads - 1) / nthreads;
  pthread_t th[256];
  job_t jobs[256];
  int used = 0;
  for (int w = 0; w < nthreads; ++w) {
    int s = w * per, e = s + per;
    if (e > n) e = n;
    if (s >= e) break;
    jobs[used].fn = fn;
    jobs[used].arg = arg;
    jobs[used].start = s;
    jobs[used].end = e;
    if (pthread_create(&th[used], NULL, job_main, &jobs[used]) != 0) {
      fn(arg, s, e);
      continue;
    }
    ++used;
  }
  for (int i = 0; i < used; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------ param layout
 * Params() order (pkg/train/trainer.go:217,242-247,253):
 *   reference: TokenEmbed[V,d], PosEmbed[maxSeq,d],
 *              per layer AttnNorm[d], WQ[d,d], WK[d,d], WV[d,d], WO[d,d],
 *                        FFNNorm[d], WGate[F,d], WUp[F,d], WDown[d,F],
 *              OutputNorm[d]
 *   llama:     no PosEmbed; WK and WV are [Hkv*hd, d].                       */
enum { P_ATTN_NORM = 0, P_WQ, P_WK, P_WV, P_WO, P_FFN_NORM, P_WGATE, P_WUP, P_WDOWN, P_PER_LAYER };

static int head_dim(const orc_config* c) { return c->hidden / c->heads; }
static int kvh(const orc_config* c) { return c->mode == ORC_MODE_LLAMA ? c->kv_heads : c->heads; }
static int n_global_front(const orc_config* c) { return c->mode == ORC_MODE_LLAMA ? 1 : 2; }

int FN(num_params)(const orc_config* c) { return n_global_front(c) + c->layers * P_PER_LAYER + 1; }

static void shape_of(const orc_config* c, int idx, int64_t* rows, int64_t* cols) {
  const int64_t d = c->hidden, F = c->inter, kvd = (int64_t)kvh(c) * head_dim(c);
  int nf = n_global_front(c);
  if (idx == 0) { *rows = c->vocab; *cols = d; return; }
  if (nf == 2 && idx == 1) { *rows = c->max_seq; *cols = d; return; }
  int li = idx - nf;
  if (li >= c->layers * P_PER_LAYER) { *rows = 1; *cols = d; return; } /* OutputNorm */
  switch (li % P_PER_LAYER) {
    case P_ATTN_NORM: case P_FFN_NORM: *rows = 1; *cols = d; return;
    case P_WQ: case P_WO: *rows = d; *cols = d; return;
    case P_WK: case P_WV: *rows = kvd; *cols = d; return;
    case P_WGATE: case P_WUP: *rows = F; *cols = d; return;
    default: *rows = d; *cols = F; return; /* WDown */
  }
}

void FN(param_info)(const orc_config* c, int idx, int64_t* offset, int64_t* rows, int64_t* cols) {
  int64_t off = 0, r, cc;
  for (int i = 0; i < idx; ++i) {
    shape_of(c, i, &r, &cc);
    off += r * cc;
  }
  shape_of(c, idx, rows, cols);
  *offset = off;
}

int64_t FN(param_total)(const orc_config* c) {
  int64_t off, r, cc;
  int n = FN(num_params)(c);
  FN(param_info)(c, n - 1, &off, &r, &cc);
  return off + r * cc;
}

static int layer_param(const orc_config* c, int layer, int which) {
  return n_global_front(c) + layer * P_PER_LAYER + which;
}
static int out_norm_param(const orc_config* c) { return FN(num_params)(c) - 1; }

/* ------------------------------------------------------------------ MatMulTransposeB
 * pkg/tensor/matmul.go:145-234 with dotProduct :237-259 (8 partial sums). */
static inline real dot8(const real* a, const real* b, int K) {
  real s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
  int k = 0;
  for (; k <= K - 8; k += 8) {
    s0 += a[k] * b[k];
    s1 += a[k + 1] * b[k + 1];
    s2 += a[k + 2] * b[k + 2];
    s3 += a[k + 3] * b[k + 3];
    s4 += a[k + 4] * b[k + 4];
    s5 += a[k + 5] * b[k + 5];
    s6 += a[k + 6] * b[k + 6];
    s7 += a[k + 7] * b[k + 7];
  }
  real sum = s0 + s1 + s2 + s3 + s4 + s5 + s6 + s7;
  for (; k < K; ++k) sum += a[k] * b[k];
  return sum;
}

typedef struct {
  const real *a, *b;
  real* out;
  int M, K, N;
} mm_args;

static void mtb_rows(void* p, int s, int e) {
  mm_args* g = (mm_args*)p;
  for (int i = s; i < e; ++i)
    for (int j = 0; j < g->N; ++j) g->out[(int64_t)i * g->N + j] = dot8(g->a + (int64_t)i * g->K, g->b + (int64_t)j * g->K, g->K);
}
static void mtb_cols_m1(void* p, int s, int e) {
  mm_args* g = (mm_args*)p;
  for (int j = s; j < e; ++j) g->out[j] = dot8(g->a, g->b + (int64_t)j * g->K, g->K);
}

void FN(matmul_transpose_b)(const real* a, const real* b, real* out, int M, int K, int N) {
  mm_args g = {a, b, out, M, K, N};
  if (M == 1 && N >= g_threads) { /* matmul.go:172-195 */
    parallel_for(N, g_threads, mtb_cols_m1, &g);
    return;
  }
  if (g_literal && !(M > 1 && (int64_t)M * N * K > 50000)) { /* matmul.go:225-233 */
    mtb_rows(&g, 0, M);
    return;
  }
  parallel_for(M, g_threads, mtb_rows, &g); /* matmul.go:198-223 */
}

/* ------------------------------------------------------------------ MatMulGrad dA
 * pkg/tensor/grad.go:106-115: dA[m,k] += sum_n dC[m,n]*B[n,k], n ascending. */
NOVEC static void da_literal(const real* dc, const real* b, real* da, int M, int K, int N) {
  for (int m = 0; m < M; ++m)
    for (int k = 0; k < K; ++k) {
      real sum = 0;
      for (int n = 0; n < N; ++n) sum += dc[(int64_t)m * N + n] * b[(int64_t)n * K + k];
      da[(int64_t)m * K + k] += sum;
    }
}

static void da_rows(void* p, int s, int e) {
  mm_args* g = (mm_args*)p; /* a = dC, b = B, out = dA */
  const int K = g->K, N = g->N;
  for (int m = s; m < e; ++m) {
    const real* dcr = g->a + (int64_t)m * N;
    int k0 = 0;
    for (; k0 + 8 <= K; k0 += 8) {
      real acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int n = 0; n < N; ++n) {
        const real c = dcr[n];
        const real* br = g->b + (int64_t)n * K + k0;
        for (int j = 0; j < 8; ++j) acc[j] += c * br[j];
      }
      for (int j = 0; j < 8; ++j) g->out[(int64_t)m * K + k0 + j] += acc[j];
    }
    for (int k = k0; k < K; ++k) {
      real sum = 0;
      for (int n = 0; n < N; ++n) sum += dcr[n] * g->b[(int64_t)n * K + k];
      g->out[(int64_t)m * K + k] += sum;
    }
  }
}

void FN(matmul_grad_da)(const real* dc, const real* b, real* da, int M, int K, int N) {
  if (g_literal) {
    da_literal(dc, b, da, M, K, N); /* single-threaded in the reference */
    return;
  }
  mm_args g = {dc, b, da, M, K, N};
  parallel_for(M, g_threads, da_rows, &g);
}

/* ------------------------------------------------------------------ MatMulGrad dB
 * pkg/tensor/grad.go:124-151: dB[n,k] += sum_m dC[m,n]*A[m,k], m ascending,
 * rows of N split over GOMAXPROCS workers. */
NOVEC static void db_literal_rows(void* p, int s, int e) {
  mm_args* g = (mm_args*)p; /* a = dC, b = A, out = dB */
  const int M = g->M, K = g->K, N = g->N;
  for (int n = s; n < e; ++n)
    for (int k = 0; k < K; ++k) {
      real sum = 0;
      for (int m = 0; m < M; ++m) sum += g->a[(int64_t)m * N + n] * g->b[(int64_t)m * K + k];
      g->out[(int64_t)n * K + k] += sum;
    }
}

static void db_rows(void* p, int s, int e) {
  mm_args* g = (mm_args*)p;
  const int M = g->M, K = g->K, N = g->N;
  for (int n = s; n < e; ++n) {
    int k0 = 0;
    for (; k0 + 8 <= K; k0 += 8) {
      real acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int m = 0; m < M; ++m) {
        const real c = g->a[(int64_t)m * N + n];
        const real* ar = g->b + (int64_t)m * K + k0;
        for (int j = 0; j < 8; ++j) acc[j] += c * ar[j];
      }
      for (int j = 0; j < 8; ++j) g->out[(int64_t)n * K + k0 + j] += acc[j];
    }
    for (int k = k0; k < K; ++k) {
      real sum = 0;
      for (int m = 0; m < M; ++m) sum += g->a[(int64_t)m * N + n] * g->b[(int64_t)m * K + k];
      g->out[(int64_t)n * K + k] += sum;
    }
  }
}

void FN(matmul_grad_db)(const real* dc, const real* a, real* db, int M, int K, int N) {
  mm_args g = {dc, a, db, M, K, N};
  parallel_for(N, g_threads, g_literal ? db_literal_rows : db_rows, &g);
}

/* ------------------------------------------------------------------ elementwise */
static void add_into(real* dst, const real* src, int64_t n) { /* addInplace, grad.go:200-204 */
  for (int64_t i = 0; i < n; ++i) dst[i] += src[i];
}

/* ------------------------------------------------------------------ RMSNorm
 * Forward: pkg/train/trainer.go:157-168.  rms = float32(sqrt(float64(ss)/cols
 * + float64(eps))) with ss a float32 running sum; out = (x/rms)*w. */
void FN(rmsnorm_fwd)(const real* x, const real* w, real* out, real* rms, int rows, int cols, float eps) {
  for (int i = 0; i < rows; ++i) {
    const real* xr = x + (int64_t)i * cols;
    real ss = 0;
    for (int j = 0; j < cols; ++j) ss += xr[j] * xr[j];
    const real r = (real)sqrt((double)ss / (double)cols + (double)eps);
    rms[i] = r;
    for (int j = 0; j < cols; ++j) out[(int64_t)i * cols + j] = (xr[j] / r) * w[j];
  }
}

/* Backward.  full = 0: the reference's simplified form (trainer.go:182-199):
 *   dw[j] += dout*x/rms, dx += dout*w/rms.
 * full = 1 (Llama mode): the true gradient
 *   dx_k += dout_k*w_k/rms - x_k * (sum_j dout_j*w_j*x_j) / (cols*rms^3).
 * dx or dw may be NULL when that gradient is not required. */
void FN(rmsnorm_bwd)(const real* x, const real* w, const real* rms, const real* dout, real* dx, real* dw,
                     int rows, int cols, int full) {
  for (int i = 0; i < rows; ++i) {
    const int64_t off = (int64_t)i * cols;
    const real r = rms[i];
    real c = 0;
    if (full && dx) {
      real s = 0;
      for (int j = 0; j < cols; ++j) s += dout[off + j] * w[j] * x[off + j];
      c = s / ((real)cols * r * r * r);
    }
    for (int j = 0; j < cols; ++j) {
      const real d = dout[off + j];
      if (dw) dw[j] += d * x[off + j] / r;
      if (dx) {
        if (full)
          dx[off + j] += d * w[j] / r - x[off + j] * c;
        else
          dx[off + j] += d * w[j] / r;
      }
    }
  }
}

/* ------------------------------------------------------------------ exp/log
 * The reference's own approximations, pkg/tensor/grad.go:283-381. */
double FN(go_exp)(double x) { /* _exp, grad.go:310-352 */
  const double Ln2Hi = 6.93147180369123816490e-01, Ln2Lo = 1.90821492927058770002e-10,
               Log2e = 1.44269504088896338700e+00, Overflow = 7.09782712893383973096e+02,
               Underflow = -7.45133219101941108420e+02;
  if (x > Overflow) return 1.7976931348623157e+308;
  if (x < Underflow) return 0;
  int k = (int)(x * Log2e + 0.5);
  if (x < 0) k = (int)(x * Log2e - 0.5);
  double r = x - (double)k * Ln2Hi - (double)k * Ln2Lo;
  double r2 = r * r;
  double p = r - r2 * (0.16666666666666602 + r2 * (0.0027777777777015593 + r2 * 6.613756321437934e-05));
  double result = 1 - (r * p / (p - 2) - r);
  if (k > 0) {
    for (int i = 0; i < k; ++i) result *= 2;
  } else {
    for (int i = 0; i < -k; ++i) result /= 2;
  }
  return result;
}

double FN(go_log)(double x) { /* _log, grad.go:354-381 */
  if (x <= 0) return -1e100;
  int k = 0;
  while (x >= 2) { x /= 2; k++; }
  while (x < 1) { x *= 2; k--; }
  double f = x - 1;
  double s = f / (2 + f);
  double s2 = s * s;
  double s4 = s2 * s2;
  double t1 = s2 * (0.6666666666666735 + s4 * (0.2857142874366239 + s4 * 0.1818357216161805));
  double t2 = s4 * (0.3999999999940942 + s4 * 0.22222198432149784);
  double R = t1 + t2;
  return (double)k * 0.6931471805599453 + f - s * (f - R);
}

float FN(exp32)(float x) { /* grad.go:283-293 */
  if (x < -88) return 0;
  if (x > 88) return 3.4e38f;
  return (float)FN(go_exp)((double)x);
}

void FN(exp32_array)(const float* x, float* y, int64_t n) { /* exp32 over an array (test vectors) */
  for (int64_t i = 0; i < n; ++i) y[i] = FN(exp32)(x[i]);
}

float FN(log32)(float x) { return (float)FN(go_log)((double)x); } /* grad.go:296-298 */

/* ------------------------------------------------------------------ frozen quantized weights
 * pkg/quant/dequant.go.  Type codes are GGUF's (pkg/gguf/format.go:40-58):
 * 0 F32, 1 F16, 2 Q4_0, 3 Q4_1, 6 Q5_0, 7 Q5_1, 8 Q8_0, 12 Q4_K, 14 Q6_K. */
#ifndef ORC_QTYPES
#define ORC_QTYPES
enum {
  ORC_Q_F32 = 0, ORC_Q_F16 = 1, ORC_Q_Q4_0 = 2, ORC_Q_Q4_1 = 3, ORC_Q_Q5_0 = 6, ORC_Q_Q5_1 = 7, ORC_Q_Q8_0 = 8,
  ORC_Q_Q4_K = 12, ORC_Q_Q6_K = 14
};
#endif

/* fp16ToFp32 (dequant.go:9-41): exact widening; a subnormal half is
 * normalised by shifting its mantissa up until the implicit bit appears. */
float FN(fp16_to_fp32)(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) & 1u, e = (uint32_t)(h >> 10) & 0x1fu, m = (uint32_t)h & 0x3ffu, bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign << 31;
    } else {
      int32_t ex = 1;
      while (!(m & 0x400u)) {
        m <<= 1;
        --ex;
      }
      m &= 0x3ffu;
      bits = (sign << 31) | ((uint32_t)(ex + 127 - 15) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = (sign << 31) | 0x7f800000u | (m << 13);
  } else {
    bits = (sign << 31) | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); } /* little endian */

static uint32_t rd_u32(const uint8_t* p) { return (uint32_t)rd_u16(p) | ((uint32_t)rd_u16(p + 2) << 16); }

/* The K-quant and 5-bit formats (dequant.go:141-344), each in the
 * reference's loop order: per block the half scales, then per byte (or per
 * element) the codes; every product and sum is one float32 operation. */
static int dequant_more(const uint8_t* data, real* out, int64_t n, int type) {
  if (type == ORC_Q_Q4_1 || type == ORC_Q_Q5_0 || type == ORC_Q_Q5_1) {
    if (n % 32) return -1;
    const int bpb = type == ORC_Q_Q4_1 ? 20 : type == ORC_Q_Q5_0 ? 22 : 24;
    for (int64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = data + (int64_t)bpb * b;
      const float scale = FN(fp16_to_fp32)(rd_u16(blk));
      if (type == ORC_Q_Q4_1) { /* :141-163: scale*q + min */
        const float mn = FN(fp16_to_fp32)(rd_u16(blk + 2));
        for (int i = 0; i < 16; ++i) {
          const uint8_t q = blk[4 + i];
          const float q0 = (float)(q & 0x0f), q1 = (float)(q >> 4);
          const float p0 = scale * q0, p1 = scale * q1;
          out[32 * b + 2 * i] = p0 + mn;
          out[32 * b + 2 * i + 1] = p1 + mn;
        }
      } else if (type == ORC_Q_Q5_0) { /* :167-199: high bit k of qh for element k, then - 16 */
        const uint32_t qh = rd_u32(blk + 2);
        for (int i = 0; i < 16; ++i) {
          const uint8_t q = blk[6 + i];
          int8_t q0 = (int8_t)(q & 0x0f), q1 = (int8_t)(q >> 4);
          if ((qh >> (i * 2)) & 1u) q0 |= 0x10;
          if ((qh >> (i * 2 + 1)) & 1u) q1 |= 0x10;
          out[32 * b + 2 * i] = scale * (float)(int8_t)(q0 - 16);
          out[32 * b + 2 * i + 1] = scale * (float)(int8_t)(q1 - 16);
        }
      } else { /* Q5_1, :203-233: scale*q + min */
        const float mn = FN(fp16_to_fp32)(rd_u16(blk + 2));
        const uint32_t qh = rd_u32(blk + 4);
        for (int i = 0; i < 16; ++i) {
          const uint8_t q = blk[8 + i];
          uint8_t q0 = (uint8_t)(q & 0x0f), q1 = (uint8_t)(q >> 4);
          if ((qh >> (i * 2)) & 1u) q0 |= 0x10;
          if ((qh >> (i * 2 + 1)) & 1u) q1 |= 0x10;
          const float p0 = scale * (float)q0, p1 = scale * (float)q1;
          out[32 * b + 2 * i] = p0 + mn;
          out[32 * b + 2 * i + 1] = p1 + mn;
        }
      }
    }
    return 0;
  }
  if (type == ORC_Q_Q4_K) { /* :237-300 */
    if (n % 256) return -1;
    for (int64_t b = 0; b < n / 256; ++b) {
      const uint8_t* blk = data + 144 * b;
      const float d = FN(fp16_to_fp32)(rd_u16(blk)), dmin = FN(fp16_to_fp32)(rd_u16(blk + 2));
      const uint8_t* sc6 = blk + 4;
      const uint8_t* qs = blk + 16;
      uint8_t sc[8], m[8];
      for (int j = 0; j < 4; ++j) {
        sc[j] = sc6[j] & 63;
        m[j] = sc6[j + 4] & 63;
      }
      sc[4] = (uint8_t)((sc6[8] & 0xF) | ((sc6[0] >> 6) << 4));
      sc[5] = (uint8_t)((sc6[8] >> 4) | ((sc6[1] >> 6) << 4));
      sc[6] = (uint8_t)((sc6[9] & 0xF) | ((sc6[2] >> 6) << 4));
      sc[7] = (uint8_t)((sc6[9] >> 4) | ((sc6[3] >> 6) << 4));
      m[4] = (uint8_t)((sc6[10] & 0xF) | ((sc6[4] >> 6) << 4));
      m[5] = (uint8_t)((sc6[10] >> 4) | ((sc6[5] >> 6) << 4));
      m[6] = (uint8_t)((sc6[11] & 0xF) | ((sc6[6] >> 6) << 4));
      m[7] = (uint8_t)((sc6[11] >> 4) | ((sc6[7] >> 6) << 4));
      for (int j = 0; j < 8; ++j) {
        const float scale_val = d * (float)sc[j];
        const float min_val = dmin * (float)m[j];
        for (int i = 0; i < 16; ++i) {
          const uint8_t q = qs[j * 16 + i];
          const float p0 = scale_val * (float)(q & 0x0F), p1 = scale_val * (float)(q >> 4);
          out[256 * b + j * 32 + i * 2] = p0 - min_val;
          out[256 * b + j * 32 + i * 2 + 1] = p1 - min_val;
        }
      }
    }
    return 0;
  }
  if (type == ORC_Q_Q6_K) { /* :304-344 */
    if (n % 256) return -1;
    for (int64_t b = 0; b < n / 256; ++b) {
      const uint8_t* blk = data + 210 * b;
      const uint8_t* ql = blk;
      const uint8_t* qh = blk + 128;
      const uint8_t* scales = blk + 192;
      const float d = FN(fp16_to_fp32)(rd_u16(blk + 208));
      for (int j = 0; j < 16; ++j) {
        const float scale_val = d * (float)(int8_t)scales[j];
        for (int i = 0; i < 16; ++i) {
          const int idx = j * 16 + i;
          const uint8_t q = (idx % 2 == 0) ? (uint8_t)(ql[idx / 2] & 0x0F) : (uint8_t)(ql[idx / 2] >> 4);
          const uint8_t q_high = (uint8_t)((qh[idx / 4] >> ((idx % 4) * 2)) & 0x03);
          const int8_t q6 = (int8_t)((int8_t)(q | (q_high << 4)) - 32);
          out[256 * b + idx] = scale_val * (float)q6;
        }
      }
    }
    return 0;
  }
  return -1;
}

/* Dequantize (dequant.go:367-393) for F32, F16 (:50-56), Q8_0 (:68-85: per
 * 32-element block a half scale then 32 int8 codes, w = scale * q), Q4_0
 * (:99-119: a half scale then 16 bytes; element 2i is the low nibble - 8,
 * element 2i+1 the high nibble - 8) and, through dequant_more, Q4_1, Q5_0,
 * Q5_1, Q4_K and Q6_K.  n counts output elements; block types need a whole
 * number of blocks.  Products are float32 like the reference's. */
int FN(dequantize)(const uint8_t* data, real* out, int64_t n, int type) {
  if (type == ORC_Q_F32) {
    for (int64_t i = 0; i < n; ++i) {
      float f;
      memcpy(&f, data + 4 * i, 4);
      out[i] = f;
    }
    return 0;
  }
  if (type == ORC_Q_F16) {
    for (int64_t i = 0; i < n; ++i) out[i] = FN(fp16_to_fp32)(rd_u16(data + 2 * i));
    return 0;
  }
  if (n % 32) return -1;
  if (type == ORC_Q_Q8_0) {
    for (int64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = data + 34 * b;
      const float scale = FN(fp16_to_fp32)(rd_u16(blk));
      for (int i = 0; i < 32; ++i) out[32 * b + i] = scale * (float)(int8_t)blk[2 + i];
    }
    return 0;
  }
  if (type == ORC_Q_Q4_0) {
    for (int64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = data + 18 * b;
      const float scale = FN(fp16_to_fp32)(rd_u16(blk));
      for (int i = 0; i < 16; ++i) {
        const uint8_t q = blk[2 + i];
        out[32 * b + 2 * i] = scale * (float)((int)(q & 0x0f) - 8);
        out[32 * b + 2 * i + 1] = scale * (float)((int)(q >> 4) - 8);
      }
    }
    return 0;
  }
  return dequant_more(data, out, n, type);
}

/* dX[M,K] += dY[M,N] . deq(W)[N,K] with W's rows (out features) stored as
 * quantized rows of K (in features): the reference dequantizes the weight
 * (dequant.go) and runs MatMulGrad's dA loop (grad.go:102-116). */
int FN(linear_bwd_dx_q)(const real* dy, const uint8_t* wq, int type, real* dx, int M, int K, int N) {
  real* w = (real*)malloc(sizeof(real) * (size_t)N * (size_t)K);
  if (!w) return -1;
  int rc = FN(dequantize)(wq, w, (int64_t)N * K, type);
  if (rc == 0) FN(matmul_grad_da)(dy, w, dx, M, K, N);
  free(w);
  return rc;
}

/* ------------------------------------------------------------------ exponential of the current semantics
 * Reference semantics use the reference's exp32/log32 (grad.go:283-298).
 * Llama semantics use the C library's expf/logf: the benchmark's decoder is
 * not the reference trainer's model, and its tolerance (loss 1e-4, gradients
 * 2e-3) is far above the 1.4e-5 by which exp32 differs from e^x.  The flag is
 * set only for the duration of a whole-model forward/backward in llama mode;
 * the single-op entry points always use exp32/log32. */
static int g_libm_exp = 0;
static float mode_exp32(float x) { return g_libm_exp ? expf(x) : FN(exp32)(x); }
static float mode_log32(float x) { return g_libm_exp ? logf(x) : FN(log32)(x); }

/* ------------------------------------------------------------------ SiLU (SiLUGrad, grad.go:417-449) */
void FN(silu_fwd)(const real* x, real* out, real* sig, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const real v = x[i];
#ifdef ORC_DOUBLE
    sig[i] = 1.0 / (1.0 + exp(-v));
#else
    sig[i] = 1.0f / (1.0f + mode_exp32(-v));
#endif
    out[i] = v * sig[i];
  }
}

void FN(silu_bwd)(const real* x, const real* sig, const real* dout, real* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const real s = sig[i];
    const real g = s * (1 + x[i] * (1 - s));
    dx[i] += dout[i] * g;
  }
}

/* ------------------------------------------------------------------ softmax cross-entropy
 * SoftmaxCrossEntropyGrad forward, grad.go:210-246.  probs may be NULL.  Rows
 * whose target is outside [0,V) add no loss but count in the mean. */
typedef struct {
  const real* logits;
  const int64_t* targets;
  int V;
  real* probs;
  real* row_loss;
} ce_args;

static void ce_rows(void* p, int s, int e) {
  ce_args* g = (ce_args*)p;
  const int V = g->V;
  real* tmp = g->probs ? NULL : (real*)malloc(sizeof(real) * (size_t)V);
  for (int b = s; b < e; ++b) {
    const real* l = g->logits + (int64_t)b * V;
    real* pr = g->probs ? g->probs + (int64_t)b * V : tmp;
    real maxv = l[0];
    for (int v = 1; v < V; ++v)
      if (l[v] > maxv) maxv = l[v];
    real sum = 0;
    for (int v = 0; v < V; ++v) {
#ifdef ORC_DOUBLE
      pr[v] = exp(l[v] - maxv);
#else
      pr[v] = mode_exp32(l[v] - maxv);
#endif
      sum += pr[v];
    }
    for (int v = 0; v < V; ++v) pr[v] /= sum;
    const int64_t t = g->targets[b];
    real loss = 0;
    if (t >= 0 && t < V) {
#ifdef ORC_DOUBLE
      loss = -log(pr[t] + 1e-10);
#else
      loss = -mode_log32(pr[t] + 1e-10f);
#endif
    }
    g->row_loss[b] = loss;
  }
  free(tmp);
}

real FN(softmax_ce)(const real* logits, const int64_t* targets, int rows, int V, real* probs) {
  real* row_loss = (real*)malloc(sizeof(real) * (size_t)(rows > 0 ? rows : 1));
  ce_args g = {logits, targets, V, probs, row_loss};
  parallel_for(rows, g_literal ? 1 : g_threads, ce_rows, &g);
  /* totalLoss -= log32(...) accumulated row by row in order (grad.go:239-243) */
  real total = 0;
  for (int b = 0; b < rows; ++b) {
    const int64_t t = targets[b];
    if (t >= 0 && t < V) total -= -row_loss[b];
  }
  free(row_loss);
  return total / (real)rows;
}

/* GradFn of the loss node, grad.go:266-276: dlogits += (probs - onehot)/rows. */
void FN(softmax_ce_grad)(const real* probs, const int64_t* targets, int rows, int V, real* dlogits) {
  const real scale = (real)1.0 / (real)rows;
  for (int b = 0; b < rows; ++b) {
    const int64_t t = targets[b];
    for (int v = 0; v < V; ++v) {
      real g = probs[(int64_t)b * V + v] * scale;
      if (v == t) g -= scale;
      dlogits[(int64_t)b * V + v] += g;
    }
  }
}

/* ------------------------------------------------------------------ RoPE
 * precomputeFreqs (pkg/model/rope.go:33-48): freq = 1/theta^(2i/dim) in
 * float64, cos/sin rounded to float32.  apply3D (:96-126): consecutive pairs
 * (2i, 2i+1); the training position of token t is t % S.  inverse = 1 rotates
 * by -angle (the backward of the rotation). */
void FN(rope_table)(int dim, int max_seq, float theta, real* cos_t, real* sin_t) {
  const int half = dim / 2;
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const double freq = 1.0 / pow((double)theta, (double)(2 * i) / (double)dim);
      const double angle = (double)pos * freq;
      cos_t[pos * half + i] = (real)cos(angle);
      sin_t[pos * half + i] = (real)sin(angle);
    }
}

void FN(rope_apply)(real* x, int T, int S, int nh, int hd, const real* cos_t, const real* sin_t, int inverse) {
  const int half = hd / 2;
  for (int t = 0; t < T; ++t) {
    const int pos = t % S;
    for (int h = 0; h < nh; ++h) {
      real* base = x + ((int64_t)t * nh + h) * hd;
      for (int i = 0; i < half; ++i) {
        const real c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const real x0 = base[2 * i], x1 = base[2 * i + 1];
        if (!inverse) {
          base[2 * i] = x0 * c - x1 * s;
          base[2 * i + 1] = x0 * s + x1 * c;
        } else {
          base[2 * i] = x0 * c + x1 * s;
          base[2 * i + 1] = -x0 * s + x1 * c;
        }
      }
    }
  }
}

/* ------------------------------------------------------------------ attention
 * forwardAttention (pkg/train/trainer.go:331-386): per token i and head h,
 * causal over j <= i within its sequence, scale float32(1/sqrt(hd)), softmax
 * with float32(math.Exp(float64(s - max))), float32 sums.  Heads sharing a KV
 * head follow pkg/model/attention.go:118,149 (kvHead = h / (H/Hkv)); q rows
 * have stride H*hd, k/v rows Hkv*hd. */
typedef struct {
  const real *q, *k, *v, *dout;
  real *out, *dq, *dk, *dv;
  int T, S, H, Hkv, hd;
} att_args;

static void att_fwd_rows(void* p, int s, int e) {
  att_args* g = (att_args*)p;
  const int S = g->S, H = g->H, Hkv = g->Hkv, hd = g->hd, group = H / Hkv;
  const int qs = H * hd, ks = Hkv * hd;
  const real scale = (real)(1.0 / sqrt((double)hd));
  real* scores = (real*)malloc(sizeof(real) * (size_t)S);
  for (int i = s; i < e; ++i) {
    const int pos = i % S, b = i / S;
    for (int h = 0; h < H; ++h) {
      const int kh = h / group;
      const real* qi = g->q + (int64_t)i * qs + h * hd;
      real maxs = (real)-1e10;
      for (int j = 0; j <= pos; ++j) {
        const real* kj = g->k + (int64_t)(b * S + j) * ks + kh * hd;
        real dot = 0;
        for (int d = 0; d < hd; ++d) dot += qi[d] * kj[d];
        scores[j] = dot * scale;
        if (scores[j] > maxs) maxs = scores[j];
      }
      real sum = 0;
      for (int j = 0; j <= pos; ++j) {
        scores[j] = (real)exp((double)(scores[j] - maxs));
        sum += scores[j];
      }
      for (int j = 0; j <= pos; ++j) scores[j] /= sum;
      for (int d = 0; d < hd; ++d) {
        real acc = 0;
        for (int j = 0; j <= pos; ++j) acc += scores[j] * g->v[(int64_t)(b * S + j) * ks + kh * hd + d];
        g->out[(int64_t)i * qs + h * hd + d] = acc;
      }
    }
  }
  free(scores);
}

void FN(attention_fwd)(const real* q, const real* k, const real* v, real* out, int T, int S, int H, int Hkv,
                       int hd) {
  att_args g = {q, k, v, NULL, out, NULL, NULL, NULL, T, S, H, Hkv, hd};
  parallel_for(T, g_literal ? 1 : g_threads, att_fwd_rows, &g);
}

/* Backward of the attention above (Llama mode only; the reference attaches no
 * GradFn, trainer.go:335-337).  With P the softmax probabilities:
 *   dV_j += P_ij dO_i;  dP_ij = dO_i.V_j;  dS_ij = P_ij (dP_ij - sum_l P_il dP_il)
 *   dQ_i += scale sum_j dS_ij K_j;  dK_j += scale sum_i dS_ij Q_i.
 * Parallel over (sequence, kv head): each task owns its dk/dv rows. */
static void att_bwd_tasks(void* p, int s, int e) {
  att_args* g = (att_args*)p;
  const int S = g->S, H = g->H, Hkv = g->Hkv, hd = g->hd, group = H / Hkv;
  const int qs = H * hd, ks = Hkv * hd;
  const real scale = (real)(1.0 / sqrt((double)hd));
  real* P = (real*)malloc(sizeof(real) * (size_t)S);
  real* dP = (real*)malloc(sizeof(real) * (size_t)S);
  for (int task = s; task < e; ++task) {
    const int b = task / Hkv, kh = task % Hkv;
    for (int h = kh * group; h < (kh + 1) * group; ++h) {
      for (int pos = 0; pos < S; ++pos) {
        const int i = b * S + pos;
        const real* qi = g->q + (int64_t)i * qs + h * hd;
        const real* doi = g->dout + (int64_t)i * qs + h * hd;
        real maxs = (real)-1e10;
        for (int j = 0; j <= pos; ++j) {
          const real* kj = g->k + (int64_t)(b * S + j) * ks + kh * hd;
          real dot = 0;
          for (int d = 0; d < hd; ++d) dot += qi[d] * kj[d];
          P[j] = dot * scale;
          if (P[j] > maxs) maxs = P[j];
        }
        real sum = 0;
        for (int j = 0; j <= pos; ++j) {
          P[j] = (real)exp((double)(P[j] - maxs));
          sum += P[j];
        }
        for (int j = 0; j <= pos; ++j) P[j] /= sum;
        real Di = 0;
        for (int j = 0; j <= pos; ++j) {
          const real* vj = g->v + (int64_t)(b * S + j) * ks + kh * hd;
          real dot = 0;
          for (int d = 0; d < hd; ++d) dot += doi[d] * vj[d];
          dP[j] = dot;
          Di += P[j] * dot;
        }
        real* dqi = g->dq + (int64_t)i * qs + h * hd;
        for (int j = 0; j <= pos; ++j) {
          const real ds = P[j] * (dP[j] - Di) * scale;
          const real* kj = g->k + (int64_t)(b * S + j) * ks + kh * hd;
          real* dkj = g->dk + (int64_t)(b * S + j) * ks + kh * hd;
          real* dvj = g->dv + (int64_t)(b * S + j) * ks + kh * hd;
          for (int d = 0; d < hd; ++d) {
            dqi[d] += ds * kj[d];
            dkj[d] += ds * qi[d];
            dvj[d] += P[j] * doi[d];
          }
        }
      }
    }
  }
  free(P);
  free(dP);
}

void FN(attention_bwd)(const real* q, const real* k, const real* v, const real* dout, real* dq, real* dk,
                       real* dv, int T, int S, int H, int Hkv, int hd) {
  att_args g = {q, k, v, dout, NULL, dq, dk, dv, T, S, H, Hkv, hd};
  parallel_for((T / S) * Hkv, g_threads, att_bwd_tasks, &g);
}

/* ------------------------------------------------------------------ clipping / AdamW / LR */
double FN(grad_clip)(real* grads, const uint8_t* has_grad, const orc_config* c, float max_norm) {
  /* GradientClipping, pkg/train/optimizer.go:169-196 */
  const int np = FN(num_params)(c);
  double total = 0;
  for (int p = 0; p < np; ++p) {
    if (!has_grad[p]) continue;
    int64_t off, r, cc;
    FN(param_info)(c, p, &off, &r, &cc);
    for (int64_t i = 0; i < r * cc; ++i) total += (double)grads[off + i] * (double)grads[off + i];
  }
  total = sqrt(total);
  if ((float)total > max_norm) {
    const real scale = (real)((double)max_norm / total);
    for (int p = 0; p < np; ++p) {
      if (!has_grad[p]) continue;
      int64_t off, r, cc;
      FN(param_info)(c, p, &off, &r, &cc);
      for (int64_t i = 0; i < r * cc; ++i) grads[off + i] *= scale;
    }
  }
  return total;
}

void FN(adamw_step)(real* params, const real* grads, const uint8_t* has_grad, real* m, real* v,
                    const orc_config* c, orc_optim_state* st) {
  /* AdamW.Step, pkg/train/optimizer.go:37-76 (float32 state, float64 update) */
  st->adam_step++;
  const double bc1 = 1.0 - pow((double)st->beta1, (double)st->adam_step);
  const double bc2 = 1.0 - pow((double)st->beta2, (double)st->adam_step);
  const real b1 = st->beta1, b2 = st->beta2, lr = st->lr, wd = st->weight_decay;
  const int np = FN(num_params)(c);
  for (int p = 0; p < np; ++p) {
    if (!has_grad[p]) continue;
    int64_t off, r, cc;
    FN(param_info)(c, p, &off, &r, &cc);
    for (int64_t i = off; i < off + r * cc; ++i) {
      const real g = grads[i];
      m[i] = b1 * m[i] + (1 - b1) * g;
      v[i] = b2 * v[i] + (1 - b2) * g * g;
      const double mhat = (double)m[i] / bc1;
      const double vhat = (double)v[i] / bc2;
      const real update = (real)(mhat / (sqrt(vhat) + (double)st->eps));
      params[i] -= lr * (update + wd * params[i]);
    }
  }
}

float FN(get_lr)(const orc_optim_state* st, int step) { /* LRScheduler.GetLR, optimizer.go:157-166 */
  if (step < st->warmup_steps) return st->initial_lr * (float)step / (float)st->warmup_steps;
  const double progress = (double)(step - st->warmup_steps) / (double)(st->total_steps - st->warmup_steps);
  return st->initial_lr * (float)(0.5 * (1 + cos(M_PI * progress)));
}

/* ------------------------------------------------------------------ the model
 * TrainableModel.Forward (trainer.go:271-305), forwardLayer (:308-320),
 * forwardAttention (:323-389), forwardFFN (:392-426), then the backward the
 * tape runs (grad.go:43-76) in its reverse topological order. */
typedef struct {
  real *x, *n1, *rms1, *q, *k, *v, *att, *x1, *n2, *rms2, *gate, *sig, *gs, *up, *h;
} layer_acts;

static real* zalloc(int64_t n) { return (real*)calloc((size_t)(n > 0 ? n : 1), sizeof(real)); }

real FN(forward_backward)(const orc_config* c, const real* params, real* grads, uint8_t* has_grad,
                          const int64_t* inputs, const int64_t* targets, int B, int S, int backward) {
  const int T = B * S, d = c->hidden, F = c->inter, V = c->vocab, L = c->layers, H = c->heads;
  const int hd = head_dim(c), Hkv = kvh(c), kvd = Hkv * hd;
  const int llama = c->mode == ORC_MODE_LLAMA;
  g_libm_exp = llama;
  int64_t off, r, cc;
#define PARAM(idx) (FN(param_info)(c, (idx), &off, &r, &cc), params + off)
#define GRAD(idx) (FN(param_info)(c, (idx), &off, &r, &cc), has_grad[(idx)] = 1, grads + off)

  real *cos_t = NULL, *sin_t = NULL;
  if (llama) {
    cos_t = zalloc((int64_t)S * (hd / 2));
    sin_t = zalloc((int64_t)S * (hd / 2));
    FN(rope_table)(hd, S, c->rope_theta, cos_t, sin_t);
  }

  /* embedding (trainer.go:276-291): out-of-range ids read row 0 */
  real* x0 = zalloc((int64_t)T * d);
  const real* E = PARAM(0);
  const real* P = llama ? NULL : PARAM(1);
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s) {
      int64_t tok = inputs[(int64_t)b * S + s];
      if (tok < 0 || tok >= V) tok = 0;
      for (int j = 0; j < d; ++j) {
        real e = E[tok * d + j];
        x0[((int64_t)b * S + s) * d + j] = llama ? e : e + P[(int64_t)s * d + j];
      }
    }

  layer_acts* A = (layer_acts*)calloc((size_t)L, sizeof(layer_acts));
  real* x = x0;
  for (int l = 0; l < L; ++l) {
    layer_acts* a = &A[l];
    a->x = x;
    a->n1 = zalloc((int64_t)T * d);
    a->rms1 = zalloc(T);
    FN(rmsnorm_fwd)(x, PARAM(layer_param(c, l, P_ATTN_NORM)), a->n1, a->rms1, T, d, c->norm_eps);
    a->q = zalloc((int64_t)T * d);
    a->k = zalloc((int64_t)T * kvd);
    a->v = zalloc((int64_t)T * kvd);
    FN(matmul_transpose_b)(a->n1, PARAM(layer_param(c, l, P_WQ)), a->q, T, d, d);
    FN(matmul_transpose_b)(a->n1, PARAM(layer_param(c, l, P_WK)), a->k, T, d, kvd);
    FN(matmul_transpose_b)(a->n1, PARAM(layer_param(c, l, P_WV)), a->v, T, d, kvd);
    if (llama) { /* RoPE on q and k, stored rotated */
      FN(rope_apply)(a->q, T, S, H, hd, cos_t, sin_t, 0);
      FN(rope_apply)(a->k, T, S, Hkv, hd, cos_t, sin_t, 0);
    }
    a->att = zalloc((int64_t)T * d);
    FN(attention_fwd)(a->q, a->k, a->v, a->att, T, S, H, Hkv, hd);
    real* o = zalloc((int64_t)T * d);
    FN(matmul_transpose_b)(a->att, PARAM(layer_param(c, l, P_WO)), o, T, d, d);
    a->x1 = zalloc((int64_t)T * d);
    for (int64_t i = 0; i < (int64_t)T * d; ++i) a->x1[i] = x[i] + o[i]; /* Add, ops.go:6-17 */
    free(o);
    a->n2 = zalloc((int64_t)T * d);
    a->rms2 = zalloc(T);
    FN(rmsnorm_fwd)(a->x1, PARAM(layer_param(c, l, P_FFN_NORM)), a->n2, a->rms2, T, d, c->norm_eps);
    a->gate = zalloc((int64_t)T * F);
    a->up = zalloc((int64_t)T * F);
    FN(matmul_transpose_b)(a->n2, PARAM(layer_param(c, l, P_WGATE)), a->gate, T, d, F);
    FN(matmul_transpose_b)(a->n2, PARAM(layer_param(c, l, P_WUP)), a->up, T, d, F);
    a->sig = zalloc((int64_t)T * F);
    a->gs = zalloc((int64_t)T * F);
    FN(silu_fwd)(a->gate, a->gs, a->sig, (int64_t)T * F);
    a->h = zalloc((int64_t)T * F);
    for (int64_t i = 0; i < (int64_t)T * F; ++i) a->h[i] = a->gs[i] * a->up[i]; /* trainer.go:405-407 */
    real* dn = zalloc((int64_t)T * d);
    FN(matmul_transpose_b)(a->h, PARAM(layer_param(c, l, P_WDOWN)), dn, T, F, d);
    real* x2 = zalloc((int64_t)T * d);
    for (int64_t i = 0; i < (int64_t)T * d; ++i) x2[i] = a->x1[i] + dn[i];
    free(dn);
    x = x2;
  }
  real* nF = zalloc((int64_t)T * d);
  real* rmsF = zalloc(T);
  FN(rmsnorm_fwd)(x, PARAM(out_norm_param(c)), nF, rmsF, T, d, c->norm_eps);
  real* logits = zalloc((int64_t)T * V);
  FN(matmul_transpose_b)(nF, E, logits, T, d, V);

  /* TrainStep flattens targets b*seqLen+s (trainer.go:480-485) */
  real* probs = backward && llama ? zalloc((int64_t)T * V) : NULL;
  const real loss = FN(softmax_ce)(logits, targets, T, V, probs);

  if (backward) {
    /* seed: reference mode calls logits.Backward() with a nil grad -> ones
     * (grad.go:45-50); Llama mode runs the loss node's GradFn. */
    real* dlogits = logits; /* logits are not needed any more */
    if (llama) {
      memset(dlogits, 0, sizeof(real) * (size_t)T * V);
      FN(softmax_ce_grad)(probs, targets, T, V, dlogits);
      free(probs);
    } else {
      for (int64_t i = 0; i < (int64_t)T * V; ++i) dlogits[i] = 1;
    }
    /* LM head MatMulGrad(nF, TokenEmbed): dA then dB */
    real* dnF = zalloc((int64_t)T * d);
    FN(matmul_grad_da)(dlogits, E, dnF, T, d, V);
    FN(matmul_grad_db)(dlogits, nF, GRAD(0), T, d, V);
    /* OutputNorm */
    real* dx = zalloc((int64_t)T * d);
    FN(rmsnorm_bwd)(x, PARAM(out_norm_param(c)), rmsF, dnF, dx, GRAD(out_norm_param(c)), T, d, llama);
    free(dnF);
    for (int l = L - 1; l >= 0; --l) {
      layer_acts* a = &A[l];
      /* x2 = AddGrad(x1, ffnOut): x1.Grad starts as a copy of dx2, ffnOut.Grad = dx2 */
      real* dx1 = zalloc((int64_t)T * d);
      add_into(dx1, dx, (int64_t)T * d);
      /* ffnOut = MatMulGrad(h, WDown) */
      real* dh = zalloc((int64_t)T * F);
      FN(matmul_grad_da)(dx, PARAM(layer_param(c, l, P_WDOWN)), dh, T, F, d);
      FN(matmul_grad_db)(dx, a->h, GRAD(layer_param(c, l, P_WDOWN)), T, F, d);
      /* product node (trainer.go:418-421) */
      real* dgs = zalloc((int64_t)T * F);
      real* dup = zalloc((int64_t)T * F);
      for (int64_t i = 0; i < (int64_t)T * F; ++i) {
        dgs[i] += dh[i] * a->up[i];
        dup[i] += dh[i] * a->gs[i];
      }
      free(dh);
      /* up = MatMulGrad(n2, WUp) runs before the SiLU node in reverse topo order */
      real* dn2 = zalloc((int64_t)T * d);
      FN(matmul_grad_da)(dup, PARAM(layer_param(c, l, P_WUP)), dn2, T, d, F);
      FN(matmul_grad_db)(dup, a->n2, GRAD(layer_param(c, l, P_WUP)), T, d, F);
      free(dup);
      real* dgate = zalloc((int64_t)T * F);
      FN(silu_bwd)(a->gate, a->sig, dgs, dgate, (int64_t)T * F);
      free(dgs);
      FN(matmul_grad_da)(dgate, PARAM(layer_param(c, l, P_WGATE)), dn2, T, d, F);
      FN(matmul_grad_db)(dgate, a->n2, GRAD(layer_param(c, l, P_WGATE)), T, d, F);
      free(dgate);
      FN(rmsnorm_bwd)(a->x1, PARAM(layer_param(c, l, P_FFN_NORM)), a->rms2, dn2, dx1,
                      GRAD(layer_param(c, l, P_FFN_NORM)), T, d, llama);
      free(dn2);
      /* x1 = AddGrad(x, attnOut) */
      real* dx0 = zalloc((int64_t)T * d);
      add_into(dx0, dx1, (int64_t)T * d);
      real* datt = zalloc((int64_t)T * d);
      FN(matmul_grad_da)(dx1, PARAM(layer_param(c, l, P_WO)), datt, T, d, d);
      FN(matmul_grad_db)(dx1, a->att, GRAD(layer_param(c, l, P_WO)), T, d, d);
      free(dx1);
      if (llama) {
        real* dq = zalloc((int64_t)T * d);
        real* dk = zalloc((int64_t)T * kvd);
        real* dv = zalloc((int64_t)T * kvd);
        FN(attention_bwd)(a->q, a->k, a->v, datt, dq, dk, dv, T, S, H, Hkv, hd);
        FN(rope_apply)(dq, T, S, H, hd, cos_t, sin_t, 1);
        FN(rope_apply)(dk, T, S, Hkv, hd, cos_t, sin_t, 1);
        /* reverse topo order of the attention parents [q, k, v]: v, k, q */
        real* dn1 = zalloc((int64_t)T * d);
        FN(matmul_grad_da)(dv, PARAM(layer_param(c, l, P_WV)), dn1, T, d, kvd);
        FN(matmul_grad_db)(dv, a->n1, GRAD(layer_param(c, l, P_WV)), T, d, kvd);
        FN(matmul_grad_da)(dk, PARAM(layer_param(c, l, P_WK)), dn1, T, d, kvd);
        FN(matmul_grad_db)(dk, a->n1, GRAD(layer_param(c, l, P_WK)), T, d, kvd);
        FN(matmul_grad_da)(dq, PARAM(layer_param(c, l, P_WQ)), dn1, T, d, d);
        FN(matmul_grad_db)(dq, a->n1, GRAD(layer_param(c, l, P_WQ)), T, d, d);
        free(dq);
        free(dk);
        free(dv);
        FN(rmsnorm_bwd)(a->x, PARAM(layer_param(c, l, P_ATTN_NORM)), a->rms1, dn1, dx0,
                        GRAD(layer_param(c, l, P_ATTN_NORM)), T, d, 1);
        free(dn1);
      }
      free(datt);
      free(dx);
      dx = dx0;
    }
    if (llama) { /* embedding GradFn: dE[tok] += dx0[t], t ascending */
      real* dE = GRAD(0);
      for (int t = 0; t < T; ++t) {
        int64_t tok = inputs[t];
        if (tok < 0 || tok >= V) tok = 0;
        for (int j = 0; j < d; ++j) dE[tok * d + j] += dx[(int64_t)t * d + j];
      }
    }
    free(dx);
  }
  free(logits);
  free(nF);
  free(rmsF);
  if (x != x0) free(x);
  for (int l = 0; l < L; ++l) {
    layer_acts* a = &A[l];
    if (a->x != x0) free(a->x);
    free(a->n1); free(a->rms1); free(a->q); free(a->k); free(a->v); free(a->att); free(a->x1);
    free(a->n2); free(a->rms2); free(a->gate); free(a->sig); free(a->gs); free(a->up); free(a->h);
  }
  free(A);
  free(x0);
  free(cos_t);
  free(sin_t);
#undef PARAM
#undef GRAD
  g_libm_exp = 0;
  return loss;
}

/* Trainer.TrainStep, trainer.go:462-505: LR, ZeroGrad, forward, loss,
 * backward, clip, AdamW.  grads/has_grad persist across steps like the
 * reference's lazily allocated GradTensor.Grad. */
real FN(train_step)(const orc_config* c, real* params, real* grads, uint8_t* has_grad, real* m, real* v,
                    orc_optim_state* st, const int64_t* inputs, const int64_t* targets, int B, int S,
                    double* grad_norm) {
  st->trainer_step++;
  st->lr = FN(get_lr)(st, st->trainer_step);
  const int np = FN(num_params)(c);
  for (int p = 0; p < np; ++p) { /* ZeroGrad zeroes only existing grads (grad.go:34-41) */
    if (!has_grad[p]) continue;
    int64_t off, r, cc;
    FN(param_info)(c, p, &off, &r, &cc);
    memset(grads + off, 0, sizeof(real) * (size_t)(r * cc));
  }
  const real loss = FN(forward_backward)(c, params, grads, has_grad, inputs, targets, B, S, 1);
  const double norm = FN(grad_clip)(grads, has_grad, c, st->grad_clip);
  if (grad_norm) *grad_norm = norm;
  FN(adamw_step)(params, grads, has_grad, m, v, c, st);
  return loss;
}
