/* CPU oracle for the grxcp-b200 hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
 * load this library, and only as the checker (or the timed CPU baseline); the
 * product path never calls it.
 *
 * Each function restates one CPU reference of kubeworkz/grxcp (cited) or, for
 * operations the reference does not have, the mathematical definition in fp64:
 *
 *   ora_sgemm_ref     tests/libs/test_grxblas.cpp:36-80      fp32 GEMM, fp64 accumulate
 *   ora_sgemm_kernel  src/libs/grxblas/kernels/sgemm.cpp:62-85  fp32 accumulate in k order
 *   ora_gemm_f32seq   tests/libs/test_grxblas_ex.cpp:45-63   fp16 GemmEx gate (exact inputs)
 *   ora_igemm         tests/libs/test_grxblas_ex.cpp:267-281 int8 -> int32 gate
 *   ora_igemm_npu     tests/libs/test_grxblas_npu.cpp:50-66  int8, int64 accumulate, row-major
 *   ora_saxpy / ora_sscal / ora_sgemv  tests/libs/test_grxblas_l12.cpp:79-175 (level 1/2)
 *   ora_gemm_f64      fp64 GEMM + epilogue (bias, scales, beta) for bf16/fp8/int8-scaled
 *                     GemmEx (no reference code: parity unpinned by the reference)
 *   ora_softmax / ora_gelu  fp64 definitions (grxDNN softmax / GELU, planned only)
 *   ora_rmsnorm / ora_layernorm / ora_attention   fp64 definitions (grxDNN is planned only
 *                     in the reference: parity unpinned by the reference)
 *   conversions       bf16 / fp16 round-to-nearest-even, e4m3 RNE with saturation to +-448
 *
 * Built with plain gcc, no -ffast-math and no FMA contraction, so float
 * expressions round exactly as written (the reference's gates are compiled the
 * same way for x86-64).
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ conversions */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t ora_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float ora_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* IEEE binary16, round to nearest even, subnormals included. */
uint16_t ora_f32_to_f16(float f) {
  const uint32_t u = f2u(f);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t au = u & 0x7fffffffu;
  if (au > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  if (au >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
  if (au < 0x38800000u) {                                    /* below 2^-14: subnormal or zero */
    const double a = (double)u2f(au);
    const double q = nearbyint(a * 16777216.0); /* units of 2^-24 */
    return (uint16_t)(sign | (uint32_t)q);
  }
  uint32_t h = sign | (((au >> 23) - 112u) << 10) | ((au >> 13) & 0x3ffu);
  const uint32_t rem = au & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)h;
}

float ora_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) {
    const float v = (float)m * 5.9604644775390625e-08f; /* 2^-24 */
    return (h & 0x8000u) ? -v : v;
  }
  if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
  return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* OCP fp8 E4M3 ("fn"): bias 7, no infinities, max finite 448, NaN = S.1111.111. */
uint8_t ora_f32_to_e4m3(float f) {
  const uint8_t sign = (f2u(f) >> 24) & 0x80u;
  double a = fabs((double)f);
  if (isnan(f)) return (uint8_t)(sign | 0x7fu);
  if (a >= 448.0) return (uint8_t)(sign | 0x7eu); /* saturate */
  if (a < 0.015625) {                             /* subnormal: steps of 2^-9 */
    const double q = nearbyint(a * 512.0);
    if (q >= 8.0) return (uint8_t)(sign | 0x08u);
    return (uint8_t)(sign | (uint8_t)q);
  }
  int E;
  const double fr = frexp(a, &E); /* a = fr * 2^E, fr in [0.5, 1) */
  int e = E - 1;
  double q = nearbyint((fr * 2.0 - 1.0) * 8.0);
  if (q >= 8.0) { q = 0.0; ++e; }
  if (e > 8 || (e == 8 && q > 6.0)) return (uint8_t)(sign | 0x7eu);
  return (uint8_t)(sign | (uint8_t)((e + 7) << 3) | (uint8_t)q);
}

float ora_e4m3_to_f32(uint8_t b) {
  const int s = b & 0x80, e = (b >> 3) & 0xf, m = b & 7;
  float v;
  if (e == 15 && m == 7) v = NAN;
  else if (e == 0) v = (float)m * 0.001953125f; /* 2^-9 */
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

/* kind: 0 bf16, 1 fp16, 2 e4m3 */
void ora_encode(int kind, const float* in, void* out, long long n) {
  for (long long i = 0; i < n; ++i) {
    if (kind == 0) ((uint16_t*)out)[i] = ora_f32_to_bf16(in[i]);
    else if (kind == 1) ((uint16_t*)out)[i] = ora_f32_to_f16(in[i]);
    else ((uint8_t*)out)[i] = ora_f32_to_e4m3(in[i]);
  }
}
void ora_decode(int kind, const void* in, float* out, long long n) {
  for (long long i = 0; i < n; ++i) {
    if (kind == 0) out[i] = ora_bf16_to_f32(((const uint16_t*)in)[i]);
    else if (kind == 1) out[i] = ora_f16_to_f32(((const uint16_t*)in)[i]);
    else out[i] = ora_e4m3_to_f32(((const uint8_t*)in)[i]);
  }
}

/* ------------------------------------------------------------ GEMM gates */

/* tests/libs/test_grxblas.cpp:36-80: unpack op(A), op(B) to row-major in a
 * separate step, then accumulate in fp64; beta == 0 never reads C. */
void ora_sgemm_ref(int ta, int tb, int m, int n, int k, float alpha, const float* A, int lda, const float* B,
                   int ldb, float beta, float* C, int ldc) {
  double* a = (double*)malloc(sizeof(double) * (size_t)(m > 0 ? m : 1) * (size_t)(k > 0 ? k : 1));
  double* b = (double*)malloc(sizeof(double) * (size_t)(k > 0 ? k : 1) * (size_t)(n > 0 ? n : 1));
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < k; ++c) {
      const int sr = ta ? c : r, sc = ta ? r : c;
      a[(size_t)r * k + c] = A[(size_t)sr + (size_t)sc * lda];
    }
  for (int r = 0; r < k; ++r)
    for (int c = 0; c < n; ++c) {
      const int sr = tb ? c : r, sc = tb ? r : c;
      b[(size_t)r * n + c] = B[(size_t)sr + (size_t)sc * ldb];
    }
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < m; ++i) {
      double acc = 0.0;
      for (int l = 0; l < k; ++l) acc += a[(size_t)i * k + l] * b[(size_t)l * n + j];
      const size_t ci = (size_t)i + (size_t)j * ldc;
      C[ci] = (beta == 0.0f) ? (float)(alpha * acc) : (float)(alpha * acc + (double)beta * C[ci]);
    }
  free(a);
  free(b);
}

/* src/libs/grxblas/kernels/sgemm.cpp:62-85: one accumulator per output, fp32,
 * k in ascending order, alpha*acc (+ beta*C), batch at signed strides. */
void ora_sgemm_kernel(int ta, int tb, int m, int n, int k, float alpha, const float* A, int lda, long long sA,
                      const float* B, int ldb, long long sB, float beta, float* C, int ldc, long long sC, int batch) {
  for (int bt = 0; bt < batch; ++bt) {
    const float* Ab = A + bt * sA;
    const float* Bb = B + bt * sB;
    float* Cb = C + bt * sC;
    for (int col = 0; col < n; ++col)
      for (int row = 0; row < m; ++row) {
        float acc = 0.0f;
        for (int l = 0; l < k; ++l) {
          const float a = ta ? Ab[l + (long long)row * lda] : Ab[row + (long long)l * lda];
          const float b = tb ? Bb[col + (long long)l * ldb] : Bb[l + (long long)col * ldb];
          const float p = a * b;
          acc = acc + p;
        }
        const long long ci = row + (long long)col * ldc;
        if (beta == 0.0f) Cb[ci] = alpha * acc;
        else {
          const float t1 = alpha * acc, t2 = beta * Cb[ci];
          Cb[ci] = t1 + t2;
        }
      }
  }
}

/* tests/libs/test_grxblas_ex.cpp:45-63: fp32 accumulate from the (exact) float
 * values the fp16 inputs were made from. */
void ora_gemm_f32seq(int ta, int tb, int m, int n, int k, float alpha, const float* A, int lda, const float* B,
                     int ldb, float beta, float* C, int ldc) {
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < m; ++i) {
      float acc = 0.0f;
      for (int l = 0; l < k; ++l) {
        const float a = ta ? A[(size_t)l + (size_t)i * lda] : A[(size_t)i + (size_t)l * lda];
        const float b = tb ? B[(size_t)j + (size_t)l * ldb] : B[(size_t)l + (size_t)j * ldb];
        const float p = a * b;
        acc = acc + p;
      }
      const size_t ci = (size_t)i + (size_t)j * ldc;
      if (beta == 0.0f) C[ci] = alpha * acc;
      else {
        const float t1 = alpha * acc, t2 = beta * C[ci];
        C[ci] = t1 + t2;
      }
    }
}

/* tests/libs/test_grxblas_ex.cpp:267-281, int32 arithmetic with two's
 * complement wrap-around (done in uint32 to keep C's overflow rules out). */
void ora_igemm(int ta, int tb, int m, int n, int k, int alpha, const int8_t* A, int lda, const int8_t* B, int ldb,
               int beta, int32_t* C, int ldc) {
  for (int j = 0; j < n; ++j)
    for (int i = 0; i < m; ++i) {
      uint32_t acc = 0;
      for (int l = 0; l < k; ++l) {
        const int32_t av = ta ? A[(size_t)l + (size_t)i * lda] : A[(size_t)i + (size_t)l * lda];
        const int32_t bv = tb ? B[(size_t)j + (size_t)l * ldb] : B[(size_t)l + (size_t)j * ldb];
        acc += (uint32_t)(av * bv);
      }
      const size_t ci = (size_t)i + (size_t)j * ldc;
      uint32_t v = (uint32_t)alpha * acc;
      if (beta != 0) v += (uint32_t)beta * (uint32_t)C[ci];
      C[ci] = (int32_t)v;
    }
}

/* tests/libs/test_grxblas_npu.cpp:50-66: row-major, int64 accumulate. */
void ora_igemm_npu(int m, int n, int k, int alpha, int beta, const int8_t* A, int lda, const int8_t* B, int ldb,
                   int32_t* C, int ldc) {
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      int64_t acc = 0;
      for (int l = 0; l < k; ++l) acc += (int64_t)A[i * lda + l] * (int64_t)B[l * ldb + j];
      const size_t ci = (size_t)i * ldc + j;
      C[ci] = (beta == 0) ? (int32_t)(alpha * acc) : (int32_t)(alpha * acc + beta * C[ci]);
    }
}

/* ------------------------------------------------------------ fp64 GEMM */

typedef struct {
  int ta, tb, m, n, k, batch;
  double alpha, beta;
  const float *A, *B;
  int lda, ldb, ldc;
  long long sA, sB, sC, sBias, ssa, ssb;
  const double* Cin;
  double* Cout;
  const float* bias;
  int scale_mode;
  const float *sa, *sb;
  int j0, j1;
  int tid, nthreads;
} GemmJob;

static void* gemm_worker(void* arg) {
  const GemmJob* g = (const GemmJob*)arg;
  for (int bt = 0; bt < g->batch; ++bt) {
    const float* Ab = g->A + bt * g->sA;
    const float* Bb = g->B + bt * g->sB;
    for (int j = g->j0 + g->tid; j < g->j1; j += g->nthreads) {
      for (int i = 0; i < g->m; ++i) {
        double acc = 0.0;
        for (int l = 0; l < g->k; ++l) {
          const double a = g->ta ? Ab[l + (long long)i * g->lda] : Ab[i + (long long)l * g->lda];
          const double b = g->tb ? Bb[j + (long long)l * g->ldb] : Bb[l + (long long)j * g->ldb];
          acc += a * b;
        }
        double s = 1.0;
        if (g->scale_mode == 1) s = (double)g->sa[bt * g->ssa] * (double)g->sb[bt * g->ssb];
        if (g->scale_mode == 2) s = (double)g->sa[bt * g->ssa + i] * (double)g->sb[bt * g->ssb + j];
        const long long ci = bt * g->sC + i + (long long)j * g->ldc;
        double v = g->alpha * s * acc;
        if (g->beta != 0.0) v += g->beta * g->Cin[ci];
        if (g->bias) v += (double)g->bias[bt * g->sBias + j];
        g->Cout[ci] = v;
      }
    }
  }
  return 0;
}

/* D = alpha * s(i,j) * (op(A) op(B)) + beta * Cin + bias[j] in fp64 over
 * columns [j0, j1) of every batch member, on `nthreads` threads. Operands are
 * the decoded (exact) float values of the low-precision inputs. */
void ora_gemm_f64(int ta, int tb, int m, int n, int k, double alpha, const float* A, int lda, long long sA,
                  const float* B, int ldb, long long sB, double beta, const double* Cin, double* Cout, int ldc,
                  long long sC, int batch, const float* bias, long long sBias, int scale_mode, const float* sa,
                  const float* sb, long long ssa, long long ssb, int j0, int j1, int nthreads) {
  (void)n;
  if (nthreads < 1) nthreads = 1;
  GemmJob* jobs = (GemmJob*)calloc((size_t)nthreads, sizeof(GemmJob));
  pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
  for (int t = 0; t < nthreads; ++t) {
    GemmJob g = {ta, tb, m, n, k, batch, alpha, beta, A, B, lda, ldb, ldc, sA, sB, sC, sBias, ssa, ssb,
                 Cin, Cout, bias, scale_mode, sa, sb, j0, j1, t, nthreads};
    jobs[t] = g;
    if (nthreads > 1) pthread_create(&th[t], 0, gemm_worker, &jobs[t]);
    else gemm_worker(&jobs[t]);
  }
  if (nthreads > 1)
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], 0);
  free(jobs);
  free(th);
}

/* ------------------------------------------------------------ norms */

typedef struct {
  int rows, hidden, ln;
  const float* x;
  long long ldx;
  const float *gamma, *beta;
  double eps;
  double *y, *mean, *rstd;
  int tid, nthreads;
} NormJob;

static void* norm_worker(void* arg) {
  const NormJob* g = (const NormJob*)arg;
  for (int r = g->tid; r < g->rows; r += g->nthreads) {
    const float* xr = g->x + (long long)r * g->ldx;
    double mu = 0.0, var = 0.0;
    if (g->ln) {
      for (int c = 0; c < g->hidden; ++c) mu += xr[c];
      mu /= g->hidden;
      for (int c = 0; c < g->hidden; ++c) var += ((double)xr[c] - mu) * ((double)xr[c] - mu);
      var /= g->hidden;
    } else {
      for (int c = 0; c < g->hidden; ++c) var += (double)xr[c] * (double)xr[c];
      var /= g->hidden;
    }
    const double rs = 1.0 / sqrt(var + g->eps);
    for (int c = 0; c < g->hidden; ++c) {
      double v = ((double)xr[c] - mu) * rs * (double)g->gamma[c];
      if (g->ln && g->beta) v += (double)g->beta[c];
      g->y[(long long)r * g->hidden + c] = v;
    }
    if (g->mean) g->mean[r] = mu;
    if (g->rstd) g->rstd[r] = rs;
  }
  return 0;
}

static void run_norm(NormJob proto, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  NormJob* jobs = (NormJob*)calloc((size_t)nthreads, sizeof(NormJob));
  pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
  for (int t = 0; t < nthreads; ++t) {
    jobs[t] = proto;
    jobs[t].tid = t;
    jobs[t].nthreads = nthreads;
    if (nthreads > 1) pthread_create(&th[t], 0, norm_worker, &jobs[t]);
    else norm_worker(&jobs[t]);
  }
  if (nthreads > 1)
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], 0);
  free(jobs);
  free(th);
}

/* y = x * rsqrt(mean(x^2) + eps) * gamma   (y dense [rows, hidden]) */
void ora_rmsnorm(int rows, int hidden, const float* x, long long ldx, const float* gamma, double eps, double* y,
                 double* rstd, int nthreads) {
  NormJob p = {rows, hidden, 0, x, ldx, gamma, 0, eps, y, 0, rstd, 0, 1};
  run_norm(p, nthreads);
}

/* y = (x - mu) * rsqrt(var + eps) * gamma + beta, population variance */
void ora_layernorm(int rows, int hidden, const float* x, long long ldx, const float* gamma, const float* beta,
                   double eps, double* y, double* mean, double* rstd, int nthreads) {
  NormJob p = {rows, hidden, 1, x, ldx, gamma, beta, eps, y, mean, rstd, 0, 1};
  run_norm(p, nthreads);
}

/* Norm backward in fp64 from the definitions (the derivative of the forward
 * above with respect to x and gamma / beta; no reference code exists).
 * Statistics are recomputed from x in fp64. dx dense [rows, hidden];
 * dgamma / dbeta [hidden] (dbeta only for ln; either may be NULL). */
void ora_norm_bwd(int ln, int rows, int hidden, const float* x, const float* dy, const float* gamma, double eps,
                  double* dx, double* dgamma, double* dbeta) {
  if (dgamma)
    for (int c = 0; c < hidden; ++c) dgamma[c] = 0.0;
  if (dbeta)
    for (int c = 0; c < hidden; ++c) dbeta[c] = 0.0;
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (long long)r * hidden;
    const float* dr = dy + (long long)r * hidden;
    double mu = 0.0, var = 0.0;
    if (ln) {
      for (int c = 0; c < hidden; ++c) mu += xr[c];
      mu /= hidden;
      for (int c = 0; c < hidden; ++c) var += ((double)xr[c] - mu) * ((double)xr[c] - mu);
    } else {
      for (int c = 0; c < hidden; ++c) var += (double)xr[c] * (double)xr[c];
    }
    var /= hidden;
    const double rs = 1.0 / sqrt(var + eps);
    double sa = 0.0, sb = 0.0;
    for (int c = 0; c < hidden; ++c) {
      const double xh = ((double)xr[c] - mu) * rs, dxh = (double)dr[c] * (double)gamma[c];
      sa += ln ? dxh : dxh * xr[c];
      sb += dxh * xh;
      if (dgamma) dgamma[c] += (double)dr[c] * xh;
      if (dbeta) dbeta[c] += dr[c];
    }
    for (int c = 0; c < hidden; ++c) {
      const double xh = ((double)xr[c] - mu) * rs, dxh = (double)dr[c] * (double)gamma[c];
      dx[(long long)r * hidden + c] =
          ln ? rs * (dxh - sa / hidden - xh * sb / hidden) : rs * dxh - (double)xr[c] * rs * rs * rs * sa / hidden;
    }
  }
}

/* ------------------------------------------------------------ attention */

typedef struct {
  int H, Sq, Sk, D, causal;
  const float *q, *k, *v;
  double scale;
  const int* pairs;
  int npairs, q0, q1;
  double *o, *lse;
  int tid, nthreads;
} AttnJob;

static void* attn_worker(void* arg) {
  const AttnJob* g = (const AttnJob*)arg;
  const int nq = g->q1 - g->q0;
  double* s = (double*)malloc(sizeof(double) * (size_t)g->Sk);
  for (long long w = g->tid; w < (long long)g->npairs * nq; w += g->nthreads) {
    const int pi = (int)(w / nq), qi = g->q0 + (int)(w % nq);
    const int bh = g->pairs[pi];
    const float* qr = g->q + ((long long)bh * g->Sq + qi) * g->D;
    const float* kb = g->k + (long long)bh * g->Sk * g->D;
    const float* vb = g->v + (long long)bh * g->Sk * g->D;
    const int kend = g->causal ? (qi + 1 < g->Sk ? qi + 1 : g->Sk) : g->Sk;
    double mx = -INFINITY;
    for (int j = 0; j < kend; ++j) {
      double d = 0.0;
      for (int c = 0; c < g->D; ++c) d += (double)qr[c] * (double)kb[(long long)j * g->D + c];
      s[j] = d * g->scale;
      if (s[j] > mx) mx = s[j];
    }
    double sum = 0.0;
    for (int j = 0; j < kend; ++j) {
      s[j] = exp(s[j] - mx);
      sum += s[j];
    }
    double* orow = g->o + ((long long)pi * nq + (qi - g->q0)) * g->D;
    for (int c = 0; c < g->D; ++c) orow[c] = 0.0;
    for (int j = 0; j < kend; ++j) {
      const double p = s[j] / sum;
      for (int c = 0; c < g->D; ++c) orow[c] += p * (double)vb[(long long)j * g->D + c];
    }
    g->lse[(long long)pi * nq + (qi - g->q0)] = mx + log(sum);
  }
  free(s);
  return 0;
}

/* softmax(scale Q K^T + causal mask) V and its natural-log LSE, fp64, for the
 * (batch*heads) indices in `pairs` and query rows [q0, q1). q/k/v are dense
 * [B*H, S, D] float arrays; o is [npairs, q1-q0, D], lse [npairs, q1-q0]. */
void ora_attention(int BH, int Sq, int Sk, int D, const float* q, const float* k, const float* v, double scale,
                   int causal, const int* pairs, int npairs, int q0, int q1, double* o, double* lse, int nthreads) {
  (void)BH;
  if (nthreads < 1) nthreads = 1;
  AttnJob* jobs = (AttnJob*)calloc((size_t)nthreads, sizeof(AttnJob));
  pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
  for (int t = 0; t < nthreads; ++t) {
    AttnJob g = {0, Sq, Sk, D, causal, q, k, v, scale, pairs, npairs, q0, q1, o, lse, t, nthreads};
    jobs[t] = g;
    if (nthreads > 1) pthread_create(&th[t], 0, attn_worker, &jobs[t]);
    else attn_worker(&jobs[t]);
  }
  if (nthreads > 1)
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], 0);
  free(jobs);
  free(th);
}

/* Attention backward in fp64 from the definitions (the reference has no
 * attention): for each (b, h) pair and query row i, with P the masked softmax
 * of scale * q_i . k_j, O_i = sum_j P_ij v_j, Delta_i = dO_i . O_i:
 *   dV_j += P_ij dO_i,  dS_ij = P_ij (dO_i . v_j - Delta_i),
 *   dQ_i += scale dS_ij k_j,  dK_j += scale dS_ij q_i.
 * q, dout [BH, Sq, D]; k, v [BH, Sk, D]; outputs dense fp64 of the same
 * shapes, threaded over (b, h). */
typedef struct {
  int BH, Sq, Sk, D, causal;
  const float *q, *k, *v, *dout;
  double scale;
  double *dq, *dk, *dv;
  int tid, nthreads;
} AttnBwdJob;

static void* attn_bwd_worker(void* arg) {
  const AttnBwdJob* g = (const AttnBwdJob*)arg;
  const int D = g->D;
  double* pr = (double*)malloc(sizeof(double) * (size_t)g->Sk);
  double* o = (double*)malloc(sizeof(double) * (size_t)D);
  for (int bh = g->tid; bh < g->BH; bh += g->nthreads) {
    const float* qb = g->q + (long long)bh * g->Sq * D;
    const float* db = g->dout + (long long)bh * g->Sq * D;
    const float* kb = g->k + (long long)bh * g->Sk * D;
    const float* vb = g->v + (long long)bh * g->Sk * D;
    double* dqb = g->dq + (long long)bh * g->Sq * D;
    double* dkb = g->dk + (long long)bh * g->Sk * D;
    double* dvb = g->dv + (long long)bh * g->Sk * D;
    for (long long e = 0; e < (long long)g->Sq * D; ++e) dqb[e] = 0.0;
    for (long long e = 0; e < (long long)g->Sk * D; ++e) dkb[e] = dvb[e] = 0.0;
    for (int i = 0; i < g->Sq; ++i) {
      const float* qi = qb + (long long)i * D;
      const float* di = db + (long long)i * D;
      const int kend = g->causal ? (i + 1 < g->Sk ? i + 1 : g->Sk) : g->Sk;
      double mx = -INFINITY;
      for (int j = 0; j < kend; ++j) {
        double d = 0.0;
        for (int c = 0; c < D; ++c) d += (double)qi[c] * (double)kb[(long long)j * D + c];
        pr[j] = d * g->scale;
        if (pr[j] > mx) mx = pr[j];
      }
      double sum = 0.0;
      for (int j = 0; j < kend; ++j) {
        pr[j] = exp(pr[j] - mx);
        sum += pr[j];
      }
      for (int c = 0; c < D; ++c) o[c] = 0.0;
      for (int j = 0; j < kend; ++j) {
        pr[j] /= sum;
        for (int c = 0; c < D; ++c) o[c] += pr[j] * (double)vb[(long long)j * D + c];
      }
      double delta = 0.0;
      for (int c = 0; c < D; ++c) delta += (double)di[c] * o[c];
      for (int j = 0; j < kend; ++j) {
        double dp = 0.0;
        for (int c = 0; c < D; ++c) dp += (double)di[c] * (double)vb[(long long)j * D + c];
        const double ds = pr[j] * (dp - delta);
        for (int c = 0; c < D; ++c) {
          dvb[(long long)j * D + c] += pr[j] * (double)di[c];
          dqb[(long long)i * D + c] += g->scale * ds * (double)kb[(long long)j * D + c];
          dkb[(long long)j * D + c] += g->scale * ds * (double)qi[c];
        }
      }
    }
  }
  free(pr);
  free(o);
  return 0;
}

void ora_attention_bwd(int BH, int Sq, int Sk, int D, const float* q, const float* k, const float* v,
                       const float* dout, double scale, int causal, double* dq, double* dk, double* dv,
                       int nthreads) {
  if (nthreads < 1) nthreads = 1;
  AttnBwdJob* jobs = (AttnBwdJob*)calloc((size_t)nthreads, sizeof(AttnBwdJob));
  pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
  for (int t = 0; t < nthreads; ++t) {
    AttnBwdJob g = {BH, Sq, Sk, D, causal, q, k, v, dout, scale, dq, dk, dv, t, nthreads};
    jobs[t] = g;
    if (nthreads > 1) pthread_create(&th[t], 0, attn_bwd_worker, &jobs[t]);
    else attn_bwd_worker(&jobs[t]);
  }
  if (nthreads > 1)
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], 0);
  free(jobs);
  free(th);
}

/* conv2d in fp64 (NHWC x, KRSC w, NHWC y; no reference code exists): the
 * definition y[n,p,q,k] = sum_{r,s,c} x[n, p sh - ph + r dh, q sw - pw + s dw, c]
 * w[k,r,s,c], taps outside the image contributing 0. */
void ora_conv2d(int n, int h, int w, int c, int k, int r, int s, int ph, int pw, int sh, int sw, int dh, int dw,
                int P, int Q, const float* x, const float* f, double* y) {
  for (int ni = 0; ni < n; ++ni)
    for (int p = 0; p < P; ++p)
      for (int q = 0; q < Q; ++q)
        for (int ki = 0; ki < k; ++ki) {
          double acc = 0.0;
          for (int ri = 0; ri < r; ++ri) {
            const int hh = p * sh - ph + ri * dh;
            if (hh < 0 || hh >= h) continue;
            for (int si = 0; si < s; ++si) {
              const int ww = q * sw - pw + si * dw;
              if (ww < 0 || ww >= w) continue;
              const float* xr = x + (((long long)ni * h + hh) * w + ww) * c;
              const float* fr = f + (((long long)ki * r + ri) * s + si) * c;
              for (int ci = 0; ci < c; ++ci) acc += (double)xr[ci] * (double)fr[ci];
            }
          }
          y[(((long long)ni * P + p) * Q + q) * k + ki] = acc;
        }
}

/* ------------------------------------------------------------ level 1 / 2 */

/* BLAS increment addressing (tests/libs/test_grxblas_l12.cpp:27-31). */
static long long ora_vec_index(long long i, long long n, int inc) {
  return inc > 0 ? i * inc : (n - 1 - i) * (long long)(-inc);
}

/* y = alpha*x + y (tests/libs/test_grxblas_l12.cpp:79-92) */
void ora_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy) {
  for (int i = 0; i < n; ++i) {
    const float t = alpha * x[ora_vec_index(i, n, incx)];
    y[ora_vec_index(i, n, incy)] = t + y[ora_vec_index(i, n, incy)];
  }
}

/* x = alpha*x, incx > 0 (tests/libs/test_grxblas_l12.cpp:110-117) */
void ora_sscal(int n, float alpha, float* x, int incx) {
  for (int i = 0; i < n; ++i) x[ora_vec_index(i, n, incx)] = alpha * x[ora_vec_index(i, n, incx)];
}

/* y = alpha*op(A)*x + beta*y, A stored m x n column-major; beta == 0 never
 * reads y (tests/libs/test_grxblas_l12.cpp:135-175). */
void ora_sgemv(int trans, int m, int n, float alpha, const float* A, int lda, const float* x, int incx, float beta,
               float* y, int incy) {
  const int rows = trans ? n : m, depth = trans ? m : n;
  for (int o = 0; o < rows; ++o) {
    float acc = 0.0f;
    for (int d = 0; d < depth; ++d) {
      const int ar = trans ? d : o, ac = trans ? o : d;
      const float p = A[(size_t)ar + (size_t)ac * (size_t)lda] * x[ora_vec_index(d, depth, incx)];
      acc = acc + p;
    }
    const long long yi = ora_vec_index(o, rows, incy);
    if (beta == 0.0f) y[yi] = alpha * acc;
    else {
      const float t1 = alpha * acc, t2 = beta * y[yi];
      y[yi] = t1 + t2;
    }
  }
}

/* ------------------------------------------------------------ softmax / GELU */

/* Row softmax in fp64 with the max-subtraction identity (definition). */
void ora_softmax(int rows, int cols, const float* x, long long ldx, double* y) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (long long)r * ldx;
    double mx = -INFINITY, s = 0.0;
    for (int c = 0; c < cols; ++c) mx = xr[c] > mx ? xr[c] : mx;
    for (int c = 0; c < cols; ++c) s += exp((double)xr[c] - mx);
    for (int c = 0; c < cols; ++c) y[(long long)r * cols + c] = exp((double)xr[c] - mx) / s;
  }
}

/* GELU in fp64: mode 0 x*Phi(x) via erf, mode 1 the tanh approximation. */
void ora_gelu(long long n, const float* x, double* y, int mode) {
  for (long long i = 0; i < n; ++i) {
    const double v = x[i];
    y[i] = mode == 0 ? 0.5 * v * (1.0 + erf(v / sqrt(2.0)))
                     : 0.5 * v * (1.0 + tanh(sqrt(2.0 / M_PI) * (v + 0.044715 * v * v * v)));
  }
}
