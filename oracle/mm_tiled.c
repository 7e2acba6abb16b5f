/*
 * mm_tiled.c -- CPU oracle for tilec.ext.matrix_mul.  TEST INFRASTRUCTURE ONLY:
 * used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker, never by the product path.
 *
 * tilec_oracle_mm_tiled restates the reference kernel tilec/ext.py:13-24
 * (_matmul_tiled) together with its launch grid tilec/ext.py:62:
 *   - one program per (pid0, pid1) in (cdiv(M,BM), cdiv(N,BN))          ext.py:62
 *   - rm = pid0*BM + arange(BM), rn = pid1*BN + arange(BN)             ext.py:15-16
 *   - acc = zeros((BM, BN))                                            ext.py:18
 *   - for k in range(0, K, BK): ka = k + arange(BK)                     ext.py:19-20
 *       x = load(a[rm, ka], mask rm<M & ka<K, other 0.0)               ext.py:21
 *       y = load(b[ka, rn], mask ka<K & rn<N, other 0.0)               ext.py:22
 *       acc = acc + dot(x, y)                                          ext.py:23
 *   - store(c[rm, rn], acc, mask rm<M & rn<N)                          ext.py:24
 * dot(x, y) is computed in fp32 with the products summed in k order, then added
 * to acc (the DSL evaluates the dot first, then the add).  Built with
 * -ffp-contract=off so no FMA contraction changes the rounding.
 *
 * tilec_oracle_mm_f64 is the fp64-accumulating reference the fp32 oracle is
 * verified against (relative Frobenius error ~3e-7 on N(0,1) data).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

/* Programs are independent (each owns its output tile), so they are spread over
 * pthreads by pid0 stripes; the result does not depend on the thread count. */
typedef struct {
  const float *a, *b;
  float* c;
  int64_t M, N, K, lda, ldb, ldc;
  int BM, BN, BK;
  int64_t p0_begin, p0_step;
} tiled_job;

static void* tiled_worker(void* arg) {
  const tiled_job* j = (const tiled_job*)arg;
  const float *a = j->a, *b = j->b;
  float* c = j->c;
  const int64_t M = j->M, N = j->N, K = j->K, lda = j->lda, ldb = j->ldb, ldc = j->ldc;
  const int BM = j->BM, BN = j->BN, BK = j->BK;
  const int64_t gm = cdiv64(M, BM), gn = cdiv64(N, BN);
  for (int64_t pid0 = j->p0_begin; pid0 < gm; pid0 += j->p0_step) {
    for (int64_t pid1 = 0; pid1 < gn; ++pid1) {
      float* acc = (float*)calloc((size_t)BM * BN, sizeof(float));
      float* x = (float*)malloc((size_t)BM * BK * sizeof(float));
      float* y = (float*)malloc((size_t)BK * BN * sizeof(float));
      for (int64_t k = 0; k < K; k += BK) {
        for (int i = 0; i < BM; ++i) {
          const int64_t rm = pid0 * BM + i;
          for (int kk = 0; kk < BK; ++kk) {
            const int64_t ka = k + kk;
            x[i * BK + kk] = (rm < M && ka < K) ? a[rm * lda + ka] : 0.0f;
          }
        }
        for (int kk = 0; kk < BK; ++kk) {
          const int64_t ka = k + kk;
          for (int j = 0; j < BN; ++j) {
            const int64_t rn = pid1 * BN + j;
            y[kk * BN + j] = (ka < K && rn < N) ? b[ka * ldb + rn] : 0.0f;
          }
        }
        for (int i = 0; i < BM; ++i) {
          for (int j = 0; j < BN; ++j) {
            float d = 0.0f;
            for (int kk = 0; kk < BK; ++kk) d += x[i * BK + kk] * y[kk * BN + j];
            acc[i * BN + j] = acc[i * BN + j] + d;
          }
        }
      }
      for (int i = 0; i < BM; ++i) {
        const int64_t rm = pid0 * BM + i;
        if (rm >= M) continue;
        for (int j = 0; j < BN; ++j) {
          const int64_t rn = pid1 * BN + j;
          if (rn < N) c[rm * ldc + rn] = acc[i * BN + j];
        }
      }
      free(acc);
      free(x);
      free(y);
    }
  }
  return NULL;
}

static int oracle_threads(void) {
  const char* env = getenv("TILEC_ORACLE_THREADS");
  long n = env ? strtol(env, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

int tilec_oracle_mm_tiled(const float* a, const float* b, float* c, int64_t M, int64_t N, int64_t K, int64_t lda,
                          int64_t ldb, int64_t ldc, int BM, int BN, int BK) {
  if (M < 0 || N < 0 || K < 0 || BM <= 0 || BN <= 0 || BK <= 0) return 1;
  int nt = oracle_threads();
  const int64_t gm = cdiv64(M, BM);
  if (nt > gm) nt = (int)(gm > 0 ? gm : 1);
  pthread_t th[256];
  tiled_job jobs[256];
  for (int t = 0; t < nt; ++t) {
    tiled_job jb = {a, b, c, M, N, K, lda, ldb, ldc, BM, BN, BK, t, nt};
    jobs[t] = jb;
  }
  int started = 1;
  for (; started < nt; ++started)
    if (pthread_create(&th[started], NULL, tiled_worker, &jobs[started]) != 0) break;
  /* Stripes whose thread could not start run on this thread. */
  for (int t = started; t < nt; ++t) tiled_worker(&jobs[t]);
  tiled_worker(&jobs[0]);
  for (int t = 1; t < started; ++t) pthread_join(th[t], NULL);
  return 0;
}

int tilec_oracle_mm_f64(const float* a, const float* b, double* c, int64_t M, int64_t N, int64_t K, int64_t lda,
                        int64_t ldb, int64_t ldc) {
  if (M < 0 || N < 0 || K < 0) return 1;
  for (int64_t m = 0; m < M; ++m) {
    double* row = c + m * ldc;
    for (int64_t n = 0; n < N; ++n) row[n] = 0.0;
    for (int64_t k = 0; k < K; ++k) {
      const double av = (double)a[m * lda + k];
      const float* brow = b + k * ldb;
      for (int64_t n = 0; n < N; ++n) row[n] += av * (double)brow[n];
    }
  }
  return 0;
}
