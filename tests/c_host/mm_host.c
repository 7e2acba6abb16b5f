/* mm_host.c -- a C host of the ABI in include/tilec_mm.h, the way a non-Python caller (a cgo,
 * JNI or N-API binding) drives it: device buffers and a stream from the CUDA runtime,
 * tilec_mm_workspace_bytes + tilec_mm_f32 per product, tilec_mm_f32_splitk_noalloc without
 * a workspace, status words and error strings.  Each product is checked against an fp64 sum
 * computed here; the program prints one line per case and exits 0 only if every case passes.
 * Test infrastructure (tests/test_c_host.py builds and runs it); not part of the library. */
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tilec_mm.h"

#define CHECK_CUDA(x)                                                              \
  do {                                                                             \
    cudaError_t e_ = (x);                                                          \
    if (e_ != cudaSuccess) {                                                       \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      exit(2);                                                                     \
    }                                                                              \
  } while (0)

static unsigned long long g_rng = 88172645463325252ull;
static float next_value(void) { /* uniform in [-1, 1), xorshift64 */
  g_rng ^= g_rng << 13;
  g_rng ^= g_rng >> 7;
  g_rng ^= g_rng << 17;
  return (float)((double)(g_rng >> 11) / 9007199254740992.0 * 2.0 - 1.0);
}

/* relFrob of C (ldc) against the fp64 product of A (lda) and B (ldb), all row-major. */
static double rel_frob(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb, int64_t ldc) {
  double num = 0.0, den = 0.0;
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      double ref = 0.0;
      for (int64_t k = 0; k < K; ++k) ref += (double)A[i * lda + k] * (double)B[k * ldb + j];
      const double d = (double)C[i * ldc + j] - ref;
      num += d * d;
      den += ref * ref;
    }
  return den > 0.0 ? sqrt(num / den) : sqrt(num);
}

static int run_case(const char* name, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int variant,
                    int noalloc, cudaStream_t s) {
  const size_t na = (size_t)(M * lda), nb = (size_t)(K * ldb), nc = (size_t)(M * N);
  float* hA = (float*)malloc(na * sizeof(float));
  float* hB = (float*)malloc(nb * sizeof(float));
  float* hC = (float*)malloc(nc * sizeof(float));
  for (size_t i = 0; i < na; ++i) hA[i] = next_value();
  for (size_t i = 0; i < nb; ++i) hB[i] = next_value();
  float *dA, *dB, *dC;
  CHECK_CUDA(cudaMalloc((void**)&dA, na * sizeof(float)));
  CHECK_CUDA(cudaMalloc((void**)&dB, nb * sizeof(float)));
  CHECK_CUDA(cudaMalloc((void**)&dC, nc * sizeof(float)));
  CHECK_CUDA(cudaMemcpyAsync(dA, hA, na * sizeof(float), cudaMemcpyHostToDevice, s));
  CHECK_CUDA(cudaMemcpyAsync(dB, hB, nb * sizeof(float), cudaMemcpyHostToDevice, s));
  int rc;
  void* ws = NULL;
  size_t ws_bytes = 0;
  if (noalloc) {
    rc = tilec_mm_f32_splitk_noalloc(dA, dB, dC, M, N, K, lda, ldb, N, 0, s);
  } else {
    tilec_mm_cfg cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.variant = variant;
    ws_bytes = tilec_mm_workspace_bytes(dA, dB, dC, M, N, K, lda, ldb, N, &cfg);
    if (ws_bytes) CHECK_CUDA(cudaMalloc(&ws, ws_bytes));
    rc = tilec_mm_f32(dA, dB, dC, M, N, K, lda, ldb, N, &cfg, ws, ws_bytes, s);
  }
  int ok = rc == TILEC_OK;
  if (!ok) fprintf(stderr, "%s: tilec call returned %d (%s)\n", name, rc, tilec_strerror(rc));
  CHECK_CUDA(cudaMemcpyAsync(hC, dC, nc * sizeof(float), cudaMemcpyDeviceToHost, s));
  CHECK_CUDA(cudaStreamSynchronize(s));
  int32_t status = -1;
  if (tilec_mm_device_status(s, &status) != TILEC_OK || status != 0) ok = 0;
  const double err = ok ? rel_frob(hA, hB, hC, M, N, K, lda, ldb, N) : 1.0;
  const double gate = variant == TILEC_MM_TF32 ? 5e-3 : 1e-5;
  ok = ok && err <= gate;
  printf("%-28s M=%lld N=%lld K=%lld lda=%lld ldb=%lld ws=%zu relFrob=%.3e %s\n", name, (long long)M,
         (long long)N, (long long)K, (long long)lda, (long long)ldb, ws_bytes, err, ok ? "ok" : "FAIL");
  if (ws) CHECK_CUDA(cudaFree(ws));
  CHECK_CUDA(cudaFree(dA));
  CHECK_CUDA(cudaFree(dB));
  CHECK_CUDA(cudaFree(dC));
  free(hA);
  free(hB);
  free(hC);
  return ok;
}

int main(void) {
  if (tilec_mm_abi_version() != TILEC_MM_ABI_VERSION) {
    fprintf(stderr, "ABI version %d, header %d\n", tilec_mm_abi_version(), TILEC_MM_ABI_VERSION);
    return 1;
  }
  /* Argument errors come back as codes, before any device work. */
  if (tilec_mm_f32(NULL, NULL, NULL, -1, 4, 4, 4, 4, 4, NULL, NULL, 0, NULL) != TILEC_ERR_BAD_ARG) return 1;
  cudaStream_t s;
  CHECK_CUDA(cudaStreamCreate(&s));
  int ok = 1;
  ok &= run_case("auto, split-K (config 1)", 512, 64, 4096, 4096, 64, TILEC_MM_AUTO, 0, s);
  ok &= run_case("auto, CTA pair", 1024, 512, 768, 768, 512, TILEC_MM_AUTO, 0, s);
  ok &= run_case("auto, unaligned rows", 300, 333, 999, 1001, 335, TILEC_MM_AUTO, 0, s);
  ok &= run_case("3xtf32, ragged", 129, 260, 77, 77, 260, TILEC_MM_3XTF32, 0, s);
  ok &= run_case("tf32", 256, 256, 512, 512, 256, TILEC_MM_TF32, 0, s);
  ok &= run_case("simt", 200, 130, 300, 300, 130, TILEC_MM_SIMT, 0, s);
  ok &= run_case("split-K without workspace", 256, 64, 8192, 8192, 64, TILEC_MM_SPLITK, 1, s);
  CHECK_CUDA(cudaStreamDestroy(s));
  printf("%s\n", ok ? "ALL OK" : "FAILED");
  return ok ? 0 : 1;
}
