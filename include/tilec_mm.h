/*
 * tilec_mm.h -- C ABI of the B200 (sm_100a) fp32 GEMM library behind
 * tilec_b200.ext.matrix_mul.
 *
 * Replaces, for the one op the reference ships, the path
 *   tilec/ext.py:54-63  _matrix_mul_tiled(x1, x2)  (host: shape check, contiguous, new_empty, launch)
 *   tilec/ext.py:13-24  _matmul_tiled[grid](...)   (device: masked 64x64x16 tiled C = A.B)
 *   tilec/jit.py:88-105 _launch(...)               (kernel launch through torch.mps.compile_shader)
 * with plain pointers, sizes and a stream.  No torch type appears here; any FFI
 * (ctypes, cgo, JNI, N-API) can bind these symbols.
 *
 * Semantics (all entry points):
 *   C[m, n] = sum_k A[m, k] * B[k, n] for 0 <= m < M, 0 <= n < N, fp32 in, fp32 out,
 *   A row-major with row stride lda, B row-major with row stride ldb, C row-major
 *   with row stride ldc (strides in elements).  cfg->flags may instead declare A
 *   stored transposed (TILEC_MM_TRANS_A: A[m, k] at A[k*lda + m]) and/or B stored
 *   transposed (TILEC_MM_TRANS_B: B[k, n] at B[n*ldb + k]), i.e. the column-major
 *   views x.t() of row-major tensors, read in place by the tensor-core variants
 *   (the reference copies them, tilec/ext.py:59-60).  Elements of A/B outside [M,K]/[K,N]
 *   are never read (the reference reads them as 0.0, tilec/ext.py:21-22); elements
 *   of C outside [M,N] are never written (tilec/ext.py:24).  K == 0 writes zeros.
 *   M == 0 or N == 0 is a no-op.
 *
 * Calls are asynchronous and stream-ordered on `stream` (a cudaStream_t, NULL = the
 * legacy default stream).  They allocate no memory, never synchronise the device and
 * never throw; errors come back as a tilec_status code.  Kernels never trap: a fault
 * detected on the device is recorded in a device status word that
 * tilec_mm_device_status() reads.  Every wait inside a kernel is bounded (2 s by default,
 * tilec_mm_set_wait_limit); a kernel that gives up sets TILEC_DEV_STATUS_TIMEOUT, lets
 * its in-flight copies and MMAs land, and writes NaN over every output tile it owns
 * (C, or the split-K / stream-K partial sums, whose NaN then reaches C), so a product
 * that did not finish never reads as a finished one.  Callers that cannot tolerate NaN
 * check the status word after the call.
 */
#ifndef TILEC_MM_H
#define TILEC_MM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TILEC_MM_ABI_VERSION 6

#if defined(__GNUC__)
#define TILEC_API __attribute__((visibility("default")))
#else
#define TILEC_API
#endif

/* Return codes.  0 is success; tilec_strerror() names every code. */
typedef enum tilec_status {
  TILEC_OK = 0,
  TILEC_ERR_BAD_ARG = 1,      /* negative size, null pointer with non-empty operand, ld < row length */
  TILEC_ERR_MISALIGNED = 2,   /* a variant that needs 16-byte aligned rows was forced on unaligned operands */
  TILEC_ERR_NO_DEVICE = 3,    /* no CUDA device, or the device is not sm_100 */
  TILEC_ERR_LAUNCH = 4,       /* a kernel launch failed (cudaGetLastError after the launch) */
  TILEC_ERR_DEVICE = 5,       /* a device-side check failed (see tilec_mm_device_status) */
  TILEC_ERR_WORKSPACE = 6,    /* workspace is NULL or smaller than tilec_mm_workspace_bytes() */
  TILEC_ERR_UNSUPPORTED = 7,  /* variant/size combination not built (e.g. K > 2^31 on the TMA path) */
  TILEC_ERR_TOO_LARGE = 8     /* request exceeds a fixed limit of the entry point */
} tilec_status;

/* Kernel variants.  AUTO lets the library choose (tilec_mm_plan shows the choice). */
typedef enum tilec_mm_variant {
  TILEC_MM_AUTO = 0,
  TILEC_MM_SIMT = 1,      /* fp32 FFMA, exact fp32 products; any strides / alignment */
  TILEC_MM_SPLITK = 2,    /* SIMT with K split over CTAs + ordered reduction (skinny / small-M shapes) */
  TILEC_MM_TF32 = 3,      /* tcgen05 kind::tf32, TMEM accumulators; rows must be 16-byte aligned */
  TILEC_MM_3XTF32 = 4,    /* tcgen05 kind::tf32 with hi/lo operand split (3 MMAs) and fp32 promotion of
                             K-chunk partial sums: fp32-class accuracy; hi(x) is the tensor core's own
                             tf32 reading of x (its low 13 mantissa bits ignored) */
  TILEC_MM_3XTF32_MASKED = 5, /* as 3XTF32 with hi(x) written explicitly (low 13 bits cleared) in shared
                                memory; same results, one more shared store per element (cross-check) */
  TILEC_MM_3XMIXED = 6    /* ABI version 5.  The same three-product split with the two small cross terms,
                             a.lo(b) and lo(a).hi(b), on the bf16 tensor pipe (kind::f16, twice the tf32
                             rate): 4 tf32-MMA slots per 16 of K instead of 6.  hi(a).hi(b) stays tf32.
                             Error per product at most 3 * 2^-18 (about 1.1e-5) relative, against
                             3 * 2^-20 for 3XTF32 (bf16 rounding of terms below 2^-10 of the
                             product); relFrob about 1.5e-6 on random data (3XTF32: 1.2e-6).  Runs on the
                             CTA-pair kernel (M >= 256, N > 128), one pair per tile (TILEC_MM_STREAM_K
                             is ignored); other shapes run 3XTF32 instead (tilec_mm_plan reports the
                             variant that runs) */
} tilec_mm_variant;

/* Per-call configuration.  Zero-initialise, then set what you need. */
typedef struct tilec_mm_cfg {
  int32_t variant;     /* tilec_mm_variant */
  int32_t split_k;     /* SPLITK / tensor variants: number of K slices (0 = choose) */
  int32_t flags;       /* TILEC_MM_TRANS_A | TILEC_MM_TRANS_B (operand storage order), TILEC_MM_STREAM_K,
                          TILEC_MM_TILE_M64 | TILEC_MM_TILE_M128; 0 = row-major, library's choice */
  int32_t activation;  /* TILEC_MM_ACT_*: applied to every element of C as it is written */
  int32_t reserved[4]; /* must be zero */
} tilec_mm_cfg;

/* cfg->activation: C = act(A.B + bias) (bias only through tilec_mm_f32_ex). */
#define TILEC_MM_ACT_NONE 0
#define TILEC_MM_ACT_RELU 1 /* max(x, 0) */
#define TILEC_MM_ACT_GELU 2 /* x * (1 + erf(x / sqrt(2))) / 2 */

/* cfg->flags.  With TRANS_A, lda >= M (A is K rows of M); with TRANS_B, ldb >= K (B is N
 * rows of K).  The tensor-core variants read either order in place (TMA boxes and UMMA
 * descriptors for K-major or MN-major tiles); SIMT / SPLITK first transpose a
 * transposed operand into the workspace.  (ABI version 1 had no flags or activation word:
 * they were reserved[0..1] and had to be zero, so version-1 callers keep their meaning.) */
#define TILEC_MM_TRANS_A 1
#define TILEC_MM_TRANS_B 2

/* cfg->flags (ABI version 4): stream-K for the CTA-pair tensor-core kernel (256 x 256
 * tiles; M >= 256, N > 128).  The GEMM then runs as one wave of CTA pairs that share out
 * the K blocks of the tiles beyond the last complete wave, instead of one pair per tile,
 * and the pairs add each tile's partial sums in a fixed order (results are deterministic
 * and independent of timing, but differ in rounding from the one-pair-per-tile form).
 * AUTO with split_k == 0 uses it where it pays (81 tiles on 74 pair slots: 1.47x on B200);
 * setting the flag asks for it whenever the pair kernel runs and split_k <= 1; split_k >= 2
 * (K slices) never uses it.  tilec_mm_plan sets the flag in its output when the plan is
 * stream-K, so feeding that output back reproduces the plan.  Needs workspace (partial
 * tiles, 256 KiB per pair): ask tilec_mm_workspace_bytes. */
#define TILEC_MM_STREAM_K 4

/* cfg->flags (ABI version 6): rows per output tile of the 1-CTA tensor-core kernel.  AUTO
 * takes 64-row tiles (tcgen05 M = 64) for products of at most 64 rows and 128-row tiles
 * otherwise; these bits force one or the other (TILE_M64 also rules out the
 * CTA-pair kernel; setting both is TILEC_ERR_BAD_ARG).  tilec_mm_plan sets the bit of the
 * tile that runs whenever the 1-CTA tensor-core kernel is the plan. */
#define TILEC_MM_TILE_M64 8
#define TILEC_MM_TILE_M128 16

/* C = A . B  (see the semantics block above).
 * cfg may be NULL (= AUTO).  workspace/ws_bytes: scratch for split-K partial sums;
 * may be NULL/0 when tilec_mm_workspace_bytes() returns 0 for the same arguments.
 * Replaces tilec/ext.py:54-63 + tilec/jit.py:88-105 (one launch per call). */
TILEC_API int tilec_mm_f32(const float* A, const float* B, float* C,
                 int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int64_t ldc,
                 const tilec_mm_cfg* cfg,
                 void* workspace, size_t ws_bytes,
                 void* stream);

/* Batched products with a fused epilogue (no counterpart in the reference; the next op
 * surface its README names).  For b < batch:
 *   C_b = act(A_b . B_b + bias)   A_b = A + b*stride_a, B_b = B + b*stride_b, C_b = C + b*stride_c
 * (strides in elements; a zero stride_a / stride_b shares that operand across the batch;
 * the batches of C must not overlap: stride_c >= (M-1)*ldc + N when batch > 1).  bias is
 * N floats added per column, or NULL; act = cfg->activation.  Layout flags, variants and
 * workspace rules as tilec_mm_f32 (size from tilec_mm_workspace_bytes_ex).  The tensor-
 * core kernels take the batch as a grid dimension (3-D tensor maps) and apply the epilogue
 * in their output stores (in the split-K reduction when K is split); batches beyond 65535
 * run as consecutive launches. */
TILEC_API int tilec_mm_f32_ex(const float* A, const float* B, float* C, const float* bias,
                    int64_t M, int64_t N, int64_t K,
                    int64_t lda, int64_t ldb, int64_t ldc,
                    int64_t batch, int64_t stride_a, int64_t stride_b, int64_t stride_c,
                    const tilec_mm_cfg* cfg,
                    void* workspace, size_t ws_bytes,
                    void* stream);

/* Bytes of workspace tilec_mm_f32_ex needs (0 when none); NULL operands as below. */
TILEC_API size_t tilec_mm_workspace_bytes_ex(const float* A, const float* B, const float* C,
                                   int64_t M, int64_t N, int64_t K,
                                   int64_t lda, int64_t ldb, int64_t ldc,
                                   int64_t batch, int64_t stride_a, int64_t stride_b, int64_t stride_c,
                                   const tilec_mm_cfg* cfg);

/* Bytes of workspace tilec_mm_f32 needs for these arguments (0 when none).
 * Pointer alignment affects the AUTO choice, so pass the same pointers (or NULL
 * to assume 16-byte aligned operands). */
TILEC_API size_t tilec_mm_workspace_bytes(const float* A, const float* B, const float* C,
                                int64_t M, int64_t N, int64_t K,
                                int64_t lda, int64_t ldb, int64_t ldc,
                                const tilec_mm_cfg* cfg);

/* Resolve AUTO (and split_k == 0) to the concrete variant/split tilec_mm_f32 would
 * launch, without launching.  Writes the resolved config to *out.
 * Counterpart of the reference's per-shape config pick (tilec/tune.py:143-151). */
TILEC_API int tilec_mm_plan(const float* A, const float* B, const float* C,
                  int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc,
                  const tilec_mm_cfg* cfg, tilec_mm_cfg* out);

/* Install a per-shape selection table used by AUTO.  Each row is
 * {log2M_lo, log2M_hi, log2N_lo, log2N_hi, log2K_lo, log2K_hi, variant, split_k}
 * (int32, bounds inclusive-exclusive, first matching row wins).  rows == 0 clears
 * the table (built-in rules apply).  Not thread-safe against concurrent calls. */
TILEC_API int tilec_mm_set_table(const int32_t* rows, int32_t nrows);

/* Bits of the device status word. */
#define TILEC_DEV_STATUS_TIMEOUT 1    /* a bounded wait gave up (time limit); the kernel unwound */
#define TILEC_DEV_STATUS_TMEM 2       /* TMEM allocation returned an unexpected address */
#define TILEC_DEV_STATUS_BAD_LAUNCH 4 /* a kernel was launched with a block shape it was not built for */

/* Read and clear the device status word of the current device (0 = clean).
 * Synchronises `stream`. */
TILEC_API int tilec_mm_device_status(void* stream, int32_t* status_out);

/* Failure-detection control (no counterpart in the reference).  Sets the limit of every
 * bounded wait inside this library's kernels on the current device to `limit_ns`
 * nanoseconds (0 restores the default of 2 s; larger values are clamped to 2 s), in
 * stream order on `stream`, and synchronises `stream`.  Tests shorten it so that a real
 * GEMM launch gives up -- its output tiles then read NaN and the status word reads
 * TILEC_DEV_STATUS_TIMEOUT -- and then restore it; the context stays usable throughout.
 * Device-wide state: do not lower it while products of other callers run on the device. */
TILEC_API int tilec_mm_set_wait_limit(int64_t limit_ns, void* stream);

/* Failure-detection self-test (no counterpart in the reference).  Launches one CTA on
 * `stream` that waits on a shared-memory mbarrier nothing ever arrives on, through the
 * same bounded wait every GEMM kernel uses, with a limit of `limit_ns` nanoseconds
 * (clamped to [1 ms, 2 s]).  The wait gives up, records TILEC_DEV_STATUS_TIMEOUT and the
 * kernel returns: no trap, no fault, the context stays usable.  Returns the launch status;
 * read the outcome with tilec_mm_device_status. */
TILEC_API int tilec_mm_selftest_wait(int64_t limit_ns, void* stream);

/* Text for a tilec_status code (static storage). */
TILEC_API const char* tilec_strerror(int code);

/* ABI version (TILEC_MM_ABI_VERSION) and the sm arch the library was built for. */
TILEC_API int tilec_mm_abi_version(void);
TILEC_API int tilec_mm_built_arch(void);

/* Size of the device-resident scratch behind tilec_mm_f32_splitk_noalloc (per GPU). */
#define TILEC_MM_NOALLOC_SCRATCH_BYTES (16u << 20)

/* C = A . B with the SPLITK kernel, for callers that cannot allocate device memory.
 * No counterpart in the reference (whose op always allocates its result, tilec/ext.py:61).
 *
 * Who needs it: a host that binds only this C ABI through an FFI (cgo, JNI, N-API) and
 * owns no device allocator; a process that reserves all device memory up front and may
 * not allocate afterwards; code for which cudaMalloc/cudaFree are off limits because
 * they synchronise the whole device and would stall other streams.  The caller still
 * provides A, B and C.
 *
 * The split-K partial sums live in a fixed array of TILEC_MM_NOALLOC_SCRATCH_BYTES that
 * the library holds on every GPU it is loaded on until the process exits.  The first call
 * on a device looks up that array's device address (cudaGetSymbolAddress) with the device
 * current; make that first call before any stream capture.  Nothing is allocated and
 * nothing is freed, here or in any later call.
 *
 * split_k: number of K slices, or 0 to let the library choose (it then picks at most as
 * many as fit).  An explicit split_k is capped at 64 and then rounded to whole 16-deep
 * K blocks per slice, so the slices that run are S = cdiv(K, round_up(cdiv(K, s), 16))
 * with s = min(split_k, 64); when S > 1 and their partial sums, S * M * round_up(N, 4) * 4
 * bytes, exceed TILEC_MM_NOALLOC_SCRATCH_BYTES, the call returns TILEC_ERR_TOO_LARGE and
 * launches nothing.  Every partial sum the reduction reads is written earlier in the
 * same call, so the array needs no clearing between calls; but all calls share it, so
 * calls that may overlap on the GPU (different streams, or different host threads without
 * ordering) race: serialise them on one stream. */
TILEC_API int tilec_mm_f32_splitk_noalloc(const float* A, const float* B, float* C,
                                          int64_t M, int64_t N, int64_t K,
                                          int64_t lda, int64_t ldb, int64_t ldc,
                                          int32_t split_k, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TILEC_MM_H */
