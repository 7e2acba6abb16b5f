// tilec_mm.cu -- C ABI (include/tilec_mm.h) and host-side dispatch of the sm_100a GEMMs.
//
// Host logic of the reference op tilec/ext.py:54-63 (_matrix_mul_tiled) and its launcher
// tilec/jit.py:88-105 (_launch), minus what the Python wrapper keeps (shape errors,
// output allocation).  Differences from the reference launcher, by design:
//   * M, N, K and strides are passed by value as int64 (the reference packs them into
//     three 1-element int32 device tensors per call, jit.py:93-94, and its i32 indexing
//     overflows past 2^31 elements);
//   * the launch shape is chosen per call from the operands (variant, tile, split-K),
//     where the reference always launches 64x64 tiles (ext.py:54,62).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/tilec_mm.h"
#include "common.cuh"
#include "simt.cuh"
#include "tc_gemm.cuh"
#include "tc2_gemm.cuh"

static_assert(TILEC_DEV_STATUS_TIMEOUT == tilec::TILEC_DEV_TIMEOUT && TILEC_DEV_STATUS_TMEM == tilec::TILEC_DEV_TMEM &&
                  TILEC_DEV_STATUS_BAD_LAUNCH == tilec::TILEC_DEV_BAD_LAUNCH,
              "status bits in include/tilec_mm.h match the device enum");
static_assert(TILEC_MM_TRANS_A == tilec::kOpAMN && TILEC_MM_TRANS_B == tilec::kOpBK,
              "cfg->flags are passed to the kernels as their operand layout");

namespace tilec {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxSplit = 64;

struct DeviceInfo {
  int dev = 0;
  int sms = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
  cudaError_t init_err = cudaSuccess;
};

DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

std::mutex g_table_mu;
std::vector<int32_t> g_table;  // rows of 8 int32

template <int BN, int BK, int STAGES, bool SPLIT3, bool HI>
cudaError_t set_tc_attr() {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3>;
  return cudaFuncSetAttribute(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
}

// Stages per mode (a 3XTF32 stage holds raw + lo tiles): BN 256: 4 x 48 KB; 128: 6 x 32 KB;
// 64: 8 x 24 KB; 32: 8 x 20 KB.
#ifndef TILEC_3X_BK
#define TILEC_3X_BK 16
#endif
constexpr int k3xBK = TILEC_3X_BK;  // K per stage of the 1-CTA 3XTF32 kernel
template <int BN>
struct TcShape {
  static constexpr int kTf32Stages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int k3xStages = (BN == 256 ? 4 : (BN == 128 ? 6 : 8)) * 16 / k3xBK;
};



// CTA-pair 3XTF32 kernel (tc2_gemm_kernel): 256 x 256 tiles, stages of 32 KB, used for
// M >= TILEC_PAIR_MIN_M and N > 128 (B200: 245 vs 210 TFLOP/s for the 1-CTA kernel at 8192^3).
#ifndef TILEC_PAIR_STAGES
#define TILEC_PAIR_STAGES 6
#endif
#ifndef TILEC_PAIR_MIN_M
#define TILEC_PAIR_MIN_M 256
#endif
constexpr int kPairStages = TILEC_PAIR_STAGES;

cudaError_t init_device_attrs() {
  cudaError_t e = cudaSuccess;
  auto acc = [&](cudaError_t x) {
    if (e == cudaSuccess && x != cudaSuccess) e = x;
  };
  acc(cudaFuncSetAttribute(simt_gemm_kernel<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           simt_smem_bytes<128>()));
  acc(cudaFuncSetAttribute(simt_gemm_kernel<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           simt_smem_bytes<128>()));
  acc(cudaFuncSetAttribute(simt_gemm_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           simt_smem_bytes<64>()));
  acc(cudaFuncSetAttribute(simt_gemm_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           simt_smem_bytes<64>()));
  acc(set_tc_attr<256, 32, TcShape<256>::kTf32Stages, false, false>());
  acc(set_tc_attr<128, 32, TcShape<128>::kTf32Stages, false, false>());
  acc(set_tc_attr<64, 32, TcShape<64>::kTf32Stages, false, false>());
  acc(set_tc_attr<256, k3xBK, TcShape<256>::k3xStages, true, true>());
  acc(set_tc_attr<128, k3xBK, TcShape<128>::k3xStages, true, true>());
  acc(set_tc_attr<64, k3xBK, TcShape<64>::k3xStages, true, true>());
  acc(set_tc_attr<256, k3xBK, TcShape<256>::k3xStages, true, false>());
  acc(set_tc_attr<128, k3xBK, TcShape<128>::k3xStages, true, false>());
  acc(set_tc_attr<64, k3xBK, TcShape<64>::k3xStages, true, false>());
  acc(cudaFuncSetAttribute(tc2_gemm_kernel<256, kPairStages, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Tc2Cfg<256, kPairStages>::kSmemBytes));
  acc(cudaFuncSetAttribute(tc2_gemm_kernel<256, kPairStages, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Tc2Cfg<256, kPairStages>::kSmemBytes));
  return e;
}

int current_device(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return TILEC_ERR_NO_DEVICE;
  }
  std::call_once(g_dev_once[dev], [dev]() {
    DeviceInfo& d = g_dev[dev];
    d.dev = dev;
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess && d.cc_major != 10) e = cudaErrorNoKernelImageForDevice;
    if (e == cudaSuccess) e = init_device_attrs();
    d.init_err = e;
    cudaGetLastError();
  });
  if (g_dev[dev].init_err != cudaSuccess) return TILEC_ERR_NO_DEVICE;
  *out = &g_dev[dev];
  return TILEC_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    cudaGetLastError();
  });
  return g_encode;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

// Workspace layout (each region 256-byte aligned):
//   [packed A: M x round_up(K,4)] [packed B: K x round_up(N,4)] [split-K slabs: split x M x round_up(N,4)]
// Packed copies exist only for operands whose rows are not 16-byte aligned and only on
// the tensor-core path (TMA needs 16-byte aligned bases and row strides).
struct Plan {
  int variant = TILEC_MM_SIMT;
  int split = 1;
  int64_t k_chunk = 0;
  int bn = 128;
  size_t ws_bytes = 0;
  int64_t ldw = 0;
  int flags = 0;      // TILEC_MM_TRANS_A / TILEC_MM_TRANS_B: how A and B are stored
  bool pack_a = false, pack_b = false;    // tensor variants: aligned copy, same storage order
  bool tpose_a = false, tpose_b = false;  // SIMT variants: transposed operand -> row-major copy
  bool pair = false;  // 3XTF32 on a CTA pair (tc2_gemm_kernel, 256 x 256 tiles)
  size_t off_a = 0, off_b = 0, off_slabs = 0;
};

inline bool rows_aligned(const float* X, int64_t ld) { return aligned16(X) && (ld % 4 == 0); }

bool tensor_dims_ok(int64_t M, int64_t N, int64_t K) {
  const int64_t lim = (int64_t(1) << 31) - 256;
  return M < lim && N < lim && K < lim;
}

bool tensor_path_ok(const float* A, const float* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb) {
  return rows_aligned(A, lda) && rows_aligned(B, ldb) && tensor_dims_ok(M, N, K);
}

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int ilog2_floor(int64_t v) {
  int r = 0;
  while (v > 1) { v >>= 1; ++r; }
  return r;
}

// Built-in AUTO rules (a table installed with tilec_mm_set_table overrides them).
void choose_auto(const DeviceInfo& d, const float* A, const float* B, int64_t M, int64_t N, int64_t K,
                 int64_t lda, int64_t ldb, int* variant, int* split) {
  {
    std::lock_guard<std::mutex> lk(g_table_mu);
    if (!g_table.empty()) {
      const int lm = ilog2_floor(M), ln = ilog2_floor(N), lk2 = ilog2_floor(K);
      for (size_t r = 0; r + 8 <= g_table.size(); r += 8) {
        const int32_t* t = &g_table[r];
        if (lm >= t[0] && lm < t[1] && ln >= t[2] && ln < t[3] && lk2 >= t[4] && lk2 < t[5]) {
          int v = t[6];
          const bool tc = v == TILEC_MM_TF32 || v == TILEC_MM_3XTF32 || v == TILEC_MM_3XTF32_MASKED;
          if (tc && !tensor_dims_ok(M, N, K)) v = TILEC_MM_SIMT;
          *variant = v;
          *split = t[7];
          return;
        }
      }
    }
  }
  (void)d;
  *split = 0;
  const double flops = 2.0 * double(M) * double(N) * double(K);
  const bool aligned = tensor_path_ok(A, B, M, N, K, lda, ldb);
  // Misaligned operands are packed first (2 x (MK + KN) x 4 bytes of traffic): worth it
  // once the product is large enough for the tensor cores to win by a wide margin.
  if (tensor_dims_ok(M, N, K) && flops >= (aligned ? 1.0e8 : 5.0e8)) {
    *variant = TILEC_MM_3XTF32;
    return;
  }
  const int64_t tiles = cdiv(M, kSimtBM) * cdiv(N, N <= 64 ? 64 : 128);
  *variant = (tiles < d.sms && K >= 1024) ? TILEC_MM_SPLITK : TILEC_MM_SIMT;
}

// K slices for a grid of `tiles` output tiles: minimise (waves of CTAs) / slices, i.e. the
// time of one full-K tile divided across slices, plus the reduction's traffic (each slice
// writes and the reduction reads an M x N slab) and a fixed cost for its extra launch.
// flops_per_sm: sustained useful FLOP/s of one SM on this kernel.
// K-split count for a grid of `ctas` CTAs per K slice on `sms` SMs, each CTA needing
// `cta_s` seconds for the full K on an SM of its own and writing `slab_bytes` per extra
// slice.  Cost of s slices: waves(s) * cta_s / s (CTAs sharing an SM run one after the
// other) + s * slab_bytes / 3 TB/s (slab written by the GEMM and read back by the
// reduction) + 1.5 us (the reduction kernel).  Measured on B200 over 20 shapes, the
// tcgen05 kernels lose 1.2-1.7x whenever a split spills into a second wave (their
// per-wave set-up, pipeline fill and epilogue are long), so for them (`one_wave`) only
// one-wave counts are considered; the SIMT kernel's second wave costs only its share of
// the work.  `smax` bounds the count (at least four K-blocks per slice).
int choose_split(int64_t ctas, int64_t sms, double cta_s, double slab_bytes, int64_t smax, int requested,
                 bool one_wave) {
  if (requested > 0) return requested > kMaxSplit ? kMaxSplit : requested;
  if (ctas >= sms || ctas <= 0) return 1;
  if (smax > kMaxSplit) smax = kMaxSplit;
  int64_t top = one_wave ? sms / ctas : smax;
  if (top > smax) top = smax;
  int best = 1;
  double best_cost = cta_s;
  for (int64_t sp = 2; sp <= top; ++sp) {
    const double waves = double(cdiv(ctas * sp, sms));
    const double cost = waves * cta_s / double(sp) + double(sp) * slab_bytes / 3.0e12 + 1.5e-6;
    if (cost < best_cost) {
      best_cost = cost;
      best = static_cast<int>(sp);
    }
  }
  return best;
}

// Per-CTA time for the full K: the larger of its arithmetic (at `flops` per CTA) and its
// operand streaming (at `bw` bytes/s per CTA).
double cta_seconds(int64_t rows, int64_t cols, int64_t b_cols, int64_t K, double flops, double bw) {
  const double compute = 2.0 * double(rows) * double(cols) * double(K) / flops;
  const double stream = double(rows + b_cols) * double(K) * 4.0 / bw;
  return compute > stream ? compute : stream;
}

// Measured per-SM rates on B200: 3xTF32 ~1.7 TFLOP/s (250 TFLOP/s / 148), TF32 ~4.3, SIMT
// FMA ~0.31; HBM share ~38 GB/s per SM with every SM streaming.
constexpr double kRate3x = 1.7e12, kRateTf32 = 4.3e12, kRateSimt = 0.31e12, kBwPerSm = 38.0e9;

int make_plan(const DeviceInfo& d, const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K,
              int64_t lda, int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg, Plan* p) {
  (void)C;
  (void)ldc;
  int variant = cfg ? cfg->variant : TILEC_MM_AUTO;
  int requested_split = cfg ? cfg->split_k : 0;
  const int flags = cfg ? cfg->flags : 0;
  if (flags & ~(TILEC_MM_TRANS_A | TILEC_MM_TRANS_B)) return TILEC_ERR_BAD_ARG;
  if (cfg) {
    for (int i = 0; i < 5; ++i)
      if (cfg->reserved[i] != 0) return TILEC_ERR_BAD_ARG;
  }
  p->flags = flags;
  if (requested_split < 0) return TILEC_ERR_BAD_ARG;
  if (variant == TILEC_MM_AUTO) choose_auto(d, A, B, M, N, K, lda, ldb, &variant, &requested_split);
  if (variant < TILEC_MM_SIMT || variant > TILEC_MM_3XTF32_MASKED) return TILEC_ERR_BAD_ARG;
  const bool tensor = variant == TILEC_MM_TF32 || variant == TILEC_MM_3XTF32 || variant == TILEC_MM_3XTF32_MASKED;
  if (tensor && !tensor_dims_ok(M, N, K)) return TILEC_ERR_UNSUPPORTED;
  if (tensor) {
    p->pack_a = !rows_aligned(A, lda);
    p->pack_b = !rows_aligned(B, ldb);
  } else {
    p->tpose_a = (flags & TILEC_MM_TRANS_A) != 0;
    p->tpose_b = (flags & TILEC_MM_TRANS_B) != 0;
  }

  p->variant = variant;
  if (tensor) {
    p->bn = N <= 64 ? 64 : (N <= 128 ? 128 : 256);
    p->pair = variant != TILEC_MM_TF32 && p->bn == 256 && M > 128 && M >= TILEC_PAIR_MIN_M;
    const int bk = variant == TILEC_MM_TF32 ? 32 : (p->pair ? 16 : k3xBK);
    const int64_t tiles = cdiv(M, kTcBM) * cdiv(N, p->bn);
    // The CTA pair launches two CTAs per 256-row x 256-column tile; each computes 128 rows
    // and loads half of the B columns.
    const int64_t ctas = p->pair ? 2 * cdiv(M, 256) * cdiv(N, 256) : tiles;
    const double cta_s = cta_seconds(kTcBM, p->bn, p->pair ? p->bn / 2 : p->bn, K,
                                     variant == TILEC_MM_TF32 ? kRateTf32 : kRate3x, kBwPerSm);
    p->split = choose_split(ctas, d.sms, cta_s, double(M) * double(round_up(N, 4)) * 4.0, K / (int64_t(bk) * 4),
                            requested_split, /*one_wave=*/true);
    p->k_chunk = round_up(cdiv(K, p->split), bk);
    p->split = static_cast<int>(cdiv(K, p->k_chunk > 0 ? p->k_chunk : 1));
    if (p->split < 1) p->split = 1;
  } else {
    p->bn = N <= 64 ? 64 : 128;
    const int64_t tiles = cdiv(M, kSimtBM) * cdiv(N, p->bn);
    int split = 1;
    if (variant == TILEC_MM_SPLITK) {
      const double cta_s = cta_seconds(kSimtBM, p->bn, p->bn, K, kRateSimt, kBwPerSm);
      split = choose_split(tiles, d.sms, cta_s, double(M) * double(round_up(N, 4)) * 4.0, K / (int64_t(kSimtBK) * 4),
                           requested_split, /*one_wave=*/false);
    }
    p->k_chunk = round_up(cdiv(K, split), kSimtBK);
    split = static_cast<int>(cdiv(K, p->k_chunk > 0 ? p->k_chunk : 1));
    p->split = split < 1 ? 1 : split;
  }
  if (p->k_chunk <= 0) p->k_chunk = 16;
  p->ldw = round_up(N, 4);
  // An aligned copy keeps the stored order (K x M for a transposed A); a SIMT transpose
  // writes the row-major M x K (K x N) operand.
  const bool ta = (flags & TILEC_MM_TRANS_A) != 0, tb = (flags & TILEC_MM_TRANS_B) != 0;
  size_t off = 0;
  if (p->pack_a || p->tpose_a) {
    p->off_a = off;
    const size_t elems = (p->pack_a && ta) ? size_t(K) * size_t(round_up(M, 4)) : size_t(M) * size_t(round_up(K, 4));
    off += align256(elems * sizeof(float));
  }
  if (p->pack_b || p->tpose_b) {
    p->off_b = off;
    const size_t elems = (p->pack_b && tb) ? size_t(N) * size_t(round_up(K, 4)) : size_t(K) * size_t(round_up(N, 4));
    off += align256(elems * sizeof(float));
  }
  p->off_slabs = off;
  if (p->split > 1) off += size_t(p->split) * size_t(M) * size_t(p->ldw) * sizeof(float);
  p->ws_bytes = off;
  return TILEC_OK;
}

// need_c: tilec_mm_f32 writes C; tilec_mm_plan / tilec_mm_workspace_bytes accept C == NULL.
int check_args(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
               int64_t ldb, int64_t ldc, bool need_c = true, int flags = 0) {
  if (M < 0 || N < 0 || K < 0) return TILEC_ERR_BAD_ARG;
  if (M == 0 || N == 0) return TILEC_OK;
  if ((need_c && C == nullptr) || ldc < N) return TILEC_ERR_BAD_ARG;
  const int64_t min_lda = (flags & TILEC_MM_TRANS_A) ? M : K;
  const int64_t min_ldb = (flags & TILEC_MM_TRANS_B) ? K : N;
  if (K > 0 && (A == nullptr || B == nullptr || lda < min_lda || ldb < min_ldb)) return TILEC_ERR_BAD_ARG;
  return TILEC_OK;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TILEC_OK : TILEC_ERR_LAUNCH;
}

// Tensor maps for the operand tiles (`layout`: kOpAMN / kOpBK, see common.cuh).  A K-major:
// box {bk, 128} with a bk*4-byte swizzle; A MN-major (stored K x M): boxes {32, bk} with
// the 128-byte / 32-byte-granule swizzle.  B MN-major: boxes {32, bk}, same swizzle; B
// K-major (stored N x K): box {bk, b_rows}, bk*4-byte swizzle.
int encode_maps(const float* A, const float* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                int bk, int layout, int b_rows, CUtensorMap* ma, CUtensorMap* mb) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode();
  if (!enc) return TILEC_ERR_NO_DEVICE;
  const CUtensorMapSwizzle k_sw = bk * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  auto encode = [&](CUtensorMap* m, const float* base, int64_t inner, int64_t outer, int64_t ld, int box_in,
                    int box_out, CUtensorMapSwizzle sw) {
    cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
    cuuint32_t box[2] = {cuuint32_t(box_in), cuuint32_t(box_out)};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  const bool ok_a = (layout & kOpAMN) ? encode(ma, A, M, K, lda, 32, bk, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                                      : encode(ma, A, K, M, lda, bk, kTcBM, k_sw);
  const bool ok_b = (layout & kOpBK) ? encode(mb, B, K, N, ldb, bk, b_rows, k_sw)
                                     : encode(mb, B, N, K, ldb, 32, bk, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  return ok_a && ok_b ? TILEC_OK : TILEC_ERR_BAD_ARG;
}

// Programmatic dependent launch is on unless TILEC_MM_PDL=0 (read once per process).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TILEC_MM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Launches `kern`, with programmatic stream serialisation when `pdl` (every kernel here
// calls pdl_wait() before touching global memory) and, when cluster_x > 1, a cluster of
// cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
int launch_kx(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_x,
              Args... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl && pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  lc.attrs = attr;
  lc.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return TILEC_ERR_LAUNCH;
  }
  return launch_status();
}

template <typename... KArgs, typename... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_x,
             Args... args) {
  return launch_kx(true, kern, grid, block, smem, s, cluster_x, args...);
}

template <int BN, int BK, int STAGES, bool SPLIT3, bool HI>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, float* out, int64_t M, int64_t N, int64_t ldo,
              int64_t slab, int64_t K, int64_t k_chunk, int split, int vec_out, int layout, cudaStream_t s) {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3>;
  const int m_tiles = static_cast<int>(cdiv(M, kTcBM));
  const int n_tiles = static_cast<int>(cdiv(N, BN));
  const int group_m = 16;
  dim3 grid(static_cast<unsigned>(int64_t(m_tiles) * n_tiles), 1, static_cast<unsigned>(split));
  return launch_k(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI>, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, s, 1, ma,
                  mb, out, static_cast<int>(M), static_cast<int>(N), ldo, slab, static_cast<int>(K),
                  static_cast<int>(k_chunk), m_tiles, n_tiles, group_m, vec_out, layout);
}

template <int BN, bool SPLIT3, bool HI>
int launch_tc_mode(const CUtensorMap& ma, const CUtensorMap& mb, float* out, int64_t M, int64_t N, int64_t ldo,
                   int64_t slab, int64_t K, int64_t k_chunk, int split, int vec_out, int layout, cudaStream_t s) {
  if constexpr (SPLIT3)
    return launch_tc<BN, k3xBK, TcShape<BN>::k3xStages, true, HI>(ma, mb, out, M, N, ldo, slab, K, k_chunk, split,
                                                                  vec_out, layout, s);
  else
    return launch_tc<BN, 32, TcShape<BN>::kTf32Stages, false, false>(ma, mb, out, M, N, ldo, slab, K, k_chunk,
                                                                     split, vec_out, layout, s);
}

template <bool HI>
int launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, float* out, int64_t M, int64_t N, int64_t ldo,
               int64_t slab, int64_t K, int64_t k_chunk, int split, int vec_out, int layout, cudaStream_t s) {
  using Cfg = Tc2Cfg<256, kPairStages>;
  const int mp_tiles = static_cast<int>(cdiv(M, 256));
  const int n_tiles = static_cast<int>(cdiv(N, 256));
  const int group_m = 8;
  const dim3 grid(static_cast<unsigned>(2 * int64_t(mp_tiles) * n_tiles), 1, static_cast<unsigned>(split));
  return launch_k(tc2_gemm_kernel<256, kPairStages, HI>, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, s, 2, ma, mb,
                  out, static_cast<int>(M), static_cast<int>(N), ldo, slab, static_cast<int>(K),
                  static_cast<int>(k_chunk), mp_tiles, n_tiles, group_m, vec_out, layout);
}

template <bool SPLIT3, bool HI>
int dispatch_tc_bn(int bn, const CUtensorMap& ma, const CUtensorMap& mb, float* out, int64_t M, int64_t N,
                   int64_t ldo, int64_t slab, int64_t K, int64_t k_chunk, int split, int vec_out, int layout, cudaStream_t s) {
  switch (bn) {
    case 64: return launch_tc_mode<64, SPLIT3, HI>(ma, mb, out, M, N, ldo, slab, K, k_chunk, split, vec_out, layout, s);
    case 128: return launch_tc_mode<128, SPLIT3, HI>(ma, mb, out, M, N, ldo, slab, K, k_chunk, split, vec_out, layout, s);
    default: return launch_tc_mode<256, SPLIT3, HI>(ma, mb, out, M, N, ldo, slab, K, k_chunk, split, vec_out, layout, s);
  }
}

// dst[r, 0:cols] = src[r, 0:cols] with row strides lds / ldd (one CTA per row, grid-stride).
__global__ void __launch_bounds__(256) pack_rows_kernel(const float* __restrict__ src, int64_t lds,
                                                        float* __restrict__ dst, int64_t ldd, int64_t rows,
                                                        int64_t cols) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* s = src + r * lds;
    float* d = dst + r * ldd;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) d[c] = s[c];
  }
}

// dst[c, r] = src[r, c] for r < rows, c < cols: 32 x 32 tiles through shared memory (the
// +1 column keeps the transposed reads free of bank conflicts), coalesced on both sides.
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ src, int64_t lds,
                                                        float* __restrict__ dst, int64_t ldd, int64_t rows,
                                                        int64_t cols) {
  __shared__ float t[32][33];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t tr = (rows + 31) / 32, tc = (cols + 31) / 32;
  const int tx = static_cast<int>(threadIdx.x) & 31, ty = static_cast<int>(threadIdx.x) >> 5;  // 32 x 8
  for (int64_t tile = blockIdx.x; tile < tr * tc; tile += gridDim.x) {
    const int64_t r0 = (tile / tc) * 32, c0 = (tile % tc) * 32;
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, c = c0 + tx;
      if (r < rows && c < cols) t[i][tx] = src[r * lds + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int64_t c = c0 + i, r = r0 + tx;
      if (r < rows && c < cols) dst[c * ldd + r] = t[tx][i];
    }
    __syncthreads();
  }
}

int launch_transpose(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows, int64_t cols,
                     const DeviceInfo& d, cudaStream_t s) {
  int64_t blocks = cdiv(rows, 32) * cdiv(cols, 32);
  if (blocks > int64_t(d.sms) * 8) blocks = int64_t(d.sms) * 8;
  if (blocks < 1) blocks = 1;
  return launch_k(transpose_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, 1, src, lds, dst, ldd, rows,
                  cols);
}

int launch_pack(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows, int64_t cols,
                const DeviceInfo& d, cudaStream_t s) {
  int64_t blocks = rows < int64_t(d.sms) * 16 ? rows : int64_t(d.sms) * 16;
  if (blocks < 1) blocks = 1;
  return launch_k(pack_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, 1, src, lds, dst, ldd, rows,
                  cols);
}

template <int P>
int launch_reduce_p(int U, dim3 grid, const float* ws, float* C, int64_t M, int64_t N, int64_t ldw, int64_t ldc,
                    int64_t slab, int split, int vec_out, cudaStream_t s) {
  switch (U) {
    case 4: return launch_k(splitk_reduce_kernel<P, 4>, grid, dim3(256), 0, s, 1, ws, C, M, N, ldw, ldc, slab, split, vec_out);
    case 2: return launch_k(splitk_reduce_kernel<P, 2>, grid, dim3(256), 0, s, 1, ws, C, M, N, ldw, ldc, slab, split, vec_out);
    default: return launch_k(splitk_reduce_kernel<P, 1>, grid, dim3(256), 0, s, 1, ws, C, M, N, ldw, ldc, slab, split, vec_out);
  }
}

int launch_reduce(const float* ws, float* C, int64_t M, int64_t N, int64_t ldw, int64_t ldc, int split,
                  const DeviceInfo& d, cudaStream_t s) {
  const int P = split >= 8 ? 8 : (split >= 4 ? 4 : (split >= 2 ? 2 : 1));
  const int64_t G = 256 / P;
  const int64_t groups = M * cdiv(N, 4);
  const int64_t resident = int64_t(d.sms) * 8;  // 256-thread blocks resident at once
  const int U = groups <= resident * G ? 1 : (groups <= 2 * resident * G ? 2 : 4);
  int64_t blocks = cdiv(groups, G * U);
  if (blocks > resident) blocks = resident;
  if (blocks < 1) blocks = 1;
  const int vec_out = aligned16(C) && (ldc % 4 == 0);
  const dim3 grid(static_cast<unsigned>(blocks));
  const int64_t slab = M * ldw;
  switch (P) {
    case 8: return launch_reduce_p<8>(U, grid, ws, C, M, N, ldw, ldc, slab, split, vec_out, s);
    case 4: return launch_reduce_p<4>(U, grid, ws, C, M, N, ldw, ldc, slab, split, vec_out, s);
    case 2: return launch_reduce_p<2>(U, grid, ws, C, M, N, ldw, ldc, slab, split, vec_out, s);
    default: return launch_reduce_p<1>(U, grid, ws, C, M, N, ldw, ldc, slab, split, vec_out, s);
  }
}

// One warp waits, through mbar_wait, for phase 0 of a barrier nothing arrives on; the wait
// must give up after limit_ns and record TILEC_DEV_TIMEOUT (tilec_mm_selftest_wait).
__global__ void __launch_bounds__(32) selftest_wait_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  pdl_wait();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, limit_ns);
  __syncwarp();
}

int launch_fill_zero(float* C, int64_t M, int64_t N, int64_t ldc, const DeviceInfo& d, cudaStream_t s) {
  int64_t blocks = cdiv(M * N, 256);
  if (blocks > int64_t(d.sms) * 8) blocks = int64_t(d.sms) * 8;
  return launch_k(fill_zero_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, 1, C, M, N, ldc);
}

int launch_simt(int bn, bool vec, dim3 grid, const float* A, const float* B, float* out, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldo, int64_t slab, int64_t k_chunk, int vec_out,
                cudaStream_t s) {
  // Launched without programmatic serialisation: a SIMT CTA fits twice on an SM, and CTAs
  // placed while the previous kernel still occupies the GPU were measured to double up on
  // some SMs (a 128-CTA grid ran 40% slower).
  const dim3 block(kSimtThreads);
  auto go = [&](auto kern, size_t smem) {
    return launch_kx(false, kern, grid, block, smem, s, 1, A, B, out, M, N, K, lda, ldb, ldo, slab, k_chunk,
                     vec_out);
  };
  if (bn == 64)
    return vec ? go(simt_gemm_kernel<64, true>, simt_smem_bytes<64>())
               : go(simt_gemm_kernel<64, false>, simt_smem_bytes<64>());
  return vec ? go(simt_gemm_kernel<128, true>, simt_smem_bytes<128>())
             : go(simt_gemm_kernel<128, false>, simt_smem_bytes<128>());
}

}  // namespace
}  // namespace tilec

using namespace tilec;

extern "C" {

int tilec_mm_plan(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                  int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg, tilec_mm_cfg* out) {
  if (!out) return TILEC_ERR_BAD_ARG;
  int rc = check_args(A, B, C, M, N, K, lda, ldb, ldc, /*need_c=*/false, cfg ? cfg->flags : 0);
  if (rc) return rc;
  DeviceInfo* d = nullptr;
  rc = current_device(&d);
  if (rc) return rc;
  Plan p;
  rc = make_plan(*d, A, B, C, M, N, K, lda, ldb, ldc, cfg, &p);
  if (rc) return rc;
  std::memset(out, 0, sizeof(*out));
  out->variant = p.variant;
  out->split_k = p.split;
  out->flags = p.flags;
  return TILEC_OK;
}

size_t tilec_mm_workspace_bytes(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K,
                                int64_t lda, int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  DeviceInfo* d = nullptr;
  if (current_device(&d)) return 0;
  // NULL operands: assume 16-byte aligned pointers (documented in the header).
  const float* a = A ? A : reinterpret_cast<const float*>(uintptr_t(256));
  const float* b = B ? B : reinterpret_cast<const float*>(uintptr_t(256));
  Plan p;
  if (make_plan(*d, a, b, C, M, N, K, lda, ldb, ldc, cfg, &p)) return 0;
  return p.ws_bytes;
}

int tilec_mm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                 int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg, void* workspace, size_t ws_bytes,
                 void* stream) {
  int rc = check_args(A, B, C, M, N, K, lda, ldb, ldc, true, cfg ? cfg->flags : 0);
  if (rc) return rc;
  if (M == 0 || N == 0) return TILEC_OK;
  DeviceInfo* d = nullptr;
  rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  if (K == 0) return launch_fill_zero(C, M, N, ldc, *d, s);

  Plan p;
  rc = make_plan(*d, A, B, C, M, N, K, lda, ldb, ldc, cfg, &p);
  if (rc) return rc;
  if (p.ws_bytes > 0) {
    if (!workspace || ws_bytes < p.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
      return TILEC_ERR_WORKSPACE;
  }
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  const bool ta = (p.flags & TILEC_MM_TRANS_A) != 0, tb = (p.flags & TILEC_MM_TRANS_B) != 0;
  // Stored shapes: A is M x K (K x M when transposed), B is K x N (N x K when transposed).
  const int64_t a_rows = ta ? K : M, a_cols = ta ? M : K;
  const int64_t b_rows = tb ? N : K, b_cols = tb ? K : N;
  if (p.pack_a || p.tpose_a) {
    float* pa = reinterpret_cast<float*>(wsb + p.off_a);
    if (p.pack_a) {
      rc = launch_pack(A, lda, pa, round_up(a_cols, 4), a_rows, a_cols, *d, s);
      lda = round_up(a_cols, 4);
    } else {
      rc = launch_transpose(A, lda, pa, round_up(K, 4), K, M, *d, s);
      lda = round_up(K, 4);
    }
    if (rc) return rc;
    A = pa;
  }
  if (p.pack_b || p.tpose_b) {
    float* pb = reinterpret_cast<float*>(wsb + p.off_b);
    if (p.pack_b) {
      rc = launch_pack(B, ldb, pb, round_up(b_cols, 4), b_rows, b_cols, *d, s);
      ldb = round_up(b_cols, 4);
    } else {
      rc = launch_transpose(B, ldb, pb, round_up(N, 4), N, K, *d, s);
      ldb = round_up(N, 4);
    }
    if (rc) return rc;
    B = pb;
  }
  // The tensor-core kernels read either storage order in place; SIMT operands are now
  // row-major.
  const bool simt = p.variant == TILEC_MM_SIMT || p.variant == TILEC_MM_SPLITK;
  const int layout = simt ? 0 : p.flags;
  float* slabs = reinterpret_cast<float*>(wsb + p.off_slabs);
  float* out = p.split > 1 ? slabs : C;
  const int64_t ldo = p.split > 1 ? p.ldw : ldc;
  const int64_t slab = p.split > 1 ? M * p.ldw : 0;
  const int vec_out = p.split > 1 ? 1 : (aligned16(C) && (ldc % 4 == 0) ? 1 : 0);

  if (simt) {
    const bool vec = aligned16(A) && aligned16(B) && (lda % 4 == 0) && (ldb % 4 == 0);
    const int64_t mt = cdiv(M, kSimtBM), nt = cdiv(N, p.bn);
    if (nt > 65535) return TILEC_ERR_UNSUPPORTED;
    dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt), static_cast<unsigned>(p.split));
    rc = launch_simt(p.bn, vec, grid, A, B, out, M, N, K, lda, ldb, ldo, slab, p.k_chunk, vec_out, s);
  } else {
    CUtensorMap ma, mb;
    const int bk = p.variant == TILEC_MM_TF32 ? 32 : (p.pair ? 16 : k3xBK);
    rc = encode_maps(A, B, M, N, K, lda, ldb, bk, layout, p.pair ? 128 : p.bn, &ma, &mb);
    if (rc) return rc;
    if (p.pair)
      rc = p.variant == TILEC_MM_3XTF32
               ? launch_tc2<false>(ma, mb, out, M, N, ldo, slab, K, p.k_chunk, p.split, vec_out, layout, s)
               : launch_tc2<true>(ma, mb, out, M, N, ldo, slab, K, p.k_chunk, p.split, vec_out, layout, s);
    else if (p.variant == TILEC_MM_TF32)
      rc = dispatch_tc_bn<false, false>(p.bn, ma, mb, out, M, N, ldo, slab, K, p.k_chunk, p.split, vec_out, layout,
                                        s);
    else if (p.variant == TILEC_MM_3XTF32)
      rc = dispatch_tc_bn<true, false>(p.bn, ma, mb, out, M, N, ldo, slab, K, p.k_chunk, p.split, vec_out, layout,
                                       s);
    else
      rc = dispatch_tc_bn<true, true>(p.bn, ma, mb, out, M, N, ldo, slab, K, p.k_chunk, p.split, vec_out, layout, s);
  }
  if (rc) return rc;
  if (p.split > 1) rc = launch_reduce(slabs, C, M, N, p.ldw, ldc, p.split, *d, s);
  return rc;
}

int tilec_mm_set_table(const int32_t* rows, int32_t nrows) {
  if (nrows < 0 || (nrows > 0 && rows == nullptr)) return TILEC_ERR_BAD_ARG;
  for (int32_t r = 0; r < nrows; ++r) {
    const int32_t v = rows[r * 8 + 6];
    if (v < TILEC_MM_SIMT || v > TILEC_MM_3XTF32_MASKED || rows[r * 8 + 7] < 0) return TILEC_ERR_BAD_ARG;
  }
  std::lock_guard<std::mutex> lk(g_table_mu);
  g_table.assign(rows, rows + size_t(nrows) * 8);
  return TILEC_OK;
}

int tilec_mm_selftest_wait(int64_t limit_ns, void* stream) {
  DeviceInfo* d = nullptr;
  const int rc = current_device(&d);
  if (rc) return rc;
  unsigned long long lim = limit_ns < 1000000 ? 1000000ull : static_cast<unsigned long long>(limit_ns);
  if (lim > kWaitLimitNs) lim = kWaitLimitNs;
  return launch_k(selftest_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1, lim);
}

int tilec_mm_device_status(void* stream, int32_t* status_out) {
  if (!status_out) return TILEC_ERR_BAD_ARG;
  DeviceInfo* d = nullptr;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return TILEC_ERR_DEVICE;
  }
  *status_out = v;
  return TILEC_OK;
}

const char* tilec_strerror(int code) {
  switch (code) {
    case TILEC_OK: return "ok";
    case TILEC_ERR_BAD_ARG: return "bad argument (negative size, null pointer, or leading dimension too small)";
    case TILEC_ERR_MISALIGNED: return "tensor-core variant needs 16-byte aligned operands and row strides";
    case TILEC_ERR_NO_DEVICE: return "no usable sm_100 CUDA device";
    case TILEC_ERR_LAUNCH: return "kernel launch failed";
    case TILEC_ERR_DEVICE: return "device-side check failed";
    case TILEC_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case TILEC_ERR_UNSUPPORTED: return "unsupported size for this variant";
    case TILEC_ERR_TOO_LARGE: return "request exceeds the entry point's fixed limit";
    default: return "unknown tilec status";
  }
}

int tilec_mm_abi_version(void) { return TILEC_MM_ABI_VERSION; }
int tilec_mm_built_arch(void) { return 100; }

}  // extern "C"

// ------------------------------------------------------------------ allocation-free split-K
// Scratch for tilec_mm_f32_splitk_noalloc: split-K partial-sum slabs, shared by every call
// on a device.  Host code must not pass the symbol itself to a kernel (on the host it
// names a host-side stand-in); the device address is looked up once per device below.
namespace {
static __device__ __align__(256) float g_noalloc_scratch[TILEC_MM_NOALLOC_SCRATCH_BYTES / sizeof(float)];

std::once_flag g_noalloc_once[kMaxDevices];
float* g_noalloc_ptr[kMaxDevices];
cudaError_t g_noalloc_err[kMaxDevices];

// Device address of g_noalloc_scratch on the current device (set up on first use).
int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return TILEC_ERR_NO_DEVICE;
  }
  std::call_once(g_noalloc_once[dev], [dev]() {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc_err[dev] = e;
    g_noalloc_ptr[dev] = e == cudaSuccess ? static_cast<float*>(p) : nullptr;
    if (e != cudaSuccess) cudaGetLastError();
  });
  if (g_noalloc_err[dev] != cudaSuccess || g_noalloc_ptr[dev] == nullptr) return TILEC_ERR_DEVICE;
  *out = g_noalloc_ptr[dev];
  return TILEC_OK;
}
}  // namespace

extern "C" int tilec_mm_f32_splitk_noalloc(const float* A, const float* B, float* C, int64_t M, int64_t N,
                                           int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int32_t split_k,
                                           void* stream) {
  int rc = check_args(A, B, C, M, N, K, lda, ldb, ldc);
  if (rc) return rc;
  if (split_k < 0) return TILEC_ERR_BAD_ARG;
  if (M == 0 || N == 0) return TILEC_OK;
  DeviceInfo* d = nullptr;
  rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) return launch_fill_zero(C, M, N, ldc, *d, s);
  float* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;

  const int bn = N <= 64 ? 64 : 128;
  const int64_t mt = cdiv(M, kSimtBM), nt = cdiv(N, bn);
  if (nt > 65535) return TILEC_ERR_UNSUPPORTED;
  const int64_t ldw = round_up(N, 4);
  const int64_t slab = M * ldw;
  const int64_t fit = static_cast<int64_t>(TILEC_MM_NOALLOC_SCRATCH_BYTES / sizeof(float)) / slab;
  int64_t split;
  if (split_k > 0) {
    split = split_k > kMaxSplit ? kMaxSplit : split_k;
    if (split > 1 && split > fit) return TILEC_ERR_TOO_LARGE;
  } else {
    const double cta_s = cta_seconds(kSimtBM, bn, bn, K, kRateSimt, kBwPerSm);
    split = choose_split(mt * nt, d->sms, cta_s, double(slab) * 4.0, K / (int64_t(kSimtBK) * 4), 0,
                         /*one_wave=*/false);
    if (split > fit) split = fit < 1 ? 1 : fit;
  }
  const int64_t k_chunk = round_up(cdiv(K, split), kSimtBK);
  split = cdiv(K, k_chunk);

  float* out = split > 1 ? scratch : C;
  const int64_t ldo = split > 1 ? ldw : ldc;
  const int64_t out_slab = split > 1 ? slab : 0;
  const int vec_out = split > 1 ? 1 : (aligned16(C) && (ldc % 4 == 0) ? 1 : 0);
  const bool vec = aligned16(A) && aligned16(B) && (lda % 4 == 0) && (ldb % 4 == 0);
  dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt), static_cast<unsigned>(split));
  rc = launch_simt(bn, vec, grid, A, B, out, M, N, K, lda, ldb, ldo, out_slab, k_chunk, vec_out, s);
  if (rc || split == 1) return rc;
  return launch_reduce(scratch, C, M, N, ldw, ldc, static_cast<int>(split), *d, s);
}
