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
#include "tc2_sk.cuh"
#include "tc2_tf32p.cuh"

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
  int pair_slots = 0;  // CTA pairs of the stream-K pair kernel resident at once (0: stream-K off)
  int tf32p_slots = 0; // CTA pairs of the persistent TF32 pair kernel resident at once (0: not used)
  cudaError_t init_err = cudaSuccess;
};

DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

std::mutex g_table_mu;
std::vector<int32_t> g_table;  // rows of 8 int32

template <int BN, int BK, int STAGES, bool SPLIT3, bool HI, int BM = kTcBM>
cudaError_t set_tc_attr() {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3, BM>;
  const cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI, false, BM>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI, true, BM>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
}

// Stages per mode (a 3XTF32 stage holds raw + lo tiles): BN 256: 4 x 48 KB; 128: 6 x 32 KB;
// 64: 8 x 24 KB.  K per stage of the 1-CTA 3XTF32 kernel: 16.  32 was measured twice: first
// no faster and with twice the error (promotion every 256 of K), then, promoting every 128
// of K, from 6 % faster (256x16384x64) to 16 % slower (200x4096x4096), config 1 1.5 % slower.
// (The CTA-pair kernel does take 32: see kPair3xStages.)
constexpr int k3xBK = 16;
template <int BN>
struct TcShape {
  static constexpr int kTf32Stages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int k3xStages = (BN == 256 ? 4 : (BN == 128 ? 6 : 8)) * 16 / k3xBK;
};
// 64-row tiles (16 / 24 / 40 KB stages at BN 64 / 128 / 256 in both modes).  Where the
// registers allow two CTAs per SM (4 epilogue warps: TF32 at BN <= 128, 3XTF32 at BN 64)
// the stages stop at 96 KB so that two CTAs fit; otherwise (one CTA per SM) 3XTF32 takes 8
// stages at BN 128 and both modes 4 at BN 256.
template <int BN>
struct TcShape64 {
  static constexpr int kTf32Stages = BN == 256 ? 4 : (BN == 128 ? 4 : 6);
  static constexpr int k3xStages = BN == 256 ? 4 : (BN == 128 ? 8 : 6);
};
constexpr int kTcBM64 = 64;



// CTA-pair kernels (tc2_gemm_kernel, tc2_sk_kernel): 256 x 256 tiles (256 x 128 for
// 256 < N <= 384), used for M >= kPairMinM and N > 128 (B200: 245 vs 210 TFLOP/s for the
// 1-CTA kernel at 8192^3).
// TF32: 6 stages of 32 KB (4 were measured slower).
constexpr int kPairStages = 6;
// 3XTF32 (both forms) and the mixed split: 3 stages of K = 32 (64 KB each), the same depth
// in K as 6 stages of 16 with half the per-stage barrier handshakes and commits.
constexpr int kPair3xStages = 3;
constexpr int64_t kPairMinM = 256;

cudaError_t init_device_attrs() {
  cudaError_t e = cudaSuccess;
  auto acc = [&](cudaError_t x) {
    if (e == cudaSuccess && x != cudaSuccess) e = x;
  };
  // Up to kSimtSpreadSmem: small grids ask for that much to keep to one CTA per SM.
  auto simt_attr = [&](auto kern) {
    acc(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSimtSpreadSmem));
  };
  simt_attr(simt_gemm_kernel<128, kBScalar>);
  simt_attr(simt_gemm_kernel<128, kBVec>);
  simt_attr(simt_gemm_kernel<128, kBTma>);
  simt_attr(simt_gemm_kernel<64, kBScalar>);
  simt_attr(simt_gemm_kernel<64, kBVec>);
  simt_attr(simt_gemm_kernel<64, kBTma>);
  acc(set_tc_attr<256, 32, TcShape<256>::kTf32Stages, false, false>());
  acc(set_tc_attr<128, 32, TcShape<128>::kTf32Stages, false, false>());
  acc(set_tc_attr<64, 32, TcShape<64>::kTf32Stages, false, false>());
  acc(set_tc_attr<256, k3xBK, TcShape<256>::k3xStages, true, true>());
  acc(set_tc_attr<128, k3xBK, TcShape<128>::k3xStages, true, true>());
  acc(set_tc_attr<64, k3xBK, TcShape<64>::k3xStages, true, true>());
  acc(set_tc_attr<256, k3xBK, TcShape<256>::k3xStages, true, false>());
  acc(set_tc_attr<128, k3xBK, TcShape<128>::k3xStages, true, false>());
  acc(set_tc_attr<64, k3xBK, TcShape<64>::k3xStages, true, false>());
  acc(set_tc_attr<256, 32, TcShape64<256>::kTf32Stages, false, false, kTcBM64>());
  acc(set_tc_attr<128, 32, TcShape64<128>::kTf32Stages, false, false, kTcBM64>());
  acc(set_tc_attr<64, 32, TcShape64<64>::kTf32Stages, false, false, kTcBM64>());
  acc(set_tc_attr<256, k3xBK, TcShape64<256>::k3xStages, true, true, kTcBM64>());
  acc(set_tc_attr<128, k3xBK, TcShape64<128>::k3xStages, true, true, kTcBM64>());
  acc(set_tc_attr<64, k3xBK, TcShape64<64>::k3xStages, true, true, kTcBM64>());
  acc(set_tc_attr<256, k3xBK, TcShape64<256>::k3xStages, true, false, kTcBM64>());
  acc(set_tc_attr<128, k3xBK, TcShape64<128>::k3xStages, true, false, kTcBM64>());
  acc(set_tc_attr<64, k3xBK, TcShape64<64>::k3xStages, true, false, kTcBM64>());
  auto pair_attr = [&](auto kern, int smem) {
    acc(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  };
  // Every (mode, layout) instantiation of both pair kernels that the launch paths use.
  constexpr int k3x = Tc2Cfg<256, kPair3xStages, true, false, 32>::kSmemBytes;
  constexpr int kMix = Tc2Cfg<256, kPair3xStages, true, false, 32>::kSmemBytes;
  constexpr int kTf = Tc2Cfg<256, kPairStages, false>::kSmemBytes;
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, false, false>, k3x);
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, true, false>, k3x);
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, false, true>, k3x);
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, true, true>, k3x);
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, false, false, true>, kMix);
  pair_attr(tc2_gemm_kernel<256, kPair3xStages, true, false, true, true>, kMix);
  pair_attr(tc2_gemm_kernel<256, kPairStages, false, false, false>, kTf);
  pair_attr(tc2_gemm_kernel<256, kPairStages, false, false, true>, kTf);
  constexpr int s3x = Tc2Cfg<256, kPair3xStages, true, true, 32>::kSmemBytes;
  constexpr int sTf = Tc2Cfg<256, kPairStages, false, true, 32>::kSmemBytes;
  pair_attr(tc2_sk_kernel<256, kPair3xStages, true, false, false>, s3x);
  pair_attr(tc2_sk_kernel<256, kPair3xStages, true, true, false>, s3x);
  pair_attr(tc2_sk_kernel<256, kPair3xStages, true, false, true>, s3x);
  pair_attr(tc2_sk_kernel<256, kPair3xStages, true, true, true>, s3x);
  pair_attr(tc2_sk_kernel<256, kPairStages, false, false, false>, sTf);
  pair_attr(tc2_sk_kernel<256, kPairStages, false, false, true>, sTf);
  // 256 x 128 pair tiles (N columns that pad badly to 256): 3XTF32, its masked form and TF32.
  constexpr int k3x128 = Tc2Cfg<128, kPair3xStages, true, false, 32>::kSmemBytes;
  constexpr int kTf128 = Tc2Cfg<128, kPairStages, false>::kSmemBytes;
  constexpr int s3x128 = Tc2Cfg<128, kPair3xStages, true, true, 32>::kSmemBytes;
  constexpr int sTf128 = Tc2Cfg<128, kPairStages, false, true, 32>::kSmemBytes;
  pair_attr(tc2_gemm_kernel<128, kPair3xStages, true, false, false>, k3x128);
  pair_attr(tc2_gemm_kernel<128, kPair3xStages, true, true, false>, k3x128);
  pair_attr(tc2_gemm_kernel<128, kPair3xStages, true, false, true>, k3x128);
  pair_attr(tc2_gemm_kernel<128, kPair3xStages, true, true, true>, k3x128);
  pair_attr(tc2_gemm_kernel<128, kPairStages, false, false, false>, kTf128);
  pair_attr(tc2_gemm_kernel<128, kPairStages, false, false, true>, kTf128);
  pair_attr(tc2_sk_kernel<128, kPair3xStages, true, false, false>, s3x128);
  pair_attr(tc2_sk_kernel<128, kPair3xStages, true, true, false>, s3x128);
  pair_attr(tc2_sk_kernel<128, kPair3xStages, true, false, true>, s3x128);
  pair_attr(tc2_sk_kernel<128, kPair3xStages, true, true, true>, s3x128);
  pair_attr(tc2_sk_kernel<128, kPairStages, false, false, false>, sTf128);
  pair_attr(tc2_sk_kernel<128, kPairStages, false, false, true>, sTf128);
  pair_attr(tc2_tf32p_kernel<false>, Tc2PCfg::kSmemBytes);
  pair_attr(tc2_tf32p_kernel<true>, Tc2PCfg::kSmemBytes);
  return e;
}

// CTA pairs of the stream-K kernel that fit on the device at once (clusters must sit within
// one GPC, so this can be below SMs / 2).  A stream-K launch never asks for more: its pairs
// wait on one another's partial tiles.  0 disables stream-K.
// CTA pairs of the persistent TF32 pair kernel that fit on the device at once (its grid).
int query_tf32p_slots() {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(2, 1, 1);
  lc.blockDim = dim3(Tc2PCfg::kThreads);
  lc.dynamicSmemBytes = Tc2PCfg::kSmemBytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc2_tf32p_kernel<false>, &lc) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int query_pair_slots() {
  using Cfg = Tc2Cfg<256, kPair3xStages, true, true, 32>;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(2, 1, 1);
  lc.blockDim = dim3(Cfg::kThreads);
  lc.dynamicSmemBytes = Cfg::kSmemBytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc2_sk_kernel<256, kPair3xStages, true, false, false>, &lc) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
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
    if (e == cudaSuccess) d.pair_slots = query_pair_slots();
    if (e == cudaSuccess) d.tf32p_slots = query_tf32p_slots();
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
//   [stream-K: pairs x 256 x 256 fp32 partial tiles][pairs x 16 int ready flags]
// One call's arguments: a single product is batch 1 (batch strides unused).  Batch b reads
// A + b*stride_a and B + b*stride_b (a zero stride shares that operand) and writes
// C + b*stride_c; bias (per column, or nullptr) and act form the fused epilogue.
struct Problem {
  const float* A = nullptr;
  const float* B = nullptr;
  float* C = nullptr;
  const float* bias = nullptr;
  int64_t M = 0, N = 0, K = 0, lda = 0, ldb = 0, ldc = 0;
  int64_t batch = 1, stride_a = 0, stride_b = 0, stride_c = 0;
};

// Packed copies exist only for operands whose rows (or batch strides) are not 16-byte
// aligned and only on the tensor-core path (TMA needs 16-byte aligned bases and strides).
struct Plan {
  int variant = TILEC_MM_SIMT;
  int split = 1;
  int64_t k_chunk = 0;
  int bn = 128;
  int bm = kTcBM;     // tensor variants, 1-CTA kernel: rows per output tile (128 or 64)
  size_t ws_bytes = 0;
  int64_t ldw = 0;
  int flags = 0;      // TILEC_MM_TRANS_A / TILEC_MM_TRANS_B: how A and B are stored
  bool pack_a = false, pack_b = false;    // tensor variants: aligned copy, same storage order
  bool tpose_a = false, tpose_b = false;  // SIMT variants: transposed operand -> row-major copy
  bool pair = false;  // 3XTF32 on a CTA pair (tc2_gemm_kernel, 256 x 256 tiles)
  bool sk = false;    // pair kernel in its stream-K form (split == 1)
  bool persist = false;  // TF32 on the persistent pair kernel (split == 1, more tiles than pairs fit)
  int persist_pairs = 0;
  int bk = 16;        // tensor variants: K per pipeline stage of the kernel that runs (TMA box depth)
  int sk_pairs = 0, sk_dp_tiles = 0, sk_tiles = 0, sk_tiles_per_batch = 0;
  size_t off_sk = 0;  // [sk_pairs partial tiles][sk_pairs x 16 ready flags]
  bool a_shared = false, b_shared = false;  // batch > 1 with a zero batch stride
  int act = 0;                              // TILEC_MM_ACT_*
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
                 int64_t lda, int64_t ldb, int64_t batch, int* variant, int* split) {
  {
    std::lock_guard<std::mutex> lk(g_table_mu);
    if (!g_table.empty()) {
      const int lm = ilog2_floor(M), ln = ilog2_floor(N), lk2 = ilog2_floor(K);
      for (size_t r = 0; r + 8 <= g_table.size(); r += 8) {
        const int32_t* t = &g_table[r];
        if (lm >= t[0] && lm < t[1] && ln >= t[2] && ln < t[3] && lk2 >= t[4] && lk2 < t[5]) {
          int v = t[6];
          const bool tc = v == TILEC_MM_TF32 || v == TILEC_MM_3XTF32 || v == TILEC_MM_3XTF32_MASKED ||
                          v == TILEC_MM_3XMIXED;
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
  const double flops = 2.0 * double(M) * double(N) * double(K) * double(batch);
  const bool aligned = tensor_path_ok(A, B, M, N, K, lda, ldb);
  // Thresholds from B200 timings of small products, eager (back-to-back calls through the
  // Python binding) and in CUDA graphs: from about 1e5 FLOPs the tcgen05 kernel, whose
  // set-up overlaps the previous kernel (programmatic launch), beats the SIMT kernel
  // (64^3: 8.0 / 4.3 us against 8.9 / 6.4; 100^3: 8.2 / 7.8 against 16.4 / 15.0; 32 x 2048
  // x 32: 10.7 / 6.3 against 11.6 / 8.4).  Misaligned operands are packed first, one more
  // launch, which pays from about 2e5 FLOPs when K >= 64 (5 x 306 x 169: 12.5 / 9.9
  // against 14.3 / 12.2); with a smaller K the product is mostly the store of C and the
  // SIMT kernel does it in one launch (2780 x 2 x 235: 8.8 against 11.3 us eager).  Smaller
  // products (1 x 4096 x 1, 445 x 4 x 1, 2 x 283 x 13) go to the SIMT kernel, split over K
  // when their tiles leave SMs idle (the split rule picks 1 when it would not pay).
  if (tensor_dims_ok(M, N, K) && (aligned ? flops >= 1.0e5 : (flops >= 2.0e5 && K >= 64))) {
    *variant = TILEC_MM_3XTF32;
    return;
  }
  const int64_t tiles = cdiv(M, kSimtBM) * cdiv(N, N <= 64 ? 64 : 128) * batch;
  *variant = tiles < d.sms ? TILEC_MM_SPLITK : TILEC_MM_SIMT;
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
constexpr double kRate3x = 1.7e12, kRateMix = 2.4e12, kRateTf32 = 4.3e12, kRateSimt = 0.31e12, kBwPerSm = 38.0e9;

// Stream-K form of the pair kernel (Plan::sk).  T tiles on P pair slots take ceil(T / P)
// waves of tile-times as one pair per tile, and T / P tile-times as stream-K, times a
// per-k-block penalty measured on B200 at 2048^3 (all 148 SMs streaming their own k
// offsets run 6 % slower per k-block in 3XTF32 than 128 SMs in lockstep, 17 % in the
// L2-bound TF32), plus ~5 us for the partial tiles' round trip and the flag reset.  Chosen,
// unless `forced`, when that is at least 3 % faster, every tile has at most three pairs
// (T >= P / 2) and K has at least 8 blocks.  The tiles of all waves but the last complete
// one stay one per pair (sk_dp_tiles); the rest, P to 2P - 1 tiles, are shared out.
constexpr size_t kPartialBytes = size_t(Tc2Cfg<256, kPair3xStages, true, true, 32>::kPartialFloats) * sizeof(float);
constexpr int kSkFlagsPerPair = 2 * Tc2Cfg<256, kPair3xStages, true, true, 32>::kEpiWarps;

void plan_stream_k(const DeviceInfo& d, int64_t M, int64_t N, int64_t K, int64_t nb, int bk, bool tf32,
                   double cta_s, bool forced, Plan* p) {
  const int64_t P = d.pair_slots;
  if (P <= 0) return;
  const int64_t per_batch = cdiv(M, 256) * cdiv(N, p->bn);
  const int64_t T = per_batch * nb, nkb = cdiv(K, bk);
  if (T >= (int64_t(1) << 30)) return;
  if (!forced) {
    if (nkb < 8 || 2 * T < P) return;
    const double penalty = tf32 ? 1.17 : 1.08;
    const double dp = double(cdiv(T, P)) * cta_s;
    const double sk = double(T) / double(P) * cta_s * penalty + 5.0e-6;
    if (!(sk < 0.97 * dp)) return;
  }
  const int64_t dp_tiles = T >= 2 * P ? (T / P - 1) * P : 0;
  const int64_t units = (T - dp_tiles) * nkb;  // >= P whenever dp_tiles > 0
  if (units * P >= (int64_t(1) << 31)) return;  // the kernel's share arithmetic is 32-bit
  p->sk = true;
  p->split = 1;
  p->k_chunk = round_up(K, bk);
  p->sk_pairs = static_cast<int>(units < P ? units : P);
  p->sk_dp_tiles = static_cast<int>(dp_tiles);
  p->sk_tiles = static_cast<int>(T);
  p->sk_tiles_per_batch = static_cast<int>(per_batch);
}

int make_plan(const DeviceInfo& d, const Problem& q, const tilec_mm_cfg* cfg, Plan* p) {
  const int64_t M = q.M, N = q.N, K = q.K, nb = q.batch;
  int variant = cfg ? cfg->variant : TILEC_MM_AUTO;
  int requested_split = cfg ? cfg->split_k : 0;
  const int flags = cfg ? cfg->flags : 0;
  const int act = cfg ? cfg->activation : 0;
  if (flags & ~(TILEC_MM_TRANS_A | TILEC_MM_TRANS_B | TILEC_MM_STREAM_K | TILEC_MM_TILE_M64 | TILEC_MM_TILE_M128))
    return TILEC_ERR_BAD_ARG;
  if ((flags & TILEC_MM_TILE_M64) && (flags & TILEC_MM_TILE_M128)) return TILEC_ERR_BAD_ARG;
  const bool want_sk = (flags & TILEC_MM_STREAM_K) != 0;
  if (act < TILEC_MM_ACT_NONE || act > TILEC_MM_ACT_GELU) return TILEC_ERR_BAD_ARG;
  if (cfg) {
    for (int i = 0; i < 4; ++i)
      if (cfg->reserved[i] != 0) return TILEC_ERR_BAD_ARG;
  }
  p->flags = flags & (TILEC_MM_TRANS_A | TILEC_MM_TRANS_B);
  p->act = act;
  p->a_shared = nb > 1 && q.stride_a == 0;
  p->b_shared = nb > 1 && q.stride_b == 0;
  if (requested_split < 0) return TILEC_ERR_BAD_ARG;
  if (variant == TILEC_MM_AUTO) choose_auto(d, q.A, q.B, M, N, K, q.lda, q.ldb, nb, &variant, &requested_split);
  if (variant < TILEC_MM_SIMT || variant > TILEC_MM_3XMIXED) return TILEC_ERR_BAD_ARG;
  const bool tensor = variant == TILEC_MM_TF32 || variant == TILEC_MM_3XTF32 || variant == TILEC_MM_3XTF32_MASKED ||
                      variant == TILEC_MM_3XMIXED;
  if (tensor && !tensor_dims_ok(M, N, K)) return TILEC_ERR_UNSUPPORTED;
  if (tensor) {
    // TMA also needs each batch's base 16-byte aligned: batch strides a multiple of 4.
    p->pack_a = !rows_aligned(q.A, q.lda) || (nb > 1 && q.stride_a % 4 != 0);
    p->pack_b = !rows_aligned(q.B, q.ldb) || (nb > 1 && q.stride_b % 4 != 0);
  } else {
    p->tpose_a = (flags & TILEC_MM_TRANS_A) != 0;
    p->tpose_b = (flags & TILEC_MM_TRANS_B) != 0;
  }

  p->variant = variant;
  if (tensor) {
    p->bn = N <= 64 ? 64 : (N <= 128 ? 128 : 256);
    p->pair = p->bn == 256 && M >= kPairMinM && !(flags & TILEC_MM_TILE_M64);
    // Pair tiles 128 columns wide for 256 < N <= 384, where 256-wide tiles pad N to 512
    // columns of MMAs and 128-wide ones to 384.  A 128-column pair reads 4/3 of the shared
    // memory per FLOP of a 256-column one, and on B200 ran each FLOP ~1.3x slower
    // (8192 x 4096 x 1100: 420 against 307 us), so narrower tiles pay only where they cut
    // the padding by a third (1024 x 4096 x 300 3xTF32: 28.4 against 30.8 us; TF32 19.5
    // against 22.2 us).  N = 777 keeps 256 (56.7 against 47.9 us).  The mixed split keeps 256.
    if (p->pair && variant != TILEC_MM_3XMIXED && N > 256 && N <= 384) p->bn = 128;
    if (!p->pair) {
      // 64-row tiles: asked for, or products of at most 64 rows (a 128-row tile would be
      // half empty).  Skinny products that split K keep 128-row tiles: 64-row tiles halve
      // their partial-sum slabs but double each CTA's share of B, and measured slower on B200
      // (512 x 4096 x 64: 10.2-12.4 us against 9.4 us).
      const bool want64 = (flags & TILEC_MM_TILE_M64) || (!(flags & TILEC_MM_TILE_M128) && M <= 64);
      if (want64) p->bm = kTcBM64;
    }
    // The mixed split exists only in the one-pair-per-tile kernel.
    if (variant == TILEC_MM_3XMIXED && !p->pair) p->variant = variant = TILEC_MM_3XTF32;
    const bool mixed = variant == TILEC_MM_3XMIXED;
    // K per stage: 32 for TF32 and every pair-kernel variant, 16 in the 1-CTA 3XTF32 kernel.
    // K slices of the pair kernel are multiples of 32, so 3XTF32, its masked form and
    // 3XMIXED cut K at the same points.
    const int bk = (variant == TILEC_MM_TF32 || p->pair) ? 32 : k3xBK;
    const int slice_align = p->pair ? 32 : bk;
    const int64_t tiles = cdiv(M, p->bm) * cdiv(N, p->bn);
    // The CTA pair launches two CTAs per 256-row x 256-column tile; each computes 128 rows
    // and loads half of the B columns.
    const int64_t ctas = (p->pair ? 2 * cdiv(M, 256) * cdiv(N, p->bn) : tiles) * nb;
    const double cta_s = cta_seconds(p->bm, p->bn, p->pair ? p->bn / 2 : p->bn, K,
                                     variant == TILEC_MM_TF32 ? kRateTf32 : (mixed ? kRateMix : kRate3x), kBwPerSm);
    p->split = choose_split(ctas, d.sms, cta_s, double(M) * double(round_up(N, 4)) * 4.0 * double(nb),
                            K / (int64_t(slice_align) * 4), requested_split, /*one_wave=*/true);
    p->k_chunk = round_up(cdiv(K, p->split), slice_align);
    p->split = static_cast<int>(cdiv(K, p->k_chunk > 0 ? p->k_chunk : 1));
    if (p->split < 1) p->split = 1;
    p->bk = bk;
    if (p->pair && !mixed && K > 0 && requested_split <= 1 && (want_sk || (requested_split == 0 && p->split == 1))) {
      plan_stream_k(d, M, N, K, nb, bk, variant == TILEC_MM_TF32, cta_s, want_sk, p);
    }
    // TF32 tiles beyond one wave of pairs run on the persistent pair kernel: each pair walks
    // its tiles with two TMEM accumulators, so a tile's epilogue overlaps the next tile's MMAs.
    // Its per-tile MMA sequence is the one-pair-per-tile kernel's, so the results are the same.
    const int64_t pair_tiles = cdiv(M, 256) * cdiv(N, 256) * nb;
    if (p->pair && p->bn == 256 && !p->sk && variant == TILEC_MM_TF32 && p->split == 1 && d.tf32p_slots > 0 &&
        pair_tiles > d.tf32p_slots && pair_tiles < (int64_t(1) << 30)) {
      p->persist = true;
      p->persist_pairs = d.tf32p_slots;
    }
  } else {
    p->bn = N <= 64 ? 64 : 128;
    const int64_t tiles = cdiv(M, kSimtBM) * cdiv(N, p->bn) * nb;
    int split = 1;
    if (variant == TILEC_MM_SPLITK) {
      const double cta_s = cta_seconds(kSimtBM, p->bn, p->bn, K, kRateSimt, kBwPerSm);
      split = choose_split(tiles, d.sms, cta_s, double(M) * double(round_up(N, 4)) * 4.0 * double(nb),
                           K / (int64_t(kSimtBK) * 4), requested_split, /*one_wave=*/false);
    }
    p->k_chunk = round_up(cdiv(K, split), kSimtBK);
    split = static_cast<int>(cdiv(K, p->k_chunk > 0 ? p->k_chunk : 1));
    p->split = split < 1 ? 1 : split;
  }
  if (p->k_chunk <= 0) p->k_chunk = 16;
  p->ldw = round_up(N, 4);
  // An aligned copy keeps the stored order (K x M for a transposed A); a SIMT transpose
  // writes the row-major M x K (K x N) operand.  One copy per batch (one when shared).
  const bool ta = (flags & TILEC_MM_TRANS_A) != 0, tb = (flags & TILEC_MM_TRANS_B) != 0;
  const size_t na = p->a_shared ? 1 : size_t(nb), nbb = p->b_shared ? 1 : size_t(nb);
  size_t off = 0;
  if (p->pack_a || p->tpose_a) {
    p->off_a = off;
    const size_t elems = (p->pack_a && ta) ? size_t(K) * size_t(round_up(M, 4)) : size_t(M) * size_t(round_up(K, 4));
    off += align256(na * elems * sizeof(float));
  }
  if (p->pack_b || p->tpose_b) {
    p->off_b = off;
    const size_t elems = (p->pack_b && tb) ? size_t(N) * size_t(round_up(K, 4)) : size_t(K) * size_t(round_up(N, 4));
    off += align256(nbb * elems * sizeof(float));
  }
  p->off_slabs = off;
  if (p->split > 1) off += size_t(nb) * size_t(p->split) * size_t(M) * size_t(p->ldw) * sizeof(float);
  if (p->sk) {
    off = align256(off);
    p->off_sk = off;
    off += size_t(p->sk_pairs) * (kPartialBytes + kSkFlagsPerPair * sizeof(int));
  }
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

// check_args for every product of a batch, plus: non-negative batch and strides, and
// batches of C that do not overlap (they are written concurrently).
int check_problem(const Problem& q, bool need_c, int flags) {
  const int rc = check_args(q.A, q.B, q.C, q.M, q.N, q.K, q.lda, q.ldb, q.ldc, need_c, flags);
  if (rc) return rc;
  if (q.batch < 0 || q.stride_a < 0 || q.stride_b < 0 || q.stride_c < 0) return TILEC_ERR_BAD_ARG;
  if (q.batch > 1 && q.M > 0 && q.N > 0 && q.stride_c < (q.M - 1) * q.ldc + q.N) return TILEC_ERR_BAD_ARG;
  return TILEC_OK;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TILEC_OK : TILEC_ERR_LAUNCH;
}

// Tensor maps for the operand tiles (`layout`: kOpAMN / kOpBK, see common.cuh), 3-D with
// the batch outermost (extent 1 for a single or shared operand).  A K-major: box {bk, 128}
// with a bk*4-byte swizzle; A MN-major (stored K x M): boxes {32, bk} with the 128-byte /
// 32-byte-granule swizzle.  B MN-major: boxes {32, bk}, same swizzle; B K-major (stored
// N x K): box {bk, b_rows}, bk*4-byte swizzle.
int encode_maps(const float* A, const float* B, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                int64_t stride_a, int64_t nba, int64_t stride_b, int64_t nbb, int bk, int layout, int b_rows,
                CUtensorMap* ma, CUtensorMap* mb, int a_rows = kTcBM) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode();
  if (!enc) return TILEC_ERR_NO_DEVICE;
  const CUtensorMapSwizzle k_sw = bk * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  auto encode = [&](CUtensorMap* m, const float* base, int64_t inner, int64_t outer, int64_t ld, int64_t bstride,
                    int64_t nbatch, int box_in, int box_out, CUtensorMapSwizzle sw) {
    cuuint64_t dims[3] = {cuuint64_t(inner), cuuint64_t(outer), cuuint64_t(nbatch)};
    const int64_t bs = nbatch > 1 ? bstride : round_up(outer * ld, 4);
    cuuint64_t strides[2] = {cuuint64_t(ld) * 4, cuuint64_t(bs) * 4};
    cuuint32_t box[3] = {cuuint32_t(box_in), cuuint32_t(box_out), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  const bool ok_a = (layout & kOpAMN)
                        ? encode(ma, A, M, K, lda, stride_a, nba, 32, bk, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                        : encode(ma, A, K, M, lda, stride_a, nba, bk, a_rows, k_sw);
  const bool ok_b = (layout & kOpBK) ? encode(mb, B, K, N, ldb, stride_b, nbb, bk, b_rows, k_sw)
                                     : encode(mb, B, N, K, ldb, stride_b, nbb, 32, bk,
                                              CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  return ok_a && ok_b ? TILEC_OK : TILEC_ERR_BAD_ARG;
}

// B of the SIMT kernel as a TMA map: {N, K, batch} with a dense {bn, 16, 1} box (no swizzle:
// the kernel reads the [16][bn] tile as written); extent N and K zero-fill ragged edges.
int encode_simt_b_map(const float* B, int64_t N, int64_t K, int64_t ldb, int64_t stride_b, int64_t nbb, int bn,
                      CUtensorMap* mb) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode();
  if (!enc) return TILEC_ERR_NO_DEVICE;
  cuuint64_t dims[3] = {cuuint64_t(N), cuuint64_t(K), cuuint64_t(nbb)};
  const int64_t bs = nbb > 1 ? stride_b : round_up(K * ldb, 4);
  cuuint64_t strides[2] = {cuuint64_t(ldb) * 4, cuuint64_t(bs) * 4};
  cuuint32_t box[3] = {cuuint32_t(bn), cuuint32_t(kSimtBK), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(B), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? TILEC_OK
             : TILEC_ERR_BAD_ARG;
}

// Programmatic dependent launch is on unless TILEC_MM_PDL=0 (read once per process).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TILEC_MM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Raster band height (pair-rows) of the one-pair-per-tile kernel: 8 unless TILEC_MM_PAIR_BAND
// (1..64, read once) says otherwise.  8 reads least from DRAM on B200 (16384x8192x8192: 4 /
// 8 / 16 pair-rows read 5.84 / 4.65 / 5.32 GB, same speed within 1.2 %); the variable exists
// to reproduce that measurement.
int pair_band() {
  static const int band = [] {
    const char* e = std::getenv("TILEC_MM_PAIR_BAND");
    const int v = e ? std::atoi(e) : 0;
    return v >= 1 && v <= 64 ? v : 8;
  }();
  return band;
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

// Per-launch arguments of the GEMM kernels: where the output goes (C, or the split-K
// slabs: slab z of batch b at out + z*out_slab + b*out_batch), the fused epilogue (only
// when writing C), the batch count (grid y) and the shared-operand bits.
struct Launch {
  float* out = nullptr;
  int64_t ldo = 0, out_slab = 0, out_batch = 0, k_chunk = 0;
  int split = 1, vec_out = 0, layout = 0, batch = 1, shared = 0, act = 0;
  const float* bias = nullptr;
};

template <int BN, int BK, int STAGES, bool SPLIT3, bool HI, int BM = kTcBM>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K, const Launch& L,
              cudaStream_t s) {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3, BM>;
  const int m_tiles = static_cast<int>(cdiv(M, BM));
  const int n_tiles = static_cast<int>(cdiv(N, BN));
  const int group_m = 16;
  const dim3 grid(static_cast<unsigned>(int64_t(m_tiles) * n_tiles), static_cast<unsigned>(L.batch),
                  static_cast<unsigned>(L.split));
  auto go = [&](auto kern) {
    return launch_k(kern, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, s, 1, ma, mb, L.out, static_cast<int>(M),
                    static_cast<int>(N), L.ldo, L.out_slab, static_cast<int>(K), static_cast<int>(L.k_chunk), m_tiles,
                    n_tiles, group_m, L.vec_out, L.layout, L.out_batch, L.bias, L.act, L.shared);
  };
  return L.layout ? go(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI, true, BM>)
                  : go(tc_gemm_kernel<BN, BK, STAGES, SPLIT3, HI, false, BM>);
}

template <int BN, bool SPLIT3, bool HI>
int launch_tc_mode(int bm, const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K,
                   const Launch& L, cudaStream_t s) {
  if (bm == kTcBM64) {
    if constexpr (SPLIT3)
      return launch_tc<BN, k3xBK, TcShape64<BN>::k3xStages, true, HI, kTcBM64>(ma, mb, M, N, K, L, s);
    else
      return launch_tc<BN, 32, TcShape64<BN>::kTf32Stages, false, false, kTcBM64>(ma, mb, M, N, K, L, s);
  }
  if constexpr (SPLIT3)
    return launch_tc<BN, k3xBK, TcShape<BN>::k3xStages, true, HI>(ma, mb, M, N, K, L, s);
  else
    return launch_tc<BN, 32, TcShape<BN>::kTf32Stages, false, false>(ma, mb, M, N, K, L, s);
}

template <int BN, bool SPLIT3, bool HI, bool MIXED = false>
int launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K, const Launch& L,
               cudaStream_t s) {
  constexpr int kStages = SPLIT3 ? kPair3xStages : kPairStages;
  using Cfg = Tc2Cfg<BN, kStages, SPLIT3, false, kTc2Bk<SPLIT3, MIXED>>;
  const int mp_tiles = static_cast<int>(cdiv(M, 256));
  const int n_tiles = static_cast<int>(cdiv(N, BN));
  const int group_m = pair_band();
  const dim3 grid(static_cast<unsigned>(2 * int64_t(mp_tiles) * n_tiles), static_cast<unsigned>(L.batch),
                  static_cast<unsigned>(L.split));
  auto go = [&](auto kern) {
    return launch_k(kern, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, s, 2, ma, mb, L.out, static_cast<int>(M),
                    static_cast<int>(N), L.ldo, L.out_slab, static_cast<int>(K), static_cast<int>(L.k_chunk),
                    mp_tiles, n_tiles, group_m, L.vec_out, L.layout, L.out_batch, L.bias, L.act, L.shared);
  };
  return L.layout ? go(tc2_gemm_kernel<BN, kStages, SPLIT3, HI, true, MIXED>)
                  : go(tc2_gemm_kernel<BN, kStages, SPLIT3, HI, false, MIXED>);
}

// Stream-K form: the flag reset (programmatic serialisation on both sides, so the GEMM's
// set-up still overlaps the previous kernel) and a grid of `pairs` pairs.
template <int BN, bool SPLIT3, bool HI>
int launch_tc2_sk(const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K, const Launch& L,
                  const Tc2StreamK& sk, int pairs, cudaStream_t s) {
  int rc = launch_k(sk_flags_reset_kernel, dim3(1), dim3(256), 0, s, 1, sk.flags, pairs * kSkFlagsPerPair);
  if (rc) return rc;
  constexpr int kStages = SPLIT3 ? kPair3xStages : kPairStages;
  using Cfg = Tc2Cfg<BN, kStages, SPLIT3, true, 32>;
  const int mp_tiles = static_cast<int>(cdiv(M, 256));
  const int n_tiles = static_cast<int>(cdiv(N, BN));
  const int group_m = 8;
  auto go = [&](auto kern) {
    return launch_k(kern, dim3(static_cast<unsigned>(2 * pairs)), dim3(Cfg::kThreads), Cfg::kSmemBytes, s, 2, ma,
                    mb, L.out, static_cast<int>(M), static_cast<int>(N), L.ldo, static_cast<int>(K), mp_tiles,
                    n_tiles, group_m, L.vec_out, L.layout, L.out_batch, L.bias, L.act, L.shared, sk);
  };
  return L.layout ? go(tc2_sk_kernel<BN, kStages, SPLIT3, HI, true>)
                  : go(tc2_sk_kernel<BN, kStages, SPLIT3, HI, false>);
}

// Persistent TF32 pair kernel: `pairs` pairs share out the 256 x 256 tiles of all batches.
int launch_tc2p(const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K, const Launch& L,
                int pairs, cudaStream_t s) {
  const int mp_tiles = static_cast<int>(cdiv(M, 256));
  const int n_tiles = static_cast<int>(cdiv(N, 256));
  const int per_batch = mp_tiles * n_tiles;
  const int total = per_batch * L.batch;
  const int group_m = 8;
  if (pairs > total) pairs = total;
  auto go = [&](auto kern) {
    return launch_k(kern, dim3(static_cast<unsigned>(2 * pairs)), dim3(Tc2PCfg::kThreads), Tc2PCfg::kSmemBytes, s, 2,
                    ma, mb, L.out, static_cast<int>(M), static_cast<int>(N), L.ldo, static_cast<int>(K), mp_tiles,
                    n_tiles, group_m, per_batch, total, L.vec_out, L.layout, L.out_batch, L.bias, L.act, L.shared);
  };
  return L.layout ? go(tc2_tf32p_kernel<true>) : go(tc2_tf32p_kernel<false>);
}

template <bool SPLIT3, bool HI>
int dispatch_tc_bn(int bm, int bn, const CUtensorMap& ma, const CUtensorMap& mb, int64_t M, int64_t N, int64_t K,
                   const Launch& L, cudaStream_t s) {
  switch (bn) {
    case 64: return launch_tc_mode<64, SPLIT3, HI>(bm, ma, mb, M, N, K, L, s);
    case 128: return launch_tc_mode<128, SPLIT3, HI>(bm, ma, mb, M, N, K, L, s);
    default: return launch_tc_mode<256, SPLIT3, HI>(bm, ma, mb, M, N, K, L, s);
  }
}

// One operand copy of pack_rows_kernel: dst[b][r, 0:cols] = src[b][r, 0:cols] for b <
// batches (src batch stride sstride, dst dense: batch stride rows*ldd), over grid-x
// blocks [first, first + blocks).
struct PackJob {
  const float* src = nullptr;
  float* dst = nullptr;
  int64_t lds = 0, sstride = 0, ldd = 0, rows = 0, cols = 0, batches = 0;
  int64_t first = 0, blocks = 0;
};

// Copies rows into a buffer with 16-byte aligned rows (dst 16-byte aligned, ldd a multiple
// of 4), for one or two operands in one launch (job 1 takes the blocks after job 0's; batch
// b = blockIdx.y).  Source rows are only 4-byte aligned, so each thread reads the two
// 16-byte-aligned float4s that hold its output chunk and shifts them into place: 16-byte
// loads and stores throughout.  An aligned float4 never crosses a page, so reading one that
// holds at least one element of the row cannot fault; the padding columns of the copy
// (cols .. ldd) receive whatever the last chunk held and are never read by the GEMM.
// Short rows share a block: a warp per row when cols <= 1024 (B200, 1000x3001x777 with both
// operands packed: 47.9 -> 46.2 us, same box; taller rows are left at 256 threads per row).
__global__ void __launch_bounds__(256) pack_rows_kernel(const PackJob j0, const PackJob j1) {
  pdl_wait();
  pdl_launch_dependents();
  const bool second = blockIdx.x >= j0.blocks;
  const float* src = second ? j1.src : j0.src;
  float* dst = second ? j1.dst : j0.dst;
  const int64_t lds = second ? j1.lds : j0.lds, ldd = second ? j1.ldd : j0.ldd;
  const int64_t rows = second ? j1.rows : j0.rows, cols = second ? j1.cols : j0.cols;
  const int64_t blocks = second ? j1.blocks : j0.blocks;
  const int64_t bx = static_cast<int64_t>(blockIdx.x) - (second ? j1.first : j0.first);
  if (static_cast<int64_t>(blockIdx.y) >= (second ? j1.batches : j0.batches)) return;
  src += static_cast<int64_t>(blockIdx.y) * (second ? j1.sstride : j0.sstride);
  dst += static_cast<int64_t>(blockIdx.y) * rows * ldd;
  const int64_t lanes = cols <= 1024 ? 32 : blockDim.x;
  const int64_t rows_per_block = blockDim.x / lanes;
  const int64_t sub = threadIdx.x / lanes, t = threadIdx.x % lanes;
  const int64_t chunks = (cols + 3) / 4;
  for (int64_t r = bx * rows_per_block + sub; r < rows; r += blocks * rows_per_block) {
    const float* s = src + r * lds;
    const int shift = static_cast<int>((reinterpret_cast<uintptr_t>(s) >> 2) & 3);
    const float4* base = reinterpret_cast<const float4*>(s - shift);
    const int64_t last = (shift + cols - 1) / 4;  // last aligned float4 holding row data
    float4* d = reinterpret_cast<float4*>(dst + r * ldd);
    for (int64_t q0 = t; q0 < chunks; q0 += 2 * lanes) {
      float4 lo[2], hi[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int64_t q = q0 + j * lanes;
        if (q < chunks) {
          lo[j] = __ldg(base + q);
          hi[j] = q + 1 <= last ? __ldg(base + q + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int64_t q = q0 + j * lanes;
        if (q >= chunks) continue;
        const float w[8] = {lo[j].x, lo[j].y, lo[j].z, lo[j].w, hi[j].x, hi[j].y, hi[j].z, hi[j].w};
        float4 o;
        switch (shift) {
          case 0: o = lo[j]; break;
          case 1: o = make_float4(w[1], w[2], w[3], w[4]); break;
          case 2: o = make_float4(w[2], w[3], w[4], w[5]); break;
          default: o = make_float4(w[3], w[4], w[5], w[6]); break;
        }
        d[q] = o;
      }
    }
  }
}

// dst[b][c, r] = src[b][r, c] for r < rows, c < cols, batch b = blockIdx.y (src batch
// stride sstride, dst dense: batch stride cols*ldd): 32 x 32 tiles through shared memory (the
// +1 column keeps the transposed reads free of bank conflicts), coalesced on both sides.
__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ src, int64_t lds, int64_t sstride,
                                                        float* __restrict__ dst, int64_t ldd, int64_t rows,
                                                        int64_t cols, int64_t batches) {
  __shared__ float t[32][33];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t tr = (rows + 31) / 32, tc = (cols + 31) / 32;
  const int tx = static_cast<int>(threadIdx.x) & 31, ty = static_cast<int>(threadIdx.x) >> 5;  // 32 x 8
  (void)batches;
  const float* sb = src + static_cast<int64_t>(blockIdx.y) * sstride;
  float* db = dst + static_cast<int64_t>(blockIdx.y) * cols * ldd;
  for (int64_t tile = blockIdx.x; tile < tr * tc; tile += gridDim.x) {
    const int64_t r0 = (tile / tc) * 32, c0 = (tile % tc) * 32;
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, c = c0 + tx;
      if (r < rows && c < cols) t[i][tx] = sb[r * lds + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int64_t c = c0 + i, r = r0 + tx;
      if (r < rows && c < cols) db[c * ldd + r] = t[tx][i];
    }
    __syncthreads();
  }
}

int launch_transpose(const float* src, int64_t lds, int64_t sstride, float* dst, int64_t ldd, int64_t rows,
                     int64_t cols, int64_t batches, const DeviceInfo& d, cudaStream_t s) {
  int64_t blocks = cdiv(rows, 32) * cdiv(cols, 32);
  const int64_t cap = int64_t(d.sms) * 8 / batches + 1;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return launch_k(transpose_kernel, dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(batches)), dim3(256), 0,
                  s, 1, src, lds, sstride, dst, ldd, rows, cols, batches);
}

// A pack job over up to 8 resident 256-thread blocks per SM (split between the batches).
PackJob pack_job(const float* src, int64_t lds, int64_t sstride, float* dst, int64_t ldd, int64_t rows,
                 int64_t cols, int64_t batches, const DeviceInfo& d) {
  PackJob j;
  j.src = src;
  j.dst = dst;
  j.lds = lds;
  j.sstride = sstride;
  j.ldd = ldd;
  j.rows = rows;
  j.cols = cols;
  j.batches = batches;
  const int64_t cap = int64_t(d.sms) * 8 / batches + 1;
  const int64_t per_block = cols <= 1024 ? 8 : 1;  // rows per 256-thread block (warp per row up to 1024)
  j.blocks = cdiv(rows, per_block) < cap ? cdiv(rows, per_block) : cap;
  if (j.blocks < 1) j.blocks = 1;
  return j;
}

// One launch for one or two jobs (j1.blocks == 0: none): both operands of a product pack
// together instead of paying a second launch and ramp (B200, 1000x3001x777 end to end:
// 53.6 -> 50.6 us).
int launch_pack(PackJob j0, PackJob j1, cudaStream_t s) {
  j0.first = 0;
  j1.first = j0.blocks;
  const int64_t batches = j0.batches > j1.batches ? j0.batches : j1.batches;
  return launch_k(pack_rows_kernel, dim3(static_cast<unsigned>(j0.blocks + j1.blocks), static_cast<unsigned>(batches)),
                  dim3(256), 0, s, 1, j0, j1);
}

// The split-K reduction of all batches (slabs of batch b at ws + b*split*M*ldw) into C,
// with the fused epilogue.
struct Reduce {
  const float* ws = nullptr;
  float* C = nullptr;
  int64_t M = 0, N = 0, ldw = 0, ldc = 0, batches = 1, stride_c = 0;
  int split = 1, act = 0;
  const float* bias = nullptr;
};

template <int P>
int launch_reduce_p(int U, dim3 grid, const Reduce& r, int vec_out, cudaStream_t s) {
  const int64_t slab = r.M * r.ldw;
  auto go = [&](auto kern) {
    return launch_k(kern, grid, dim3(256), 0, s, 1, r.ws, r.C, r.M, r.N, r.ldw, r.ldc, slab, r.split, vec_out,
                    r.stride_c, r.bias, r.act);
  };
  switch (U) {
    case 4: return go(splitk_reduce_kernel<P, 4>);
    case 2: return go(splitk_reduce_kernel<P, 2>);
    default: return r.N > 64 ? go(splitk_reduce_kernel<P, 1, 4>) : go(splitk_reduce_kernel<P, 1>);
  }
}

int launch_reduce(const Reduce& r, const DeviceInfo& d, cudaStream_t s) {
  const int P = r.split >= 8 ? 8 : (r.split >= 4 ? 4 : (r.split >= 2 ? 2 : 1));
  const int64_t G = 256 / P;
  const int64_t groups = r.M * cdiv(r.N, 4);                       // per batch
  const int64_t resident = int64_t(d.sms) * 8 / r.batches + 1;       // 256-thread blocks per batch at once
  const int U = groups <= resident * G ? 1 : (groups <= 2 * resident * G ? 2 : 4);
  int64_t blocks = cdiv(groups, G * U);
  if (blocks > resident) blocks = resident;
  if (blocks < 1) blocks = 1;
  const int vec_out = aligned16(r.C) && (r.ldc % 4 == 0) && (r.batches == 1 || r.stride_c % 4 == 0);
  const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(r.batches));
  switch (P) {
    case 8: return launch_reduce_p<8>(U, grid, r, vec_out, s);
    case 4: return launch_reduce_p<4>(U, grid, r, vec_out, s);
    case 2: return launch_reduce_p<2>(U, grid, r, vec_out, s);
    default: return launch_reduce_p<1>(U, grid, r, vec_out, s);
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

int launch_fill_zero(float* C, int64_t M, int64_t N, int64_t ldc, int64_t batches, int64_t stride_c,
                     const float* bias, int act, const DeviceInfo& d, cudaStream_t s) {
  int64_t blocks = cdiv(M * N * batches, 256);
  if (blocks > int64_t(d.sms) * 8) blocks = int64_t(d.sms) * 8;
  if (blocks < 1) blocks = 1;
  return launch_k(fill_zero_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, 1, C, M, N, ldc, batches,
                  stride_c, bias, act);
}

// grid: (M tiles, N tiles, batches * L.split).  A / B advance by stride_a / stride_b per
// batch (0 = shared).
// mb: B's tensor map for TMA staging (encode_simt_b_map), or nullptr for cp.async copies
// (16-byte ones when `vec`).
int launch_simt(int bn, bool vec, const CUtensorMap* mb, dim3 grid, const float* A, const float* B, int64_t M,
                int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t stride_a, int64_t stride_b, const Launch& L,
                int sms, cudaStream_t s) {
  // Launched without programmatic serialisation: two SIMT CTAs fit on an SM, and CTAs
  // placed while the previous kernel still occupies the GPU were measured to double up on
  // some SMs (a 128-CTA grid ran 40% slower).  For the same reason a grid of at most one
  // CTA per SM asks for more than half an SM's shared memory, so that no SM takes two
  // (B200, config 1 as SPLITK, 148 CTAs: 12.2 us with two allowed, 11.6 us spread).
  const dim3 block(kSimtThreads);
  const bool spread = int64_t(grid.x) * grid.y * grid.z <= sms;
  CUtensorMap unused{};
  const CUtensorMap& map = mb ? *mb : unused;
  auto go = [&](auto kern, size_t smem) {
    return launch_kx(false, kern, grid, block, spread ? size_t(kSimtSpreadSmem) : smem, s, 1, map, A, B, L.out, M,
                     N, K, lda, ldb, L.ldo, L.out_slab, L.k_chunk, L.vec_out, L.split, stride_a, stride_b,
                     L.out_batch, L.bias, L.act);
  };
  if (bn == 64)
    return mb ? go(simt_gemm_kernel<64, kBTma>, simt_smem_bytes<64>())
              : vec ? go(simt_gemm_kernel<64, kBVec>, simt_smem_bytes<64>())
                    : go(simt_gemm_kernel<64, kBScalar>, simt_smem_bytes<64>());
  return mb ? go(simt_gemm_kernel<128, kBTma>, simt_smem_bytes<128>())
            : vec ? go(simt_gemm_kernel<128, kBVec>, simt_smem_bytes<128>())
                  : go(simt_gemm_kernel<128, kBScalar>, simt_smem_bytes<128>());
}

constexpr int64_t kMaxBatch = 65535;  // grid y / z limit; larger batches run in chunks

// One launch sequence for a batch chunk (batch <= kMaxBatch): packing / transposition
// into the workspace when needed, the GEMM, and the split-K reduction.
int run_chunk(const DeviceInfo& d, const Problem& q, const tilec_mm_cfg* cfg, void* workspace, size_t ws_bytes,
              cudaStream_t s) {
  Plan p;
  int rc = make_plan(d, q, cfg, &p);
  if (rc) return rc;
  if (p.ws_bytes > 0) {
    if (!workspace || ws_bytes < p.ws_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
      return TILEC_ERR_WORKSPACE;
  }
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  const int64_t M = q.M, N = q.N, K = q.K, nb = q.batch;
  const float* A = q.A;
  const float* B = q.B;
  int64_t lda = q.lda, ldb = q.ldb, sa = p.a_shared ? 0 : q.stride_a, sb = p.b_shared ? 0 : q.stride_b;
  const bool ta = (p.flags & TILEC_MM_TRANS_A) != 0, tb = (p.flags & TILEC_MM_TRANS_B) != 0;
  // Stored shapes: A is M x K (K x M when transposed), B is K x N (N x K when transposed).
  const int64_t a_rows = ta ? K : M, a_cols = ta ? M : K;
  const int64_t b_rows = tb ? N : K, b_cols = tb ? K : N;
  const int64_t na = p.a_shared ? 1 : nb, nbb = p.b_shared ? 1 : nb;
  // Tensor variants: aligned copies (both in one launch); SIMT: row-major transposes.
  PackJob jobs[2];
  int njobs = 0;
  if (p.pack_a || p.tpose_a) {
    float* pa = reinterpret_cast<float*>(wsb + p.off_a);
    if (p.pack_a) {
      const int64_t ld = round_up(a_cols, 4);
      jobs[njobs++] = pack_job(A, lda, sa, pa, ld, a_rows, a_cols, na, d);
      lda = ld;
      sa = p.a_shared ? 0 : a_rows * ld;
    } else {
      const int64_t ld = round_up(K, 4);
      rc = launch_transpose(A, lda, sa, pa, ld, K, M, na, d, s);
      if (rc) return rc;
      lda = ld;
      sa = p.a_shared ? 0 : M * ld;
    }
    A = pa;
  }
  if (p.pack_b || p.tpose_b) {
    float* pb = reinterpret_cast<float*>(wsb + p.off_b);
    if (p.pack_b) {
      const int64_t ld = round_up(b_cols, 4);
      jobs[njobs++] = pack_job(B, ldb, sb, pb, ld, b_rows, b_cols, nbb, d);
      ldb = ld;
      sb = p.b_shared ? 0 : b_rows * ld;
    } else {
      const int64_t ld = round_up(N, 4);
      rc = launch_transpose(B, ldb, sb, pb, ld, N, K, nbb, d, s);
      if (rc) return rc;
      ldb = ld;
      sb = p.b_shared ? 0 : K * ld;
    }
    B = pb;
  }
  if (njobs > 0) {
    rc = launch_pack(jobs[0], njobs > 1 ? jobs[1] : PackJob{}, s);
    if (rc) return rc;
  }
  // The tensor-core kernels read either storage order in place; SIMT operands are now
  // row-major.
  const bool simt = p.variant == TILEC_MM_SIMT || p.variant == TILEC_MM_SPLITK;
  float* slabs = reinterpret_cast<float*>(wsb + p.off_slabs);
  Launch L;
  L.layout = simt ? 0 : p.flags;
  L.batch = static_cast<int>(nb);
  L.shared = (p.a_shared ? 1 : 0) | (p.b_shared ? 2 : 0);
  L.split = p.split;
  L.k_chunk = p.k_chunk;
  if (p.split > 1) {  // partial sums to the slabs; the reduction applies the epilogue
    L.out = slabs;
    L.ldo = p.ldw;
    L.out_slab = M * p.ldw;
    L.out_batch = int64_t(p.split) * M * p.ldw;
    L.vec_out = 1;
  } else {
    L.out = q.C;
    L.ldo = q.ldc;
    L.out_batch = q.stride_c;
    L.vec_out = aligned16(q.C) && (q.ldc % 4 == 0) && (nb == 1 || q.stride_c % 4 == 0) ? 1 : 0;
    L.bias = q.bias;
    L.act = p.act;
  }

  if (simt) {
    const bool vec = aligned16(A) && aligned16(B) && (lda % 4 == 0) && (ldb % 4 == 0) && (sa % 4 == 0) &&
                     (sb % 4 == 0);
    const int64_t mt = cdiv(M, kSimtBM), nt = cdiv(N, p.bn);
    if (nt > 65535 || nb * p.split > 65535) return TILEC_ERR_UNSUPPORTED;
    const dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt), static_cast<unsigned>(nb * p.split));
    // B with 16-byte aligned rows (and batch strides) is staged by TMA.
    CUtensorMap mbs;
    const bool tma_b = rows_aligned(B, ldb) && (nbb == 1 || sb % 4 == 0) && tensor_dims_ok(M, N, K) &&
                       nbb < (int64_t(1) << 31) && encode_simt_b_map(B, N, K, ldb, sb, nbb, p.bn, &mbs) == TILEC_OK;
    rc = launch_simt(p.bn, vec, tma_b ? &mbs : nullptr, grid, A, B, M, N, K, lda, ldb, sa, sb, L, d.sms, s);
  } else {
    CUtensorMap ma, mb;
    const int bk = p.bk;
    rc = encode_maps(A, B, M, N, K, lda, ldb, sa, na, sb, nbb, bk, L.layout, p.pair ? p.bn / 2 : p.bn, &ma, &mb, p.bm);
    if (rc) return rc;
    if (p.sk) {
      Tc2StreamK sk{};
      sk.partial = reinterpret_cast<float*>(wsb + p.off_sk);
      sk.flags = reinterpret_cast<int*>(wsb + p.off_sk + size_t(p.sk_pairs) * kPartialBytes);
      sk.dp_tiles = p.sk_dp_tiles;
      sk.tiles = p.sk_tiles;
      sk.tiles_per_batch = p.sk_tiles_per_batch;
      if (p.bn == 128)
        rc = p.variant == TILEC_MM_TF32     ? launch_tc2_sk<128, false, false>(ma, mb, M, N, K, L, sk, p.sk_pairs, s)
             : p.variant == TILEC_MM_3XTF32 ? launch_tc2_sk<128, true, false>(ma, mb, M, N, K, L, sk, p.sk_pairs, s)
                                            : launch_tc2_sk<128, true, true>(ma, mb, M, N, K, L, sk, p.sk_pairs, s);
      else
        rc = p.variant == TILEC_MM_TF32     ? launch_tc2_sk<256, false, false>(ma, mb, M, N, K, L, sk, p.sk_pairs, s)
             : p.variant == TILEC_MM_3XTF32 ? launch_tc2_sk<256, true, false>(ma, mb, M, N, K, L, sk, p.sk_pairs, s)
                                            : launch_tc2_sk<256, true, true>(ma, mb, M, N, K, L, sk, p.sk_pairs, s);
    } else if (p.persist) {
      rc = launch_tc2p(ma, mb, M, N, K, L, p.persist_pairs, s);
    } else if (p.pair)
      rc = p.bn == 128 ? (p.variant == TILEC_MM_TF32     ? launch_tc2<128, false, false>(ma, mb, M, N, K, L, s)
                          : p.variant == TILEC_MM_3XTF32 ? launch_tc2<128, true, false>(ma, mb, M, N, K, L, s)
                                                         : launch_tc2<128, true, true>(ma, mb, M, N, K, L, s))
           : p.variant == TILEC_MM_TF32      ? launch_tc2<256, false, false>(ma, mb, M, N, K, L, s)
           : p.variant == TILEC_MM_3XTF32  ? launch_tc2<256, true, false>(ma, mb, M, N, K, L, s)
           : p.variant == TILEC_MM_3XMIXED ? launch_tc2<256, true, false, true>(ma, mb, M, N, K, L, s)
                                           : launch_tc2<256, true, true>(ma, mb, M, N, K, L, s);
    else if (p.variant == TILEC_MM_TF32)
      rc = dispatch_tc_bn<false, false>(p.bm, p.bn, ma, mb, M, N, K, L, s);
    else if (p.variant == TILEC_MM_3XTF32)
      rc = dispatch_tc_bn<true, false>(p.bm, p.bn, ma, mb, M, N, K, L, s);
    else
      rc = dispatch_tc_bn<true, true>(p.bm, p.bn, ma, mb, M, N, K, L, s);
  }
  if (rc) return rc;
  if (p.split > 1) {
    Reduce r;
    r.ws = slabs;
    r.C = q.C;
    r.M = M;
    r.N = N;
    r.ldw = p.ldw;
    r.ldc = q.ldc;
    r.batches = nb;
    r.stride_c = q.stride_c;
    r.split = p.split;
    r.act = p.act;
    r.bias = q.bias;
    rc = launch_reduce(r, d, s);
  }
  return rc;
}

int run_problem(const Problem& q, const tilec_mm_cfg* cfg, void* workspace, size_t ws_bytes, void* stream) {
  int rc = check_problem(q, true, cfg ? cfg->flags : 0);
  if (rc) return rc;
  if (q.M == 0 || q.N == 0 || q.batch == 0) return TILEC_OK;
  DeviceInfo* d = nullptr;
  rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (q.K == 0) {
    const int act = cfg ? cfg->activation : 0;
    if (act < TILEC_MM_ACT_NONE || act > TILEC_MM_ACT_GELU) return TILEC_ERR_BAD_ARG;
    return launch_fill_zero(q.C, q.M, q.N, q.ldc, q.batch, q.stride_c, q.bias, act, *d, s);
  }
  for (int64_t b0 = 0; b0 < q.batch; b0 += kMaxBatch) {
    Problem c = q;
    c.batch = q.batch - b0 < kMaxBatch ? q.batch - b0 : kMaxBatch;
    c.A = q.A + b0 * q.stride_a;
    c.B = q.B + b0 * q.stride_b;
    c.C = q.C + b0 * q.stride_c;
    rc = run_chunk(*d, c, cfg, workspace, ws_bytes, s);
    if (rc) return rc;
  }
  return TILEC_OK;
}

size_t workspace_for(Problem q, const tilec_mm_cfg* cfg) {
  if (q.M <= 0 || q.N <= 0 || q.K <= 0 || q.batch <= 0) return 0;
  DeviceInfo* d = nullptr;
  if (current_device(&d)) return 0;
  // NULL operands: assume 16-byte aligned pointers (documented in the header).
  if (!q.A) q.A = reinterpret_cast<const float*>(uintptr_t(256));
  if (!q.B) q.B = reinterpret_cast<const float*>(uintptr_t(256));
  if (q.batch > kMaxBatch) q.batch = kMaxBatch;  // batches run in chunks of this size
  Plan p;
  if (make_plan(*d, q, cfg, &p)) return 0;
  return p.ws_bytes;
}

Problem single(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
               int64_t ldb, int64_t ldc) {
  Problem q;
  q.A = A;
  q.B = B;
  q.C = const_cast<float*>(C);
  q.M = M;
  q.N = N;
  q.K = K;
  q.lda = lda;
  q.ldb = ldb;
  q.ldc = ldc;
  return q;
}

Problem batched(const float* A, const float* B, const float* C, const float* bias, int64_t M, int64_t N, int64_t K,
                int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t stride_a, int64_t stride_b,
                int64_t stride_c) {
  Problem q = single(A, B, C, M, N, K, lda, ldb, ldc);
  q.bias = bias;
  q.batch = batch;
  q.stride_a = stride_a;
  q.stride_b = stride_b;
  q.stride_c = stride_c;
  return q;
}

}  // namespace
}  // namespace tilec

using namespace tilec;

extern "C" {

int tilec_mm_plan(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                  int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg, tilec_mm_cfg* out) {
  if (!out) return TILEC_ERR_BAD_ARG;
  const Problem q = single(A, B, C, M, N, K, lda, ldb, ldc);
  int rc = check_problem(q, /*need_c=*/false, cfg ? cfg->flags : 0);
  if (rc) return rc;
  DeviceInfo* d = nullptr;
  rc = current_device(&d);
  if (rc) return rc;
  Plan p;
  rc = make_plan(*d, q, cfg, &p);
  if (rc) return rc;
  std::memset(out, 0, sizeof(*out));
  out->variant = p.variant;
  out->split_k = p.split;
  const bool tensor = p.variant == TILEC_MM_TF32 || p.variant == TILEC_MM_3XTF32 ||
                      p.variant == TILEC_MM_3XTF32_MASKED || p.variant == TILEC_MM_3XMIXED;
  out->flags = p.flags | (p.sk ? TILEC_MM_STREAM_K : 0) |
               (tensor && !p.pair ? (p.bm == kTcBM64 ? TILEC_MM_TILE_M64 : TILEC_MM_TILE_M128) : 0);
  out->activation = p.act;
  return TILEC_OK;
}

size_t tilec_mm_workspace_bytes(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K,
                                int64_t lda, int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg) {
  return workspace_for(single(A, B, C, M, N, K, lda, ldb, ldc), cfg);
}

size_t tilec_mm_workspace_bytes_ex(const float* A, const float* B, const float* C, int64_t M, int64_t N, int64_t K,
                                   int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t stride_a,
                                   int64_t stride_b, int64_t stride_c, const tilec_mm_cfg* cfg) {
  return workspace_for(batched(A, B, C, nullptr, M, N, K, lda, ldb, ldc, batch, stride_a, stride_b, stride_c), cfg);
}

int tilec_mm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K, int64_t lda,
                 int64_t ldb, int64_t ldc, const tilec_mm_cfg* cfg, void* workspace, size_t ws_bytes,
                 void* stream) {
  return run_problem(single(A, B, C, M, N, K, lda, ldb, ldc), cfg, workspace, ws_bytes, stream);
}

int tilec_mm_f32_ex(const float* A, const float* B, float* C, const float* bias, int64_t M, int64_t N, int64_t K,
                    int64_t lda, int64_t ldb, int64_t ldc, int64_t batch, int64_t stride_a, int64_t stride_b,
                    int64_t stride_c, const tilec_mm_cfg* cfg, void* workspace, size_t ws_bytes, void* stream) {
  return run_problem(batched(A, B, C, bias, M, N, K, lda, ldb, ldc, batch, stride_a, stride_b, stride_c), cfg,
                     workspace, ws_bytes, stream);
}

int tilec_mm_set_table(const int32_t* rows, int32_t nrows) {
  if (nrows < 0 || (nrows > 0 && rows == nullptr)) return TILEC_ERR_BAD_ARG;
  for (int32_t r = 0; r < nrows; ++r) {
    const int32_t v = rows[r * 8 + 6];
    if (v < TILEC_MM_SIMT || v > TILEC_MM_3XMIXED || rows[r * 8 + 7] < 0) return TILEC_ERR_BAD_ARG;
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

int tilec_mm_set_wait_limit(int64_t limit_ns, void* stream) {
  if (limit_ns < 0) return TILEC_ERR_BAD_ARG;
  DeviceInfo* d = nullptr;
  const int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned long long v =
      static_cast<unsigned long long>(limit_ns) > kWaitLimitNs ? kWaitLimitNs : static_cast<unsigned long long>(limit_ns);
  if (cudaMemcpyToSymbolAsync(g_wait_limit_ns, &v, sizeof(v), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return TILEC_ERR_DEVICE;
  }
  return TILEC_OK;
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
  if (K == 0) return launch_fill_zero(C, M, N, ldc, 1, 0, nullptr, TILEC_MM_ACT_NONE, *d, s);
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
  } else {
    const double cta_s = cta_seconds(kSimtBM, bn, bn, K, kRateSimt, kBwPerSm);
    split = choose_split(mt * nt, d->sms, cta_s, double(slab) * 4.0, K / (int64_t(kSimtBK) * 4), 0,
                         /*one_wave=*/false);
    if (split > fit) split = fit < 1 ? 1 : fit;
  }
  // The slices that run: whole 16-deep K blocks per slice, so rounding can only lower the
  // count.  Only those must fit in the scratch (the library's own choice always does).
  const int64_t k_chunk = round_up(cdiv(K, split), kSimtBK);
  split = cdiv(K, k_chunk);
  if (split > 1 && split > fit) return TILEC_ERR_TOO_LARGE;

  Launch L;
  L.out = split > 1 ? scratch : C;
  L.ldo = split > 1 ? ldw : ldc;
  L.out_slab = split > 1 ? slab : 0;
  L.vec_out = split > 1 ? 1 : (aligned16(C) && (ldc % 4 == 0) ? 1 : 0);
  L.split = static_cast<int>(split);
  L.k_chunk = k_chunk;
  const bool vec = aligned16(A) && aligned16(B) && (lda % 4 == 0) && (ldb % 4 == 0);
  dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt), static_cast<unsigned>(split));
  rc = launch_simt(bn, vec, nullptr, grid, A, B, M, N, K, lda, ldb, 0, 0, L, d->sms, s);
  if (rc || split == 1) return rc;
  Reduce r;
  r.ws = scratch;
  r.C = C;
  r.M = M;
  r.N = N;
  r.ldw = ldw;
  r.ldc = ldc;
  r.split = static_cast<int>(split);
  return launch_reduce(r, *d, s);
}
