// tc_gemm.cuh -- tcgen05 (5th-gen tensor core) GEMM for sm_100a: variants TF32 and 3XTF32.
//
// Same contraction as the reference kernel tilec/ext.py:13-24: C[M,N] = A[M,K] . B[K,N],
// out-of-range operand elements read as 0.0 (TMA zero fill, matching ext.py:21-22),
// out-of-range outputs never stored (ext.py:24).
//
// One CTA owns a 128 x BN output tile (BN = 64/128/256) whose fp32 accumulator lives in
// TMEM (BN columns x 128 lanes).  192 threads, warp-specialised:
//   warp 0      TMA producer: A tile [128 x BK] K-major (128B/64B swizzle), B tile as
//               BN/32 slabs of [BK x 32] MN-major (128B swizzle); one mbarrier per stage.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=8 per
//               instruction) and tcgen05.commit to release stages / signal the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32x32b rows out of TMEM, masked stores to C (or to a
//               split-K workspace slab).  In 3XTF32 mode they first act as the "split"
//               stage: for every landed stage they write lo = x - hi(x) next to the raw
//               tile (hi(x) = x with the low 13 mantissa bits cleared; optionally written
//               back in place) so the MMA warp can issue  A_lo.B_hi + A_hi.B_lo + A_hi.B_hi.
//
// Operands: A = x1 row-major (K contiguous) -> K-major; B = x2 row-major (N contiguous)
// -> MN-major.  kind::tf32 accepts MN-major B, so x2 is consumed in place (no transpose).
// TMA needs 16-byte aligned bases and row strides (lda, ldb multiples of 4); the host
// routes anything else to the SIMT kernel.
#pragma once

#include "common.cuh"

namespace tilec {

constexpr int kTcBM = 128;
constexpr int kTcThreads = 192;

template <int BN, int BK, int STAGES, bool SPLIT3>
struct TcCfg {
  static constexpr int kABytes = kTcBM * BK * 4;
  static constexpr int kBBytes = BK * BN * 4;
  static constexpr int kStageBytes = (kABytes + kBBytes) * (SPLIT3 ? 2 : 1);
  static constexpr int kTxBytes = kABytes + kBBytes;
  static constexpr int kBarBytes = 1024;  // barriers + tmem slot + flags
  static constexpr int kSmemBytes = STAGES * kStageBytes + kBarBytes + 1024;  // +1024 alignment slack
  static constexpr uint32_t kALayout = (BK == 32) ? kLayoutSw128 : kLayoutSw64;
  static constexpr uint32_t kASbo = (BK == 32) ? 1024u : 512u;  // 8 rows x (BK*4) bytes
  static constexpr uint32_t kBLbo = BK * 128u;                  // stride between 32-column slabs
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  static_assert(BK == 16 || BK == 32, "BK");
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
};

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Bounded wait that ignores the abort flag (used while draining after an abort).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > 100000000ull) return;  // 100 ms
  }
}

// Grid: x = tile index (grouped raster, see tile_coords), z = K split.
template <int BN, int BK, int STAGES, bool SPLIT3, bool HI_EXPLICIT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   float* __restrict__ out, int M, int N, int64_t ldo, int64_t out_slab, int K, int k_chunk,
                   int m_tiles, int n_tiles, int group_m, int vec_out) {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  auto a_raw = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto b_raw = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes; };
  auto a_lo = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes; };
  auto b_lo = [&](int s) { return smem + s * Cfg::kStageBytes + 2 * Cfg::kABytes + Cfg::kBBytes; };

  uint8_t* bar_area = smem + STAGES * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + STAGES;
  uint64_t* split = empty + STAGES;
  uint64_t* acc_bar = split + STAGES;
  uint64_t* drain_bar = acc_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (blockDim.x != kTcThreads) {
    if (threadIdx.x == 0) record_status(TILEC_DEV_BAD_LAUNCH);
    return;
  }

  // Grouped rasterisation: consecutive CTAs sweep N inside a band of group_m M-tiles,
  // so a wave of CTAs shares a few A bands and B panels in L2.
  const int tile = blockIdx.x;
  const int band = tile / (group_m * n_tiles);
  const int first_m = band * group_m;
  const int band_rows = min(group_m, m_tiles - first_m);
  const int in_band = tile - band * group_m * n_tiles;
  const int tile_m = first_m + in_band % band_rows;
  const int tile_n = in_band / band_rows;
  const int m0 = tile_m * kTcBM;
  const int n0 = tile_n * BN;

  const int k_begin = blockIdx.z * k_chunk;
  const int k_end = min(K, k_begin + k_chunk);
  const int nkb = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
  out += static_cast<int64_t>(blockIdx.z) * out_slab;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&split[s], 128);
    }
    mbar_init(acc_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], Cfg::kTxBytes);
        const int k0 = k_begin + kb * BK;
        tma_load_2d(a_raw(s), &tmA, &full[s], k0, m0);
#pragma unroll
        for (int j = 0; j < BN / 32; ++j) tma_load_2d(b_raw(s) + j * BK * 128, &tmB, &full[s], n0 + 32 * j, k0);
        ++issued;
      }
      if (!ok) {
        // Let copies already in flight land before the CTA's shared memory goes away.
        for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb)
          mbar_drain(&full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_tf32(kTcBM, BN);
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(SPLIT3 ? &split[s] : &full[s], ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_hi_addr = smem_u32(a_raw(s));
        const uint32_t b_hi_addr = smem_u32(b_raw(s));
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t ad = make_smem_desc(a_hi_addr + kk * 32, 16, Cfg::kASbo, Cfg::kALayout);
          const uint64_t bd = make_smem_desc(b_hi_addr + kk * 1024, Cfg::kBLbo, 1024, kLayoutSw128);
          const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
          if constexpr (SPLIT3) {
            const uint64_t adl = make_smem_desc(smem_u32(a_lo(s)) + kk * 32, 16, Cfg::kASbo, Cfg::kALayout);
            const uint64_t bdl = make_smem_desc(smem_u32(b_lo(s)) + kk * 1024, Cfg::kBLbo, 1024, kLayoutSw128);
            umma_tf32(tmem, adl, bd, idesc, accum);  // small terms first
            umma_tf32(tmem, ad, bdl, idesc, 1u);
            umma_tf32(tmem, ad, bd, idesc, 1u);
          } else {
            umma_tf32(tmem, ad, bd, idesc, accum);
          }
        }
        umma_commit(&empty[s]);
      }
      if (ok) {
        if (nkb > 0) umma_commit(acc_bar);
      } else {
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ split + epilogue (warps 2..5)
    const int et = threadIdx.x - 64;  // 0..127
    bool ok = true;
    if constexpr (SPLIT3) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
        float4* src_a = reinterpret_cast<float4*>(a_raw(s));
        float4* dst_a = reinterpret_cast<float4*>(a_lo(s));
#pragma unroll 4
        for (int i = et; i < Cfg::kABytes / 16; i += 128) {
          const float4 x = src_a[i];
          const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
          dst_a[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
          if constexpr (HI_EXPLICIT) src_a[i] = h;
        }
        float4* src_b = reinterpret_cast<float4*>(b_raw(s));
        float4* dst_b = reinterpret_cast<float4*>(b_lo(s));
#pragma unroll 4
        for (int i = et; i < Cfg::kBBytes / 16; i += 128) {
          const float4 x = src_b[i];
          const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
          dst_b[i] = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
          if constexpr (HI_EXPLICIT) src_b[i] = h;
        }
        fence_proxy_async_smem();
        mbar_arrive(&split[s]);
      }
    }
    if (ok && nkb > 0) ok = mbar_wait(acc_bar, 0, abort_flag);
    if (ok) {
      tc_fence_after();
      const int q = warp & 3;  // TMEM lane quadrant this warp may access
      const int row = m0 + 32 * q + lane;
      float* crow = out + static_cast<int64_t>(row) * ldo;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        if (nkb > 0) {
          tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + c * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        if (row < M) {
          const int col = n0 + c * 32;
          if (vec_out && col + 31 < N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(crow + col + j) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                              __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col + j < N) crow[col + j] = __uint_as_float(r[j]);
          }
        }
      }
    }
  }

  __syncwarp();  // lanes 1..31 of warps 0/1 wait here for their lane 0
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace tilec
