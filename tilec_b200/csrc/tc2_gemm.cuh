// tc2_gemm.cuh -- 3XTF32 GEMM on a CTA pair (tcgen05 cta_group::2), sm_100a.
//
// Same contraction and edge semantics as tc_gemm.cuh (tilec/ext.py:13-24: zero-filled
// out-of-range operands, masked stores), same hi/lo split and K-chunk promotion; the
// difference is the MMA shape.  Two CTAs of a cluster (2,1,1) own a 256 x BN output tile:
// CTA r holds A rows [128r, 128r+128) and the BN/2 columns [r*BN/2, (r+1)*BN/2) of B, and
// the leader (r = 0) issues tcgen05.mma.cta_group::2 with M = 256, N = BN, which reads A
// and B from both CTAs' shared memory and writes each CTA's 128 rows of the accumulator
// into that CTA's TMEM.  Per SM the tensor core then reads 8 KB of operands per K=8 step
// instead of 12 KB (1-CTA M=128 x N=256), which is what keeps the shared-memory port
// (TMA writes + split stage + MMA operand reads) below its bandwidth.
//
// Data movement stays local: each CTA TMA-loads only its own halves into its own shared
// memory with its own mbarriers (plain cta_group::1 TMA, no multicast).  Cross-CTA
// signalling:
//   split[s]      (leader)  <- 8 split warps of each CTA, mbarrier arrive on the leader's barrier (release.cta)
//   empty[s]      (each)    <- leader's tcgen05.commit, multicast to the same barrier in both CTAs
//   chunk_full[b] (each)    <- leader's tcgen05.commit, multicast to both CTAs
//   chunk_empty[b](leader)  <- 8 epilogue warps of each CTA after draining their TMEM rows
// TMEM is allocated and freed by warp 1 of both CTAs together (cta_group::2).  A cluster
// barrier after set-up and another before teardown keep either CTA from touching the
// peer's barriers before they exist or after they are gone.
#pragma once

#include "common.cuh"
#include "tc_gemm.cuh"

// The split warps and the epilogue warps signal the leader CTA with a remote mbarrier
// arrive whose release is at CTA scope, after fence.proxy.async.shared::cta has made the
// warp's shared-memory writes visible to the async proxy (the tensor core reads them only
// after the leader observes the arrive).  Measured alternatives, slower on B200: the same
// arrive with a cluster-scope release (a cluster memory barrier per warp and stage: 147
// vs 245 TFLOP/s at 8192^3), and eight local arrives followed by one cluster-scope release
// per stage (139 TFLOP/s).

namespace tilec {

// SPLIT3: 3XTF32 (raw + lo tiles per stage, K-chunk promotion every 128 of K through two
// TMEM buffers); otherwise TF32 (raw tiles only, one accumulator over all of K, the split
// warps only relay "stage full" to the leader).  BK: K per stage, 32 in every pair kernel
// (BKX = 16 builds the 16-deep form).  With raw + lo tiles a 32-deep stage is 64 KB, so
// 3XTF32 runs 3 stages: half the per-stage handshakes of 6 stages of 16 for the same depth
// in K, 282.7 -> 300.0 TFLOP/s at 8192^3 and 246.7 -> 264.4 on 65536x8192x8192, same box.
// SK: the stream-K kernel (tc2_sk.cuh) on the same stages: two TMEM buffers in both modes
// (a segment's sums are read out while the next segment's MMAs run), a smaller barrier
// area and a 32 x 33 float block per epilogue warp for stores made while the stages
// still stream.  SK = false is the one-pair-per-tile kernel below.
template <int BN, int STAGES, bool SPLIT3 = true, bool SK = false, int BKX = 0>
struct Tc2Cfg {
  static constexpr int BK = BKX ? BKX : 32;
  static_assert(BK == 16 || BK == 32, "BK");
  static constexpr int kBNHalf = BN / 2;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kABytes = 128 * BK * 4;          // own A rows
  static constexpr int kBBytes = BK * kBNHalf * 4;      // own half of B
  static constexpr int kStageBytes = (SPLIT3 ? 2 : 1) * (kABytes + kBBytes);  // raw (+ lo)
  static constexpr int kTxBytes = kABytes + kBBytes;
  static constexpr int kBarBytes = SK ? 256 : 1024;
  static constexpr int kBlockPitch = 33;                // 32 x 33 floats: conflict-free both ways
  static constexpr int kBlockBytes = SK ? kEpiWarps * 32 * kBlockPitch * 4 : 0;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024 + kBarBytes + kBlockBytes;
  static constexpr uint32_t kASbo = 8u * BK * 4u;       // 8 rows x BK*4 bytes (K-major)
  static constexpr uint32_t kALayout = BK == 32 ? kLayoutSw128 : kLayoutSw64;  // BK*4-byte rows
  static constexpr uint32_t kBLbo = BK * 128u;          // stride between 32-column slabs
  static constexpr uint32_t kBSbo = 512u;               // stride between 4-row K groups
  static constexpr uint32_t kTmemCols = (SPLIT3 || SK) ? 2 * BN : BN;  // chunk buffers of BN columns
  static constexpr int kColsPerThread = BN / 2;
  static constexpr int kChunkBlocks = SPLIT3 ? 128 / BK : (1 << 30);  // TF32: one chunk (per segment)
  static constexpr int kPartialFloats = 2 * kEpiWarps * 32 * kColsPerThread;  // one pair's tile
  static_assert(BN == 256 || BN == 128, "BN");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kEpiWarps * 32 * (kColsPerThread + 4) * 4 <= STAGES * kStageBytes, "output staging");
  static_assert((3 * STAGES + 5) * 8 + 8 <= kBarBytes, "barrier area");  // mbarriers + TMEM slot + abort flag
};

// K per stage of the one-pair-per-tile kernel (every variant): 32.
template <bool SPLIT3, bool MIXED>
constexpr int kTc2Bk = 32;

// Operand readers for the mixed split (MIXED below): 8 consecutive k of one row of an fp32
// stage tile of depth BK as TMA left it.
//   K-major tile ([rows x BK] fp32, BK*4-byte rows, BK*4-byte swizzle: the 16-byte granule
//   index is XORed with (row >> 1) & 3 for 64-byte rows, with row & 7 for 128-byte rows):
//   chunk kc holds k 8kc .. 8kc+7.
template <int BK>
__device__ __forceinline__ void read_kmajor8(const uint8_t* tile, int r, int kc, float (&v)[8]) {
  const uint8_t* row = tile + r * (BK * 4);
  const int sw = BK == 32 ? (r & 7) : ((r >> 1) & 3);
  const float4 x0 = *reinterpret_cast<const float4*>(row + 16 * ((2 * kc) ^ sw));
  const float4 x1 = *reinterpret_cast<const float4*>(row + 16 * ((2 * kc + 1) ^ sw));
  v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
  v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
}
// 8 consecutive MN indices 8q..8q+7 at one k of an MN-major fp32 stage tile (slabs of
// [BK k x 32] fp32 BK*128 bytes apart, 128-byte rows with 32-byte granules: granule index,
// address bits 5-6, XORed with bits 7-8, i.e. with k & 3): one granule, two 16-byte loads.
// Odd slabs read their upper half first, so a quarter warp's eight loads cover all 32 banks.
template <int BK>
__device__ __forceinline__ void read_mnmajor_chunk8(const uint8_t* tile, int k, int q, float (&v)[8]) {
  const int j = q >> 2, h0 = j & 1;
  const uint8_t* g = tile + j * (BK * 128) + k * 128 + 32 * ((q & 3) ^ (k & 3));
  const float4 x0 = *reinterpret_cast<const float4*>(g + 16 * h0);
  const float4 x1 = *reinterpret_cast<const float4*>(g + 16 * (h0 ^ 1));
  const float4 lo = h0 ? x1 : x0, hi = h0 ? x0 : x1;
  v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
  v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
}
// Byte offset of MN indices 8q..8q+7 at k (16 bytes) in a [BK x 128] bf16 tile laid out
// MN-major with the 128-byte swizzle: 64-element (128-byte) rows along MN, the 16-byte chunk
// index XORed with k & 7; the two 64-wide MN halves 1 KB apart (LBO), 8-row K groups 2 KB
// apart (SBO).  A quarter warp storing one k's 8 chunks fills one 128-byte row.
__device__ __forceinline__ uint32_t bf16_mn_tile_offset(int k, int q) {
  return (k >> 3) * 2048 + (q >> 3) * 1024 + (k & 7) * 128 + (((q & 7) ^ (k & 7)) << 4);
}
// Byte offset of row r, chunk kc (k 8kc .. 8kc+7, 16 bytes) in a [128 x BK] bf16 tile laid
// out K-major with the BK*2-byte swizzle, as the kind::f16 descriptors describe it: BK*2-byte
// rows, the 16-byte chunk index XORed with (r >> 2) & 1 (32-byte rows) or (r >> 1) & 3
// (64-byte rows); 8-row groups BK*16 bytes apart (SBO).  A quarter warp storing 8 consecutive
// rows of one chunk covers all 32 banks.  (A no-swizzle layout with the K halves 2 KB apart
// measured 3 % slower at BK 16.)
template <int BK>
__device__ __forceinline__ uint32_t bf16_tile_offset(int r, int kc) {
  return BK == 32 ? r * 64 + 16 * (kc ^ ((r >> 1) & 3)) : r * 32 + 16 * (kc ^ ((r >> 2) & 1));
}

// M = 256 (pair), N = BN, kind::tf32; A K-major and B MN-major unless `layout` flips
// them (kOpAMN / kOpBK, operands stored transposed).
// ANY_LAYOUT as in tc_gemm_kernel.
// MIXED (with SPLIT3): the 3-product split with the two cross terms on the bf16 pipe.  With
// h(x) the tensor core's tf32 reading of x and l(x) = x - h(x) (exact in fp32),
//   a.b = h(a).h(b) + a.l(b) + l(a).h(b)      (exactly),
// and the cross terms are about 2^-11 of the product, so their operands need only bf16's
// 8 bits: h.h runs as two kind::tf32 MMAs (K = 8) on the raw tiles, a.l(b) and l(a).h(b) as
// one kind::f16 MMA each (K = 16) on bf16 tiles the split warps write.  Per 16 of K that is
// 4 tensor slots of a tf32 K=8 MMA's length instead of 6.  Rounding the cross-term operands
// to bf16 (relative error <= 2^-8 each, on terms below 2^-10 of the product) adds at most
// 3 * 2^-18 relative error per product (2^-18 from bf16(a) and from bf16(h(b)), 2^-19 from
// each rounded l()), about 1e-6 rms on random data.
template <int BN, int STAGES, bool SPLIT3, bool HI_EXPLICIT, bool ANY_LAYOUT, bool MIXED = false>
__global__ void __launch_bounds__(Tc2Cfg<BN, STAGES, SPLIT3, false, kTc2Bk<SPLIT3, MIXED>>::kThreads, 1)
    tc2_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    float* __restrict__ out, int M, int N, int64_t ldo, int64_t out_slab, int K, int k_chunk,
                    int mp_tiles, int n_tiles, int group_m, int vec_out, int layout_arg, int64_t out_batch,
                    const float* __restrict__ bias, int act, int shared) {
  const int layout = ANY_LAYOUT ? layout_arg : 0;
  using Cfg = Tc2Cfg<BN, STAGES, SPLIT3, false, kTc2Bk<SPLIT3, MIXED>>;
  static_assert(!MIXED || (SPLIT3 && !HI_EXPLICIT && BN == 256 && (Cfg::BK == 16 || Cfg::BK == 32)),
                "mixed split: 3-product stages, 128-row tiles");
  constexpr int BK = Cfg::BK;
  constexpr int KC = Cfg::kChunkBlocks;
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
  uint64_t* chunk_full = split + STAGES;
  uint64_t* chunk_empty = chunk_full + 2;
  uint64_t* drain_bar = chunk_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (blockDim.x != Cfg::kThreads) {  // uniform across the cluster: every CTA returns
    if (threadIdx.x == 0) record_status(TILEC_DEV_BAD_LAUNCH);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  // Grouped raster over pair tiles (256 x BN).
  const int tile = blockIdx.x >> 1;
  const int band = tile / (group_m * n_tiles);
  const int first_m = band * group_m;
  const int band_rows = min(group_m, mp_tiles - first_m);
  const int in_band = tile - band * group_m * n_tiles;
  const int tile_m = first_m + in_band % band_rows;
  const int tile_n = in_band / band_rows;
  const int m0 = tile_m * 256 + static_cast<int>(rank) * 128;  // this CTA's rows
  const int n0 = tile_n * BN;                                   // the pair's columns
  const int nb0 = n0 + static_cast<int>(rank) * Cfg::kBNHalf;   // this CTA's B columns

  const int k_begin = blockIdx.z * k_chunk;
  const int k_end = min(K, k_begin + k_chunk);
  const int nkb = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
  const int n_chunks = (nkb + KC - 1) / KC;
  const int batch = static_cast<int>(blockIdx.y);
  const int a_batch = (shared & 1) ? 0 : batch, b_batch = (shared & 2) ? 0 : batch;
  out += static_cast<int64_t>(blockIdx.z) * out_slab + static_cast<int64_t>(batch) * out_batch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&split[s], 2 * Cfg::kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&chunk_full[b], 1);
      mbar_init(&chunk_empty[b], 2 * Cfg::kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncwarp();
  cluster_sync();  // both CTAs' barriers exist before anyone arrives remotely
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Barrier init, TMEM allocation and descriptor prefetch overlap the previous kernel.
  pdl_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait_cluster(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[s], Cfg::kTxBytes);
        const int k0 = k_begin + kb * BK;
        if (layout & kOpAMN) {
#pragma unroll
          for (int j = 0; j < 128 / 32; ++j)
            tma_load_3d(a_raw(s) + j * BK * 128, &tmA, &full[s], m0 + 32 * j, k0, a_batch);
        } else {
          tma_load_3d(a_raw(s), &tmA, &full[s], k0, m0, a_batch);
        }
        if (layout & kOpBK) {
          tma_load_3d(b_raw(s), &tmB, &full[s], k0, nb0, b_batch);
        } else {
#pragma unroll
          for (int j = 0; j < Cfg::kBNHalf / 32; ++j)
            tma_load_3d(b_raw(s) + j * BK * 128, &tmB, &full[s], nb0 + 32 * j, k0, b_batch);
        }
        ++issued;
      }
      if (ok) {
        // Producer tail: wait for the release (leader's commit) of each of the last fills,
        // so no arrival targets this CTA's barriers after it exits.
        for (int kb = nkb - STAGES < 0 ? 0 : nkb - STAGES; kb < nkb; ++kb)
          if (!mbar_wait_cluster(&empty[kb % STAGES], (kb / STAGES) & 1, abort_flag)) { ok = false; break; }
      }
      if (!ok) {
        // Gave up: let the last fills' copies land (a landed fill passes at once).
        for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb)
          mbar_drain(&full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA only)
    if (leader && lane == 0) {
      const bool a_mn = (layout & kOpAMN) != 0, b_k = (layout & kOpBK) != 0;
      const uint32_t idesc = make_idesc_tf32(256, BN, a_mn, !b_k);
      auto desc_a = [&](uint32_t base, int kk) {
        return a_mn ? make_smem_desc(base + kk * 1024, Cfg::kBLbo, Cfg::kBSbo, kLayoutSw128Base32)
                    : make_smem_desc(base + kk * 32, 16, Cfg::kASbo, Cfg::kALayout);
      };
      auto desc_b = [&](uint32_t base, int kk) {
        return b_k ? make_smem_desc(base + kk * 32, 16, Cfg::kASbo, Cfg::kALayout)
                   : make_smem_desc(base + kk * 1024, Cfg::kBLbo, Cfg::kBSbo, kLayoutSw128Base32);
      };
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        const int chunk = kb / KC;
        const bool chunk_start = (kb % KC == 0);
        const uint32_t dcol = static_cast<uint32_t>((chunk & 1) * BN);
        if (chunk_start && chunk >= 2) {
          if (!mbar_wait_cluster(&chunk_empty[chunk & 1], ((chunk >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
        }
        if (!mbar_wait_cluster(&split[s], ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_hi = smem_u32(a_raw(s)), b_hi = smem_u32(b_raw(s));
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t ad = desc_a(a_hi, kk), bd = desc_b(b_hi, kk);
          const uint32_t accum = (chunk_start && kk == 0) ? 0u : 1u;
          if constexpr (MIXED) {
            if (kk == 0) {  // the stage's cross terms first: two bf16 MMAs (K = 16) per 16 of K
              constexpr uint32_t kTile = 128 * BK * 2;  // one bf16 tile
              const uint32_t la = smem_u32(a_lo(s)), lb = smem_u32(b_lo(s));
              const uint32_t idesc16 = make_idesc_bf16(256, BN, a_mn, !b_k);
              // K step h (16 of K): 32 bytes along a K-major row, or two 8-row K groups of an
              // MN-major tile.
              auto d16 = [](uint32_t base, bool mn, int h) {
                return mn ? make_smem_desc(base + h * 4096, 1024, 2048, kLayoutSw128)
                          : make_smem_desc(base + h * 32, 16, BK * 16, BK == 32 ? kLayoutSw64 : kLayoutSw32);
              };
#pragma unroll
              for (int h = 0; h < BK / 16; ++h) {
                umma_bf16_pair(tmem + dcol, d16(la, a_mn, h), d16(lb, !b_k, h), idesc16,
                               h == 0 ? accum : 1u);                                             // a . l(b)
                umma_bf16_pair(tmem + dcol, d16(la + kTile, a_mn, h), d16(lb + kTile, !b_k, h), idesc16,
                               1u);                                                              // l(a) . h(b)
              }
            }
            umma_tf32_pair(tmem + dcol, ad, bd, idesc, 1u);
          } else if constexpr (SPLIT3) {
            const uint64_t adl = desc_a(smem_u32(a_lo(s)), kk), bdl = desc_b(smem_u32(b_lo(s)), kk);
            umma_tf32_pair(tmem + dcol, adl, bd, idesc, accum);  // small terms first
            umma_tf32_pair(tmem + dcol, ad, bdl, idesc, 1u);
            umma_tf32_pair(tmem + dcol, ad, bd, idesc, 1u);
          } else {
            umma_tf32_pair(tmem + dcol, ad, bd, idesc, accum);
          }
        }
        const uint32_t e_local = smem_u32(&empty[s]);
        umma_commit_pair_both(e_local);
        if (kb % KC == KC - 1 || kb == nkb - 1) {
          const uint32_t c_local = smem_u32(&chunk_full[chunk & 1]);
          umma_commit_pair_both(c_local);
        }
      }
      // Every MMA issued here completes before this thread leaves its role, on every path
      // (an epilogue that gave up must not let the pair free TMEM or exit under a running
      // MMA, which also reads the peer CTA's shared memory).
      umma_commit_pair(smem_u32(drain_bar));
      mbar_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ split + promotion epilogue (both CTAs)
    constexpr int COLS = Cfg::kColsPerThread;
    const int e = warp - 2;
    const int q = warp & 3;
    const int h = e >> 2;
    const int et = threadIdx.x - 64;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    bool ok = true;
    float tot[COLS];
#pragma unroll
    for (int j = 0; j < COLS; ++j) tot[j] = 0.f;

    auto drain = [&](int c) {
      const int buf = c & 1;
      if (!mbar_wait_cluster(&chunk_full[buf], (c >> 1) & 1, abort_flag)) return false;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < COLS / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_base + buf * BN + h * COLS + j * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) tot[j * 32 + i] += __uint_as_float(r[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(mapa_shared(smem_u32(&chunk_empty[buf]), 0));
      return true;
    };

    constexpr int kLag = 2;
    int drained = 0;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (kb / STAGES) & 1;
      if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
      if constexpr (MIXED) {
        // Each operand tile's bf16 copies keep its major-ness.  BK / 16 units per thread.
        // K-major: (row, 8-k chunk) units, warps 0-3 of the eight taking the even chunks and
        // warps 4-7 the odd ones for 32 consecutive rows each; MN-major: (k, 8 MN indices)
        // chunks, 16 per k.  Either way each quarter warp's 16-byte loads and stores cover all
        // 32 banks.
        constexpr uint32_t kTile = 128 * BK * 2;  // one bf16 tile
        auto to_bf16 = [&](const uint8_t* raw, uint8_t* dst, bool mn, bool lhs, int u) {
          float v[8];
          uint32_t off;
          if (mn) {
            const int k = (et >> 4) + 16 * u, q = et & 15;
            read_mnmajor_chunk8<BK>(raw, k, q, v);
            off = bf16_mn_tile_offset(k, q);
          } else {
            const int r = (e & 3) * 32 + lane, kc = (e >> 2) + 2 * u;
            read_kmajor8<BK>(raw, r, kc, v);
            off = bf16_tile_offset<BK>(r, kc);
          }
          uint4 o0, o1;
          uint32_t* p0 = &o0.x;
          uint32_t* p1 = &o1.x;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float x0 = v[2 * i], x1 = v[2 * i + 1];
            const float h0 = tf32_hi(x0), h1 = tf32_hi(x1);
            if (lhs) {  // A side: bf16(a), bf16(l(a))
              p0[i] = pack_bf16x2(x0, x1);
              p1[i] = pack_bf16x2(x0 - h0, x1 - h1);
            } else {    // B side: bf16(l(b)), bf16(h(b))
              p0[i] = pack_bf16x2(x0 - h0, x1 - h1);
              p1[i] = pack_bf16x2(h0, h1);
            }
          }
          *reinterpret_cast<uint4*>(dst + off) = o0;
          *reinterpret_cast<uint4*>(dst + kTile + off) = o1;
        };
#pragma unroll
        for (int u = 0; u < BK / 16; ++u) {
          to_bf16(a_raw(s), a_lo(s), (layout & kOpAMN) != 0, true, u);
          to_bf16(b_raw(s), b_lo(s), (layout & kOpBK) == 0, false, u);
        }
        fence_proxy_async_smem();
      } else if constexpr (SPLIT3) {
        float4* src_a = reinterpret_cast<float4*>(a_raw(s));
        float4* dst_a = reinterpret_cast<float4*>(a_lo(s));
#pragma unroll
        for (int i = et; i < Cfg::kABytes / 16; i += 32 * Cfg::kEpiWarps) {
          const float4 x = src_a[i];
          const float4 hv = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
          dst_a[i] = make_float4(x.x - hv.x, x.y - hv.y, x.z - hv.z, x.w - hv.w);
          if constexpr (HI_EXPLICIT) src_a[i] = hv;
        }
        float4* src_b = reinterpret_cast<float4*>(b_raw(s));
        float4* dst_b = reinterpret_cast<float4*>(b_lo(s));
#pragma unroll
        for (int i = et; i < Cfg::kBBytes / 16; i += 32 * Cfg::kEpiWarps) {
          const float4 x = src_b[i];
          const float4 hv = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
          dst_b[i] = make_float4(x.x - hv.x, x.y - hv.y, x.z - hv.z, x.w - hv.w);
          if constexpr (HI_EXPLICIT) src_b[i] = hv;
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(mapa_shared(smem_u32(&split[s]), 0));
      if (kb % KC == (kLag < KC ? kLag : KC - 1) && kb / KC >= 1 && drained < kb / KC) {
        if (!drain(drained)) { ok = false; break; }
        ++drained;
      }
    }
    while (ok && drained < n_chunks) {
      if (!drain(drained)) { ok = false; break; }
      ++drained;
    }

    // Every MMA of the pair has completed (the last chunk was drained), so this CTA's stage
    // buffers are free for the output staging.
    pdl_launch_dependents();
    if (ok) {
      float* stage = reinterpret_cast<float*>(smem) + e * 32 * (COLS + 4);
      store_rows_coalesced<COLS>(stage, tot, out, ldo, m0 + 32 * q, n0 + h * COLS, M, N, vec_out, lane, bias, act);
    }
  }

  __syncwarp();
  pdl_launch_dependents();
  tc_fence_before();
  cluster_sync();  // every remote arrive / commit targeting either CTA has landed
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::kTmemCols);
  }
  // This CTA gave up: both CTAs' copies and MMAs have landed (cluster barrier above), so
  // its epilogue warps overwrite its 128 rows of the tile with NaN.
  if (*abort_flag && warp >= 2) {
    const int e = warp - 2;
    poison_rows(out, ldo, m0 + 32 * (warp & 3), 32, n0 + (e >> 2) * Cfg::kColsPerThread, Cfg::kColsPerThread, M,
                N, lane);
  }
}

}  // namespace tilec
