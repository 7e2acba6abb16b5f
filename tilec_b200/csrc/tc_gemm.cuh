// tc_gemm.cuh -- tcgen05 (5th-gen tensor core) GEMM for sm_100a: variants TF32 and 3XTF32.
//
// Same contraction as the reference kernel tilec/ext.py:13-24: C[M,N] = A[M,K] . B[K,N],
// out-of-range operand elements read as 0.0 (TMA zero fill, matching ext.py:21-22),
// out-of-range outputs never stored (ext.py:24).
//
// One CTA owns a BM x BN output tile (BM = 128 or 64, BN = 64/128/256); fp32 accumulators
// live in TMEM.  BM = 64 (tcgen05.mma M = 64) serves products of at most 64 rows (batched
// 64-row slices, GEMV-like shapes) without computing a half-empty tile, and halves the
// partial-sum slabs of skinny split-K products.  Its accumulator holds tile row 16q + i in
// TMEM lane 32q + i (i < 16) of quadrant q, so each epilogue warp drains 16 rows.
// Warp-specialised:
//   warp 0      TMA producer: A tile [128 x BK] K-major (128B/64B swizzle), B tile as
//               BN/32 slabs of [BK x 32] MN-major (128B swizzle with 32-byte granules,
//               the only MN-major layout kind::tf32 reads); one mbarrier per stage.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=8 per
//               instruction) and tcgen05.commit to release stages / publish results.
//   warps 2..   epilogue.
//
// TF32 (SPLIT3 = false): one TMEM accumulator over all of K; 4 epilogue warps read it
// once (tcgen05.ld 32x32b) and store rows of C.
//
// 3XTF32 (SPLIT3 = true): C = A_lo.B_hi + A_hi.B_lo + A_hi.B_hi with hi(x) = x with the
// low 13 mantissa bits cleared and lo(x) = x - hi(x) (exact in fp32).  The tensor core
// reads only the top 19 bits of a tf32 operand, so the raw fp32 tile already *is* hi(x)
// (HI_EXPLICIT = true writes the masked copy anyway; a GPU test checks both agree bit
// for bit).  8 epilogue warps first act as the split stage (write lo next to each landed
// tile, fence.proxy.async, arrive), then as accumulator drains:
//   the tensor core accumulates with truncation, which biases long sums (relative error
//   grows ~linearly with K: 5.8e-5 at K = 8192 measured on B200 with one accumulator).
//   So the MMA accumulates K-chunks of KC_BLOCKS*BK into two ping-pong TMEM buffers, and
//   every finished chunk is added into fp32 registers (round-to-nearest FADD) by the
//   epilogue warps while the next chunk's MMAs run.  Each epilogue thread owns one row
//   (TMEM lane) and BN/2 columns.
//
// Operands: A = x1 row-major (K contiguous) -> K-major; B = x2 row-major (N contiguous)
// -> MN-major, consumed in place (no transpose).  `layout` (kOpAMN / kOpBK) flips either
// for operands stored transposed (x.t() views): A as MN-major slabs, B as a K-major tile.
// TMA needs 16-byte aligned bases and row strides (multiples of 4 elements); the host
// packs anything else into an aligned copy first.
#pragma once

#include "common.cuh"

namespace tilec {

constexpr int kTcBM = 128;

template <int BN, int BK, int STAGES, bool SPLIT3, int BM = kTcBM>
struct TcCfg {
  static_assert(BM == 128 || BM == 64, "BM");
  static constexpr int kEpiWarps = (SPLIT3 && BN >= 128) ? 8 : 4;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kRowsPerWarp = BM / 4;  // tile rows an epilogue warp drains (TMEM lanes 0..rows-1 of its quadrant)
  static constexpr int kABytes = BM * BK * 4;
  static constexpr int kBBytes = BK * BN * 4;
  // A stage holds the raw TMA tiles and, for 3XTF32, their lo(x) tiles next to them.  (A
  // separate, shallower lo ring was measured slower: it bounds how far the split stage can
  // run ahead of the MMA.)
  static constexpr int kStageBytes = (kABytes + kBBytes) * (SPLIT3 ? 2 : 1);
  static constexpr int kTxBytes = kABytes + kBBytes;
  static constexpr int kBarBytes = 1024;  // barriers + tmem slot + flags
  static constexpr int kSmemBytes = STAGES * kStageBytes + kBarBytes + 1024;  // +1024 alignment slack
  static constexpr uint32_t kALayout = (BK == 32) ? kLayoutSw128 : kLayoutSw64;
  static constexpr uint32_t kASbo = (BK == 32) ? 1024u : 512u;  // 8 rows x (BK*4) bytes
  static constexpr uint32_t kBLbo = BK * 128u;                  // stride between 32-column slabs
  static constexpr uint32_t kBSbo = 512u;                       // stride between 4-row K groups
  static constexpr uint32_t kTmemCols = SPLIT3 ? 2 * BN : BN;   // 3XTF32: two chunk buffers
  static constexpr int kColsPerThread = SPLIT3 ? BN / (kEpiWarps / 4) : 32;  // register totals per thread
  static constexpr int kChunkBlocks = 8;                        // K-blocks per promoted chunk
  static_assert(BK == 16 || BK == 32, "BK");
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "BN");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kColsPerThread % 32 == 0, "epilogue reads 32 TMEM columns at a time");
  // Output staging (reuses the stage buffers once every MMA has completed).
  static constexpr int kStoreCols = SPLIT3 ? kColsPerThread : 32;
  static constexpr int kStageFloatsPerWarp = 32 * (kStoreCols + 4);
  static_assert(kEpiWarps * kStageFloatsPerWarp * 4 <= STAGES * kStageBytes, "output staging");
};

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}


// Writes a 32-row x NC-column block, held one row per lane in v[], to rows row0.. and
// columns col0.. of `out` (masked at M and N).  The warp transposes it through its own
// staging buffer `stage` (32 x (NC + 4) floats; the pitch of NC + 4 keeps both passes
// free of bank conflicts) so that consecutive lanes store consecutive 16-byte pieces of
// one row: the warp writes whole row runs instead of 32 rows 16 bytes at a time.
//
// `bias` (per column, or nullptr) and `act` (kAct*) apply the fused epilogue on the way;
// the test is made once, outside the store loop (EPI instantiates the loop with it).
// ROWS: how many of the 32 staged rows to store (16 for a 64-row tile's warp).
template <int NC, bool EPI, int ROWS = 32>
__device__ __forceinline__ void store_rows_pass(const float* stage, float* out, int64_t ldo, int row0, int col0,
                                                int M, int N, int vec_out, int lane, const float* __restrict__ bias,
                                                int act) {
  constexpr int kPitch = NC + 4;
  constexpr int kChunks = NC / 4;  // 16-byte pieces per row
#pragma unroll 4
  for (int c = lane; c < ROWS * kChunks; c += 32) {
    const int r = c / kChunks, piece = c % kChunks;
    const int grow = row0 + r, gcol = col0 + 4 * piece;
    if (grow < M) {
      float4 x = *reinterpret_cast<const float4*>(stage + r * kPitch + 4 * piece);
      if constexpr (EPI) {
        float bv[4] = {0.f, 0.f, 0.f, 0.f};
        if (bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 4; ++j) bv[j] = gcol + j < N ? __ldg(bias + gcol + j) : 0.f;
        }
        x = make_float4(epilogue(x.x, bv[0], act), epilogue(x.y, bv[1], act), epilogue(x.z, bv[2], act),
                        epilogue(x.w, bv[3], act));
      }
      float* dst = out + static_cast<int64_t>(grow) * ldo + gcol;
      if (vec_out && gcol + 3 < N) {
        *reinterpret_cast<float4*>(dst) = x;
      } else {
        const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gcol + j < N) dst[j] = xs[j];
      }
    }
  }
}

template <int NC, int ROWS = 32>
__device__ __forceinline__ void store_rows_coalesced(float* stage, const float (&v)[NC], float* out, int64_t ldo,
                                                     int row0, int col0, int M, int N, int vec_out, int lane,
                                                     const float* __restrict__ bias = nullptr, int act = kActNone) {
  constexpr int kPitch = NC + 4;
#pragma unroll
  for (int j = 0; j < NC; j += 4)
    *reinterpret_cast<float4*>(stage + lane * kPitch + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  __syncwarp();
  if (bias != nullptr || act != kActNone)
    store_rows_pass<NC, true, ROWS>(stage, out, ldo, row0, col0, M, N, vec_out, lane, bias, act);
  else
    store_rows_pass<NC, false, ROWS>(stage, out, ldo, row0, col0, M, N, vec_out, lane, nullptr, kActNone);
  __syncwarp();
}

// Grid: x = tile index (grouped raster), y = batch index, z = K split (slabs of `out`).
// Operand tensor maps are 3-D (x inner, y outer, z batch); an operand's batch coordinate
// is 0 when it is shared by all batches (`shared` bit 0 = A, bit 1 = B).  `out` advances by out_batch per batch and out_slab per K slice; bias / act
// are the fused epilogue (only when C is written directly, i.e. without a K split).
// ANY_LAYOUT = false fixes `layout` to row-major operands at compile time: the flipped
// tile paths are then not in the kernel (keeping them there cost the common case 4-6 %
// on B200, measured at 8192^3 and 65536x8192x8192).
template <int BN, int BK, int STAGES, bool SPLIT3, bool HI_EXPLICIT, bool ANY_LAYOUT, int BM = kTcBM>
__global__ void __launch_bounds__(TcCfg<BN, BK, STAGES, SPLIT3, BM>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   float* __restrict__ out, int M, int N, int64_t ldo, int64_t out_slab, int K, int k_chunk,
                   int m_tiles, int n_tiles, int group_m, int vec_out, int layout_arg, int64_t out_batch,
                   const float* __restrict__ bias, int act, int shared) {
  using Cfg = TcCfg<BN, BK, STAGES, SPLIT3, BM>;
  constexpr int RW = Cfg::kRowsPerWarp;
  const int layout = ANY_LAYOUT ? layout_arg : 0;
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
  uint64_t* split = empty + STAGES;        // [STAGES] split warps -> MMA (3XTF32)
  uint64_t* chunk_full = split + STAGES;   // [2] MMA -> epilogue (3XTF32)
  uint64_t* chunk_empty = chunk_full + 2;  // [2] epilogue -> MMA (3XTF32)
  uint64_t* acc_bar = chunk_empty + 2;     // TF32: accumulator complete
  uint64_t* drain_bar = acc_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (blockDim.x != Cfg::kThreads) {
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
  const int kslice = static_cast<int>(blockIdx.z);
  const int batch = static_cast<int>(blockIdx.y);
  const int a_batch = (shared & 1) ? 0 : batch, b_batch = (shared & 2) ? 0 : batch;
  out += static_cast<int64_t>(blockIdx.z) * out_slab + static_cast<int64_t>(batch) * out_batch;
  const int m0 = tile_m * BM;
  const int n0 = tile_n * BN;

  const int k_begin = kslice * k_chunk;
  const int k_end = min(K, k_begin + k_chunk);
  const int nkb = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
  const int n_chunks = (nkb + KC - 1) / KC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&split[s], 32 * Cfg::kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&chunk_full[b], 1);
      mbar_init(&chunk_empty[b], Cfg::kEpiWarps);
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
  // Barrier init, TMEM allocation and descriptor prefetch overlap the previous kernel.
  pdl_wait();

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
        if (layout & kOpAMN) {
#pragma unroll
          for (int j = 0; j < BM / 32; ++j)
            tma_load_3d(a_raw(s) + j * BK * 128, &tmA, &full[s], m0 + 32 * j, k0, a_batch);
        } else {
          tma_load_3d(a_raw(s), &tmA, &full[s], k0, m0, a_batch);
        }
        if (layout & kOpBK) {
          tma_load_3d(b_raw(s), &tmB, &full[s], k0, n0, b_batch);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j)
            tma_load_3d(b_raw(s) + j * BK * 128, &tmB, &full[s], n0 + 32 * j, k0, b_batch);
        }
        ++issued;
      }
      if (ok) {
        // Tail: the MMA's release of the last fills has arrived before the CTA exits.
        for (int kb = nkb - STAGES < 0 ? 0 : nkb - STAGES; kb < nkb; ++kb)
          if (!mbar_wait(&empty[kb % STAGES], (kb / STAGES) & 1, abort_flag)) { ok = false; break; }
      }
      if (!ok) {
        // Gave up (here or elsewhere): let the last fills' copies land before the CTA's
        // shared memory goes away (a fill that already landed passes at once).
        for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb)
          mbar_drain(&full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const bool a_mn = (layout & kOpAMN) != 0, b_k = (layout & kOpBK) != 0;
      const uint32_t idesc = make_idesc_tf32(BM, BN, a_mn, !b_k);
      // K step kk (8 elements) of a tile: 32 bytes along a K-major row, or 8 rows of 128
      // bytes in an MN-major slab.
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
        const int chunk = SPLIT3 ? kb / KC : 0;
        const bool chunk_start = SPLIT3 ? (kb % KC == 0) : (kb == 0);
        const uint32_t dcol = SPLIT3 ? static_cast<uint32_t>((chunk & 1) * BN) : 0u;
        if (SPLIT3 && chunk_start && chunk >= 2) {
          // Reuse of this buffer: its previous chunk must have been drained.
          if (!mbar_wait(&chunk_empty[chunk & 1], ((chunk >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
        }
        if (!mbar_wait(SPLIT3 ? &split[s] : &full[s], ph, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_hi_addr = smem_u32(a_raw(s));
        const uint32_t b_hi_addr = smem_u32(b_raw(s));
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t ad = desc_a(a_hi_addr, kk);
          const uint64_t bd = desc_b(b_hi_addr, kk);
          const uint32_t accum = (chunk_start && kk == 0) ? 0u : 1u;
          if constexpr (SPLIT3) {
            const uint64_t adl = desc_a(smem_u32(a_lo(s)), kk);
            const uint64_t bdl = desc_b(smem_u32(b_lo(s)), kk);
            umma_tf32(tmem + dcol, adl, bd, idesc, accum);  // small terms first
            umma_tf32(tmem + dcol, ad, bdl, idesc, 1u);
            umma_tf32(tmem + dcol, ad, bd, idesc, 1u);
          } else {
            umma_tf32(tmem, ad, bd, idesc, accum);
          }
        }
        umma_commit(&empty[s]);
        if (SPLIT3 && (kb % KC == KC - 1 || kb == nkb - 1)) umma_commit(&chunk_full[chunk & 1]);
      }
      if (ok && !SPLIT3 && nkb > 0) umma_commit(acc_bar);
      // Every MMA issued here completes before this thread leaves its role, on every path:
      // an epilogue that gave up must not let the CTA free TMEM or exit under a running MMA.
      if (nkb > 0) {
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int e = warp - 2;                  // 0 .. kEpiWarps-1
    const int q = warp & 3;                  // TMEM lane quadrant this warp may access
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    bool ok = true;

    if constexpr (SPLIT3) {
      constexpr int COLS = Cfg::kColsPerThread;   // BN / 2
      const int h = e >> 2;                       // which half of the BN columns
      const int et = threadIdx.x - 64;            // 0 .. 255
      float tot[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) tot[j] = 0.f;

      auto drain = [&](int c) {
        const int buf = c & 1;
        if (!mbar_wait(&chunk_full[buf], (c >> 1) & 1, abort_flag)) return false;
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
        if (lane == 0) mbar_arrive(&chunk_empty[buf]);
        return true;
      };

      constexpr int kLag = 2;  // drain chunk c-1 after splitting this many blocks of chunk c
      int drained = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
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
        mbar_arrive(&split[s]);
        // Chunk c-1 is finished once the MMAs of the first blocks of chunk c are queued.
        if (kb % KC == (kLag < KC ? kLag : KC - 1) && kb / KC >= 1 && drained < kb / KC) {
          if (!drain(drained)) { ok = false; break; }
          ++drained;
        }
      }
      while (ok && drained < n_chunks) {
        if (!drain(drained)) { ok = false; break; }
        ++drained;
      }

      // Every MMA has completed (the last chunk was drained), so the stage buffers are free.
      pdl_launch_dependents();
      if (ok) {
        float* stage = reinterpret_cast<float*>(smem) + e * Cfg::kStageFloatsPerWarp;
        store_rows_coalesced<COLS, RW>(stage, tot, out, ldo, m0 + RW * q, n0 + h * COLS, M, N, vec_out, lane, bias,
                                       act);
      }
    } else {
      if (nkb > 0) ok = mbar_wait(acc_bar, 0, abort_flag);
      pdl_launch_dependents();
      if (ok) {
        tc_fence_after();
        float* stage = reinterpret_cast<float*>(smem) + e * Cfg::kStageFloatsPerWarp;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          if (nkb > 0) {
            tmem_ld_32x32b_x32(tmem + lane_base + c * 32, r);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = 0u;
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          store_rows_coalesced<32, RW>(stage, v, out, ldo, m0 + RW * q, n0 + c * 32, M, N, vec_out, lane, bias, act);
        }
      }
    }
  }

  __syncwarp();  // lanes 1..31 of warps 0/1 wait here for their lane 0
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  // A role gave up: every copy and MMA of this CTA has landed (drained above), so the
  // epilogue warps overwrite the CTA's tile with NaN, each the 32 rows x cols it stores.
  if (*abort_flag && warp >= 2) {
    constexpr int kWarpCols = BN / (Cfg::kEpiWarps / 4);
    const int e = warp - 2;
    poison_rows(out, ldo, m0 + RW * (warp & 3), RW, n0 + (e >> 2) * kWarpCols, kWarpCols, M, N, lane);
  }
}

}  // namespace tilec
