// tc2_sk.cuh -- stream-K form of the CTA-pair tf32 / 3XTF32 GEMM (tc2_gemm.cuh), sm_100a.
//
// A grid of one pair per 256 x 256 tile leaves pair slots idle in its last wave whenever
// the tile count is not a multiple of the slots (T = 81 tiles on 74 slots: two waves,
// the second 7 % full).  This kernel launches exactly P pairs, the slots that are
// resident at once, and gives each an equal share of the work:
//   * tiles [0, dp_tiles) -- the complete waves but the last -- go whole to pairs
//     p, p + P, ... as in the one-pair-per-tile kernel;
//   * the k-blocks of tiles [dp_tiles, tiles) (P to 2P - 1 tiles) are split into P equal
//     contiguous ranges of (tile, k-block) units, tile-major.
// A pair walks its units as segments (a tile and a k-block range); the pipeline stages and
// the two TMEM chunk buffers count on across segments, so the pipeline does not drain
// between them.  A segment that does not end at its tile's last k-block is a partial: the
// pair writes its fp32 sums to its slot of the workspace and raises one ready flag per
// epilogue warp.  The pair that holds the last k-block adds the partials of the
// lower-numbered pairs sharing the tile, in pair order (a fixed order: results do not
// depend on timing), then stores the tile with the fused epilogue.  A pair visits its
// stream-K tiles last one first, so its one partial is its first piece of work: a wait is
// only ever on a lower-numbered pair, for the work it started with.  The host launches no
// more pairs than fit at once; and should other kernels hold SMs (another stream), a
// resident pair still only waits on lower-numbered pairs, which the block scheduler has
// placed no later than it, so waits end either way.  Every wait is bounded all the same
// (kWaitLimitNs, then TILEC_DEV_TIMEOUT and an orderly unwind).
//
// Roles, barriers, TMEM and the hi/lo split are those of tc2_gemm_kernel (see there).
#pragma once

#include "common.cuh"
#include "tc2_gemm.cuh"

namespace tilec {

// Stream-K arguments of tc2_sk_kernel.
struct Tc2StreamK {
  float* partial;       // [pairs][2 CTAs][8 warps][BN/8 x 32 float4]: one partial tile per pair
  int* flags;           // [pairs][2 CTAs][8 warps] ready flags, zeroed before every launch
  int dp_tiles;         // tiles [0, dp_tiles): whole tiles, pair p taking p, p + P, ...
  int tiles;            // tiles of all batches; [dp_tiles, tiles) are shared out by k-block
  int tiles_per_batch;  // tile t belongs to batch t / tiles_per_batch
  int pad;
};

// Clears the stream-K ready flags of the next launch.  Launched between stream-K GEMMs with
// programmatic serialisation: it lets the GEMM after it start its set-up at once, then
// waits for the GEMM before it to finish with the flags.
__global__ void sk_flags_reset_kernel(int* __restrict__ flags, int n) {
  pdl_launch_dependents();
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) flags[i] = 0;
}

// Writes a 32-row x NC-column block, held one row per lane in v[], to rows row0.. and
// columns col0.. of `out` (masked at M and N) through the warp's 32 x 33 float buffer
// `blk`, one 32-column block at a time: every lane writes its row of the block, then the
// warp stores the block row by row, 128 contiguous bytes per row.  For tiles finished
// while the stage buffers still stream the next segment.
template <int NC>
__device__ __forceinline__ void store_rows_blocked(float* blk, const float (&v)[NC], float* out, int64_t ldo,
                                                   int row0, int col0, int M, int N, int lane,
                                                   const float* __restrict__ bias, int act) {
  constexpr int kPitch = 33;
  const bool epi = bias != nullptr || act != kActNone;
#pragma unroll
  for (int b = 0; b < NC / 32; ++b) {
#pragma unroll
    for (int i = 0; i < 32; ++i) blk[lane * kPitch + i] = v[b * 32 + i];
    __syncwarp();
    const int gcol = col0 + b * 32 + lane;
    if (gcol < N) {
      const float bv = bias != nullptr ? __ldg(bias + gcol) : 0.f;
      const int rows = min(32, M - row0);
      float* dst = out + static_cast<int64_t>(row0) * ldo + gcol;
#pragma unroll 4
      for (int r = 0; r < rows; ++r) {
        const float x = blk[r * kPitch + lane];
        dst[static_cast<int64_t>(r) * ldo] = epi ? epilogue(x, bv, act) : x;
      }
    }
    __syncwarp();
  }
}

// One piece of a pair's work: k-blocks [kb_lo, kb_hi) of tile `tile`; `owner` when it
// ends at the tile's last k-block (the pair then stores the tile).
struct PairSeg {
  int tile, kb_lo, kb_hi;
  bool owner;
};

// Grid: x = 2 x pairs, y = z = 1 (batch and tile come from the schedule); other arguments
// as tc2_gemm_kernel (no K slices: k_chunk is unused, out_slab 0).
template <int BN, int STAGES, bool SPLIT3, bool HI_EXPLICIT, bool ANY_LAYOUT>
__global__ void __launch_bounds__(Tc2Cfg<BN, STAGES, SPLIT3, true, 32>::kThreads, 1)
    tc2_sk_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  float* __restrict__ out, int M, int N, int64_t ldo, int K, int mp_tiles, int n_tiles,
                  int group_m, int vec_out, int layout_arg, int64_t out_batch, const float* __restrict__ bias,
                  int act, int shared, const Tc2StreamK sk) {
  const int layout = ANY_LAYOUT ? layout_arg : 0;
  using Cfg = Tc2Cfg<BN, STAGES, SPLIT3, true, 32>;
  constexpr int BK = Cfg::BK;
  constexpr int KC = Cfg::kChunkBlocks;
  constexpr int COLS = Cfg::kColsPerThread;
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

  // ---- schedule (the same arithmetic in every role of both CTAs).  The host keeps
  // units x pairs below 2^31, so the shares are exact in 32-bit arithmetic.
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int nkb = (K + BK - 1) / BK;
  const int units = (sk.tiles - sk.dp_tiles) * nkb;
  const int u0 = units * pair / npairs, u1 = units * (pair + 1) / npairs;
  const int t_hi = u1 > u0 ? (u1 - 1) / nkb : 0;
  const int n_sk = u1 > u0 ? t_hi - u0 / nkb + 1 : 0;
  const int n_seg = n_sk + (pair < sk.dp_tiles ? (sk.dp_tiles - pair + npairs - 1) / npairs : 0);
  auto segment = [&](int i) -> PairSeg {
    if (i < n_sk) {
      const int t = t_hi - i;
      const int base = t * nkb;
      const int hi = min(u1, base + nkb) - base;
      return PairSeg{sk.dp_tiles + t, max(u0, base) - base, hi, hi == nkb};
    }
    return PairSeg{pair + (i - n_sk) * npairs, 0, nkb, true};
  };
  // Grouped raster over the 256 x BN tiles of one batch: this CTA's first row, the pair's
  // first column and the batch of tile t.
  struct TileAt {
    int m0, n0, batch;
  };
  auto tile_at = [&](int t) -> TileAt {
    const int batch = t / sk.tiles_per_batch;
    t -= batch * sk.tiles_per_batch;
    const int band = t / (group_m * n_tiles);
    const int first_m = band * group_m;
    const int band_rows = min(group_m, mp_tiles - first_m);
    const int in_band = t - band * group_m * n_tiles;
    const int tile_m = first_m + in_band % band_rows;
    const int tile_n = in_band / band_rows;
    return TileAt{tile_m * 256 + static_cast<int>(rank) * 128, tile_n * BN, batch};
  };
  auto chunks_of = [](int n) { return SPLIT3 ? (n + KC - 1) / KC : (n > 0 ? 1 : 0); };

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
  pdl_wait();
  bool published = false;  // epilogue warps: this warp's partial (if it has one) is out

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int g = 0;  // stage fills issued, over all segments
      bool ok = true;
      for (int si = 0; si < n_seg && ok; ++si) {
        const PairSeg sg = segment(si);
        const TileAt ta = tile_at(sg.tile);
        const int nb0 = ta.n0 + static_cast<int>(rank) * Cfg::kBNHalf;  // this CTA's B columns
        const int a_batch = (shared & 1) ? 0 : ta.batch, b_batch = (shared & 2) ? 0 : ta.batch;
        const int g_end = g + (sg.kb_hi - sg.kb_lo);
        const int k_shift = (sg.kb_lo - g) * BK;  // k0 of fill g is k_shift + g * BK
        for (; g < g_end; ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!mbar_wait_cluster(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kTxBytes);
          const int k0 = k_shift + g * BK;
          if (layout & kOpAMN) {
#pragma unroll
            for (int j = 0; j < 128 / 32; ++j)
              tma_load_3d(a_raw(s) + j * BK * 128, &tmA, &full[s], ta.m0 + 32 * j, k0, a_batch);
          } else {
            tma_load_3d(a_raw(s), &tmA, &full[s], k0, ta.m0, a_batch);
          }
          if (layout & kOpBK) {
            tma_load_3d(b_raw(s), &tmB, &full[s], k0, nb0, b_batch);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::kBNHalf / 32; ++j)
              tma_load_3d(b_raw(s) + j * BK * 128, &tmB, &full[s], nb0 + 32 * j, k0, b_batch);
          }
        }
      }
      if (ok) {
        // Producer tail: wait for the release (leader's commit) of each of the last fills,
        // so no arrival targets this CTA's barriers after it exits.
        for (int f = g - STAGES < 0 ? 0 : g - STAGES; f < g; ++f)
          if (!mbar_wait_cluster(&empty[f % STAGES], (f / STAGES) & 1, abort_flag)) { ok = false; break; }
      }
      if (!ok) {
        // Gave up: let the last fills' copies land (a landed fill passes at once).
        for (int f = g - STAGES < 0 ? 0 : g - STAGES; f < g; ++f) mbar_drain(&full[f % STAGES], (f / STAGES) & 1);
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
      int g = 0, gc = 0;  // stages consumed and TMEM chunks started, over all segments
      for (int si = 0; si < n_seg && ok; ++si) {
        const PairSeg sg = segment(si);
        const int n = sg.kb_hi - sg.kb_lo;
        const int g0 = g, g_end = g + n;
        for (; g < g_end; ++g) {
          const int r = g - g0;  // k-block within the segment
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          const int chunk = gc + r / KC;
          const bool chunk_start = (r % KC == 0);
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
            if constexpr (SPLIT3) {
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
          if (r % KC == KC - 1 || r == n - 1) {
            const uint32_t c_local = smem_u32(&chunk_full[chunk & 1]);
            umma_commit_pair_both(c_local);
          }
        }
        gc += chunks_of(n);
      }
      // Every MMA issued here completes before this thread leaves its role, on every path
      // (an epilogue that gave up must not let the pair free TMEM or exit under a running
      // MMA, which also reads the peer CTA's shared memory).
      umma_commit_pair(smem_u32(drain_bar));
      mbar_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ split + promotion epilogue (both CTAs)
    const int e = warp - 2;
    const int q = warp & 3;
    const int h = e >> 2;
    const int et = threadIdx.x - 64;
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    bool ok = true;
    float tot[COLS];

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

    // This warp's block of a pair's partial tile: COLS/4 float4 columns of 32 lanes (rows),
    // so every access of the warp is 512 contiguous bytes.
    const int64_t warp_slot = (static_cast<int64_t>(rank) * Cfg::kEpiWarps + e) * (COLS * 32);
    const int flag_slot = static_cast<int>(rank) * Cfg::kEpiWarps + e;
    constexpr int kLag = 2;
    int g = 0, gc = 0;  // stages split and TMEM chunks drained, over all segments
    for (int si = 0; si < n_seg && ok; ++si) {
      const PairSeg sg = segment(si);
      const int n = sg.kb_hi - sg.kb_lo, n_chunks = chunks_of(n);
#pragma unroll
      for (int j = 0; j < COLS; ++j) tot[j] = 0.f;
      int drained = 0;
      const int g0 = g, g_end = g + n;
      for (; g < g_end; ++g) {
        const int r = g - g0;
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
        if constexpr (SPLIT3) {
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
        if (r % KC == (kLag < KC ? kLag : KC - 1) && r / KC >= 1 && drained < r / KC) {
          if (!drain(gc + drained)) { ok = false; break; }
          ++drained;
        }
      }
      while (ok && drained < n_chunks) {
        if (!drain(gc + drained)) { ok = false; break; }
        ++drained;
      }
      gc += n_chunks;
      if (!ok) break;

      const bool last = si == n_seg - 1;
      // After the last segment's last chunk every MMA of the pair has completed, so this
      // CTA's stage buffers are free for the output staging.
      if (last) pdl_launch_dependents();
      if (!sg.owner) {
        float4* slot = reinterpret_cast<float4*>(sk.partial + static_cast<int64_t>(pair) * Cfg::kPartialFloats +
                                                 warp_slot);
#pragma unroll
        for (int j = 0; j < COLS / 4; ++j)
          __stcg(slot + j * 32 + lane, make_float4(tot[4 * j], tot[4 * j + 1], tot[4 * j + 2], tot[4 * j + 3]));
        __threadfence();
        __syncwarp();
        if (lane == 0) flag_release(sk.flags + pair * 2 * Cfg::kEpiWarps + flag_slot, 1);
        published = true;
        continue;
      }
      if (sg.kb_lo > 0) {
        // Lower-numbered pairs holding k-blocks [0, kb_lo) of this tile, in pair order.
        const int base = (sg.tile - sk.dp_tiles) * nkb;
        const int first = ((base + 1) * npairs + units - 1) / units - 1;
        for (int p2 = first; p2 < pair; ++p2) {
          // Every lane acquires the flag itself before reading the partial.
          const bool ready = flag_wait(sk.flags + p2 * 2 * Cfg::kEpiWarps + flag_slot, abort_flag);
          if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
          const float4* slot = reinterpret_cast<const float4*>(
              sk.partial + static_cast<int64_t>(p2) * Cfg::kPartialFloats + warp_slot);
#pragma unroll
          for (int j = 0; j < COLS / 4; ++j) {
            const float4 v = __ldcg(slot + j * 32 + lane);
            tot[4 * j] += v.x;
            tot[4 * j + 1] += v.y;
            tot[4 * j + 2] += v.z;
            tot[4 * j + 3] += v.w;
          }
        }
        if (!ok) break;
      }
      const TileAt ta = tile_at(sg.tile);
      float* out_t = out + static_cast<int64_t>(ta.batch) * out_batch;
      const int row0 = ta.m0 + 32 * q, col0 = ta.n0 + h * COLS;
      if (last) {
        float* stage = reinterpret_cast<float*>(smem) + e * 32 * (COLS + 4);
        store_rows_coalesced<COLS>(stage, tot, out_t, ldo, row0, col0, M, N, vec_out, lane, bias, act);
      } else {
        float* blk = reinterpret_cast<float*>(bar_area + Cfg::kBarBytes) + e * 32 * Cfg::kBlockPitch;
        store_rows_blocked<COLS>(blk, tot, out_t, ldo, row0, col0, M, N, lane, bias, act);
      }
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
  // This CTA gave up (copies and MMAs of both CTAs have landed): each epilogue warp
  // overwrites its block of every tile the pair owns with NaN, and publishes a NaN partial
  // in place of one it did not publish, so the owner of that tile finishes with NaN
  // instead of waiting out its own limit.
  if (*abort_flag && warp >= 2) {
    const int e = warp - 2, q = warp & 3, h = e >> 2;
    const int flag_slot = static_cast<int>(rank) * Cfg::kEpiWarps + e;
    for (int si = 0; si < n_seg; ++si) {
      const PairSeg sg = segment(si);
      if (!sg.owner) {
        if (published) continue;
        float* slot = sk.partial + static_cast<int64_t>(pair) * Cfg::kPartialFloats +
                      (static_cast<int64_t>(rank) * Cfg::kEpiWarps + e) * (COLS * 32);
        poison_rows(slot, COLS * 32, 0, 1, 0, COLS * 32, 1, COLS * 32, lane);
        __threadfence();
        __syncwarp();
        if (lane == 0) flag_release(sk.flags + pair * 2 * Cfg::kEpiWarps + flag_slot, 1);
        continue;
      }
      const TileAt ta = tile_at(sg.tile);
      poison_rows(out + static_cast<int64_t>(ta.batch) * out_batch, ldo, ta.m0 + 32 * q, 32, ta.n0 + h * COLS, COLS,
                  M, N, lane);
    }
  }
}

}  // namespace tilec
