// tc2_tf32p.cuh -- persistent TF32 GEMM on CTA pairs (tcgen05 cta_group::2), sm_100a.
//
// Same contraction and edge semantics as tc2_gemm.cuh in its TF32 mode (tilec/ext.py:13-24:
// zero-filled out-of-range operands, masked stores) and the same MMA sequence per output
// element (one TMEM accumulator over all of K, K = 8 per instruction in K order), so its
// results equal the one-pair-per-tile kernel's bit for bit.  What changes is the schedule:
// a pair computes many 256 x 256 tiles (tile t of all batches goes to pair t % P, P pairs
// in the grid), so a tile's pipeline fill and epilogue no longer leave the tensor core idle.
//
//   * two TMEM accumulators of 256 columns: the MMAs of a pair's tile i run into buffer
//     i % 2 while the epilogue warps drain tile i - 1 from the other one (acc_full /
//     acc_empty barriers, the latter arrived by the 16 epilogue warps of both CTAs);
//   * the TMA producer of each CTA runs straight on across tiles through a 5-stage ring;
//   * "the peer's stage landed" reaches the leader through one relay thread in the peer CTA
//     (its warp 1, otherwise idle there), so the epilogue warps do nothing per stage: they
//     wait for a finished accumulator, read it in 32-column pieces (tcgen05.ld) and store
//     each through a staging buffer of their own, which leaves the stage ring alone;
//   * every wait is bounded; a CTA that gives up lets its copies and MMAs land and writes
//     NaN over the tiles it had not stored.
//
// Operands as in tc2_gemm.cuh: A K-major (x1 row-major), B MN-major (x2 row-major), either
// flipped by `layout` (kOpAMN / kOpBK) when stored transposed.  No K split, no stream-K.
#pragma once

#include "common.cuh"
#include "tc_gemm.cuh"

namespace tilec {

struct Tc2PCfg {
  static constexpr int BN = 256;
  static constexpr int BK = 32;
  static constexpr int kStages = 5;
  static constexpr int kBNHalf = BN / 2;
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kABytes = 128 * BK * 4;      // own A rows
  static constexpr int kBBytes = BK * kBNHalf * 4;  // own half of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTxBytes = kStageBytes;
  static constexpr int kStorePitch = 36;            // 32 rows x (32 + 4) floats per epilogue warp
  static constexpr int kStoreFloatsPerWarp = 32 * kStorePitch;
  static constexpr int kStoreBytes = kEpiWarps * kStoreFloatsPerWarp * 4;
  static constexpr int kBarBytes = 512;
  static constexpr int kSmemBytes = kStages * kStageBytes + kStoreBytes + kBarBytes + 1024;
  static constexpr uint32_t kASbo = 8u * BK * 4u;   // 8 rows x 128 bytes (K-major)
  static constexpr uint32_t kBLbo = BK * 128u;      // stride between 32-column slabs
  static constexpr uint32_t kBSbo = 512u;           // stride between 4-row K groups
  static constexpr uint32_t kTmemCols = 2 * BN;     // two accumulators
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert((3 * kStages + 5) * 8 + 8 <= kBarBytes, "barrier area");
};

// Grid: 2 x P CTAs in clusters of 2 (P pairs), y = z = 1.  Tiles: `total_tiles` = batches x
// tiles_per_batch, tile t of batch t / tiles_per_batch in the grouped raster of tc2_gemm.cuh.
template <bool ANY_LAYOUT>
__global__ void __launch_bounds__(Tc2PCfg::kThreads, 1)
    tc2_tf32p_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     float* __restrict__ out, int M, int N, int64_t ldo, int K, int mp_tiles, int n_tiles,
                     int group_m, int tiles_per_batch, int total_tiles, int vec_out, int layout_arg,
                     int64_t out_batch, const float* __restrict__ bias, int act, int shared) {
  using Cfg = Tc2PCfg;
  constexpr int STAGES = Cfg::kStages, BK = Cfg::BK, BN = Cfg::BN;
  const int layout = ANY_LAYOUT ? layout_arg : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto a_tile = [&](int s) { return smem + s * Cfg::kStageBytes; };
  auto b_tile = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kABytes; };
  float* store_area = reinterpret_cast<float*>(smem + STAGES * Cfg::kStageBytes);
  uint8_t* bar_area = smem + STAGES * Cfg::kStageBytes + Cfg::kStoreBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);  // [STAGES] own TMA landed
  uint64_t* empty = full + STAGES;                          // [STAGES] leader's MMAs released the stage
  uint64_t* peer_full = empty + STAGES;                     // [STAGES] (leader) the peer's TMA landed
  uint64_t* acc_full = peer_full + STAGES;                  // [2] accumulator holds a finished tile
  uint64_t* acc_empty = acc_full + 2;                       // [2] (leader) both CTAs drained it
  uint64_t* drain_bar = acc_empty + 2;
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
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int n_my = pair < total_tiles ? (total_tiles - pair + npairs - 1) / npairs : 0;
  const int nkb = (K + BK - 1) / BK;

  struct TileAt {
    int m0, n0, batch;
  };
  auto tile_at = [&](int i) -> TileAt {
    int t = pair + i * npairs;
    const int batch = t / tiles_per_batch;
    t -= batch * tiles_per_batch;
    const int band = t / (group_m * n_tiles);
    const int first_m = band * group_m;
    const int band_rows = min(group_m, mp_tiles - first_m);
    const int in_band = t - band * group_m * n_tiles;
    const int tile_m = first_m + in_band % band_rows;
    const int tile_n = in_band / band_rows;
    return TileAt{tile_m * 256 + static_cast<int>(rank) * 128, tile_n * BN, batch};
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&peer_full[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * Cfg::kEpiWarps);
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

  int stored = 0;  // epilogue warps: tiles of this pair whose rows this warp has stored
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int g = 0;  // fills issued, over all tiles
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const TileAt ta = tile_at(i);
        const int nb0 = ta.n0 + static_cast<int>(rank) * Cfg::kBNHalf;
        const int a_batch = (shared & 1) ? 0 : ta.batch, b_batch = (shared & 2) ? 0 : ta.batch;
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!mbar_wait_cluster(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], Cfg::kTxBytes);
          const int k0 = kb * BK;
          if (layout & kOpAMN) {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_3d(a_tile(s) + j * BK * 128, &tmA, &full[s], ta.m0 + 32 * j, k0, a_batch);
          } else {
            tma_load_3d(a_tile(s), &tmA, &full[s], k0, ta.m0, a_batch);
          }
          if (layout & kOpBK) {
            tma_load_3d(b_tile(s), &tmB, &full[s], k0, nb0, b_batch);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::kBNHalf / 32; ++j)
              tma_load_3d(b_tile(s) + j * BK * 128, &tmB, &full[s], nb0 + 32 * j, k0, b_batch);
          }
          ++g;
        }
      }
      if (ok) {
        // Tail: the leader's release of each of the last fills has arrived before the CTA exits.
        for (int f = g - STAGES < 0 ? 0 : g - STAGES; f < g; ++f)
          if (!mbar_wait_cluster(&empty[f % STAGES], (f / STAGES) & 1, abort_flag)) { ok = false; break; }
      }
      if (!ok) {
        for (int f = g - STAGES < 0 ? 0 : g - STAGES; f < g; ++f) mbar_drain(&full[f % STAGES], (f / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------------------------------------------------- MMA issuer (leader CTA)
      const bool a_mn = (layout & kOpAMN) != 0, b_k = (layout & kOpBK) != 0;
      const uint32_t idesc = make_idesc_tf32(256, BN, a_mn, !b_k);
      auto desc_a = [&](uint32_t base, int kk) {
        return a_mn ? make_smem_desc(base + kk * 1024, Cfg::kBLbo, Cfg::kBSbo, kLayoutSw128Base32)
                    : make_smem_desc(base + kk * 32, 16, Cfg::kASbo, kLayoutSw128);
      };
      auto desc_b = [&](uint32_t base, int kk) {
        return b_k ? make_smem_desc(base + kk * 32, 16, Cfg::kASbo, kLayoutSw128)
                   : make_smem_desc(base + kk * 1024, Cfg::kBLbo, Cfg::kBSbo, kLayoutSw128Base32);
      };
      int g = 0;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const int b = i & 1;
        const uint32_t dcol = static_cast<uint32_t>(b * BN);
        // Buffer b last held tile i - 2: both CTAs' epilogues must have drained it.
        if (i >= 2 && !mbar_wait_cluster(&acc_empty[b], ((i >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag) || !mbar_wait_cluster(&peer_full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(a_tile(s)), b0 = smem_u32(b_tile(s));
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk)
            umma_tf32_pair(tmem + dcol, desc_a(a0, kk), desc_b(b0, kk), idesc, (kb == 0 && kk == 0) ? 0u : 1u);
          umma_commit_pair_both(smem_u32(&empty[s]));
          ++g;
        }
        if (ok) umma_commit_pair_both(smem_u32(&acc_full[b]));
      }
      // Every MMA issued here completes before this thread leaves its role, on every path.
      umma_commit_pair(smem_u32(drain_bar));
      mbar_drain(drain_bar, 0);
    } else if (!leader && lane == 0) {
      // ---------------------------------------------------------- relay (peer CTA)
      // The leader's MMAs read this CTA's half of each stage: tell it when the stage landed.
      const uint32_t pf = mapa_shared(smem_u32(peer_full), 0);
      const int fills = n_my * nkb;
      for (int g = 0; g < fills; ++g) {
        const int s = g % STAGES;
        if (!mbar_wait(&full[s], (g / STAGES) & 1, abort_flag)) break;
        mbar_arrive_remote_cta(pf + static_cast<uint32_t>(s * 8));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warps (both CTAs)
    const int e = warp - 2;
    const int q = warp & 3;  // TMEM lane quadrant of this warp: rows 32q .. 32q + 31 of the CTA's half
    const int h = e >> 2;    // which 128 of the 256 columns
    const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
    float* stage = store_area + e * Cfg::kStoreFloatsPerWarp;
    const uint32_t ae = mapa_shared(smem_u32(acc_empty), 0);
    for (int i = 0; i < n_my; ++i) {
      const int b = i & 1;
      if (!mbar_wait_cluster(&acc_full[b], (i >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      if (i == n_my - 1) pdl_launch_dependents();
      const TileAt ta = tile_at(i);
      float* out_t = out + static_cast<int64_t>(ta.batch) * out_batch;
#pragma unroll 1
      for (int c = 0; c < Cfg::kBNHalf / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>(b * BN + h * Cfg::kBNHalf + c * 32), r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        store_rows_coalesced<32>(stage, v, out_t, ldo, ta.m0 + 32 * q, ta.n0 + h * Cfg::kBNHalf + c * 32, M, N,
                                 vec_out, lane, bias, act);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_cta(ae + static_cast<uint32_t>(b * 8));
      ++stored;
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
  // This CTA gave up: both CTAs' copies and MMAs have landed (cluster barrier above), so each
  // epilogue warp overwrites its block of every tile it had not stored with NaN.
  if (*abort_flag && warp >= 2) {
    const int e = warp - 2, q = warp & 3, h = e >> 2;
    for (int i = stored; i < n_my; ++i) {
      const TileAt ta = tile_at(i);
      poison_rows(out + static_cast<int64_t>(ta.batch) * out_batch, ldo, ta.m0 + 32 * q, 32,
                  ta.n0 + h * Cfg::kBNHalf, Cfg::kBNHalf, M, N, lane);
    }
  }
}

}  // namespace tilec
