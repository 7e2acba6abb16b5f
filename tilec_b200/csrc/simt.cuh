// simt.cuh -- fp32 FFMA GEMM for sm_100a (variant SIMT, and SPLITK when gridDim.z > 1).
//
// Arithmetic of the reference kernel tilec/ext.py:13-24 (_matmul_tiled): one CTA owns
// an output tile, walks K in BK-wide steps, reads out-of-range elements of A and B as
// 0.0 (ext.py:21-22) and stores only in-range elements of C (ext.py:24).  Every
// product is a single fp32 FFMA accumulated in k order, so results are fp32-exact
// in the usual GEMM sense.
//
// B200 mapping:
//   * CTA tile 128 x BN x 16 (BN = 128 or 64), 256 threads, each thread an 8 x (BN/16)
//     register block (2-D register blocking, 64 or 32 FFMA per k), at most 128 registers
//     so that two CTAs (16 warps) share an SM.
//   * 4-stage pipeline global -> shared.  B tiles with 16-byte aligned rows are staged by
//     TMA (one [16 x BN] box per stage, completion on a per-stage mbarrier; the tensor
//     map's extent zero-fills ragged edges); others, and A always, by cp.async, whose
//     src-size operand zero-fills the tail of a ragged tile, so no out-of-range address is
//     read.  TMA cannot stage A: the kernel wants A k-major and TMA does not transpose
//     4-byte elements.
//   * Both shared tiles are k-major: A as [16][128 + 4] (transposed on the way in by
//     4-byte copies; a warp copies 4 rows x 8 k, 32-byte runs of global memory, and the
//     pitch of 132 puts its 32 stores in 32 banks), B as [16][BN] (the dense box TMA
//     writes, or 16-byte / 4-byte cp.async copies).  A thread owns the 8 consecutive
//     rows tm*8.. and reads them at one k with two 16-byte loads, as it reads its B
//     columns: 4 shared loads per 64 FFMA and only 16 operand registers live.
//   * Split-K (gridDim.z = S > 1): CTA z covers K range [z*k_chunk, min(K,(z+1)*k_chunk))
//     and writes its partial tile to slab z of the workspace; splitk_reduce_kernel
//     sums the slabs in z order (deterministic).
#pragma once

#include "common.cuh"

namespace tilec {

constexpr int kSimtBM = 128;
constexpr int kSimtBK = 16;
constexpr int kSimtStages = 4;
constexpr int kSimtThreads = 256;
constexpr int kSimtAPitch = kSimtBM + 4;  // floats per k row of the k-major A tile
constexpr int kSimtBarBytes = 64;         // TMA-staged B: kSimtStages mbarriers + abort flag

// How B reaches shared memory: 4-byte cp.async (any alignment), 16-byte cp.async, TMA.
enum : int { kBScalar = 0, kBVec = 1, kBTma = 2 };

template <int BN>
constexpr int simt_smem_bytes() {
  return kSimtStages * (kSimtBK * kSimtAPitch + kSimtBK * BN) * 4 + kSimtBarBytes;
}
// Dynamic shared memory asked for by grids of at most one CTA per SM: more than half of an
// SM's 228 KB, so the block scheduler cannot place two such CTAs on one SM.
constexpr int kSimtSpreadSmem = 120 * 1024;
static_assert(simt_smem_bytes<128>() <= kSimtSpreadSmem, "spread request covers the tiles");

// Per-thread copy plan of the SIMT tiles, fixed for the CTA, so that a tile costs one
// pointer step per operand:
//   A (4-byte copies, transposed to k-major): blocks of 4 rows x 8 k, lane = 8 * (row % 4)
//     + k % 8 (32-byte runs of global memory; with the 132-float pitch, which is 4 mod 32,
//     the warp's 32 shared stores hit 32 banks).  Copy j of warp w is block 8 j + w: k
//     group (8 j + w) % G = w % G of the G = BK / 8, so a thread always copies the same k
//     a_k, of rows a_row + (32 / G) j.
//   B: 16-byte chunk (VEC) or element b_n of rows b_row + kBRowStep * i.
// Out-of-range elements are zero-filled through cp.async's src-size operand, with the
// operand's base address as the (unread) source.
template <int BN, int BMODE>
struct SimtCopy {
  static constexpr bool VEC = BMODE != kBScalar;
  static constexpr int kAPerThread = kSimtBM * kSimtBK / kSimtThreads;
  static constexpr int kKGroups = kSimtBK / 8;            // G
  static constexpr int kARowStep = 4 * (8 / kKGroups);    // rows between a thread's copies
  static constexpr int kBPerRow = VEC ? BN / 4 : BN;      // copies per B row
  static constexpr int kBPerThread = kSimtBK * kBPerRow / kSimtThreads;
  static constexpr int kBRowStep = kSimtThreads / kBPerRow;
  static_assert(kSimtBK % 8 == 0 && 8 % kKGroups == 0 && kAPerThread <= 32, "A copy plan");
  static_assert(kSimtThreads % kBPerRow == 0 && kBPerThread >= 1, "B copy plan");
  const float* a_src;  // A + (m0 + a_row) * lda + a_k
  const float* b_src;  // B + b_row * ldb + n0 + b_n
  int64_t a_step;      // kARowStep rows of A
  int64_t b_step;      // kBRowStep rows of B
  int64_t ldb;
  int a_dst, b_dst;    // shared offsets within a stage
  int a_k, b_row;
  uint32_t a_rows_ok;  // bit j: row a_row + kARowStep j is below M
  uint32_t b_bytes;    // per B copy: 16 or fewer at a ragged N edge (VEC), 4 or 0 (scalar)

  __device__ __forceinline__ SimtCopy(const float* A, const float* B, int64_t M, int64_t N, int64_t lda,
                                      int64_t ldb_, int64_t m0, int64_t n0, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int a_row = 4 * (warp / kKGroups) + (lane >> 3);
    a_k = 8 * (warp % kKGroups) + (lane & 7);
    a_dst = a_k * kSimtAPitch + a_row;
    a_src = A + (m0 + a_row) * lda + a_k;
    a_step = kARowStep * lda;
    a_rows_ok = 0;
#pragma unroll
    for (int j = 0; j < kAPerThread; ++j)
      if (m0 + a_row + kARowStep * j < M) a_rows_ok |= 1u << j;
    b_row = tid / kBPerRow;
    const int b_n = (tid % kBPerRow) * (VEC ? 4 : 1);
    b_dst = b_row * BN + b_n;
    b_src = B + b_row * ldb_ + n0 + b_n;
    b_step = kBRowStep * ldb_;
    ldb = ldb_;
    const int64_t rem = N - (n0 + b_n);
    if constexpr (VEC)
      b_bytes = rem >= 4 ? 16u : (rem > 0 ? static_cast<uint32_t>(rem) * 4u : 0u);
    else
      b_bytes = rem > 0 ? 4u : 0u;
  }

  // Copies the tile at k0 (rows of A and B beyond k_end read as zero) into as / bs.
  __device__ __forceinline__ void load(float* as, float* bs, const float* A, const float* B, int64_t k0,
                                       int64_t k_end) const {
    const bool ka = k0 + a_k < k_end;
    const float* pa = a_src + k0;
#pragma unroll
    for (int j = 0; j < kAPerThread; ++j) {
      const bool ok = ka && ((a_rows_ok >> j) & 1u);
      cp_async_4(as + a_dst + kARowStep * j, ok ? pa + j * a_step : A, ok ? 4u : 0u);
    }
    if constexpr (BMODE == kBTma) return;  // B arrives by TMA
    const float* pb = b_src + k0 * ldb;
#pragma unroll
    for (int i = 0; i < kBPerThread; ++i) {
      const bool ok = b_bytes != 0 && k0 + b_row + kBRowStep * i < k_end;
      if constexpr (VEC)
        cp_async_16(bs + b_dst + kBRowStep * i * BN, ok ? pb + i * b_step : B, ok ? b_bytes : 0u);
      else
        cp_async_4(bs + b_dst + kBRowStep * i * BN, ok ? pb + i * b_step : B, ok ? 4u : 0u);
    }
  }
};

// out/ldo: C (one K slice) or the split-K workspace (slab z at out + z*out_slab).
// blockIdx.z = batch * splits + K slice; batch b reads A + b*stride_a, B + b*stride_b and
// writes out + b*out_batch.  bias / act: fused epilogue (only when writing C directly).
// tmB (BMODE == kBTma): B as a 3-D map {N, K, batch} with a {BN, 16, 1} box; batch index 0
// when stride_b == 0 (shared B).  K slices start at multiples of 16, so a stage's 16 rows
// never straddle a slice boundary, and rows past K read as zero.
template <int BN, int BMODE>
__global__ void __launch_bounds__(kSimtThreads, 2)
    simt_gemm_kernel(const __grid_constant__ CUtensorMap tmB, const float* __restrict__ A,
                     const float* __restrict__ B, float* __restrict__ out,
                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldo, int64_t out_slab,
                     int64_t k_chunk, int vec_out, int splits, int64_t stride_a, int64_t stride_b,
                     int64_t out_batch, const float* __restrict__ bias, int act) {
  constexpr int TN = BN / 16;  // columns per thread: 8 (two float4 groups 64 apart) or 4
  extern __shared__ __align__(128) float smem[];
  float* As = smem;
  float* Bs = smem + kSimtStages * kSimtBK * kSimtAPitch;  // 128-byte aligned: a TMA destination
  uint64_t* full = reinterpret_cast<uint64_t*>(Bs + kSimtStages * kSimtBK * BN);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + kSimtStages);
  static_assert((kSimtStages * kSimtBK * kSimtAPitch * 4) % 128 == 0, "B tiles 128-byte aligned");
  static_assert(kSimtStages * 8 + 4 <= kSimtBarBytes, "barrier area");

  pdl_wait();
  if (blockDim.x != kSimtThreads) {
    if (threadIdx.x == 0) record_status(TILEC_DEV_BAD_LAUNCH);
    return;
  }
  const int tid = threadIdx.x;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * kSimtBM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.y) * BN;
  const int64_t batch = static_cast<int64_t>(blockIdx.z) / splits;
  const int64_t kslice = static_cast<int64_t>(blockIdx.z) % splits;
  A += batch * stride_a;
  B += batch * stride_b;
  const int64_t k_begin = kslice * k_chunk;
  const int64_t k_end = (k_begin + k_chunk < K) ? k_begin + k_chunk : K;
  const int64_t nkt = (k_end > k_begin) ? (k_end - k_begin + kSimtBK - 1) / kSimtBK : 0;
  out += kslice * out_slab + batch * out_batch;
  const SimtCopy<BN, BMODE> copy(A, B, M, N, lda, ldb, m0, n0, tid);
  // Thread 0 stages B tile `it` (k rows k_begin + 16 it ..) into stage it % kSimtStages.
  // Coordinates are recomputed from blockIdx at each use rather than held in registers.
  auto issue_b = [&](int it) {
    const int st = it % kSimtStages;
    const int bz = static_cast<int>(blockIdx.z) / splits;
    mbar_arrive_expect_tx(&full[st], kSimtBK * BN * 4);
    tma_load_3d(Bs + st * kSimtBK * BN, &tmB, &full[st], static_cast<int>(blockIdx.y) * BN,
                static_cast<int>((static_cast<int>(blockIdx.z) % splits) * k_chunk) + it * kSimtBK,
                stride_b == 0 ? 0 : bz);
  };
  if constexpr (BMODE == kBTma) {
    if (tid == 0) {
      for (int s = 0; s < kSimtStages; ++s) mbar_init(&full[s], 1);
      *abort_flag = 0;
      fence_barrier_init();
      tma_prefetch_desc(&tmB);
    }
    __syncthreads();
  }

  const int tm = tid >> 4;
  const int tn = tid & 15;

  float acc[8][TN];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

#pragma unroll
  for (int s = 0; s < kSimtStages - 1; ++s) {
    if (s < nkt) {
      copy.load(As + s * kSimtBK * kSimtAPitch, Bs + s * kSimtBK * BN, A, B, k_begin + s * kSimtBK, k_end);
      if (BMODE == kBTma && tid == 0) issue_b(s);
    }
    cp_async_commit();
  }

  bool ok = true;
  int64_t kt = 0;
  for (; kt < nkt; ++kt) {
    cp_async_wait<kSimtStages - 2>();
    if constexpr (BMODE == kBTma) {
      // Thread 0 waits (bounded) for the stage's B tile; the barrier below then orders the
      // TMA's writes, which its wait acquired, before every thread's reads.  On a timeout it
      // raises the abort flag, which every thread reads after the barrier, so the whole CTA
      // leaves the loop together.
      if (tid == 0) {
        const int it = static_cast<int>(kt);
        mbar_wait(&full[it % kSimtStages], static_cast<uint32_t>((it / kSimtStages) & 1), abort_flag);
      }
    }
    __syncthreads();
    if constexpr (BMODE == kBTma) {
      if (*abort_flag) {
        ok = false;
        break;
      }
    }
    const int64_t nt = kt + kSimtStages - 1;
    if (nt < nkt) {
      const int ns = static_cast<int>(nt % kSimtStages);
      copy.load(As + ns * kSimtBK * kSimtAPitch, Bs + ns * kSimtBK * BN, A, B, k_begin + nt * kSimtBK, k_end);
      if (BMODE == kBTma && tid == 0) issue_b(static_cast<int>(nt));
    }
    cp_async_commit();

    const int cs = static_cast<int>(kt % kSimtStages);
    const float* as = As + cs * kSimtBK * kSimtAPitch + tm * 8;
    const float* bs = Bs + cs * kSimtBK * BN + tn * 4;
#pragma unroll
    for (int k = 0; k < kSimtBK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(as + k * kSimtAPitch);
      const float4 a1 = *reinterpret_cast<const float4*>(as + k * kSimtAPitch + 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float b[TN];
      const float4 b0 = *reinterpret_cast<const float4*>(bs + k * BN);
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      if constexpr (TN == 8) {
        const float4 b1 = *reinterpret_cast<const float4*>(bs + k * BN + 64);
        b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
      }
      // Packed two-wide FMAs (sm_100 FFMA2): per component exactly fmaf, half the FMA
      // instructions, so more issue slots go to the FMA pipe.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 ai = make_float2(a[i], a[i]);
#pragma unroll
        for (int j = 0; j < TN; j += 2) {
          const float2 r = __ffma2_rn(ai, make_float2(b[j], b[j + 1]), make_float2(acc[i][j], acc[i][j + 1]));
          acc[i][j] = r.x;
          acc[i][j + 1] = r.y;
        }
      }
    }
  }
  cp_async_wait<0>();
  if constexpr (BMODE == kBTma) {
    if (!ok) {
      // Let the TMA copies still in flight (tiles kt .. kt + 2) land before the CTA's
      // shared memory goes away, and overwrite the CTA's tile with NaN (the status word
      // records the timeout): each warp 16 of its 128 rows.
      if (tid == 0)
        for (int64_t it = kt; it < nkt && it < kt + kSimtStages - 1; ++it)
          mbar_drain(&full[it % kSimtStages], static_cast<uint32_t>((it / kSimtStages) & 1));
      poison_rows(out, ldo, m0 + 16 * (tid >> 5), 16, n0, BN, M, N, tid & 31);
      return;
    }
  }
  // Let the next kernel launch only now: CTAs of a dependent kernel that wait resident on
  // the SM while this FMA-bound loop runs cost it issue slots (measured 40% slower).
  pdl_launch_dependents();

  // Epilogue: masked stores (ext.py:24).  Each warp writes two 256-byte row runs.
  if (bias != nullptr || act != kActNone) {
#pragma unroll
    for (int g = 0; g < TN / 4; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + g * 64 + tn * 4 + j;
        const float bv = (bias != nullptr && gn < N) ? __ldg(bias + gn) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i][g * 4 + j] = epilogue(acc[i][g * 4 + j], bv, act);
      }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + tm * 8 + i;
    if (gm >= M) continue;
    float* crow = out + gm * ldo;
#pragma unroll
    for (int g = 0; g < TN / 4; ++g) {
      const int64_t gn = n0 + g * 64 + tn * 4;
      if (vec_out && gn + 3 < N) {
        *reinterpret_cast<float4*>(crow + gn) =
            make_float4(acc[i][g * 4 + 0], acc[i][g * 4 + 1], acc[i][g * 4 + 2], acc[i][g * 4 + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gn + j < N) crow[gn + j] = acc[i][g * 4 + j];
      }
    }
  }
}

// C[m, n] = sum_{z < S} W[z][m, n].  W slabs have row stride ldw (a multiple of 4) and
// slab stride `slab`.  A 256-thread block has P slab partitions of G = 256 / P lanes; a
// lane handles U float4 column groups (G apart, so a warp reads contiguous runs).
// Partition p sums slabs [p*S/P, (p+1)*S/P) of each group in z order, then partition 0
// adds partitions 1..P-1 in p order.  The order is fixed by (S, P), so results are
// bitwise reproducible.  P and U are chosen so that one pass of resident blocks covers
// the output with every load in flight at once (up to eight per thread at a time):
// separate grid-stride rounds would each pay the full L2 latency again.
//
// Batched: blockIdx.y is the batch; its slabs are W + blockIdx.y*S*slab and its result
// goes to C + blockIdx.y*stride_c.  bias / act: the fused epilogue, applied to the
// finished sum.
//
// LB: blocks per SM the registers are bounded for.  LB = 4 (64 registers, U = 1 only)
// leaves an SM room for the next product's GEMM CTA, which can then launch (programmatic
// dependent launch), allocate TMEM and prefetch its first operand tiles into L2 while this
// kernel still runs: on B200 1.7-1.8 us faster for 1024x8192x128 and 512x2048x256, but
// 0.5-0.9 us slower for N = 64 products (fewer loads in flight per thread), which keep LB = 2.
template <int P, int U, int LB = 2>
__global__ void __launch_bounds__(256, LB) splitk_reduce_kernel(const float* __restrict__ W, float* __restrict__ C,
                                                            int64_t M, int64_t N, int64_t ldw, int64_t ldc,
                                                            int64_t slab, int S, int vec_out, int64_t stride_c,
                                                            const float* __restrict__ bias, int act) {
  static_assert(8 % U == 0, "U divides the load batch");
  static_assert(LB == 2 || (LB == 4 && U == 1), "64-register bound only for one column group per thread");
  constexpr int G = 256 / P;
  __shared__ float4 part[P > 1 ? P - 1 : 1][P > 1 ? U * G : 1];
  pdl_wait();
  pdl_launch_dependents();
  W += static_cast<int64_t>(blockIdx.y) * S * slab;
  C += static_cast<int64_t>(blockIdx.y) * stride_c;
  const int p = static_cast<int>(threadIdx.x) / G;
  const int gi = static_cast<int>(threadIdx.x) % G;
  const int z0 = (S * p) / P, nz = (S * (p + 1)) / P - z0;
  const int64_t groups_per_row = (N + 3) / 4;
  const int64_t total = M * groups_per_row;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * G * U; base < total;
       base += static_cast<int64_t>(gridDim.x) * G * U) {
    const float* w[U];
    int64_t mm[U], nn[U];
    bool live[U];
    float4 acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = base + u * G + gi;
      live[u] = g < total;
      mm[u] = live[u] ? g / groups_per_row : 0;
      nn[u] = live[u] ? (g % groups_per_row) * 4 : 0;
      w[u] = W + mm[u] * ldw + nn[u] + static_cast<int64_t>(z0) * slab;
      acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live[u] && nz > 0) acc[u] = __ldg(reinterpret_cast<const float4*>(w[u]));
    }
    // Load t covers group t % U, slab z0 + t / U; batches of eight keep each group's adds
    // in z order.
    for (int t0 = U; t0 < U * nz; t0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (t0 + j < U * nz && live[j % U])
          v[j] = __ldg(reinterpret_cast<const float4*>(w[j % U] + static_cast<int64_t>((t0 + j) / U) * slab));
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (t0 + j < U * nz && live[j % U]) {
          float4& a = acc[j % U];
          a.x += v[j].x; a.y += v[j].y; a.z += v[j].z; a.w += v[j].w;
        }
    }
    if constexpr (P > 1) {
      if (p > 0) {
#pragma unroll
        for (int u = 0; u < U; ++u) part[p - 1][u * G + gi] = acc[u];
      }
      __syncthreads();
    }
    if (p == 0) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!live[u]) continue;
        float4 s = acc[u];
#pragma unroll
        for (int q = 1; q < P; ++q) {
          const float4 v = part[q - 1][u * G + gi];
          s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
        }
        if (bias != nullptr || act != kActNone) {
          float bv[4] = {0.f, 0.f, 0.f, 0.f};
          if (bias != nullptr) {
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = nn[u] + j < N ? __ldg(bias + nn[u] + j) : 0.f;
          }
          s = make_float4(epilogue(s.x, bv[0], act), epilogue(s.y, bv[1], act), epilogue(s.z, bv[2], act),
                          epilogue(s.w, bv[3], act));
        }
        float* c = C + mm[u] * ldc + nn[u];
        if (vec_out && nn[u] + 3 < N) {
          *reinterpret_cast<float4*>(c) = s;
        } else {
          const float sv[4] = {s.x, s.y, s.z, s.w};
          for (int j = 0; j < 4 && nn[u] + j < N; ++j) c[j] = sv[j];
        }
      }
    }
    if constexpr (P > 1) __syncthreads();
  }
}

// K == 0: the reference's accumulator stays 0 and is stored (ext.py:18,24); with a fused
// epilogue C = act(bias) per column.  All batches (C + b*stride_c) in one pass.
__global__ void __launch_bounds__(256) fill_zero_kernel(float* __restrict__ C, int64_t M, int64_t N, int64_t ldc,
                                                        int64_t batches, int64_t stride_c,
                                                        const float* __restrict__ bias, int act) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t total = batches * M * N;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = e / N, n = e % N, b = row / M, m = row - b * M;
    C[b * stride_c + m * ldc + n] =
        (bias != nullptr || act != kActNone) ? epilogue(0.f, bias != nullptr ? bias[n] : 0.f, act) : 0.f;
  }
}

}  // namespace tilec
