// common.cuh -- sm_100a PTX helpers shared by the GEMM kernels.
//
// Every wait in this library is bounded: a wait that runs past kWaitLimitNs
// records TILEC_DEV_TIMEOUT in the device status word, raises the CTA's abort
// flag and returns false, and the kernel then unwinds (no __trap, no endless spin).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace tilec {

// Device status word bits (read by tilec_mm_device_status()).
enum : int {
  TILEC_DEV_TIMEOUT = 1,      // an mbarrier wait exceeded kWaitLimitNs
  TILEC_DEV_TMEM = 2,         // TMEM allocation returned an unexpected address
  TILEC_DEV_BAD_LAUNCH = 4,   // kernel launched with a block shape it was not built for
};

// Defined here: the library is built as a single translation unit (tilec_mm.cu).
__device__ int g_status = 0;

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Limit of every bounded wait of the GEMM kernels on this device, in ns; 0 means
// kWaitLimitNs.  Set only by tilec_mm_set_wait_limit (failure-detection tests shorten it so
// that a real GEMM launch gives up, then restore it).
__device__ unsigned long long g_wait_limit_ns = 0;

__device__ __forceinline__ unsigned long long wait_limit() {
  const unsigned long long v = *const_cast<volatile unsigned long long*>(&g_wait_limit_ns);
  return v ? v : kWaitLimitNs;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int bits) { atomicOr(&g_status, bits); }

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of this library is launched with programmatic stream serialisation, so it
// may start while the previous kernel in the stream is still running.  pdl_wait() blocks
// until that kernel has completed and its writes are visible; each kernel calls it before
// its first global-memory access (only shared-memory / TMEM set-up runs before it).
// Without the launch attribute it returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream start launching its CTAs (they block in pdl_wait()).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// try_wait with an explicit suspend-time hint: a waiting thread is parked for up to
// TILEC_WAIT_HINT_NS (or until the phase completes) instead of returning after the
// implementation's default slice.  Measured on B200 over the tcgen05 kernels this is
// 4-8% faster on large GEMMs than the hint-less form (8192^3 3xTF32: 237 -> 256 TFLOP/s;
// 2048^3: 194 -> 208) and slower never; the hint value itself (8..512 ns) did not matter.
// A non-suspending test_wait spin was slightly slower than both.
#ifndef TILEC_WAIT_HINT_NS
#define TILEC_WAIT_HINT_NS 64
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(uint32_t(TILEC_WAIT_HINT_NS))
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  `abort_flag` (shared) lets
// one role that gave up release every other role quickly.  limit_ns == 0: the device's
// limit (wait_limit()); the clock is read every 64 polls at the default limit and on
// every poll below it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  if (limit_ns == 0) limit_ns = wait_limit();
  const uint32_t mask = limit_ns < kWaitLimitNs ? 0u : 63u;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & mask) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        record_status(TILEC_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

// Bounded wait that ignores the abort flag (used while draining after an abort).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > 100000000ull) return;  // 100 ms
  }
}

// ---------------------------------------------------------------- flags between CTAs in global memory
// A producer CTA publishes data with plain stores, then one thread raises a flag with a
// release at GPU scope; the consumer polls the flag with acquire loads.
__device__ __forceinline__ void flag_release(int* f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ int flag_acquire(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
// Bounded wait for a nonzero flag, with the same limit, abort flag and status bit as mbar_wait.
__device__ __forceinline__ bool flag_wait(const int* f, volatile int* abort_flag, unsigned long long limit_ns = 0) {
  if (flag_acquire(f)) return true;
  const unsigned long long t0 = global_ns();
  if (limit_ns == 0) limit_ns = wait_limit();
  const uint32_t mask = limit_ns < kWaitLimitNs ? 0u : 15u;
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);
    if (flag_acquire(f)) return true;
    if ((it & mask) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        record_status(TILEC_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- proxies / fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load global -> shared, completion signalled on `bar` (complete_tx).
// x is the innermost coordinate (elements); callers keep x * 4 bytes a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load (x innermost, z = batch index); same rules as tma_load_2d.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- epilogue
// Element-wise epilogue applied where C is written: v + bias (when given), then the
// activation (TILEC_MM_ACT_*: 0 none, 1 ReLU, 2 GELU with the exact erf form).
enum : int { kActNone = 0, kActRelu = 1, kActGelu = 2 };
__device__ __forceinline__ float epilogue(float v, float bias, int act) {
  v += bias;
  if (act == kActRelu) return fmaxf(v, 0.f);
  if (act == kActGelu) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  return v;
}

// ---------------------------------------------------------------- abort: poisoned output
// A kernel that gave up (a bounded wait expired, TILEC_DEV_TIMEOUT recorded) writes NaN
// over the part of its output it owns -- C, a split-K slab or a stream-K partial -- once
// every copy and MMA it issued has landed, so that an unfinished result is never left
// looking like a finished one (NaN also propagates through a split-K reduction).  One
// warp writes rows [row0, row0 + rows) x columns [col0, col0 + cols) of `out`, masked at
// M and N: lane j takes columns col0 + j, col0 + j + 32, ...
__device__ __forceinline__ void poison_rows(float* out, int64_t ldo, int64_t row0, int64_t rows, int64_t col0,
                                            int64_t cols, int64_t M, int64_t N, int lane) {
  const float nan = __int_as_float(0x7fc00000);
  const int64_t r_end = row0 + rows < M ? row0 + rows : M;
  const int64_t c_end = col0 + cols < N ? col0 + cols : N;
  for (int64_t r = row0; r < r_end; ++r)
    for (int64_t c = col0 + lane; c < c_end; c += 32) out[r * ldo + c] = nan;
}

// ---------------------------------------------------------------- cp.async (SIMT path)
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, issued by one thread.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row (lane base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- clusters (CTA pairs)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}
// Arrive on an mbarrier given by a shared::cluster address (own or peer CTA), release at
// CTA scope (orders this thread's prior operations for its own CTA only).
__device__ __forceinline__ void mbar_arrive_remote_cta(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(uint32_t(TILEC_WAIT_HINT_NS))
      : "memory");
  return ok != 0;
}
// Bounded wait with acquire at cluster scope (for barriers the peer CTA arrives on); the
// device's wait limit, as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  const unsigned long long limit_ns = wait_limit();
  const uint32_t mask = limit_ns < kWaitLimitNs ? 0u : 63u;
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & mask) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        record_status(TILEC_DEV_TIMEOUT);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// CTA-pair (cta_group::2) forms: allocation / deallocation by the same warp of both CTAs,
// MMA and commit issued by one thread of the leader CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same, kind::f16 with bf16 operands (both A and B bf16, K = 16 per instruction).
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at `cluster_addr` (either CTA of the pair) when every
// cta_group::2 tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}
// One arrive on the mbarrier at the same offset (`local_addr`, this CTA's shared-memory
// address) in both CTAs of the pair, from a single commit.  Each tcgen05 instruction the
// MMA thread issues costs it issue time; two single-CTA commits per stage instead of this
// one held the CTA-pair 3XTF32 kernel at 262-268 vs 286 TFLOP/s at 8192^3 (B200).
__device__ __forceinline__ void umma_commit_pair_both(uint32_t local_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          local_addr),
      "h"(static_cast<unsigned short>(3))
      : "memory");
}

// ---------------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor (tcgen05 format, version 1).
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1)
//   bits 49-51 base offset (0: tiles are 1024-byte aligned)  bits 61-63 layout type
//   Layout types: 2 = 128B swizzle (16-byte granules, 8-row atoms), 4 = 64B, 6 = 32B,
//   1 = 128B swizzle with 32-byte granules (4-row atoms of 128-byte rows) -- the only
//   layout the tensor core accepts for MN-major 32-bit (tf32) operands.
enum : uint32_t { kLayoutSw128 = 2, kLayoutSw64 = 4, kLayoutSw32 = 6, kLayoutSw128Base32 = 1 };

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::tf32, fp32 accumulate.
//   bits 4-5 D format (1 = f32), 7-9 A format (2 = tf32), 10-12 B format (2 = tf32),
//   15 A major (0 = K, 1 = MN), 16 B major (0 = K, 1 = MN), 17-22 N >> 3, 24-28 M >> 4.
// x1 row-major gives a K-major A and x2 row-major an MN-major B; their transposed views
// flip each.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int m, int n, bool a_mn = false, bool b_mn = true) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         ((uint32_t(n) >> 3) << 17) | ((uint32_t(m) >> 4) << 24);
}

// Instruction descriptor for kind::f16 with bf16 A and B (format 1), fp32 accumulate;
// major bits as in make_idesc_tf32.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int m, int n, bool a_mn = false, bool b_mn = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         ((uint32_t(n) >> 3) << 17) | ((uint32_t(m) >> 4) << 24);
}

// Two floats rounded to nearest-even bf16 and packed: `lo` in bits 0-15 (the lower
// address in shared memory), `hi` in bits 16-31.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Operand tile layouts of the tcgen05 kernels (runtime flags; the same bits as
// TILEC_MM_TRANS_A / TILEC_MM_TRANS_B).
//   default     A tile [128 x BK] K-major (one TMA box {BK, 128}, 64/128-byte swizzle);
//               B tile as slabs of [BK x 32] MN-major (boxes {32, BK}, 128-byte swizzle
//               with 32-byte granules).
//   kOpAMN      A stored K x M: A tile as 128/32 slabs of [BK x 32] MN-major, like B.
//   kOpBK       B stored N x K: B tile [BN x BK] K-major (one box {BK, BN}), like A.
enum : int { kOpAMN = 1, kOpBK = 2 };

}  // namespace tilec
