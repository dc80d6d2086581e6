// Shared device helpers for the gemq-b200 kernels (sm_100a only).
//
// * bounded mbarrier waits: every spin gives up after a wall-clock limit, records
//   where in the device error word and returns false, so no kernel can hang the GPU;
// * TMA (cp.async.bulk.tensor, no multicast), tcgen05 (MMA, TMEM alloc/ld, commit);
// * UMMA shared-memory / instruction descriptors for kind::f16 with f32 accumulate;
// * the packed-code -> fp16 dequant that reproduces the reference exactly:
//   w = fma.rn.f16(fp16(q), s, z')  (gemq/triton_kernels/utils.py:206-210).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#if !defined(__CUDA_ARCH__) || (__CUDA_ARCH__ >= 1000)
#else
#error "gemq-b200 kernels target sm_100a only"
#endif

namespace gemq {

// ------------------------------------------------------------------ device error word
// Bit layout of the error word: low 8 bits = error kind, upper bits = site id.
enum DeviceError : uint32_t {
  kDevOk = 0,
  kDevTimeoutTmaFull = 1,
  kDevTimeoutTmaEmpty = 2,
  kDevTimeoutAFull = 3,
  kDevTimeoutAEmpty = 4,
  kDevTimeoutAccFull = 5,
  kDevTimeoutAccEmpty = 6,
  kDevTimeoutDrain = 7,
  kDevBadExpert = 8,
  kDevBadBits = 9,
  kDevBadCachePos = 10,  // a KV-cache write past the cache's length (model harness)
  kDevTimeoutChain = 11,  // a down-projection item waited too long for its gate/up tiles
};

// g_device_error: first error recorded (any kind), reported by gemq_get_device_error.
// g_device_abort: set only when a wait expired; every other pending wait then gives
// up at once so a broken pipeline drains quickly. Input errors (an out-of-range
// expert id, a bad bit-width) are recorded without aborting other kernels.
extern __device__ uint32_t g_device_error;
extern __device__ uint32_t g_device_abort;

__device__ __forceinline__ void set_device_error(uint32_t code) { atomicCAS(&g_device_error, 0u, code); }
__device__ __forceinline__ void set_device_abort(uint32_t code) {
  set_device_error(code);
  atomicExch(&g_device_abort, 1u);
}
__device__ __forceinline__ bool device_error_set() {
  return *((volatile uint32_t*)&g_device_abort) != 0u;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wall-clock limit for any single wait inside a kernel (2 s). A healthy wait in
// these kernels lasts microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) { mbar_arrive(smem_u32(bar)); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may sleep up to `hint_ns` for the phase to
// complete (it wakes as soon as it does), so waiting warps do not re-issue polls
// that would steal issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Each sleeping poll lasts at most this long (the bound of every wait is checked
// between polls).
constexpr uint32_t kPollSleepNs = 100000;

// Waits until the phase with the given parity has completed. A try_wait suspends
// only briefly, so a polling warp takes issue slots from the warps that do the work
// on its sub-partition: a waiter off the critical path passes `sleep_ns` to sleep
// between polls. The abort word and the time bound are checked every 16 polls.
// Returns false (recording `code`) if the wait exceeds kWaitLimitNs, or once another
// wait expired (so a failed pipeline drains instead of spinning).
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, uint32_t code, uint32_t sleep_ns = 0) {
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t polls = 1;; ++polls) {
    if (sleep_ns != 0) __nanosleep(sleep_ns);
    if (mbar_try_wait_sleep(a, parity, kPollSleepNs)) return true;
    if ((polls & 15) == 0) {
      if (device_error_set()) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_device_abort(code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t code, uint32_t sleep_ns = 0) {
  return mbar_wait(smem_u32(bar), parity, code, sleep_ns);
}

// Bounded wait by every lane of a converged warp; the lanes agree on the outcome so
// the warp stays converged on every path. `bar` is a shared-memory address.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, uint32_t code, uint32_t sleep_ns = 0) {
  const bool ok = mbar_wait(bar, parity, code, sleep_ns);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t code, uint32_t sleep_ns = 0) {
  return warp_wait(smem_u32(bar), parity, code, sleep_ns);
}

// Completes a wait whose first try_wait (`tok`) was issued earlier, so that its
// latency overlapped other work; polls only if that try found the phase open.
__device__ __forceinline__ bool warp_wait_tok(uint32_t bar, uint32_t parity, bool tok, uint32_t code,
                                              uint32_t sleep_ns = 0) {
  if (__all_sync(0xffffffffu, tok)) return true;
  return warp_wait(bar, parity, code, sleep_ns);
}

// Waits for copies still in flight before a CTA exits: bounded by time only, so it
// also waits after another wait expired (the copies write this CTA's shared memory).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(a, parity, kPollSleepNs)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_abort(kDevTimeoutDrain);
      return false;
    }
  }
}

// ------------------------------------------------------------------ dependent launch
// The decode-path kernels are launched with programmatic stream serialization and
// call grid_dep_wait() before they touch any global buffer; the wait returns once the
// previous kernel in the stream has finished and its writes are visible (at once when
// launched without the attribute). No kernel triggers its dependents early: measured
// on B200, letting the next kernel become resident before this one finished slowed
// the decode stack by 5-10% (early kernels hold shared memory on SMs that a
// one-CTA-per-SM kernel behind them needs), while launching at completion through the
// programmatic edge gains about 1% over plain stream order.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// The one exception: the gate/up GEMM of a layer forward lets its down-projection
// GEMM be scheduled (onto SMs its own CTAs have left) once each of its CTAs has begun
// its last item; the down GEMM then waits per token tile on counters instead of on
// grid completion (tile_done_signal / tile_done_wait).
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Counter handshake between CTAs of two kernels. The producer: every lane stores its
// part, the warp converges, then one lane orders the warp's stores for the async proxy
// and at GPU scope and adds 1. The consumer: one lane polls with acquire loads until the
// count is reached, then a proxy fence so that its later TMA loads read those stores.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void tile_done_signal(int32_t* cnt) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    fence_proxy_async_global();
    __threadfence();
    atomicAdd(cnt, 1);
  }
  __syncwarp();
}
__device__ __forceinline__ int32_t ld_acquire_gpu(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// One thread; bounded like every wait (records kDevTimeoutChain and returns false).
__device__ __forceinline__ bool tile_done_wait(const int32_t* cnt, int32_t target) {
  if (ld_acquire_gpu(cnt) < target) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t polls = 1;; ++polls) {
      __nanosleep(200);
      if (ld_acquire_gpu(cnt) >= target) break;
      if ((polls & 15) == 0) {
        if (device_error_set()) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_device_abort(kDevTimeoutChain);
          return false;
        }
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// ------------------------------------------------------------------ TMA (no multicast)
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// L2 policy for data read once per launch (packed weights, scales, zeros): evicted
// first, so that streaming gigabytes of weights through L2 does not push out what is
// reused (activations, routing tables, the small kernels' code and data).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// As tma_load_2d, with an L2 cache policy (no multicast).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                                 int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from this GPU's global memory to shared memory, completing on `bar`, with an L2
// cache policy (no multicast).
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
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
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once all previously issued tcgen05.mma of this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp gets lane (base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Thread i of the warp writes 32 consecutive 32-bit columns of lane (base + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// Thread i of the warp writes 16 consecutive 32-bit columns of lane (base + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, one CTA: A is M lanes x K fp16, two
// consecutive k per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The eight K=16 steps of one 128-wide K stage, D[tmem] (+)= A[tmem] * B[smem]^T,
// issued from one asm block: step j reads A at column a_tmem + 8j and B through the
// descriptor advanced by 2j (j < 4) or BHI + 2(j - 4) (j >= 4) descriptor units of 16
// bytes (B is two 64-wide SW128 sub-tiles, the second BHI units on). Step 0
// accumulates when `accumulate` is non-zero, the others always. With no compiler
// barrier between the steps their operands are formed back to back: issued one asm
// statement (and one memory clobber) per MMA, each MMA cost about 28 cycles of issue,
// several times its execution at a 16-token tile, and the MMA warp paced the kernel.
// The descriptor's start field (bits 0-13, address >> 4) cannot carry: shared memory
// addresses stay below 2^18.
template <int BHI>
__device__ __forceinline__ void umma_f16_ts_k128(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      ".reg .b32 a1, a2, a3, a4, a5, a6, a7;\n\t"
      ".reg .b64 b1, b2, b3, b4, b5, b6, b7;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.u32 q, 0, 0;\n\t"
      "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\tadd.u32 a4, %1, 32;\n\t"
      "add.u32 a5, %1, 40;\n\tadd.u32 a6, %1, 48;\n\tadd.u32 a7, %1, 56;\n\t"
      "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\tadd.u64 b4, %2, %5;\n\t"
      "add.u64 b5, %2, %6;\n\tadd.u64 b6, %2, %7;\n\tadd.u64 b7, %2, %8;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], b5, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], b6, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], b7, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "n"(BHI), "n"(BHI + 2), "n"(BHI + 4), "n"(BHI + 6)
      : "memory");
}

// The four K=16 steps of one 64-wide K stage, D[tmem] (+)= A[smem] * B[smem]^T, both
// operands SW128 K-major: step j advances both descriptors by 2j units (32 bytes).
__device__ __forceinline__ void umma_f16_k64(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      ".reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.u32 q, 0, 0;\n\t"
      "add.u64 a1, %1, 2;\n\tadd.u64 a2, %1, 4;\n\tadd.u64 a3, %1, 6;\n\t"
      "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, q;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the canonical 128-byte
// swizzle: rows of 64 fp16 (128 B), 8-row atoms of 1024 B stacked along M/N.
// Fields per the sm100 UMMA descriptor: start>>4 [0,14), LBO>>4 [16,30) (unused
// for swizzled K-major), SBO>>4 [32,46), version=1 [46,48), layout [61,64) = 2.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: A,B fp16 K-major, D fp32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------ dequant helpers
// Byte offset of 16-byte chunk `c` (k = 8c..8c+7) of row `r` in a 128B-swizzled
// K-major tile (row = 128 bytes = 64 fp16).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
  return (r >> 3) * 1024u + (r & 7u) * 128u + ((c ^ (r & 7u)) << 4);
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// (1024 + q_lo, 1024 + q_hi) as fp16 pair -> exact (q_lo, q_hi) -> fma.rn.f16x2.
// fp16(q) for q < 1024 is exact, 1024+q is exact, the subtraction is exact, so the
// only rounding is the single one of the fused multiply-add, as in the reference.
__device__ __forceinline__ uint32_t dq_pair(uint32_t magic_pair, __half2 s2, __half2 z2) {
  const __half2 kMagic = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  __half2 q = __hsub2(u32_as_h2(magic_pair), kMagic);
  return h2_as_u32(__hfma2(q, s2, z2));
}

// fp16 exponent field of 2^(10 - o): a code placed at mantissa bit o (o + width <= 10)
// under this exponent reads as 2^(10 - o) + code, exactly.
__host__ __device__ constexpr uint32_t magic_exp(int o) { return static_cast<uint32_t>(25 - o) << 10; }

// Two codes of width NB at mantissa offset OA of the low half and OB of the high half
// of x -> exact (q_lo, q_hi) -> fma.rn.f16x2 with (s, z'). One lop3 extracts both
// codes and sets the exponents; the subtraction of the exponent's value is exact.
template <int NB, int OA, int OB>
__device__ __forceinline__ uint32_t dq_pair_at(uint32_t x, __half2 s2, __half2 z2) {
  static_assert(OA >= 0 && OB >= 0 && OA + NB <= 10 && OB + NB <= 10, "code must sit inside the fp16 mantissa");
  constexpr uint32_t cm = (1u << NB) - 1u;
  constexpr uint32_t mask = (cm << OA) | (cm << (OB + 16));
  constexpr uint32_t magic = (magic_exp(OB) << 16) | magic_exp(OA);
  const uint32_t m = (x & mask) | magic;
  __half2 q = __hsub2(u32_as_h2(m), u32_as_h2(magic));
  return h2_as_u32(__hfma2(q, s2, z2));
}

// Elects one lane of a converged warp (the lowest active one). Issuing tensor-core
// and bulk-copy instructions from an elected lane of a converged warp, rather than
// from a branch only lane 0 takes, lets the compiler keep their operands warp-uniform;
// measured on B200 the issue cost per tcgen05.mma drops about threefold.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// Scalar form, the definition the kernels must reproduce bit-exactly.
__device__ __forceinline__ __half dq_scalar(uint32_t q, __half s, __half z) {
  return __hfma(__uint2half_rn(q), s, z);
}

// One 3-bit code pair (ten codes per word, bits 30-31 unused) as the magic pair
// expected by dq_pair: codes at (word a, slot sa) and (word b, slot sb).
__device__ __forceinline__ uint32_t magic3(uint32_t wa, int sa, uint32_t wb, int sb) {
  return ((wa >> (3 * sa)) & 7u) | (((wb >> (3 * sb)) & 7u) << 16) | 0x64006400u;
}

// Decode the 32/NB codes of one word (NB in {1,2,4}) to fp16 and write them as
// consecutive-k 16-byte chunks through `emit(chunk_index, uint4)`.
template <int NB, typename Emit>
__device__ __forceinline__ void dq_word_pow2(uint32_t w, __half2 s2, __half2 z2, Emit&& emit) {
  constexpr int kCodes = 32 / NB;   // codes per word
  constexpr int kPairs = kCodes / 2;  // pairs (j, j + kPairs): half-words are kPairs codes apart
  constexpr uint32_t kMask = ((1u << NB) - 1u) * 0x00010001u;
  uint32_t p[kPairs];
#pragma unroll
  for (int j = 0; j < kPairs; ++j) p[j] = dq_pair(((w >> (NB * j)) & kMask) | 0x64006400u, s2, z2);
  // p[j] = (c_j, c_{j+kPairs}); regroup into chunks of 8 consecutive codes. Output
  // word m of chunk c holds codes (i, i+1), i = 8c + 2m: the low halves of p[i],
  // p[i+1] when i < kPairs, else the high halves of p[i-kPairs], p[i-kPairs+1].
#pragma unroll
  for (int c = 0; c < kCodes / 8; ++c) {
    uint32_t o[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i = 8 * c + 2 * m;
      o[m] = (i < kPairs) ? __byte_perm(p[i], p[i + 1], 0x5410u)
                          : __byte_perm(p[i - kPairs], p[i - kPairs + 1], 0x7632u);
    }
    emit(c, make_uint4(o[0], o[1], o[2], o[3]));
  }
}

__host__ __device__ constexpr int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace gemq
