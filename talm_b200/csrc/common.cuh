// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and the host-side error plumbing of
// the C ABI. Everything here is hand-written inline PTX for sm_100a.
#pragma once

#include <cuda.h>  // CUtensorMap (type only; the driver entry point is fetched at run time)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/talm.h"

namespace talm {

// ------------------------------------------------------------------------------------------
// host-side error plumbing
// ------------------------------------------------------------------------------------------
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
int current_sm_count();
bool device_is_sm100();
// Per-device caches of the library (kernel attributes, scratch addresses) hold this many
// devices; current_device() reports an ordinal beyond it as TALM_ERANGE.
constexpr int kMaxDevices = 64;
int current_device(int* dev);

// Launch timing (talm_profile_begin / talm_profile_end): a scope around one kernel launch that
// records CUDA events on the launch stream while profiling is on, and does nothing otherwise.
struct LaunchTimer {
  LaunchTimer(int kind, cudaStream_t stream);
  ~LaunchTimer();
  int kind_;
  cudaStream_t stream_;
  void* start_;
};

// Device status word set by bounded waits that gave up (read by talm_device_status). The
// library is built as one translation unit (talm.cu), so this header is seen once.
__device__ int g_device_status = 0;

// ------------------------------------------------------------------------------------------
// basic device helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may
// start (and run its set-up) before the previous kernel of its stream has finished; it waits
// here until that kernel has completed and its writes are visible. A no-op for a kernel
// launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Lets the next kernel of the stream (launched with programmatic stream serialization) start
// its set-up now; it still waits in grid_dependency_wait until this grid has completed.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait limit for every spin in this library: a wait that has not completed after this long
// records TALM_ETIMEOUT in g_device_status and gives up (the kernel then drains and returns).
// The limit of each device lives in g_wait_limit_ns (talm_set_wait_limit_ns changes it, for
// tests that let a wait run out); each wait reads it once, when it starts to spin.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s, the default
__device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint64_t wait_limit_ns() {
  return *const_cast<const volatile uint64_t*>(&g_wait_limit_ns);
}

__device__ __forceinline__ void record_timeout() {
  atomicCAS(&g_device_status, 0, TALM_ETIMEOUT);
}

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. `abort` (shared) is set by the
// first wait of the CTA that gives up, so that every other role stops waiting at once.
// Returns false when the wait gave up or the CTA is aborting.
// The polls of a bounded wait between two looks at the clock: the loop that reacts to the
// barrier holds no clock read and no global load, so a phase that completes while the thread
// spins is seen at once; the clock (and the limit, a global load) is read every 64 polls, which
// is a few microseconds at most.
constexpr uint32_t kPollsPerClockCheck = 64;

// Bounded wait for the phase with the given parity to complete. `abort` (shared) is set by the
// first wait of the CTA that gives up, so that every other role stops waiting at once.
// Returns false when the wait gave up or the CTA is aborting.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  uint64_t t0 = 0, limit = 0;
  for (uint32_t poll = 1;; ++poll) {
    if (mbar_test(bar, parity)) return true;
    if (*abort) return false;
    if (poll % kPollsPerClockCheck == 0) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
        limit = wait_limit_ns();
      } else if (now - t0 > limit) {
        *abort = 1;
        record_timeout();
        return false;
      }
    }
  }
}

// Bounded wait that ignores the CTA's abort flag: used on the way out, to let copies and MMAs
// already in flight land before shared memory and TMEM are released.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = 0, limit = 0;
  for (uint32_t poll = 1; !mbar_test(bar, parity); ++poll) {
    if (poll % kPollsPerClockCheck == 0) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
        limit = wait_limit_ns();
      } else if (now - t0 > limit) {
        record_timeout();
        return false;
      }
    }
  }
  return true;
}

// ------------------------------------------------------------------------------------------
// TMA tile loads (each CTA loads its own tiles)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// TMA tile store / reduce-add from shared memory (bulk groups; coordinates never negative)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t c0,
                                             int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src,
                                                  int32_t c0, int32_t c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// wait until at most N bulk groups of this thread still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until every bulk group of this thread has completed (writes performed)
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// named barrier among `count` threads (ids 1.. are free; 0 is __syncthreads)
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// named barrier that also ORs a predicate over the participating threads
__device__ __forceinline__ bool named_barrier_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// generic-proxy writes to shared memory -> visible to the async proxy (UMMA operand reads)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05: TMEM, UMMA
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane (base lane + t),
// columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 layout: version 1, base offset 0).
//   K-major tiles: rows of 128 B (64 fp16 of K), 8-row atoms -> SBO = 1024, LBO unused (1).
//   MN-major tiles: K-rows of 128 B (64 fp16 of MN), 8-row atoms -> SBO = 1024 between
//   8-row K groups, LBO = bytes between successive 64-element MN groups.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: fp16 A and B, fp32 D.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn_major,
                                                     bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (0u << 7) | (0u << 10)                    // A, B format: f16
         | ((a_mn_major ? 1u : 0u) << 15)            // A major
         | ((b_mn_major ? 1u : 0u) << 16)            // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ------------------------------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA tile load whose completion is counted on the pair leader's mbarrier (cta_group::2);
// `bar_cluster` is the shared::cluster address of that barrier. Each CTA loads
// its own half of the operands.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int32_t c0, int32_t c1,
                                                 int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem, both CTAs] (+)= A[smem, both CTAs] * B[smem, both CTAs]: M = 256 (128 rows per CTA),
// B split along N between the CTAs. Issued by one thread of the pair leader.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` (same shared-memory offset) in both CTAs of the pair when every UMMA
// issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// ------------------------------------------------------------------------------------------
// memory helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
// 16-byte store marked streaming (evict-first in L2): output that this kernel never reads back
__device__ __forceinline__ void st_v4_stream(void* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace talm

// Host: build a 2-D fp16 / fp32 tensor map with 128-byte swizzle. dims/strides in elements.
int talm_make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer);
int talm_make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer);
// Host: a row-major fp16 [rows][k] matrix (k % 64 == 0) as a 3-D tensor map {64, rows, k / 64}
// (128-byte swizzle) whose box {64, box_rows, 2} is two consecutive 64-column chunks of
// box_rows rows: one request fills two 128-byte-swizzled tiles of box_rows rows, back to back.
int talm_make_tmap_kchunks_f16(CUtensorMap* map, const void* base, uint64_t k, uint64_t rows,
                               uint64_t row_stride_elems, uint32_t box_rows);
