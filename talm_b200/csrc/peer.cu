// The exchange step of the vocabulary-parallel head over NVLink peer memory.
//
// Every rank holds one "peer buffer" (allocated by the caller, the same size on every rank) and
// maps the other ranks' buffers into its address space (CUDA IPC handles, exchanged by the
// caller). Kernels then read and write peers' memory with plain loads and stores over NVLink.
// The buffer holds, at offsets every rank computes the same way (peer_layout):
//
//   flags     [3][world] u32  phase flags: flags[ph][src] = epoch once rank src finished phase ph
//                              of call `epoch` (written by src with a system-scope release)
//   counters  [3] u32         local: CTAs of this rank's kernel of phase ph that are done
//   stats     [world][n][8]   every rank's per-row statistics (phase 0 writes slot `rank` on
//                              every rank)
//   recv      [world][rpr][h] fp32 partial gradients of the rows this rank owns (rows
//                              rank * rpr ..), one slot per source rank (phase 1)
//   dh        [n][h] fp16     the reduced gradient, every row (phase 2 writes this rank's rows
//                              on every rank)
//
// Per call: publish statistics (phase 0) -> wait + merge -> finalize the partial gradient and
// scatter each row to its owner (phase 1) -> wait + reduce the owned rows in rank order, round
// to fp16 and write them to every rank (phase 2) -> wait + copy the gradient out. This replaces
// NCCL's all_gather of the statistics and all_reduce of the fp32 gradient: the partial gradient
// crosses NVLink once (to its owner) instead of twice, and the gathered result is fp16.
//
// A phase ends when the last CTA of the writing kernel (a device-scope counter) raises the
// phase flag of its rank on every rank, after every CTA fenced its stores at system scope. A
// waiting CTA polls its own flags with acquire loads; every wait is bounded (g_wait_limit_ns,
// 2 s by default) and records TALM_ETIMEOUT on expiry, after which the kernel returns without
// its work. Data that other GPUs write while a kernel runs is read with L2-only loads (__ldcg).
#include <string.h>

#include "common.cuh"

namespace talm {
namespace peer {

constexpr int kPhases = 3;

struct PeerLayout {
  size_t flags, counters, stats, recv, dh, bytes;
  int64_t rpr;  // rows per rank
};

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

inline PeerLayout peer_layout(int64_t world, int64_t n, int64_t hidden) {
  PeerLayout L;
  size_t off = 0;
  L.flags = off;
  off = align256(off + sizeof(uint32_t) * kPhases * world);
  L.counters = off;
  off = align256(off + sizeof(uint32_t) * kPhases);
  L.stats = off;
  off = align256(off + sizeof(float) * world * n * TALM_HEAD_STATS);
  L.rpr = (n + world - 1) / world;
  L.recv = off;
  off = align256(off + sizeof(float) * world * L.rpr * hidden);
  L.dh = off;
  off = align256(off + sizeof(uint16_t) * n * hidden);
  L.bytes = off;
  return L;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// CTA-wide: thread 0 waits (bounded) until every rank's flag of the phase reached `epoch`;
// every thread gets the outcome.
__device__ bool cta_wait_phase(const uint8_t* own, size_t flags_off, int phase, int world,
                               uint32_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(own + flags_off) + phase * world;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = wait_limit_ns();
    int good = 1;
    for (int q = 0; q < world && good; ++q) {
      while (static_cast<int32_t>(ld_acquire_sys(f + q) - epoch) < 0) {
        if (globaltimer_ns() - t0 > limit) {
          record_timeout();
          good = 0;
          break;
        }
        __nanosleep(100);
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

// CTA-wide, at the end of a writing kernel: every thread fences its stores at system scope;
// the last CTA of the grid raises flag (phase, rank) on every rank.
__device__ void cta_signal_phase(uint8_t* own, const unsigned long long* peers, size_t flags_off,
                                 size_t counters_off, int phase, int rank, int world,
                                 uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* counter = reinterpret_cast<uint32_t*>(own + counters_off) + phase;
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      *counter = 0;  // ready for the next call (stream-ordered after this kernel)
      __threadfence_system();
      for (int q = 0; q < world; ++q)
        st_release_sys(reinterpret_cast<uint32_t*>(peers[q] + flags_off) + phase * world + rank,
                       epoch);
    }
  }
}

// Phase 0: this rank's [n][8] statistics into slot `rank` of every rank's stats region.
__global__ void __launch_bounds__(256) publish_stats_kernel(const float4* __restrict__ stats,
                                                            long long n4,
                                                            const unsigned long long* peers,
                                                            PeerLayout L, int rank, int world,
                                                            uint32_t epoch) {
  uint8_t* own = reinterpret_cast<uint8_t*>(peers[rank]);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = stats[i];
    for (int k = 1; k <= world; ++k) {  // ranks after this one first: no common first receiver
      const int q = (rank + k) % world;
      reinterpret_cast<float4*>(peers[q] + L.stats)[rank * n4 + i] = v;
    }
  }
  cta_signal_phase(own, peers, L.flags, L.counters, 0, rank, world, epoch);
}

// Phase 2: the rows this rank owns, summed over the source ranks in rank order, rounded to fp16
// and written to every rank's dh region. 8 columns per thread (hidden % 8 == 0).
__global__ void __launch_bounds__(256) reduce_gather_kernel(const unsigned long long* peers,
                                                            PeerLayout L, int rank, int world,
                                                            int n, int hidden, uint32_t epoch) {
  uint8_t* own = reinterpret_cast<uint8_t*>(peers[rank]);
  if (!cta_wait_phase(own, L.flags, 1, world, epoch)) return;
  const long long row0 = static_cast<long long>(rank) * L.rpr;
  const long long rows = max(0LL, min(static_cast<long long>(L.rpr), n - row0));
  const int per_row = hidden / 8;
  const float* recv = reinterpret_cast<const float*>(own + L.recv);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < rows * per_row; i += stride) {
    const long long j = i / per_row;
    const int c = static_cast<int>(i - j * per_row) * 8;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r) {
      const float4* src =
          reinterpret_cast<const float4*>(recv + ((static_cast<long long>(r) * L.rpr + j) * hidden + c));
      const float4 x = __ldcg(src), y = __ldcg(src + 1);
      a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
      a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
    }
    const uint4 h = make_uint4(pack_half2(a[0], a[1]), pack_half2(a[2], a[3]),
                               pack_half2(a[4], a[5]), pack_half2(a[6], a[7]));
    const long long o = (row0 + j) * hidden + c;
    for (int k = 1; k <= world; ++k) {  // ranks after this one first: no common first receiver
      const int q = (rank + k) % world;
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(peers[q] + L.dh) + o) = h;
    }
  }
  cta_signal_phase(own, peers, L.flags, L.counters, 2, rank, world, epoch);
}

// After phase 2: the gathered fp16 gradient out of the peer buffer into the caller's tensor.
__global__ void __launch_bounds__(256) gather_finish_kernel(const uint8_t* own, PeerLayout L,
                                                            int world, long long n16,
                                                            uint32_t epoch,
                                                            uint4* __restrict__ out) {
  if (!cta_wait_phase(own, L.flags, 2, world, epoch)) return;
  const uint4* src = reinterpret_cast<const uint4*>(own + L.dh);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
       i += stride)
    out[i] = __ldcg(src + i);
}

int grid_for(long long items) {
  const int sms = current_sm_count();
  const long long want = (items + 255) / 256;
  const long long cap = static_cast<long long>(sms > 0 ? sms : 1) * 4;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  }
  return fn;
}

int check_peer_args(int64_t world, int64_t rank, int64_t n_tokens, int64_t hidden) {
  if (world < 1 || rank < 0 || rank >= world || n_tokens < 0)
    return set_error(TALM_EINVAL, "need 0 <= rank < world and n_tokens >= 0");
  if (hidden < 8 || hidden % 8 != 0)
    return set_error(TALM_EINVAL, "hidden columns must be a positive multiple of 8");
  if (n_tokens >= (int64_t{1} << 30)) return set_error(TALM_ERANGE, "n_tokens beyond 2^30");
  return TALM_OK;
}

}  // namespace peer
}  // namespace talm

extern "C" {

int talm_peer_buffer_size(int64_t world, int64_t n_tokens, int64_t hidden, size_t* bytes) {
  using namespace talm;
  int st = peer::check_peer_args(world, 0, n_tokens, hidden);
  if (st != TALM_OK) return st;
  if (!bytes) return set_error(TALM_EINVAL, "null pointer");
  *bytes = peer::peer_layout(world, n_tokens, hidden).bytes;
  return TALM_OK;
}

int talm_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  using namespace talm;
  if (!ptr || !handle || !offset) return set_error(TALM_EINVAL, "null pointer");
  peer::AddressRangeFn range = peer::address_range_fn();
  if (!range) return set_error(TALM_ECUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(TALM_ECUDA, "cuMemGetAddressRange failed for %p", ptr);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return set_error(TALM_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == TALM_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return TALM_OK;
}

int talm_ipc_import(const void* handle, int64_t offset, void** ptr) {
  using namespace talm;
  if (!handle || !ptr || offset < 0) return set_error(TALM_EINVAL, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return set_error(TALM_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return TALM_OK;
}

int talm_ipc_close(void* ptr, int64_t offset) {
  using namespace talm;
  if (!ptr || offset < 0) return set_error(TALM_EINVAL, "bad argument");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (e != cudaSuccess)
    return set_error(TALM_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return TALM_OK;
}

int talm_head_publish_stats(const float* stats, int64_t n_tokens, int64_t hidden, int64_t rank,
                            int64_t world, const uint64_t* peers, uint32_t epoch, void* stream) {
  using namespace talm;
  int st = peer::check_peer_args(world, rank, n_tokens, hidden);
  if (st != TALM_OK) return st;
  if (!peers || (n_tokens > 0 && !stats)) return set_error(TALM_EINVAL, "null pointer");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden);
  const long long n4 = n_tokens * (TALM_HEAD_STATS / 4);
  LaunchTimer timer(TALM_KERNEL_PEER_PUBLISH, static_cast<cudaStream_t>(stream));
  peer::publish_stats_kernel<<<peer::grid_for(n4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(stats), n4,
      reinterpret_cast<const unsigned long long*>(peers), L, static_cast<int>(rank),
      static_cast<int>(world), epoch);
  return check_launch("publish stats kernel");
}

int talm_head_reduce_gather(int64_t n_tokens, int64_t hidden, int64_t rank, int64_t world,
                            const uint64_t* peers, uint32_t epoch, void* stream) {
  using namespace talm;
  int st = peer::check_peer_args(world, rank, n_tokens, hidden);
  if (st != TALM_OK) return st;
  if (!peers) return set_error(TALM_EINVAL, "null pointer");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden);
  const long long items = L.rpr * (hidden / 8);
  LaunchTimer timer(TALM_KERNEL_PEER_REDUCE, static_cast<cudaStream_t>(stream));
  peer::reduce_gather_kernel<<<peer::grid_for(items), 256, 0,
                               static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const unsigned long long*>(peers), L, static_cast<int>(rank),
      static_cast<int>(world), static_cast<int>(n_tokens), static_cast<int>(hidden), epoch);
  return check_launch("reduce gather kernel");
}

int talm_head_gather_finish(int64_t n_tokens, int64_t hidden, int64_t world,
                            const void* own_buffer, uint32_t epoch, uint16_t* out,
                            void* stream) {
  using namespace talm;
  int st = peer::check_peer_args(world, 0, n_tokens, hidden);
  if (st != TALM_OK) return st;
  if (!own_buffer || (n_tokens > 0 && !out)) return set_error(TALM_EINVAL, "null pointer");
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0)
    return set_error(TALM_EINVAL, "out must be 16-byte aligned");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden);
  const long long n16 = n_tokens * hidden / 8;
  LaunchTimer timer(TALM_KERNEL_PEER_FINISH, static_cast<cudaStream_t>(stream));
  peer::gather_finish_kernel<<<peer::grid_for(n16), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(own_buffer), L, static_cast<int>(world), n16, epoch,
      reinterpret_cast<uint4*>(out));
  return check_launch("gather finish kernel");
}

}  // extern "C"
