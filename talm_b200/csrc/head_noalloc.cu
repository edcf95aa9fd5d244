// talm_head_shard_noalloc: the fused-head slice walk with its scratch in a static device array.
//
// Who needs it: callers that cannot allocate device memory at the point where they call the
// head - code running inside a pre-planned memory pool that must not grow, an embedding host
// whose allocator is owned by another runtime, or a caller that has no allocator binding at all
// (a C program linking only this library). talm_head_shard asks such callers for a workspace
// they cannot produce; this entry point takes the same inputs and outputs and uses a scratch
// region that lives in the library image instead.
//
// The scratch is one file-scope __device__ array of kScratchBytes (16 MiB). Every GPU on which
// the library is loaded holds it until the process exits. A call whose slice walk needs more
// (see talm_head_workspace_size: it grows with n_grad x vocab_chunk) is refused with TALM_ERANGE
// before anything is enqueued; a smaller vocab_chunk or fewer rows per call fit.
//
// Set-up: host code cannot use the array's name as a device address (on the host it names a
// stand-in object). The first call on each device, with that device current, looks the device
// address up with cudaGetSymbolAddress and caches it; make that first call before any stream
// capture begins. Later calls only read the cache.
//
// Sharing: every call on a device uses the same scratch, and it keeps what the last call left.
// No scratch state carries from one call to the next: the scratch holds the slice
// probabilities and the per-part statistics, and a call writes each of them before it reads
// them; what must start at zero (the caller's stats and acc) is cleared by talm_head_shard
// itself. Two calls whose kernels overlap on the GPU (different streams without an ordering
// between them) race on the scratch: order them, or use talm_head_shard.
//
// No allocation happens here: no device-memory allocation or release call, no allocating
// library routine.
#include <mutex>

#include "common.cuh"

namespace talm {
namespace head_noalloc {

constexpr size_t kScratchBytes = size_t{16} << 20;  // 16 MiB per device

static __device__ __align__(256) unsigned char g_head_scratch[kScratchBytes];

static void* g_scratch_address[kMaxDevices];
static std::mutex g_scratch_mutex;

// Device address of g_head_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = 0;
  const int st = current_device(&dev);
  if (st != TALM_OK) return st;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_head_scratch);
    if (err != cudaSuccess || p == nullptr)
      return set_error(TALM_ECUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                       cudaGetErrorString(err));
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return TALM_OK;
}

}  // namespace head_noalloc
}  // namespace talm

extern "C" {

int talm_head_shard_noalloc(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                            int64_t ld_weight, const int64_t* targets, int64_t n_tokens,
                            int64_t n_grad, int64_t hidden_size, int64_t vocab_cols,
                            int64_t vocab_col0, int64_t vocab_chunk, float* stats, float* acc,
                            void* stream) {
  using namespace talm;
  size_t need = 0;
  int st = talm_head_workspace_size(n_tokens, n_grad, hidden_size, vocab_cols, vocab_chunk,
                                    &need);
  if (st != TALM_OK) return st;
  if (need > head_noalloc::kScratchBytes)
    return set_error(TALM_ERANGE,
                     "this call needs %zu bytes of scratch but the static scratch holds %zu "
                     "(lower vocab_chunk or the labelled rows per call, or pass a workspace to "
                     "talm_head_shard)",
                     need, head_noalloc::kScratchBytes);
  void* scratch = nullptr;
  st = head_noalloc::scratch_address(&scratch);
  if (st != TALM_OK) return st;
  return talm_head_shard(hidden, ld_hidden, weight, ld_weight, targets, n_tokens, n_grad,
                         hidden_size, vocab_cols, vocab_col0, vocab_chunk, stats, acc, scratch,
                         head_noalloc::kScratchBytes, stream);
}

}  // extern "C"
