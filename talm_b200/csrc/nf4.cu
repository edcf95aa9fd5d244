// NF4 -> fp16 dequantisation (bandwidth-bound).
//
// Format (bitsandbytes NF4, as the reference uses it: solution/nf4_dequant.py:38-80,
// solution/qgroup.py:72-91): byte i of the packed buffer holds element 2i in its high nibble and
// element 2i+1 in its low nibble; a nibble selects one of 16 NormalFloat levels; the value is
// fp16(level * scale) with the product rounded to fp32 first (one multiply, no fusion), then
// rounded to nearest-even fp16. The scale of a block of `blocksize` elements is either an fp32
// absmax (per-projection path) or rebuilt from a double-quantised absmax:
// fp32(fp32(code[absmax8] * absmax2) + offset2) with two separate roundings (grouped path).
//
// Layout of the work: a warp expands 512-byte pieces of packed bytes (1024 outputs, 2 KiB of
// fp16). Lane l takes the 32-bit words l, 32+l, 64+l, 96+l of a piece (each read instruction
// covers 128 contiguous bytes) and writes each word's 8 outputs as one 16-byte store (each store
// instruction writes 512 contiguous bytes). The level table sits in shared memory: 16 floats in
// 16 distinct banks, so the per-nibble lookups never conflict.
//
// Three kernels share that layout. nf4_tma_kernel is the main path (16-byte aligned buffers,
// power-of-two block sizes 64..1024, whole 8 KiB tiles): the packed bytes and block scales reach
// shared memory through a cp.async.bulk ring fed by a producer warp. nf4_chunks_kernel covers the
// remaining whole pieces and the other word-aligned cases with direct loads, and
// nf4_bytes_kernel the ragged tail and any alignment, one byte per thread.
#include "common.cuh"

namespace talm {
namespace {

// The 16 NormalFloat levels, as listed in solution/nf4_dequant.py:32-35 (NF4_TABLE).
__constant__ float kNf4Levels[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

struct Fp32Scale {
  const float* absmax;
  int64_t base = 0;  // absolute index of block 0 of the launch
  __device__ __forceinline__ float operator()(int64_t block) const {
    return __ldg(absmax + base + block);
  }
};

struct DoubleQuantScale {
  const uint8_t* absmax8;
  const float* code;
  const float* absmax2;
  const float* offset2;
  int64_t qblock2;
  int64_t base = 0;  // absolute index of block 0 of the launch
  __device__ __forceinline__ float operator()(int64_t block) const {
    block += base;
    const int64_t b2 = block / qblock2;
    const float c = __ldg(code + __ldg(absmax8 + block));
    // qgroup.py:82-83 with enable_fp_fusion=False (:99): product rounded, then the sum.
    return __fadd_rn(__fmul_rn(c, __ldg(absmax2 + b2)), __ldg(offset2 + b2));
  }
};

__device__ __forceinline__ uint32_t nf4_pair(const float* lut, uint32_t byte, float scale) {
  const float first = __fmul_rn(lut[(byte >> 4) & 15u], scale);
  const float second = __fmul_rn(lut[byte & 15u], scale);
  return pack_half2(first, second);  // element 2i in the low half (little-endian order)
}

// Main kernel: whole 512-byte chunks. kWarpScale: block scales computed once per chunk by the
// lanes and shuffled (needs blocksize >= 64 so that a chunk touches at most 17 blocks).
template <class Scale, bool kWarpScale>
__global__ void __launch_bounds__(256) nf4_chunks_kernel(const uint8_t* __restrict__ packed,
                                                         uint32_t* __restrict__ out_pairs,
                                                         int64_t n_chunks, int64_t n_blocks,
                                                         int block_shift, int64_t blocksize,
                                                         Scale scale,
                                                         const float* __restrict__ levels) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = levels ? levels[threadIdx.x] : kNf4Levels[threadIdx.x];
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint32_t* words = reinterpret_cast<const uint32_t*>(packed);

  // Two chunks per iteration: all eight 128-byte loads of the pair are issued before any of
  // them is consumed, so each warp keeps 1 KiB of reads in flight.
  for (int64_t c = warp; c < n_chunks; c += 2 * n_warps) {
    const int64_t cc[2] = {c, c + n_warps};
    const bool second = cc[1] < n_chunks;
    uint32_t w[2][4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[0][k] = ld_stream_u32(words + cc[0] * 128 + k * 32 + lane);
    if (second) {
#pragma unroll
      for (int k = 0; k < 4; ++k) w[1][k] = ld_stream_u32(words + cc[1] * 128 + k * 32 + lane);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !second) break;
      float sc[4];
      const int64_t e0 = cc[h] * 1024;  // first element of the chunk
      if constexpr (kWarpScale) {
        const int64_t b0 = block_shift >= 0 ? (e0 >> block_shift) : e0 / blocksize;
        const float mine = (lane <= 16 && b0 + lane < n_blocks) ? scale(b0 + lane) : 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t e = e0 + static_cast<int64_t>(k * 32 + lane) * 8;
          const int64_t b = block_shift >= 0 ? (e >> block_shift) : e / blocksize;
          sc[k] = __shfl_sync(0xffffffffu, mine, static_cast<int>(b - b0));
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t e = e0 + static_cast<int64_t>(k * 32 + lane) * 8;
          sc[k] = scale(block_shift >= 0 ? (e >> block_shift) : e / blocksize);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t v = w[h][k];
        const uint32_t p0 = nf4_pair(lut, v & 0xffu, sc[k]);
        const uint32_t p1 = nf4_pair(lut, (v >> 8) & 0xffu, sc[k]);
        const uint32_t p2 = nf4_pair(lut, (v >> 16) & 0xffu, sc[k]);
        const uint32_t p3 = nf4_pair(lut, v >> 24, sc[k]);
        st_v4(out_pairs + (cc[h] * 128 + k * 32 + lane) * 4, p0, p1, p2, p3);
      }
    }
  }
}

// Byte-granular kernel for the ragged tail (and for any alignment / odd block size):
// bytes [byte0, byte1), one byte per thread, two fp16 stores each.
template <class Scale>
__global__ void __launch_bounds__(256) nf4_bytes_kernel(const uint8_t* __restrict__ packed,
                                                        __half* __restrict__ out, int64_t byte0,
                                                        int64_t byte1, int64_t blocksize,
                                                        Scale scale,
                                                        const float* __restrict__ levels) {
  __shared__ float lut[16];
  if (threadIdx.x < 16) lut[threadIdx.x] = levels ? levels[threadIdx.x] : kNf4Levels[threadIdx.x];
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = byte0 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < byte1; i += stride) {
    const uint32_t byte = packed[i];
    const float s = scale((2 * i) / blocksize);
    out[2 * i] = __float2half_rn(__fmul_rn(lut[byte >> 4], s));
    out[2 * i + 1] = __float2half_rn(__fmul_rn(lut[byte & 15u], s));
  }
}

// ------------------------------------------------------------------------------------------
// Bulk-copy pipelined kernel (the main path for aligned buffers and block sizes 64..1024).
// A tile is 8 KiB of packed bytes (16384 weights). A producer warp streams tiles and their block
// scales into a shared-memory ring with cp.async.bulk, so the loads run ahead of the
// arithmetic; each compute warp expands 512-byte pieces of a landed tile and writes them out
// with coalesced 16-byte stores (512 contiguous bytes per warp instruction), which need no
// wait. Scale modes: 0 = fp32 absmax per block, 1 = double-quantised.
// ------------------------------------------------------------------------------------------
// Output stores of the bulk kernel: streaming (evict-first) by default.
#ifndef NF4_STORE
#define NF4_STORE st_v4_stream
#endif
// The bulk kernel is launched with programmatic stream serialization (1) unless built with 0.
#ifndef NF4_PDL
#define NF4_PDL 1
#endif
constexpr int kTileBytes = 8192;          // packed bytes per tile
constexpr int kTmaStages = 4;
constexpr int kScaleBytes = 1024;         // room for a tile's scales (fp32 at blocksize 64)
constexpr int kComputeWarps = 8;
constexpr int kPiecesPerWarp = kTileBytes / 512 / kComputeWarps;
static_assert(kPiecesPerWarp == 2, "the scale exchange pairs 16 lanes with each of two pieces");
static_assert(kPiecesPerWarp * kComputeWarps * 512 == kTileBytes, "pieces must cover a tile");
static_assert(kScaleBytes >= kTileBytes / 8, "room for fp32 scales at blocksize 64");
constexpr int kNf4TmaThreads = 32 * (kComputeWarps + 1);
constexpr int kStageBytes = kTileBytes + kScaleBytes;
constexpr int kNf4TmaSmem = kTmaStages * kStageBytes + 256 * 4 + 64 + 128 + 128;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// q2_shift >= 0: every tile lies inside one second-level block (its index is tile >> q2_shift);
// otherwise each block's second-level index is a division by qblock2.
template <int MODE>
__global__ void __launch_bounds__(kNf4TmaThreads) nf4_tma_kernel(
    const uint8_t* __restrict__ packed, const void* __restrict__ scales,
    const float* __restrict__ code, const float* __restrict__ absmax2,
    const float* __restrict__ offset2, int64_t qblock2, int q2_shift,
    uint32_t* __restrict__ out_pairs, int64_t n_tiles, int bs_shift,
    const float* __restrict__ levels) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 127) &
                                           ~uintptr_t(127));
  uint8_t* stage_base = sm;                                              // [stages][tile+scales]
  float* code_s = reinterpret_cast<float*>(sm + kTmaStages * kStageBytes);  // [256]
  float* lut = code_s + 256;                                                // [16]
  uint64_t* full = reinterpret_cast<uint64_t*>(lut + 16);                   // [stages]
  uint64_t* empty = full + kTmaStages;                                      // [stages]
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int blocks_per_tile = (2 * kTileBytes) >> bs_shift;
  const uint32_t scale_bytes = MODE == 0 ? blocks_per_tile * 4 : blocks_per_tile;

  const int producer = 32 * kComputeWarps;  // lane 0 of the last warp
  auto issue = [&](int64_t tile, int stage) {
    uint8_t* st = stage_base + stage * kStageBytes;
    mbar_arrive_expect_tx(&full[stage], kTileBytes + scale_bytes);
    bulk_load(st, packed + tile * kTileBytes, kTileBytes, &full[stage]);
    bulk_load(st + kTileBytes,
              static_cast<const uint8_t*>(scales) + tile * static_cast<int64_t>(scale_bytes),
              scale_bytes, &full[stage]);
  };
  int issued = 0;  // producer lane: tiles issued
  if (tid == producer) {
    for (int i = 0; i < kTmaStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kComputeWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  // Launched with programmatic stream serialization: everything above overlapped the previous
  // kernel's tail; every read of an input and every write of the output comes after it has
  // completed. The next layer's launch may then start its own set-up at once.
  grid_dependency_wait();
  grid_launch_dependents();
  if (tid == producer) {
    // The first pass over the ring needs no wait for a free slot: with only the 64-byte level
    // table to fill, start it at once. The double-quantised path first fills its 1 KiB code
    // table, which every CTA reads from the same addresses; a burst of tile loads queued ahead
    // of those reads delays the first tile more than the early start gains (measured).
    if (MODE == 0)
      for (int64_t tile = blockIdx.x; tile < n_tiles && issued < kTmaStages; tile += gridDim.x)
        issue(tile, issued++);
  }
  if (tid < 16) lut[tid] = levels ? levels[tid] : kNf4Levels[tid];
  if (MODE == 1)
    for (int i = tid; i < 256; i += blockDim.x) code_s[i] = code[i];
  __syncthreads();
  volatile int* abort = &abort_flag;

  if (warp == kComputeWarps) {  // producer
    if (lane == 0) {
      int stage = issued % kTmaStages;
      uint32_t phase = issued / kTmaStages;
      for (int64_t tile = blockIdx.x + int64_t{issued} * gridDim.x; tile < n_tiles && !*abort;
           tile += gridDim.x) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort)) break;
        issue(tile, stage);
        ++issued;
        if (++stage == kTmaStages) { stage = 0; phase ^= 1; }
      }
      for (int i = 0; i < kTmaStages && i < issued; ++i) {  // copies land before exit
        if (--stage < 0) { stage = kTmaStages - 1; phase ^= 1; }
        mbar_drain(&full[stage], phase);
      }
    }
    return;
  }

  // compute warps: warp w takes pieces w, w + 8, ... of every tile (512 packed bytes each)
  int stage = 0;
  uint32_t phase = 0;
  // second-level scale of the next tile, loaded one tile ahead so its latency is hidden
  const bool tile_q2 = MODE == 1 && q2_shift >= 0;
  float a2_next = 0.0f, o2_next = 0.0f;
  if (tile_q2 && blockIdx.x < n_tiles) {
    a2_next = __ldg(absmax2 + (int64_t{blockIdx.x} >> q2_shift));
    o2_next = __ldg(offset2 + (int64_t{blockIdx.x} >> q2_shift));
  }
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const float a2 = a2_next, o2 = o2_next;
    if (tile_q2 && tile + gridDim.x < n_tiles) {
      a2_next = __ldg(absmax2 + ((tile + gridDim.x) >> q2_shift));
      o2_next = __ldg(offset2 + ((tile + gridDim.x) >> q2_shift));
    }
    if (!mbar_wait(&full[stage], phase, abort)) break;
    const uint8_t* st = stage_base + stage * kStageBytes;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(st);
    const int64_t tile_block0 = (tile * 2 * kTileBytes) >> bs_shift;
    constexpr int kWords = 4 * kPiecesPerWarp;  // words per lane per tile
    uint32_t v[kWords];
    float sc[kWords];
    // Double-quantised scales: the warp's two pieces span at most 32 blocks of >= 64 weights.
    // Lane L computes the scale at weight 64 * (L % 16) of piece L / 16 (every block of the
    // pieces holds one such sample) and the lanes exchange them by shuffle.
    float mine = 0.0f;
    if (MODE == 1) {
      const int blk = ((warp + kComputeWarps * (lane >> 4)) * 1024 + (lane & 15) * 64) >> bs_shift;
      float a = a2, o = o2;
      if (q2_shift < 0) {
        const int64_t b2 = (tile_block0 + blk) / qblock2;
        a = __ldg(absmax2 + b2);
        o = __ldg(offset2 + b2);
      }
      mine = __fadd_rn(__fmul_rn(code_s[st[kTileBytes + blk]], a), o);
    }
#pragma unroll
    for (int k = 0; k < kWords; ++k) {  // load phase: the lane's words and their scales
      const int byte = (warp + kComputeWarps * (k >> 2)) * 512 + (k & 3) * 128 + lane * 4;
      v[k] = words[byte >> 2];
      if (MODE == 0)
        sc[k] = reinterpret_cast<const float*>(st + kTileBytes)[(2 * byte) >> bs_shift];
      else  // this word's weights start at 256 * (k % 4) + 8 * lane of piece k / 4
        sc[k] = __shfl_sync(0xffffffffu, mine, (k >> 2) * 16 + (k & 3) * 4 + (lane >> 3));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);  // the stage is free once read into registers
    uint4* out4 = reinterpret_cast<uint4*>(out_pairs) + tile * (kTileBytes / 4);
#pragma unroll
    for (int k = 0; k < kWords; ++k) {
      const int byte = (warp + kComputeWarps * (k >> 2)) * 512 + (k & 3) * 128 + lane * 4;
      const uint32_t w = v[k];
      const uint32_t p0 = nf4_pair(lut, w & 0xffu, sc[k]);
      const uint32_t p1 = nf4_pair(lut, (w >> 8) & 0xffu, sc[k]);
      const uint32_t p2 = nf4_pair(lut, (w >> 16) & 0xffu, sc[k]);
      const uint32_t p3 = nf4_pair(lut, w >> 24, sc[k]);
      NF4_STORE(out4 + (byte >> 2), p0, p1, p2, p3);
    }
    if (++stage == kTmaStages) { stage = 0; phase ^= 1; }
  }
}

int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int s = 0;
  while ((int64_t{1} << s) < v) ++s;
  return s;
}

// The bulk-copy kernel for whole tiles; returns the bytes it covers (0 when it does not apply).
template <int MODE>
int64_t run_nf4_tma(const uint8_t* packed, const void* scales, const float* code,
                    const float* absmax2, const float* offset2, int64_t qblock2, uint16_t* out,
                    int64_t n_bytes, int64_t blocksize, const float* levels, cudaStream_t stream,
                    int* status) {
  *status = TALM_OK;
  const int shift = log2_exact(blocksize);
  const int64_t n_tiles = n_bytes / kTileBytes;
  const bool ok = shift >= 6 && shift <= 10 && n_tiles > 0 &&
                  (reinterpret_cast<uintptr_t>(packed) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(scales) & 15) == 0;
  if (!ok) return 0;
  // per device: the shared-memory opt-in and the resident CTAs per SM it allows
  static int per_sm_cache[2][kMaxDevices];
  int dev = 0;
  if ((*status = current_device(&dev)) != TALM_OK) return 0;
  int per_sm = per_sm_cache[MODE][dev];
  if (per_sm == 0) {
    cudaError_t e = cudaFuncSetAttribute(
        nf4_tma_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kNf4TmaSmem);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, nf4_tma_kernel<MODE>,
                                                        kNf4TmaThreads, kNf4TmaSmem);
    if (e != cudaSuccess) {
      *status = set_error(TALM_ECUDA, "nf4 bulk kernel set-up: %s", cudaGetErrorString(e));
      return 0;
    }
    if (per_sm < 1) per_sm = 1;
    per_sm_cache[MODE][dev] = per_sm;
  }
  const int64_t cap = int64_t{current_sm_count()} * per_sm;
  const int grid = static_cast<int>(n_tiles < cap ? n_tiles : cap);
  // one second-level block spans whole tiles when qblock * qblock2 is a multiple of the tile
  const int64_t span = blocksize * qblock2;
  const int q2_shift = span % (2 * kTileBytes) == 0 && log2_exact(span / (2 * kTileBytes)) >= 0
                           ? log2_exact(span / (2 * kTileBytes))
                           : -1;
  {
    LaunchTimer timer(TALM_KERNEL_NF4, stream);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(kNf4TmaThreads, 1, 1);
    cfg.dynamicSmemBytes = kNf4TmaSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = NF4_PDL;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, nf4_tma_kernel<MODE>, packed, scales, code, absmax2, offset2,
                       qblock2, q2_shift, reinterpret_cast<uint32_t*>(out), n_tiles, shift,
                       levels);
  }
  *status = check_launch("nf4 bulk kernel");
  return *status == TALM_OK ? n_tiles * kTileBytes : 0;
}

template <class Scale>
int run_nf4(const uint8_t* packed, uint16_t* out, int64_t n_elems, int64_t blocksize,
            Scale scale, const float* levels, cudaStream_t stream, int64_t done = 0) {
  const int64_t n_bytes = n_elems / 2;
  if (n_bytes == 0) return TALM_OK;
  const int sms = current_sm_count();
  if (sms <= 0) return set_error(TALM_ENODEV, "no CUDA device");
  // bytes [0, done) were handled by the bulk kernel: continue behind them
  packed += done;
  out += 2 * done;
  scale.base += (2 * done) / blocksize;
  n_elems -= 2 * done;
  const int64_t n_blocks = (n_elems + blocksize - 1) / blocksize;
  const int64_t n_left = n_elems / 2;
  const bool aligned = (reinterpret_cast<uintptr_t>(packed) & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const bool word_blocks = blocksize % 8 == 0;  // a 4-byte word never straddles two blocks
  done = 0;
  if (n_left == 0) return TALM_OK;
  if (aligned && word_blocks) {
    const int64_t n_chunks = n_left / 512;
    if (n_chunks > 0) {
      const int shift = log2_exact(blocksize);
      uint32_t* pairs = reinterpret_cast<uint32_t*>(out);
      // one resident wave: SMs x the blocks per SM the kernel's registers allow
      auto kernel = blocksize >= 64 ? nf4_chunks_kernel<Scale, true>
                                    : nf4_chunks_kernel<Scale, false>;
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess ||
          per_sm < 1)
        per_sm = 4;
      const int64_t want = (n_chunks + 15) / 16;  // 8 warps per block, 2 chunks per warp
      const int64_t cap = int64_t{sms} * per_sm;
      const int grid = static_cast<int>(want < cap ? want : cap);
      LaunchTimer timer(TALM_KERNEL_NF4, stream);
      kernel<<<grid, 256, 0, stream>>>(packed, pairs, n_chunks, n_blocks, shift, blocksize, scale,
                                      levels);
      int st = check_launch("nf4 chunk kernel");
      if (st != TALM_OK) return st;
      done = n_chunks * 512;
    }
  }
  if (done < n_left) {
    const int64_t rest = n_left - done;
    const int64_t want = (rest + 255) / 256;
    const int grid = static_cast<int>(want < int64_t{sms} * 8 ? want : int64_t{sms} * 8);
    LaunchTimer timer(TALM_KERNEL_NF4_TAIL, stream);
    nf4_bytes_kernel<Scale><<<grid, 256, 0, stream>>>(
        packed, reinterpret_cast<__half*>(out), done, n_left, blocksize, scale, levels);
    int st = check_launch("nf4 byte kernel");
    if (st != TALM_OK) return st;
  }
  return TALM_OK;
}

}  // namespace
}  // namespace talm

extern "C" {

int talm_nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n_elems,
                        int64_t blocksize, uint16_t* out, void* stream) {
  using namespace talm;
  if (n_elems < 0 || n_elems % 2 != 0)
    return set_error(TALM_EINVAL, "n_elems must be even and >= 0 (got %lld)", (long long)n_elems);
  if (blocksize < 2 || blocksize % 2 != 0)
    return set_error(TALM_EINVAL, "blocksize must be even and >= 2 (got %lld)",
                     (long long)blocksize);
  if (n_elems > 0 && (packed == nullptr || absmax == nullptr || out == nullptr))
    return set_error(TALM_EINVAL, "null pointer");
  int st = TALM_OK;
  const int64_t done = run_nf4_tma<0>(packed, absmax, nullptr, nullptr, nullptr, 1, out,
                                      n_elems / 2, blocksize, nullptr,
                                      static_cast<cudaStream_t>(stream), &st);
  if (st != TALM_OK) return st;
  return run_nf4(packed, out, n_elems, blocksize, Fp32Scale{absmax}, nullptr,
                 static_cast<cudaStream_t>(stream), done);
}

int talm_nf4_group_dequant(const uint8_t* packed, const uint8_t* absmax8, const float* code,
                           const float* absmax2, const float* offset2, const float* levels,
                           uint16_t* out, int64_t n_rows, int64_t qblock, int64_t qblock2,
                           void* stream) {
  using namespace talm;
  if (qblock < 2 || qblock % 2 != 0 || log2_exact(qblock / 2) < 0)
    return set_error(TALM_EINVAL, "qblock must be even with qblock/2 a power of two (got %lld)",
                     (long long)qblock);
  if (qblock2 < 1) return set_error(TALM_EINVAL, "qblock2 must be >= 1");
  if (n_rows < 0) return set_error(TALM_EINVAL, "n_rows must be >= 0");
  if (n_rows * (qblock / 2) >= (int64_t{1} << 31))
    return set_error(TALM_ERANGE, "layer of %lld pairs exceeds 2^31",
                     (long long)(n_rows * (qblock / 2)));
  if (n_rows > 0 && (!packed || !absmax8 || !code || !absmax2 || !offset2 || !levels || !out))
    return set_error(TALM_EINVAL, "null pointer");
  int st = TALM_OK;
  const int64_t done = run_nf4_tma<1>(packed, absmax8, code, absmax2, offset2, qblock2, out,
                                      n_rows * qblock / 2, qblock, levels,
                                      static_cast<cudaStream_t>(stream), &st);
  if (st != TALM_OK) return st;
  DoubleQuantScale scale{absmax8, code, absmax2, offset2, qblock2};
  return run_nf4(packed, out, n_rows * qblock, qblock, scale, levels,
                 static_cast<cudaStream_t>(stream), done);
}

}  // extern "C"
