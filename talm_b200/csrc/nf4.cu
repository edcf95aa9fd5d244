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
// Layout of the work: one warp handles a 512-byte chunk of packed bytes (1024 outputs, 2 KiB of
// fp16). Lane l loads the 32-bit words l, 32+l, 64+l, 96+l of the chunk (each load instruction
// reads 128 contiguous bytes) and writes each word's 8 outputs as one 16-byte store (each store
// instruction writes 512 contiguous bytes). The block scales of a chunk (at most 17 for
// blocksize >= 64) are computed once by lanes 0..16 and broadcast with shuffles. The level table
// sits in shared memory: 16 floats in 16 distinct banks, so the per-nibble lookups never
// conflict. Chunks are distributed grid-stride over a grid sized to the SM count.
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
  __device__ __forceinline__ float operator()(int64_t block) const { return __ldg(absmax + block); }
};

struct DoubleQuantScale {
  const uint8_t* absmax8;
  const float* code;
  const float* absmax2;
  const float* offset2;
  int64_t qblock2;
  __device__ __forceinline__ float operator()(int64_t block) const {
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

int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int s = 0;
  while ((int64_t{1} << s) < v) ++s;
  return s;
}

template <class Scale>
int run_nf4(const uint8_t* packed, uint16_t* out, int64_t n_elems, int64_t blocksize,
            Scale scale, const float* levels, cudaStream_t stream) {
  const int64_t n_bytes = n_elems / 2;
  if (n_bytes == 0) return TALM_OK;
  const int64_t n_blocks = (n_elems + blocksize - 1) / blocksize;
  const int sms = current_sm_count();
  if (sms <= 0) return set_error(TALM_ENODEV, "no CUDA device");
  const bool aligned = (reinterpret_cast<uintptr_t>(packed) & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const bool word_blocks = blocksize % 8 == 0;  // a 4-byte word never straddles two blocks
  int64_t done = 0;
  if (aligned && word_blocks) {
    const int64_t n_chunks = n_bytes / 512;
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
  if (done < n_bytes) {
    const int64_t rest = n_bytes - done;
    const int64_t want = (rest + 255) / 256;
    const int grid = static_cast<int>(want < int64_t{sms} * 8 ? want : int64_t{sms} * 8);
    LaunchTimer timer(TALM_KERNEL_NF4_TAIL, stream);
    nf4_bytes_kernel<Scale><<<grid, 256, 0, stream>>>(
        packed, reinterpret_cast<__half*>(out), done, n_bytes, blocksize, scale, levels);
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
  return run_nf4(packed, out, n_elems, blocksize, Fp32Scale{absmax}, nullptr,
                 static_cast<cudaStream_t>(stream));
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
  DoubleQuantScale scale{absmax8, code, absmax2, offset2, qblock2};
  return run_nf4(packed, out, n_rows * qblock, qblock, scale, levels,
                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
