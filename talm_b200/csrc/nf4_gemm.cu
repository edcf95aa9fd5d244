// Fused NF4 dequantisation + GEMM (W4A16) on tcgen05: the products of a layer's 4-bit
// projections without the fp16 copy of their weights.
//
// The grouped path (solution/qgroup.py:346-355, GroupLinear) dequantises a whole layer into an
// fp16 buffer (one launch, 93.6 MB written and read back per layer and pass) and multiplies with
// cuBLAS. Here the weights stay packed in HBM: eight converter warps per CTA read the packed
// bytes of the tile's weight rows (4 KiB per stage instead of 16 KiB of fp16; two stages ahead,
// from L2 for all but the first pair row) and expand them to fp16 in the 128-byte-swizzled
// operand layout the tensor cores read, and the MMA warp of the CTA pair issues tcgen05.mma on
// them. Each weight is rebuilt exactly as the grouped
// kernel rebuilds it: fp16(level * scale), scale = fp32(fp32(code[absmax8] * absmax2) + offset2)
// with both products rounded to fp32 separately (solution/qgroup.py:82-83).
//
//   forward  (TRANS = false): y[T, R] = x[T, K] . W[R, K]^T (+ bias[R]); B = W, K-major
//   backward (TRANS = true):  y[T, K] = g[T, R] . W[R, K] (the input gradient of the frozen
//                             projection, GroupLinear.backward); B = W, MN-major
//
// W is R consecutive rows of K weights in a LayerGroup's buffers: packed bytes (row r at byte
// r * K / 2, element 2i in the high nibble of byte i), one coded scale per 64 weights (qblock
// 64: absmax8[r * K / 64 + k / 64]) and the group's second-level scales and offsets indexed by
// the group-wide absmax row (absmax_row0 + that index) / qblock2.
//
// CTA pairs (cluster of 2, cta_group::2), tiles of 256 x 256 outputs, K staged 64 at a time:
//   warp 0       TMA producer: this CTA's 128 rows of A (counted on the leader's barrier)
//   warp 1       MMA issuer (pair leader): 4 x tcgen05.mma (K = 16) per stage into TMEM
//   warps 2-9    converters: half a weight row (forward) or half of a row's 64 columns
//                (backward) per thread and stage, 64 bytes of fp16 into the stage's B tile,
//                then a cluster-scope arrive per warp on the leader's stage barrier
//   warps 10-17  epilogue: TMEM -> fp32 (+ bias) -> fp16 -> swizzled staging -> TMA store
// Every wait is bounded (2 s); a wait that gives up aborts the CTA's roles, drains what is in
// flight, frees TMEM and records TALM_ETIMEOUT in the device status word.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace talm {
namespace nf4g {

constexpr int BM = 128;                 // A rows per CTA = TMEM lanes
constexpr int PAIR_ROWS = 2 * BM;
constexpr int BN = 256;                 // output columns of a pair tile (128 per CTA's B half)
constexpr int BK = 64;                  // reduction per stage = one absmax block (qblock 64)
constexpr int STAGES = 5;
constexpr int A_BYTES = BM * BK * 2;          // 16 KiB
constexpr int B_BYTES = (BN / 2) * BK * 2;    // 16 KiB: this CTA's half of B, fp16, swizzled
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 32 KiB
constexpr int TMEM_COLS = 2 * BN;
constexpr int STAGING_PER_GROUP = 2;
constexpr int STAGING_BYTES = 2 * STAGING_PER_GROUP * 16384;
constexpr int TABLE_BYTES = (256 + 16) * 4;  // second-level code table + NF4 levels
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + STAGING_BYTES + TABLE_BYTES + 1024 + 512;
constexpr int CONV_WARPS = 8;
constexpr int EPI_GROUPS = 2;
constexpr int EPI_COLS = BN / EPI_GROUPS;  // 128
constexpr int EPI_WARPS = 4 * EPI_GROUPS;
constexpr int EPI_THREADS = 128;
constexpr int THREADS = 32 * (2 + CONV_WARPS + EPI_WARPS);  // 576
constexpr int FIRST_EPI_WARP = 2 + CONV_WARPS;

static_assert(SMEM_BYTES <= 232448, "shared memory of one CTA");
static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1 KiB alignment of swizzled tiles");

template <bool TRANS>
__host__ __device__ constexpr uint32_t idesc() {
  return idesc_f16_f32(PAIR_ROWS, BN, false, TRANS);
}

struct Ctl {
  uint64_t full[STAGES];      // leader: A bytes of both CTAs + 2 x CONV_WARPS warp arrivals
  uint64_t empty[STAGES];     // each CTA: the pair's MMAs finished reading the stage
  uint64_t tfull[2];          // each CTA: its half of an accumulator buffer is complete
  uint64_t tempty[2];         // leader: both CTAs' epilogues drained the buffer
  uint64_t drain;             // MMA issuer: every UMMA issued has completed
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int n_rows;         // T: rows of A and of the output
  int n_out;          // output columns: R (forward) or K (backward)
  int k_blocks;       // reduction / 64: K / 64 (forward) or R / 64 (backward)
  int n_pair_rows;    // ceil(T / 256)
  int n_col_tiles;    // ceil(n_out / 256)
  int n_tiles;        // n_pair_rows * n_col_tiles
  int w_rows;         // R
  int w_blocks;       // K / 64: coded scales per weight row
  long long absmax_row0;  // group-wide absmax index of this weight's first block
  int qblock2;
  const uint8_t* packed;   // this weight's packed bytes (row r at r * K / 2)
  const uint8_t* absmax8;  // this weight's coded scales
  const float* absmax2;    // the group's second-level scales
  const float* offset2;    // the group's per-second-level-block offsets
  const float* code;       // 256 entries
  const float* levels;     // 16 entries
  const __half* bias;      // [n_out] or null (forward only)
};

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// Bounded wait with cluster-scope acquire: the stage barrier also counts the peer CTA's
// converter warps, which arrive with cluster-scope release after writing their B half.
__device__ __forceinline__ bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  if (mbar_test_cluster(bar, parity)) return true;
  uint64_t t0 = 0, limit = 0;
  for (uint32_t poll = 1;; ++poll) {
    if (mbar_test_cluster(bar, parity)) return true;
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

// 16 bytes of row r, chunk q (0..7) of a 128-byte-swizzled tile of 128-byte rows.
__device__ __forceinline__ void put_chunk(uint8_t* tile, int r, int q, uint4 v) {
  *reinterpret_cast<uint4*>(tile + r * 128 + ((q ^ (r & 7)) << 4)) = v;
}

// The eight fp16 weights of four packed bytes (little-endian word w: byte j holds weights 2j
// (high nibble) and 2j + 1 (low nibble)), each fp16(level * scale).
__device__ __forceinline__ uint4 expand8(uint32_t w, float scale, const float* lv) {
  uint32_t h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b = (w >> (8 * j)) & 0xFFu;
    h[j] = pack_half2(__fmul_rn(lv[b >> 4], scale), __fmul_rn(lv[b & 15u], scale));
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// Tile t of this pair: rows [pr * 256, +256) x output columns [ct * 256, +256); the pairs
// running at the same time share the column tile (its weights stay in L2).
__device__ __forceinline__ void tile_of(const Params& p, int t, int& pr, int& ct) {
  pr = t % p.n_pair_rows;
  ct = t / p.n_pair_rows;
}

template <bool TRANS>
__global__ void __launch_bounds__(THREADS, 1)
    nf4_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_y, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  float* code_s = reinterpret_cast<float*>(staging + STAGING_BYTES);
  float* level_s = code_s + 256;
  Ctl* ctl = reinterpret_cast<Ctl*>(level_s + 16);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  for (int i = threadIdx.x; i < 256 + 16; i += THREADS)
    code_s[i] = i < 256 ? p.code[i] : p.levels[i - 256];
  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_y);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1 + 2 * CONV_WARPS);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], 2 * EPI_WARPS);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers, tables and TMEM of both CTAs ready
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer (both CTAs)
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = pair; t < p.n_tiles && !*abort; t += n_pairs) {
        int pr, ct;
        tile_of(p, t, pr, ct);
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort)) { ok = false; break; }
          uint8_t* st = smem + stage * STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&ctl->full[stage], 2 * A_BYTES);
          tma_load_2d_pair(st, &tm_a, mapa_shared(smem_u32(&ctl->full[stage]), 0), kb * BK,
                           pr * PAIR_ROWS + static_cast<int>(rank) * BM);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // every copy issued must land before the pair releases its shared memory: the last
      // min(issued, STAGES) slots hold the outstanding ones (counted on the leader)
      if (leader) {
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          mbar_drain(&ctl->full[stage], phase);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issuer (pair leader)
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int t = pair; t < p.n_tiles; t += n_pairs) {
        if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_cluster(&ctl->full[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: K-major rows of 128 B, +32 B per 16 K. B forward: K-major likewise; B
            // backward: MN-major, two 64-column groups of 64 K-rows x 128 B (LBO 8 KiB),
            // +2 KiB per 16 K-rows.
            const uint64_t bd = TRANS ? smem_desc_sw128(b + k * 2048, 64 * BK * 2, 1024)
                                      : smem_desc_sw128(b + k * 32, 16, 1024);
            umma_f16_pair(d, smem_desc_sw128(a + k * 32, 16, 1024), bd, idesc<TRANS>(),
                          kb != 0 || k != 0);
          }
          umma_commit_pair(&ctl->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&ctl->tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit_pair(&ctl->drain);
      mbar_drain(&ctl->drain, 0);
    }
  } else if (warp < FIRST_EPI_WARP) {  // converters
    const int c = threadIdx.x - 64;    // 0 .. 32 * CONV_WARPS - 1
    const int h = c & 1;               // which 16 of the row's 32 packed bytes (chunks 4h..4h+3)
    // forward: weight row n0 + (c >> 1), 64 weights of K-block kb. backward: weight row
    // kb * 64 + jr, the 64 columns n0 + jg * 64 .. +64 (one absmax block).
    const int jr = TRANS ? ((c >> 1) & 63) : (c >> 1);
    const int jg = TRANS ? (c >> 7) : 0;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = pair; t < p.n_tiles; t += n_pairs) {
      int pr, ct;
      tile_of(p, t, pr, ct);
      (void)pr;
      const int n0 = ct * BN + static_cast<int>(rank) * (BN / 2);
      bool ok = true;
      // the packed bytes and scale inputs of block kb are loaded from global memory (L2: the
      // pairs running at the same time read the same weight tile) two stages before they are
      // converted, so the loads overlap two stages' work
      const long long row_bytes = static_cast<long long>(p.w_blocks) * (BK / 2);
      auto fetch = [&](int kb, uint4& w, uint32_t& a8, float& s2, float& o2) {
        const int wrow = TRANS ? kb * BK + jr : n0 + jr;
        const int wblk = TRANS ? (n0 / BK + jg) : kb;
        if (kb >= p.k_blocks || wrow >= p.w_rows || wblk >= p.w_blocks) {
          w = make_uint4(0, 0, 0, 0);
          a8 = 0;
          s2 = 0.0f;
          o2 = 0.0f;
          return;
        }
        const long long li = static_cast<long long>(wrow) * p.w_blocks + wblk;
        const long long b2 = (p.absmax_row0 + li) / p.qblock2;
        w = __ldg(reinterpret_cast<const uint4*>(p.packed + wrow * row_bytes + wblk * (BK / 2) +
                                                 h * 16));
        a8 = __ldg(p.absmax8 + li);
        s2 = __ldg(p.absmax2 + b2);
        o2 = __ldg(p.offset2 + b2);
      };
      uint4 w_0, w_1;
      uint32_t a8_0, a8_1;
      float s2_0, s2_1, o2_0, o2_1;
      fetch(0, w_0, a8_0, s2_0, o2_0);
      fetch(1, w_1, a8_1, s2_1, o2_1);
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        const float scale = __fadd_rn(__fmul_rn(code_s[a8_0], s2_0), o2_0);
        const uint4 w = w_0;
        w_0 = w_1;
        a8_0 = a8_1;
        s2_0 = s2_1;
        o2_0 = o2_1;
        fetch(kb + 2, w_1, a8_1, s2_1, o2_1);
        // the pair's MMAs of this stage's previous round are done with its B tile
        if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort)) { ok = false; break; }
        uint8_t* btile = smem + stage * STAGE_BYTES + A_BYTES;
        // forward: row jr of a 128-row K-major tile; backward: K-row jr of column group jg
        uint8_t* dst = TRANS ? btile + jg * (64 * BK * 2) : btile;
        put_chunk(dst, jr, 4 * h + 0, expand8(w.x, scale, level_s));
        put_chunk(dst, jr, 4 * h + 1, expand8(w.y, scale, level_s));
        put_chunk(dst, jr, 4 * h + 2, expand8(w.z, scale, level_s));
        put_chunk(dst, jr, 4 * h + 3, expand8(w.w, scale, level_s));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->full[stage]), 0));
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  } else {  // epilogue: the last 8 warps of both CTAs; TMEM lane quarter = warp % 4
    const int q = warp & 3;
    const int g = (warp - FIRST_EPI_WARP) >> 2;
    const int bar_id = 1 + g;
    const int r_in_tile = q * 32 + lane;
    const bool elected = (warp - FIRST_EPI_WARP) % 4 == 0 && lane == 0;
    uint8_t* const bufs = staging + g * STAGING_PER_GROUP * 16384;
    int nb = 0, acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.n_tiles; t += n_pairs) {
      int pr, ct;
      tile_of(p, t, pr, ct);
      const bool landed = mbar_wait(&ctl->tfull[acc], acc_phase, abort);
      if (named_barrier_or(bar_id, EPI_THREADS, !landed)) break;
      tc_fence_after();
      const int row0 = pr * PAIR_ROWS + static_cast<int>(rank) * BM;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int h = 0; h < EPI_COLS / 64; ++h) {  // 64 output columns per staged store
        const int c0 = g * EPI_COLS + h * 64;    // tile column of the block
        const int col0 = ct * BN + c0;           // output column
        uint8_t* buf = bufs + nb * 16384;
        nb = (nb + 1) % STAGING_PER_GROUP;
        if (elected) bulk_wait_read<STAGING_PER_GROUP - 1>();
        named_barrier(bar_id, EPI_THREADS);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + c0 + half * 32, v);
          tmem_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            float y0 = __uint_as_float(v[j]), y1 = __uint_as_float(v[j + 1]);
            if (!TRANS && p.bias != nullptr) {
              const int col = col0 + half * 32 + j;
              if (col < p.n_out) y0 += __half2float(p.bias[col]);
              if (col + 1 < p.n_out) y1 += __half2float(p.bias[col + 1]);
            }
            packed[j / 2] = pack_half2(y0, y1);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            put_chunk(buf, r_in_tile, half * 4 + u,
                      make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2],
                                 packed[4 * u + 3]));
        }
        fence_proxy_async_smem();
        named_barrier(bar_id, EPI_THREADS);
        if (elected && col0 < p.n_out && row0 < p.n_rows) {
          tma_store_2d(&tm_y, buf, col0, row0);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (elected) bulk_wait_all();
  }
  tc_fence_before();
  cluster_sync();  // the peer's shared memory stays alive until the leader's MMAs are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// Shared-memory opt-in of both kernel variants, once per device (see head.cu's set_attrs).
std::mutex g_attr_mutex;
bool g_attrs_set[kMaxDevices] = {};

int set_attrs() {
  int dev = 0;
  int st = current_device(&dev);
  if (st != TALM_OK) return st;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (g_attrs_set[dev]) return TALM_OK;
  cudaError_t e = cudaFuncSetAttribute(nf4_gemm_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(nf4_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES);
  if (e != cudaSuccess) return set_error(TALM_ECUDA, "smem attribute: %s", cudaGetErrorString(e));
  g_attrs_set[dev] = true;
  return TALM_OK;
}

}  // namespace nf4g
}  // namespace talm

extern "C" {

int talm_nf4_linear(const uint16_t* a, int64_t ld_a, int64_t n_rows, const uint8_t* packed,
                    const uint8_t* absmax8, const float* code, const float* absmax2,
                    const float* offset2, const float* levels, int64_t absmax_row0,
                    int64_t w_rows, int64_t w_cols, int64_t qblock, int64_t qblock2,
                    int transpose, const uint16_t* bias, uint16_t* y, int64_t ld_y,
                    void* stream_) {
  using namespace talm;
  using namespace talm::nf4g;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (qblock != BK) return set_error(TALM_EINVAL, "the fused NF4 GEMM takes qblock 64 only");
  if (qblock2 < 1 || absmax_row0 < 0) return set_error(TALM_EINVAL, "bad second-level blocks");
  if (w_rows < 64 || w_rows % 64 != 0 || w_cols < 128 || w_cols % 128 != 0)
    return set_error(TALM_EINVAL, "weight rows must be a multiple of 64, columns of 128");
  if (n_rows < 0) return set_error(TALM_EINVAL, "negative row count");
  if (n_rows >= (int64_t{1} << 31) || w_rows >= (int64_t{1} << 24) ||
      w_cols >= (int64_t{1} << 24))
    return set_error(TALM_ERANGE, "sizes beyond the kernel's 32-bit tile indices");
  if (transpose && bias != nullptr)
    return set_error(TALM_EINVAL, "the input-gradient product takes no bias");
  const int64_t red = transpose ? w_rows : w_cols;   // reduction length
  const int64_t n_out = transpose ? w_cols : w_rows;  // output columns
  if (ld_a < red || ld_a % 8 != 0 || ld_y < n_out || ld_y % 8 != 0)
    return set_error(TALM_EINVAL, "row strides must cover the rows and be multiples of 8");
  if (n_rows == 0) return TALM_OK;
  if (!a || !packed || !absmax8 || !code || !absmax2 || !offset2 || !levels || !y)
    return set_error(TALM_EINVAL, "null pointer");
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(y) |
        reinterpret_cast<uintptr_t>(packed)) & 15) != 0)
    return set_error(TALM_EINVAL, "operands must be 16-byte aligned");
  if (!device_is_sm100()) return set_error(TALM_ENODEV, "the fused NF4 GEMM needs an sm_100 GPU");
  int st = set_attrs();
  if (st != TALM_OK) return st;
  const int sms = current_sm_count();
  if (sms <= 0) return set_error(TALM_ENODEV, "no CUDA device");

  CUtensorMap tm_a, tm_y;
  st = talm_make_tmap_2d_f16(&tm_a, a, red, n_rows, ld_a, BK, BM);
  if (st == TALM_OK) st = talm_make_tmap_2d_f16(&tm_y, y, n_out, n_rows, ld_y, 64, BM);
  if (st != TALM_OK) return st;

  Params p;
  p.n_rows = static_cast<int>(n_rows);
  p.n_out = static_cast<int>(n_out);
  p.k_blocks = static_cast<int>(red / BK);
  p.n_pair_rows = static_cast<int>((n_rows + PAIR_ROWS - 1) / PAIR_ROWS);
  p.n_col_tiles = static_cast<int>((n_out + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(p.n_pair_rows) * p.n_col_tiles;
  if (tiles >= (int64_t{1} << 31)) return set_error(TALM_ERANGE, "too many tiles");
  p.n_tiles = static_cast<int>(tiles);
  p.w_rows = static_cast<int>(w_rows);
  p.w_blocks = static_cast<int>(w_cols / BK);
  p.absmax_row0 = absmax_row0;
  p.qblock2 = static_cast<int>(qblock2);
  p.packed = packed;
  p.absmax8 = absmax8;
  p.absmax2 = absmax2;
  p.offset2 = offset2;
  p.code = code;
  p.levels = levels;
  p.bias = reinterpret_cast<const __half*>(bias);

  const int pairs = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles, sms / 2)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  LaunchTimer timer(TALM_KERNEL_NF4_GEMM, stream);
  const cudaError_t e =
      transpose ? cudaLaunchKernelEx(&cfg, nf4_gemm_kernel<true>, tm_a, tm_y, p)
                : cudaLaunchKernelEx(&cfg, nf4_gemm_kernel<false>, tm_a, tm_y, p);
  if (e != cudaSuccess)
    return set_error(TALM_ECUDA, "fused NF4 GEMM launch: %s", cudaGetErrorString(e));
  return TALM_OK;
}

}  // extern "C"
