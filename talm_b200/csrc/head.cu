// Fused LM head + cross-entropy, forward and backward, without materialised logits.
//
// The vocabulary (or this rank's shard of it) is walked in slices of `vocab_chunk` columns. Per
// slice three launches run back to back on the caller's stream:
//
//   1. head_logits_kernel  (tcgen05, TMA-fed, persistent): tiles of 128 token rows x 256 vocab
//      columns of z = fp16(h . W^T), K = hidden. The fp32 accumulator lives in TMEM (two
//      256-column buffers, so the epilogue of one tile overlaps the MMAs of the next). The
//      epilogue (4 warps, one token row per thread) rounds each logit to fp16 as the
//      reference's cuBLAS output does, and computes the tile's row statistics: max m_t, first
//      argmax, s_t = sum exp(z - m_t), t_t = sum exp(z - m_t) z, the target logit. For the
//      labelled rows it writes p = fp16(exp(z - m_t)) into the slice's probability buffer (the
//      only [rows, chunk] buffer of the head; it stays in L2 at the configured sizes).
//   2. head_combine_kernel: one warp per row merges the slice's tile statistics with the running
//      statistics of the earlier slices (log-sum-exp merge), and for labelled rows writes
//      per-tile factors exp(m_t - m_new) and the accumulator rescale alpha = exp(m_old - m_new)
//      (the online-softmax rescale of solution/fused_head.py:170-177).
//   3. head_accum_kernel (tcgen05, persistent): acc[128 rows, 256 hidden] = alpha * acc +
//      P' W_slice, K = slice columns. P arrives by TMA; four transform warps rescale it in shared
//      memory to p * exp(m_t - m_new) (so the GEMM operand equals fp16(exp(z - m_new)), the
//      reference's in-place softmax weights) before the MMA warp consumes the stage. W_slice is
//      read MN-major (hidden contiguous) straight from the weight rows.
//
// A last launch (head_finalize_kernel) turns the statistics into loss / entropy / correctness
// and the accumulator into dH = acc / s - fp16(W[target]) (fused_head.py:111-125, :160-169),
// writing rows in the caller's original order.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace talm {
namespace head {

constexpr int BM = 128;  // token rows per tile = TMEM lanes
constexpr int BN = 256;  // columns per tile (vocab in the logits GEMM, hidden in the acc GEMM)
constexpr int BK = 64;   // K per pipeline stage: one 128-byte swizzle row of fp16
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;     // double-buffered fp32 accumulator
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr float kLog2e = 1.4426950408889634f;
// Slack of the lazy reference: a row's probabilities and accumulator stay relative to REF while
// its running max is at most REF + kRefSlack, so p = exp(z - REF) <= e^8 (fits fp16).
constexpr float kRefSlack = 8.0f;

constexpr uint32_t kIdescLogits = idesc_f16_f32(BM, BN, false, false);  // A, B K-major
constexpr uint32_t kIdescAccum = idesc_f16_f32(BM, BN, false, true);    // B (W) MN-major

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

struct SharedCtl {
  uint64_t full[STAGES];
  uint64_t ready[STAGES];  // accum kernel: stage transformed and ready for the MMA
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;          // MMA issuer: every UMMA issued has completed
  uint64_t ring_full[4];   // tile-id ring (dynamic scheduler): id published
  uint64_t ring_empty[4];  // every consumer role has read the id
  int ring_id[4];
  uint32_t tmem_base;
  int abort;
};

// Dynamic tile scheduler. The TMA thread claims tiles from a global counter (one per launch,
// zeroed by the host) and publishes each id through a 4-slot ring in shared memory; the MMA
// thread and the epilogue / transform warps read the same sequence. CTAs that start late (the
// other kernel of the pipeline still holds their SM) simply claim fewer tiles.
__device__ __forceinline__ int ring_publish(SharedCtl* ctl, int i, int* counter, int n_tiles,
                                            volatile int* abort) {
  const int slot = i & 3;
  if (!mbar_wait(&ctl->ring_empty[slot], ((i >> 2) & 1) ^ 1, abort)) return -1;
  int tile = atomicAdd(counter, 1);
  if (tile >= n_tiles) tile = -1;
  ctl->ring_id[slot] = tile;
  mbar_arrive(&ctl->ring_full[slot]);
  return tile;
}

// One thread's read of ring entry i (then the caller releases the slot with ring_release).
__device__ __forceinline__ int ring_take(SharedCtl* ctl, int i, volatile int* abort) {
  const int slot = i & 3;
  if (!mbar_wait(&ctl->ring_full[slot], (i >> 2) & 1, abort)) return -1;
  return *reinterpret_cast<volatile int*>(&ctl->ring_id[slot]);
}

// A warp's read of ring entry i: every lane gets the id (or -1 when done / aborting), lane 0
// releases the slot.
__device__ __forceinline__ int ring_take_warp(SharedCtl* ctl, int i, volatile int* abort,
                                              int lane) {
  const int slot = i & 3;
  if (!__all_sync(0xffffffffu, mbar_wait(&ctl->ring_full[slot], (i >> 2) & 1, abort))) return -1;
  const int tile = *reinterpret_cast<volatile int*>(&ctl->ring_id[slot]);
  __syncwarp();
  if (lane == 0) mbar_arrive(&ctl->ring_empty[slot]);
  return tile;
}

__device__ __forceinline__ void init_ring(SharedCtl* ctl, int consumers) {
  for (int r = 0; r < 4; ++r) {
    mbar_init(&ctl->ring_full[r], 1);
    mbar_init(&ctl->ring_empty[r], consumers);
  }
}

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// On the way out of the producer: every TMA copy issued must have landed before the CTA
// releases its shared memory. (stage, phase) is the next slot the producer would have used;
// the last min(issued, STAGES) slots before it hold the outstanding copies. On the normal path
// they have all been consumed and each wait returns at once.
__device__ __forceinline__ void drain_copies(SharedCtl* ctl, int stage, uint32_t phase,
                                             int issued) {
  for (int i = 0; i < STAGES && i < issued; ++i) {
    if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
    mbar_drain(&ctl->full[stage], phase);
  }
}

// On the way out of the MMA issuer: wait until every UMMA it issued has completed, so that no
// MMA is still writing TMEM when it is released.
__device__ __forceinline__ void drain_mmas(SharedCtl* ctl) {
  umma_commit(&ctl->drain);
  mbar_drain(&ctl->drain, 0);
}

// ------------------------------------------------------------------------------------------
// 1. logits GEMM + tile statistics
// ------------------------------------------------------------------------------------------
struct LogitsParams {
  int n_tokens;
  int n_grad;
  int k_blocks;       // ceil(hidden / BK)
  int slice_row0;     // first weight row (of this call's range) of the slice
  int cols;           // valid columns of the slice
  int n_col_tiles;    // ceil(cols / BN)
  int n_row_tiles;    // ceil(n_tokens / BM)
  long long col_base; // global column id of slice column 0
  int has_ref;        // 0 on the first slice: no reference yet
  int* tile_counter;  // dynamic scheduler counter of this launch (zeroed by the host)
  const long long* targets;
  float4* partial;    // [n_tokens][n_col_tiles]: m_t, s_t, t_t, first argmax (int bits)
  __half* probs;      // [n_grad][ldp]
  long long ldp;
  float* stats;       // [n_tokens][TALM_HEAD_STATS]
};

__global__ void __launch_bounds__(192, 1)
    head_logits_kernel(const __grid_constant__ CUtensorMap tm_hidden,
                       const __grid_constant__ CUtensorMap tm_weight, LogitsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(&ctl->drain, 1);
    init_ring(ctl, 1 + 4);  // MMA thread + 4 epilogue warps
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_hidden);
    prefetch_tmap(&tm_weight);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;
  const int n_tiles = p.n_row_tiles * p.n_col_tiles;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int i = 0;; ++i) {
        const int tile = ring_publish(ctl, i, p.tile_counter, n_tiles, abort);
        if (tile < 0) break;
        const int rt = tile % p.n_row_tiles, ct = tile / p.n_row_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort)) break;
          uint8_t* a = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[stage], STAGE_BYTES);
          tma_load_2d(a, &tm_hidden, &ctl->full[stage], kb * BK, rt * BM);
          tma_load_2d(a + A_BYTES, &tm_weight, &ctl->full[stage], kb * BK,
                      p.slice_row0 + ct * BN);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      drain_copies(ctl, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int i = 0;; ++i) {
        const int tile = ring_take(ctl, i, abort);
        if (tile < 0) break;
        mbar_arrive(&ctl->ring_empty[i & 3]);
        if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl->full[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16(d, smem_desc_sw128(a + k * 32, 16, 1024), smem_desc_sw128(b + k * 32, 16, 1024),
                     kIdescLogits, (kb | k) != 0);
          }
          umma_commit(&ctl->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&ctl->tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      drain_mmas(ctl);
    }
  } else {  // epilogue: warps 2..5, TMEM lane quarter = warp % 4
    const int q = warp & 3;
    const int r_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      const int tile = ring_take_warp(ctl, i, abort, lane);
      if (tile < 0) break;
      const int rt = tile % p.n_row_tiles, ct = tile / p.n_row_tiles;
      // warp-uniform decision (each lane's wait is bounded, so every lane reaches the vote)
      if (!__all_sync(0xffffffffu, mbar_wait(&ctl->tfull[acc], acc_phase, abort))) break;
      tc_fence_after();
      const int row = rt * BM + r_in_tile;
      const bool valid_row = row < p.n_tokens;
      const long long tgt = valid_row ? p.targets[row] : -1;
      const long long tile_col0 = p.col_base + static_cast<long long>(ct) * BN;
      const long long tcol_ll = tgt - tile_col0;
      const int tcol = (tgt >= 0 && tcol_ll >= 0 && tcol_ll < BN) ? static_cast<int>(tcol_ll) : -1;
      const int ncols = min(BN, p.cols - ct * BN);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;

      // pass 1: max, first argmax, target logit
      float mx = -INFINITY;
      int arg = 0;
      float zt = 0.0f;
      uint32_t r[32];
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = c * 32 + j;
          const float z = round_f16(__uint_as_float(r[j]));
          if (col < ncols && z > mx) { mx = z; arg = col; }
          if (col == tcol) zt = z;
        }
      }
      // pass 2: sums and probabilities relative to the row's reference when the tile max stays
      // within its slack (the common case), else relative to the tile max; the combine kernel
      // recomputes the same choice from (mx, REF)
      const float ref = (p.has_ref && valid_row)
                            ? p.stats[static_cast<long long>(row) * TALM_HEAD_STATS + TALM_STAT_REF]
                            : 0.0f;
      const float base = (p.has_ref && mx <= ref + kRefSlack) ? ref : mx;
      float s = 0.0f, t = 0.0f;
      const bool write_p = row < p.n_grad;
      __half* prow = p.probs + static_cast<long long>(row) * p.ldp + static_cast<long long>(ct) * BN;
      const float mscaled = base * kLog2e;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_wait_ld();
        uint32_t packed[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const int col = c * 32 + j;
          const float z0 = round_f16(__uint_as_float(r[j]));
          const float z1 = round_f16(__uint_as_float(r[j + 1]));
          const float e0 = col < ncols ? ex2(fmaf(z0, kLog2e, -mscaled)) : 0.0f;
          const float e1 = col + 1 < ncols ? ex2(fmaf(z1, kLog2e, -mscaled)) : 0.0f;
          s += e0;
          s += e1;
          if (col < ncols) t = fmaf(e0, z0, t);
          if (col + 1 < ncols) t = fmaf(e1, z1, t);
          packed[j / 2] = pack_half2(e0, e1);
        }
        if (write_p) {
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_v4(prow + c * 32 + v * 8, packed[4 * v], packed[4 * v + 1], packed[4 * v + 2],
                  packed[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
      if (valid_row) {
        p.partial[static_cast<long long>(row) * p.n_col_tiles + ct] =
            make_float4(mx, s, t, __int_as_float(static_cast<int>(tile_col0 + arg)));
        if (tcol >= 0 && tcol < ncols) {
          float* st = p.stats + static_cast<long long>(row) * TALM_HEAD_STATS;
          st[TALM_STAT_ZT] = zt;
          st[TALM_STAT_HIT] = 1.0f;
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------------------------------
// 2. per-slice combine of tile statistics with the running statistics
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void better_arg(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(256) head_combine_kernel(const float4* __restrict__ partial,
                                                           int n_col_tiles, int n_tokens,
                                                           int n_grad, int first,
                                                           float* __restrict__ stats,
                                                           float* __restrict__ tile_scale,
                                                           float* __restrict__ alpha,
                                                           int* __restrict__ block_jump) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= n_tokens) return;
  const float4* pr = partial + static_cast<long long>(row) * n_col_tiles;
  float* st = stats + static_cast<long long>(row) * TALM_HEAD_STATS;
  // every lane reads the running statistics before lane 0 overwrites them
  const float ref = first ? 0.0f : st[TALM_STAT_REF];
  const float m_old = first ? -INFINITY : st[TALM_STAT_M];
  const float s_old = first ? 0.0f : st[TALM_STAT_S];
  const float t_old = first ? 0.0f : st[TALM_STAT_T];
  const float best_old = first ? -INFINITY : st[TALM_STAT_BEST];
  __syncwarp();
  // the slice's max and first argmax
  float M = -INFINITY, bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = lane; j < n_col_tiles; j += 32) {
    const float4 v = pr[j];
    M = fmaxf(M, v.x);
    better_arg(bv, bi, v.x, __float_as_int(v.w));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    better_arg(bv, bi, v2, i2);
  }
  const float m_new = fmaxf(m_old, M);
  // the reference moves (a "jump") on the first slice and when the max outgrows its slack
  const bool jump = first || m_new > ref + kRefSlack;
  const float ref_new = jump ? m_new : ref;
  // tile sums were taken relative to base_j = (has ref and m_j <= ref + slack) ? ref : m_j
  float S = 0.0f, T = 0.0f;
  float* sc = tile_scale + static_cast<long long>(row) * n_col_tiles;
  for (int j = lane; j < n_col_tiles; j += 32) {
    const float4 v = pr[j];
    const float base = (!first && v.x <= ref + kRefSlack) ? ref : v.x;
    const float w = ex2((base - ref_new) * kLog2e);
    S = fmaf(v.y, w, S);
    T = fmaf(v.z, w, T);
    if (row < n_grad) sc[j] = w;  // the accumulator GEMM's factor for this tile (1 if stable)
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    S += __shfl_xor_sync(0xffffffffu, S, o);
    T += __shfl_xor_sync(0xffffffffu, T, o);
  }
  const float a = first ? 0.0f : ex2((ref - ref_new) * kLog2e);
  if (lane == 0) {
    st[TALM_STAT_REF] = ref_new;
    st[TALM_STAT_M] = m_new;
    st[TALM_STAT_S] = s_old * a + S;
    st[TALM_STAT_T] = t_old * a + T;
    if (first || bv > best_old) {  // earlier slices win ties: lower columns
      st[TALM_STAT_BEST] = bv;
      st[TALM_STAT_IDX] = __int_as_float(bi);
    }
    if (row < n_grad) {
      alpha[row] = a;
      if (jump) atomicOr(block_jump + row / BM, 1);
    }
  }
}

// ------------------------------------------------------------------------------------------
// 3. accumulator GEMM: acc = alpha * acc + P' W_slice
// ------------------------------------------------------------------------------------------
struct AccumParams {
  int n_grad;
  int hidden;
  int k_blocks;      // slice columns / BK (padded slice: a multiple of BN / BK)
  int slice_row0;    // first weight row of the slice
  int n_col_tiles;   // tiles of the slice (for the scale table)
  int n_row_tiles;   // ceil(n_grad / BM)
  int n_h_tiles;     // ceil(hidden / BN)
  int first;
  const float* tile_scale;  // [n_grad][n_col_tiles]
  const float* alpha;       // [n_grad]
  const int* block_jump;    // [n_row_tiles]: some row of the block moved its reference
  int* tile_counter;        // dynamic scheduler counter of this launch (zeroed by the host)
  float* acc;               // [n_grad][hidden]
};

__global__ void __launch_bounds__(320, 1)
    head_accum_kernel(const __grid_constant__ CUtensorMap tm_probs,
                      const __grid_constant__ CUtensorMap tm_weight_mn, AccumParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->ready[s], 4);  // one arrive per transform warp
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(&ctl->drain, 1);
    init_ring(ctl, 1 + 4 + 4);  // MMA thread + 4 epilogue warps + 4 transform warps
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_probs);
    prefetch_tmap(&tm_weight_mn);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;
  const int n_tiles = p.n_row_tiles * p.n_h_tiles;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int i = 0;; ++i) {
        const int tile = ring_publish(ctl, i, p.tile_counter, n_tiles, abort);
        if (tile < 0) break;
        const int ht = tile % p.n_h_tiles, rt = tile / p.n_h_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort)) break;
          uint8_t* a = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[stage], STAGE_BYTES);
          tma_load_2d(a, &tm_probs, &ctl->full[stage], kb * BK, rt * BM);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(a + A_BYTES + j * (64 * BK * 2), &tm_weight_mn, &ctl->full[stage],
                        ht * BN + j * 64, p.slice_row0 + kb * BK);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      drain_copies(ctl, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t ready_phase = 0;  // bit s: parity of the next phase of ready[s]
      for (int i = 0;; ++i) {
        const int tile = ring_take(ctl, i, abort);
        if (tile < 0) break;
        mbar_arrive(&ctl->ring_empty[i & 3]);
        if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        // tiles whose rows all kept their reference need no rescaling: the MMA consumes the
        // TMA'd stage directly; otherwise it waits for the transform warps
        const bool transformed = __ldg(p.block_jump + tile / p.n_h_tiles) != 0;
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          bool landed;
          if (transformed) {
            landed = mbar_wait(&ctl->ready[stage], (ready_phase >> stage) & 1u, abort);
            ready_phase ^= 1u << stage;
          } else {
            landed = mbar_wait(&ctl->full[stage], phase, abort);
          }
          if (!landed) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: K-major rows of 128 B, +32 B per 16 K. B: MN-major, 64-wide hidden groups of
            // BK rows x 128 B (LBO = 8 KiB), 16 K-rows = +2 KiB.
            umma_f16(d, smem_desc_sw128(a + k * 32, 16, 1024),
                     smem_desc_sw128(b + k * 2048, 64 * BK * 2, 1024), kIdescAccum,
                     (kb | k) != 0);
          }
          umma_commit(&ctl->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&ctl->tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      drain_mmas(ctl);
    }
  } else if (warp >= 6) {  // transform: p -> p * exp(m_t - m_new), one row per thread
    const int r_in_tile = (warp - 6) * 32 + lane;
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0;; ++i) {
      const int tile = ring_take_warp(ctl, i, abort, lane);
      if (tile < 0) break;
      const int rt = tile / p.n_h_tiles;
      if (__ldg(p.block_jump + rt) == 0) {  // the MMA consumes these stages untouched
        const int adv = p.k_blocks % STAGES;
        phase ^= static_cast<uint32_t>((p.k_blocks / STAGES) & 1);
        if (stage + adv >= STAGES) phase ^= 1;
        stage = (stage + adv) % STAGES;
        continue;
      }
      const int row = min(rt * BM + r_in_tile, p.n_grad - 1);
      const float* sc_row = p.tile_scale + static_cast<long long>(row) * p.n_col_tiles;
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (!__all_sync(0xffffffffu, mbar_wait(&ctl->full[stage], phase, abort))) {
          ok = false;
          break;
        }
        const float sc = __ldg(sc_row + (kb * BK) / BN);
        uint4* line = reinterpret_cast<uint4*>(smem + stage * STAGE_BYTES + r_in_tile * 128);
        // Visit the row's 16-byte chunks in logical order: logical chunk c sits at c ^ (row & 7)
        // (128-byte swizzle), so the 32 lanes of a warp spread over all 8 chunk positions and
        // each 512-byte warp access takes the minimum 4 shared-memory wavefronts.
#pragma unroll
        for (int c0 = 0; c0 < 8; ++c0) {
          const int c = c0 ^ (r_in_tile & 7);
          uint4 v = line[c];
          uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            __half2 h = *reinterpret_cast<__half2*>(&w[i]);
            const float2 f = __half22float2(h);
            w[i] = pack_half2(f.x * sc, f.y * sc);
          }
          line[c] = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->ready[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  } else {  // epilogue: warps 2..5
    const int q = warp & 3;
    const int r_in_tile = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      const int tile = ring_take_warp(ctl, i, abort, lane);
      if (tile < 0) break;
      const int ht = tile % p.n_h_tiles, rt = tile / p.n_h_tiles;
      // warp-uniform decision (each lane's wait is bounded, so every lane reaches the vote)
      if (!__all_sync(0xffffffffu, mbar_wait(&ctl->tfull[acc], acc_phase, abort))) break;
      tc_fence_after();
      const int row = rt * BM + r_in_tile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      const float al = (row < p.n_grad && !p.first) ? p.alpha[row] : 0.0f;
      float* arow = p.acc + static_cast<long long>(row) * p.hidden + ht * BN;
      uint32_t r[32];
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld_32x32b_x32(taddr + c * 32, r);
        tmem_wait_ld();
        const int h0 = ht * BN + c * 32;
        if (row < p.n_grad) {
          if (h0 + 32 <= p.hidden) {
            float4* dst = reinterpret_cast<float4*>(arow + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 o;
              if (p.first) {
                o = make_float4(0.f, 0.f, 0.f, 0.f);
              } else {
                o = dst[v];
              }
              o.x = fmaf(o.x, al, __uint_as_float(r[4 * v + 0]));
              o.y = fmaf(o.y, al, __uint_as_float(r[4 * v + 1]));
              o.z = fmaf(o.z, al, __uint_as_float(r[4 * v + 2]));
              o.w = fmaf(o.w, al, __uint_as_float(r[4 * v + 3]));
              dst[v] = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (h0 + j < p.hidden) {
                float* dst = arow + c * 32 + j;
                const float old = p.first ? 0.0f : *dst;
                *dst = fmaf(old, al, __uint_as_float(r[j]));
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------------------------------
// 4. finalize: per-row outputs and the hidden gradient
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) head_finalize_kernel(
    const float* __restrict__ stats, const long long* __restrict__ targets, int n_tokens,
    int n_grad, const float* __restrict__ acc, const float* __restrict__ acc_scale,
    const __half* __restrict__ weight, long long ld_weight, long long col0, long long vcols,
    int hidden, const long long* __restrict__ grad_rows, float* __restrict__ token_loss,
    float* __restrict__ token_entropy, int* __restrict__ correct, void* __restrict__ grad,
    int grad_f32) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= n_tokens) return;
  const float* st = stats + static_cast<long long>(row) * TALM_HEAD_STATS;
  const long long tgt = targets[row];
  const bool labelled = tgt >= 0;
  const long long out = grad_rows ? grad_rows[row] : row;
  const float ref = st[TALM_STAT_REF], s = st[TALM_STAT_S], t = st[TALM_STAT_T];
  if (lane == 0) {
    const float ls = logf(s);
    const float lse = ref + ls;
    if (token_entropy) token_entropy[out] = lse - t / s;
    if (token_loss) token_loss[out] = labelled ? ls + (ref - st[TALM_STAT_ZT]) : 0.0f;
    if (correct)
      correct[out] = (labelled && static_cast<long long>(__float_as_int(st[TALM_STAT_IDX])) == tgt)
                         ? 1 : 0;
  }
  if (grad == nullptr) return;
  const bool live = labelled && row < n_grad && acc != nullptr;
  const bool own = live && tgt >= col0 && tgt < col0 + vcols;
  const float* arow = acc + static_cast<long long>(row) * hidden;
  const __half* wrow = weight + (own ? (tgt - col0) * ld_weight : 0);
  const float scale = acc_scale ? acc_scale[row] : 0.0f;
  for (int h = lane; h < hidden; h += 32) {
    float g = 0.0f;
    if (live) {
      const float a = arow[h];
      g = acc_scale ? a * scale : a / s;
      if (own) g -= __half2float(wrow[h]);
    }
    if (grad_f32) {
      reinterpret_cast<float*>(grad)[out * hidden + h] = g;
    } else {
      reinterpret_cast<__half*>(grad)[out * hidden + h] = __float2half_rn(g);
    }
  }
}

// ------------------------------------------------------------------------------------------
// vocabulary-parallel merge of shard statistics
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) head_merge_shards_kernel(const float* __restrict__ gathered,
                                                                int n_shards, int n_tokens,
                                                                int rank, int n_grad,
                                                                float* __restrict__ out,
                                                                float* __restrict__ acc_scale) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n_tokens) return;
  float M = -INFINITY, R = -INFINITY, bv = -INFINITY, zt = 0.0f, hit = 0.0f;
  int bi = 0x7fffffff;
  for (int r = 0; r < n_shards; ++r) {
    const float* st = gathered + (static_cast<long long>(r) * n_tokens + row) * TALM_HEAD_STATS;
    M = fmaxf(M, st[TALM_STAT_M]);
    R = fmaxf(R, st[TALM_STAT_REF]);
    better_arg(bv, bi, st[TALM_STAT_BEST], __float_as_int(st[TALM_STAT_IDX]));
    if (st[TALM_STAT_HIT] != 0.0f) { zt = st[TALM_STAT_ZT]; hit = 1.0f; }
  }
  float S = 0.0f, T = 0.0f, mine = 0.0f;
  for (int r = 0; r < n_shards; ++r) {
    const float* st = gathered + (static_cast<long long>(r) * n_tokens + row) * TALM_HEAD_STATS;
    const float w = ex2((st[TALM_STAT_REF] - R) * kLog2e);
    S = fmaf(st[TALM_STAT_S], w, S);
    T = fmaf(st[TALM_STAT_T], w, T);
    if (r == rank) mine = w;
  }
  float* o = out + static_cast<long long>(row) * TALM_HEAD_STATS;
  o[TALM_STAT_M] = M;
  o[TALM_STAT_S] = S;
  o[TALM_STAT_T] = T;
  o[TALM_STAT_ZT] = zt;
  o[TALM_STAT_BEST] = bv;
  o[TALM_STAT_IDX] = __int_as_float(bi);
  o[TALM_STAT_HIT] = hit;
  o[TALM_STAT_REF] = R;
  if (acc_scale != nullptr && row < n_grad) acc_scale[row] = mine / S;
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
// Slice buffers come in pairs: the accumulator GEMM of slice k (side stream) reads pair k % 2
// while the logits GEMM and the combine of slice k + 1 (caller's stream) write the other one.
struct Workspace {
  __half* probs[2];      // [n_grad][chunk] each
  float4* partial;       // [n_tokens][chunk / BN]
  float* tile_scale[2];  // [n_grad][chunk / BN] each
  float* alpha[2];       // [n_grad] each
  int* block_jump;       // [n_slices][flag_stride]
  int* counters;         // [n_slices][2]: dynamic scheduler counters (logits, accum)
  size_t bytes;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline int64_t chunk_cols(int64_t vocab_cols, int64_t vocab_chunk) {
  int64_t c = vocab_chunk < 1 ? 1 : vocab_chunk;
  if (c > vocab_cols) c = vocab_cols;
  c = (c + BN - 1) / BN * BN;  // whole tiles
  return c < BN ? BN : c;
}

Workspace layout(int64_t n_tokens, int64_t n_grad, int64_t vocab_cols, int64_t vocab_chunk,
                 uint8_t* base) {
  const int64_t chunk = chunk_cols(vocab_cols, vocab_chunk);
  const int64_t tiles = chunk / BN;
  const int64_t n_slices = (vocab_cols + chunk - 1) / chunk;
  const int n_buf = n_slices > 1 ? 2 : 1;
  Workspace w;
  size_t off = 0;
  for (int b = 0; b < 2; ++b) {
    w.probs[b] = reinterpret_cast<__half*>(base + off);
    if (b < n_buf) off = align_up(off + static_cast<size_t>(n_grad) * chunk * 2, 256);
  }
  w.partial = reinterpret_cast<float4*>(base + off);
  off = align_up(off + static_cast<size_t>(n_tokens) * tiles * 16, 256);
  for (int b = 0; b < 2; ++b) {
    w.tile_scale[b] = reinterpret_cast<float*>(base + off);
    if (b < n_buf) off = align_up(off + static_cast<size_t>(n_grad) * tiles * 4, 256);
  }
  for (int b = 0; b < 2; ++b) {
    w.alpha[b] = reinterpret_cast<float*>(base + off);
    if (b < n_buf) off = align_up(off + static_cast<size_t>(n_grad) * 4, 256);
  }
  w.block_jump = reinterpret_cast<int*>(base + off);
  off = align_up(off + static_cast<size_t>(n_slices) * ((n_grad + BM - 1) / BM + 1) * 4, 256);
  w.counters = reinterpret_cast<int*>(base + off);
  off = align_up(off + static_cast<size_t>(n_slices) * 2 * 4, 256);
  w.bytes = off + 256;  // slack for base alignment
  return w;
}

// The accumulator GEMM runs on a library-owned stream per device, forked from and joined back
// into the caller's stream with events, so that it overlaps the next slice's logits GEMM. The
// stream and its events are created once per device; calls from several host threads serialise
// their enqueueing on a mutex (the GPU work of the calls then orders on the side stream).
struct SidePipe {
  cudaStream_t stream = nullptr;
  cudaEvent_t combined[2] = {nullptr, nullptr};  // slice k's statistics ready (caller's stream)
  cudaEvent_t drained[2] = {nullptr, nullptr};   // slice k's accumulator GEMM done (side stream)
  bool ready = false;
};
constexpr int kMaxPipeDevices = 64;
SidePipe g_pipes[kMaxPipeDevices];
std::mutex g_pipe_mutex;

int side_pipe(SidePipe** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxPipeDevices)
    return set_error(TALM_ENODEV, "no usable current device");
  SidePipe& p = g_pipes[dev];
  if (!p.ready) {
    cudaError_t e = cudaStreamCreateWithFlags(&p.stream, cudaStreamNonBlocking);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) {
      e = cudaEventCreateWithFlags(&p.combined[i], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.drained[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess)
      return set_error(TALM_ECUDA, "side stream set-up: %s", cudaGetErrorString(e));
    p.ready = true;
  }
  *out = &p;
  return TALM_OK;
}

bool g_attrs_set = false;

int set_attrs() {
  if (g_attrs_set) return TALM_OK;
  cudaError_t e = cudaFuncSetAttribute(head_logits_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(head_accum_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES);
  if (e != cudaSuccess) return set_error(TALM_ECUDA, "smem attribute: %s", cudaGetErrorString(e));
  g_attrs_set = true;
  return TALM_OK;
}

}  // namespace head
}  // namespace talm

extern "C" {

int talm_head_workspace_size(int64_t n_tokens, int64_t n_grad, int64_t hidden,
                             int64_t vocab_cols, int64_t vocab_chunk, size_t* bytes) {
  using namespace talm;
  if (bytes == nullptr) return set_error(TALM_EINVAL, "bytes is NULL");
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens || hidden < 1 || vocab_cols < 1)
    return set_error(TALM_EINVAL, "bad sizes");
  *bytes = head::layout(n_tokens, n_grad, vocab_cols, vocab_chunk, nullptr).bytes;
  return TALM_OK;
}

int talm_head_shard(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                    int64_t ld_weight, const int64_t* targets, int64_t n_tokens, int64_t n_grad,
                    int64_t hidden_size, int64_t vocab_cols, int64_t vocab_col0,
                    int64_t vocab_chunk, float* stats, float* acc, void* workspace,
                    size_t ws_bytes, void* stream_) {
  using namespace talm;
  using namespace talm::head;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  if (hidden_size < 8 || hidden_size % 8 != 0 || ld_hidden % 8 != 0 || ld_weight % 8 != 0 ||
      ld_hidden < hidden_size || ld_weight < hidden_size)
    return set_error(TALM_EINVAL, "hidden size and row strides must be multiples of 8 elements");
  if (vocab_cols < 1 || vocab_col0 < 0) return set_error(TALM_EINVAL, "empty vocabulary range");
  if (n_tokens >= (int64_t{1} << 30) || vocab_cols >= (int64_t{1} << 31) ||
      hidden_size >= (int64_t{1} << 20))
    return set_error(TALM_ERANGE, "sizes beyond the kernels' 32-bit tile indices");
  if (n_tokens == 0) return TALM_OK;
  if (!hidden || !weight || !targets || !stats || (n_grad > 0 && !acc) || !workspace)
    return set_error(TALM_EINVAL, "null pointer");
  if (!device_is_sm100()) return set_error(TALM_ENODEV, "the head kernels need an sm_100 GPU");
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  Workspace ws = layout(n_tokens, n_grad, vocab_cols, vocab_chunk, base);
  if (ws.bytes > ws_bytes)
    return set_error(TALM_EINVAL, "workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
  int st = set_attrs();
  if (st != TALM_OK) return st;
  const int64_t chunk = chunk_cols(vocab_cols, vocab_chunk);
  const int sms = current_sm_count();

  CUtensorMap tm_hidden, tm_weight, tm_weight_mn;
  st = talm_make_tmap_2d_f16(&tm_hidden, hidden, hidden_size, n_tokens, ld_hidden, BK, BM);
  if (st == TALM_OK)
    st = talm_make_tmap_2d_f16(&tm_weight, weight, hidden_size, vocab_cols, ld_weight, BK, BN);
  if (st == TALM_OK && n_grad > 0)
    st = talm_make_tmap_2d_f16(&tm_weight_mn, weight, hidden_size, vocab_cols, ld_weight, 64, BK);
  if (st != TALM_OK) return st;

  const int64_t n_slices = (vocab_cols + chunk - 1) / chunk;
  const int64_t flag_stride = (n_grad + BM - 1) / BM + 1;
  std::lock_guard<std::mutex> lock(g_pipe_mutex);
  // The accumulator GEMM goes to the side stream (overlapping the next slice's logits GEMM)
  // only when it has fewer tiles than the GPU has SMs; a GEMM that fills the GPU on its own
  // gains nothing from sharing it and runs in order on the caller's stream.
  const int64_t grad_tiles = ((n_grad + BM - 1) / BM) * ((hidden_size + BN - 1) / BN);
  SidePipe* pipe = nullptr;
  if (n_grad > 0 && n_slices > 1 && grad_tiles < sms && (st = side_pipe(&pipe)) != TALM_OK)
    return st;

  if (cudaMemsetAsync(stats, 0, sizeof(float) * TALM_HEAD_STATS * n_tokens, stream) != cudaSuccess)
    return check_launch("stats memset");
  // flags and scheduler counters are contiguous in the workspace: one memset for both
  const size_t zero_bytes = reinterpret_cast<uint8_t*>(ws.counters + n_slices * 2) -
                            reinterpret_cast<uint8_t*>(ws.block_jump);
  if (cudaMemsetAsync(ws.block_jump, 0, zero_bytes, stream) != cudaSuccess)
    return check_launch("flag memset");

  const int k_blocks = static_cast<int>((hidden_size + BK - 1) / BK);
  const int n_row_tiles = static_cast<int>((n_tokens + BM - 1) / BM);
  for (int64_t k = 0; k < n_slices; ++k) {
    const int64_t s0 = k * chunk;
    const int buf = static_cast<int>(k & 1);
    const int cols = static_cast<int>(vocab_cols - s0 < chunk ? vocab_cols - s0 : chunk);
    const int n_col_tiles = (cols + BN - 1) / BN;
    int* slice_jump = ws.block_jump + k * flag_stride;
    // the pair of buffers this slice writes is free once slice k - 2's accumulator GEMM is done
    if (pipe && k >= 2 && cudaStreamWaitEvent(stream, pipe->drained[buf], 0) != cudaSuccess)
      return check_launch("wait for slice buffers");
    LogitsParams lp;
    lp.n_tokens = static_cast<int>(n_tokens);
    lp.n_grad = static_cast<int>(n_grad);
    lp.k_blocks = k_blocks;
    lp.slice_row0 = static_cast<int>(s0);
    lp.cols = cols;
    lp.n_col_tiles = n_col_tiles;
    lp.n_row_tiles = n_row_tiles;
    lp.col_base = vocab_col0 + s0;
    lp.has_ref = k != 0;
    lp.tile_counter = ws.counters + 2 * k;
    lp.targets = reinterpret_cast<const long long*>(targets);
    lp.partial = ws.partial;
    lp.probs = ws.probs[buf];
    lp.ldp = chunk;
    lp.stats = stats;
    const int tiles = n_row_tiles * n_col_tiles;
    {
      LaunchTimer timer(TALM_KERNEL_HEAD_LOGITS, stream);
      head_logits_kernel<<<tiles < sms ? tiles : sms, 192, SMEM_BYTES, stream>>>(
          tm_hidden, tm_weight, lp);
    }
    if ((st = check_launch("head logits kernel")) != TALM_OK) return st;
    {
      LaunchTimer timer(TALM_KERNEL_HEAD_COMBINE, stream);
      head_combine_kernel<<<static_cast<int>((n_tokens + 7) / 8), 256, 0, stream>>>(
          ws.partial, n_col_tiles, static_cast<int>(n_tokens), static_cast<int>(n_grad), k == 0,
          stats, ws.tile_scale[buf], ws.alpha[buf], slice_jump);
    }
    if ((st = check_launch("head combine kernel")) != TALM_OK) return st;

    if (n_grad > 0) {
      cudaStream_t acc_stream = pipe ? pipe->stream : stream;
      if (pipe && (cudaEventRecord(pipe->combined[buf], stream) != cudaSuccess ||
                   cudaStreamWaitEvent(pipe->stream, pipe->combined[buf], 0) != cudaSuccess))
        return check_launch("fork to the side stream");
      CUtensorMap tm_probs;
      if ((st = talm_make_tmap_2d_f16(&tm_probs, ws.probs[buf], chunk, n_grad, chunk, BK, BM)) !=
          TALM_OK)
        return st;
      AccumParams ap;
      ap.n_grad = static_cast<int>(n_grad);
      ap.hidden = static_cast<int>(hidden_size);
      ap.k_blocks = n_col_tiles * (BN / BK);
      ap.slice_row0 = static_cast<int>(s0);
      ap.n_col_tiles = n_col_tiles;
      ap.n_row_tiles = static_cast<int>((n_grad + BM - 1) / BM);
      ap.n_h_tiles = static_cast<int>((hidden_size + BN - 1) / BN);
      ap.first = k == 0;
      ap.tile_scale = ws.tile_scale[buf];
      ap.alpha = ws.alpha[buf];
      ap.block_jump = slice_jump;
      ap.tile_counter = ws.counters + 2 * k + 1;
      ap.acc = acc;
      const int atiles = ap.n_row_tiles * ap.n_h_tiles;
      {
        LaunchTimer timer(TALM_KERNEL_HEAD_ACCUM, acc_stream);
        head_accum_kernel<<<atiles < sms ? atiles : sms, 320, SMEM_BYTES, acc_stream>>>(
            tm_probs, tm_weight_mn, ap);
      }
      if ((st = check_launch("head accumulator kernel")) != TALM_OK) return st;
      if (pipe && cudaEventRecord(pipe->drained[buf], pipe->stream) != cudaSuccess)
        return check_launch("side stream event");
    }
  }
  // join: the caller's stream continues after the last accumulator GEMM
  if (pipe && cudaStreamWaitEvent(stream, pipe->drained[(n_slices - 1) & 1], 0) != cudaSuccess)
    return check_launch("join the side stream");
  return TALM_OK;
}

int talm_head_finalize(const float* stats, const int64_t* targets, int64_t n_tokens,
                       int64_t n_grad, const float* acc, const float* acc_scale,
                       const uint16_t* weight, int64_t ld_weight, int64_t vocab_col0,
                       int64_t vocab_cols, int64_t hidden_size, const int64_t* grad_rows,
                       float* token_loss, float* token_entropy, int32_t* correct, void* grad,
                       int grad_is_f32, void* stream) {
  using namespace talm;
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  if (n_tokens == 0) return TALM_OK;
  if (!stats || !targets) return set_error(TALM_EINVAL, "null pointer");
  if (grad != nullptr && n_grad > 0 && (acc == nullptr || weight == nullptr))
    return set_error(TALM_EINVAL, "gradient needs acc and weight");
  LaunchTimer timer(TALM_KERNEL_HEAD_FINALIZE, static_cast<cudaStream_t>(stream));
  head::head_finalize_kernel<<<static_cast<int>((n_tokens + 7) / 8), 256, 0,
                               static_cast<cudaStream_t>(stream)>>>(
      stats, reinterpret_cast<const long long*>(targets), static_cast<int>(n_tokens),
      static_cast<int>(n_grad), acc, acc_scale, reinterpret_cast<const __half*>(weight),
      ld_weight, vocab_col0, vocab_cols, static_cast<int>(hidden_size),
      reinterpret_cast<const long long*>(grad_rows), token_loss, token_entropy, correct, grad,
      grad_is_f32);
  return check_launch("head finalize kernel");
}

int talm_head_combine(const float* gathered, int64_t n_shards, int64_t n_tokens, int64_t rank,
                      int64_t n_grad, float* stats_out, float* acc_scale, void* stream) {
  using namespace talm;
  if (n_shards < 1 || rank < 0 || rank >= n_shards || n_tokens < 0 || n_grad < 0 ||
      n_grad > n_tokens)
    return set_error(TALM_EINVAL, "bad shard arguments");
  if (n_tokens == 0) return TALM_OK;
  if (!gathered || !stats_out) return set_error(TALM_EINVAL, "null pointer");
  LaunchTimer timer(TALM_KERNEL_HEAD_MERGE, static_cast<cudaStream_t>(stream));
  head::head_merge_shards_kernel<<<static_cast<int>((n_tokens + 255) / 256), 256, 0,
                                   static_cast<cudaStream_t>(stream)>>>(
      gathered, static_cast<int>(n_shards), static_cast<int>(n_tokens), static_cast<int>(rank),
      static_cast<int>(n_grad), stats_out, acc_scale);
  return check_launch("head merge kernel");
}

}  // extern "C"
