// Fused LM head + cross-entropy, forward and backward, without materialised logits.
//
// The vocabulary (or this rank's shard of it) is walked in slices (a narrow first slice, then
// equal slices of at most `vocab_chunk` columns). Two kinds of work run per slice:
//
//   * the logits GEMM (tcgen05, TMA-fed, CTA pairs): tiles of 256 token rows x 256 vocab columns
//     of z = fp16(h . W^T), K = hidden. The fp32 accumulator lives in TMEM (two 256-column
//     buffers, so the epilogue of one tile overlaps the MMAs of the next). The epilogue (two
//     groups of 4 warps, one token row per thread) rounds each logit to fp16 as the reference's
//     cuBLAS output does, and computes per 128-column part: max m_t, first argmax,
//     s_t = sum exp(z - base), t_t = sum exp(z - base) z, the target logit; for the labelled
//     rows it stores p = fp16(exp(z - base)) into the slice's probability buffer (the only
//     [rows, chunk] buffer of the head), base = the row's reference REF (the part's max on the
//     first slice, or where the max outgrew REF + 8);
//   * the accumulator GEMM (same tiles, K = slice columns): acc[256 rows, 256 hidden] +=
//     P W_slice by TMA reduce-add into an acc that starts at zero, P and W_slice TMA -> MMA
//     untouched (W read MN-major, hidden contiguous, straight from the weight rows).
//
// head_slice_kernel runs the logits GEMM of slice s together with the accumulator GEMM of
// slice s - 1 in one persistent launch (one list of whole tiles per CTA pair, balanced in
// K-blocks: the logits tiles fill what the accumulator tiles leave), then head_combine_kernel
// merges slice s's part statistics
// into the running ones (log-sum-exp merge). A row whose reference moved in slice s (every row
// on the first slice, afterwards only a row whose max outgrew REF + 8) has its probability row
// rescaled in place to fp16(exp(z - REF_new)), the reference's in-place softmax weights, and its
// acc row multiplied by alpha = exp(REF_old - REF_new) (the online-softmax rescale of
// solution/fused_head.py:170-177) before the accumulator GEMM of slice s reads them.
//
// A last launch (head_finalize_kernel) turns the statistics into loss / entropy / correctness
// and the accumulator into dH = acc / s - fp16(W[target]) (fused_head.py:111-125, :160-169),
// writing rows in the caller's original order.
//
// Operands reach shared memory in stages of two 64-column K sub-blocks (one barrier wait and
// one commit per 128 of K), each operand of a stage by one 3-D TMA request where the hidden
// size allows. In the vocabulary-parallel walk under the peer exchange, the walk's last step
// (the accumulator GEMM of the last slice) can run after the ranks' statistics are merged
// (talm_head_shard_begin / talm_head_shard_finish_scatter): its epilogue then finishes each
// gradient row piece and stores it at the rank that owns the row.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace talm {
namespace head {

constexpr int BM = 128;  // token rows per CTA = TMEM lanes; a CTA pair covers 2 * BM rows
constexpr int PAIR_ROWS = 2 * BM;
// Pair rows per band of the logits tile order (logits_tile). Measured at config 4 (64 pair
// rows): bands of 8 read 654 MB of DRAM per slice launch against 760 MB for one band of all
// 64 (the hidden rows re-read as the probability streams evict them), and the step ran 2 %
// faster; bands of 4 and 16 timed the same as 8.
constexpr int kBandRows = 8;
constexpr int BN = 256;  // columns of a pair tile (vocab in the logits GEMM, hidden in the acc GEMM)
constexpr int BK = 64;   // K per sub-block: one 128-byte swizzle row of fp16
// A pipeline stage holds KSUB sub-blocks of BK (each its own A and B tiles), so that the MMA
// warp waits for one stage and commits one release per KSUB * BK of K. Measured on these GPUs
// with operands fixed in shared memory and a producer thread on the same barriers: a wait +
// commit per 64 of K holds the tensor pipe to 0.75-0.79 of its rate, one per 128 of K to
// 0.90-0.93, whatever the number of stages (3 to 12); in this kernel 3 stages of 2 sub-blocks
// ran 5 % faster than 5 stages of 1, and 2 stages of 3 sub-blocks 9 % slower (too little
// latency hidden).
constexpr int KSUB = 2;
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;        // 16 KiB: this CTA's 128 rows of A
constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KiB: this CTA's half of B's columns
constexpr int SUB_BYTES = A_BYTES + B_BYTES;
constexpr int STAGE_BYTES = KSUB * SUB_BYTES;
constexpr int TMEM_COLS = 2 * BN;           // double-buffered fp32 accumulator (128 x 256 per CTA)
// Epilogue staging: one 16 KiB buffer (128 rows x 128 bytes, 128-byte swizzle) per epilogue
// group, through which the epilogue's outputs leave by TMA store / reduce-add instead of
// per-lane global stores; before refilling it the group's TMA-issuing thread waits until the
// previous store has read it (the three pipeline stages leave room for one buffer per group).
constexpr int STAGING_PER_GROUP = 1;  // staging buffers per epilogue group
constexpr int STAGING_BYTES = 2 * STAGING_PER_GROUP * 16384;
constexpr int SMEM_BYTES =
    STAGES * STAGE_BYTES + STAGING_BYTES + 1024 /*align slack*/ + 512 /*barriers*/;
// Two epilogue groups of 4 warps (one warp per TMEM lane quarter in each group); group g owns
// columns [g * 128, g * 128 + 128) of the tile, so two warps per SM sub-partition interleave
// and hide each other's latencies. Each group has its own named barrier (ids 1, 2), staging
// buffer and TMA-issuing thread; per row and tile it leaves one statistics record ("part").
constexpr int EPI_GROUPS = 2;
constexpr int EPI_COLS = BN / EPI_GROUPS;      // 128 columns per group
constexpr int EPI_WARPS = 4 * EPI_GROUPS;      // 8
constexpr int EPI_THREADS = 128;               // threads per group
constexpr int PARTS = EPI_GROUPS;              // statistics records per (row, tile)
constexpr int SLICE_THREADS = 32 * (2 + EPI_WARPS);  // producer, MMA, epilogue warps
constexpr float kLog2e = 1.4426950408889634f;
// Slack of the lazy reference: a row's probabilities and accumulator stay relative to REF while
// its running max is at most REF + kRefSlack, so p = exp(z - REF) <= e^8 (fits fp16).
constexpr float kRefSlack = 8.0f;

// M = 256 across the CTA pair, N = 256 (128 columns of B in each CTA's shared memory)
constexpr uint32_t kIdescLogits = idesc_f16_f32(PAIR_ROWS, BN, false, false);  // A, B K-major
constexpr uint32_t kIdescAccum = idesc_f16_f32(PAIR_ROWS, BN, false, true);    // B (W) MN-major

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Barriers of a CTA of a pair. The pair leader (cluster rank 0) issues every MMA; `full` and
// `tempty` are waited on in the leader only and receive arrivals / transaction bytes from both
// CTAs; `empty` and `tfull` live in each CTA.
struct SharedCtl {
  uint64_t full[STAGES];   // leader: both CTAs' operands of the stage landed (TMA bytes)
  uint64_t empty[STAGES];  // each CTA: the pair's MMAs finished reading the stage
  uint64_t tfull[2];       // each CTA: its half of an accumulator buffer is complete
  uint64_t tempty[2];      // leader: both CTAs' epilogues drained the buffer
  uint64_t drain;          // MMA issuer: every UMMA issued has completed
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// Write 16 bytes of row r (0..127), 16-byte chunk q (0..7), into a staging buffer laid out as
// a TMA box of 128 rows x 128 bytes with the 128-byte swizzle (chunk q of row r sits at
// q ^ (r & 7)): a warp's 32 rows spread over all 8 chunk positions, so every 512-byte warp
// access takes the minimum 4 shared-memory wavefronts.
__device__ __forceinline__ void stage_chunk(uint8_t* buf, int r, int q, uint32_t a, uint32_t b,
                                            uint32_t c, uint32_t d) {
  *reinterpret_cast<uint4*>(buf + r * 128 + ((q ^ (r & 7)) << 4)) = make_uint4(a, b, c, d);
}

// Set-up shared by both GEMMs: barriers, TMEM for the pair, cluster-wide visibility.
__device__ __forceinline__ void pair_setup(SharedCtl* ctl, int warp) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->tfull[a], 1);
      mbar_init(&ctl->tempty[a], 2 * EPI_WARPS);  // every epilogue warp of both CTAs
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
  cluster_sync();
  tc_fence_after();
}

__device__ __forceinline__ void pair_teardown(SharedCtl* ctl, int warp, uint32_t tmem_base) {
  tc_fence_before();
  cluster_sync();  // the peer's shared memory stays alive until the leader's MMAs are done
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// On the way out of the leader's producer: every copy counted on its `full` barriers (both
// CTAs' halves) must have landed before the pair releases its shared memory. (stage, phase) is
// the next slot; the last min(issued, STAGES) slots hold the outstanding copies.
__device__ __forceinline__ void drain_copies(SharedCtl* ctl, int stage, uint32_t phase,
                                             int issued) {
  for (int i = 0; i < STAGES && i < issued; ++i) {
    if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
    mbar_drain(&ctl->full[stage], phase);
  }
}

// On the way out of the MMA issuer: wait until every UMMA it issued has completed.
__device__ __forceinline__ void drain_mmas(SharedCtl* ctl) {
  umma_commit_pair(&ctl->drain);
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
  int n_parts;        // n_col_tiles * PARTS: statistics records per row
  int n_pair_rows;    // ceil(n_tokens / PAIR_ROWS)
  int band_rows;      // pair rows per band of the tile order (logits_tile)
  int k3d;            // stages of two sub-blocks load through the 3-D k-chunk maps
  long long col_base; // global column id of slice column 0
  int has_ref;        // 0 on the first slice: no reference yet
  const long long* targets;
  float4* partial;    // [n_tokens][n_parts]: m, s, t, first argmax (int bits) per part
  float* stats;       // [n_tokens][TALM_HEAD_STATS]
};

// Logits tile t of a slice -> (pair row block pr, column tile ct). The tiles go in bands of
// band_rows pair rows (the last band may be shorter), column after column within a band, so
// that the tiles running at the same time on the pairs share a band of hidden rows and a few
// weight tiles in L2.
__device__ __forceinline__ void logits_tile(const LogitsParams& lp, int t, int& pr, int& ct) {
  const int per_band = lp.band_rows * lp.n_col_tiles;
  const int band = t / per_band;
  const int r = t - band * per_band;
  const int rows = min(lp.band_rows, lp.n_pair_rows - band * lp.band_rows);
  ct = r / rows;
  pr = band * lp.band_rows + (r - ct * rows);
}

// ------------------------------------------------------------------------------------------
// 2. per-slice combine of tile statistics with the running statistics
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void better_arg(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(256) head_combine_kernel(const float4* __restrict__ partial,
                                                           int n_parts, int n_tokens,
                                                           int n_grad, int first,
                                                           float* __restrict__ stats,
                                                           __half* __restrict__ probs,
                                                           int probs_ld,
                                                           float* __restrict__ acc, int hidden) {
  grid_dependency_wait();  // the slice's part statistics and probabilities
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= n_tokens) return;
  const float4* pr = partial + static_cast<long long>(row) * n_parts;
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
  for (int j = lane; j < n_parts; j += 32) {
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
  // (the factor w_j below is 1 exactly for every part of a row that kept its reference)
  auto part_factor = [&](const float4& v) {
    const float base = (!first && v.x <= ref + kRefSlack) ? ref : v.x;
    return ex2((base - ref_new) * kLog2e);
  };
  float S = 0.0f, T = 0.0f;
  for (int j = lane; j < n_parts; j += 32) {
    const float4 v = pr[j];
    const float w = part_factor(v);
    S = fmaf(v.y, w, S);
    T = fmaf(v.z, w, T);
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
  }
  if (!jump || row >= n_grad) return;
  // The row moved its reference: its probabilities of this slice become p * w_j, i.e.
  // fp16(exp(z - REF_new)) (the stored p was taken relative to base_j), read and written in
  // 16-byte pieces of 8 columns, EPI_COLS / 8 pieces per part.
  if (probs != nullptr) {
    uint4* prow = reinterpret_cast<uint4*>(probs + static_cast<long long>(row) * probs_ld);
    const int n_pieces = n_parts * (EPI_COLS / 8);
    for (int c = lane; c < n_pieces; c += 32) {
      const float w = part_factor(pr[c / (EPI_COLS / 8)]);
      uint4 q = prow[c];
      uint32_t* h = reinterpret_cast<uint32_t*>(&q);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h[i]));
        h[i] = pack_half2(f.x * w, f.y * w);
      }
      prow[c] = q;
    }
  }
  // acc = alpha * acc (alpha = 1 for every row that kept its reference); the earlier slices'
  // accumulator GEMMs precede this launch, the current slice's follows it
  if (!first && acc != nullptr) {
    float4* arow = reinterpret_cast<float4*>(acc + static_cast<long long>(row) * hidden);
    for (int v = lane; v < hidden / 4; v += 32) {
      float4 o = arow[v];
      o.x *= a;
      o.y *= a;
      o.z *= a;
      o.w *= a;
      arow[v] = o;
    }
  }
}

// ------------------------------------------------------------------------------------------
// 3. accumulator GEMM: acc += P W_slice (acc starts at zero; moved rows rescaled by combine)
// ------------------------------------------------------------------------------------------
struct AccumParams {
  int n_grad;
  int hidden;
  int k_blocks;      // slice columns / BK (padded slice: a multiple of BN / BK)
  int slice_row0;    // first weight row of the slice
  int n_pair_rows;   // ceil(n_grad / PAIR_ROWS)
  int n_h_tiles;     // ceil(hidden / BN)
  int k3d;           // stages load through the 3-D k-chunk maps (hidden % 64 == 0)
};

// ------------------------------------------------------------------------------------------
// One launch per slice step: the logits GEMM of slice s and the accumulator GEMM of slice s - 1
// share one persistent grid of CTA pairs, so that the accumulator work fills the logits GEMM's
// last, partial wave (and vice versa) and a slice costs two launches (this and the combine).
// ------------------------------------------------------------------------------------------
// One element of a gradient row under a merged scale (the vocabulary-parallel flows):
// a * scale, minus the target's weight where this rank holds the target column, 0 for a row
// without gradient; each operation rounded on its own (no contraction into an FMA), so that
// the scatter epilogue and head_finalize_kernel give the same bits.
__device__ __forceinline__ float grad_value(bool live, bool own, float a, float scale, float w) {
  if (!live) return 0.0f;
  const float g = __fmul_rn(a, scale);
  return own ? __fsub_rn(g, w) : g;
}

// The last accumulator step of a vocabulary-parallel walk under the peer exchange
// (talm_head_shard_finish_scatter): instead of adding its tiles into acc, the epilogue
// finishes each piece of a gradient row -- (acc + D) * scale[row], minus the target's weight
// row where this rank holds the target column, 0 for an unlabelled row; the arithmetic of
// head_finalize_kernel after a reduce-add of D -- and stores it in fp32 straight into the
// owning rank's receive slot over NVLink, so that the scatter overlaps the step's MMAs. The
// last CTA to finish raises this rank's phase-1 flag on every rank.
struct ScatterParams {
  int on;
  int tile_shift;                   // accumulator tiles are taken from this one on (rotated)
  const float* acc;                 // [n_grad][hidden]: the earlier slices' sum
  const float* scale;               // [n_grad]: e^(REF - REF_merged) / S_merged
  const long long* targets;         // [n_tokens], in row order
  const long long* grad_rows;       // output row of each row (null: the row itself)
  const __half* weight;             // this rank's weight rows
  long long ld_weight, col0, vcols;
  const unsigned long long* peers;  // every rank's peer buffer, mapped here
  peer::PeerLayout L;
  int rank, world;
  uint32_t epoch;
};

struct SliceParams {
  LogitsParams lg;  // logits GEMM of slice s: n_tiles_l pair tiles (0: none, the last step)
  AccumParams ac;   // accumulator GEMM of slice s - 1: n_tiles_a pair tiles (0: none)
  ScatterParams sc; // sc.on: the accumulator tiles finish the rows and scatter them
  int n_tiles_l;
  int n_tiles_a;
};

// A unit of work: a whole logits tile (type 0) or accumulator tile (type 1), K-blocks
// [kb0, kb1).
struct Unit {
  int type, tile, kb0, kb1;
};

// This pair's share of a step, in whole tiles (so that every acc element receives exactly one
// addition per slice: the sums are the same bits on every run). Accumulator tiles go
// round-robin over the pairs; when their count is not a multiple of the pair count, the
// first nA pairs hold one more accumulator tile than the other nB pairs, so the logits tiles
// first go round-robin over those nB pairs (d each, d = K_a / K_l rounded: one accumulator
// tile's worth of K-blocks), then round-robin over all pairs. Tiles that run at the same time
// on different pairs stay neighbours in the tile order (logits tiles: one band of row blocks
// and a few weight column tiles; accumulator tiles: a few row blocks of probabilities and
// every hidden column tile), which keeps their operands shared in L2. Every role of both CTAs
// computes the same plan and walks the same unit sequence: the accumulator tiles, then the
// logits tiles.
struct PairPlan {
  int n_a;      // accumulator tiles: pair + i * n_pairs
  int n_l1;     // logits tiles of the first round-robin: (pair - nA) + i * nB
  int n_l2;     // logits tiles of the second: base2 + pair + i * n_pairs
  int nA, nB, base2;
};

__device__ __forceinline__ PairPlan plan_pair(const SliceParams& p, int pair, int n_pairs) {
  const int ta = p.n_tiles_a, tl = p.n_tiles_l;
  PairPlan r;
  r.n_a = ta / n_pairs + (pair < ta % n_pairs ? 1 : 0);
  r.nA = ta % n_pairs;
  r.nB = n_pairs - r.nA;
  int d = 0;
  if (r.nA > 0 && tl > 0 && p.lg.k_blocks > 0)
    d = min((p.ac.k_blocks + p.lg.k_blocks / 2) / p.lg.k_blocks, tl / r.nB);
  r.n_l1 = pair >= r.nA ? d : 0;
  r.base2 = d * r.nB;
  r.n_l2 = tl - r.base2 > pair ? (tl - r.base2 - pair + n_pairs - 1) / n_pairs : 0;
  return r;
}

__device__ __forceinline__ bool slice_unit(const SliceParams& p, const PairPlan& plan, int pair,
                                           int n_pairs, int u, Unit& out) {
  out.kb0 = 0;
  if (u < plan.n_a) {
    out.type = 1;
    out.tile = pair + u * n_pairs;
    if (p.sc.on) out.tile = (out.tile + p.sc.tile_shift) % p.n_tiles_a;
    out.kb1 = p.ac.k_blocks;
    return true;
  }
  u -= plan.n_a;
  out.type = 0;
  out.kb1 = p.lg.k_blocks;
  if (u < plan.n_l1) {
    out.tile = (pair - plan.nA) + u * plan.nB;
    return true;
  }
  u -= plan.n_l1;
  if (u < plan.n_l2) {
    out.tile = plan.base2 + pair + u * n_pairs;
    return true;
  }
  return false;
}

// Logits tile t covers rows [pr * 256, +256) x slice columns [ct * 256, +256) (pr = t % pair
// rows); the CTA of rank r owns rows pr * 256 + r * 128 + [0, 128) (its TMEM lanes) and loads
// weight rows ct * 256 + r * 128 + [0, 128) (K-major B): the pair's accumulator columns
// 0..127 come from the leader's B half, 128..255 from the peer's. Accumulator tile t covers
// labelled rows [pr * 256, +256) x hidden columns [ht * 256, +256) (ht = t % hidden tiles); the
// CTA of rank r owns rows pr * 256 + r * 128 + [0, 128) and loads hidden columns
// ht * 256 + r * 128 + [0, 128) of W (two 64-wide MN-major boxes per stage).
__global__ void __launch_bounds__(SLICE_THREADS, 1)
    head_slice_kernel(const __grid_constant__ CUtensorMap tm_hidden,
                      const __grid_constant__ CUtensorMap tm_weight,
                      const __grid_constant__ CUtensorMap tm_probs_out,
                      const __grid_constant__ CUtensorMap tm_probs_in,
                      const __grid_constant__ CUtensorMap tm_weight_mn,
                      const __grid_constant__ CUtensorMap tm_acc,
                      const __grid_constant__ CUtensorMap tm_hidden3,
                      const __grid_constant__ CUtensorMap tm_weight3,
                      const __grid_constant__ CUtensorMap tm_probs3_in, SliceParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(staging + STAGING_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const LogitsParams& lp = p.lg;
  const AccumParams& ap = p.ac;
  if (threadIdx.x == 0) {
    if (p.n_tiles_l > 0) {
      prefetch_tmap(&tm_hidden);
      prefetch_tmap(&tm_weight);
      if (lp.n_grad > 0) prefetch_tmap(&tm_probs_out);
    }
    if (p.n_tiles_a > 0) {
      prefetch_tmap(&tm_probs_in);
      prefetch_tmap(&tm_weight_mn);
      prefetch_tmap(&tm_acc);
    }
  }
  pair_setup(ctl, warp);
  grid_dependency_wait();  // the previous kernel's outputs (statistics, probabilities, acc)
  const uint32_t tmem_base = ctl->tmem_base;
  volatile int* abort = &ctl->abort;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const PairPlan plan = plan_pair(p, pair, n_pairs);
  Unit unit;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer (both CTAs): this CTA's halves, counted on the leader
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int u = 0; !*abort && slice_unit(p, plan, pair, n_pairs, u, unit); ++u) {
        for (int kb0 = unit.kb0; kb0 < unit.kb1; kb0 += KSUB) {
          const int nsub = min(KSUB, unit.kb1 - kb0);
          if (!mbar_wait(&ctl->empty[stage], phase ^ 1, abort)) break;
          const uint32_t lfull = mapa_shared(smem_u32(&ctl->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&ctl->full[stage], 2 * nsub * SUB_BYTES);
          uint8_t* const st = smem + stage * STAGE_BYTES;
          if (nsub == 2 && (unit.type == 0 ? lp.k3d : ap.k3d)) {
            // one request per operand for both sub-blocks (3-D k-chunk boxes): the stage
            // holds A0 A1 B0 B1 (logits) or A0 A1 and the two 64-column weight groups of
            // 128 K-rows each (accumulator); TMA requests, not bytes, limit the operand feed
            if (unit.type == 0) {
              int pr, ct;
              logits_tile(lp, unit.tile, pr, ct);
              tma_load_3d_pair(st, &tm_hidden3, lfull, 0, pr * PAIR_ROWS + rank * BM, kb0);
              tma_load_3d_pair(st + 2 * A_BYTES, &tm_weight3, lfull, 0,
                               lp.slice_row0 + ct * BN + rank * (BN / 2), kb0);
            } else {
              const int ht = unit.tile % ap.n_h_tiles, pr = unit.tile / ap.n_h_tiles;
              tma_load_3d_pair(st, &tm_probs3_in, lfull, 0, pr * PAIR_ROWS + rank * BM, kb0);
              tma_load_3d_pair(st + 2 * A_BYTES, &tm_weight3, lfull, 0,
                               ap.slice_row0 + kb0 * BK, (ht * BN + rank * (BN / 2)) / 64);
            }
          } else {
            // 2-D boxes, one sub-block at a time (an odd last sub-block, or a hidden size that
            // is not a multiple of 64): A then B per sub-block
            for (int j = 0; j < nsub; ++j) {
              const int kb = kb0 + j;
              uint8_t* a = st + j * SUB_BYTES;
              if (unit.type == 0) {
                int pr, ct;
                logits_tile(lp, unit.tile, pr, ct);
                tma_load_2d_pair(a, &tm_hidden, lfull, kb * BK, pr * PAIR_ROWS + rank * BM);
                tma_load_2d_pair(a + A_BYTES, &tm_weight, lfull, kb * BK,
                                 lp.slice_row0 + ct * BN + rank * (BN / 2));
              } else {
                const int ht = unit.tile % ap.n_h_tiles, pr = unit.tile / ap.n_h_tiles;
                tma_load_2d_pair(a, &tm_probs_in, lfull, kb * BK, pr * PAIR_ROWS + rank * BM);
#pragma unroll
                for (int h = 0; h < BN / 2 / 64; ++h)
                  tma_load_2d_pair(a + A_BYTES + h * (64 * BK * 2), &tm_weight_mn, lfull,
                                   ht * BN + rank * (BN / 2) + h * 64, ap.slice_row0 + kb * BK);
              }
            }
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (leader) drain_copies(ctl, stage, phase, issued);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // MMA issuer (leader only)
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int u = 0; slice_unit(p, plan, pair, n_pairs, u, unit); ++u) {
        if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb0 = unit.kb0; kb0 < unit.kb1; kb0 += KSUB) {
          const int nsub = min(KSUB, unit.kb1 - kb0);
          if (!mbar_wait(&ctl->full[stage], phase, abort)) { ok = false; break; }
          tc_fence_after();
          const bool s3 = nsub == 2 && (unit.type == 0 ? lp.k3d : ap.k3d);
          const uint32_t st = smem_u32(smem + stage * STAGE_BYTES);
          for (int j = 0; j < nsub; ++j) {
            const uint32_t a = s3 ? st + j * A_BYTES : st + j * SUB_BYTES;
            // 3-D stages: B0 B1 after A0 A1 (logits); the accumulator's weight groups of 128
            // K-rows each, 16 KiB apart, sub-block j at +8 KiB
            const uint32_t b = s3 ? st + 2 * A_BYTES + j * (unit.type == 0 ? B_BYTES : 64 * BK * 2)
                                  : a + A_BYTES;
            const uint32_t lbo_acc = s3 ? 2 * 64 * BK * 2 : 64 * BK * 2;
            const bool first_kb = kb0 + j == unit.kb0;
            if (unit.type == 0) {
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)  // A and B K-major rows of 128 B, +32 B per 16 K
                umma_f16_pair(d, smem_desc_sw128(a + k * 32, 16, 1024),
                              smem_desc_sw128(b + k * 32, 16, 1024), kIdescLogits,
                              !first_kb || k != 0);
            } else {
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                // A: K-major rows of 128 B, +32 B per 16 K. B: MN-major, two 64-wide hidden
                // groups of 128 B rows (LBO = the group distance: 8 KiB for a 2-D stage, 16 KiB
                // for a 3-D one), 16 K-rows = +2 KiB.
                umma_f16_pair(d, smem_desc_sw128(a + k * 32, 16, 1024),
                              smem_desc_sw128(b + k * 2048, lbo_acc, 1024), kIdescAccum,
                              !first_kb || k != 0);
            }
          }
          umma_commit_pair(&ctl->empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&ctl->tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      drain_mmas(ctl);
    }
  } else {  // epilogue: warps 2..9 of both CTAs, TMEM lane quarter = warp % 4
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;                    // epilogue group: columns g*128..+128
    const int bar_id = 1 + g;
    const int r_in_tile = q * 32 + lane;
    const bool elected = (warp - 2) % 4 == 0 && lane == 0;  // the group's TMA-issuing thread
    uint8_t* const bufs = staging + g * STAGING_PER_GROUP * 16384;  // the group's buffers
    int nb = 0;                                     // the one to fill next
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = 0; slice_unit(p, plan, pair, n_pairs, u, unit); ++u) {
      // CTA-uniform decision among the 4 epilogue warps (named barriers follow; every lane's
      // wait is bounded, so every thread reaches the vote)
      const bool landed = mbar_wait(&ctl->tfull[acc], acc_phase, abort);
      if (named_barrier_or(bar_id, EPI_THREADS, !landed)) break;
      tc_fence_after();
      if (unit.type == 0) {  // logits tile: statistics and probabilities
        int pr, ct;
        logits_tile(lp, unit.tile, pr, ct);
        const int row0 = pr * PAIR_ROWS + rank * BM;  // first row of this CTA's half
        const int row = row0 + r_in_tile;
        const bool valid_row = row < lp.n_tokens;
        const long long tgt = valid_row ? lp.targets[row] : -1;
        const long long tile_col0 = lp.col_base + static_cast<long long>(ct) * BN;
        const long long tcol_ll = tgt - tile_col0;
        const int tcol = (tgt >= 0 && tcol_ll >= g * EPI_COLS && tcol_ll < (g + 1) * EPI_COLS)
                             ? static_cast<int>(tcol_ll) : -1;
        const int ncols = min(BN, lp.cols - ct * BN);  // valid columns of the tile (tile-relative)
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
        // probabilities leave through the staging buffers by TMA store (64 columns = 16 KiB per
        // store); CTAs whose rows are all unlabelled (or no gradient) skip them
        const bool store_p = row0 < lp.n_grad;

        // Rows with a reference (every slice after the first) take ONE pass over TMEM: logits
        // rounded to fp16, running max / first argmax / target logit, and s, t, p relative to
        // REF. If some row's tile max outgrows REF + slack (its reference moves: rare), the CTA
        // takes a second pass in which those rows use their tile max. The first slice (no
        // reference yet) takes a max pass, then the sum pass relative to the tile max.
        const float ref = (lp.has_ref && valid_row)
                              ? lp.stats[static_cast<long long>(row) * TALM_HEAD_STATS + TALM_STAT_REF]
                              : 0.0f;
        const bool full_tile = ncols >= (g + 1) * EPI_COLS;  // the group's columns all valid
        // is this warp's target column anywhere in the tile (then the per-element test runs)
        const bool any_target = __any_sync(0xffffffffu, tcol >= 0);
        float mx = -INFINITY, zt = 0.0f, s = 0.0f, t = 0.0f;
        int arg = g * EPI_COLS;
        uint32_t r[32];
        // One 32-column chunk: `track` = max / argmax / target, `sum` = s, t and the
        // probabilities (written to `buf`, 16-byte chunks qbase..qbase+3 of this row). The TMEM
        // load is warp-collective (.sync.aligned): every lane executes it. `full` (a compile-time
        // flag: the group's columns are all valid) drops the per-column bounds tests.
        uint32_t packed[16];  // the last chunk's probabilities, fp16 pairs
        auto chunk = [&](auto full, int c, bool track, bool sum, float mscaled) {
          constexpr bool kFull = decltype(full)::value;
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_wait_ld();
  #pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const int col = c * 32 + j;
            // fp16 rounding of the pair as the reference's fp16 GEMM output (one packed cvt)
            const float2 z = __half22float2(
                __floats2half2_rn(__uint_as_float(r[j]), __uint_as_float(r[j + 1])));
            const bool ok0 = kFull || col < ncols;
            const bool ok1 = kFull || col + 1 < ncols;
            if (track) {
              if (ok0 && z.x > mx) { mx = z.x; arg = col; }
              if (ok1 && z.y > mx) { mx = z.y; arg = col + 1; }
              if (any_target) {
                if (col == tcol) zt = z.x;
                if (col + 1 == tcol) zt = z.y;
              }
            }
            if (sum) {
              const float e0 = ok0 ? ex2(fmaf(z.x, kLog2e, -mscaled)) : 0.0f;
              const float e1 = ok1 ? ex2(fmaf(z.y, kLog2e, -mscaled)) : 0.0f;
              s += e0 + e1;
              t = fmaf(e0, z.x, t);
              t = fmaf(e1, z.y, t);
              packed[j / 2] = pack_half2(e0, e1);
            }
          }
        };
        // the last chunk's probabilities into 16-byte pieces qbase..qbase+3 of this row
        auto stage = [&](uint8_t* buf, int qbase) {
  #pragma unroll
          for (int v = 0; v < 4; ++v)
            stage_chunk(buf, r_in_tile, qbase + v, packed[4 * v], packed[4 * v + 1],
                        packed[4 * v + 2], packed[4 * v + 3]);
        };
        // A pass with sums over the group's columns: 2 blocks of 64 columns, each staged and
        // stored. `base` per lane; `track` for the single-pass case. The first chunk of a block
        // is loaded and computed before the wait for the staging buffer (the previous block's
        // store may still be reading it), so that the wait overlaps that work.
        auto sum_pass = [&](auto full, bool track, float base) {
          const float mscaled = base * kLog2e;
  #pragma unroll 1
          for (int kb = g * (EPI_COLS / 64); kb < (g + 1) * (EPI_COLS / 64); ++kb) {
            uint8_t* buf = bufs + nb * 16384;
            chunk(full, 2 * kb, track, true, mscaled);
            if (store_p) {
              // the store issued from this buffer two blocks ago has read it (at most the last
              // store, from the other buffer, may still be reading)
              if (elected) bulk_wait_read<STAGING_PER_GROUP - 1>();
              named_barrier(bar_id, EPI_THREADS);
              nb = (nb + 1) % STAGING_PER_GROUP;
              stage(buf, 0);
            }
            chunk(full, 2 * kb + 1, track, true, mscaled);
            if (store_p) {
              stage(buf, 4);
              fence_proxy_async_smem();
              named_barrier(bar_id, EPI_THREADS);
              if (elected) {
                tma_store_2d(&tm_probs_out, buf, ct * BN + kb * 64, row0);
                bulk_commit();
              }
            }
          }
        };
        auto epilogue = [&](auto full) {
          if (lp.has_ref) {
            s = 0.0f;
            t = 0.0f;
            sum_pass(full, true, ref);
            const bool jump = mx > ref + kRefSlack;
            if (named_barrier_or(bar_id, EPI_THREADS, jump)) {
              // some row's reference moves in the group's columns: they are redone (rows
              // without a move recompute the same values); earlier stores must land before the
              // new ones
              if (elected) bulk_wait_all();
              named_barrier(bar_id, EPI_THREADS);
              s = 0.0f;
              t = 0.0f;
              sum_pass(full, false, jump ? mx : ref);
            }
          } else {
  #pragma unroll 1
            for (int c = g * (EPI_COLS / 32); c < (g + 1) * (EPI_COLS / 32); ++c)
              chunk(full, c, true, false, 0.0f);
            sum_pass(full, false, mx);
          }
        };
        if (full_tile) {
          epilogue(std::true_type{});
        } else {
          epilogue(std::false_type{});
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->tempty[acc]), 0));
        if (valid_row) {
          lp.partial[static_cast<long long>(row) * lp.n_parts + ct * PARTS + g] =
              make_float4(mx, s, t, __int_as_float(static_cast<int>(tile_col0 + arg)));
          if (tcol >= 0 && tcol < ncols) {
            float* st = lp.stats + static_cast<long long>(row) * TALM_HEAD_STATS;
            st[TALM_STAT_ZT] = zt;
            st[TALM_STAT_HIT] = 1.0f;
          }
        }
      } else if (p.sc.on) {  // the walk's last accumulator step: finish the rows, send them
        // Per 32-column chunk: D (one row per thread, as TMEM gives it) goes through the
        // group's staging buffer, then 8 lanes per row (4 columns each) finish 4 rows per
        // step, so that every row piece leaves as one 128-byte line (a store of a lane per row
        // would split each line into 16-byte writes over NVLink).
        const ScatterParams& sc = p.sc;
        const int ht = unit.tile % ap.n_h_tiles, pr = unit.tile / ap.n_h_tiles;
        const int row0 = pr * PAIR_ROWS + static_cast<int>(rank) * BM;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
        uint8_t* const buf = bufs;
        const int sub = lane >> 3, piece = lane & 7;
  #pragma unroll 1
        for (int c = g * (EPI_COLS / 32); c < (g + 1) * (EPI_COLS / 32); ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_wait_ld();
  #pragma unroll
          for (int v = 0; v < 8; ++v)
            stage_chunk(buf, r_in_tile, v, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
          named_barrier(bar_id, EPI_THREADS);
          const int h = ht * BN + c * 32 + piece * 4;
          if (h < ap.hidden) {
  #pragma unroll 2
            for (int i = 0; i < 8; ++i) {
              const int rl = q * 32 + i * 4 + sub;  // the tile row (of this CTA's 128)
              const int row = row0 + rl;
              if (row >= ap.n_grad) continue;
              const long long tgt = sc.targets[row];
              const bool live = tgt >= 0;
              const bool own = live && tgt >= sc.col0 && tgt < sc.col0 + sc.vcols;
              const float scale = live ? sc.scale[row] : 0.0f;
              const long long out = sc.grad_rows ? sc.grad_rows[row] : row;
              const long long owner = out / sc.L.rpr;
              float* const dst =
                  reinterpret_cast<float*>(sc.peers[owner] + sc.L.recv) +
                  (static_cast<long long>(sc.rank) * sc.L.rpr + (out - owner * sc.L.rpr)) *
                      ap.hidden + h;
              const float4 a =
                  *reinterpret_cast<const float4*>(sc.acc + static_cast<long long>(row) * ap.hidden + h);
              const uint4 d =
                  *reinterpret_cast<const uint4*>(buf + rl * 128 + ((piece ^ (rl & 7)) << 4));
              float w[4] = {0.0f, 0.0f, 0.0f, 0.0f};
              if (own) {
                const uint2 wv = *reinterpret_cast<const uint2*>(
                    sc.weight + (tgt - sc.col0) * sc.ld_weight + h);
                const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
                const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
                w[0] = w01.x; w[1] = w01.y; w[2] = w23.x; w[3] = w23.y;
              }
              // acc + D as the reduce-add of the other steps forms it, then the finalize
              *reinterpret_cast<float4*>(dst) = make_float4(
                  grad_value(live, own, __fadd_rn(a.x, __uint_as_float(d.x)), scale, w[0]),
                  grad_value(live, own, __fadd_rn(a.y, __uint_as_float(d.y)), scale, w[1]),
                  grad_value(live, own, __fadd_rn(a.z, __uint_as_float(d.z)), scale, w[2]),
                  grad_value(live, own, __fadd_rn(a.w, __uint_as_float(d.w)), scale, w[3]));
            }
          }
          named_barrier(bar_id, EPI_THREADS);  // read out before the next chunk refills it
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->tempty[acc]), 0));
      } else {  // accumulator K range: acc += D
        const int ht = unit.tile % ap.n_h_tiles, pr = unit.tile / ap.n_h_tiles;
        const int row0 = pr * PAIR_ROWS + static_cast<int>(rank) * BM;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
        // acc += D by TMA reduce-add (acc starts at zero; a moved reference was applied to acc
        // by the combine kernel before this launch)
        const bool any_rows = row0 < ap.n_grad;
  #pragma unroll 1
        for (int c = g * (EPI_COLS / 32); c < (g + 1) * (EPI_COLS / 32); ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          tmem_wait_ld();
          if (any_rows && ht * BN + c * 32 < ap.hidden) {
            uint8_t* buf = bufs + nb * 16384;
            nb = (nb + 1) % STAGING_PER_GROUP;
            // the reduce issued from this buffer two chunks ago has read it
            if (elected) bulk_wait_read<STAGING_PER_GROUP - 1>();
            named_barrier(bar_id, EPI_THREADS);
  #pragma unroll
            for (int v = 0; v < 8; ++v)
              stage_chunk(buf, r_in_tile, v, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
            fence_proxy_async_smem();
            named_barrier(bar_id, EPI_THREADS);
            if (elected) {
              tma_reduce_add_2d(&tm_acc, buf, ht * BN + c * 32, row0);
              bulk_commit();
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctl->tempty[acc]), 0));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (elected) bulk_wait_all();  // every store and reduce has landed before the CTA leaves
  }
  pair_teardown(ctl, warp, tmem_base);
  if (p.sc.on)  // every gradient row piece of this CTA has been stored at its owner
    peer::cta_signal_phase(reinterpret_cast<uint8_t*>(p.sc.peers[p.sc.rank]), p.sc.peers,
                           p.sc.L.flags, p.sc.L.counters, 1, p.sc.rank, p.sc.world, p.sc.epoch);
}

// ------------------------------------------------------------------------------------------
// 4. finalize: per-row outputs and the hidden gradient
// ------------------------------------------------------------------------------------------
// Where a gradient row goes: the caller's [n, hidden] array (fp16 or fp32), or, under the
// peer exchange, slot `rank` of the owning rank's receive region (fp32).
struct GradDest {
  void* grad;                       // local array (null: no gradient)
  int grad_f32;
  const unsigned long long* peers;  // non-null: scatter to the owners
  size_t recv_off;
  long long rpr;                    // rows per rank
  int rank;
  long long grad_from;              // rows below this one get no gradient row here
  int signal;                       // peers: the kernel ends phase 1 (raises the flags)
  __device__ __forceinline__ void* row_ptr(long long out, int hidden) const {
    if (peers == nullptr) {
      return grad_f32 ? static_cast<void*>(static_cast<float*>(grad) + out * hidden)
                      : static_cast<void*>(static_cast<__half*>(grad) + out * hidden);
    }
    const long long q = out / rpr;
    float* recv = reinterpret_cast<float*>(peers[q] + recv_off);
    return recv + (static_cast<long long>(rank) * rpr + (out - q * rpr)) * hidden;
  }
};

__device__ __forceinline__ void finalize_row(
    int row, int lane, const float* __restrict__ stats, const long long* __restrict__ targets,
    int n_grad, const float* __restrict__ acc, const float* __restrict__ acc_scale,
    const __half* __restrict__ weight, long long ld_weight, long long col0, long long vcols,
    int hidden, const long long* __restrict__ grad_rows, float* __restrict__ token_loss,
    float* __restrict__ token_entropy, int* __restrict__ correct, const GradDest& dest,
    int vec4) {
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
  if ((dest.grad == nullptr && dest.peers == nullptr) || row < dest.grad_from) return;
  const int grad_f32 = dest.peers != nullptr ? 1 : dest.grad_f32;
  void* const grow = dest.row_ptr(out, hidden);
  const bool live = labelled && row < n_grad && acc != nullptr;
  const bool own = live && tgt >= col0 && tgt < col0 + vcols;
  const float* arow = acc + static_cast<long long>(row) * hidden;
  const __half* wrow = weight + (own ? (tgt - col0) * ld_weight : 0);
  const float scale = acc_scale ? acc_scale[row] : 0.0f;
  auto value = [&](float a, __half w) {
    if (acc_scale) return grad_value(live, own, a, scale, __half2float(w));
    if (!live) return 0.0f;
    const float g = a / s;
    return own ? g - __half2float(w) : g;
  };
  if (vec4) {  // 4 columns per lane and step: 16-byte acc loads, 8- or 16-byte stores
    const __half zero = __float2half_rn(0.0f);
    for (int h = 4 * lane; h < hidden; h += 128) {
      const float4 a = live ? *reinterpret_cast<const float4*>(arow + h) : make_float4(0, 0, 0, 0);
      __half2 w01 = __halves2half2(zero, zero), w23 = w01;
      if (own) {
        const uint2 wv = *reinterpret_cast<const uint2*>(wrow + h);
        w01 = *reinterpret_cast<const __half2*>(&wv.x);
        w23 = *reinterpret_cast<const __half2*>(&wv.y);
      }
      const float g0 = value(a.x, __low2half(w01)), g1 = value(a.y, __high2half(w01));
      const float g2 = value(a.z, __low2half(w23)), g3 = value(a.w, __high2half(w23));
      if (grad_f32) {
        *reinterpret_cast<float4*>(static_cast<float*>(grow) + h) = make_float4(g0, g1, g2, g3);
      } else {
        *reinterpret_cast<uint2*>(static_cast<__half*>(grow) + h) =
            make_uint2(pack_half2(g0, g1), pack_half2(g2, g3));
      }
    }
    return;
  }
  for (int h = lane; h < hidden; h += 32) {
    const float g = value(live ? arow[h] : 0.0f, own ? wrow[h] : __float2half_rn(0.0f));
    if (grad_f32) {
      static_cast<float*>(grow)[h] = g;
    } else {
      static_cast<__half*>(grow)[h] = __float2half_rn(g);
    }
  }
}

// One warp per row. With dest.peers (the peer exchange) the kernel ends phase 1: the last CTA
// raises this rank's flag on every rank once every gradient row has reached its owner.
__global__ void __launch_bounds__(256) head_finalize_kernel(
    const float* __restrict__ stats, const long long* __restrict__ targets, int n_tokens,
    int n_grad, const float* __restrict__ acc, const float* __restrict__ acc_scale,
    const __half* __restrict__ weight, long long ld_weight, long long col0, long long vcols,
    int hidden, const long long* __restrict__ grad_rows, float* __restrict__ token_loss,
    float* __restrict__ token_entropy, int* __restrict__ correct, GradDest dest, int vec4,
    peer::PeerLayout L, int world, uint32_t epoch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Under the peer exchange the gradient rows go to their owners: rows [q * rpr, +rpr) to rank
  // q. CTAs start roughly in index order, so every rank walking the rows from 0 would send to
  // rank 0 first, then rank 1, ... (all ranks into one receiver at a time). Rank r starts its
  // walk at the rows of rank r + 1 instead: at any moment the ranks send to different owners.
  int block = blockIdx.x;
  if (dest.peers != nullptr && world > 1) {
    const long long first = (static_cast<long long>((dest.rank + 1) % world) * dest.rpr) / 8;
    block = static_cast<int>((block + first) % gridDim.x);
  }
  const int row = block * 8 + warp;
  if (row < n_tokens)
    finalize_row(row, lane, stats, targets, n_grad, acc, acc_scale, weight, ld_weight, col0,
                 vcols, hidden, grad_rows, token_loss, token_entropy, correct, dest, vec4);
  if (dest.peers != nullptr && dest.signal) {
    peer::cta_signal_phase(reinterpret_cast<uint8_t*>(dest.peers[dest.rank]), dest.peers,
                           L.flags, L.counters, 1, dest.rank, world, epoch);
  } else if (dest.peers != nullptr) {
    __threadfence_system();  // the zero rows; the scatter step after this kernel signals
  }
}

// ------------------------------------------------------------------------------------------
// labelled-first row order on the device (solution/fused_head.py:290-299)
// ------------------------------------------------------------------------------------------
// One CTA scans the labelled flags (target >= 0) 1024 rows at a time: with c(r) the labelled
// rows among 0..r, dest[r] = c(r) - 1 for a labelled row and r - c(r) + n_labelled for an
// unlabelled one (labelled rows first, each group in input order), src[dest[r]] = r. A
// dest outside [0, n) (n_labelled not the true count) is not written and records TALM_ERANGE.
__global__ void __launch_bounds__(1024) head_order_kernel(const long long* __restrict__ targets,
                                                          int n, int n_labelled,
                                                          long long* __restrict__ src,
                                                          long long* __restrict__ dest) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int r = base + static_cast<int>(threadIdx.x);
    const int f = (r < n && targets[r] >= 0) ? 1 : 0;
    int x = f;  // inclusive count within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;  // inclusive over the warps
    }
    __syncthreads();
    const int incl = carry + x + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (r < n) {
      const long long d = f ? incl - 1 : static_cast<long long>(r) - incl + n_labelled;
      if (d >= 0 && d < n) {
        if (dest != nullptr) dest[r] = d;
        src[d] = r;
      } else {
        atomicCAS(&g_device_status, 0, TALM_ERANGE);
      }
    }
    __syncthreads();  // every thread has read `carry` and `warp_sums`
    if (threadIdx.x == 1023) carry = incl;
    __syncthreads();
  }
}

// Rows in src order: out[i] = in[src[i]] (16-byte pieces), targets_out[i] = targets[src[i]].
__global__ void __launch_bounds__(256) head_gather_rows_kernel(
    const uint4* __restrict__ in, long long ld16, int n, int row16,
    const long long* __restrict__ src, const long long* __restrict__ targets,
    uint4* __restrict__ out, long long* __restrict__ targets_out) {
  const long long total = static_cast<long long>(n) * row16;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const long long row = i / row16;
    const int c = static_cast<int>(i - row * row16);
    const long long from = src[row];
    out[i] = in[from * ld16 + c];
    if (c == 0) targets_out[row] = targets[from];
  }
}

// ------------------------------------------------------------------------------------------
// 5. backward: the saved gradient times grad_loss / denom, in the hidden's dtype
// ------------------------------------------------------------------------------------------
template <int OUT>
__device__ __forceinline__ void store_scaled(void* out, long long i, float v) {
  if (OUT == TALM_DTYPE_F16) {
    reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
  } else if (OUT == TALM_DTYPE_BF16) {
    reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<float*>(out)[i] = v;
  }
}

// One thread per 4 consecutive columns of a row (the row length is a multiple of 4 on the
// vector path, checked by the host); any other shape goes one element per thread.
template <int OUT, bool IN_F32, bool VEC4>
__global__ void __launch_bounds__(256) head_scale_grad_kernel(
    const void* __restrict__ grad, long long ld, const float* __restrict__ grad_loss,
    const float* __restrict__ denom, long long n_rows, long long n_cols, void* __restrict__ out) {
  const float d = *denom;
  // fused_head.py:280-287: (grad_loss / denom, then 0 where denom == 0) in fp32
  const float sc = d != 0.0f ? *grad_loss / d : 0.0f;
  const long long per_row = VEC4 ? n_cols / 4 : n_cols;
  const long long n = n_rows * per_row;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const long long r = i / per_row, c = (i - r * per_row) * (VEC4 ? 4 : 1);
    float v[4];
    constexpr int W = VEC4 ? 4 : 1;
    if (IN_F32) {
      const float* src = reinterpret_cast<const float*>(grad) + r * ld + c;
      if (VEC4) {
        const float4 q = *reinterpret_cast<const float4*>(src);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
      } else {
        v[0] = *src;
      }
#pragma unroll
      for (int k = 0; k < W; ++k) v[k] = __half2float(__float2half_rn(v[k]));
    } else {
      const __half* src = reinterpret_cast<const __half*>(grad) + r * ld + c;
      if (VEC4) {
        const uint2 q = *reinterpret_cast<const uint2*>(src);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
      } else {
        v[0] = __half2float(*src);
      }
    }
    const long long o = r * n_cols + c;
#pragma unroll
    for (int k = 0; k < W; ++k) store_scaled<OUT>(out, o + k, v[k] * sc);
  }
}

// ------------------------------------------------------------------------------------------
// vocabulary-parallel merge of shard statistics
// ------------------------------------------------------------------------------------------
// `wait_own` (the peer exchange): first wait until every rank published its statistics into
// this rank's peer buffer (phase 0). The gathered records are read with L2-only loads: under
// the peer exchange other GPUs wrote them while this grid may already run.
__global__ void __launch_bounds__(256) head_merge_shards_kernel(const float* gathered,
                                                                int n_shards, int n_tokens,
                                                                int rank, int n_grad,
                                                                float* __restrict__ out,
                                                                float* __restrict__ acc_scale,
                                                                const uint8_t* wait_own,
                                                                size_t flags_off,
                                                                uint32_t epoch) {
  if (wait_own != nullptr && !peer::cta_wait_phase(wait_own, flags_off, 0, n_shards, epoch))
    return;
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n_tokens) return;
  float M = -INFINITY, R = -INFINITY, bv = -INFINITY, zt = 0.0f, hit = 0.0f;
  int bi = 0x7fffffff;
  for (int r = 0; r < n_shards; ++r) {
    const float4* st4 = reinterpret_cast<const float4*>(
        gathered + (static_cast<long long>(r) * n_tokens + row) * TALM_HEAD_STATS);
    const float4 a = __ldcg(st4), b = __ldcg(st4 + 1);  // (M, S, T, ZT), (BEST, IDX, HIT, REF)
    M = fmaxf(M, a.x);
    R = fmaxf(R, b.w);
    better_arg(bv, bi, b.x, __float_as_int(b.y));
    if (b.z != 0.0f) { zt = a.w; hit = 1.0f; }
  }
  float S = 0.0f, T = 0.0f, mine = 0.0f;
  for (int r = 0; r < n_shards; ++r) {
    const float4* st4 = reinterpret_cast<const float4*>(
        gathered + (static_cast<long long>(r) * n_tokens + row) * TALM_HEAD_STATS);
    const float4 a = __ldcg(st4), b = __ldcg(st4 + 1);
    const float w = ex2((b.w - R) * kLog2e);
    S = fmaf(a.y, w, S);
    T = fmaf(a.z, w, T);
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
// Probability buffers come in pairs: the slice step that runs the accumulator GEMM of slice k
// reads buffer k % 2 while its logits GEMM of slice k + 1 writes the other one.
struct Workspace {
  __half* probs[2];      // [n_grad][chunk] each
  float4* partial;       // [n_tokens][chunk / EPI_COLS]
  size_t bytes;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline int64_t chunk_cols(int64_t vocab_cols, int64_t vocab_chunk) {
  int64_t c = vocab_chunk < 1 ? 1 : vocab_chunk;
  if (c > vocab_cols) c = vocab_cols;
  c = (c + BN - 1) / BN * BN;  // whole tiles
  return c < BN ? BN : c;
}

// Width of the first slice. Every row's reference REF is set from the first slice, which has
// no reference to work against: its probabilities are taken relative to each 128-column part's
// own max and rescaled in place by the combine kernel (read + write of the slice's fp16
// probability rows). A narrow first slice keeps that pass small (2048 columns of 16384 rows:
// 67 MB, L2-resident); the later slices then run against REF and move it only when a row's
// max outgrows REF + kRefSlack.
constexpr int64_t kFirstSliceCols = 2048;

// The slices of a walk over `vocab_cols` columns: a first slice of at most kFirstSliceCols,
// then the rest in equal slices of whole tiles, none wider than `chunk` (no narrow tail slice).
struct Slices {
  int64_t first, width, count;
  int64_t begin(int64_t k) const { return k == 0 ? 0 : first + (k - 1) * width; }
};

inline Slices slices_of(int64_t vocab_cols, int64_t chunk) {
  Slices s;
  s.first = std::min<int64_t>(std::min<int64_t>(kFirstSliceCols, chunk), vocab_cols);
  s.first = (s.first + BN - 1) / BN * BN;
  const int64_t rest = vocab_cols > s.first ? vocab_cols - s.first : 0;
  const int64_t n_rest = (rest + chunk - 1) / chunk;
  s.width = n_rest > 0 ? ((rest + n_rest - 1) / n_rest + BN - 1) / BN * BN : chunk;
  s.count = 1 + n_rest;
  return s;
}

Workspace layout(int64_t n_tokens, int64_t n_grad, int64_t vocab_cols, int64_t vocab_chunk,
                 uint8_t* base) {
  const int64_t chunk = chunk_cols(vocab_cols, vocab_chunk);
  const int64_t tiles = chunk / BN * PARTS;  // statistics records per row and slice
  const int64_t n_slices = slices_of(vocab_cols, chunk).count;
  const int n_buf = n_slices > 1 ? 2 : 1;
  Workspace w;
  size_t off = 0;
  for (int b = 0; b < 2; ++b) {
    w.probs[b] = reinterpret_cast<__half*>(base + off);
    if (b < n_buf) off = align_up(off + static_cast<size_t>(n_grad) * chunk * 2, 256);
  }
  w.partial = reinterpret_cast<float4*>(base + off);
  off = align_up(off + static_cast<size_t>(n_tokens) * tiles * 16, 256);
  w.bytes = off + 256;  // slack for base alignment
  return w;
}

// The shared-memory opt-in of a kernel is a property of the kernel on one device: it is set
// once per device (the current one at the call), under a lock.
std::mutex g_attr_mutex;
bool g_attrs_set[kMaxDevices] = {};

int set_attrs() {
  int dev = 0;
  int st = current_device(&dev);
  if (st != TALM_OK) return st;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (g_attrs_set[dev]) return TALM_OK;
  const cudaError_t e = cudaFuncSetAttribute(
      head_slice_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return set_error(TALM_ECUDA, "smem attribute: %s", cudaGetErrorString(e));
  g_attrs_set[dev] = true;
  return TALM_OK;
}

// Launch one slice step: clusters of 2 CTAs, at most one pair per 2 SMs, with programmatic
// dependent launch (the launch and the kernel's set-up overlap the previous kernel).
int launch_slice_step(const CUtensorMap& tm_hidden, const CUtensorMap& tm_weight,
                      const CUtensorMap& tm_probs_out, const CUtensorMap& tm_probs_in,
                      const CUtensorMap& tm_weight_mn, const CUtensorMap& tm_acc,
                      const CUtensorMap& tm_hidden3, const CUtensorMap& tm_weight3,
                      const CUtensorMap& tm_probs3_in, const SliceParams& sp,
                      cudaStream_t stream, int max_pairs) {
  // one pair per tile at most
  const long long want = static_cast<long long>(sp.n_tiles_l) + sp.n_tiles_a;
  const int pairs = static_cast<int>(std::max(1LL, std::min<long long>(want, max_pairs)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(SLICE_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, head_slice_kernel, tm_hidden, tm_weight,
                                           tm_probs_out, tm_probs_in, tm_weight_mn, tm_acc,
                                           tm_hidden3, tm_weight3, tm_probs3_in, sp);
  if (e != cudaSuccess) return set_error(TALM_ECUDA, "slice kernel launch: %s", cudaGetErrorString(e));
  return TALM_OK;
}

// Pairs that fit on the GPU at once (one CTA per SM: shared memory and TMEM are taken whole).
int max_pairs_of(int sms) { return sms / 2 > 0 ? sms / 2 : 1; }

// Which steps of a walk one call runs: all of them; all but the last (accumulator-only) step,
// whose accumulator GEMM talm_head_shard_finish_scatter then runs with the scatter epilogue
// once the statistics are merged; or only that last step.
enum WalkPart { WALK_ALL, WALK_BEGIN, WALK_LAST };

// The vocabulary walk over weight rows [0, vocab_cols) of `weight` (global columns vocab_col0..):
// step k < n_slices runs the logits GEMM of slice k together with the accumulator GEMM of slice
// k - 1, then the combine of slice k; step n_slices runs the accumulator GEMM of the last
// slice. `sc` (WALK_LAST only) turns that last accumulator GEMM into the scatter step.
int shard_walk(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
               int64_t ld_weight, const int64_t* targets, int64_t n_tokens, int64_t n_grad,
               int64_t hidden_size, int64_t vocab_cols, int64_t vocab_col0, int64_t vocab_chunk,
               float* stats, float* acc, void* workspace, size_t ws_bytes, cudaStream_t stream,
               WalkPart part, const ScatterParams* sc) {
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  if (hidden_size < 8 || hidden_size % 8 != 0 || ld_hidden % 8 != 0 || ld_weight % 8 != 0 ||
      ld_hidden < hidden_size || ld_weight < hidden_size)
    return set_error(TALM_EINVAL, "hidden size and row strides must be multiples of 8 elements");
  if (vocab_cols < 1 || vocab_col0 < 0) return set_error(TALM_EINVAL, "empty vocabulary range");
  if (n_tokens >= (int64_t{1} << 30) || vocab_cols >= (int64_t{1} << 31) ||
      hidden_size >= (int64_t{1} << 20))
    return set_error(TALM_ERANGE, "sizes beyond the kernels' 32-bit tile indices");
  if (n_tokens == 0 || (part == WALK_LAST && n_grad == 0)) return TALM_OK;
  const bool logits_steps = part != WALK_LAST;
  if ((logits_steps && !hidden) || !weight || !targets || !stats || (n_grad > 0 && !acc) ||
      !workspace)
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
  st = TALM_OK;
  if (logits_steps) {
    st = talm_make_tmap_2d_f16(&tm_hidden, hidden, hidden_size, n_tokens, ld_hidden, BK, BM);
    if (st == TALM_OK)
      st = talm_make_tmap_2d_f16(&tm_weight, weight, hidden_size, vocab_cols, ld_weight, BK,
                                 BN / 2);
  }
  if (st == TALM_OK && n_grad > 0)
    st = talm_make_tmap_2d_f16(&tm_weight_mn, weight, hidden_size, vocab_cols, ld_weight, 64, BK);
  if (st != TALM_OK) return st;
  if (!logits_steps) tm_hidden = tm_weight = tm_weight_mn;  // unused by an accumulator step
  // 3-D k-chunk maps (two 64-column chunks per request) where the hidden size is a multiple
  // of 64; the weight map serves the logits tiles (rows = vocabulary rows, chunks along K =
  // hidden) and the accumulator tiles (rows = K, chunks = hidden column groups) alike
  const int k3d = hidden_size % 64 == 0 ? 1 : 0;
  CUtensorMap tm_hidden3 = tm_hidden, tm_weight3 = tm_hidden;
  if (k3d) {
    if (logits_steps)
      st = talm_make_tmap_kchunks_f16(&tm_hidden3, hidden, hidden_size, n_tokens, ld_hidden, BM);
    if (st == TALM_OK)
      st = talm_make_tmap_kchunks_f16(&tm_weight3, weight, hidden_size, vocab_cols, ld_weight,
                                      BN / 2);
    if (st != TALM_OK) return st;
  }
  CUtensorMap tm_acc = tm_hidden;
  if (n_grad > 0 && (st = talm_make_tmap_2d_f32(&tm_acc, acc, hidden_size, n_grad, hidden_size,
                                                32, BM)) != TALM_OK)
    return st;

  const Slices sl = slices_of(vocab_cols, chunk);
  const int64_t n_slices = sl.count;
  const int64_t k_first = part == WALK_LAST ? n_slices : 0;
  const int64_t k_last = part == WALK_BEGIN ? n_slices - 1 : n_slices;

  if (k_first == 0) {
    if (cudaMemsetAsync(stats, 0, sizeof(float) * TALM_HEAD_STATS * n_tokens, stream) !=
        cudaSuccess)
      return check_launch("stats memset");
    // every accumulator GEMM adds into acc (TMA reduce-add): it starts at zero
    if (n_grad > 0 &&
        cudaMemsetAsync(acc, 0, sizeof(float) * n_grad * hidden_size, stream) != cudaSuccess)
      return check_launch("acc memset");
  }

  const int k_blocks = static_cast<int>((hidden_size + BK - 1) / BK);
  const int n_pair_rows = static_cast<int>((n_tokens + PAIR_ROWS - 1) / PAIR_ROWS);
  const int max_pairs = max_pairs_of(sms);
  // The slices' probability buffers alternate: step k writes buffer k % 2 while its
  // accumulator part reads buffer (k - 1) % 2. The combine of slice k follows the accumulator
  // GEMM of slice k - 1 (its acc rescale needs that) and precedes the one of slice k (which
  // reads the rows it rescales). Steps before k_first are only planned, not launched.
  AccumParams prev_ap{};
  CUtensorMap prev_tm_probs = tm_hidden, prev_tm_probs3 = tm_hidden;
  for (int64_t k = 0; k <= k_last; ++k) {
    const bool run = k >= k_first;
    SliceParams sp{};
    sp.n_tiles_l = 0;
    sp.n_tiles_a = 0;
    CUtensorMap tm_probs_out = tm_hidden;  // unused when no probabilities are stored
    CUtensorMap tm_probs3 = tm_hidden;     // the same buffer as k chunks, read next step
    int n_col_tiles = 0;
    const int buf = static_cast<int>(k & 1);
    const int64_t s0 = k < n_slices ? sl.begin(k) : 0;
    if (k < n_slices) {
      const int64_t s1 = std::min<int64_t>(vocab_cols, k == 0 ? sl.first : s0 + sl.width);
      const int cols = static_cast<int>(s1 - s0);
      n_col_tiles = (cols + BN - 1) / BN;
      LogitsParams& lp = sp.lg;
      lp.n_tokens = static_cast<int>(n_tokens);
      lp.n_grad = static_cast<int>(n_grad);
      lp.k_blocks = k_blocks;
      lp.slice_row0 = static_cast<int>(s0);
      lp.cols = cols;
      lp.n_col_tiles = n_col_tiles;
      lp.n_parts = n_col_tiles * PARTS;
      lp.n_pair_rows = n_pair_rows;
      lp.band_rows = std::min(n_pair_rows, kBandRows);
      lp.k3d = k3d;
      lp.col_base = vocab_col0 + s0;
      lp.has_ref = k != 0;
      lp.targets = reinterpret_cast<const long long*>(targets);
      lp.partial = ws.partial;
      lp.stats = stats;
      sp.n_tiles_l = n_pair_rows * n_col_tiles;
      if (n_grad > 0 && (st = talm_make_tmap_2d_f16(&tm_probs_out, ws.probs[buf], chunk, n_grad,
                                                    chunk, 64, BM)) != TALM_OK)
        return st;
      if (n_grad > 0 && k3d &&
          (st = talm_make_tmap_kchunks_f16(&tm_probs3, ws.probs[buf], chunk, n_grad, chunk,
                                           BM)) != TALM_OK)
        return st;
    }
    if (k >= 1 && n_grad > 0) {
      sp.ac = prev_ap;
      sp.n_tiles_a = prev_ap.n_pair_rows * prev_ap.n_h_tiles;
    }
    if (k == n_slices && sc != nullptr) sp.sc = *sc;
    if (run && sp.n_tiles_l + sp.n_tiles_a > 0) {
      LaunchTimer timer(TALM_KERNEL_HEAD_SLICE, stream);
      st = launch_slice_step(tm_hidden, tm_weight, tm_probs_out, prev_tm_probs, tm_weight_mn,
                             tm_acc, tm_hidden3, tm_weight3, prev_tm_probs3, sp, stream,
                             max_pairs);
      if (st != TALM_OK) return st;
    }
    if (k == n_slices) break;
    if (run) {
      LaunchTimer timer(TALM_KERNEL_HEAD_COMBINE, stream);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>((n_tokens + 7) / 8), 1, 1);
      cfg.blockDim = dim3(256, 1, 1);
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      const cudaError_t e = cudaLaunchKernelEx(
          &cfg, head_combine_kernel, static_cast<const float4*>(ws.partial),
          static_cast<int>(n_col_tiles * PARTS), static_cast<int>(n_tokens),
          static_cast<int>(n_grad), static_cast<int>(k == 0), stats,
          n_grad > 0 ? ws.probs[buf] : static_cast<__half*>(nullptr), static_cast<int>(chunk),
          n_grad > 0 ? acc : static_cast<float*>(nullptr), static_cast<int>(hidden_size));
      if (e != cudaSuccess)
        return set_error(TALM_ECUDA, "head combine launch: %s", cudaGetErrorString(e));
    }
    // the accumulator GEMM of this slice runs in the next step
    prev_ap.n_grad = static_cast<int>(n_grad);
    prev_ap.hidden = static_cast<int>(hidden_size);
    prev_ap.k_blocks = n_col_tiles * (BN / BK);
    prev_ap.slice_row0 = static_cast<int>(s0);
    prev_ap.n_pair_rows = static_cast<int>((n_grad + PAIR_ROWS - 1) / PAIR_ROWS);
    prev_ap.n_h_tiles = static_cast<int>((hidden_size + BN - 1) / BN);
    prev_ap.k3d = k3d;
    prev_tm_probs = tm_probs_out;
    prev_tm_probs3 = tm_probs3;
  }
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
                    size_t ws_bytes, void* stream) {
  return talm::head::shard_walk(hidden, ld_hidden, weight, ld_weight, targets, n_tokens, n_grad,
                                hidden_size, vocab_cols, vocab_col0, vocab_chunk, stats, acc,
                                workspace, ws_bytes, static_cast<cudaStream_t>(stream),
                                talm::head::WALK_ALL, nullptr);
}

int talm_head_shard_begin(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                          int64_t ld_weight, const int64_t* targets, int64_t n_tokens,
                          int64_t n_grad, int64_t hidden_size, int64_t vocab_cols,
                          int64_t vocab_col0, int64_t vocab_chunk, float* stats, float* acc,
                          void* workspace, size_t ws_bytes, void* stream) {
  return talm::head::shard_walk(hidden, ld_hidden, weight, ld_weight, targets, n_tokens, n_grad,
                                hidden_size, vocab_cols, vocab_col0, vocab_chunk, stats, acc,
                                workspace, ws_bytes, static_cast<cudaStream_t>(stream),
                                talm::head::WALK_BEGIN, nullptr);
}

int talm_head_shard_finish_scatter(const uint16_t* weight, int64_t ld_weight,
                                   const int64_t* targets, int64_t n_tokens, int64_t n_grad,
                                   int64_t hidden_size, int64_t vocab_cols, int64_t vocab_col0,
                                   int64_t vocab_chunk, const float* stats, float* acc,
                                   const float* acc_scale, void* workspace, size_t ws_bytes,
                                   const int64_t* grad_rows, float* token_loss,
                                   float* token_entropy, int32_t* correct, int64_t rank,
                                   int64_t world, const uint64_t* peers, uint32_t epoch,
                                   void* stream) {
  using namespace talm;
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  int st = peer::check_peer_args(world, rank, n_tokens, hidden_size);
  if (st != TALM_OK) return st;
  if (n_grad == 0)  // no accumulator: the finalize kernel ends phase 1 itself
    return talm_head_finalize_scatter(stats, targets, n_tokens, 0, nullptr, nullptr, weight,
                                      ld_weight, vocab_col0, vocab_cols, hidden_size,
                                      grad_rows, token_loss, token_entropy, correct, rank,
                                      world, peers, epoch, stream);
  if (!peers || !stats || !targets || !acc || !acc_scale || !weight)
    return set_error(TALM_EINVAL, "null pointer");
  if (ld_weight % 4 != 0 || (reinterpret_cast<uintptr_t>(weight) & 7) != 0 ||
      (reinterpret_cast<uintptr_t>(acc) & 15) != 0)
    return set_error(TALM_EINVAL, "acc must be 16-byte and the weight rows 8-byte aligned");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    // the per-row outputs, and zero gradient rows for the rows without one (n_grad and on);
    // the rows below n_grad leave from the scatter step
    LaunchTimer timer(TALM_KERNEL_HEAD_FINALIZE, s);
    head::head_finalize_kernel<<<static_cast<int>((n_tokens + 7) / 8), 256, 0, s>>>(
        stats, reinterpret_cast<const long long*>(targets), static_cast<int>(n_tokens),
        static_cast<int>(n_grad), acc, acc_scale, reinterpret_cast<const __half*>(weight),
        ld_weight, vocab_col0, vocab_cols, static_cast<int>(hidden_size),
        reinterpret_cast<const long long*>(grad_rows), token_loss, token_entropy, correct,
        head::GradDest{nullptr, 1, reinterpret_cast<const unsigned long long*>(peers), L.recv,
                       L.rpr, static_cast<int>(rank), n_grad, 0},
        1, L, static_cast<int>(world), epoch);
    st = check_launch("head finalize kernel (per-row outputs)");
    if (st != TALM_OK) return st;
  }
  head::ScatterParams sc{};
  sc.on = 1;
  // the ranks start on different owners: rank r on the tiles of the rows rank r + 1 owns
  const int64_t n_h_tiles = (hidden_size + head::BN - 1) / head::BN;
  const int64_t n_pair_rows = (n_grad + head::PAIR_ROWS - 1) / head::PAIR_ROWS;
  sc.tile_shift = static_cast<int>(
      ((((rank + 1) % world) * L.rpr / head::PAIR_ROWS) % n_pair_rows) * n_h_tiles);
  sc.acc = acc;
  sc.scale = acc_scale;
  sc.targets = reinterpret_cast<const long long*>(targets);
  sc.grad_rows = reinterpret_cast<const long long*>(grad_rows);
  sc.weight = reinterpret_cast<const __half*>(weight);
  sc.ld_weight = ld_weight;
  sc.col0 = vocab_col0;
  sc.vcols = vocab_cols;
  sc.peers = reinterpret_cast<const unsigned long long*>(peers);
  sc.L = L;
  sc.rank = static_cast<int>(rank);
  sc.world = static_cast<int>(world);
  sc.epoch = epoch;
  return head::shard_walk(nullptr, hidden_size, weight, ld_weight, targets, n_tokens, n_grad,
                          hidden_size, vocab_cols, vocab_col0, vocab_chunk,
                          const_cast<float*>(stats), acc, workspace, ws_bytes, s,
                          head::WALK_LAST, &sc);
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
  // 4 columns per lane when every row of acc, grad and weight starts on the needed boundary
  auto aligned = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
  const int vec4 = hidden_size % 4 == 0 && ld_weight % 4 == 0 && aligned(acc, 16) &&
                   aligned(weight, 8) && aligned(grad, grad_is_f32 ? 16 : 8);
  LaunchTimer timer(TALM_KERNEL_HEAD_FINALIZE, static_cast<cudaStream_t>(stream));
  head::head_finalize_kernel<<<static_cast<int>((n_tokens + 7) / 8), 256, 0,
                               static_cast<cudaStream_t>(stream)>>>(
      stats, reinterpret_cast<const long long*>(targets), static_cast<int>(n_tokens),
      static_cast<int>(n_grad), acc, acc_scale, reinterpret_cast<const __half*>(weight),
      ld_weight, vocab_col0, vocab_cols, static_cast<int>(hidden_size),
      reinterpret_cast<const long long*>(grad_rows), token_loss, token_entropy, correct,
      head::GradDest{grad, grad_is_f32, nullptr, 0, 1, 0}, vec4, peer::PeerLayout{}, 1, 0u);
  return check_launch("head finalize kernel");
}

int talm_head_finalize_scatter(const float* stats, const int64_t* targets, int64_t n_tokens,
                               int64_t n_grad, const float* acc, const float* acc_scale,
                               const uint16_t* weight, int64_t ld_weight, int64_t vocab_col0,
                               int64_t vocab_cols, int64_t hidden_size,
                               const int64_t* grad_rows, float* token_loss,
                               float* token_entropy, int32_t* correct, int64_t rank,
                               int64_t world, const uint64_t* peers, uint32_t epoch,
                               void* stream) {
  using namespace talm;
  if (n_tokens < 0 || n_grad < 0 || n_grad > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  int st = peer::check_peer_args(world, rank, n_tokens, hidden_size);
  if (st != TALM_OK) return st;
  if (!peers || (n_tokens > 0 && (!stats || !targets)) ||
      (n_grad > 0 && (!acc || !acc_scale || !weight)))
    return set_error(TALM_EINVAL, "null pointer");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden_size);
  auto aligned = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
  const int vec4 = ld_weight % 4 == 0 && aligned(acc, 16) && aligned(weight, 8);
  // every CTA takes part in the phase signal, so the grid is never empty
  const int grid = static_cast<int>(n_tokens > 0 ? (n_tokens + 7) / 8 : 1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchTimer timer(TALM_KERNEL_HEAD_FINALIZE, s);
  head::head_finalize_kernel<<<grid, 256, 0, s>>>(
      stats, reinterpret_cast<const long long*>(targets), static_cast<int>(n_tokens),
      static_cast<int>(n_grad), acc, acc_scale, reinterpret_cast<const __half*>(weight),
      ld_weight, vocab_col0, vocab_cols, static_cast<int>(hidden_size),
      reinterpret_cast<const long long*>(grad_rows), token_loss, token_entropy, correct,
      head::GradDest{nullptr, 1, reinterpret_cast<const unsigned long long*>(peers), L.recv,
                     L.rpr, static_cast<int>(rank), 0, 1},
      vec4, L, static_cast<int>(world), epoch);
  return check_launch("head finalize scatter kernel");
}

int talm_head_scale_grad(const void* grad, int64_t ld_grad, int grad_is_f32,
                         const float* grad_loss, const float* denom, int64_t n_rows,
                         int64_t n_cols, void* out, int out_dtype, void* stream) {
  using namespace talm;
  if (n_rows < 0 || n_cols < 0 || ld_grad < n_cols)
    return set_error(TALM_EINVAL, "need n_rows, n_cols >= 0 and ld_grad >= n_cols");
  if (out_dtype < TALM_DTYPE_F16 || out_dtype > TALM_DTYPE_F32)
    return set_error(TALM_EINVAL, "out_dtype must be TALM_DTYPE_F16, _BF16 or _F32");
  if (n_rows == 0 || n_cols == 0) return TALM_OK;
  if (!grad || !grad_loss || !denom || !out) return set_error(TALM_EINVAL, "null pointer");
  const int in_bytes = grad_is_f32 ? 4 : 2, out_bytes = out_dtype == TALM_DTYPE_F32 ? 4 : 2;
  auto aligned = [](const void* q, uintptr_t a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
  const bool vec4 = n_cols % 4 == 0 && ld_grad % 4 == 0 && aligned(grad, 4 * in_bytes) &&
                    aligned(out, 4 * out_bytes);
  const long long items = n_rows * (vec4 ? n_cols / 4 : n_cols);
  const int sms = current_sm_count();
  if (sms <= 0) return set_error(TALM_ENODEV, "no CUDA device");
  const long long want = (items + 255) / 256;
  const int grid = static_cast<int>(want < int64_t{sms} * 8 ? want : int64_t{sms} * 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchTimer timer(TALM_KERNEL_HEAD_SCALE, s);
#define TALM_SCALE_LAUNCH(OUT, F32, V)                                                        \
  head::head_scale_grad_kernel<OUT, F32, V><<<grid, 256, 0, s>>>(grad, ld_grad, grad_loss, \
                                                                 denom, n_rows, n_cols, out)
#define TALM_SCALE_BY_INPUT(OUT)                                          \
  do {                                                                    \
    if (grad_is_f32) {                                                    \
      if (vec4) TALM_SCALE_LAUNCH(OUT, true, true); else TALM_SCALE_LAUNCH(OUT, true, false);   \
    } else {                                                              \
      if (vec4) TALM_SCALE_LAUNCH(OUT, false, true); else TALM_SCALE_LAUNCH(OUT, false, false); \
    }                                                                     \
  } while (0)
  if (out_dtype == TALM_DTYPE_F16) {
    TALM_SCALE_BY_INPUT(TALM_DTYPE_F16);
  } else if (out_dtype == TALM_DTYPE_BF16) {
    TALM_SCALE_BY_INPUT(TALM_DTYPE_BF16);
  } else {
    TALM_SCALE_BY_INPUT(TALM_DTYPE_F32);
  }
#undef TALM_SCALE_BY_INPUT
#undef TALM_SCALE_LAUNCH
  return check_launch("head scale kernel");
}

int talm_head_labelled_first(const int64_t* targets, int64_t n_tokens, int64_t n_labelled,
                             const uint16_t* hidden, int64_t ld_hidden, int64_t cols,
                             int64_t* src, int64_t* dest, uint16_t* hidden_out,
                             int64_t* targets_out, void* stream) {
  using namespace talm;
  if (n_tokens < 0 || n_labelled < 0 || n_labelled > n_tokens)
    return set_error(TALM_EINVAL, "need 0 <= n_labelled <= n_tokens");
  if (n_tokens >= (int64_t{1} << 31)) return set_error(TALM_ERANGE, "n_tokens beyond 2^31");
  if (n_tokens == 0) return TALM_OK;
  if (!targets || !src) return set_error(TALM_EINVAL, "null pointer");
  const bool rows = hidden_out != nullptr;
  if (rows) {
    if (!hidden || !targets_out) return set_error(TALM_EINVAL, "null pointer");
    if (cols < 8 || cols % 8 != 0 || ld_hidden % 8 != 0 || ld_hidden < cols ||
        (reinterpret_cast<uintptr_t>(hidden) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(hidden_out) & 15) != 0)
      return set_error(TALM_EINVAL, "hidden rows must be 16-byte aligned multiples of 8 columns");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  head::head_order_kernel<<<1, 1024, 0, s>>>(reinterpret_cast<const long long*>(targets),
                                             static_cast<int>(n_tokens),
                                             static_cast<int>(n_labelled),
                                             reinterpret_cast<long long*>(src),
                                             reinterpret_cast<long long*>(dest));
  int st = check_launch("head order kernel");
  if (st != TALM_OK || !rows) return st;
  const int row16 = static_cast<int>(cols / 8);
  const long long items = n_tokens * row16;
  const int sms = current_sm_count();
  if (sms <= 0) return set_error(TALM_ENODEV, "no CUDA device");
  const long long want = (items + 255) / 256;
  const int grid = static_cast<int>(want < int64_t{sms} * 8 ? want : int64_t{sms} * 8);
  head::head_gather_rows_kernel<<<grid, 256, 0, s>>>(
      reinterpret_cast<const uint4*>(hidden), ld_hidden / 8, static_cast<int>(n_tokens), row16,
      reinterpret_cast<const long long*>(src), reinterpret_cast<const long long*>(targets),
      reinterpret_cast<uint4*>(hidden_out), reinterpret_cast<long long*>(targets_out));
  return check_launch("head gather rows kernel");
}

int talm_head_combine(const float* gathered, int64_t n_shards, int64_t n_tokens, int64_t rank,
                      int64_t n_grad, float* stats_out, float* acc_scale, void* stream) {
  using namespace talm;
  if (n_shards < 1 || rank < 0 || rank >= n_shards || n_tokens < 0 || n_grad < 0 ||
      n_grad > n_tokens)
    return set_error(TALM_EINVAL, "bad shard arguments");
  if (n_tokens == 0) return TALM_OK;
  if (!gathered || !stats_out) return set_error(TALM_EINVAL, "null pointer");
  if ((reinterpret_cast<uintptr_t>(gathered) & 15) != 0)
    return set_error(TALM_EINVAL, "gathered statistics must be 16-byte aligned");
  LaunchTimer timer(TALM_KERNEL_HEAD_MERGE, static_cast<cudaStream_t>(stream));
  head::head_merge_shards_kernel<<<static_cast<int>((n_tokens + 255) / 256), 256, 0,
                                   static_cast<cudaStream_t>(stream)>>>(
      gathered, static_cast<int>(n_shards), static_cast<int>(n_tokens), static_cast<int>(rank),
      static_cast<int>(n_grad), stats_out, acc_scale, nullptr, 0, 0u);
  return check_launch("head merge kernel");
}

int talm_head_merge_peers(int64_t n_tokens, int64_t hidden, int64_t rank, int64_t world,
                          int64_t n_grad, const void* own_buffer, uint32_t epoch,
                          float* stats_out, float* acc_scale, void* stream) {
  using namespace talm;
  int st = peer::check_peer_args(world, rank, n_tokens, hidden);
  if (st != TALM_OK) return st;
  if (n_grad < 0 || n_grad > n_tokens) return set_error(TALM_EINVAL, "need 0 <= n_grad <= n_tokens");
  if (n_tokens == 0) return TALM_OK;
  if (!own_buffer || !stats_out || (n_grad > 0 && !acc_scale))
    return set_error(TALM_EINVAL, "null pointer");
  const peer::PeerLayout L = peer::peer_layout(world, n_tokens, hidden);
  const uint8_t* own = static_cast<const uint8_t*>(own_buffer);
  LaunchTimer timer(TALM_KERNEL_HEAD_MERGE, static_cast<cudaStream_t>(stream));
  head::head_merge_shards_kernel<<<static_cast<int>((n_tokens + 255) / 256), 256, 0,
                                   static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float*>(own + L.stats), static_cast<int>(world),
      static_cast<int>(n_tokens), static_cast<int>(rank), static_cast<int>(n_grad), stats_out,
      acc_scale, own, L.flags, epoch);
  return check_launch("head merge peers kernel");
}

}  // extern "C"
