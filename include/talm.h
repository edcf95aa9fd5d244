/*
 * talm.h - C ABI of libtalm_b200.so, the sm_100a kernels behind the two hot paths of
 * otarernazar-eng/Talm's QLoRA step:
 *
 *   (1) the vocabulary-sliced fused LM head + cross-entropy (reference: solution/fused_head.py)
 *   (2) the grouped / per-projection NF4 dequantisation (reference: solution/qgroup.py,
 *       solution/nf4_dequant.py)
 *
 * Conventions shared by every entry point:
 *   - plain pointers to device memory and sizes; no framework types;
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream);
 *   - every call is asynchronous on `stream`: it validates its arguments on the host,
 *     enqueues its kernels and returns; it never synchronises, never allocates device memory
 *     (the caller passes any workspace) and keeps no pointer after it returns;
 *   - the return value is a TALM_* status; 0 means the work was enqueued. talm_last_error()
 *     gives a one-line reason for the last non-zero status on the calling thread.
 *   - fp16 tensors are passed as uint16_t* (IEEE binary16 bit patterns).
 */
#ifndef TALM_H_
#define TALM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TALM_OK 0
#define TALM_EINVAL 1   /* an argument violates a documented precondition */
#define TALM_ECUDA 2    /* a CUDA runtime call or kernel launch failed */
#define TALM_ERANGE 3   /* a size beyond what the kernels support */
#define TALM_ENODEV 4   /* no sm_100 device is current */
#define TALM_ETIMEOUT 5 /* a device-side wait gave up (read back by talm_device_status) */

/* ABI version of this header (bumped on any signature change). */
int talm_abi_version(void);

/* One-line reason for the last non-zero status returned on this thread ("" if none). */
const char* talm_last_error(void);

/* Human-readable name of a status code. */
const char* talm_status_string(int status);

/* Reads and clears the device-side status word that kernels with bounded waits set when a
 * wait gives up (TALM_OK when nothing was recorded). Synchronises the current device. No
 * reference counterpart: the reference's Triton kernels have no device-side waits. */
int talm_device_status(int* status_out);

/* Sets how long every bounded device-side wait of this library (pipeline barriers, the peer
 * exchange's phase flags) spins before it gives up with TALM_ETIMEOUT, on the current device;
 * 0 restores the default of 2 s. Synchronous (a copy to device memory): call it between
 * launches, not while kernels of this library run. For tests that make a wait run out on
 * purpose without a fault. No reference counterpart (the reference has no device-side waits). */
int talm_set_wait_limit_ns(uint64_t limit_ns);

/* Kernel-level timing (the counterpart of the reference's Triton launch timer,
 * harness/_train.py:44-85): between talm_profile_begin and talm_profile_end every kernel this
 * library launches is bracketed by CUDA events on its own stream. talm_profile_end synchronises
 * on those events and returns, per kernel kind, the summed device milliseconds and the launch
 * count (arrays of n_kinds entries, n_kinds <= TALM_KERNEL_KINDS). Off by default; when off the
 * launches carry no events. Not thread-safe: profile from one host thread. */
#define TALM_KERNEL_HEAD_SLICE 0    /* head_slice_kernel (tcgen05 logits GEMM of a slice + stats,
                                       with the accumulator GEMM of the slice before)    */
#define TALM_KERNEL_HEAD_COMBINE 1  /* head_combine_kernel  (per-slice merge)             */
#define TALM_KERNEL_HEAD_RESERVED 2 /* unused (the accumulator GEMM is part of HEAD_SLICE) */
#define TALM_KERNEL_HEAD_FINALIZE 3 /* head_finalize_kernel                               */
#define TALM_KERNEL_HEAD_MERGE 4    /* head_merge_shards_kernel                           */
#define TALM_KERNEL_NF4 5           /* nf4 bulk-copy and chunk kernels (main body)        */
#define TALM_KERNEL_NF4_TAIL 6      /* nf4 byte kernel (tails, unaligned pointers)        */
#define TALM_KERNEL_HEAD_SCALE 7    /* head_scale_grad_kernel (backward scaling)          */
#define TALM_KERNEL_PEER_PUBLISH 8  /* publish_stats_kernel (peer exchange, phase 0)      */
#define TALM_KERNEL_PEER_REDUCE 9   /* reduce_gather_kernel (peer exchange, phase 2)      */
#define TALM_KERNEL_PEER_FINISH 10  /* gather_finish_kernel (wait + copy out)             */
#define TALM_KERNEL_NF4_GEMM 11     /* nf4_gemm_kernel (fused NF4 dequant + tcgen05 GEMM)  */
#define TALM_KERNEL_KINDS 12
int talm_profile_begin(void);
int talm_profile_end(double* ms_out, int64_t* launches_out, int n_kinds);

/* ------------------------------------------------------------------------------------------
 * NF4 dequantisation
 * ---------------------------------------------------------------------------------------- */

/* Per-projection NF4 -> fp16 with an fp32 absmax per block.
 * Replaces: solution/nf4_dequant.py:83-91 `nf4_dequantize(packed, absmax, blocksize, out)`
 * (kernel `nf4_dequant_pairs_kernel`, nf4_dequant.py:38-80).
 *   packed   : n_elems/2 bytes; byte i holds element 2i in its high nibble, 2i+1 in its low one
 *   absmax   : ceil(n_elems / blocksize) fp32 scales
 *   out      : n_elems fp16, out[e] = fp16(NF4[code(e)] * absmax[e / blocksize]) (fp32 product,
 *              one round-to-nearest-even to fp16)
 * Preconditions: n_elems even and >= 0, blocksize even and >= 2. Any alignment is accepted;
 * the fast path needs packed 4-byte and out 16-byte aligned. */
int talm_nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n_elems,
                        int64_t blocksize, uint16_t* out, void* stream);

/* Grouped NF4 -> fp16 over a layer's packed buffers with double-quantised absmax: one launch
 * for the seven projections of a decoder layer.
 * Replaces: solution/qgroup.py:94-99 `launch(packed, absmax8, code, absmax2, offset2, levels,
 * out, n_rows, qblock, qblock2)` (kernel `nf4_group_dequant_kernel`, qgroup.py:72-91).
 *   row r (one absmax block of qblock weights) has the scale
 *     scale[r] = fp32(fp32(code[absmax8[r]] * absmax2[r / qblock2]) + offset2[r / qblock2])
 *   (two separate roundings, no fused multiply-add), and
 *     out[r*qblock + 2j]   = fp16(levels[packed[r*qblock/2 + j] >> 4] * scale[r])
 *     out[r*qblock + 2j+1] = fp16(levels[packed[r*qblock/2 + j] & 15] * scale[r])
 *   packed : n_rows*qblock/2 bytes     absmax8 : n_rows bytes        code : 256 fp32
 *   absmax2, offset2 : ceil(n_rows / qblock2) fp32                  levels : 16 fp32
 * Preconditions: qblock even, qblock/2 a power of two, n_rows*qblock/2 < 2^31, qblock2 >= 1. */
int talm_nf4_group_dequant(const uint8_t* packed, const uint8_t* absmax8, const float* code,
                           const float* absmax2, const float* offset2, const float* levels,
                           uint16_t* out, int64_t n_rows, int64_t qblock, int64_t qblock2,
                           void* stream);

/* Fused NF4 dequantisation + GEMM (tcgen05): the product of an fp16 activation with R
 * consecutive 4-bit weight rows of a layer group, the weights rebuilt in shared memory exactly
 * as talm_nf4_group_dequant rebuilds them, never written to HBM. Replaces the grouped path's
 * dequant launch + cuBLAS product (solution/qgroup.py:346-355, GroupLinear):
 *   transpose = 0: y[n_rows, w_rows] = a[n_rows, w_cols] . W^T (+ bias[w_rows])   (forward)
 *   transpose = 1: y[n_rows, w_cols] = a[n_rows, w_rows] . W  (input gradient; bias NULL)
 *   a, y    : fp16 rows, strides ld_a, ld_y elements (multiples of 8, 16-byte aligned bases)
 *   packed  : w_rows * w_cols / 2 bytes, row-major (16-byte aligned)
 *   absmax8 : w_rows * w_cols / 64 coded scales of this weight (qblock 64)
 *   absmax2, offset2 : the group's second-level arrays, indexed by
 *             (absmax_row0 + absmax index within this weight) / qblock2
 *   code    : 256 fp32         levels : 16 fp32
 * Preconditions: qblock == 64, w_rows % 64 == 0, w_cols % 128 == 0, fp32 accumulation; the
 * output is rounded to fp16 once (after the bias). */
int talm_nf4_linear(const uint16_t* a, int64_t ld_a, int64_t n_rows, const uint8_t* packed,
                    const uint8_t* absmax8, const float* code, const float* absmax2,
                    const float* offset2, const float* levels, int64_t absmax_row0,
                    int64_t w_rows, int64_t w_cols, int64_t qblock, int64_t qblock2,
                    int transpose, const uint16_t* bias, uint16_t* y, int64_t ld_y,
                    void* stream);

/* ------------------------------------------------------------------------------------------
 * Fused LM head + cross-entropy (vocabulary-sliced, no materialised logits)
 * ---------------------------------------------------------------------------------------- */

/* Per-row statistics, one float[TALM_HEAD_STATS] record per token row, relative to the part of
 * the vocabulary a call covered (all of it on one GPU, the rank's shard under vocabulary
 * parallelism). Argmax and the target logit are over fp16-rounded logits, as the reference's
 * cuBLAS fp16 GEMM output (solution/fused_head.py:136-169). The sums S and T and the
 * accumulator are kept relative to a per-row reference REF that trails the running max M by at
 * most 8 (REF <= M <= REF + 8): the reference moves only when the max outgrows it, so most
 * slices need no rescaling of the probabilities or of the accumulator. */
#define TALM_HEAD_STATS 8
#define TALM_STAT_M 0      /* running max of z                                      */
#define TALM_STAT_S 1      /* sum exp(z - REF)                                       */
#define TALM_STAT_T 2      /* sum exp(z - REF) * z                                   */
#define TALM_STAT_ZT 3     /* z[target] if the target column is covered, else 0       */
#define TALM_STAT_BEST 4   /* max z (same as M, kept for the argmax key)               */
#define TALM_STAT_IDX 5    /* first global column attaining BEST, as int32 bits        */
#define TALM_STAT_HIT 6    /* 1.0 if the target column is covered by the call, else 0  */
#define TALM_STAT_REF 7    /* reference of S, T and the accumulator                    */

/* Device bytes of workspace talm_head_shard needs. */
int talm_head_workspace_size(int64_t n_tokens, int64_t n_grad, int64_t hidden,
                             int64_t vocab_cols, int64_t vocab_chunk, size_t* bytes);

/* Logits GEMM + online log-sum-exp / entropy numerator / argmax / target logit over the
 * vocabulary columns [vocab_col0, vocab_col0 + vocab_cols) of the weight, in slices of
 * vocab_chunk columns, and (n_grad > 0) the accumulator acc[i] = sum_v exp(z_iv - REF_i) W[v]
 * of the first n_grad rows (the labelled rows, placed first by the caller).
 * Replaces the slice loop of solution/fused_head.py:356-371 (`torch.mm` logits GEMM,
 * `fused_head_vocab_kernel` stats mode :126-182, `torch.addmm` accumulator GEMM).
 *   hidden  : fp16 [n_tokens, hidden], row stride ld_hidden elements
 *   weight  : fp16 rows [vocab_cols, hidden] of this call's columns (pointer to row vocab_col0
 *             is NOT implied: `weight` points at the first row of the covered range), row
 *             stride ld_weight elements
 *   targets : int64 [n_tokens] global column ids, negative = ignored row
 *   stats   : float [n_tokens, TALM_HEAD_STATS] (written)
 *   acc     : float [n_grad, hidden] (written when n_grad > 0)
 * Preconditions: hidden % 8 == 0 and ld_* % 8 == 0 (16-byte rows for TMA), hidden/weight
 * 16-byte aligned, 0 <= n_grad <= n_tokens, vocab_chunk >= 1, ws_bytes >=
 * talm_head_workspace_size(...). */
int talm_head_shard(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                    int64_t ld_weight, const int64_t* targets, int64_t n_tokens, int64_t n_grad,
                    int64_t hidden_size, int64_t vocab_cols, int64_t vocab_col0,
                    int64_t vocab_chunk, float* stats, float* acc, void* workspace,
                    size_t ws_bytes, void* stream);

/* talm_head_shard with no workspace argument, for callers that cannot allocate device memory
 * where they call the head (a fixed memory plan that must not grow, an allocator owned by
 * another runtime, a C caller with no allocator binding). No counterpart in the reference: its
 * head allocates its temporaries through PyTorch. The scratch is a static 16 MiB device array
 * inside this library, held on every GPU that loads it until the process exits; calls needing
 * more scratch than that (talm_head_workspace_size) return TALM_ERANGE before enqueuing
 * anything. The first call on a device looks up the array's device address (make it before any
 * stream capture). All calls on a device share the scratch: calls whose kernels overlap on the
 * GPU race and must be ordered by the caller. Everything else is as talm_head_shard. */
int talm_head_shard_noalloc(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                            int64_t ld_weight, const int64_t* targets, int64_t n_tokens,
                            int64_t n_grad, int64_t hidden_size, int64_t vocab_cols,
                            int64_t vocab_col0, int64_t vocab_chunk, float* stats, float* acc,
                            void* stream);

/* Per-row outputs and the hidden gradient from complete statistics (one shard covering the
 * whole vocabulary, or the combination of all shards).
 * Replaces the last-slice branch of `fused_head_vocab_kernel` (fused_head.py:160-169) and its
 * finalize mode (fused_head.py:111-125).
 *   token_loss[i]    = labelled ? REF + log(S) - zt : 0
 *   token_entropy[i] = REF + log(S) - T / S
 *   correct[i]       = labelled && idx == target
 *   grad ([n_tokens, hidden], fp16, or fp32 when grad_is_f32 != 0; skipped when NULL):
 *     grad[i] = labelled && i < n_grad ? acc[i] * acc_scale[i] - fp16(W[target_i]) : 0
 *     with acc_scale[i] = 1/s when acc_scale == NULL.
 *   weight/ld_weight/vocab_col0: the rows of the vocabulary range the caller owns; the
 *   subtraction of W[target] is done only for targets inside [vocab_col0, vocab_col0 +
 *   vocab_cols) (the owning rank under vocabulary parallelism).
 *   grad_rows (optional): output row of compacted row i (the inverse of the labelled-first
 *   order); NULL = identity. */
int talm_head_finalize(const float* stats, const int64_t* targets, int64_t n_tokens,
                       int64_t n_grad, const float* acc, const float* acc_scale,
                       const uint16_t* weight, int64_t ld_weight, int64_t vocab_col0,
                       int64_t vocab_cols, int64_t hidden_size, const int64_t* grad_rows,
                       float* token_loss, float* token_entropy, int32_t* correct,
                       void* grad, int grad_is_f32, void* stream);

/* Merges the statistics of n_shards vocabulary shards (gathered as [n_shards, n_tokens,
 * TALM_HEAD_STATS], shard r covering the columns of rank r) into one record per row, and
 * writes acc_scale[i] = exp(REF_rank - REF) / S for this rank's accumulator rows (n_grad rows).
 * No reference counterpart: the reference is single-GPU; this is the exchange step of the
 * vocabulary-parallel head (log-sum-exp merge of online-softmax partials). */
int talm_head_combine(const float* gathered, int64_t n_shards, int64_t n_tokens, int64_t rank,
                      int64_t n_grad, float* stats_out, float* acc_scale, void* stream);

/* The labelled-first row order (solution/fused_head.py:290-299 labelled_first) on the device,
 * and the rows gathered in that order. targets: [n_tokens] int64 (-100 = unlabelled);
 * n_labelled: the exact count of targets >= 0 (a wrong count leaves rows unwritten and records
 * TALM_ERANGE in talm_device_status). src[i] = input row at position i (labelled rows first,
 * each group in input order); dest (optional, NULL to skip) its inverse. With hidden_out
 * (NULL to skip): hidden_out[i] = hidden[src[i]] ([n_tokens, cols] fp16, contiguous; rows of
 * 16-byte multiples on 16-byte boundaries) and targets_out[i] = targets[src[i]]. Replaces the
 * labelled_first call and the two index_select of FusedHeadLossVocab.forward (:326-336). */
int talm_head_labelled_first(const int64_t* targets, int64_t n_tokens, int64_t n_labelled,
                             const uint16_t* hidden, int64_t ld_hidden, int64_t cols,
                             int64_t* src, int64_t* dest, uint16_t* hidden_out,
                             int64_t* targets_out, void* stream);

/* The head's backward: out = out_dtype(float(fp16(grad)) * s), s = grad_loss / denom, or 0
 * when denom == 0 (grad_loss, denom: fp32 scalars in device memory). grad is [n_rows, n_cols]
 * with a row stride of ld_grad elements, fp16 (grad_is_f32 == 0) or fp32 (grad_is_f32 != 0:
 * rounded to fp16 first, the value the single-GPU forward saves); out is a contiguous
 * [n_rows, n_cols] array of out_dtype (TALM_DTYPE_*).
 * Replaces _head_backward (fused_head.py:280-287): the reference's chain of four elementwise
 * torch passes (to fp32, scale, where, to the hidden's dtype) in one. */
#define TALM_DTYPE_F16 0
#define TALM_DTYPE_BF16 1
#define TALM_DTYPE_F32 2
int talm_head_scale_grad(const void* grad, int64_t ld_grad, int grad_is_f32,
                         const float* grad_loss, const float* denom, int64_t n_rows,
                         int64_t n_cols, void* out, int out_dtype, void* stream);

/* ---- vocabulary-parallel exchange over NVLink peer memory ---------------------------------
 * No reference counterpart (the reference is single-GPU): these replace the NCCL all_gather of
 * the statistics and all_reduce of the fp32 gradient of the vocabulary-parallel head.
 *
 * Every rank allocates one peer buffer of talm_peer_buffer_size bytes (zero-filled, the same
 * size on every rank), exports it with talm_ipc_export, exchanges the handles and maps the
 * other ranks' buffers with talm_ipc_import. `peers` is a device array of `world` uint64 device
 * addresses: peers[q] = rank q's buffer as mapped in this process (peers[rank] = its own).
 * `epoch` numbers the call (1, 2, ...; the same on every rank). One call is, in stream order:
 *   talm_head_shard -> talm_head_publish_stats -> talm_head_merge_peers
 *   -> talm_head_finalize_scatter -> talm_head_reduce_gather -> talm_head_gather_finish
 * or, with the scatter inside the walk's last accumulator GEMM:
 *   talm_head_shard_begin -> talm_head_publish_stats -> talm_head_merge_peers
 *   -> talm_head_shard_finish_scatter -> talm_head_reduce_gather -> talm_head_gather_finish
 * Kernels of different ranks wait on each other through flags in the peer buffers; every wait
 * is bounded (2 s, then TALM_ETIMEOUT in talm_device_status and the kernel returns). */
#define TALM_IPC_HANDLE_BYTES 64
int talm_peer_buffer_size(int64_t world, int64_t n_tokens, int64_t hidden, size_t* bytes);
/* handle: TALM_IPC_HANDLE_BYTES bytes; offset: of ptr within its allocation. */
int talm_ipc_export(const void* ptr, void* handle, int64_t* offset);
int talm_ipc_import(const void* handle, int64_t offset, void** ptr);
int talm_ipc_close(void* ptr, int64_t offset);
/* Phase 0: this rank's [n_tokens][TALM_HEAD_STATS] statistics into every rank's buffer. */
int talm_head_publish_stats(const float* stats, int64_t n_tokens, int64_t hidden, int64_t rank,
                            int64_t world, const uint64_t* peers, uint32_t epoch, void* stream);
/* Waits for every rank's statistics, then merges them as talm_head_combine does. */
int talm_head_merge_peers(int64_t n_tokens, int64_t hidden, int64_t rank, int64_t world,
                          int64_t n_grad, const void* own_buffer, uint32_t epoch,
                          float* stats_out, float* acc_scale, void* stream);
/* talm_head_finalize with the partial fp32 gradient row of output row o stored by the kernel
 * straight into the buffer of rank o / ceil(n_tokens / world) (phase 1) instead of a local
 * array. */
int talm_head_finalize_scatter(const float* stats, const int64_t* targets, int64_t n_tokens,
                               int64_t n_grad, const float* acc, const float* acc_scale,
                               const uint16_t* weight, int64_t ld_weight, int64_t vocab_col0,
                               int64_t vocab_cols, int64_t hidden_size,
                               const int64_t* grad_rows, float* token_loss,
                               float* token_entropy, int32_t* correct, int64_t rank,
                               int64_t world, const uint64_t* peers, uint32_t epoch,
                               void* stream);
/* talm_head_shard without its last step (the accumulator GEMM of the last slice, which no
 * logits GEMM precedes): the statistics are final when it returns, acc still lacks the last
 * slice. Same arguments and preconditions as talm_head_shard. */
int talm_head_shard_begin(const uint16_t* hidden, int64_t ld_hidden, const uint16_t* weight,
                          int64_t ld_weight, const int64_t* targets, int64_t n_tokens,
                          int64_t n_grad, int64_t hidden_size, int64_t vocab_cols,
                          int64_t vocab_col0, int64_t vocab_chunk, float* stats, float* acc,
                          void* workspace, size_t ws_bytes, void* stream);
/* Phase 1 for a walk run by talm_head_shard_begin, in place of talm_head_finalize_scatter:
 * the per-row outputs from the merged `stats` (and zero gradient rows for rows n_grad..), then
 * the walk's last step, whose epilogue finishes each gradient row -- (acc + last slice) *
 * acc_scale minus the owned target weight row, the values talm_head_finalize_scatter computes
 * -- and stores it in fp32 at its owner, overlapping the scatter with the step's MMAs. The walk
 * arguments (weight .. vocab_chunk, acc, workspace) are those of the talm_head_shard_begin
 * call; acc 16-byte and the weight rows 8-byte aligned. */
int talm_head_shard_finish_scatter(const uint16_t* weight, int64_t ld_weight,
                                   const int64_t* targets, int64_t n_tokens, int64_t n_grad,
                                   int64_t hidden_size, int64_t vocab_cols, int64_t vocab_col0,
                                   int64_t vocab_chunk, const float* stats, float* acc,
                                   const float* acc_scale, void* workspace, size_t ws_bytes,
                                   const int64_t* grad_rows, float* token_loss,
                                   float* token_entropy, int32_t* correct, int64_t rank,
                                   int64_t world, const uint64_t* peers, uint32_t epoch,
                                   void* stream);
/* Phase 2: waits for every rank's rows, sums the rows this rank owns over the ranks in rank
 * order (fp32), rounds them to fp16 and writes them into every rank's buffer. */
int talm_head_reduce_gather(int64_t n_tokens, int64_t hidden, int64_t rank, int64_t world,
                            const uint64_t* peers, uint32_t epoch, void* stream);
/* Waits for every rank's rows, then copies the [n_tokens][hidden] fp16 gradient to `out`
 * (16-byte aligned). */
int talm_head_gather_finish(int64_t n_tokens, int64_t hidden, int64_t world,
                            const void* own_buffer, uint32_t epoch, uint16_t* out,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TALM_H_ */
