"""Vocabulary-parallel fused head over torch.distributed (one process per GPU, NCCL on NVLink).

The reference is single-GPU; its head walks the vocabulary in slices with an online softmax
(solution/fused_head.py:356-371). The same walk shards naturally by vocabulary: rank r owns the
weight rows [col0_r, col0_r + cols_r). Every rank holds the full hidden states and targets.

  1. each rank runs the sm_100a head over its rows (`talm_head_shard`): per-row statistics
     (m_r, s_r, t_r, z_target if owned, first argmax) and the accumulator
     acc_r = sum_{v in shard} exp(z_v - m_r) W[v] of the labelled rows;
  2. all_gather of the [N, 8] fp32 statistics (16 bytes of payload per row and rank);
  3. each rank merges them locally and deterministically (`talm_head_combine`): M = max m_r,
     S = sum s_r e^{m_r - M}, T likewise, argmax = the first column among the shards' maxima,
     and its own accumulator scale e^{m_r - M} / S;
  4. `talm_head_finalize` writes the per-row outputs (identical on every rank) and the rank's
     partial gradient acc_r * scale_r - [target owned] W[target] in fp32;
  5. all_reduce(SUM) of the [N, H] fp32 partial gradients.

The kernels and the collectives are behind `HeadOps` so that the exchange logic can be exercised
with CPU ranks (gloo) by the tests; the product path is `CudaHeadOps`.
"""

import torch
import torch.distributed as dist

from . import _lib
from .fused_head import _denominator, _head_backward, _operand, _pad8, labelled_first


def shard_bounds(vocab, world, rank):
    """[col0, col0 + cols) of rank `rank`: contiguous, sizes differing by at most one."""
    base, extra = divmod(vocab, world)
    col0 = rank * base + min(rank, extra)
    return col0, base + (1 if rank < extra else 0)


class CudaHeadOps:
    """The three kernel steps of the sharded head through the C ABI."""

    def shard(self, h16, w16, ld_w, targets, n_grad, hidden_cols, col0, vocab_chunk):
        lib = _lib.load()
        device = h16.device
        n_tokens, cols = h16.shape[0], w16.shape[0]
        stream = _lib.stream_of(device)
        stats = torch.empty(n_tokens, _lib.HEAD_STATS, dtype=torch.float32, device=device)
        acc = torch.empty(n_grad, hidden_cols, dtype=torch.float32, device=device) \
            if n_grad else None
        size = _lib._SZ(0)
        _lib.check(lib.talm_head_workspace_size(n_tokens, n_grad, hidden_cols, cols, vocab_chunk,
                                                size), "talm_head_workspace_size")
        ws = torch.empty(size.value, dtype=torch.uint8, device=device)
        _lib.check(lib.talm_head_shard(_lib.ptr(h16), h16.stride(0), _lib.ptr(w16), ld_w,
                                       _lib.ptr(targets), n_tokens, n_grad, hidden_cols, cols,
                                       col0, vocab_chunk, _lib.ptr(stats), _lib.ptr(acc),
                                       _lib.ptr(ws), size.value, stream), "talm_head_shard")
        return stats, acc

    def combine(self, gathered, rank, n_grad):
        lib = _lib.load()
        n_shards, n_tokens = gathered.shape[0], gathered.shape[1]
        stats = torch.empty(n_tokens, _lib.HEAD_STATS, dtype=torch.float32,
                            device=gathered.device)
        scale = torch.empty(max(n_grad, 1), dtype=torch.float32, device=gathered.device)
        _lib.check(lib.talm_head_combine(_lib.ptr(gathered), n_shards, n_tokens, rank, n_grad,
                                         _lib.ptr(stats), _lib.ptr(scale),
                                         _lib.stream_of(gathered.device)), "talm_head_combine")
        return stats, scale

    def finalize(self, stats, targets, n_grad, acc, acc_scale, w16, ld_w, col0, hidden_cols,
                 grad_rows, want_grad):
        lib = _lib.load()
        device = stats.device
        n_tokens = stats.shape[0]
        token_loss = torch.empty(n_tokens, dtype=torch.float32, device=device)
        token_entropy = torch.empty_like(token_loss)
        correct = torch.empty(n_tokens, dtype=torch.int32, device=device)
        grad = (torch.empty(n_tokens, hidden_cols, dtype=torch.float32, device=device)
                if want_grad else None)
        _lib.check(lib.talm_head_finalize(
            _lib.ptr(stats), _lib.ptr(targets), n_tokens, n_grad, _lib.ptr(acc),
            _lib.ptr(acc_scale), _lib.ptr(w16), ld_w, col0, w16.shape[0], hidden_cols,
            _lib.ptr(grad_rows), _lib.ptr(token_loss), _lib.ptr(token_entropy),
            _lib.ptr(correct), _lib.ptr(grad), 1, _lib.stream_of(device)), "talm_head_finalize")
        return token_loss, token_entropy, correct, grad


OPS = CudaHeadOps()


def sharded_head(hidden, weight_shard, targets, vocab, col0, num_items=None, vocab_chunk=8192,
                 need_grad=True, n_labelled=None, group=None, ops=None):
    """One rank's part of the vocabulary-parallel head. Returns (loss, token_loss, entropy,
    correct, grad_hidden) with grad_hidden the all-reduced dH in fp32 (unscaled by the loss
    denominator; the backward rounds it to fp16, the value the single-GPU head saves) or None;
    every rank gets the same values."""
    ops = ops or OPS
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n_tokens, hidden_size = hidden.shape
    cols = _pad8(hidden_size)
    h16, _ = _operand(hidden.detach().to(torch.float16), cols)
    w16, ld_w = _operand(weight_shard.detach(), cols)
    targets = targets.contiguous().to(torch.int64)
    labelled = targets >= 0
    n_grad, src, rows_targets = (n_tokens if need_grad else 0), None, targets
    if need_grad and n_tokens > 0:
        if n_labelled is None:
            n_labelled = int(labelled.sum())
        n_grad = int(n_labelled)
        if 0 < n_grad < n_tokens:
            _dest, src = labelled_first(labelled, n_grad)
            h16 = h16.index_select(0, src)
            rows_targets = targets.index_select(0, src)

    stats, acc = ops.shard(h16, w16, ld_w, rows_targets, n_grad, cols, col0, int(vocab_chunk))
    gathered = torch.empty(world * n_tokens, _lib.HEAD_STATS, dtype=torch.float32,
                           device=stats.device)
    dist.all_gather_into_tensor(gathered, stats, group=group)
    gathered = gathered.view(world, n_tokens, _lib.HEAD_STATS)
    merged, scale = ops.combine(gathered, rank, n_grad)
    token_loss, token_entropy, correct, grad = ops.finalize(
        merged, rows_targets, n_grad, acc, scale, w16, ld_w, col0, cols, src, need_grad)
    if grad is not None:
        dist.all_reduce(grad, group=group)
        grad = grad[:, :hidden_size]
    denom = _denominator(num_items, labelled.sum())
    loss = token_loss.sum() / denom
    return loss, token_loss, token_entropy, correct.to(torch.bool), grad


class VocabParallelHeadLoss(torch.autograd.Function):
    """Autograd wrapper of `sharded_head`: forward computes everything, backward scales the
    saved gradient exactly as the single-GPU head (fused_head.py:280-287)."""

    @staticmethod
    def forward(ctx, hidden, weight_shard, targets, vocab, col0, num_items, vocab_chunk,
                need_grad, n_labelled, group):
        loss, token_loss, token_entropy, correct, grad = sharded_head(
            hidden, weight_shard, targets, vocab, col0, num_items, vocab_chunk, need_grad,
            n_labelled, group)
        ctx.denom = _denominator(num_items, (targets >= 0).sum())
        ctx.out_dtype = hidden.dtype
        if need_grad:
            ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(token_loss, token_entropy, correct)
        return loss, token_loss, token_entropy, correct

    @staticmethod
    def backward(ctx, grad_loss, *_):
        return (_head_backward(ctx, grad_loss),) + (None,) * 9


def vocab_parallel_head_loss(hidden, weight_shard, targets, vocab, col0, num_items=None,
                             vocab_chunk=8192, *, n_labelled=None, group=None):
    """The fused head with this rank's weight rows [col0, col0 + weight_shard.shape[0]) of a
    vocabulary of `vocab` columns; the same outputs as `fused_head_loss` on every rank."""
    need_grad = torch.is_grad_enabled() and hidden.requires_grad
    return VocabParallelHeadLoss.apply(hidden, weight_shard, targets, vocab, col0, num_items,
                                       vocab_chunk, need_grad, n_labelled, group)
