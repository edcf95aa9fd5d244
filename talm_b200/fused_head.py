"""Fused output head + causal-LM loss on sm_100a, without a [N, V] logits tensor (drop-in for
solution/fused_head.py).

`fused_head_loss(hidden, weight, targets, num_items=None, vocab_chunk=None, *, token_chunk=None,
n_labelled=None)` returns (loss, token_loss[N], token_entropy[N], correct[N]) with the
reference's semantics (fused_head.py:53-58, :447-462):

  loss      = sum over labelled t of (lse_t - z[t, y_t]) / num_items (or / #labelled)
  entropy_t = lse_t - sum_v softmax(z_t)_v z_tv, for every row
  correct_t = argmax_v z_tv == y_t (first column on ties), labelled rows only
  z         = fp16(h16 . W16^T), the logits as the reference's fp16 cuBLAS GEMM rounds them

and the hidden gradient computed in the same forward (dH = softmax(z) W16 - W16[y]), saved for a
backward that only scales it (fused_head.py:280-287). The whole vocabulary walk runs in
libtalm_b200 (csrc/head.cu) as one persistent tcgen05 launch per vocabulary slice -- the logits
tiles of slice s, with the row statistics fused into their epilogue, together with the
accumulator tiles (softmax(z) W over the labelled rows) of slice s-1 -- each followed by a
per-row merge launch. The host code here keeps the reference's contract around it: the
labelled-first row order (`labelled_first`; `labelled_first_rows` is the same order built on
the device), the denominator, the autograd Function and the module switches.

That host code restates otarernazar-eng/Talm's solution/fused_head.py (Apache License 2.0,
"Soup Kernel Challenge starter kit", Copyright 2026 Makazhan Alpamys and the Soup contributors):
`labelled_first`, `_denominator`, `_head_backward`'s expression, the autograd contract and the
`fused_head_loss` dispatch follow that file, because callers and tests depend on them; the
kernels are this package's own.
"""

import os

import torch

from . import _lib
from .engaged import FELL_BACK, RAN

BLOCK_V = 4096            # reference row-kernel block; kept for callers reading it
NUM_WARPS = 8
DEFAULT_CHUNK = 256
VOCAB_CHUNK = int(os.environ.get("SOLUTION_HEAD_VCHUNK", "8192"))
BLOCK_H = 512
VOCAB_PATH = os.environ.get("SOLUTION_DISABLE_HEAD_VCHUNK") != "1"
COMPACT = os.environ.get("SOLUTION_DISABLE_HEAD_COMPACT") != "1"
ROW_UNIT = 1 if os.environ.get("SOLUTION_DISABLE_HEAD_ROWS") == "1" else 8


def _denominator(num_items, labelled_count):
    """solution/fused_head.py:272-277."""
    if num_items is None:
        return labelled_count.clamp(min=1).to(torch.float32)
    if torch.is_tensor(num_items):
        return num_items.to(device=labelled_count.device, dtype=torch.float32)
    return torch.tensor(float(num_items), device=labelled_count.device)


_OUT_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}  # TALM_DTYPE_*


def _head_backward(ctx, grad_loss):
    """dH * grad_loss / denom, 0 when denom == 0, in the hidden's dtype (fused_head.py:280-287),
    in one kernel (talm_head_scale_grad). The saved gradient is fp16, or the fp32 all-reduced
    one of the vocabulary-parallel head (rounded to fp16 inside the kernel first)."""
    (grad_hidden,) = ctx.saved_tensors
    if ctx.out_dtype not in _OUT_DTYPES:
        raise TypeError(f"hidden dtype {ctx.out_dtype} not supported by the head's backward")
    lib = _lib.load()
    device = grad_hidden.device
    n_rows, n_cols = grad_hidden.shape
    out = torch.empty(n_rows, n_cols, dtype=ctx.out_dtype, device=device)
    if grad_hidden.stride(1) != 1:
        grad_hidden = grad_hidden.contiguous()
    gl = grad_loss.detach().to(device=device, dtype=torch.float32).reshape(())
    denom = ctx.denom.detach().to(device=device, dtype=torch.float32).reshape(())
    _lib.check(lib.talm_head_scale_grad(
        _lib.ptr(grad_hidden), grad_hidden.stride(0), int(grad_hidden.dtype == torch.float32),
        _lib.ptr(gl), _lib.ptr(denom), n_rows, n_cols, _lib.ptr(out), _OUT_DTYPES[ctx.out_dtype],
        _lib.stream_of(device)), "talm_head_scale_grad")
    return out


def labelled_first(labelled, n_labelled):
    """The order that puts the labelled rows first, each group in its original order, without a
    host sync: (dest, src) with input row r at position dest[r] of the reordered rows and src the
    inverse (fused_head.py:290-299)."""
    n = labelled.shape[0]
    pos = torch.arange(n, device=labelled.device)
    seen = torch.cumsum(labelled, 0)
    dest = torch.where(labelled, seen - 1, pos - seen + n_labelled)
    src = torch.empty_like(dest).index_copy_(0, dest, pos)
    return dest, src


def labelled_first_rows(h16, targets, n_labelled):
    """Device-side labelled-first compaction (talm_head_labelled_first): the fp16 rows and
    their targets in the order of `labelled_first`, and `src` (the input row of each position),
    in two launches instead of labelled_first + two index_select. h16: [N, cols] fp16 rows of
    16-byte multiples on 16-byte boundaries; n_labelled: the exact count of targets >= 0 (a
    count that does not match records TALM_ERANGE in the device status word)."""
    lib = _lib.load()
    n, cols = h16.shape
    src = torch.empty(n, dtype=torch.int64, device=h16.device)
    rows = torch.empty(n, cols, dtype=torch.float16, device=h16.device)
    rows_targets = torch.empty(n, dtype=torch.int64, device=h16.device)
    _lib.check(lib.talm_head_labelled_first(
        _lib.ptr(targets), n, n_labelled, _lib.ptr(h16), h16.stride(0), cols, _lib.ptr(src), None,
        _lib.ptr(rows), _lib.ptr(rows_targets), _lib.stream_of(h16.device)),
        "talm_head_labelled_first")
    return rows, rows_targets, src


def _pad8(n):
    return (n + 7) // 8 * 8


def _operand(t, cols):
    """fp16 rows usable by TMA: 16-byte aligned base, row stride a multiple of 8 elements,
    `cols` (>= the tensor's width, a multiple of 8) addressable columns. Views when the tensor
    already is one; a zero-padded fp16 copy otherwise (odd widths, fp32/bf16 storage, rows
    that are not contiguous)."""
    rows, width = t.shape
    if (t.dtype == torch.float16 and t.stride(1) == 1 and width == cols
            and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0):
        return t, t.stride(0)
    out = torch.zeros(rows, cols, dtype=torch.float16, device=t.device)
    out[:, :width].copy_(t)
    return out, cols


def _check_cuda(*tensors):
    for t in tensors:
        if torch.is_tensor(t) and not t.is_cuda:
            raise RuntimeError("fused_head_loss runs on CUDA tensors only (sm_100a kernels; "
                               "there is no CPU path)")


def head_forward(h16, w16, ld_w, targets, n_grad, hidden_cols, vocab_chunk, grad_rows=None,
                 want_grad=True):
    """The C-ABI call sequence of one single-GPU head: talm_head_shard over the whole vocabulary,
    then talm_head_finalize. h16 [N, hidden_cols] fp16 TMA rows, w16 [V, >= hidden_cols] fp16
    rows with stride ld_w, targets [N] int64 in h16's row order (labelled rows first when
    n_grad < N). Returns token_loss, token_entropy, correct (int32), grad [N, hidden_cols] fp16
    (rows placed through grad_rows) or None."""
    lib = _lib.load()
    device = h16.device
    n_tokens = h16.shape[0]
    vocab = w16.shape[0]
    stream = _lib.stream_of(device)
    stats = torch.empty(n_tokens, _lib.HEAD_STATS, dtype=torch.float32, device=device)
    acc = torch.empty(n_grad, hidden_cols, dtype=torch.float32, device=device) if n_grad else None
    size = _lib._SZ(0)
    _lib.check(lib.talm_head_workspace_size(n_tokens, n_grad, hidden_cols, vocab, vocab_chunk,
                                            size), "talm_head_workspace_size")
    ws = torch.empty(size.value, dtype=torch.uint8, device=device)
    _lib.check(lib.talm_head_shard(_lib.ptr(h16), h16.stride(0), _lib.ptr(w16), ld_w,
                                   _lib.ptr(targets), n_tokens, n_grad, hidden_cols, vocab, 0,
                                   vocab_chunk, _lib.ptr(stats), _lib.ptr(acc), _lib.ptr(ws),
                                   size.value, stream), "talm_head_shard")
    token_loss = torch.empty(n_tokens, dtype=torch.float32, device=device)
    token_entropy = torch.empty_like(token_loss)
    correct = torch.empty(n_tokens, dtype=torch.int32, device=device)
    grad = (torch.empty(n_tokens, hidden_cols, dtype=torch.float16, device=device)
            if want_grad else None)
    _lib.check(lib.talm_head_finalize(_lib.ptr(stats), _lib.ptr(targets), n_tokens, n_grad,
                                      _lib.ptr(acc), None, _lib.ptr(w16), ld_w, 0, vocab,
                                      hidden_cols, _lib.ptr(grad_rows), _lib.ptr(token_loss),
                                      _lib.ptr(token_entropy), _lib.ptr(correct),
                                      _lib.ptr(grad), 0, stream), "talm_head_finalize")
    return token_loss, token_entropy, correct, grad


class FusedHeadLossVocab(torch.autograd.Function):
    """loss, per-token loss, per-token entropy, per-token correctness from hidden states and the
    frozen output weight, walking the vocabulary in slices (fused_head.py:302-397). Saves only
    the fp16 hidden gradient. With the gradient on and COMPACT, the rows are put labelled-first
    so the accumulator GEMM covers the labelled rows only; every output comes back in the input
    order."""

    @staticmethod
    def forward(ctx, hidden, weight, targets, num_items, vocab_chunk, need_grad, n_labelled):
        _check_cuda(hidden, weight, targets)
        n_tokens, hidden_size = hidden.shape
        cols = _pad8(hidden_size)
        h16, _ = _operand(hidden.detach().to(torch.float16), cols)
        w16, ld_w = _operand(weight.detach(), cols)
        targets = targets.contiguous().to(torch.int64)

        n_grad, src, rows_targets = (n_tokens if need_grad else 0), None, targets
        if need_grad and COMPACT and n_tokens > 0:
            if n_labelled is None:
                n_labelled = int((targets >= 0).sum())
            n_grad = int(n_labelled)
            if 0 < n_grad < n_tokens:
                # the order of labelled_first, built on the device in two launches
                # (talm_head_labelled_first) instead of ten torch ops
                h16, rows_targets, src = labelled_first_rows(h16, targets, n_grad)
                RAN["compact"] += 1

        if n_tokens > 0:
            token_loss, token_entropy, correct, grad = head_forward(
                h16, w16, ld_w, rows_targets, n_grad, cols, int(vocab_chunk), grad_rows=src,
                want_grad=need_grad)
        else:
            token_loss = torch.empty(0, dtype=torch.float32, device=hidden.device)
            token_entropy = torch.empty_like(token_loss)
            correct = torch.empty(0, dtype=torch.int32, device=hidden.device)
            grad = torch.empty(0, cols, dtype=torch.float16, device=hidden.device)
        if need_grad and cols != hidden_size:
            grad = grad[:, :hidden_size]

        if num_items is None and n_labelled is not None:
            # the labelled count is known on the host: the reference's denominator
            # (count clamped to 1, fp32) in one fill instead of a device count
            denom = torch.full((), float(max(int(n_labelled), 1)), dtype=torch.float32,
                               device=hidden.device)
        else:
            denom = _denominator(num_items, (targets >= 0).sum())
        loss = token_loss.sum() / denom
        correct = correct.to(torch.bool)
        ctx.denom = denom
        ctx.out_dtype = hidden.dtype
        if need_grad:
            ctx.save_for_backward(grad)
        ctx.mark_non_differentiable(token_loss, token_entropy, correct)
        return loss, token_loss, token_entropy, correct

    @staticmethod
    def backward(ctx, grad_loss, _grad_token_loss, _grad_entropy, _grad_correct):
        return _head_backward(ctx, grad_loss), None, None, None, None, None, None


class FusedHeadLoss(torch.autograd.Function):
    """Token-chunked entry point (fused_head.py:400-444), same signature. The reference's
    token-chunked kernel is replaced by the vocabulary-sliced CUDA path (same outputs); `chunk`
    is accepted and ignored."""

    @staticmethod
    def forward(ctx, hidden, weight, targets, num_items, chunk, need_grad):
        outs = FusedHeadLossVocab.forward(ctx, hidden, weight, targets, num_items, VOCAB_CHUNK,
                                          need_grad, None)
        return outs

    @staticmethod
    def backward(ctx, grad_loss, _grad_token_loss, _grad_entropy, _grad_correct):
        return _head_backward(ctx, grad_loss), None, None, None, None, None


def fused_head_loss(hidden, weight, targets, num_items=None, vocab_chunk=None, *,
                    token_chunk=None, n_labelled=None):
    """hidden [N, H] (fp16/fp32/bf16, may require grad), weight [V, H] frozen, targets [N] int64
    already shifted (-100 = ignore). Returns (loss, token_loss[N], token_entropy[N], correct[N])
    (fused_head.py:447-462). `n_labelled`: the host count of targets >= 0 when the caller has it
    (saves a host sync); it must be exact."""
    need_grad = torch.is_grad_enabled() and hidden.requires_grad
    if token_chunk is None and VOCAB_PATH and weight.dim() == 2 and weight.stride(1) == 1:
        RAN["vchunk"] += 1
        return FusedHeadLossVocab.apply(hidden, weight, targets, num_items,
                                        vocab_chunk or VOCAB_CHUNK, need_grad, n_labelled)
    if VOCAB_PATH:
        FELL_BACK["vchunk"] += 1
    return FusedHeadLoss.apply(hidden, weight, targets, num_items, token_chunk or DEFAULT_CHUNK,
                               need_grad)
