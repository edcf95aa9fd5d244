"""Vocabulary-parallel fused head over torch.distributed (one process per GPU, NCCL on NVLink).

The reference is single-GPU; its head walks the vocabulary in slices with an online softmax
(solution/fused_head.py:356-371). The same walk shards naturally by vocabulary: rank r owns the
weight rows [col0_r, col0_r + cols_r). Every rank holds the full hidden states and targets.

  1. each rank runs the sm_100a head over its rows (`talm_head_shard`): per-row statistics
     (m_r, s_r, t_r, z_target if owned, first argmax) and the accumulator
     acc_r = sum_{v in shard} exp(z_v - m_r) W[v] of the labelled rows;
  2. every rank's [N, 8] fp32 statistics reach every rank;
  3. each rank merges them locally and deterministically: M = max m_r, S = sum s_r e^{m_r - M},
     T likewise, argmax = the first column among the shards' maxima, and its own accumulator
     scale e^{m_r - M} / S;
  4. the per-row outputs (identical on every rank) and the rank's partial gradient
     acc_r * scale_r - [target owned] W[target] in fp32;
  5. the partial gradients are summed over the ranks.

On CUDA ranks that can map each other's memory (one node, NVLink) steps 2-5 run as the peer
exchange of the library (`PeerExchange`, talm_head_publish_stats ... talm_head_gather_finish):
kernels write the statistics and the gradient rows straight into the other GPUs' buffers, each
row is reduced once by its owner and the fp16 result is written to every rank. Step 1 then stops
before its last accumulator GEMM (talm_head_shard_begin), which runs after the merge
(talm_head_shard_finish_scatter) and performs step 4 in its epilogue: each finished gradient
row piece leaves for its owner while the tensor cores work on the remaining tiles. Otherwise
(TALM_B200_PEER_EXCHANGE=0, or ranks that cannot map each other's memory) step 2 is an NCCL
all_gather and step 5 an all_reduce of the fp32 gradient.

The kernels are behind `HeadOps` so that the collective flow can be exercised with CPU ranks
(gloo) by the tests; the product path is `CudaHeadOps`.
"""

import ctypes
import os

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

    def shard(self, h16, w16, ld_w, targets, n_grad, hidden_cols, col0, vocab_chunk,
              begin=False):
        """The walk over this rank's rows: (stats, acc). With `begin`, every step but the last
        accumulator GEMM (talm_head_shard_begin), and the workspace is returned as well: the
        peer flow finishes the walk with talm_head_shard_finish_scatter once the statistics
        are merged."""
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
        fn, name = ((lib.talm_head_shard_begin, "talm_head_shard_begin") if begin
                    else (lib.talm_head_shard, "talm_head_shard"))
        _lib.check(fn(_lib.ptr(h16), h16.stride(0), _lib.ptr(w16), ld_w, _lib.ptr(targets),
                      n_tokens, n_grad, hidden_cols, cols, col0, vocab_chunk, _lib.ptr(stats),
                      _lib.ptr(acc), _lib.ptr(ws), size.value, stream), name)
        return (stats, acc, ws) if begin else (stats, acc)

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

PEER_EXCHANGE = os.environ.get("TALM_B200_PEER_EXCHANGE", "1") != "0"
# Under the peer exchange, the walk's last accumulator GEMM finishes the gradient rows and
# stores them at their owners from its epilogue (talm_head_shard_finish_scatter), instead of a
# separate finalize pass over acc after it; 0 keeps the separate pass.
FUSED_SCATTER = os.environ.get("TALM_B200_FUSED_SCATTER", "1") != "0"


class PeerExchange:
    """One rank's peer buffer and its mappings of the other ranks' buffers (CUDA IPC), for one
    process group and device. The buffer grows (in lockstep on every rank: the sizes depend only
    on replicated shapes) when a call needs more. `ok` is False when some rank could not map
    the others' memory; the caller then uses the NCCL flow."""

    def __init__(self, group, device):
        self.group, self.device = group, device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.size = 0
        self.buf = None
        self.mapped = []      # (pointer, offset) of the imported peer buffers
        self.peers = None     # device int64 [world]: every rank's buffer in this process
        self.epoch = 0
        self.ok = True

    def _release(self):
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still writes into the old buffers
        for p, off in self.mapped:
            lib.talm_ipc_close(p, off)
        self.mapped, self.buf, self.peers = [], None, None

    def ensure(self, n_tokens, hidden_cols):
        lib = _lib.load()
        need = _lib._SZ(0)
        _lib.check(lib.talm_peer_buffer_size(self.world, n_tokens, hidden_cols, need),
                   "talm_peer_buffer_size")
        if self.buf is not None and need.value <= self.size:
            return self.ok
        if self.buf is not None:
            self._release()
        self.size = max(need.value, 2 * self.size)
        self.buf = torch.zeros(self.size, dtype=torch.uint8, device=self.device)
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        offset = _lib._I64(0)
        _lib.check(lib.talm_ipc_export(_lib.ptr(self.buf), ctypes.cast(handle, ctypes.c_void_p),
                                       ctypes.byref(offset)), "talm_ipc_export")
        mine = torch.tensor(list(bytes(handle)) + list(offset.value.to_bytes(8, "little")),
                            dtype=torch.uint8, device=self.device)
        everyone = torch.empty(self.world * mine.numel(), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(everyone, mine, group=self.group)
        records = everyone.view(self.world, -1).cpu()
        addrs, good = [], 1
        for q in range(self.world):
            if q == self.rank:
                addrs.append(self.buf.data_ptr())
                continue
            raw = bytes(records[q].tolist())
            h = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(raw[:_lib.IPC_HANDLE_BYTES])
            off = int.from_bytes(raw[_lib.IPC_HANDLE_BYTES:], "little")
            p = ctypes.c_void_p(0)
            if lib.talm_ipc_import(ctypes.cast(h, ctypes.c_void_p), off, ctypes.byref(p)) != 0:
                good = 0
                addrs.append(0)
                continue
            self.mapped.append((p.value, off))
            addrs.append(p.value)
        flag = torch.tensor([good], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        self.ok = bool(flag.item())
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=self.device)
        return self.ok

    def next_epoch(self):
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        return self.epoch


_EXCHANGES = {}


def _exchange(group, device, n_tokens, hidden_cols):
    key = (id(group) if group is not None else None, device.index)
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = _EXCHANGES[key] = PeerExchange(group, device)
    return ex if ex.ensure(n_tokens, hidden_cols) else None


def _peer_flow(ex, stats, acc, rows_targets, n_grad, w16, ld_w, col0, cols, src, need_grad,
               walk=None):
    """Steps 2-5 through the peer buffers: returns token_loss, token_entropy, correct (int32)
    and the reduced fp16 gradient [N, cols] (or None). `walk` = (workspace, vocab_chunk) of a
    walk run by talm_head_shard_begin: its last accumulator GEMM then runs here, after the
    merge, and scatters the finished gradient rows itself."""
    lib = _lib.load()
    device = stats.device
    stream = _lib.stream_of(device)
    n_tokens = stats.shape[0]
    epoch = ex.next_epoch()
    peers, own = _lib.ptr(ex.peers), _lib.ptr(ex.buf)
    _lib.check(lib.talm_head_publish_stats(_lib.ptr(stats), n_tokens, cols, ex.rank, ex.world,
                                           peers, epoch, stream), "talm_head_publish_stats")
    merged = torch.empty(n_tokens, _lib.HEAD_STATS, dtype=torch.float32, device=device)
    scale = torch.empty(max(n_grad, 1), dtype=torch.float32, device=device)
    _lib.check(lib.talm_head_merge_peers(n_tokens, cols, ex.rank, ex.world, n_grad, own, epoch,
                                         _lib.ptr(merged), _lib.ptr(scale), stream),
               "talm_head_merge_peers")
    token_loss = torch.empty(n_tokens, dtype=torch.float32, device=device)
    token_entropy = torch.empty_like(token_loss)
    correct = torch.empty(n_tokens, dtype=torch.int32, device=device)
    if not need_grad:
        _lib.check(lib.talm_head_finalize(
            _lib.ptr(merged), _lib.ptr(rows_targets), n_tokens, 0, None, None, _lib.ptr(w16),
            ld_w, col0, w16.shape[0], cols, _lib.ptr(src), _lib.ptr(token_loss),
            _lib.ptr(token_entropy), _lib.ptr(correct), None, 0, stream), "talm_head_finalize")
        return token_loss, token_entropy, correct, None
    if walk is not None:
        ws, vocab_chunk = walk
        _lib.check(lib.talm_head_shard_finish_scatter(
            _lib.ptr(w16), ld_w, _lib.ptr(rows_targets), n_tokens, n_grad, cols, w16.shape[0],
            col0, vocab_chunk, _lib.ptr(merged), _lib.ptr(acc), _lib.ptr(scale), _lib.ptr(ws),
            ws.numel(), _lib.ptr(src), _lib.ptr(token_loss), _lib.ptr(token_entropy),
            _lib.ptr(correct), ex.rank, ex.world, peers, epoch, stream),
            "talm_head_shard_finish_scatter")
    else:
        _lib.check(lib.talm_head_finalize_scatter(
            _lib.ptr(merged), _lib.ptr(rows_targets), n_tokens, n_grad, _lib.ptr(acc),
            _lib.ptr(scale), _lib.ptr(w16), ld_w, col0, w16.shape[0], cols, _lib.ptr(src),
            _lib.ptr(token_loss), _lib.ptr(token_entropy), _lib.ptr(correct), ex.rank, ex.world,
            peers, epoch, stream), "talm_head_finalize_scatter")
    _lib.check(lib.talm_head_reduce_gather(n_tokens, cols, ex.rank, ex.world, peers, epoch,
                                           stream), "talm_head_reduce_gather")
    grad = torch.empty(n_tokens, cols, dtype=torch.float16, device=device)
    _lib.check(lib.talm_head_gather_finish(n_tokens, cols, ex.world, own, epoch,
                                           _lib.ptr(grad), stream), "talm_head_gather_finish")
    return token_loss, token_entropy, correct, grad


def sharded_head(hidden, weight_shard, targets, vocab, col0, num_items=None, vocab_chunk=8192,
                 need_grad=True, n_labelled=None, group=None, ops=None):
    """One rank's part of the vocabulary-parallel head. Returns (loss, token_loss, entropy,
    correct, grad_hidden) with grad_hidden the summed dH (unscaled by the loss denominator;
    fp16 from the peer exchange, fp32 from the NCCL flow, which the backward rounds to fp16 as
    the single-GPU head saves it) or None; every rank gets the same values."""
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

    ex = (_exchange(group, hidden.device, n_tokens, cols)
          if PEER_EXCHANGE and isinstance(ops, CudaHeadOps) and world > 1 and n_tokens > 0
          else None)
    walk = None
    if ex is not None and FUSED_SCATTER and need_grad and n_grad > 0:
        stats, acc, ws = ops.shard(h16, w16, ld_w, rows_targets, n_grad, cols, col0,
                                   int(vocab_chunk), begin=True)
        walk = (ws, int(vocab_chunk))
    else:
        stats, acc = ops.shard(h16, w16, ld_w, rows_targets, n_grad, cols, col0,
                               int(vocab_chunk))
    if ex is not None:
        token_loss, token_entropy, correct, grad = _peer_flow(
            ex, stats, acc, rows_targets, n_grad, w16, ld_w, col0, cols, src, need_grad, walk)
        if grad is not None:
            grad = grad[:, :hidden_size]
        denom = _denominator(num_items, labelled.sum())
        loss = token_loss.sum() / denom
        return loss, token_loss, token_entropy, correct.to(torch.bool), grad
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
