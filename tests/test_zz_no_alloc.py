"""talm_head_shard_noalloc: the head's slice walk for callers that cannot allocate device memory
(a fixed memory plan, an allocator owned by another runtime, a plain C caller). It must give
what talm_head_shard gives with a caller workspace, call after call, and refuse work that does
not fit its static scratch. Called through the C ABI.

This file is collected last on purpose (pytest orders files by name), so that a run stopping at
the first failure has run every other test before it; it also passes on its own in a fresh
process."""

import ctypes

import pytest
import torch

from talm_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH_BYTES = 16 << 20


def _case(seed, n, vocab, size):
    g = torch.Generator(device=DEV).manual_seed(seed)
    hidden = torch.randn(n, size, generator=g, device=DEV).half()
    weight = (torch.randn(vocab, size, generator=g, device=DEV) * 0.05).half()
    targets = torch.randint(0, vocab, (n,), generator=g, device=DEV)
    # a row whose maximum jumps in a later slice, so the rescaling path runs too
    hidden[3] = (weight[vocab - 5].float() * 30).half()
    targets[3] = vocab - 5
    return hidden, weight, targets


def _with_workspace(lib, hidden, weight, targets, n_grad, chunk):
    n, size = hidden.shape
    vocab = weight.shape[0]
    stats = torch.full((n, _lib.HEAD_STATS), float("nan"), device=DEV)
    acc = torch.full((n_grad, size), float("nan"), device=DEV)
    need = ctypes.c_size_t(0)
    _lib.check(lib.talm_head_workspace_size(n, n_grad, size, vocab, chunk, ctypes.byref(need)),
               "talm_head_workspace_size")
    ws = torch.empty(need.value, dtype=torch.uint8, device=DEV)
    _lib.check(lib.talm_head_shard(hidden.data_ptr(), size, weight.data_ptr(), size,
                                   targets.data_ptr(), n, n_grad, size, vocab, 0, chunk,
                                   stats.data_ptr(), acc.data_ptr(), ws.data_ptr(), need.value,
                                   _lib.stream_of(hidden.device)), "talm_head_shard")
    return stats, acc


def _without_workspace(lib, hidden, weight, targets, n_grad, chunk):
    n, size = hidden.shape
    vocab = weight.shape[0]
    stats = torch.full((n, _lib.HEAD_STATS), float("nan"), device=DEV)
    acc = torch.full((n_grad, size), float("nan"), device=DEV)
    _lib.check(lib.talm_head_shard_noalloc(hidden.data_ptr(), size, weight.data_ptr(), size,
                                           targets.data_ptr(), n, n_grad, size, vocab, 0, chunk,
                                           stats.data_ptr(), acc.data_ptr(),
                                           _lib.stream_of(hidden.device)),
               "talm_head_shard_noalloc")
    return stats, acc


def test_no_alloc_matches_the_workspace_entry_point_on_consecutive_calls():
    lib = _lib.load()
    # two different problems back to back: the second call finds the first call's leftovers in
    # the shared scratch and must not be affected by them
    for seed, (n, vocab, size, n_grad, chunk) in ((21, (300, 5000, 256, 180, 2048)),
                                                  (22, (129, 3001, 128, 129, 1024))):
        hidden, weight, targets = _case(seed, n, vocab, size)
        ref_stats, ref_acc = _with_workspace(lib, hidden, weight, targets, n_grad, chunk)
        stats, acc = _without_workspace(lib, hidden, weight, targets, n_grad, chunk)
        torch.cuda.synchronize()
        for field in (_lib.STAT_M, _lib.STAT_S, _lib.STAT_T, _lib.STAT_ZT, _lib.STAT_BEST,
                      _lib.STAT_HIT, 7):
            torch.testing.assert_close(stats[:, field], ref_stats[:, field], rtol=1e-5,
                                       atol=1e-6)
        assert torch.equal(stats[:, _lib.STAT_IDX].view(torch.int32),
                           ref_stats[:, _lib.STAT_IDX].view(torch.int32))
        torch.testing.assert_close(acc, ref_acc, rtol=1e-3,
                                   atol=float(ref_acc.abs().max()) * 2 ** -10)
    assert _lib.device_status() == 0


def test_no_alloc_refuses_work_beyond_its_scratch():
    lib = _lib.load()
    n, vocab, size, n_grad, chunk = 4096, 20000, 256, 4096, 8192
    need = ctypes.c_size_t(0)
    _lib.check(lib.talm_head_workspace_size(n, n_grad, size, vocab, chunk, ctypes.byref(need)),
               "talm_head_workspace_size")
    assert need.value > SCRATCH_BYTES
    # nothing is read or launched for a refused call: dummy pointers are never dereferenced
    status = lib.talm_head_shard_noalloc(16, size, 16, size, 16, n, n_grad, size, vocab, 0, chunk,
                                         16, 16, None)
    assert status == 3
    assert b"scratch" in lib.talm_last_error()
