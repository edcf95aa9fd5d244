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


def _case(seed, n, vocab, size, dev=DEV):
    g = torch.Generator(device=dev).manual_seed(seed)
    hidden = torch.randn(n, size, generator=g, device=dev).half()
    weight = (torch.randn(vocab, size, generator=g, device=dev) * 0.05).half()
    targets = torch.randint(0, vocab, (n,), generator=g, device=dev)
    # a row whose maximum jumps in a later slice, so the rescaling path runs too
    hidden[3] = (weight[vocab - 5].float() * 30).half()
    targets[3] = vocab - 5
    return hidden, weight, targets


def _with_workspace(lib, hidden, weight, targets, n_grad, chunk):
    n, size = hidden.shape
    vocab = weight.shape[0]
    dev = hidden.device
    stats = torch.full((n, _lib.HEAD_STATS), float("nan"), device=dev)
    acc = torch.full((n_grad, size), float("nan"), device=dev)
    need = ctypes.c_size_t(0)
    _lib.check(lib.talm_head_workspace_size(n, n_grad, size, vocab, chunk, ctypes.byref(need)),
               "talm_head_workspace_size")
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    _lib.check(lib.talm_head_shard(hidden.data_ptr(), size, weight.data_ptr(), size,
                                   targets.data_ptr(), n, n_grad, size, vocab, 0, chunk,
                                   stats.data_ptr(), acc.data_ptr(), ws.data_ptr(), need.value,
                                   _lib.stream_of(hidden.device)), "talm_head_shard")
    return stats, acc


def _without_workspace(lib, hidden, weight, targets, n_grad, chunk):
    n, size = hidden.shape
    vocab = weight.shape[0]
    dev = hidden.device
    stats = torch.full((n, _lib.HEAD_STATS), float("nan"), device=dev)
    acc = torch.full((n_grad, size), float("nan"), device=dev)
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
        _same_bits(stats, ref_stats, acc, ref_acc)
    assert _lib.device_status() == 0


def _same_bits(stats, ref_stats, acc, ref_acc):
    # both entry points run the same whole-tile kernels, which add every accumulator element
    # in the same order on every call: the results are the same bits
    assert torch.equal(stats.view(torch.int32), ref_stats.view(torch.int32))
    assert torch.equal(acc.view(torch.int32), ref_acc.view(torch.int32))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_both_entry_points_on_two_devices_in_one_process():
    # the shared-memory opt-in of the slice kernel and the scratch address are per device: a
    # process that drives two GPUs must get a working launch and its own scratch on each
    lib = _lib.load()
    for index in (0, 1, 0):
        dev = torch.device("cuda", index)
        with torch.cuda.device(dev):
            hidden, weight, targets = _case(30 + index, 260, 3000, 256, dev)
            ref_stats, ref_acc = _with_workspace(lib, hidden, weight, targets, 200, 1024)
            stats, acc = _without_workspace(lib, hidden, weight, targets, 200, 1024)
            torch.cuda.synchronize(dev)
            _same_bits(stats, ref_stats, acc, ref_acc)
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
