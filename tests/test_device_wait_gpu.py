"""Bounded device-side waits: a wait that is never released gives up with TALM_ETIMEOUT, the
kernel returns without its work, and the library keeps working afterwards.

The wait used here is the peer exchange's phase-flag wait (talm_head_merge_peers), run for a
world of 2 on one GPU over a freshly zeroed peer buffer: no other rank exists, so no flag is ever
raised and the wait runs out. Nothing faults or hangs: the wait limit is lowered to 20 ms for the
call (talm_set_wait_limit_ns) and restored afterwards. The host-side counterpart of this fault
model in the reference is its fallback test (solution/test_fallback.py:24-73)."""

import ctypes
import time

import pytest
import torch

from talm_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
TALM_ETIMEOUT = 5


def test_a_peer_flag_wait_that_nobody_releases_times_out():
    lib = _lib.load()
    n, hidden, world = 256, 64, 2
    need = ctypes.c_size_t(0)
    _lib.check(lib.talm_peer_buffer_size(world, n, hidden, ctypes.byref(need)),
               "talm_peer_buffer_size")
    own = torch.zeros(need.value, dtype=torch.uint8, device=DEV)  # every phase flag is 0
    merged = torch.full((n, _lib.HEAD_STATS), float("nan"), device=DEV)
    scale = torch.full((n,), float("nan"), device=DEV)
    assert _lib.device_status() == 0
    _lib.check(lib.talm_set_wait_limit_ns(20_000_000), "talm_set_wait_limit_ns")
    try:
        t0 = time.perf_counter()
        _lib.check(lib.talm_head_merge_peers(n, hidden, 0, world, n, own.data_ptr(), 1,
                                             merged.data_ptr(), scale.data_ptr(),
                                             _lib.stream_of(own.device)),
                   "talm_head_merge_peers")
        status = _lib.device_status()  # synchronises
        waited = time.perf_counter() - t0
    finally:
        _lib.check(lib.talm_set_wait_limit_ns(0), "talm_set_wait_limit_ns")
    assert status == TALM_ETIMEOUT
    assert waited < 1.5, waited  # the lowered limit, not the 2 s default
    # the kernel gave up without merging anything
    assert torch.isnan(merged).all() and torch.isnan(scale).all()
    # the status word was cleared by the read, and the library still computes
    assert _lib.device_status() == 0
    from talm_b200.fused_head import fused_head_loss

    g = torch.Generator(device=DEV).manual_seed(5)
    h = torch.randn(64, 128, generator=g, device=DEV).half().requires_grad_(True)
    w = (torch.randn(1000, 128, generator=g, device=DEV) * 0.05).half()
    t = torch.randint(0, 1000, (64,), generator=g, device=DEV)
    loss, *_ = fused_head_loss(h, w, t)
    loss.backward()
    ref = torch.nn.functional.cross_entropy((h.detach() @ w.T).float(), t)
    torch.testing.assert_close(loss.detach(), ref, rtol=1e-3, atol=1e-3)
    assert _lib.device_status() == 0

