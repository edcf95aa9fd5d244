"""The C-ABI library builds, loads and exports every entry point include/talm.h declares; the
argument checks that run before any CUDA call answer on any machine. No kernel is launched."""

import ctypes
import os
import re
import subprocess

import pytest

from talm_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "talm.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(talm_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_the_abi():
    names = declared_functions()
    assert "talm_nf4_dequantize" in names and "talm_nf4_group_dequant" in names
    assert "talm_head_shard" in names and "talm_head_finalize" in names
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", build.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (talm_\w+)", out))
    missing = set(declared_functions()) - exported
    assert not missing, f"declared in talm.h but not exported: {sorted(missing)}"
    for name in declared_functions():
        assert getattr(lib, name) is not None


def test_no_library_allocates_or_batches_copies():
    """The C ABI never allocates (callers pass workspace) and never uses batched copies."""
    csrc = os.path.join(ROOT, "talm_b200", "csrc")
    for name in os.listdir(csrc):
        text = open(os.path.join(csrc, name)).read()
        assert "cudaMalloc" not in text, name
        assert "Batch" + "Async" not in text, name


def test_status_strings_and_version(lib):
    assert lib.talm_abi_version() == 1
    assert lib.talm_status_string(0) == b"ok"
    assert lib.talm_status_string(1) == b"invalid argument"


def test_argument_errors_are_reported_before_any_launch(lib):
    # odd element count and odd block size: rejected on the host
    assert lib.talm_nf4_dequantize(None, None, 3, 64, None, None) == 1
    assert b"even" in lib.talm_last_error()
    assert lib.talm_nf4_dequantize(None, None, 4, 63, None, None) == 1
    assert lib.talm_nf4_group_dequant(None, None, None, None, None, None, None, 4, 96, 256,
                                      None) == 1
    assert lib.talm_nf4_group_dequant(None, None, None, None, None, None, None,
                                      1 << 26, 64, 256, None) == 3
    # head: n_grad > n_tokens, odd hidden size
    assert lib.talm_head_shard(None, 8, None, 8, None, 4, 5, 8, 10, 0, 8, None, None, None, 0,
                               None) == 1
    assert lib.talm_head_shard(None, 12, None, 12, None, 4, 2, 12, 10, 0, 8, None, None, None,
                               0, None) == 1
    assert lib.talm_head_combine(None, 2, 4, 2, 0, None, None, None) == 1
    # zero-sized work is a no-op
    assert lib.talm_nf4_dequantize(None, None, 0, 64, None, None) == 0


def test_workspace_size_is_host_only(lib):
    size = ctypes.c_size_t(0)
    assert lib.talm_head_workspace_size(2048, 1126, 1536, 151936, 8192, ctypes.byref(size)) == 0
    # the pair of probability slices (2 x n_grad x chunk fp16) dominates
    assert 2 * 1126 * 8192 * 2 < size.value < 2 * 1126 * 8192 * 2 + 4 * 2**20
    # a single slice needs a single buffer
    assert lib.talm_head_workspace_size(64, 64, 64, 1000, 8192, ctypes.byref(size)) == 0
    assert 64 * 1024 * 2 < size.value < 2 * 64 * 1024 * 2


def test_peer_buffer_layout_is_host_only(lib):
    """The peer-exchange buffer holds flags, every rank's statistics, the fp32 rows the rank
    owns from every rank and the fp16 gradient: at config 4 on 8 GPUs about 154 MB."""
    size = ctypes.c_size_t(0)
    n, h, w = 16384, 1536, 8
    assert lib.talm_peer_buffer_size(w, n, h, ctypes.byref(size)) == 0
    payload = w * n * 8 * 4 + w * (n // w) * h * 4 + n * h * 2
    assert payload < size.value < payload + 8192
    # rows per rank round up: every row has an owner
    assert lib.talm_peer_buffer_size(3, 10, 8, ctypes.byref(size)) == 0
    assert size.value >= 3 * 4 * 8 * 4 + 10 * 8 * 2
    # hidden columns must be a multiple of 8, rank inside the group
    assert lib.talm_peer_buffer_size(2, 10, 12, ctypes.byref(size)) == 1
    assert lib.talm_peer_buffer_size(0, 10, 8, ctypes.byref(size)) == 1


def test_peer_exchange_and_backward_reject_bad_arguments(lib):
    assert lib.talm_head_publish_stats(None, 4, 8, 2, 2, None, 1, None) == 1    # rank >= world
    assert lib.talm_head_reduce_gather(4, 8, 0, 2, None, 1, None) == 1          # no peer table
    assert lib.talm_head_gather_finish(4, 8, 2, None, 1, None, None) == 1
    assert lib.talm_ipc_export(None, None, None) == 1
    # backward: out_dtype outside TALM_DTYPE_*, a row stride shorter than the row
    assert lib.talm_head_scale_grad(None, 8, 0, None, None, 4, 8, None, 7, None) == 1
    assert lib.talm_head_scale_grad(None, 4, 0, None, None, 4, 8, None, 0, None) == 1
    assert lib.talm_head_scale_grad(None, 8, 0, None, None, 0, 8, None, 0, None) == 0


def test_labelled_first_rejects_bad_arguments(lib):
    assert lib.talm_head_labelled_first(None, 4, 5, None, 8, 8, None, None, None, None, None) == 1
    assert lib.talm_head_labelled_first(None, 0, 0, None, 8, 8, None, None, None, None, None) == 0


def test_fused_nf4_gemm_rejects_bad_arguments(lib):
    """talm_nf4_linear validates its shapes before it touches a pointer or the device."""
    def call(n_rows=8, qblock=64, rows=128, cols=256, transpose=0, bias=None, ld_a=256,
             ld_y=128, qblock2=256):
        return lib.talm_nf4_linear(None, ld_a, n_rows, None, None, None, None, None, None, 0,
                                   rows, cols, qblock, qblock2, transpose, bias, None, ld_y, None)
    assert call(qblock=128) == 1                 # qblock 64 only
    assert call(rows=96) == 1                    # rows: multiples of 64
    assert call(cols=192) == 1                   # columns: multiples of 128
    assert call(transpose=1, bias=16, ld_a=128, ld_y=256) == 1   # no bias on the gradient
    assert call(ld_a=200) == 1                   # stride below the reduction length
    assert call(ld_y=100) == 1                   # stride not a multiple of 8
    assert call(qblock2=0) == 1
    assert call(n_rows=-1) == 1
    assert call(n_rows=0) == 0                   # nothing to do: no pointer read
    assert b"qblock" in (call(qblock=32) and lib.talm_last_error())


def test_split_walk_rejects_bad_arguments(lib):
    """talm_head_shard_begin / talm_head_shard_finish_scatter validate sizes and the rank
    before they touch a pointer or the device."""
    # the walk's first part: n_grad above n_tokens, hidden not a multiple of 8
    assert lib.talm_head_shard_begin(None, 8, None, 8, None, 4, 5, 8, 100, 0, 64, None, None,
                                     None, 0, None) == 1
    assert lib.talm_head_shard_begin(None, 12, None, 12, None, 4, 4, 12, 100, 0, 64, None,
                                     None, None, 0, None) == 1
    assert lib.talm_head_shard_begin(None, 8, None, 8, None, 0, 0, 8, 100, 0, 64, None, None,
                                     None, 0, None) == 0     # no rows: nothing to do

    def finish(n=4, n_grad=2, hidden=8, rank=0, world=2, acc=None):
        return lib.talm_head_shard_finish_scatter(None, 8, None, n, n_grad, hidden, 100, 0, 64,
                                                  None, acc, None, None, 0, None, None, None,
                                                  None, rank, world, None, 1, None)
    assert finish(n_grad=5) == 1                 # more gradient rows than rows
    assert finish(rank=2) == 1                   # rank outside the group
    assert finish(hidden=12) == 1                # hidden columns: multiples of 8
    assert finish() == 1                         # null peer table, statistics and acc
    assert b"null" in lib.talm_last_error()
