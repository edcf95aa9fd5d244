"""ctypes binding of libtalm_b200.so (the C ABI declared in include/talm.h).

This is the thin layer between the PyTorch host code and the sm_100a kernels: tensors go in as
device pointers (`Tensor.data_ptr()`), the current CUDA stream as a raw handle. A missing library,
a tensor that is not on a CUDA device or a non-zero status raises: there is no CPU path.
"""

import ctypes
import os

import torch

from . import build as _build

_C = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_SZ = ctypes.c_size_t
_U32 = ctypes.c_uint32

SIGNATURES = {
    "talm_abi_version": (_INT, []),
    "talm_last_error": (ctypes.c_char_p, []),
    "talm_status_string": (ctypes.c_char_p, [_INT]),
    "talm_device_status": (_INT, [ctypes.POINTER(_INT)]),
    "talm_set_wait_limit_ns": (_INT, [ctypes.c_uint64]),
    "talm_profile_begin": (_INT, []),
    "talm_profile_end": (_INT, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_I64), _INT]),
    "talm_nf4_dequantize": (_INT, [_P, _P, _I64, _I64, _P, _P]),
    "talm_nf4_group_dequant": (_INT, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "talm_nf4_linear": (_INT, [_P, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                               _I64, _INT, _P, _P, _I64, _P]),
    "talm_head_workspace_size": (_INT, [_I64, _I64, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    "talm_head_shard": (_INT, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P,
                               _P, _P, _SZ, _P]),
    "talm_head_shard_noalloc": (_INT, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64,
                                       _I64, _P, _P, _P]),
    "talm_head_finalize": (_INT, [_P, _P, _I64, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _P,
                                  _P, _P, _P, _P, _INT, _P]),
    "talm_head_combine": (_INT, [_P, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "talm_head_scale_grad": (_INT, [_P, _I64, _INT, _P, _P, _I64, _I64, _P, _INT, _P]),
    "talm_head_labelled_first": (_INT, [_P, _I64, _I64, _P, _I64, _I64, _P, _P, _P, _P, _P]),
    "talm_peer_buffer_size": (_INT, [_I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    "talm_ipc_export": (_INT, [_P, _P, ctypes.POINTER(_I64)]),
    "talm_ipc_import": (_INT, [_P, _I64, ctypes.POINTER(_P)]),
    "talm_ipc_close": (_INT, [_P, _I64]),
    "talm_head_publish_stats": (_INT, [_P, _I64, _I64, _I64, _I64, _P, _U32, _P]),
    "talm_head_merge_peers": (_INT, [_I64, _I64, _I64, _I64, _I64, _P, _U32, _P, _P, _P]),
    "talm_head_finalize_scatter": (_INT, [_P, _P, _I64, _I64, _P, _P, _P, _I64, _I64, _I64,
                                          _I64, _P, _P, _P, _P, _I64, _I64, _P, _U32, _P]),
    "talm_head_shard_begin": (_INT, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64,
                                     _I64, _P, _P, _P, _SZ, _P]),
    "talm_head_shard_finish_scatter": (_INT, [_P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                              _P, _P, _P, _P, _SZ, _P, _P, _P, _P, _I64, _I64,
                                              _P, _U32, _P]),
    "talm_head_reduce_gather": (_INT, [_I64, _I64, _I64, _I64, _P, _U32, _P]),
    "talm_head_gather_finish": (_INT, [_I64, _I64, _I64, _P, _U32, _P, _P]),
}
IPC_HANDLE_BYTES = 64

# Mirrors include/talm.h.
HEAD_STATS = 8
STAT_M, STAT_S, STAT_T, STAT_ZT, STAT_BEST, STAT_IDX, STAT_HIT = range(7)


def library_path():
    return os.environ.get("TALM_B200_LIB", _build.LIB_PATH)


def load(path=None):
    """Load (once) and return the ctypes handle of the library, with every signature set."""
    global _C
    if _C is not None:
        return _C
    path = path or library_path()
    if not os.path.exists(path):
        raise RuntimeError(f"libtalm_b200.so not built ({path}); run `python -m talm_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _C = lib
    return lib


def check(status, what):
    if status != 0:
        lib = load()
        detail = lib.talm_last_error().decode(errors="replace")
        name = lib.talm_status_string(status).decode(errors="replace")
        raise RuntimeError(f"{what}: {name} ({status}): {detail}")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise RuntimeError("talm_b200 kernels run on CUDA tensors only (no CPU path)")
    return t.data_ptr()


def stream_of(device):
    return torch.cuda.current_stream(device).cuda_stream


KERNEL_KINDS = ("head_slice", "head_combine", "head_reserved", "head_finalize", "head_merge",
                "nf4", "nf4_tail", "head_scale", "peer_publish", "peer_reduce", "peer_finish",
                "nf4_gemm")


def profile_begin():
    check(load().talm_profile_begin(), "talm_profile_begin")


def profile_end():
    """{kind: (total device ms, launches)} of the kernels launched since profile_begin."""
    n = len(KERNEL_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (_I64 * n)()
    check(load().talm_profile_end(ms, cnt, n), "talm_profile_end")
    return {k: (ms[i], cnt[i]) for i, k in enumerate(KERNEL_KINDS)}


def device_status():
    """Read and clear the device-side status word of bounded waits (synchronises)."""
    lib = load()
    out = _INT(0)
    check(lib.talm_device_status(ctypes.byref(out)), "talm_device_status")
    return out.value
