"""Per-projection NF4 -> fp16 dequantisation on sm_100a (drop-in for solution/nf4_dequant.py).

`nf4_dequantize(packed, absmax, blocksize, out)` keeps the reference's signature and contract
(solution/nf4_dequant.py:83-91): packed uint8 (any shape, flattened), fp32 absmax per block of
`blocksize` elements, a contiguous fp16 `out` with an even number of elements, filled in place
and returned. Byte i holds element 2i in its high nibble and 2i+1 in its low nibble; each value
is fp16(level * absmax) with the product rounded to fp32 first. The work is one launch of the
bandwidth-bound kernel in csrc/nf4.cu (no Triton, no CPU path).

`patch_bnb_dequant()` routes bitsandbytes' `_dequantize_4bit_impl` through it for NF4 fp16 on
CUDA, after a bit-exact self-check against bitsandbytes' own kernel (nf4_dequant.py:94-149).

Interface and semantics follow otarernazar-eng/Talm's solution/nf4_dequant.py (Apache License
2.0, "Soup Kernel Challenge starter kit", Copyright 2026 Makazhan Alpamys and the Soup
contributors): the function names and signatures, the NF4 level table and the set of calls
that the patch takes over are that file's.
"""

import torch

from . import _lib
from .engaged import FELL_BACK, ON, RAN
from .state import DISABLED, fallback

BLOCK = 2048  # reference launch granularity (pairs per program); kept as a module constant

# The 16 NormalFloat levels (solution/nf4_dequant.py:32-35).
NF4_TABLE = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
             -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
             0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
             0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]


def nf4_dequantize(packed, absmax, blocksize, out):
    """packed: uint8 [(n+1)//2, 1] or flat; absmax: fp32 [ceil(n / blocksize)]; out: contiguous
    fp16 tensor with an even number of elements (solution/nf4_dequant.py:83-91)."""
    if out.dtype != torch.float16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous fp16 tensor")
    n = out.numel()
    if n % 2:
        raise ValueError("out must have an even number of elements")
    if absmax.dtype != torch.float32:
        raise ValueError("absmax must be fp32")
    packed = packed.contiguous().view(-1)
    absmax = absmax.contiguous()
    if packed.numel() < n // 2:
        raise ValueError(f"packed holds {packed.numel()} bytes, {n // 2} needed")
    lib = _lib.load()
    _lib.check(lib.talm_nf4_dequantize(_lib.ptr(packed), _lib.ptr(absmax), n, int(blocksize),
                                       _lib.ptr(out), _lib.stream_of(out.device)),
               "talm_nf4_dequantize")
    return out


def _self_check(original_impl):
    """Before taking over, one comparison with bitsandbytes' own kernel: a 1 M-element NF4 buffer
    of random codes with random fp32 block scales (block size 64), dequantised by both; True
    only when every fp16 bit agrees (the reference runs the same gate, nf4_dequant.py:94-107)."""
    g = torch.Generator(device="cuda").manual_seed(20260)
    n = 1 << 20
    codes = torch.randint(0, 256, (n // 2, 1), generator=g, device="cuda", dtype=torch.uint8)
    scales = torch.rand(n // 64, generator=g, device="cuda") * 0.25 + 0.005
    theirs = torch.empty(n, dtype=torch.float16, device="cuda")
    original_impl(codes, scales, 64, "nf4", torch.float16, out=theirs)
    mine = nf4_dequantize(codes, scales, 64, torch.empty_like(theirs))
    torch.cuda.synchronize()
    return torch.equal(mine, theirs)


def _covered(A, absmax, blocksize, quant_type, dtype, out):
    """Whether a bitsandbytes dequantisation call is one this kernel performs: NF4 codes on a
    CUDA device, fp32 block scales, an even block size, an fp16 result written into a
    contiguous fp16 buffer of even length, and the component not switched off. Anything else
    stays with bitsandbytes."""
    if "nf4_dequant" in DISABLED or quant_type != "nf4" or not A.is_cuda:
        return False
    if absmax.dtype is not torch.float32 or blocksize % 2 != 0:
        return False
    if dtype is not torch.float16 or out.dtype is not torch.float16:
        return False
    return out.is_contiguous() and out.numel() % 2 == 0


def patch_bnb_dequant(verify=True):
    """Route `bitsandbytes.backends.cuda.ops._dequantize_4bit_impl` through `nf4_dequantize`
    for NF4 fp16 on CUDA (solution/nf4_dequant.py:110-149). Inputs outside that case keep
    bitsandbytes' path and count as FELL_BACK; a failure of ours records the component and
    re-raises (no silent detour)."""
    try:
        import bitsandbytes.backends.cuda.ops as ops
    except Exception:  # noqa: BLE001 - bitsandbytes absent: nothing to patch
        return False
    original = ops._dequantize_4bit_impl
    if getattr(original, "_talm_patched", False):
        return True
    if verify:
        if not torch.cuda.is_available():
            return False
        try:
            if not _self_check(original):
                return False
        except Exception:  # noqa: BLE001
            return False

    def impl(A, absmax, blocksize, quant_type, dtype, out):
        if not _covered(A, absmax, blocksize, quant_type, dtype, out):
            FELL_BACK["nf4_dequant"] += 1
            return original(A, absmax, blocksize, quant_type, dtype, out=out)
        try:
            nf4_dequantize(A, absmax, blocksize, out)
        except Exception as exc:
            fallback("nf4_dequant", exc)  # recorded once, then raised: no second kernel here
            raise
        RAN["nf4_dequant"] += 1
        return None

    impl._talm_patched = True
    impl._original = original
    ops._dequantize_4bit_impl = impl
    ON.add("nf4_dequant")
    return True
