"""NF4 dequantisation restated in numpy - TEST INFRASTRUCTURE (oracle), not product code.

Byte/integer work with one fp32 product and one fp16 rounding per element, so numpy gives the
exact answer: numpy's float32 multiply is IEEE round-to-nearest-even and its float32 -> float16
conversion rounds to nearest even, which is what the reference's kernels compute
(tl.float32 product, `.to(tl.float16)`).
"""

import numpy as np

# solution/nf4_dequant.py:32-35 (NF4_TABLE) == solution/qgroup.py:60-63 (NF4_LEVELS)
NF4_LEVELS = np.array([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                       -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                       0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
                       0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                       0.7229568362236023, 1.0], dtype=np.float32)


def unpack_levels(packed, n_elems, levels=NF4_LEVELS):
    """fp32 levels of the n_elems codes: element 2i = high nibble of byte i, 2i+1 = low nibble
    (solution/nf4_dequant.py:49, :64; solution/test_fuzz.py:866)."""
    codes = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(codes.size * 2, dtype=np.float32)
    out[0::2] = levels[codes >> 4]
    out[1::2] = levels[codes & 15]
    return out[:n_elems]


def dequant_fp32_absmax(packed, absmax, blocksize, n_elems, levels=NF4_LEVELS):
    """fp16(level * absmax[e // blocksize]) (solution/test_fuzz.py:860-869, the per-projection
    kernel nf4_dequant.py:38-80)."""
    vals = unpack_levels(packed, n_elems, levels)
    scale = np.repeat(np.asarray(absmax, dtype=np.float32), blocksize)[:n_elems]
    return (vals * scale).astype(np.float16)


def double_quant_absmax(absmax8, code, absmax2, offset2, qblock2):
    """fp32(fp32(code[absmax8] * absmax2[r // qblock2]) + offset2[r // qblock2]): two separate
    roundings, no fused multiply-add (solution/qgroup.py:82-83 with enable_fp_fusion=False,
    :99; bitsandbytes' dequantize_blockwise + offset)."""
    a8 = np.asarray(absmax8, dtype=np.uint8).reshape(-1)
    rows = np.arange(a8.size) // qblock2
    prod = np.asarray(code, dtype=np.float32)[a8] * np.asarray(absmax2, dtype=np.float32)[rows]
    return (prod.astype(np.float32) + np.asarray(offset2, dtype=np.float32)[rows]).astype(
        np.float32)


def group_dequant(packed, absmax8, code, absmax2, offset2, n_rows, qblock, qblock2,
                  levels=NF4_LEVELS):
    """The grouped kernel's output over n_rows absmax blocks (solution/qgroup.py:72-91)."""
    scale = double_quant_absmax(np.asarray(absmax8).reshape(-1)[:n_rows], code, absmax2, offset2,
                                qblock2)
    return dequant_fp32_absmax(np.asarray(packed).reshape(-1)[:n_rows * qblock // 2], scale,
                               qblock, n_rows * qblock, levels)
