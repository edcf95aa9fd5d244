"""The CPU oracle pinned against the golden fixtures the reference's own functions produced
(tests/golden/make_golden.py). CPU only."""

import os

import numpy as np
import torch

from oracle import head as ohead
from oracle import nf4 as onf4


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_nf4_fp32_oracle_matches_reference_manual(golden_dir):
    """oracle.nf4.dequant_fp32_absmax == solution/test_fuzz.py:860-869 `_nf4_manual`, bit for
    bit, on every fixture case (block sizes 64..4096, odd row counts, zero / subnormal /
    overflowing scales)."""
    g = _load(golden_dir, "nf4_fp32.npz")
    for i in range(int(g["n_cases"])):
        rows, cols, bs = (int(v) for v in g[f"c{i}_meta"])
        n = rows * cols
        ours = onf4.dequant_fp32_absmax(g[f"c{i}_packed"], g[f"c{i}_absmax"], bs, n)
        assert np.array_equal(ours.view(np.uint16), g[f"c{i}_expected"]), f"case {i}"


def test_nf4_group_oracle_matches_reference(golden_dir):
    """oracle.nf4.group_dequant over the layer buffers the reference's LayerGroup packs equals
    the reference's per-projection `_nf4_manual` with the double-quantised absmax."""
    g = _load(golden_dir, "nf4_group.npz")
    qblock, qblock2 = int(g["qblock"]), int(g["qblock2"])
    shapes = g["shapes"]
    packed = np.concatenate([g[f"p{i}_packed"] for i in range(7)])
    absmax8 = np.concatenate([g[f"p{i}_absmax8"] for i in range(7)])
    absmax2 = np.concatenate([g[f"p{i}_absmax2"] for i in range(7)])
    out = onf4.group_dequant(packed, absmax8, g["code"], absmax2, g["offset2"],
                             int(g["n_rows"]), qblock, qblock2)
    bounds = g["elem_bounds"]
    for i, (o, n_in) in enumerate(shapes):
        piece = out[bounds[i]:bounds[i + 1]]
        assert piece.size == o * n_in
        assert np.array_equal(piece.view(np.uint16), g[f"p{i}_expected"]), f"projection {i}"


def test_nf4_levels_are_the_reference_table():
    from talm_b200.nf4_dequant import NF4_TABLE
    from talm_b200.qgroup import NF4_LEVELS

    assert NF4_TABLE == NF4_LEVELS
    assert np.array_equal(np.array(NF4_TABLE, dtype=np.float32), onf4.NF4_LEVELS)


def test_head_oracle_matches_reference_head(golden_dir):
    """oracle.head.reference_head against solution/test_kernels.py:70-83 `reference_head` (and
    its autograd gradient) on the fixture cases: loss / per-token loss / entropy to 1e-5
    relative, correctness exact outside the reference's fragile near-tie rows, dH within
    rtol 1e-3 + 2^-10 max|dH|."""
    g = _load(golden_dir, "head_small.npz")
    scale = float(g["grad_scale"])
    for i in range(int(g["n_cases"])):
        n, vocab, size, chunk, items = (int(v) for v in g[f"c{i}_meta"])
        hidden = torch.from_numpy(g[f"c{i}_hidden"].view(np.float16))
        weight = torch.from_numpy(g[f"c{i}_weight"].view(np.float16))
        targets = torch.from_numpy(g[f"c{i}_targets"])
        loss, token_loss, entropy, correct, grad = ohead.reference_head(
            hidden, weight, targets, None if items < 0 else items, grad_scale=scale)
        torch.testing.assert_close(loss, torch.tensor(float(g[f"c{i}_loss"])), rtol=1e-5,
                                   atol=1e-6)
        torch.testing.assert_close(token_loss, torch.from_numpy(g[f"c{i}_token_loss"]),
                                   rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(entropy, torch.from_numpy(g[f"c{i}_entropy"]), rtol=1e-5,
                                   atol=1e-5)
        ref_correct = torch.from_numpy(g[f"c{i}_correct"])
        fragile = torch.from_numpy(g[f"c{i}_fragile"])
        assert not bool(((correct != ref_correct) & ~fragile).any()), f"case {i}"
        assert int(ref_correct.sum()) > 0, "planted hits must make accuracy non-trivial"
        ref_grad = torch.from_numpy(g[f"c{i}_grad"])
        torch.testing.assert_close(grad, ref_grad, rtol=1e-3,
                                   atol=float(ref_grad.abs().max()) * 2 ** -10)
        grad64 = torch.from_numpy(g[f"c{i}_grad64"])
        torch.testing.assert_close(grad, grad64, rtol=1e-4,
                                   atol=float(grad64.abs().max()) * 2 ** -14)


def test_labelled_first_matches_reference(golden_dir):
    from talm_b200.fused_head import labelled_first

    g = _load(golden_dir, "labelled_first.npz")
    mask = torch.from_numpy(g["mask"])
    dest, src = labelled_first(mask, int(mask.sum()))
    assert np.array_equal(dest.numpy(), g["dest"])
    assert np.array_equal(src.numpy(), g["src"])
