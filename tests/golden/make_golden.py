"""Generate the golden fixtures of tests/golden/ from the reference's own Python code.

    python tests/golden/make_golden.py [/path/to/reference]

Run on a machine where the reference (otarernazar-eng/Talm) is checked out; it imports the
reference's `solution` package on CPU (triton imports without a GPU; no kernel is launched) and
records what its functions compute:

  nf4_fp32.npz     solution/test_fuzz.py:860-869 `_nf4_manual` (the NF4 format as the reference's
                   tests state it) on seeded packed bytes / fp32 absmax, several block sizes
  nf4_group.npz    a 7-projection layer packed by the reference's `LayerGroup`
                   (solution/qgroup.py:124-192) with SimpleNamespace quant states as
                   solution/test_fuzz.py:919-929 builds them; its bounds / offset2 /
                   splittable, and `_nf4_manual` of each projection with the double-quantised
                   absmax rebuilt as code[absmax8] * absmax2 + offset (qgroup.py:82-83)
  head_small.npz   solution/test_kernels.py:70-83 `reference_head` (loss, per-token loss,
                   entropy, correctness, and the hidden gradient by autograd) and
                   solution/test_fuzz.py:145-185 `_head_reference` (float64, `fragile` rows)
  labelled_first.npz  solution/fused_head.py:290-299 on a seeded mask

Inputs come from numpy's seeded PCG64 generator, so the fixtures are reproducible anywhere.
"""

import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path):
    sys.path.insert(0, path)
    import solution.fused_head as fused_head  # noqa: F401
    import solution.qgroup as qgroup  # noqa: F401
    import solution.test_fuzz as test_fuzz  # noqa: F401
    import solution.test_kernels as test_kernels  # noqa: F401
    return fused_head, qgroup, test_fuzz, test_kernels


def nf4_fp32(test_fuzz):
    rng = np.random.default_rng(20261201)
    out = {}
    cases = [((64, 254), 64), ((16, 130), 64), ((8, 512), 128), ((4, 1024), 4096),
             ((3, 2048), 2048), ((1, 64), 64), ((2, 200), 256), ((7, 96), 1024)]
    for i, (shape, bs) in enumerate(cases):
        n = shape[0] * shape[1]
        packed = rng.integers(0, 256, size=(n + 1) // 2, dtype=np.uint8)
        absmax = rng.uniform(0.01, 0.2, size=(n + bs - 1) // bs).astype(np.float32)
        if i == 0:
            absmax[:3] = [0.0, 1e-30, 65000.0]  # zero, subnormal products, fp16 overflow
        ref = test_fuzz._nf4_manual(torch.from_numpy(packed), torch.from_numpy(absmax), bs, n)
        out[f"c{i}_packed"] = packed
        out[f"c{i}_absmax"] = absmax
        out[f"c{i}_meta"] = np.array([shape[0], shape[1], bs], dtype=np.int64)
        out[f"c{i}_expected"] = ref.numpy().view(np.uint16)
    out["n_cases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "nf4_fp32.npz"), **out)


def _fake_layer(rng, shapes, qblock, qblock2):
    modules, refs = [], []
    code = np.sort(rng.uniform(-1, 1, size=256)).astype(np.float32)
    code[0], code[-1] = -1.0, 1.0
    code_t = torch.from_numpy(code)
    for i, (o, n_in) in enumerate(shapes):
        n = o * n_in
        packed = torch.from_numpy(rng.integers(0, 256, size=(n // 2, 1), dtype=np.uint8))
        absmax8 = torch.from_numpy(rng.integers(0, 256, size=n // qblock, dtype=np.uint8))
        absmax2 = torch.from_numpy(
            rng.uniform(0.01, 0.2, size=n // (qblock * qblock2)).astype(np.float32))
        offset = torch.tensor(float(rng.uniform(0.01, 0.05)), dtype=torch.float32)
        state = SimpleNamespace(quant_type="nf4", nested=True, blocksize=qblock,
                                shape=torch.Size([o, n_in]), absmax=absmax8, offset=offset,
                                state2=SimpleNamespace(blocksize=qblock2, code=code_t.clone(),
                                                       absmax=absmax2))
        packed.quant_state = state
        modules.append(SimpleNamespace(weight=packed, bias=None))
        refs.append((packed.clone(), absmax8.clone(), absmax2.clone(), offset.clone()))
    return modules, refs, code


def nf4_group(qgroup, test_fuzz):
    rng = np.random.default_rng(7)
    qblock, qblock2 = 64, 256
    shapes = [(64, 256), (64, 256), (64, 256), (64, 256), (128, 256), (128, 256), (64, 512)]
    modules, refs, code = _fake_layer(rng, shapes, qblock, qblock2)
    group = qgroup.LayerGroup(modules)
    out = {"shapes": np.array(shapes, dtype=np.int64), "qblock": np.array(qblock),
           "qblock2": np.array(qblock2), "code": code}
    for i, (packed, absmax8, absmax2, offset) in enumerate(refs):
        out[f"p{i}_packed"] = packed.numpy().reshape(-1)
        out[f"p{i}_absmax8"] = absmax8.numpy()
        out[f"p{i}_absmax2"] = absmax2.numpy()
        out[f"p{i}_offset"] = np.array(offset.item(), dtype=np.float32)
        # bitsandbytes' dequantize_blockwise (code[absmax8] * absmax2, fp32) + offset: two ops
        code_t = torch.from_numpy(code)
        absmax32 = code_t[absmax8.long()] * absmax2.repeat_interleave(qblock2)
        absmax32 = absmax32 + offset
        numel = shapes[i][0] * shapes[i][1]
        ref = test_fuzz._nf4_manual(packed, absmax32, qblock, numel)
        out[f"p{i}_expected"] = ref.numpy().view(np.uint16)
    out["pair_bounds"] = np.array(group.pair_bounds, dtype=np.int64)
    out["elem_bounds"] = np.array(group.elem_bounds, dtype=np.int64)
    out["row_bounds"] = np.array(group.row_bounds, dtype=np.int64)
    out["offset2"] = group.offset2.numpy()
    out["splittable"] = np.array(group.splittable)
    out["n_rows"] = np.array(group.n_rows)
    out["n_pairs"] = np.array(group.n_pairs)
    # a layer the grouped kernel cannot tile: one size not a multiple of the double block
    bad = list(shapes)
    bad[3] = (bad[3][0] + 8, bad[3][1])
    out["bad_shapes"] = np.array(bad, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "nf4_group.npz"), **out)


def head_small(fused_head, test_fuzz, test_kernels):
    rng = np.random.default_rng(11)
    out = {}
    cases = [(37, 4097, 32, 4096, 2.0, "int"), (5, 1000, 64, 384, 2.0, None),
             (64, 2304, 64, 1024, 1.5, "int"), (19, 600, 32, 256, 1.0, None)]
    for i, (n, vocab, size, chunk, scale, items_kind) in enumerate(cases):
        hidden = (rng.standard_normal((n, size)) * scale).astype(np.float32)
        weight = (rng.standard_normal((vocab, size)) * 0.05).astype(np.float16)
        targets = rng.integers(0, vocab, size=n).astype(np.int64)
        targets[rng.uniform(size=n) < 0.45] = -100
        targets[0] = -100
        # planted hits at slice / block edges (solution/test_kernels.py:104-131)
        cols = [c for c in (0, chunk - 1, chunk, vocab - 1, 4095, 4096) if 0 <= c < vocab]
        for j, c in enumerate(cols):
            r = 1 + j
            if r >= n - 1:
                break
            hidden[r] = weight[c].astype(np.float32) * 40.0
            targets[r] = c if j % 2 == 0 else (c + 1 if c + 1 < vocab else c - 1)
        h = torch.from_numpy(hidden.astype(np.float16)).requires_grad_(True)
        w = torch.from_numpy(weight)
        t = torch.from_numpy(targets)
        n_lab = int((t >= 0).sum())
        items = n_lab + 3 if items_kind == "int" else None
        loss, token_loss, entropy, correct = test_kernels.reference_head(h, w, t, items)
        grad_scale = 3.0
        (loss * grad_scale).backward()
        ref64 = test_fuzz._head_reference(h, w, t, items)
        out[f"c{i}_hidden"] = h.detach().numpy().view(np.uint16)
        out[f"c{i}_weight"] = weight.view(np.uint16)
        out[f"c{i}_targets"] = targets
        out[f"c{i}_meta"] = np.array([n, vocab, size, chunk, -1 if items is None else items],
                                     dtype=np.int64)
        out[f"c{i}_loss"] = np.array(loss.item(), dtype=np.float32)
        out[f"c{i}_token_loss"] = token_loss.detach().numpy()
        out[f"c{i}_entropy"] = entropy.detach().numpy()
        out[f"c{i}_correct"] = correct.numpy()
        out[f"c{i}_grad"] = h.grad.float().numpy()
        out[f"c{i}_fragile"] = ref64["fragile"].numpy()
        out[f"c{i}_grad64"] = (ref64["grad"] * (grad_scale / ref64["denom"])).float().numpy()
    out["n_cases"] = np.array(len(cases))
    out["grad_scale"] = np.array(3.0)
    np.savez_compressed(os.path.join(HERE, "head_small.npz"), **out)


def labelled_first(fused_head):
    rng = np.random.default_rng(3)
    mask = rng.uniform(size=1000) < 0.4
    lab = torch.from_numpy(mask)
    dest, src = fused_head.labelled_first(lab, int(lab.sum()))
    np.savez_compressed(os.path.join(HERE, "labelled_first.npz"), mask=mask, dest=dest.numpy(),
                        src=src.numpy())


def main():
    path = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    fused_head, qgroup, test_fuzz, test_kernels = _import_reference(path)
    torch.manual_seed(0)
    nf4_fp32(test_fuzz)
    nf4_group(qgroup, test_fuzz)
    head_small(fused_head, test_fuzz, test_kernels)
    labelled_first(fused_head)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
