"""NF4 dequantisation on the GPU through the C ABI, bit for bit against the oracle and the
golden fixtures (torch.equal, as the reference's tests assert: solution/test_kernels.py:580-600,
:1015-1034; solution/test_fuzz.py:889-918, :949-1030)."""

import os
import random
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fp16_bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def test_golden_fp32_absmax_cases(golden_dir):
    from talm_b200.nf4_dequant import nf4_dequantize

    g = np.load(os.path.join(golden_dir, "nf4_fp32.npz"))
    for i in range(int(g["n_cases"])):
        rows, cols, bs = (int(v) for v in g[f"c{i}_meta"])
        packed = torch.from_numpy(g[f"c{i}_packed"]).to(DEV)
        absmax = torch.from_numpy(g[f"c{i}_absmax"]).to(DEV)
        out = torch.full((rows, cols), float("nan"), dtype=torch.float16, device=DEV)
        nf4_dequantize(packed, absmax, bs, out)
        assert np.array_equal(_fp16_bits(out).reshape(-1), g[f"c{i}_expected"]), f"case {i}"


@pytest.mark.parametrize("shape", [(8960, 1536), (256, 1536), (1536, 8960), (64, 4094)])
def test_reference_shapes_bit_exact(shape):
    """solution/test_kernels.py:580 shapes, blocksize 64."""
    from talm_b200.nf4_dequant import nf4_dequantize

    rng = np.random.default_rng(4)
    n = shape[0] * shape[1]
    packed = rng.integers(0, 256, n // 2, dtype=np.uint8)
    absmax = rng.uniform(0.001, 0.2, (n + 63) // 64).astype(np.float32)
    out = torch.empty(shape, dtype=torch.float16, device=DEV)
    nf4_dequantize(torch.from_numpy(packed).to(DEV), torch.from_numpy(absmax).to(DEV), 64, out)
    ref = onf4.dequant_fp32_absmax(packed, absmax, 64, n)
    assert np.array_equal(_fp16_bits(out).reshape(-1), ref.view(np.uint16))


def test_fuzz_block_sizes_alignments_and_tails():
    """Random sizes, every bitsandbytes block size plus odd even ones, and pointers off the
    16-byte grid (the byte-granular path) - all bit-exact."""
    from talm_b200.nf4_dequant import nf4_dequantize

    r = random.Random("nf4-fuzz")
    for case in range(60):
        bs = r.choice([64, 64, 128, 256, 512, 1024, 2048, 4096, 2, 6, 8, 32, 192])
        n = 2 * r.randint(1, 300_000)
        rng = np.random.default_rng(case)
        packed = rng.integers(0, 256, n // 2 + 8, dtype=np.uint8)
        absmax = rng.uniform(0.0, 0.5, (n + bs - 1) // bs + 1).astype(np.float32)
        pk_off = r.choice([0, 0, 0, 1, 3, 4])
        out_off = r.choice([0, 0, 0, 1, 8])
        pk = torch.from_numpy(packed).to(DEV)[pk_off:pk_off + n // 2]
        am = torch.from_numpy(absmax).to(DEV)
        base = torch.full((n + out_off,), float("nan"), dtype=torch.float16, device=DEV)
        out = base[out_off:]
        nf4_dequantize(pk, am, bs, out)
        ref = onf4.dequant_fp32_absmax(packed[pk_off:pk_off + n // 2], absmax, bs, n)
        assert np.array_equal(_fp16_bits(out), ref.view(np.uint16)), \
            f"case {case}: n={n} bs={bs} offsets={pk_off},{out_off}"


def _qwen_layer(seed, qblock=64, qblock2=256, device=DEV):
    """Seven Qwen2.5-1.5B projections as SimpleNamespace modules with seeded NF4 data."""
    shapes = [(1536, 1536), (256, 1536), (256, 1536), (1536, 1536), (8960, 1536), (8960, 1536),
              (1536, 8960)]
    return _layer(seed, shapes, qblock, qblock2, device)


def _layer(seed, shapes, qblock, qblock2, device):
    g = torch.Generator().manual_seed(seed)
    code = torch.sort(torch.rand(256, generator=g) * 2 - 1).values
    code[0], code[-1] = -1.0, 1.0
    mods, raw = [], []
    for o, n_in in shapes:
        n = o * n_in
        packed = torch.randint(0, 256, (n // 2, 1), generator=g, dtype=torch.uint8)
        absmax8 = torch.randint(0, 256, (n // qblock,), generator=g, dtype=torch.uint8)
        absmax2 = torch.rand(n // (qblock * qblock2), generator=g) * 0.19 + 0.01
        offset = torch.rand((), generator=g) * 0.04 + 0.01
        raw.append((packed.numpy().reshape(-1).copy(), absmax8.numpy().copy(),
                    absmax2.numpy().copy(), float(offset)))
        packed = packed.to(device)
        packed.quant_state = SimpleNamespace(
            quant_type="nf4", nested=True, blocksize=qblock, shape=torch.Size([o, n_in]),
            absmax=absmax8.to(device), offset=offset.to(device),
            state2=SimpleNamespace(blocksize=qblock2, code=code.to(device),
                                   absmax=absmax2.to(device)))
        mods.append(SimpleNamespace(weight=packed, bias=None))
    return mods, raw, code.numpy()


def _expected(raw, code, qblock, qblock2):
    outs = []
    for packed, absmax8, absmax2, offset in raw:
        off2 = np.full(absmax2.shape, offset, dtype=np.float32)
        outs.append(onf4.group_dequant(packed, absmax8, code, absmax2, off2, absmax8.size,
                                       qblock, qblock2))
    return outs


def test_group_golden_layer(golden_dir):
    from talm_b200.qgroup import LayerGroup

    g = np.load(os.path.join(golden_dir, "nf4_group.npz"))
    qblock, qblock2 = int(g["qblock"]), int(g["qblock2"])
    code = torch.from_numpy(g["code"]).to(DEV)
    mods = []
    for i, (o, n_in) in enumerate(g["shapes"]):
        packed = torch.from_numpy(g[f"p{i}_packed"].copy()).to(DEV).view(-1, 1)
        packed.quant_state = SimpleNamespace(
            quant_type="nf4", nested=True, blocksize=qblock, shape=torch.Size([int(o), int(n_in)]),
            absmax=torch.from_numpy(g[f"p{i}_absmax8"].copy()).to(DEV),
            offset=torch.tensor(float(g[f"p{i}_offset"]), device=DEV),
            state2=SimpleNamespace(blocksize=qblock2, code=code.clone(),
                                   absmax=torch.from_numpy(g[f"p{i}_absmax2"].copy()).to(DEV)))
        mods.append(SimpleNamespace(weight=packed, bias=None))
    group = LayerGroup(mods)
    full = group.dequantize_all()
    for i in range(7):
        piece = full[group.elem_bounds[i]:group.elem_bounds[i + 1]]
        assert np.array_equal(_fp16_bits(piece), g[f"p{i}_expected"]), f"projection {i}"
        if group.splittable:
            assert np.array_equal(_fp16_bits(group.dequantize_one(i)).reshape(-1),
                                  g[f"p{i}_expected"]), f"slice launch {i}"


@pytest.mark.parametrize("seed", [3, 4])
def test_group_qwen_layer_bit_exact(seed):
    """The Qwen2.5-1.5B layer (46.8 M weights) with double-quantised absmax: the whole-layer
    launch and every per-projection launch equal the oracle bit for bit."""
    from talm_b200.qgroup import LayerGroup

    mods, raw, code = _qwen_layer(seed)
    group = LayerGroup(mods)
    assert group.n_pairs * 2 == 46_792_704
    full = group.dequantize_all()
    expected = _expected(raw, code, 64, 256)
    for i, ref in enumerate(expected):
        piece = full[group.elem_bounds[i]:group.elem_bounds[i + 1]]
        assert np.array_equal(_fp16_bits(piece), ref.view(np.uint16)), f"projection {i}"
        if group.splittable:
            one = group.dequantize_one(i)
            assert np.array_equal(_fp16_bits(one).reshape(-1), ref.view(np.uint16))


def test_group_random_layers_and_block_sizes():
    """solution/test_fuzz.py:949-1030 style: random conforming shapes, qblock 64/128/256."""
    from talm_b200.qgroup import LayerGroup

    r = random.Random("group-dequant")
    for case in range(12):
        qblock = r.choice([64, 64, 128, 256])
        double = qblock * 256
        shapes = []
        for _ in range(7):
            n_in = r.choice([64, 128, 256, 512, 1536, 192, 320])
            step = double // np.gcd(n_in, double)
            shapes.append((int(step * r.randint(1, max(1, 1024 // step))), n_in))
        mods, raw, code = _layer(case, shapes, qblock, 256, DEV)
        try:
            group = LayerGroup(mods)
        except ValueError:
            continue  # the reference's tiling check; its layers take the per-projection path
        full = group.dequantize_all()
        for i, ref in enumerate(_expected(raw, code, qblock, 256)):
            piece = full[group.elem_bounds[i]:group.elem_bounds[i + 1]]
            assert np.array_equal(_fp16_bits(piece), ref.view(np.uint16)), f"case {case} p{i}"


def test_group_linear_launches_once_per_pass(monkeypatch):
    """Forward: one grouped launch for the seven projections; backward: one more; outputs and
    input gradients equal F.linear on the oracle's weights (solution/test_kernels.py:1037-1098)."""
    from talm_b200 import qgroup
    from talm_b200.qgroup import GroupLinear, LayerGroup

    monkeypatch.setattr(qgroup, "SPLIT_LAYERS", {"fwd": 0, "bwd": 0})
    shapes = [(256, 256), (64, 256), (64, 256), (256, 256), (512, 256), (512, 256), (256, 512)]
    mods, raw, code = _layer(12, shapes, 64, 256, DEV)
    refs = [torch.from_numpy(w.view(np.float16).copy()).view(s).to(DEV)
            for w, s in zip(_expected(raw, code, 64, 256), shapes)]
    group = LayerGroup(mods)
    launches = {"n": 0}
    original = LayerGroup.dequantize_all

    def counted(self):
        launches["n"] += 1
        return original(self)

    monkeypatch.setattr(LayerGroup, "dequantize_all", counted)
    torch.manual_seed(0)
    x = torch.randn(3, 40, 256, device=DEV, dtype=torch.float16, requires_grad=True)
    h = torch.randn(3, 40, 512, device=DEV, dtype=torch.float16, requires_grad=True)
    inputs = [x] * 6 + [h]
    outs = []
    group.start_forward()
    for i, inp in enumerate(inputs):
        group.expected_bwd += 1
        outs.append(GroupLinear.apply(inp, group, i))
    assert launches["n"] == 1 and group.cache["fwd"][0] is None
    for o, inp, w in zip(outs, inputs, refs):
        assert torch.equal(o, F.linear(inp, w))
    sum((o.float() ** 2).mean() for o in outs).backward()
    assert launches["n"] == 2 and group.cache["bwd"][0] is None
    x2 = x.detach().clone().requires_grad_(True)
    h2 = h.detach().clone().requires_grad_(True)
    sum((F.linear(inp, w).float() ** 2).mean()
        for inp, w in zip([x2] * 6 + [h2], refs)).backward()
    assert torch.equal(x.grad, x2.grad) and torch.equal(h.grad, h2.grad)


@pytest.mark.parametrize("n_tokens", [2048, 37])
def test_fused_linear_matches_dequant_and_cublas(n_tokens):
    """The fused NF4 dequant + tcgen05 GEMM (talm_nf4_linear) on the Qwen layer's spans (q|k|v
    with bias, o, gate|up, down, k alone), forward and input gradient, against F.linear / matmul
    on the grouped kernel's dequantised weights. Both accumulate in fp32 and round once to fp16;
    they agree to an fp16 ulp (measured: bit-identical on almost every element)."""
    from talm_b200 import _lib
    from talm_b200.qgroup import LayerGroup, fused_linear

    mods, _, _ = _qwen_layer(5)
    group = LayerGroup(mods)
    full = group.dequantize_all()
    torch.manual_seed(1)
    for first, last in ((0, 3), (3, 4), (4, 6), (6, 7), (1, 2)):
        rows = sum(group.shapes[i][0] for i in range(first, last))
        cols = group.shapes[first][1]
        w = full[group.elem_bounds[first]:group.elem_bounds[last]].view(rows, cols)
        x = torch.randn(n_tokens, cols, device=DEV, dtype=torch.float16)
        bias = (torch.randn(rows, device=DEV) * 0.1).half() if first == 0 else None
        ref = F.linear(x, w, bias)
        out = fused_linear(x, group, first, last, bias=bias)
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-3,
                                   atol=float(ref.abs().max()) * 1e-3)
        g = torch.randn(n_tokens, rows, device=DEV, dtype=torch.float16)
        ref = g @ w
        out = fused_linear(g, group, first, last, transpose=True)
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-3,
                                   atol=float(ref.abs().max()) * 1e-3)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
