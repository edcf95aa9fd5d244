"""The two bitsandbytes patches (solution/qgroup.py:498-545, solution/nf4_dequant.py:110-149)
exercised through a stand-in `bitsandbytes` package placed in sys.modules (bitsandbytes itself
is not installed here): which calls they take over, which they leave to bitsandbytes (counted
as FELL_BACK), and that what they compute equals bitsandbytes' arithmetic bit for bit.

The stand-in's `_dequantize_4bit_impl` is the reference's NF4 formula in torch (the oracle's
`_nf4_manual`, solution/test_fuzz.py:860-869: level of each nibble, high nibble first, times the
block's fp32 absmax, one rounding to fp16); its `Linear4bit.forward` records that it ran. Test
infrastructure only."""

import sys
import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import nf4 as onf4
from talm_b200 import engaged, nf4_dequant, qgroup
from talm_b200.nf4_dequant import NF4_TABLE

HAS_GPU = torch.cuda.is_available()


def _torch_nf4(A, absmax, blocksize, quant_type, dtype, out):
    """bitsandbytes' dequantisation restated in torch (the oracle's formula)."""
    assert quant_type == "nf4"
    levels = torch.tensor(NF4_TABLE, dtype=torch.float32, device=A.device)
    b = A.reshape(-1).to(torch.int64)
    codes = torch.stack([b >> 4, b & 15], 1).reshape(-1)[:out.numel()]
    scale = absmax.to(torch.float32).repeat_interleave(blocksize)[:out.numel()]
    out.copy_((levels[codes] * scale).to(dtype).view(out.shape))
    return out


@pytest.fixture
def fake_bnb(monkeypatch):
    """A minimal `bitsandbytes` package: backends.cuda.ops._dequantize_4bit_impl and
    nn.Linear4bit, with call logs."""
    calls = {"dequant": 0, "linear": 0}

    def original_impl(A, absmax, blocksize, quant_type, dtype, out):
        calls["dequant"] += 1
        return _torch_nf4(A, absmax, blocksize, quant_type, dtype, out)

    class Linear4bit(torch.nn.Module):
        def forward(self, x):
            calls["linear"] += 1
            return F.linear(x, self.dense_weight.to(x.dtype))

    root = types.ModuleType("bitsandbytes")
    backends = types.ModuleType("bitsandbytes.backends")
    cuda = types.ModuleType("bitsandbytes.backends.cuda")
    ops = types.ModuleType("bitsandbytes.backends.cuda.ops")
    nn = types.ModuleType("bitsandbytes.nn")
    ops._dequantize_4bit_impl = original_impl
    nn.Linear4bit = Linear4bit
    root.backends, backends.cuda, cuda.ops, root.nn = backends, cuda, ops, nn
    for name, mod in (("bitsandbytes", root), ("bitsandbytes.backends", backends),
                      ("bitsandbytes.backends.cuda", cuda),
                      ("bitsandbytes.backends.cuda.ops", ops), ("bitsandbytes.nn", nn)):
        monkeypatch.setitem(sys.modules, name, mod)
    # the decoder-layer hook is installed on transformers' class: restore it afterwards
    from transformers.models.qwen2 import modeling_qwen2

    monkeypatch.setattr(modeling_qwen2.Qwen2DecoderLayer, "forward",
                        modeling_qwen2.Qwen2DecoderLayer.forward)
    engaged.reset()
    yield types.SimpleNamespace(ops=ops, nn=nn, calls=calls, original=original_impl)
    engaged.reset()


def test_dequant_patch_installs_once_and_leaves_cpu_calls_to_bitsandbytes(fake_bnb):
    assert nf4_dequant.patch_bnb_dequant(verify=False)
    impl = fake_bnb.ops._dequantize_4bit_impl
    assert impl is not fake_bnb.original and impl._original is fake_bnb.original
    assert nf4_dequant.patch_bnb_dequant(verify=False)  # installed: not wrapped twice
    assert fake_bnb.ops._dequantize_4bit_impl is impl
    rng = np.random.default_rng(0)
    packed = torch.from_numpy(rng.integers(0, 256, (512, 1), dtype=np.uint8))
    absmax = torch.from_numpy(rng.uniform(0.01, 0.2, 16).astype(np.float32))
    out = torch.empty(1024, dtype=torch.float16)
    impl(packed, absmax, 64, "nf4", torch.float16, out)  # a CPU tensor: bitsandbytes' path
    assert fake_bnb.calls["dequant"] == 1
    assert engaged.FELL_BACK["nf4_dequant"] == 1 and engaged.RAN["nf4_dequant"] == 0
    ref = onf4.dequant_fp32_absmax(packed.numpy().reshape(-1), absmax.numpy(), 64, 1024)
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), ref.view(np.uint16))


def test_dequant_patch_declines_without_a_gpu_to_check_on(fake_bnb, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert nf4_dequant.patch_bnb_dequant(verify=True) is False
    assert fake_bnb.ops._dequantize_4bit_impl is fake_bnb.original


def test_group_patch_installs_both_hooks_once(fake_bnb):
    from transformers.models.qwen2 import modeling_qwen2

    assert qgroup.patch_group_dequant()
    fwd = fake_bnb.nn.Linear4bit.forward
    layer_fwd = modeling_qwen2.Qwen2DecoderLayer.forward
    assert fwd._talm_group and layer_fwd._talm_group
    assert qgroup.patch_group_dequant()
    assert fake_bnb.nn.Linear4bit.forward is fwd
    assert modeling_qwen2.Qwen2DecoderLayer.forward is layer_fwd
    # an untagged module (not packed into a layer group) keeps bitsandbytes' forward
    lin = fake_bnb.nn.Linear4bit()
    lin.dense_weight = torch.randn(8, 16)
    x = torch.randn(3, 16)
    torch.testing.assert_close(lin(x), F.linear(x, lin.dense_weight))
    assert fake_bnb.calls["linear"] == 1 and engaged.FELL_BACK["group"] == 1


@pytest.mark.gpu
@pytest.mark.skipif(not HAS_GPU, reason="needs a GPU")
def test_dequant_patch_routes_nf4_fp16_cuda_calls_to_the_kernel(fake_bnb):
    assert nf4_dequant.patch_bnb_dequant(verify=True)  # the self-check against the stand-in
    impl = fake_bnb.ops._dequantize_4bit_impl
    assert fake_bnb.calls["dequant"] == 1  # the self-check's reference call
    g = torch.Generator(device="cuda").manual_seed(3)
    packed = torch.randint(0, 256, (8960 * 1536 // 2, 1), generator=g, device="cuda",
                           dtype=torch.uint8)
    absmax = torch.rand(8960 * 1536 // 64, generator=g, device="cuda") * 0.19 + 0.01
    ours = torch.empty(8960, 1536, dtype=torch.float16, device="cuda")
    assert impl(packed, absmax, 64, "nf4", torch.float16, ours) is None
    assert engaged.RAN["nf4_dequant"] == 1 and fake_bnb.calls["dequant"] == 1
    ref = _torch_nf4(packed, absmax, 64, "nf4", torch.float16, torch.empty_like(ours))
    assert torch.equal(ours, ref)
    # calls outside the kernel's case stay with bitsandbytes, each counted
    declined = [
        (packed, absmax, 64, "fp4", torch.float16, torch.empty_like(ours)),
        (packed, absmax.half(), 64, "nf4", torch.float16, torch.empty_like(ours)),
        (packed, absmax, 64, "nf4", torch.bfloat16, torch.empty_like(ours, dtype=torch.bfloat16)),
        (packed, absmax, 64, "nf4", torch.float16, torch.empty(1536, 8960, dtype=torch.float16,
                                                                device="cuda").t()),
    ]
    for i, args in enumerate(declined):
        before = fake_bnb.calls["dequant"]
        if args[3] == "fp4":
            with pytest.raises(AssertionError):  # the stand-in knows NF4 only
                impl(*args)
        else:
            impl(*args)
        assert fake_bnb.calls["dequant"] == before + 1, f"declined case {i}"
        assert engaged.FELL_BACK["nf4_dequant"] == i + 1
    assert engaged.RAN["nf4_dequant"] == 1
    # the transposed buffer got bitsandbytes' values in its own layout
    assert torch.equal(declined[3][5], ref)


@pytest.mark.gpu
@pytest.mark.skipif(not HAS_GPU, reason="needs a GPU")
def test_dequant_patch_refuses_a_kernel_that_disagrees_with_bitsandbytes(fake_bnb, monkeypatch):
    def off_by_a_bit(A, absmax, blocksize, quant_type, dtype, out):
        _torch_nf4(A, absmax, blocksize, quant_type, dtype, out)
        out.view(-1)[7] = out.view(-1)[7] + 1
        return out

    monkeypatch.setattr(fake_bnb.ops, "_dequantize_4bit_impl", off_by_a_bit)
    assert nf4_dequant.patch_bnb_dequant(verify=True) is False
    assert fake_bnb.ops._dequantize_4bit_impl is off_by_a_bit


@pytest.mark.gpu
@pytest.mark.skipif(not HAS_GPU, reason="needs a GPU")
def test_group_patch_routes_packed_fp16_modules_through_group_linear(fake_bnb, monkeypatch):
    from tests.test_nf4_gpu import _expected, _layer

    monkeypatch.setattr(qgroup, "SPLIT_LAYERS", {"fwd": 0, "bwd": 0})
    assert qgroup.patch_group_dequant()
    shapes = [(256, 256), (64, 256), (64, 256), (256, 256), (512, 256), (512, 256), (256, 512)]
    raw_mods, raw, code = _layer(21, shapes, 64, 256, "cuda")
    weights = [torch.from_numpy(w.view(np.float16).copy()).view(s).to("cuda")
               for w, s in zip(_expected(raw, code, 64, 256), shapes)]
    mods = []
    for m, w in zip(raw_mods, weights):
        lin = fake_bnb.nn.Linear4bit()
        lin.weight, lin.bias = m.weight, None
        lin.dense_weight = w
        mods.append(lin)
    group = qgroup.LayerGroup(mods)
    for idx, lin in enumerate(mods):
        lin._talm_group = (group, idx)
    group.start_forward()
    x = torch.randn(2, 9, 256, device="cuda", dtype=torch.float16, requires_grad=True)
    out = mods[4](x)  # gate: through GroupLinear, not bitsandbytes' forward
    assert fake_bnb.calls["linear"] == 0 and engaged.FELL_BACK["group"] == 0
    assert group.expected_bwd == 1
    assert torch.equal(out, F.linear(x, weights[4]))
    out.float().square().mean().backward()
    y = x.detach().clone().requires_grad_(True)
    F.linear(y, weights[4]).float().square().mean().backward()
    assert torch.equal(x.grad, y.grad)
    # an fp32 input is not the fused case: bitsandbytes' forward runs and the detour is counted
    x32 = torch.randn(4, 256, device="cuda")
    torch.testing.assert_close(mods[4](x32), F.linear(x32, weights[4].float()))
    assert fake_bnb.calls["linear"] == 1 and engaged.FELL_BACK["group"] == 1
