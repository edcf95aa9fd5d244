"""Host-side logic of the drop-in modules, on CPU tensors (no kernel launches): LayerGroup packing
against the reference's, its validation, the head's denominator and row order, the vocabulary
shards, the engagement counters and apply()."""

import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from talm_b200 import fused_head, qgroup, vocab_parallel


def _modules_from_golden(g, shapes=None):
    from_fixture = shapes is None
    shapes = g["shapes"] if from_fixture else shapes
    qblock, qblock2 = int(g["qblock"]), int(g["qblock2"])
    code = torch.from_numpy(g["code"])
    mods = []
    rng = np.random.default_rng(0)
    for i, (o, n_in) in enumerate(shapes):
        n = int(o) * int(n_in)
        if from_fixture:
            packed = torch.from_numpy(g[f"p{i}_packed"].copy()).view(-1, 1)
            absmax8 = torch.from_numpy(g[f"p{i}_absmax8"].copy())
            absmax2 = torch.from_numpy(g[f"p{i}_absmax2"].copy())
            offset = torch.tensor(float(g[f"p{i}_offset"]))
        else:
            packed = torch.from_numpy(rng.integers(0, 256, (n // 2, 1), dtype=np.uint8))
            absmax8 = torch.from_numpy(rng.integers(0, 256, n // qblock, dtype=np.uint8))
            absmax2 = torch.rand(max(1, n // (qblock * qblock2)))
            offset = torch.tensor(0.01)
        state = SimpleNamespace(quant_type="nf4", nested=True, blocksize=qblock,
                                shape=torch.Size([int(o), int(n_in)]), absmax=absmax8,
                                offset=offset,
                                state2=SimpleNamespace(blocksize=qblock2, code=code.clone(),
                                                       absmax=absmax2))
        packed.quant_state = state
        mods.append(SimpleNamespace(weight=packed, bias=None))
    return mods


def test_layer_group_packing_matches_reference(golden_dir):
    """Bounds, per-block offsets, splittability and row count equal what the reference's
    LayerGroup computed for the same layer (solution/qgroup.py:124-192); the parameters become
    views of the packed buffers holding the same bytes."""
    g = np.load(os.path.join(golden_dir, "nf4_group.npz"))
    mods = _modules_from_golden(g)
    originals = [m.weight.clone() for m in mods]
    group = qgroup.LayerGroup(mods)
    assert group.pair_bounds == g["pair_bounds"].tolist()
    assert group.elem_bounds == g["elem_bounds"].tolist()
    assert group.row_bounds == g["row_bounds"].tolist()
    assert np.array_equal(group.offset2.numpy(), g["offset2"])
    assert group.splittable == bool(g["splittable"])
    assert group.n_rows == int(g["n_rows"]) and group.n_pairs == int(g["n_pairs"])
    for m, orig in zip(mods, originals):
        assert m.weight.data.untyped_storage().data_ptr() == \
            group.packed.untyped_storage().data_ptr()
        assert torch.equal(m.weight.data.view(-1), orig.view(-1))


def test_layer_group_rejects_untileable_layer_before_repacking(golden_dir):
    """A size that is not a multiple of the absmax double block raises ValueError and leaves the
    parameters untouched (the per-projection path then serves the layer)."""
    g = np.load(os.path.join(golden_dir, "nf4_group.npz"))
    mods = _modules_from_golden(g, shapes=g["bad_shapes"])
    ptrs = [(m.weight.data_ptr(), m.weight.quant_state.absmax.data_ptr()) for m in mods]
    with pytest.raises(ValueError):
        qgroup.LayerGroup(mods)
    assert ptrs == [(m.weight.data_ptr(), m.weight.quant_state.absmax.data_ptr()) for m in mods]


def test_layer_group_pass_bookkeeping_without_kernels(golden_dir, monkeypatch):
    """Forward: one dequantisation for the seven projections, buffer dropped after the 7th use.
    Backward: one per pass, sized by expected_bwd. Split passes of the last layers dequantise
    per projection (solution/qgroup.py:252-308). The kernel is replaced by a counter: this is
    the host logic only."""
    g = np.load(os.path.join(golden_dir, "nf4_group.npz"))
    group = qgroup.LayerGroup(_modules_from_golden(g))
    calls = {"all": 0, "one": 0}

    def fake_all(self):
        calls["all"] += 1
        return torch.zeros(self.n_pairs * 2, dtype=torch.float16)

    def fake_one(self, idx):
        calls["one"] += 1
        return torch.zeros(self.shapes[idx], dtype=torch.float16)

    monkeypatch.setattr(qgroup.LayerGroup, "dequantize_all", fake_all)
    monkeypatch.setattr(qgroup.LayerGroup, "dequantize_one", fake_one)
    group.start_forward()
    for i in range(7):
        assert group.weight("fwd", i).shape == group.shapes[i]
    assert calls["all"] == 1 and group.cache["fwd"][0] is None
    group.expected_bwd = 7
    for i in reversed(range(7)):
        group.weight("bwd", i)
    assert calls["all"] == 2 and group.cache["bwd"][0] is None and group.expected_bwd == 0
    # q|k|v as one span counts three uses
    group.start_forward()
    span = group.span("fwd", 0, 3)
    assert span.shape == (sum(group.shapes[i][0] for i in range(3)), group.shapes[0][1])
    assert group.cache["fwd"][1] == 4
    # split pass of the last layer
    monkeypatch.setattr(qgroup, "SPLIT_LAYERS", {"fwd": 1, "bwd": 2})
    group.start_forward()
    group.depth = 0
    if group.splittable:
        for i in range(7):
            group.weight("fwd", i)
        assert calls["one"] == 7
        assert group.span("fwd", 0, 3) is None


def test_denominator_and_backward_scale():
    count = torch.tensor(0)
    assert float(fused_head._denominator(None, count)) == 1.0
    assert float(fused_head._denominator(7, count)) == 7.0
    assert float(fused_head._denominator(torch.tensor(5), count)) == 5.0
    # the backward's semantics (the oracle restatement the GPU kernel is checked against)
    from oracle.head import scale_grad

    ones = torch.ones(2, 3, dtype=torch.float16)
    out = scale_grad(ones, torch.tensor(2.0), torch.tensor(0.0), torch.float32)
    assert out.dtype == torch.float32 and torch.equal(out, torch.zeros(2, 3))
    assert torch.equal(scale_grad(ones, torch.tensor(2.0), torch.tensor(4.0), torch.float32),
                       torch.full((2, 3), .5))
    # an fp32 gradient is rounded to fp16 first
    g = torch.tensor([[1.0 + 2 ** -13]])
    assert float(scale_grad(g, torch.tensor(1.0), torch.tensor(1.0), torch.float32)) == 1.0


def test_labelled_first_is_order_stable():
    torch.manual_seed(3)
    labelled = torch.rand(1000) < 0.4
    n_lab = int(labelled.sum())
    dest, src = fused_head.labelled_first(labelled, n_lab)
    rows = torch.arange(1000)
    assert torch.equal(src[dest], rows) and torch.equal(dest[src], rows)
    assert labelled[src[:n_lab]].all() and not labelled[src[n_lab:]].any()
    assert (src[1:n_lab] > src[:n_lab - 1]).all() and (src[n_lab + 1:] > src[n_lab:-1]).all()


@pytest.mark.parametrize("vocab,world", [(151936, 8), (151936, 3), (1000, 7), (5, 8)])
def test_shard_bounds_cover_the_vocabulary(vocab, world):
    spans = [vocab_parallel.shard_bounds(vocab, world, r) for r in range(world)]
    assert spans[0][0] == 0
    for (a, n), (b, _) in zip(spans, spans[1:]):
        assert a + n == b
    assert spans[-1][0] + spans[-1][1] == vocab
    assert max(n for _, n in spans) - min(n for _, n in spans) <= 1


def test_fused_head_refuses_cpu_tensors():
    """No CPU path: the product fails loudly on CPU tensors."""
    hidden = torch.randn(4, 16, requires_grad=True)
    weight = torch.randn(10, 16)
    targets = torch.tensor([1, 2, -100, 3])
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_head.fused_head_loss(hidden, weight, targets)


def test_apply_installs_what_is_importable():
    """apply() never raises for an absent dependency (bitsandbytes here); the fused head patch
    installs on transformers' Qwen2ForCausalLM and a second call installs nothing twice."""
    import talm_b200
    from transformers.models.qwen2 import modeling_qwen2

    before = modeling_qwen2.Qwen2ForCausalLM.forward
    try:
        talm_b200.apply()
        patched = modeling_qwen2.Qwen2ForCausalLM.forward
        assert getattr(patched, "_talm_fused_lm", False)
        talm_b200.apply()
        assert modeling_qwen2.Qwen2ForCausalLM.forward is patched
    finally:
        modeling_qwen2.Qwen2ForCausalLM.forward = before


def test_fused_linear_checks_the_span_before_any_launch(golden_dir):
    """qgroup.fused_linear refuses spans whose projections differ in input size and inputs of
    the wrong width on the host (CPU tensors: nothing reaches the library)."""
    g = np.load(os.path.join(golden_dir, "nf4_group.npz"))
    group = qgroup.LayerGroup(_modules_from_golden(g))
    # golden shapes: six projections of 256 inputs, the last of 512
    with pytest.raises(ValueError, match="share"):
        qgroup.fused_linear(torch.zeros(4, 256, dtype=torch.float16), group, 5, 7)
    with pytest.raises(ValueError, match="last dimension"):
        qgroup.fused_linear(torch.zeros(4, 128, dtype=torch.float16), group, 0, 2)
    with pytest.raises(ValueError, match="last dimension"):
        qgroup.fused_linear(torch.zeros(4, 256, dtype=torch.float16), group, 0, 2,
                            transpose=True)
    packed, absmax8, row0, rows, cols = qgroup._span(group, 4, 6)
    assert (rows, cols) == (256, 256) and row0 == group.row_bounds[4]
    assert packed.numel() == rows * cols // 2 and absmax8.numel() == rows * cols // 64
