"""The QLoRA step (talm_b200/qlora.py) with both hot paths plugged in.

CPU tests run the whole step on a tiny Qwen2 (V=1000, H=512, 3 layers, the size of the
reference's own end-to-end parity model: solution/test_parity.py:1-60) with the grouped kernel's
launch replaced by the oracle, and compare it with a twin model whose projections are plain fp16
`nn.Linear` modules holding the same dequantised weights: the packing, the pass bookkeeping,
the adapters and the hooks must give the same loss and the same adapter gradients, bit for bit.
The GPU test runs the real kernels and the fused head against the twin with the transformers
loss on materialised logits."""

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4
from talm_b200 import qgroup, qlora
from talm_b200.engaged import RAN

TINY = dict(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
            num_attention_heads=8, num_key_value_heads=2)


def _oracle_launch(packed, absmax8, code, absmax2, offset2, levels, out, n_rows, qblock, qblock2):
    full = onf4.group_dequant(packed.cpu().numpy(), absmax8.cpu().numpy(), code.cpu().numpy(),
                              absmax2.cpu().numpy(), offset2.cpu().numpy(), n_rows, qblock,
                              qblock2)
    out.copy_(torch.from_numpy(full[:out.numel()]))


def _dense_weights(group):
    full = onf4.group_dequant(group.packed.cpu().numpy(), group.absmax8.cpu().numpy(),
                              group.code.cpu().numpy(), group.absmax2.cpu().numpy(),
                              group.offset2.cpu().numpy(), group.n_rows, group.qblock,
                              group.qblock2)
    return [torch.from_numpy(full[a:b].copy()).view(shape) for a, b, shape in
            zip(group.elem_bounds[:-1], group.elem_bounds[1:], group.shapes)]


def _twin(config, device, **kwargs):
    """The same model (same seed) with every 4-bit projection a plain fp16 nn.Linear holding the
    oracle's dequantised weight (and the same bias), no layer groups."""
    model = qlora.build_model(config, device, **kwargs)
    for layer in model.model.layers:
        group = layer._talm_layer_group
        for path, weight, bias in zip(qgroup.PROJECTIONS, _dense_weights(group), group.biases):
            holder = qlora._child(layer, path)
            dense = torch.nn.Linear(weight.shape[1], weight.shape[0], bias=bias is not None,
                                    dtype=torch.float16, device=device)
            dense.weight.data.copy_(weight)
            if bias is not None:
                dense.bias.data.copy_(bias)
            dense.requires_grad_(False)
            if isinstance(holder, qlora.LoraLinear):
                holder.base = dense
            else:
                qlora._replace(layer, path, dense)
        layer._talm_layer_group = None
    return model


def _grads(model):
    return {n: p.grad.clone() for n, p in model.named_parameters() if p.requires_grad}


def test_projection_shapes_of_the_qwen_layer():
    shapes = qlora.projection_shapes(qlora.qwen25_15b_config())
    assert list(shapes) == list(qgroup.PROJECTIONS)
    assert sum(o * i for o, i in shapes.values()) == 46_792_704


def test_make_batch_pads_the_tail_of_each_row():
    batch = qlora.make_batch(4, 512, 151936, "cpu", seed=3)
    mask, labels, ids = batch["attention_mask"], batch["labels"], batch["input_ids"]
    assert mask.shape == labels.shape == ids.shape == (4, 512)
    assert torch.equal(labels == -100, mask == 0)
    assert torch.equal(labels[mask == 1], ids[mask == 1])
    for row in mask:
        n = int(row.sum())
        assert n > 0 and row[:n].all() and not row[n:].any()
    assert abs(float((mask == 0).float().mean()) - 0.45) < 0.01


def test_build_model_trains_only_the_adapters():
    model = qlora.build_model(qlora.qwen25_15b_config(**TINY), "cpu")
    names = [n for n, p in model.named_parameters() if p.requires_grad]
    assert len(names) == TINY["num_hidden_layers"] * 2 * 2
    assert all(n.endswith(("lora_A", "lora_B")) for n in names)
    for layer in model.model.layers:
        group = layer._talm_layer_group
        assert group is not None and group.depth == TINY["num_hidden_layers"] - 1 - \
            layer.self_attn.layer_idx
        assert layer.self_attn.q_proj.base.weight.untyped_storage().data_ptr() == \
            group.packed.untyped_storage().data_ptr()
        assert float(layer.self_attn.v_proj.lora_B.detach().abs().sum()) == 0.0


def test_step_equals_plain_linear_twin_on_cpu(monkeypatch):
    """Two steps of the 4-bit model (oracle launch) and of the dense twin: identical losses,
    adapter gradients and updated adapters; each layer dequantised once per pass (grouped, or
    per projection in the split passes of the last layers)."""
    monkeypatch.setattr(qgroup, "launch", _oracle_launch)
    config = qlora.qwen25_15b_config(**TINY)
    kw = dict(seed=5, lora_dropout=0.0, lora_b_std=0.02)
    model, twin = qlora.build_model(config, "cpu", **kw), _twin(config, "cpu", **kw)
    qlora.patch()
    model.train()
    twin.train()
    batch = qlora.make_batch(2, 64, TINY["vocab_size"], "cpu", seed=1)
    opts = [torch.optim.AdamW(qlora.adapters(m), lr=1e-3) for m in (model, twin)]
    n_layers = TINY["num_hidden_layers"]
    for _ in range(2):
        before = dict(RAN)
        losses, grads = [], []
        for m, opt in zip((model, twin), opts):
            out = m(**batch)
            out.loss.backward()
            grads.append(_grads(m))
            opt.step()
            opt.zero_grad(set_to_none=True)
            losses.append(out.loss.detach())
        assert torch.equal(losses[0], losses[1])
        assert grads[0].keys() == grads[1].keys()
        for name in grads[0]:
            assert torch.equal(grads[0][name], grads[1][name]), name
            assert bool(grads[0][name].abs().sum() > 0), name
        grouped = RAN["group"] - before.get("group", 0)
        split = RAN["split"] - before.get("split", 0)
        assert grouped * qgroup.NSEG + split == 2 * n_layers * qgroup.NSEG
    for (na, a), (nb, b) in zip(model.named_parameters(), twin.named_parameters()):
        if a.requires_grad:
            assert torch.equal(a, b), na


def test_prepared_mask_gives_the_decoder_the_same_output(monkeypatch):
    """The 4-D mask the graphed step passes equals what transformers builds from the [B, S] mask:
    the same hidden states, bit for bit (pad rows included)."""
    monkeypatch.setattr(qgroup, "launch", _oracle_launch)
    model = qlora.build_model(qlora.qwen25_15b_config(**TINY), "cpu", seed=3, lora_dropout=0.0,
                              lora_b_std=0.02)
    qlora.patch()
    batch = qlora.make_batch(3, 40, TINY["vocab_size"], "cpu", seed=2)
    with torch.no_grad():
        two = model.model(input_ids=batch["input_ids"], attention_mask=batch["attention_mask"],
                          use_cache=False).last_hidden_state
        four = qlora._Decoder(model)(batch["input_ids"],
                                     qlora.causal_padding_mask(batch["attention_mask"]))
    assert torch.equal(two, four)
    assert qlora.labelled_count(batch["labels"]) == int(
        (torch.nn.functional.pad(batch["labels"], (0, 1), value=-100)[:, 1:] >= 0).sum())


def test_pack_batch_keeps_each_rows_tokens_positions_and_targets():
    batch = qlora.make_batch(4, 64, TINY["vocab_size"], "cpu", seed=6)
    packed = qlora.pack_batch(batch, "cpu", bucket=32)
    mask, ids = batch["attention_mask"].bool(), batch["input_ids"]
    shift = torch.nn.functional.pad(batch["labels"], (0, 1), value=-100)[:, 1:]
    n_real = int(mask.sum())
    total = packed["input_ids"].shape[1]
    assert packed["n_real"] == n_real and total % 32 == 0 and total - n_real < 32
    at = 0
    for row in range(4):
        n = int(mask[row].sum())
        assert torch.equal(packed["input_ids"][0, at:at + n], ids[row, :n])
        assert torch.equal(packed["position_ids"][0, at:at + n], torch.arange(n))
        assert torch.equal(packed["targets"][at:at + n], shift[row, :n])
        assert int(packed["targets"][at + n - 1]) == -100
        assert (packed["segments"][at:at + n] == row).all()
        at += n
    assert (packed["targets"][at:] == -100).all() and (packed["segments"][at:] == 4).all()
    assert packed["n_labelled"] == int((shift >= 0).sum())


def test_packed_decoder_matches_the_padded_rows(monkeypatch):
    """The decoder over the packed real tokens (block-causal mask, per-row positions) gives the
    padded batch's hidden states at the real positions, and the same next-token loss (fp16 on
    the CPU: within fp16 rounding of differently blocked GEMMs)."""
    monkeypatch.setattr(qgroup, "launch", _oracle_launch)
    model = qlora.build_model(qlora.qwen25_15b_config(**TINY), "cpu", seed=8, lora_dropout=0.0,
                              lora_b_std=0.02)
    qlora.patch()
    batch = qlora.make_batch(3, 48, TINY["vocab_size"], "cpu", seed=9)
    packed = qlora.pack_batch(batch, "cpu", bucket=16)
    with torch.no_grad():
        padded = qlora._Decoder(model)(batch["input_ids"],
                                       qlora.causal_padding_mask(batch["attention_mask"]))
        flat = qlora._Decoder(model)(packed["input_ids"],
                                     qlora.block_causal_mask(packed["segments"]),
                                     packed["position_ids"])
    real = flat[0, :packed["n_real"]].float()
    ref = padded[batch["attention_mask"].bool()].float()
    torch.testing.assert_close(real, ref, rtol=2e-2, atol=2e-2)
    w = model.lm_head.weight.float()
    shift = torch.nn.functional.pad(batch["labels"], (0, 1), value=-100)[:, 1:].reshape(-1)
    loss_padded = torch.nn.functional.cross_entropy(padded.reshape(-1, padded.shape[-1]).float()
                                                    @ w.t(), shift, ignore_index=-100)
    loss_packed = torch.nn.functional.cross_entropy(flat[0].float() @ w.t(), packed["targets"],
                                                    ignore_index=-100)
    torch.testing.assert_close(loss_packed, loss_padded, rtol=1e-3, atol=0)


def test_train_step_reduces_the_loss_with_dropout(monkeypatch):
    monkeypatch.setattr(qgroup, "launch", _oracle_launch)
    model = qlora.build_model(qlora.qwen25_15b_config(**TINY), "cpu", seed=2, lora_dropout=0.1)
    qlora.patch()
    model.train()
    opt = torch.optim.AdamW(qlora.adapters(model), lr=5e-3)
    batch = qlora.make_batch(2, 32, TINY["vocab_size"], "cpu", seed=4)
    losses = [float(qlora.train_step(model, opt, batch)) for _ in range(4)]
    assert all(np.isfinite(losses)) and losses[-1] < losses[0]


@pytest.mark.gpu
def test_step_on_the_gpu_matches_the_dense_twin():
    """The real grouped kernel and the fused head against the dense twin with transformers' loss
    on materialised fp16 logits: loss within 1e-3 relative, adapter gradients within 2e-2 in
    relative norm (the head's dH differs from autograd's through fp16 logits by fp16 roundings),
    the same after an optimizer step."""
    torch.manual_seed(0)
    config = qlora.qwen25_15b_config(**TINY)
    kw = dict(seed=7, lora_dropout=0.0, lora_b_std=0.02)
    model, twin = qlora.build_model(config, "cuda", **kw), _twin(config, "cuda", **kw)
    qlora.patch()
    model.train()
    twin.train()
    batch = qlora.make_batch(4, 128, TINY["vocab_size"], "cuda", seed=1)
    RAN.clear()
    for _ in range(2):
        out = model(**batch)
        assert out.logits is None
        out.loss.backward()
        logits = twin(input_ids=batch["input_ids"],
                      attention_mask=batch["attention_mask"]).logits
        shift = torch.nn.functional.pad(batch["labels"], (0, 1), value=-100)[:, 1:]
        ref = torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                                                shift.reshape(-1), ignore_index=-100)
        ref.backward()
        torch.testing.assert_close(out.loss.detach(), ref.detach(), rtol=1e-3, atol=0)
        ga, gb = _grads(model), _grads(twin)
        for name in ga:
            err = float((ga[name] - gb[name]).norm() / gb[name].norm().clamp(min=1e-30))
            assert err < 2e-2, (name, err)
        for m in (model, twin):
            with torch.no_grad():
                for p in qlora.adapters(m):
                    p.add_(p.grad, alpha=-1e-2)
                    p.grad = None
    assert RAN["head"] >= 2 and RAN["group"] + RAN["split"] > 0


@pytest.mark.gpu
def test_graphed_step_matches_the_eager_step():
    """The step with the decoder replayed as CUDA graphs gives the eager step's losses and
    adapters over three steps (the same kernels in the same order; dropout off)."""
    config = qlora.qwen25_15b_config(**TINY)
    kw = dict(seed=11, lora_dropout=0.0, lora_b_std=0.02)
    eager, graphed = qlora.build_model(config, "cuda", **kw), qlora.build_model(config, "cuda", **kw)
    qlora.patch()
    eager.train()
    graphed.train()
    batch = qlora.make_batch(4, 128, TINY["vocab_size"], "cuda", seed=5)
    n_lab = qlora.labelled_count(batch["labels"])
    opts = [torch.optim.AdamW(qlora.adapters(m), lr=1e-3) for m in (eager, graphed)]
    step = qlora.GraphedStep(graphed, opts[1], batch)
    for _ in range(3):
        a = qlora.train_step(eager, opts[0], batch)
        b = step(batch, n_lab)
        torch.testing.assert_close(b, a, rtol=1e-5, atol=0)
    for (na, pa), (_, pb) in zip(eager.named_parameters(), graphed.named_parameters()):
        if pa.requires_grad:
            torch.testing.assert_close(pb, pa, rtol=1e-3, atol=1e-5, msg=na)


@pytest.mark.gpu
def test_packed_steps_match_the_padded_step():
    """The packed step (real tokens only), eager and with the decoder as CUDA graphs, against the
    padded eager step on the same batch: the same loss within 2e-3, adapter gradients within
    3e-2 in relative norm; packed graphed equals packed eager."""
    config = qlora.qwen25_15b_config(**TINY)
    kw = dict(seed=13, lora_dropout=0.0, lora_b_std=0.02)
    models = [qlora.build_model(config, "cuda", **kw) for _ in range(3)]
    qlora.patch()
    for m in models:
        m.train()
    host = qlora.make_batch(4, 128, TINY["vocab_size"], "cpu", seed=3)
    batch = {k: v.cuda() for k, v in host.items()}
    packed = qlora.pack_batch(host, "cuda", bucket=128)
    assert packed["n_labelled"] == qlora.labelled_count(host["labels"])
    step = qlora.GraphedStep(models[2], torch.optim.SGD(qlora.adapters(models[2]), lr=0.0))
    out = models[0](**batch)
    out.loss.backward()
    eager = qlora._packed_loss(models[1], qlora._Decoder(models[1])(
        packed["input_ids"], qlora.block_causal_mask(packed["segments"]),
        packed["position_ids"]), packed)
    eager.backward()
    graphed = step.packed(packed)
    torch.testing.assert_close(eager.detach(), out.loss.detach(), rtol=2e-3, atol=0)
    torch.testing.assert_close(graphed, eager.detach(), rtol=1e-5, atol=0)
    ga, gb = _grads(models[0]), _grads(models[1])
    for name in ga:
        err = float((gb[name] - ga[name]).norm() / ga[name].norm().clamp(min=1e-30))
        assert err < 3e-2, (name, err)


def test_device_unpad_matches_the_host_packing():
    """unpad_batch (on the batch's own device, one host read) keeps the same tokens, positions
    and targets in the same order as pack_batch, and its row bounds are the packed rows'."""
    batch = qlora.make_batch(4, 96, TINY["vocab_size"], "cpu", seed=21)
    dev = qlora.unpad_batch(batch)
    host = qlora.pack_batch(batch, "cpu", bucket=0)
    for key in ("input_ids", "position_ids", "targets"):
        assert torch.equal(dev[key], host[key]), key
    assert (dev["n_real"], dev["n_labelled"]) == (host["n_real"], host["n_labelled"])
    lengths = batch["attention_mask"].sum(1)
    assert dev["cu_seqlens"].tolist() == [0] + torch.cumsum(lengths, 0).tolist()
    assert dev["max_len"] == int(lengths.max())
    bucketed = qlora.unpad_batch(batch, bucket=64)
    total = bucketed["input_ids"].shape[1]
    assert total % 64 == 0 and total >= dev["n_real"]
    assert bucketed["cu_seqlens"].tolist()[:-1] == dev["cu_seqlens"].tolist()
    assert bucketed["cu_seqlens"].tolist()[-1] == total
    assert (bucketed["targets"][dev["n_real"]:] == -100).all()


@pytest.mark.gpu
def test_varlen_step_matches_the_padded_step():
    """The step with the padding removed on the device and variable-length attention over the
    packed rows against the padded eager step on the same batch: the same loss within 2e-3 and
    adapter gradients within 3e-2 in relative norm (as the host-packed step's test)."""
    config = qlora.qwen25_15b_config(**TINY)
    kw = dict(seed=13, lora_dropout=0.0, lora_b_std=0.02)
    models = [qlora.build_model(config, "cuda", **kw) for _ in range(2)]
    qlora.patch()
    for m in models:
        m.train()
    host = qlora.make_batch(4, 128, TINY["vocab_size"], "cpu", seed=3)
    batch = {k: v.cuda() for k, v in host.items()}
    out = models[0](**batch)
    out.loss.backward()
    packed = qlora.unpad_batch(batch)
    loss = qlora._packed_loss(models[1], qlora._varlen_hidden(models[1], packed), packed)
    loss.backward()
    torch.testing.assert_close(loss.detach(), out.loss.detach(), rtol=2e-3, atol=0)
    ga, gb = _grads(models[0]), _grads(models[1])
    for name in ga:
        err = float((gb[name] - ga[name]).norm() / ga[name].norm().clamp(min=1e-30))
        assert err < 3e-2, (name, err)
    # a whole step through the public helper runs and changes the adapters
    opt = torch.optim.SGD(qlora.adapters(models[1]), lr=1e-2)
    before = [p.detach().clone() for p in qlora.adapters(models[1])]
    assert torch.isfinite(qlora.varlen_train_step(models[1], opt, batch))
    assert any(not torch.equal(a, p) for a, p in zip(before, qlora.adapters(models[1])))
