"""The NF4 double-quant storage format loader (talm_b200/nf4_format.py).

The checkpoints here are written key by key in the format bitsandbytes' `Linear4bit` state dict
uses (packed uint8 weight, coded absmax, NF4 quant_map, nested absmax and code, and the JSON
scalars tensor), from the arrays of the golden layer that the reference's `LayerGroup` packed
(tests/golden/nf4_group.npz). CPU tests cover reading, validation, the contiguous buffers, the
writer and safetensors files; the GPU test runs the grouped kernel and the NF4Linear product on
a loaded layer against the golden dequantised weights."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4
from talm_b200 import nf4_format, qgroup

PREFIX = "model.layers.0."


def _golden(golden_dir):
    return np.load(os.path.join(golden_dir, "nf4_group.npz"))


def _checkpoint(g, prefix=PREFIX, with_bias=False):
    """The golden layer in bitsandbytes' serialised form, written out explicitly."""
    sd = {}
    qblock, qblock2 = int(g["qblock"]), int(g["qblock2"])
    for i, path in enumerate(qgroup.PROJECTIONS):
        o, n_in = (int(d) for d in g["shapes"][i])
        w = f"{prefix}{path}.weight"
        sd[w] = torch.from_numpy(g[f"p{i}_packed"].copy()).view(-1, 1)
        sd[w + ".absmax"] = torch.from_numpy(g[f"p{i}_absmax8"].copy())
        sd[w + ".quant_map"] = torch.tensor(qgroup.NF4_LEVELS, dtype=torch.float32)
        sd[w + ".nested_absmax"] = torch.from_numpy(g[f"p{i}_absmax2"].copy())
        sd[w + ".nested_quant_map"] = torch.from_numpy(g["code"].copy())
        scalars = {"quant_type": "nf4", "blocksize": qblock, "dtype": "float16",
                   "shape": [o, n_in], "nested_blocksize": qblock2,
                   "nested_offset": float(g[f"p{i}_offset"]), "nested_dtype": "float32"}
        sd[w + ".quant_state.bitsandbytes__nf4"] = torch.tensor(
            list(json.dumps(scalars).encode("utf-8")), dtype=torch.uint8)
        if with_bias:
            sd[f"{prefix}{path}.bias"] = torch.arange(o, dtype=torch.float16) / 64
    return sd


def _oracle_weights(group):
    """The oracle's fp16 weights of every projection of a loaded group, from its own buffers."""
    full = onf4.group_dequant(group.packed.cpu().numpy(), group.absmax8.cpu().numpy(),
                              group.code.cpu().numpy(), group.absmax2.cpu().numpy(),
                              group.offset2.cpu().numpy(), group.n_rows, group.qblock,
                              group.qblock2)
    return [full[a:b] for a, b in zip(group.elem_bounds[:-1], group.elem_bounds[1:])]


def test_load_layer_packs_into_adopted_buffers(golden_dir):
    """The seven projections land in one buffer per array, in projection order, and the group
    adopts those buffers (every parameter and scale is a view; no concatenated copy); the
    packing bookkeeping equals the reference's for the same layer."""
    g = _golden(golden_dir)
    group, modules = nf4_format.load_layer(_checkpoint(g), PREFIX, "cpu")
    assert list(modules) == list(qgroup.PROJECTIONS)
    assert group.pair_bounds == g["pair_bounds"].tolist()
    assert group.row_bounds == g["row_bounds"].tolist()
    assert np.array_equal(group.offset2.numpy(), g["offset2"])
    assert group.splittable == bool(g["splittable"])
    ptr = group.packed.untyped_storage().data_ptr()
    ptr8 = group.absmax8.untyped_storage().data_ptr()
    ptr2 = group.absmax2.untyped_storage().data_ptr()
    for i, m in enumerate(modules.values()):
        state = m.weight.quant_state
        assert m.weight.untyped_storage().data_ptr() == ptr
        assert state.absmax.untyped_storage().data_ptr() == ptr8
        assert state.state2.absmax.untyped_storage().data_ptr() == ptr2
        assert np.array_equal(m.weight.data.view(-1).numpy(), g[f"p{i}_packed"])
        assert np.array_equal(state.absmax.numpy(), g[f"p{i}_absmax8"])
        assert (m.out_features, m.in_features) == tuple(int(d) for d in g["shapes"][i])
        assert m._talm_group == (group, i)
    # the buffers are exactly the size of the layer: nothing was concatenated around them
    assert group.packed.untyped_storage().nbytes() == group.n_pairs


def test_loaded_layer_dequantises_to_the_golden_weights(golden_dir):
    """The oracle on the loaded group's buffers gives the golden fp16 weights bit for bit."""
    g = _golden(golden_dir)
    group, _ = nf4_format.load_layer(_checkpoint(g), PREFIX, "cpu")
    for i, w in enumerate(_oracle_weights(group)):
        assert np.array_equal(w.view(np.uint16), g[f"p{i}_expected"]), f"projection {i}"


def test_unadjacent_projections_are_still_concatenated(golden_dir):
    """Modules whose tensors do not lie back to back keep the reference's concatenation."""
    g = _golden(golden_dir)
    sd = _checkpoint(g)
    mods = [nf4_format.NF4Linear(*nf4_format.read_projection(sd, f"{PREFIX}{p}."))
            for p in qgroup.PROJECTIONS]
    group = qgroup.LayerGroup(mods)
    assert group.packed.untyped_storage().data_ptr() != sd[
        f"{PREFIX}{qgroup.PROJECTIONS[0]}.weight"].untyped_storage().data_ptr()
    for i, w in enumerate(_oracle_weights(group)):
        assert np.array_equal(w.view(np.uint16), g[f"p{i}_expected"])


def test_writer_round_trip_and_safetensors(golden_dir, tmp_path):
    """layer_state_dict writes back the tensors and scalars it read; a safetensors file of the
    checkpoint loads to the same buffers, one tensor at a time."""
    from safetensors.torch import save_file

    g = _golden(golden_dir)
    sd = _checkpoint(g, with_bias=True)
    group, modules = nf4_format.load_layer(sd, PREFIX, "cpu")
    back = nf4_format.layer_state_dict(modules, PREFIX)
    assert set(back) == set(sd)
    for k, v in sd.items():
        if k.endswith(nf4_format.QUANT_STATE_KEY):
            assert nf4_format.unpack_scalars(back[k]) == nf4_format.unpack_scalars(v), k
        else:
            assert back[k].dtype == v.dtype and torch.equal(back[k], v), k
    path = str(tmp_path / "layer.safetensors")
    save_file(back, path)
    group2, modules2 = nf4_format.load_layer(path, PREFIX, "cpu")
    assert torch.equal(group2.packed, group.packed)
    assert torch.equal(group2.absmax8, group.absmax8)
    assert torch.equal(group2.absmax2, group.absmax2)
    assert torch.equal(group2.offset2, group.offset2)
    assert all(torch.equal(a, b) for a, b in zip(group2.biases, group.biases))


def test_load_layers_orders_layers_and_sets_depth(golden_dir):
    g = _golden(golden_dir)
    sd = {}
    for i in (2, 0, 1):
        sd.update(_checkpoint(g, prefix=f"model.layers.{i}."))
    assert nf4_format.layer_indices(sd) == [0, 1, 2]
    layers = nf4_format.load_layers(sd, "cpu")
    assert [grp.depth for grp, _ in layers] == [2, 1, 0]
    assert all(torch.equal(grp.packed, layers[0][0].packed) for grp, _ in layers)


def _broken(g, edit):
    sd = _checkpoint(g)
    w = f"{PREFIX}{qgroup.PROJECTIONS[3]}.weight"
    edit(sd, w)
    return sd


def _set_scalar(key, value):
    def edit(sd, w):
        scalars = nf4_format.unpack_scalars(sd[w + ".quant_state.bitsandbytes__nf4"])
        if value is None:
            del scalars[key]
        else:
            scalars[key] = value
        sd[w + ".quant_state.bitsandbytes__nf4"] = nf4_format.pack_scalars(scalars)
    return edit


@pytest.mark.parametrize("edit, message", [
    (_set_scalar("quant_type", "fp4"), "quant_type"),
    (_set_scalar("nested_blocksize", None), "double-quantised"),
    (lambda sd, w: sd.pop(w + ".nested_absmax"), "double-quantised"),
    (lambda sd, w: sd.pop(w + ".absmax"), "missing"),
    (_set_scalar("shape", [64, 255]), "expected"),
    (_set_scalar("shape", [64]), "shape"),
    (_set_scalar("dtype", "float8"), "dtypes"),
    (lambda sd, w: sd[w + ".quant_map"].__setitem__(3, 0.5), "NF4 level table"),
    (lambda sd, w: sd.__setitem__(w + ".absmax", sd[w + ".absmax"][:-1]), "expected"),
    (lambda sd, w: sd.__setitem__(w + ".nested_absmax", sd[w + ".nested_absmax"].double()),
     "expected"),
    (lambda sd, w: sd.__setitem__(w + ".quant_state.bitsandbytes__nf4",
                                  torch.tensor([0xFF, 0xFE], dtype=torch.uint8)), "not JSON"),
])
def test_malformed_projection_is_refused(golden_dir, edit, message):
    g = _golden(golden_dir)
    with pytest.raises(ValueError, match=message):
        nf4_format.load_layer(_broken(g, edit), PREFIX, "cpu")


def test_missing_projection_and_ungrouped_module_raise(golden_dir):
    g = _golden(golden_dir)
    sd = _checkpoint(g)
    del sd[f"{PREFIX}mlp.down_proj.weight"]
    with pytest.raises(KeyError, match="down_proj"):
        nf4_format.load_layer(sd, PREFIX, "cpu")
    module = nf4_format.NF4Linear(*nf4_format.read_projection(_checkpoint(g),
                                                              f"{PREFIX}self_attn.q_proj."))
    with pytest.raises(RuntimeError, match="layer group"):
        module(torch.zeros(1, module.in_features, dtype=torch.float16))


def test_untileable_layer_is_refused_by_the_group(golden_dir):
    """A layer whose sizes the grouped kernel cannot tile loads its arrays but LayerGroup
    refuses it, as it refuses the same layer built from bitsandbytes modules."""
    g = _golden(golden_dir)
    sd = _checkpoint(g)
    w = f"{PREFIX}{qgroup.PROJECTIONS[6]}.weight"
    scalars = nf4_format.unpack_scalars(sd[w + ".quant_state.bitsandbytes__nf4"])
    scalars["shape"] = [16, 512]
    sd[w + ".quant_state.bitsandbytes__nf4"] = nf4_format.pack_scalars(scalars)
    sd[w] = sd[w][:4096]
    sd[w + ".absmax"] = sd[w + ".absmax"][:128]
    sd[w + ".nested_absmax"] = sd[w + ".nested_absmax"][:1]
    with pytest.raises(ValueError, match="double-block"):
        nf4_format.load_layer(sd, PREFIX, "cpu")


@pytest.mark.gpu
def test_loaded_layer_on_the_gpu(golden_dir):
    """Loaded to the device from pinned host tensors: the grouped kernel gives the golden weights
    bit for bit, and NF4Linear's product (forward and input gradient through GroupLinear) equals
    the same product with the golden weights."""
    g = _golden(golden_dir)
    sd = {k: v.pin_memory() for k, v in _checkpoint(g, with_bias=True).items()}
    group, modules = nf4_format.load_layer(sd, PREFIX, "cuda")
    full = group.dequantize_all()
    for i in range(len(qgroup.PROJECTIONS)):
        piece = full[group.elem_bounds[i]:group.elem_bounds[i + 1]].view(torch.int16).cpu()
        assert np.array_equal(piece.numpy().view(np.uint16), g[f"p{i}_expected"]), i
    qgroup.reset_passes()
    group.start_forward()
    torch.manual_seed(0)
    for i, (path, m) in enumerate(modules.items()):
        w = torch.from_numpy(g[f"p{i}_expected"].view(np.float16).copy()).cuda()
        w = w.view(m.out_features, m.in_features)
        x = torch.randn(8, m.in_features, device="cuda", dtype=torch.float16, requires_grad=True)
        out = m(x)
        ref = torch.nn.functional.linear(x.detach(), w, m.bias)
        torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)
        grad = torch.randn_like(out)
        (dx,) = torch.autograd.grad(out, x, grad)
        torch.testing.assert_close(dx, grad @ w, rtol=1e-3, atol=1e-3)
