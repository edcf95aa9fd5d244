"""The NF4 double-quant storage format, read straight into a layer's contiguous buffers.

A 4-bit checkpoint of the reference's model stores each frozen projection the way bitsandbytes
(0.50.2, the version the reference pins: README.md:58) serialises a `Linear4bit` whose
`Params4bit` carries a double-quantised `QuantState` (`QuantState.as_dict(packed=True)` under the
module's `weight.` prefix):

  <p>weight                                  uint8 [n/2, 1]  code of element 2i in the high
                                                             nibble of byte i, 2i+1 in the low
  <p>weight.absmax                           uint8 [n/qblock]  first-level block scales, coded
  <p>weight.quant_map                        fp32 [16]       the NF4 levels
  <p>weight.nested_absmax                    fp32 [n/(qblock*qblock2)]  second-level scales
  <p>weight.nested_quant_map                 fp32 [256]      code of the first-level scales
  <p>weight.quant_state.bitsandbytes__nf4    uint8 [k]       UTF-8 JSON of the scalars:
        quant_type, blocksize, dtype, shape, nested_blocksize, nested_offset, nested_dtype
  <p>bias                                    fp16 [out]      optional

The reference never reads this format itself: transformers and bitsandbytes build its
`Linear4bit` modules, and `LayerGroup` then concatenates the seven projections of a layer into
three buffers (solution/qgroup.py:124-192). `load_layer` instead allocates those three buffers
once, on the device, and copies every projection's arrays into its slice of them, so the layer
is packed with no intermediate per-projection copy and no concatenation; `LayerGroup` adopts the
buffers as they are (qgroup._joined). `NF4Linear` is the module that holds one such projection
(the attributes of `Linear4bit` that the grouped path reads) and runs its product through
`GroupLinear`, the cached grouped dequantisation. `layer_state_dict` writes the format back.
"""

import json
import re

import torch

from . import qgroup

QUANT_STATE_KEY = "quant_state.bitsandbytes__nf4"
_TENSOR_KEYS = ("absmax", "quant_map", "nested_absmax", "nested_quant_map")
_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


class QuantState:
    """The quantisation state of one NF4 weight, with the attribute names of bitsandbytes'
    `QuantState` that `LayerGroup` reads (quant_type, blocksize, shape, dtype, absmax, code,
    offset, nested, state2). `state2` is a QuantState of the first-level scales (its own
    blocksize, code table and fp32 absmax); it is None for a weight that is not
    double-quantised."""

    def __init__(self, absmax, blocksize, code, dtype, quant_type=None, shape=None, offset=None,
                 state2=None):
        self.absmax, self.blocksize, self.code, self.dtype = absmax, blocksize, code, dtype
        self.quant_type, self.shape, self.offset, self.state2 = quant_type, shape, offset, state2
        self.nested = state2 is not None


def _dtype_name(dtype):
    return str(dtype).split(".")[-1]


def pack_scalars(scalars):
    """The JSON tensor bitsandbytes stores beside the arrays: uint8 bytes of json.dumps."""
    return torch.tensor(list(json.dumps(scalars).encode("utf-8")), dtype=torch.uint8)


def unpack_scalars(tensor):
    """The dictionary of `pack_scalars`' tensor."""
    if tensor.dtype != torch.uint8 or tensor.dim() != 1:
        raise ValueError("the packed quant state is not a 1-D uint8 tensor")
    try:
        return json.loads(bytes(tensor.cpu().numpy().tobytes()).decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"the packed quant state is not JSON: {exc}") from None


class _Source:
    """Tensors by name from a state-dict mapping, or lazily from a safetensors file."""

    def __init__(self, source):
        self._file = None
        if isinstance(source, str):
            from safetensors import safe_open

            self._file = safe_open(source, framework="pt", device="cpu")
            self._keys = set(self._file.keys())
        else:
            self._map = source
            self._keys = set(source.keys())

    def keys(self):
        return self._keys

    def __contains__(self, key):
        return key in self._keys

    def get(self, key):
        if key not in self._keys:
            raise KeyError(f"missing tensor {key!r}")
        return self._file.get_tensor(key) if self._file is not None else self._map[key]


def read_projection(source, prefix):
    """(packed, state, bias) of the projection stored under `prefix` ("...q_proj."), on the host
    (or wherever the mapping holds them), checked against each other. Raises ValueError for
    anything `LayerGroup` cannot run: not NF4, not double-quantised, levels that are not the NF4
    levels, sizes that disagree with the shape."""
    src = source if isinstance(source, _Source) else _Source(source)
    w = prefix + "weight"
    packed = src.get(w)
    scalars = unpack_scalars(src.get(f"{w}.{QUANT_STATE_KEY}"))
    arrays = {k: src.get(f"{w}.{k}") for k in _TENSOR_KEYS if f"{w}.{k}" in src}
    if scalars.get("quant_type") != "nf4":
        raise ValueError(f"{w}: quant_type {scalars.get('quant_type')!r}, not 'nf4'")
    if "nested_absmax" not in arrays or "nested_blocksize" not in scalars:
        raise ValueError(f"{w}: not double-quantised (no nested absmax)")
    for k in _TENSOR_KEYS:
        if k not in arrays:
            raise ValueError(f"{w}: missing {w}.{k}")
    shape = scalars.get("shape")
    if not isinstance(shape, list) or len(shape) != 2 or min(shape) <= 0:
        raise ValueError(f"{w}: shape {shape!r} is not [out, in]")
    qblock, qblock2 = int(scalars["blocksize"]), int(scalars["nested_blocksize"])
    if qblock <= 0 or qblock2 <= 0:
        raise ValueError(f"{w}: block sizes {qblock}, {qblock2}")
    n = shape[0] * shape[1]
    n_blocks = -(-n // qblock)
    expect = {"weight": (packed, torch.uint8, (n + 1) // 2),
              "absmax": (arrays["absmax"], torch.uint8, n_blocks),
              "quant_map": (arrays["quant_map"], torch.float32, 16),
              "nested_absmax": (arrays["nested_absmax"], torch.float32, -(-n_blocks // qblock2)),
              "nested_quant_map": (arrays["nested_quant_map"], torch.float32, 256)}
    for name, (t, dtype, numel) in expect.items():
        if t.dtype != dtype or t.numel() != numel:
            raise ValueError(f"{w}: {name} is {t.dtype} x {t.numel()}, expected {dtype} x {numel}")
    levels = torch.tensor(qgroup.NF4_LEVELS, dtype=torch.float32)
    if not torch.equal(arrays["quant_map"].cpu(), levels):
        raise ValueError(f"{w}: quant_map is not the NF4 level table")
    dtype = _DTYPES.get(scalars.get("dtype"))
    nested_dtype = _DTYPES.get(scalars.get("nested_dtype"))
    if dtype is None or nested_dtype is None:
        raise ValueError(f"{w}: dtypes {scalars.get('dtype')!r}, {scalars.get('nested_dtype')!r}")
    state2 = QuantState(absmax=arrays["nested_absmax"], blocksize=qblock2,
                        code=arrays["nested_quant_map"], dtype=nested_dtype)
    state = QuantState(absmax=arrays["absmax"], blocksize=qblock, code=arrays["quant_map"],
                       dtype=dtype, quant_type="nf4", shape=torch.Size(shape),
                       offset=torch.tensor(float(scalars["nested_offset"]), dtype=torch.float32),
                       state2=state2)
    bias = src.get(prefix + "bias") if prefix + "bias" in src else None
    return packed, state, bias


class NF4Linear(torch.nn.Module):
    """One frozen NF4 projection: `weight` is the packed uint8 parameter with its `quant_state`,
    `bias` an optional fp16 parameter. The product runs through the layer's `GroupLinear` (the
    grouped dequantisation, cached per pass), counted for the backward the way the patched
    `Linear4bit.forward` counts it (solution/qgroup.py:498-545); inputs are cast to fp16 and the
    result back, as `Linear4bit` does with its compute dtype. A module outside a layer group has
    no dequantisation path and raises."""

    def __init__(self, packed, state, bias=None):
        super().__init__()
        self.out_features, self.in_features = (int(d) for d in state.shape)
        self.weight = torch.nn.Parameter(packed, requires_grad=False)
        self.weight.quant_state = state
        self.bias = None if bias is None else torch.nn.Parameter(bias, requires_grad=False)
        self.compute_dtype = torch.float16
        self._talm_group = None

    def forward(self, x):
        if self._talm_group is None:
            raise RuntimeError("NF4Linear is not packed into a layer group (nf4_format.load_layer)")
        group, idx = self._talm_group
        in_dtype = x.dtype
        out = qgroup.GroupLinear.apply(x.to(torch.float16), group, idx)
        if torch.is_grad_enabled() and x.requires_grad:
            group.expected_bwd += 1
        return out.to(in_dtype)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, nf4"


def load_layer(source, prefix, device, projections=qgroup.PROJECTIONS):
    """The seven projections of the decoder layer stored under `prefix` ("model.layers.3."), as
    `NF4Linear` modules packed into one `LayerGroup` on `device`.

    `source` is a state-dict mapping (host or device tensors; pinned host tensors copy
    asynchronously) or the path of a safetensors file, read one tensor at a time. The packed
    weights, coded scales and second-level scales of the seven projections are copied into one
    buffer each, in projection order, and every module's tensors are views of those buffers;
    the returned group has adopted them (no second copy). Returns (group, {path: module})."""
    src = source if isinstance(source, _Source) else _Source(source)
    device = torch.device(device)
    read = [read_projection(src, f"{prefix}{p}.") for p in projections]
    sizes = [(p.numel(), s.absmax.numel(), s.state2.absmax.numel()) for p, s, _ in read]
    packed_buf = torch.empty(sum(s[0] for s in sizes), dtype=torch.uint8, device=device)
    absmax8_buf = torch.empty(sum(s[1] for s in sizes), dtype=torch.uint8, device=device)
    absmax2_buf = torch.empty(sum(s[2] for s in sizes), dtype=torch.float32, device=device)
    code = None
    modules = {}
    at = [0, 0, 0]
    for path, (packed, state, bias), size in zip(projections, read, sizes):
        views = []
        for k, (buf, src_t) in enumerate(((packed_buf, packed), (absmax8_buf, state.absmax),
                                          (absmax2_buf, state.state2.absmax))):
            view = buf[at[k]:at[k] + size[k]]
            view.copy_(src_t.reshape(-1), non_blocking=True)
            views.append(view)
            at[k] += size[k]
        if code is None or not torch.equal(state.state2.code.cpu(), code.cpu()):
            code = state.state2.code.to(device)
        state2 = QuantState(absmax=views[2], blocksize=state.state2.blocksize, code=code,
                            dtype=state.state2.dtype)
        dev_state = QuantState(absmax=views[1], blocksize=state.blocksize,
                               code=state.code.to(device), dtype=state.dtype,
                               quant_type=state.quant_type, shape=state.shape,
                               offset=state.offset.to(device), state2=state2)
        if bias is not None:
            bias = bias.to(device=device, dtype=torch.float16)
        modules[path] = NF4Linear(views[0].view(-1, 1), dev_state, bias)
    group = qgroup.LayerGroup(list(modules.values()))
    for idx, module in enumerate(modules.values()):
        module._talm_group = (group, idx)
    qgroup.track(group)
    return group, modules


def layer_indices(source, prefix="model.layers."):
    """The decoder-layer indices that have 4-bit projections under `prefix`, ascending."""
    pattern = re.compile(re.escape(prefix) + r"(\d+)\..*weight\." + re.escape(QUANT_STATE_KEY))
    src = source if isinstance(source, _Source) else _Source(source)
    return sorted({int(m.group(1)) for k in src.keys() for m in [pattern.fullmatch(k)] if m})


def load_layers(source, device, prefix="model.layers."):
    """Every decoder layer of a 4-bit checkpoint: [(group, modules)] in layer order, with each
    group's depth (layers after it) set as `qgroup` sets it for the split passes."""
    src = source if isinstance(source, _Source) else _Source(source)
    indices = layer_indices(src, prefix)
    out = []
    for i in indices:
        group, modules = load_layer(src, f"{prefix}{i}.", device)
        group.depth = indices[-1] - i
        out.append((group, modules))
    return out


def projection_state_dict(module, prefix=""):
    """The stored form of one NF4 projection (module with `weight.quant_state`), host tensors."""
    w = module.weight
    state = w.quant_state
    if not state.nested:
        raise ValueError("only double-quantised weights are written")
    scalars = {"quant_type": state.quant_type, "blocksize": int(state.blocksize),
               "dtype": _dtype_name(state.dtype), "shape": [int(d) for d in state.shape],
               "nested_blocksize": int(state.state2.blocksize),
               "nested_offset": float(state.offset), "nested_dtype":
               _dtype_name(state.state2.dtype)}
    out = {f"{prefix}weight": w.detach().reshape(-1, 1).cpu().clone(),
           f"{prefix}weight.absmax": state.absmax.detach().cpu().clone(),
           f"{prefix}weight.quant_map": state.code.detach().cpu().clone(),
           f"{prefix}weight.nested_absmax": state.state2.absmax.detach().cpu().clone(),
           f"{prefix}weight.nested_quant_map": state.state2.code.detach().cpu().clone(),
           f"{prefix}weight.{QUANT_STATE_KEY}": pack_scalars(scalars)}
    if getattr(module, "bias", None) is not None:
        out[f"{prefix}bias"] = module.bias.detach().cpu().clone()
    return out


def layer_state_dict(modules, prefix):
    """The stored form of a loaded layer ({path: module} of `load_layer`) under `prefix`."""
    out = {}
    for path, module in modules.items():
        out.update(projection_state_dict(module, f"{prefix}{path}."))
    return out
