"""One NF4 dequantisation launch per decoder layer (drop-in for solution/qgroup.py).

A `LayerGroup` owns the seven NF4 projections of one Qwen2 decoder layer. Their packed weights,
uint8 absmax and second-level fp32 absmax are concatenated into three buffers and the modules'
parameters become views of them (no memory duplicated), exactly as the reference packs them
(solution/qgroup.py:124-192). One call of the grouped sm_100a kernel (csrc/nf4.cu,
`talm_nf4_group_dequant`) then rebuilds every block scale as
fp32(fp32(code[absmax8] * absmax2) + offset2) and writes the whole layer's fp16 weights; the
other six projections slice the cached buffer. The per-pass cache (`fwd` / `bwd`), the split
passes of the last layers, the gradient-checkpointing mode and the use counting are the
reference's host logic (qgroup.py:194-328), restated here; only the kernel differs.

Failures: the reference answers an unexpected error with bitsandbytes' own dequantization. Here
the error is recorded (state.fallback) and raised: there is no second implementation.

The host logic restates otarernazar-eng/Talm's solution/qgroup.py (Apache License 2.0, "Soup
Kernel Challenge starter kit", Copyright 2026 Makazhan Alpamys and the Soup contributors): the
packing of the seven projections (`LayerGroup.__init__`), the per-pass cache and its use
counting (`reset` ... `span_bias`), `GroupLinear`, the level table and the layer / Linear4bit
patches follow that file statement for statement, because callers and tests depend on their
exact behaviour; the CUDA kernels they call are this package's own.
"""

import os
import weakref

import torch
import torch.nn.functional as F

from . import _lib
from .engaged import FELL_BACK, ON, RAN
from .state import DISABLED, fallback

ROWS = 64          # absmax blocks per tile of the reference kernel; still the layer granularity
NUM_WARPS = 4
NSEG = 7           # projections per decoder layer
WARMUP_QBLOCK, WARMUP_QBLOCK2 = 64, 256

# The 16 NormalFloat levels (solution/qgroup.py:60-63).
NF4_LEVELS = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
              -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
              0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
              0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0]

_SPLIT_OFF = os.environ.get("SOLUTION_DISABLE_SPLIT_DEQUANT") == "1"
# passes of the last layers that dequantise one projection at a time (qgroup.py:66-69)
SPLIT_LAYERS = {"fwd": 0 if _SPLIT_OFF else 1, "bwd": 0 if _SPLIT_OFF else 2}

PROJECTIONS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def launch(packed, absmax8, code, absmax2, offset2, levels, out, n_rows, qblock, qblock2):
    """The grouped kernel over `n_rows` absmax blocks of `qblock` weights into the contiguous
    fp16 `out` (solution/qgroup.py:94-99)."""
    lib = _lib.load()
    _lib.check(lib.talm_nf4_group_dequant(
        _lib.ptr(packed), _lib.ptr(absmax8), _lib.ptr(code), _lib.ptr(absmax2),
        _lib.ptr(offset2), _lib.ptr(levels), _lib.ptr(out), int(n_rows), int(qblock),
        int(qblock2), _lib.stream_of(out.device)), "talm_nf4_group_dequant")


_LEVELS = {}


def _levels(device):
    """The NF4 level table on `device`, shared by all layers."""
    key = str(device)
    if key not in _LEVELS:
        _LEVELS[key] = torch.tensor(NF4_LEVELS, dtype=torch.float32, device=device)
    return _LEVELS[key]


def _state_ok(state, first):
    """The quant states the grouped kernel handles (solution/qgroup.py:110-118): NF4,
    double-quantised, one block size pair and one second-level code table for the layer."""
    return (state is not None and state.quant_type == "nf4" and state.nested
            and state.blocksize == first.blocksize
            and state.state2.blocksize == first.state2.blocksize
            and len(state.shape) == 2 and state.absmax.dtype == torch.uint8
            and state.state2.absmax.dtype == torch.float32
            and torch.equal(state.state2.code, first.state2.code))


def _joined(parts):
    """One flat tensor holding `parts` in order. Parts that already lie back to back in one
    allocation (a loader wrote them there: nf4_format.load_layer) are adopted as one view of it;
    anything else is concatenated into a new buffer."""
    first = parts[0]
    storage, offset = first.untyped_storage().data_ptr(), first.storage_offset()
    for p in parts:
        if (p.dtype != first.dtype or p.device != first.device or not p.is_contiguous()
                or p.untyped_storage().data_ptr() != storage or p.storage_offset() != offset):
            return torch.cat(parts)
        offset += p.numel()
    return first.as_strided((offset - first.storage_offset(),), (1,), first.storage_offset())


class LayerGroup:
    """The seven 4-bit projections of one decoder layer, packed, with per-pass caches."""

    def __init__(self, modules):
        if len(modules) != NSEG:
            raise ValueError(f"a layer group has {NSEG} projections, got {len(modules)}")
        states = [m.weight.quant_state for m in modules]
        head = states[0]
        if not all(_state_ok(s, head) for s in states):
            raise ValueError("unsupported quant state")
        qblock, qblock2 = head.blocksize, head.state2.blocksize
        if qblock % 2 or (qblock * qblock2) % 2:
            raise ValueError("odd block size")
        double = qblock * qblock2
        numels = [int(s.shape[0]) * int(s.shape[1]) for s in states]
        if any(n % double for n in numels):
            raise ValueError("weight size not a multiple of the absmax double-block")
        half = qblock // 2
        total_pairs = sum(numels) // 2
        if half & (half - 1) or total_pairs % (ROWS * half) or total_pairs >= 2 ** 31:
            raise ValueError("layer size does not fit the kernel's tiling")

        device = modules[0].weight.device
        self.qblock, self.qblock2 = qblock, qblock2
        self.shapes = [tuple(int(d) for d in s.shape) for s in states]
        self.numels = numels
        # cumulative bounds of each projection in pairs (bytes), elements and absmax rows
        self.pair_bounds = [0]
        for n in numels:
            self.pair_bounds.append(self.pair_bounds[-1] + n // 2)
        self.elem_bounds = [2 * b for b in self.pair_bounds]
        self.row_bounds = [e // qblock for e in self.elem_bounds]

        # One buffer per array; each parameter / quant state becomes a view into it.
        self.packed = _joined([m.weight.data.reshape(-1) for m in modules])
        self.absmax8 = _joined([s.absmax.reshape(-1) for s in states])
        self.absmax2 = _joined([s.state2.absmax.reshape(-1) for s in states])
        byte = row = row2 = 0
        for m, s, n in zip(modules, states, numels):
            m.weight.data = self.packed[byte:byte + n // 2].view(-1, 1)
            s.absmax = self.absmax8[row:row + n // qblock]
            s.state2.absmax = self.absmax2[row2:row2 + n // double]
            byte, row, row2 = byte + n // 2, row + n // qblock, row2 + n // double
        self.code = head.state2.code
        self.offsets = torch.stack([s.offset.reshape(()).to(torch.float32)
                                    for s in states]).to(device)
        # the offset of each second-level block (no per-element segment search in the kernel)
        self.offset2 = torch.cat([self.offsets[i:i + 1].expand(n // double)
                                  for i, n in enumerate(numels)])
        self.n_pairs = total_pairs
        self.n_rows = total_pairs // half
        self.levels = _levels(device)
        self.biases = [None if m.bias is None else m.bias.detach().to(torch.float16)
                       for m in modules]
        self.params = [m.weight for m in modules]
        self._span_biases = {}
        self.cache = {"fwd": [None, 0], "bwd": [None, 0]}
        self.expected_bwd = 0
        self.split_left = 0
        self.checkpointed = False
        self.depth = None
        # a projection can be dequantised alone when its absmax rows tile by ROWS and start on
        # a second-level block that keeps the slice pointers 16-byte aligned (qgroup.py:185-192)
        self.splittable = all(
            (r1 - r0) % ROWS == 0 and r0 % (4 * qblock2) == 0
            for r0, r1 in zip(self.row_bounds[:-1], self.row_bounds[1:]))

    def dequantize_all(self):
        out = torch.empty(self.n_pairs * 2, dtype=torch.float16, device=self.packed.device)
        launch(self.packed, self.absmax8, self.code, self.absmax2, self.offset2, self.levels,
               out, self.n_rows, self.qblock, self.qblock2)
        return out

    def dequantize_one(self, idx):
        """fp16 [out, in] of projection `idx` alone: the kernel on that weight's slice of the
        packed buffers (it starts on a second-level block, so block indices stay right)."""
        r0, r1 = self.row_bounds[idx], self.row_bounds[idx + 1]
        b0 = r0 // self.qblock2
        out = torch.empty(self.numels[idx], dtype=torch.float16, device=self.packed.device)
        launch(self.packed[r0 * (self.qblock // 2):], self.absmax8[r0:], self.code,
               self.absmax2[b0:], self.offset2[b0:], self.levels, out, r1 - r0, self.qblock,
               self.qblock2)
        return out.view(self.shapes[idx])

    def weight(self, which, idx):
        """fp16 [out, in] of projection `idx` for pass `which` (qgroup.py:213-223)."""
        try:
            return self._weight(which, idx)
        except Exception as exc:
            fallback("qgroup", exc)
            raise

    def reset(self):
        """Forget the pass state: cached weights and backward counts."""
        self.cache = {"fwd": [None, 0], "bwd": [None, 0]}
        self.expected_bwd = 0
        self.split_left = 0

    def refund(self, which, uses=1):
        """Give back uses of the pass cache taken by a call whose result was dropped."""
        entry = self.cache[which]
        if entry[0] is not None:
            entry[1] += uses

    def start_forward(self, checkpointed=False):
        """The layer's forward begins: drop whatever a step cut short left (qgroup.py:252-264)."""
        for which in ("fwd", "bwd"):
            self.cache[which][0] = None
            self.cache[which][1] = 0
        self.expected_bwd = 0
        self.split_left = 0
        self.checkpointed = checkpointed

    def split_now(self, which):
        """True when the next use in pass `which` dequantises one projection alone
        (qgroup.py:266-271)."""
        if self.checkpointed:
            return True
        return (self.cache[which][0] is None and self.depth is not None
                and self.depth < SPLIT_LAYERS[which] and self.splittable)

    def _take(self, which, uses):
        """The layer's buffer for pass `which`, dequantised at the first use of the pass and
        dropped after the last expected use (qgroup.py:273-288)."""
        entry = self.cache[which]
        if entry[0] is None:
            entry[0] = self.dequantize_all()
            RAN["group"] += 1
            if which == "fwd":
                entry[1] = NSEG
            else:
                entry[1] = max(self.expected_bwd, 1)
                self.expected_bwd = 0
        buf = entry[0]
        entry[1] -= uses
        if entry[1] <= 0:
            entry[0] = None
        return buf

    def _slice(self, buf, first, last):
        return buf[self.elem_bounds[first]:self.elem_bounds[last]]

    def _weight(self, which, idx):
        if self.split_now(which):
            if self.checkpointed:
                self.expected_bwd = 0
                if not self.splittable:
                    RAN["group"] += 1
                    return self._slice(self.dequantize_all(), idx, idx + 1).view(self.shapes[idx])
            elif which == "bwd":
                if self.split_left == 0:
                    self.split_left = max(self.expected_bwd, 1)
                    self.expected_bwd = 0
                self.split_left -= 1
            RAN["split"] += 1
            return self.dequantize_one(idx)
        return self._slice(self._take(which, 1), idx, idx + 1).view(self.shapes[idx])

    def span(self, which, first, last):
        """fp16 [sum of out, in] of adjacent projections first .. last - 1 as one view of the
        layer's buffer, counted as last - first uses; None in a split pass (qgroup.py:310-328)."""
        if "qgroup" in DISABLED:
            return None
        try:
            if self.split_now(which):
                return None
            buf = self._take(which, last - first)
        except Exception as exc:
            fallback("qgroup", exc)
            raise
        rows = sum(self.shapes[i][0] for i in range(first, last))
        return self._slice(buf, first, last).view(rows, self.shapes[first][1])

    def span_bias(self, first, last):
        """The fp16 biases of projections first .. last - 1 concatenated (zeros where a
        projection has none), or None when none has one; built once."""
        key = (first, last)
        if key not in self._span_biases:
            parts = self.biases[first:last]
            if all(b is None for b in parts):
                self._span_biases[key] = None
            else:
                like = next(b for b in parts if b is not None)
                self._span_biases[key] = torch.cat([
                    b if b is not None else like.new_zeros(self.shapes[first + i][0])
                    for i, b in enumerate(parts)])
        return self._span_biases[key]


def _span(group, first, last):
    """The packed bytes, coded scales, group-wide first absmax row and [rows, cols] of the
    adjacent projections first .. last - 1 (one weight of sum-of-rows x shared columns)."""
    cols = group.shapes[first][1]
    if any(group.shapes[i][1] != cols for i in range(first, last)):
        raise ValueError("projections of a span share their input size")
    rows = sum(group.shapes[i][0] for i in range(first, last))
    b0, b1 = group.pair_bounds[first], group.pair_bounds[last]
    r0, r1 = group.row_bounds[first], group.row_bounds[last]
    return group.packed[b0:b1], group.absmax8[r0:r1], r0, rows, cols


def fused_linear(x, group, first, last=None, bias=None, transpose=False):
    """The fused NF4 dequant + tcgen05 GEMM (talm_nf4_linear) on projections first .. last - 1
    of `group` (default: `first` alone): x [..., in] -> x W^T (+ bias) [..., sum of out], or with
    transpose=True the input gradient g [..., sum of out] -> g W [..., in]. The weights are
    rebuilt in shared memory bit for bit as the grouped kernel writes them (the same fp16
    values F.linear would read from the dequantised buffer); the products accumulate in fp32.
    Needs qblock 64, spans of 64-row multiples and input sizes of 128-column multiples."""
    last = first + 1 if last is None else last
    packed, absmax8, row0, rows, cols = _span(group, first, last)
    red, n_out = (rows, cols) if transpose else (cols, rows)
    if x.shape[-1] != red:
        raise ValueError(f"last dimension {x.shape[-1]}, expected {red}")
    a = x.reshape(-1, red)
    if a.dtype != torch.float16 or a.stride(1) != 1 or a.stride(0) % 8 or a.data_ptr() % 16:
        a = a.to(torch.float16).contiguous()
    y = torch.empty(a.shape[0], n_out, dtype=torch.float16, device=a.device)
    if bias is not None:
        bias = bias.to(torch.float16).contiguous()
    lib = _lib.load()
    _lib.check(lib.talm_nf4_linear(
        _lib.ptr(a), a.stride(0), a.shape[0], _lib.ptr(packed), _lib.ptr(absmax8),
        _lib.ptr(group.code), _lib.ptr(group.absmax2), _lib.ptr(group.offset2),
        _lib.ptr(group.levels), row0, rows, cols, group.qblock, group.qblock2, int(transpose),
        _lib.ptr(bias), _lib.ptr(y), y.stride(0), _lib.stream_of(a.device)), "talm_nf4_linear")
    return y.view(*x.shape[:-1], n_out)


class GroupLinear(torch.autograd.Function):
    """x @ W^T (+ b) with W from the layer's dequantised buffer; the frozen weight gets no
    gradient (solution/qgroup.py:346-355)."""

    @staticmethod
    def forward(ctx, x, group, idx):
        ctx.group, ctx.idx = group, idx
        return F.linear(x, group.weight("fwd", idx), group.biases[idx])

    @staticmethod
    def backward(ctx, grad_out):
        weight = ctx.group.weight("bwd", ctx.idx)
        return torch.matmul(grad_out, weight), None, None


_GROUPS = []


def track(group):
    """Count `group` among the live layer groups that `reset_passes` resets."""
    _GROUPS.append(weakref.ref(group))


def reset_passes():
    """Reset every live layer group's pass state (qgroup.py:362-373)."""
    alive = []
    for ref in _GROUPS:
        group = ref()
        if group is not None:
            group.reset()
            alive.append(ref)
    _GROUPS[:] = alive


def _bnb_linear(module):
    """The bitsandbytes Linear4bit under a PEFT wrapper (or the module itself); None for any
    other module, and for every module when bitsandbytes is not installed."""
    try:
        import bitsandbytes as bnb
    except ImportError:
        return None

    base = getattr(module, "base_layer", module)
    return base if isinstance(base, bnb.nn.Linear4bit) else None


def _projections(layer):
    modules = []
    for path in PROJECTIONS:
        obj = layer
        for part in path.split("."):
            obj = getattr(obj, part, None)
            if obj is None:
                return None
        modules.append(obj)
    return modules


def _pack(layer):
    """The layer's seven frozen 4-bit projections as one LayerGroup, or None (qgroup.py:402-434)."""
    found = _projections(layer)
    if found is None:
        return None
    modules = []
    for obj in found:
        base = _bnb_linear(obj)
        if base is None or base.weight.requires_grad or not base.weight.is_cuda:
            return None
        if base.bias is not None and base.bias.requires_grad:
            return None
        if getattr(base, "compute_dtype", None) not in (None, torch.float16):
            return None
        modules.append(base)
    try:
        group = LayerGroup(modules)
    except ValueError:
        return None
    attn = getattr(layer, "self_attn", None)
    layer_idx = getattr(attn, "layer_idx", None)
    n_layers = getattr(getattr(attn, "config", None), "num_hidden_layers", None)
    if isinstance(layer_idx, int) and isinstance(n_layers, int) and 0 <= layer_idx < n_layers:
        group.depth = n_layers - 1 - layer_idx
    for idx, base in enumerate(modules):
        base._talm_group = (group, idx)
    track(group)
    return group


def setup_layer(layer):
    """Pack the layer's seven projections once; tag each module with its group."""
    if getattr(layer, "_talm_group_done", False):
        return
    layer._talm_group_done = True
    layer._talm_layer_group = _pack(layer)


def _wrapped(layer):
    """An instance-level forward on the layer or its attention (a checkpointing wrapper)."""
    attention = getattr(layer, "_modules", {}).get("self_attn")
    return "forward" in getattr(layer, "__dict__", {}) or (
        attention is not None and "forward" in attention.__dict__)


def enter_layer(layer):
    """The decoder layer's forward begins: pack on first use, start the passes afresh
    (qgroup.py:474-492)."""
    if "qgroup" in DISABLED:
        return
    try:
        if not getattr(layer, "_talm_group_done", False):
            setup_layer(layer)
        group = getattr(layer, "_talm_layer_group", None)
        if group is not None:
            group.start_forward(bool(getattr(layer, "training", False) and (
                getattr(layer, "gradient_checkpointing", False) or _wrapped(layer))))
    except Exception as exc:
        fallback("qgroup", exc)
        raise


prepare_layer = enter_layer


def patch_decoder_layer():
    """`Qwen2DecoderLayer.forward` packs its layer on first use and starts its passes afresh
    (qgroup.py:474-492); installed once."""
    from transformers.models.qwen2 import modeling_qwen2

    layer_cls = modeling_qwen2.Qwen2DecoderLayer
    ON.add("group")
    if not getattr(layer_cls.forward, "_talm_group", False):
        layer_forward = layer_cls.forward

        def forward(self, *args, **kwargs):
            enter_layer(self)
            return layer_forward(self, *args, **kwargs)

        forward._talm_group = True
        forward._original = layer_forward
        layer_cls.forward = forward


def patch_group_dequant():
    """`Qwen2DecoderLayer.forward` packs its layer on first use and starts its passes afresh;
    `bitsandbytes.nn.Linear4bit.forward` routes packed modules through GroupLinear for fp16
    CUDA inputs (qgroup.py:498-545)."""
    import bitsandbytes as bnb

    patch_decoder_layer()
    lin_cls = bnb.nn.Linear4bit
    if getattr(lin_cls.forward, "_talm_group", False):
        return True
    lin_forward = lin_cls.forward

    def linear_forward(self, x):
        tag = getattr(self, "_talm_group", None)
        if tag is not None and "qgroup" not in DISABLED and x.is_cuda \
                and x.dtype == torch.float16:
            group, idx = tag
            out = GroupLinear.apply(x, group, idx)
            if torch.is_grad_enabled() and x.requires_grad:
                group.expected_bwd += 1
            return out
        FELL_BACK["group"] += 1
        return lin_forward(self, x)

    linear_forward._talm_group = True
    linear_forward._original = lin_forward
    lin_cls.forward = linear_forward
    return True
