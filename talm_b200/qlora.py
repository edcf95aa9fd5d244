"""A QLoRA training step of the Qwen2 architecture with both hot paths plugged in.

`build_model(config, device)` makes transformers' `Qwen2ForCausalLM` in fp16 (random init),
replaces the seven projections of every decoder layer by `NF4Linear` modules packed into one
`LayerGroup` (read by `nf4_format.load_layer` from a seeded 4-bit checkpoint in the stored
format) and wraps q_proj and v_proj in `LoraLinear` adapters. Only the adapters train. With
`patch()` installed (the decoder-layer hook of `qgroup` and the fused head of `patches`), one
`train_step` is: forward with labels (each layer's seven weights dequantised by one grouped
launch per pass, the loss by the fused head with no logits tensor), backward (the head's saved
dH scaled by one kernel, each layer dequantised once more), and one AdamW step on the adapters.
The reference's step plugs the same two paths into the same model (solution/patches.py:173-260
for the head call, solution/qgroup.py:474-545 for the layer hooks, solution/lora.py:151-231 for
the adapter arithmetic).

Padding removal (solution/unpad.py) comes in two forms: `varlen_train_step` gathers the real
tokens on the device after one host read of the row lengths (`unpad_batch`, as the reference
does) and runs attention in PyTorch's variable-length mode over the packed rows
(`varlen_attention`); `pack_batch` builds the same packed tokens on the host before upload, for
the CUDA-graph replay (`GraphedStep.packed`, a block-causal mask). What the reference's step has
that this one does not: PEFT and trl around the model, a gradient scaler for fp16 training (here
the frozen model is fp16 and the adapters fp32, with no loss scaling), and gradient
checkpointing.
"""

import math

import torch
import torch.nn.functional as F

from . import nf4_format, qgroup

LORA_TARGETS = ("self_attn.q_proj", "self_attn.v_proj")


def qwen25_15b_config(**overrides):
    """The Qwen2.5-1.5B architecture: 28 layers, hidden 1536, 12 query / 2 key-value heads of
    128, SwiGLU 8960, tied vocabulary of 151936, RMSNorm eps 1e-6, RoPE theta 1e6."""
    from transformers import Qwen2Config

    args = dict(vocab_size=151936, hidden_size=1536, intermediate_size=8960,
                num_hidden_layers=28, num_attention_heads=12, num_key_value_heads=2,
                rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True,
                max_position_embeddings=32768, attention_dropout=0.0)
    args.update(overrides)
    return Qwen2Config(**args)


class LoraLinear(torch.nn.Module):
    """base(x) + scaling * B(A(dropout(x))): the adapter of PEFT's 4-bit Linear under fp16
    autocast, which the reference's LoraProjectionTorch reproduces op for op
    (solution/lora.py:151-231): dropout of the input, the fp32 adapter weights cast to fp16, two
    fp16 GEMMs ([T, in] x [in, r], then [T, r] x [r, out]), the product times scaling, added to
    the base output. A is Kaiming-uniform and B zero at initialisation, as PEFT does; autograd
    derives the backward."""

    def __init__(self, base, r, alpha, dropout, generator=None, b_std=0.0):
        super().__init__()
        self.base = base
        self.r, self.scaling, self.dropout = r, alpha / r, dropout
        device = base.weight.device
        a = torch.empty(r, base.in_features, dtype=torch.float32, device=device)
        torch.nn.init.kaiming_uniform_(a, a=math.sqrt(5), generator=generator)
        b = torch.zeros(base.out_features, r, dtype=torch.float32, device=device)
        if b_std:
            b.normal_(0.0, b_std, generator=generator)
        self.lora_A = torch.nn.Parameter(a)
        self.lora_B = torch.nn.Parameter(b)

    @property
    def in_features(self):
        return self.base.in_features

    @property
    def out_features(self):
        return self.base.out_features

    def forward(self, x):
        out = self.base(x)
        xd = F.dropout(x, self.dropout, self.training) if self.dropout > 0 else x
        t = torch.matmul(xd.to(torch.float16), self.lora_A.to(torch.float16).t())
        branch = torch.matmul(t, self.lora_B.to(torch.float16).t())
        return out + (branch * self.scaling).to(out.dtype)


def projection_shapes(config):
    """[out, in] of the seven projections of one decoder layer, in `qgroup.PROJECTIONS` order."""
    hidden, inter = config.hidden_size, config.intermediate_size
    head_dim = getattr(config, "head_dim", None) or hidden // config.num_attention_heads
    q, kv = config.num_attention_heads * head_dim, config.num_key_value_heads * head_dim
    shapes = [(q, hidden), (kv, hidden), (kv, hidden), (hidden, q), (inter, hidden),
              (inter, hidden), (hidden, inter)]
    return dict(zip(qgroup.PROJECTIONS, shapes))


def code_table(generator, device):
    """A seeded, sorted 256-entry code for the first-level scales, spanning [-1, 1] (the role of
    bitsandbytes' dynamic map in a double-quantised checkpoint)."""
    code = torch.sort(torch.rand(256, generator=generator, device=device) * 2 - 1).values
    code[0], code[-1] = -1.0, 1.0
    return code


def synthetic_layer_checkpoint(shapes, prefix, generator, device, code, qblock=64, qblock2=256,
                               scale=0.035, biases=None):
    """A seeded 4-bit layer in the stored format (nf4_format): uniform codes and coded scales,
    second-level scales in [0.2, 0.4] * scale and offset `scale`, so that every block scale is
    code * absmax2 + offset in [0.6, 1.4] * scale (weights of standard deviation ~0.58 * scale:
    ~0.02 at the default). `biases` maps a projection to an fp16 bias to store with it."""
    sd = {}
    levels = torch.tensor(qgroup.NF4_LEVELS, dtype=torch.float32, device=device)
    for path, (o, i) in shapes.items():
        n = o * i
        n_blocks = n // qblock
        w = f"{prefix}{path}.weight"
        sd[w] = torch.randint(0, 256, (n // 2, 1), generator=generator, device=device,
                              dtype=torch.uint8)
        sd[w + ".absmax"] = torch.randint(0, 256, (n_blocks,), generator=generator,
                                          device=device, dtype=torch.uint8)
        sd[w + ".quant_map"] = levels.clone()
        sd[w + ".nested_absmax"] = (torch.rand(-(-n_blocks // qblock2), generator=generator,
                                               device=device) * 0.2 + 0.2) * scale
        sd[w + ".nested_quant_map"] = code
        sd[f"{w}.{nf4_format.QUANT_STATE_KEY}"] = nf4_format.pack_scalars(
            {"quant_type": "nf4", "blocksize": qblock, "dtype": "float16", "shape": [o, i],
             "nested_blocksize": qblock2, "nested_offset": float(scale),
             "nested_dtype": "float32"})
        if biases is not None and biases.get(path) is not None:
            sd[f"{prefix}{path}.bias"] = biases[path]
    return sd


def _child(root, path):
    obj = root
    for part in path.split("."):
        obj = getattr(obj, part)
    return obj


def _replace(root, path, module):
    parent, _, name = path.rpartition(".")
    setattr(_child(root, parent) if parent else root, name, module)


def build_model(config, device, seed=0, lora_r=16, lora_alpha=32, lora_dropout=0.05,
                lora_targets=LORA_TARGETS, qblock=64, qblock2=256, weight_scale=0.035,
                lora_b_std=0.0):
    """`Qwen2ForCausalLM(config)` in fp16 on `device` (random init from `seed`), its decoder
    projections 4-bit (`NF4Linear`, one `LayerGroup` per layer, loaded from a synthetic stored
    checkpoint) and LoRA on `lora_targets`; every parameter but the adapters frozen. The fp16
    projection weights the constructor made are freed layer by layer before the 4-bit ones are
    loaded. `lora_b_std` > 0 starts B at random instead of zero (tests use it to give A a
    gradient on the first step)."""
    from transformers import Qwen2ForCausalLM

    device = torch.device(device)
    torch.manual_seed(seed)
    previous = torch.get_default_dtype()
    torch.set_default_dtype(torch.float16)
    try:
        with device:
            model = Qwen2ForCausalLM(config)
    finally:
        torch.set_default_dtype(previous)
    generator = torch.Generator(device=device).manual_seed(seed + 1)
    lora_generator = torch.Generator(device=device).manual_seed(seed + 2)
    code = code_table(generator, device)
    shapes = projection_shapes(config)
    layers = model.model.layers
    for index, layer in enumerate(layers):
        prefix = f"model.layers.{index}."
        biases = {}
        for path in qgroup.PROJECTIONS:
            bias = _child(layer, path).bias
            biases[path] = None if bias is None else bias.detach().to(torch.float16)
            _replace(layer, path, None)
        sd = synthetic_layer_checkpoint(shapes, prefix, generator, device, code, qblock,
                                        qblock2, weight_scale, biases)
        group, modules = nf4_format.load_layer(sd, prefix, device)
        del sd
        group.depth = len(layers) - 1 - index
        for path, module in modules.items():
            if path in lora_targets:
                module = LoraLinear(module, lora_r, lora_alpha, lora_dropout, lora_generator,
                                    lora_b_std)
            _replace(layer, path, module)
        layer._talm_layer_group = group
        layer._talm_group_done = True
    for name, param in model.named_parameters():
        param.requires_grad_(name.rsplit(".", 1)[-1] in ("lora_A", "lora_B"))
    model.config.use_cache = False
    return model


def adapters(model):
    """The trainable parameters (the LoRA A and B of every adapted projection)."""
    return [p for p in model.parameters() if p.requires_grad]


def patch():
    """Install what the step runs through: the decoder-layer hook that starts each layer's
    dequantisation passes, and the fused head in Qwen2ForCausalLM.forward."""
    from .patches import patch_qwen2_causal_lm

    qgroup.patch_decoder_layer()
    patch_qwen2_causal_lm()


def make_batch(batch, seq, vocab, device, seed=0, pad_fraction=0.45):
    """Token ids uniform over the vocabulary, each row with a seeded trailing pad of 35-55 % of
    the sequence, the last row's adjusted so the batch has ~`pad_fraction` pad (BASELINE config
    5's batch shape); attention mask 0 and label -100 on the pad."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq), generator=g)
    lo, hi = int(0.35 * seq), int(0.55 * seq)
    pads = torch.randint(lo, max(hi, lo + 1), (batch,), generator=g)
    if batch > 1:
        rest = int(round(pad_fraction * batch * seq)) - int(pads[:-1].sum())
        pads[-1] = min(max(rest, 0), seq - 1)
    keep = torch.arange(seq)[None, :] < (seq - pads)[:, None]
    labels = ids.masked_fill(~keep, -100)
    return {"input_ids": ids.to(device), "attention_mask": keep.to(torch.long).to(device),
            "labels": labels.to(device)}


def train_step(model, optimizer, batch):
    """Forward with labels, backward, one optimizer step; returns the loss (a device scalar)."""
    out = model(**batch)
    out.loss.backward()
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return out.loss.detach()


def causal_padding_mask(attention_mask):
    """[B, 1, S, S] bool: query i of row b sees key j when j <= i and key j is not pad -- the
    mask transformers builds from a right-padded [B, S] mask for SDPA, made here once so that
    the decoder's forward reads no mask values on the host."""
    seq = attention_mask.shape[1]
    causal = torch.ones(seq, seq, dtype=torch.bool, device=attention_mask.device).tril()
    return causal[None, None] & attention_mask.bool()[:, None, None, :]


class _Decoder(torch.nn.Module):
    """input ids + prepared 4-D mask (+ position ids) -> last hidden state of the decoder."""

    def __init__(self, model):
        super().__init__()
        self.decoder = model.model

    def forward(self, input_ids, mask4d, position_ids=None):
        return self.decoder(input_ids=input_ids, attention_mask=mask4d, position_ids=position_ids,
                            use_cache=False).last_hidden_state


def pack_batch(batch, device, bucket=256):
    """The real tokens of a right-padded HOST batch packed into one sequence, built on the host
    (where the collator has the batch) so that the device sees no data-dependent shape and no
    host sync: the reference's padding removal (solution/unpad.py:66-95) does the same gather on
    the device after one host read of the row lengths.

    Row b's first len_b tokens follow one another in row order; each keeps its position in its
    row (the rotary positions of the padded batch) and its next-token target within the row
    (the padded batch's shifted label: the last real token's target is the pad's -100). The
    packed length is rounded up to a multiple of `bucket` with filler tokens (id 0, target
    -100, a segment of their own), so that a few captured graphs serve every batch. Returns
    device tensors input_ids [1, T], position_ids [1, T], segments [T] and targets [T], and the
    host counts n_real and n_labelled."""
    ids, mask, labels = batch["input_ids"], batch["attention_mask"], batch["labels"]
    if ids.is_cuda or mask.is_cuda or labels.is_cuda:
        raise ValueError("pack_batch packs the host batch (before it is copied to the GPU)")
    rows, seq = ids.shape
    keep = mask.bool()
    shift = F.pad(labels, (0, 1), value=-100)[:, 1:]
    pos = torch.arange(seq).expand(rows, seq)
    seg = torch.arange(rows)[:, None].expand(rows, seq)
    real_ids, real_pos, real_seg, real_tgt = ids[keep], pos[keep], seg[keep], shift[keep]
    n_real = int(real_ids.numel())
    total = -(-n_real // bucket) * bucket if bucket else n_real
    fill = total - n_real
    packed = {
        "input_ids": torch.cat([real_ids, torch.zeros(fill, dtype=ids.dtype)])[None],
        "position_ids": torch.cat([real_pos, torch.arange(fill)])[None],
        "segments": torch.cat([real_seg, torch.full((fill,), rows)]),
        "targets": torch.cat([real_tgt, torch.full((fill,), -100, dtype=labels.dtype)]),
    }
    n_labelled = int((packed["targets"] >= 0).sum())
    out = {k: v.to(device, non_blocking=True) for k, v in packed.items()}
    out.update(n_real=n_real, n_labelled=n_labelled)
    return out


def unpad_batch(batch, bucket=0):
    """Padding removal on the device (solution/unpad.py:66-95): the real tokens of a right-padded
    DEVICE batch packed row after row into one sequence, with one host read (the row lengths and
    the labelled count, in a single copy). Returns input_ids [1, T], position_ids [1, T] (each
    token's position in its row), targets [T] (the padded batch's shifted labels at the kept
    positions), cu_seqlens int32 [rows + 1] (row bounds in the packed sequence; with `bucket`,
    T is rounded up to a multiple of it and one more bound closes a filler segment of id-0
    tokens with target -100), max_len (the longest segment) and the host counts n_real and
    n_labelled."""
    ids, mask, labels = batch["input_ids"], batch["attention_mask"], batch["labels"]
    rows, seq = ids.shape
    device = ids.device
    lengths_dev = mask.to(torch.int64).sum(1)
    shift = F.pad(labels, (0, 1), value=-100)[:, 1:]
    inside = torch.arange(seq, device=device)[None] < lengths_dev[:, None]
    n_lab_dev = ((shift >= 0) & inside).sum()
    values = torch.cat((lengths_dev, n_lab_dev[None])).tolist()  # the one host read
    lengths, n_labelled = [int(v) for v in values[:rows]], int(values[rows])
    n_real = sum(lengths)
    total = -(-n_real // bucket) * bucket if bucket else n_real
    fill = total - n_real
    idx = torch.cat([torch.arange(n, device=device) + b * seq for b, n in enumerate(lengths)])
    pos = torch.cat([torch.arange(n, device=device) for n in lengths]
                    + ([torch.arange(fill, device=device)] if fill else []))
    flat_ids, flat_tgt = ids.reshape(-1)[idx], shift.reshape(-1)[idx]
    if fill:
        flat_ids = torch.cat([flat_ids, flat_ids.new_zeros(fill)])
        flat_tgt = torch.cat([flat_tgt, flat_tgt.new_full((fill,), -100)])
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    if fill:
        bounds.append(total)
    cu = torch.tensor(bounds, dtype=torch.int32).to(device, non_blocking=True)
    max_len = max([b - a for a, b in zip(bounds[:-1], bounds[1:])] + [1])
    return {"input_ids": flat_ids[None], "position_ids": pos[None], "targets": flat_tgt,
            "cu_seqlens": cu, "max_len": max_len, "n_real": n_real, "n_labelled": n_labelled}


VARLEN = "talm_varlen"


def varlen_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0,
                     **kwargs):
    """Causal attention over a packed sequence whose segments are given by `cu_seq_lens_q` /
    `max_length_q` (transformers passes the model's keyword arguments through), in one call of
    PyTorch's variable-length flash-attention kernel: no [T, T] mask, no attention across
    segments, grouped key/value heads used as they are. The reference runs the
    memory-efficient kernel's variable-length mode for the same purpose
    (solution/unpad.py:199-295). query [1, Hq, T, D], key/value [1, Hkv, T, D] -> [1, T, Hq, D]."""
    from torch.nn.attention.varlen import varlen_attn

    if dropout:
        raise ValueError("the packed attention path has no attention dropout")
    cu, max_len = kwargs["cu_seq_lens_q"], int(kwargs["max_length_q"])
    q = query[0].transpose(0, 1)
    k = key[0].transpose(0, 1)
    v = value[0].transpose(0, 1)
    out = varlen_attn(q, k, v, cu, cu, max_len, max_len, scale=scaling, window_size=(-1, 0))
    return out[None], None


def _register_varlen():
    from transformers import AttentionInterface

    AttentionInterface.register(VARLEN, varlen_attention)


def _varlen_hidden(model, packed):
    """The decoder over a packed batch (`unpad_batch`) with the variable-length attention."""
    _register_varlen()
    config = model.config
    previous = config._attn_implementation
    config._attn_implementation = VARLEN
    try:
        cu = packed["cu_seqlens"]
        return model.model(input_ids=packed["input_ids"], position_ids=packed["position_ids"],
                           cu_seq_lens_q=cu, cu_seq_lens_k=cu, max_length_q=packed["max_len"],
                           max_length_k=packed["max_len"], use_cache=False).last_hidden_state
    finally:
        config._attn_implementation = previous


def varlen_train_step(model, optimizer, batch, bucket=0):
    """The training step with the padding removed on the device (`unpad_batch`: one host read)
    and variable-length attention over the packed rows; the fused head over the kept tokens'
    targets, backward, one optimizer step."""
    packed = unpad_batch(batch, bucket)
    loss = _packed_loss(model, _varlen_hidden(model, packed), packed)
    loss.backward()
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()


def block_causal_mask(segments):
    """[1, 1, T, T] bool: token i sees token j when j <= i and both are in the same segment (a
    row of the packed batch)."""
    same = segments[:, None] == segments[None, :]
    return (same & torch.ones_like(same).tril())[None, None]


def _packed_loss(model, hidden, packed):
    from .fused_head import fused_head_loss

    return fused_head_loss(hidden.reshape(-1, hidden.shape[-1]), model.lm_head.weight,
                           packed["targets"], None, n_labelled=packed["n_labelled"])[0]


def packed_train_step(model, optimizer, packed):
    """The training step on a packed batch (`pack_batch`): the decoder over the real tokens only,
    the fused head over their targets, backward, one optimizer step."""
    hidden = _Decoder(model)(packed["input_ids"], block_causal_mask(packed["segments"]),
                             packed["position_ids"])
    loss = _packed_loss(model, hidden, packed)
    loss.backward()
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()


class GraphedStep:
    """The training step with the decoder's forward and backward replayed as CUDA graphs.

    The decoder (embedding, 28 layers, final norm) issues thousands of small launches per step
    from Python; captured once per input shape (`torch.cuda.make_graphed_callables`), each
    direction is one graph launch. Inside the graphs every layer still dequantises its seven
    weights with one grouped launch per pass. The head stays eager: its row compaction depends
    on the batch's labelled count (`n_labelled`, taken from the host batch, so no host sync),
    and it is a handful of launches. The optimizer step runs eagerly after the backward.
    Padded batches (`__call__`) must keep the shape of `batch`, captured at construction;
    packed batches (`packed`) capture one graph pair per packed length (a multiple of
    pack_batch's bucket) on first use. The LayerGroups' pass bookkeeping runs during each
    capture and the graphs replay its launches."""

    def __init__(self, model, optimizer, batch=None, warmup=3):
        self.model, self.optimizer, self.warmup = model, optimizer, warmup
        self.graphs = {}
        self.shape = None
        if batch is not None:
            ids, mask = batch["input_ids"], batch["attention_mask"]
            self.shape = tuple(ids.shape)
            self._graph(("padded", self.shape), (ids, causal_padding_mask(mask)))

    def _graph(self, key, args):
        if key not in self.graphs:
            # the sample arguments become the graphs' static inputs: copies, not the caller's
            self.graphs[key] = torch.cuda.make_graphed_callables(
                _Decoder(self.model), tuple(a.clone() for a in args),
                num_warmup_iters=self.warmup)
        return self.graphs[key]

    def _finish(self, loss):
        loss.backward()
        self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        return loss.detach()

    def __call__(self, batch, n_labelled):
        ids, mask, labels = batch["input_ids"], batch["attention_mask"], batch["labels"]
        if tuple(ids.shape) != self.shape:
            raise ValueError(f"batch shape {tuple(ids.shape)} is not the captured {self.shape}")
        from .fused_head import fused_head_loss

        hidden = self.graphs[("padded", self.shape)](ids, causal_padding_mask(mask))
        shift = F.pad(labels, (0, 1), value=-100)[:, 1:].reshape(-1)
        loss = fused_head_loss(hidden.reshape(-1, hidden.shape[-1]), self.model.lm_head.weight,
                               shift, None, n_labelled=n_labelled)[0]
        return self._finish(loss)

    def packed(self, packed):
        """One step on a packed batch (`pack_batch`)."""
        args = (packed["input_ids"], block_causal_mask(packed["segments"]),
                packed["position_ids"])
        graph = self._graph(("packed", tuple(packed["input_ids"].shape)), args)
        return self._finish(_packed_loss(self.model, graph(*args), packed))


def labelled_count(labels):
    """Host count of the shifted targets >= 0 of a [B, S] label batch (the head's n_labelled)."""
    return int((labels[:, 1:] >= 0).sum())
