"""The fused LM head + cross-entropy restated on CPU with torch - TEST INFRASTRUCTURE (oracle),
not product code.

`reference_head` is the base run's computation as the reference's tests state it
(solution/test_kernels.py:70-83): fp16 logits of an fp16 GEMM, transformers' ForCausalLMLoss
(fp32 upcast, sum / num_items), TRL's entropy and accuracy (first column on ties), per-token
losses; and the hidden gradient of the loss (softmax - onehot) W16 / denom. `head_reference64`
is the float64 variant with the `fragile` near-tie rows of solution/test_fuzz.py:145-185. Both
walk the vocabulary in chunks so that the [N, V] logits never exist at once.

The fp16 logits are computed as fp32 dot products of the fp16 values, rounded once to fp16: the
value a tensor-core GEMM with fp32 accumulation returns, up to the fp32 summation order.
"""

import torch

F16 = torch.float16


def _chunks(vocab, rows):
    step = max(1, (1 << 24) // max(rows, 1))
    for s in range(0, vocab, step):
        yield s, min(vocab, s + step)


def logits16(h16, w16, s, e):
    """fp16-rounded logits of columns [s, e) as fp32 values."""
    return (h16.float() @ w16[s:e].float().t()).to(F16).float()


def row_stats(hidden, weight, targets, col0=0):
    """Per-row statistics of the columns `weight` holds (global ids col0 + j): m (max z), s =
    sum exp(z - m), t = sum exp(z - m) z, zt (target logit if covered, else 0), hit, idx (first
    global column of the max), in float64 - the quantities of the reference's stats mode
    (solution/fused_head.py:126-169)."""
    h16 = hidden.detach().to(F16)
    w16 = weight.detach().to(F16)
    n = h16.shape[0]
    vocab = w16.shape[0]
    m = torch.full((n,), -float("inf"), dtype=torch.float64)
    s = torch.zeros(n, dtype=torch.float64)
    t = torch.zeros(n, dtype=torch.float64)
    zt = torch.zeros(n, dtype=torch.float64)
    hit = torch.zeros(n, dtype=torch.bool)
    idx = torch.zeros(n, dtype=torch.int64)
    rel = targets.to(torch.int64) - col0
    for a, b in _chunks(vocab, n):
        z = logits16(h16, w16, a, b).double()
        cm, ci = z.max(-1)                       # torch.max returns the first maximum
        better = cm > m
        idx = torch.where(better, ci + a + col0, idx)
        m_new = torch.maximum(m, cm)
        alpha = torch.exp(m - m_new)
        e = torch.exp(z - m_new[:, None])
        s = s * alpha + e.sum(-1)
        t = t * alpha + (e * z).sum(-1)
        m = m_new
        here = (rel >= a) & (rel < b) & (targets >= 0)
        if here.any():
            rows = here.nonzero().squeeze(1)
            zt[rows] = z[rows, rel[rows] - a]
            hit[rows] = True
    return {"m": m, "s": s, "t": t, "zt": zt, "hit": hit, "idx": idx}


def reference_head(hidden, weight, targets, num_items=None, grad_scale=1.0):
    """(loss, token_loss, entropy, correct, dH) of the base run (solution/test_kernels.py:70-83)
    with dH = d(loss * grad_scale)/d hidden, in fp32 (float64 internally)."""
    st = row_stats(hidden, weight, targets)
    labelled = targets >= 0
    lse = st["m"] + torch.log(st["s"])
    token_loss = torch.where(labelled, lse - st["zt"], torch.zeros_like(lse))
    entropy = lse - st["t"] / st["s"]
    correct = labelled & (st["idx"] == targets)
    n_lab = int(labelled.sum())
    denom = float(num_items) if num_items is not None else float(max(n_lab, 1))
    loss = token_loss.sum() / denom if denom != 0 else token_loss.sum() * 0.0
    grad = head_grad(hidden, weight, targets, lse)
    scale = grad_scale / denom if denom != 0 else 0.0
    return (loss.float(), token_loss.float(), entropy.float(), correct,
            (grad * scale).float())


def head_grad(hidden, weight, targets, lse):
    """(softmax(z) - onehot(target)) W16 for labelled rows, 0 for the others (float64)."""
    h16 = hidden.detach().to(F16)
    w16 = weight.detach().to(F16)
    n, size = h16.shape
    vocab = w16.shape[0]
    labelled = targets >= 0
    grad = torch.zeros(n, size, dtype=torch.float64)
    for a, b in _chunks(vocab, n):
        z = logits16(h16, w16, a, b).double()
        p = torch.exp(z - lse[:, None])
        grad += p @ w16[a:b].double()
    tc = targets.clamp(min=0)
    grad -= w16[tc].double()
    grad[~labelled] = 0
    return grad


def head_reference64(hidden, weight, targets, num_items=None):
    """solution/test_fuzz.py:145-185 restated: float64 per-token loss, entropy, first-max
    correctness, max |z| per row, the `fragile` rows (target within 8 fp16 ulps of the row max
    with another logit as close) and the hidden gradient of sum(token loss)."""
    h16 = hidden.detach().to(F16)
    w16 = weight.detach().to(F16)
    n = h16.shape[0]
    vocab = w16.shape[0]
    st = row_stats(hidden, weight, targets)
    labelled = targets >= 0
    lse = st["m"] + torch.log(st["s"])
    ulp = torch.exp2(torch.floor(torch.log2(st["m"].abs().clamp(min=torch.finfo(F16).tiny)))) \
        * torch.finfo(F16).eps
    near_lo = st["m"] - 8 * ulp
    near_count = torch.zeros(n, dtype=torch.int64)
    target_near = torch.zeros(n, dtype=torch.bool)
    zmax = torch.zeros(n, dtype=torch.float64)
    tc = targets.clamp(min=0)
    for a, b in _chunks(vocab, n):
        z = logits16(h16, w16, a, b).double()
        zmax = torch.maximum(zmax, z.abs().max(-1).values)
        near = z >= near_lo[:, None]
        near_count += near.sum(-1)
        here = (tc >= a) & (tc < b)
        rows = here.nonzero().squeeze(1)
        target_near[rows] = near[rows, tc[rows] - a]
    n_lab = int(labelled.sum())
    return {
        "token_loss": torch.where(labelled, lse - st["zt"], torch.zeros_like(lse)),
        "entropy": lse - st["t"] / st["s"],
        "correct": labelled & (st["idx"] == targets),
        "zmax": zmax,
        "fragile": labelled & target_near & (near_count >= 2),
        "grad": head_grad(hidden, weight, targets, lse),
        "denom": float(num_items) if num_items is not None else float(max(n_lab, 1)),
        "labelled": labelled,
        "max_w": float(w16.float().abs().max()) if w16.numel() else 0.0,
    }


def scale_grad(grad_hidden, grad_loss, denom, out_dtype):
    """The head's backward (solution/fused_head.py:280-287): the saved fp16 hidden gradient
    times grad_loss / denom in fp32, 0 where denom == 0, in the hidden's dtype."""
    scale = grad_loss.to(torch.float32) / denom
    scale = torch.where(denom != 0, scale, 0.0)
    return (grad_hidden.to(F16).to(torch.float32) * scale).to(out_dtype)


class CpuHeadOps:
    """The three kernel steps of talm_b200.vocab_parallel (shard / combine / finalize) restated
    on CPU tensors, so that the exchange logic runs on gloo ranks in the tests."""

    def shard(self, h16, w16, ld_w, targets, n_grad, hidden_cols, col0, vocab_chunk):
        st = row_stats(h16, w16[:, :hidden_cols], targets, col0)
        n = h16.shape[0]
        stats = torch.zeros(n, 8, dtype=torch.float32)
        stats[:, 0] = st["m"].float()
        stats[:, 1] = st["s"].float()
        stats[:, 2] = st["t"].float()
        stats[:, 3] = st["zt"].float()
        stats[:, 4] = st["m"].float()
        stats[:, 5] = st["idx"].to(torch.int32).view(torch.float32)
        stats[:, 6] = st["hit"].float()
        stats[:, 7] = st["m"].float()        # reference of s, t and acc: the max itself
        acc = None
        if n_grad:
            acc = torch.zeros(n_grad, hidden_cols, dtype=torch.float64)
            hh = h16[:n_grad].to(F16)
            ww = w16[:, :hidden_cols].to(F16)
            for a, b in _chunks(ww.shape[0], n_grad):
                z = logits16(hh, ww, a, b).double()
                acc += torch.exp(z - st["m"][:n_grad, None]) @ ww[a:b].double()
            acc = acc.float()
        return stats, acc

    def combine(self, gathered, rank, n_grad):
        m = gathered[:, :, 0].double()
        ref = gathered[:, :, 7].double()
        big = ref.max(0).values
        w = torch.exp(ref - big)
        s = (gathered[:, :, 1].double() * w).sum(0)
        t = (gathered[:, :, 2].double() * w).sum(0)
        best = gathered[:, :, 4]
        idx = gathered[:, :, 5].contiguous().view(torch.int32).to(torch.int64)
        # first column among the shards' maxima: max value, then the lowest column
        key_best = best.max(0).values
        cand = torch.where(best == key_best, idx, torch.full_like(idx, 2 ** 62))
        hit = gathered[:, :, 6] != 0
        zt = (gathered[:, :, 3] * hit).sum(0)
        out = torch.zeros(gathered.shape[1], 8, dtype=torch.float32)
        out[:, 0] = m.max(0).values.float()
        out[:, 7] = big.float()
        out[:, 1] = s.float()
        out[:, 2] = t.float()
        out[:, 3] = zt
        out[:, 4] = key_best
        out[:, 5] = cand.min(0).values.to(torch.int32).view(torch.float32)
        out[:, 6] = hit.any(0).float()
        scale = (w[rank] / s)[:max(n_grad, 1)].float()
        return out, scale

    def finalize(self, stats, targets, n_grad, acc, acc_scale, w16, ld_w, col0, hidden_cols,
                 grad_rows, want_grad):
        n = stats.shape[0]
        s, t, zt = (stats[:, i].double() for i in range(1, 4))
        m = stats[:, 7].double()             # lse = ref + log(s)
        idx = stats[:, 5].contiguous().view(torch.int32).to(torch.int64)
        labelled = targets >= 0
        ls = torch.log(s)
        out_rows = grad_rows if grad_rows is not None else torch.arange(n)
        token_loss = torch.zeros(n, dtype=torch.float32)
        entropy = torch.zeros(n, dtype=torch.float32)
        correct = torch.zeros(n, dtype=torch.int32)
        token_loss[out_rows] = torch.where(labelled, ls + (m - zt), torch.zeros_like(ls)).float()
        entropy[out_rows] = (m + ls - t / s).float()
        correct[out_rows] = (labelled & (idx == targets)).to(torch.int32)
        grad = None
        if want_grad:
            grad = torch.zeros(n, hidden_cols, dtype=torch.float32)
            if n_grad:
                g = acc.double() * acc_scale[:n_grad, None].double()
                tg = targets[:n_grad]
                own = (tg >= col0) & (tg < col0 + w16.shape[0]) & (tg >= 0)
                rows = own.nonzero().squeeze(1)
                g[rows] -= w16[tg[rows] - col0, :hidden_cols].double()
                g[~labelled[:n_grad]] = 0
                grad[out_rows[:n_grad]] = g.float()
        return token_loss, entropy, correct, grad
