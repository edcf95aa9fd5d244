"""Test helper: the reference head computed with PyTorch on the GPU (cuBLAS fp16 GEMM -> fp16
logits, then fp32/fp64 statistics), for sizes the CPU oracle would take minutes on, and the
reference's tolerance checks. Test infrastructure only.

The formulas are solution/test_kernels.py:70-83 (`reference_head`) and the float64 variant of
solution/test_fuzz.py:145-185 (first-maximum argmax, `fragile` near-tie rows, dH =
(softmax - onehot) W16), walked in vocabulary chunks so the [N, V] logits never exist at once.
"""

import torch

F16 = torch.float16


@torch.no_grad()
def gpu_reference(hidden, weight, targets, num_items=None, grad_scale=1.0, chunk=16384):
    h16 = hidden.detach().to(F16)
    w16 = weight.detach().to(F16)
    n = h16.shape[0]
    vocab = w16.shape[0]
    dev = h16.device
    m = torch.full((n,), -float("inf"), dtype=torch.float64, device=dev)
    s = torch.zeros(n, dtype=torch.float64, device=dev)
    t = torch.zeros(n, dtype=torch.float64, device=dev)
    zt = torch.zeros(n, dtype=torch.float64, device=dev)
    idx = torch.zeros(n, dtype=torch.int64, device=dev)
    zmax = torch.zeros(n, dtype=torch.float64, device=dev)
    tc = targets.clamp(min=0)
    labelled = targets >= 0
    for a in range(0, vocab, chunk):
        b = min(vocab, a + chunk)
        z = (h16 @ w16[a:b].t()).double()          # fp16 GEMM output, as the reference
        cm, ci = z.max(-1)
        better = cm > m
        idx = torch.where(better, ci + a, idx)
        m_new = torch.maximum(m, cm)
        e = torch.exp(z - m_new[:, None])
        alpha = torch.exp(m - m_new)
        s = s * alpha + e.sum(-1)
        t = t * alpha + (e * z).sum(-1)
        m = m_new
        zmax = torch.maximum(zmax, z.abs().max(-1).values)
        here = (tc >= a) & (tc < b)
        rows = here.nonzero().squeeze(1)
        zt[rows] = z[rows, tc[rows] - a]
    lse = m + torch.log(s)
    token_loss = torch.where(labelled, lse - zt, torch.zeros_like(lse))
    entropy = lse - t / s
    correct = labelled & (idx == targets)
    # fragile rows: the target within 8 fp16 ulps of the row max, next to another such logit
    ulp = torch.exp2(torch.floor(torch.log2(m.abs().clamp(min=torch.finfo(F16).tiny)))) \
        * torch.finfo(F16).eps
    near_lo = m - 8 * ulp
    count = torch.zeros(n, dtype=torch.int64, device=dev)
    tnear = torch.zeros(n, dtype=torch.bool, device=dev)
    grad = torch.zeros(n, h16.shape[1], dtype=torch.float32, device=dev)
    for a in range(0, vocab, chunk):
        b = min(vocab, a + chunk)
        z = (h16 @ w16[a:b].t()).double()
        near = z >= near_lo[:, None]
        count += near.sum(-1)
        here = (tc >= a) & (tc < b)
        rows = here.nonzero().squeeze(1)
        tnear[rows] = near[rows, tc[rows] - a]
        p = torch.exp(z - lse[:, None]).float()
        grad += p @ w16[a:b].float()
    grad -= w16[tc].float()
    grad[~labelled] = 0
    n_lab = int(labelled.sum())
    denom = float(num_items) if num_items is not None else float(max(n_lab, 1))
    scale = grad_scale / denom if denom != 0 else 0.0
    return {
        "loss": (token_loss.sum() / denom).float() if denom else token_loss.sum().float() * 0,
        "token_loss": token_loss.float(), "entropy": entropy.float(), "correct": correct,
        "fragile": labelled & tnear & (count >= 2), "grad": grad * scale, "zmax": zmax,
        "labelled": labelled,
    }


def check_head(out, ref, grad=None, what=""):
    """The reference's tolerances (solution/test_kernels.py:172-183; the north star's 1e-3
    relative on loss and dH): loss rtol 1e-4, per-token loss / entropy 1e-4 (scaled by |z| for
    large logits), correctness exact outside fragile rows, dH rtol 1e-3 + atol 2^-10 max|dH|."""
    loss, token_loss, entropy, correct = out
    torch.testing.assert_close(loss.float(), ref["loss"], rtol=1e-4, atol=1e-5, msg=what)
    tol = 1e-4 + 2e-6 * ref["zmax"].float()
    assert bool(((token_loss - ref["token_loss"]).abs() <= tol + 1e-4 * ref["token_loss"].abs())
                .all()), f"{what}: per-token loss, max err " \
        f"{float((token_loss - ref['token_loss']).abs().max()):.3g}"
    assert bool(((entropy - ref["entropy"]).abs() <= tol + 1e-4 * ref["entropy"].abs()).all()), \
        f"{what}: entropy, max err {float((entropy - ref['entropy']).abs().max()):.3g}"
    flips = correct != ref["correct"]
    assert not bool((flips & ~ref["fragile"]).any()), \
        f"{what}: correctness differs on {int((flips & ~ref['fragile']).sum())} non-fragile rows"
    assert bool((token_loss[~ref["labelled"]] == 0).all()), f"{what}: loss on unlabelled rows"
    if grad is not None:
        rg = ref["grad"]
        # plus one ulp of an output dtype coarser than fp16 (bf16 hidden states get a bf16
        # gradient), as solution/test_fuzz.py:332-338 adds _ulp(ref_grad, grad.dtype)
        rtol = 1e-3 + (torch.finfo(grad.dtype).eps if grad.dtype == torch.bfloat16 else 0.0)
        torch.testing.assert_close(grad.float(), rg, rtol=rtol,
                                   atol=float(rg.abs().max()) * 2 ** -10, msg=what)
        assert bool((grad[~ref["labelled"]] == 0).all()), f"{what}: gradient on unlabelled rows"
        assert bool(torch.isfinite(grad).all()), f"{what}: non-finite gradient"
