"""The fused head on the GPU through the C ABI against the reference's formulas: golden fixtures
(CPU reference outputs), the reference's own test matrix (solution/test_kernels.py:134-413) and
edge cases, compared with the tolerances the reference's tests use."""

import os

import numpy as np
import pytest
import torch

from tests.head_reference import check_head, gpu_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(hidden, weight, targets, num_items=None, grad_scale=3.0, **kw):
    from talm_b200.fused_head import fused_head_loss

    x = hidden.detach().clone().requires_grad_(True)
    loss, token_loss, entropy, correct = fused_head_loss(x, weight, targets, num_items, **kw)
    (loss * grad_scale).backward()
    assert x.grad.dtype == hidden.dtype and x.grad.shape == hidden.shape
    return (loss.detach(), token_loss, entropy, correct), x.grad


def test_golden_small_cases(golden_dir):
    g = np.load(os.path.join(golden_dir, "head_small.npz"))
    for i in range(int(g["n_cases"])):
        n, vocab, size, chunk, items = (int(v) for v in g[f"c{i}_meta"])
        hidden = torch.from_numpy(g[f"c{i}_hidden"].view(np.float16)).to(DEV)
        weight = torch.from_numpy(g[f"c{i}_weight"].view(np.float16)).to(DEV)
        targets = torch.from_numpy(g[f"c{i}_targets"]).to(DEV)
        out, grad = _run(hidden, weight, targets, None if items < 0 else items,
                         grad_scale=float(g["grad_scale"]), vocab_chunk=chunk)
        loss, token_loss, entropy, correct = out
        torch.testing.assert_close(loss.cpu(), torch.tensor(float(g[f"c{i}_loss"])), rtol=1e-4,
                                   atol=1e-5)
        torch.testing.assert_close(token_loss.cpu(), torch.from_numpy(g[f"c{i}_token_loss"]),
                                   rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(entropy.cpu(), torch.from_numpy(g[f"c{i}_entropy"]),
                                   rtol=1e-4, atol=1e-4)
        ref_correct = torch.from_numpy(g[f"c{i}_correct"])
        fragile = torch.from_numpy(g[f"c{i}_fragile"])
        assert not bool(((correct.cpu() != ref_correct) & ~fragile).any()), f"case {i}"
        ref_grad = torch.from_numpy(g[f"c{i}_grad"])
        torch.testing.assert_close(grad.float().cpu(), ref_grad, rtol=1e-3,
                                   atol=float(ref_grad.abs().max()) * 2 ** -10)


def _plant(hidden, weight, targets, columns, scale):
    """solution/test_kernels.py:104-131: rows along a weight row make that column the clear
    argmax; every other planted row targets the column next to it (a miss)."""
    vocab = weight.shape[0]
    hits = 0
    for i, col in enumerate(columns):
        row = 1 + i
        if row >= hidden.shape[0] - 1:
            break
        hidden[row] = (weight[col].float() * scale).to(hidden.dtype)
        if i % 2 == 0:
            targets[row] = col
            hits += 1
        else:
            targets[row] = col + 1 if col + 1 < vocab else col - 1
    return hits


@pytest.mark.parametrize("hidden_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("n_tokens,vocab,vocab_chunk",
                         [(2048, 151936, None), (37, 151936, 20000), (300, 1000, 384),
                          (5, 4097, 4096)])
@pytest.mark.parametrize("num_items", ["tensor", "int", None])
def test_matches_reference(hidden_dtype, n_tokens, vocab, vocab_chunk, num_items):
    """solution/test_kernels.py:134-184."""
    torch.manual_seed(0)
    size = 1536 if vocab > 10000 else 64
    hidden = torch.randn(n_tokens, size, device=DEV, dtype=hidden_dtype) * 2
    weight = torch.randn(vocab, size, device=DEV) * 0.05
    targets = torch.randint(0, vocab, (n_tokens,), device=DEV)
    targets[torch.rand(n_tokens, device=DEV) < 0.45] = -100
    targets[0] = -100
    if n_tokens > 2:
        targets[-1] = -100
    chunk = vocab_chunk or 8192
    last = (vocab - 1) // chunk * chunk
    cols = [c for c in dict.fromkeys([0, 4095, 4096, chunk - 1, chunk, last, vocab - 1])
            if 0 <= c < vocab]
    planted = _plant(hidden, weight, targets, cols, 40.0)
    labelled = int((targets >= 0).sum())
    items = {"tensor": torch.tensor(labelled + 3, device=DEV), "int": labelled + 3,
             None: None}[num_items]
    ref = gpu_reference(hidden, weight, targets, None if items is None else int(items),
                        grad_scale=3.0)
    out, grad = _run(hidden, weight, targets, items, vocab_chunk=vocab_chunk)
    check_head(out, ref, grad, f"N={n_tokens} V={vocab} {hidden_dtype} items={num_items}")
    assert int(ref["correct"].sum()) >= planted > 0
    assert torch.equal(out[3], ref["correct"]) or bool(ref["fragile"].any())


@pytest.mark.parametrize("vocab_chunk", [1, 256, 300, 8192, 200000])
def test_vocab_chunk_widths(vocab_chunk):
    """Slice widths below a tile, not a multiple of it, and wider than the vocabulary."""
    torch.manual_seed(2)
    n, vocab, size = 200, 5000, 128
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16)
    weight = (torch.randn(vocab, size, device=DEV) * 0.1).half()
    targets = torch.randint(0, vocab, (n,), device=DEV)
    targets[::3] = -100
    ref = gpu_reference(hidden, weight, targets, grad_scale=3.0)
    out, grad = _run(hidden, weight, targets, vocab_chunk=vocab_chunk)
    check_head(out, ref, grad, f"chunk={vocab_chunk}")


def test_argmax_ties_report_the_first_column():
    """solution/test_kernels.py:250-282: exact ties inside a tile, across tiles, slices and the
    narrower last slice resolve to the first column."""
    from talm_b200.fused_head import fused_head_loss

    torch.manual_seed(13)
    n, size, vocab = 16, 256, 151936
    pairs = [(4096 + 10, 4096 + 20), (1000, 4096 + 1000), (100, 8192 + 50),
             (vocab - 4000, vocab - 1), (255, 256), (511, 8191)]
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16) * 2
    weight = torch.randn(vocab, size, device=DEV) * 0.05
    targets = torch.full((n,), -100, dtype=torch.long, device=DEV)
    signs = torch.randint(0, 2, (len(pairs), size), device=DEV).float() * 2 - 1
    for i, (first, second) in enumerate(pairs):
        weight[first] = weight[second] = signs[i] / 16
        hidden[2 * i] = hidden[2 * i + 1] = (signs[i] * 4).half()
        targets[2 * i], targets[2 * i + 1] = first, second
    logits = hidden @ weight.half().t()
    for i, (first, second) in enumerate(pairs):
        for row in (2 * i, 2 * i + 1):
            assert logits[row, first] == logits[row, second] == logits[row].max() == 64
    ref_correct = (logits.argmax(-1) == targets) & (targets >= 0)
    with torch.no_grad():
        *_, correct = fused_head_loss(hidden, weight, targets, None)
    assert torch.equal(correct, ref_correct)
    assert correct[:2 * len(pairs)].tolist() == [True, False] * len(pairs)


def test_no_grad_path():
    from talm_b200.fused_head import fused_head_loss

    torch.manual_seed(1)
    hidden = torch.randn(64, 1536, device=DEV, dtype=torch.float16)
    weight = torch.randn(151936, 1536, device=DEV) * 0.05
    targets = torch.randint(0, 151936, (64,), device=DEV)
    with torch.no_grad():
        out = fused_head_loss(hidden, weight, targets, None)
    check_head(out, gpu_reference(hidden, weight, targets), None, "no grad")


def test_unlabelled_rows_never_produce_nan():
    """solution/test_kernels.py:667-680: large logits on unlabelled rows."""
    torch.manual_seed(6)
    hidden = torch.randn(512, 1536, device=DEV) * 60
    weight = torch.randn(151936, 1536, device=DEV) * 0.5
    targets = torch.randint(0, 151936, (512,), device=DEV)
    targets[::2] = -100
    _, grad = _run(hidden, weight, targets, grad_scale=4096.0)
    assert torch.isfinite(grad).all()
    assert (grad[targets < 0] == 0).all()


def test_large_accumulator_matches_reference():
    """Enough labelled rows (about 5400, 132 accumulator tiles) that each slice step's
    accumulator tiles outnumber the CTA pairs and share the launch with the next slice's
    logits tiles; planted confident rows move their reference in late slices, so their
    probability and accumulator rows are rescaled between slices."""
    torch.manual_seed(5)
    n, vocab, size = 6000, 151936, 1536
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16) * 2
    weight = torch.randn(vocab, size, device=DEV) * 0.05
    targets = torch.randint(0, vocab, (n,), device=DEV)
    targets[torch.rand(n, device=DEV) < 0.1] = -100
    cols = [0, 8191, 8192, 65536, 131071, 147455, vocab - 1]
    planted = _plant(hidden, weight, targets, cols * 40, 40.0)
    ref = gpu_reference(hidden, weight, targets, grad_scale=3.0)
    out, grad = _run(hidden, weight, targets, vocab_chunk=8192)
    check_head(out, ref, grad, "large accumulator")
    assert int(ref["correct"].sum()) >= planted > 0
    assert torch.equal(out[3], ref["correct"]) or bool(ref["fragile"].any())


def test_repeated_calls_are_bit_identical():
    """Every acc element receives exactly one addition per slice (whole tiles, no split K), so
    two calls on the same inputs return the same bits - at a size where the accumulator GEMM
    has more tiles than the GPU has CTA pairs."""
    torch.manual_seed(17)
    n, vocab, size = 5000, 151936, 1536
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16) * 2
    weight = (torch.randn(vocab, size, device=DEV) * 0.05).half()
    targets = torch.randint(0, vocab, (n,), device=DEV)
    targets[torch.rand(n, device=DEV) < 0.2] = -100
    runs = [_run(hidden, weight, targets, vocab_chunk=8192) for _ in range(2)]
    for a, b in zip(runs[0][0], runs[1][0]):
        assert torch.equal(a, b)
    assert torch.equal(runs[0][1], runs[1][1])


@pytest.mark.parametrize("n_tokens,vocab,unlabelled",
                         [(700, 151936, 0.45), (37, 151936, 0.3), (300, 1000, 0.0),
                          (300, 1000, 1.0), (5, 4097, 0.5)])
def test_compaction_matches_full_accumulator(monkeypatch, n_tokens, vocab, unlabelled):
    """solution/test_kernels.py:345-381: loss / per-token outputs identical with the accumulator
    over the labelled rows only or over all rows; the gradient within the compaction bound;
    the same result whether the caller passes the labelled count or the head counts it."""
    from talm_b200 import fused_head

    torch.manual_seed(13)
    size = 1536 if vocab > 10000 else 64
    weight = torch.randn(vocab, size, device=DEV) * 0.03
    hidden = (torch.randn(n_tokens, size, device=DEV) * 1.5).half()
    targets = torch.randint(0, vocab, (n_tokens,), device=DEV)
    targets[torch.rand(n_tokens, device=DEV) < unlabelled] = -100
    n_lab = int((targets >= 0).sum())
    outs = {}
    for name, compact, given in (("full", False, None), ("compact", True, n_lab),
                                 ("counted", True, None)):
        monkeypatch.setattr(fused_head, "COMPACT", compact)
        out, grad = _run(hidden, weight, targets, None, 1024.0, n_labelled=given)
        outs[name] = (*out, grad)
    for a, b in zip(outs["full"][:4], outs["compact"][:4]):
        assert torch.equal(a, b)
    for a, b in zip(outs["compact"], outs["counted"]):
        assert torch.equal(a, b)
    full, compact = outs["full"][4].float(), outs["compact"][4].float()
    torch.testing.assert_close(compact, full, rtol=1e-3, atol=float(full.abs().max()) * 2 ** -10)
    assert (outs["compact"][4][targets < 0] == 0).all()


@pytest.mark.parametrize("size", [8, 40, 77, 100, 192, 255, 320])
def test_odd_hidden_sizes_and_layouts(size):
    """Hidden sizes that are not multiples of 8 / 64, an fp32 weight, a padded-row weight and a
    bf16 hidden (the wrapper casts and pads; the kernels see fp16 TMA rows). 192 and 320 are
    odd numbers of 64-column blocks: their walks mix two-sub-block stages fetched by one 3-D
    request per operand with a last stage of one sub-block fetched by 2-D boxes, and their
    accumulator tiles reach past the last weight column group."""
    torch.manual_seed(size)
    n, vocab = 90, 3000
    hidden = torch.randn(n, size, device=DEV, dtype=torch.bfloat16)
    base = torch.randn(vocab, size + 8, device=DEV) * 0.1
    weight = base[:, :size]                       # padded rows, fp32
    targets = torch.randint(0, vocab, (n,), device=DEV)
    targets[::4] = -100
    ref = gpu_reference(hidden, weight, targets, grad_scale=3.0)
    out, grad = _run(hidden, weight, targets)
    check_head(out, ref, grad, f"H={size}")


@pytest.mark.parametrize("labels", ["none", "all"])
def test_all_or_no_labels(labels):
    torch.manual_seed(9)
    n, vocab, size = 130, 2000, 64
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16)
    weight = torch.randn(vocab, size, device=DEV) * 0.1
    targets = torch.randint(0, vocab, (n,), device=DEV)
    if labels == "none":
        targets.fill_(-100)
    ref = gpu_reference(hidden, weight, targets, grad_scale=3.0)
    out, grad = _run(hidden, weight, targets)
    check_head(out, ref, grad, labels)
    if labels == "none":
        assert float(out[0]) == 0.0 and (grad == 0).all()


def test_zero_num_items_gives_zero_gradient():
    """solution/test_robustness.py:369-443: num_items = 0 -> inf/nan loss as transformers has it,
    but a zero gradient."""
    torch.manual_seed(10)
    hidden = torch.randn(33, 64, device=DEV, dtype=torch.float16)
    weight = torch.randn(700, 64, device=DEV) * 0.1
    targets = torch.randint(0, 700, (33,), device=DEV)
    _, grad = _run(hidden, weight, targets, num_items=0)
    assert (grad == 0).all()


def test_device_status_clean_after_runs():
    from talm_b200 import _lib

    assert _lib.device_status() == 0


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_backward_scale_kernel_matches_oracle(out_dtype):
    """talm_head_scale_grad against the reference's backward expression (fused_head.py:280-287):
    fp16 and fp32 saved gradients, a padded row stride, an odd row length, denom 0 - bit-exact."""
    from types import SimpleNamespace

    from oracle.head import scale_grad
    from talm_b200.fused_head import _head_backward

    torch.manual_seed(11)
    cases = [torch.randn(37, 40, device=DEV).half(),
             torch.randn(37, 48, device=DEV).half()[:, :40],
             torch.randn(1000, 1536, device=DEV) * 3,
             torch.randn(5, 13, device=DEV).half(),
             torch.randn(6, 13, device=DEV)]
    for g in cases:
        for gl, dn in ((2.5, 7.0), (1.0, 3.0), (4.0, 0.0)):
            gl_t = torch.tensor(gl, device=DEV)
            ctx = SimpleNamespace(saved_tensors=(g,), denom=torch.tensor(dn, device=DEV),
                                  out_dtype=out_dtype)
            out = _head_backward(ctx, gl_t)
            ref = scale_grad(g, gl_t, ctx.denom, out_dtype)
            assert out.dtype == out_dtype and out.shape == g.shape
            assert torch.equal(out, ref), (tuple(g.shape), g.dtype, gl, dn)


@pytest.mark.parametrize("n,frac", [(1, 0.5), (1000, 0.45), (1024, 0.0), (3001, 1.0), (20000, 0.3)])
def test_device_labelled_first_matches_reference_order(n, frac):
    """talm_head_labelled_first (one scanning CTA + a row gather) against labelled_first
    (fused_head.py:290-299) and index_select: identical order, rows and targets."""
    from talm_b200.fused_head import labelled_first, labelled_first_rows

    g = torch.Generator(device=DEV).manual_seed(n)
    targets = torch.randint(0, 1000, (n,), generator=g, device=DEV)
    targets[torch.rand(n, generator=g, device=DEV) < frac] = -100
    hidden = torch.randn(n, 40, generator=g, device=DEV).half()
    n_lab = int((targets >= 0).sum())
    rows, rows_targets, src = labelled_first_rows(hidden, targets, n_lab)
    _dest, ref_src = labelled_first(targets >= 0, n_lab)
    assert torch.equal(src, ref_src)
    assert torch.equal(rows, hidden.index_select(0, ref_src))
    assert torch.equal(rows_targets, targets.index_select(0, ref_src))


def test_token_chunked_entry_point_matches_the_vocab_path():
    """solution/test_kernels.py:285-330: `token_chunk=` selects FusedHeadLoss (the reference's
    token-chunked path, routed here to the same sm_100a walk) - the same loss, per-token loss,
    entropy and accuracy as the vocabulary-sliced entry point, both against the reference's
    formulas, with confident rows among ordinary ones; the dispatch counters move as the
    reference's do (fused_head.py:447-462)."""
    from talm_b200.engaged import FELL_BACK, RAN
    from talm_b200.fused_head import fused_head_loss

    torch.manual_seed(11)
    n, size, vocab = 700, 1536, 151936
    weight = (torch.randn(vocab, size, device=DEV) * 0.03).half()
    targets = torch.randint(0, vocab, (n,), device=DEV)
    targets[torch.rand(n, device=DEV) < 0.35] = -100
    hidden = torch.randn(n, size, device=DEV, dtype=torch.float16) * 1.5
    confident = (torch.rand(n, device=DEV) < 0.3) & (targets >= 0)
    hidden[confident] = (weight[targets[confident]].float() * 400).half()
    outs = {}
    for path, kw in (("tokens", {"token_chunk": 256}), ("vocab", {})):
        ran, fell = RAN["vchunk"], FELL_BACK["vchunk"]
        x = hidden.clone().requires_grad_(True)
        loss, token_loss, entropy, correct = fused_head_loss(x, weight, targets, None, **kw)
        (loss * 1024.0).backward()
        outs[path] = (loss.detach(), token_loss, entropy, correct, x.grad)
        if path == "tokens":
            assert (RAN["vchunk"], FELL_BACK["vchunk"]) == (ran, fell + 1)
        else:
            assert (RAN["vchunk"], FELL_BACK["vchunk"]) == (ran + 1, fell)
    for a, b in zip(outs["tokens"], outs["vocab"]):
        assert torch.equal(a, b)
    ref = gpu_reference(hidden, weight, targets, grad_scale=1024.0)
    check_head(outs["tokens"][:4], ref, outs["tokens"][4], "token_chunk=256")
    assert (outs["tokens"][4][targets < 0] == 0).all()
