"""The vocabulary-parallel exchange (all_gather of per-row statistics, local merge, all_reduce of
the partial gradients) on world_size 2 and 3 CPU ranks over gloo, with the kernel steps taken by
the oracle's CPU restatement; every rank's outputs must equal the single-device oracle head."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed, n, vocab, size):
    g = torch.Generator().manual_seed(seed)
    hidden = (torch.randn(n, size, generator=g) * 2).half()
    weight = (torch.randn(vocab, size, generator=g) * 0.05).half()
    targets = torch.randint(0, vocab, (n,), generator=g)
    targets[torch.rand(n, generator=g) < 0.4] = -100
    targets[0] = -100
    # planted hits on shard boundaries and a tie across two shards
    hidden[1] = (weight[vocab // 2].float() * 40).half()
    targets[1] = vocab // 2
    weight[vocab - 1] = weight[3]
    hidden[2] = (weight[3].float() * 40).half()
    targets[2] = vocab - 1          # tie with column 3: the first column wins, a miss
    return hidden, weight, targets


def _worker(rank, world, port, out_q, seed, n, vocab, size):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.head import CpuHeadOps
        from talm_b200 import vocab_parallel

        hidden, weight, targets = _case(seed, n, vocab, size)
        col0, cols = vocab_parallel.shard_bounds(vocab, world, rank)
        loss, token_loss, entropy, correct, grad = vocab_parallel.sharded_head(
            hidden, weight[col0:col0 + cols], targets, vocab, col0, None, 64, True,
            None, None, CpuHeadOps())
        out_q.put((rank, loss, token_loss, entropy, correct, grad))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_head_matches_single_device_oracle(world):
    from oracle.head import reference_head

    seed, n, vocab, size = 5, 23, 301, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, seed, n, vocab, size))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    hidden, weight, targets = _case(seed, n, vocab, size)
    ref_loss, ref_tl, ref_ent, ref_corr, ref_grad = reference_head(hidden, weight, targets)
    assert not bool(ref_corr[2]) and bool(ref_corr[1])
    for rank, loss, tl, ent, corr, grad in results:
        torch.testing.assert_close(loss, ref_loss, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(tl, ref_tl, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ent, ref_ent, rtol=1e-5, atol=1e-5)
        assert torch.equal(corr, ref_corr), f"rank {rank}"
        # the shards' gradients sum to the full one (unscaled by the loss denominator)
        denom = float(max(int((targets >= 0).sum()), 1))
        torch.testing.assert_close(grad.float() / denom, ref_grad, rtol=1e-3,
                                   atol=float(ref_grad.abs().max()) * 2 ** -10)
        assert (grad[targets < 0] == 0).all()
