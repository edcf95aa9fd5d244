"""The vocabulary-parallel head over NCCL on 2+ GPUs (one process per GPU) against the
single-GPU fused head on the same inputs: identical per-token outputs (up to fp32 merge order),
the same accuracy, and the gradient within the head's tolerance. The peer flow with the scatter
inside the walk's last accumulator GEMM must give the same bits as the peer flow with a
separate finalize pass. Skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(n, vocab, size, device, unlabelled=0.4):
    g = torch.Generator(device=device).manual_seed(31)
    hidden = torch.randn(n, size, generator=g, device=device).half()
    weight = (torch.randn(vocab, size, generator=g, device=device) * 0.05).half()
    targets = torch.randint(0, vocab, (n,), generator=g, device=device)
    targets[torch.rand(n, generator=g, device=device) < unlabelled] = -100
    hidden[1] = (weight[vocab - 3].float() * 30).half()   # a confident row in the last shard
    targets[1] = vocab - 3
    # an ordinary labelled row in every case: the confident row's gradient alone is almost
    # all cancellation, too small to set the gradient tolerance
    targets[2] = 7
    return hidden, weight, targets


def _worker(rank, world, port, q, sizes, vocab, size, flow):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from talm_b200 import vocab_parallel
        from talm_b200.fused_head import fused_head_loss
        from talm_b200.vocab_parallel import shard_bounds, vocab_parallel_head_loss

        vocab_parallel.PEER_EXCHANGE = flow != "nccl"
        col0, cols = shard_bounds(vocab, world, rank)

        def sharded(hidden, weight, targets, fused):
            vocab_parallel.FUSED_SCATTER = fused
            x = hidden.clone().requires_grad_(True)
            out = vocab_parallel_head_loss(x, weight[col0:col0 + cols], targets, vocab, col0,
                                           None, 2048)
            (out[0] * 7.0).backward()
            return [t.detach().cpu() for t in out], x.grad.cpu()

        results = []
        # several calls: the peer buffers are reused (epochs) and grow once (600 -> 1500 rows);
        # partly labelled rows (compacted), every row labelled, and only rows 1 and 2 labelled
        for n, unlabelled in sizes:
            hidden, weight, targets = _case(n, vocab, size, dev, unlabelled)
            out, grad = sharded(hidden, weight, targets, True)
            # the same exchange with a separate finalize pass (peer flow only)
            split = sharded(hidden, weight, targets, False) if flow == "peer" else None
            y = hidden.clone().requires_grad_(True)
            ref = fused_head_loss(y, weight, targets, None, 2048)
            (ref[0] * 7.0).backward()
            results.append((out, grad, [t.detach().cpu() for t in ref], y.grad.cpu(), split))
        from talm_b200 import _lib
        q.put((rank, results, _lib.device_status()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("flow", ["peer", "nccl"])
def test_vocab_parallel_matches_single_gpu(flow):
    """Both exchange flows: the library's NVLink peer exchange and NCCL collectives."""
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    sizes, vocab, size = ((600, 0.4), (1500, 0.0), (600, 0.4), (300, 1.0)), 30011, 512
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, sizes, vocab, size, flow))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, calls, status in results:
        assert status == 0, f"rank {rank}: device status {status}"
        for out, grad, ref, ref_grad, split in calls:
            if split is not None:  # scatter in the last accumulator GEMM: the same bits
                for a, b in zip(out + [grad], split[0] + [split[1]]):
                    assert torch.equal(a, b), f"rank {rank}: fused scatter differs"
            loss, token_loss, entropy, correct = out
            r_loss, r_tl, r_ent, r_corr = ref
            torch.testing.assert_close(loss, r_loss, rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(token_loss, r_tl, rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(entropy, r_ent, rtol=1e-5, atol=1e-5)
            assert torch.equal(correct, r_corr), f"rank {rank}"
            torch.testing.assert_close(grad.float(), ref_grad.float(), rtol=1e-3,
                                       atol=float(ref_grad.abs().max()) * 2 ** -10)
