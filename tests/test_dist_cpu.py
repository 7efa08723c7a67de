"""Data-parallel host logic on CPU ranks (gloo, world size 2): the per-layer
gradient buckets sum correctly and in the same order on every rank, the rank
windows reproduce one global batch, and a rank that never joins makes the
others' collective fail within the process-group timeout (host-side failure,
no GPU involved)."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _bucket_worker(rank, world, port, queue):
    try:
        import sys
        sys.path.insert(0, os.getcwd())
        from reversability_b200.dist import GradBuckets
        from reversability_b200 import data as rdata
        _init(rank, world, port)
        torch.manual_seed(rank)
        flat = torch.randn(1000)
        sizes = [100, 250, 50, 400, 200]
        offs = [0]
        for n in sizes:
            offs.append(offs[-1] + n)
        slices = [flat[offs[i]:offs[i + 1]] for i in range(len(sizes))]
        expected = torch.zeros(1000)
        for r in range(world):
            torch.manual_seed(r)
            expected += torch.randn(1000)
        b = GradBuckets(slices, None, torch.device("cpu"))
        for i in reversed(range(3)):  # layers finish in reverse order
            b.launch(i)
        b.launch(3)
        b.launch(4)
        order = b.finish()
        orders = [None] * world
        dist.all_gather_object(orders, order)
        ok_sum = torch.allclose(flat, expected, rtol=1e-6, atol=1e-6)
        # data windows: concatenating the ranks' batches equals one global batch_at
        B, T, acc = 2, 8, 2
        stream = rdata.synthetic_stream(world * acc * B * T * 2 + 1, seed=4, vocab_size=101, eos=100, mean_doc=30.0)
        batches, targets = rdata.update_batches(stream, 0, rank, world, B, T, acc, len(stream) - 1)
        mine = torch.stack([x for x, _, _ in batches])
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        gx, _, gc = rdata.batch_at(stream, 0, world * acc * B, T, world * acc * B * T)
        pieces = [gathered[r][m] for m in range(acc) for r in range(world)]
        ok_data = torch.equal(torch.cat(pieces), gx) and targets == gc
        queue.put((rank, ok_sum, orders[0] == orders[1], ok_data))
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        queue.put((rank, repr(exc), False, False))


def _timeout_worker(rank, world, port, queue):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            os._exit(0)  # leaves between steps: nothing of this rank is in flight
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
            queue.put((rank, "no error", time.time() - t0))
        except Exception as exc:
            queue.put((rank, type(exc).__name__, time.time() - t0))
    except Exception as exc:
        queue.put((rank, "setup:" + repr(exc), 0.0))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            results.append(queue.get(timeout=1))
        except Exception:
            if all(not p.is_alive() for p in procs) and queue.empty():
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return results


def test_grad_buckets_and_rank_windows_gloo():
    res = _run(_bucket_worker)
    assert len(res) == 2, res
    for rank, ok_sum, same_order, ok_data in res:
        assert ok_sum is True, (rank, ok_sum)
        assert same_order and ok_data, (rank, same_order, ok_data)


def test_missing_rank_makes_collective_fail_within_timeout():
    res = _run(_timeout_worker)
    survivors = [r for r in res if r[0] == 0]
    assert survivors, res
    _, outcome, elapsed = survivors[0]
    assert outcome != "no error" and not outcome.startswith("setup"), survivors
    assert elapsed < 60


def _tied_split_worker(rank, world, port, queue):
    """The trainer's bucket order with the tied-gradient split: the loss sum,
    then the head share of the tied gradient (before the sweep), the layer
    buckets in reverse, then the embedding scatter share, position and final
    norm; the two reduced shares summed equal the reduced total."""
    try:
        import sys
        sys.path.insert(0, os.getcwd())
        from reversability_b200.dist import GradBuckets
        _init(rank, world, port)
        g = torch.Generator().manual_seed(100 + rank)
        n_layers, V, d = 3, 11, 4
        flat = torch.randn(n_layers * 20 + V * d + 6 + 3, generator=g)
        layers = [flat[i * 20:(i + 1) * 20] for i in range(n_layers)]
        o = n_layers * 20
        g_tok, g_pos, g_final = flat[o:o + V * d].view(V, d), flat[o + V * d:o + V * d + 6], flat[-3:]
        loss = torch.randn((), generator=g)
        g_head = torch.randn(V, d, generator=g)
        total = [None] * world
        dist.all_gather_object(total, (flat.clone(), g_head.clone(), loss.clone()))
        b = GradBuckets(layers + [g_tok, g_pos, g_final, loss, g_head], None, torch.device("cpu"))
        b.launch(n_layers + 3)  # loss
        b.launch(n_layers + 4)  # head share, beside the sweep
        for i in reversed(range(n_layers)):
            b.launch(i)
        for i in range(n_layers, n_layers + 3):
            b.launch(i)
        order = b.finish()
        g_tok.add_(g_head)
        exp_flat = sum(t[0] for t in total)
        exp_tok = sum(t[0][o:o + V * d].view(V, d) + t[1] for t in total)
        ok = (torch.allclose(g_tok, exp_tok, rtol=1e-6, atol=1e-6)
              and torch.allclose(flat[:o], exp_flat[:o], rtol=1e-6, atol=1e-6)
              and torch.allclose(flat[o + V * d:], exp_flat[o + V * d:], rtol=1e-6, atol=1e-6)
              and torch.allclose(loss, sum(t[2] for t in total), rtol=1e-6))
        queue.put((rank, ok, order))
        dist.destroy_process_group()
    except Exception as exc:
        queue.put((rank, repr(exc), None))


def test_tied_gradient_split_buckets_gloo():
    res = _run(_tied_split_worker)
    assert len(res) == 2, res
    assert all(ok is True for _, ok, _ in res), res
    assert res[0][2] == res[1][2]
