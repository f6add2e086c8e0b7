"""Data-parallel gradient averaging on world_size-2 gloo process groups (CPU), including a
rank that fails before the collective: the surviving rank must end with an error from the
short process-group timeout instead of hanging."""

import datetime
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


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _average_worker(rank, world, port, queue):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "poly-tensors_b200"))
    from polytensors_b200 import PolyTensor
    from polytensors_b200.parallel import allreduce_gradients

    _init(rank, world, port)
    try:
        params = []
        for i, shape in enumerate([(5, 3), (7,), (2, 2, 2)]):
            p = PolyTensor(tuple(torch.zeros(shape) for _ in range(4)), requires_grad=True)
            p.grad = PolyTensor(tuple(torch.full(shape, float(rank * 10 + i * 100 + k)) for k in range(4)))
            params.append(p)
        allreduce_gradients(params, bucket_bytes=64)   # several buckets
        # plain lists: a tensor sent through the queue lives in shared memory that this process
        # removes when it exits, possibly before the parent has received it
        got = [[c.tolist() for c in p.grad.coeffs] for p in params]
        queue.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_allreduce_averages_every_plane():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_average_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        for i, planes in enumerate(results[rank]):
            for k, c in enumerate(planes):
                assert torch.all(torch.tensor(c) == (0 + 10) / 2 + i * 100 + k)


def _failing_worker(rank, world, port, queue):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "poly-tensors_b200"))
    from polytensors_b200 import PolyTensor
    from polytensors_b200.parallel import allreduce_gradients

    _init(rank, world, port, timeout_s=5)
    p = PolyTensor((torch.zeros(4), torch.zeros(4)), requires_grad=True)
    p.grad = PolyTensor((torch.ones(4), torch.ones(4)))
    if rank == 1:
        os._exit(3)   # the rank dies between steps, before the collective
    try:
        allreduce_gradients([p])
        queue.put((rank, "completed"))
    except Exception as e:   # the short timeout ends the collective with an error
        queue.put((rank, "error: " + type(e).__name__))


def test_failed_rank_surfaces_as_error_not_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    rank, message = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    assert rank == 0 and message.startswith("error"), message


def _overlap_worker(rank, world, port, queue):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "poly-tensors_b200"))
    from polytensors_b200.parallel import OverlappedAllReduce

    _init(rank, world, port)
    try:
        torch.manual_seed(0)
        layers = [torch.nn.Linear(6, 6) for _ in range(4)]
        unused = torch.nn.Parameter(torch.zeros(3))   # never gets a gradient (skipped on every rank)
        params = [p for l in layers for p in l.parameters()] + [unused]
        ar = OverlappedAllReduce(params, bucket_bytes=200)   # several buckets
        x_all = torch.randn(2, 3, 6, generator=torch.Generator().manual_seed(1))
        for step in range(2):   # the first step finds the unused parameter, the second runs without it
            for p in params:
                p.grad = None
            for micro in range(3):   # gradient accumulation; only the last backward launches buckets
                x = x_all[rank] * (micro + 1)
                for l in layers:
                    x = torch.tanh(l(x))
                if micro == 2:
                    ar.arm()
                x.sum().backward()
            launched_during = ar.next_launch
            ar.finish()
        got = [p.grad.tolist() if p.grad is not None else None for p in params]
        queue.put((rank, got, launched_during, len(ar.buckets)))
    finally:
        dist.destroy_process_group()


def test_overlapped_allreduce_matches_the_average():
    """Buckets are launched from the gradient hooks during the last backward (several of them before
    finish()), and the result equals the average over ranks of each rank's accumulated gradient."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_overlap_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: (g, n, nb) for r, g, n, nb in (queue.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # reference: each rank's accumulated gradients computed here, then averaged
    torch.manual_seed(0)
    layers = [torch.nn.Linear(6, 6) for _ in range(4)]
    x_all = torch.randn(2, 3, 6, generator=torch.Generator().manual_seed(1))
    per_rank = []
    for rank in range(world):
        for l in layers:
            l.zero_grad()
        for micro in range(3):
            x = x_all[rank] * (micro + 1)
            for l in layers:
                x = torch.tanh(l(x))
            x.sum().backward()
        per_rank.append([p.grad.clone() for l in layers for p in l.parameters()])
    want = [(a + b) / 2 for a, b in zip(*per_rank)]
    for rank in range(world):
        got, launched, nbuckets = results[rank]
        assert nbuckets > 2 and launched >= nbuckets - 1, (launched, nbuckets)
        assert got[-1] is None
        for g, w in zip(got[:-1], want):
            assert torch.allclose(torch.tensor(g), w, atol=1e-6)
