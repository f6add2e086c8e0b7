"""Batch-sharded data parallelism on 2 GPUs (NCCL): each rank trains the reduced transformer on
its half of every batch and the gradient series are averaged by polytensors_b200.parallel; the
trajectory must match the reference's single-process trajectory (tests/golden) as closely as a
single-GPU run does.  Skipped with fewer than 2 GPUs."""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue, overlapped=False):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "..", "poly-tensors_b200"))
    sys.path.insert(0, os.path.join(here, ".."))
    sys.path.insert(0, here)
    import torch.distributed as dist
    import torch.nn.functional as F
    from polytensors_b200 import PolyTensor
    from polytensors_b200.parallel import OverlappedAllReduce, allreduce_gradients

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = torch.load(os.path.join(here, "golden", "tiny_transformer_f32_n3.pt"), weights_only=False)
        cfg, init = g["config"], g["init"]
        n, d, H, V, T, Bt = cfg["degree"], cfg["d"], cfg["heads"], cfg["vocab"], cfg["seq"], cfg["batch"]
        P = {k: torch.nn.Parameter(PolyTensor((v.to(dev),), degree=n)) for k, v in init.items()}
        Z = PolyTensor((torch.tensor(0.0, device=dev), 1.0), degree=n)
        opt = torch.optim.SGD(list(P.values()), lr=cfg["lr"], foreach=False)
        reducer = OverlappedAllReduce(list(P.values()), bucket_bytes=1 << 16) if overlapped else None
        per = Bt // world
        ids = g["ids"][:, rank * per:(rank + 1) * per].to(dev)
        losses = []
        with PolyTensor.plain_range():
            for step in range(cfg["steps"]):
                opt.zero_grad(set_to_none=True)
                with PolyTensor.retain_wrappers():
                    inp, tgt = ids[step, :, :-1], ids[step, :, 1:]
                    x = F.embedding(inp, P["emb"])
                    for l in range(cfg["layers"]):
                        h = F.rms_norm(x, (d,), P[f"n1.{l}"])
                        q, k, v = (F.linear(h, P[f"{nm}.{l}"]).view(per, T, H, d // H).transpose(1, 2)
                                   for nm in ("wq", "wk", "wv"))
                        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(per, T, d)
                        x = x + F.linear(a, P[f"wo.{l}"])
                        h = F.rms_norm(x, (d,), P[f"n2.{l}"])
                        x = x + F.linear(F.gelu(F.linear(h, P[f"w1.{l}"])), P[f"w2.{l}"])
                    logits = F.linear(F.rms_norm(x, (d,), P["nf"]), P["head"])
                    loss = F.cross_entropy(logits.reshape(-1, V), tgt.reshape(-1)) * (1 - cfg["lam"] * Z)
                    if reducer is not None:
                        reducer.arm()
                    loss.backward()
                    if reducer is not None:
                        reducer.finish()
                    else:
                        allreduce_gradients(list(P.values()))
                    opt.step()
        # numpy arrays travel by value; a tensor would travel through shared memory that this
        # process removes when it exits, possibly before the parent has received it
        final = {k: [c.detach().cpu().numpy() for c in p.coeffs] for k, p in P.items()}
        queue.put((rank, final))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("overlapped", [False, True])
def test_two_rank_training_matches_reference(golden, overlapped):
    import torch.multiprocessing as mp

    from test_training_gpu import _as_accurate

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, overlapped)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: {k: [torch.from_numpy(c) for c in v] for k, v in final.items()}
               for r, final in (queue.get(timeout=600) for _ in range(world))}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g32, g64 = golden("tiny_transformer_f32_n3"), golden("tiny_transformer_f64_n3")
    for name in g32["final"]:
        for k, (a, b) in enumerate(zip(results[0][name], results[1][name])):
            assert torch.equal(a, b), (name, k)   # replicas stay bit-identical
        _as_accurate(results[0][name], g32["final"][name], g64["final"][name], name)
