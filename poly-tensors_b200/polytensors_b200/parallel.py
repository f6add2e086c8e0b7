"""Batch-sharded data parallelism for PolyTensor training.

The reference has no distributed code (its notes list distributed execution as not
established); the transformer benchmark shards the global batch across GPUs and needs one
exchange step per optimizer step: the average of every parameter's gradient series.
DistributedDataParallel does not understand the wrapper subclass, so the coefficient planes
of all gradients are packed into flat buckets and all-reduced with ``torch.distributed``
(NCCL over NVLink on GPUs, gloo on CPU for tests).
"""

import torch
import torch.distributed as dist


def _grad_planes(params):
    planes = []
    for p in params:
        g = p.grad
        if g is None:
            continue
        planes.extend(g.coeffs if hasattr(g, "coeffs") else (g,))
    return planes


def allreduce_gradients(params, group=None, bucket_bytes=512 << 20):
    """Average the gradient series of ``params`` over the ranks of ``group``, in place.

    Gradient planes are packed (in parameter order) into flat buckets of at most
    ``bucket_bytes`` per dtype, each reduced by one collective and unpacked again, so the
    collective count per step is small and independent of the series degree.  Every rank
    must call this with the same parameters in the same order."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    planes = _grad_planes(params)
    by_dtype = {}
    for t in planes:
        by_dtype.setdefault((t.dtype, t.device), []).append(t)
    use_avg = dist.get_backend(group) == "nccl"
    for (dtype, device), items in sorted(by_dtype.items(), key=lambda kv: str(kv[0])):
        bucket, size = [], 0
        for t in items + [None]:
            if t is not None and (not bucket or size + t.numel() * t.element_size() <= bucket_bytes):
                bucket.append(t)
                size += t.numel() * t.element_size()
                continue
            if bucket:
                flat = torch.cat([b.reshape(-1) for b in bucket])
                if use_avg:
                    dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=group)
                else:
                    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
                    flat.div_(world)
                offset = 0
                for b in bucket:
                    n = b.numel()
                    b.copy_(flat[offset:offset + n].view_as(b))
                    offset += n
            bucket, size = ([t], t.numel() * t.element_size()) if t is not None else ([], 0)
