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


class OverlappedAllReduce:
    """Average gradient series across ranks while backward is still running.

    The parameters are split, in reverse order (the order backward finishes their gradients), into
    fixed buckets of at most ``bucket_bytes`` of gradient planes per dtype and device.  After
    ``arm()``, each parameter's post-accumulate-grad hook counts it in; when a bucket is complete
    its planes are packed into one flat buffer and an asynchronous all-reduce is launched (NCCL
    runs it on its own stream while backward computes the remaining gradients).  Buckets are
    launched strictly in their fixed order, so every rank issues the same collectives in the same
    order.  ``finish()`` launches what is left (parameters without a gradient are skipped on every
    rank alike), waits for the collectives on the current stream and unpacks the averages.

    With gradient accumulation, call ``arm()`` before the LAST micro-batch's backward only.  Every
    rank must construct it with the same parameters in the same order."""

    def __init__(self, params, group=None, bucket_bytes=128 << 20):
        self.group = group
        self.bucket_bytes = bucket_bytes
        self.world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.params = [p for p in params if p.requires_grad]
        self._build(self.params)
        self.armed = False
        self.hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in self.params] if self.world > 1 else []
        self._reset()

    def _build(self, params):
        self.buckets = []
        current, size, key = [], 0, None
        bucket_bytes = self.bucket_bytes
        for p in reversed(params):
            planes = len(p.coeffs) if hasattr(p, "coeffs") else 1
            nbytes = planes * p.numel() * p.element_size()
            k = (p.dtype, p.device)
            if current and (k != key or size + nbytes > bucket_bytes):
                self.buckets.append(current)
                current, size = [], 0
            current.append(p)
            size += nbytes
            key = k
        if current:
            self.buckets.append(current)
        self.bucket_of = {id(p): i for i, b in enumerate(self.buckets) for p in b}

    def _reset(self):
        self.pending = [0] * len(self.buckets)
        self.next_launch = 0
        self.inflight = []
        self.seen = set()

    def arm(self):
        """Launch buckets from the gradient hooks of the backward that follows."""
        self._reset()
        self.armed = self.world > 1

    def _ready(self, p):
        if not self.armed or id(p) not in self.bucket_of:
            return
        self.seen.add(id(p))
        b = self.bucket_of[id(p)]
        self.pending[b] += 1
        while self.next_launch < len(self.buckets) and \
                self.pending[self.next_launch] == len(self.buckets[self.next_launch]):
            self._launch(self.next_launch)
            self.next_launch += 1

    def _launch(self, b):
        planes = []
        for p in self.buckets[b]:
            g = p.grad
            if g is not None:
                planes.extend(g.coeffs if hasattr(g, "coeffs") else (g,))
        if not planes:
            return
        flat = torch.cat([t.reshape(-1) for t in planes])
        use_avg = dist.get_backend(self.group) == "nccl"
        work = dist.all_reduce(flat, op=dist.ReduceOp.AVG if use_avg else dist.ReduceOp.SUM, group=self.group,
                               async_op=True)
        self.inflight.append((work, flat, planes, use_avg))

    def finish(self):
        """Launch the remaining buckets, wait for every collective and write the averages back."""
        if self.world == 1:
            return
        if self.armed:
            while self.next_launch < len(self.buckets):
                self._launch(self.next_launch)
                self.next_launch += 1
            # parameters the graph never reached would hold their bucket (and every later one)
            # back until finish() in every step: leave them out from now on (all ranks run the same
            # graph, so they all drop the same parameters)
            unused = [p for p in self.params if id(p) in self.bucket_of and id(p) not in self.seen]
            if unused:
                self._build([p for p in self.params if id(p) in self.seen])
        self.armed = False
        for work, flat, planes, use_avg in self.inflight:
            work.wait()
            if not use_avg:
                flat.div_(self.world)
            torch._foreach_copy_(planes, [v.view_as(t) for v, t in zip(flat.split([t.numel() for t in planes]),
                                                                      planes)])
        self.inflight = []

    def remove(self):
        for h in self.hooks:
            h.remove()
        self.hooks = []
