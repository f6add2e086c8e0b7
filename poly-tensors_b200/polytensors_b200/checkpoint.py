"""Checkpoints of PolyTensor state as stacked coefficient planes.

A PolyTensor of degree n is n+1 same-shape planes (a real constant plane, possibly complex
directions).  ``save`` writes any nesting of dicts, lists and tuples whose leaves are PolyTensors,
ordinary tensors or plain Python values with ``torch.save``; each PolyTensor becomes a record

    {"degree": n, "shape": (...), "requires_grad": bool,
     "planes": (n+1, *shape) tensor}                      all planes one dtype, or
     "base": (*shape) real tensor, "directions": (n, *shape) complex tensor
                                                          real constant with complex directions

so a plane stack loads as one contiguous tensor (``load(..., stacked=True)`` returns them as is, e.g.
for a collective or a memory map) and ``load`` rebuilds the PolyTensors on a chosen device.  The
reference keeps PolyTensor state only in memory (its PolyTensor is not picklable as a subclass); the
format is this library's addition (``FORMAT`` names its version).
"""

import torch

FORMAT = "polytensors_b200.planes/1"


def _poly_cls():
    from ._tensor import PolyTensor

    return PolyTensor


def _encode(obj):
    P = _poly_cls()
    if isinstance(obj, torch.nn.Parameter) and isinstance(obj.data, P):
        obj = obj.data
    if isinstance(obj, P):
        planes = [c.detach().cpu() for c in obj.coeffs]
        rec = {"__polytensor__": True, "degree": len(planes) - 1, "shape": tuple(planes[0].shape),
               "requires_grad": bool(obj.requires_grad)}
        if all(p.dtype == planes[0].dtype for p in planes):
            rec["planes"] = torch.stack(planes)
        else:
            rec["base"] = planes[0]
            rec["directions"] = torch.stack(planes[1:])
        return rec
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {k: _encode(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        out = [_encode(v) for v in obj]
        return out if isinstance(obj, list) else tuple(out)
    return obj


def _decode(obj, device, stacked):
    P = _poly_cls()
    if isinstance(obj, dict) and obj.get("__polytensor__"):
        if stacked:
            return obj
        if "planes" in obj:
            planes = list(obj["planes"].to(device).unbind(0))
        else:
            planes = [obj["base"].to(device)] + list(obj["directions"].to(device).unbind(0))
        planes = [p.clone() for p in planes]  # independent storage per plane, as constructed ones
        return P(tuple(planes), degree=obj["degree"], requires_grad=obj["requires_grad"])
    if isinstance(obj, torch.Tensor):
        return obj.to(device) if device is not None else obj
    if isinstance(obj, dict):
        return {k: _decode(v, device, stacked) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        out = [_decode(v, device, stacked) for v in obj]
        return out if isinstance(obj, list) else tuple(out)
    return obj


def save(obj, path):
    """Write ``obj`` (PolyTensors, tensors, nested containers) to ``path``."""
    torch.save({"format": FORMAT, "items": _encode(obj)}, path)


def load(path, device=None, stacked=False):
    """Read a checkpoint written by ``save``; PolyTensors are rebuilt on ``device`` (the stored CPU
    planes if None).  With ``stacked=True`` PolyTensor records are returned as stored."""
    data = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(data, dict) or data.get("format") != FORMAT:
        raise ValueError(f"{path}: not a {FORMAT} checkpoint")
    return _decode(data["items"], device, stacked)
