"""Diagonal extraction of the Cartesian down output + slot-order weighted reduce +
sigmoid-gated shared merge (reference ``fnx/moe_epilogue.py:6-21`` ->
``fnx_moe_epilogue``).  Accepts any ``[k, k*W]`` instead of only ``(10, 25600)``."""
import torch

from . import _lib


def merge(cartesian, weights, shared, gate):
    tensors = (cartesian, weights, shared, gate)
    if cartesian.ndim != 2 or weights.ndim != 2 or weights.shape[0] != 1:
        return None
    k = weights.shape[1]
    W = shared.shape[-1]
    if (cartesian.shape != (k, k * W) or shared.shape != (1, W) or gate.numel() != 1
            or cartesian.device.type != "cuda"
            or any(t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != cartesian.device for t in tensors)):
        return None
    out = torch.empty_like(shared)
    rc = _lib.lib().fnx_moe_epilogue_ex(*(t.data_ptr() for t in (*tensors, out)), k, W, _lib.stream(cartesian.device))
    _lib.check(rc, "MoE epilogue")
    return out
