"""BF16-rounded products accumulated in fp32 in slot order (reference
``fnx/weighted_reduce.py:10-42`` -> ``fnx_weighted_reduce``).

``mean=True`` is mode 0 (mean of 4 groups with elementwise weights); otherwise mode 1,
or mode 2 when ``inverse`` gives the source row of every (token, slot).  The reference
requires ``width == 2560`` and top-10; this build accepts any width and 1..64 groups."""
import torch

from . import _lib


def reduce(values, weights, *, inverse=None, mean=False, order=0):
    if mean:
        if values.shape != weights.shape or values.ndim != 3 or values.shape[1] != 4:
            return None
        batch, groups, width = values.shape
        if not values.is_contiguous() or not weights.is_contiguous():
            return None
        x = values.view(-1, width)
        w = weights
        mode = 0
    else:
        if weights.ndim != 2 or not 1 <= weights.shape[1] <= 64:
            return None
        batch, groups = weights.shape
        width = values.shape[-1]
        x = values.view(-1, width)
        w = weights.float().contiguous()
        mode = 2 if inverse is not None else 1
    if values.dtype != torch.bfloat16 or weights.dtype != torch.bfloat16 or x.stride(1) != 1:
        return None
    if x.device != w.device or x.device.type != "cuda":
        return None
    if inverse is not None and (inverse.dtype != torch.int64 or not inverse.is_contiguous()
                                or inverse.numel() != batch * groups or inverse.device != x.device):
        return None
    if inverse is None and not mean and x.shape[0] != batch * groups:
        return None
    output = torch.empty((batch, width), dtype=torch.bfloat16, device=x.device)
    rc = _lib.lib().fnx_weighted_reduce(x.data_ptr(), w.data_ptr(), inverse.data_ptr() if inverse is not None else None,
                                        output.data_ptr(), batch, groups, width, x.stride(0), mode, order,
                                        _lib.stream(x.device))
    _lib.check(rc, "weighted reduction")
    return output
