"""``moe_merge`` = bf16(e + bf16(shared * bf16(sigmoid(gate)))) (reference
``fnx/post_ops.py:36-39`` -> ``fnx_moe_merge``), for any ``[batch, W]`` with one gate
value per row.  The reference's hyper-connection helpers (``activate``, ``mix_reduce``,
``mul_cast``) belong to the attention side and are not part of this build."""
import torch

from . import _lib


def moe_merge(experts, shared, gate):
    if (experts.ndim != 2 or shared.shape != experts.shape or gate.numel() != experts.shape[0]
            or experts.device.type != "cuda"
            or any(t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != experts.device
                   for t in (experts, shared, gate))):
        return None
    out = torch.empty_like(experts)
    rc = _lib.lib().fnx_moe_merge_ex(experts.data_ptr(), shared.data_ptr(), gate.data_ptr(), out.data_ptr(),
                                     experts.shape[0], experts.shape[1], _lib.stream(experts.device))
    _lib.check(rc, "decode postprocessing")
    return out
