"""Post-ops of the reference's ``fnx/post_ops.py`` on ``libfnx_b200.so``:

* ``moe_merge`` = bf16(e + bf16(shared * bf16(sigmoid(gate)))) (``fnx/post_ops.py:36-39`` ->
  ``fnx_moe_merge``), for any ``[batch, W]`` with one gate value per row;
* ``activate`` and ``mix_reduce``, the hyper-connection steps of ``gated_residual`` that
  produce the MoE layer's input (``fnx/post_ops.py:22-30``), for any batch, width and branch
  count.  (``mul_cast`` serves the attention-side norm and is not part of this build.)"""
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


def _bf16_cuda(*tensors):
    d = tensors[0].device
    return d.type == "cuda" and all(t.dtype == torch.bfloat16 and t.is_contiguous() and t.device == d for t in tensors)


def activate(di, hc=4, mode=0):
    """The hyper-connection activation (reference ``fnx/post_ops.py:22-26`` ->
    ``fnx_hc_activation``): ``di`` bf16 ``[b, 1, n_mix + hc]`` -> ``(mixed [b, 1, n_mix],
    gate [b, 1, hc])`` with ``mixed = silu(dp / hc)``, ``gate = 2 * sigmoid(ip / hc)``."""
    if di.ndim != 3 or di.shape[1] != 1 or di.shape[2] <= hc or not _bf16_cuda(di):
        return None
    b, n_mix = di.shape[0], di.shape[2] - hc
    mixed = torch.empty(b, 1, n_mix, device=di.device, dtype=di.dtype)
    gate = torch.empty(b, 1, hc, device=di.device, dtype=di.dtype)
    rc = _lib.lib().fnx_hc_activation_ex(di.data_ptr(), mixed.data_ptr(), gate.data_ptr(), b, n_mix, hc, mode,
                                         _lib.stream(di.device))
    _lib.check(rc, "hyper-connection activation")
    return mixed, gate


def mix_reduce(values, logits, hc=4):
    """The branch mix (reference ``fnx/post_ops.py:27-30`` -> ``fnx_hc_sigmoid_reduce``):
    ``values`` (hn), ``logits`` bf16 ``[b, 1, hc*H]`` -> ``[b, 1, H]`` =
    mean over branches of ``sigmoid(logits) * values``."""
    if (values.ndim != 3 or logits.shape != values.shape or values.shape[2] % hc
            or not _bf16_cuda(values, logits)):
        return None
    b, H = values.shape[0], values.shape[2] // hc
    out = torch.empty(b, 1, H, device=values.device, dtype=values.dtype)
    rc = _lib.lib().fnx_hc_sigmoid_reduce_ex(values.data_ptr(), logits.data_ptr(), out.data_ptr(), b, H, hc,
                                             _lib.stream(values.device))
    _lib.check(rc, "hyper-connection mix")
    return out
