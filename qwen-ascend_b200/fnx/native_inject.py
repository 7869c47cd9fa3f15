"""Residual injection (``fnx/native_inject.py`` of the reference): ``hyper + y * inj`` over the
hyper-connection branches with the intermediate bf16 rounding, on ``libfnx_b200.so``
(``fnx_inject_ex``; the reference's AscendC shim ``fnx_inject`` is exported too).

``inject(hyper, gate, values)`` keeps the reference's signature and its ``None``-for-unsupported
convention: ``hyper`` bf16 ``[b, 1, HC*H]``, ``gate`` bf16 ``[b, 1, HC]``, ``values`` bf16
``[b, 1, H]`` (any batch and width here; the AscendC kernel took one token at H=2560).
"""
from __future__ import annotations

import torch

from . import _lib


def inject(hyper, gate, values):
    b = hyper.shape[0]
    if b < 1 or values.numel() % b or gate.numel() % b:
        return None
    H, HC = values.numel() // b, gate.numel() // b
    if hyper.numel() != b * HC * H or H % 8 or HC > 64:
        return None
    if any(t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != hyper.device
           for t in (hyper, gate, values)) or hyper.device.type != "cuda":
        return None
    output = torch.empty_like(hyper)
    rc = _lib.lib().fnx_inject_ex(hyper.data_ptr(), values.data_ptr(), gate.data_ptr(), output.data_ptr(), b, H, HC,
                                  _lib.stream(hyper.device))
    if rc:
        raise RuntimeError(f"residual injection launch rejected: {rc}")
    return output
