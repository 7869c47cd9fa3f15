"""Gather the selected experts' expert-major W4 words and bf16 scales into the K-major
concatenated layout (reference ``fnx/expert_gather.py:9-31`` -> ``fnx_gather_pair``).

The reference accepts only its two production shapes; this build accepts any
``N % 8 == 0`` and any number of ids, validates ids against ``E`` on the device and
returns ``None`` for inputs it does not handle (the caller falls back)."""
import torch

from . import _lib


def gather(projection, ids):
    if (not getattr(projection, "expert_major", False) or getattr(projection, "_scales", None) is None
            or ids.ndim != 1 or ids.dtype != torch.int64 or not ids.is_contiguous()):
        return None
    w, s = projection.w4, projection._scales
    if (w.dtype != torch.int32 or s.dtype != torch.bfloat16 or not w.is_contiguous() or not s.is_contiguous()
            or w.device != s.device or w.device != ids.device or w.device.type != "cuda" or projection.N % 8):
        return None
    k = ids.numel()
    ow = torch.empty((projection.K, k * projection.N // 8), dtype=torch.int32, device=w.device)
    oscale = torch.empty((projection.G, k * projection.N), dtype=torch.bfloat16, device=w.device)
    rc = _lib.lib().fnx_gather_pair_ex(w.data_ptr(), s.data_ptr(), ids.data_ptr(), ow.data_ptr(), oscale.data_ptr(),
                                       projection.E, projection.K, projection.G, projection.N, k,
                                       _lib.stream(w.device))
    _lib.check(rc, "expert gather")
    return ow, oscale
