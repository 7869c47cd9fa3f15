"""Loader for ``libfnx_b200.so`` (the sm_100a kernels behind a C ABI).

The library is found through ``$FNX_B200_SO`` or next to this file, mirroring the
reference's ``FNX_*_SO`` override convention (``fnx/expert_gather.py:21``).  There is
no fallback: if the library or a CUDA device is missing, the call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

P = ctypes.c_void_p
I = ctypes.c_int
LL = ctypes.c_longlong
SZ = ctypes.c_size_t

# name -> (argtypes, restype)
SIGNATURES = {
    "fnx_b200_version": ([], ctypes.c_char_p),
    "fnx_device_errors": ([I], ctypes.c_uint),
    "fnx_weighted_reduce": ([P] * 4 + [I] * 6 + [P], I),
    "fnx_moe_merge": ([P] * 4 + [I, P], I),
    "fnx_moe_merge_ex": ([P] * 4 + [I, I, P], I),
    "fnx_moe_epilogue": ([P] * 6, I),
    "fnx_moe_epilogue_ex": ([P] * 5 + [I, I, P], I),
    "fnx_gather_pair": ([P] * 5 + [I] * 3 + [P], I),
    "fnx_gather_pair_ex": ([P] * 5 + [I] * 5 + [P], I),
    "fnx_moe_combine": ([P] * 5 + [LL, P, I, I, I, P], I),
    "fnx_moe_combine_inject": ([P] * 5 + [LL, P, P, P, P, I, I, I, I, P], I),
    "fnx_inject": ([P] * 4 + [I, P], I),
    "fnx_hc_rms_norm": ([P] * 3 + [I, I, I, ctypes.c_float, P], I),
    "fnx_hc_activation": ([P] * 3 + [I, I, P], I),
    "fnx_hc_activation_ex": ([P] * 3 + [I] * 4 + [P], I),
    "fnx_hc_sigmoid_reduce": ([P] * 3 + [I, P], I),
    "fnx_hc_sigmoid_reduce_ex": ([P] * 3 + [I] * 3 + [P], I),
    "fnx_inject_ex": ([P] * 4 + [I, I, I, P], I),
    "fnx_router_topk": ([P, LL, P, P, P, P, I, I, I, P], I),
    "fnx_moe_permute_workspace": ([I, I], SZ),
    "fnx_moe_permute": ([P] * 5 + [I, I, P, SZ, P], I),
    "fnx_ep_layout_workspace": ([I, I], SZ),
    "fnx_ep_dispatch_layout": ([P, I, I, I, P, P, P, P, SZ, P], I),
    "fnx_ep_gather_rows": ([P, LL, LL, P, I, P, I, P, LL, P, LL, I, P], I),
    "fnx_ep_p2p_region_bytes": ([I, I, I, I], SZ),
    "fnx_ep_p2p_alloc": ([SZ, ctypes.POINTER(P)], I),
    "fnx_ep_p2p_free": ([P], I),
    "fnx_ep_p2p_export": ([P, P], I),
    "fnx_ep_p2p_import": ([P, ctypes.POINTER(P)], I),
    "fnx_ep_p2p_close": ([P], I),
    "fnx_ep_p2p_desc_bytes": ([], SZ),
    "fnx_ep_p2p_desc": ([P, I, I, ctypes.POINTER(P), I, I, I, I], I),
    "fnx_ep_p2p_local": ([P, I], P),
    "fnx_ep_p2p_capacity": ([P, I], LL),
    "fnx_ep_p2p_received": ([P], LL),
    "fnx_ep_p2p_dedup": ([P, P, P, I, P, P, P], I),
    "fnx_ep_p2p_counts": ([P, P, P, P], I),
    "fnx_ep_p2p_push": ([P, P, I, P, P, P, P], I),
    "fnx_ep_p2p_push_ex": ([P, P, I, P, P, P, I, I, P], I),
    "fnx_ep_p2p_wait": ([P, I, P], I),
    "fnx_ep_p2p_signal": ([P, I, P], I),
    "fnx_ep_p2p_recv_workspace": ([P], SZ),
    "fnx_ep_p2p_recv_layout": ([P, I, P, P, P, P, P, P, SZ, P], I),
    "fnx_ep_p2p_recv_layout_routed": ([P, P, P, P, P, P, SZ, P], I),
    "fnx_moe_grouped_w4_rows": ([P, LL, LL, P, I, P, P, P, I, I, I, I, P], I),
    "fnx_moe_grouped_w4": ([P, LL, LL, P, I, P, P, P, LL] + [I] * 5 + [P], I),
    "fnx_moe_grouped_w4_lim": ([P, LL, LL, P, I, P, P, P, LL] + [I] * 6 + [P], I),
    "fnx_moe_grouped_w4_sel": ([P, LL, LL, P, I, P, I, P, P, P, LL] + [I] * 5 + [P], I),
    "fnx_weighted_sum_f32": ([P, P, P, I, I, P], I),
    "fnx_repack_v2o": ([P, I, I, I, I, P, P], I),
    "fnx_w4_tiles_bytes": ([I] * 3, SZ),
    "fnx_repack_w4_tiles": ([P] * 3 + [I] * 5 + [P], I),
    "fnx_w8a16_gemm": ([P] * 4 + [I] * 4 + [P], I),
    "fnx_w8a16_gemm_workspace": ([I] * 4, SZ),
    "fnx_w8a16_gemm_ws": ([P] * 4 + [I] * 4 + [P, SZ, P], I),
    "fnx_bf16_gemm_nt": ([P, LL, P, P, LL, I, I, I, P], I),
    "fnx_moe_decode_workspace": ([I] * 5, SZ),
    "fnx_moe_decode_w4": ([P] * 10 + [I] * 5 + [P, SZ, P], I),
    "fnx_moe_decode_w4_ex": ([P] * 10 + [I] * 5 + [P, SZ, I, P], I),
    "fnx_hc_mix_router": ([P] * 5 + [SZ] + [I] * 6 + [P], I),
    "fnx_moe_decode_w4_noalloc": ([P] * 10 + [I] * 5 + [P], I),
    "fnx_w4gemv_launch": ([P] * 7 + [I] * 5 + [P], I),
    "fnx_w4gemv_launch_layers": ([ctypes.POINTER(P)] * 4 + [I] * 6 + [P, P], I),
}

_lib = None


def library_path() -> Path:
    return Path(os.environ.get("FNX_B200_SO", str(Path(__file__).with_name("libfnx_b200.so"))))


def lib():
    """The loaded library (raises ``OSError`` when it cannot be found or loaded)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not path.exists():
            raise OSError(f"fnx: {path} not found -- build it with `python qwen-ascend_b200/build.py` "
                          "(there is no CPU or torch fallback)")
        h = ctypes.CDLL(str(path))
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = h
    return _lib


def stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def check(rc: int, what: str):
    if rc:
        raise RuntimeError(f"{what} launch rejected: {rc}")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError(f"fnx: expected CUDA tensors, got {t.device}")


def device_errors(clear: bool = True) -> int:
    """Bits recorded by kernels since the last clear (1 timeout, 2 bad expert id, 4 overflow,
    8 a logits-ready decode without fresh router logits)."""
    return int(lib().fnx_device_errors(1 if clear else 0))
