"""The legacy W4A16 GEMV op (reference ``fnx/w4gemv_op.py:37-265``, used with
``FNX_MOE_KERNEL=1``) on the B200 library.

Same class, method names and argument meaning: ``p4`` ``[E, N, K/2]`` packed bytes
(``lay=1`` two nibbles per byte along K, ``lay=2`` the v2 layout), ``s4t`` fp16
``[E, K/32, N]``, fp32 ``x`` ``[nE, K]`` and fp32 ``y`` ``[nE, N]``; weights and scales are
indexed by expert id, ``x``/``y`` by slot.  ``so_path`` defaults to this package's
``libfnx_b200.so``; ``nblk`` and ``dbg_elems`` are accepted and unused (the kernel sizes
its own grid and writes no debug buffer)."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import _lib

GS = 32


class W4GemvOp:
    def __init__(self, so_path=None, nblk=20, dbg_elems=65536, device=None):
        if so_path is not None and not os.path.exists(so_path):
            raise FileNotFoundError(so_path)
        if so_path is not None:
            os.environ.setdefault("FNX_B200_SO", str(so_path))
        self.lib = _lib.lib()
        self.nblk = nblk
        self._dev = device if device is not None else "cuda:0"
        self._dbg_elems = dbg_elems
        self._xe = self._xo = None
        self._ids = None

    def prepare_layer(self, s4_np):
        """``s4`` fp16 ``[E, N, K/gs]`` (numpy) -> device ``[E, K/gs, N]``, once at load time."""
        s4t = np.ascontiguousarray(np.transpose(s4_np, (0, 2, 1)), dtype=np.float16)
        return torch.from_numpy(s4t).to(self._dev)

    @staticmethod
    def _split_x(x_np):
        xe = np.ascontiguousarray(x_np[:, 0::2], dtype=np.float32)
        xo = np.ascontiguousarray(x_np[:, 1::2], dtype=np.float32)
        return xe, xo

    def run(self, p4_dev, s4t_dev, x_dev, n_exp, N, K, expert_ids=None, lay=1, out=None):
        """``p4_dev`` int8/uint8 ``[E, N, K/2]``, ``s4t_dev`` fp16 ``[E, K/32, N]``, ``x_dev`` fp32
        ``[nE, K]`` (device tensor or numpy) -> fp32 ``[nE, N]``."""
        dev = x_dev.device if isinstance(x_dev, torch.Tensor) else torch.device(self._dev)
        if isinstance(expert_ids, torch.Tensor) and expert_ids.device.type == "cuda":
            dev = expert_ids.device
        if isinstance(x_dev, np.ndarray):
            xt = torch.from_numpy(np.ascontiguousarray(x_dev, dtype=np.float32)).to(dev)
        else:
            xt = x_dev if (x_dev.dtype == torch.float32 and x_dev.is_contiguous()) else x_dev.float().contiguous()
        if lay == 2:
            self._xe = self._xo = xt.contiguous()
        else:
            self._xe = xt[:, 0::2].contiguous()
            self._xo = xt[:, 1::2].contiguous()
        if expert_ids is None:
            if self._ids is None or self._ids.numel() != n_exp or self._ids.device != dev:
                self._ids = torch.arange(n_exp, dtype=torch.int32, device=dev)
            ids_dev = self._ids
        elif isinstance(expert_ids, torch.Tensor):
            ids_dev = expert_ids.to(device=dev, dtype=torch.int32).contiguous()
        else:
            ids_dev = torch.from_numpy(np.ascontiguousarray(expert_ids, dtype=np.int32)).to(dev)
        y = out if out is not None else torch.empty((n_exp, N), dtype=torch.float32, device=dev)
        for name, t in (("p4", p4_dev), ("s4t", s4t_dev), ("ids", ids_dev)):
            if isinstance(t, torch.Tensor) and t.device != y.device:
                raise RuntimeError(f"w4gemv device mismatch: {name} on {t.device}, x/y on {y.device}")
        rc = self.lib.fnx_w4gemv_launch(p4_dev.data_ptr(), s4t_dev.data_ptr(), self._xe.data_ptr(),
                                        self._xo.data_ptr(), y.data_ptr(), None, ids_dev.data_ptr(), int(N), int(K),
                                        int(n_exp), int(self.nblk), int(lay), _lib.stream(y.device))
        if rc != 0:
            raise RuntimeError(f"fnx_w4gemv_launch rc={rc}")
        return y

    def run_layers(self, p4_list, s4t_list, x_list, y_list, N, K, n_exp, lay=2):
        """One launch for ``len(p4_list)`` layers (natural ``x``; ids = slot order)."""
        nL = len(p4_list)
        if nL == 0:
            return y_list

        def arr(ts):
            return (ctypes.c_void_p * nL)(*[ctypes.c_void_p(t.data_ptr()) for t in ts])
        dev = p4_list[0].device
        rc = self.lib.fnx_w4gemv_launch_layers(arr(p4_list), arr(s4t_list), arr(x_list), arr(y_list), nL, int(N),
                                               int(K), int(n_exp), int(self.nblk), int(lay), None, _lib.stream(dev))
        if rc != 0:
            raise RuntimeError(f"fnx_w4gemv_launch_layers rc={rc}")
        return y_list

    def make_x_dev(self, x_np, lay=2):
        if lay == 2:
            return torch.from_numpy(np.ascontiguousarray(x_np, dtype=np.float32)).to(self._dev)
        xe, _ = self._split_x(np.asarray(x_np, dtype=np.float32))
        return torch.from_numpy(xe).to(self._dev)

    def moe_forward(self, p4_dev, s4t_dev, x_np, topk_ids, topk_w, N, K):
        """One token through ``nE`` experts, then the weighted sum -> fp32 ``[N]``."""
        nE = len(topk_ids)
        x_b = np.repeat(np.asarray(x_np, dtype=np.float32).reshape(1, K), nE, axis=0)
        y = self.run(p4_dev, s4t_dev, x_b, nE, N, K, expert_ids=np.asarray(topk_ids, dtype=np.int32))
        return self.weighted_sum(y, topk_w)

    @staticmethod
    def to_v2_layout(p4_old, N, K):
        """Old layout (byte j: lo=W[2j], hi=W[2j+1]) -> v2 (byte 64s+j: lo=W[128s+j],
        hi=W[128s+64+j]); ``[nE, N, K/2]`` or ``[N, K/2]``; an int8 container ``[.., K]``
        (one value per byte) is accepted too."""
        squeeze = p4_old.ndim == 2
        a = p4_old[None] if squeeze else p4_old
        nE, Nx, X = a.shape
        if X == K:
            w = a.reshape(nE * Nx, K).astype(np.int8)
        else:
            assert X == K // 2, (a.shape, N, K)
            b = a.reshape(nE * Nx, K // 2).astype(np.int8).view(np.uint8)
            w = np.empty((nE * Nx, K), dtype=np.int8)
            w[:, 0::2] = ((b & 0x0F).astype(np.int8) ^ 8) - 8
            w[:, 1::2] = (((b >> 4) & 0x0F).astype(np.int8) ^ 8) - 8
        v = (w.reshape(nE * Nx, K // 128, 2, 64).astype(np.int16) & 0x0F)
        out = (v[:, :, 0, :] | (v[:, :, 1, :] << 4)).astype(np.uint8).reshape(nE, N, K // 2)
        return out[0] if squeeze else out

    @staticmethod
    def weighted_sum(y_dev, w):
        """sum_e w_e * y_e (``fnx/w4gemv_op.py:252-264``): one kernel, fp32 products rounded
        and summed in expert order.  y ``[nE, N]`` (cast to fp32 if needed), w ``[nE]``."""
        _lib.require_cuda(y_dev)
        y = (y_dev if y_dev.dtype == torch.float32 else y_dev.float()).contiguous()
        if isinstance(w, torch.Tensor):
            wt = w.to(device=y.device, dtype=torch.float32).contiguous().view(-1)
        else:
            wt = torch.from_numpy(np.asarray(w, dtype=np.float32).reshape(-1)).to(y.device)
        nE, N = y.shape
        if wt.numel() != nE:
            raise ValueError(f"weighted_sum: {wt.numel()} weights for {nE} rows")
        if nE == 0 or N == 0:
            return torch.zeros(N, dtype=torch.float32, device=y.device)
        out = torch.empty(N, dtype=torch.float32, device=y.device)
        rc = _lib.lib().fnx_weighted_sum_f32(y.data_ptr(), wt.data_ptr(), out.data_ptr(), nE, N,
                                             _lib.stream(y.device))
        _lib.check(rc, "weighted sum")
        return out
