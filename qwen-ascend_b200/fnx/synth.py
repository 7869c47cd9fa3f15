"""Seeded synthetic MoE-layer tensors in the reference's artifact layouts.

No real checkpoint exists on the B200 boxes (the reference's weights live under
``/models/Qwen3.8-Flash-Next-*``), so every test and benchmark runs on synthetic
tensors with the shapes and value distributions the workload definition names:

* routed experts: int4 weights uniform in [-8, 7], stored expert-major int4pack
  ``int32 [E, K, N/8]`` (nibble ``t`` of word ``j`` = ``W[k, 8j+t]``, low nibble first,
  two's complement -- the layout ``tools/repack_w4a16.py:64-70`` writes and
  ``tools/repack_w4_em.py:16`` transposes to expert-major).  A uniformly random 32-bit
  word is exactly eight independent uniform int4 values, so the words are drawn directly.
* per-group scales: ``bf16 [E, K/gs, N]`` drawn ``|N(0, 0.02)|`` -- the cached
  ``ExpW4._scales`` layout (``fnx/engine.py:653-659``).
* router ``gate_w`` ``bf16 [E, H]`` and shared-expert gate row ``bf16 [1, H]`` drawn
  ``N(0, 1/H)`` so that logits of an ``N(0,1)`` token are ``N(0,1)``.
* shared expert: one always-on W4 expert (gate_up ``[H, 2I]``, down ``[I, H]``) with
  the same distributions.
* activations ``bf16 [T, H]`` drawn ``N(0, 1)``.

This module has no package-relative imports so that fixture generators can load it by
file path.  CPU generation uses numpy's PCG64 so the bits are identical on every host
with the same numpy; ``device='cuda'`` generation uses torch's CUDA generator (same
distributions, different bits) and is meant for benchmarks only.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class MoEShape:
    """Hidden size H, expert intermediate I, experts E, top-k, W4 group size gs."""
    H: int = 2048
    I: int = 512
    E: int = 512
    k: int = 10
    gs: int = 128

    def check(self):
        if self.H % self.gs or self.I % self.gs:
            raise ValueError(f"H={self.H} and I={self.I} must be multiples of gs={self.gs}")
        if (2 * self.I) % 8 or self.H % 8:
            raise ValueError("N dimensions must be multiples of 8 (int4pack words)")
        if not 1 <= self.k <= self.E:
            raise ValueError(f"top-k {self.k} out of range for E={self.E}")
        return self


# Shapes named by the workload definition (H=2048, I=512, group 128).
CFG1 = MoEShape(H=2048, I=512, E=64, k=8, gs=128)     # CPU-runnable parity layer
CFG2 = MoEShape(H=2048, I=512, E=512, k=10, gs=128)   # decode / prefill layer
PROD = MoEShape(H=2560, I=640, E=512, k=10, gs=64)    # the reference's production shape


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def _words(rng: np.random.Generator, shape) -> torch.Tensor:
    w = rng.integers(0, 2 ** 32, size=shape, dtype=np.uint32).view(np.int32)
    return torch.from_numpy(w)


def _scales(rng: np.random.Generator, shape, std=0.02) -> torch.Tensor:
    return _bf16(np.abs(rng.standard_normal(size=shape, dtype=np.float32)) * std)


def make_layer(shape: MoEShape, seed: int = 0, device="cpu", shared: bool = True) -> dict:
    """One MoE layer's weights.  Keys:

    ``gu_w4 [E,H,2I/8] int32``, ``gu_scales [E,H/gs,2I] bf16``,
    ``dn_w4 [E,I,H/8] int32``, ``dn_scales [E,I/gs,H] bf16``, ``gate_w [E,H] bf16``,
    and with ``shared``: ``sh_gu_w4 [H,2I/8]``, ``sh_gu_scales [H/gs,2I]``,
    ``sh_dn_w4 [I,H/8]``, ``sh_dn_scales [I/gs,H]``, ``sh_gate [1,H] bf16``.
    """
    s = shape.check()
    H, I, E, gs = s.H, s.I, s.E, s.gs
    if str(device).startswith("cuda"):
        return _make_layer_cuda(s, seed, device, shared)
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {
        "gu_w4": _words(rng, (E, H, 2 * I // 8)),
        "gu_scales": _scales(rng, (E, H // gs, 2 * I)),
        "dn_w4": _words(rng, (E, I, H // 8)),
        "dn_scales": _scales(rng, (E, I // gs, H)),
        "gate_w": _bf16(rng.standard_normal(size=(E, H), dtype=np.float32) / np.sqrt(H)),
    }
    if shared:
        out.update({
            "sh_gu_w4": _words(rng, (H, 2 * I // 8)),
            "sh_gu_scales": _scales(rng, (H // gs, 2 * I)),
            "sh_dn_w4": _words(rng, (I, H // 8)),
            "sh_dn_scales": _scales(rng, (I // gs, H)),
            "sh_gate": _bf16(rng.standard_normal(size=(1, H), dtype=np.float32) / np.sqrt(H)),
        })
    return {k: v.to(device) for k, v in out.items()} if str(device) != "cpu" else out


def _make_layer_cuda(s: MoEShape, seed: int, device, shared: bool) -> dict:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I, E, gs = s.H, s.I, s.E, s.gs

    def words(*shape):
        return torch.randint(-2 ** 31, 2 ** 31, shape, generator=g, device=device, dtype=torch.int64).to(torch.int32)

    def scales(*shape):
        return (torch.randn(shape, generator=g, device=device).abs_() * 0.02).to(torch.bfloat16)

    out = {
        "gu_w4": words(E, H, 2 * I // 8),
        "gu_scales": scales(E, H // gs, 2 * I),
        "dn_w4": words(E, I, H // 8),
        "dn_scales": scales(E, I // gs, H),
        "gate_w": (torch.randn((E, H), generator=g, device=device) / H ** 0.5).to(torch.bfloat16),
    }
    if shared:
        out.update({
            "sh_gu_w4": words(H, 2 * I // 8),
            "sh_gu_scales": scales(H // gs, 2 * I),
            "sh_dn_w4": words(I, H // 8),
            "sh_dn_scales": scales(I // gs, H),
            "sh_gate": (torch.randn((1, H), generator=g, device=device) / H ** 0.5).to(torch.bfloat16),
        })
    return out


def make_tokens(T: int, H: int, seed: int = 1, device="cpu") -> torch.Tensor:
    """Activations ``bf16 [T, H]`` drawn ``N(0, 1)``."""
    if str(device).startswith("cuda"):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        return torch.randn((T, H), generator=g, device=device).to(torch.bfloat16)
    rng = np.random.Generator(np.random.PCG64(seed))
    return _bf16(rng.standard_normal(size=(T, H), dtype=np.float32))


def zipf_bias(E: int, s: float = 1.1, seed: int = 7) -> torch.Tensor:
    """fp32 ``[E]`` log-popularity bias with Zipf(s) popularity over a seeded expert ranking.

    Added to the router logits before the softmax it skews expert load the way the
    48-layer expert-parallel workload asks for (popularity of the r-th expert ~ r^-s).
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    rank = rng.permutation(E) + 1
    p = rank.astype(np.float64) ** (-s)
    p /= p.sum()
    b = np.log(p * E)
    return torch.from_numpy(b.astype(np.float32))


def make_dense_w8(K: int, N: int, seed: int = 3, G: int = 1) -> dict:
    """W8A16 dense projection in ``DenseW8`` layout: ``w8t int8 [K,N]`` uniform in
    [-127, 127], ``sc bf16 [G,N]`` drawn ``|N(0, 0.01)|`` (per output channel for G=1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w8t = torch.from_numpy(rng.integers(-127, 128, size=(K, N), dtype=np.int8))
    sc = _bf16(np.abs(rng.standard_normal(size=(G, N), dtype=np.float32)) * 0.01)
    return {"w8t": w8t, "sc": sc}
