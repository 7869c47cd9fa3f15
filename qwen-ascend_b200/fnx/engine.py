"""Quantised weight containers and the MoE layer, backed by ``libfnx_b200.so``.

Mirrors the reference's MoE/quant section of ``fnx/engine.py``:

* ``ExpW4``  (reference ``fnx/engine.py:619-753``): int4pack experts + bf16 group scales;
  ``apply`` / ``apply_diag`` / ``apply_grouped`` run the tcgen05 grouped GEMM.
* ``ExpQ``   (reference ``fnx/engine.py:411-616``): experts from int4 values or straight from
  the LQP ``v2o`` artifact; ``matmul`` runs the same grouped GEMM per selected expert.
* ``DenseW8`` (reference ``fnx/engine.py:297-384``): int8 ``[K, N]`` + bf16 ``[G, N]``
  scales, N-concatenation by ``merge``; calls run the W8A16 kernels.
* ``MoELayer`` (reference ``FnLayer._moe``, ``fnx/engine.py:1782-1930``): shared expert,
  router top-k, expert-major permutation, grouped gate/up + SwiGLU, grouped down,
  slot-order combine and sigmoid-gated shared merge.  ``T <= 16`` tokens take the fused
  decode kernels, larger batches the prefill pipeline.

All tensors live on a CUDA device; nothing here computes on the CPU.
"""
from __future__ import annotations

import os

import torch

from . import _lib

BF16 = torch.bfloat16
EPI_PLAIN, EPI_SWIGLU_F32, EPI_SWIGLU_BF16, EPI_SWIGLU_MIXED = 0, 1, 2, 3
DECODE_MAX_TOKENS = 16
DECODE_MAX_EXPERTS = 512         # the fused decode kernel's router width; wider ones take the grouped path


TILE_BLOCK_WORDS = 1088          # 1024 words of int4 + 128 bf16 scales per (tile, k-block)
# prefill: the shared expert on a second stream while the routing runs (FNX_PREFILL_OVERLAP=0: one
# stream), leaving SHARED_RESERVE_SMS SMs to the routing kernels
OVERLAP_SHARED = os.environ.get("FNX_PREFILL_OVERLAP", "1") != "0"
SHARED_RESERVE_SMS = int(os.environ.get("FNX_PREFILL_RESERVE_SMS", "64"))


def repack_w4(w4, scales, swiglu):
    """Expert-major int4pack ``[E, K, N/8]`` + bf16 scales ``[E, K/gs, N]`` -> the tile blocks
    the kernels stream (``fnx_repack_w4_tiles``): int32 ``[E, N/128, K/64, 1088]``, each block
    the 8x128 words of one (feature tile, k-block) followed by the 128 rows' scales.
    ``swiglu`` orders the rows of a tile as gate/up pairs (for the fused SwiGLU epilogue);
    otherwise rows are consecutive features.  Runs once at load; the artifact layout itself
    is read unchanged."""
    _lib.require_cuda(w4, scales)
    E, K, n8 = w4.shape
    N, G = n8 * 8, scales.shape[1]
    t = torch.empty(E, N // 128, K // 64, TILE_BLOCK_WORDS, dtype=torch.int32, device=w4.device)
    rc = _lib.lib().fnx_repack_w4_tiles(w4.contiguous().data_ptr(), scales.contiguous().data_ptr(), t.data_ptr(),
                                        E, K, N, K // G, 1 if swiglu else 0, _lib.stream(w4.device))
    _lib.check(rc, "W4 tile repack")
    return t


def repack_v2o(v2o, K, expert_major=False):
    """The LQP artifact's experts ``v2o`` uint8 ``[E, N, K/2]`` (offset-binary, byte ``64s+j`` =
    ``W[128s+j] + 8`` low | ``W[128s+64+j] + 8`` high) as int4pack words: ``int32 [K, E, N/8]``
    (the layout ``tools/repack_w4a16.py:58-70`` writes, there with CANN's
    ``npu_convert_weight_to_int4pack``) or ``[E, K, N/8]`` with ``expert_major``
    (``tools/repack_w4_em.py``).  Byte-exact, on the GPU (``fnx_repack_v2o``)."""
    _lib.require_cuda(v2o)
    E, N = v2o.shape[0], v2o.shape[1]
    shape = (E, K, N // 8) if expert_major else (K, E, N // 8)
    out = torch.empty(shape, dtype=torch.int32, device=v2o.device)
    rc = _lib.lib().fnx_repack_v2o(v2o.contiguous().data_ptr(), E, N, K, 1 if expert_major else 0, out.data_ptr(),
                                   _lib.stream(v2o.device))
    _lib.check(rc, "v2o repack")
    return out


def _grouped_w4(act, tiles, ends, out, *, E, M, K, Nw, epilogue, row_index=None, index_div=1):
    """Grouped GEMM over the tile blocks of ``repack_w4`` (the SwiGLU epilogues need the
    SwiGLU row order)."""
    rc = _lib.lib().fnx_moe_grouped_w4(act.data_ptr(), act.stride(0), act.shape[0], _lib.ptr(row_index), index_div,
                                       tiles.data_ptr(), _lib.ptr(ends), out.data_ptr(), out.stride(0), E, M, K, Nw,
                                       epilogue, _lib.stream(act.device))
    _lib.check(rc, "grouped W4A16 GEMM")
    return out


def mm_nt(x, w):
    """``x [M, K] @ w[N, K]^T`` -> bf16 ``[M, N]`` on this library's tcgen05 bf16 GEMM
    (``fnx_bf16_gemm_nt``: fp32 accumulation, one rounding).  K is zero-padded to a multiple of
    64 when it is not one (exact: the padding adds zero products)."""
    _lib.require_cuda(x, w)
    x = (x if x.dtype == BF16 else x.to(BF16)).contiguous()
    w = (w if w.dtype == BF16 else w.to(BF16)).contiguous()
    M, K = x.shape
    N = w.shape[0]
    Kp = (K + 63) // 64 * 64
    if Kp != K:
        x = torch.nn.functional.pad(x, (0, Kp - K))
        w = torch.nn.functional.pad(w, (0, Kp - K))
    out = torch.empty(M, N, dtype=BF16, device=x.device)
    if M:
        rc = _lib.lib().fnx_bf16_gemm_nt(x.data_ptr(), x.stride(0), w.data_ptr(), out.data_ptr(), N, M, Kp, N,
                                         _lib.stream(x.device))
        _lib.check(rc, "bf16 GEMM")
    return out


def gated_residual(h, hc_norm_w, w_down, w_up, w_inj=None, n_inj=0, hc=4, eps=1e-6, moe=None):
    """The hyper-connection mix that produces a layer's MoE input (``fnx/engine.py:818-857``):
    ``h`` bf16 ``[b, 1, hc*H]`` -> ``(mixed [b, 1, H], inj [b, 1, hc])``.  ``w_down`` bf16
    ``[r (+ hc), hc*H]`` (with ``n_inj == hc`` its last rows are the inject weights, as the
    reference's loader concatenates them), ``w_up`` bf16 ``[hc*H, r]``, ``w_inj`` bf16
    ``[hc, hc*H]`` when not concatenated.  RMSNorm, activation and branch mix run on this
    library's kernels with the reference's roundings, the two small GEMMs on its tcgen05 bf16
    GEMM (``mm_nt``).  ``moe``: the ``MoELayer`` whose decode follows (``b <= 16``, ``moe.H == H``;
    ``ValueError`` otherwise, before any launch): its router GEMV is fused into the mix
    (``MoELayer.mix_and_route``) and its decode must be called next with ``logits_ready=True``.
    Same bits either way; on B200 the fused pair is the slower one (25.6 against 23.0 us per layer
    at b = 1), because the decode kernel already overlaps its own router GEMV with the
    expert-weight stream."""
    from . import post_ops
    b, HCH = h.shape[0], h.shape[-1]
    H = HCH // hc
    if moe is not None and (b > DECODE_MAX_TOKENS or moe.E > DECODE_MAX_EXPERTS or moe.H != H):
        raise ValueError(f"gated_residual: the fused router needs b <= {DECODE_MAX_TOKENS}, E <= "
                         f"{DECODE_MAX_EXPERTS} and the layer's H = {H} (got b={b}, E={moe.E}, H={moe.H})")
    h2 = h.reshape(b, HCH).contiguous()
    hn = torch.empty_like(h2)
    rc = _lib.lib().fnx_hc_rms_norm(h2.data_ptr(), hc_norm_w.contiguous().data_ptr(), hn.data_ptr(), b, H, hc, eps,
                                    _lib.stream(h.device))
    _lib.check(rc, "hyper-connection rms_norm")
    if not n_inj:
        if w_inj is None:
            raise ValueError("gated_residual: pass w_inj, or w_down with the inject rows and n_inj = hc")
        w_down = torch.cat([w_down, w_inj])
    di = mm_nt(hn, w_down)
    mix, inj = post_ops.activate(di.view(b, 1, -1).contiguous(), hc)
    logits = mm_nt(mix.view(b, -1), w_up)
    if moe is not None:
        # the router GEMV of the MoE layer that follows, fused into the mix; its decode call must
        # come next on this stream, as moe.decode(mixed, logits_ready=True)
        mixed = moe.mix_and_route(hn, logits, hc)
        return mixed.view(b, 1, H), inj
    mixed = post_ops.mix_reduce(hn.view(b, 1, HCH), logits.view(b, 1, HCH).contiguous(), hc)
    return mixed, inj


class ExpW4:
    """Experts in the W4A16 artifact layout (``tools/repack_w4a16.py``):
    ``w4`` int32 ``[K, E, N/8]`` (or ``[E, K, N/8]`` with ``expert_major``), ``s8t`` int8
    ``[G, E, N]`` and ``base`` bf16 ``[E, N]``; the real scale is
    ``bf16(bf16(s8t) * base)``, cached as ``_scales [E, G, N]`` exactly as
    ``FNX_W4_SCALE_CACHE=1`` does (``fnx/engine.py:653-659``).  The kernels read the
    expert-major words, so a K-major artifact is transposed once here (the byte-exact
    transpose of ``tools/repack_w4_em.py``)."""

    def __init__(self, w4, s8t, base, gs, expert_major=False):
        _lib.require_cuda(w4)
        self.expert_major = True
        self.w4 = (w4 if expert_major else w4.permute(1, 0, 2)).contiguous()
        self.E, self.K = self.w4.shape[0], self.w4.shape[1]
        self.N = self.w4.shape[2] * 8
        self.G = s8t.shape[0]
        self.gs = gs
        self._scales = (s8t.permute(1, 0, 2).to(BF16) * base.to(BF16)[:, None, :]).contiguous()
        self.s8t = self.base = None

    @classmethod
    def from_lqp(cls, v2o, s8, base, gs):
        """Experts straight from the LQP artifact (``v2o [E,N,K/2]`` uint8, ``s8 [E,N,G]`` int8,
        ``base [E,N]`` fp16), with the conversion ``tools/repack_w4a16.py`` does offline: the
        int4 values repacked on the GPU, ``s8t = s8`` as ``[G,E,N]`` and ``base`` in bf16."""
        K = v2o.shape[2] * 2
        w4 = repack_v2o(v2o, K, expert_major=True)
        return cls(w4, s8.permute(2, 0, 1).contiguous(), base.to(BF16), gs, expert_major=True)

    @classmethod
    def from_scales(cls, w4_em, scales, gs):
        """Expert-major words ``[E, K, N/8]`` and ready bf16 scales ``[E, G, N]``."""
        _lib.require_cuda(w4_em, scales)
        o = cls.__new__(cls)
        o.expert_major = True
        o.w4 = w4_em.contiguous()
        o.E, o.K = o.w4.shape[0], o.w4.shape[1]
        o.N = o.w4.shape[2] * 8
        o.G = scales.shape[1]
        o.gs = gs
        o._scales = scales.contiguous()
        o.s8t = o.base = None
        return o

    def tiles(self):
        """The tile blocks the GEMM reads (built once, then cached)."""
        t = getattr(self, "_tiles", None)
        if t is None:
            t = repack_w4(self.w4, self._scales, swiglu=False)
            self._tiles = t
        return t

    def _groups(self, k, M, device):
        """Cached group ends and the source row of every grouped row (row m of every group
        reads x[m]) for k groups of M rows each (the reference keeps ``_dg``/``_ends`` for the
        same purpose, ``fnx/engine.py:661-669``)."""
        cache = self.__dict__.setdefault("_group_cache", {})
        key = (k, M, str(device))
        g = cache.get(key)
        if g is None:
            ends = torch.arange(1, k + 1, device=device, dtype=torch.int64) * M
            rows = torch.arange(k * M, device=device, dtype=torch.int64) % M
            g = cache[key] = (ends, rows)
        return g

    def _ids(self, ids, device):
        if isinstance(ids, torch.Tensor):
            return ids.to(device=device, dtype=torch.int64).contiguous().view(-1)
        return torch.tensor(ids, dtype=torch.int64, device=device).view(-1)

    def _sel(self, x, ids, out, k, M, rows_per_group, diagonal=False):
        """Grouped GEMM over experts ``ids`` read in place from the cached tile blocks (an
        expert-id table, no copy of the selected experts).  ``diagonal``: grouped row j reads
        x[j] (no row index)."""
        ends, rows = self._groups(k, rows_per_group, x.device)
        if diagonal:
            rows = None
        rc = _lib.lib().fnx_moe_grouped_w4_sel(x.data_ptr(), x.stride(0), x.shape[0], _lib.ptr(rows), 1,
                                               self.tiles().data_ptr(), self.E, ids.data_ptr(), ends.data_ptr(),
                                               out.data_ptr(), out.stride(0), k, M, self.K, self.N, EPI_PLAIN,
                                               _lib.stream(x.device))
        _lib.check(rc, "grouped W4A16 GEMM (selected experts)")
        return out

    def apply(self, x, ids):
        """x ``[M, K]`` bf16, ids ``[k]`` -> ``[M, k*N]``: every row times every selected expert."""
        M = x.shape[0]
        x = (x if x.dtype == BF16 else x.to(BF16)).contiguous()
        ids = self._ids(ids, x.device)
        k = ids.numel()
        out = torch.empty(k * M, self.N, dtype=BF16, device=x.device)
        if k and M:
            self._sel(x, ids, out, k, k * M, M)
        return out.view(k, M, self.N).transpose(0, 1).reshape(M, k * self.N)

    def apply_diag(self, x, ids):
        """Row j of x uses expert ids[j] -> ``[k, N]`` (the diagonal of the Cartesian product)."""
        k = x.shape[0]
        x = (x if x.dtype == BF16 else x.to(BF16)).contiguous()
        ids = self._ids(ids, x.device)
        if ids.numel() != k:
            raise ValueError(f"apply_diag: {ids.numel()} expert ids for {k} rows")
        out = torch.empty(k, self.N, dtype=BF16, device=x.device)
        if k:
            self._sel(x, ids, out, k, k, 1, diagonal=True)
        return out

    def apply_grouped(self, x, group_ends, host_ends=None):
        """Rows sorted by expert (cumulative ``group_ends`` over all E experts)."""
        out = torch.empty(x.shape[0], self.N, dtype=BF16, device=x.device)
        return _grouped_w4(x.to(BF16).contiguous(), self.tiles(), group_ends.contiguous(), out, E=self.E,
                           M=x.shape[0], K=self.K, Nw=self.N, epilogue=EPI_PLAIN)


def _values_to_v2o(q):
    """int8 ``[E, N, K]`` values in [-8, 7] -> the LQP ``v2o`` bytes ``[E, N, K/2]`` (byte
    ``64s+j`` = ``W[128s+j] + 8`` low | ``W[128s+64+j] + 8`` high), on q's device."""
    E, N, K = q.shape
    v = (q.to(torch.int16) + 8).to(torch.uint8).view(E, N, K // 128, 2, 64)
    return (v[..., 0, :] | (v[..., 1, :] << 4)).reshape(E, N, K // 2).contiguous()


class ExpQ:
    """Experts given as int4 values or as the LQP artifact (reference ``ExpQ``,
    ``fnx/engine.py:411-616``): ``ExpQ(q, s, gs, packed=True, base=None)`` with ``q`` int8
    ``[E, N, K]`` in [-8, 7] and scales ``s [E, N, K/gs]`` (times ``base [E, N]`` when given),
    or ``ExpQ.from_packed(qv2, s8, base, dev)`` straight from the artifact's offset-binary
    ``v2o [E, N, K/2]``, int8 ``s8 [E, N, G]`` and fp16 ``base [E, N]``.  The real weight is
    ``bf16(q * bf16(bf16(s) * bf16(base)))`` as in ``_deq_v2`` (``fnx/engine.py:503-565``).

    ``matmul(xb, idx)``: row j of ``xb [k, 1, K]`` times expert ``idx[j]`` -> bf16 ``[k, N]``.
    The reference dequantises the selected experts with torch ops and adds two bf16 GEMMs over
    the lo/hi halves of every 128-k block (``_gemm2``, ``fnx/engine.py:772-776``).  Here the
    values are repacked once on the GPU into the W4A16 tile blocks and every call is one
    fp32-accumulated tcgen05 GEMM rounded once, so results agree with the reference's within
    the floating-point tolerance, not bit for bit; no dequantised weight is ever stored.
    ``packed`` is accepted for signature compatibility (storage is always 4-bit)."""

    def __init__(self, q, s, gs, packed=True, base=None):
        _lib.require_cuda(q, s)
        self.gs, self.K, self.N = gs, q.shape[-1], q.shape[1]
        if self.K % 128:
            raise ValueError(f"ExpQ: K={self.K} is not a multiple of 128")
        self.packed, self.dev = True, q.device
        self._init(_values_to_v2o(q), s, base)

    def _init(self, v2o, s, base):
        sc = s.to(BF16)
        if base is not None:
            sc = sc * base.to(BF16).unsqueeze(-1)
        w4 = repack_v2o(v2o, self.K, expert_major=True)
        self.w = ExpW4.from_scales(w4, sc.permute(0, 2, 1).contiguous(), self.gs)
        self.w.tiles()
        self.w.w4 = self.w._scales = None           # the tile blocks carry both

    @classmethod
    def from_packed(cls, qv2, s8, base, dev):
        """``fnx/engine.py:478-501``: ``gs`` is inferred from the artifact (``K / G``)."""
        o = cls.__new__(cls)
        o.dev = torch.device(dev)
        o.N, o.K = qv2.shape[1], qv2.shape[2] * 2
        if o.K % 128:
            raise ValueError(f"ExpQ: K={o.K} is not a multiple of 128")
        o.gs, o.packed = o.K // s8.shape[-1], True
        v2o = qv2.to(o.dev)
        _lib.require_cuda(v2o)
        o._init(v2o, s8.to(o.dev), None if base is None else base.to(o.dev))
        return o

    def matmul(self, xb, idx):
        x = xb.reshape(-1, self.K)
        idx = idx.to(self.dev)
        if x.shape[0] != idx.numel():
            raise ValueError(f"ExpQ.matmul: {x.shape[0]} rows for {idx.numel()} expert ids")
        return self.w.apply_diag(x, idx)

    def to_host_offload(self):
        """Host offload is not part of this build (weights stay in HBM); returns False, as the
        reference does when there is nothing to offload."""
        return False


class DenseW8:
    """Dense int8 weights, per-group bf16 scales (``fnx/engine.py:297-384``):
    ``q`` int8 ``[N, K(+pad)]``, ``s`` ``[N, G]`` -> ``w8t [K, N]``, ``sc [G, N]`` bf16."""

    def __init__(self, q, s, K=None):
        gs = q.shape[-1] // s.shape[-1]
        kk = q.shape[-1] if K is None else K
        if kk % gs:
            raise ValueError(f"DenseW8: K={kk} is not a multiple of gs={gs}")
        g = kk // gs
        self.w8t = q[:, :kk].t().contiguous()
        self.sc = s[:, :g].t().contiguous().to(BF16)
        self.gs = gs
        self.K = kk
        self.N = self.w8t.shape[1]
        self.chunks = None

    def make_chunks(self, chunk_n):
        """Kept for interface parity; the B200 kernel has no N limit, so nothing is split."""
        return None

    def deq_w(self):
        w = self.w8t.to(BF16) * self.sc.repeat_interleave(self.gs, dim=0)
        return w.t().contiguous()

    def __call__(self, x):
        sh = x.shape
        x2 = (x if x.dtype == BF16 else x.to(BF16)).reshape(-1, sh[-1]).contiguous()
        _lib.require_cuda(x2, self.w8t)
        L = _lib.lib()
        M, G = x2.shape[0], self.sc.shape[0]
        y = torch.empty(M, self.N, dtype=BF16, device=x2.device)
        # split-K partials for mid-sized M (stream-ordered by the caching allocator)
        nws = L.fnx_w8a16_gemm_workspace(M, self.K, self.N, G)
        ws = torch.empty(nws, dtype=torch.uint8, device=x2.device) if nws else None
        rc = L.fnx_w8a16_gemm_ws(x2.data_ptr(), self.w8t.data_ptr(), self.sc.data_ptr(), y.data_ptr(), M, self.K,
                                 self.N, G, _lib.ptr(ws), nws, _lib.stream(x2.device))
        _lib.check(rc, "W8A16 GEMM")
        return y if x.dim() <= 2 else y.view(*sh[:-1], self.N)

    @staticmethod
    def merge(parts):
        assert parts and all(p is not None for p in parts)
        gs = parts[0].gs
        assert all(p.gs == gs and p.K == parts[0].K for p in parts), "group size / K differ, cannot merge"
        o = DenseW8.__new__(DenseW8)
        o.w8t = torch.cat([p.w8t for p in parts], dim=1)
        o.sc = torch.cat([p.sc for p in parts], dim=1)
        o.gs, o.K, o.N = gs, parts[0].K, o.w8t.shape[1]
        o.chunks = None
        return o


class MoELayer:
    """One W4A16 MoE layer: routed experts (expert-major int4pack + bf16 group scales, kept
    as the tile blocks of ``repack_w4``), an always-on W4 shared expert with a sigmoid
    gate, and a bf16 router.

    ``router_cat`` concatenates the router rows and the shared-expert gate row into one
    bf16 ``[R, H]`` GEMM operand (the reference's load-time concat,
    ``fnx/engine.py:1223-1236``), padded to a multiple of 128 rows with zeros."""

    def __init__(self, gu_w4, gu_scales, dn_w4, dn_scales, gate_w, sh_gu_w4, sh_gu_scales, sh_dn_w4, sh_dn_scales,
                 sh_gate, k, gs, bias=None):
        _lib.require_cuda(gu_w4, dn_w4, gate_w, sh_gu_w4, sh_dn_w4)
        self.E, self.H = gate_w.shape
        self.I = gu_w4.shape[2] * 8 // 2
        # tile blocks (the artifact tensors are not kept): routed experts 0..E-1 and the
        # shared expert as expert E, so prefill runs both in one grouped launch per projection
        E = self.E
        self.gu_all = repack_w4(torch.cat([gu_w4, sh_gu_w4[None]]), torch.cat([gu_scales, sh_gu_scales[None]]),
                                swiglu=True)
        self.dn_all = repack_w4(torch.cat([dn_w4, sh_dn_w4[None]]), torch.cat([dn_scales, sh_dn_scales[None]]),
                                swiglu=False)
        self.gu_t, self.sh_gu_t = self.gu_all[:E], self.gu_all[E:]
        self.dn_t, self.sh_dn_t = self.dn_all[:E], self.dn_all[E:]
        self._init_router(gate_w, sh_gate, k, gs, bias)

    def _init_router(self, gate_w, sh_gate, k, gs, bias):
        self.E, self.H = gate_w.shape
        self.k, self.gs = k, gs
        R = self.E + 1
        self.R = R
        self.R_pad = (R + 127) // 128 * 128
        rc = torch.zeros(self.R_pad, self.H, dtype=BF16, device=gate_w.device)
        rc[:self.E] = gate_w
        rc[self.E] = sh_gate.reshape(-1)
        self.router_cat = rc
        self.bias = None if bias is None else bias.to(torch.float32).to(gate_w.device).contiguous()
        self._ws = {}
        self._routed = set()        # decode workspaces holding logits from mix_and_route
        self._prefill_bufs = {}

    @classmethod
    def from_synth(cls, t, shape, bias=None):
        return cls(t["gu_w4"], t["gu_scales"], t["dn_w4"], t["dn_scales"], t["gate_w"], t["sh_gu_w4"],
                   t["sh_gu_scales"], t["sh_dn_w4"], t["sh_dn_scales"], t["sh_gate"], shape.k, shape.gs, bias=bias)

    def weight_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.gu_all, self.dn_all, self.router_cat))

    # ---------------------------------------------------------------- routing
    def logits(self, x, native=True):
        """bf16 ``[T, R_pad]``: router logits in columns ``[0, E)``, shared gate in column E:
        one bf16 GEMM over the concatenated router (fp32 accumulation, rounded once) on this
        library's tcgen05 bf16 GEMM.  ``native=False`` runs the same product on cuBLAS, for
        comparisons."""
        if not native:
            return torch.mm(x, self.router_cat.t())
        T = x.shape[0]
        out = torch.empty(T, self.R_pad, dtype=BF16, device=x.device)
        rc = _lib.lib().fnx_bf16_gemm_nt(x.data_ptr(), x.stride(0), self.router_cat.data_ptr(), out.data_ptr(),
                                         out.stride(0), T, self.H, self.R_pad, _lib.stream(x.device))
        _lib.check(rc, "router GEMM")
        return out

    def topk(self, logits, ld=None):
        T = logits.shape[0]
        w = torch.empty(T, self.k, dtype=BF16, device=logits.device)
        idx = torch.empty(T, self.k, dtype=torch.int64, device=logits.device)
        wf = torch.empty(T, self.k, dtype=torch.float32, device=logits.device)
        rc = _lib.lib().fnx_router_topk(logits.data_ptr(), ld or logits.stride(0), _lib.ptr(self.bias), w.data_ptr(),
                                        idx.data_ptr(), wf.data_ptr(), T, self.E, self.k, _lib.stream(logits.device))
        _lib.check(rc, "router top-k")
        return w, idx, wf

    def permute(self, idx, order=None, ends=None):
        n = idx.numel()
        dev = idx.device
        order = torch.empty(n, dtype=torch.int64, device=dev) if order is None else order
        inverse = torch.empty(n, dtype=torch.int64, device=dev)
        ends = torch.empty(self.E, dtype=torch.int64, device=dev) if ends is None else ends
        wsb = _lib.lib().fnx_moe_permute_workspace(n, self.E)
        ws = torch.empty(max(1, wsb), dtype=torch.uint8, device=dev)
        rc = _lib.lib().fnx_moe_permute(idx.data_ptr(), order.data_ptr(), inverse.data_ptr(), ends.data_ptr(), None, n,
                                        self.E, ws.data_ptr(), wsb, _lib.stream(dev))
        _lib.check(rc, "expert permutation")
        return order, inverse, ends

    # ---------------------------------------------------------------- paths
    def forward(self, x):
        x = x.reshape(-1, self.H)
        if x.dtype != BF16:
            x = x.to(BF16)
        x = x.contiguous()
        if x.shape[0] <= DECODE_MAX_TOKENS and self.E <= DECODE_MAX_EXPERTS:
            return self.decode(x)[0]
        return self.prefill(x)

    __call__ = forward

    def capture(self, T, device=None):
        """This layer's call on ``T`` tokens captured into one CUDA graph over static buffers
        (the reference's graph-level caller, ``FnModel.capture`` ``fnx/model.py:288-358``:
        three warm-up calls on a side stream, then the capture).  Returns a
        ``CapturedLayer``; its replay launches the same kernels as a direct call."""
        return CapturedLayer(self, T, device or self.router_cat.device)

    def moe_inject(self, x, hyper, inj):
        """The MoE half of a layer's tail, ``inject(h, inj, self._moe(mixed))``
        (``fnx/engine.py:1945-1946``): ``hyper`` bf16 ``[b, 1, HC*H]`` (the hyper-connection
        state), ``inj`` bf16 ``[b, 1, HC]``; returns the new state.  The grouped path applies
        the inject inside the combine pass; the decode path runs it after the fused layer."""
        from . import native_inject
        x2 = x.reshape(-1, self.H)
        if x2.dtype != BF16:
            x2 = x2.to(BF16)
        x2 = x2.contiguous()
        hyper, inj = hyper.contiguous(), inj.contiguous()
        if x2.shape[0] <= DECODE_MAX_TOKENS and self.E <= DECODE_MAX_EXPERTS:
            y = self.decode(x2)[0]
            out = native_inject.inject(hyper, inj, y.view(x2.shape[0], 1, self.H))
            if out is None:
                raise ValueError("moe_inject: unsupported hyper / inj shapes")
            return out
        return self.prefill(x2, inject=(hyper, inj))

    def prefill(self, x, details=False, inject=None, logits=None):
        """Grouped path (``fnx/engine.py:1815-1853``) for ``T`` tokens.  The routed and the shared
        expert share one grouped launch per projection; the per-call buffers of the extended
        permutation are cached per token count (calls on one layer must not overlap).
        ``logits``: bf16 ``[T, >= E+1]`` router logits (columns ``[0, E)``) and shared-expert gate
        (column ``E``) computed elsewhere, in place of this layer's router GEMM."""
        T, H, I, k, E = x.shape[0], self.H, self.I, self.k, self.E
        dev = x.device
        M = T * k
        if logits is None:
            logits = self.logits(x)
        elif logits.dtype != BF16 or logits.dim() != 2 or logits.shape[0] != T or logits.shape[1] <= E \
                or logits.stride(1) != 1 or logits.device != dev:
            raise ValueError("prefill: logits must be bf16 [T, >= E+1], row-major, on x's device")
        # expert-major rows of the routed experts, then the shared expert (expert E) over all
        # T tokens: its rows M .. M+T-1 read token t (row index t*k, divided by k)
        key = (T, str(dev))
        bufs = self._prefill_bufs.get(key)
        if bufs is None:
            order_x = torch.empty(M + T, dtype=torch.int64, device=dev)
            order_x[M:] = torch.arange(T, dtype=torch.int64, device=dev) * k
            ends_x = torch.empty(E + 1, dtype=torch.int64, device=dev)
            ends_x[E] = M + T
            bufs = self._prefill_bufs[key] = (order_x, ends_x)
        order_x, ends_x = bufs
        act = torch.empty(M + T, I, dtype=BF16, device=dev)
        yd = torch.empty(M + T, H, dtype=BF16, device=dev)
        side = self._shared_side_stream(dev) if T else None
        if side is not None:
            # the shared expert (expert E, all T tokens) on a second stream while this one routes
            # and permutes, on all but SHARED_RESERVE_SMS SMs; then the routed experts alone
            main = torch.cuda.current_stream(dev)
            side.wait_stream(main)
            sh_ends = self._sh_ends_for(T, dev)
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            ctas = max(2, (sms - SHARED_RESERVE_SMS) // 2 * 2)
            L = _lib.lib()
            gu_sh = self.gu_all[E:E + 1]
            dn_sh = self.dn_all[E:E + 1]
            with torch.cuda.stream(side):
                ss = side.cuda_stream
                _lib.check(L.fnx_moe_grouped_w4_lim(x.data_ptr(), x.stride(0), T, None, 1, gu_sh.data_ptr(),
                                                    sh_ends.data_ptr(), act[M:].data_ptr(), I, 1, T, H, 2 * I,
                                                    EPI_SWIGLU_BF16, ctas, ss), "shared expert gate/up")
                _lib.check(L.fnx_moe_grouped_w4_lim(act[M:].data_ptr(), I, T, None, 1, dn_sh.data_ptr(),
                                                    sh_ends.data_ptr(), yd[M:].data_ptr(), H, 1, T, I, H, EPI_PLAIN,
                                                    ctas, ss), "shared expert down")
        w, idx, wf = self.topk(logits)
        order, inverse, ends = self.permute(idx, order=order_x[:M], ends=ends_x[:E])
        if side is not None:
            if M:
                _grouped_w4(x, self.gu_all, ends_x, act, E=E, M=M, K=H, Nw=2 * I, epilogue=EPI_SWIGLU_F32,
                            row_index=order_x, index_div=k)
                _grouped_w4(act, self.dn_all, ends_x, yd, E=E, M=M, K=I, Nw=H, epilogue=EPI_PLAIN)
            main.wait_stream(side)
        else:
            _grouped_w4(x, self.gu_all, ends_x, act, E=E + 1, M=M + T, K=H, Nw=2 * I, epilogue=EPI_SWIGLU_MIXED,
                        row_index=order_x, index_div=k)
            _grouped_w4(act, self.dn_all, ends_x, yd, E=E + 1, M=M + T, K=I, Nw=H, epilogue=EPI_PLAIN)
        sh_act, sh = act[M:], yd[M:]
        gate = logits[:, E:E + 1]
        if inject is not None:              # combine + residual inject in one pass
            hyper, inj = inject
            HC = inj.numel() // T
            if hyper.numel() != T * HC * H:
                raise ValueError("prefill inject: hyper must hold T * HC * H values")
            out_h = torch.empty_like(hyper)
            rc = _lib.lib().fnx_moe_combine_inject(yd.data_ptr(), wf.data_ptr(), inverse.data_ptr(), sh.data_ptr(),
                                                   gate.data_ptr(), logits.stride(0), hyper.data_ptr(), inj.data_ptr(),
                                                   out_h.data_ptr(), None, T, k, H, HC, _lib.stream(dev))
            _lib.check(rc, "MoE combine + inject")
            return out_h
        out = torch.empty(T, H, dtype=BF16, device=dev)
        rc = _lib.lib().fnx_moe_combine(yd.data_ptr(), wf.data_ptr(), inverse.data_ptr(), sh.data_ptr(),
                                        gate.data_ptr(), logits.stride(0), out.data_ptr(), T, k, H, _lib.stream(dev))
        _lib.check(rc, "MoE combine")
        if details:
            return out, dict(logits=logits[:, :E], gate=gate, w=w, idx=idx, order=order, inverse=inverse, ends=ends,
                             act=act[:M], yd=yd[:M], sh=sh, sh_act=sh_act)
        return out

    def permute_experts(self, perm):
        """Renumber the routed experts in place: new expert j is old expert perm[j] (its router row,
        bias and tile blocks move together), e.g. to give the contiguous expert blocks of an
        expert-parallel split equal loads.  The layer computes the same function, except where two
        experts have exactly equal probability: the tie rule orders them by their (new) ids."""
        E = self.E
        perm = torch.as_tensor(perm, dtype=torch.int64).reshape(-1)
        if perm.numel() != E or not torch.equal(torch.sort(perm).values, torch.arange(E)):
            raise ValueError(f"permute_experts: not a permutation of {E} experts")
        p = perm.to(self.router_cat.device)
        self.router_cat[:E] = self.router_cat[:E].index_select(0, p)
        if self.bias is not None:
            self.bias = self.bias.index_select(0, p).contiguous()
        self.gu_all[:E] = self.gu_all[:E].index_select(0, p)
        self.dn_all[:E] = self.dn_all[:E].index_select(0, p)
        return self

    def _shared_side_stream(self, dev):
        """The second stream of the overlapped prefill (None when `overlap_shared` is off)."""
        if not getattr(self, "overlap_shared", OVERLAP_SHARED):
            return None
        streams = self.__dict__.setdefault("_side_streams", {})
        st = streams.get(str(dev))
        if st is None:
            st = streams[str(dev)] = torch.cuda.Stream(dev)
        return st

    def _sh_ends_for(self, T, dev):
        cache = self.__dict__.setdefault("_sh_ends", {})
        t = cache.get((T, str(dev)))
        if t is None:
            t = cache[(T, str(dev))] = torch.full((1,), T, dtype=torch.int64, device=dev)
        return t

    def decode_workspace(self, M, device):
        key = (M, str(device))
        ws = self._ws.get(key)
        if ws is None:
            n = _lib.lib().fnx_moe_decode_workspace(M, self.H, self.I, self.E, self.k)
            ws = torch.zeros(n, dtype=torch.uint8, device=device)      # tickets start at zero
            self._ws[key] = ws
        return ws

    def decode(self, x, out=None, w_out=None, idx_out=None, logits_ready=False):
        """Fused decode kernels for ``M <= 16`` tokens; returns ``(out, w, idx)``.
        ``logits_ready``: ``x`` came from ``mix_and_route`` just before, which left its router logits
        in this layer's decode workspace, so the launch skips its router items."""
        M = x.shape[0]
        dev = x.device
        out = torch.empty(M, self.H, dtype=BF16, device=dev) if out is None else out
        w_out = torch.empty(M, self.k, dtype=BF16, device=dev) if w_out is None else w_out
        idx_out = torch.empty(M, self.k, dtype=torch.int64, device=dev) if idx_out is None else idx_out
        ws = self.decode_workspace(M, dev)
        key = (M, str(dev))
        if logits_ready and key not in self._routed:
            raise RuntimeError("decode(logits_ready=True) needs mix_and_route on the same rows just before")
        self._routed.discard(key)
        rc = _lib.lib().fnx_moe_decode_w4_ex(
            x.data_ptr(), self.router_cat.data_ptr(), self.gu_t.data_ptr(), self.dn_t.data_ptr(),
            self.sh_gu_t.data_ptr(), self.sh_dn_t.data_ptr(), _lib.ptr(self.bias), out.data_ptr(), w_out.data_ptr(),
            idx_out.data_ptr(), M, self.H, self.I, self.E, self.k, ws.data_ptr(), ws.numel(),
            1 if logits_ready else 0, _lib.stream(dev))
        _lib.check(rc, "MoE decode")
        return out, w_out, idx_out

    def mix_and_route(self, hn, mix_logits, hc=4):
        """The branch mix that produces this layer's decode input, with the router GEMV fused behind
        it (``fnx_hc_mix_router``): ``hn``, ``mix_logits`` bf16 ``[M, hc*H]`` -> ``mixed [M, H]``
        (the bits of ``post_ops.mix_reduce``), the router logits of ``mixed`` left in this layer's
        decode workspace for the next ``decode(mixed, logits_ready=True)`` on the same stream."""
        _lib.require_cuda(hn, mix_logits)
        M = hn.shape[0]
        dev = hn.device
        hn = hn.reshape(M, -1).contiguous()
        mix_logits = mix_logits.reshape(M, -1).contiguous()
        if hn.shape[1] != hc * self.H or mix_logits.shape != hn.shape:
            raise ValueError(f"mix_and_route: rows of {hc}*{self.H} expected, got {tuple(hn.shape)}")
        mixed = torch.empty(M, self.H, dtype=BF16, device=dev)
        ws = self.decode_workspace(M, dev)
        rc = _lib.lib().fnx_hc_mix_router(hn.data_ptr(), mix_logits.data_ptr(), mixed.data_ptr(),
                                          self.router_cat.data_ptr(), ws.data_ptr(), ws.numel(), M, self.H, self.I,
                                          self.E, self.k, hc, _lib.stream(dev))
        _lib.check(rc, "hyper-connection mix + router")
        self._routed.add((M, str(dev)))
        return mixed


class CapturedLayer:
    """One MoE layer call replayed from a CUDA graph.  ``x`` is the static bf16 ``[T, H]``
    input and ``out`` the static output; ``replay()`` runs the layer on whatever ``x``
    holds, ``__call__(x)`` copies ``x`` in first.  The layer's own buffers stay bound to the
    graph, so one layer object backs one capture at a time."""

    def __init__(self, layer, T, device):
        self.layer = layer
        self.x = torch.zeros(T, layer.H, dtype=BF16, device=device)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(3):
                layer(self.x)
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            out = layer(self.x)
        self.out = out[0] if isinstance(out, tuple) else out

    def replay(self):
        self.graph.replay()
        return self.out

    def __call__(self, x):
        if x.data_ptr() != self.x.data_ptr():
            self.x.copy_(x.reshape(self.x.shape), non_blocking=True)
        return self.replay()


class HostPipeline:
    """Layer calls on batches that live in pinned host memory, with the copies overlapped:
    while batch i's graph replays on the compute stream, batch i+1's input goes up and batch
    i-1's output comes down on two copy streams (the two directions of the host link run at
    once).  ``slots`` are ``CapturedLayer`` objects used round-robin (at least two); batch i
    runs on slot ``i % len(slots)``.  A slot's input buffer is refilled once its previous
    batch's replay is done (that replay is the only reader of the input), and its next replay
    waits until the previous output has been copied out, so the upload of batch i+1 does not
    wait for the download of batch i-1: per batch the pipeline takes the longest of the replay,
    the upload and the download, not the replay or their sum."""

    def __init__(self, slots):
        if len(slots) < 2:
            raise ValueError("HostPipeline needs at least two captured slots")
        self.slots = list(slots)
        self.device = self.slots[0].x.device
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)

    def run(self, xs_host, outs_host):
        """``outs_host[i] <- layer(xs_host[i])`` for every i (pinned host tensors); returns
        when the work is queued (synchronise the device, or the last output's stream, to
        read the results)."""
        n, S = len(xs_host), len(self.slots)
        comp = torch.cuda.current_stream(self.device)
        ev = lambda: torch.cuda.Event()                       # noqa: E731
        in_ready, done, out_free = [None] * n, [None] * n, [None] * n
        start = ev()
        start.record(comp)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)

        def upload(i):
            s = self.slots[i % S]
            if i >= S:                                      # the slot's previous replay read its input
                self.h2d.wait_event(done[i - S])
            with torch.cuda.stream(self.h2d):
                s.x.copy_(xs_host[i].reshape(s.x.shape), non_blocking=True)
            in_ready[i] = ev()
            in_ready[i].record(self.h2d)

        if n:
            upload(0)
        for i in range(n):
            s = self.slots[i % S]
            if i + 1 < n:
                upload(i + 1)
            comp.wait_event(in_ready[i])
            if i >= S:                                      # the slot's previous output is copied out
                comp.wait_event(out_free[i - S])
            s.replay()
            done[i] = ev()
            done[i].record(comp)
            self.d2h.wait_event(done[i])
            with torch.cuda.stream(self.d2h):
                outs_host[i].copy_(s.out, non_blocking=True)
            out_free[i] = ev()
            out_free[i].record(self.d2h)
        # the caller's stream sees every output copied
        end = ev()
        end.record(self.d2h)
        comp.wait_event(end)
