"""Expert-parallel MoE layer: the routed experts split over the ranks of a process group,
token rows dispatched to the experts' owners and the expert outputs combined back with
all-to-all exchanges (NCCL over NVLink on B200; any ``torch.distributed`` backend works).

The reference runs the whole MoE layer on one device (``FnLayer._moe``,
``fnx/engine.py:1782-1930``); this layer partitions its 512 experts in contiguous blocks of
E/G over G ranks.  Per call on rank r (experts ``[r*E/G, (r+1)*E/G)`` live here; the router
and the shared expert live on every rank):

1. route the rank's own T tokens (router GEMM, top-k), as the one-device layer does;
2. sort the T*k (token, slot) entries by owner rank, stable (``fnx_ep_dispatch_layout``),
   and pack one token row per entry in that order with its owner-local expert id
   (``fnx_ep_gather_rows``);
3. exchange the per-owner counts, then the rows and ids (all-to-all-v);
4. on the owner: sort the received entries expert-major (``fnx_moe_permute``) and run the
   grouped gate/up + SwiGLU and down launches over them, with the shared expert over the
   rank's own T tokens appended as local expert E/G of the same two launches;
5. gather the down rows back into received order and send them home (all-to-all-v);
6. the slot-order weighted reduce and sigmoid-gated shared merge (``fnx_moe_combine``),
   reading slot q's row through the dispatch layout's inverse.

Every slot's down row comes from the same kernel and operands as on one device, and step 6
reduces in the reference's slot order, so the output equals ``MoELayer`` on one GPU bit for
bit.  Rows are exchanged per slot (a token with three experts on one owner is sent three
times) so that the owner never reduces: the combine stays the reference's fixed-order sum.

Two transports move the rows:

* ``"p2p"`` (default on CUDA): this library's kernels write each row straight into its
  destination's exchange region through NVLink peer mappings (CUDA IPC), the per-owner
  counts travel the same way behind release/acquire flags, and nothing waits on the host --
  the layer is one stream of launches, capturable in a CUDA graph;
* ``"collective"``: ``torch.distributed.all_to_all_single`` (NCCL, or gloo on CPU ranks)
  with the counts exchanged first and read on the host to size the transfers.
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib
from .engine import BF16, EPI_PLAIN, EPI_SWIGLU_BF16, EPI_SWIGLU_F32, EPI_SWIGLU_MIXED, MoELayer, _grouped_w4, repack_w4

I64 = torch.int64
EPI_SWIGLU_SHARED_FIRST = 4      # EPI_SWIGLU_MIXED with the shared expert as expert 0


class _PeerExchange:
    """The ranks' exchange regions (``fnx_ep_p2p_*``): one zero-filled ``cudaMalloc`` per
    rank, mapped into every peer through CUDA IPC, and the kernels' descriptor."""

    def __init__(self, rank, world, group, H, k, max_tokens, e_local, device):
        L = _lib.lib()
        self.world, self.group = world, group
        self.H, self.k, self.max_tokens, self.e_local = H, k, max_tokens, e_local
        nbytes = L.fnx_ep_p2p_region_bytes(world, H, k, max_tokens)
        if not nbytes:
            raise ValueError(f"peer exchange: unsupported shape (world={world}, H={H}, k={k}, T={max_tokens})")
        self.imported = []
        with torch.cuda.device(device):
            base = ctypes.c_void_p()
            _lib.check(L.fnx_ep_p2p_alloc(nbytes, ctypes.byref(base)), "exchange region allocation")
            self.base = base
            bases = [0] * world
            bases[rank] = base.value
            if world > 1:
                h = ctypes.create_string_buffer(64)
                _lib.check(L.fnx_ep_p2p_export(base, h), "exchange region IPC export")
                handles = [None] * world
                dist.all_gather_object(handles, h.raw, group=group)
                for q in range(world):
                    if q == rank:
                        continue
                    p = ctypes.c_void_p()
                    hq = ctypes.create_string_buffer(handles[q], 64)
                    _lib.check(L.fnx_ep_p2p_import(hq, ctypes.byref(p)), f"exchange region IPC import (rank {q})")
                    self.imported.append(p)
                    bases[q] = p.value
            self._desc = ctypes.create_string_buffer(L.fnx_ep_p2p_desc_bytes())
            self.desc = ctypes.addressof(self._desc)
            _lib.check(L.fnx_ep_p2p_desc(self.desc, rank, world, (ctypes.c_void_p * world)(*bases), H, k, max_tokens,
                                         e_local), "exchange descriptor")
        self.cap = L.fnx_ep_p2p_capacity(self.desc, 0)          # received slots
        self.cap_tok = L.fnx_ep_p2p_capacity(self.desc, 1)      # received token rows
        self.recv_x = L.fnx_ep_p2p_local(self.desc, 0)
        self.yb = L.fnx_ep_p2p_local(self.desc, 2)

    def close(self):
        L = _lib.lib()
        torch.cuda.synchronize()
        for p in self.imported:
            L.fnx_ep_p2p_close(p)
        self.imported = []
        if self.world > 1:
            dist.barrier(group=self.group)        # no peer maps this region any more
        L.fnx_ep_p2p_free(self.base)
        self.base = None


def balanced_expert_order(counts, world):
    """An expert order (new id j = old expert order[j]) whose contiguous blocks of E/world experts,
    one per rank, carry near-equal loads: experts by descending count (ties by id) each go to the
    least loaded rank that still has room (longest-processing-time first with equal block sizes).
    ``counts``: slots per expert from a calibration batch.  The heaviest rank is at most the mean
    plus the largest single expert; a single expert above the mean share bounds it from below."""
    c = torch.as_tensor(counts, dtype=torch.float64).reshape(-1).cpu()
    E = c.numel()
    if world < 1 or E % world:
        raise ValueError(f"balanced_expert_order: {E} experts over {world} ranks")
    per = E // world
    order = sorted(range(E), key=lambda e: (-float(c[e]), e))
    load = [0.0] * world
    blocks = [[] for _ in range(world)]
    for e in order:
        r = min((q for q in range(world) if len(blocks[q]) < per), key=lambda q: (load[q], q))
        blocks[r].append(e)
        load[r] += float(c[e])
    return torch.tensor([e for b in blocks for e in sorted(b)], dtype=torch.int64)


class ExpertParallelMoE(MoELayer):
    """One MoE layer whose routed experts are sharded over ``world`` ranks.

    ``gu_w4 / gu_scales / dn_w4 / dn_scales`` hold this rank's experts only (expert-major
    int4pack and bf16 group scales of experts ``[rank*E/world, (rank+1)*E/world)``);
    ``gate_w`` is the full router ``[E, H]``; the shared expert is replicated.  ``group``
    is the process group of the ``world`` ranks (``None``: the default group; unused when
    ``world == 1``)."""

    def __init__(self, gu_w4, gu_scales, dn_w4, dn_scales, gate_w, sh_gu_w4, sh_gu_scales, sh_dn_w4, sh_dn_scales,
                 sh_gate, k, gs, *, rank=0, world=1, group=None, bias=None, transport="auto", max_tokens=4096):
        _lib.require_cuda(gu_w4, dn_w4, gate_w, sh_gu_w4, sh_dn_w4)
        self._init_router(gate_w, sh_gate, k, gs, bias)
        self._init_shard(rank, world, group, gu_w4.shape[0], transport, max_tokens)
        self.I = gu_w4.shape[2] * 8 // 2
        self.gu_loc = self._arrange(repack_w4(torch.cat([gu_w4, sh_gu_w4[None]]),
                                              torch.cat([gu_scales, sh_gu_scales[None]]), swiglu=True))
        self.dn_loc = self._arrange(repack_w4(torch.cat([dn_w4, sh_dn_w4[None]]),
                                              torch.cat([dn_scales, sh_dn_scales[None]]), swiglu=False))
        self._setup_transport(gate_w.device)

    def _init_shard(self, rank, world, group, e_local, transport="collective", max_tokens=4096):
        if world < 1 or not 0 <= rank < world or self.E % world or e_local != self.E // world:
            raise ValueError(f"ExpertParallelMoE: {e_local} local experts of E={self.E} on rank {rank} of {world}")
        if transport == "auto":
            nccl = world == 1 or (dist.is_initialized() and dist.get_backend(group) == "nccl")
            transport = "p2p" if nccl else "collective"
        if transport not in ("p2p", "collective"):
            raise ValueError(f"ExpertParallelMoE: unknown transport {transport!r}")
        self.rank, self.world, self.group = rank, world, group
        self.E_local = e_local
        self.transport = transport
        self.max_tokens = max_tokens
        self.last_counts = None
        self._p2p = None
        # p2p: run the shared expert (which needs only this rank's own tokens) on a second stream
        # while the exchange kernels run, on all but `reserve_sms` SMs, which the exchange keeps
        # (FNX_EP_OVERLAP=0: the single-stream form, for comparisons)
        self.overlap_shared = os.environ.get("FNX_EP_OVERLAP", "1") != "0"
        self.reserve_sms = int(os.environ.get("FNX_EP_RESERVE_SMS", "64"))
        self._side = None
        self._sh_ends = {}

    def _arrange(self, tiles):
        """Routed experts then the shared one (collective transport), or the shared expert
        first (p2p: its rows precede the received slots, whose count only the device knows)."""
        if self.transport == "p2p":
            return torch.cat([tiles[-1:], tiles[:-1]]).contiguous()
        return tiles

    def _setup_transport(self, device, exchange=None):
        self._own_p2p = exchange is None
        if self.transport == "p2p":
            if exchange is not None:
                if (exchange.world != self.world or exchange.H != self.H or exchange.k != self.k
                        or exchange.max_tokens < self.max_tokens or exchange.e_local != self.E_local):
                    raise ValueError("ExpertParallelMoE: the shared exchange was made for another shape")
                self._p2p = exchange
            else:
                self._p2p = _PeerExchange(self.rank, self.world, self.group, self.H, self.k, self.max_tokens,
                                          self.E_local, device)

    @property
    def exchange(self):
        """The peer exchange (p2p transport), for other layers of the same stack to share."""
        return self._p2p

    @classmethod
    def from_layer(cls, layer: MoELayer, rank, world, group=None, transport="auto", max_tokens=4096,
                   exchange=None):
        """This rank's shard of a one-device ``MoELayer`` (its tile blocks are copied, so the
        full layer may be dropped afterwards).  Collective over the group when the transport
        is ``"p2p"`` (the ranks exchange their regions' IPC handles).  ``exchange``: the peer
        exchange of another layer of the same shape, to share (the layers of a stack run one
        after another, and the exchange's device-side call epochs order them); the layer that
        made it releases it."""
        o = cls.__new__(cls)
        o.E, o.H, o.I, o.k, o.gs = layer.E, layer.H, layer.I, layer.k, layer.gs
        o.R, o.R_pad, o.router_cat, o.bias = layer.R, layer.R_pad, layer.router_cat, layer.bias
        o._ws, o._prefill_bufs = {}, {}
        o._init_shard(rank, world, group, layer.E // world if layer.E % world == 0 else -1, transport, max_tokens)
        lo, hi = rank * o.E_local, (rank + 1) * o.E_local
        o.gu_loc = o._arrange(torch.cat([layer.gu_all[lo:hi], layer.gu_all[layer.E:]]))
        o.dn_loc = o._arrange(torch.cat([layer.dn_all[lo:hi], layer.dn_all[layer.E:]]))
        o._setup_transport(layer.router_cat.device, exchange)
        return o

    def capture(self, T, device=None):
        """The layer's call on ``T`` tokens as one CUDA graph (``MoELayer.capture``); every
        rank captures, and replays, in step.  Needs the p2p transport: the collective one
        reads the exchange counts on the host."""
        if self.transport != "p2p":
            raise RuntimeError("ExpertParallelMoE.capture needs transport='p2p'")
        return super().capture(T, device)

    def close(self):
        """Release the peer exchange if this layer made it (collective over the group)."""
        if self._p2p is not None and getattr(self, "_own_p2p", True):
            self._p2p.close()
        self._p2p = None

    # ---------------------------------------------------------------- stages
    def route(self, x):
        """Step 1: ``(logits, w, idx, wf)`` of the rank's tokens."""
        logits = self.logits(x)
        w, idx, wf = self.topk(logits)
        return logits, w, idx, wf

    def dispatch_layout(self, idx):
        """Step 2a: owner-major order of the ``T*k`` slots, its inverse, per-owner counts."""
        n = idx.numel()
        dev = idx.device
        order = torch.empty(n, dtype=I64, device=dev)
        inverse = torch.empty(n, dtype=I64, device=dev)
        counts = torch.empty(self.world, dtype=I64, device=dev)
        L = _lib.lib()
        wsb = L.fnx_ep_layout_workspace(n, self.world)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = L.fnx_ep_dispatch_layout(idx.data_ptr(), n, self.E, self.world, order.data_ptr(), inverse.data_ptr(),
                                      counts.data_ptr(), ws.data_ptr(), wsb, _lib.stream(dev))
        _lib.check(rc, "expert-parallel dispatch layout")
        return order, inverse, counts

    def gather_rows(self, src, index, div, n, ids=None, mod=1, out=None):
        """``out[p] = src[index[p] // div]`` (and owner-local ids ``ids[index[p]] % mod``)."""
        dev = src.device
        H = src.shape[1]
        out = torch.empty(n, H, dtype=BF16, device=dev) if out is None else out
        ids_out = torch.empty(n, dtype=I64, device=dev) if ids is not None else None
        rc = _lib.lib().fnx_ep_gather_rows(src.data_ptr(), src.stride(0), src.shape[0], _lib.ptr(index), div,
                                           _lib.ptr(ids), mod, out.data_ptr(), out.stride(0), _lib.ptr(ids_out), n, H,
                                           _lib.stream(dev))
        _lib.check(rc, "expert-parallel row gather")
        return out, ids_out

    def pack(self, x, idx, order):
        """Step 2b: one token row per slot in owner-major order and its owner-local expert."""
        return self.gather_rows(x, order, self.k, idx.numel(), ids=idx.reshape(-1), mod=self.E_local)

    def local_experts(self, act, recv_e, R):
        """Step 4 (collective transport): ``act`` holds the ``R`` received rows followed by
        the rank's own ``T`` tokens; returns the down rows ``[R+T, H]`` (the received slots
        expert-major, then the shared expert's rows) and the received slots' rows in it
        (``inverse``)."""
        assert self.transport == "collective", "the p2p transport runs its own receive side"
        dev = act.device
        T = act.shape[0] - R
        Eg, H, I = self.E_local, self.H, self.I
        order_x = torch.empty(R + T, dtype=I64, device=dev)
        ends_x = torch.empty(Eg + 1, dtype=I64, device=dev)
        inverse = torch.empty(R, dtype=I64, device=dev)
        L = _lib.lib()
        wsb = L.fnx_moe_permute_workspace(R, Eg)
        ws = torch.empty(max(1, wsb), dtype=torch.uint8, device=dev)
        rc = L.fnx_moe_permute(recv_e.data_ptr(), order_x.data_ptr(), inverse.data_ptr(), ends_x.data_ptr(), None, R,
                               Eg, ws.data_ptr(), wsb, _lib.stream(dev))
        _lib.check(rc, "expert permutation")
        torch.add(self._arange(T, dev), R, out=order_x[R:])
        ends_x[Eg:].fill_(R + T)
        a2 = torch.empty(R + T, I, dtype=BF16, device=dev)
        _grouped_w4(act, self.gu_loc, ends_x, a2, E=Eg + 1, M=R + T, K=H, Nw=2 * I, epilogue=EPI_SWIGLU_MIXED,
                    row_index=order_x, index_div=1)
        yd = torch.empty(R + T, H, dtype=BF16, device=dev)
        _grouped_w4(a2, self.dn_loc, ends_x, yd, E=Eg + 1, M=R + T, K=I, Nw=H, epilogue=EPI_PLAIN)
        return yd, inverse

    def unpack(self, yd, inverse, R):
        """Step 5a: the received slots' down rows in received order."""
        return self.gather_rows(yd, inverse, 1, R)[0]

    def combine(self, yb, wf, inverse_d, sh, logits):
        """Step 6: slot-order reduce of the returned rows + gated shared merge."""
        T = wf.shape[0]
        out = torch.empty(T, self.H, dtype=BF16, device=yb.device)
        gate = logits[:, self.E:self.E + 1]
        rc = _lib.lib().fnx_moe_combine(yb.data_ptr(), wf.data_ptr(), inverse_d.data_ptr(), sh.data_ptr(),
                                        gate.data_ptr(), logits.stride(0), out.data_ptr(), T, self.k, self.H,
                                        _lib.stream(yb.device))
        _lib.check(rc, "MoE combine")
        return out

    def _arange(self, T, dev):
        key = ("arange", T, str(dev))
        a = self._prefill_bufs.get(key)
        if a is None:
            a = self._prefill_bufs[key] = torch.arange(T, dtype=I64, device=dev)
        return a

    # ---------------------------------------------------------------- exchange
    def _exchange_counts(self, send_counts):
        recv = torch.empty_like(send_counts)
        dist.all_to_all_single(recv, send_counts, group=self.group)
        both = torch.cat([send_counts, recv]).cpu().tolist()       # the host needs the split sizes
        return both[:self.world], both[self.world:]

    def _exchange(self, out, inp, out_splits, in_splits):
        if out.dtype == BF16:          # moved as bytes: every backend carries uint8
            out, inp = out.view(torch.uint8), inp.view(torch.uint8)
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    # ---------------------------------------------------------------- layer
    def forward(self, x):
        """The layer for this rank's tokens ``x`` ``[T, H]`` (every rank calls it, with its
        own T; T may be 0).  Returns bf16 ``[T, H]``."""
        x = x.reshape(-1, self.H)
        if x.dtype != BF16:
            x = x.to(BF16)
        x = x.contiguous()
        if self.transport == "p2p":
            return self._forward_p2p(x)
        T, H = x.shape
        dev = x.device
        logits, w, idx, wf = self.route(x)
        order_d, inverse_d, send_counts = self.dispatch_layout(idx)
        if self.world == 1:
            n = idx.numel()
            act = torch.empty(n + T, H, dtype=BF16, device=dev)
            _, recv_e = self.gather_rows(x, order_d, self.k, n, ids=idx.reshape(-1), mod=self.E_local, out=act[:n])
            act[n:].copy_(x)
            yd, inverse = self.local_experts(act, recv_e, n)
            yb = self.unpack(yd, inverse, n)
            self.last_counts = ([n], [n])
            return self.combine(yb, wf, inverse_d, yd[n:], logits)
        send_x, send_e = self.pack(x, idx, order_d)
        sc, rc = self._exchange_counts(send_counts)
        self.last_counts = (sc, rc)
        R = sum(rc)
        act = torch.empty(R + T, H, dtype=BF16, device=dev)
        recv_e = torch.empty(R, dtype=I64, device=dev)
        self._exchange(act[:R], send_x, rc, sc)
        self._exchange(recv_e, send_e, rc, sc)
        act[R:].copy_(x)
        yd, inverse = self.local_experts(act, recv_e, R)
        back = self.unpack(yd, inverse, R)
        yb = torch.empty(idx.numel(), H, dtype=BF16, device=dev)
        self._exchange(yb, back, sc, rc)
        return self.combine(yb, wf, inverse_d, yd[R:], logits)

    __call__ = forward

    def _forward_p2p(self, x):
        if self.overlap_shared:
            return self._forward_p2p_overlap(x)
        T, H = x.shape
        if T > self.max_tokens:
            raise ValueError(f"ExpertParallelMoE: {T} tokens exceed max_tokens={self.max_tokens}")
        ex = self._p2p
        dev = x.device
        L, st, D = _lib.lib(), _lib.stream(dev), ex.desc
        Eg, I, cap = self.E_local, self.I, ex.cap
        logits, w, idx, wf = self.route(x)
        order_d, inverse_d, counts = self.dispatch_layout(idx)
        tok_index = torch.empty(max(idx.numel(), 1), dtype=torch.int32, device=dev)
        tcounts = torch.empty(self.world, dtype=I64, device=dev)
        self.last_counts = (counts, tcounts)
        _lib.check(L.fnx_ep_p2p_dedup(D, order_d.data_ptr(), counts.data_ptr(), T, tok_index.data_ptr(),
                                      tcounts.data_ptr(), st), "EP token dedup")
        _lib.check(L.fnx_ep_p2p_counts(D, counts.data_ptr(), tcounts.data_ptr(), st), "EP count exchange")
        _lib.check(L.fnx_ep_p2p_push(D, x.data_ptr(), T, order_d.data_ptr(), idx.data_ptr(), tok_index.data_ptr(), st),
                   "EP dispatch")
        _lib.check(L.fnx_ep_p2p_wait(D, 1, st), "EP dispatch wait")
        M = T + cap
        order_x = torch.empty(M, dtype=I64, device=dev)
        ends_x = torch.empty(Eg + 1, dtype=I64, device=dev)
        pos = torch.empty(cap, dtype=I64, device=dev)
        rows = torch.empty(M, dtype=I64, device=dev)              # down-row destinations (pointers)
        sh = torch.empty(max(T, 1), H, dtype=BF16, device=dev)
        wsb = L.fnx_ep_p2p_recv_workspace(D)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        _lib.check(L.fnx_ep_p2p_recv_layout(D, T, order_x.data_ptr(), ends_x.data_ptr(), pos.data_ptr(),
                                            rows.data_ptr(), sh.data_ptr(), ws.data_ptr(), wsb, st), "EP receive layout")
        a2 = torch.empty(M, I, dtype=BF16, device=dev)
        _lib.check(L.fnx_moe_grouped_w4(ex.recv_x, H, ex.cap_tok + self.max_tokens, order_x.data_ptr(), 1,
                                        self.gu_loc.data_ptr(), ends_x.data_ptr(), a2.data_ptr(), I, Eg + 1, M, H,
                                        2 * I, EPI_SWIGLU_SHARED_FIRST, st), "grouped W4A16 GEMM")
        _lib.check(L.fnx_moe_grouped_w4_rows(a2.data_ptr(), I, M, None, 1, self.dn_loc.data_ptr(), ends_x.data_ptr(),
                                             rows.data_ptr(), Eg + 1, M, I, H, st), "grouped W4A16 GEMM (return)")
        _lib.check(L.fnx_ep_p2p_signal(D, 2, st), "EP return signal")
        _lib.check(L.fnx_ep_p2p_wait(D, 2, st), "EP return wait")
        out = torch.empty(T, H, dtype=BF16, device=dev)
        gate = logits[:, self.E:self.E + 1]
        _lib.check(L.fnx_moe_combine(ex.yb, wf.data_ptr(), inverse_d.data_ptr(), sh.data_ptr(), gate.data_ptr(),
                                     logits.stride(0), out.data_ptr(), T, self.k, H, st), "MoE combine")
        return out

    def _forward_p2p_overlap(self, x):
        """The p2p call with the shared expert on a second stream: its gate/up and down run from x
        on all but `reserve_sms` SMs while this stream lays out, deduplicates, exchanges counts
        and pushes the token rows (on the reserved SMs) and lays out what it received; the routed
        experts then run over the received slots alone and the streams join before the combine.
        Every row meets the same kernels and operands as in the single-stream form, so the output
        is the same bit for bit."""
        T, H = x.shape
        if T > self.max_tokens:
            raise ValueError(f"ExpertParallelMoE: {T} tokens exceed max_tokens={self.max_tokens}")
        ex = self._p2p
        dev = x.device
        L, D = _lib.lib(), ex.desc
        Eg, I, cap = self.E_local, self.I, ex.cap
        main = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = torch.cuda.Stream(dev)
        side = self._side
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        reserve = max(2, min(self.reserve_sms, sms - 2))
        side_ctas = (sms - reserve) // 2 * 2
        sh_ends = self._sh_ends.get((T, str(dev)))
        if sh_ends is None:
            sh_ends = self._sh_ends[(T, str(dev))] = torch.full((1,), T, dtype=I64, device=dev)
        x = x.contiguous()
        logits, w, idx, wf = self.route(x)
        # buffers of both streams, allocated here (on this stream) before the fork
        a_sh = torch.empty(max(T, 1), I, dtype=BF16, device=dev)
        sh = torch.empty(max(T, 1), H, dtype=BF16, device=dev)
        order_r = torch.empty(max(cap, 1), dtype=I64, device=dev)
        ends_r = torch.empty(Eg, dtype=I64, device=dev)
        pos = torch.empty(max(cap, 1), dtype=I64, device=dev)
        rows = torch.empty(max(cap, 1), dtype=I64, device=dev)
        wsb = L.fnx_ep_p2p_recv_workspace(D)
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        a2 = torch.empty(max(cap, 1), I, dtype=BF16, device=dev)
        out = torch.empty(T, H, dtype=BF16, device=dev)
        side.wait_stream(main)
        if T:
            ss = side.cuda_stream
            with torch.cuda.stream(side):
                _lib.check(L.fnx_moe_grouped_w4_lim(x.data_ptr(), H, T, None, 1, self.gu_loc.data_ptr(),
                                                    sh_ends.data_ptr(), a_sh.data_ptr(), I, 1, T, H, 2 * I,
                                                    EPI_SWIGLU_BF16, side_ctas, ss), "shared expert gate/up")
                _lib.check(L.fnx_moe_grouped_w4_lim(a_sh.data_ptr(), I, T, None, 1, self.dn_loc.data_ptr(),
                                                    sh_ends.data_ptr(), sh.data_ptr(), H, 1, T, I, H, EPI_PLAIN,
                                                    side_ctas, ss), "shared expert down")
        st = _lib.stream(dev)
        order_d, inverse_d, counts = self.dispatch_layout(idx)
        tok_index = torch.empty(max(idx.numel(), 1), dtype=torch.int32, device=dev)
        tcounts = torch.empty(self.world, dtype=I64, device=dev)
        self.last_counts = (counts, tcounts)
        _lib.check(L.fnx_ep_p2p_dedup(D, order_d.data_ptr(), counts.data_ptr(), T, tok_index.data_ptr(),
                                      tcounts.data_ptr(), st), "EP token dedup")
        _lib.check(L.fnx_ep_p2p_counts(D, counts.data_ptr(), tcounts.data_ptr(), st), "EP count exchange")
        _lib.check(L.fnx_ep_p2p_push_ex(D, x.data_ptr(), T, order_d.data_ptr(), idx.data_ptr(), tok_index.data_ptr(),
                                        1, 4 * reserve, st), "EP dispatch")
        _lib.check(L.fnx_ep_p2p_wait(D, 1, st), "EP dispatch wait")
        _lib.check(L.fnx_ep_p2p_recv_layout_routed(D, order_r.data_ptr(), ends_r.data_ptr(), pos.data_ptr(),
                                                   rows.data_ptr(), ws.data_ptr(), wsb, st), "EP receive layout")
        one = self.gu_loc[0].numel() * self.gu_loc.element_size()
        one_d = self.dn_loc[0].numel() * self.dn_loc.element_size()
        if cap:
            _lib.check(L.fnx_moe_grouped_w4(ex.recv_x, H, ex.cap_tok + self.max_tokens, order_r.data_ptr(), 1,
                                            self.gu_loc.data_ptr() + one, ends_r.data_ptr(), a2.data_ptr(), I, Eg, cap,
                                            H, 2 * I, EPI_SWIGLU_F32, st), "grouped W4A16 GEMM")
            _lib.check(L.fnx_moe_grouped_w4_rows(a2.data_ptr(), I, cap, None, 1, self.dn_loc.data_ptr() + one_d,
                                                 ends_r.data_ptr(), rows.data_ptr(), Eg, cap, I, H, st),
                       "grouped W4A16 GEMM (return)")
        _lib.check(L.fnx_ep_p2p_signal(D, 2, st), "EP return signal")
        _lib.check(L.fnx_ep_p2p_wait(D, 2, st), "EP return wait")
        main.wait_stream(side)
        gate = logits[:, self.E:self.E + 1]
        _lib.check(L.fnx_moe_combine(ex.yb, wf.data_ptr(), inverse_d.data_ptr(), sh.data_ptr(), gate.data_ptr(),
                                     logits.stride(0), out.data_ptr(), T, self.k, H, st), "MoE combine")
        return out

    def exchange_stats(self):
        """Rows this rank moved in its last call (synchronises): ``dispatch_rows`` token rows
        sent to other ranks, ``return_rows`` slot rows that came back from other ranks,
        ``received_slots`` slots this rank's experts processed."""
        if self.last_counts is None:
            return None
        r = self.rank
        if self.transport == "p2p":
            sc, tc = (t.cpu().tolist() for t in self.last_counts)
            return dict(dispatch_rows=sum(tc) - tc[r], return_rows=sum(sc) - sc[r],
                        received_slots=int(_lib.lib().fnx_ep_p2p_received(self._p2p.desc)))
        sc, rc = self.last_counts
        return dict(dispatch_rows=sum(sc) - sc[r], return_rows=sum(sc) - sc[r], received_slots=sum(rc))

    # ---------------------------------------------------------------- one-process emulation
    @staticmethod
    def emulate(shards, xs):
        """Run ``world`` shards (one per rank, in rank order, ``transport="collective"``) on the
        tokens ``xs`` in this process, moving the exchanged rows with copies in place of the
        all-to-all.  Checks the dispatch, expert and combine stages of a multi-rank layer on
        one device."""
        G = len(shards)
        st = []
        for s, x in zip(shards, xs):
            x = x.reshape(-1, s.H).to(BF16).contiguous()
            logits, w, idx, wf = s.route(x)
            order_d, inverse_d, counts = s.dispatch_layout(idx)
            send_x, send_e = s.pack(x, idx, order_d)
            st.append(dict(x=x, logits=logits, wf=wf, inverse_d=inverse_d, counts=counts.cpu().tolist(),
                           send_x=send_x, send_e=send_e))
        outs = [None] * G
        backs = []
        for d, s in enumerate(shards):
            rows, ids = [], []
            for src in st:
                off = sum(src["counts"][:d])
                rows.append(src["send_x"][off:off + src["counts"][d]])
                ids.append(src["send_e"][off:off + src["counts"][d]])
            R = sum(r.shape[0] for r in rows)
            act = torch.cat(rows + [st[d]["x"]])
            yd, inverse = s.local_experts(act, torch.cat(ids), R)
            back = s.unpack(yd, inverse, R)
            st[d]["sh"] = yd[R:]
            backs.append(back)
        for r, s in enumerate(shards):
            parts = []
            for d in range(G):
                off = sum(st[q]["counts"][d] for q in range(r))
                parts.append(backs[d][off:off + st[r]["counts"][d]])
            yb = torch.cat(parts)
            outs[r] = s.combine(yb, st[r]["wf"], st[r]["inverse_d"], st[r]["sh"], st[r]["logits"])
        return outs
