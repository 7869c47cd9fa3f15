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
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .engine import BF16, EPI_PLAIN, EPI_SWIGLU_MIXED, MoELayer, _grouped_w4, repack_w4

I64 = torch.int64


class ExpertParallelMoE(MoELayer):
    """One MoE layer whose routed experts are sharded over ``world`` ranks.

    ``gu_w4 / gu_scales / dn_w4 / dn_scales`` hold this rank's experts only (expert-major
    int4pack and bf16 group scales of experts ``[rank*E/world, (rank+1)*E/world)``);
    ``gate_w`` is the full router ``[E, H]``; the shared expert is replicated.  ``group``
    is the process group of the ``world`` ranks (``None``: the default group; unused when
    ``world == 1``)."""

    def __init__(self, gu_w4, gu_scales, dn_w4, dn_scales, gate_w, sh_gu_w4, sh_gu_scales, sh_dn_w4, sh_dn_scales,
                 sh_gate, k, gs, *, rank=0, world=1, group=None, bias=None):
        _lib.require_cuda(gu_w4, dn_w4, gate_w, sh_gu_w4, sh_dn_w4)
        self._init_router(gate_w, sh_gate, k, gs, bias)
        self._init_shard(rank, world, group, gu_w4.shape[0])
        self.I = gu_w4.shape[2] * 8 // 2
        self.gu_loc = repack_w4(torch.cat([gu_w4, sh_gu_w4[None]]), torch.cat([gu_scales, sh_gu_scales[None]]),
                                swiglu=True)
        self.dn_loc = repack_w4(torch.cat([dn_w4, sh_dn_w4[None]]), torch.cat([dn_scales, sh_dn_scales[None]]),
                                swiglu=False)

    def _init_shard(self, rank, world, group, e_local):
        if world < 1 or not 0 <= rank < world or self.E % world or e_local != self.E // world:
            raise ValueError(f"ExpertParallelMoE: {e_local} local experts of E={self.E} on rank {rank} of {world}")
        self.rank, self.world, self.group = rank, world, group
        self.E_local = e_local
        self.last_counts = None

    @classmethod
    def from_layer(cls, layer: MoELayer, rank, world, group=None):
        """This rank's shard of a one-device ``MoELayer`` (its tile blocks are copied, so the
        full layer may be dropped afterwards)."""
        o = cls.__new__(cls)
        o.E, o.H, o.I, o.k, o.gs = layer.E, layer.H, layer.I, layer.k, layer.gs
        o.R, o.R_pad, o.router_cat, o.bias = layer.R, layer.R_pad, layer.router_cat, layer.bias
        o._ws, o._prefill_bufs = {}, {}
        o._init_shard(rank, world, group, layer.E // world if layer.E % world == 0 else -1)
        lo, hi = rank * o.E_local, (rank + 1) * o.E_local
        o.gu_loc = torch.cat([layer.gu_all[lo:hi], layer.gu_all[layer.E:]]).contiguous()
        o.dn_loc = torch.cat([layer.dn_all[lo:hi], layer.dn_all[layer.E:]]).contiguous()
        return o

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
        """Step 4: ``act`` holds the ``R`` received rows followed by the rank's own ``T``
        tokens; returns the down rows ``[R+T, H]`` (the received slots expert-major, then
        the shared expert's rows) and the received slots' rows in it (``inverse``)."""
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

    # ---------------------------------------------------------------- one-process emulation
    @staticmethod
    def emulate(shards, xs):
        """Run ``world`` shards (one per rank, in rank order) on the tokens ``xs`` in this
        process, moving the exchanged rows with copies in place of the all-to-all.  Checks the
        dispatch, expert and combine stages of a multi-rank layer on one device."""
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
