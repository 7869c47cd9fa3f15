"""Expert-parallel layer (``fnx/ep.py``) on CPU ranks over ``gloo``.

The exchange logic -- owner-major dispatch order, per-owner counts, the all-to-all-v of
rows and owner-local expert ids, the owner's expert-major sort, the return of the down rows
in received order and the slot-order combine through the dispatch inverse -- runs unchanged
in ``ExpertParallelMoE.forward``; only the per-rank compute stages are replaced by the CPU
oracle (``CpuShard`` below, test infrastructure).  A G-rank run must give, bit for bit, the
one-rank output over the same tokens, because each slot's expert row is computed from the
same operands and the combine reduces in the same slot order.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from fnx import synth
from fnx.ep import ExpertParallelMoE

BF16 = torch.bfloat16
SHAPE = dict(H=256, I=128, E=8, k=3, gs=128)


class CpuShard(ExpertParallelMoE):
    """The compute stages of one rank on the CPU oracle (fp64 accumulation, so a row's
    result does not depend on which other rows share its GEMM)."""

    def __init__(self, L, k, rank, world, group=None):
        self.E, self.H, self.I, self.k, self.gs = L.E, L.H, L.I, k, L.gs
        self._prefill_bufs = {}
        self._init_shard(rank, world, group, L.E // world)
        self.L = L
        self.W = torch.cat([L.t["gate_w"], L.t["sh_gate"]]).to(BF16)      # router rows + shared gate

    def route(self, x):
        logits = (x.double() @ self.W.double().t()).float().to(BF16)
        w, idx, _ = O.route(logits[:, :self.E], self.k)
        return logits, w, idx, w.float()

    def dispatch_layout(self, idx):
        ids = idx.reshape(-1)
        dest = ids // self.E_local
        order = torch.sort(dest, stable=True).indices
        inverse = torch.empty_like(order)
        inverse[order] = torch.arange(order.numel())
        return order, inverse, torch.bincount(dest, minlength=self.world).to(torch.int64)

    def gather_rows(self, src, index, div, n, ids=None, mod=1, out=None):
        rows = src[index // div] if index is not None else src[:n]
        if out is not None:
            out.copy_(rows)
            rows = out
        return rows, (ids[index] % mod if ids is not None else None)

    def local_experts(self, act, recv_e, R):
        L, lo = self.L, self.rank * self.E_local
        order = torch.sort(recv_e, stable=True).indices
        inverse = torch.empty_like(order)
        inverse[order] = torch.arange(R)
        ends = torch.bincount(recv_e, minlength=self.E_local).cumsum(0)
        rows = act[:R][order]
        gu = O.grouped_matmul(rows, ends, lambda e: L.gu(lo + e))
        yd = O.grouped_matmul(O.swiglu_fp32(gu, self.I), ends, lambda e: L.dn(lo + e))
        xs = act[R:]
        sh = O.w4a16_matmul(O.swiglu_shared(O.w4a16_matmul(xs, L.sh_gu), self.I), L.sh_dn)
        return torch.cat([yd, sh]), inverse

    def combine(self, yb, wf, inverse_d, sh, logits):
        y = O.weighted_reduce(yb, wf.to(BF16), inverse=inverse_d)
        return O.moe_merge(y, sh, logits[:, self.E:self.E + 1])


def _layer():
    shape = synth.MoEShape(**SHAPE)
    return O.Layer(synth.make_layer(shape, seed=7), shape.gs)


def _tokens(Ts):
    return [synth.make_tokens(T, SHAPE["H"], seed=100 + r) for r, T in enumerate(Ts)]


def _worker(rank, world, port, Ts, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        torch.set_num_threads(1)
        layer = CpuShard(_layer(), SHAPE["k"], rank, world)
        out = layer(_tokens(Ts)[rank])
        q.put((rank, out.view(torch.int16).numpy().copy(), layer.last_counts))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(Ts):
    world = len(Ts)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, Ts, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out, counts = q.get(timeout=240)
            res[r] = (out, counts)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return [res[r] for r in range(world)]


@pytest.mark.parametrize("Ts", [(12, 7), (5, 0, 9, 3)], ids=["world2", "world4-empty-rank"])
def test_ep_gloo_matches_one_rank(Ts):
    world = len(Ts)
    res = _run(Ts)
    L = _layer()
    one = CpuShard(L, SHAPE["k"], 0, 1)
    x_all = torch.cat(_tokens(Ts))
    ref = one(x_all)
    got = np.concatenate([o for o, _ in res])
    assert np.array_equal(got, ref.view(torch.int16).numpy())
    # the exchanged counts: what rank r sends to d is what d receives from r, and every
    # rank sends T*k slots in all
    for r, (_, (sc, rc)) in enumerate(res):
        assert sum(sc) == Ts[r] * SHAPE["k"]
        for d in range(world):
            assert sc[d] == res[d][1][1][r]
    # the one-rank layer itself is the oracle's MoE layer (same routing)
    logits, w, idx, _ = one.route(x_all)
    ref2 = O.moe_forward(x_all, L, SHAPE["k"], routing=(w, idx))
    assert O.within_tolerance(ref, ref2)


def test_balanced_expert_order():
    """Equal blocks per rank, every expert once, and the heaviest block within one expert of the
    mean (LPT bound); a uniform load stays uniform."""
    from fnx.ep import balanced_expert_order
    g = torch.Generator().manual_seed(3)
    for E, G in ((512, 8), (64, 4), (8, 2)):
        ranks = torch.randperm(E, generator=g)
        counts = 1.0 / (1.0 + ranks.double()) ** 1.1 * 1e5            # Zipf-like over a random ranking
        order = balanced_expert_order(counts, G)
        assert sorted(order.tolist()) == list(range(E))
        loads = counts[order].view(G, E // G).sum(1)
        assert float(loads.max()) <= float(loads.mean()) + float(counts.max()) + 1e-6
        contiguous = counts.view(G, E // G).sum(1)
        assert float(loads.max()) <= float(contiguous.max()) + 1e-6
    order = balanced_expert_order(torch.ones(16), 4)
    assert sorted(order.tolist()) == list(range(16))
    with pytest.raises(ValueError):
        balanced_expert_order(torch.ones(10), 4)
