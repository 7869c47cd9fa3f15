"""Expert-parallel layer on the GPU: the dispatch-layout and row-gather kernels bit-exact
against torch index arithmetic, a G-rank layer emulated in one process (exchange by copies)
bit-identical to the one-GPU layer on every rank's tokens, and -- with two or more GPUs --
the NCCL all-to-all path."""
import os
import socket
from datetime import timedelta

import pytest
import torch

from fnx import _lib, synth
from fnx.engine import MoELayer
from fnx.ep import ExpertParallelMoE

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _errors():
    _lib.lib()
    _lib.device_errors()
    yield
    assert _lib.device_errors() == 0


def _layout(idx, E, G):
    n = idx.numel()
    order = torch.empty(n, dtype=torch.int64, device=DEV)
    inverse = torch.empty(n, dtype=torch.int64, device=DEV)
    counts = torch.empty(G, dtype=torch.int64, device=DEV)
    L = _lib.lib()
    wsb = L.fnx_ep_layout_workspace(n, G)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    rc = L.fnx_ep_dispatch_layout(idx.data_ptr(), n, E, G, order.data_ptr(), inverse.data_ptr(), counts.data_ptr(),
                                  ws.data_ptr(), wsb, _lib.stream(idx.device))
    return rc, order, inverse, counts


@pytest.mark.parametrize("T,k,E,G", [(4096, 10, 512, 1), (4096, 10, 512, 2), (4096, 10, 512, 8), (333, 6, 64, 4),
                                     (1, 10, 512, 8), (0, 10, 512, 4)])
def test_dispatch_layout(T, k, E, G):
    g = torch.Generator().manual_seed(T + G)
    idx = torch.randint(0, E, (T, k), generator=g)
    rc, order, inverse, counts = _layout(idx.to(DEV), E, G)
    assert rc == 0
    dest = (idx // (E // G)).reshape(-1)
    ref_order = torch.sort(dest, stable=True).indices
    assert torch.equal(order.cpu(), ref_order)
    assert torch.equal(inverse.cpu()[ref_order], torch.arange(T * k))
    assert torch.equal(counts.cpu(), torch.bincount(dest, minlength=G))


def test_dispatch_layout_rejects():
    idx = torch.zeros(8, dtype=torch.int64, device=DEV)
    assert _layout(idx, 10, 4)[0] != 0          # E % G != 0
    assert _layout(idx, 4, 8)[0] != 0           # more ranks than experts


@pytest.mark.parametrize("n,H,div,src_rows", [(5000, 2048, 10, 900), (77, 100, 1, 50), (0, 2048, 1, 4)])
def test_gather_rows(n, H, div, src_rows):
    g = torch.Generator().manual_seed(n + H)
    src = torch.randn(src_rows, H, generator=g).to(BF16).to(DEV)
    index = torch.randint(0, src_rows * div, (n,), generator=g).to(DEV)
    ids = torch.randint(0, 512, (src_rows * div,), generator=g).to(DEV)
    out = torch.full((n, H), float("nan"), dtype=BF16, device=DEV)
    ids_out = torch.empty(n, dtype=torch.int64, device=DEV)
    rc = _lib.lib().fnx_ep_gather_rows(src.data_ptr(), H, src_rows, index.data_ptr(), div, ids.data_ptr(), 64,
                                       out.data_ptr(), H, ids_out.data_ptr(), n, H, _lib.stream(src.device))
    assert rc == 0
    assert torch.equal(out.view(torch.int16), src[index // div].view(torch.int16))
    assert torch.equal(ids_out, ids[index] % 64)


def test_gather_rows_bad_index_flags():
    src = torch.ones(4, 256, dtype=BF16, device=DEV)
    index = torch.tensor([0, 9, 3], dtype=torch.int64, device=DEV)
    out = torch.full((3, 256), 7.0, dtype=BF16, device=DEV)
    _lib.device_errors()
    rc = _lib.lib().fnx_ep_gather_rows(src.data_ptr(), 256, 4, index.data_ptr(), 1, None, 1, out.data_ptr(), 256,
                                       None, 3, 256, _lib.stream(src.device))
    assert rc == 0
    assert _lib.device_errors() & 2
    assert bool((out[1] == 0).all()) and bool((out[0] == 1).all())


@pytest.fixture(scope="module")
def cfg2_layer():
    t = synth.make_layer(synth.CFG2, seed=21, device=DEV)
    return t, MoELayer.from_synth(t, synth.CFG2)


@pytest.mark.parametrize("G,T", [(1, 200), (2, 300), (4, 128), (8, 64)])
def test_ep_emulated_bit_identical(cfg2_layer, G, T):
    _, layer = cfg2_layer
    shards = [ExpertParallelMoE.from_layer(layer, r, G, transport="collective") for r in range(G)]
    xs = [synth.make_tokens(T + 3 * r, synth.CFG2.H, seed=500 + r, device=DEV) for r in range(G)]
    outs = ExpertParallelMoE.emulate(shards, xs)
    for r in range(G):
        ref = layer.prefill(xs[r])
        assert torch.equal(outs[r].view(torch.int16), ref.view(torch.int16)), r


@pytest.mark.parametrize("transport,overlap", [("p2p", True), ("p2p", False), ("collective", True)])
def test_ep_single_rank_forward(cfg2_layer, transport, overlap):
    """Bit-identical to the one-GPU layer; p2p with the shared expert on a second stream (overlap)
    and in the single-stream form."""
    _, layer = cfg2_layer
    ep = ExpertParallelMoE.from_layer(layer, 0, 1, transport=transport, max_tokens=1024)
    ep.overlap_shared = overlap
    assert ep.transport == transport
    for T, seed in ((777, 9), (1024, 10), (17, 11), (777, 9)):
        x = synth.make_tokens(T, synth.CFG2.H, seed=seed, device=DEV)
        assert torch.equal(ep(x).view(torch.int16), layer.prefill(x).view(torch.int16)), T
    with pytest.raises(ValueError):
        if transport == "p2p":
            ep(synth.make_tokens(1025, synth.CFG2.H, seed=1, device=DEV))
        else:
            raise ValueError
    ep.close()


@pytest.mark.parametrize("overlap", [True, False])
def test_ep_p2p_graph_capture(cfg2_layer, overlap):
    """The p2p layer never waits on the host, so one call captures into a CUDA graph (with the
    shared expert's second stream forked and joined inside the capture)."""
    _, layer = cfg2_layer
    ep = ExpertParallelMoE.from_layer(layer, 0, 1, transport="p2p", max_tokens=512)
    ep.overlap_shared = overlap
    x = synth.make_tokens(512, synth.CFG2.H, seed=12, device=DEV)
    ref = layer.prefill(x)
    ep(x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ep(x)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    del g
    ep.close()


def test_ep_p2p_wait_times_out():
    """A peer that never arrives: the bounded wait gives up, records device error 1, and the
    context stays usable (the flag that nothing sets is this step's return flag)."""
    import ctypes
    from fnx.ep import _PeerExchange
    ex = _PeerExchange(0, 1, None, 256, 2, 16, 4, torch.device(DEV))
    L = _lib.lib()
    st = _lib.stream(torch.device(DEV))
    counts = torch.tensor([0], dtype=torch.int64, device=DEV)
    _lib.device_errors()
    assert L.fnx_ep_p2p_counts(ex.desc, counts.data_ptr(), counts.data_ptr(), st) == 0
    assert L.fnx_ep_p2p_wait(ex.desc, 2, st) == 0            # nothing signals RET of this epoch
    torch.cuda.synchronize()
    assert _lib.device_errors() & 1
    assert L.fnx_ep_p2p_wait(ex.desc, 0, st) == 0            # CNT of this epoch was signalled
    torch.cuda.synchronize()
    assert _lib.device_errors() == 0
    assert L.fnx_ep_p2p_received(ex.desc) == 0
    ex.close()


def test_ep_constructor_matches_shard(cfg2_layer):
    t, layer = cfg2_layer
    G, r = 4, 2
    Eg = synth.CFG2.E // G
    sl = slice(r * Eg, (r + 1) * Eg)
    ep = ExpertParallelMoE(t["gu_w4"][sl], t["gu_scales"][sl], t["dn_w4"][sl], t["dn_scales"][sl], t["gate_w"],
                           t["sh_gu_w4"], t["sh_gu_scales"], t["sh_dn_w4"], t["sh_dn_scales"], t["sh_gate"],
                           synth.CFG2.k, synth.CFG2.gs, rank=r, world=G)
    ref = ExpertParallelMoE.from_layer(layer, r, G)
    assert torch.equal(ep.gu_loc, ref.gu_loc) and torch.equal(ep.dn_loc, ref.dn_loc)
    assert torch.equal(ep.router_cat, ref.router_cat)


# ------------------------------------------------------------------ NCCL, 2+ GPUs
def _nccl_worker(rank, world, port, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        t = synth.make_layer(synth.CFG2, seed=21, device=dev)
        layer = MoELayer.from_synth(t, synth.CFG2)
        res = {}
        for transport in ("p2p", "collective"):
            ep = ExpertParallelMoE.from_layer(layer, rank, world, transport=transport, max_tokens=T + 8)
            assert ep.transport == transport
            same = True
            for i in range(3):
                x = synth.make_tokens(T + rank - 2 * i, synth.CFG2.H, seed=700 + rank + 10 * i, device=dev)
                out = ep(x)
                same = same and torch.equal(out.view(torch.int16), layer.prefill(x).view(torch.int16))
            torch.cuda.synchronize(dev)
            res[transport] = (same, ep.exchange_stats())
            ep.close()
        dist.barrier()
        q.put((rank, res, _lib.device_errors()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_nccl_bit_identical():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, 512, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, per, errs = q.get(timeout=300)
            res[r] = (per, errs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        per, errs = res[r]
        assert errs == 0, (r, errs)
        for transport, (same, stats) in per.items():
            assert same, (r, transport)
        # both transports returned the same slot rows and processed the same slots; the p2p
        # dispatch sends each token once per owner, so never more rows than the collective
        p, c = per["p2p"][1], per["collective"][1]
        assert p["return_rows"] == c["return_rows"] and p["received_slots"] == c["received_slots"], (r, per)
        assert p["dispatch_rows"] <= c["dispatch_rows"], (r, per)
