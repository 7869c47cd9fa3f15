"""GPU parity of the byte/rounding-exact kernels against the oracle and the reference
goldens, called through the C ABI (drop-in modules)."""
import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda"


def bits_equal(a, b):
    return a.shape == b.shape and torch.equal(a.cpu().view(torch.int16), b.cpu().view(torch.int16))


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from fnx import _lib
    _lib.lib()
    _lib.device_errors()
    yield
    assert _lib.device_errors() == 0


def test_weighted_reduce_goldens(golden):
    from fnx.weighted_reduce import reduce
    cases = golden("reduce_cases")
    c = cases["adversarial"]
    got = reduce(c["values"].to(DEV).view(-1, c["values"].shape[-1]), c["weights"].to(DEV))
    assert bits_equal(got, c["expected"])
    for B in (1, 3, 9):
        c = cases[f"inverse{B}"]
        got = reduce(c["values"].to(DEV), c["weights"].to(DEV), inverse=c["inverse"].to(DEV))
        assert bits_equal(got, c["expected"])
    c = cases["mean4"]
    got = reduce(c["values"].to(DEV), c["weights"].to(DEV), mean=True)
    assert bits_equal(got, c["expected"])


@pytest.mark.parametrize("B,k,H", [(1, 10, 2560), (128, 10, 2048), (513, 8, 2048), (4096, 10, 2048), (7, 3, 100)])
def test_weighted_reduce_random(B, k, H):
    from fnx.weighted_reduce import reduce
    g = torch.Generator().manual_seed(B * 131 + k)
    v = (torch.randn(B * k, H, generator=g) * 10).to(BF16)
    w = torch.rand(B, k, generator=g).to(BF16)
    inv = torch.randperm(B * k, generator=g)
    got = reduce(v.to(DEV), w.to(DEV), inverse=inv.to(DEV))
    assert bits_equal(got, O.weighted_reduce(v, w, inverse=inv))
    got1 = reduce(v.to(DEV), w.to(DEV))
    assert bits_equal(got1, O.weighted_reduce(v, w))


def test_epilogue_and_merge(golden):
    from fnx import moe_epilogue, post_ops
    c = golden("reduce_cases")["epilogue"]
    got = moe_epilogue.merge(c["cartesian"].to(DEV), c["weights"].to(DEV), c["shared"].to(DEV), c["gate"].to(DEV))
    assert bits_equal(got, c["expected"])
    g = torch.Generator().manual_seed(141)
    for i in range(16):
        B, W = (1, 2560) if i % 2 else (5, 2048)
        e = (torch.randn(B, W, generator=g) * (0.01 if i % 4 else 10)).to(BF16)
        s = (torch.randn(B, W, generator=g) * 0.1).to(BF16)
        gt = (torch.randn(B, 1, generator=g) * 8).to(BF16)
        got = post_ops.moe_merge(e.to(DEV), s.to(DEV), gt.to(DEV))
        assert bits_equal(got, O.moe_merge(e, s, gt))


def test_gather_pair():
    from fnx import engine, expert_gather
    from fnx import _lib
    g = torch.Generator().manual_seed(138)
    E, K, N, G = 512, 256, 1024, 2
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K, N // 8), generator=g, dtype=torch.int64).to(torch.int32)
    s = (torch.randn(E, G, N, generator=g) * .01).to(BF16)
    proj = engine.ExpW4.from_scales(w.to(DEV), s.to(DEV), K // G)
    for step in range(8):
        ids = torch.randperm(E, generator=g)[:10] if step % 4 else torch.tensor([0, 511, 0, 123, 12, 510, 50, 100, 300, 399])
        ow, os_ = expert_gather.gather(proj, ids.to(DEV))
        rw, rs = O.gather_pair(w, s, ids)
        assert torch.equal(ow.cpu(), rw) and bits_equal(os_, rs)
    # the reference-signature export (10 slots, no range check)
    ids = torch.tensor([3, 17, 61, 200, 255, 256, 400, 401, 510, 511], device=DEV)
    ow = torch.empty(K, 10 * N // 8, dtype=torch.int32, device=DEV)
    os_ = torch.empty(G, 10 * N, dtype=BF16, device=DEV)
    rc = _lib.lib().fnx_gather_pair(proj.w4.data_ptr(), proj._scales.data_ptr(), ids.data_ptr(), ow.data_ptr(),
                                    os_.data_ptr(), K, G, N, _lib.stream(ow.device))
    assert rc == 0
    rw, rs = O.gather_pair(w, s, ids.cpu())
    assert torch.equal(ow.cpu(), rw) and bits_equal(os_, rs)


@pytest.mark.parametrize("T,E,k", [(64, 64, 8), (4096, 512, 10), (3, 16, 4), (100, 1000, 32)])
def test_router_topk_and_permute(T, E, k):
    from fnx import _lib
    g = torch.Generator().manual_seed(T + E)
    logits = torch.randn(T, E, generator=g).to(BF16)
    dl = logits.to(DEV)
    w = torch.empty(T, k, dtype=BF16, device=DEV)
    idx = torch.empty(T, k, dtype=torch.int64, device=DEV)
    wf = torch.empty(T, k, dtype=torch.float32, device=DEV)
    rc = _lib.lib().fnx_router_topk(dl.data_ptr(), E, None, w.data_ptr(), idx.data_ptr(), wf.data_ptr(), T, E, k,
                                    _lib.stream(dl.device))
    assert rc == 0
    rw, ridx, probs = O.route(logits, k)
    assert torch.equal(idx.cpu(), ridx), "routing ids must be bit-exact given the logits"
    ulp = O.bf16_ulp_diff(w.cpu(), rw)
    assert int(ulp.max()) <= 1 and float((ulp == 0).float().mean()) > 0.99
    assert torch.equal(wf.cpu(), w.cpu().float())
    # permutation
    from fnx.engine import MoELayer
    lay = MoELayer.__new__(MoELayer)
    lay.E = E
    order, inverse, ends = lay.permute(idx)
    ro, _, rends, rinv = O.permute(idx.cpu(), E)
    assert torch.equal(order.cpu(), ro) and torch.equal(ends.cpu(), rends) and torch.equal(inverse.cpu(), rinv)
    assert O.is_within_group_permutation(order.cpu(), torch.argsort(idx.cpu().reshape(-1).float()), idx.cpu().reshape(-1))


def test_invalid_routing_is_contained():
    """NaN logits still give k valid distinct ids; ids outside [0, E) are flagged and leave
    no row (inverse = -1) that a later gather could follow out of bounds."""
    from fnx import _lib
    from fnx.engine import MoELayer
    T, E, k = 6, 64, 8
    logits = torch.full((T, E), float("nan"), dtype=BF16, device=DEV)
    logits[1, 5] = 1.0
    w = torch.empty(T, k, dtype=BF16, device=DEV)
    idx = torch.empty(T, k, dtype=torch.int64, device=DEV)
    rc = _lib.lib().fnx_router_topk(logits.data_ptr(), E, None, w.data_ptr(), idx.data_ptr(), None, T, E, k,
                                    _lib.stream(logits.device))
    assert rc == 0
    ids = idx.cpu()
    assert int(ids.min()) >= 0 and int(ids.max()) < E
    assert all(len(set(r.tolist())) == k for r in ids)
    lay = MoELayer.__new__(MoELayer)
    lay.E = 8
    bad = torch.tensor([3, 9, 1, -2, 3, 7], dtype=torch.int64)
    order, inverse, ends = lay.permute(bad.to(DEV))
    torch.cuda.synchronize()
    assert _lib.device_errors() & 2
    assert int(ends[-1]) == 4 and inverse.cpu()[[1, 3]].tolist() == [-1, -1]
    # the combine skips the missing rows instead of following them
    H = 64
    yd = torch.randn(6, H, device=DEV).to(BF16)
    wf = torch.ones(2, 3, device=DEV)
    sh = torch.zeros(2, H, dtype=BF16, device=DEV)
    gate = torch.zeros(2, 1, dtype=BF16, device=DEV)
    out = torch.empty(2, H, dtype=BF16, device=DEV)
    rc = _lib.lib().fnx_moe_combine(yd.data_ptr(), wf.data_ptr(), inverse.data_ptr(), sh.data_ptr(), gate.data_ptr(), 1,
                                    out.data_ptr(), 2, 3, H, _lib.stream(yd.device))
    assert rc == 0
    torch.cuda.synchronize()
    assert _lib.device_errors() & 2
    assert bool(torch.isfinite(out.float()).all())


def test_permute_edge_cases():
    from fnx.engine import MoELayer
    lay = MoELayer.__new__(MoELayer)
    for E, ids in ((8, torch.zeros(37, dtype=torch.int64)), (8, torch.full((5,), 7, dtype=torch.int64)),
                   (512, torch.arange(2048 + 17) % 512), (4, torch.tensor([3, 0, 3, 0, 1]))):
        lay.E = E
        order, inverse, ends = lay.permute(ids.to(DEV))
        ro, _, rends, rinv = O.permute(ids, E)
        assert torch.equal(order.cpu(), ro) and torch.equal(ends.cpu(), rends) and torch.equal(inverse.cpu(), rinv)


def test_w4gemv_goldens(golden):
    from fnx.w4gemv_op import W4GemvOp
    gd = golden("w4gemv")
    op = W4GemvOp()
    p4, N, K = gd["p4"].numpy(), gd["N"], gd["K"]
    s4t = op.prepare_layer(gd["s4"].numpy())
    x = gd["x"].numpy()
    for lay, p in ((1, p4), (2, op.to_v2_layout(p4, N, K))):
        pd = torch.from_numpy(np.ascontiguousarray(p)).to(DEV)
        y = op.run(pd, s4t, x, x.shape[0], N, K, expert_ids=gd["perm"].numpy(), lay=lay).cpu().numpy()
        assert np.abs(y - gd["y_perm"].numpy()).max() < 1e-4
    assert np.array_equal(op.to_v2_layout(p4, N, K), gd["v2"].numpy())
    # moe_forward and run_layers
    ids = np.array([2, 0, 1], dtype=np.int32)
    wts = np.array([0.5, 0.25, 0.125], dtype=np.float32)
    pd = torch.from_numpy(np.ascontiguousarray(p4)).to(DEV)
    got = op.moe_forward(pd, s4t, x[0], ids, wts, N, K).cpu().numpy()
    ref = (O.w4gemv(p4, np.ascontiguousarray(np.transpose(gd["s4"].numpy(), (0, 2, 1))), np.repeat(x[:1], 3, 0),
                    ids, N, K, 1) * wts[:, None]).sum(0)
    assert np.abs(got - ref).max() < 1e-4
    v2 = torch.from_numpy(op.to_v2_layout(p4, N, K)).to(DEV)
    xs = [torch.from_numpy(x).to(DEV) for _ in range(2)]
    ys = [torch.empty(3, N, device=DEV) for _ in range(2)]
    op.run_layers([v2, v2], [s4t, s4t], xs, ys, N, K, 3, lay=2)
    ref = O.w4gemv(gd["v2"].numpy(), np.ascontiguousarray(np.transpose(gd["s4"].numpy(), (0, 2, 1))), x,
                   np.arange(3), N, K, 2)
    assert np.abs(ys[1].cpu().numpy() - ref).max() < 1e-4


@pytest.mark.parametrize("E,N,K", [(3, 24, 384), (2, 1024, 2048)])
def test_repack_v2o_bit_exact(E, N, K):
    """fnx_repack_v2o (K-major and expert-major) equals the oracle's restatement of
    tools/repack_w4a16.py byte for byte."""
    from fnx.engine import repack_v2o
    rng = np.random.Generator(np.random.PCG64(E * N + K))
    v2o = rng.integers(0, 256, size=(E, N, K // 2), dtype=np.uint8)
    ref = O.repack_v2o(v2o, K)
    vd = torch.from_numpy(v2o).to(DEV)
    assert torch.equal(repack_v2o(vd, K).cpu(), ref)
    assert torch.equal(repack_v2o(vd, K, expert_major=True).cpu(), ref.permute(1, 0, 2).contiguous())


def test_expw4_from_lqp():
    """ExpW4.from_lqp: the LQP artifact through the GPU repack and the grouped GEMM matches the
    oracle's dequant matmul of the same values."""
    from fnx.engine import ExpW4
    E, N, K, gs = 2, 256, 256, 64
    rng = np.random.Generator(np.random.PCG64(3))
    v2o = rng.integers(0, 256, size=(E, N, K // 2), dtype=np.uint8)
    s8 = rng.integers(1, 127, size=(E, N, K // gs), dtype=np.int8)
    base = (np.abs(rng.standard_normal((E, N))) * 1e-3).astype(np.float16)
    w = ExpW4.from_lqp(torch.from_numpy(v2o).to(DEV), torch.from_numpy(s8).to(DEV), torch.from_numpy(base).to(DEV), gs)
    x = torch.randn(5, K, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    ends = torch.tensor([3, 5], dtype=torch.int64)
    got = w.apply_grouped(x.to(DEV), ends.to(DEV)).cpu()
    q = torch.from_numpy(O.unpack_v2o(v2o, K)).to(torch.int8).transpose(1, 2)        # [E, K, N]
    scales = (torch.from_numpy(s8).permute(0, 2, 1).to(torch.bfloat16)
              * torch.from_numpy(base).to(torch.bfloat16)[:, None, :])           # [E, G, N]
    ref = O.grouped_matmul(x, ends, lambda e: O.deq_w4(q[e], scales[e], gs))
    assert O.within_tolerance(got, ref), O.tolerance_report(got, ref)


@pytest.mark.parametrize("gs", [64, 128])
def test_expq_from_packed_golden(golden, gs):
    """ExpQ.from_packed + matmul (the reference's ``ExpQ`` surface) on the reference's own
    fixture: within tolerance of the reference's three-rounding torch result, and close to
    the oracle's once-rounded specification; the value constructor gives the same bits."""
    from fnx.engine import ExpQ
    g = golden("expq_packed")
    c, idx = g["cases"][f"g{gs}"], g["idx"]
    q = ExpQ.from_packed(c["v2o"], c["s8"], c["base"], DEV)
    assert (q.K, q.N, q.gs) == (g["K"], g["N"], gs)
    got = q.matmul(c["xb"].to(DEV), idx).cpu()
    r = O.tolerance_report(got, c["y"])
    assert r["rel_l2"] < 5e-3 and r["max_abs_norm"] < 2e-2, r
    spec = O.expq_matmul(c["xb"], c["v2o"], c["s8"], c["base"], idx)
    r = O.tolerance_report(got, spec)
    assert r["rel_l2"] < 1e-3 and r["exact_fraction"] > 0.9, r
    vals = torch.from_numpy(O.unpack_v2o(c["v2o"].numpy(), g["K"])).to(torch.int8)
    q2 = ExpQ(vals.to(DEV), c["s8"].to(DEV), gs, base=c["base"].to(DEV))
    assert bits_equal(q2.matmul(c["xb"].to(DEV), idx.to(DEV)), got)
    assert q.to_host_offload() is False


def _ordered(t):
    b = t.contiguous().view(torch.int16).to(torch.int32)
    return torch.where(b < 0, -(b & 0x7FFF), b)          # bf16 bit patterns in value order (+0 == -0)


def _ulp_ok(got, ref, min_exact=0.99):
    d = (_ordered(got) - _ordered(ref)).abs()
    return int(d.max()) <= 1 and float((d == 0).float().mean()) >= min_exact


@pytest.mark.parametrize("b,H,HC,LR", [(3, 2560, 4, 320), (5, 256, 4, 32), (2, 512, 3, 64)])
def test_hyper_connection_kernels(b, H, HC, LR):
    """rms_norm (its own sum order: within 1 bf16 ulp), the activation and the branch mix
    (CUDA expf: within 1 ulp) against the oracle's torch path on the same inputs."""
    from fnx import _lib as fl, post_ops
    g = torch.Generator().manual_seed(b * H + HC)
    h = torch.randn(b, HC * H, generator=g).to(torch.bfloat16)
    w = (0.1 * torch.randn(HC * H, generator=g)).to(torch.bfloat16)
    hn = torch.empty(b, HC * H, dtype=torch.bfloat16, device=DEV)
    hd, wd = h.to(DEV), w.to(DEV)                       # alive until the kernel has read them
    rc = fl.lib().fnx_hc_rms_norm(hd.data_ptr(), wd.data_ptr(), hn.data_ptr(), b, H, HC, 1e-6, fl.stream(hn.device))
    torch.cuda.synchronize()
    assert rc == 0
    assert _ulp_ok(hn.cpu(), O.hc_rms_norm(h, w, H))
    di = (3 * torch.randn(b, 1, LR + HC, generator=g)).to(torch.bfloat16)
    mix, inj = post_ops.activate(di.to(DEV), HC)
    rmix, rinj = O.hc_activation(di, HC)
    assert _ulp_ok(mix.cpu(), rmix, 0.97) and _ulp_ok(inj.cpu(), rinj, 0.5)
    logits = (2 * torch.randn(b, 1, HC * H, generator=g)).to(torch.bfloat16)
    vals = torch.randn(b, 1, HC * H, generator=g).to(torch.bfloat16)
    mixed = post_ops.mix_reduce(vals.to(DEV), logits.to(DEV), HC)
    assert _ulp_ok(mixed.cpu(), O.hc_mix_reduce(vals, logits, HC), 0.97)


def test_hyper_connection_reference_shims():
    """fnx_hc_activation / fnx_hc_sigmoid_reduce with the reference shims' fixed shapes."""
    from fnx import _lib as fl, post_ops
    g = torch.Generator().manual_seed(8)
    di = (3 * torch.randn(2, 324, generator=g)).to(torch.bfloat16).to(DEV)
    m = torch.empty(2, 320, dtype=torch.bfloat16, device=DEV)
    gt = torch.empty(2, 4, dtype=torch.bfloat16, device=DEV)
    L, st = fl.lib(), fl.stream(di.device)
    assert L.fnx_hc_activation(di.data_ptr(), m.data_ptr(), gt.data_ptr(), 2, 0, st) == 0
    rm, rg = post_ops.activate(di.view(2, 1, 324), 4)
    assert torch.equal(m, rm.view(2, 320)) and torch.equal(gt, rg.view(2, 4))
    x = torch.randn(2, 10240, generator=g).to(torch.bfloat16).to(DEV)
    lg = torch.randn(2, 10240, generator=g).to(torch.bfloat16).to(DEV)
    y = torch.empty(2, 2560, dtype=torch.bfloat16, device=DEV)
    assert L.fnx_hc_sigmoid_reduce(x.data_ptr(), lg.data_ptr(), y.data_ptr(), 2, st) == 0
    assert torch.equal(y, post_ops.mix_reduce(x.view(2, 1, 10240), lg.view(2, 1, 10240), 4).view(2, 2560))


def test_gated_residual_end_to_end(golden):
    """engine.gated_residual on the reference golden's inputs: the GEMMs run on the GPU's
    library, so within tolerance of the reference's output."""
    from fnx.engine import gated_residual
    g = golden("hc")
    mixed, inj = gated_residual(g["h"].to(DEV), g["norm_w"].to(DEV), g["w_di"].to(DEV), g["w_up"].to(DEV),
                                n_inj=g["HC"], hc=g["HC"])
    assert O.within_tolerance(mixed.cpu(), g["mixed"]), O.tolerance_report(mixed.cpu(), g["mixed"])
    assert int((_ordered(inj.cpu()) - _ordered(g["inj"])).abs().max()) <= 2
