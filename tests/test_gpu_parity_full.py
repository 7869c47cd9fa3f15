"""GPU parity at the workload's own sizes (the configurations the bench times), through the
public layer API and the C ABI, against the CPU oracle and the reference-produced goldens.

* the prefill layer at T=4096 (E=512, top-10, H=2048, I=512, g128; the bench's first layer
  and tokens): router logits, routing from the CPU logits (bit-exact ids), the number of
  tokens whose routing flips when routed from the GPU's own logits, and the layer output
  against the oracle on every token whose routing agrees;
* the reference's grouped ``_moe`` at E=512, top-10 on 512 tokens (fixture made by running
  the reference's code): the GPU top-k kernel on the reference's CPU logits reproduces its
  ``torch.topk`` ids (up to ties at the k-th place), and the layer fed those logits
  reproduces its output;
* the W8A16 concatenated projection (K=2048, N=5120) at M = 256 and 4096;
* W8A16 split-K at splits that are not powers of two (3, 6, 12).

Tolerance (bf16 outputs, fp32 accumulation): relative-L2 <= 5e-3 and max-abs <= 2e-2 of the
reference's largest magnitude (``O.within_tolerance``).
"""
import numpy as np
import pytest
import torch

import oracle as O
from fnx import _lib, synth

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _errors():
    _lib.lib()
    _lib.device_errors()
    yield
    assert _lib.device_errors() == 0


def _gpu_layer(t, shape):
    from fnx.engine import MoELayer
    return MoELayer.from_synth({k: v.to(DEV) for k, v in t.items()}, shape)


def _logits_with(layer, logits, gate):
    """A ``[T, R_pad]`` logits operand holding the given router logits and shared gate."""
    T = logits.shape[0]
    lg = torch.zeros(T, layer.R_pad, dtype=BF16)
    lg[:, :layer.E] = logits
    lg[:, layer.E] = gate.reshape(-1)
    return lg.to(DEV)


def _set_differs(a, b):
    """Per row: the two top-k id sets differ."""
    sa, sb = torch.sort(a, dim=-1).values, torch.sort(b, dim=-1).values
    return (sa != sb).any(dim=-1)


def test_prefill_layer_T4096_full_size():
    """The bench's headline layer (seed 100, tokens seed 1000) against the oracle."""
    shape, T = synth.CFG2, 4096
    t = synth.make_layer(shape, seed=100)
    L = O.Layer(t, shape.gs)
    layer = _gpu_layer(t, shape)
    x = synth.make_tokens(T, shape.H, seed=1000)
    xd = x.to(DEV)
    out, d = layer.prefill(xd, details=True)
    sh, gate, rlogits = O.shared_and_logits(x, L)
    # router GEMM within tolerance of the CPU bf16 GEMM
    rep = O.tolerance_report(d["logits"].float().cpu(), rlogits.float())
    assert rep["rel_l2"] < 5e-3, rep
    # routing from the CPU logits on the GPU top-k kernel: the oracle's ids bit for bit
    lg = _logits_with(layer, rlogits, gate)
    w_c, idx_c, _ = layer.topk(lg)
    rw, ridx, probs = O.route(rlogits, shape.k)
    assert torch.equal(idx_c.cpu(), ridx)
    assert int(O.bf16_ulp_diff(rw, w_c.cpu()).max()) <= 1
    # routing from the GPU's own logits: a token flips only where a logit differs by an ulp
    flips = _set_differs(d["idx"].cpu(), ridx)
    nflip = int(flips.sum())
    print(f"T=4096: {nflip} of {T} tokens route differently from the GPU logits than from the CPU logits")
    assert nflip <= T // 50
    # the layer output against the oracle on its own routing, every token that routes alike
    ref = O.moe_forward(x, L, shape.k)
    keep = ~flips
    rep = O.tolerance_report(out.cpu()[keep], ref[keep])
    assert O.within_tolerance(out.cpu()[keep], ref[keep]), rep
    # fed the CPU logits, the whole batch (every token) matches
    out_c = layer.prefill(xd, logits=lg)
    rep = O.tolerance_report(out_c.cpu(), ref)
    assert O.within_tolerance(out_c.cpu(), ref), rep


def test_prefill_cfg2_T512_reference_golden(golden):
    """The reference's grouped branch at E=512, top-10, 512 tokens (its own torch.topk,
    argsort and combine; closed operators restated)."""
    g = golden("cfg2_grouped_T512")
    H, I, E, k, gs = g["shape"]
    shape = synth.MoEShape(H, I, E, k, gs)
    t = synth.make_layer(shape, seed=g["seed"])
    x = synth.make_tokens(g["T"], H, seed=g["xseed"])
    T = g["T"]
    layer = _gpu_layer(t, shape)
    lg = _logits_with(layer, g["logits"], g["gate"])
    w, idx, _ = layer.topk(lg)
    probs = torch.softmax(g["logits"].float(), -1)
    wr = (g["probs_topk"] / g["probs_topk"].sum(-1, keepdim=True)).to(BF16)
    assert bool(O.same_topk(idx.cpu(), w.cpu(), g["idx"], wr, probs, k).all())
    differ = _set_differs(idx.cpu(), g["idx"])
    assert bool(O.boundary_tie(probs, k)[differ].all()), "ids differ only where the k-th place is tied"
    out, d = layer.prefill(x.to(DEV), details=True, logits=lg)
    assert torch.equal(d["ends"].cpu(), g["ends"].reshape(-1)[:E]) or bool(differ.any())
    if not bool(differ.any()):
        assert O.is_within_group_permutation(d["order"].cpu(), g["order"], g["idx"].reshape(-1))
    ref = g["out"].clone()
    if bool(differ.any()):
        # a tie at the k-th place: the reference's topk picked another tied expert; those tokens
        # are checked against the reference formulation with this routing
        L = O.Layer(t, gs)
        rows = differ.nonzero().reshape(-1)
        ref[rows] = O.moe_forward(x[rows], L, k, routing=(w.cpu()[rows], idx.cpu()[rows]))
    rep = O.tolerance_report(out.cpu(), ref)
    assert O.within_tolerance(out.cpu(), ref), rep
    # routed from the GPU's own logits instead: count the tokens that flip
    _, idx_g, _ = layer.topk(layer.logits(x.to(DEV)))
    nflip = int((_set_differs(idx_g.cpu(), g["idx"]) & ~O.boundary_tie(probs, k)).sum())
    print(f"T=512: {nflip} of {T} tokens route differently from the GPU logits than from the reference's")
    assert nflip <= T // 50


def _w8_cfg5(seed=7):
    K, N = 2048, 5120
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8)
    sc = (torch.randn(N, 1, generator=g).abs() * 0.01).to(BF16)
    return q, sc, g


@pytest.mark.parametrize("M", [256, 4096])
def test_w8a16_cfg5_large_m(M):
    """The qkv+z projection (K=2048, N=5120, per-channel int8) on the tensor-core GEMM; at
    M=4096 a seeded sample of 512 rows is checked (rows are independent)."""
    from fnx.engine import DenseW8
    q, sc, g = _w8_cfg5()
    x = torch.randn(M, 2048, generator=g).to(BF16)
    w = DenseW8(q.to(DEV), sc.to(DEV))
    got = w(x.to(DEV)).cpu()
    rows = torch.arange(M) if M <= 256 else torch.randperm(M, generator=g)[:512]
    ref = O.dense_w8(x[rows], w.w8t.cpu(), w.sc.cpu())
    rep = O.tolerance_report(got[rows], ref)
    assert O.within_tolerance(got[rows], ref), rep
    assert torch.equal(w(x.to(DEV)).cpu().view(torch.int16), got.view(torch.int16))


@pytest.mark.parametrize("M,K,split", [(12, 1536, 12), (64, 1536, 6), (100, 1536, 3), (64, 3072, 12)])
def test_w8a16_split_k_not_power_of_two(M, K, split):
    """Splits of 3, 6 and 12 K ranges (K/64 = 24 or 48 k-blocks): the split and unsplit entry
    points match the oracle, and the split result repeats bit for bit."""
    from fnx.engine import DenseW8
    L = _lib.lib()
    N = 640
    g = torch.Generator().manual_seed(M + K)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8)
    sc = (torch.randn(N, 1, generator=g).abs() * 0.01).to(BF16)
    x = torch.randn(M, K, generator=g).to(BF16)
    w = DenseW8(q.to(DEV), sc.to(DEV))
    xd = x.to(DEV)
    nws = L.fnx_w8a16_gemm_workspace(M, K, N, 1)
    assert nws == split * M * N * 4
    ws = torch.empty(nws, dtype=torch.uint8, device=DEV)
    ref = O.dense_w8(x, w.w8t.cpu(), w.sc.cpu())
    outs = []
    for use_split in (True, True, False):
        y = torch.full((M, N), float("nan"), dtype=BF16, device=DEV)
        if use_split:
            rc = L.fnx_w8a16_gemm_ws(xd.data_ptr(), w.w8t.data_ptr(), w.sc.data_ptr(), y.data_ptr(), M, K, N, 1,
                                     ws.data_ptr(), nws, _lib.stream(xd.device))
        else:
            rc = L.fnx_w8a16_gemm(xd.data_ptr(), w.w8t.data_ptr(), w.sc.data_ptr(), y.data_ptr(), M, K, N, 1,
                                  _lib.stream(xd.device))
        assert rc == 0
        outs.append(y.cpu())
        assert O.within_tolerance(outs[-1], ref), O.tolerance_report(outs[-1], ref)
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
