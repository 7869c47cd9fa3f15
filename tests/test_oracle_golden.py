"""Pin the CPU oracle against golden vectors produced by the reference's own code.

The fixtures under ``tests/golden/`` come from ``tests/golden/make_golden.py``, which
imports the reference's ``fnx`` package and runs ``FnLayer._moe`` (grouped prefill branch
and production decode branch), the pure-torch ``ExpQ`` branch, the ``QW``/``DenseW8``
containers, the reduce/epilogue torch fallbacks and ``W4GemvOp.to_v2_layout``.
"""
import hashlib

import numpy as np
import pytest
import torch

import oracle as O
from fnx import synth

BF16 = torch.bfloat16


def bits_equal(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.int16), b.view(torch.int16))


def sha(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != BF16
                 else t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def load_case(g):
    H, I, E, k, gs = g["shape"]
    shp = synth.MoEShape(H, I, E, k, gs)
    t = synth.make_layer(shp, seed=g["seed"])
    x = synth.make_tokens(g["T"], H, seed=g["xseed"])
    assert sha(*t.values(), x) == g["input_sha"], "synthetic generator drifted from the fixture"
    return shp, t, x


def canonical_rows(t, order):
    """Rows of an expert-major tensor re-indexed by flat (token*k + slot) position."""
    out = torch.empty_like(t)
    out[order] = t
    return out


@pytest.mark.parametrize("name", ["pin_grouped", "cfg1_grouped", "cfg2_grouped_T512"])
def test_grouped_layer(golden, name):
    g = golden(name)
    shp, t, x = load_case(g)
    L = O.Layer(t, shp.gs)
    sh, gate, logits = O.shared_and_logits(x, L)
    assert bits_equal(logits, g["logits"])
    assert bits_equal(gate, g["gate"])
    if g["sh"] is not None:                 # the larger fixtures keep no shared-expert rows
        assert bits_equal(sh, g["sh"])
    w, idx, probs = O.route(logits, shp.k)
    # reference weights: renormalise the top-k probabilities it selected
    wr = (g["probs_topk"] / g["probs_topk"].sum(-1, keepdim=True)).to(BF16)
    assert bool(O.same_topk(idx, w, g["idx"], wr, probs, shp.k).all())
    order, counts, ends, inverse = O.permute(g["idx"], shp.E)
    assert torch.equal(ends, g["ends"])
    assert O.is_within_group_permutation(order, g["order"], g["idx"].reshape(-1))
    out, d = O.moe_forward(x, L, shp.k, routing=(wr, g["idx"]), details=True)
    assert bits_equal(out, g["out"])
    if "gu" in g:
        assert bits_equal(canonical_rows(d["gu"], d["order"]), canonical_rows(g["gu"], g["order"]))
        assert bits_equal(canonical_rows(d["act"], d["order"]), canonical_rows(g["act"], g["order"]))
        assert bits_equal(canonical_rows(d["yd"], d["order"]), canonical_rows(g["yd"], g["order"]))
    if g.get("inverse") is not None:
        assert torch.equal(g["order"][g["inverse"]], torch.arange(g["order"].numel()))


@pytest.mark.parametrize("name", ["pin_decode", "cfg2_decode"])
def test_decode_branch(golden, name):
    """The production decode branch (K-major expert gather + Cartesian down + diagonal
    epilogue) equals the grouped formulation for one token."""
    g = golden(name)
    shp, t, x = load_case(g)
    L = O.Layer(t, shp.gs)
    sh, gate, logits = O.shared_and_logits(x, L)
    assert bits_equal(logits, g["logits"])
    wr = (g["probs_topk"] / g["probs_topk"].sum(-1, keepdim=True)).to(BF16)
    out = O.moe_forward(x, L, shp.k, routing=(wr, g["idx"]))
    assert bits_equal(out, g["out"])
    ow, os_ = O.gather_pair(t["gu_w4"], t["gu_scales"], g["idx"][0])
    assert sha(ow) == g["wcat_sha"] and sha(os_) == g["scat_sha"]
    if g.get("scat") is not None:
        assert bits_equal(os_, g["scat"])


def test_expq_torch_path(golden):
    """The reference's pure-torch ExpQ path (dequant + bf16 bmm per row) agrees with the
    oracle's fp32-accumulated grouped formulation within rounding."""
    g = golden("cfg1_expq")
    shp, t, x = load_case(g)
    L = O.Layer(t, shp.gs)
    ref_route = golden("cfg1_grouped")
    wr = (ref_route["probs_topk"] / ref_route["probs_topk"].sum(-1, keepdim=True)).to(BF16)
    out = O.moe_forward(x, L, shp.k, routing=(wr, ref_route["idx"]))
    r = O.tolerance_report(out, g["out"])
    assert r["rel_l2"] < 1e-3 and r["max_abs_norm"] < 2e-2 and r["exact_fraction"] > 0.9, r
    gd = golden("pin_expq_decode")
    shp, t, x = load_case(gd)
    out = O.moe_forward(x, O.Layer(t, shp.gs), shp.k)
    r = O.tolerance_report(out, gd["out"])
    assert r["rel_l2"] < 1e-3 and r["max_abs_norm"] < 2e-2, r


def test_reduce_cases(golden):
    cases = golden("reduce_cases")
    c = cases["adversarial"]
    got = O.weighted_reduce(c["values"].view(-1, c["values"].shape[-1]), c["weights"])
    assert bits_equal(got, c["expected"])
    assert got[0, 0].item() == 1.0 and got[0, 1].item() == 2.0      # sequential, not tree order
    for B in (1, 3, 9):
        c = cases[f"inverse{B}"]
        assert bits_equal(O.weighted_reduce(c["values"], c["weights"], inverse=c["inverse"]), c["expected"])
    c = cases["mean4"]
    assert bits_equal(O.weighted_mean4(c["values"], c["weights"]), c["expected"])
    c = cases["epilogue"]
    assert bits_equal(O.moe_epilogue(c["cartesian"], c["weights"], c["shared"], c["gate"]), c["expected"])


def test_dense_w8(golden):
    g = golden("dense_w8")
    rng = np.random.Generator(np.random.PCG64(g["seed"]))
    parts = []
    for N in g["Ns"]:
        q = torch.from_numpy(rng.integers(-127, 128, size=(N, g["K"]), dtype=np.int8))
        s = torch.from_numpy(np.abs(rng.standard_normal((N, 1), dtype=np.float32)) * 0.01).to(BF16)
        parts.append((q, s))
    assert sha(*[t for p in parts for t in p]) == g["parts_sha"]
    w8t = torch.cat([q.t() for q, _ in parts], 1).contiguous()          # DenseW8.merge layout
    sc = torch.cat([s.t() for _, s in parts], 1).contiguous()
    assert sha(w8t) == g["w8t_sha"] and bits_equal(sc, g["sc"])
    assert bits_equal(O.dense_w8_deq(w8t, sc).t()[:64].contiguous(), g["deq_w"])
    y = O.dense_w8(g["x"], w8t, sc)
    r = O.tolerance_report(y, g["qw_out"])
    assert r["rel_l2"] < 1e-3 and r["max_abs_norm"] < 2e-2, r


def test_w4gemv_layout(golden):
    g = golden("w4gemv")
    p4, N, K = g["p4"].numpy(), g["N"], g["K"]
    assert np.array_equal(O.to_v2_layout(p4, N, K), g["v2"].numpy())
    s4t = np.ascontiguousarray(np.transpose(g["s4"].numpy(), (0, 2, 1)))
    for lay, p in ((1, p4), (2, g["v2"].numpy())):
        y = O.w4gemv(p, s4t, g["x"].numpy(), g["perm"].numpy(), N, K, lay)
        assert np.abs(y - g["y_perm"].numpy()).max() < 1e-4


def test_int4pack_roundtrip():
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-8, 8, (3, 16, 24), generator=g, dtype=torch.int8)
    w = O.pack_int4pack(q)
    assert w.dtype == torch.int32 and w.shape == (3, 16, 3)
    assert torch.equal(O.unpack_int4pack(w), q)
    # nibble t of word j = W[k, 8j+t], low nibble first
    assert (int(w[0, 0, 0]) & 15) == (int(q[0, 0, 0]) & 15)
    assert ((int(w[0, 0, 0]) >> 28) & 15) == (int(q[0, 0, 7]) & 15)
    em = O.to_expert_major(w.permute(1, 0, 2).contiguous())
    assert torch.equal(em, w)


def test_topk_tie_rule():
    logits = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0]], dtype=BF16)
    w, idx, probs = O.route(logits, 2)
    assert idx.tolist() == [[1, 2]]                   # ties broken by ascending id
    assert bool(O.boundary_tie(probs, 2)[0])
    w2 = w.clone()
    assert bool(O.same_topk(idx, w, torch.tensor([[1, 4]]), w2, probs, 2)[0])
    assert not bool(O.same_topk(idx, w, torch.tensor([[1, 3]]), w2, probs, 2)[0])


def test_v2o_unpack_and_repack_pinned(golden):
    """LQP v2o: the oracle's unpack equals the reference's own ``unpack_v2``
    (``tools/repack_w4a16.py:41-55``) on the fixture, and its int4pack repack round-trips."""
    g = golden("v2o")
    v2o, K = g["v2o"].numpy(), g["K"]
    q = O.unpack_v2o(v2o, K)
    assert np.array_equal(q, g["q"].numpy())
    art = O.repack_v2o(v2o, K)                                    # [K, E, N/8]
    back = O.unpack_int4pack(art.permute(1, 0, 2))                # [E, K, N]
    assert torch.equal(back.transpose(1, 2).to(torch.int32), torch.from_numpy(q))


@pytest.mark.parametrize("gs", [64, 128])
def test_expq_packed_pinned(golden, gs):
    """``ExpQ.from_packed`` + ``matmul`` (the reference's torch dequant path straight from the
    LQP tensors): the oracle's dequantised halves equal the reference's bit for bit, and its
    once-rounded product agrees with the reference's three-rounding one within tolerance."""
    g = golden("expq_packed")
    c = g["cases"][f"g{gs}"]
    w = O.expq_deq(c["v2o"], c["s8"], c["base"], g["idx"])
    wlo, whi = O.expq_halves(w)
    assert sha(wlo) == c["wlo_sha"] and sha(whi) == c["whi_sha"]
    y = O.expq_matmul(c["xb"], c["v2o"], c["s8"], c["base"], g["idx"])
    r = O.tolerance_report(y, c["y"])
    assert r["rel_l2"] < 5e-3 and r["max_abs_norm"] < 2e-2, r


def test_inject_pinned(golden):
    """The oracle's inject equals the reference's ``inject`` (torch path) bit for bit."""
    g = golden("inject")
    got = O.inject(g["hyper"], g["inj"], g["y"])
    assert torch.equal(got.view(torch.int16), g["out"].view(torch.int16))


def test_gated_residual_pinned(golden):
    """The oracle's gated_residual (rms_norm, linears, activation, branch mix) equals the
    reference's function (torch path) bit for bit."""
    g = golden("hc")
    mixed, inj = O.gated_residual(g["h"], g["norm_w"], g["w_di"], g["w_up"], g["HC"], g["H"])
    assert torch.equal(mixed.view(torch.int16), g["mixed"].view(torch.int16))
    assert torch.equal(inj.view(torch.int16), g["inj"].view(torch.int16))
