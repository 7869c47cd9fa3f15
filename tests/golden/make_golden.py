"""Generate golden vectors by running the reference's own Python code on CPU.

Run where the reference tree is available, with its location in ``$FNX_REFERENCE``::

    FNX_REFERENCE=<path of the qwen-ascend tree> python tests/golden/make_golden.py

The reference imports ``torch_npu`` at module load; a stub module is injected whose
closed CANN operators (``npu_weight_quant_batchmatmul``, ``npu_grouped_matmul``,
``npu_swiglu``, ``npu_convert_weight_to_int4pack``) are restated on CPU by the oracle.  Everything else -- ``FnLayer._moe``
routing / permutation / inverse / combine fallbacks, ``ExpW4._wcat/_scat``, ``ExpQ``
packing and torch dequant + bmm, ``DenseW8`` layout, ``QW`` torch dequant and
``W4GemvOp.to_v2_layout`` -- is the reference's unmodified code.

Synthetic inputs are regenerated from seeds by ``fnx/synth.py`` (loaded by file path, so
the reference's ``fnx`` package and this repository's do not collide); each fixture
stores a SHA-256 of its inputs so a drift in the generator is detected.
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("FNX_REFERENCE"):
    raise SystemExit("make_golden.py: set FNX_REFERENCE to the reference (qwen-ascend) source tree")
REF = Path(os.environ["FNX_REFERENCE"])


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


synth = _load("b200_synth", REPO / "qwen-ascend_b200" / "fnx" / "synth.py")
sys.path.insert(0, str(REPO))
import oracle as O  # noqa: E402


def _install_stub():
    stub = types.ModuleType("torch_npu")

    def wqbm(x, w, scale, antiquant_group_size=None, **_):
        q = O.unpack_int4pack(w) if w.dtype == torch.int32 else w
        gs = antiquant_group_size or q.shape[0] // scale.shape[0]
        wd = O.deq_w4(q, scale, gs) if w.dtype == torch.int32 else O.dense_w8_deq(q, scale)
        return O.w4a16_matmul(x, wd)

    def gmm(xs, ws, antiquant_scale=None, group_list=None, split_item=3, group_type=0, output_dtype=None, **_):
        x, w, s = xs[0], ws[0], antiquant_scale[0]
        gs = w.shape[1] // s.shape[1]
        return [O.grouped_matmul(x, group_list, lambda e: O.deq_w4(O.unpack_int4pack(w[e]), s[e], gs))]

    def swiglu(x, dim=-1):
        n = x.shape[dim] // 2
        return torch.nn.functional.silu(x[..., :n]) * x[..., n:]

    def int4pack(q):
        # npu_convert_weight_to_int4pack restated (used only by the tools module's import)
        return O.pack_int4pack(q.to(torch.int8))

    stub.npu_weight_quant_batchmatmul = wqbm
    stub.npu_grouped_matmul = gmm
    stub.npu_swiglu = swiglu
    stub.npu_convert_weight_to_int4pack = int4pack
    sys.modules["torch_npu"] = stub


def sha(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def ref_engine(shape):
    _install_stub()
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import fnx.engine as E
    E.H, E.MI, E.TOPK, E.NEXP = shape.H, shape.I, shape.k, shape.E
    return E


def build_ref_layer(E, t, shape, expq=False):
    """A SimpleNamespace carrying exactly the attributes ``FnLayer._moe`` reads."""
    L = O.Layer(t, shape.gs)
    ns = SimpleNamespace(idx=0)
    ns.sh_gu = E.Raw(L.sh_cat)                       # sh_gate | sh_up | gate2 | router
    ns.sh_gw = True
    ns.sh_down = E.Raw(L.sh_dn.t().contiguous())
    if expq:
        # ExpQ stores [E, N, K] int8 (-8..7) + scales [E, N, G]; pack4 packs it.
        def mk(w4, sc):
            q = O.unpack_int4pack(w4).transpose(1, 2).contiguous()        # [E, N, K]
            return E.ExpQ(q, sc.transpose(1, 2).contiguous(), shape.gs, packed=True)
        ns.exp_gu = mk(t["gu_w4"], t["gu_scales"])
        ns.exp_dn = mk(t["dn_w4"], t["dn_scales"])
    else:
        os.environ["FNX_W4_SCALE_CACHE"] = "0"
        def mk(w4, sc):
            Ex, K, n8 = w4.shape
            dummy_s8t = torch.ones(K // shape.gs, Ex, n8 * 8, dtype=torch.int8)
            dummy_base = torch.ones(Ex, n8 * 8, dtype=torch.bfloat16)
            # a dict-carrying subclass so the recorder can wrap methods per instance
            rec_cls = type("RecordingExpW4", (E.ExpW4,), {})
            o = rec_cls(w4, dummy_s8t, dummy_base, shape.gs, expert_major=True)
            o._scales = sc.contiguous()                       # the FNX_W4_SCALE_CACHE layout
            o.s8t = o.base = None
            return o
        ns.exp_gu = mk(t["gu_w4"], t["gu_scales"])
        ns.exp_dn = mk(t["dn_w4"], t["dn_scales"])
    return L, ns


def run_moe(E, ns, x, flags):
    for k_, v in flags.items():
        os.environ[k_] = v
    try:
        with torch.no_grad():
            return E.FnLayer._moe(ns, x.view(x.shape[0], 1, -1)).view(x.shape[0], -1)
    finally:
        for k_ in flags:
            os.environ.pop(k_, None)


GROUPED = {"FNX_MOE_GROUP": "1", "FNX_MOE_INVERSE": "1", "FNX_MOE_INVERSE_SORT": "1",
           "FNX_MOE_SWIGLU_FP32": "1", "FNX_MOE_REDUCE": "0"}
DECODE = {"FNX_POST_NATIVE": "1", "FNX_MOE_EPILOGUE": "1", "FNX_MOE_REDUCE": "1",
          "FNX_MOE_SWIGLU_FP32": "1", "FNX_EXPERT_GATHER": "1", "FNX_DECODE_DN_GMM": "0"}


def capture_intermediates(E, ns, x, flags, shape):
    """Run ``_moe`` while recording the routing / permutation tensors it builds."""
    rec = {}
    orig_topk, orig_argsort = torch.topk, torch.argsort
    orig_lin = E.lin

    def lin(x_, w_):
        r = orig_lin(x_, w_)
        rec.setdefault("lin", []).append(r.clone())
        return r

    def topk(*a, **k):
        r = orig_topk(*a, **k)
        rec.setdefault("topk", (r[0].clone(), r[1].clone()))
        return r

    def argsort(t, *a, **k):
        r = orig_argsort(t, *a, **k)
        rec.setdefault("argsort", []).append(r.clone())
        return r

    grouped = ns.exp_gu.apply_grouped
    def apply_grouped(x_, ends, host_ends=None):
        rec.setdefault("grouped_in", []).append((x_.clone(), ends.clone()))
        y = grouped(x_, ends, host_ends)
        rec.setdefault("grouped_out", []).append(y.clone())
        return y
    ns.exp_gu.apply_grouped = apply_grouped
    dgrouped = ns.exp_dn.apply_grouped
    def dn_grouped(x_, ends, host_ends=None):
        rec.setdefault("grouped_in", []).append((x_.clone(), ends.clone()))
        y = dgrouped(x_, ends, host_ends)
        rec.setdefault("grouped_out", []).append(y.clone())
        return y
    ns.exp_dn.apply_grouped = dn_grouped
    torch.topk, torch.argsort, E.lin = topk, argsort, lin
    try:
        out = run_moe(E, ns, x, flags)
    finally:
        torch.topk, torch.argsort, E.lin = orig_topk, orig_argsort, orig_lin
    return out, rec


def lin_outputs(rec, shape):
    """(sh, shared_gate, logits) as the reference's own concat GEMM produced them."""
    gu, sh = rec["lin"][0], rec["lin"][1]
    I = shape.I
    return sh, gu[:, 2 * I:2 * I + 1].contiguous(), gu[:, 2 * I + 1:].contiguous()


def golden_grouped(name, shape, T, seed, xseed, light=False):
    """The grouped prefill branch; ``light`` keeps the routing, permutation and output only
    (not the shared-expert rows), for the larger token counts."""
    E = ref_engine(shape)
    t = synth.make_layer(shape, seed=seed)
    x = synth.make_tokens(T, shape.H, seed=xseed)
    L, ns = build_ref_layer(E, t, shape)
    out, rec = capture_intermediates(E, ns, x, GROUPED, shape)
    sh, gate, logits = lin_outputs(rec, shape)
    w_raw, idx = rec["topk"]
    g = dict(kind="grouped", shape=list(map(int, (shape.H, shape.I, shape.E, shape.k, shape.gs))),
             T=T, seed=seed, xseed=xseed, input_sha=sha(*t.values(), x),
             logits=logits, gate=gate, sh=None if light else sh, probs_topk=w_raw, idx=idx, out=out,
             order=rec["argsort"][0], inverse=rec["argsort"][1] if len(rec["argsort"]) > 1 else None,
             ends=rec["grouped_in"][0][1])
    if T * shape.k <= 256:
        g.update(gu=rec["grouped_out"][0], act=rec["grouped_in"][1][0], yd=rec["grouped_out"][1])
    torch.save(g, HERE / f"{name}.pt")
    print(name, "saved", out.shape, flush=True)


def golden_expq(name, shape, T, seed, xseed):
    """The pure-torch ExpQ path (dequant + bf16 bmm): b>1 batch branch or b=1 branch."""
    E = ref_engine(shape)
    t = synth.make_layer(shape, seed=seed)
    x = synth.make_tokens(T, shape.H, seed=xseed)
    L, ns = build_ref_layer(E, t, shape, expq=True)
    out = run_moe(E, ns, x, {})
    torch.save(dict(kind="expq", shape=list(map(int, (shape.H, shape.I, shape.E, shape.k, shape.gs))),
                    T=T, seed=seed, xseed=xseed, input_sha=sha(*t.values(), x), out=out),
               HERE / f"{name}.pt")
    print(name, "saved", out.shape, flush=True)


def golden_decode(name, shape, seed, xseed):
    """The production decode branch (b=1, ExpW4 + K-major gather + Cartesian down)."""
    E = ref_engine(shape)
    t = synth.make_layer(shape, seed=seed)
    x = synth.make_tokens(1, shape.H, seed=xseed)
    L, ns = build_ref_layer(E, t, shape)
    rec = {}
    wcat, scat = ns.exp_gu._wcat, ns.exp_gu._scat
    def wcat_(ids):
        r = wcat(ids)
        rec.setdefault("wcat", r.clone())
        return r
    def scat_(ids):
        r = scat(ids)
        rec.setdefault("scat", r.clone())
        return r
    ns.exp_gu._wcat, ns.exp_gu._scat = wcat_, scat_
    out, rec2 = capture_intermediates(E, ns, x, DECODE, shape)
    rec.update(rec2)
    sh, gate, logits = lin_outputs(rec, shape)
    torch.save(dict(kind="decode", shape=list(map(int, (shape.H, shape.I, shape.E, shape.k, shape.gs))),
                    T=1, seed=seed, xseed=xseed, input_sha=sha(*t.values(), x), out=out,
                    logits=logits, gate=gate, sh=sh, idx=rec["topk"][1], probs_topk=rec["topk"][0],
                    wcat_sha=sha(rec["wcat"]), scat_sha=sha(rec["scat"]),
                    scat=rec["scat"] if rec["scat"].numel() <= 1 << 20 else None),
               HERE / f"{name}.pt")
    print(name, "saved", flush=True)


def golden_reduce():
    """Adversarial cancellation rows (``tests/r118_weighted_reduce.py:38-43``) and random
    batches through the reference's torch fallback expressions."""
    _install_stub()
    torch.manual_seed(117)
    H = 2560
    cases = {}
    values = torch.randn(1, 10, H, dtype=torch.bfloat16)
    weights = torch.ones(1, 10, dtype=torch.bfloat16)
    values[0, :, 0] = 0; values[0, 0, 0] = 1e8; values[0, 1, 0] = 1; values[0, 2, 0] = -1e8; values[0, 3, 0] = 1
    values[0, :, 1] = 0; values[0, 0, 1] = 1e8; values[0, 1, 1] = -1e8; values[0, 2, 1] = 1; values[0, 3, 1] = 1
    cases["adversarial"] = dict(values=values.clone(), weights=weights.clone(),
                                expected=(values * weights.unsqueeze(-1)).sum(1))
    for B in (1, 3, 9):
        v = torch.randn(B, 10, H, dtype=torch.bfloat16) * .1
        w = torch.rand(B, 10, dtype=torch.bfloat16)
        inv = torch.randperm(B * 10)
        src = v.view(-1, H)
        restored = src.index_select(0, inv).view(B, 10, H)
        cases[f"inverse{B}"] = dict(values=src.clone(), weights=w, inverse=inv,
                                    expected=(restored * w.unsqueeze(-1)).sum(1))
    mv = torch.randn(5, 4, H, dtype=torch.bfloat16)
    mw = torch.rand(5, 4, H, dtype=torch.bfloat16)
    cases["mean4"] = dict(values=mv, weights=mw, expected=(mv * mw).mean(1))
    # moe_merge / epilogue reference compositions (benchmarks/r141-moe-epilogue/probe.py:9-18)
    y = torch.randn(10, 10 * H, dtype=torch.bfloat16) * 10
    w = torch.softmax(torch.randn(1, 10).float() * 3, -1).bfloat16()
    shared = torch.randn(1, H, dtype=torch.bfloat16) * .1
    gate = (torch.randn(1, 1) * 8).bfloat16()
    dg = torch.arange(10)
    diag = y.view(10, 10, H)[dg, dg]
    red = (diag * w[0].unsqueeze(-1)).sum(dim=0, keepdim=True)
    merged = red + torch.sigmoid(gate) * shared
    cases["epilogue"] = dict(cartesian=y, weights=w, shared=shared, gate=gate, expected=merged)
    torch.save(cases, HERE / "reduce_cases.pt")
    print("reduce_cases saved", flush=True)


def golden_dense_w8():
    """``DenseW8`` layout + merge and the ``QW`` torch dequant path (``fnx/engine.py:259-384``)."""
    E = ref_engine(synth.CFG1)
    rng = np.random.Generator(np.random.PCG64(5))
    K = 2048
    parts = []
    for N in (2048, 512, 512, 2048):
        q = torch.from_numpy(rng.integers(-127, 128, size=(N, K), dtype=np.int8))
        s = torch.from_numpy(np.abs(rng.standard_normal((N, 1), dtype=np.float32)) * 0.01).to(torch.bfloat16)
        parts.append((q, s))
    dws = [E.DenseW8(q, s, K=K) for q, s in parts]
    merged = E.DenseW8.merge(dws)
    x = torch.from_numpy(rng.standard_normal((16, K), dtype=np.float32)).to(torch.bfloat16)
    qw_out = torch.cat([E.QW(q, s)(x) for q, s in parts], dim=1)        # the torch dequant path
    # the weights regenerate from PCG64(5); only their digests, the merged scales and outputs are stored
    torch.save(dict(seed=5, K=K, Ns=[2048, 512, 512, 2048], parts_sha=sha(*[t for p_ in parts for t in p_]),
                    x=x, w8t_sha=sha(merged.w8t), sc=merged.sc, gs=merged.gs, N=merged.N,
                    qw_out=qw_out, deq_w=merged.deq_w()[:64].clone()), HERE / "dense_w8.pt")
    print("dense_w8 saved", flush=True)


def golden_w4gemv():
    """``W4GemvOp.to_v2_layout`` on random packed bytes (``fnx/w4gemv_op.py:222-250``)."""
    _install_stub()
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from fnx.w4gemv_op import W4GemvOp
    rng = np.random.Generator(np.random.PCG64(9))
    nE, N, K = 3, 40, 256
    p4 = rng.integers(-128, 128, size=(nE, N, K // 2), dtype=np.int8)
    v2 = W4GemvOp.to_v2_layout(p4, N, K)
    s4 = (np.abs(rng.standard_normal((nE, N, K // 32))) * 0.02).astype(np.float16)
    x = rng.standard_normal((nE, K)).astype(np.float32)
    # the self-test's numpy contract (fnx/w4gemv_op.py:302-319), reversed-id index table
    b = p4.view(np.uint8)
    lo = ((b & 0x0F).astype(np.int8) ^ 8) - 8
    hi = (((b >> 4) & 0x0F).astype(np.int8) ^ 8) - 8
    w4 = np.empty((nE, N, K), dtype=np.int8)
    w4[:, :, 0::2] = lo
    w4[:, :, 1::2] = hi
    wf = w4.astype(np.float32) * np.repeat(s4.astype(np.float32), 32, axis=2)
    perm = np.arange(nE - 1, -1, -1)
    y_perm = np.einsum("enk,ek->en", wf[perm], x)
    torch.save(dict(p4=torch.from_numpy(p4), v2=torch.from_numpy(v2), s4=torch.from_numpy(s4),
                    x=torch.from_numpy(x), perm=torch.from_numpy(perm), y_perm=torch.from_numpy(y_perm),
                    N=N, K=K), HERE / "w4gemv.pt")
    print("w4gemv saved", flush=True)


def golden_v2o():
    """The LQP v2o unpack of ``tools/repack_w4a16.py:41-55`` (the reference function itself, run
    on random bytes): the layout the GPU v2o -> int4pack repack reads."""
    _install_stub()
    spec = importlib.util.spec_from_file_location("ref_repack_w4a16", REF / "tools" / "repack_w4a16.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.Generator(np.random.PCG64(17))
    E, N, K = 3, 24, 384
    v2o = rng.integers(0, 256, size=(E, N, K // 2), dtype=np.uint8)
    q = mod.unpack_v2(v2o, K)
    torch.save(dict(v2o=torch.from_numpy(v2o), K=K, q=torch.from_numpy(q)), HERE / "v2o.pt")
    print("v2o saved", flush=True)


def golden_expq_packed():
    """``ExpQ.from_packed`` (``fnx/engine.py:478-501``) on random LQP tensors and its ``matmul``
    (``_deq_v2`` + ``_gemm2``, ``fnx/engine.py:503-572,772-776``), default flags: the torch
    dequant path built straight from the artifact, at 64- and 128-wide scale groups.  The
    dequantised lo/hi halves are kept as SHA-256 digests, the products in full."""
    E = ref_engine(synth.CFG1)
    rng = np.random.Generator(np.random.PCG64(31))
    nE, N, K = 3, 256, 384
    idx = torch.tensor([2, 0, 2, 1])                    # a repeated expert, one left out
    cases = {}
    for gs in (64, 128):
        v2o = torch.from_numpy(rng.integers(0, 256, size=(nE, N, K // 2), dtype=np.uint8))
        s8 = torch.from_numpy(rng.integers(1, 128, size=(nE, N, K // gs), dtype=np.int8))
        base = torch.from_numpy((np.abs(rng.standard_normal((nE, N))) * 1e-3 + 1e-4).astype(np.float16))
        xb = torch.from_numpy(rng.standard_normal((idx.numel(), 1, K), dtype=np.float32)).to(torch.bfloat16)
        q = E.ExpQ.from_packed(v2o, s8, base, "cpu")
        wlo, whi = q._deq_v2(idx)
        y = q.matmul(xb, idx)
        cases[f"g{gs}"] = dict(v2o=v2o, s8=s8, base=base, xb=xb, y=y, wlo_sha=sha(wlo), whi_sha=sha(whi))
    torch.save(dict(K=K, N=N, E=nE, idx=idx, cases=cases), HERE / "expq_packed.pt")
    print("expq_packed saved", flush=True)


def golden_inject():
    """``inject`` (``fnx/engine.py:859-877``, the torch path) on random bf16 tensors at the
    reference's production width (H=2560, HC=4): ``hyper + y * inj`` broadcast over branches."""
    E = ref_engine(synth.PROD)
    g = torch.Generator().manual_seed(23)
    b = 3
    hyper = torch.randn(b, 1, E.HC * E.H, generator=g).to(torch.bfloat16)
    inj = (2 * torch.rand(b, 1, E.HC, generator=g)).to(torch.bfloat16)
    y = torch.randn(b, 1, E.H, generator=g).to(torch.bfloat16)
    out = E.inject(hyper, inj, y)
    torch.save(dict(hyper=hyper, inj=inj, y=y, out=out, H=int(E.H), HC=int(E.HC)), HERE / "inject.pt")
    print("inject saved", flush=True)


def golden_hc():
    """``gated_residual`` (``fnx/engine.py:818-857``, torch path, with the concatenated
    down+inject weight as the loader builds it) at H=256, HC=4, low rank 32: the step that
    produces the MoE input ``mixed`` and the inject gates."""
    E = ref_engine(synth.PROD)
    g = torch.Generator().manual_seed(29)
    # a narrow instance of the production shape (H=2560, LOWRANK=320) keeps the fixture small;
    # gated_residual reads H and HC from the module and the low rank from the weights
    H, HC, LR, b = 256, int(E.HC), 32, 3
    E.H = H
    h = torch.randn(b, 1, HC * H, generator=g).to(torch.bfloat16)
    norm_w = (0.1 * torch.randn(HC * H, generator=g)).to(torch.bfloat16)
    w_di = (torch.randn(LR + HC, HC * H, generator=g) / (HC * H) ** 0.5).to(torch.bfloat16)
    w_up = (torch.randn(HC * H, LR, generator=g) / LR ** 0.5).to(torch.bfloat16)
    mixed, inj = E.gated_residual(h, norm_w, w_di, w_up, None, n_inj=HC)
    torch.save(dict(h=h, norm_w=norm_w, w_di=w_di, w_up=w_up, mixed=mixed, inj=inj, H=H, HC=HC, LR=LR),
               HERE / "hc.pt")
    print("hc saved", flush=True)


PIN = synth.MoEShape(H=256, I=128, E=16, k=4, gs=128)

if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count())
    which = set(sys.argv[1:]) or {"pin", "cfg1", "cfg2", "decode", "reduce", "w8", "w4gemv", "expq", "v2o", "inject", "hc"}
    if "v2o" in which:
        golden_v2o()
    if "inject" in which:
        golden_inject()
    if "hc" in which:
        golden_hc()
    if "pin" in which:
        golden_grouped("pin_grouped", PIN, T=48, seed=11, xseed=12)
        golden_decode("pin_decode", PIN, seed=11, xseed=13)
    if "cfg1" in which:
        golden_grouped("cfg1_grouped", synth.CFG1, T=64, seed=0, xseed=1)
    if "cfg2" in which:
        # the prefill configuration's layer shape (E=512, top-10) at 512 tokens
        golden_grouped("cfg2_grouped_T512", synth.CFG2, T=512, seed=2, xseed=5, light=True)
    if "expq" in which:
        golden_expq("cfg1_expq", synth.CFG1, T=64, seed=0, xseed=1)
        golden_expq("pin_expq_decode", PIN, T=1, seed=11, xseed=13)
        golden_expq_packed()
    if "decode" in which:
        golden_decode("cfg2_decode", synth.CFG2, seed=2, xseed=3)
    if "reduce" in which:
        golden_reduce()
    if "w8" in which:
        golden_dense_w8()
    if "w4gemv" in which:
        golden_w4gemv()
