"""Benchmark of the B200 W4A16 MoE expert path (one JSON line on rank 0).

Headline (``value``): MoE-layer prefill tokens/s at T=4096 tokens per GPU, H=2048,
E=512 experts, I=512, top-10, W4 group 128 (the prefill configuration of the workload
definition; synthetic seeded weights and activations).  A step is one full MoE layer:
router GEMM, top-k, expert-major permutation, grouped gate/up + SwiGLU, grouped down,
shared expert, slot-order combine and sigmoid-gated merge.  Inputs are resident in HBM;
each layer's weights (0.83 GB) exceed the 126 MB L2, and steps rotate over distinct
layers.  ``decode`` reports the decode configuration (M=1 and M=4 tokens, microseconds
per layer) over a CUDA-graphed rotation of 16 distinct layers (13 GB of weights).

With ``--gpus N`` under torchrun each rank brings its own T=4096 tokens (weak scaling); the
experts are sharded expert-parallel (E/N per GPU, ``fnx.ep``) and token rows go to their
experts' owners and back over NVLink peer stores (the shared expert runs on a second stream
meanwhile).  Decode is reported at N=1 only.

``--impl reference`` times the reference's algorithm on the host CPU (the oracle port of
``FnLayer._moe``; the reference itself is Python + torch_npu and cannot run here) on a
bounded token sample of the same layer, with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "qwen-ascend_b200"))

import torch  # noqa: E402

H, I, E, K_TOP, GS = 2048, 512, 512, 10, 128
T_PREFILL = 4096
METRIC = "MoE-layer prefill tokens/s @T=4096 (E=512, top-10, H=2048, I=512, W4 g128)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def prefill_flops(T):
    routed = 2 * T * K_TOP * (H * 2 * I + I * H)
    shared = 2 * T * 3 * H * I
    router = 2 * T * H * E
    return routed + shared + router


def decode_bytes(U, M):
    per_expert = H * 2 * I // 2 + (H // GS) * 2 * I * 2 + I * H // 2 + (I // GS) * H * 2
    return U * per_expert + per_expert + (E + 1) * H * 2 + M * H * 2 * 2


class ClockSampler:
    """nvidia-smi samples of SM clock / reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) >= 9:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU baseline
_CPU_INPUTS = {}


def cpu_baseline(sample_tokens=T_PREFILL, seed=0):
    """The oracle port of the reference's torch path on this host's cores: one MoE layer
    over ``sample_tokens`` tokens with fp32 accumulation, dequantising every touched
    expert inside the timed region (as the reference's ExpQ path does per call)."""
    import oracle as O
    from fnx import synth
    threads = len(os.sched_getaffinity(0)) or 1
    torch.set_num_threads(threads)
    key = (seed, sample_tokens)
    if key not in _CPU_INPUTS:                  # synthesis stays outside the timed region
        _CPU_INPUTS[key] = (synth.make_layer(synth.CFG2, seed=seed), synth.make_tokens(sample_tokens, H, seed=seed + 1))
    t, x = _CPU_INPUTS[key]
    t0 = time.perf_counter()
    L = O.Layer(t, GS)
    O.moe_forward(x, L, K_TOP, acc=torch.float32)
    dt = time.perf_counter() - t0
    return {"value": sample_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample_tokens} tokens through one layer of the T=4096 configuration (E=512, top-10): "
                      f"oracle port of FnLayer._moe, fp32 accumulation, per-call dequantisation; {dt:.1f} s"}


def cpu_baseline_median(sample_tokens=T_PREFILL, runs=3, warm=1):
    """``cpu_baseline`` after ``warm`` untimed calls (first-touch allocation, thread-pool start),
    the median of ``runs`` timed calls, as the reference arm measures it."""
    for _ in range(warm):
        cpu_baseline(sample_tokens)
    rs = [cpu_baseline(sample_tokens) for _ in range(runs)]
    v = statistics.median(r["value"] for r in rs)
    r = dict(rs[0], value=v)
    r["sample"] += f"; median of {runs} calls after {warm} untimed"
    return r


# ------------------------------------------------------------------ B200 arm
def make_layers(n, dev, seed0=100):
    from fnx import synth
    from fnx.engine import MoELayer
    layers = []
    for i in range(n):
        t = synth.make_layer(synth.CFG2, seed=seed0 + i, device=dev)
        layers.append(MoELayer.from_synth(t, synth.CFG2))
    return layers


def time_events(fn, iters, stream):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(iters):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / iters


def bench_prefill(args, world, rank, dev):
    from fnx import synth
    from fnx import _lib
    from fnx.engine import EPI_SWIGLU_F32, _grouped_w4
    nl = 2
    full = make_layers(nl, dev)
    if world > 1:
        # expert parallel: rank r keeps experts [r*E/N, (r+1)*E/N) of every layer (the same
        # seeded layers on every rank) and exchanges token rows with NCCL all-to-all
        from fnx.ep import ExpertParallelMoE
        layers = [ExpertParallelMoE.from_layer(lay, rank, world) for lay in full]
        full = full[:1]
        torch.cuda.empty_cache()
    else:
        layers = full
    xs = [synth.make_tokens(T_PREFILL, H, seed=1000 + rank * 10 + i, device=dev) for i in range(nl)]
    # each layer call runs as one CUDA graph (the public MoELayer.capture; the expert-parallel
    # layer waits on nothing on the host, so it captures whole as well)
    caps = [layers[i].capture(T_PREFILL) for i in range(nl)]
    for i in range(nl):
        caps[i].x.copy_(xs[i])
    stream = torch.cuda.current_stream(dev)
    step = [0]

    def run():
        i = step[0] % nl
        step[0] += 1
        return caps[i].replay()

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        ms = time_events(run, args.steps, stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ms, world)
    value = world * T_PREFILL / (ms * 1e-3)

    ep = None
    if world > 1:
        # multi-GPU parity: this rank's tokens through the expert-parallel layer (graph replay)
        # against the one-GPU layer holding all experts, bit for bit, on every rank
        got = caps[0](xs[0]).clone()
        ref = full[0].prefill(xs[0])
        same = torch.tensor([1 if torch.equal(got.view(torch.int16), ref.view(torch.int16)) else 0],
                            dtype=torch.int32, device=dev)
        torch.distributed.all_reduce(same, op=torch.distributed.ReduceOp.MIN)
        ep_bit_identical = bool(same.item())
        del got, ref
        st = layers[(step[0] - 1) % nl].exchange_stats()
        t = torch.tensor([st["received_slots"], st["dispatch_rows"] + st["return_rows"]], dtype=torch.float64,
                         device=dev)
        tmax, tsum = t.clone(), t.clone()
        torch.distributed.all_reduce(tmax, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(tsum)
        row = H * 2
        ep = {"experts_per_gpu": E // world,
              "exchange": "NVLink peer stores: token rows once per owner (dispatch kernel), per-slot down rows "
                          "written to the source by the down GEMM's epilogue; device-side count exchange, no host "
                          "sync",
              "bit_identical_to_one_gpu": ep_bit_identical,
              "recv_rows_max_over_mean": round(float(tmax[0] / (tsum[0] / world)), 4),
              "nvlink_bytes_per_step_per_gpu_max": int(tmax[1] * row)}

    # dominant kernel: routed gate/up grouped GEMM + fused SwiGLU (one-GPU form), timed alone
    lay = full[0]
    _, d = lay.prefill(xs[0], details=True)
    act = torch.empty(T_PREFILL * K_TOP, I, dtype=torch.bfloat16, device=dev)

    def gu():
        _grouped_w4(xs[0], lay.gu_t, d["ends"], act, E=E, M=T_PREFILL * K_TOP, K=H, Nw=2 * I,
                    epilogue=EPI_SWIGLU_F32, row_index=d["order"], index_div=K_TOP)
    for _ in range(3):
        gu()
    gu_ms = time_events(gu, 10, stream)
    gu_flops = 2 * T_PREFILL * K_TOP * H * 2 * I
    pk, src = peaks()
    achieved = gu_flops / (gu_ms * 1e-3) / 1e12
    roofline = {"kernel": "grouped_gemm_pair_kernel<SwiGLU> (routed gate/up)", "bound": "tensor",
                "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "peak_source": f"{src} bf16 burst",
                # dram__bytes_read.sum + dram__bytes_write.sum of this launch (587.6 + 8.3 MB) from one
                # ncu capture of `bench.py --profile-case gu`
                "traffic": 595.9e6, "traffic_unit": "B", "ms_per_launch": round(gu_ms, 4),
                "algorithmic_flops_per_launch": gu_flops}
    layer_tflops = prefill_flops(T_PREFILL) / (ms * 1e-3) / 1e12
    # the router + shared-gate logits GEMM ([T, 2048] x [640, 2048]^T): this library's tcgen05 GEMM
    # (what the layer runs) beside cuBLAS on the same operands
    rg = {}
    for name, native in (("native", True), ("cublas", False)):
        for _ in range(3):
            lay.logits(xs[0], native=native)
        rg[f"{name}_us"] = round(time_events(lambda: lay.logits(xs[0], native=native), 20, stream) * 1e3, 2)

    # end to end through the public API with host buffers
    xh = [xs[i].cpu().pin_memory() for i in range(nl)]
    outh = torch.empty(T_PREFILL, H, dtype=torch.bfloat16).pin_memory()

    # HostPipeline: batch i+1's tokens go up and batch i-1's output comes down while batch i
    # runs; every step still copies its own input from and its output to pinned host memory
    from fnx.engine import HostPipeline
    pipe = HostPipeline(caps)
    outs_h = [torch.empty(T_PREFILL, H, dtype=torch.bfloat16).pin_memory() for _ in range(nl)]
    xs_w = [xh[i % nl] for i in range(args.warmup)]
    pipe.run(xs_w, [outs_h[i % nl] for i in range(args.warmup)])
    torch.cuda.synchronize()
    barrier(world)
    xs_t = [xh[i % nl] for i in range(args.steps)]
    os_t = [outs_h[i % nl] for i in range(args.steps)]
    e2e_ms = max_over_ranks(time_events(lambda: pipe.run(xs_t, os_t), 1, stream) / args.steps, world)
    ref_out = caps[0](xs[0]).cpu()
    torch.cuda.synchronize()
    pipe.run([xh[0]], [outh])
    torch.cuda.synchronize()
    assert torch.equal(outh.view(torch.int16), ref_out.view(torch.int16)), "host pipeline output differs"
    # this library's kernels per layer: router logits GEMM, top-k, permute (hist, scan, scatter),
    # gate/up, down, combine, with the shared expert's gate/up and down as launches of their own on
    # the second stream (10; 8 in the single-launch form).  Expert parallel (peer exchange): router
    # GEMM, top-k, dispatch layout (3), token dedup (2), count exchange, dispatch push, wait, receive
    # layout (4 + row destinations), routed gate/up, down with the return in its epilogue, signal,
    # wait, combine, and the shared expert's two launches (23; 21 in the single-stream form).
    from fnx import engine as _eng
    if world > 1:
        launches_per_step = 23 if layers[0].overlap_shared else 21
    else:
        launches_per_step = 10 if _eng.OVERLAP_SHARED else 8
    # the host link's ceiling for e2e: both directions at once (the pipeline's copies overlap the
    # replays), so a step takes at least the device step and each direction's copy time
    link = bench_host_link(world, dev, T_PREFILL * H * 2)
    link_ms = max(ms, T_PREFILL * H * 2 / (link["duplex_gbs"] * 1e9) * 1e3)
    link["e2e_ceiling_tokens_per_s"] = round(world * T_PREFILL / (link_ms * 1e-3), 1)
    del caps
    torch.cuda.synchronize()
    if world > 1:
        barrier(world)
        for lay in layers:
            lay.close()
    return dict(value=value, ms=ms, clocks=clk.summary(), roofline=roofline, layer_tflops=layer_tflops, ep=ep,
                router_gemm=rg,
                e2e={"value": world * T_PREFILL / (e2e_ms * 1e-3), "unit": "tokens/s",
                     "h2d_bytes_per_step": T_PREFILL * H * 2, "d2h_bytes_per_step": T_PREFILL * H * 2,
                     "ms_per_step": round(e2e_ms, 4), "host_link": link},
                gpu_launches=launches_per_step * args.steps)


def bench_host_link(world, dev, nbytes, iters=20):
    """Host-link bandwidth with the bench's own kind of buffers (pinned host, allocated after
    the NUMA binding): ``nbytes`` up alone, down alone, and both directions at once on two
    streams (as ``HostPipeline`` runs them), every rank copying at the same time.  GB/s of the
    slowest rank (time max over ranks)."""
    hin = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    hout = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    din = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dout = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    sa, sb = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def timed(up, down):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(comp)
        for st, on, fn in ((sa, up, lambda: din.copy_(hin, non_blocking=True)),
                           (sb, down, lambda: hout.copy_(dout, non_blocking=True))):
            if not on:
                continue
            st.wait_event(ev[0])
            with torch.cuda.stream(st):
                for _ in range(iters):
                    fn()
        ev[1].record(sa)
        ev[2].record(sb)
        comp.wait_event(ev[1])
        comp.wait_event(ev[2])
        torch.cuda.synchronize()
        return max(ev[0].elapsed_time(ev[1]) if up else 0.0, ev[0].elapsed_time(ev[2]) if down else 0.0)

    res = {}
    for name, up, down in (("h2d", True, False), ("d2h", False, True), ("duplex", True, True)):
        timed(up, down)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(timed(up, down), world)
        res[f"{name}_gbs"] = round(nbytes * iters / (ms * 1e-3) / 1e9, 1)
    res["bytes_per_copy"] = nbytes
    return res


def bench_ep_stack(args, world, rank, dev, n_layers=48, T=8192, steps=2, warmup=1, balance=None):
    """The expert-parallel stack of the workload definition: 48 independently seeded layers of the
    prefill shape (E=512, top-10, H=2048, I=512, W4 g128), T=8192 tokens per GPU, router logits
    biased by a Zipf(1.1) expert popularity (so the experts, and with them the owner GPUs, are
    unevenly loaded).  Each layer's experts are first renumbered so that equal contiguous blocks
    carry equal loads (`balanced_expert_order` on a calibration batch's counts; FNX_EP_BALANCE=0
    keeps the seeded numbering), then rank r keeps experts [r*E/N, (r+1)*E/N); the layers share one
    peer exchange and run one after another on the rank's tokens (each layer gets the same input:
    the stack times the MoE path, not a model, and the model's residuals and norms are not part of
    it).  Reports tokens/s over the stack, NVLink bytes per GPU per step, and the load imbalance
    (max / mean received rows over the GPUs, and max / mean rows per expert)."""
    from fnx import synth
    from fnx.engine import MoELayer
    bias = synth.zipf_bias(E, 1.1).to(dev)
    if balance is None:
        balance = os.environ.get("FNX_EP_BALANCE", "1") != "0"
    layers, shared = [], None
    # expert placement: each layer's experts are renumbered so that the ranks' contiguous blocks
    # carry equal loads by the slot counts of a calibration batch (other tokens than the timed ones)
    xc = synth.make_tokens(T, H, seed=7000 + rank, device=dev)
    for i in range(n_layers):
        full = MoELayer.from_synth(synth.make_layer(synth.CFG2, seed=5000 + i, device=dev), synth.CFG2, bias=bias)
        if world > 1:
            from fnx.ep import ExpertParallelMoE, balanced_expert_order
            if balance:
                _, idc, _ = full.topk(full.logits(xc))
                cnt = torch.bincount(idc.reshape(-1), minlength=E).to(torch.float64)
                torch.distributed.all_reduce(cnt)
                full.permute_experts(balanced_expert_order(cnt.cpu(), world))
            lay = ExpertParallelMoE.from_layer(full, rank, world, transport="p2p", max_tokens=T, exchange=shared)
            shared = lay.exchange
            del full
        else:
            lay = full
        layers.append(lay)
    torch.cuda.empty_cache()
    x = synth.make_tokens(T, H, seed=9000 + rank, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for lay in layers:
            lay(x)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(time_events(step, steps, stream), world)
    # routing skew: rows per expert in layer 0 on this rank's tokens
    _, idx, _ = layers[0].topk(layers[0].logits(x))
    per_expert = torch.bincount(idx.reshape(-1), minlength=E).double()
    res = {"layers": n_layers, "tokens_per_gpu": T, "routing_bias": "zipf(1.1) over a seeded expert ranking",
           "inputs": "the same seeded tokens into every layer", "ms_per_step": round(ms, 3),
           "tokens_per_s": round(world * T / (ms * 1e-3), 1), "ms_per_layer": round(ms / n_layers, 4),
           "experts_per_gpu": E // world,
           "placement": ("experts renumbered per layer for equal rank loads by a calibration batch's slot counts"
                         if balance and world > 1 else "contiguous blocks of expert ids"),
           "expert_rows_max_over_mean_layer0": round(float(per_expert.max() / per_expert.mean()), 3)}
    if world > 1:
        sends = torch.stack([lay.last_counts[0] for lay in layers]).to(torch.float64)       # [L, world] slots sent
        toks = torch.stack([lay.last_counts[1] for lay in layers]).to(torch.float64)        # [L, world] token rows
        recv = sends.clone()
        torch.distributed.all_reduce(recv)
        imb = recv.max(dim=1).values / recv.mean(dim=1)
        moved = (toks.sum(1) - toks[:, rank]) + (sends.sum(1) - sends[:, rank])             # rows out + rows back
        mx = torch.tensor([float(moved.sum()) * H * 2], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        res.update(recv_rows_max_over_mean_mean=round(float(imb.mean()), 4),
                   recv_rows_max_over_mean_max=round(float(imb.max()), 4),
                   nvlink_bytes_per_step_per_gpu_max=int(mx.item()))
        torch.cuda.synchronize()
        barrier(world)
        for lay in layers[1:]:
            lay.close()
        layers[0].close()
    del layers
    torch.cuda.empty_cache()
    return res


def profile_case(case, dev):
    """Small cases for ncu captures (one layer of the bench workload):
    gu / dn  two launches of the routed gate/up or down grouped GEMM (its real routing), nothing
             else of the grouped-GEMM kind (`-k regex:grouped_gemm -s 1 -c 1` takes the second);
             before them one router logits GEMM (`-k regex:gemm_bf16_tma -c 1`);
    dec      four decode calls at M=1 (`-k regex:decode_stream -s 2 -c 1` takes the third);
    ep       three calls of the expert-parallel layer with the peer exchange on one rank
             (every kernel of the p2p path, the exchange kept on this GPU);
    w8       four W8A16 projections at M=1 (K=2048, N=5120; `-k regex:w8a16 -s 2 -c 1`);
    w8s      four at M=16, the split-K tensor-core GEMM and its reduce (`-s 4 -c 4` takes the last two)."""
    from fnx import synth
    from fnx.engine import EPI_PLAIN, EPI_SWIGLU_F32, _grouped_w4
    if case in ("w8", "w8s"):
        from fnx.engine import DenseW8
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        q = torch.randint(-127, 128, (5120, 2048), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
        sc = (torch.randn(5120, 1, generator=g, device=dev).abs_() * 0.01).to(torch.bfloat16)
        w = DenseW8(q, sc)
        x = torch.randn(1 if case == "w8" else 16, 2048, generator=g, device=dev).to(torch.bfloat16)
        for _ in range(4):
            w(x)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    lay = make_layers(1, dev)[0]
    if case == "dec":
        x = synth.make_tokens(1, H, seed=3, device=dev)
        for _ in range(4):
            lay.decode(x)
        torch.cuda.synchronize()
        print(json.dumps({"profile_case": case, "ok": True}))
        return
    if case == "ep":
        from fnx.ep import ExpertParallelMoE
        ep = ExpertParallelMoE.from_layer(lay, 0, 1, transport="p2p")
        x = synth.make_tokens(T_PREFILL, H, seed=1000, device=dev)
        for _ in range(3):
            out = ep(x)
        torch.cuda.synchronize()
        ok = bool(torch.equal(out.view(torch.int16), lay.prefill(x).view(torch.int16)))
        ep.close()
        print(json.dumps({"profile_case": case, "ok": ok}))
        return
    x = synth.make_tokens(T_PREFILL, H, seed=1000, device=dev)
    _, idx, _ = lay.topk(lay.logits(x))
    order, _, ends = lay.permute(idx)
    M = T_PREFILL * K_TOP
    if case == "gu":
        out = torch.empty(M, I, dtype=torch.bfloat16, device=dev)

        def fn():
            _grouped_w4(x, lay.gu_t, ends, out, E=E, M=M, K=H, Nw=2 * I, epilogue=EPI_SWIGLU_F32, row_index=order,
                        index_div=K_TOP)
    else:
        a_in = synth.make_tokens(M, I, seed=4, device=dev)
        out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)

        def fn():
            _grouped_w4(a_in, lay.dn_t, ends, out, E=E, M=M, K=I, Nw=H, epilogue=EPI_PLAIN)
    fn()
    fn()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "ok": True}))


def bench_decode(dev, nl=16, iters=20):
    from fnx import synth
    layers = make_layers(nl, dev, seed0=200)
    stream = torch.cuda.current_stream(dev)
    res = {}
    pk, src = peaks()
    for M in (1, 4):
        xs = [synth.make_tokens(M, H, seed=300 + i, device=dev) for i in range(nl)]
        for i in range(nl):
            layers[i].decode(xs[i])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = [layers[i].decode(xs[i]) for i in range(nl)]
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        ms = time_events(g.replay, iters, stream)
        us = ms * 1e3 / nl
        U = statistics.mean(int(torch.unique(o[2]).numel()) for o in outs)
        nbytes = decode_bytes(U, M)
        gbs = nbytes / (us * 1e-6) / 1e9
        res[f"M{M}"] = {"us_per_layer": round(us, 3), "distinct_experts": U, "bytes_per_layer": int(nbytes),
                        "achieved_gbs": round(gbs, 1), "frac_hbm": round(gbs / pk["hbm_gbs"], 4)}
        del g
    res["hbm_peak_gbs"] = pk["hbm_gbs"]
    res["peak_source"] = src
    res["layers_in_rotation"] = nl
    return res


def bench_w8(dev, nw=16, iters=10):
    """The W8A16 concatenated dense projection (qkv+z fused: K=2048, N=5120, per-channel
    int8 weights, bf16 scales |N(0, 0.01)|) at M = 1, 16, 256, 4096.  16 distinct weight
    sets (168 MB, beyond L2) are called in turn inside one CUDA graph; the time per call is
    the graph's time over its 16 calls."""
    from fnx.engine import DenseW8
    K, N = 2048, 5120
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    mats = []
    for _ in range(nw):
        q = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
        sc = (torch.randn(N, 1, generator=g, device=dev).abs_() * 0.01).to(torch.bfloat16)
        mats.append(DenseW8(q, sc))
    pk, src = peaks()
    stream = torch.cuda.current_stream(dev)
    res = {"shape": {"K": K, "N": N, "weights": "int8 per output channel"}, "peak_source": src}
    for M in (1, 16, 256, 4096):
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        for w in mats:
            w(x)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for w in mats:
                w(x)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        ms = time_events(gr.replay, iters, stream) / nw
        nbytes = K * N + 2 * N + 2 * M * K + 2 * M * N
        flops = 2 * M * K * N
        gbs = nbytes / (ms * 1e-3) / 1e9
        tfl = flops / (ms * 1e-3) / 1e12
        r = {"us": round(ms * 1e3, 2), "achieved_gbs": round(gbs, 1), "achieved_tflops": round(tfl, 1)}
        if M <= 16:
            r.update(bound="hbm", frac=round(gbs / pk["hbm_gbs"], 4))
        else:
            r.update(bound="tensor", frac=round(tfl / pk["bf16_tflops"], 4))
        res[f"M{M}"] = r
        del gr
    return res


def bench_apply(dev, ncalls=16, iters=20):
    """ExpW4.apply at M=1, the reference's drop-in decode entry (one token times its top-10
    experts of the E=512 gate/up bank, K=H=2048, N=2I=1024).  16 calls with different expert
    sets (178 MB of tile blocks, beyond L2) run in one CUDA graph; the expert-id path (the
    experts read in place) is timed beside the earlier form that copied the selected tile
    blocks out first (index_select, then the GEMM on the copy)."""
    from fnx.engine import ExpW4, EPI_PLAIN, _grouped_w4
    from fnx import _lib
    K, N, G = H, 2 * I, H // GS
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    w4 = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, K, N // 8), generator=g, device=dev, dtype=torch.int32)
    sc = (torch.rand(E, G, N, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    ex = ExpW4.from_scales(w4, sc, GS)
    del w4, sc
    ex.tiles()
    ex.w4 = ex._scales = None          # only the tile blocks are read
    ids = [torch.randperm(E, generator=g, device=dev)[:K_TOP].contiguous() for _ in range(ncalls)]
    x = torch.randn(1, K, generator=g, device=dev).to(torch.bfloat16)
    ends = torch.arange(1, K_TOP + 1, device=dev, dtype=torch.int64)
    rows = torch.zeros(K_TOP, device=dev, dtype=torch.int64)
    outc = torch.empty(K_TOP, N, dtype=torch.bfloat16, device=dev)

    def copied(i):
        sel = ex.tiles().index_select(0, ids[i]).contiguous()
        _grouped_w4(x, sel, ends, outc, E=K_TOP, M=K_TOP, K=K, Nw=N, epilogue=EPI_PLAIN, row_index=rows)

    stream = torch.cuda.current_stream(dev)
    pk, src = peaks()
    per_expert = int(_lib.lib().fnx_w4_tiles_bytes(1, K, N))
    nbytes = K_TOP * per_expert + 2 * K + 2 * K_TOP * N
    res = {"M": 1, "experts": K_TOP, "K": K, "N": N, "bytes_per_call": nbytes, "peak_source": src}
    for name, fn in (("in_place", lambda i: ex.apply(x, ids[i])), ("copy_then_gemm", copied)):
        for i in range(ncalls):
            fn(i)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for i in range(ncalls):
                fn(i)
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        us = time_events(gr.replay, iters, stream) * 1e3 / ncalls
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"us": round(us, 2), "achieved_gbs": round(gbs, 1), "frac_hbm": round(gbs / pk["hbm_gbs"], 4)}
        del gr
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-stack", action="store_true", help="skip the 48-layer expert-parallel stack")
    ap.add_argument("--cpu-sample", type=int, default=T_PREFILL,
                    help="tokens per CPU-baseline sample (both arms; default the whole T=4096 batch)")
    ap.add_argument("--profile-case", choices=["gu", "dn", "dec", "ep", "w8", "w8s"], default=None,
                    help="run only a small case for ncu captures (see profile_case)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    config = {"workload": "moe_layer_prefill_T4096", "tokens_per_gpu": T_PREFILL, "H": H, "I": I, "E": E,
              "top_k": K_TOP, "w4_group": GS, "shared_expert": "W4, sigmoid gate",
              "l2": "inputs larger than L2 (0.83 GB weights per layer, 2-layer rotation)",
              "execution": "one CUDA graph per layer call (MoELayer.capture), replayed"}

    if args.impl == "reference":
        if rank != 0:
            return
        steps = []
        for s in range(args.warmup + args.steps):
            r = cpu_baseline(sample_tokens=args.cpu_sample, seed=s % 2)
            if s >= args.warmup:
                steps.append(r["value"])
        v = statistics.median(steps)
        r["value"] = v
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * args.cpu_sample / v,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic", "config": config, "cpu_baseline": r,
                          "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # pinned host buffers on the GPU's NUMA node: the GPU part of the run is bound to the CPUs
    # local to this rank's GPU; the CPU baseline afterwards gets every CPU back
    from fnx.hostmem import bind_to_device
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_device(dev)
    import __graft_entry__
    __graft_entry__.build()
    if args.profile_case:
        profile_case(args.profile_case, dev)
        return

    r = bench_prefill(args, world, rank, dev)
    stack = None if args.no_stack else bench_ep_stack(args, world, rank, dev)
    dec = None if (args.no_decode or world > 1) else bench_decode(dev)
    w8 = None if (args.no_decode or world > 1) else bench_w8(dev)
    app = None if (args.no_decode or world > 1) else bench_apply(dev)
    os.sched_setaffinity(0, all_cpus)
    cpu = cpu_baseline_median(args.cpu_sample) if (rank == 0 and world == 1) else None
    if rank == 0:
        line = {"metric": METRIC, "value": round(r["value"], 1), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms"], 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded; shapes/distributions of the workload definition)",
                "config": dict(config, parallelism=f"ep{world}" if world > 1 else "single GPU",
                               **({"expert_parallel": r["ep"]} if r["ep"] else {})),
                **({"ep_bit_identical": r["ep"]["bit_identical_to_one_gpu"]} if r["ep"] else {}),
                "clocks": r["clocks"], "e2e": dict(r["e2e"], numa=numa), "gpu_launches": r["gpu_launches"],
                "roofline": r["roofline"], "layer_tflops": round(r["layer_tflops"], 1),
                "router_gemm": r["router_gemm"], "ep_stack": stack, "decode": dec, "w8a16": w8, "expw4_apply": app,
                "cpu_baseline": cpu}
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
