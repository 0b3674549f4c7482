#!/usr/bin/env python3
"""Benchmark of the MXFP4 grouped-MoE expert path on B200.

Workload (the headline metric's configuration): one
Qwen3-30B-A3B-shaped MoE layer (H = 2048, 128 experts, top-8, Mi = 768,
SwiGLU experts, MXFP4 weights N(0, 0.02) quantised on the device) at decode
size T tokens per GPU (default 64), bf16 N(0, 1) activations quantised on the
fly, routing from a random N(0, 0.02) router (near-uniform load).

A *step* is one decode step's worth of MoE work: the T tokens pass through 48
MoE layers, each with its own weights (48 x 320.9 MB = 15.4 GB resident), so
consecutive layer calls never find their weights in the 126 MB L2.  ``value``
is MoE-layer token throughput: tokens x layer calls / second, over all GPUs.

Arms:
  default            this library, inputs resident in HBM (``value``) and end to
                     end through ``MoELayer.forward`` with pinned host buffers
                     (``e2e``: H2D of the step's activations, D2H of its outputs);
  --impl reference   the reference's CPU dequantise-then-matmul path
                     (runtime/model_runner.py:99-132, ported in oracle/moe_ref.py)
                     on the host cores, same metric and config, rank 0 only.

Multi-GPU (torchrun, N ranks): expert parallelism (BASELINE config 5's
sharding) — each rank holds 128/N experts of every layer and the full router,
routes its own T tokens, and dispatch / combine are NCCL all-to-alls over
NVLink (moe_fused_inference_b200/ep.py).  Per-GPU tokens stay at T (weak
scaling); the step is timed on the device and reduced with a max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, MI, E, TOPK = 2048, 768, 128, 8
N_LAYERS = 48
EXPERT_BYTES = 3 * (MI * H // 2 + MI * H // 32)  # 2,506,752 B packed gate+up+down
ROUTER_BYTES = E * (H // 2 + H // 32)            # 139,264 B (MXFP4 router)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=64, help="decode tokens per GPU (T)")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="distinct MoE layers per step (48 = the model; fewer for profiling)")
    ap.add_argument("--workload", choices=["decode", "prefill", "linear"], default="decode",
                    help="decode (BASELINE config 2, the headline), prefill (config 3: "
                         "T = 16384 by default, Zipf(1.2)-skewed routing) or linear (the "
                         "static decode projections and lm_head through lin_pq)")
    ap.add_argument("--zipf-alpha", type=float, default=0.5,
                    help="prefill: scale of the Zipf(1.2) per-expert logit bias")
    ap.add_argument("--ep-zipf", action="store_true",
                    help="expert parallelism: add the Zipf(1.2) logit bias (--zipf-alpha) to "
                         "the router, for the skewed-load scaling report")
    ap.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                    help="multi-GPU token exchange: peer-memory stores fused into the kernels "
                         "(p2p) or two NCCL all_to_all_single calls (nccl)")
    ap.add_argument("--no-graph", action="store_true",
                    help="time plain launches instead of a captured CUDA graph")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample-s", type=float, default=15.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_gpu{gpu_index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            # sampling must be live before the timed region starts
            t0 = time.time()
            while time.time() - t0 < 5.0 and self.proc.poll() is None:
                self.f.flush()
                if os.path.getsize(self.path) > 0:
                    break
                time.sleep(0.02)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            p = [c.strip() for c in line.split(",")]
            if len(p) < 9:
                continue
            try:
                rows.append((float(p[1]), float(p[2]), float(p[3]), p[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return None
    return None


# ---------------------------------------------------------------------------
def make_cpu_layer(layer_weights=None):
    """The reference's CPU dequantise-then-matmul MoE layer (oracle/moe_ref.py,
    a port of runtime/model_runner.py:99-132) with bf16 experts dequantised up
    front (outside any timing, like the reference's expert cache)."""
    from oracle import moe_ref

    if layer_weights is not None:
        from oracle import mxfp4 as mx
        w = layer_weights
        c = lambda t: t.cpu().numpy()
        deq = lambda p, s, k: torch.from_numpy(mx.dequantize_rows(p, s, k)).bfloat16()
        gp, gs, up, us, dp, ds = (c(w.gate_wp), c(w.gate_sc), c(w.up_wp), c(w.up_sc),
                                  c(w.down_wp), c(w.down_sc))
        wg = [deq(gp[e], gs[e], H) for e in range(E)]
        wu = [deq(up[e], us[e], H) for e in range(E)]
        wd = [deq(dp[e], ds[e], MI) for e in range(E)]
    else:
        g = torch.Generator().manual_seed(0)
        mk = lambda n, k: moe_ref.quant_dequant_bf16((torch.randn(n, k, generator=g) * 0.02).bfloat16())
        wg = list(mk(E * MI, H).view(E, MI, H).unbind(0))
        wu = list(mk(E * MI, H).view(E, MI, H).unbind(0))
        wd = list(mk(E * H, MI).view(E, H, MI).unbind(0))
    gr = torch.Generator().manual_seed(1)
    wr = (torch.randn(E, H, generator=gr) * 0.02).bfloat16()
    return moe_ref.CpuMoELayer.from_bf16(wg, wu, wd, wr, top_k=TOPK)


def time_cpu_layer(layer, T, seconds=None, calls=None):
    """Time layer.forward on T tokens for about ``seconds`` or exactly ``calls``
    calls; returns (tokens/s, calls, seconds per call)."""
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).bfloat16()
    layer.forward(x)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        layer.forward(x)
        n += 1
        el = time.perf_counter() - t0
        if (calls is not None and n >= calls) or (calls is None and (el >= seconds or n >= 1000)):
            break
    return T * n / el, n, el / n


def run_reference(args, world, rank):
    """--impl reference: rank 0 times the reference's CPU path; other ranks exit."""
    if rank != 0:
        barrier(world)
        return
    T = args.tokens
    layer = make_cpu_layer()
    x = torch.randn(T, H).bfloat16()
    for _ in range(max(args.warmup, 1)):
        layer.forward(x)
    t0 = time.perf_counter()
    layer.forward(x)
    per_call = time.perf_counter() - t0
    steps = max(1, min(args.steps, int(120.0 / max(per_call, 1e-6))))
    tok_s, n, per = time_cpu_layer(layer, T, calls=steps)
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": "MXFP4 MoE layer tokens/s (decode)", "value": tok_s,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
        "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (dequantised MXFP4 weights)", "data": "synthetic",
        "config": {"workload": f"decode MoE layer, T={T} tokens, H=2048, E=128, top-8, Mi=768",
                   "step": "one MoE layer call on the host CPU", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} layer calls x T={T} tokens, torch CPU bf16 "
                                   "(runtime/model_runner.py:99-132 ported)"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    barrier(world)


# ---------------------------------------------------------------------------
def timed_region(args, world, dev, stream, step):
    """Clock-sampled, barrier-bracketed device timing of args.steps calls of
    step(); returns (max-over-ranks ms, clocks)."""
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    return max_over_ranks(t0.elapsed_time(t1), world), clocks


def capture(dev, stream, fn, warm):
    """Capture fn() into a CUDA graph on a side stream (after `warm` eager calls)."""
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(graph, stream=cap):
            fn()
    stream.wait_stream(cap)
    torch.cuda.synchronize(dev)
    return graph


def cpu_baseline(args, T, weights):
    cpu_layer = make_cpu_layer(weights)
    tok_s, n, _ = time_cpu_layer(cpu_layer, T, seconds=args.cpu_sample_s)
    return {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} layer calls x T={T} tokens, torch CPU bf16 with layer 0's weights "
                      "dequantised (runtime/model_runner.py:99-132 ported)"}


def run_prefill(args, world, rank, local):
    """one prefill-sized MoE layer call per layer (T tokens,
    default 16384) with Zipf(1.2)-skewed routing; FLOP rate of the layer
    against the dense FP4 tensor peak.  Single GPU; under torchrun every rank
    runs its own copy (weak scaling)."""
    from moe_fused_inference_b200.layer import MoELayer, random_layer_weights
    from oracle import mxfp4 as mx

    dev = torch.device("cuda", local if world > 1 else 0)
    T = args.tokens if args.tokens != 64 else 16384
    NL = args.layers if args.layers != N_LAYERS else 4
    bias = torch.from_numpy(mx.zipf_bias(E, args.zipf_alpha, seed=3))
    layers = [MoELayer(random_layer_weights(E, H, MI, 0.02, seed=l, device=dev), TOPK,
                       logit_bias=bias) for l in range(NL)]
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
    out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
    topi = torch.empty((NL, T, TOPK), dtype=torch.int32, device=dev)
    topw = torch.empty((NL, T, TOPK), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for l in range(NL):
            layers[l](X[l], out=out[l], topi=topi[l], topw=topw[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ms, clocks = timed_region(args, world, dev, stream, step)
    ms_per_step = ms / args.steps
    flop_tok = TOPK * (2 * H * 2 * MI + 2 * MI * H) + 2 * H * E   # experts + router
    flops = flop_tok * T * NL
    tflops = flops / (ms_per_step / 1e3) / 1e12
    counts = torch.bincount(topi[0].flatten().long(), minlength=E).float()
    fp4_peak = 9000.0  # dense MXFP4 tensor peak, nominal (no measured FP4 figure on this pool)
    # algorithmic bytes of one layer call: every expert with tokens once, the
    # MXFP4 router, bf16 in, fp32 out, ids and weights
    hbm_bytes = (int((counts > 0).sum()) * EXPERT_BYTES + ROUTER_BYTES + T * H * 2 + T * H * 4
                 + T * TOPK * 8)
    hbm_gbs = hbm_bytes / (ms_per_step / NL / 1e3) / 1e9
    hbm_peak, hbm_kind = measured_peaks()

    # ---- dense mxfp4_linear of the attention projections at T tokens (config 3):
    # lin_pq on pre-quantised activations (the GEMM incl. its scale re-layout)
    from moe_fused_inference_b200 import fp4_ext
    from moe_fused_inference_b200.layer import quantize_rows
    dec = fp4_ext.get_decode_ext()
    dense = {}
    del X, out
    torch.cuda.empty_cache()
    for name, (n_out, k_in) in {"q": (4096, 2048), "k": (512, 2048), "v": (512, 2048),
                                "o": (2048, 4096)}.items():
        wq, wsc = quantize_rows((torch.randn((n_out, k_in), generator=g, device=dev) * 0.02).bfloat16())
        xq, xsc = quantize_rows(torch.randn((T, k_in), generator=g, device=dev).bfloat16())
        for _ in range(2):
            dec.lin_pq(xq, xsc, wq, wsc, T, n_out, k_in)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            dec.lin_pq(xq, xsc, wq, wsc, T, n_out, k_in)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / 5 * 1e3
        dense[name] = {"us": us, "tflops": 2.0 * T * n_out * k_in / us / 1e6}
        del wq, wsc, xq, xsc
    if rank != 0:
        return
    line = {
        "metric": "MXFP4 MoE layer tokens/s (prefill)", "value": T * NL * args.steps * world / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"prefill MoE layer, T={T} tokens, H=2048, E=128, top-8, Mi=768, "
                               f"Zipf(1.2) logit bias alpha={args.zipf_alpha}",
                   "step": f"{NL} MoE layers with distinct weights, plain launches",
                   "expert_load_max_over_mean": float(counts.max() / counts.mean()),
                   "experts_with_tokens": int((counts > 0).sum())},
        "gpu_launches": 5 * NL * args.steps,  # quantise, route, scatter, experts, combine
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": tflops / fp4_peak, "peak_kind": "nominal dense FP4 (no measured FP4 peak)",
                     "flops_per_layer": flop_tok * T,
                     "dense_projections": {k: {"us": v["us"], "tflops": v["tflops"],
                                               "frac": v["tflops"] / fp4_peak}
                                           for k, v in dense.items()},
                     # the other roof: at small T the weights, not the math, set the time
                     "hbm": {"bytes_per_layer": hbm_bytes, "achieved": hbm_gbs, "peak": hbm_peak,
                             "unit": "GB/s", "frac": hbm_gbs / hbm_peak, "peak_kind": hbm_kind}},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_linear(args, world, rank, local):
    """Static MXFP4 projections of a decode step through lin_pq (the lm_head,
    151936 x 2048, and the attention projections q 4096 x 2048, k/v 512 x
    2048, o 2048 x 4096) at T in {1, 8} rows: weight-stream GB/s against the
    measured HBM peak.  Each shape runs 24 calls over distinct weight copies
    (one for the 165 MB lm_head) captured in one CUDA graph, so the time is
    the kernels' and the weights come from HBM."""
    from moe_fused_inference_b200 import fp4_ext
    from moe_fused_inference_b200.layer import quantize_rows

    dev = torch.device("cuda", local if world > 1 else 0)
    dec = fp4_ext.get_decode_ext()
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    peak, peak_kind = measured_peaks()
    shapes = {"lm_head": (151936, 2048), "q": (4096, 2048), "kv": (512, 2048), "o": (2048, 4096)}
    res = {}
    stream = torch.cuda.current_stream(dev)
    for name, (n_out, k_in) in shapes.items():
        nw = 1 if name == "lm_head" else 24
        ws = [quantize_rows((torch.randn((n_out, k_in), generator=g, device=dev) * 0.02).bfloat16())
              for _ in range(nw)]
        w_bytes = n_out * (k_in // 2 + k_in // 32)
        for T in (1, 8):
            xq, xsc = quantize_rows(torch.randn((T, k_in), generator=g, device=dev).bfloat16())
            reps = 24

            def calls():
                for i in range(reps):
                    dec.lin_pq(xq, xsc, ws[i % nw][0], ws[i % nw][1], T, n_out, k_in)

            graph = capture(dev, stream, calls, 1)
            for _ in range(max(args.warmup, 1)):
                graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / (args.steps * reps) * 1e3
            res[f"{name}_T{T}"] = {"us": us, "GBps": w_bytes / us / 1e3,
                                   "frac": w_bytes / us / 1e3 / peak}
            del graph
        del ws
        torch.cuda.empty_cache()
    if rank != 0:
        return
    head = res["lm_head_T1"]
    line = {
        "metric": "MXFP4 lin_pq weight stream GB/s (decode lm_head, T=1)", "value": head["GBps"],
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["us"] * 24 / 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": "decode static projections through lin_pq: lm_head 151936x2048, "
                               "q 4096x2048, k/v 512x2048, o 2048x4096 at T in {1, 8}",
                   "step": "24 lin_pq calls in one CUDA graph"},
        "gpu_launches": 24 * args.steps,  # per shape: one kernel per lin_pq call
        "roofline": {"bound": "hbm", "achieved": head["GBps"], "peak": peak, "unit": "GB/s",
                     "frac": head["frac"], "peak_kind": peak_kind, "shapes": res},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    if args.workload == "prefill":
        return run_prefill(args, world, rank, local)
    if args.workload == "linear":
        return run_linear(args, world, rank, local)
    if world > 1:
        return run_ep(args, world, rank, local)
    from moe_fused_inference_b200.layer import MoELayer, random_layer_weights

    dev = torch.device("cuda", 0)
    T, NL = args.tokens, args.layers
    layers = [MoELayer(random_layer_weights(E, H, MI, 0.02, seed=l, device=dev), TOPK)
              for l in range(NL)]
    g = torch.Generator(device=dev).manual_seed(7)
    X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
    out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
    topi = torch.empty((NL, T, TOPK), dtype=torch.int32, device=dev)
    topw = torch.empty((NL, T, TOPK), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(NL)]
    for row in evs:
        for e in row:
            e.record(stream)  # creates the event handles before the library records them

    def step(with_events=False):
        for l in range(NL):
            layers[l](X[l], out=out[l], topi=topi[l], topw=topw[l],
                      events=evs[l] if with_events else None)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # One step (NL layer calls) is captured in a CUDA graph and replayed:
    # decode serving runs graphs, and replay removes the host's per-launch cost
    # from the device-side measurement.  The timed graph has no stage events
    # (each event node costs the timeline ~2-3 us); a second graph with the
    # stage events is replayed once afterwards for the per-kernel breakdown.
    graph = graph_ev = None
    if not args.no_graph:
        graph = capture(dev, stream, step, 1)
        graph_ev = capture(dev, stream, lambda: step(True), 0)
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize(dev)

    ms, clocks = timed_region(args, world, dev, stream, graph.replay if graph else step)
    ms_per_step = ms / args.steps
    tokens = T * NL * args.steps
    value = tokens / (ms / 1e3)

    # ---- per-stage times (stage events, after the timed region) ----
    if graph_ev is not None:
        graph_ev.replay()
    else:
        step(True)
    torch.cuda.synchronize(dev)
    stage = [0.0] * 5
    for l in range(NL):
        for i in range(5):
            stage[i] += evs[l][i].elapsed_time(evs[l][i + 1])
    uniq = sum(int(torch.unique(topi[l]).numel()) for l in range(NL))

    # ---- roofline of the dominant kernel (tensor-core expert GEMMs: gate/up + down) ----
    peak, peak_kind = measured_peaks()
    gemm_ms = stage[2] + stage[3]  # per step, summed over the NL layer calls
    w_bytes = uniq * EXPERT_BYTES  # per step
    achieved = w_bytes / (gemm_ms / 1e3) / 1e9
    layer_bytes = (uniq * EXPERT_BYTES + NL * (ROUTER_BYTES + T * H * 2 + T * H * 4 + T * TOPK * 8))
    traffic = committed_traffic()

    del graph, graph_ev
    # ---- e2e through the public API with host buffers (plain per-call launches) ----
    Xh = X.cpu().pin_memory()
    Oh = torch.empty((NL, T, H), dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)

    def e2e_step():
        Xd.copy_(Xh, non_blocking=True)
        for l in range(NL):
            layers[l](Xd[l], out=out[l], topi=topi[l], topw=topw[l])
        Oh.copy_(out, non_blocking=True)

    e2e_ms, _ = timed_region(args, world, dev, stream, e2e_step)
    e2e_value = tokens / (e2e_ms / 1e3)

    line = {
        "metric": "MXFP4 MoE layer tokens/s (decode)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"decode MoE layer, T={T} tokens/GPU, H=2048, E=128, top-8, Mi=768",
                   "step": f"T tokens through {NL} MoE layers with distinct weights, "
                           + ("plain launches" if args.no_graph else "replayed as one captured CUDA graph")
                           + " (e2e: plain API calls)",
                   "global_batch": T, "parallelism": "single GPU",
                   "l2": f"inputs larger than L2: {NL} distinct layer weight sets "
                         f"({NL * E * EXPERT_BYTES / 1e9:.1f} GB) per step",
                   "unique_experts_per_layer": uniq / NL},
        "gpu_launches": 3 * NL * args.steps,  # route (+quantise), experts (gate/up + down), combine
        "roofline": {"bound": "hbm", "kernel": "moe_experts_kernel (gate/up + down, one launch)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind,
                     "algorithmic_bytes_per_step": w_bytes,
                     "algorithmic_bytes_per_layer_call": w_bytes / NL,
                     "traffic": (traffic or {}).get("bytes_per_layer_call"),
                     "traffic_source": (traffic or {}).get("source"),
                     "layer": {"achieved": layer_bytes / (ms_per_step / 1e3) / 1e9,
                               "frac": layer_bytes / (ms_per_step / 1e3) / 1e9 / peak,
                               "stage_ms_per_step": {"route": stage[0],
                                                     "experts": stage[2] + stage[3],
                                                     "combine": stage[4]}}},
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(Xh.numel() * Xh.element_size()),
                "d2h_bytes_per_step": int(Oh.numel() * Oh.element_size())},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, T, layers[0].w)
    print(json.dumps(line), flush=True)


def run_ep(args, world, rank, local):
    """Expert-parallel step over the torchrun ranks (peer-memory exchange fused
    into the kernels, or NCCL all-to-all with --ep-transport nccl)."""
    from moe_fused_inference_b200.ep import EPMoELayer, random_shard

    dev = torch.device("cuda", local)
    T, NL = args.tokens, args.layers
    bias = None
    if args.ep_zipf:
        from oracle import mxfp4 as mx
        bias = torch.from_numpy(mx.zipf_bias(E, args.zipf_alpha, seed=3)).to(dev)
    layers = [EPMoELayer(random_shard(E, world, rank, H, MI, 0.02, seed=l, device=dev), TOPK, T,
                         transport=args.ep_transport, logit_bias=bias)
              for l in range(NL)]
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
    out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for l in range(NL):
            layers[l](X[l], out=out[l])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    graph, graph_note = None, "plain launches"
    if not args.no_graph:
        # NCCL collectives are captured with the kernels; every rank must take
        # the same path, so a capture failure anywhere makes all ranks time
        # plain launches
        import torch.distributed as dist
        err = ""
        try:
            graph = capture(dev, stream, step, 1)
        except Exception as e:  # noqa: BLE001
            graph, err = None, f"{type(e).__name__}: {e}"[:200]
        ok = torch.tensor([0.0 if graph is None else 1.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() < 1.0:
            graph = None
            graph_note = "plain launches (graph capture failed: " + (err or "on another rank") + ")"
        else:
            graph_note = "one captured CUDA graph"
            for _ in range(args.warmup):
                graph.replay()
        torch.cuda.synchronize(dev)

    ms, clocks = timed_region(args, world, dev, stream, graph.replay if graph else step)
    ms_per_step = ms / args.steps
    tokens = T * NL * args.steps * world
    value = tokens / (ms / 1e3)

    # ---- expert-compute time per step (events around the local expert part) ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(NL)]
    import torch.distributed as dist
    from moe_fused_inference_b200.ep import ep_row_bytes
    recvs = []
    for l in range(NL):
        L = layers[l]
        if L.transport == "p2p":
            L.p2p_dispatch(X[l])
            evs[l][0].record(stream)
            L.p2p_experts()  # includes the wait for the peers' dispatch
            evs[l][1].record(stream)
            L.p2p_finish(T, out[l])
            rv = torch.empty((world, T + 1, ep_row_bytes(H, TOPK)), dtype=torch.uint8, device=dev)
            L.xch.copy_recv_to(rv)
            recvs.append(rv)
        else:
            L.dispatch_prepare(X[l])
            dist.all_to_all_single(L.recv.view(-1), L.send.view(-1))
            evs[l][0].record(stream)
            L.compute()
            evs[l][1].record(stream)
            dist.all_to_all_single(L.ret_back.view(-1), L.ret.view(-1))
            L.finish(T, out[l])
            recvs.append(L.recv)
    torch.cuda.synchronize(dev)
    experts_ms = sum(a.elapsed_time(b) for a, b in evs)
    # unique local experts touched per layer on this rank
    uniq = 0
    rows_recv = 0
    for l in range(NL):
        rv = recvs[l]
        cnt = rv[:, 0, :4].contiguous().view(torch.int32)[:, 0]
        rows_recv += int(cnt.sum())
        sel = torch.cat([rv[s, 1:1 + int(cnt[s])] for s in range(world)])
        if sel.shape[0]:
            from moe_fused_inference_b200.ep import row_offsets
            _, _, so, _ = row_offsets(H, TOPK)
            ids = sel[:, so:so + 4 * TOPK].contiguous().view(torch.int32)
            uniq += int(torch.unique(ids[ids >= 0]).numel())
    w_bytes = uniq * EXPERT_BYTES
    peak, peak_kind = measured_peaks()
    achieved = w_bytes / (experts_ms / 1e3) / 1e9
    stats = torch.tensor([achieved, experts_ms, rows_recv / NL, uniq / NL], dtype=torch.float64,
                         device=dev)
    allstats = [torch.zeros_like(stats) for _ in range(world)]
    dist.all_gather(allstats, stats)
    allstats = torch.stack(allstats).cpu()
    # expert load over all ranks' tokens (layer 0's routing)
    load = torch.bincount(layers[0].topi[:T].flatten().long(), minlength=E).to(torch.float64)
    dist.all_reduce(load)
    load_max_over_mean = float(load.max() / load.mean())

    # ---- e2e: host activations in, host outputs back, plain launches ----
    if graph is not None:
        del graph
    del recvs
    Xh = X.cpu().pin_memory()
    Oh = torch.empty((NL, T, H), dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)

    def e2e_step():
        Xd.copy_(Xh, non_blocking=True)
        for l in range(NL):
            layers[l](Xd[l], out=out[l])
        Oh.copy_(out, non_blocking=True)

    e2e_ms, _ = timed_region(args, world, dev, stream, e2e_step)
    e2e_value = tokens / (e2e_ms / 1e3)
    torch.cuda.synchronize(dev)
    barrier(world)
    for L in layers:
        L.close()  # unmap the peers' memory before the process group goes away
    barrier(world)
    if rank != 0:
        return
    worst = int(torch.argmin(allstats[:, 0]))
    line = {
        "metric": "MXFP4 MoE layer tokens/s (decode)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"decode MoE layer, T={T} tokens/GPU, H=2048, E=128, top-8, Mi=768",
                   "step": f"T tokens per rank through {NL} expert-parallel MoE layers, " + (
                       "router storing rows into the owners' receive buffers over NVLink, "
                       "tcgen05 experts storing weighted sums back, rank-ordered unpack"
                       if args.ep_transport == "p2p" else
                       "route, pack, NCCL all-to-all dispatch, tcgen05 experts, all-to-all "
                       "return, unpack") + ", " + graph_note,
                   "ep_transport": args.ep_transport,
                   "routing": (f"Zipf(1.2) logit bias alpha={args.zipf_alpha}" if args.ep_zipf
                               else "near-uniform (random router)"),
                   "expert_load_max_over_mean": load_max_over_mean,
                   "global_batch": T * world, "parallelism": f"ep{world} ({E // world} experts/GPU)",
                   "l2": f"inputs larger than L2: {NL} distinct layer shards "
                         f"({NL * (E // world) * EXPERT_BYTES / 1e9:.1f} GB/GPU) per step",
                   "rows_received_per_layer": [float(v) for v in allstats[:, 2]],
                   "unique_local_experts_per_layer": [float(v) for v in allstats[:, 3]]},
        # per layer: p2p route+dispatch, scatter, experts, combine+return, unpack;
        # nccl: route, pack, header, mask, scatter, experts, combine, unpack (+ NCCL's own)
        "gpu_launches": (5 if args.ep_transport == "p2p" else 8) * NL * args.steps,
        "roofline": {"bound": "hbm", "kernel": "mfi_moe_experts (scatter, gate/up, down, combine)",
                     "achieved": float(allstats[worst, 0]), "peak": peak, "unit": "GB/s",
                     "frac": float(allstats[worst, 0]) / peak, "peak_kind": peak_kind,
                     "rank": worst, "experts_ms_per_step": float(allstats[worst, 1]),
                     "traffic": None},
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(Xh.numel() * Xh.element_size()),
                "d2h_bytes_per_step": int(Oh.numel() * Oh.element_size())},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
