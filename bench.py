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

Multi-GPU (torchrun): each rank runs the same per-GPU workload on its own GPU
(weak scaling, no collective on the data path; expert parallelism is not in
this benchmark yet), timed on the device and reduced with a max over ranks.
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
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
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
def run_ours(args, world, rank, local):
    from moe_fused_inference_b200.layer import MoELayer, random_layer_weights

    dev = torch.device("cuda", local if world > 1 else 0)
    T = args.tokens
    layers = [MoELayer(random_layer_weights(E, H, MI, 0.02, seed=1000 * rank + l, device=dev), TOPK)
              for l in range(N_LAYERS)]
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    X = torch.randn((N_LAYERS, T, H), generator=g, device=dev).bfloat16()
    out = torch.empty((N_LAYERS, T, H), dtype=torch.float32, device=dev)
    topi = torch.empty((N_LAYERS, T, TOPK), dtype=torch.int32, device=dev)
    topw = torch.empty((N_LAYERS, T, TOPK), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(N_LAYERS)]
    for row in evs:
        for e in row:
            e.record(stream)  # creates the event handles before the library records them

    def step(with_events):
        for l in range(N_LAYERS):
            layers[l](X[l], out=out[l], topi=topi[l], topw=topw[l],
                      events=evs[l] if with_events else None)

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize(dev)

    # One step (48 layer calls) is captured in a CUDA graph and replayed:
    # decode serving runs graphs, and replay removes the host's per-launch cost
    # from the device-side measurement.  The timed graph has no stage events
    # (each event node costs the timeline ~2-3 us); a second graph with the
    # stage events is replayed once afterwards for the per-kernel breakdown.
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    graph_ev = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        step(True)  # warm the capture stream
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(graph, stream=cap):
            step(False)
        with torch.cuda.graph(graph_ev, stream=cap):
            step(True)
    stream.wait_stream(cap)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)

    # ---- device-resident timed region ----
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1)
    ms_max = max_over_ranks(ms, world)
    ms_per_step = ms_max / args.steps
    tokens = T * N_LAYERS * args.steps * world
    value = tokens / (ms_max / 1e3)

    # ---- per-stage times (graph with stage events, replayed after the timed region) ----
    graph_ev.replay()
    torch.cuda.synchronize(dev)
    stage = [0.0] * 5
    for l in range(N_LAYERS):
        for i in range(5):
            stage[i] += evs[l][i].elapsed_time(evs[l][i + 1])
    uniq = sum(int(torch.unique(topi[l]).numel()) for l in range(N_LAYERS))

    # ---- roofline of the dominant kernel (tensor-core expert GEMMs: gate/up + down) ----
    peak, peak_kind = measured_peaks()
    gemm_ms = stage[2] + stage[3]  # per step, summed over the 48 layer calls
    w_bytes = uniq * EXPERT_BYTES  # per step
    achieved = w_bytes / (gemm_ms / 1e3) / 1e9
    layer_ms = ms_per_step
    layer_bytes = (uniq * EXPERT_BYTES + N_LAYERS * (ROUTER_BYTES + T * H * 2 + T * H * 4 + T * TOPK * 8))
    traffic = committed_traffic()

    del graph, graph_ev
    # ---- e2e through the public API with host buffers (plain per-call launches) ----
    Xh = X.cpu().pin_memory()
    Oh = torch.empty((N_LAYERS, T, H), dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)
    barrier(world)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        Xd.copy_(Xh, non_blocking=True)
        for l in range(N_LAYERS):
            layers[l](Xd[l], out=out[l], topi=topi[l], topw=topw[l])
        Oh.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = tokens / (e2e_ms / 1e3)

    if rank != 0:
        return
    line = {
        "metric": "MXFP4 MoE layer tokens/s (decode)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"decode MoE layer, T={T} tokens/GPU, H=2048, E=128, top-8, Mi=768",
                   "step": f"T tokens through {N_LAYERS} MoE layers with distinct weights, "
                           "replayed as one captured CUDA graph (e2e: plain API calls)",
                   "global_batch": T * world, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: 48 distinct layer weight sets (15.4 GB) per step",
                   "unique_experts_per_layer": uniq / N_LAYERS},
        "gpu_launches": 6 * N_LAYERS * args.steps,  # quant, route, gather, gate/up, down, combine
        "roofline": {"bound": "hbm", "kernel": "moe_tc_kernel (gate/up + down launches)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind,
                     "algorithmic_bytes_per_step": w_bytes,
                     "traffic": (traffic or {}).get("bytes_per_layer_call"),
                     "traffic_source": (traffic or {}).get("source"),
                     "layer": {"achieved": layer_bytes / (layer_ms / 1e3) / 1e9,
                               "frac": layer_bytes / (layer_ms / 1e3) / 1e9 / peak,
                               "stage_ms_per_step": dict(zip(
                                   ["route", "gather", "gate_up", "down", "combine"], stage))}},
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(Xh.numel() * Xh.element_size()),
                "d2h_bytes_per_step": int(Oh.numel() * Oh.element_size())},
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        cpu_layer = make_cpu_layer(layers[0].w)
        tok_s, n, _ = time_cpu_layer(cpu_layer, T, seconds=args.cpu_sample_s)
        line["cpu_baseline"] = {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"{n} layer calls x T={T} tokens, torch CPU bf16 with "
                                          "layer 0's weights dequantised (runtime/model_runner.py:99-132 ported)"}
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
