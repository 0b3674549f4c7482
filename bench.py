#!/usr/bin/env python3
"""Benchmark of the MXFP4 grouped-MoE expert path on B200.

Headline (the metric's configuration): one
Qwen3-30B-A3B-shaped MoE layer (H = 2048, 128 experts, top-8, Mi = 768,
SwiGLU experts, MXFP4 weights N(0, 0.02) quantised on the device) at decode
size T tokens per GPU (default 64), bf16 N(0, 1) activations quantised on the
fly, routing from a random N(0, 0.02) router (near-uniform load).

A *step* is one decode step's worth of MoE work: the T tokens pass through 48
MoE layers, each with its own weights (48 x 320.9 MB = 15.4 GB resident), so
consecutive layer calls never find their weights in the 126 MB L2.  ``value``
is MoE-layer token throughput: tokens x layer calls / second, over all GPUs.

The same single-GPU line also carries every other configuration of the path:
  decode_sweep   T in {1, 8, 32, 64}: per-layer time, per-stage times, the
                 expert kernel's and the whole layer's HBM roofline fraction;
  prefill        BASELINE config 3: T in {2048, 16384} with Zipf(1.2)-skewed
                 routing (FP4 tensor fraction, HBM fraction, per-stage times)
                 and the dense q/k/v/o mxfp4_linear GEMMs at T = 16384;
  dropin         the reference's own call sequence, unchanged
                 (runtime/model_runner_v2.py:185-207: prequant -> lin_pq router
                 -> host softmax/top-k -> .tolist() -> host pointer tables ->
                 moe_gateup -> moe_down -> moe_combine) through the drop-in
                 fp4_ext module, with its kernel-only HBM roofline;
  cpu_baseline   the reference's CPU dequantise-then-matmul layer
                 (runtime/model_runner.py:99-132, ported in oracle/moe_ref.py)
                 at T = 64 and at config 1's T = 4.

Arms:
  default            this library, inputs resident in HBM (``value``) and end to
                     end through ``MoELayer.forward`` with pinned host buffers
                     (``e2e``: H2D of the step's activations, D2H of its outputs);
  --impl reference   the reference's CPU dequantise-then-matmul path on the host
                     cores, same metric and config, rank 0 only.

Multi-GPU (torchrun, N ranks): expert parallelism (BASELINE config 5's
sharding) — each rank holds 128/N experts of every layer and the full router,
routes its own T tokens, and the token exchange runs over peer memory: the
router stores each token's row straight into the owning ranks' receive
buffers over NVLink and the experts store their weighted sums straight back
(the default, ``--ep-transport p2p``), or two NCCL all-to-alls
(``--ep-transport nccl``).  Per-GPU tokens stay at T (weak scaling); the step
is timed on the device and reduced with a max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, MI, E, TOPK = 2048, 768, 128, 8
N_LAYERS = 48
EXPERT_BYTES = 3 * (MI * H // 2 + MI * H // 32)  # 2,506,752 B packed gate+up+down
ROUTER_BYTES = E * (H // 2 + H // 32)            # 139,264 B (MXFP4 router)
FLOP_TOKEN = TOPK * (2 * H * 2 * MI + 2 * MI * H) + 2 * H * E  # experts + router
FP4_PEAK = 9000.0  # dense MXFP4 tensor TFLOP/s, nominal (no measured FP4 figure on this pool)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=64, help="decode tokens per GPU (T)")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="distinct MoE layers per step (48 = the model; fewer for profiling)")
    ap.add_argument("--workload", choices=["decode", "prefill", "linear", "model", "dropin",
                                           "attn"],
                    default="decode",
                    help="decode (BASELINE config 2, the headline, with every other "
                         "configuration in the same line), prefill (config 3 alone: T = 16384 "
                         "by default, Zipf(1.2)-skewed routing), linear (the static decode "
                         "projections and lm_head through lin_pq), model (config 4: greedy "
                         "decode of the 48-layer synthetic model at batch 1 / 16 / 64, each "
                         "step one CUDA graph), dropin (the decode line's drop-in block "
                         "alone: the reference's call sequence at T = 1 and 16 over --layers "
                         "layers) or attn (the decode line's attention block alone)")
    ap.add_argument("--headline-only", action="store_true",
                    help="decode: skip the sweep, prefill, drop-in and T=4 blocks")
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
    ap.add_argument("--cpu-sample-s", type=float, default=12.0,
                    help="seconds of CPU work for each cpu_baseline sample")
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
    """nvidia-smi clocks/throttle sampling during the timed region (samples
    go to a temporary file that is removed afterwards)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"mfi_clocks_gpu{gpu_index}_", suffix=".csv")
        os.close(fd)

    def start(self):
        try:
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
            self._remove()
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
        self._remove()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded)}

    def _remove(self):
        try:
            os.remove(self.path)
        except OSError:
            pass


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


def decode_layer_bytes(uniq_per_layer: float, T: int) -> float:
    """Algorithmic HBM bytes of one decode layer call: every expert with
    tokens once, the MXFP4 router, bf16 in, fp32 out, ids and weights."""
    return uniq_per_layer * EXPERT_BYTES + ROUTER_BYTES + T * H * 2 + T * H * 4 + T * TOPK * 8


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
        if (calls is not None and n >= calls) or (calls is None and (el >= seconds or n >= 2000)):
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
    line = {
        "impl": "reference", "metric": "MXFP4 MoE layer tokens/s (decode)", "value": tok_s,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": n, "warmup": args.warmup,
        "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (dequantised MXFP4 weights)", "data": "synthetic",
        "config": {"workload": f"decode MoE layer, T={T} tokens, H=2048, E=128, top-8, Mi=768",
                   "step": "one MoE layer call on the host CPU", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "cpu_count": os.cpu_count(), "kind": "port",
                         "sample": f"{n} layer calls x T={T} tokens, torch CPU bf16 "
                                   "(runtime/model_runner.py:99-132 ported)"},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    barrier(world)


# ---------------------------------------------------------------------------
def timed_region(args, world, dev, stream, step, steps=None):
    """Clock-sampled, barrier-bracketed device timing of `steps` (default
    args.steps) calls of step(); returns (max-over-ranks ms, clocks)."""
    steps = args.steps if steps is None else steps
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    return max_over_ranks(t0.elapsed_time(t1), world), clocks


def event_time(dev, stream, step, steps):
    """Device time (ms) of `steps` calls of step() between two events."""
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1)


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


def overlapped_e2e_step(dev, layers, Xh, Xd, Oh, out, call, stream, graph=True):
    """One end-to-end step: per layer l, the H2D copy of Xh[l] on a copy
    stream, the layer (call(l, Xd[l], out[l])) once its input is in, the D2H
    copy of out[l] on a second copy stream once the layer is done; captured
    as one CUDA graph when `graph` (falls back to plain launches if capture
    fails).  Returns (step function, note)."""
    NL = len(layers)
    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(NL)]
    ev_done = [torch.cuda.Event() for _ in range(NL)]

    def body():
        main = torch.cuda.current_stream(dev)
        cs_in.wait_stream(main)
        cs_out.wait_stream(main)
        with torch.cuda.stream(cs_in):
            for l in range(NL):
                Xd[l].copy_(Xh[l], non_blocking=True)
                ev_in[l].record(cs_in)
        for l in range(NL):
            main.wait_event(ev_in[l])
            call(l, Xd[l], out[l])
            ev_done[l].record(main)
            cs_out.wait_event(ev_done[l])
            with torch.cuda.stream(cs_out):
                Oh[l].copy_(out[l], non_blocking=True)
        main.wait_stream(cs_in)
        main.wait_stream(cs_out)

    if graph:
        try:
            g = capture(dev, stream, body, 1)
            return g.replay, "per-layer H2D / D2H overlapping the layers, one CUDA graph"
        except Exception:  # noqa: BLE001 - fall back to plain launches
            torch.cuda.synchronize(dev)
    return body, "per-layer H2D / D2H overlapping the layers, plain launches"


def cpu_baseline(args, T, cpu_layer):
    tok_s, n, _ = time_cpu_layer(cpu_layer, T, seconds=args.cpu_sample_s)
    return {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "cpu_count": os.cpu_count(), "kind": "port",
            "sample": f"{n} layer calls x T={T} tokens, torch CPU bf16 with layer 0's weights "
                      "dequantised (runtime/model_runner.py:99-132 ported)"}


# ---------------------------------------------------------------------------
class DecodePoint:
    """The decode step at T tokens: NL layer calls of the fused layer with
    distinct weights, captured in one CUDA graph, plus a second graph that
    records the library's stage events for the per-kernel breakdown."""

    def __init__(self, layers, T, dev, stream, seed=7, graph=True):
        self.layers, self.T, self.dev, self.stream = layers, T, dev, stream
        NL = len(layers)
        g = torch.Generator(device=dev).manual_seed(seed)
        self.X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
        self.out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
        self.topi = torch.empty((NL, T, TOPK), dtype=torch.int32, device=dev)
        self.topw = torch.empty((NL, T, TOPK), dtype=torch.float32, device=dev)
        self.evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(NL)]
        for row in self.evs:
            for e in row:
                e.record(stream)  # creates the event handles before the library records them
        self.graph = self.graph_ev = None
        self.use_graph = graph

    def step(self, with_events=False):
        for l, layer in enumerate(self.layers):
            layer(self.X[l], out=self.out[l], topi=self.topi[l], topw=self.topw[l],
                  events=self.evs[l] if with_events else None)

    def prepare(self, warmup):
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize(self.dev)
        # The timed graph has no stage events (each event node costs the
        # timeline ~2-3 us); the graph with the stage events is replayed once
        # afterwards for the per-kernel breakdown.
        if self.use_graph:
            self.graph = capture(self.dev, self.stream, self.step, 1)
            self.graph_ev = capture(self.dev, self.stream, lambda: self.step(True), 0)
            for _ in range(warmup):
                self.graph.replay()
            torch.cuda.synchronize(self.dev)

    def run(self):
        (self.graph.replay if self.graph is not None else self.step)()

    def breakdown(self):
        """Per-step stage times (ms, summed over the layers) and unique experts
        per layer, from one replay of the stage-event graph."""
        if self.graph_ev is not None:
            self.graph_ev.replay()
        else:
            self.step(True)
        torch.cuda.synchronize(self.dev)
        NL = len(self.layers)
        stage = [0.0] * 5
        for l in range(NL):
            for i in range(5):
                stage[i] += self.evs[l][i].elapsed_time(self.evs[l][i + 1])
        uniq = sum(int(torch.unique(self.topi[l]).numel()) for l in range(NL)) / NL
        return stage, uniq

    def release(self):
        self.graph = self.graph_ev = None


def decode_summary(pt: DecodePoint, ms_per_step: float, peak: float) -> dict:
    """Per-layer time, stage times and the HBM roofline of one decode point."""
    NL = len(pt.layers)
    stage, uniq = pt.breakdown()
    gemm_ms = stage[2] + stage[3]
    w_bytes = uniq * EXPERT_BYTES
    layer_bytes = decode_layer_bytes(uniq, pt.T)
    us_layer = ms_per_step / NL * 1e3
    exp_gbs = w_bytes / (gemm_ms / NL / 1e3) / 1e9
    lay_gbs = layer_bytes / (us_layer / 1e6) / 1e9
    return {"tokens_per_s": pt.T * NL / (ms_per_step / 1e3), "us_per_layer": us_layer,
            "unique_experts_per_layer": uniq,
            "stage_us_per_layer": {"route": stage[0] / NL * 1e3, "experts": gemm_ms / NL * 1e3,
                                   "combine": stage[4] / NL * 1e3},
            "experts_kernel": {"bytes": w_bytes, "GBps": exp_gbs, "frac": exp_gbs / peak},
            "layer": {"bytes": layer_bytes, "GBps": lay_gbs, "frac": lay_gbs / peak}}


# ---------------------------------------------------------------------------
def prefill_point(T, NL, dev, stream, zipf_alpha, steps, warmup, seed_base=100, layer_weights=None):
    """BASELINE config 3 at T tokens: NL prefill layer calls (distinct weights,
    Zipf(1.2)-skewed routing), plain launches; returns the summary dict."""
    from moe_fused_inference_b200.layer import MoELayer, random_layer_weights
    from moe_fused_inference_b200.synthetic import zipf_bias

    bias = torch.from_numpy(zipf_bias(E, zipf_alpha, seed=3))
    if layer_weights is None:
        layer_weights = [random_layer_weights(E, H, MI, 0.02, seed=seed_base + l, device=dev)
                         for l in range(NL)]
    layers = [MoELayer(w, TOPK, logit_bias=bias) for w in layer_weights[:NL]]
    g = torch.Generator(device=dev).manual_seed(7)
    X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
    out = torch.empty((NL, T, H), dtype=torch.float32, device=dev)
    topi = torch.empty((NL, T, TOPK), dtype=torch.int32, device=dev)
    topw = torch.empty((NL, T, TOPK), dtype=torch.float32, device=dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(NL)]
    for row in evs:
        for e in row:
            e.record(stream)  # creates the event handles before the library records them

    def step(with_events=False):
        # T * top_k > 4096: mfi_moe_layer takes the prefill path by itself
        for l in range(NL):
            layers[l](X[l], out=out[l], topi=topi[l], topw=topw[l],
                      events=evs[l] if with_events else None)

    for _ in range(warmup):
        step()
    ms = event_time(dev, stream, step, steps)
    ms_per_layer = ms / steps / NL
    step(True)
    torch.cuda.synchronize(dev)
    names = ["route", "scatter", "experts", "combine"]
    st = {n: 0.0 for n in names}
    for l in range(NL):
        t = [evs[l][i].elapsed_time(evs[l][i + 1]) for i in range(5)]
        st["route"] += t[0]
        st["scatter"] += t[1]
        st["experts"] += t[2] + t[3]
        st["combine"] += t[4]
    counts = torch.bincount(topi[0].flatten().long(), minlength=E).float()
    flops = FLOP_TOKEN * T
    tflops = flops / (ms_per_layer / 1e3) / 1e12
    exp_flops = TOPK * (2 * H * 2 * MI + 2 * MI * H) * T
    exp_ms = st["experts"] / NL
    hbm_peak, hbm_kind = measured_peaks()
    hbm_bytes = (int((counts > 0).sum()) * EXPERT_BYTES + ROUTER_BYTES + T * H * 2 + T * H * 4
                 + T * TOPK * 8)
    hbm_gbs = hbm_bytes / (ms_per_layer / 1e3) / 1e9
    res = {"tokens_per_s": T / (ms_per_layer / 1e3), "us_per_layer": ms_per_layer * 1e3,
           "flops_per_layer": flops, "tflops": tflops, "frac": tflops / FP4_PEAK,
           "stage_us_per_layer": {k: v / NL * 1e3 for k, v in st.items()},
           "experts_kernel": {"us": exp_ms * 1e3, "tflops": exp_flops / (exp_ms / 1e3) / 1e12,
                              "frac": exp_flops / (exp_ms / 1e3) / 1e12 / FP4_PEAK},
           "hbm": {"bytes_per_layer": hbm_bytes, "GBps": hbm_gbs, "frac": hbm_gbs / hbm_peak,
                   "peak_kind": hbm_kind},
           "expert_load_max_over_mean": float(counts.max() / counts.mean()),
           "experts_with_tokens": int((counts > 0).sum()),
           "layers": NL, "steps": steps}
    del layers, X, out, topi, topw
    torch.cuda.empty_cache()
    return res


def dense_projections(T, dev, stream, seed=5):
    """Dense mxfp4_linear of the attention projections at T tokens (config 3)
    through lin_pq on pre-quantised activations."""
    from moe_fused_inference_b200 import fp4_ext
    from moe_fused_inference_b200.layer import quantize_rows

    dec = fp4_ext.get_decode_ext()
    g = torch.Generator(device=dev).manual_seed(seed)
    dense = {}
    for name, (n_out, k_in) in {"q": (4096, 2048), "k": (512, 2048), "v": (512, 2048),
                                "o": (2048, 4096)}.items():
        wq, wsc = quantize_rows((torch.randn((n_out, k_in), generator=g, device=dev) * 0.02).bfloat16())
        xq, xsc = quantize_rows(torch.randn((T, k_in), generator=g, device=dev).bfloat16())
        for _ in range(2):
            dec.lin_pq(xq, xsc, wq, wsc, T, n_out, k_in)
        ms = event_time(dev, stream, lambda: dec.lin_pq(xq, xsc, wq, wsc, T, n_out, k_in), 5)
        us = ms / 5 * 1e3
        tf = 2.0 * T * n_out * k_in / us / 1e6
        dense[name] = {"us": us, "tflops": tf, "frac": tf / FP4_PEAK}
        del wq, wsc, xq, xsc
    torch.cuda.empty_cache()
    return dense


def dropin_point(layers, T, dev, stream, steps, warmup, peak):
    """The reference's decode MoE block through the drop-in operators, with
    its host steps unchanged (runtime/model_runner_v2.py:185-207 for T = 1,
    :266-290 for T = M): prequant, lin_pq router, softmax/top-k/renormalise in
    torch, .tolist(), per-token pointer lists, moe_gateup, moe_down,
    moe_combine.  Returns the whole chain's time and the gate/up + down
    kernels' HBM roofline (CUDA events around them)."""
    from moe_fused_inference_b200 import fp4_ext
    import torch.nn.functional as F

    dext = fp4_ext.get_decode_ext()
    NL = len(layers)
    # per-expert tensors, as the reference WeightStore hands them out
    # (runtime/weight_store.py:283-285)
    views = []
    for L in layers:
        w = L.w
        views.append({e: {"gate": (w.gate_wp[e], w.gate_sc[e]), "up": (w.up_wp[e], w.up_sc[e]),
                          "down": (w.down_wp[e], w.down_sc[e])} for e in range(E)})
    g = torch.Generator(device=dev).manual_seed(17)
    X = torch.randn((NL, T, H), generator=g, device=dev).bfloat16()
    uniq = [0] * NL
    tabs = [None] * NL
    outs = [None] * NL

    def step(keep_tables=False):
        for l in range(NL):
            w = layers[l].w
            hq, hs = dext.prequant(X[l])
            gate = dext.lin_pq(hq, hs, w.router_wp, w.router_sc, T, E, H)
            rp = F.softmax(gate.float(), -1)
            tv, ti = torch.topk(rp, TOPK, dim=-1)
            tv = tv / tv.sum(-1, keepdim=True)
            ids = ti.reshape(-1).tolist()
            ex = views[l]
            gu_tab, gsu_tab, dw_tab, ds_tab = [], [], [], []
            for m in range(T):
                sel = ids[m * TOPK:(m + 1) * TOPK]
                gu_tab += [ex[e]["gate"][0] for e in sel] + [ex[e]["up"][0] for e in sel]
                gsu_tab += [ex[e]["gate"][1] for e in sel] + [ex[e]["up"][1] for e in sel]
                dw_tab += [ex[e]["down"][0] for e in sel]
                ds_tab += [ex[e]["down"][1] for e in sel]
            guv = dext.moe_gateup(hq, hs, gu_tab, gsu_tab, TOPK, T, MI, H)
            ydv = dext.moe_down(guv, dw_tab, ds_tab, TOPK, T, H, MI)
            outs[l] = dext.moe_combine(ydv, tv.reshape(T, TOPK).float(), T)
            if keep_tables:
                uniq[l] = len(set(ids))
                ptr = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64,
                                              device=dev)
                tabs[l] = (hq, hs, ptr(gu_tab), ptr(gsu_tab), ptr(dw_tab), ptr(ds_tab))

    for _ in range(warmup):
        step()
    ms = event_time(dev, stream, step, steps)
    ms_per_layer = ms / steps / NL
    step(True)
    torch.cuda.synchronize(dev)

    # the operators' kernels alone: the graph-friendly _tab forms with the
    # same routing's device pointer tables (built above, outside the timing),
    # all layers captured in one CUDA graph
    def kernels():
        for l in range(NL):
            hq, hs, gt, gs, dt, ds = tabs[l]
            guv = dext.moe_gateup_tab(hq, hs, gt, gs, TOPK, T, MI, H)
            dext.moe_down_tab(guv, dt, ds, TOPK, T, H, MI)

    graph = capture(dev, stream, kernels, 1)
    for _ in range(warmup):
        graph.replay()
    k_ms = event_time(dev, stream, graph.replay, steps) / steps / NL
    del graph
    u = sum(uniq) / NL
    k_gbs = u * EXPERT_BYTES / (k_ms / 1e3) / 1e9
    lay_gbs = decode_layer_bytes(u, T) / (ms_per_layer / 1e3) / 1e9
    return {"tokens_per_s": T / (ms_per_layer / 1e3), "us_per_layer": ms_per_layer * 1e3,
            "unique_experts_per_layer": u,
            "gateup_down_kernels": {"us_per_layer": k_ms * 1e3, "GBps": k_gbs, "frac": k_gbs / peak,
                                    "how": "moe_gateup_tab + moe_down_tab of every layer in one "
                                           "CUDA graph, tables built outside the timing"},
            "layer": {"GBps": lay_gbs, "frac": lay_gbs / peak},
            "note": "host steps (.tolist(), pointer lists) inside the timed chain, as the "
                    "reference runner runs them"}


def attn_point(dev, stream, steps, warmup, peak, ctx=4096, M=1, n_caches=48):
    """FP8-KV decode attention (config 4's attention: 32 query / 4 KV heads,
    head_dim 128) of M query rows at context `ctx` over n_caches distinct
    layer caches (n_caches x ctx x 4 x 128 x 2 B, larger than L2), all calls
    in one CUDA graph.  Bytes per call: the live K and V positions."""
    from moe_fused_inference_b200 import _lib
    lib = _lib.load()
    Hq, Hkv, D = 32, 4, 128
    max_pos = ctx + M
    g = torch.Generator(device=dev).manual_seed(23)
    caches = [(torch.randint(0, 120, (max_pos, Hkv, D), generator=g, device=dev,
                             dtype=torch.int32).to(torch.uint8),
               torch.randint(0, 120, (max_pos, Hkv, D), generator=g, device=dev,
                             dtype=torch.int32).to(torch.uint8)) for _ in range(n_caches)]
    q = torch.randn((M, Hq, D), generator=g, device=dev).bfloat16()
    dpos = torch.tensor([ctx - 1], dtype=torch.int32, device=dev)
    o = torch.empty((M, Hq, D), dtype=torch.float32, device=dev)
    nws = int(lib.mfi_attn_decode_workspace_bytes(M, Hq, Hkv, D, max_pos))
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    def calls():
        # the reference-codec cache (no scales), through the C entry with a
        # preallocated output and workspace (as the model runner calls it),
        # on the stream being captured
        st = torch.cuda.current_stream(dev).cuda_stream
        for kk, vv in caches:
            _lib.check(lib.mfi_attn_decode(q.data_ptr(), kk.data_ptr(), vv.data_ptr(),
                                           dpos.data_ptr(), o.data_ptr(), M, Hq, Hkv, D, max_pos,
                                           None, None, ws.data_ptr(), nws, st), "attn_decode")

    graph = capture(dev, stream, calls, 1)
    for _ in range(warmup):
        graph.replay()
    us = event_time(dev, stream, graph.replay, steps) / steps / n_caches * 1e3
    del graph, caches
    torch.cuda.empty_cache()
    kv_bytes = (ctx - 1 + M) * Hkv * D * 2
    gbs = kv_bytes / us / 1e3
    return {"us": us, "kv_bytes": kv_bytes, "GBps": gbs, "frac": gbs / peak,
            "note": "mfi_attn_decode (partial + merge kernels), graph-captured"}


# ---------------------------------------------------------------------------
def run_prefill(args, world, rank, local):
    """--workload prefill: BASELINE config 3 alone (T tokens, default 16384,
    Zipf(1.2)-skewed routing) with its own JSON line.  Under torchrun every
    rank runs its own copy (weak scaling)."""
    dev = torch.device("cuda", local if world > 1 else 0)
    T = args.tokens if args.tokens != 64 else 16384
    NL = args.layers if args.layers != N_LAYERS else 4
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(dev.index)
    sampler.start()
    barrier(world)
    pf = prefill_point(T, NL, dev, stream, args.zipf_alpha, args.steps, args.warmup)
    barrier(world)
    clocks = sampler.stop()
    ms_layer = max_over_ranks(pf["us_per_layer"] / 1e3, world)
    dense = dense_projections(T, dev, stream)
    if rank != 0:
        return
    line = {
        "metric": "MXFP4 MoE layer tokens/s (prefill)", "value": T * world / (ms_layer / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_layer * NL, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"prefill MoE layer, T={T} tokens, H=2048, E=128, top-8, Mi=768, "
                               f"Zipf(1.2) logit bias alpha={args.zipf_alpha}",
                   "step": f"{NL} MoE layers with distinct weights, plain launches",
                   "expert_load_max_over_mean": pf["expert_load_max_over_mean"],
                   "experts_with_tokens": pf["experts_with_tokens"]},
        "gpu_launches": 5 * NL * args.steps,  # quantise, route, scatter, experts, combine
        "roofline": {"bound": "tensor", "achieved": pf["tflops"], "peak": FP4_PEAK,
                     "unit": "TFLOP/s", "frac": pf["frac"],
                     "peak_kind": "nominal dense FP4 (no measured FP4 peak)",
                     "flops_per_layer": pf["flops_per_layer"], "experts_kernel": pf["experts_kernel"],
                     "stage_us_per_layer": pf["stage_us_per_layer"], "dense_projections": dense,
                     "hbm": pf["hbm"]},
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
            ms = event_time(dev, stream, graph.replay, args.steps)
            us = ms / (args.steps * reps) * 1e3
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


def run_model(args, world, rank, local):
    """the random-init 48-layer Qwen3-30B-A3B-shaped model
    on the library (model.py), 1024-token prompts with the repeated motif,
    then greedy decode steps, each replayed from one CUDA graph
    (GraphDecoder), at batch 1, 16 and 64.  Decode tokens/s = batch x steps /
    the device time of the steps; the eager step time is reported beside it."""
    from moe_fused_inference_b200.model import (GraphDecoder, LibBackend, QwenConfig, Runner,
                                                SyntheticQwen, synthetic_prompts)
    dev = torch.device("cuda", local if world > 1 else 0)
    stream = torch.cuda.current_stream(dev)
    t0 = time.time()
    model = SyntheticQwen.build(QwenConfig(), seed=1, device=dev)
    lib = LibBackend(model)
    torch.cuda.synchronize(dev)
    build_s = time.time() - t0
    P, S = 1024, max(args.steps, 8)
    per = {}
    sampler = ClockSampler(dev.index if dev.index is not None else 0)
    sampler.start()
    for B in (1, 16, 64):
        prompt = synthetic_prompts(B, P, model.cfg.vocab, seed=101 + B, device=dev)
        runner = Runner(model, lib, B, P + S + 8)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        runner.prefill(prompt)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        prefill_ms = e0.elapsed_time(e1)
        # eager decode steps (for comparison), then the graph
        pos = P - 1
        last = prompt[:, -1:]
        eager_ms = event_time(dev, stream, lambda: runner.forward(last, pos, last_only=True), 3) / 3
        gd = GraphDecoder(runner, S)
        gd.start(prompt, prefill=False)
        ms = event_time(dev, stream, lambda: gd.decode(S), 1)
        per[f"B{B}"] = {"decode_tokens_per_s": B * S / (ms / 1e3), "ms_per_step": ms / S,
                        "eager_ms_per_step": eager_ms, "steps": S,
                        "prefill_ms": prefill_ms, "prefill_tokens_per_s": B * (P - 1) / (prefill_ms / 1e3)}
        del gd, runner
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    if rank != 0:
        return
    line = {
        "metric": "config 4 greedy decode tokens/s (48-layer synthetic Qwen3-30B-A3B)",
        "value": per["B64"]["decode_tokens_per_s"], "unit": "tokens/s", "n_gpus": 1,
        "steps": S, "warmup": 1, "ms_per_step": per["B64"]["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 experts and projections, bf16 activations, FP8 KV cache",
        "data": "synthetic (random-init weights, uniform random prompts with a repeated "
                "32-token motif, seeded)",
        "config": {"workload": "config 4: 48 layers, 32/4 heads, head_dim 128, vocab 151936, "
                               "128 experts top-8; 1024-token prompts, greedy decode",
                   "step": "one decode step of B sequences, replayed from one CUDA graph "
                           "(GraphDecoder); prefill in 64-token chunks, eager",
                   "model_build_s": build_s},
        "per_batch": per, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_dropin(args, world, rank, local):
    """--workload dropin: the decode line's drop-in block alone (the
    reference's decode MoE block through moe_gateup / moe_down / moe_combine
    with its host steps, T = 1 and 16), for profiling that chain."""
    from moe_fused_inference_b200.layer import MoELayer, random_layer_weights

    dev = torch.device("cuda", local if world > 1 else 0)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peaks()
    layers = [MoELayer(random_layer_weights(E, H, MI, 0.02, seed=l, device=dev), TOPK)
              for l in range(args.layers)]
    res = {f"T{t}": dropin_point(layers, t, dev, stream, args.steps, max(args.warmup, 1), peak)
           for t in (1, 16)}
    if rank != 0:
        return
    head = res["T1"]
    line = {
        "metric": "drop-in decode MoE block tokens/s (T=1, the reference's call sequence)",
        "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["us_per_layer"] / 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 (e2m1 x e2m1, fp32 accumulate)",
        "data": "synthetic (random-init weights N(0,0.02), activations N(0,1), seeded)",
        "config": {"workload": f"drop-in moe_gateup/moe_down/moe_combine chain, {args.layers} "
                               "layers, T in {1, 16}", "peak_kind": peak_kind},
        "dropin": res,
    }
    print(json.dumps(line), flush=True)


def run_attn(args, world, rank, local):
    """--workload attn: the decode line's attention block alone (FP8-KV
    decode attention, context 4096, M = 1 and 5 query rows)."""
    dev = torch.device("cuda", local if world > 1 else 0)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peaks()
    res = {f"M{m}_ctx4096": attn_point(dev, stream, args.steps, max(args.warmup, 1), peak, M=m)
           for m in (1, 5)}
    if rank != 0:
        return
    head = res["M1_ctx4096"]
    line = {
        "metric": "FP8-KV decode attention us per call (M=1, context 4096)", "value": head["us"],
        "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["us"] / 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8 e4m3 KV, fp32 softmax",
        "data": "synthetic (seeded queries and caches)",
        "config": {"workload": "mfi_attn_decode, 32 query / 4 KV heads, head_dim 128, "
                               "context 4096, M in {1, 5}", "peak_kind": peak_kind},
        "attn_decode": res,
    }
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    if args.workload == "dropin":
        return run_dropin(args, world, rank, local)
    if args.workload == "attn":
        return run_attn(args, world, rank, local)
    if args.workload == "model":
        return run_model(args, world, rank, local)
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
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peaks()

    # ---- headline: decode at T, one CUDA graph per step (decode serving runs
    # graphs; replay removes the host's per-launch cost from the measurement)
    head = DecodePoint(layers, T, dev, stream, graph=not args.no_graph)
    head.prepare(args.warmup)
    ms, clocks = timed_region(args, world, dev, stream, head.run)
    ms_per_step = ms / args.steps
    tokens = T * NL * args.steps
    value = tokens / (ms / 1e3)
    hs = decode_summary(head, ms_per_step, peak)
    head.release()
    traffic = committed_traffic()

    # ---- e2e through the public API with host buffers ----
    # every step copies its inputs in from pinned host memory and its outputs
    # back; the copies run per layer on two copy streams, overlapping the
    # layers (layer l waits for its own input only, the D2H of its output
    # starts when it is done), and the whole step is one CUDA graph
    Xh = head.X.cpu().pin_memory()
    Oh = torch.empty((NL, T, H), dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(head.X)
    e2e_step, e2e_note = overlapped_e2e_step(dev, layers, Xh, Xd, Oh, head.out,
                                             lambda l, x, o: layers[l](x, out=o, topi=head.topi[l],
                                                                        topw=head.topw[l]),
                                             stream, graph=not args.no_graph)
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
                           + " (e2e: " + e2e_note + ")",
                   "global_batch": T, "parallelism": "single GPU",
                   "l2": f"inputs larger than L2: {NL} distinct layer weight sets "
                         f"({NL * E * EXPERT_BYTES / 1e9:.1f} GB) per step",
                   "unique_experts_per_layer": hs["unique_experts_per_layer"]},
        "gpu_launches": 3 * NL * args.steps,  # route (+quantise), experts (gate/up + down), combine
        "roofline": {"bound": "hbm", "kernel": "moe_experts_kernel (gate/up + down, one launch)",
                     "achieved": hs["experts_kernel"]["GBps"], "peak": peak, "unit": "GB/s",
                     "frac": hs["experts_kernel"]["frac"], "peak_kind": peak_kind,
                     "algorithmic_bytes_per_layer_call": hs["experts_kernel"]["bytes"],
                     "algorithmic_bytes_per_step": hs["experts_kernel"]["bytes"] * NL,
                     "traffic": (traffic or {}).get("bytes_per_layer_call"),
                     "traffic_source": (traffic or {}).get("source"),
                     "layer": {"achieved": hs["layer"]["GBps"], "frac": hs["layer"]["frac"],
                               "stage_us_per_layer": hs["stage_us_per_layer"]}},
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(Xh.numel() * Xh.element_size()),
                "d2h_bytes_per_step": int(Oh.numel() * Oh.element_size())},
        "clocks": clocks,
    }
    del Xh, Oh, Xd, head
    torch.cuda.empty_cache()

    if not args.headline_only:
        # ---- decode sweep (config 2's other batch sizes) ----
        sweep = {str(T): hs}
        for t in (1, 8, 32):
            if t == T:
                continue
            pt = DecodePoint(layers, t, dev, stream, seed=70 + t, graph=not args.no_graph)
            pt.prepare(args.warmup)
            pms = event_time(dev, stream, pt.run, args.steps) / args.steps
            sweep[str(t)] = decode_summary(pt, pms, peak)
            pt.release()
            del pt
        line["decode_sweep"] = {k: sweep[k] for k in sorted(sweep, key=int)}
        # ---- the reference's drop-in call sequence (unchanged callers) ----
        line["dropin"] = {f"T{t}": dropin_point(layers, t, dev, stream, max(args.steps // 4, 3),
                                                 2, peak) for t in (1, 16)}
        torch.cuda.empty_cache()
        # ---- FP8-KV decode attention (config 4's attention, context 4096) ----
        line["attn_decode"] = {f"M{m}_ctx4096": attn_point(dev, stream, args.steps, 2, peak, M=m)
                               for m in (1, 5)}
        # ---- prefill (config 3) on 4 of the decode weight sets ----
        pf = {}
        for t in (2048, 16384):
            pf[f"T{t}"] = prefill_point(t, 4, dev, stream, args.zipf_alpha,
                                        steps=5 if t > 4096 else 10, warmup=2,
                                        layer_weights=[L.w for L in layers[:4]])
        pf["dense_projections_T16384"] = dense_projections(16384, dev, stream)
        pf["peak_kind"] = "nominal dense FP4 9000 TFLOP/s (no measured FP4 peak)"
        line["prefill"] = pf

    if not args.no_cpu_baseline:
        cpu_layer = make_cpu_layer(layers[0].w)
        line["cpu_baseline"] = cpu_baseline(args, T, cpu_layer)
        if not args.headline_only:
            line["cpu_baseline"]["config1_T4"] = cpu_baseline(args, 4, cpu_layer)
    print(json.dumps(line), flush=True)


def ep_prefill_point(args, world, rank, dev, T_total=16384, NL=2, steps=5, warmup=2):
    """BASELINE config 5's prefill: T_total tokens split over the ranks
    (T_total / world each), NL expert-parallel layers (128/N experts per GPU)
    with Zipf(1.2)-skewed routing, NCCL all-to-all dispatch and return, the
    prefill tcgen05 kernels on the received rows.  Device time max over
    ranks; one extra step with events between the calls gives the stages."""
    import torch.distributed as dist
    from moe_fused_inference_b200.ep import EPMoELayer, random_shard
    from moe_fused_inference_b200.synthetic import zipf_bias

    Tr = T_total // world
    bias = torch.from_numpy(zipf_bias(E, args.zipf_alpha, seed=3)).to(dev)
    layers = [EPMoELayer(random_shard(E, world, rank, H, MI, 0.02, seed=200 + l, device=dev),
                         TOPK, Tr, transport="nccl", logit_bias=bias) for l in range(NL)]
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    X = torch.randn((NL, Tr, H), generator=g, device=dev).bfloat16()
    out = torch.empty((NL, Tr, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for l in range(NL):
            layers[l](X[l], out=out[l])

    for _ in range(warmup):
        step()
    barrier(world)
    ms = max_over_ranks(event_time(dev, stream, step, steps), world)
    names = ["route_pack", "a2a_dispatch", "experts", "a2a_return", "unpack"]
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(NL)]
    barrier(world)
    for l in range(NL):
        L, ev = layers[l], evs[l]
        ev[0].record(stream)
        L.dispatch_prepare(X[l])
        ev[1].record(stream)
        dist.all_to_all_single(L.recv.view(-1), L.send.view(-1))
        ev[2].record(stream)
        L.compute()
        ev[3].record(stream)
        dist.all_to_all_single(L.ret_back.view(-1), L.ret.view(-1))
        ev[4].record(stream)
        L.finish(Tr, out[l])
        ev[5].record(stream)
    torch.cuda.synchronize(dev)
    st = torch.tensor([sum(evs[l][i].elapsed_time(evs[l][i + 1]) for l in range(NL)) / NL * 1e3
                       for i in range(5)], dtype=torch.float64, device=dev)
    allst = [torch.zeros_like(st) for _ in range(world)]
    dist.all_gather(allst, st)
    load = torch.bincount(layers[0].topi[:Tr].flatten().long(), minlength=E).to(torch.float64)
    dist.all_reduce(load)
    for L in layers:
        L.close()
    del layers, X, out
    torch.cuda.empty_cache()
    us_layer = ms / steps / NL * 1e3
    tflops = FLOP_TOKEN * T_total / (us_layer / 1e6) / 1e12
    return {"tokens_total": T_total, "tokens_per_rank": Tr, "layers": NL, "steps": steps,
            "us_per_layer": us_layer, "tokens_per_s": T_total / (us_layer / 1e6),
            "tflops_all_gpus": tflops, "frac_of_nominal_fp4_per_gpu": tflops / world / 9000.0,
            "stage_us_per_layer": {n: [float(v[i]) for v in allst] for i, n in enumerate(names)},
            "expert_load_max_over_mean": float(load.max() / load.mean()),
            "routing": f"Zipf(1.2) logit bias alpha={args.zipf_alpha}",
            "transport": "NCCL all_to_all_single (fixed-capacity blocks)"}


def run_ep(args, world, rank, local):
    """Expert-parallel step over the torchrun ranks (peer-memory exchange fused
    into the kernels, or NCCL all-to-all with --ep-transport nccl)."""
    from moe_fused_inference_b200.ep import EPMoELayer, random_shard

    dev = torch.device("cuda", local)
    T, NL = args.tokens, args.layers
    bias = None
    if args.ep_zipf:
        from moe_fused_inference_b200.synthetic import zipf_bias
        bias = torch.from_numpy(zipf_bias(E, args.zipf_alpha, seed=3)).to(dev)
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

    # ---- per-stage device times of one step (events between the calls) ----
    import torch.distributed as dist
    from moe_fused_inference_b200.ep import ep_row_bytes
    stage_names = (["route_dispatch", "experts_return", "unpack_wait"] if args.ep_transport == "p2p"
                   else ["route_pack", "a2a_dispatch", "experts", "a2a_return", "unpack"])
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(stage_names) + 1)]
           for _ in range(NL)]
    recvs = []
    barrier(world)
    for l in range(NL):
        L = layers[l]
        ev = evs[l]
        ev[0].record(stream)
        if L.transport == "p2p":
            L.p2p_dispatch(X[l])
            ev[1].record(stream)
            L.p2p_experts()  # includes the wait for the peers' dispatch
            ev[2].record(stream)
            L.p2p_finish(T, out[l])
            ev[3].record(stream)
            rv = torch.empty((world, T + 1, ep_row_bytes(H, TOPK)), dtype=torch.uint8, device=dev)
            L.xch.copy_recv_to(rv)
            recvs.append(rv)
        else:
            L.dispatch_prepare(X[l])
            ev[1].record(stream)
            dist.all_to_all_single(L.recv.view(-1), L.send.view(-1))
            ev[2].record(stream)
            L.compute()
            ev[3].record(stream)
            dist.all_to_all_single(L.ret_back.view(-1), L.ret.view(-1))
            ev[4].record(stream)
            L.finish(T, out[l])
            ev[5].record(stream)
            recvs.append(L.recv)
    torch.cuda.synchronize(dev)
    stage_ms = [sum(evs[l][i].elapsed_time(evs[l][i + 1]) for l in range(NL))
                for i in range(len(stage_names))]
    experts_ms = stage_ms[1] if args.ep_transport == "p2p" else stage_ms[2]
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
    # the rate of the rank's local expert weights over the device-timed step
    # (graph replay, max over ranks): the eager stage times below include
    # each rank's waits on the other ranks' launches, so they cannot serve as
    # the kernel's duration
    achieved = w_bytes / (ms_per_step / 1e3) / 1e9
    stats = torch.tensor([achieved, experts_ms, rows_recv / NL, uniq / NL] + stage_ms,
                         dtype=torch.float64, device=dev)
    allstats = [torch.zeros_like(stats) for _ in range(world)]
    dist.all_gather(allstats, stats)
    allstats = torch.stack(allstats).cpu()
    # expert load over all ranks' tokens (layer 0's routing)
    load = torch.bincount(layers[0].topi[:T].flatten().long(), minlength=E).to(torch.float64)
    dist.all_reduce(load)
    load_max_over_mean = float(load.max() / load.mean())

    # ---- e2e: host activations in, host outputs back (per-layer copies on
    # copy streams overlapping the layers; one graph when the timed run
    # captured one on every rank) ----
    use_graph = graph is not None
    if graph is not None:
        del graph
    del recvs
    Xh = X.cpu().pin_memory()
    Oh = torch.empty((NL, T, H), dtype=torch.float32).pin_memory()
    Xd = torch.empty_like(X)
    e2e_step, e2e_note = overlapped_e2e_step(dev, layers, Xh, Xd, Oh, out,
                                             lambda l, x, o: layers[l](x, out=o), stream,
                                             graph=use_graph)
    ok = torch.tensor([1.0 if e2e_note.endswith("graph") or not use_graph else 0.0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() < 1.0 and use_graph:
        # a rank fell back to plain launches: all ranks take the same path
        e2e_step, e2e_note = overlapped_e2e_step(dev, layers, Xh, Xd, Oh, out,
                                                 lambda l, x, o: layers[l](x, out=o), stream,
                                                 graph=False)
    e2e_ms, _ = timed_region(args, world, dev, stream, e2e_step)
    e2e_value = tokens / (e2e_ms / 1e3)
    torch.cuda.synchronize(dev)
    barrier(world)
    for L in layers:
        L.close()  # unmap the peers' memory before the process group goes away
    barrier(world)
    del layers, X, out, Xd
    torch.cuda.empty_cache()
    ep_prefill = None if args.headline_only else ep_prefill_point(args, world, rank, dev)
    barrier(world)
    if rank != 0:
        return
    worst = int(torch.argmin(allstats[:, 0]))
    per_rank_stages = {n: [float(v) / NL * 1e3 for v in allstats[:, 4 + i]]
                       for i, n in enumerate(stage_names)}
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
                       "return, unpack") + ", " + graph_note + " (e2e: " + e2e_note + ")",
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
        "roofline": {"bound": "hbm", "kernel": "expert-parallel layer (local expert weights)",
                     "achieved": float(allstats[worst, 0]), "peak": peak, "unit": "GB/s",
                     "frac": float(allstats[worst, 0]) / peak, "peak_kind": peak_kind,
                     "basis": "local expert weight bytes per step / device-timed step "
                              "(max over ranks), lowest rank",
                     "rank": worst, "experts_ms_per_step_eager": float(allstats[worst, 1]),
                     "traffic": None},
        # one eager step with events between the calls (plain launches; each
        # call's time includes its waits on the other ranks)
        "stage_us_per_layer": per_rank_stages,
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": int(Xh.numel() * Xh.element_size()),
                "d2h_bytes_per_step": int(Oh.numel() * Oh.element_size())},
        "clocks": clocks,
    }
    if ep_prefill is not None:
        line["ep_prefill"] = ep_prefill
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
