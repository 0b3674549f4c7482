"""GPU tests of the layer halves (mfi_moe_route, mfi_moe_experts) and of the
expert-parallel exchange kernels (mfi_ep_pack / mask_recv / unpack).

All ranks of an expert-parallel layer are driven from one process on one GPU
with the two all-to-alls done by copies (the blocks a rank sends are exactly
what NCCL would deliver), so the sharded path is checked against the
single-GPU layer on any box; the multi-process NCCL form of the same test
runs when two GPUs are visible.
"""

import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from moe_fused_inference_b200.synthetic import zipf_bias
from oracle import ep as oep
from oracle import mxfp4 as mx
from tests.conftest import cosine, max_rel_err

pytestmark = pytest.mark.gpu


def _lib():
    from moe_fused_inference_b200 import _lib as L
    return L


def _layer_w(E, H, Mi, seed=3):
    from moe_fused_inference_b200.layer import random_layer_weights
    return random_layer_weights(E, H, Mi, seed=seed, device="cuda")


def _x(T, H, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)


def _emulate(w, xs, world, k, capacity):
    """Run an EP layer (all-to-all transport) over `world` virtual ranks in
    this process, the all-to-alls done by copies."""
    from moe_fused_inference_b200.ep import EPMoELayer, EPShard
    layers = [EPMoELayer(EPShard.from_layer(w, r, world), k, capacity, world=world, rank=r,
                         transport="nccl")
              for r in range(world)]
    for L, x in zip(layers, xs):
        L.dispatch_prepare(x)
    for d in range(world):
        for s in range(world):
            layers[d].recv[s].copy_(layers[s].send[d])
    for L in layers:
        L.compute()
    for s in range(world):
        for d in range(world):
            layers[s].ret_back[d].copy_(layers[d].ret[s])
    outs = []
    for L, x in zip(layers, xs):
        out = torch.empty((x.shape[0], w.hidden), dtype=torch.float32, device="cuda")
        L.finish(x.shape[0], out)
        outs.append(out)
    torch.cuda.synchronize()
    return layers, outs


@pytest.mark.parametrize("world,counts", [(2, [64, 64]), (4, [64, 17, 0, 33]),
                                          (8, [64] * 8), (8, [1, 0, 5, 64, 2, 31, 8, 3])])
def test_ep_emulated_matches_single_gpu(world, counts):
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k = 128, 2048, 768, 8
    w = _layer_w(E, H, Mi)
    xs = [_x(t, H, 50 + r) for r, t in enumerate(counts)]
    layers, outs = _emulate(w, xs, world, k, max(counts))
    single = MoELayer(w, top_k=k)
    for r, x in enumerate(xs):
        if x.shape[0] == 0:
            continue
        ref, topi, topw = single(x)
        torch.cuda.synchronize()
        assert torch.equal(layers[r].topi[: x.shape[0]], topi)
        assert torch.equal(layers[r].topw[: x.shape[0]], topw)
        a, b = outs[r].cpu().numpy(), ref.cpu().numpy()
        # same expert outputs; the combine sums local slots, then ranks
        assert max_rel_err(a, b) <= 1e-5
        assert cosine(a, b) >= 0.999999


@pytest.mark.parametrize("world,counts,zipf", [(2, [1100, 700], False), (4, [600, 0, 2100, 900], True),
                                               (8, [2048] * 8, True)])
def test_ep_prefill_emulated_matches_single_gpu(world, counts, zipf):
    """Expert-parallel prefill (BASELINE config 5 at its per-rank sizes): more
    than 16384 (row, slot) pairs per rank, so the expert step runs the prefill
    tcgen05 kernels on the received rows, with ragged per-rank token counts
    (one rank empty) and Zipf-skewed routing.  Every rank here has more than
    512 tokens, so the single-GPU layer takes its prefill path too: the expert
    outputs are the same bf16 rows and only the combine's summation order
    (local slots, then ranks) differs."""
    from moe_fused_inference_b200.ep import EPMoELayer, EPShard
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k = 128, 2048, 768, 8
    w = _layer_w(E, H, Mi, seed=9)
    bias = torch.from_numpy(zipf_bias(E, 0.5, seed=3)).cuda() if zipf else None
    C = max(counts)
    xs = [_x(t, H, 80 + r) for r, t in enumerate(counts)]
    layers = [EPMoELayer(EPShard.from_layer(w, r, world), k, C, world=world, rank=r,
                         logit_bias=bias) for r in range(world)]
    assert all(L.transport == "nccl" for L in layers)  # too large for the peer-memory transport
    for L, x in zip(layers, xs):
        L.dispatch_prepare(x)
    for d in range(world):
        for s in range(world):
            layers[d].recv[s].copy_(layers[s].send[d])
    for L in layers:
        L.compute()
    for s in range(world):
        for d in range(world):
            layers[s].ret_back[d].copy_(layers[d].ret[s])
    outs = []
    for L, x in zip(layers, xs):
        out = torch.empty((x.shape[0], H), dtype=torch.float32, device="cuda")
        L.finish(x.shape[0], out)
        outs.append(out)
    torch.cuda.synchronize()
    assert _lib().load().mfi_device_error(1) == 0
    single = MoELayer(w, top_k=k, logit_bias=bias)
    for r, x in enumerate(xs):
        if x.shape[0] == 0:
            continue
        ref, topi, topw = single(x)
        torch.cuda.synchronize()
        assert torch.equal(layers[r].topi[: x.shape[0]], topi)
        assert torch.equal(layers[r].topw[: x.shape[0]], topw)
        a, b = outs[r].cpu().numpy(), ref.cpu().numpy()
        assert max_rel_err(a, b) <= 1e-5
        assert cosine(a, b) >= 0.999999
    for L in layers:
        L.close()


def _emulate_p2p(w, xs, world, k, capacity, calls=1, logit_bias=None):
    """The peer-memory transport over `world` virtual ranks on one GPU: every
    rank's block is an allocation of this process, so the peer table holds
    plain device addresses.  Launch order keeps every wait already satisfied
    when it runs: all dispatches, then all expert steps, then all unpacks."""
    from moe_fused_inference_b200.ep import EPMoELayer, EPShard
    layers = [EPMoELayer(EPShard.from_layer(w, r, world), k, capacity, world=world, rank=r,
                         transport="p2p", connect=False, logit_bias=logit_bias)
              for r in range(world)]
    bases = [L.xch.base for L in layers]
    for L in layers:
        L.xch.connect(bases)
    outs = []
    for _ in range(calls):
        for L, x in zip(layers, xs):
            L.p2p_dispatch(x)
        for L in layers:
            L.p2p_experts()
        outs = []
        for L, x in zip(layers, xs):
            out = torch.full((x.shape[0], w.hidden), float("nan"), dtype=torch.float32,
                             device="cuda")
            L.p2p_finish(x.shape[0], out)
            outs.append(out)
        torch.cuda.synchronize()
    return layers, outs


@pytest.mark.parametrize("world,counts", [(2, [64, 64]), (4, [64, 17, 0, 33]),
                                          (8, [1, 0, 5, 64, 2, 31, 8, 3])])
def test_ep_p2p_emulated_matches_all_to_all(world, counts):
    """Peer-memory transport: same routing, bit-identical outputs to the
    all-to-all transport (same rows, same sums, same order), over three
    consecutive calls (call ids advance, buffers are reused)."""
    E, H, Mi, k = 128, 2048, 768, 8
    w = _layer_w(E, H, Mi, seed=21)
    xs = [_x(t, H, 90 + r) for r, t in enumerate(counts)]
    ref_layers, ref = _emulate(w, xs, world, k, max(counts))
    layers, outs = _emulate_p2p(w, xs, world, k, max(counts), calls=3)
    try:
        lib = _lib().load()
        assert lib.mfi_device_error(1) == 0
        for r, x in enumerate(xs):
            T = x.shape[0]
            assert torch.equal(layers[r].topi[:T], ref_layers[r].topi[:T])
            assert torch.equal(outs[r], ref[r])
    finally:
        for L in layers:
            L.close()


def test_ep_pack_rows_match_restatement():
    """The packed rows (keyed by token: row order inside a block follows
    atomics) equal the CPU restatement byte for byte."""
    from moe_fused_inference_b200.ep import EPMoELayer, EPShard
    E, H, Mi, k, world, T = 32, 512, 256, 4, 4, 23
    w = _layer_w(E, H, Mi, seed=11)
    x = _x(T, H, 5)
    L = EPMoELayer(EPShard.from_layer(w, 1, world), k, T, world=world, rank=1, transport="nccl")
    L.dispatch_prepare(x)
    torch.cuda.synchronize()
    W = mx.MoELayerWeights(*(t.cpu().numpy() for t in (w.gate_wp, w.gate_sc, w.up_wp, w.up_sc,
                                                        w.down_wp, w.down_sc, w.router_wp,
                                                        w.router_sc)))
    cpu = oep.CpuEPOps(W, 1, world, k, T)
    send = torch.zeros((world, T + 1, oep.row_bytes(H, k)), dtype=torch.uint8)
    counts = torch.zeros(world, dtype=torch.int32)
    pos = torch.zeros((T, world), dtype=torch.int32)
    xq, xsc = L.xq.cpu(), L.xsc.cpu()
    topi, topw = L.topi.cpu(), L.topw.cpu()
    cpu.pack(xq, xsc, topi, topw, T, counts, send, pos)
    g_send, g_pos = L.send.cpu().numpy(), L.pack_pos[:T].cpu().numpy()
    assert np.array_equal(L.counts.cpu().numpy(), counts.numpy())
    assert np.array_equal(g_pos >= 0, pos.numpy() >= 0)
    _, meta, _, _ = oep.offsets(H, k)
    for d in range(world):
        n = int(counts[d])
        assert int(np.frombuffer(g_send[d, 0, :4].tobytes(), np.int32)[0]) == n
        got = {int(np.frombuffer(g_send[d, 1 + i, meta:meta + 4].tobytes(), np.int32)[0]):
               g_send[d, 1 + i] for i in range(n)}
        want = {int(np.frombuffer(send[d, 1 + i, meta:meta + 4].numpy().tobytes(), np.int32)[0]):
                send[d, 1 + i].numpy() for i in range(n)}
        assert got.keys() == want.keys()
        for t in got:
            assert np.array_equal(got[t][: meta + 4], want[t][: meta + 4])
            assert np.array_equal(got[t][meta + 16:meta + 16 + 8 * k],
                                  want[t][meta + 16:meta + 16 + 8 * k])
            assert g_pos[t, d] >= 0


def test_route_matches_layer():
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k, T = 128, 2048, 768, 8, 40
    w = _layer_w(E, H, Mi, seed=4)
    x = _x(T, H, 9)
    lib = _lib().load()
    cw = _lib().MoEWeights(0, 0, 0, 0, 0, 0, w.router_wp.data_ptr(), w.router_sc.data_ptr(),
                           E, H, Mi, k, None)
    xq = torch.empty((T, H // 2), dtype=torch.uint8, device="cuda")
    xsc = torch.empty((T, H // 32), dtype=torch.uint8, device="cuda")
    topi = torch.empty((T, k), dtype=torch.int32, device="cuda")
    topw = torch.empty((T, k), dtype=torch.float32, device="cuda")
    logits = torch.empty((T, E), dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib().check(lib.mfi_moe_route(ctypes.byref(cw), x.data_ptr(), T, xq.data_ptr(), xsc.data_ptr(),
                                   topi.data_ptr(), topw.data_ptr(), logits.data_ptr(), st),
                 "moe_route")
    lg2 = torch.empty_like(logits)
    _, ti2, tw2 = MoELayer(w, top_k=k)(x, logits=lg2)
    torch.cuda.synchronize()
    assert torch.equal(logits, lg2) and torch.equal(topi, ti2) and torch.equal(topw, tw2)
    q, s = mx.quantize_rows(x.float().cpu().numpy())
    assert np.array_equal(xq.cpu().numpy(), q) and np.array_equal(xsc.cpu().numpy(), s)


def _experts_call(w, prepared, xq, xsc, sel, selw, R, k, out):
    L = _lib()
    lib = L.load()
    E, H, Mi = w.n_experts, w.hidden, w.inter
    cw = L.MoEWeights(w.gate_wp.data_ptr(), w.gate_sc.data_ptr(), w.up_wp.data_ptr(),
                      w.up_sc.data_ptr(), w.down_wp.data_ptr(), w.down_sc.data_ptr(), 0, 0,
                      E, H, Mi, k, prepared.data_ptr())
    nws = int(lib.mfi_moe_experts_workspace_bytes(R, H, Mi, E, k))
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    return lib.mfi_moe_experts(ctypes.byref(cw), xq.data_ptr(), xq.stride(0), xsc.data_ptr(),
                               xsc.stride(0), sel.data_ptr(), sel.stride(0), selw.data_ptr(),
                               selw.stride(0), R, out.data_ptr(), out.stride(0), ws.data_ptr(),
                               nws, st)


def test_experts_equal_layer_bit_exact():
    """mfi_moe_experts fed the layer's own routing reproduces mfi_moe_layer
    bit for bit (same expert GEMMs, same slot-ordered combine)."""
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k, T = 128, 2048, 768, 8, 64
    w = _layer_w(E, H, Mi, seed=6)
    x = _x(T, H, 12)
    layer = MoELayer(w, top_k=k)
    ref, topi, topw = layer(x)
    q, s = mx.quantize_rows(x.float().cpu().numpy())
    xq, xsc = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    _lib().check(_experts_call(w, layer.prepared, xq, xsc, topi, topw, T, k, out), "moe_experts")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_experts_masked_slots_and_empty_rows():
    E, H, Mi, k, R = 16, 512, 256, 4, 37
    from moe_fused_inference_b200.layer import MoELayer
    w = _layer_w(E, H, Mi, seed=8)
    layer = MoELayer(w, top_k=k)
    x = _x(R, H, 2)
    q, s = mx.quantize_rows(x.float().cpu().numpy())
    rng = np.random.default_rng(0)
    sel = np.full((R, k), -1, np.int32)
    for r in range(R):
        m = rng.integers(0, k + 1)  # 0..k valid slots, some rows none
        ids = rng.choice(E, size=m, replace=False)
        slots = rng.choice(k, size=m, replace=False)
        sel[r, slots] = ids
    selw = rng.random((R, k)).astype(np.float32)
    out = torch.full((R, H), 7.0, dtype=torch.float32, device="cuda")
    _lib().check(_experts_call(w, layer.prepared, torch.from_numpy(q).cuda(),
                               torch.from_numpy(s).cuda(), torch.from_numpy(sel).cuda(),
                               torch.from_numpy(selw).cuda(), R, k, out), "moe_experts")
    torch.cuda.synchronize()
    W = mx.MoELayerWeights(*(t.cpu().numpy() for t in (w.gate_wp, w.gate_sc, w.up_wp, w.up_sc,
                                                        w.down_wp, w.down_sc, w.router_wp,
                                                        w.router_sc)))
    want = np.zeros((R, H), np.float32)
    for r in range(R):
        for j in range(k):
            if sel[r, j] >= 0:
                y = oep.expert_row(q[r:r + 1], s[r:r + 1], W, int(sel[r, j]))[0]
                want[r] = (want[r] + (selw[r, j] * y).astype(np.float32)).astype(np.float32)
    got = out.cpu().numpy()
    empty = (sel < 0).all(axis=1)
    assert empty.any() and np.all(got[empty] == 0)
    # layer contract vs the float64-accumulated oracle
    assert max_rel_err(got, want) <= 1e-2
    assert cosine(got, want) >= 0.999


def test_experts_rejects_bad_args():
    L = _lib()
    lib = L.load()
    cw = L.MoEWeights(0, 0, 0, 0, 0, 0, 0, 0, 16, 512, 96, 4, None)
    st = lib.mfi_moe_experts(ctypes.byref(cw), 0, 256, 0, 16, 0, 4, 0, 4, 4, 0, 512, 0, 0, 0)
    assert st == 1 and b"multiples of 256" in lib.mfi_last_error()
    cw.inter = 256
    # past the prefill kernels' 262144 (row, slot) pairs
    st = lib.mfi_moe_experts(ctypes.byref(cw), 0, 256, 0, 16, 0, 4, 0, 4, 70000, 0, 512, 0, 0, 0)
    assert st == 1 and b"262144" in lib.mfi_last_error()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, outdir, transport):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from moe_fused_inference_b200.ep import EPMoELayer, EPShard
        from moe_fused_inference_b200.layer import MoELayer
        w = _layer_w(128, 2048, 768)
        counts = [64, 40]
        x = _x(counts[rank], 2048, 70 + rank)
        ep = EPMoELayer(EPShard.from_layer(w, rank, world), 8, 64, transport=transport)
        out = ep(x)
        out = ep(x)  # a second call: the call ids advance
        ref, topi, _ = MoELayer(w, top_k=8)(x)
        torch.cuda.synchronize()
        ep.close()
        np.save(os.path.join(outdir, f"nccl{rank}.npy"),
                np.array([max_rel_err(out.cpu().numpy(), ref.cpu().numpy()),
                          float(torch.equal(ep.topi[: counts[rank]], topi))]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_ep_nccl_two_ranks(tmp_path, transport):
    import torch.multiprocessing as mp
    mp.start_processes(_nccl_worker, args=(2, _free_port(), str(tmp_path), transport), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        rel, same = np.load(os.path.join(tmp_path, f"nccl{r}.npy"))
        assert same == 1.0 and rel <= 1e-5


def test_ep_p2p_zipf_bias_routes_like_single_gpu():
    """The Zipf(1.2) logit bias of the skewed scaling runs: the expert-parallel
    router applies it like the single-GPU layer (bit-identical top-k), and the
    outputs agree to the rank-ordered summation."""
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k, world = 128, 2048, 768, 8, 4
    w = _layer_w(E, H, Mi, seed=23)
    bias = torch.from_numpy(zipf_bias(E, alpha=0.5, seed=3))
    counts = [64, 40, 64, 9]
    xs = [_x(t, H, 130 + r) for r, t in enumerate(counts)]
    layers, outs = _emulate_p2p(w, xs, world, k, max(counts), logit_bias=bias.cuda())
    try:
        single = MoELayer(w, top_k=k, logit_bias=bias)
        for r, x in enumerate(xs):
            ref, topi, _ = single(x)
            torch.cuda.synchronize()
            T = x.shape[0]
            assert torch.equal(layers[r].topi[:T], topi)
            a, b = outs[r].cpu().numpy(), ref.cpu().numpy()
            assert max_rel_err(a, b) <= 1e-5
        assert _lib().load().mfi_device_error(1) == 0
    finally:
        for L in layers:
            L.close()


def test_ep_p2p_missing_peer_times_out():
    """A virtual rank that never dispatches (two ranks emulated on one GPU,
    rank 1 launches nothing): rank 0's expert step waits for rank 1's
    dispatch flag, a flag nothing sets, gives up after its bounded wait (2 s)
    and treats the block as empty; its unpack likewise gives up on rank 1's
    return.  Both calls return, the device error flag reads 7 (missing
    dispatch: the first failure wins over the later 8), and the GPU stays
    usable: a fresh single-GPU layer afterwards runs clean."""
    import time

    from moe_fused_inference_b200.ep import EPMoELayer, EPShard
    from moe_fused_inference_b200.layer import MoELayer
    E, H, Mi, k, world, C = 128, 2048, 768, 8, 2, 8
    w = _layer_w(E, H, Mi, seed=31)
    L = _lib().load()
    assert L.mfi_device_error(1) == 0
    layers = [EPMoELayer(EPShard.from_layer(w, r, world), k, C, world=world, rank=r,
                         transport="p2p", connect=False) for r in range(world)]
    try:
        bases = [x.xch.base for x in layers]
        for x in layers:
            x.xch.connect(bases)
        xin = _x(C, H, 150)
        out = torch.full((C, H), float("nan"), dtype=torch.float32, device="cuda")
        t0 = time.time()
        layers[0].p2p_dispatch(xin)
        layers[0].p2p_experts()
        layers[0].p2p_finish(C, out)
        torch.cuda.synchronize()
        elapsed = time.time() - t0
        assert L.mfi_device_error(1) == 7
        assert elapsed < 30.0
        # rank 0's own experts answered; rank 1's share of each token is missing
        assert bool(torch.isfinite(out).all())
    finally:
        for x in layers:
            x.close()
    # the context is still good and the flag was cleared: later calls are not
    # affected by the failure
    single = MoELayer(w, top_k=k)
    o, _, _ = single(xin)
    torch.cuda.synchronize()
    assert L.mfi_device_error(1) == 0
    assert bool(torch.isfinite(o).all())
