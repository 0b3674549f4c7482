"""Expert-parallel exchange protocol on CPU: two gloo ranks run EPMoELayer with
the CPU restatement of its per-step operations (oracle/ep.py), so the
all-to-all dispatch / return, the fixed-capacity blocks, ragged token counts
and the rank-ordered combine are checked without a GPU.

Expected values: oracle/ep.py:ep_layer (bit-exact: same per-row arithmetic
and summation order) and the single-device oracle layer (oracle/mxfp4.py:
moe_layer, which sums the slots in one sequence) to fp32 rounding.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep as oep
from oracle import mxfp4 as mx

E, H, MI, K = 8, 256, 256, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer():
    return mx.make_layer(np.random.default_rng(7), n_experts=E, hidden=H, inter=MI)


def _tokens(rank, t):
    rng = np.random.default_rng(100 + rank)
    return mx.bf16_round(rng.standard_normal((t, H)).astype(np.float32))


def _worker(rank, world, port, counts, capacity, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from moe_fused_inference_b200.ep import EPMoELayer, EPShard

        W = _layer()
        el = E // world
        s = slice(rank * el, (rank + 1) * el)
        t = torch.from_numpy
        shard = EPShard(t(W.wg[s]), t(W.sg[s]), t(W.wu[s]), t(W.su[s]), t(W.wd[s]), t(W.sd[s]),
                        t(W.wr), t(W.sr))
        ops = oep.CpuEPOps(W, rank, world, K, capacity)
        layer = EPMoELayer(shard, K, capacity, ops=ops, device="cpu")
        outs = []
        for step, tr in enumerate(counts[rank]):
            x = torch.from_numpy(_tokens(rank + 10 * step, tr)).to(torch.bfloat16)
            out = layer(x)
            outs.append((out.numpy().copy(), layer.topi[:tr].numpy().copy()))
        np.save(os.path.join(outdir, f"rank{rank}.npy"), np.array(outs, dtype=object),
                allow_pickle=True)
    finally:
        dist.destroy_process_group()


def _run(world, counts, capacity, tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, counts, capacity, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    return [np.load(os.path.join(tmp_path, f"rank{r}.npy"), allow_pickle=True)
            for r in range(world)]


def test_ep_two_ranks_ragged(tmp_path):
    # step 0: ragged counts; step 1: one rank sends nothing
    counts = [[5, 0], [3, 4]]
    res = _run(2, counts, 5, tmp_path)
    W = _layer()
    for step in range(2):
        xs = [_tokens(r + 10 * step, counts[r][step]) for r in range(2)]
        want = oep.ep_layer(xs, W, K, 2)
        for r in range(2):
            out, topi = res[r][step]
            assert out.shape == (counts[r][step], H)
            if counts[r][step] == 0:
                continue
            np.testing.assert_array_equal(topi, want[r]["idx"])
            np.testing.assert_array_equal(out, want[r]["out"])
            # single-device layer: same expert outputs, one summation sequence
            single = mx.moe_layer(xs[r], W, K)["out"]
            np.testing.assert_allclose(out, single, rtol=0, atol=1e-5 * np.abs(single).max())


def test_ep_row_layout_matches_library_header():
    from moe_fused_inference_b200 import ep
    for h, k in [(2048, 8), (256, 4), (4096, 1), (128, 32)]:
        assert ep.ep_row_bytes(h, k) == oep.row_bytes(h, k)
        assert ep.row_offsets(h, k) == oep.offsets(h, k)
        assert ep.ep_row_bytes(h, k) % 16 == 0
    # Qwen3-30B-A3B: 1,024 B nibbles + 64 B scales + 16 B meta + 64 B slots
    assert ep.ep_row_bytes(2048, 8) == 1168


def test_ep_layer_rejects_bad_shapes():
    from moe_fused_inference_b200.ep import EPShard
    W = _layer()
    t = torch.from_numpy
    shard = EPShard(t(W.wg[:3]), t(W.sg[:3]), t(W.wu[:3]), t(W.su[:3]), t(W.wd[:3]),
                    t(W.sd[:3]), t(W.wr), t(W.sr))
    assert shard.local_experts == 3 and shard.n_experts == E and shard.hidden == H
