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


# ---------------------------------------------------------------------------
# Failures made on the host (no GPU involved): a rank that leaves between
# steps, and a corrupted block count.  The surviving ranks must raise within
# the process group's timeout instead of hanging.

def _fail_worker(rank, world, port, mode, capacity, outdir):
    import datetime
    import json
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=15))
    res = {"rank": rank, "steps_done": 0, "raised": None}
    t0 = time.time()
    try:
        from moe_fused_inference_b200.ep import EPMoELayer, EPShard

        W = _layer()
        el = E // world
        s = slice(rank * el, (rank + 1) * el)
        t = torch.from_numpy
        shard = EPShard(t(W.wg[s]), t(W.sg[s]), t(W.wu[s]), t(W.su[s]), t(W.wd[s]), t(W.sd[s]),
                        t(W.wr), t(W.sr))
        layer = EPMoELayer(shard, K, capacity, ops=oep.CpuEPOps(W, rank, world, K, capacity),
                           device="cpu")
        for step in range(2):
            if mode == "dead" and rank == 1 and step == 1:
                break  # this rank leaves between steps: nothing of step 1 in flight
            x = torch.from_numpy(_tokens(rank + 10 * step, 3)).to(torch.bfloat16)
            layer.dispatch_prepare(x)
            if mode == "corrupt" and rank == 1 and step == 0:
                # the header of the block bound for rank 0 claims more rows than fit
                layer.send[0, 0, :4] = torch.from_numpy(
                    np.frombuffer(np.int32(capacity + 3).tobytes(), np.uint8).copy())
            dist.all_to_all_single(layer.recv.view(-1), layer.send.view(-1))
            layer.compute()
            dist.all_to_all_single(layer.ret_back.view(-1), layer.ret.view(-1))
            out = torch.empty((3, H), dtype=torch.float32)
            layer.finish(3, out)
            res["steps_done"] = step + 1
    except Exception as e:  # noqa: BLE001 - the failure under test
        res["raised"] = f"{type(e).__name__}: {e}"[:300]
    res["seconds"] = time.time() - t0
    with open(os.path.join(outdir, f"fail{rank}.json"), "w") as f:
        json.dump(res, f)
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - the group may already be broken
        pass


def _run_fail(mode, tmp_path, world=2, capacity=4):
    import json
    port = _free_port()
    mp.start_processes(_fail_worker, args=(world, port, mode, capacity, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    return [json.load(open(os.path.join(tmp_path, f"fail{r}.json"))) for r in range(world)]


def test_ep_rank_leaves_between_steps(tmp_path):
    """Rank 1 completes step 0 and exits; rank 0's step-1 dispatch (a
    collective with a departed peer) must raise, not hang."""
    res = _run_fail("dead", tmp_path)
    assert res[1]["steps_done"] == 1 and res[1]["raised"] is None
    assert res[0]["steps_done"] == 1
    assert res[0]["raised"] is not None
    assert res[0]["seconds"] < 60


def test_ep_corrupted_block_count(tmp_path):
    """Rank 1 sends rank 0 a block whose header claims capacity + 3 rows:
    rank 0's expert step rejects it (the GPU library treats such a block as
    empty and reports device error 9) and leaves; rank 1, waiting for rank
    0's return, must then raise too."""
    res = _run_fail("corrupt", tmp_path)
    assert res[0]["steps_done"] == 0 and "row count" in (res[0]["raised"] or "")
    assert res[1]["steps_done"] == 0 and res[1]["raised"] is not None
    assert res[0]["seconds"] < 60 and res[1]["seconds"] < 60
