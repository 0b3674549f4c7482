"""MXFP4 mirror I/O (moe_fused_inference_b200/mirror.py) against a mirror
written by the reference's own quantiser (tests/golden/mirror_ref, made by
tests/golden/make_golden.py from the seeded mini checkpoint it defines).

CPU: the reader parses the reference's shards, index and manifest and hands
out tensors whose bytes equal the oracle quantiser on the same inputs.
GPU: the writer, quantising on the device, reproduces the reference's
mirror file for file — every tensor, the shard assignment, the index and the
manifest (all but its creation time); a Qwen-shaped layer read back from a
mirror runs in the fused layer with the same results as the weights it was
written from.
"""

import json
import os

import numpy as np
import pytest
import torch

from oracle import mxfp4 as mx
from tests.conftest import GOLDEN
from tests.golden.make_golden import MIRROR_PATTERN, MIRROR_SHARD_GB, mini_checkpoint

REF = os.path.join(GOLDEN, "mirror_ref")


def _oracle_codes(name, ckpt):
    t = ckpt[name]
    s_inv = ckpt.get(name + "_scale_inv")
    if s_inv is not None:
        from moe_fused_inference_b200.mirror import dequant_fp8_blocks
        x = dequant_fp8_blocks(t, s_inv).numpy()
    else:
        x = t.float().numpy()
    return mx.quantize_rows(x)


def test_reader_parses_reference_mirror():
    from moe_fused_inference_b200.mirror import MirrorReader
    r = MirrorReader(REF, device="cpu")
    ckpt = mini_checkpoint()
    assert r.index is not None and len(r.handles) == 4  # sharded: 4 files and an index
    names = sorted(r.info)
    assert len(names) == 4 * 3 + 1 + 1  # bf16 experts, the FP8 expert, the router
    for name in names:
        spec = r.spec(name)
        p, c = _oracle_codes(name, ckpt)
        assert torch.equal(spec["wp"], torch.from_numpy(p)), name
        assert torch.equal(spec["wsc"], torch.from_numpy(c)), name
        assert spec["K"] == ckpt[name].shape[1]
    # non-expert tensors are float32 copies
    nw = ckpt["model.layers.0.post_attention_layernorm.weight"]
    assert np.array_equal(r.tensor("model.layers.0.post_attention_layernorm.weight"),
                          nw.float().numpy())
    ex = r.load_layer_experts(0, active={1, 3}, n_experts=4)
    assert sorted(ex) == [1, 3] and ex[1]["down"]["wp"].shape == (100, 32)
    static = r.load_static_v2()
    assert list(static) == ["model.layers.0.mlp.gate.weight"]
    assert r.manifest["tensors"]["model.layers.0.mlp.experts.4.gate_proj.weight"][
        "fp8_scale_inv_present"] is True


@pytest.mark.gpu
def test_writer_reproduces_reference_mirror(tmp_path):
    from safetensors import safe_open

    from moe_fused_inference_b200.mirror import write_mirror
    ckpt = mini_checkpoint()
    # the reference walks the checkpoint's tensors in safetensors key order
    names = sorted(ckpt)
    scale_inv = {k[: -len("_scale_inv")]: v for k, v in ckpt.items() if k.endswith("_scale_inv")}
    out = str(tmp_path / "mirror")
    write_mirror(out, [(k, ckpt[k]) for k in names], pattern=MIRROR_PATTERN, scale_inv=scale_inv,
                 copy_others=True, shard_gb=MIRROR_SHARD_GB)
    assert sorted(os.listdir(out)) == sorted(os.listdir(REF))
    a = json.load(open(os.path.join(out, "manifest.json")))
    b = json.load(open(os.path.join(REF, "manifest.json")))
    a.pop("created"), b.pop("created")
    assert a == b
    ia = json.load(open(os.path.join(out, "model.safetensors.index.json")))
    ib = json.load(open(os.path.join(REF, "model.safetensors.index.json")))
    assert ia["weight_map"] == ib["weight_map"]
    for fn in sorted(set(ib["weight_map"].values())):
        fa = safe_open(os.path.join(out, fn), framework="numpy")
        fb = safe_open(os.path.join(REF, fn), framework="numpy")
        assert sorted(fa.keys()) == sorted(fb.keys())
        for k in fb.keys():
            ta, tb = fa.get_tensor(k), fb.get_tensor(k)
            assert ta.dtype == tb.dtype and ta.shape == tb.shape and np.array_equal(ta, tb), k


@pytest.mark.gpu
def test_layer_round_trip_through_mirror(tmp_path):
    """A Qwen-shaped layer (16 experts to keep the files small) written to a
    mirror and read back stacks into the same packed weights, and the fused
    layer gives the same routing and output bit for bit."""
    from moe_fused_inference_b200.layer import MoELayer
    from moe_fused_inference_b200.mirror import MirrorReader, write_mirror
    E, H, Mi = 16, 2048, 768
    g = torch.Generator(device="cuda").manual_seed(5)
    bf = lambda *s: (torch.randn(s, generator=g, device="cuda") * 0.02).bfloat16()
    tensors = {"model.layers.3.mlp.gate.weight": bf(E, H)}
    for e in range(E):
        pre = f"model.layers.3.mlp.experts.{e}"
        tensors[f"{pre}.gate_proj.weight"] = bf(Mi, H)
        tensors[f"{pre}.up_proj.weight"] = bf(Mi, H)
        tensors[f"{pre}.down_proj.weight"] = bf(H, Mi)
    out = str(tmp_path / "m")
    write_mirror(out, tensors, pattern=MIRROR_PATTERN)
    w = MirrorReader(out).load_layer(3, n_experts=E)
    from moe_fused_inference_b200.layer import quantize_rows
    gp, gs = quantize_rows(tensors["model.layers.3.mlp.experts.7.gate_proj.weight"])
    assert torch.equal(w.gate_wp[7], gp) and torch.equal(w.gate_sc[7], gs)
    x = torch.randn((8, H), generator=g, device="cuda").bfloat16()
    o1, t1, _ = MoELayer(w, top_k=4)(x)
    # the same weights stacked directly from the device quantiser
    q = {k: quantize_rows(v) for k, v in tensors.items()}
    st = lambda p, i: torch.stack([q[f"model.layers.3.mlp.experts.{e}.{p}_proj.weight"][i]
                                   for e in range(E)]).contiguous()
    from moe_fused_inference_b200.layer import MoELayerWeights
    w2 = MoELayerWeights(st("gate", 0), st("gate", 1), st("up", 0), st("up", 1), st("down", 0),
                         st("down", 1), *q["model.layers.3.mlp.gate.weight"])
    o2, t2, _ = MoELayer(w2, top_k=4)(x)
    torch.cuda.synchronize()
    assert torch.equal(t1, t2) and torch.equal(o1, o2)
