#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is available (its path is the
first argument, default ``../reference`` next to the repository root or the
REFERENCE_ROOT environment variable).  It imports the reference's own Python
(quant/fp4_format.py, quant/quantize_mxfp4.py, runtime/weight_store.py,
runtime/model_runner.py), runs it on seeded inputs and writes small ``.npz``
fixtures next to this script.  The fixtures are committed; tests only read
them, so nothing at test time needs the reference.

Fixtures:
  quant_cases.npz      quantize_expert_tensor on bf16 inputs of the reference
                       tests' shapes (tests/correctness/test_mxfp4_decode.py:57,
                       quant/quantize_mxfp4.py:303-313) plus edge blocks.
  quant_exhaustive.npz one 32-element block per positive finite bf16 amax
                       (32,512 blocks): the reference's E8M0 codes and a
                       SHA-256 of its packed nibbles.
  quant_f32.npz        quantize_expert_tensor on float32 (non-bf16) inputs, the
                       form the down-projection input h takes.
  dequant.npz          mxfp4_reconstruct_gpu(device="cpu") of a packed tensor.
  route_moe.npz        ModelRunner.moe_route + moe_compute(variant="mxfp4") on
                       a small layer (BASELINE config 1 semantics, reduced size).
  rms_norm.npz         model_runner.rms_norm (runtime/model_runner.py:20-25) on
                       64 bf16 rows of width 2048 with a bf16 weight.
  mirror_ref/          an MXFP4 mirror (safetensors shards, index, manifest)
                       written by the reference's run_quantization
                       (quant/quantize_mxfp4.py:175-223) from the seeded mini
                       checkpoint of mini_checkpoint().
"""

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref_root():
    if len(sys.argv) > 1:
        return sys.argv[1]
    return os.environ.get("REFERENCE_ROOT", os.path.join(HERE, "..", "..", "..", "reference"))


def main():
    root = os.path.abspath(_ref_root())
    sys.path.insert(0, os.path.join(root, "quant"))
    sys.path.insert(0, os.path.join(root, "runtime"))
    from quantize_mxfp4 import quantize_expert_tensor  # noqa: E402
    from weight_store import mxfp4_reconstruct_gpu  # noqa: E402
    from model_runner import ModelRunner  # noqa: E402

    def qet(t):
        packed, codes, info = quantize_expert_tensor(t)
        n, kp = info["orig_shape"][0], info["padded_k"]
        return packed.reshape(n, kp // 2), codes

    # ---- 1. quantiser cases on bf16 inputs --------------------------------
    rng = np.random.default_rng(0)
    cases = {}
    shapes = [(1, 64), (1, 2048), (3, 768), (2, 100), (96, 128), (128, 100), (4, 40), (5, 33)]
    for i, (m, k) in enumerate(shapes):
        x = rng.standard_normal((m, k)).astype(np.float32) * 0.5
        x[rng.random((m, k)) < 0.01] *= 4.0
        xb = torch.from_numpy(x).bfloat16()
        p, c = qet(xb)
        cases[f"x{i}"] = xb.view(torch.int16).numpy().astype(np.uint16)
        cases[f"p{i}"] = p
        cases[f"c{i}"] = c
    # edge blocks: zeros, negative zeros, tiny (subnormal-range) values, huge values,
    # exact powers of two times 6, small negatives that round to zero magnitude
    edge = np.zeros((8, 64), np.float32)
    edge[1, :] = -0.0
    edge[2, :32] = np.ldexp(1.0, -133) * np.arange(32)          # bf16 subnormals
    edge[2, 32:] = np.ldexp(1.0, -126) * (np.arange(32) - 16)    # around min normal
    edge[3, :32] = 6.0 * np.ldexp(1.0, np.arange(32) - 10)
    edge[3, 32:] = -(2.0 ** 120) * (1 + np.arange(32) / 64.0)
    edge[4, :32] = 0.25 * np.array([1, -1] * 16)
    edge[4, 32:] = np.linspace(-6, 6, 32)
    edge[5, :] = 1e-3
    edge[5, 0] = 7.0
    edge[5, 1] = -1e-3
    edge[6, :] = rng.standard_normal(64) * 1e-38
    edge[7, :] = rng.uniform(-1.0, 1.0, 64) * 3e38
    eb = torch.from_numpy(edge).bfloat16()
    p, c = qet(eb)
    cases["edge_x"] = eb.view(torch.int16).numpy().astype(np.uint16)
    cases["edge_p"] = p
    cases["edge_c"] = c
    cases["n_cases"] = np.array(len(shapes))
    np.savez_compressed(os.path.join(HERE, "quant_cases.npz"), **cases)

    # ---- 2. exhaustive bf16 amax sweep ------------------------------------
    bits = np.arange(0x0001, 0x7F80, dtype=np.uint32)  # positive finite bf16
    amax = (bits << 16).view(np.float32)
    frac = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    blk = (amax[:, None] * frac[None, :]).astype(np.float32)
    blk[:, 0] = -amax
    blk[:, 31] = amax
    bb = torch.from_numpy(blk).bfloat16()
    p, c = qet(bb)
    np.savez_compressed(
        os.path.join(HERE, "quant_exhaustive.npz"),
        bits=bits.astype(np.uint16),
        frac=frac,
        codes=c.reshape(-1),
        packed_sha256=np.frombuffer(hashlib.sha256(p.tobytes()).digest(), np.uint8),
    )

    # ---- 3. float32 (non-bf16) inputs -------------------------------------
    rng = np.random.default_rng(3)
    xf = (rng.standard_normal((16, 768)).astype(np.float32)
          * np.exp(rng.standard_normal((16, 1))).astype(np.float32))
    p, c = qet(torch.from_numpy(xf))
    np.savez_compressed(os.path.join(HERE, "quant_f32.npz"), x=xf, p=p, c=c)

    # ---- 4. dequantisation -----------------------------------------------
    rng = np.random.default_rng(4)
    w = torch.from_numpy(rng.standard_normal((48, 100)).astype(np.float32)).bfloat16()
    packed, codes, info = quantize_expert_tensor(w)
    rec = mxfp4_reconstruct_gpu(packed, codes, 48, info["padded_k"], 100, "cpu")
    np.savez_compressed(os.path.join(HERE, "dequant.npz"),
                        p=packed.reshape(48, -1), c=codes, rec=rec.numpy())

    # ---- 5. moe_route + moe_compute("mxfp4"), reduced layer ---------------
    rng = np.random.default_rng(5)
    E, H, MI, T, K = 8, 128, 64, 4, 4
    cfg = {"num_experts_per_tok": K, "norm_topk_prob": True}
    runner = ModelRunner(None, cfg)
    wr = torch.from_numpy(rng.standard_normal((E, H)).astype(np.float32) * 0.02).bfloat16()
    runner.static = {"model.layers.0.mlp.gate.weight": wr}
    experts, packs = {}, {}
    for e in range(E):
        ed = {}
        for name, (n, k) in (("gate", (MI, H)), ("up", (MI, H)), ("down", (H, MI))):
            wt = torch.from_numpy(rng.standard_normal((n, k)).astype(np.float32) * 0.02).bfloat16()
            pk, cd, inf = quantize_expert_tensor(wt)
            rec = mxfp4_reconstruct_gpu(pk, cd, n, inf["padded_k"], k, "cpu")
            ed[name] = rec.to(torch.bfloat16)
            packs[f"{name}_p{e}"] = pk.reshape(n, -1)
            packs[f"{name}_c{e}"] = cd
        experts[e] = ed
    h = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).bfloat16()
    logits, topi, scores = runner.moe_route(h, 0)
    out = runner.moe_compute(h, topi, scores, experts, "mxfp4")
    np.savez_compressed(
        os.path.join(HERE, "route_moe.npz"),
        h=h.view(torch.int16).numpy().astype(np.uint16),
        wr=wr.view(torch.int16).numpy().astype(np.uint16),
        logits=logits.float().numpy(), topi=topi.numpy(),
        scores=scores.float().numpy(), out=out.float().numpy(),
        dims=np.array([E, H, MI, T, K]), **packs,
    )

    # ---- 6. rms_norm (the MoE block's post-attention layernorm) ------------
    from model_runner import rms_norm  # noqa: E402
    rng = np.random.default_rng(6)
    rows = rng.standard_normal((64, 2048)).astype(np.float32)
    rows *= np.power(2.0, rng.integers(-8, 9, size=(64, 1))).astype(np.float32)
    x = torch.from_numpy(rows).bfloat16()
    w = torch.from_numpy(1.0 + 0.1 * rng.standard_normal(2048).astype(np.float32)).bfloat16()
    y = rms_norm(x, w, 1e-6)
    np.savez_compressed(
        os.path.join(HERE, "rms_norm.npz"),
        x=x.view(torch.int16).numpy().astype(np.uint16),
        w=w.view(torch.int16).numpy().astype(np.uint16),
        y=y.view(torch.int16).numpy().astype(np.uint16), eps=np.float32(1e-6))

    # ---- 7. an MXFP4 mirror written by the reference's own quantiser -------
    import shutil
    import tempfile
    from safetensors.torch import save_file as save_torch
    from quantize_mxfp4 import run_quantization  # noqa: E402
    src = tempfile.mkdtemp(prefix="mfi_mini_ckpt_")
    save_torch(mini_checkpoint(), os.path.join(src, "model.safetensors"))
    out = os.path.join(HERE, "mirror_ref")
    shutil.rmtree(out, ignore_errors=True)
    run_quantization(src, out, MIRROR_PATTERN, MIRROR_SHARD_GB, True)
    shutil.rmtree(src)
    print("golden fixtures written to", HERE)


# The mirror fixture's inputs: one layer of 4 bf16 experts (K = 100, not a
# multiple of 32), a fifth expert stored as FP8 with a 128 x 128 block
# scale_inv (the official checkpoint's form), the router and a norm weight.
# Shared with the tests, which rebuild the same checkpoint.
MIRROR_PATTERN = r"(experts\.\d+\.(gate|up|down)_proj|mlp\.gate)\.weight$"
MIRROR_SHARD_GB = 16e-6  # about 17 KB: several shards and an index


def mini_checkpoint():
    rng = np.random.default_rng(7)
    t = {}
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).bfloat16()
    pre = "model.layers.0.mlp"
    for e in range(4):
        t[f"{pre}.experts.{e}.gate_proj.weight"] = bf(rng.standard_normal((64, 100)) * 0.02)
        t[f"{pre}.experts.{e}.up_proj.weight"] = bf(rng.standard_normal((64, 100)) * 0.02)
        t[f"{pre}.experts.{e}.down_proj.weight"] = bf(rng.standard_normal((100, 64)) * 0.02)
    w8 = torch.from_numpy(rng.standard_normal((128, 256)).astype(np.float32) * 8.0)
    t[f"{pre}.experts.4.gate_proj.weight"] = w8.to(torch.float8_e4m3fn)
    t[f"{pre}.experts.4.gate_proj.weight_scale_inv"] = torch.from_numpy(
        (0.001 + 0.01 * rng.random((1, 2))).astype(np.float32))
    t[f"{pre}.gate.weight"] = bf(rng.standard_normal((4, 100)) * 0.02)
    t["model.layers.0.post_attention_layernorm.weight"] = bf(1.0 + 0.1 * rng.standard_normal(100))
    return t


if __name__ == "__main__":
    main()
