"""MXFP4 mirror I/O: the reference's on-disk weight format, written from the
GPU quantiser and read back for the kernels.

Format (written by the reference's quant/quantize_mxfp4.py:41-87, 175-223 and
read by runtime/weight_store.py:178-198, 265-286):

  <dir>/model.safetensors, or model-XXXXX-of-XXXXX.safetensors shards plus
      model.safetensors.index.json ({"metadata": {"total_size"}, "weight_map"})
      <name>.fp4_data   uint8, flat: the packed E2M1 nibbles of the (N, Kp)
                        weight, LSB first, Kp = K rounded up to 32
      <name>.fp4_scale  uint8 (N, Kp/32): E8M0 codes
      other tensors     float32 copies of non-quantised weights (norms, ...)
  <dir>/manifest.json
      {"format": "mxfp4-1x32-e8m0-e2m1", "block_size": 32,
       "scale_type": "e8m0_power_of_2", "created": ..., "stats": {...},
       "tensors": {<name>: {"orig_shape", "orig_dtype", "padded_k", "pad",
                            "n_elements", "scale_shape", "scale_dtype",
                            "data_key", "scale_key", "fp8_scale_inv_present"}}}

``write_mirror`` quantises with the library's bit-exact device form of
quantize_expert_tensor (mfi_quantize_rows), so a checkpoint that takes the
reference's CPU quantiser about 73 s per layer is quantised in milliseconds,
with identical bytes.  ``MirrorReader`` hands the tensors out as the
reference's spec dicts ({"wp", "wsc", "K"}, runtime/weight_store.py:283-285),
as a static-weights dict (load_static_v2) or stacked into one layer's
``MoELayerWeights`` for the fused layer.
"""

from __future__ import annotations

import json
import os
import re
import time

import numpy as np
import torch

from .layer import MoELayerWeights, quantize_rows

FORMAT = "mxfp4-1x32-e8m0-e2m1"
BLOCK = 32
EXPERT_RE = r"experts\.\d+\.(gate|up|down)_proj\.weight$"


def _save_file(tensors: dict, path: str) -> None:
    from safetensors.numpy import save_file
    save_file(tensors, path)


def dequant_fp8_blocks(w8: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """FP8 checkpoint weight with a 128 x 128 block scale_inv -> fp32 (the
    official checkpoint's form, reference quant/quantize_mxfp4.py:95-104):
    w[b, i] = float(w8[b, i]) * scale_inv[b // 128, i // 128]."""
    out, inp = w8.shape
    if out % block or inp % block:
        raise RuntimeError(f"FP8 block dequantisation needs dimensions divisible by {block}: "
                           f"{tuple(w8.shape)}")
    w = w8.float().view(out // block, block, inp // block, block)
    w = w * scale_inv.view(out // block, 1, inp // block, 1).float()
    return w.reshape(out, inp)


class _ShardWriter:
    """Accumulates tensors and writes a shard each time max_bytes is reached;
    finalize() names the shards as the reference does (one file:
    model.safetensors; several: model-XXXXX-of-XXXXX.safetensors and an
    index)."""

    def __init__(self, out_dir: str, max_bytes: int):
        self.out_dir, self.max_bytes = out_dir, max_bytes
        os.makedirs(out_dir, exist_ok=True)
        self.buf, self.nbytes = {}, 0
        self.tmp, self.weight_map = [], {}

    def add(self, name: str, arr: np.ndarray) -> None:
        self.buf[name] = np.ascontiguousarray(arr)
        self.nbytes += arr.nbytes
        if self.nbytes >= self.max_bytes:
            self._flush()

    def _flush(self) -> None:
        if not self.buf:
            return
        fn = f"tmp-{len(self.tmp) + 1:05d}.safetensors"
        _save_file(self.buf, os.path.join(self.out_dir, fn))
        for k in self.buf:
            self.weight_map[k] = fn
        self.tmp.append(fn)
        self.buf, self.nbytes = {}, 0

    def finalize(self) -> None:
        self._flush()
        n = len(self.tmp)
        if n == 1:
            os.replace(os.path.join(self.out_dir, self.tmp[0]),
                       os.path.join(self.out_dir, "model.safetensors"))
            return
        rename = {}
        for i, t in enumerate(self.tmp, 1):
            final = f"model-{i:05d}-of-{n:05d}.safetensors"
            os.replace(os.path.join(self.out_dir, t), os.path.join(self.out_dir, final))
            rename[t] = final
        wm = {k: rename[v] for k, v in self.weight_map.items()}
        total = sum(os.path.getsize(os.path.join(self.out_dir, f)) for f in set(wm.values()))
        with open(os.path.join(self.out_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": int(total)}, "weight_map": wm}, f, indent=2)


def write_mirror(out_dir: str, tensors, pattern: str = EXPERT_RE, scale_inv=None,
                 copy_others: bool = False, shard_gb: float = 2.0, device="cuda") -> dict:
    """Write a mirror of ``tensors`` (an iterable of (name, tensor) pairs, or a
    dict): every 2-D tensor whose name matches ``pattern`` is quantised on the
    GPU (bit-exact quantize_expert_tensor) and stored as <name>.fp4_data /
    <name>.fp4_scale; others are copied as float32 when ``copy_others``.
    ``scale_inv`` maps a name to its FP8 128 x 128 block scale (the FP8
    checkpoint's <name>_scale_inv), applied before quantisation; tensors
    whose name ends in _scale_inv are never written.  Returns the manifest."""
    rx = re.compile(pattern)
    items = tensors.items() if isinstance(tensors, dict) else tensors
    scale_inv = scale_inv or {}
    w = _ShardWriter(out_dir, int(shard_gb * 1024 ** 3))
    manifest = {"format": FORMAT, "block_size": BLOCK, "scale_type": "e8m0_power_of_2",
                "created": time.strftime("%Y-%m-%d %H:%M:%S"), "tensors": {}}
    stats = {"expert_tensors": 0, "copied_tensors": 0, "skipped_tensors": 0,
             "consumed_scale_inv": 0, "input_bytes": 0, "fp4_bytes": 0, "scale_bytes": 0}
    for name, t in items:
        stats["input_bytes"] += t.element_size() * t.numel()
        if rx.search(name):
            if t.dim() != 2:
                raise RuntimeError(f"{name}: only 2-D weights are quantised")
            s_inv = scale_inv.get(name)
            x = t.to(device)
            if s_inv is not None:
                x = dequant_fp8_blocks(x, s_inv.to(device))
            elif x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                x = x.float()
            n, k = x.shape
            wp, wsc = quantize_rows(x)
            kp = wp.shape[1] * 2
            dk, sk = name + ".fp4_data", name + ".fp4_scale"
            data = wp.reshape(-1).cpu().numpy()
            codes = wsc.cpu().numpy()
            w.add(dk, data)
            w.add(sk, codes)
            manifest["tensors"][name] = {
                "orig_shape": [int(n), int(k)], "orig_dtype": str(t.dtype), "padded_k": int(kp),
                "pad": int(kp - k), "n_elements": int(n * k), "scale_shape": list(codes.shape),
                "scale_dtype": "e8m0_uint8", "data_key": dk, "scale_key": sk,
                "fp8_scale_inv_present": s_inv is not None}
            stats["expert_tensors"] += 1
            stats["fp4_bytes"] += data.nbytes
            stats["scale_bytes"] += codes.nbytes
            if s_inv is not None:
                stats["consumed_scale_inv"] += 1
        elif name.endswith("_scale_inv"):
            continue
        elif copy_others:
            w.add(name, t.float().cpu().numpy())
            stats["copied_tensors"] += 1
        else:
            stats["skipped_tensors"] += 1
    w.finalize()
    manifest["stats"] = stats
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


class MirrorReader:
    """Read access to a mirror directory (safetensors handles opened once)."""

    def __init__(self, mirror_dir: str, device="cuda"):
        from safetensors import safe_open
        self.dir = mirror_dir
        self.device = device
        with open(os.path.join(mirror_dir, "manifest.json")) as f:
            self.manifest = json.load(f)
        if self.manifest.get("format") != FORMAT:
            raise RuntimeError(f"{mirror_dir}: unknown mirror format {self.manifest.get('format')!r}")
        self.info = self.manifest["tensors"]
        idx = os.path.join(mirror_dir, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                self.index = json.load(f)["weight_map"]
            files = sorted(set(self.index.values()))
        else:
            self.index = None
            files = sorted(f for f in os.listdir(mirror_dir) if f.endswith(".safetensors"))
        self.handles = {fn: safe_open(os.path.join(mirror_dir, fn), framework="numpy")
                        for fn in files}

    def _get(self, key: str) -> np.ndarray:
        if self.index is not None:
            return self.handles[self.index[key]].get_tensor(key)
        for h in self.handles.values():
            if key in h.keys():
                return h.get_tensor(key)
        raise KeyError(key)

    def tensor(self, name: str) -> np.ndarray:
        """A non-quantised tensor (float32 copy) of the mirror."""
        return self._get(name)

    def spec(self, name: str) -> dict:
        """{"wp": uint8 (N, Kp/2), "wsc": uint8 (N, Kp/32), "K": K} on the
        reader's device — the reference's spec dict (runtime/weight_store.py:
        283-285)."""
        info = self.info[name]
        n, kp = info["orig_shape"][0], info["padded_k"]
        data = np.ascontiguousarray(self._get(info["data_key"]))
        codes = np.ascontiguousarray(self._get(info["scale_key"]))
        if data.size != n * kp // 2 or codes.shape != (n, kp // BLOCK):
            raise RuntimeError(f"{name}: stored sizes do not match the manifest")
        return {"wp": torch.from_numpy(data.reshape(n, kp // 2)).to(self.device),
                "wsc": torch.from_numpy(codes).to(self.device), "K": int(info["orig_shape"][1])}

    def load_static_v2(self) -> dict:
        """Every quantised tensor that is not an expert weight, as spec dicts
        (the fp4 half of runtime/weight_store.py:178-198)."""
        rx = re.compile(EXPERT_RE)
        return {k: self.spec(k) for k in self.info if not rx.search(k)}

    def load_layer_experts(self, layer: int, active=None, n_experts: int = 128) -> dict:
        """eid -> {"gate", "up", "down"} spec dicts (the "mxfp4_mma" variant of
        runtime/weight_store.py:265-286)."""
        ids = range(n_experts) if active is None else sorted(active)
        out = {}
        for e in ids:
            pre = f"model.layers.{layer}.mlp.experts.{e}"
            out[e] = {p: self.spec(f"{pre}.{p}_proj.weight") for p in ("gate", "up", "down")}
        return out

    def load_layer(self, layer: int, n_experts: int = 128,
                   router_key: str | None = None) -> MoELayerWeights:
        """One layer stacked for the fused MoE layer: experts 0..n-1 and the
        router (model.layers.<L>.mlp.gate.weight, quantised in the mirror)."""
        ex = self.load_layer_experts(layer, n_experts=n_experts)
        r = self.spec(router_key or f"model.layers.{layer}.mlp.gate.weight")

        def st(p, k):
            return torch.stack([ex[e][p][k] for e in range(n_experts)]).contiguous()

        return MoELayerWeights(st("gate", "wp"), st("gate", "wsc"), st("up", "wp"), st("up", "wsc"),
                               st("down", "wp"), st("down", "wsc"), r["wp"].contiguous(),
                               r["wsc"].contiguous())
