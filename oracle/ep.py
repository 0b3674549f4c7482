"""CPU restatement of the expert-parallel exchange — TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module; the product path (moe_fused_inference_b200)
never does.  The reference has no multi-GPU path (it runs the MoE block of
runtime/model_runner_v2.py:183-208 on one device), so there is no reference
code to pin this against: it restates the library's own exchange format
(include/moe_fp4.h, "Expert-parallel exchange") on top of the pinned
single-device oracle (oracle/mxfp4.py), and its expected outputs are the
single-device expert results summed in the exchange's order:

    out[t] = sum over ranks d (ascending) of
             sum over slots j of t whose expert lives on d (ascending) of
             w[t, j] * y[t, j]                      (float32 multiply, add)

``CpuEPOps`` implements the per-step operations of
moe_fused_inference_b200.ep.EPMoELayer on CPU tensors with the same byte
layout, so the all-to-all protocol runs under the gloo backend without a GPU.
"""

from __future__ import annotations

import numpy as np

from . import mxfp4 as mx


def row_bytes(hidden: int, top_k: int) -> int:
    b = hidden // 2 + hidden // 32 + 16 + 8 * top_k
    return (b + 15) // 16 * 16


def offsets(hidden: int, top_k: int):
    sc = hidden // 2
    meta = sc + hidden // 32
    return sc, meta, meta + 16, meta + 16 + 4 * top_k


def expert_row(xq, xsc, W: mx.MoELayerWeights, e: int) -> np.ndarray:
    """One expert on one quantised row: the per-pair computation of
    mx.moe_layer (gate/up -> SwiGLU -> requantise -> down), float32 result."""
    g = mx.mx_gemm_f64(xq, xsc, W.wg[e], W.sg[e]).astype(np.float32)
    u = mx.mx_gemm_f64(xq, xsc, W.wu[e], W.su[e]).astype(np.float32)
    h = mx.silu_mul(g, u)
    hq, hsc = mx.quantize_rows(h)
    return mx.mx_gemm_f64(hq, hsc, W.wd[e], W.sd[e]).astype(np.float32)


def ep_layer(xs, W: mx.MoELayerWeights, topk: int, world: int):
    """Expected EP layer outputs for per-rank token batches ``xs`` (list of
    float32 arrays holding bf16 values).  Returns per-rank dicts with idx, w
    and out."""
    E = W.wr.shape[0]
    el = E // world
    res = []
    for x in xs:
        x = np.asarray(x, np.float32)
        xq, xsc = mx.quantize_rows(x)
        idx, w = mx.topk_route(mx.router_logits(xq, xsc, W.wr, W.sr), topk)
        t = x.shape[0]
        out = np.zeros((t, x.shape[1]), np.float32)
        for i in range(t):
            total = np.zeros(x.shape[1], np.float32)
            for d in range(world):
                slots = [j for j in range(topk) if idx[i, j] // el == d]
                if not slots:
                    continue
                part = np.zeros(x.shape[1], np.float32)
                for j in slots:
                    y = expert_row(xq[i : i + 1], xsc[i : i + 1], W, int(idx[i, j]))[0]
                    part = (part + (w[i, j] * y).astype(np.float32)).astype(np.float32)
                total = (total + part).astype(np.float32)
            out[i] = total
        res.append(dict(idx=idx, w=w, out=out, xq=xq, xsc=xsc))
    return res


class CpuEPOps:
    """Per-step operations of EPMoELayer on CPU torch tensors (numpy inside)."""

    def __init__(self, W: mx.MoELayerWeights, rank: int, world: int, top_k: int, capacity: int):
        self.W = W
        self.rank = rank
        self.world = world
        self.k = top_k
        self.C = capacity
        self.E = W.wr.shape[0]
        self.el = self.E // world
        self.H = W.wg.shape[2] * 2
        self.rb = row_bytes(self.H, top_k)

    def route(self, x, xq, xsc, topi, topw, logits=None):
        import torch
        xf = x.to(torch.float32).numpy()
        q, s = mx.quantize_rows(xf)
        lg = mx.router_logits(q, s, self.W.wr, self.W.sr)
        idx, w = mx.topk_route(lg, self.k)
        t = xf.shape[0]
        xq[:t] = torch.from_numpy(q)
        xsc[:t] = torch.from_numpy(s)
        topi[:t] = torch.from_numpy(idx)
        topw[:t] = torch.from_numpy(w)
        if logits is not None:
            logits[:t] = torch.from_numpy(lg)

    def pack(self, xq, xsc, topi, topw, T, counts, send, pack_pos):
        H, k = self.H, self.k
        sc, meta, sel, wo = offsets(H, k)
        s = send.numpy()
        q, scs = xq.numpy(), xsc.numpy()
        ti, tw = topi.numpy(), topw.numpy()
        cnt = np.zeros(self.world, np.int32)
        pp = pack_pos.numpy()
        for t in range(T):
            for d in range(self.world):
                if not np.any(ti[t] // self.el == d):
                    pp[t, d] = -1
                    continue
                pos = cnt[d]
                cnt[d] += 1
                pp[t, d] = pos
                row = s[d, 1 + pos]
                row[:sc] = q[t]
                row[sc:meta] = scs[t]
                row[meta : meta + 4] = np.frombuffer(np.int32(t).tobytes(), np.uint8)
                ids = np.where(ti[t] // self.el == d, ti[t] % self.el, -1).astype(np.int32)
                row[sel : sel + 4 * k] = np.frombuffer(ids.tobytes(), np.uint8)
                row[wo : wo + 4 * k] = np.frombuffer(tw[t].astype(np.float32).tobytes(), np.uint8)
        for d in range(self.world):
            s[d, 0, :4] = np.frombuffer(np.int32(cnt[d]).tobytes(), np.uint8)
        counts.numpy()[:] = cnt

    def experts(self, recv, ret):
        H, k = self.H, self.k
        sc, meta, sel, wo = offsets(H, k)
        r = recv.numpy()
        out = ret.numpy()
        out[:] = 0
        for s in range(self.world):
            count = int(np.frombuffer(r[s, 0, :4].tobytes(), np.int32)[0])
            if not 0 <= count <= self.C:
                # the library treats such a block as empty and reports device
                # error 9; on the host the step raises
                raise RuntimeError(f"received block from rank {s} has row count {count}, "
                                   f"outside [0, {self.C}]")
            for i in range(count):
                row = r[s, 1 + i]
                ids = np.frombuffer(row[sel : sel + 4 * k].tobytes(), np.int32)
                ws = np.frombuffer(row[wo : wo + 4 * k].tobytes(), np.float32)
                xq, xsc = row[:sc][None, :], row[sc:meta][None, :]
                acc = np.zeros(H, np.float32)
                for j in range(k):
                    if ids[j] < 0:
                        continue
                    e = self.rank * self.el + int(ids[j])
                    y = expert_row(xq, xsc, self.W, e)[0]
                    acc = (acc + (ws[j] * y).astype(np.float32)).astype(np.float32)
                out[s, 1 + i] = acc

    def unpack(self, ret_back, pack_pos, T, out):
        rb = ret_back.numpy()
        pp = pack_pos.numpy()
        o = out.numpy()
        for t in range(T):
            acc = np.zeros(self.H, np.float32)
            for d in range(self.world):
                if pp[t, d] >= 0:
                    acc = (acc + rb[d, 1 + pp[t, d]]).astype(np.float32)
            o[t] = acc
