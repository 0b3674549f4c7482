"""Device-routed MXFP4 MoE layer and the GPU weight quantiser.

``MoELayer`` holds one Qwen3-MoE layer's packed weights stacked over experts
(the reference keeps them as per-expert tensors in WeightStore dicts,
runtime/weight_store.py:265-286) and runs the whole MoE block of
model_runner_v2 (runtime/model_runner_v2.py:183-208 for T = 1, :266-290 for
T = M) as one library call: activation quantisation, router GEMM, top-k,
grouped gate/up, SwiGLU requantisation, grouped down and the top-k combine,
with no host synchronisation in between.

``quantize_rows`` is the device form of the reference's
``quantize_expert_tensor`` (quant/quantize_mxfp4.py:110-160), bit-exact on
bf16 inputs; it is what builds the random-init model quickly (the reference's
CPU quantiser takes about 73 s per layer).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

_DT = {torch.float32: _lib.MFI_F32, torch.float16: _lib.MFI_F16, torch.bfloat16: _lib.MFI_BF16}


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def ceil32(k: int) -> int:
    return (k + 31) // 32 * 32


def quantize_rows(x: torch.Tensor, half_roundtrip: bool = False):
    """(M, K) float cuda tensor -> (packed (M, Kp/2) uint8, codes (M, Kp/32) uint8)."""
    lib = _lib.load()
    if not x.is_cuda:
        raise RuntimeError("x must be cuda")
    if x.dtype not in _DT:
        raise RuntimeError("x must be float32, float16 or bfloat16")
    if x.dim() != 2:
        raise RuntimeError("x must be 2-D")
    if x.stride(1) != 1:
        x = x.contiguous()
    M, K = x.shape
    Kp = ceil32(K)
    xq = torch.empty((M, Kp // 2), dtype=torch.uint8, device=x.device)
    xsc = torch.empty((M, Kp // 32), dtype=torch.uint8, device=x.device)
    if M and K:
        st = lib.mfi_quantize_rows(x.data_ptr(), _DT[x.dtype], x.stride(0), int(half_roundtrip),
                                   xq.data_ptr(), xsc.data_ptr(), M, K, Kp, _stream(x.device))
        _lib.check(st, "quantize_rows")
    return xq, xsc


@dataclass
class MoELayerWeights:
    """Stacked packed weights of one MoE layer (all uint8, cuda, contiguous)."""

    gate_wp: torch.Tensor   # (E, inter, hidden/2)
    gate_sc: torch.Tensor   # (E, inter, hidden/32)
    up_wp: torch.Tensor
    up_sc: torch.Tensor
    down_wp: torch.Tensor   # (E, hidden, inter/2)
    down_sc: torch.Tensor   # (E, hidden, inter/32)
    router_wp: torch.Tensor  # (E, hidden/2)
    router_sc: torch.Tensor  # (E, hidden/32)

    @property
    def n_experts(self) -> int:
        return self.gate_wp.shape[0]

    @property
    def hidden(self) -> int:
        return self.gate_wp.shape[2] * 2

    @property
    def inter(self) -> int:
        return self.gate_wp.shape[1]

    def validate(self) -> None:
        E, H, Mi = self.n_experts, self.hidden, self.inter
        want = {
            "gate_wp": (E, Mi, H // 2), "gate_sc": (E, Mi, H // 32),
            "up_wp": (E, Mi, H // 2), "up_sc": (E, Mi, H // 32),
            "down_wp": (E, H, Mi // 2), "down_sc": (E, H, Mi // 32),
            "router_wp": (E, H // 2), "router_sc": (E, H // 32),
        }
        for name, shape in want.items():
            t = getattr(self, name)
            if not (t.is_cuda and t.dtype == torch.uint8 and t.is_contiguous()):
                raise RuntimeError(f"{name} must be a contiguous cuda uint8 tensor")
            if tuple(t.shape) != shape:
                raise RuntimeError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if H % 32 or Mi % 32:
            raise RuntimeError("hidden and inter must be multiples of 32")

    @staticmethod
    def from_expert_lists(gate, up, down, router):
        """Stack per-expert (wp, wsc) pairs — the reference WeightStore spec
        dicts (runtime/weight_store.py:283-285) — into the layer layout."""
        def st(pairs, i):
            return torch.stack([p[i] for p in pairs]).contiguous()
        return MoELayerWeights(st(gate, 0), st(gate, 1), st(up, 0), st(up, 1),
                               st(down, 0), st(down, 1),
                               router[0].contiguous(), router[1].contiguous())


def random_layer_weights(n_experts=128, hidden=2048, inter=768, std=0.02, seed=0,
                         device="cuda") -> MoELayerWeights:
    """Random-init layer: bf16 N(0, std) weights (router included), quantised on
    the GPU with the quantize_expert_tensor rules."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def q(rows, k):
        w = (torch.randn((rows, k), generator=g, device=device, dtype=torch.float32) * std)
        return quantize_rows(w.to(torch.bfloat16))

    gwp, gsc = q(n_experts * inter, hidden)
    uwp, usc = q(n_experts * inter, hidden)
    dwp, dsc = q(n_experts * hidden, inter)
    rwp, rsc = q(n_experts, hidden)
    E, H, Mi = n_experts, hidden, inter
    return MoELayerWeights(
        gwp.view(E, Mi, H // 2), gsc.view(E, Mi, H // 32),
        uwp.view(E, Mi, H // 2), usc.view(E, Mi, H // 32),
        dwp.view(E, H, Mi // 2), dsc.view(E, H, Mi // 32),
        rwp, rsc)


class MoELayer:
    """One device-routed MoE layer call per forward (library entry mfi_moe_layer)."""

    def __init__(self, weights: MoELayerWeights, top_k: int = 8, logit_bias=None,
                 norm_weight=None, norm_eps: float = 1e-6):
        """``logit_bias``: optional cuda float32 (E,) added to the router logits
        before top-k (a synthetic load skew; the reference has no such term).
        ``norm_weight``: optional bf16 (hidden,) RMSNorm weight — the MoE
        block's post-attention layernorm (runtime/model_runner.py:20-25) fused
        into the router: forward() then takes the residual stream x and
        normalises each row before quantising it."""
        weights.validate()
        if not 1 <= top_k <= min(weights.n_experts, 32):
            raise RuntimeError("top_k must be in [1, min(E, 32)]")
        self.w = weights
        self.top_k = top_k
        lib = _lib.load()
        self._cw = _lib.MoEWeights(
            weights.gate_wp.data_ptr(), weights.gate_sc.data_ptr(),
            weights.up_wp.data_ptr(), weights.up_sc.data_ptr(),
            weights.down_wp.data_ptr(), weights.down_sc.data_ptr(),
            weights.router_wp.data_ptr(), weights.router_sc.data_ptr(),
            weights.n_experts, weights.hidden, weights.inter, top_k, None, None)
        self.logit_bias = None
        if logit_bias is not None:
            lb = logit_bias.to(device=weights.gate_wp.device, dtype=torch.float32).contiguous()
            if lb.shape != (weights.n_experts,):
                raise RuntimeError("logit_bias must have shape (E,)")
            self.logit_bias = lb
            self._cw.logit_bias = lb.data_ptr()
        self.norm_weight = None
        if norm_weight is not None:
            nw = norm_weight.to(device=weights.gate_wp.device, dtype=torch.bfloat16).contiguous()
            if nw.shape != (weights.hidden,):
                raise RuntimeError("norm_weight must have shape (hidden,)")
            self.norm_weight = nw
            self._cw.norm_weight = nw.data_ptr()
            self._cw.norm_eps = float(norm_eps)
        # tensor-core scale atoms, built once per weight set (mfi_moe_prepare)
        nprep = int(lib.mfi_moe_prepared_bytes(weights.n_experts, weights.hidden, weights.inter))
        self.prepared = None
        if nprep:
            dev = weights.gate_wp.device
            self.prepared = torch.empty(nprep, dtype=torch.uint8, device=dev)
            self._cw.prepared = self.prepared.data_ptr()
            _lib.check(lib.mfi_moe_prepare(ctypes.byref(self._cw), self.prepared.data_ptr(), nprep,
                                           _stream(dev)), "moe_prepare")
        self._ws = {}

    def workspace_bytes(self, T: int) -> int:
        return int(_lib.load().mfi_moe_layer_workspace_bytes(
            T, self.w.hidden, self.w.inter, self.w.n_experts, self.top_k))

    def _workspace(self, T: int, device) -> torch.Tensor:
        ws = self._ws.get(T)
        if ws is None:
            lib = _lib.load()
            ws = torch.empty(self.workspace_bytes(T), dtype=torch.uint8, device=device)
            _lib.check(lib.mfi_moe_layer_init_workspace(
                ws.data_ptr(), ws.numel(), T, self.w.hidden, self.w.inter, self.w.n_experts,
                self.top_k, _stream(device)), "moe_layer_init_workspace")
            self._ws[T] = ws
        return ws

    def prefill(self, x: torch.Tensor, out=None, topi=None, topw=None, logits=None):
        """The prefill path (mfi_moe_layer_prefill) for any T: compact
        count-based expert placement and 128-token tensor-core tiles.  forward()
        takes it by itself when T * top_k > 4096."""
        lib = _lib.load()
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("x must be a cuda bfloat16 tensor")
        x = x.contiguous()
        T, H = x.shape
        dev = x.device
        k = self.top_k
        out = torch.empty((T, H), dtype=torch.float32, device=dev) if out is None else out
        topi = torch.empty((T, k), dtype=torch.int32, device=dev) if topi is None else topi
        topw = torch.empty((T, k), dtype=torch.float32, device=dev) if topw is None else topw
        nbytes = int(lib.mfi_moe_layer_prefill_workspace_bytes(T, self.w.hidden, self.w.inter,
                                                                self.w.n_experts, k))
        ws = self._ws.get(("prefill", T))
        if ws is None:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            self._ws[("prefill", T)] = ws
        st = lib.mfi_moe_layer_prefill(ctypes.byref(self._cw), x.data_ptr(), T, out.data_ptr(),
                                       topi.data_ptr(), topw.data_ptr(),
                                       0 if logits is None else logits.data_ptr(),
                                       ws.data_ptr(), ws.numel(), _stream(dev))
        _lib.check(st, "moe_layer_prefill")
        return out, topi, topw

    def forward(self, x: torch.Tensor, out=None, topi=None, topw=None, logits=None, events=None):
        """x bf16 (T, hidden) -> (out fp32 (T, hidden), topi int32 (T, k), topw fp32 (T, k)).

        ``logits`` (fp32 (T, E)) is filled when given.  Output tensors may be
        passed in to keep the call allocation-free (CUDA-graph capture).
        ``events``: six torch.cuda.Event(enable_timing=True) recorded at the
        stage boundaries (see mfi_moe_layer_ex in include/moe_fp4.h)."""
        lib = _lib.load()
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("x must be a cuda bfloat16 tensor")
        x = x.contiguous()
        T, H = x.shape
        if H != self.w.hidden:
            raise RuntimeError(f"x must have {self.w.hidden} columns")
        dev = x.device
        k = self.top_k
        out = torch.empty((T, H), dtype=torch.float32, device=dev) if out is None else out
        topi = torch.empty((T, k), dtype=torch.int32, device=dev) if topi is None else topi
        topw = torch.empty((T, k), dtype=torch.float32, device=dev) if topw is None else topw
        ws = self._workspace(T, dev)
        if events is None:
            st = lib.mfi_moe_layer(ctypes.byref(self._cw), x.data_ptr(), T, out.data_ptr(),
                                   topi.data_ptr(), topw.data_ptr(),
                                   0 if logits is None else logits.data_ptr(),
                                   ws.data_ptr(), ws.numel(), _stream(dev))
        else:
            evs = (ctypes.c_void_p * 6)(*[e.cuda_event for e in events])
            st = lib.mfi_moe_layer_ex(ctypes.byref(self._cw), x.data_ptr(), T, out.data_ptr(),
                                      topi.data_ptr(), topw.data_ptr(),
                                      0 if logits is None else logits.data_ptr(),
                                      ws.data_ptr(), ws.numel(), evs, 6, _stream(dev))
        _lib.check(st, "moe_layer")
        return out, topi, topw

    __call__ = forward
