"""Synthetic Qwen3-30B-A3B decode runner over the MXFP4 path.

The reference's model runner (runtime/model_runner_v2.py) is the caller of
this library's operators; it cannot run on a B200 box as shipped (its
extensions build for sm_120a only), so this module restates its per-layer
operation sequence — the same ops, in the same order, with the same dtypes —
over a pluggable backend, for B independent sequences at once:

  embedding rows      dequant_rows_gpu of the MXFP4 embedding
                      (runtime/weight_store.py:47-65)
  per layer           rms_norm -> prequant -> q/k/v lin_pq -> q_norm/k_norm ->
                      RoPE -> FP8 KV write (torch float8_e4m3fn cast) ->
                      attention -> prequant -> o lin_pq -> residual add ->
                      rms_norm -> MoE block (router, top-8, experts, combine)
                      -> residual add      (runtime/model_runner_v2.py:244-290)
  head                rms_norm -> prequant -> lm_head lin_pq   (:292-297)

Rows of one forward are B sequences x M tokens: M = 1 is a decode step,
M = L + 1 the prompt-lookup speculative verify (runtime/spec_decoder.py:94-122),
M = a prompt chunk for prefill.  Attention of the M rows of a sequence runs
over its own FP8 cache with the reference's attn_decode semantics (row m sees
positions up to base + m).

The library backend (``LibBackend``) runs the MoE block as the fused device-
routed layer (mfi_moe_layer) and everything else through the drop-in
operators (fp4_ext: prequant, lin_pq, attn_decode).  A test backend with the
same interface restates the operators in torch (dequantise, fp32 matmul) so
greedy token ids can be compared step by step.

Weights are random-init (N(0, 0.02), the norms 1 + N(0, 0.02)), quantised on
the device; there is no checkpoint or tokenizer on this path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .layer import MoELayer, MoELayerWeights, quantize_rows, random_layer_weights


@dataclass
class QwenConfig:
    hidden: int = 2048
    layers: int = 48
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    vocab: int = 151936
    experts: int = 128
    top_k: int = 8
    inter: int = 768
    rope_theta: float = 1e6
    eps: float = 1e-6


# ---- reference helpers restated (runtime/model_runner.py:20-42,
# runtime/weight_store.py:47-65) ------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dtype = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(dtype) * weight


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float) -> torch.Tensor:
    """x (T, H, D), positions (T,): half-layout RoPE."""
    D = x.shape[-1]
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, device=x.device).float() / D))
    freqs = positions.float()[:, None] * inv_freq[None, :]
    cos = torch.cat([freqs.cos(), freqs.cos()], dim=-1)[:, None]
    sin = torch.cat([freqs.sin(), freqs.sin()], dim=-1)[:, None]
    x1, x2 = x.chunk(2, dim=-1)
    rot = torch.cat((-x2, x1), dim=-1)
    return (x * cos + rot * sin).to(x.dtype)


_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
_E2M1_DEV: dict = {}


def _e2m1_table(device) -> torch.Tensor:
    """The E2M1 magnitudes on `device` (made once, so the gather can run while
    a CUDA graph is being captured)."""
    key = str(device)
    t = _E2M1_DEV.get(key)
    if t is None:
        t = _E2M1_DEV[key] = torch.tensor(_E2M1, device=device)
    return t


def dequant_rows(wp: torch.Tensor, wsc: torch.Tensor, K: int, ids: torch.Tensor) -> torch.Tensor:
    """Rows `ids` of a packed MXFP4 matrix as bf16 (the embedding gather)."""
    data = wp[ids]
    T, half = data.shape
    kp = half * 2
    codes = torch.empty((T, kp), dtype=torch.uint8, device=wp.device)
    codes[:, 0::2] = data & 0xF
    codes[:, 1::2] = (data >> 4) & 0xF
    codes = codes.view(T, kp // 32, 32)
    sign = torch.where((codes & 0x8) != 0, -1.0, 1.0)
    vals = _e2m1_table(wp.device)[(codes & 0x7).long()]
    scales = torch.exp2(wsc[ids].float() - 127.0)
    return ((sign * vals) * scales[..., None]).reshape(T, kp)[:, :K].to(torch.bfloat16)


# ---- weights ------------------------------------------------------------------
@dataclass
class LayerWeights:
    q: tuple
    k: tuple
    v: tuple
    o: tuple
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    moe: MoELayerWeights


@dataclass
class SyntheticQwen:
    cfg: QwenConfig
    embed: tuple
    lm_head: tuple
    final_norm: torch.Tensor
    layers: list = field(default_factory=list)

    @staticmethod
    def build(cfg: QwenConfig, seed: int = 0, device="cuda", std: float = 0.02) -> "SyntheticQwen":
        g = torch.Generator(device=device).manual_seed(seed)

        def packed(n, k):
            w = (torch.randn((n, k), generator=g, device=device) * std).bfloat16()
            return quantize_rows(w)

        def norm(n):
            return (1.0 + std * torch.randn(n, generator=g, device=device)).bfloat16()

        H, D = cfg.hidden, cfg.head_dim
        m = SyntheticQwen(cfg, packed(cfg.vocab, H), packed(cfg.vocab, H), norm(H))
        for L in range(cfg.layers):
            m.layers.append(LayerWeights(
                packed(cfg.heads * D, H), packed(cfg.kv_heads * D, H), packed(cfg.kv_heads * D, H),
                packed(H, cfg.heads * D), norm(D), norm(D), norm(H), norm(H),
                random_layer_weights(cfg.experts, H, cfg.inter, std, seed=seed * 1000 + L + 1,
                                     device=device)))
        return m


# ---- the library backend ---------------------------------------------------------
class LibBackend:
    """The library: drop-in operators for the dense projections and the
    attention, the fused device-routed layer for the MoE block."""

    name = "library"

    def __init__(self, model: SyntheticQwen):
        from . import fp4_ext
        self.dext = fp4_ext.get_decode_ext()
        self.model = model
        cfg = model.cfg
        self.moe = [MoELayer(lw.moe, top_k=cfg.top_k) for lw in model.layers]

    def prequant(self, x):
        return self.dext.prequant(x)

    def linear(self, xq, xsc, w, M, N, K):
        return self.dext.lin_pq(xq, xsc, w[0], w[1], M, N, K)

    def moe_block(self, L, h):
        out, topi, _ = self.moe[L](h.contiguous())
        return out, topi

    def attention(self, q, kvk, kvv, base, M):
        """q (B, M, Hq, D) bf16 of B sequences at the same base position,
        kvk/kvv (B, max_pos, Hkv, D) -> (B, M, Hq, D) fp32: one
        mfi_attn_decode_batched launch (the reference's attn_decode per
        sequence).  `base` is an int or a device int32 tensor of one element
        (read by the kernel, as in a captured decode step)."""
        from . import _lib
        lib = _lib.load()
        B, _, Hq, D = q.shape
        max_pos, Hkv = kvk.shape[1], kvk.shape[2]
        q = q.contiguous()
        if torch.is_tensor(base):
            dpos = base
        else:
            dpos = torch.full((1,), base, dtype=torch.int32, device=q.device)
        o = torch.empty((B, M, Hq, D), dtype=torch.float32, device=q.device)
        nws = int(lib.mfi_attn_decode_batched_workspace_bytes(B, M, Hq, Hkv, D, max_pos))
        ws = torch.empty(nws, dtype=torch.uint8, device=q.device)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _lib.check(lib.mfi_attn_decode_batched(
            q.data_ptr(), kvk.data_ptr(), kvv.data_ptr(), kvk.stride(0), dpos.data_ptr(),
            o.data_ptr(), B, M, Hq, Hkv, D, max_pos, None, None, ws.data_ptr(), nws, stream),
            "attn_decode_batched")
        return o


class Runner:
    """B sequences of the synthetic model with per-sequence FP8 KV caches."""

    def __init__(self, model: SyntheticQwen, backend, batch: int, max_len: int):
        cfg = model.cfg
        self.model, self.be, self.B, self.max_len = model, backend, batch, max_len
        dev = model.final_norm.device
        shape = (cfg.layers, batch, max_len, cfg.kv_heads, cfg.head_dim)
        self.kvk = torch.zeros(shape, dtype=torch.uint8, device=dev)
        self.kvv = torch.zeros(shape, dtype=torch.uint8, device=dev)

    def forward(self, ids: torch.Tensor, base: int, last_only: bool = False, trace=None):
        """ids (B, M) at positions base .. base + M - 1 of every sequence;
        returns fp32 logits (B, M, V) (or (B, V) of the last row) and the
        top-k expert ids of every layer.  ``trace`` (a list) receives the
        residual stream after every layer's attention and MoE block."""
        cfg, be, m = self.model.cfg, self.be, self.model
        B, M = ids.shape
        T = B * M
        H, Hq, Hkv, D = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim
        x = dequant_rows(m.embed[0], m.embed[1], H, ids.reshape(-1))
        # `base` may be a device int32 tensor of one element (a captured
        # decode step): positions and the KV rows then come from the device
        on_device = torch.is_tensor(base)
        if on_device:
            kv_idx = base.long() + torch.arange(M, device=ids.device)
            positions = kv_idx.repeat(B)
        else:
            positions = torch.arange(base, base + M, device=ids.device).repeat(B)
        routing = []
        for L, lw in enumerate(m.layers):
            hp = rms_norm(x, lw.in_norm, cfg.eps)
            hq, hs = be.prequant(hp.contiguous())
            q = be.linear(hq, hs, lw.q, T, Hq * D, H)
            k = be.linear(hq, hs, lw.k, T, Hkv * D, H)
            v = be.linear(hq, hs, lw.v, T, Hkv * D, H)
            q = rms_norm(q.view(T, Hq, D), lw.q_norm, cfg.eps).bfloat16()
            k = rms_norm(k.view(T, Hkv, D), lw.k_norm, cfg.eps).bfloat16()
            v = v.view(T, Hkv, D).bfloat16()
            q = apply_rope(q, positions, cfg.rope_theta)
            k = apply_rope(k, positions, cfg.rope_theta)
            kb = k.view(B, M, Hkv, D)
            vb = v.view(B, M, Hkv, D)
            k8 = kb.to(torch.float8_e4m3fn).view(torch.uint8)
            v8 = vb.to(torch.float8_e4m3fn).view(torch.uint8)
            if on_device:
                self.kvk[L].index_copy_(1, kv_idx, k8)
                self.kvv[L].index_copy_(1, kv_idx, v8)
            else:
                self.kvk[L, :, base:base + M] = k8
                self.kvv[L, :, base:base + M] = v8
            o = be.attention(q.view(B, M, Hq, D), self.kvk[L], self.kvv[L], base, M)
            of = o.reshape(T, Hq * D).to(torch.bfloat16).contiguous()
            aq, asc = be.prequant(of)
            x = x + be.linear(aq, asc, lw.o, T, H, Hq * D).bfloat16()
            if trace is not None:
                trace.append(("attn", L, x.clone()))
            h2 = rms_norm(x, lw.post_norm, cfg.eps)
            moe, topi = be.moe_block(L, h2)
            x = x + moe.bfloat16()
            routing.append(topi)
            if trace is not None:
                trace.append(("moe", L, x.clone()))
        if last_only:
            x = x.view(B, M, H)[:, -1]
        xn = rms_norm(x, m.final_norm, cfg.eps)
        lq, ls = be.prequant(xn.contiguous())
        logits = be.linear(lq, ls, m.lm_head, xn.shape[0], cfg.vocab, H)
        return (logits if last_only else logits.view(B, M, cfg.vocab)), routing

    # ---- generation ------------------------------------------------------
    def prefill(self, prompt: torch.Tensor, chunk: int = 64) -> None:
        """Write the KV of prompt[:, :-1] (its last token is fed by the first
        decode step, as runtime/spec_decoder.py:94-104 re-feeds it)."""
        P = prompt.shape[1] - 1
        for s in range(0, P, chunk):
            self.forward(prompt[:, s:min(s + chunk, P)], s, last_only=True)

    def greedy(self, prompt: torch.Tensor, steps: int, chunk: int = 64):
        """Plain greedy decoding: returns token ids (B, steps) and each step's
        top-2 logit margin (B, steps)."""
        self.prefill(prompt, chunk)
        pos = prompt.shape[1] - 1
        last = prompt[:, -1:]
        toks, margins = [], []
        for _ in range(steps):
            logits, _ = self.forward(last, pos, last_only=True)
            top2 = torch.topk(logits, 2, dim=-1).values
            nxt = logits.argmax(-1)
            toks.append(nxt)
            margins.append(top2[:, 0] - top2[:, 1])
            last = nxt[:, None]
            pos += 1
        return torch.stack(toks, 1), torch.stack(margins, 1)

    def score(self, prompt: torch.Tensor, tokens: torch.Tensor, chunk: int = 64):
        """Teacher-forced next-token predictions along a given continuation:
        the prompt, then tokens (B, S) fed as history, in chunks of rows;
        returns this backend's argmax (B, S) and top-2 margins (B, S) for each
        position of `tokens` (prediction i sees the prompt and tokens[:, :i])."""
        self.prefill(prompt, chunk)
        P = prompt.shape[1] - 1
        feed = torch.cat([prompt[:, -1:], tokens[:, :-1]], dim=1)
        am, mg = [], []
        for s in range(0, feed.shape[1], chunk):
            logits, _ = self.forward(feed[:, s:s + chunk], P + s)
            top2 = torch.topk(logits, 2, dim=-1).values
            am.append(logits.argmax(-1))
            mg.append(top2[..., 0] - top2[..., 1])
            del logits
        return torch.cat(am, 1), torch.cat(mg, 1)

    def speculative(self, prompt: torch.Tensor, steps: int, n_gram: int = 7, draft_len: int = 4):
        """Prompt-lookup speculative decoding of one sequence (B = 1), the
        reference's PromptLookup (runtime/spec_decoder.py:22-122): drafts are
        the draft_len tokens that followed the last earlier occurrence of the
        current n-gram, verified in one forward of 1 + draft_len rows; the
        longest agreeing prefix plus the model's own next token are kept.
        Returns (token ids, verify forwards, drafted tokens accepted);
        ``self.spec_stats`` also counts the drafted tokens proposed."""
        assert self.B == 1
        self.prefill(prompt)
        hist = [int(t) for t in prompt[0]]
        P = len(hist)
        pos = P
        dev = prompt.device
        first = {}
        for i in range(len(hist) - n_gram + 1):
            first.setdefault(tuple(hist[i:i + n_gram]), i)
        forwards = accepted = drafted = 0
        while len(hist) - P < steps:
            tail = tuple(hist[-n_gram:])
            j = first.get(tail)
            drafts = hist[j + n_gram:j + n_gram + draft_len] if (j is not None and
                                                                  j + n_gram < len(hist)) else []
            ids = torch.tensor([[hist[-1]] + drafts], dtype=torch.long, device=dev)
            logits, _ = self.forward(ids, pos - 1)
            am = logits[0].argmax(-1).tolist()
            forwards += 1
            drafted += len(drafts)
            a = 0
            while a < len(drafts) and am[a] == drafts[a]:
                a += 1
            accepted += a
            new = drafts[:a] + [am[a]]
            for t in new:
                hist.append(int(t))
                if len(hist) >= n_gram:
                    first.setdefault(tuple(hist[-n_gram:]), len(hist) - n_gram)
            pos += len(new)
        self.spec_stats = {"forwards": forwards, "drafted": drafted, "accepted": accepted}
        return torch.tensor(hist[P:P + steps]), forwards, accepted


class GraphDecoder:
    """Greedy decoding of a Runner on the library backend with every decode
    step replayed from one captured CUDA graph.

    The reference's own graph attempt for its runner failed on the per-layer
    `.tolist()` of the routing (runtime/model_runner_v2.py:194); with the
    device-routed MoE layer nothing on the step needs the host, so the whole
    step — 48 layers of projections, FP8 KV write, attention, MoE block, the
    lm_head and the argmax — is one graph.  The position lives in a device
    tensor that the graph advances; each replay feeds the previous step's
    token and records the new one.  Same kernels in the same order as
    Runner.greedy, so the tokens are identical (tests/test_gpu_model.py)."""

    def __init__(self, runner: "Runner", max_steps: int):
        dev = runner.model.final_norm.device
        B = runner.B
        self.runner, self.max_steps = runner, max_steps
        self.ids = torch.zeros((B, 1), dtype=torch.long, device=dev)
        self.base = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.step = torch.zeros((1,), dtype=torch.long, device=dev)
        self.tokens = torch.zeros((B, max_steps), dtype=torch.long, device=dev)
        self.graph = None

    def _body(self):
        logits, _ = self.runner.forward(self.ids, self.base, last_only=True)
        nxt = logits.argmax(-1)
        self.tokens.index_copy_(1, self.step, nxt[:, None])
        self.ids.copy_(nxt[:, None])
        self.base.add_(1)
        self.step.add_(1)

    def _set(self, last_ids: torch.Tensor, base: int):
        self.ids.copy_(last_ids)
        self.base.fill_(base)
        self.step.zero_()

    def start(self, prompt: torch.Tensor, chunk: int = 64, prefill: bool = True) -> None:
        """Prefill the prompt (eager; skipped with prefill=False when the
        runner's caches already hold it) and make the graph of one decode step
        (captured once, after an eager warm-up step whose KV row and token
        the replays then write again)."""
        r = self.runner
        if prefill:
            r.prefill(prompt, chunk)
        pos = prompt.shape[1] - 1
        dev = self.ids.device
        if self.graph is None:
            self._set(prompt[:, -1:], pos)
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                self._body()  # allocates the layers' workspaces, initialises state
                torch.cuda.synchronize(dev)
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph, stream=side):
                    self._body()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
        self._set(prompt[:, -1:], pos)

    def decode(self, steps: int) -> torch.Tensor:
        """`steps` greedy tokens (B, steps) after start()."""
        if steps > self.max_steps:
            raise RuntimeError(f"at most {self.max_steps} steps")
        for _ in range(steps):
            self.graph.replay()
        return self.tokens[:, :steps]


def synthetic_prompts(batch: int, length: int, vocab: int, seed: int = 0, motif: int = 32,
                      device="cuda") -> torch.Tensor:
    """Uniform random token ids with a repeated 32-token motif (BASELINE
    config 4): the motif recurs every 256 tokens, so the prompt-lookup
    drafts have n-grams to reuse."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, length), generator=g)
    mot = torch.randint(0, vocab, (batch, motif), generator=g)
    for s in range(0, length - motif + 1, 256):
        ids[:, s:s + motif] = mot
    ids[:, length - motif:] = mot  # the prompt ends inside the motif
    return ids.to(device)
