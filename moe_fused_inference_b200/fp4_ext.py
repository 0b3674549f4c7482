"""Drop-in replacement for the reference's ``runtime/fp4_ext.py``.

The reference JIT-builds two torch extensions for sm_120a
(runtime/fp4_ext.py:21-62):

* ``get_ext()`` -> module ``mxfp4_linear_ext`` with ``forward(x, wp, wsc)``
  (src/ext/mxfp4_binding.cpp:21-50);
* ``get_decode_ext()`` -> module ``mxfp4_decode_ext`` with ``prequant``,
  ``lin_pq``, ``moe_gateup``, ``moe_down``, ``moe_combine``,
  ``moe_gateup_tab``, ``moe_down_tab``, ``attn_decode`` and ``kv_write``
  (src/ext/mxfp4_decode_binding.cpp:232-243).

This module returns objects with the same function names, argument meaning,
output shapes/dtypes and error type (``RuntimeError`` with the binding's
TORCH_CHECK wording), backed by the sm_100a kernels of libmoe_fp4.so through
its C ABI (include/moe_fp4.h).  ``model_runner_v2.py`` and ``spec_decoder.py``
use it by replacing their ``runtime/fp4_ext.py`` with a two-line shim
(INTEGRATION.md).

Differences on purpose:
* pointer tables are uploaded with an asynchronous copy from pinned memory
  instead of the reference's blocking pageable copy
  (src/ext/mxfp4_decode_binding.cpp:44-60);
* weights shared by several (token, slot) entries are streamed once;
* the stale call arities used by the reference's own tests and v3 runner
  (``moe_down`` with 6 arguments, ``moe_combine`` with 2, ``attn_decode`` and
  ``kv_write`` with 5) are accepted and mean M = 1;
* ``attn_decode`` does not write the score buffer ``sc`` (the reference
  leaves raw scores there; no caller reads them) and splits the positions
  over the grid; ``attn_decode`` / ``kv_write`` take optional per-KV-head
  FP8 scales (the reference's cache has none).
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["get_ext", "get_decode_ext"]


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _ceil32(k: int) -> int:
    return (k + 31) // 32 * 32


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _require_f32(t: torch.Tensor, name: str) -> None:
    _check(t.dtype == torch.float32,
           f"expected scalar type Float but found {str(t.dtype).replace('torch.', '')} ({name})")


class _PinnedRing:
    """Reusable pinned staging buffers for pointer-table uploads: allocating
    pinned memory per call (cudaHostAlloc) costs far more than the copy.  A
    slot is reused only after the copy that last read it has completed (an
    event recorded behind the copy), so the host never overwrites a table the
    GPU has not yet read."""

    SLOTS = 16
    ENTRIES = 8192

    def __init__(self):
        self.buf = torch.empty((self.SLOTS, self.ENTRIES), dtype=torch.int64).pin_memory()
        self.np = self.buf.numpy()
        self.events = [None] * self.SLOTS
        self.next = 0

    def upload(self, ptrs, dev: torch.device) -> torch.Tensor:
        n = len(ptrs)
        if n > self.ENTRIES:
            return torch.tensor(ptrs, dtype=torch.int64).to(dev)
        i = self.next
        self.next = (i + 1) % self.SLOTS
        if self.events[i] is not None:
            self.events[i].synchronize()
        self.np[i, :n] = ptrs
        out = torch.empty(n, dtype=torch.int64, device=dev)
        out.copy_(self.buf[i, :n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(dev))
        self.events[i] = ev
        return out


_RING: dict = {}


def _ptr_table(ts, dev: torch.device) -> torch.Tensor:
    """Device int64 table of data pointers (reference make_ptr_table,
    src/ext/mxfp4_decode_binding.cpp:44-60), uploaded asynchronously from a
    reusable pinned buffer."""
    _check(len(ts) > 0, "empty pointer table")
    ptrs = []
    for t in ts:
        _check(t.is_cuda and t.dtype == torch.uint8, "ptr table entries must be cuda uint8")
        ptrs.append(t.data_ptr())
    ring = _RING.get(dev.index)
    if ring is None:
        ring = _RING[dev.index] = _PinnedRing()
    return ring.upload(ptrs, dev)


def _workspace(nbytes: int, dev: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)


_DTYPE = {torch.float32: _lib.MFI_F32, torch.float16: _lib.MFI_F16, torch.bfloat16: _lib.MFI_BF16}


class _LinearExt:
    """Stand-in for the ``mxfp4_linear_ext`` module."""

    __name__ = "mxfp4_linear_ext"

    @staticmethod
    def forward(x: torch.Tensor, wp: torch.Tensor, wsc: torch.Tensor) -> torch.Tensor:
        """y (M, N) fp32 = Q(half(x)) . W^T — reference src/ext/mxfp4_binding.cpp:21-45.

        x: (M, K) half/bf16/fp32 cuda (non-half inputs are rounded through fp16,
        as the reference binding casts them); wp (N, Kp/2) and wsc (N, Kp/32)
        uint8 cuda.  Columns of x beyond Kp are ignored and missing ones are
        zero, as in the reference kernel."""
        lib = _lib.load()
        _check(x.is_cuda, "x must be cuda")
        _check(wp.is_cuda and wsc.is_cuda, "weights must be cuda")
        _check(wp.dtype == torch.uint8 and wsc.dtype == torch.uint8, "weight tensors must be uint8")
        _check(x.dim() == 2 and wp.dim() == 2 and wsc.dim() == 2, "x, wp, wsc must be 2-D")
        if x.dtype not in _DTYPE:
            x = x.to(torch.float16)
        x = x.contiguous()
        wp = wp.contiguous()
        wsc = wsc.contiguous()
        M, K = x.shape
        N, Kp = wp.shape[0], wp.shape[1] * 2
        _check(wsc.shape[0] == N and wsc.shape[1] * 32 == Kp, "wsc must be (N, Kp/32)")
        y = torch.empty((M, N), dtype=torch.float32, device=x.device)
        if M == 0 or N == 0:
            return y
        ws = _workspace(lib.mfi_linear_workspace_bytes(M, N, Kp), x.device)
        st = lib.mfi_mxfp4_linear(_ptr(x), _DTYPE[x.dtype], K, _ptr(wp), _ptr(wsc), _ptr(y),
                                  M, N, Kp, _ptr(ws), ws.numel(), _stream(x.device))
        _lib.check(st, "forward")
        return y


class _DecodeExt:
    """Stand-in for the ``mxfp4_decode_ext`` module."""

    __name__ = "mxfp4_decode_ext"

    @staticmethod
    def prequant(x: torch.Tensor):
        """bf16 (M, K) -> [xq (M, Kp/2) u8, xsc (M, Kp/32) u8], Kp = ceil32(K)
        (reference src/ext/mxfp4_decode_binding.cpp:65-81)."""
        lib = _lib.load()
        _check(x.is_cuda, "x must be cuda")
        _check(x.dtype == torch.bfloat16, "x must be bfloat16")
        x = x.contiguous()
        M, K = x.shape
        Kp = _ceil32(K)
        xq = torch.empty((M, Kp // 2), dtype=torch.uint8, device=x.device)
        xsc = torch.empty((M, Kp // 32), dtype=torch.uint8, device=x.device)
        if M and K:
            _lib.check(lib.mfi_prequant(_ptr(x), _ptr(xq), _ptr(xsc), M, K, Kp, _stream(x.device)),
                       "prequant")
        else:
            xq.zero_()
            xsc.fill_(127)
        return [xq, xsc]

    @staticmethod
    def lin_pq(xq, xsc, wp, wsc, M, N, K):
        """y (M, N) fp32 = Q(x) . W^T from pre-quantised x; Kp = wp.size(1)*2
        (reference src/ext/mxfp4_decode_binding.cpp:84-98)."""
        lib = _lib.load()
        xq, xsc, wp, wsc = xq.contiguous(), xsc.contiguous(), wp.contiguous(), wsc.contiguous()
        M, N, K = int(M), int(N), int(K)
        Kp = wp.shape[1] * 2
        _check(xq.shape[1] * 2 == Kp, "xq must be (M, Kp/2) with the weight's Kp")
        _check(xq.shape[0] >= M, "xq has fewer than M rows")
        y = torch.empty((M, N), dtype=torch.float32, device=xq.device)
        if M and N:
            ws = _workspace(lib.mfi_lin_pq_workspace_bytes(M, N, Kp), xq.device)
            _lib.check(lib.mfi_lin_pq(_ptr(xq), _ptr(xsc), _ptr(wp), _ptr(wsc), _ptr(y), M, N, K, Kp,
                                      _ptr(ws), ws.numel(), _stream(xq.device)), "lin_pq")
        return y

    @staticmethod
    def _gateup(xq, xsc, wp_tab, wsc_tab, E, M, N, K, Kp):
        lib = _lib.load()
        gu = torch.empty((M * E, 2 * N), dtype=torch.float32, device=xq.device)
        ws = _workspace(lib.mfi_moe_gateup_workspace_bytes(E, M), xq.device)
        st = lib.mfi_moe_gateup(_ptr(xq), _ptr(xsc), _ptr(wp_tab), _ptr(wsc_tab), _ptr(gu),
                                E, M, N, K, Kp, _ptr(ws), ws.numel(), _stream(xq.device))
        _lib.check(st, "moe_gateup")
        return gu

    @staticmethod
    def moe_gateup(xq, xsc, wps, wscs, E, M, N, K):
        """gu (M*E, 2N) fp32; wps/wscs: 2*E*M tensors ordered per token
        [gate e0..e(E-1), up e0..e(E-1)] (reference
        src/ext/mxfp4_decode_binding.cpp:101-120)."""
        E, M, N, K = int(E), int(M), int(N), int(K)
        _check(len(wps) == 2 * E * M, "wps must be 2E*M")
        _check(len(wscs) == 2 * E * M, "wscs must be 2E*M")
        Kp = wps[0].shape[1] * 2
        xq, xsc = xq.contiguous(), xsc.contiguous()
        wp_tab = _ptr_table(wps, xq.device)
        wsc_tab = _ptr_table(wscs, xq.device)
        return _DecodeExt._gateup(xq, xsc, wp_tab, wsc_tab, E, M, N, K, Kp)

    @staticmethod
    def moe_gateup_tab(xq, xsc, wps_tab, wscs_tab, E, M, N, K):
        """As moe_gateup with caller-owned device int64 pointer tables; Kp =
        xq.size(1)*2 (reference src/ext/mxfp4_decode_binding.cpp:177-192)."""
        E, M, N, K = int(E), int(M), int(N), int(K)
        _check(wps_tab.dtype == torch.int64 and wscs_tab.dtype == torch.int64,
               "pointer tables must be int64")
        _check(wps_tab.numel() >= 2 * E * M and wscs_tab.numel() >= 2 * E * M,
               "pointer tables must hold 2E*M entries")
        return _DecodeExt._gateup(xq.contiguous(), xsc.contiguous(), wps_tab, wscs_tab,
                                  E, M, N, K, xq.shape[1] * 2)

    @staticmethod
    def _down(gu, wp_tab, wsc_tab, E, M, N, K, Kp):
        lib = _lib.load()
        _require_f32(gu, "gu")
        gu = gu.contiguous()
        yd = torch.empty((M * E, N), dtype=gu.dtype, device=gu.device)
        ws = _workspace(lib.mfi_moe_down_workspace_bytes(E, M, K), gu.device)
        st = lib.mfi_moe_down(_ptr(gu), _ptr(wp_tab), _ptr(wsc_tab), _ptr(yd), E, M, N, K, Kp,
                              _ptr(ws), ws.numel(), _stream(gu.device))
        _lib.check(st, "moe_down")
        return yd

    @staticmethod
    def moe_down(gu, wps, wscs, E, *args):
        """yd (M*E, N) fp32 = Q(silu(g)*u) . Wd^T (reference
        src/ext/mxfp4_decode_binding.cpp:123-142).  Signature
        ``(gu, wps, wscs, E, M, N, K)``; the stale 6-argument form
        ``(gu, wps, wscs, E, N, K)`` means M = 1."""
        if len(args) == 3:
            M, N, K = (int(a) for a in args)
        elif len(args) == 2:
            M, (N, K) = 1, (int(a) for a in args)
        else:
            raise TypeError("moe_down(gu, wps, wscs, E, M, N, K)")
        E = int(E)
        _check(len(wps) == E * M, "wps must be E*M")
        Kp = wps[0].shape[1] * 2
        _check(gu.shape[0] == M * E and gu.shape[1] == 2 * K, "gu (M*E,2K)")
        _check(Kp == _ceil32(K), "down weights must have Kp = ceil32(K)")
        wp_tab = _ptr_table(wps, gu.device)
        wsc_tab = _ptr_table(wscs, gu.device)
        return _DecodeExt._down(gu, wp_tab, wsc_tab, E, M, N, K, Kp)

    @staticmethod
    def moe_down_tab(gu, wps_tab, wscs_tab, E, M, N, K):
        """As moe_down with caller-owned device pointer tables; Kp =
        ceil32(gu.size(1)/2) (reference src/ext/mxfp4_decode_binding.cpp:194-209)."""
        E, M, N, K = int(E), int(M), int(N), int(K)
        _check(wps_tab.dtype == torch.int64 and wscs_tab.dtype == torch.int64,
               "pointer tables must be int64")
        _check(wps_tab.numel() >= E * M and wscs_tab.numel() >= E * M,
               "pointer tables must hold E*M entries")
        Kp = _ceil32(gu.shape[1] // 2)
        return _DecodeExt._down(gu, wps_tab, wscs_tab, E, M, N, K, Kp)

    @staticmethod
    def moe_combine(yd, w, M=1):
        """out (M, N) fp32, out[m,c] = sum_{e<min(E,8)} w[m,e]*yd[m*E+e,c]
        (reference src/ext/mxfp4_decode_binding.cpp:145-158; the 2-argument
        form means M = 1)."""
        lib = _lib.load()
        yd, w = yd.contiguous(), w.contiguous()
        M = int(M)
        _check(M > 0, "M must be positive")
        E = w.numel() // M
        N = yd.shape[1]
        _check(M * E == w.numel(), "w (M,E)")
        _check(yd.shape[0] == M * E, "yd (M*E,N)")
        _require_f32(yd, "yd")
        _require_f32(w, "w")
        out = torch.empty((M, N), dtype=yd.dtype, device=yd.device)
        if N:
            _lib.check(lib.mfi_moe_combine(_ptr(yd), N, _ptr(w), E, _ptr(out), M, N,
                                           _stream(yd.device)), "moe_combine")
        return out

    @staticmethod
    def attn_decode(q, kvk, kvv, dpos, sc, M=1, k_scale=None, v_scale=None):
        """o fp32 (M, Hq, D): decode attention of M query rows of one sequence
        over the layer's FP8 cache kvk/kvv (max_pos, Hkv, D) up to position
        dpos[0] + m (reference src/ext/mxfp4_decode_binding.cpp:213-230).
        ``sc`` (the reference's score buffer) is accepted and left untouched;
        the stale 5-argument call and a 2-D q (Hq, D) mean M = 1.  Optional
        per-KV-head ``k_scale``/``v_scale`` (fp32 (Hkv,)) select the standard
        e4m3fn cache format with scales (this library's addition)."""
        lib = _lib.load()
        M = int(M)
        _check(q.is_cuda and kvk.is_cuda and kvv.is_cuda and dpos.is_cuda, "tensors must be cuda")
        _check(q.dtype == torch.bfloat16, "q must be bfloat16")
        if q.dim() == 2:
            q = q.unsqueeze(0)
        q = q.contiguous()
        kvk = kvk.view(torch.uint8) if kvk.dtype != torch.uint8 else kvk
        kvv = kvv.view(torch.uint8) if kvv.dtype != torch.uint8 else kvv
        _check(kvk.dim() == 3 and kvv.shape == kvk.shape and kvk.is_contiguous()
               and kvv.is_contiguous(), "kvk/kvv must be contiguous (max_pos, Hkv, D)")
        _check(dpos.dtype == torch.int32, "dpos must be int32")
        Hq, D = int(q.shape[1]), int(q.shape[2])
        max_pos, Hkv = int(kvk.shape[0]), int(kvk.shape[1])
        _check(q.shape[0] >= M, "q has fewer than M rows")
        o = torch.empty((M, Hq, D), dtype=torch.float32, device=q.device)
        ks = vs = 0
        if k_scale is not None or v_scale is not None:
            _check(k_scale is not None and v_scale is not None, "give both scales or neither")
            k_scale = k_scale.to(q.device, torch.float32).contiguous()
            v_scale = v_scale.to(q.device, torch.float32).contiguous()
            _check(k_scale.numel() == Hkv and v_scale.numel() == Hkv, "one scale per KV head")
            ks, vs = k_scale.data_ptr(), v_scale.data_ptr()
        ws = _workspace(lib.mfi_attn_decode_workspace_bytes(M, Hq, Hkv, D, max_pos), q.device)
        _lib.check(lib.mfi_attn_decode(_ptr(q), _ptr(kvk), _ptr(kvv), _ptr(dpos), _ptr(o), M, Hq,
                                       Hkv, D, max_pos, ks, vs, _ptr(ws), ws.numel(),
                                       _stream(q.device)), "attn_decode")
        return o

    @staticmethod
    def kv_write(k, v, kvk, kvv, dpos, M=1, k_scale=None, v_scale=None):
        """Write M rows of k, v (bf16 (M, Hkv, D)) into the FP8 cache slices
        kvk/kvv (max_pos, Hkv, D) at positions dpos[0] + m (reference
        src/ext/mxfp4_decode_binding.cpp:161-173; the stale 5-argument call
        means M = 1).  Without scales the bytes are the reference encoder's,
        bit for bit; with per-KV-head scales, standard e4m3fn of x / scale."""
        lib = _lib.load()
        M = int(M)
        kvk = kvk.view(torch.uint8) if kvk.dtype != torch.uint8 else kvk
        kvv = kvv.view(torch.uint8) if kvv.dtype != torch.uint8 else kvv
        _check(k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16, "k and v must be bfloat16")
        _check(dpos.dtype == torch.int32, "dpos must be int32")
        _check(kvk.dim() == 3 and kvv.shape == kvk.shape and kvk.is_contiguous()
               and kvv.is_contiguous(), "kvk/kvv must be contiguous (max_pos, Hkv, D)")
        k, v = k.contiguous(), v.contiguous()
        max_pos, Hkv, D = (int(s) for s in kvk.shape)
        _check(k.numel() >= M * Hkv * D and v.numel() >= M * Hkv * D, "k/v smaller than (M, Hkv, D)")
        ks = vs = 0
        if k_scale is not None or v_scale is not None:
            _check(k_scale is not None and v_scale is not None, "give both scales or neither")
            k_scale = k_scale.to(k.device, torch.float32).contiguous()
            v_scale = v_scale.to(k.device, torch.float32).contiguous()
            _check(k_scale.numel() == Hkv and v_scale.numel() == Hkv, "one scale per KV head")
            ks, vs = k_scale.data_ptr(), v_scale.data_ptr()
        _lib.check(lib.mfi_kv_write(_ptr(k), _ptr(v), _ptr(kvk), _ptr(kvv), _ptr(dpos), M, Hkv, D,
                                    max_pos, ks, vs, _stream(k.device)), "kv_write")


_EXT = _LinearExt()
_DEXT = _DecodeExt()


def get_ext():
    """Reference runtime/fp4_ext.py:21-39 — returns the linear module."""
    _lib.load()
    return _EXT


def get_decode_ext():
    """Reference runtime/fp4_ext.py:46-62 — returns the decode module."""
    _lib.load()
    return _DEXT
