"""Expert-parallel MoE layer: 128/N experts per rank, token dispatch and
combine as NCCL all-to-all over NVLink.

The reference runs the MoE block on one GPU (runtime/model_runner_v2.py:183-208,
:266-290) and has no collective anywhere; this module is the multi-GPU form of
the same block.  Two transports move the same rows:

``transport="p2p"`` (default on GPUs): the exchange is fused into the kernels.
The router stores each token's row straight into the receive buffer of every
rank that owns one of its experts (NVLink stores through CUDA IPC mappings,
mfi_ep_route_dispatch); the expert side waits on per-source flags, runs the
local experts and stores each row's weighted slot sum straight back into the
source's return buffer (mfi_ep_experts_return); the source waits for every
rank's return and sums in rank order (mfi_ep_unpack_wait).  Only the rows that
exist cross NVLink, no collective library runs on the data path and flags
carry call ids, so a whole decode step can be captured in one CUDA graph.

``transport="nccl"``: the same rows in fixed-capacity blocks exchanged with
two ``all_to_all_single`` calls.  Per layer and rank, with no host
synchronisation:

  route     mfi_moe_route: quantise the rank's tokens, router GEMM, top-k
            (full router on every rank, so the routing is the single-GPU one)
  pack      mfi_ep_pack: one MXFP4 row per (token, destination rank) pair
            with the token's local expert ids and weights; fixed capacity
            (C = max tokens per rank) so the split sizes are known up front
  dispatch  all_to_all_single of the equal-size blocks
  experts   mfi_ep_mask_recv + mfi_moe_experts on every received row: the
            same tcgen05 expert GEMMs as the single-GPU layer, followed by the
            weighted sum of the row's local slots
  return    all_to_all_single of the fp32 partial sums
  unpack    mfi_ep_unpack: out[t] = sum over ranks, in rank order

Expert outputs are bit-identical to the single-GPU layer; only the fp32
summation order of the combine differs (local slots first, then ranks), so
layer outputs agree to fp32 rounding, not bit for bit.

The per-step operations go through an ``ops`` object so the exchange protocol
can be exercised without a GPU; the product path is ``CudaEPOps`` (the C-ABI
library) and has no fallback.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib
from .layer import MoELayerWeights, _stream


@dataclass
class EPShard:
    """One rank's part of a layer: its experts and the full router."""

    gate_wp: torch.Tensor   # (El, inter, hidden/2)
    gate_sc: torch.Tensor   # (El, inter, hidden/32)
    up_wp: torch.Tensor
    up_sc: torch.Tensor
    down_wp: torch.Tensor   # (El, hidden, inter/2)
    down_sc: torch.Tensor   # (El, hidden, inter/32)
    router_wp: torch.Tensor  # (E, hidden/2), E = El * world
    router_sc: torch.Tensor  # (E, hidden/32)

    @property
    def local_experts(self) -> int:
        return self.gate_wp.shape[0]

    @property
    def n_experts(self) -> int:
        return self.router_wp.shape[0]

    @property
    def hidden(self) -> int:
        return self.gate_wp.shape[2] * 2

    @property
    def inter(self) -> int:
        return self.gate_wp.shape[1]

    @staticmethod
    def from_layer(w: MoELayerWeights, rank: int, world: int) -> "EPShard":
        """Experts [rank*El, (rank+1)*El) of a full layer, El = E / world."""
        E = w.n_experts
        if E % world:
            raise RuntimeError(f"{E} experts do not split over {world} ranks")
        el = E // world
        s = slice(rank * el, (rank + 1) * el)
        return EPShard(w.gate_wp[s].contiguous(), w.gate_sc[s].contiguous(),
                       w.up_wp[s].contiguous(), w.up_sc[s].contiguous(),
                       w.down_wp[s].contiguous(), w.down_sc[s].contiguous(),
                       w.router_wp, w.router_sc)


def random_shard(n_experts: int, world: int, rank: int, hidden: int = 2048, inter: int = 768,
                 std: float = 0.02, seed: int = 0, device="cuda") -> EPShard:
    """Random-init shard of a layer: bf16 N(0, std) weights quantised on the
    GPU with the quantize_expert_tensor rules; the router (all experts) is
    drawn from ``seed`` so every rank holds the same one, the rank's experts
    from (seed, rank)."""
    from .layer import quantize_rows
    if n_experts % world:
        raise RuntimeError(f"{n_experts} experts do not split over {world} ranks")
    el = n_experts // world
    g = torch.Generator(device=device)

    def q(rows, k):
        w = torch.randn((rows, k), generator=g, device=device, dtype=torch.float32) * std
        return quantize_rows(w.to(torch.bfloat16))

    g.manual_seed(seed)
    rwp, rsc = q(n_experts, hidden)
    g.manual_seed(seed * 1009 + 17 + rank)
    gwp, gsc = q(el * inter, hidden)
    uwp, usc = q(el * inter, hidden)
    dwp, dsc = q(el * hidden, inter)
    H, Mi = hidden, inter
    return EPShard(gwp.view(el, Mi, H // 2), gsc.view(el, Mi, H // 32),
                   uwp.view(el, Mi, H // 2), usc.view(el, Mi, H // 32),
                   dwp.view(el, H, Mi // 2), dsc.view(el, H, Mi // 32), rwp, rsc)


# mfi_ep_experts_return: world * (capacity + 1) * top_k (row, slot) pairs at most
P2P_MAX_PAIRS = 16384


def ep_row_bytes(hidden: int, top_k: int) -> int:
    """Bytes of one exchanged row (mfi_ep_row_bytes)."""
    b = hidden // 2 + hidden // 32 + 16 + 8 * top_k
    return (b + 15) // 16 * 16


def row_offsets(hidden: int, top_k: int):
    """Byte offsets inside an exchanged row: (scales, token, sel, weights)."""
    sc = hidden // 2
    meta = sc + hidden // 32
    return sc, meta, meta + 16, meta + 16 + 4 * top_k


class CudaEPOps:
    """The per-step operations on the GPU, through libmoe_fp4.so."""

    def __init__(self, shard: EPShard, top_k: int, capacity: int, world: int,
                 logit_bias: torch.Tensor | None = None):
        lib = _lib.load()
        self.lib = lib
        self.shard = shard
        self.k = top_k
        self.C = capacity
        self.world = world
        H, Mi, El = shard.hidden, shard.inter, shard.local_experts
        self.H = H
        self.El = El
        if lib.mfi_ep_row_bytes(H, top_k) != ep_row_bytes(H, top_k):
            raise RuntimeError("row size mismatch between library and host")
        self.rb = ep_row_bytes(H, top_k)
        self._route_w = _lib.MoEWeights(0, 0, 0, 0, 0, 0, shard.router_wp.data_ptr(),
                                        shard.router_sc.data_ptr(), shard.n_experts, H, Mi,
                                        top_k, None)
        # optional per-expert logit bias (E fp32), added before the top-k
        self.logit_bias = None
        if logit_bias is not None:
            self.logit_bias = logit_bias.to(shard.router_wp.device, torch.float32).contiguous()
            if self.logit_bias.numel() != shard.n_experts:
                raise RuntimeError("logit_bias needs one value per expert")
            self._route_w.logit_bias = self.logit_bias.data_ptr()
        self._exp_w = _lib.MoEWeights(
            shard.gate_wp.data_ptr(), shard.gate_sc.data_ptr(), shard.up_wp.data_ptr(),
            shard.up_sc.data_ptr(), shard.down_wp.data_ptr(), shard.down_sc.data_ptr(),
            0, 0, El, H, Mi, top_k, None)
        dev = shard.gate_wp.device
        nprep = int(lib.mfi_moe_prepared_bytes(El, H, Mi))
        if nprep == 0:
            raise RuntimeError("expert parallelism needs hidden and inter multiples of 256")
        self.prepared = torch.empty(nprep, dtype=torch.uint8, device=dev)
        self._exp_w.prepared = self.prepared.data_ptr()
        _lib.check(lib.mfi_moe_prepare(ctypes.byref(self._exp_w), self.prepared.data_ptr(), nprep,
                                       _stream(dev)), "moe_prepare")
        self.route_ws = None
        self.R = world * (capacity + 1)
        nws = int(lib.mfi_moe_experts_workspace_bytes(self.R, H, Mi, El, top_k))
        # zero once: the peer-memory transport keeps its counters here between
        # calls (each call leaves them at zero)
        self.ws = torch.zeros(nws, dtype=torch.uint8, device=dev)

    def route(self, x, xq, xsc, topi, topw, logits=None):
        T = x.shape[0]
        nws = int(self.lib.mfi_moe_route_workspace_bytes(T, self.H, self.shard.n_experts))
        if nws and (self.route_ws is None or self.route_ws.numel() < nws):
            # the tensor-core router's scratch (prefill-sized batches)
            self.route_ws = torch.empty(nws, dtype=torch.uint8, device=x.device)
        ws = self.route_ws if nws else None
        _lib.check(self.lib.mfi_moe_route_ex(ctypes.byref(self._route_w), x.data_ptr(), T,
                                             xq.data_ptr(), xsc.data_ptr(), topi.data_ptr(),
                                             topw.data_ptr(),
                                             0 if logits is None else logits.data_ptr(),
                                             0 if ws is None else ws.data_ptr(),
                                             0 if ws is None else ws.numel(),
                                             _stream(x.device)), "moe_route")

    def pack(self, xq, xsc, topi, topw, T, counts, send, pack_pos):
        _lib.check(self.lib.mfi_ep_pack(xq.data_ptr(), xsc.data_ptr(), topi.data_ptr(),
                                        topw.data_ptr(), T, self.H, self.k, self.world, self.El,
                                        self.C, counts.data_ptr(), send.data_ptr(),
                                        pack_pos.data_ptr(), _stream(send.device)), "ep_pack")

    def experts(self, recv, ret):
        lib = self.lib
        st = _stream(recv.device)
        _lib.check(lib.mfi_ep_mask_recv(recv.data_ptr(), self.world, self.C, self.H, self.k, st),
                   "ep_mask_recv")
        sc, _, sel, w = row_offsets(self.H, self.k)
        base = recv.data_ptr()
        rb = self.rb
        _lib.check(lib.mfi_moe_experts(ctypes.byref(self._exp_w), base, rb, base + sc, rb,
                                       base + sel, rb // 4, base + w, rb // 4, self.R,
                                       ret.data_ptr(), self.H, self.ws.data_ptr(), self.ws.numel(),
                                       st), "moe_experts")

    def unpack(self, ret_back, pack_pos, T, out):
        _lib.check(self.lib.mfi_ep_unpack(ret_back.data_ptr(), pack_pos.data_ptr(), T, self.world,
                                          self.C, self.H, out.data_ptr(), _stream(out.device)),
                   "ep_unpack")

    # ---- peer-memory transport ----
    def p2p_dispatch(self, x, topi, topw, pack_pos, xch, C):
        rank = xch.rank
        _lib.check(self.lib.mfi_ep_route_dispatch(
            ctypes.byref(self._route_w), x.data_ptr(), x.shape[0], rank, self.world, C,
            xch.table.data_ptr(), xch.flags, topi.data_ptr(), topw.data_ptr(),
            pack_pos.data_ptr(), _stream(x.device)), "ep_route_dispatch")

    def p2p_experts(self, xch, C):
        dev = self.ws.device
        _lib.check(self.lib.mfi_ep_experts_return(
            ctypes.byref(self._exp_w), xch.rank, self.world, C, xch.table.data_ptr(), xch.flags,
            xch.recv, self.ws.data_ptr(), self.ws.numel(), _stream(dev)), "ep_experts_return")

    def p2p_finish(self, T, out, pack_pos, xch, C):
        _lib.check(self.lib.mfi_ep_unpack_wait(
            self.world, C, self.H, T, xch.flags, xch.ret, pack_pos.data_ptr(), out.data_ptr(),
            _stream(out.device)), "ep_unpack_wait")


class P2PExchange:
    """This rank's exchange memory — receive buffer, return buffer and flag
    area in one block that the peers map through CUDA IPC — and the device
    table of every rank's addresses as seen from this rank."""

    def __init__(self, world: int, rank: int, capacity: int, hidden: int, top_k: int, device):
        lib = _lib.load()
        self.lib = lib
        self.world, self.rank = world, rank
        self.recv_bytes = int(lib.mfi_ep_recv_bytes(world, capacity, hidden, top_k))
        self.ret_bytes = int(lib.mfi_ep_ret_bytes(world, capacity, hidden))
        self.flag_bytes = int(lib.mfi_ep_flag_bytes())
        if not (self.recv_bytes and self.ret_bytes and self.flag_bytes):
            raise RuntimeError("invalid exchange shape")
        up = lambda v: (v + 255) // 256 * 256
        self.off_ret = up(self.recv_bytes)
        self.off_flags = self.off_ret + up(self.ret_bytes)
        self.total = self.off_flags + up(self.flag_bytes)
        ptr = ctypes.c_void_p()
        _lib.check(lib.mfi_ipc_alloc(self.total, ctypes.byref(ptr)), "ipc_alloc")
        self.base = int(ptr.value)
        self.table = torch.empty(int(lib.mfi_ep_table_bytes()), dtype=torch.uint8, device=device)
        self._opened: list[int] = []

    @property
    def recv(self) -> int:
        return self.base

    @property
    def ret(self) -> int:
        return self.base + self.off_ret

    @property
    def flags(self) -> int:
        return self.base + self.off_flags

    def copy_recv_to(self, dst: torch.Tensor) -> None:
        """Copy this rank's receive buffer into a cuda tensor (inspection)."""
        if dst.numel() * dst.element_size() < self.recv_bytes or not dst.is_contiguous():
            raise RuntimeError("destination too small")
        _lib.check(self.lib.mfi_copy_async(dst.data_ptr(), self.recv, self.recv_bytes,
                                           _stream(dst.device)), "copy")

    def handle(self) -> bytes:
        h = ctypes.create_string_buffer(64)
        _lib.check(self.lib.mfi_ipc_handle(self.base, h), "ipc_handle")
        return h.raw

    def connect(self, bases) -> None:
        """bases[d]: rank d's block address as seen from this rank."""
        n = self.world
        if len(bases) != n:
            raise RuntimeError("one base address per rank")
        arr = lambda off: (ctypes.c_void_p * n)(*[b + off for b in bases])
        _lib.check(self.lib.mfi_ep_table_set(self.table.data_ptr(), n, arr(0), arr(self.off_ret),
                                             arr(self.off_flags)), "ep_table_set")

    def connect_group(self, group=None) -> None:
        """Exchange IPC handles over the process group and map every peer."""
        handles = [None] * self.world
        dist.all_gather_object(handles, self.handle(), group=group)
        bases = []
        for d, h in enumerate(handles):
            if d == self.rank:
                bases.append(self.base)
                continue
            ptr = ctypes.c_void_p()
            _lib.check(self.lib.mfi_ipc_open(h, ctypes.byref(ptr)), "ipc_open")
            self._opened.append(int(ptr.value))
            bases.append(int(ptr.value))
        self.connect(bases)

    def close(self) -> None:
        for p in self._opened:
            self.lib.mfi_ipc_close(p)
        self._opened = []
        if self.base:
            self.lib.mfi_ipc_free(self.base)
            self.base = 0


class EPMoELayer:
    """One MoE layer sharded over the ranks of ``group`` (expert parallelism).

    ``capacity`` is the largest token count any rank passes to one forward;
    every rank must call forward the same number of times (the all-to-alls
    are collective)."""

    def __init__(self, shard: EPShard, top_k: int, capacity: int, group=None, ops=None,
                 device=None, world: int | None = None, rank: int | None = None,
                 transport: str | None = None, connect: bool = True,
                 logit_bias: torch.Tensor | None = None):
        self.group = group
        # world / rank may be given to drive the steps without a process group
        # (all ranks of a test in one process, the exchange done by copies)
        self.world = dist.get_world_size(group) if world is None else int(world)
        self.rank = dist.get_rank(group) if rank is None else int(rank)
        if shard.local_experts * self.world != shard.n_experts:
            raise RuntimeError("local experts x ranks must equal the router's expert count")
        if not 1 <= top_k <= min(shard.n_experts, 32):
            raise RuntimeError("top_k must be in [1, min(E, 32)]")
        self.shard = shard
        self.k = top_k
        self.C = int(capacity)
        if ops is not None and logit_bias is not None:
            raise RuntimeError("logit_bias is applied by the GPU router only")
        self.ops = ops if ops is not None else CudaEPOps(shard, top_k, self.C, self.world,
                                                         logit_bias=logit_bias)
        dev = device if device is not None else shard.gate_wp.device
        H, n, C = shard.hidden, self.world, self.C
        rb = ep_row_bytes(H, top_k)
        self.xq = torch.empty((C, H // 2), dtype=torch.uint8, device=dev)
        self.xsc = torch.empty((C, H // 32), dtype=torch.uint8, device=dev)
        self.topi = torch.empty((C, top_k), dtype=torch.int32, device=dev)
        self.topw = torch.empty((C, top_k), dtype=torch.float32, device=dev)
        self.counts = torch.zeros(n, dtype=torch.int32, device=dev)
        self.pack_pos = torch.empty((C, n), dtype=torch.int32, device=dev)
        # the peer-memory transport runs the decode expert kernels (at most
        # 16384 (row, slot) pairs per rank); larger exchanges (prefill) take
        # the all-to-all transport, whose expert step switches to the prefill
        # kernels
        p2p_fits = n * (C + 1) * top_k <= P2P_MAX_PAIRS
        if transport is None:
            transport = ("nccl" if ops is not None or not torch.device(dev).type == "cuda"
                         or not p2p_fits else "p2p")
        if transport not in ("p2p", "nccl"):
            raise RuntimeError("transport must be 'p2p' or 'nccl'")
        if transport == "p2p" and not p2p_fits:
            raise RuntimeError(f"the p2p transport holds at most {P2P_MAX_PAIRS} (row, slot) pairs "
                               f"per rank: world * (capacity + 1) * top_k = {n * (C + 1) * top_k}")
        self.transport = transport
        self.xch = None
        if transport == "p2p":
            if not isinstance(self.ops, CudaEPOps):
                raise RuntimeError("the p2p transport runs on the GPU library only")
            self.xch = P2PExchange(n, self.rank, C, H, top_k, dev)
            if connect:
                self.xch.connect_group(group)
        else:
            self.send = torch.zeros((n, C + 1, rb), dtype=torch.uint8, device=dev)
            self.recv = torch.zeros_like(self.send)
            self.ret = torch.empty((n, C + 1, H), dtype=torch.float32, device=dev)
            self.ret_back = torch.empty_like(self.ret)

    def close(self) -> None:
        """Release the peer mappings (p2p transport)."""
        if self.xch is not None:
            self.xch.close()
            self.xch = None

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None):
        """x bf16 (T, hidden), T <= capacity -> fp32 (T, hidden); also leaves the
        routing in ``self.topi[:T]`` / ``self.topw[:T]``."""
        T, H = x.shape
        if T > self.C:
            raise RuntimeError(f"T={T} exceeds the layer's capacity {self.C}")
        if H != self.shard.hidden:
            raise RuntimeError(f"x must have {self.shard.hidden} columns")
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        if self.transport == "p2p":
            self.p2p_dispatch(x)
            self.p2p_experts()
            self.p2p_finish(T, out)
            return out
        self.dispatch_prepare(x)
        dist.all_to_all_single(self.recv.view(-1), self.send.view(-1), group=self.group)
        self.compute()
        dist.all_to_all_single(self.ret_back.view(-1), self.ret.view(-1), group=self.group)
        self.finish(T, out)
        return out

    # The three local parts of a forward, between which the two exchanges run:
    # send -> recv (block d of send goes to rank d) and ret -> ret_back.
    def dispatch_prepare(self, x: torch.Tensor) -> None:
        """Route x and pack it into ``self.send``."""
        x = x.contiguous()
        T = x.shape[0]
        self.ops.route(x, self.xq, self.xsc, self.topi, self.topw)
        self.ops.pack(self.xq, self.xsc, self.topi, self.topw, T, self.counts, self.send,
                      self.pack_pos)

    def compute(self) -> None:
        """Expert compute on ``self.recv`` into ``self.ret``."""
        self.ops.experts(self.recv, self.ret)

    def finish(self, T: int, out: torch.Tensor) -> None:
        """Sum the returned rows of ``self.ret_back`` into out (T, hidden)."""
        self.ops.unpack(self.ret_back, self.pack_pos, T, out)

    # p2p transport: the three launches groups of a forward, in order
    def p2p_dispatch(self, x: torch.Tensor) -> None:
        x = x.contiguous()
        self.ops.p2p_dispatch(x, self.topi, self.topw, self.pack_pos, self.xch, self.C)

    def p2p_experts(self) -> None:
        self.ops.p2p_experts(self.xch, self.C)

    def p2p_finish(self, T: int, out: torch.Tensor) -> None:
        self.ops.p2p_finish(T, out, self.pack_pos, self.xch, self.C)

    __call__ = forward
