"""Expert parallelism: one MoE layer with its experts sharded over the ranks of a
process group, one rank per GPU.

No counterpart in the reference, which serves from a single device
(projects/oom-inference/crates/oominf-cuda/src/lib.rs:1-5): this is the
expert-parallel form of Moe::forward's routed half (crates/oominf-models-qwen/
src/moe.rs:254-366).  Expert e lives on rank e // experts_per_rank; the router
is replicated.  A decode step on every rank, for its own t tokens:

  1. route: logits and softmax top-k (ids, weights) of the rank's tokens;
  2. meta[g][t][s]: local id on rank g of slot s's expert, or -1;
  3. all-to-all of meta and of the tokens' activations (every rank receives
     every rank's t rows: fixed sizes, so no host round trip and the step can
     be captured in a CUDA graph);
  4. group the received assignments by local expert, in (source rank, token,
     slot) order, and run gate/up+SiLU and down on them;
  5. scatter each output row to its slot's place in the return buffer of its
     source rank; reverse all-to-all;
  6. combine each token's k slots in slot order.

Steps 4 and 6 are the single-GPU kernels' arithmetic and an expert output does
not depend on what else shares its launch, so each rank's output is
bit-identical to the single-GPU decode of the same tokens.

The device steps go through an `ops` object (EpGpuOps here: the C ABI of
liboomb.so) and the exchanges through torch.distributed (NCCL on GPUs).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._lib import BF16, F32, check

# Tokens over all ranks (ranks x t) from which the peer chain runs its local
# experts on the tensor cores (oomb_moe_experts_tiled_fp8), as the single-GPU
# decode step does from 17 tokens.
EP_TILED_MIN_TOKENS = 17


class EpGpuOps:
    """The device steps of an expert-parallel layer on liboomb.so."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.L = _lib.lib()

    def _s(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def route(self, x, router_w, logits, ids, weights, t, e, k, hidden):
        xd = BF16 if x.dtype == torch.bfloat16 else F32
        check(self.L.oomb_router_logits(x.data_ptr(), xd, router_w.data_ptr(), logits.data_ptr(), t, e, hidden,
                                        self._s()), "router_logits")
        check(self.L.oomb_router_topk(logits.data_ptr(), ids.data_ptr(), weights.data_ptr(), t, e, k, self._s()),
              "router_topk")

    def meta(self, ids, t, k, epr, ranks, meta):
        check(self.L.oomb_ep_meta(ids.data_ptr(), t, k, epr, ranks, meta.data_ptr(), self._s()), "ep_meta")

    def group(self, recv_meta, ranks, t, k, epr, recs_local, n_active, off, assign_row, assign_ret, recs_active):
        check(self.L.oomb_ep_group(recv_meta.data_ptr(), ranks, t, k, epr, recs_local.data_ptr(),
                                   n_active.data_ptr(), off.data_ptr(), assign_row.data_ptr(), assign_ret.data_ptr(),
                                   recs_active.data_ptr(), self._s()), "ep_group")

    def experts(self, recs_active, off, assign_row, n_active, max_active, x, h, y, geo, max_per_expert):
        xd = BF16 if x.dtype == torch.bfloat16 else F32
        check(self.L.oomb_moe_experts_fp8(recs_active.data_ptr(), off.data_ptr(), assign_row.data_ptr(),
                                          n_active.data_ptr(), max_active, x.data_ptr(), xd, h.data_ptr(),
                                          y.data_ptr(), C.byref(geo), max_per_expert, self._s()), "moe_experts")

    def experts_tiled(self, recs_active, off, assign_row, n_active, max_active, max_assignments, x, h, y, geo,
                      max_per_expert, ws):
        """The same step on the tensor cores (oomb_moe_experts_tiled_fp8); ws from
        tiled_workspace."""
        xd = BF16 if x.dtype == torch.bfloat16 else F32
        check(self.L.oomb_moe_experts_tiled_fp8(recs_active.data_ptr(), off.data_ptr(), assign_row.data_ptr(),
                                                n_active.data_ptr(), max_active, max_assignments, x.data_ptr(), xd,
                                                h.data_ptr(), y.data_ptr(), C.byref(geo), max_per_expert,
                                                ws.data_ptr(), ws.numel(), self._s()), "moe_experts_tiled")

    def tiled_workspace(self, max_assignments, geo, x_dtype=torch.bfloat16):
        """The workspace of experts_tiled, or None when the layer's shapes are
        outside the tensor-core path."""
        xd = BF16 if x_dtype == torch.bfloat16 else F32
        n = self.L.oomb_moe_experts_tiled_fp8_workspace_bytes(max_assignments, C.byref(geo), xd)
        return torch.empty(n, dtype=torch.uint8, device=self.device) if n else None

    def scatter(self, y, n_active, off, assign_ret, hidden, max_rows, ret):
        check(self.L.oomb_ep_scatter(y.data_ptr(), n_active.data_ptr(), off.data_ptr(), assign_ret.data_ptr(),
                                     hidden, max_rows, ret.data_ptr(), self._s()), "ep_scatter")

    def combine(self, back, ids, weights, t, k, hidden, epr, ranks, out):
        od = BF16 if out.dtype == torch.bfloat16 else F32
        check(self.L.oomb_ep_combine(back.data_ptr(), ids.data_ptr(), weights.data_ptr(), t, k, hidden, epr, ranks,
                                     out.data_ptr(), od, self._s()), "ep_combine")


class EpMoeLayer:
    """A MoE layer whose experts are sharded over `group` (this rank holds experts
    [rank * epr, (rank + 1) * epr)).  recs_local: int64 device addresses of the
    local expert records; geo: their Fp8Record; router_w: bf16 [experts, hidden]
    (replicated).  Buffers are sized for up to t_max tokens per rank."""

    def __init__(self, ops, group, hidden, experts, top_k, inter, router_w, recs_local, geo, t_max,
                 x_dtype=torch.bfloat16, ranks=None, rank=None):
        self.ops, self.group = ops, group
        # ranks / rank given explicitly: virtual ranks in one process (no group)
        self.G = ranks if ranks is not None else dist.get_world_size(group)
        self.rank = rank if rank is not None else dist.get_rank(group)
        if experts % self.G:
            raise ValueError("experts must divide evenly over the ranks")
        self.H, self.E, self.K, self.I = hidden, experts, top_k, inter
        self.epr = experts // self.G
        self.router_w, self.recs_local, self.geo = router_w, recs_local, geo
        self.t_max = t_max
        dev = router_w.device
        G, T, K, H = self.G, t_max, top_k, hidden
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.logits = torch.empty((T, experts), **f32)
        self.ids = torch.empty((T, K), **i32)
        self.weights = torch.empty((T, K), **f32)
        self.meta = torch.empty((G, T, K), **i32)
        self.recv_meta = torch.empty((G, T, K), **i32)
        self.send_x = torch.empty((G, T, H), dtype=x_dtype, device=dev)
        self.recv_x = torch.empty((G, T, H), dtype=x_dtype, device=dev)
        A = G * T * K
        self.n_active = torch.zeros(1, **i32)
        self.off = torch.zeros(self.epr + 1, **i32)
        self.assign_row = torch.zeros(A, **i32)
        self.assign_ret = torch.zeros(A, **i32)
        self.recs_active = torch.zeros(self.epr, dtype=torch.int64, device=dev)
        self.h = torch.empty((A, inter), **f32)
        self.y = torch.empty((A, H), **f32)
        self.ret = torch.zeros((G, T * K, H), **f32)
        self.back = torch.empty((G, T * K, H), **f32)

    # The step in three device phases separated by the two exchanges.  Each
    # exchange is an all-to-all of equal chunks: rank g's chunk of `send` goes
    # to rank g and lands in chunk (sender) of `recv`.

    def phase_route(self, x, t: int):
        """Route, meta, staged activations; returns the first exchange's
        [(send_meta, recv_meta), (send_x, recv_x)] views."""
        if t > self.t_max:
            raise ValueError("more tokens than the layer's buffers hold")
        G, K, H = self.G, self.K, self.H
        self.ops.route(x, self.router_w, self.logits, self.ids, self.weights, t, self.E, K, H)
        self.ops.meta(self.ids, t, K, self.epr, G, self.meta)
        send_meta = self.meta.view(-1)[: G * t * K].view(G, t, K)
        recv_meta = self.recv_meta.view(-1)[: G * t * K].view(G, t, K)
        send_x = self.send_x.view(-1)[: G * t * H].view(G, t, H)
        send_x.copy_(x[:t].unsqueeze(0).expand(G, t, H))
        recv_x = self.recv_x.view(-1)[: G * t * H].view(G, t, H)
        return [(send_meta, recv_meta), (send_x, recv_x)]

    def phase_experts(self, t: int):
        """Group the received assignments, run the local experts, stage the
        outputs for their source ranks; returns the second exchange's (send, recv)."""
        G, K, H = self.G, self.K, self.H
        recv_meta = self.recv_meta.view(-1)[: G * t * K].view(G, t, K)
        recv_x = self.recv_x.view(-1)[: G * t * H].view(G * t, H)
        self.ops.group(recv_meta, G, t, K, self.epr, self.recs_local, self.n_active, self.off, self.assign_row,
                       self.assign_ret, self.recs_active)
        max_active = min(self.epr, G * t * K)
        self.ops.experts(self.recs_active, self.off, self.assign_row, self.n_active, max_active, recv_x, self.h,
                         self.y, self.geo, G * t)
        ret = self.ret.view(-1)[: G * t * K * H].view(G, t * K, H)
        self.ops.scatter(self.y, self.n_active, self.off, self.assign_ret, H, G * t * K, ret)
        back = self.back.view(-1)[: G * t * K * H].view(G, t * K, H)
        return ret, back

    def phase_combine(self, t: int, out):
        G, K, H = self.G, self.K, self.H
        back = self.back.view(-1)[: G * t * K * H].view(G, t * K, H)
        self.ops.combine(back, self.ids, self.weights, t, K, H, self.epr, G, out)
        return self.ids[:t], self.weights[:t]

    def forward(self, x, t: int, out):
        """out[t, hidden] = the routed experts' combined output for this rank's t tokens;
        returns (ids, weights) of the routing."""
        for send, recv in self.phase_route(x, t):
            dist.all_to_all_single(recv, send, group=self.group)
        ret, back = self.phase_experts(t)
        dist.all_to_all_single(back, ret, group=self.group)
        return self.phase_combine(t, out)


def exchange_local(sends, recvs):
    """The all-to-all of equal chunks between ranks that live in one process
    (virtual ranks on one device, tests): recvs[g][src] = sends[src][g]."""
    G = len(sends)
    for g in range(G):
        for src in range(G):
            recvs[g][src].copy_(sends[src][g])


# ---- the exchanges through peer memory ---------------------------------------------------

class _DeviceBytes:
    """A raw device allocation seen through __cuda_array_interface__ (no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _bytes_view(ptr: int, nbytes: int, device) -> torch.Tensor:
    return torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)


class EpPeerMailboxes:
    """The mailboxes of the peer-memory exchange (oomb_ep_peer).  With a process
    group: this process's mailbox (cudaMalloc'd by the library) mapped into every
    peer through CUDA IPC, the handles exchanged over the group.  With `ranks`
    given: virtual ranks in this process, one mailbox each (tests)."""

    def __init__(self, group, hidden, top_k, t_max, x_dtype, device, ranks=None):
        self.L = L = _lib.lib()
        self.device = torch.device(device)
        self.virtual = ranks is not None
        self.G = ranks if self.virtual else dist.get_world_size(group)
        self.rank = None if self.virtual else dist.get_rank(group)
        self.hidden, self.top_k, self.t_max = hidden, top_k, t_max
        self.x_dtype = x_dtype
        self.xd = BF16 if x_dtype == torch.bfloat16 else F32
        self.nbytes = int(L.oomb_ep_mailbox_bytes(self.G, t_max, top_k, hidden, self.xd))
        if self.nbytes == 0:
            raise ValueError("unsupported mailbox shape")
        self.x_off = int(L.oomb_ep_mailbox_x_offset(self.G, t_max, top_k, hidden, self.xd))
        self.owned, self.opened = [], []
        with torch.cuda.device(self.device):
            if self.virtual:
                bases = [self._alloc() for _ in range(self.G)]
            else:
                own = self._alloc()
                h = (C.c_ubyte * _lib.IPC_HANDLE_BYTES)()
                check(L.oomb_ipc_handle(own, h), "ipc_handle")
                handles = [None] * self.G
                dist.all_gather_object(handles, bytes(h), group=group)
                bases = []
                for g, hb in enumerate(handles):
                    if g == self.rank:
                        bases.append(own)
                        continue
                    buf = (C.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                    p = C.c_void_p()
                    check(L.oomb_ipc_open(buf, C.byref(p)), "ipc_open")
                    self.opened.append(p.value)
                    bases.append(p.value)
        self.bases = bases
        self.peers = torch.tensor(bases, dtype=torch.int64, device=self.device)

    def _alloc(self) -> int:
        p = C.c_void_p()
        check(self.L.oomb_ep_mailbox_alloc(self.nbytes, C.byref(p)), "mailbox_alloc")
        self.owned.append(p.value)
        return p.value

    def view(self, rank: int) -> _lib.EpPeer:
        """The oomb_ep_peer of `rank` (this process's rank for a real group)."""
        return _lib.EpPeer(self.peers.data_ptr(), self.bases[rank], self.G, rank, self.t_max, self.top_k,
                           self.hidden, self.xd)

    def recv_x(self, rank: int, t: int) -> torch.Tensor:
        """The received activations [G * t, hidden] in `rank`'s mailbox."""
        xb = 2 if self.x_dtype == torch.bfloat16 else 4
        raw = _bytes_view(self.bases[rank] + self.x_off, self.G * t * self.hidden * xb, self.device)
        return raw.view(self.x_dtype).view(self.G * t, self.hidden)

    def close(self):
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for p in self.opened:
                self.L.oomb_ipc_close(p)
            for p in self.owned:
                self.L.oomb_ep_mailbox_free(p)
        self.opened, self.owned = [], []


class EpPeerMoeLayer:
    """EpMoeLayer with its three all-to-alls done by the kernels over peer memory
    (oomb_ep_dispatch_peer / _group_peer / _return_peer / _combine_peer): no
    collective library on the data path, and the whole step stream-ordered on
    the device, so it captures into a CUDA graph.  Buffers as EpMoeLayer's."""

    def __init__(self, ops, mailboxes: EpPeerMailboxes, rank, hidden, experts, top_k, inter, router_w, recs_local,
                 geo, t_max):
        self.ops, self.mb = ops, mailboxes
        self.L = _lib.lib()
        self.G, self.rank = mailboxes.G, rank
        if experts % self.G:
            raise ValueError("experts must divide evenly over the ranks")
        if t_max > mailboxes.t_max:
            raise ValueError("more tokens than the mailboxes hold")
        self.H, self.E, self.K, self.I = hidden, experts, top_k, inter
        self.epr = experts // self.G
        self.router_w, self.recs_local, self.geo = router_w, recs_local, geo
        self.t_max = t_max
        self.q = mailboxes.view(rank)
        dev = router_w.device
        G, T, K = self.G, t_max, top_k
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        self.logits = torch.empty((T, experts), **f32)
        self.ids = torch.empty((T, K), **i32)
        self.weights = torch.empty((T, K), **f32)
        A = G * T * K
        self.n_active = torch.zeros(1, **i32)
        self.off = torch.zeros(self.epr + 1, **i32)
        self.assign_row = torch.zeros(A, **i32)
        self.assign_ret = torch.zeros(A, **i32)
        self.recs_active = torch.zeros(self.epr, dtype=torch.int64, device=dev)
        self.h = torch.empty((A, inter), **f32)
        self.y = torch.empty((A, hidden), **f32)
        # from EP_TILED_MIN_TOKENS tokens over the ranks the local experts run on the tensor cores
        self.tiled_ws = ops.tiled_workspace(A, geo, mailboxes.x_dtype) if G * T >= EP_TILED_MIN_TOKENS else None

    def _s(self):
        return torch.cuda.current_stream(self.router_w.device).cuda_stream

    def phase_route(self, x, t: int):
        """Route this rank's t tokens and dispatch them to every rank's mailbox."""
        if t > self.t_max:
            raise ValueError("more tokens than the layer's buffers hold")
        self.ops.route(x, self.router_w, self.logits, self.ids, self.weights, t, self.E, self.K, self.H)
        check(self.L.oomb_ep_dispatch_peer(C.byref(self.q), self.ids.data_ptr(), t, self.epr, x.data_ptr(), self._s()),
              "ep_dispatch_peer")

    def phase_experts(self, t: int):
        """Group what every rank dispatched here, run the local experts, return the rows."""
        check(self.L.oomb_ep_group_peer(C.byref(self.q), t, self.epr, self.recs_local.data_ptr(),
                                        self.n_active.data_ptr(), self.off.data_ptr(), self.assign_row.data_ptr(),
                                        self.assign_ret.data_ptr(), self.recs_active.data_ptr(), self._s()),
              "ep_group_peer")
        G, K = self.G, self.K
        max_active = min(self.epr, G * t * K)
        if self.tiled_ws is not None and G * t >= EP_TILED_MIN_TOKENS:
            self.ops.experts_tiled(self.recs_active, self.off, self.assign_row, self.n_active, max_active, G * t * K,
                                   self.mb.recv_x(self.rank, t), self.h, self.y, self.geo, G * t, self.tiled_ws)
        else:
            self.ops.experts(self.recs_active, self.off, self.assign_row, self.n_active, max_active,
                             self.mb.recv_x(self.rank, t), self.h, self.y, self.geo, G * t)
        check(self.L.oomb_ep_return_peer(C.byref(self.q), self.y.data_ptr(), self.n_active.data_ptr(),
                                         self.off.data_ptr(), self.assign_ret.data_ptr(), t, G * t * K, self._s()),
              "ep_return_peer")

    def phase_combine(self, t: int, out):
        od = BF16 if out.dtype == torch.bfloat16 else F32
        check(self.L.oomb_ep_combine_peer(C.byref(self.q), self.ids.data_ptr(), self.weights.data_ptr(), t, self.epr,
                                          out.data_ptr(), od, self._s()), "ep_combine_peer")
        return self.ids[:t], self.weights[:t]

    def forward(self, x, t: int, out):
        """out[t, hidden] = the routed experts' combined output for this rank's t tokens."""
        self.phase_route(x, t)
        self.phase_experts(t)
        return self.phase_combine(t, out)


class EpDecodeLayer:
    """The expert-parallel decode step in one launch per rank
    (oomb_moe_decode_ep_fp8): route, dispatch into the mailboxes, the local
    experts with each output value stored into its source rank's mailbox as an
    (epoch, value) word, and the slot-order combine polling those words, for up
    to 16 tokens per rank and 256 experts.  Every
    rank runs each step with the same t; the kernels of the ranks wait on one
    another (bounded waits), so each rank's runs on its own GPU."""

    def __init__(self, mailboxes: EpPeerMailboxes, rank, hidden, experts, top_k, router_w, recs_local, geo, t_max):
        self.L = L = _lib.lib()
        self.mb = mailboxes
        self.q = mailboxes.view(rank)
        self.layer = _lib.MoeLayer(hidden=hidden, experts=experts, top_k=top_k, router_w=router_w.data_ptr(),
                                   recs=recs_local.data_ptr())
        self.layer.geo = geo
        self._keep = (router_w, recs_local)
        dev = router_w.device
        self.t_max = t_max
        n = int(L.oomb_moe_decode_ep_workspace_bytes(t_max, mailboxes.G, C.byref(self.layer)))
        if n == 0:
            raise ValueError("unsupported expert-parallel layer shape")
        self.ws = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.ids = torch.empty((t_max, top_k), dtype=torch.int32, device=dev)
        self.weights = torch.empty((t_max, top_k), dtype=torch.float32, device=dev)

    def forward(self, x, t: int, out):
        """out[t, hidden] = the routed experts' combined output for this rank's t tokens."""
        xd = BF16 if x.dtype == torch.bfloat16 else F32
        od = BF16 if out.dtype == torch.bfloat16 else F32
        s = torch.cuda.current_stream(self.ws.device).cuda_stream  # x and out may be pinned host tensors
        check(self.L.oomb_moe_decode_ep_fp8(C.byref(self.layer), C.byref(self.q), x.data_ptr(), xd, t, out.data_ptr(),
                                            od, self.ids.data_ptr(), self.weights.data_ptr(), self.ws.data_ptr(),
                                            self.ws.numel(), s), "moe_decode_ep")
        return self.ids[:t], self.weights[:t]
