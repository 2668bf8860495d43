"""Expert-parallel routed-MoE layer over NCCL (NVLink / NVSwitch).

The reference keeps every expert on every TP rank and refuses expert
parallelism (engine/patches/gguf_moe.patch:57-58); its tier placement
(engine/.../experts/nvfp4_8r_tiers.py) becomes ownership here: rank r owns the
contiguous expert ids ``tiers.owner_ranges(E, world)[r]``, in either format.

Two exchanges, the same arithmetic (per rank: its own T tokens, all ranks
call in the same order):

``exchange="p2p"`` (default): the library's own kernels over NVLink peer
memory (CUDA IPC, no multicast): ``b200moe_ep_push`` stores each route's fp16
row and expert id straight into its owner's receive buffer, at a row the
route reserves with one atomic on the owner's counter (no rank waits for
another's counts); the owner runs its experts on what it received
(``b200moe_ep_forward``: top-1 rows, y2 rows out; its first launch waits for
every rank's push); ``b200moe_ep_return`` stores the y2 rows back into their
home ranks; ``b200moe_ep_combine_p2p`` sums them per token in slot order and
adds the residual.  Counts and hand-offs live on the device (bounded flag
waits), so a step needs no host sync and can be captured in a CUDA graph.

``exchange="nccl"``: ``b200moe_ep_dispatch`` + one host read of the counts +
NCCL all-to-all out and back + ``b200moe_ep_combine``.

Communication is timed with CUDA events on the launching stream
(``comm_ms()``: the exposed, non-overlapped exchange time of the last call,
waits for slower ranks included).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from . import tiers as tiersmod
from .moe import B200NativeMoe


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def gate(logits: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax top-k gating (the library's rule) without a layer object."""
    t, e = logits.shape
    ids = torch.empty((t, top_k), dtype=torch.int32, device=logits.device)
    w = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    err = torch.zeros(1, dtype=torch.int32, device=logits.device)
    _lib.check("b200moe_gate", _lib.lib().b200moe_gate(_stream(), logits.data_ptr(), t, e, top_k, ids.data_ptr(),
                                                         w.data_ptr(), err.data_ptr()))
    return ids, w


def check_placement(tier, world: int, group=None, owner=None) -> str:
    """Every rank must hold the same tier array, world size and owner map; a
    rank that differs makes every rank raise (the reference's stage digest
    check, engine/.../experts/nvfp4_8r_native.py:1657-1659)."""
    digest = tiersmod.placement_digest(tier, world, owner)
    if world == 1 or not dist.is_initialized():
        return digest
    digests = [None] * world
    dist.all_gather_object(digests, digest, group=group)
    if len(set(digests)) != 1:
        raise RuntimeError(f"expert placement differs across ranks: {sorted(set(d[:12] for d in digests))}")
    return digest


def owner_of_expert(num_experts: int, world: int) -> np.ndarray:
    """The default placement: contiguous expert-id ranges."""
    return tiersmod.owner_by_range(num_experts, world)


def exchange_counts(send_counts: torch.Tensor, world: int, group=None) -> tuple[list[int], list[int]]:
    """(routes this rank sends to each rank, routes it receives from each rank):
    one all_gather of the per-rank counts (works on NCCL and gloo)."""
    if world == 1:
        c = send_counts.cpu().tolist()
        return c, c
    gathered = [torch.empty_like(send_counts) for _ in range(world)]
    dist.all_gather(gathered, send_counts, group=group)
    rank = dist.get_rank(group)
    mat = torch.stack(gathered).cpu()  # mat[src][dst]
    return mat[rank].tolist(), mat[:, rank].tolist()


class PeerExchange:
    """The NVLink peer-memory exchange of one process group: receive buffers
    every rank maps through CUDA IPC (``b200moe_ep_*``).  Layers that run one
    after another on the same stream may share one (``ExpertParallelMoe(peer=)``);
    ``max_routes`` bounds the routes one rank sends in a step (tokens * top_k).
    Creating and closing it are collectives."""

    def __init__(self, hidden: int, max_routes: int, group=None, device: torch.device | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.hidden, self.max_routes = hidden, max_routes
        L = _lib.lib()
        ep = ctypes.c_void_p()
        _lib.check("b200moe_ep_create", L.b200moe_ep_create(self.device.index, self.world, self.rank, hidden,
                                                            max_routes, ctypes.byref(ep)))
        self.handle = ep
        h = (ctypes.c_uint8 * 64)()
        _lib.check("b200moe_ep_ipc_handle", L.b200moe_ep_ipc_handle(ep, h))
        handles = [bytes(h)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=group)
        _lib.check("b200moe_ep_connect", L.b200moe_ep_connect(ep, ctypes.c_char_p(b"".join(handles))))
        ptrs = [ctypes.c_void_p() for _ in range(5)]
        max_rows = ctypes.c_int()
        _lib.check("b200moe_ep_recv_buffers", L.b200moe_ep_recv_buffers(ep, *(ctypes.byref(p) for p in ptrs),
                                                                       ctypes.byref(max_rows)))
        self.rows, self.eids, self.n_valid, self.row_range, self.y2 = (p.value for p in ptrs)
        self.max_rows = max_rows.value
        if self.world > 1:
            dist.barrier(group=group)  # every rank mapped every buffer before the first push

    def check(self) -> int:
        return _lib.lib().b200moe_ep_check_errors(self.handle, _stream(), None)

    def received(self) -> np.ndarray:
        n = ctypes.c_int()
        ids = np.empty(self.max_rows, np.int32)
        _lib.check("b200moe_ep_received", _lib.lib().b200moe_ep_received(
            self.handle, _stream(), ctypes.byref(n), ids.ctypes.data_as(ctypes.c_void_p), ids.size))
        return ids[:n.value]

    def close(self) -> None:
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # no rank still writes into another's buffers
        _lib.lib().b200moe_ep_destroy(self.handle)
        self.handle = None


class ExpertParallelMoe:
    """One routed-MoE layer with its experts sharded over a process group.

    ``tokens`` bounds the tokens one rank passes per forward.  Local experts
    run with the skinny kernels (``gemm="skinny"``, a rank sees few routes per
    expert at decode) or, for an NVFP4 bank, the block-scaled FP4 tensor path
    (``gemm="fp4"``).  With ``split_k`` fixed here and on a single-GPU layer of
    the same ``gemm``, the outputs of the two are bit-equal (same per-route
    rows, same slot-order combine)."""

    def __init__(self, *, hidden: int, inter: int, num_experts: int, top_k: int, tokens: int, tier,
                 fp4_format: str = "nvfp4", group=None, device: torch.device | None = None,
                 split_k: tuple[int, int] | None = None, exchange: str = "p2p", peer: PeerExchange | None = None,
                 gemm: str = "skinny", owner=None, iq_types: tuple[int, int] = (16, 16)):
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange is 'p2p' or 'nccl'")
        self.exchange = exchange
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.tier = tiersmod.check_tier_array(tier, num_experts)
        owner_np = (owner_of_expert(num_experts, self.world) if owner is None
                    else tiersmod.check_owner(owner, num_experts, self.world))
        self.digest = check_placement(self.tier, self.world, group, None if owner is None else owner_np)
        self.hidden, self.inter, self.num_experts, self.top_k, self.tokens = hidden, inter, num_experts, top_k, tokens
        S = tokens * top_k
        r_max = S * self.world  # every route of every rank could land here
        self.layer = B200NativeMoe(hidden=hidden, inter=inter, num_experts=num_experts, top_k=1,
                                   max_tokens=min(64, r_max), max_prefill_tokens=r_max, tier=self.tier,
                                   fp4_format=fp4_format, device=dev, rank=self.rank, world=self.world,
                                   prefill_gemm=gemm, owner=owner_np, iq_types=iq_types)
        if split_k is not None:
            self.layer.set_split_k(*split_k)
        self.owner_np = owner_np
        self.owner = torch.from_numpy(owner_np).to(dev)
        f16 = dict(dtype=torch.float16, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        self._plan_ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]  # start, convert, plan
        self._last_plan_events = []
        self._timed = False
        self.last_routes_in = 0
        self._peer, self._own_peer = None, False
        # FP4-only block-scaled owners store their y2 rows at home from the W2 epilogue (no return launch)
        self.fused_return = exchange == "p2p" and gemm == "fp4" and self.layer.n_iq2 == 0 and self.layer.n_fp4 > 0
        if exchange == "p2p":
            if peer is None:
                peer, self._own_peer = PeerExchange(hidden, S, group, dev), True
            elif peer.hidden != hidden or peer.max_routes < S or peer.world != self.world:
                raise ValueError("the shared exchange does not fit this layer")
            self._peer = peer
            return
        self.send_rows = torch.empty((S, hidden), **f16)
        self.send_eid = torch.empty(S, **i32)
        self.route_pos = torch.empty(S, **i32)
        self.send_counts = torch.zeros(self.world, **i32)
        self.recv_rows = torch.empty((r_max, hidden), **f16) if self.world > 1 else None
        self.recv_eid = torch.empty(r_max, **i32) if self.world > 1 else None
        self.ones = torch.ones((r_max, 1), dtype=torch.float32, device=dev)
        self.y2_local = torch.empty((r_max, hidden), **f16)
        self.y2_home = torch.empty((S, hidden), **f16) if self.world > 1 else None
        nbytes = int(_lib.lib().b200moe_ep_workspace_bytes(S, self.world))
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    # weights go to the local layer (slots = this rank's experts of each format, ascending id)
    def load_fp4(self, *args, **kw):
        self.layer.load_fp4(*args, **kw)

    def load_iq2(self, *args, **kw):
        self.layer.load_iq2(*args, **kw)

    def set_iq2_tables(self, *args, **kw):
        self.layer.set_iq2_tables(*args, **kw)

    def set_iq_tables(self):
        self.layer.set_iq_tables()

    def route(self, logits: torch.Tensor):
        return gate(logits, self.top_k)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        T = x.shape[0]
        k = self.top_k
        if not 0 < T <= self.tokens or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [<= {self.tokens}, {self.hidden}], got {tuple(x.shape)}")
        if ids.shape != (T, k) or ids.dtype != torch.int32 or w.shape != (T, k) or w.dtype != torch.float32:
            raise ValueError("ids int32 [T, k] and weights fp32 [T, k] required")
        S = T * k
        dt = _lib.F16 if x.dtype == torch.float16 else _lib.BF16
        L = _lib.lib()
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=self.device)
        if residual is not None and (residual.shape != (T, self.hidden) or residual.dtype != torch.float32):
            raise ValueError("residual must be fp32 [T, hidden]")
        if self.exchange == "p2p":
            return self._forward_p2p(x, dt, ids, w, T, k, residual, out)
        _lib.check("b200moe_ep_dispatch", L.b200moe_ep_dispatch(
            _stream(), x.data_ptr(), dt, ids.data_ptr(), T, k, self.num_experts, self.world, self.owner.data_ptr(),
            self.hidden, self.send_rows.data_ptr(), self.send_eid.data_ptr(), self.route_pos.data_ptr(),
            self.send_counts.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(), self.err.data_ptr()))
        ev = self._ev
        if self.world > 1:
            ev[0].record()
        # routes whose id has no owner are sorted last and never sent
        send_split, recv_split = exchange_counts(self.send_counts, self.world, self.group)
        S_ok, R = int(sum(send_split)), int(sum(recv_split))
        self.last_routes_in = R
        if self.world > 1:
            dist.all_to_all_single(self.recv_rows[:R], self.send_rows[:S_ok], recv_split, send_split,
                                   group=self.group)
            dist.all_to_all_single(self.recv_eid[:R], self.send_eid[:S_ok], recv_split, send_split, group=self.group)
            ev[1].record()
            rows, eid = self.recv_rows, self.recv_eid
        else:
            rows, eid = self.send_rows, self.send_eid
        if R > 0:
            y = self.layer.forward_prefill(rows[:R], eid[:R].view(R, 1), self.ones[:R])
            _lib.check("b200moe_f32_to_f16", L.b200moe_f32_to_f16(_stream(), y.data_ptr(), R * self.hidden,
                                                                    self.y2_local.data_ptr()))
        if self.world > 1:
            ev[2].record()
            dist.all_to_all_single(self.y2_home[:S_ok], self.y2_local[:R], send_split, recv_split, group=self.group)
            ev[3].record()
            y2 = self.y2_home
        else:
            y2 = self.y2_local
        _lib.check("b200moe_ep_combine", L.b200moe_ep_combine(
            _stream(), y2.data_ptr(), self.route_pos.data_ptr(), w.data_ptr(), T, k, self.hidden,
            _lib.ptr(residual), out.data_ptr()))
        self._timed = self.world > 1
        return out

    def _forward_p2p(self, x, dt, ids, w, T, k, residual, out):
        L, st, ev = _lib.lib(), _stream(), self._ev
        timed = torch.cuda.is_current_stream_capturing() is False
        if timed:
            ev[0].record()
        pe = self._peer
        _lib.check("b200moe_ep_push", L.b200moe_ep_push(pe.handle, st, x.data_ptr(), dt, ids.data_ptr(), T, k,
                                                        self.num_experts, self.owner.data_ptr()))
        if timed:
            ev[1].record()
        # the receive wait sits in the forward's first launch (the route plan): time that launch too
        user_events = list(getattr(self.layer, "_timing_events", []) or [])
        plan_events = user_events if len(user_events) >= 3 else (self._plan_ev if timed else [])
        if timed and plan_events is self._plan_ev:
            self.layer.set_timing_events(self._plan_ev)
        _lib.check("b200moe_ep_forward", L.b200moe_ep_forward(pe.handle, self.layer._h, st, int(self.fused_return)))
        if timed and plan_events is self._plan_ev:
            self.layer.set_timing_events(user_events or None)
        self._last_plan_events = plan_events if timed else []
        if timed:
            ev[2].record()
        if not self.fused_return:  # otherwise the owner's W2 epilogue stored the y2 rows at home
            _lib.check("b200moe_ep_return", L.b200moe_ep_return(pe.handle, st))
        _lib.check("b200moe_ep_combine_p2p", L.b200moe_ep_combine_p2p(
            pe.handle, st, ids.data_ptr(), w.data_ptr(), T, k, self.num_experts, self.owner.data_ptr(),
            _lib.ptr(residual), out.data_ptr()))
        if timed:
            ev[3].record()
        self._timed = timed
        self.last_routes_in = -1  # on the device: read by local_experts_used()
        return out

    def received(self) -> np.ndarray:
        """Expert ids of the routes this rank's experts ran in the last forward (host sync)."""
        if self.exchange == "p2p":
            return self._peer.received()
        R = self.last_routes_in
        return (self.recv_eid if self.world > 1 else self.send_eid)[:R].cpu().numpy()

    def local_experts_used(self) -> int:
        """Distinct local experts the last forward ran (host sync)."""
        return int(np.unique(self.received()).size)

    def comm_ms(self) -> float:
        """Exchange time of the last forward (NCCL: counts + rows + ids out, y2
        back; p2p: push, the owner's route-plan launch that waits for every
        rank's push, return + combine; waits for the slower ranks included);
        waits for those events."""
        if not self._timed:
            return 0.0
        ev = self._ev
        ev[3].synchronize()
        t = ev[0].elapsed_time(ev[1]) + ev[2].elapsed_time(ev[3])
        pe = self._last_plan_events
        if self.exchange == "p2p" and len(pe) >= 3:
            t += pe[1].elapsed_time(pe[2])
        return t

    def check_errors(self) -> None:
        """Synchronize; raise if the dispatch (a route id without an owner), the
        exchange (a wait that ran out) or the local layer recorded an error
        since the last check."""
        bits = int(self.err.item())
        if bits:
            self.err.zero_()
        status = self._peer.check() if self._peer is not None else 0
        self.layer.check_errors()
        if bits:
            raise _lib.B200MoeError("expert-parallel dispatch", 5)
        _lib.check("expert-parallel exchange", status)

    def close(self) -> None:
        """Free the layer and the exchange; a collective (every rank must call it)."""
        if self._peer is not None and self._own_peer:
            self._peer.close()
        self._peer = None
        self.layer.close()
