"""Expert-parallel routed-MoE layer over NCCL (NVLink / NVSwitch).

The reference keeps every expert on every TP rank and refuses expert
parallelism (engine/patches/gguf_moe.patch:57-58); its tier placement
(engine/.../experts/nvfp4_8r_tiers.py) becomes ownership here: rank r owns the
contiguous expert ids ``tiers.owner_ranges(E, world)[r]``, in either format.

One forward (per rank: its own T tokens, all ranks call in the same order):
  1. ``b200moe_ep_dispatch``: stable sort of the T*k routes by owner rank,
     per-rank counts, fp16 row + expert id + sorted position per route;
  2. counts exchange (one host sync), then NCCL all-to-all of rows and ids;
  3. the owner runs its experts on the received routes with k = 1 and weight
     1.0, which yields exactly the fp16 y2 rows, and all-to-all returns them;
  4. ``b200moe_ep_combine``: slot-order sum of fma(y2, w) per token (the
     single-GPU combine's arithmetic) plus the residual.
Communication is timed with CUDA events on the launching stream
(``comm_ms()``: the exposed, non-overlapped exchange time of the last call).
"""

from __future__ import annotations

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


def check_placement(tier, world: int, group=None) -> str:
    """Every rank must hold the same tier array and world size; a rank that
    differs makes every rank raise (the reference's stage digest check,
    engine/.../experts/nvfp4_8r_native.py:1657-1659)."""
    digest = tiersmod.placement_digest(tier, world)
    if world == 1 or not dist.is_initialized():
        return digest
    digests = [None] * world
    dist.all_gather_object(digests, digest, group=group)
    if len(set(digests)) != 1:
        raise RuntimeError(f"expert placement differs across ranks: {sorted(set(d[:12] for d in digests))}")
    return digest


def owner_of_expert(num_experts: int, world: int) -> np.ndarray:
    out = np.empty(num_experts, np.int32)
    for r, rng in enumerate(tiersmod.owner_ranges(num_experts, world)):
        out[rng.start:rng.stop] = r
    return out


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


class ExpertParallelMoe:
    """One routed-MoE layer with its experts sharded over a process group.

    ``tokens`` bounds the tokens one rank passes per forward.  Local experts
    run with the skinny kernels (a rank sees few routes per expert at decode).
    With ``split_k`` fixed here and on a single-GPU layer, the outputs of the
    two are bit-equal (same per-route rows, same slot-order combine)."""

    def __init__(self, *, hidden: int, inter: int, num_experts: int, top_k: int, tokens: int, tier,
                 fp4_format: str = "nvfp4", group=None, device: torch.device | None = None,
                 split_k: tuple[int, int] | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.tier = tiersmod.check_tier_array(tier, num_experts)
        self.digest = check_placement(self.tier, self.world, group)
        self.hidden, self.inter, self.num_experts, self.top_k, self.tokens = hidden, inter, num_experts, top_k, tokens
        S = tokens * top_k
        r_max = S * self.world  # every route of every rank could land here
        self.layer = B200NativeMoe(hidden=hidden, inter=inter, num_experts=num_experts, top_k=1,
                                   max_tokens=min(64, r_max), max_prefill_tokens=r_max, tier=self.tier,
                                   fp4_format=fp4_format, device=dev, rank=self.rank, world=self.world,
                                   prefill_gemm="skinny")
        if split_k is not None:
            self.layer.set_split_k(*split_k)
        self.owner = torch.from_numpy(owner_of_expert(num_experts, self.world)).to(dev)
        f16 = dict(dtype=torch.float16, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
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
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        self._timed = False
        self.last_routes_in = 0

    # weights go to the local layer (slots = this rank's experts of each format, ascending id)
    def load_fp4(self, *args, **kw):
        self.layer.load_fp4(*args, **kw)

    def load_iq2(self, *args, **kw):
        self.layer.load_iq2(*args, **kw)

    def set_iq2_tables(self, *args, **kw):
        self.layer.set_iq2_tables(*args, **kw)

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
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=self.device)
        _lib.check("b200moe_ep_combine", L.b200moe_ep_combine(
            _stream(), y2.data_ptr(), self.route_pos.data_ptr(), w.data_ptr(), T, k, self.hidden,
            _lib.ptr(residual), out.data_ptr()))
        self._timed = self.world > 1
        return out

    def local_experts_used(self) -> int:
        """Distinct local experts the last forward ran (host sync)."""
        if self.last_routes_in == 0:
            return 0
        eid = (self.recv_eid if self.world > 1 else self.send_eid)[:self.last_routes_in]
        return int(torch.unique(eid).numel())

    def comm_ms(self) -> float:
        """Exchange time (counts + rows + ids out, y2 back) of the last forward;
        waits for those events."""
        if not self._timed:
            return 0.0
        ev = self._ev
        ev[3].synchronize()
        return ev[0].elapsed_time(ev[1]) + ev[2].elapsed_time(ev[3])

    def check_errors(self) -> None:
        """Synchronize; raise if the dispatch (a route id without an owner) or
        the local layer recorded an error since the last check."""
        bits = int(self.err.item())
        if bits:
            self.err.zero_()
        self.layer.check_errors()
        if bits:
            raise _lib.B200MoeError("expert-parallel dispatch", 5)

    def close(self) -> None:
        self.layer.close()
