"""Decode route counters of a layer, counted on the device.

Mirrors the reference's RouteStats (engine/src/vllm/model_executor/layers/
fused_moe/experts/nvfp4_8r_stats.py:65-110): device tensors updated only by
device work (here one launch of ``b200moe_route_stats`` per call), so a
captured decode graph keeps counting at every replay.  Per layer:

  stat       int64 [5]    calls, routes, HOST routes, distinct HOST experts
                          per call (summed), WARM routes
  gap_hist   int64 [7]    HOST routes by rounds since their expert's last HOST
                          use: <= 1, 2, <= 4, <= 16, <= 64, <= 256, more (or never)
  routes     int64 [E]    routes per expert
  last_round int32 [E+1]  the round of each expert's last HOST use

On B200 no expert is host-resident, so the HOST fields stay zero for the
layers of this library; the counters still take any tier array, and
``routes`` is the tally ``tiers.choose_tiers`` plans from.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from . import tiers as tiersmod

STAT_FIELDS = ("calls", "routes", "host_routes", "host_groups", "warm_routes")
GAP_EDGES = (1, 2, 4, 16, 64, 256)
RECENT = (4, 16, 64, 256)
NEVER = -(2**30)


class RouteStats:
    """The counters of one layer on one GPU; ``tier`` is its tier array."""

    def __init__(self, tier, device: torch.device) -> None:
        maps = tiersmod.slot_maps(tier)  # validates the array
        E = maps.hot.size
        self.num_experts = E
        self.device = device
        self.is_host = torch.from_numpy((maps.host >= 0).astype(np.uint8)).to(device)
        self.is_warm = torch.from_numpy((maps.iq >= 0).astype(np.uint8)).to(device)
        self.stat = torch.zeros(len(STAT_FIELDS), dtype=torch.int64, device=device)
        self.gap_hist = torch.zeros(len(GAP_EDGES) + 1, dtype=torch.int64, device=device)
        self.routes = torch.zeros(E, dtype=torch.int64, device=device)
        self.last_round = torch.full((E + 1,), NEVER, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def count(self, topk_ids: torch.Tensor) -> None:
        """One decode call's routes (int32 [M, k] on the layer's device): one
        launch on the current stream, no host sync (graph-capturable)."""
        if topk_ids.dtype != torch.int32 or topk_ids.device != self.device or not topk_ids.is_contiguous():
            raise ValueError("topk_ids must be a contiguous int32 tensor on the counters' device")
        _lib.check("b200moe_route_stats", _lib.lib().b200moe_route_stats(
            torch.cuda.current_stream(self.device).cuda_stream, topk_ids.data_ptr(), topk_ids.numel(),
            self.num_experts, self.is_host.data_ptr(), self.is_warm.data_ptr(), self.stat.data_ptr(),
            self.gap_hist.data_ptr(), self.routes.data_ptr(), self.last_round.data_ptr(), self.err.data_ptr()))

    def check_errors(self) -> None:
        """Raise (after a sync) if a call held an id outside the layer's experts."""
        if int(self.err.item()):
            self.err.zero_()
            raise RuntimeError("route counters: an expert id outside [0, num_experts)")

    def read(self) -> dict[str, np.ndarray]:
        """Host copies: stat, gap_hist, recent (experts whose last HOST use is
        within each RECENT window) and routes."""
        r = self.stat[0]
        age = r - self.last_round[: self.num_experts].long()
        recent = torch.stack([(age <= g).sum() for g in RECENT])
        return {"stat": self.stat.cpu().numpy(), "gap_hist": self.gap_hist.cpu().numpy(),
                "recent": recent.cpu().numpy(), "routes": self.routes.cpu().numpy()}

    def reset(self) -> None:
        self.stat.zero_()
        self.gap_hist.zero_()
        self.routes.zero_()
        self.last_round.fill_(NEVER)
