"""Tier map -> bank slot maps (host logic).

Mirrors the reference's tier model (engine/.../experts/nvfp4_8r_tiers.py:48-51,
169-179): one tier per expert, slots are ranks in ascending expert id.  On B200
every expert is HBM-resident, so the tiers are formats, not places:

  HOT   FP4 record (NVFP4 or MXFP4)   -> bank 0
  WARM  IQ2_XXS record                -> bank 1
  HOST  refused: nothing is host-resident on a 180 GB B200

Under expert parallelism the tier array is also split by owner: expert e
lives on GPU ``owner_of(e)`` (contiguous id ranges, even split) and a GPU's
maps hold only its own experts.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

HOT, WARM, HOST = 0, 1, 2


def check_tier_array(tier, num_experts: int | None = None) -> np.ndarray:
    t = np.asarray(tier)
    if t.dtype != np.int8 or t.ndim != 1 or (num_experts is not None and t.size != num_experts):
        raise ValueError(f"a tier array is int8 [{num_experts or 'E'}] of HOT/WARM/HOST")
    if np.any((t < 0) | (t > 2)):
        raise ValueError("tier values must be HOT (0), WARM (1) or HOST (2)")
    return t


@dataclass(frozen=True)
class SlotMaps:
    """int32 [E] slot of each expert per bank, -1 where absent (ascending-id ranks)."""

    hot: np.ndarray
    cold: np.ndarray
    host: np.ndarray
    iq: np.ndarray


def slot_maps(tier) -> SlotMaps:
    tier = check_tier_array(tier)

    def ranks(mask):
        out = np.full(tier.size, -1, np.int32)
        out[mask] = np.arange(int(mask.sum()), dtype=np.int32)
        return out

    cold = ranks(tier != HOT)
    return SlotMaps(ranks(tier == HOT), cold, np.where(tier == HOST, cold, -1).astype(np.int32),
                    ranks(tier == WARM))


def owner_ranges(num_experts: int, world: int) -> list[range]:
    """Expert ids of each GPU: contiguous, as even as possible (id order)."""
    if world < 1 or num_experts < world:
        raise ValueError(f"cannot split {num_experts} experts over {world} GPUs")
    base, extra = divmod(num_experts, world)
    out, lo = [], 0
    for g in range(world):
        n = base + (1 if g < extra else 0)
        out.append(range(lo, lo + n))
        lo += n
    return out


def local_maps(tier, rank: int, world: int) -> tuple[np.ndarray, np.ndarray]:
    """(fp4 slot map, iq2 slot map) of one GPU: slots rank that GPU's experts
    of each format in ascending id; every other expert maps to -1."""
    tier = check_tier_array(tier)
    if np.any(tier == HOST):
        raise ValueError("HOST tier: every expert is HBM-resident on B200 (HOT = FP4, WARM = IQ2)")
    own = np.zeros(tier.size, bool)
    own[owner_ranges(tier.size, world)[rank]] = True
    fp4 = np.full(tier.size, -1, np.int32)
    iq2 = np.full(tier.size, -1, np.int32)
    m = own & (tier == HOT)
    fp4[m] = np.arange(int(m.sum()), dtype=np.int32)
    m = own & (tier == WARM)
    iq2[m] = np.arange(int(m.sum()), dtype=np.int32)
    return fp4, iq2


def placement_digest(tier, world: int) -> str:
    """sha256 of (tier array, world size): every EP rank must hold the same
    placement (the reference checks a per-stage digest on all ranks,
    engine/.../experts/nvfp4_8r_native.py:1657-1659)."""
    tier = check_tier_array(tier)
    h = hashlib.sha256()
    h.update(np.asarray(tier, np.int8).tobytes())
    h.update(int(world).to_bytes(4, "little"))
    return h.hexdigest()


def zipf_tier(num_experts: int, n_hot: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """A seeded tier map: a permutation (seed) of expert ids ranked by Zipf
    popularity; the n_hot most popular are HOT, the rest WARM.  Returns
    (tier int8 [E], rank int32 [E] = popularity rank of each expert)."""
    rng = np.random.default_rng(seed)
    order = rng.permutation(num_experts)  # order[r] = expert of popularity rank r
    rank = np.empty(num_experts, np.int32)
    rank[order] = np.arange(num_experts, dtype=np.int32)
    tier = np.where(rank < n_hot, HOT, WARM).astype(np.int8)
    return tier, rank
