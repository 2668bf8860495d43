"""Tiers of routed experts: slot maps, placement, the tier planner and tier-map files (host logic).

Mirrors the reference's tier model (engine/.../experts/nvfp4_8r_tiers.py): one
tier per expert, slots are ranks in ascending expert id.  On B200 every expert
is HBM-resident, so the tiers are formats, not places:

  HOT   FP4 record (NVFP4 or MXFP4)   -> bank 0
  WARM  IQ2_XXS record                -> bank 1
  HOST  refused by the layers: nothing is host-resident on a 180 GB B200

Under expert parallelism the tier array is also split by owner: expert e lives
on GPU ``owner[e]`` (contiguous id ranges by default, or a placement from
``balanced_owners``) and a GPU's maps hold only its own experts.

The planner (``choose_tiers``, ``TierPlan``) and the tier-map reader
(``parse_tier_map``, ``plan_from_map``) follow the reference's rules and its
errors (ValueError at the first inconsistency).  The HBM cost of a tier is a
parameter: the reference's per-TP-rank record sizes by default, this library's
per-expert slot sizes (``slot_bytes``) for a B200 plan.  Pure numpy.
"""

from __future__ import annotations

import enum
import hashlib
import json
import math
from collections.abc import Mapping
from dataclasses import dataclass
from fractions import Fraction
from functools import cached_property
from pathlib import Path

import numpy as np

HOT, WARM, HOST = 0, 1, 2


class Tier(enum.IntEnum):
    HOT = 0
    WARM = 1
    HOST = 2


NUM_EXPERTS = 384
# One reference native record (MXFP4, one TP4 rank of one expert, W2 K padded
# to 640): engine/.../experts/nvfp4_8r_native.py:59-75.
REF_RECORD_BYTES = 4_874_240
# Bytes of one 256-weight block per GGML type (nvfp4_8r_tiers.py:35).
IQ_BLOCK_BYTES = {29: 56, 16: 66, 17: 74}  # IQ1_M, IQ2_XXS, IQ2_XS


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


# ---------------------------------------------------------------- placement
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


def owner_by_range(num_experts: int, world: int) -> np.ndarray:
    """int32 [E] owner of each expert under the contiguous split."""
    out = np.empty(num_experts, np.int32)
    for r, rng in enumerate(owner_ranges(num_experts, world)):
        out[rng.start:rng.stop] = r
    return out


def check_owner(owner, num_experts: int, world: int) -> np.ndarray:
    o = np.asarray(owner)
    if o.dtype != np.int32 or o.shape != (num_experts,) or np.any((o < 0) | (o >= world)):
        raise ValueError(f"an owner map is int32 [{num_experts}] of ranks in 0..{world - 1}")
    if np.unique(o).size != world:
        raise ValueError("every rank must own at least one expert")
    return o


def balanced_owners(tier, world: int, counts=None) -> np.ndarray:
    """A placement that balances HBM bytes and expected routes per GPU.

    Each format is dealt separately.  Its experts, by expected routes
    (``counts``, int [E]) descending with ties by ascending id (id order when
    no counts are given), each go to the rank with the fewest routes so far
    (ties: the rank earlier in the format's rank order) among the ranks with
    room left, a rank having room for floor or ceil(n / W) experts of the
    format.  So every GPU holds equal bytes of each format within one expert,
    and the routes even out unless one expert alone outweighs a GPU's share.
    The FP4 experts' rank order is 0..W-1; the IQ2 experts' puts the ranks
    short of an FP4 expert first, so expert counts per GPU differ by at most
    one as well.  Returns int32 [E]; deterministic, so every rank computes the
    same map (``placement_digest`` checks it)."""
    tier = check_tier_array(tier)
    if np.any(tier == HOST):
        raise ValueError("HOST tier: every expert is HBM-resident on B200 (HOT = FP4, WARM = IQ2)")
    E = tier.size
    if world < 1 or E < world:
        raise ValueError(f"cannot split {E} experts over {world} GPUs")
    if counts is None:
        c = np.zeros(E, np.int64)
    else:
        c = np.asarray(counts)
        if c.shape != (E,) or c.dtype.kind not in "iu" or np.any(c < 0):
            raise ValueError(f"expected routes are non-negative integers [{E}]")
        c = c.astype(np.int64)
    owner = np.full(E, -1, np.int32)
    routes = np.zeros(world, np.int64)
    order_ranks = np.arange(world)
    for t in (HOT, WARM):
        ids = np.nonzero(tier == t)[0]
        base, extra = divmod(ids.size, world)
        room = np.full(world, base, np.int64)
        room[order_ranks[:extra]] += 1
        pos = np.empty(world, np.int64)
        pos[order_ranks] = np.arange(world)  # a rank's place in this format's order
        for e in ids[np.lexsort((ids, -c[ids]))]:
            open_ranks = np.nonzero(room > 0)[0]
            r = open_ranks[np.lexsort((pos[open_ranks], routes[open_ranks]))[0]]
            owner[e] = r
            routes[r] += c[e]
            room[r] -= 1
        n_fp4 = np.bincount(owner[(owner >= 0) & (tier == HOT)], minlength=world)
        order_ranks = np.lexsort((np.arange(world), n_fp4))
    if np.unique(owner).size != world:
        raise ValueError(f"{E} experts leave a rank of {world} without an expert")
    return owner


def local_maps(tier, rank: int, world: int, owner=None) -> tuple[np.ndarray, np.ndarray]:
    """(fp4 slot map, iq2 slot map) of one GPU: slots rank that GPU's experts
    of each format in ascending id; every other expert maps to -1.  ``owner``
    (int32 [E]) places the experts; by default contiguous id ranges."""
    tier = check_tier_array(tier)
    if np.any(tier == HOST):
        raise ValueError("HOST tier: every expert is HBM-resident on B200 (HOT = FP4, WARM = IQ2)")
    if owner is None:
        own = np.zeros(tier.size, bool)
        own[owner_ranges(tier.size, world)[rank]] = True
    else:
        own = check_owner(owner, tier.size, world) == rank
    fp4 = np.full(tier.size, -1, np.int32)
    iq2 = np.full(tier.size, -1, np.int32)
    m = own & (tier == HOT)
    fp4[m] = np.arange(int(m.sum()), dtype=np.int32)
    m = own & (tier == WARM)
    iq2[m] = np.arange(int(m.sum()), dtype=np.int32)
    return fp4, iq2


def placement_digest(tier, world: int, owner=None) -> str:
    """sha256 of (tier array, world size[, owner map]): every EP rank must
    hold the same placement (the reference checks a per-stage digest on all
    ranks, engine/.../experts/nvfp4_8r_native.py:1657-1659)."""
    tier = check_tier_array(tier)
    h = hashlib.sha256()
    h.update(np.asarray(tier, np.int8).tobytes())
    h.update(int(world).to_bytes(4, "little"))
    if owner is not None:
        h.update(check_owner(owner, tier.size, world).tobytes())
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


# ---------------------------------------------------------------- record sizes
def iq_record_bytes(type13: int, type2: int, hidden: int = 5120, inter: int = 2304, tp: int = 4) -> int:
    """HBM bytes of one expert's IQ record on one of ``tp`` ranks: gate and up
    of ``type13``, down of ``type2``, each projection inter x hidden / (256 tp)
    blocks (the reference's TP4 slice: 11,520 blocks, nvfp4_8r_tiers.py:36-40,
    137-142).  ``tp = 1`` gives a whole expert, as a B200 layer holds it."""
    for t in (type13, type2):
        if t not in IQ_BLOCK_BYTES:
            raise ValueError(f"routed-expert GGML type {t!r} is not IQ1_M/IQ2_XXS/IQ2_XS")
    blocks, rem = divmod(hidden * inter, 256 * tp)
    if rem or blocks <= 0:
        raise ValueError(f"hidden x inter = {hidden} x {inter} is not whole 256-blocks over {tp} ranks")
    return blocks * (2 * IQ_BLOCK_BYTES[type13] + IQ_BLOCK_BYTES[type2])


def slot_bytes(fmt: str, hidden: int, inter: int, block_scaled: bool = False) -> int:
    """HBM bytes one expert slot takes in this library's banks: NVFP4 codes +
    E4M3 per 16 (+ 3 fp32 globals); MXFP4 codes + E8M0 per 32 (the block-scaled
    layout, ``prefill_gemm="fp4"``, keeps one scale byte per 16 weights for
    either format); IQ2_XXS 66 bytes per 256 weights."""
    w = 3 * hidden * inter
    if fmt == "nvfp4":
        return w // 2 + w // 16 + 12
    if fmt == "mxfp4":
        return w // 2 + (w // 16 if block_scaled else w // 32)
    if fmt == "iq2_xxs":
        return w // 256 * 66
    raise ValueError(f"no slot format {fmt!r} (nvfp4, mxfp4, iq2_xxs)")


# ---------------------------------------------------------------- residency
RESIDENCY_KEY = "nvfp4_8r_residency"
HOST_SHARE_KEY = "nvfp4_8r_host_route_share"
MAX_HOST_ROUTE_SHARE = 0.05
TIER_MAP_FORMAT = "nvfp4-8r-tier-map-v1"


@dataclass(frozen=True)
class TwoTier:
    """HOT experts in HBM, the rest host-resident (no tier plan)."""


@dataclass(frozen=True)
class HotIq:
    """HOT and WARM only: the B200 residency."""


@dataclass(frozen=True)
class HotIqHost:
    """HOT, WARM and a HOST tier of at most ``route_share`` of the stage's
    routes (0.0: exactly the experts never routed to)."""

    route_share: float

    def __post_init__(self) -> None:
        s = self.route_share
        if type(s) is not float or not math.isfinite(s) or not 0.0 <= s <= MAX_HOST_ROUTE_SHARE:
            raise ValueError(f"{HOST_SHARE_KEY} must be a float in [0, {MAX_HOST_ROUTE_SHARE}], got {s!r}")


def parse_residency(extra: Mapping[str, object]):
    """The residency of a loader config mapping; no defaults (the reference's
    keys and rules, nvfp4_8r_tiers.py:115-135)."""
    if RESIDENCY_KEY not in extra:
        raise ValueError(f"{RESIDENCY_KEY} is required (two_tier, hot_iq or hot_iq_host)")
    name = extra[RESIDENCY_KEY]
    if name == "hot_iq_host":
        if HOST_SHARE_KEY not in extra:
            raise ValueError(f"{RESIDENCY_KEY} hot_iq_host needs {HOST_SHARE_KEY}")
        share = extra[HOST_SHARE_KEY]
        return HotIqHost(float(share) if type(share) is int else share)  # a YAML 0 reads as int
    if name not in ("two_tier", "hot_iq"):
        raise ValueError(f"{RESIDENCY_KEY} must be two_tier, hot_iq or hot_iq_host, got {name!r}")
    if HOST_SHARE_KEY in extra:
        raise ValueError(f"{HOST_SHARE_KEY} is only valid with {RESIDENCY_KEY} hot_iq_host")
    return TwoTier() if name == "two_tier" else HotIq()


# ---------------------------------------------------------------- tier plan
def stage_digest(arrays: Mapping[int, np.ndarray], layers: range) -> str:
    """sha256 of the tier arrays (int8 bytes) in layer order."""
    h = hashlib.sha256()
    for layer in layers:
        h.update(np.asarray(arrays[layer], np.int8).tobytes())
    return h.hexdigest()


def _stage_tier_array(tier, where: str, num_experts: int) -> np.ndarray:
    if (not isinstance(tier, np.ndarray) or tier.dtype != np.int8 or tier.shape != (num_experts,)
            or bool(((tier < 0) | (tier > 2)).any())):
        raise ValueError(f"{where}: a tier array is int8 [{num_experts}] of Tier values")
    return tier


@dataclass(frozen=True, eq=False)
class TierPlan:
    """The tiers of one stage's layers under a HBM budget (nvfp4_8r_tiers.py:182-243).

    ``native_bytes`` is what a HOT expert costs (the reference's TP-rank
    record by default; ``slot_bytes`` for a B200 layer), ``iq_bytes[layer]``
    what a WARM one costs.  ``hbm_bytes`` and ``digest`` derive from the
    arrays.  Every layer holds a HOT and a WARM expert; HotIq holds no HOST."""

    layers: range
    tiers: dict
    iq_bytes: dict
    budget_bytes: int
    residency: object
    native_bytes: int = REF_RECORD_BYTES
    num_experts: int = NUM_EXPERTS

    def __post_init__(self) -> None:
        if not isinstance(self.residency, (HotIq, HotIqHost)):
            raise ValueError(f"a tier plan needs a WARM tier, got {self.residency!r}")
        if self.layers.step != 1 or len(self.layers) == 0:
            raise ValueError(f"stage layers must be a contiguous run, got {self.layers}")
        want = list(self.layers)
        if sorted(self.tiers) != want or sorted(self.iq_bytes) != want:
            raise ValueError(f"tier plan must cover exactly layers {self.layers}")
        frozen = {}
        for layer in self.layers:
            t = _stage_tier_array(self.tiers[layer], f"layer {layer}", self.num_experts).copy()
            t.setflags(write=False)
            frozen[layer] = t
            iq = self.iq_bytes[layer]
            if type(iq) is not int or not 0 < iq < self.native_bytes:
                raise ValueError(f"layer {layer}: IQ record bytes {iq!r}")
            if not bool((t == HOT).any()):
                raise ValueError(f"layer {layer} has no HOT expert: the budget is too small")
            if not bool((t == WARM).any()):
                raise ValueError(f"layer {layer} has no WARM expert")
            if isinstance(self.residency, HotIq) and bool((t == HOST).any()):
                raise ValueError(f"layer {layer}: a hot_iq plan holds a HOST expert")
        object.__setattr__(self, "tiers", frozen)
        object.__setattr__(self, "iq_bytes", dict(self.iq_bytes))
        if self.hbm_bytes > self.budget_bytes:
            raise ValueError(f"tier plan uses {self.hbm_bytes} bytes of HBM, budget {self.budget_bytes}")

    @cached_property
    def hbm_bytes(self) -> int:
        return sum(int((self.tiers[l] == HOT).sum()) * self.native_bytes
                   + int((self.tiers[l] == WARM).sum()) * self.iq_bytes[l] for l in self.layers)

    @cached_property
    def digest(self) -> str:
        return stage_digest(self.tiers, self.layers)

    def count(self, tier: int) -> int:
        return sum(int((self.tiers[l] == tier).sum()) for l in self.layers)


def choose_tiers(counts: np.ndarray, layers: range, iq_bytes: Mapping[int, int], budget_bytes: int, residency,
                 native_bytes: int = REF_RECORD_BYTES) -> TierPlan:
    """Tiers of one stage from a decode tally (int [layers, E]) and a HBM budget.

    The reference's rule (nvfp4_8r_tiers.py:246-305):
    1. HOST (HotIqHost(s) only): the longest prefix of the stage's experts in
       ascending (count, layer, expert) whose summed count is at most s x the
       stage's total (s = 0: exactly the zero-count experts).
    2. Every other expert starts WARM; the budget must hold their IQ records.
    3. WARM experts become HOT in descending count / (native - IQ bytes), ties
       by ascending (layer, expert), while the next one fits; the walk stops
       at the first that does not.
    Here both walks are prefix searches over exact integer sums."""
    if not isinstance(residency, (HotIq, HotIqHost)):
        raise ValueError(f"choose_tiers needs a residency with a WARM tier, got {residency!r}")
    counts = np.asarray(counts)
    if counts.ndim != 2 or counts.dtype.kind not in "iu":
        raise ValueError("decode tally must be integer [layers, experts]")
    E = counts.shape[1]
    if layers.step != 1 or len(layers) == 0 or layers.start < 0 or layers.stop > counts.shape[0]:
        raise ValueError(f"stage layers {layers} are not a run inside the tally")
    if sorted(iq_bytes) != list(layers):
        raise ValueError(f"IQ record bytes must cover exactly layers {layers}")
    stage = counts[layers.start:layers.stop].astype(np.int64)
    if bool((stage < 0).any()):
        raise ValueError("decode tally has a negative count")
    L = len(layers)
    flat = stage.reshape(-1)  # index = layer offset * E + expert: (layer, expert) order
    tier = np.full(L * E, WARM, np.int8)
    if isinstance(residency, HotIqHost):
        asc = np.argsort(flat, kind="stable")  # ascending count, ties in (layer, expert) order
        run = np.cumsum(flat[asc])
        num, den = Fraction(residency.route_share).as_integer_ratio()
        cap = (num * int(flat.sum())) // den  # running <= share x total <=> running <= floor(...)
        tier[asc[:int(np.searchsorted(run, cap, side="right"))]] = HOST
    iqb = np.array([iq_bytes[l] for l in layers], dtype=object)
    warm_per_layer = (tier.reshape(L, E) == WARM).sum(axis=1)
    need = sum(int(n) * int(b) for n, b in zip(warm_per_layer, iqb))
    if need > budget_bytes:
        raise ValueError(f"budget {budget_bytes} cannot hold the IQ tier of layers "
                         f"{layers.start}-{layers.stop - 1} ({need} bytes)")
    cost = [native_bytes - int(b) for b in iqb]
    if any(c <= 0 for c in cost):
        raise ValueError("an IQ record is not smaller than a native record")
    cand = np.nonzero(tier == WARM)[0]
    order = sorted(cand.tolist(), key=lambda i: (-Fraction(int(flat[i]), cost[i // E]), i))
    spend = np.cumsum([cost[i // E] for i in order], dtype=np.int64) if order else np.zeros(0, np.int64)
    n_promote = int(np.searchsorted(spend, budget_bytes - need, side="right"))
    tier[np.asarray(order[:n_promote], dtype=np.int64)] = HOT
    arrays = {l: tier[j * E:(j + 1) * E].copy() for j, l in enumerate(layers)}
    return TierPlan(layers, arrays, dict(iq_bytes), budget_bytes, residency, native_bytes, E)


# ---------------------------------------------------------------- tier-map file
@dataclass(frozen=True, eq=False)
class TierMap:
    """HOT / WARM of every routed expert from a tier-map file (no HOST tier,
    no counts).  ``stages`` maps a stage's first layer to (its layers, the
    sha256 its tier arrays must give)."""

    tiers: dict
    stages: dict

    def stage(self, layers: range) -> dict:
        if layers.start not in self.stages or self.stages[layers.start][0] != layers:
            have = [(r.start, r.stop - 1) for r, _ in self.stages.values()]
            raise ValueError(f"the tier map has no stage of layers {layers.start}-{layers.stop - 1} "
                             f"(has {have}): it was made for another pipeline split")
        return {l: self.tiers[l] for l in layers}


def _ints(*vals) -> bool:
    return all(type(v) is int for v in vals)


def parse_tier_map(doc: object, num_experts: int = NUM_EXPERTS) -> TierMap:
    """A tier-map document (format ``nvfp4-8r-tier-map-v1``), checked whole
    with the reference's rules (nvfp4_8r_tiers.py:332-396): exact keys, HOT
    ids distinct ascending and neither none nor all per layer, stages
    contiguous from layer 0, each stage's sha256 and stated counts equal to
    what its HOT ids give."""
    keys = {"format", "comment", "num_layers", "num_experts", "stages", "hot"}
    if not isinstance(doc, dict) or set(doc) != keys:
        got = sorted(doc) if isinstance(doc, dict) else type(doc).__name__
        raise ValueError(f"a tier map has exactly the keys {sorted(keys)}, got {got}")
    if doc["format"] != TIER_MAP_FORMAT:
        raise ValueError(f"tier map format {doc['format']!r}, want {TIER_MAP_FORMAT!r}")
    n, hot = doc["num_layers"], doc["hot"]
    if doc["num_experts"] != num_experts or type(n) is not int or n < 1:
        raise ValueError(f"tier map is for {doc['num_experts']!r} experts x {n!r} layers")
    if not isinstance(hot, list) or len(hot) != n:
        raise ValueError(f"tier map 'hot' must list {n} layers")
    tiers: dict[int, np.ndarray] = {}
    for layer, ids in enumerate(hot):
        ok = isinstance(ids, list) and len(ids) > 0 and all(type(e) is int for e in ids)
        ok = ok and all(a < b for a, b in zip(ids, ids[1:])) and ids[0] >= 0 and ids[-1] < num_experts
        if not ok or len(ids) == num_experts:
            raise ValueError(f"tier map layer {layer}: HOT ids must be distinct ascending ints in "
                             f"0..{num_experts - 1}, at least one and not all (a layer needs a WARM expert)")
        t = np.full(num_experts, WARM, np.int8)
        t[ids] = HOT
        t.setflags(write=False)
        tiers[layer] = t
    stages: dict[int, tuple[range, str]] = {}
    next_layer = 0
    entries = doc["stages"] if isinstance(doc["stages"], list) else [None]
    for s in entries:
        fields = {"first_layer", "last_layer", "hot", "compressed", "digest"}
        if (not isinstance(s, dict) or set(s) != fields
                or not _ints(s["first_layer"], s["last_layer"], s["hot"], s["compressed"])):
            raise ValueError(f"tier map stage entry {s!r}")
        layers = range(s["first_layer"], s["last_layer"] + 1)
        if len(layers) == 0 or layers.start != next_layer:
            raise ValueError(f"tier map stages must be contiguous from layer 0, got {s!r}")
        next_layer = layers.stop
        digest = s["digest"]
        if type(digest) is not str or len(digest) != 64:
            raise ValueError(f"tier map stage {layers.start}: digest must be a sha256 hex")
        got = stage_digest(tiers, layers) if layers.stop <= n else None
        if got != digest:
            raise ValueError(f"tier map stage {layers.start}-{layers.stop - 1}: its tiers give digest "
                             f"{(got or 'none')[:12]}, the file says {digest[:12]}")
        n_hot = sum(int((tiers[l] == HOT).sum()) for l in layers)
        if (s["hot"], s["compressed"]) != (n_hot, len(layers) * num_experts - n_hot):
            raise ValueError(f"tier map stage {layers.start}: stated counts disagree with its HOT ids")
        stages[layers.start] = (layers, digest)
    if next_layer != n:
        raise ValueError(f"tier map stages cover layers 0..{next_layer - 1}, want 0..{n - 1}")
    return TierMap(tiers, stages)


def load_tier_map(path, num_experts: int = NUM_EXPERTS) -> TierMap:
    return parse_tier_map(json.loads(Path(path).read_text()), num_experts)


def tier_map_document(arrays: Mapping[int, np.ndarray], stage_layers: list[range], comment: str = "") -> dict:
    """The tier-map document of HOT / WARM arrays (layer -> int8 [E]) split
    into the given stages: what ``parse_tier_map`` reads back."""
    n = len(arrays)
    if sorted(arrays) != list(range(n)):
        raise ValueError("tier arrays must cover layers 0..n-1")
    E = None
    hot = []
    for l in range(n):
        t = check_tier_array(arrays[l])
        E = t.size if E is None else E
        if t.size != E or np.any(t == HOST):
            raise ValueError(f"layer {l}: a tier map holds HOT / WARM arrays of one size")
        hot.append(np.nonzero(t == HOT)[0].astype(int).tolist())
    stages = []
    for r in stage_layers:
        n_hot = sum(len(hot[l]) for l in r)
        stages.append({"first_layer": r.start, "last_layer": r.stop - 1, "hot": n_hot,
                       "compressed": len(r) * E - n_hot, "digest": stage_digest(arrays, r)})
    return {"format": TIER_MAP_FORMAT, "comment": comment, "num_layers": n, "num_experts": E,
            "stages": stages, "hot": hot}


def plan_from_map(tier_map: TierMap, layers: range, iq_bytes: Mapping[int, int], budget_bytes: int, residency,
                  native_bytes: int = REF_RECORD_BYTES) -> TierPlan:
    """A stage's plan from a fixed tier map (nvfp4_8r_tiers.py:403-431): only
    hot_iq, only a stage the map holds, and only within the budget (the map's
    tiers or nothing); the plan's digest equals the map's."""
    if not isinstance(residency, HotIq):
        raise ValueError(f"a tier map serves {RESIDENCY_KEY} hot_iq only, got {residency!r}")
    arrays = tier_map.stage(layers)
    need = sum(int((arrays[l] == HOT).sum()) * native_bytes + int((arrays[l] == WARM).sum()) * iq_bytes[l]
               for l in layers)
    if need > budget_bytes:
        raise ValueError(f"the tier map's records of layers {layers.start}-{layers.stop - 1} need {need} bytes "
                         f"({need / 2**30:.4f} GiB) per GPU; the budget is {budget_bytes} bytes "
                         f"({budget_bytes / 2**30:.4f} GiB)")
    E = next(iter(arrays.values())).size
    plan = TierPlan(layers, arrays, dict(iq_bytes), budget_bytes, residency, native_bytes, E)
    if plan.digest != tier_map.stages[layers.start][1]:
        raise ValueError("the stage's plan digest differs from the tier map's")
    return plan


def hbm_budget(device, reserve_bytes: int = 0, workspace_bytes: int = 0) -> int:
    """Bytes of expert records a plan may place on ``device``: its free HBM
    now, less a reserve and the layers' workspaces (as the reference sizes a
    stage's budget, engine/.../experts/nvfp4_8r_native.py:1577-1611)."""
    import torch

    free, _ = torch.cuda.mem_get_info(device)
    budget = int(free) - int(reserve_bytes) - int(workspace_bytes)
    if budget <= 0:
        raise ValueError(f"{free} bytes free cannot hold a reserve of {reserve_bytes} and "
                         f"workspaces of {workspace_bytes}")
    return budget
