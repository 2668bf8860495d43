"""Seeded inputs of the golden fixtures.

Shared by ``make_golden.py`` (which runs the reference on them once) and the
tests (which regenerate them and run the oracle or the CUDA path on them).
Everything here is deterministic numpy; nothing reads the reference tree.
"""

from __future__ import annotations

import numpy as np

ROUTE_PLAN_SEED = 20261201
SAMPLE_ROWS = np.array([0, 1, 17, 511, 1024, 2047, 2303], np.int64)


def _e4m3_finite_bytes(rng, shape):
    b = rng.integers(0, 256, size=shape, dtype=np.uint8)
    nan = (b & 127) == 127
    b[nan] = b[nan] & 0xF7  # 0x7F -> 0x77: finite
    return b


def nvfp4_decode_inputs():
    """One w1 projection at the reference checkpoint geometry (2304 x 5120):
    random E2M1 codes, random finite E4M3 scales, a fixed global."""
    rng = np.random.default_rng(101)
    rows, cols = 2304, 5120
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = _e4m3_finite_bytes(rng, (rows, cols // 16))
    return codes, scales, np.float32(3.0517578e-05)


def mxfp4_decode_inputs():
    """A raw MXFP4 record section (codes then E8M0) for accept_p1.packed_projection."""
    rng = np.random.default_rng(102)
    rows, cols = 576, 5120
    codes = rng.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    scales = rng.integers(100, 140, size=rows * cols // 32, dtype=np.uint8)
    return np.concatenate([codes, scales]), rows, cols


def fold_inputs(foldable: bool):
    """A C0-shaped W13 projection [2816, 2048] in NVFP4.  Foldable: both
    16-halves of every 32-block share a power-of-two E4M3 scale, so the E8M0/32
    fold is exact.  Not foldable: one block pair gets scales 1.5 and 1.0."""
    rng = np.random.default_rng(103 if foldable else 104)
    rows, cols = 2816, 2048
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    # powers of two in E4M3: exponent field 1..14, mantissa 0 -> 2^(e-7)
    e = rng.integers(1, 15, size=(rows, cols // 32), dtype=np.uint8)
    bits = np.repeat((e << 3).astype(np.uint8), 2, axis=1)
    if not foldable:
        bits[5, 6] = (7 << 3) | 4  # 1.5
        bits[5, 7] = 7 << 3        # 1.0
        codes[5, 48:64] = 0x77     # every element of that 32-block is +-6 magnitude
    return codes, bits, np.float32(0.125)


def contribution_inputs():
    rng = np.random.default_rng(105)
    h, i = 96, 40
    w1 = rng.normal(0, 0.2, (i, h))
    w3 = rng.normal(0, 0.2, (i, h))
    w2 = rng.normal(0, 0.2, (h, i))
    x = rng.normal(0, 1, h).astype(np.float16)
    return w1, w3, w2, x, 0.37


SWIGLU_SPECIALS = np.array([0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E00, 0x4900, 0xC900, 0x4901, 0xC901,
                            0x7BFF, 0xFBFF, 0x0001, 0x8001, 0x0400, 0x8400], np.uint16)


def swiglu_inputs():
    """y13 fp16 [48, 2 * 576]: normal values times 4 with the fp16 specials
    (+-0, +-inf, NaN, +-10, +-10.0078, +-65504, smallest subnormal and normal)
    in the first columns of gate and up, rolled per row."""
    rng = np.random.default_rng(106)
    s, inter = 48, 576
    y = (rng.standard_normal((s, 2 * inter)) * 4).astype(np.float16)
    sp = SWIGLU_SPECIALS.view(np.float16)
    for r in range(s):
        y[r, : sp.size] = sp
        y[r, inter: inter + sp.size] = np.roll(sp, r)
    return y


def iq2_inputs():
    """Random valid IQ2_XXS blocks [64 rows, 8 blocks, 66 bytes]."""
    rng = np.random.default_rng(107)
    rows, nb = 64, 8
    out = rng.integers(0, 256, size=(rows, nb, 66), dtype=np.uint8)
    d = (0.02 / 48.0) * rng.uniform(0.5, 1.5, size=(rows, nb))
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return out


# ---------------------------------------------------------------- host readers and planner
# Tier planner tallies: 6 layers x 384 experts, heavy-tailed counts with about
# a third of the experts never routed to.
TIER_SEED = 20261202
TIER_LAYERS = 6
TIER_TYPES = [(16, 16), (29, 29), (17, 17), (17, 29), (16, 29), (29, 16)]  # (gate/up, down) per layer


def tier_tally() -> np.ndarray:
    rng = np.random.default_rng(TIER_SEED)
    c = np.floor(rng.pareto(1.1, size=(TIER_LAYERS, 384)) * 40).astype(np.int64)
    c[rng.random(size=c.shape) < 0.33] = 0
    return c


# Pack reader: a small geometry (the record's field order and padding rules at
# the reference's layout; 40 layers and 4 ranks as its manifests require).
PACK_SEED = 20261203
PACK_GEOM = dict(hidden=256, tp_inter=64, w2_k=96, tp_ranks=4, num_experts=12, num_layers=40)
PACK_LAYERS = (0, 7)


def pack_full_experts(layer: int):
    """Whole MXFP4 experts of one layer: (w13 codes, w13 scales, w2 codes, w2
    scales) with I = tp_ranks x tp_inter, E8M0 scales in 110..140."""
    g = PACK_GEOM
    rng = np.random.default_rng(PACK_SEED + layer)
    E, H, I = g["num_experts"], g["hidden"], g["tp_ranks"] * g["tp_inter"]
    w13c = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    w13s = rng.integers(110, 141, size=(E, 2 * I, H // 32), dtype=np.uint8)
    w2c = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    w2s = rng.integers(110, 141, size=(E, H, I // 32), dtype=np.uint8)
    return w13c, w13s, w2c, w2s


def pack_v1_split(layer: int, rank: int) -> dict:
    """A seeded hot / cold partition of the experts for the v1 pack."""
    rng = np.random.default_rng(PACK_SEED + 1000 * layer + rank)
    E = PACK_GEOM["num_experts"]
    hot = np.sort(rng.permutation(E)[: E // 2 + rank]).tolist()
    return {"hot": [int(e) for e in hot], "cold": [e for e in range(E) if e not in hot]}


def residency_cases():
    key, share = "nvfp4_8r_residency", "nvfp4_8r_host_route_share"
    return [
        {key: "two_tier"}, {key: "hot_iq"}, {key: "hot_iq_host", share: 0.0}, {key: "hot_iq_host", share: 0},
        {key: "hot_iq_host", share: 0.05}, {key: "hot_iq_host", share: 0.013}, {}, {key: "hot_iq_host"},
        {key: "two_tier", share: 0.0}, {key: "hot_iq", share: 0.01}, {key: "hot_iq_host", share: 0.0500001},
        {key: "hot_iq_host", share: -0.001}, {key: "hot_iq_host", share: "0.0"}, {key: "hot_iq_host", share: True},
        {key: "hot_iq_host", share: float("nan")}, {key: "three_tier"}, {key: 1}, {key: "hot_iq_host", share: None},
        {key: "hot_iq_host", share: 1},
    ]


def write_seeded_packs(root, packs):
    """Seeded v1 and v2 packs of the same records (layers PACK_LAYERS) under
    ``root``, laid out by the product's ``packs`` module (its ``split_expert``
    and ``write_id_order_pack``); returns (v1 dir, v2 dir)."""
    import json
    from pathlib import Path

    root = Path(root)
    geom = packs.PackGeometry(**PACK_GEOM)
    v1, v2 = root / "v1", root / "v2"
    v1.mkdir(parents=True)
    records = {}
    for layer in PACK_LAYERS:
        for r, rec in enumerate(packs.split_expert(*pack_full_experts(layer), geom=geom)):
            records[(layer, r)] = rec
    packs.write_id_order_pack(v2, records, geom, comment="seeded")
    layers = []
    for layer in range(geom.num_layers):
        per_rank = []
        for r in range(geom.tp_ranks):
            split = pack_v1_split(layer, r)
            per_rank.append(split)
            if layer in PACK_LAYERS:
                for temp in ("hot", "cold"):
                    records[(layer, r)][np.asarray(split[temp], np.int64)].tofile(v1 / f"L{layer:02d}-r{r}-{temp}.bin")
        layers.append(per_rank)
    (v1 / "manifest.json").write_text(json.dumps({"format": "nvfp4-8r-mxfp4-v1", "layers": layers}))
    return v1, v2


# Route counters: a tier map with all three tiers and a run of decode calls
# (M <= 6 tokens x 6 routes, the reference's decode batch), popular experts
# often and rare ones after long gaps, so every gap bucket fills.
ROUTE_STATS_SEED = 20261204
ROUTE_STATS_CALLS = 420


def route_stats_inputs():
    rng = np.random.default_rng(ROUTE_STATS_SEED)
    tier = rng.choice(np.array([0, 1, 2], np.int8), size=384, p=[0.3, 0.3, 0.4]).astype(np.int8)
    p = 1.0 / (rng.permutation(384) + 1.0) ** 1.3
    p /= p.sum()
    calls = []
    for _ in range(ROUTE_STATS_CALLS):
        m = int(rng.integers(1, 7))
        calls.append(np.stack([rng.choice(384, size=6, replace=False, p=p) for _ in range(m)]).astype(np.int32))
    return tier, calls
