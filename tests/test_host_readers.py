"""CPU tests: the tier planner, the tier-map reader, expert placement and the
pack readers against fixtures the reference's own code produced
(``tests/golden/make_host_golden.py``), plus the reference's hand-worked tier
cases and round trips of the B200 join of rank slices."""

from __future__ import annotations

import json
import math

import numpy as np
import pytest

import golden_inputs as gi

GOLDEN = gi.__file__.rsplit("/", 1)[0]


@pytest.fixture(scope="module")
def tiers(pkg):
    from b200moe import tiers as t

    return t


@pytest.fixture(scope="module")
def packs(pkg):
    from b200moe import packs as p

    return p


def _record(name):
    z = np.load(f"{GOLDEN}/{name}.npz")
    return json.loads(z["record"].tobytes()), z


def _status(fn):
    try:
        return "ok", fn()
    except ValueError:
        return "refused", None


# ------------------------------------------------------------------ tiers
def test_iq_record_bytes_golden(tiers):
    rec, _ = _record("tiers")
    for key, want in rec["iq_record_bytes"].items():
        t13, t2 = map(int, key.split(","))
        st, got = _status(lambda: tiers.iq_record_bytes(t13, t2))
        assert (got if st == "ok" else None) == want, key
    # a whole expert at the C1 shapes: 8,192 blocks per projection slice x 4 ranks
    assert tiers.iq_record_bytes(16, 16, hidden=4096, inter=2048, tp=1) == 6_488_064
    assert tiers.slot_bytes("iq2_xxs", 4096, 2048) == 6_488_064
    assert tiers.slot_bytes("nvfp4", 4096, 2048) == 14_155_776 + 12
    assert tiers.slot_bytes("mxfp4", 4096, 2048) == 13_369_344
    assert tiers.slot_bytes("mxfp4", 4096, 2048, block_scaled=True) == 14_155_776


def test_parse_residency_golden(tiers):
    rec, _ = _record("tiers")
    cases = gi.residency_cases()
    assert len(cases) == len(rec["residency"])
    for extra, want in zip(cases, rec["residency"]):
        st, got = _status(lambda: tiers.parse_residency(extra))
        desc = None
        if st == "ok":
            name = type(got).__name__
            desc = f"{name}({got.route_share!r})" if name == "HotIqHost" else f"{name}()"
        assert desc == want["outcome"], want["extra"]


def test_choose_tiers_golden(tiers):
    """Every (stage, residency, budget) case: the same refusal, or the same
    tier arrays, HBM bytes and digest as the reference's choose_tiers."""
    rec, z = _record("tiers")
    counts = gi.tier_tally()
    iq = {l: tiers.iq_record_bytes(*gi.TIER_TYPES[l]) for l in range(gi.TIER_LAYERS)}
    n_ok = 0
    for i, case in enumerate(rec["plans"]):
        stage = range(*case["stage"])
        res, share = case["residency"]
        residency = tiers.HotIq() if res == "HotIq" else tiers.HotIqHost(share)
        st, plan = _status(lambda: tiers.choose_tiers(counts, stage, {l: iq[l] for l in stage}, case["budget"],
                                                      residency))
        assert st == case["status"], (i, case)
        if st != "ok":
            continue
        n_ok += 1
        np.testing.assert_array_equal(np.stack([plan.tiers[l] for l in stage]), z[f"plan{i}"])
        assert plan.hbm_bytes == case["hbm"] and plan.digest == case["digest"]
        assert (plan.count(0), plan.count(1), plan.count(2)) == (case["hot"], case["warm"], case["host"])
    assert n_ok >= 40


# The reference's hand-worked toy stage (harness/benchmarks/nvfp4_8r/test_t3_tiers.py:96-215):
# layer 0 IQ1_M (1,935,360 B per rank record), layer 1 IQ2_XS (2,557,440 B).
IQ_TOY = {0: 1_935_360, 1: 2_557_440}
D0, D1 = 4_874_240 - 1_935_360, 4_874_240 - 2_557_440
ALL_IQ = 384 * (1_935_360 + 2_557_440)


def _toy_counts():
    c = np.zeros((2, 384), np.int64)
    c[0, 10], c[0, 20], c[0, 30] = 600, 300, 5
    c[1, 7], c[1, 8], c[1, 9] = 500, 100, 4
    return c


def _want(default, sets):
    out = {l: np.full(384, default, np.int8) for l in (0, 1)}
    for (l, e), t in sets.items():
        out[l][e] = t
    return out


@pytest.mark.parametrize("case", ["T1", "T2", "T3", "T4"])
def test_choose_tiers_hand_cases(tiers, case):
    HOT, WARM, HOST = tiers.HOT, tiers.WARM, tiers.HOST
    hbm = ALL_IQ + D1 + D0
    spec = {
        # one byte short of the third promotion: L1 e7 and L0 e10 HOT; L1 e8 would fit but follows the stop
        "T1": (hbm + D0 - 1, tiers.HotIq(), _want(WARM, {(1, 7): HOT, (0, 10): HOT}), hbm),
        "T2": (hbm + D0, tiers.HotIq(), _want(WARM, {(1, 7): HOT, (0, 10): HOT, (0, 20): HOT}), hbm + D0),
        # share 0: HOST = exactly the 762 never-routed experts
        "T3": (13_478_400 + D1 + D0, tiers.HotIqHost(0.0),
               _want(HOST, {(1, 7): HOT, (0, 10): HOT, (0, 20): WARM, (0, 30): WARM, (1, 8): WARM, (1, 9): WARM}),
               13_478_400 + D1 + D0),
        # 0.004 x 1,509 routes = 6.036: the zeros and L1 e9 (4 routes) go HOST, L0 e30 (sum 9) stops the walk
        "T4": (10_920_960 + D1 + D0, tiers.HotIqHost(0.004),
               _want(HOST, {(1, 7): HOT, (0, 10): HOT, (0, 20): WARM, (0, 30): WARM, (1, 8): WARM}),
               10_920_960 + D1 + D0),
    }[case]
    budget, residency, want, want_hbm = spec
    plan = tiers.choose_tiers(_toy_counts(), range(0, 2), IQ_TOY, budget, residency)
    for l in (0, 1):
        np.testing.assert_array_equal(plan.tiers[l], want[l])
    assert plan.hbm_bytes == want_hbm and plan.budget_bytes == budget
    import hashlib

    assert plan.digest == hashlib.sha256(want[0].tobytes() + want[1].tobytes()).hexdigest()


def test_choose_tiers_refusals(tiers):
    c = _toy_counts()
    with pytest.raises(ValueError):  # below the all-IQ tier
        tiers.choose_tiers(c, range(0, 2), IQ_TOY, ALL_IQ - 1, tiers.HotIq())
    with pytest.raises(ValueError):  # layer 0 gets no HOT expert
        tiers.choose_tiers(c, range(0, 2), IQ_TOY, ALL_IQ + D1, tiers.HotIq())
    with pytest.raises(ValueError):  # room for every routed expert: no WARM left
        tiers.choose_tiers(c, range(0, 2), IQ_TOY, 29_245_440, tiers.HotIqHost(0.0))
    with pytest.raises(ValueError):
        tiers.choose_tiers(c, range(0, 2), IQ_TOY, ALL_IQ + D0 + D1, tiers.TwoTier())
    with pytest.raises(ValueError):
        tiers.choose_tiers(c.astype(np.float32), range(0, 2), IQ_TOY, ALL_IQ + D0 + D1, tiers.HotIq())
    with pytest.raises(ValueError):
        tiers.choose_tiers(-c, range(0, 2), IQ_TOY, ALL_IQ + D0 + D1, tiers.HotIq())
    with pytest.raises(ValueError):
        tiers.choose_tiers(c, range(0, 3), IQ_TOY, ALL_IQ + D0 + D1, tiers.HotIq())
    good = _want(tiers.WARM, {(1, 7): tiers.HOT, (0, 10): tiers.HOT})
    with pytest.raises(ValueError):  # a HOST expert under hot_iq
        bad = {l: a.copy() for l, a in good.items()}
        bad[0][0] = tiers.HOST
        tiers.TierPlan(range(0, 2), bad, IQ_TOY, ALL_IQ + D0 + D1, tiers.HotIq())
    with pytest.raises(ValueError):
        tiers.TierPlan(range(0, 2), good, IQ_TOY, ALL_IQ + D0 + D1 - 1, tiers.HotIq())
    with pytest.raises(ValueError):
        tiers.TierPlan(range(0, 2), {l: a.astype(np.int64) for l, a in good.items()}, IQ_TOY, ALL_IQ + D0 + D1,
                       tiers.HotIq())


def test_b200_plan_properties(tiers):
    """A B200 plan: HOT costs an NVFP4 slot, WARM an IQ2_XXS slot, one 180 GB
    budget for 40 C4 layers; every HOT expert is at least as dense (routes per
    promoted byte) as every WARM one and no further promotion fits."""
    rng = np.random.default_rng(4000)
    counts = np.floor(rng.pareto(1.1, size=(40, 384)) * 20).astype(np.int64)
    native = tiers.slot_bytes("nvfp4", 4096, 2048)
    iqb = tiers.slot_bytes("iq2_xxs", 4096, 2048)
    budget = 120 * 2**30
    plan = tiers.choose_tiers(counts, range(0, 40), {l: iqb for l in range(40)}, budget, tiers.HotIq(),
                              native_bytes=native)
    assert plan.hbm_bytes <= budget < plan.hbm_bytes + (native - iqb)
    t = np.stack([plan.tiers[l] for l in range(40)])
    assert counts[t == tiers.HOT].min() >= counts[t == tiers.WARM].max()
    assert plan.count(tiers.HOST) == 0


def test_tier_map_golden(tiers):
    rec, z = _record("tiers")
    for case in rec["maps"]:
        doc = json.loads(case["doc"])
        st, tm = _status(lambda: tiers.parse_tier_map(doc))
        assert st == case["status"], case["name"]
        if st == "ok":
            got = {str(k): [r.start, r.stop, d] for k, (r, d) in tm.stages.items()}
            assert got == case["stages"]
            for l in range(gi.TIER_LAYERS):
                np.testing.assert_array_equal(tm.tiers[l], z["map_tiers"][l])
                assert not tm.tiers[l].flags.writeable


def test_plan_from_map_golden(tiers):
    rec, z = _record("tiers")
    tm = tiers.parse_tier_map(json.loads(rec["maps"][0]["doc"]))
    iq = {l: tiers.iq_record_bytes(*gi.TIER_TYPES[l]) for l in range(gi.TIER_LAYERS)}
    for case in rec["from_map"]:
        stage = range(*case["stage"])
        residency = tiers.HotIq() if case["residency"] == "HotIq" else tiers.HotIqHost(0.0)
        st, plan = _status(lambda: tiers.plan_from_map(tm, stage, {l: iq[l] for l in stage}, case["budget"],
                                                       residency))
        assert st == case["status"], case
        if st == "ok":
            assert plan.hbm_bytes == case["hbm"] and plan.digest == case["digest"]


def test_tier_map_document_round_trip(tiers, tmp_path):
    rng = np.random.default_rng(7)
    arrays = {l: np.where(rng.random(384) < 0.4, tiers.HOT, tiers.WARM).astype(np.int8) for l in range(5)}
    doc = tiers.tier_map_document(arrays, [range(0, 2), range(2, 5)], comment="b200")
    path = tmp_path / "map.json"
    path.write_text(json.dumps(doc))
    tm = tiers.load_tier_map(path)
    for l in range(5):
        np.testing.assert_array_equal(tm.tiers[l], arrays[l])
    assert tm.stages[2][0] == range(2, 5)
    with pytest.raises(ValueError):
        tm.stage(range(0, 5))  # made for another split


# ------------------------------------------------------------------ placement
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_balanced_owners(tiers, world):
    tier, rank = tiers.zipf_tier(384, 150, seed=2)
    counts = (1e6 / (rank.astype(np.float64) + 1) ** 1.1).astype(np.int64)
    owner = tiers.balanced_owners(tier, world, counts)
    assert owner.dtype == np.int32 and owner.shape == (384,)
    np.testing.assert_array_equal(owner, tiers.balanced_owners(tier.copy(), world, counts.copy()))
    for t in (tiers.HOT, tiers.WARM):
        per = np.bincount(owner[tier == t], minlength=world)
        assert per.max() - per.min() <= 1
    per = np.bincount(owner, minlength=world)
    assert per.max() - per.min() <= 1
    routes = np.bincount(owner, weights=counts, minlength=world)
    if world > 1:  # the contiguous split puts the popular experts wherever their ids fall
        by_range = np.bincount(tiers.owner_by_range(384, world), weights=counts, minlength=world)
        assert routes.max() / routes.mean() <= by_range.max() / by_range.mean() + 1e-9
        # within 5 % of an even share, unless one expert alone outweighs a share
        assert routes.max() <= max(1.05 * routes.mean(), 1.15 * counts.max())
    seen = np.zeros(384, int)
    for r in range(world):
        fp4, iq2 = tiers.local_maps(tier, r, world, owner)
        mine = (fp4 >= 0) | (iq2 >= 0)
        np.testing.assert_array_equal(mine, owner == r)
        np.testing.assert_array_equal(np.sort(fp4[fp4 >= 0]), np.arange(int((fp4 >= 0).sum())))
        seen += mine
    assert np.all(seen == 1)


def test_placement_checks(tiers):
    tier, _ = tiers.zipf_tier(384, 150, seed=2)
    owner = tiers.balanced_owners(tier, 4)
    assert tiers.placement_digest(tier, 4, owner) != tiers.placement_digest(tier, 4)
    assert tiers.placement_digest(tier, 4, owner) == tiers.placement_digest(tier, 4, owner.copy())
    np.testing.assert_array_equal(tiers.owner_by_range(384, 4), np.repeat(np.arange(4, dtype=np.int32), 96))
    with pytest.raises(ValueError):
        tiers.local_maps(tier, 0, 4, owner.astype(np.int64))
    with pytest.raises(ValueError):
        tiers.local_maps(tier, 0, 4, np.zeros(384, np.int32))  # ranks 1-3 own nothing
    with pytest.raises(ValueError):
        tiers.balanced_owners(np.full(384, tiers.HOST, np.int8), 2)


# ------------------------------------------------------------------ packs
def _sha(a):
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_pack_reader_golden(packs, tmp_path):
    """v1 and v2 packs of the same seeded records read back as the
    reference's read_rank_experts + _split_records read them."""
    rec, _ = _record("packs")
    geom = packs.PackGeometry(**gi.PACK_GEOM)
    assert rec["expert_bytes"] == geom.expert_bytes
    v1, v2 = gi.write_seeded_packs(tmp_path, packs)
    dirs = {"nvfp4-8r-mxfp4-v1": v1, "nvfp4-8r-mxfp4-v2-id-order": v2}
    for want in rec["reads"]:
        d = dirs[want["format"]]
        assert packs.check_packs(d, geom) == want["format"]
        raw = packs.read_rank_experts(d, want["layer"], want["rank"], geom)
        assert _sha(raw) == want["raw"]
        parts = packs.split_records(np.asarray(raw), geom)
        assert [_sha(p) for p in parts] == want["parts"]
        assert [list(p.shape) for p in parts] == want["shapes"]


def test_pack_refusals(packs, tmp_path):
    rec, _ = _record("packs")
    geom = packs.PackGeometry(**gi.PACK_GEOM)
    v1, v2 = gi.write_seeded_packs(tmp_path, packs)
    got = {}
    got["v2_layer_40"] = _status(lambda: packs.read_rank_experts(v2, 40, 0, geom))[0]
    got["v2_rank_4"] = _status(lambda: packs.read_rank_experts(v2, 0, 4, geom))[0]
    (v2 / "L00-r1.bin").write_bytes((v2 / "L00-r1.bin").read_bytes()[:-1])
    got["v2_short_file"] = _status(lambda: packs.read_rank_experts(v2, 0, 1, geom))[0]
    m = json.loads((v2 / "manifest.json").read_text())
    m["extra"] = 1
    (v2 / "manifest.json").write_text(json.dumps(m))
    got["v2_extra_key"] = _status(lambda: packs.check_packs(v2, geom))[0]
    m = json.loads((v1 / "manifest.json").read_text())
    m["layers"][0][0]["cold"] = m["layers"][0][0]["cold"][1:]
    (v1 / "manifest.json").write_text(json.dumps(m))
    got["v1_not_partition"] = _status(lambda: packs.read_rank_experts(v1, 0, 0, geom))[0]
    assert got == rec["refusals"]
    with pytest.raises(ValueError):
        packs.check_packs(tmp_path, geom)  # no manifest


def test_join_split_round_trip(packs, tmp_path):
    """Whole experts -> rank records (the reference's builder layout) -> the
    pack files -> joined again: the same bytes."""
    geom = packs.PackGeometry(**gi.PACK_GEOM)
    full = gi.pack_full_experts(7)
    _, v2 = gi.write_seeded_packs(tmp_path, packs)
    ranks = [packs.read_rank_experts(v2, 7, r, geom) for r in range(geom.tp_ranks)]
    assert isinstance(ranks[0], np.memmap)
    sel = np.array([0, 3, 4, 11])
    joined = packs.join_experts([np.asarray(r[sel]) for r in ranks], geom)
    for a, b in zip(joined, full):
        np.testing.assert_array_equal(a, b[sel])
    # the W2 padding the builder writes: zero codes, scale 127
    w2c, w2s = packs.split_records(np.asarray(ranks[1]), geom)[4:]
    assert not w2c[:, :, geom.tp_inter // 2:].any() and np.all(w2s[:, :, geom.tp_inter // 32:] == 127)


def test_join_refusals(packs):
    geom = packs.PackGeometry(**gi.PACK_GEOM)
    slices = packs.split_expert(*[a[:2] for a in gi.pack_full_experts(0)], geom=geom)
    bad = [s.copy() for s in slices]
    w2c = packs.split_records(bad[2], geom)[4]
    w2c[1, 5, geom.tp_inter // 2] = 0x10  # a padding code
    with pytest.raises(ValueError):
        packs.join_experts(bad, geom)
    bad = [s.copy() for s in slices]
    packs.split_records(bad[0], geom)[1][0, 0, 0] = 255  # E8M0 NaN
    with pytest.raises(ValueError):
        packs.join_experts(bad, geom)
    with pytest.raises(ValueError):
        packs.join_experts(slices[:3], geom)
    assert packs.REFERENCE_GEOMETRY.expert_bytes == 4_874_240
    assert packs.REFERENCE_GEOMETRY.inter == 2304
    assert math.isclose(packs.REFERENCE_GEOMETRY.expert_bytes / 4_874_240, 1.0)
