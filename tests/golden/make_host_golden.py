"""Golden fixtures for the host-side tier planner, tier-map reader and pack
reader, generated from the reference's own code.

Run where the reference project is mounted read-only, with REFERENCE_ROOT
set to its root directory.  It imports the reference's
modules (as ``make_golden.py`` does; nothing is copied) and writes
``tiers.npz`` and ``packs.npz`` beside this file.  Nothing at test time reads
the reference tree.

Pinned pieces (reference path:line, under
engine/src/vllm/model_executor/layers/fused_moe/experts/):
- nvfp4_8r_tiers.iq_record_bytes (:137-142), parse_residency (:115-135),
  choose_tiers (:246-305) with TierPlan's checks (:182-243) on a seeded tally
  over stages, budgets and residencies, parse_tier_map (:332-396) on a valid
  document and mutations of it, plan_from_map (:403-431);
- nvfp4_8r_native.read_rank_experts (:205-231), check_packs (:193-202) and
  _split_records (:234-250) on seeded v1 and v2 packs of a small geometry
  (the module's size constants are set to that geometry for the run);
- nvfp4_8r_stats.RouteStats.count / read (:65-110), run on CPU tensors over a
  seeded sequence of decode calls (counters after selected calls).
"""

from __future__ import annotations

import copy
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402
from make_golden import REF, import_reference_engine  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _outcome(fn):
    try:
        return "ok", fn()
    except ValueError as exc:
        return "refused", str(exc)


# ------------------------------------------------------------------- tiers
def describe_residency(r) -> str:
    name = type(r).__name__
    return f"{name}({r.route_share!r})" if name == "HotIqHost" else f"{name}()"


def plan_cases(tiers):
    """(stage, residency, budget) triples over the seeded tally."""
    iq = {l: tiers.iq_record_bytes(*gi.TIER_TYPES[l]) for l in range(gi.TIER_LAYERS)}
    out = []
    for stage in (range(0, 3), range(3, 6), range(0, 6), range(2, 3)):
        all_iq = sum(384 * iq[l] for l in stage)
        extra = sum(384 * (tiers.EXPERT_BYTES - iq[l]) for l in stage)
        for res in (("HotIq", None), ("HotIqHost", 0.0), ("HotIqHost", 0.003), ("HotIqHost", 0.05)):
            for frac in (-1e-9, 0.0, 0.004, 0.1, 0.37, 0.8, 1.0):
                budget = int(all_iq + frac * extra)
                out.append((stage, res, budget))
            out.append((stage, res, all_iq + tiers.EXPERT_BYTES - min(iq[l] for l in stage) - 1))
    return iq, out


def tier_map_docs(tiers, plan_tiers):
    """A valid document for 6 layers in stages 0-2 and 3-5, and mutations of it."""
    hot = [np.nonzero(plan_tiers[l] == 0)[0].astype(int).tolist() for l in range(gi.TIER_LAYERS)]
    stages = []
    for r in (range(0, 3), range(3, 6)):
        n_hot = sum(len(hot[l]) for l in r)
        stages.append({"first_layer": r.start, "last_layer": r.stop - 1, "hot": n_hot,
                       "compressed": len(r) * 384 - n_hot,
                       "digest": tiers.stage_digest({l: plan_tiers[l] for l in r}, r)})
    good = {"format": "nvfp4-8r-tier-map-v1", "comment": "seeded", "num_layers": gi.TIER_LAYERS,
            "num_experts": 384, "stages": stages, "hot": hot}
    docs = [("valid", good)]

    def mut(name, fn):
        d = copy.deepcopy(good)
        fn(d)
        docs.append((name, d))

    mut("format", lambda d: d.update(format="nvfp4-8r-tier-map-v2"))
    mut("extra_key", lambda d: d.update(extra=1))
    mut("missing_comment", lambda d: d.pop("comment"))
    mut("experts_383", lambda d: d.update(num_experts=383))
    mut("layers_zero", lambda d: d.update(num_layers=0))
    mut("layers_bool", lambda d: d.update(num_layers=True))
    mut("hot_short", lambda d: d["hot"].pop())
    mut("hot_unsorted", lambda d: d["hot"][1].reverse())
    mut("hot_duplicate", lambda d: d["hot"][2].append(d["hot"][2][-1]))
    mut("hot_empty", lambda d: d["hot"].__setitem__(0, []))
    mut("hot_all", lambda d: d["hot"].__setitem__(0, list(range(384))))
    mut("hot_out_of_range", lambda d: d["hot"][3].append(384))
    mut("hot_negative", lambda d: d["hot"][3].insert(0, -1))
    mut("hot_bool", lambda d: d["hot"][4].__setitem__(0, True) if d["hot"][4][0] == 1 else d["hot"][4].insert(0, False))
    mut("hot_float", lambda d: d["hot"][4].__setitem__(-1, float(d["hot"][4][-1])))
    mut("digest_wrong", lambda d: d["stages"][0].update(digest="0" * 64))
    mut("digest_short", lambda d: d["stages"][1].update(digest=d["stages"][1]["digest"][:63]))
    mut("counts_wrong", lambda d: d["stages"][1].update(hot=d["stages"][1]["hot"] + 1))
    mut("compressed_wrong", lambda d: d["stages"][1].update(compressed=d["stages"][1]["compressed"] - 1))
    mut("stage_gap", lambda d: d["stages"][1].update(first_layer=4))
    mut("stage_missing", lambda d: d["stages"].pop())
    mut("stages_not_list", lambda d: d.update(stages=d["stages"][0]))
    mut("stage_extra_key", lambda d: d["stages"][0].update(note="x"))
    mut("stage_past_end", lambda d: d["stages"][1].update(last_layer=6))
    mut("stage_empty", lambda d: d["stages"].insert(1, {"first_layer": 3, "last_layer": 2, "hot": 0,
                                                        "compressed": 0, "digest": "0" * 64}))
    mut("stages_empty", lambda d: d.update(stages=[]))
    mut("not_a_dict", lambda d: None)
    docs[-1] = ("not_a_dict", [1, 2])
    return docs


def make_tiers(out: Path) -> None:
    _, tiers, _, _, _ = import_reference_engine()
    counts = gi.tier_tally()
    record = {"iq_record_bytes": {}, "residency": [], "plans": [], "maps": [], "from_map": []}
    for t13 in (29, 16, 17, 15, 0):
        for t2 in (29, 16, 17, 18):
            st, v = _outcome(lambda: tiers.iq_record_bytes(t13, t2))
            record["iq_record_bytes"][f"{t13},{t2}"] = v if st == "ok" else None
    for extra in gi.residency_cases():
        st, v = _outcome(lambda: tiers.parse_residency(extra))
        record["residency"].append({"extra": repr(extra), "outcome": describe_residency(v) if st == "ok" else None})
    iq, cases = plan_cases(tiers)
    arrays = {}
    for i, (stage, (res, share), budget) in enumerate(cases):
        residency = tiers.HotIq() if res == "HotIq" else tiers.HotIqHost(share)
        st, v = _outcome(lambda: tiers.choose_tiers(counts, stage, {l: iq[l] for l in stage}, budget, residency))
        rec = {"stage": [stage.start, stage.stop], "residency": [res, share], "budget": budget, "status": st}
        if st == "ok":
            rec.update(hbm=int(v.hbm_bytes), digest=v.digest, hot=v.count(0), warm=v.count(1), host=v.count(2))
            arrays[f"plan{i}"] = np.stack([v.tiers[l] for l in stage])
        record["plans"].append(rec)
    # a whole-tally plan feeds the tier-map documents
    full = tiers.choose_tiers(counts, range(0, 6), iq, sum(384 * iq[l] for l in range(6)) + 300 * tiers.EXPERT_BYTES,
                              tiers.HotIq())
    plan_tiers = {l: np.asarray(full.tiers[l]) for l in range(6)}
    arrays["map_tiers"] = np.stack([plan_tiers[l] for l in range(6)])
    for name, doc in tier_map_docs(tiers, plan_tiers):
        st, v = _outcome(lambda: tiers.parse_tier_map(doc))
        rec = {"name": name, "doc": json.dumps(doc), "status": st}
        if st == "ok":
            rec["stages"] = {str(k): [r.start, r.stop, d] for k, (r, d) in v.stages.items()}
        record["maps"].append(rec)
    tmap = tiers.parse_tier_map(tier_map_docs(tiers, plan_tiers)[0][1])
    for stage in (range(0, 3), range(3, 6), range(0, 6), range(1, 3)):
        need = sum(int((plan_tiers[l] == 0).sum()) * tiers.EXPERT_BYTES + int((plan_tiers[l] == 1).sum()) * iq[l]
                   for l in stage)
        for res in ("HotIq", "HotIqHost"):
            for budget in (need, need - 1, need + 12345):
                residency = tiers.HotIq() if res == "HotIq" else tiers.HotIqHost(0.0)
                st, v = _outcome(lambda: tiers.plan_from_map(tmap, stage, {l: iq[l] for l in stage}, budget,
                                                             residency))
                rec = {"stage": [stage.start, stage.stop], "residency": res, "budget": budget, "status": st}
                if st == "ok":
                    rec.update(hbm=int(v.hbm_bytes), digest=v.digest)
                record["from_map"].append(rec)
    np.savez_compressed(out, record=np.frombuffer(json.dumps(record).encode(), np.uint8), **arrays)
    n_ok = sum(p["status"] == "ok" for p in record["plans"])
    print(f"tiers: {len(record['plans'])} plans ({n_ok} ok), {len(record['maps'])} maps -> {out.name}")


# ------------------------------------------------------------------- packs
def product_packs():
    """This repository's pack module (its writer lays out the seeded packs)."""
    import importlib

    sys.path.insert(0, str(HERE.parents[1]))
    from __graft_entry__ import load_package

    load_package()
    return importlib.import_module("b200moe.packs")


def make_packs(out: Path) -> None:
    import torch

    nat, _, _, _, _ = import_reference_engine()
    g = gi.PACK_GEOM
    packs = product_packs()
    geom = packs.PackGeometry(**g)
    H, Ip, K2 = g["hidden"], g["tp_inter"], g["w2_k"]
    patch = {"HIDDEN": H, "TP_INTER": Ip, "W2_K": K2, "NUM_EXPERTS": g["num_experts"],
             "_W13_CODES": Ip * H // 2, "_W13_SCALES": Ip * H // 32, "_W2_CODES": H * K2 // 2,
             "_W2_SCALES": H * K2 // 32}
    patch["EXPERT_BYTES"] = 2 * (patch["_W13_CODES"] + patch["_W13_SCALES"]) + patch["_W2_CODES"] + patch["_W2_SCALES"]
    assert patch["EXPERT_BYTES"] == geom.expert_bytes
    saved = {k: getattr(nat, k) for k in patch}
    record = {"geometry": g, "expert_bytes": geom.expert_bytes, "reads": []}
    try:
        for k, v in patch.items():
            setattr(nat, k, v)
        with tempfile.TemporaryDirectory() as tmp:
            v1, v2 = gi.write_seeded_packs(Path(tmp), packs)
            for fmt_dir in (v1, v2):
                fmt = nat.check_packs(fmt_dir)
                for layer in gi.PACK_LAYERS:
                    for r in range(g["tp_ranks"]):
                        raw = nat.read_rank_experts(fmt_dir, layer, r)
                        parts = nat._split_records(torch.from_numpy(np.ascontiguousarray(raw)))
                        record["reads"].append({"format": fmt, "layer": layer, "rank": r, "raw": sha(raw),
                                                "parts": [sha(p.numpy()) for p in parts],
                                                "shapes": [list(p.shape) for p in parts]})
            # refusals of the reference's readers
            bad = {}
            st, _ = _outcome(lambda: nat.read_rank_experts(v2, 40, 0))
            bad["v2_layer_40"] = st
            st, _ = _outcome(lambda: nat.read_rank_experts(v2, 0, 4))
            bad["v2_rank_4"] = st
            (v2 / "L00-r1.bin").write_bytes((v2 / "L00-r1.bin").read_bytes()[:-1])
            st, _ = _outcome(lambda: nat.read_rank_experts(v2, 0, 1))
            bad["v2_short_file"] = st
            m = json.loads((v2 / "manifest.json").read_text())
            m["extra"] = 1
            (v2 / "manifest.json").write_text(json.dumps(m))
            st, _ = _outcome(lambda: nat.check_packs(v2))
            bad["v2_extra_key"] = st
            m = json.loads((v1 / "manifest.json").read_text())
            m["layers"][0][0]["cold"] = m["layers"][0][0]["cold"][1:]
            (v1 / "manifest.json").write_text(json.dumps(m))
            st, _ = _outcome(lambda: nat.read_rank_experts(v1, 0, 0))
            bad["v1_not_partition"] = st
            record["refusals"] = bad
    finally:
        for k, v in saved.items():
            setattr(nat, k, v)
    np.savez_compressed(out, record=np.frombuffer(json.dumps(record).encode(), np.uint8))
    print(f"packs: {len(record['reads'])} reads, refusals {record['refusals']} -> {out.name}")


# ------------------------------------------------------------------- route counters
ROUTE_STATS_MARKS = (0, 1, 2, 50, 200, 419)


def make_route_stats(out: Path) -> None:
    import importlib

    import torch

    import_reference_engine()
    stats = importlib.import_module("vllm.model_executor.layers.fused_moe.experts.nvfp4_8r_stats")
    tier, calls = gi.route_stats_inputs()
    rs = stats.RouteStats(tier, torch.device("cpu"))
    arrays = {}
    for i, ids in enumerate(calls):
        rs.count(torch.from_numpy(ids))
        if i in ROUTE_STATS_MARKS:
            got = rs.read()
            for k in ("stat", "gap_hist", "recent", "routes"):
                arrays[f"{k}_{i}"] = np.array(got[k], np.int64, copy=True)  # CPU tensors share memory
            arrays[f"last_round_{i}"] = rs.last_round.numpy().copy()
    np.savez_compressed(out, marks=np.asarray(ROUTE_STATS_MARKS), **arrays)
    print(f"route stats: {len(calls)} calls, final stat {arrays[f'stat_{ROUTE_STATS_MARKS[-1]}'].tolist()}, "
          f"gap_hist {arrays[f'gap_hist_{ROUTE_STATS_MARKS[-1]}'].tolist()} -> {out.name}")


def main() -> None:
    if not REF.is_dir():
        raise SystemExit(f"reference tree {REF} not present")
    make_tiers(HERE / "tiers.npz")
    make_packs(HERE / "packs.npz")
    make_route_stats(HERE / "route_stats.npz")


if __name__ == "__main__":
    main()
