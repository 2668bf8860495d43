"""Generate the golden fixtures in this directory from the reference's own code.

Run where the reference project is mounted read-only, with REFERENCE_ROOT
set to its root directory.  It imports the reference's
Python modules directly (no copy of their source is made) and writes small
``.npz`` fixtures that the CPU and GPU tests read.  Nothing at test time reads
the reference tree.

Pinned pieces (reference path:line):
- route-plan chain: NativeV41Moe._groups / _split_groups / _tier_groups
  (engine/src/vllm/model_executor/layers/fused_moe/experts/nvfp4_8r_native.py:806-872)
  on placeholder banks built as harness/benchmarks/nvfp4_8r/test_group_plan.py:72-104
  does; and the IQ route slots (nvfp4_8r_native.py:878-884);
- slot maps: nvfp4_8r_tiers.slot_maps (nvfp4_8r_tiers.py:169-179);
- NVFP4 decode: accept_p1.Checkpoint.projection (harness/benchmarks/nvfp4_8r/accept_p1.py:53-84)
  on a one-expert synthetic safetensors checkpoint;
- MXFP4 decode: accept_p1.packed_projection (accept_p1.py:87-101);
- NVFP4 -> MXFP4 fold: build_packs.fold (build_packs.py:120-151), both a
  foldable projection and a refused one;
- fp64 expert: make_p2_refs.contribution (make_p2_refs.py:52-59);
- SwiGLU chain: the three torch lines of nvfp4_8r_native.py:937-939 run on CPU;
- IQ2_XXS decode: gguf-py 0.19.0 gguf.quants.dequantize (the call of
  make_t3_refs.py:61-64).

Large outputs are pinned by sha256 of their bytes plus a few sampled rows;
inputs are regenerated from the stored seed by ``golden_inputs.py``.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import os
import struct
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402

def _reference_root() -> Path:
    root = os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit("set REFERENCE_ROOT to the reference project's root directory")
    return Path(root)


REF = _reference_root()
EXP = REF / "engine/src/vllm/model_executor/layers/fused_moe/experts"
HB = REF / "harness/benchmarks"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------------------
# importing the reference
# ---------------------------------------------------------------------------

def _stub(name: str, **attrs) -> None:
    mod = types.ModuleType(name)
    mod.__dict__.update(attrs)
    sys.modules[name] = mod


def import_reference_engine():
    """nvfp4_8r_native with three (four) missing engine modules stubbed."""
    import enum

    import vllm.model_executor.layers.fused_moe.experts as experts_pkg

    if str(EXP) not in experts_pkg.__path__:
        experts_pkg.__path__.append(str(EXP))

    class QpnFragmentOrder(enum.IntEnum):
        M8N8K4 = 0

    base = "vllm.model_executor.layers"
    _stub(f"{base}.fused_moe.experts.skinny_sm70_moe", _QPN_MAX_M=16,
          QpnFragmentOrder=QpnFragmentOrder, grouped_splitk=lambda *a, **k: 1,
          qpn_fragment_order=lambda *a, **k: QpnFragmentOrder.M8N8K4,
          qpn_prepack=lambda *a, **k: None, rebase_e8m0_for_fp16=lambda *a, **k: None)
    _stub(f"{base}.fused_moe.sm70")
    _stub(f"{base}.fused_moe.sm70.reduction", _mtp_weighted_reduce=None)
    _stub(f"{base}.quantization.gguf_expert_cache", _native=None)
    _stub(f"{base}.quantization.gguf_v41_moe")
    nat = importlib.import_module(f"{base}.fused_moe.experts.nvfp4_8r_native")
    tiers = importlib.import_module(f"{base}.fused_moe.experts.nvfp4_8r_tiers")
    gplan = importlib.import_module(f"{base}.fused_moe.experts.nvfp4_8r_group_plan")
    swig = importlib.import_module(f"{base}.fused_moe.experts.nvfp4_8r_swiglu")
    return nat, tiers, gplan, swig, QpnFragmentOrder


def import_reference_harness():
    os.environ.setdefault("LANE", tempfile.gettempdir())
    if str(HB) not in sys.path:
        sys.path.insert(0, str(HB))
    accept_p1 = importlib.import_module("nvfp4_8r.accept_p1")
    build_packs = importlib.import_module("nvfp4_8r.build_packs")
    make_p2_refs = importlib.import_module("nvfp4_8r.make_p2_refs")
    return accept_p1, build_packs, make_p2_refs


# ---------------------------------------------------------------------------
# route plan
# ---------------------------------------------------------------------------

def make_route_plan(out: Path) -> None:
    import torch

    nat, tiers, gplan, swig, Order = import_reference_engine()
    dev = torch.device("cpu")
    HOT, WARM, HOST = 0, 1, 2
    kinds = ("resident", "two_tier", "three_tier_host", "three_tier_nohost")
    rng = np.random.default_rng(gi.ROUTE_PLAN_SEED)

    def pset(n):
        z = torch.zeros((n, 1), dtype=torch.uint8)
        g = torch.ones(n, dtype=torch.float32)
        return nat.NativeExpertSet(z, z, z, z, g, g, Order.M8N8K4)

    def piq(n):
        banks = []
        for role in ("w1", "w3", "w2"):
            _, rows, blocks = nat._IQ_ROWS[role]
            one = torch.zeros((1, rows, blocks * tiers.IQ_BLOCK_BYTES[16]), dtype=torch.uint8)
            banks.append(one.expand(n, -1, -1))
        return nat.IqWarmBank(banks[0], banks[1], banks[2], 16, 16)

    def build(kind, tier):
        maps = tiers.slot_maps(tier)
        to = torch.from_numpy
        kw = dict(group_plan=gplan.GroupPlan.CHAIN, swiglu=swig.Swiglu.CHAIN,
                  prefill_swiglu=swig.Swiglu.CHAIN, prefill_rb=nat.qrb.PrefillRb.RB2)
        hot = pset(int((tier == HOT).sum()))
        if kind == "resident":
            return nat.NativeV41Moe(hot, to(maps.hot), 16, **kw)
        cold = pset(int((tier != HOT).sum()))
        if kind == "two_tier":
            return nat.NativeV41Moe(hot, to(maps.hot), 16, cold=cold,
                                    cold_slot_of_expert=to(maps.cold), **kw)
        iq = piq(int((tier == WARM).sum()))
        return nat.NativeV41Moe.three_tier(hot, cold, iq, tier, 16, None,
                                           iq_tail=nat.iqt.IqTail.TORCH, **kw)

    def tier_of(kind):
        perm = rng.permutation(384)
        tier = np.full(384, HOT, np.int8)
        if kind == "resident":
            return tier
        if kind == "two_tier":
            n_host = int(rng.choice([1, 6, int(rng.integers(1, 384)), 383]))
            tier[perm[:n_host]] = HOST
            return tier
        n_hot = int(rng.choice([1, int(rng.integers(1, 383)), 382 if kind == "three_tier_host" else 383]))
        rest = perm[n_hot:]
        if kind == "three_tier_nohost":
            tier[rest] = WARM
            return tier
        n_warm = int(rng.integers(1, len(rest)))
        tier[rest[:n_warm]] = WARM
        tier[rest[n_warm:]] = HOST
        return tier

    arrays: dict[str, np.ndarray] = {}
    meta = []
    case = 0
    for j in range(24):
        kind = kinds[j % 4]
        tier = tier_of(kind)
        moe = build(kind, tier)
        maps = tiers.slot_maps(tier)
        for name in ("hot", "cold", "host", "iq"):
            arrays[f"map{j}_{name}"] = getattr(maps, name)
        arrays[f"tier{j}"] = tier
        routings = []
        for _ in range(10):
            m = int(rng.integers(1, 17))
            style = rng.integers(3)
            if style == 0:
                ids = np.stack([rng.choice(384, 6, replace=False) for _ in range(m)])
            elif style == 1:
                pool = rng.choice(384, int(rng.integers(6, 40)), replace=False)
                ids = np.stack([rng.choice(pool, 6, replace=False) for _ in range(m)])
            else:
                ids = np.full((m, 6), int(rng.integers(384)))  # repeated keys
            routings.append(ids.astype(np.int32))
        for ids in routings:
            t_ids = torch.from_numpy(ids)
            launches = moe._launches(t_ids)
            arrays[f"c{case}_ids"] = ids
            for li, (_, perm, gids, goff) in enumerate(launches):
                arrays[f"c{case}_l{li}_perm"] = perm.numpy().astype(np.int32)
                arrays[f"c{case}_l{li}_gids"] = gids.numpy().astype(np.int32)
                arrays[f"c{case}_l{li}_goff"] = goff.numpy().astype(np.int32)
            if moe.warm is not None:
                iq_ids, w_native = moe._iq_routes(t_ids, torch.ones(ids.shape, dtype=torch.float32))
                arrays[f"c{case}_iq"] = iq_ids.numpy().astype(np.int32)
            meta.append({"case": case, "map": j, "kind": kind, "launches": len(launches),
                         "n_hot": int((tier == HOT).sum()), "n_cold": int((tier != HOT).sum()),
                         "host_in_decode": bool((tier == HOST).any())})
            case += 1
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(out, **arrays)
    print(f"route plan: {case} cases -> {out.name}")


# ---------------------------------------------------------------------------
# packing and decode
# ---------------------------------------------------------------------------

def _write_checkpoint(root: Path, codes: np.ndarray, scales: np.ndarray, glob: np.float32) -> None:
    """A one-tensor-triple safetensors checkpoint for accept_p1.Checkpoint."""
    prefix = "layers.0.ffn.experts.0.w1"
    tensors = [(prefix + ".weight", "U8", codes), (prefix + ".weight_scale", "F8_E4M3", scales),
               (prefix + ".weight_scale_2", "F32", np.asarray([glob], np.float32))]
    header, blobs, off = {}, [], 0
    for name, dt, arr in tensors:
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape) if arr.ndim else [], "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hb = json.dumps(header).encode()
    with open(root / "model-00001.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    (root / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {n: "model-00001.safetensors" for n, _, _ in tensors}}))
    (root / "verify.log").write_text("ALL-VERIFIED 84\n")


def make_packing(out: Path) -> None:
    accept_p1, build_packs, make_p2_refs = import_reference_harness()
    arrays: dict[str, np.ndarray] = {}
    meta: dict = {}

    # NVFP4 decode through the reference checkpoint reader (geometry fixed at 2304 x 5120)
    codes, scales, glob = gi.nvfp4_decode_inputs()
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp)
        _write_checkpoint(root, codes, scales, glob)
        ck = accept_p1.Checkpoint(root, root / "verify.log")
        dec = ck.projection(0, 0, "w1")
    meta["nvfp4_decode_sha256"] = sha(dec.astype(np.float32))
    arrays["nvfp4_decode_rows"] = dec[gi.SAMPLE_ROWS].astype(np.float32)

    # MXFP4 record decode
    raw, rows, cols = gi.mxfp4_decode_inputs()
    dec = accept_p1.packed_projection(raw, rows, cols)
    meta["mxfp4_decode_sha256"] = sha(dec.astype(np.float32))
    arrays["mxfp4_decode_rows"] = dec[gi.SAMPLE_ROWS[gi.SAMPLE_ROWS < rows]].astype(np.float32)

    # Fold: a foldable C0-shaped W13 projection and a refused one
    for tag, foldable in (("ok", True), ("bad", False)):
        codes, scale_bits, glob = gi.fold_inputs(foldable)
        table = np.array([((b & 7) / 512 if (b & 120) == 0 else (1 + (b & 7) / 8) * 2.0 ** (((b >> 3) & 15) - 7))
                          * (-1 if b & 128 else 1) for b in range(256)], np.float32)
        proj = build_packs.Nvfp4Projection(codes, table[scale_bits], np.float32(glob))
        try:
            fc, fs = build_packs.fold(proj)
            meta[f"fold_{tag}"] = {"ok": True, "codes_sha256": sha(fc), "scales_sha256": sha(fs)}
            arrays[f"fold_{tag}_codes_rows"] = fc[:8]
            arrays[f"fold_{tag}_scales_rows"] = fs[:8]
        except ValueError as exc:
            meta[f"fold_{tag}"] = {"ok": False, "error": str(exc)}

    # fp64 contribution
    w1, w3, w2, x, wt = gi.contribution_inputs()
    c = make_p2_refs.contribution(w1, w3, w2, x, wt)
    arrays["contribution"] = c.astype(np.float64)

    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(out, **arrays)
    print(f"packing: {sorted(meta)} -> {out.name}")


def make_swiglu(out: Path) -> None:
    import torch

    y13 = gi.swiglu_inputs()
    inter = y13.shape[1] // 2
    t = torch.from_numpy(y13)
    # nvfp4_8r_native.py:937-939, verbatim semantics on CPU torch
    g = t[:, :inter].float().clamp(max=10.0)
    u = t[:, inter:].float().clamp(-10.0, 10.0)
    res = (torch.nn.functional.silu(g) * u).to(torch.float16).numpy()
    np.savez_compressed(out, y13=y13, inter=res)
    print(f"swiglu: {y13.shape} -> {out.name}")


def make_iq2(out: Path) -> None:
    import gguf

    blocks = gi.iq2_inputs()
    rows, nb, _ = blocks.shape
    dec = gguf.quants.dequantize(blocks.reshape(rows, nb * 66), gguf.GGMLQuantizationType.IQ2_XXS)
    dec = np.asarray(dec, np.float32).reshape(rows, nb * 256)
    np.savez_compressed(out, sha256=np.frombuffer(sha(dec).encode(), np.uint8),
                        rows=dec[:4], gguf_version=np.frombuffer(gguf.__version__.encode()
                                                                  if hasattr(gguf, "__version__") else b"0.19.0", np.uint8))
    print(f"iq2: {blocks.shape} -> {out.name}")


def main() -> None:
    if not REF.is_dir():
        raise SystemExit(f"reference tree {REF} not present")
    make_route_plan(HERE / "route_plan.npz")
    make_packing(HERE / "packing.npz")
    make_swiglu(HERE / "swiglu.npz")
    make_iq2(HERE / "iq2xxs.npz")


if __name__ == "__main__":
    main()
