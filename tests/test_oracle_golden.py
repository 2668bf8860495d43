"""The CPU oracle against the golden vectors made by the reference's own code.

These pin the oracle before anything is checked against it: every bit-exact
claim of the CUDA path rests on these passing.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

import golden_inputs as gi
from oracle import moe_oracle as mo

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def packing():
    with np.load(GOLDEN / "packing.npz") as z:
        d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(bytes(d["meta"]).decode())
    return d


def test_nvfp4_decode_bit_exact(packing):
    codes, scales, glob = gi.nvfp4_decode_inputs()
    dec = mo.nvfp4_decode(codes, scales, glob)
    assert np.array_equal(dec[gi.SAMPLE_ROWS].view(np.uint32), packing["nvfp4_decode_rows"].view(np.uint32))
    assert sha(dec) == packing["meta"]["nvfp4_decode_sha256"]


def test_mxfp4_decode_bit_exact(packing):
    raw, rows, cols = gi.mxfp4_decode_inputs()
    n = rows * cols // 2
    dec = mo.mxfp4_decode(raw[:n].reshape(rows, cols // 2), raw[n:].reshape(rows, cols // 32))
    assert sha(dec) == packing["meta"]["mxfp4_decode_sha256"]


def test_fold_bit_exact_and_refusal(packing):
    codes, bits, glob = gi.fold_inputs(True)
    fc, fs = mo.fold_nvfp4_to_mxfp4(codes, bits, glob)
    assert packing["meta"]["fold_ok"]["ok"]
    assert sha(fc) == packing["meta"]["fold_ok"]["codes_sha256"]
    assert sha(fs) == packing["meta"]["fold_ok"]["scales_sha256"]
    # folded values decode to exactly the NVFP4 values
    assert np.array_equal(mo.mxfp4_decode(fc, fs), mo.nvfp4_decode(codes, bits, glob))
    codes, bits, glob = gi.fold_inputs(False)
    assert not packing["meta"]["fold_bad"]["ok"]
    with pytest.raises(ValueError, match="cannot fold exactly"):
        mo.fold_nvfp4_to_mxfp4(codes, bits, glob)


def test_contribution_fp64(packing):
    w1, w3, w2, x, wt = gi.contribution_inputs()
    got = mo.contribution_fp64(np.concatenate([w1, w3]), w2, x, wt)
    assert np.array_equal(got, packing["contribution"])


def test_swiglu_chain_vs_reference_torch():
    with np.load(GOLDEN / "swiglu.npz") as z:
        y13, want = z["y13"], z["inter"]
    got = mo.swiglu_chain(y13, y13.shape[1] // 2)
    a, b = got.view(np.uint16).astype(np.int32), want.view(np.uint16).astype(np.int32)
    both_nan = np.isnan(got) & np.isnan(want)
    diff = (a != b) & ~both_nan
    # numpy's float32 exp and torch's CPU exp may differ in the last fp32 bit;
    # after the fp16 rounding that shows as at most one fp16 ulp, rarely.
    assert np.all(np.abs(a - b)[diff] <= 1)
    assert diff.sum() <= max(2, got.size // 2000)
    assert np.array_equal(np.isnan(got), np.isnan(want))


def test_iq2xxs_decode_vs_gguf():
    with np.load(GOLDEN / "iq2xxs.npz") as z:
        want_sha, rows = bytes(z["sha256"]).decode(), z["rows"]
    grid, ksigns = mo.iq2xxs_tables()
    dec = mo.iq2xxs_decode(gi.iq2_inputs(), grid, ksigns)
    assert np.array_equal(dec[:4].view(np.uint32), rows.view(np.uint32))
    assert sha(dec) == want_sha


@pytest.fixture(scope="module")
def route_plan():
    with np.load(GOLDEN / "route_plan.npz") as z:
        d = {k: z[k] for k in z.files}
    d["meta"] = json.loads(bytes(d["meta"]).decode())
    return d


def test_slot_maps(route_plan):
    for j in range(24):
        maps = mo.slot_maps(route_plan[f"tier{j}"])
        for name in ("hot", "cold", "host", "iq"):
            assert np.array_equal(maps[name], route_plan[f"map{j}_{name}"])


def test_route_plan_chain_bit_exact(route_plan):
    for c in route_plan["meta"]:
        j, kind = c["map"], c["kind"]
        ids = route_plan[f"c{c['case']}_ids"]
        maps = mo.slot_maps(route_plan[f"tier{j}"])
        if kind == "resident":
            launches = mo.groups_resident(ids, maps["hot"])
        elif kind == "two_tier":
            launches = mo.groups_split(ids, maps["hot"], maps["cold"], c["n_hot"])
        else:
            launches = mo.groups_tier(ids, maps["hot"], maps["host"], c["n_hot"], c["n_cold"],
                                      c["host_in_decode"])
        assert len(launches) == c["launches"]
        for li, (perm, gids, goff) in enumerate(launches):
            pre = f"c{c['case']}_l{li}_"
            assert np.array_equal(perm, route_plan[pre + "perm"]), (c, li)
            assert np.array_equal(gids, route_plan[pre + "gids"]), (c, li)
            assert np.array_equal(goff, route_plan[pre + "goff"]), (c, li)
        # the one-launch definition gives the same tables (EXP/nvfp4_8r_group_plan.py:13-24)
        if kind == "resident":
            gp = mo.group_plan(ids, maps["hot"], maps["hot"], 384, 1, False, False)
        elif kind == "two_tier":
            gp = mo.group_plan(ids, maps["hot"], maps["cold"], c["n_hot"], c["n_cold"], True, True)
        else:
            gp = mo.group_plan(ids, maps["hot"], maps["host"], c["n_hot"], c["n_cold"], True,
                               c["host_in_decode"], maps["iq"])
            assert np.array_equal(gp["iq"], route_plan[f"c{c['case']}_iq"].reshape(-1))
        assert np.array_equal(gp["perm"], launches[0][0])
        assert np.array_equal(gp["gids_hot"], launches[0][1])
        assert np.array_equal(gp["goff_hot"], launches[0][2])
        if len(launches) == 2:
            assert np.array_equal(gp["gids_host"], launches[1][1])
            assert np.array_equal(gp["goff_host"], launches[1][2])


def test_quantizers_round_trip():
    rng = np.random.default_rng(5)
    w = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    codes, sb, g = mo.nvfp4_quantize(w)
    dec = mo.nvfp4_decode(codes, sb, g)
    # every element decodes to the nearest representable value of its block grid
    assert mo.rel_l2(dec, w) < 0.12
    step = (mo.e4m3_to_f32(sb) * g).astype(np.float32)
    assert np.all(np.abs(dec - w).reshape(64, -1, 16) <= step[:, :, None] * 1.0 + 1e-12)
    codes2, e8 = mo.mxfp4_quantize(w)
    dec2 = mo.mxfp4_decode(codes2, e8)
    assert mo.rel_l2(dec2, w) < 0.15
    # exact values survive both quantizers
    exact = (mo.E2M1_VALUES[rng.integers(0, 16, (8, 64))] * 0.25).astype(np.float32)
    c3, e3 = mo.mxfp4_quantize(exact)
    assert np.array_equal(mo.mxfp4_decode(c3, e3), exact)


def test_e4m3_encoder_exhaustive():
    # every finite non-negative E4M3 value encodes to itself
    bits = np.arange(0, 127, dtype=np.uint8)
    vals = mo.e4m3_to_f32(bits)
    assert np.array_equal(mo.e4m3_from_f32(vals), bits)
    # midpoints round to the even code, overflow saturates
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)
    enc = mo.e4m3_from_f32(mids)
    assert np.all((enc == bits[1:]) | (enc == bits[:-1]))
    assert np.all(enc % 2 == 0)
    assert mo.e4m3_from_f32(np.array([1e6], np.float32))[0] == 0x7E


def test_gating_ties_and_weights():
    logits = np.array([[0.5, 2.0, 2.0, -1.0, 2.0, 0.0]], np.float32)
    ids, w = mo.route(logits, 3)
    assert ids.tolist() == [[1, 2, 4]]
    assert np.allclose(w, 1 / 3) and w.dtype == np.float32
    rng = np.random.default_rng(0)
    lg = rng.normal(size=(32, 384)).astype(np.float32)
    ids, w = mo.route(lg, 8)
    p = np.exp(lg.astype(np.float64) - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    ref = np.take_along_axis(p, ids, 1)
    assert np.allclose(w, ref / ref.sum(1, keepdims=True), rtol=1e-6)
    assert np.all(np.diff(np.take_along_axis(lg, ids, 1), axis=1) <= 0)


def test_route_stats_vs_reference_counters():
    """The counter restatement against the reference's RouteStats run on CPU
    tensors over the same 420 decode calls (EXP/nvfp4_8r_stats.py:81-110)."""
    z = np.load(GOLDEN / "route_stats.npz")
    tier, calls = gi.route_stats_inputs()
    c = mo.route_stats_new(384)
    is_host, is_warm = (tier == 2).astype(np.uint8), (tier == 1).astype(np.uint8)
    marks = set(z["marks"].tolist())
    for i, ids in enumerate(calls):
        mo.route_stats_count(c, ids, is_host, is_warm)
        if i in marks:
            for k in ("stat", "gap_hist", "routes", "last_round"):
                np.testing.assert_array_equal(c[k], z[f"{k}_{i}"], err_msg=f"{k} after call {i}")
            np.testing.assert_array_equal(mo.route_stats_recent(c), z[f"recent_{i}"])
    assert np.all(z[f"gap_hist_{max(marks)}"] > 0)  # every bucket was reached


@pytest.mark.parametrize("ggml_type", [17, 29])
def test_iq_formats_vs_gguf(ggml_type):
    """IQ2_XS / IQ1_M decode restatements against gguf-py 0.19.0's dequantize
    (the third-party implementation of ggml's published formats), bit for bit."""
    from gguf import GGMLQuantizationType as Q
    from gguf.quants import dequantize

    rng = np.random.default_rng(700 + ggml_type)
    blocks = mo.iq_random_blocks(rng, ggml_type, 96, 2048, 0.02)
    mine = mo.iq_decode(ggml_type, blocks)
    ref = dequantize(blocks.reshape(96, -1), Q.IQ2_XS if ggml_type == 17 else Q.IQ1_M).astype(np.float32)
    assert np.array_equal(mine.view(np.uint32), ref.reshape(mine.shape).view(np.uint32))
    assert np.abs(mine).mean() > 1e-3


def test_torch_quantizers_match_the_oracle_bit_for_bit():
    """oracle/torch_quant.py (the reference arm's packer, stock torch ops) =
    moe_oracle's quantizers, on seeded data with zero blocks, a zero row,
    binade edges, subnormal-range scales and E4M3 saturation."""
    import torch

    from oracle import torch_quant as tq

    rng = np.random.default_rng(77)
    cases = [rng.normal(0, 0.02, (64, 512)).astype(np.float32),
             (rng.normal(0, 1, (16, 256)) * np.exp2(rng.integers(-30, 10, (16, 1)))).astype(np.float32),
             rng.standard_cauchy((8, 256)).astype(np.float32)]
    edge = rng.normal(0, 1e-3, (8, 256)).astype(np.float32)
    edge[0] = 0.0
    edge[1, :32] = 0.0
    edge[2, :16] = np.float32(6.0) * np.exp2(np.arange(16) - 8).astype(np.float32)
    edge[3, 5] = 1e4  # one huge element: the other blocks' E4M3 scales fall into the subnormal range
    cases.append(edge)
    for w in cases:
        c, s, g = mo.nvfp4_quantize(w)
        tc, ts, tg = tq.nvfp4_quantize(torch.from_numpy(w))
        assert np.array_equal(tc.numpy(), c) and np.array_equal(ts.numpy(), s)
        assert np.float32(tg.item()).view(np.uint32) == np.float32(g).view(np.uint32)
        c, s = mo.mxfp4_quantize(w)
        tc, ts = tq.mxfp4_quantize(torch.from_numpy(w))
        assert np.array_equal(tc.numpy(), c) and np.array_equal(ts.numpy(), s)
