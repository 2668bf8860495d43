"""GPU parity of the CUDA path (through the C ABI) against the oracle.

Bit-exact: packing (NVFP4 / MXFP4 quantizers, the fold), the route plan
(against the reference's own tables), gating, the SwiGLU step.  Tolerance:
layer outputs within rel-L2 1e-2 of the fp32 dequant-then-matmul reference
(the reference's own acceptance rule, harness/benchmarks/nvfp4_8r/accept_p2.py:36).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import golden_inputs as gi
import torch_ref as tr
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 1e-2  # rel-L2 of a layer output vs the fp32 dequant reference


@pytest.fixture(scope="module")
def dev(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    torch.cuda.set_device(d)
    return d


def sha(a) -> str:
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ------------------------------------------------------------------ packing
def _quant_inputs():
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, (256, 2048)).astype(np.float32)
    w[3, :16] = 0.0                                     # all-zero block
    w[4, :32] = -0.0                                    # negative zeros
    w[5, 16:32] = np.float32(0.001) * mo.E2M1_MAG[rng.integers(0, 8, 16)]  # exact grid values
    w[6, :] = rng.normal(0, 50.0, 2048)                 # large values
    w[7, 32:64] = 1e-30                                 # tiny values
    return w


def test_quantize_nvfp4_bit_exact(dev, pkg):
    from b200moe import packing

    w = _quant_inputs()
    c, s, g = packing.quantize_nvfp4(torch.from_numpy(w).to(dev))
    rc, rs, rg = mo.nvfp4_quantize(w)
    assert np.float32(g.item()).view(np.uint32) == np.float32(rg).view(np.uint32)
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(c.cpu().numpy(), rc)


def test_quantize_mxfp4_bit_exact(dev, pkg):
    from b200moe import packing

    w = _quant_inputs()
    c, e = packing.quantize_mxfp4(torch.from_numpy(w).to(dev))
    rc, re_ = mo.mxfp4_quantize(w)
    assert np.array_equal(e.cpu().numpy(), re_)
    assert np.array_equal(c.cpu().numpy(), rc)


def test_fold_matches_reference_golden(dev, pkg):
    from b200moe import packing

    with np.load(GOLDEN / "packing.npz") as z:
        meta = json.loads(bytes(z["meta"]).decode())
    codes, bits, glob = gi.fold_inputs(True)
    oc, oe = packing.fold_nvfp4_to_mxfp4(torch.from_numpy(codes).to(dev), torch.from_numpy(bits).to(dev),
                                         torch.tensor([glob], device=dev))
    assert sha(oc.cpu().numpy()) == meta["fold_ok"]["codes_sha256"]
    assert sha(oe.cpu().numpy()) == meta["fold_ok"]["scales_sha256"]
    codes, bits, glob = gi.fold_inputs(False)
    with pytest.raises(packing.PackError, match="cannot fold"):
        packing.fold_nvfp4_to_mxfp4(torch.from_numpy(codes).to(dev), torch.from_numpy(bits).to(dev),
                                    torch.tensor([glob], device=dev))


# ------------------------------------------------------------------ routing
def test_route_plan_matches_reference_golden(dev, pkg):
    from b200moe import packing

    with np.load(GOLDEN / "route_plan.npz") as z:
        data = {k: z[k] for k in z.files}
    meta = json.loads(bytes(data["meta"]).decode())
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)  # noqa: E731
    for c in meta:
        j, kind = c["map"], c["kind"]
        ids = data[f"c{c['case']}_ids"]
        hot, cold, host, iq = (data[f"map{j}_{n}"] for n in ("hot", "cold", "host", "iq"))
        if kind == "resident":
            got = packing.route_plan(t(ids), t(hot), None, 384)
        elif kind == "two_tier":
            got = packing.route_plan(t(ids), t(hot), t(cold), c["n_hot"], c["n_cold"], host=True)
        else:
            got = packing.route_plan(t(ids), t(hot), t(host), c["n_hot"], c["n_cold"], host=c["host_in_decode"],
                                     iq_slot=t(iq))
            assert np.array_equal(got["iq"].cpu().numpy(), data[f"c{c['case']}_iq"].reshape(-1))
        want = [(data[f"c{c['case']}_l{li}_perm"], data[f"c{c['case']}_l{li}_gids"],
                 data[f"c{c['case']}_l{li}_goff"]) for li in range(c["launches"])]
        assert np.array_equal(got["perm"].cpu().numpy(), want[0][0]), c
        assert np.array_equal(got["gids_hot"].cpu().numpy(), want[0][1]), c
        assert np.array_equal(got["goff_hot"].cpu().numpy(), want[0][2]), c
        if len(want) == 2:
            assert np.array_equal(got["gids_host"].cpu().numpy(), want[1][1]), c
            assert np.array_equal(got["goff_host"].cpu().numpy(), want[1][2]), c


def test_route_plan_large_and_repeated(dev, pkg):
    from b200moe import packing

    rng = np.random.default_rng(9)
    tier = rng.choice([0, 1, 2], 384, p=[0.5, 0.3, 0.2]).astype(np.int8)
    maps = mo.slot_maps(tier)
    n_hot, n_cold = int((tier == 0).sum()), int((tier != 0).sum())
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)  # noqa: E731
    for ids in (rng.integers(0, 384, (512, 8)), np.full((64, 8), 7), rng.integers(0, 384, (4096, 1))):
        got = packing.route_plan(t(ids), t(maps["hot"]), t(maps["host"]), n_hot, n_cold, host=True,
                                 iq_slot=t(maps["iq"]))
        want = mo.group_plan(ids, maps["hot"], maps["host"], n_hot, n_cold, True, True, maps["iq"])
        for k, v in want.items():
            assert np.array_equal(got[k].cpu().numpy(), v), k


def test_gating_bit_exact(dev, pkg):
    from b200moe import moe

    for (T, E, K) in ((8, 64, 6), (64, 384, 8), (300, 384, 8), (16, 1000, 16), (6, 100, 3)):
        layer = moe.B200NativeMoe(hidden=256, inter=128, num_experts=E, top_k=K, max_tokens=8,
                                  tier=np.zeros(E, np.int8), device=dev)
        rng = np.random.default_rng(T)
        lg = rng.normal(0, 1, (T, E)).astype(np.float32)
        lg[0, :5] = 0.25  # ties
        lg[1, 7] = lg[1, 9] = 3.0
        lg[2, :] = 0.5  # every logit equal: the K smallest ids
        lg[3, :] = -1.0 - np.abs(lg[3, :])  # -0 and +0 on top tie: the smaller id first
        lg[3, 40], lg[3, 3] = -0.0, 0.0
        lg[4, 33::32] = 4.0  # ties in one lane's column across the K boundary
        lg[5, [i for i in (1, 33, 65, 97) if i < E]] = 2.0  # a tie held by one lane in several columns
        ids, w = layer.route(torch.from_numpy(lg).to(dev))
        rid, rw = mo.route(lg, K)
        assert np.array_equal(ids.cpu().numpy(), rid)
        assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32))
        layer.close()


# --------------------------------------------------------------- layers
def _fp4_dequant(bank, fmt, inter):
    def dq(e):
        if fmt == "nvfp4":
            g = bank.globals[e]
            w13 = torch.cat([tr.nvfp4_decode(bank.w13_codes[e, :inter], bank.w13_scales[e, :inter], g[0]),
                             tr.nvfp4_decode(bank.w13_codes[e, inter:], bank.w13_scales[e, inter:], g[1])])
            return w13, tr.nvfp4_decode(bank.w2_codes[e], bank.w2_scales[e], g[2])
        return (tr.mxfp4_decode(bank.w13_codes[e], bank.w13_scales[e]),
                tr.mxfp4_decode(bank.w2_codes[e], bank.w2_scales[e]))
    return dq


def _make_layer(dev, H, I, E, K, max_tokens, fmt="nvfp4", tier=None, seed=0, max_prefill=0, gemm="tcgen05",
                iq_types=(16, 16)):
    from b200moe import moe, synth, tiers

    tier = np.zeros(E, np.int8) if tier is None else tier
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=max_tokens, tier=tier,
                              fp4_format=fmt, device=dev, max_prefill_tokens=max_prefill, prefill_gemm=gemm,
                              iq_types=iq_types)
    n_hot, n_iq = int((tier == tiers.HOT).sum()), int((tier == tiers.WARM).sum())
    fp4 = synth.make_fp4_bank(n_hot, H, I, fmt, seed, dev) if n_hot else None
    iq2 = synth.make_iq2_bank(n_iq, H, I, seed + 1, dev, iq_types=iq_types) if n_iq else None
    if fp4 is not None:
        synth.load_bank(layer, fp4)
    if iq2 is not None:
        layer.set_iq_tables()
        synth.load_bank(layer, iq2)
    layer.check_errors()
    grid, ksigns = mo.iq2xxs_tables()
    fp4_dq = _fp4_dequant(fp4, fmt, I) if fp4 is not None else None

    def iq_dq(t, blocks):
        if t == 16:
            return tr.iq2xxs_decode(blocks, grid, ksigns)
        return torch.from_numpy(mo.iq_decode(t, blocks.cpu().numpy())).to(dev)

    def dequant(e):
        if tier[e] == tiers.HOT:
            return fp4_dq(int(layer.fp4_slot[e]))
        s = int(layer.iq2_slot[e])
        return (torch.cat([iq_dq(iq_types[0], iq2.w1[s]), iq_dq(iq_types[0], iq2.w3[s])]),
                iq_dq(iq_types[1], iq2.w2[s]))

    return layer, dequant, fp4, iq2


def test_torch_ref_matches_oracle(dev, pkg):
    codes, scales, glob = gi.nvfp4_decode_inputs()
    a = tr.nvfp4_decode(torch.from_numpy(codes[:64]).to(dev), torch.from_numpy(scales[:64]).to(dev), glob)
    assert np.array_equal(a.cpu().numpy().view(np.uint32), mo.nvfp4_decode(codes[:64], scales[:64], glob).view(np.uint32))
    grid, ksigns = mo.iq2xxs_tables()
    blocks = gi.iq2_inputs()
    b = tr.iq2xxs_decode(torch.from_numpy(blocks).to(dev), grid, ksigns)
    assert np.array_equal(b.cpu().numpy().view(np.uint32), mo.iq2xxs_decode(blocks, grid, ksigns).view(np.uint32))


def test_c0_layer_vs_numpy_oracle(dev, pkg):
    """Config 0: T=8, hidden 2048, 64 experts, top-6, I=1408, NVFP4, bf16 x."""
    H, I, E, K, T = 2048, 1408, 64, 6, 8
    layer, _, bank, _ = _make_layer(dev, H, I, E, K, 8, seed=0)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    router = torch.randn((E, H), generator=g, device=dev) * 0.02
    logits = (x.float() @ router.T).contiguous()
    ids, w = layer.route(logits)
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    nb = {k: v.cpu().numpy() for k, v in vars(bank).items() if isinstance(v, torch.Tensor)}

    def dequant(e):
        gl = nb["globals"][e]
        return (np.concatenate([mo.nvfp4_decode(nb["w13_codes"][e, :I], nb["w13_scales"][e, :I], gl[0]),
                                mo.nvfp4_decode(nb["w13_codes"][e, I:], nb["w13_scales"][e, I:], gl[1])]),
                mo.nvfp4_decode(nb["w2_codes"][e], nb["w2_scales"][e], gl[2]))

    rid, rw = mo.route(logits.cpu().numpy(), K)
    assert np.array_equal(ids.cpu().numpy(), rid)
    ref = mo.layer_forward(x.float().cpu().numpy(), rid, rw, dequant)
    err = mo.rel_l2(out.cpu().numpy(), ref)
    assert err < TOL, err
    # dequant against fp32 (config 0's check): decode = the fp32 weights' nearest grid values
    layer.close()


@pytest.fixture(scope="module")
def c1(dev, pkg):
    layer, dequant, bank, _ = _make_layer(dev, 4096, 2048, 384, 8, 64, seed=1000)
    yield layer, dequant
    layer.close()


@pytest.mark.parametrize("m", [1, 8, 32, 64])
def test_c1_decode_layer(dev, c1, m):
    layer, dequant = c1
    g = torch.Generator(device=dev).manual_seed(1000 + m)
    x = torch.randn((m, 4096), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, 384), generator=g, device=dev)
    ids, w = layer.route(logits)
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    ref = tr.layer_forward(x, ids.long(), w, dequant)
    err = tr.rel_l2(out, ref)
    assert err < TOL, err
    again = layer.forward(x, ids, w).clone()
    assert torch.equal(out, again), "forward is not deterministic"


def test_c1_graph_replay_equals_eager(dev, c1):
    layer, _ = c1
    m = 6
    g = torch.Generator(device=dev).manual_seed(77)
    x = torch.randn((m, 4096), generator=g, device=dev).to(torch.float16)
    ids, w = layer.route(torch.randn((m, 384), generator=g, device=dev))
    eager = layer.forward(x, ids, w).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward(x, ids, w)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer.forward(x, ids, w)
    layer.out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_swiglu_bit_exact_vs_torch_chain(dev, pkg):
    """The fused SwiGLU = the reference's three torch lines (nvfp4_8r_native.py:937-939)
    applied to the kernel's own fp16 y13, bit for bit."""
    H, I, E, K, M = 1024, 512, 32, 4, 16
    layer, _, _, _ = _make_layer(dev, H, I, E, K, M, seed=5)
    y13 = torch.zeros((M * K, 2 * I), dtype=torch.float16, device=dev)
    layer.set_debug_y13(y13)
    g = torch.Generator(device=dev).manual_seed(5)
    x = (torch.randn((M, H), generator=g, device=dev) * 30).to(torch.float16)  # large: exercises the clamps
    ids, w = layer.route(torch.randn((M, E), generator=g, device=dev))
    layer.forward(x, ids, w)
    inter = layer.debug_inter(M * K)
    layer.check_errors()
    gg = y13[:, :I].float().clamp(max=10.0)
    u = y13[:, I:].float().clamp(-10.0, 10.0)
    chain = (torch.nn.functional.silu(gg) * u).to(torch.float16)
    assert torch.equal(inter.view(torch.int16), chain.view(torch.int16))
    assert (y13.float().abs() > 10).any()  # the clamps were active
    layer.set_debug_y13(None)
    layer.close()


def test_mxfp4_layer(dev, pkg):
    H, I, E, K, M = 1024, 512, 32, 4, 12
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, M, fmt="mxfp4", seed=3)
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn((M, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((M, E), generator=g, device=dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()


def test_mixed_tier_layer(dev, pkg):
    """Config 2 shapes: 150 NVFP4 (HOT) + 234 IQ2_XXS (WARM) experts, Zipf routing, M=32."""
    from b200moe import synth, tiers

    tier, rank = tiers.zipf_tier(384, 150, seed=2)
    layer, dequant, _, _ = _make_layer(dev, 4096, 2048, 384, 8, 32, tier=tier, seed=2)
    g = torch.Generator(device=dev).manual_seed(2032)
    x = torch.randn((32, 4096), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(synth.zipf_logits(32, rank, 1.0, 1.1, 2032, dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    assert (tier[ids.cpu().numpy()] == tiers.WARM).any() and (tier[ids.cpu().numpy()] == tiers.HOT).any()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()


@pytest.mark.parametrize("m", [1, 16, 64])
def test_all_iq2_layer(dev, pkg, m):
    """Every expert IQ2_XXS: the int8 tensor path (two-plane int8 activations)
    against the fp32 dequant-then-matmul reference, with a tighter bar than the
    layer rule, since nothing else in the layer dilutes the IQ2 error."""
    from b200moe import tiers

    E = 64
    tier = np.full(E, tiers.WARM, np.int8)
    layer, dequant, _, _ = _make_layer(dev, 2048, 1024, E, 8, 64, tier=tier, seed=9)
    g = torch.Generator(device=dev).manual_seed(90 + m)
    x = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < 2e-3, err
    layer.close()


@pytest.mark.parametrize("iq_types,m", [((17, 17), 1), ((17, 17), 48), ((29, 29), 8), ((29, 29), 64),
                                        ((17, 29), 16), ((29, 16), 300), ((16, 17), 33)])
def test_iq_types_layer(dev, pkg, iq_types, m):
    """IQ2_XS (17) and IQ1_M (29) experts, alone and mixed per projection with
    IQ2_XXS (16): the int8 tensor path against the fp32 dequant (gguf-py's
    published decode, restated in the oracle) of the same blocks."""
    from b200moe import tiers

    E = 48
    tier = np.full(E, tiers.WARM, np.int8)
    layer, dequant, _, _ = _make_layer(dev, 2048, 1024, E, 8, 64, tier=tier, seed=19, max_prefill=300,
                                       iq_types=iq_types)
    g = torch.Generator(device=dev).manual_seed(190 + m)
    x = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    out = (layer.forward(x, ids, w) if m <= 64 else layer.forward_prefill(x, ids, w)).clone()
    layer.check_errors()
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < 2e-3, err
    layer.close()


def test_iq_types_mixed_with_fp4(dev, pkg):
    """NVFP4 HOT experts beside IQ1_M gate/up + IQ2_XS down WARM experts."""
    from b200moe import synth, tiers

    tier, rank = tiers.zipf_tier(96, 40, seed=5)
    layer, dequant, _, _ = _make_layer(dev, 2048, 1024, 96, 8, 32, tier=tier, seed=5, iq_types=(29, 17))
    g = torch.Generator(device=dev).manual_seed(55)
    x = torch.randn((32, 2048), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(synth.zipf_logits(32, rank, 1.0, 1.1, 55, dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    assert (tier[ids.cpu().numpy()] == tiers.WARM).any() and (tier[ids.cpu().numpy()] == tiers.HOT).any()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()


@pytest.mark.parametrize("m,mixed,fmt", [(1, False, "nvfp4"), (8, False, "nvfp4"), (64, False, "nvfp4"),
                                         (300, False, "nvfp4"), (32, True, "nvfp4"), (600, True, "nvfp4"),
                                         (1, False, "mxfp4"), (64, False, "mxfp4"), (300, True, "mxfp4"),
                                         (600, False, "mxfp4")])
def test_block_scaled_fp4_path(dev, pkg, m, mixed, fmt):
    """prefill_gemm="fp4": the FP4 bank on tcgen05.mma.kind::mxf4nvf4 (E2M1 x E2M1
    with E4M3 block scales per 16 for NVFP4, E8M0 per 32 for MXFP4; activations
    as four E2M1 planes), decode and prefill, against the fp32
    dequant-then-matmul reference.  Prefills of >= 4096 routes (m = 600) run
    the same weight units through the tcgen05 f16 grouped GEMM."""
    from b200moe import tiers

    H, I, E, K = 2048, 1024, 64, 8
    tier = tiers.zipf_tier(E, 40, seed=5)[0] if mixed else np.zeros(E, np.int8)
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, 64, fmt=fmt, tier=tier, seed=13, max_prefill=max(300, m),
                                       gemm="fp4")
    g = torch.Generator(device=dev).manual_seed(130 + m)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    out = (layer.forward(x, ids, w) if m <= 64 else layer.forward_prefill(x, ids, w)).clone()
    layer.check_errors()
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < 2e-3, err
    again = (layer.forward(x, ids, w) if m <= 64 else layer.forward_prefill(x, ids, w)).clone()
    layer.check_errors()
    assert torch.equal(again, out)  # deterministic
    layer.close()


@pytest.mark.parametrize("gemm,fmt", [("fp4-bs", "nvfp4"), ("fp4-bs", "mxfp4"), ("fp4", "nvfp4")])
def test_long_prefill_on_the_weight_units(dev, pkg, gemm, fmt):
    """Prefills of >= 4096 routes of a block-scaled layer: "fp4-bs" runs them
    on the block-scaled kernel with 32-route chunks (one accumulator buffer,
    the epilogue in slices of four routes); "fp4" on the tcgen05 f16 GEMM over
    the same weight units.  Both against the fp32 dequant reference, on a
    skewed mixed-tier routing (experts with 1 to ~100 routes: full, partial
    and single-route chunks)."""
    from b200moe import tiers

    H, I, E, K, m = 2048, 1024, 64, 8, 700
    tier = tiers.zipf_tier(E, 40, seed=9)[0]
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, 64, fmt=fmt, tier=tier, seed=19, max_prefill=m, gemm=gemm)
    g = torch.Generator(device=dev).manual_seed(190)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    logits[:, :8] += 2.0  # a few popular experts: chunks of 32 and partial ones
    ids, w = layer.route(logits)
    out = layer.forward_prefill(x, ids, w).clone()
    layer.check_errors()
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < 2e-3, err
    again = layer.forward_prefill(x, ids, w)
    layer.check_errors()
    assert torch.equal(again, out)
    layer.close()


def test_prefill_and_apply(dev, pkg):
    from b200moe import moe

    H, I, E, K = 1024, 512, 32, 4
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, 4, seed=4, max_prefill=300)
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn((300, H), generator=g, device=dev).to(torch.float16)
    ids, w = layer.route(torch.randn((300, E), generator=g, device=dev))
    out = layer.forward_prefill(x, ids, w)
    layer.check_errors()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    method = moe.B200NativeMoEMethod(layer)

    class FakeLayer:
        apply_router_weight_on_input = False
        activation = "silu"

    y = method.apply(FakeLayer(), x[:3], w[:3], ids[:3].long())
    assert y.dtype == torch.float16 and y.shape == (3, H)
    assert torch.equal(y, out[:3].to(torch.float16)) or tr.rel_l2(y.float(), out[:3]) < 1e-3
    y = method.apply(FakeLayer(), x, w, ids)
    assert y.shape == (300, H)
    layer.close()


def test_bad_expert_id_reports_bounds_then_recovers(dev, pkg):
    from b200moe import _lib

    H, I, E, K, M = 512, 256, 16, 4, 4
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, M, seed=6)
    x = torch.randn((M, H), device=dev).to(torch.float16)
    ids = torch.tensor([[0, 1, 2, 3], [4, 5, 999, 7], [8, 9, 10, 11], [-1, 13, 14, 15]], dtype=torch.int32, device=dev)
    w = torch.full((M, K), 0.25, device=dev)
    layer.forward(x, ids, w)
    with pytest.raises(_lib.B200MoeError, match="BOUNDS"):
        layer.check_errors()
    ids[1, 2] = 6
    ids[3, 0] = 12
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()


# ------------------------------------------------------- prefill on tcgen05
@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
def test_prefill_tcgen05_vs_reference_and_skinny(dev, pkg, fmt):
    """configs[3]-shaped layer (hidden 4096, inter 2048, top-8) at 32 experts:
    ~128 routes per expert, so token tiles are full, partial and split."""
    from b200moe import moe, synth

    H, I, E, K, T = 4096, 2048, 32, 8, 512
    outs = {}
    for mode in ("tcgen05", "skinny"):
        layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=4, tier=np.zeros(E, np.int8),
                                  fp4_format=fmt, device=dev, max_prefill_tokens=T, prefill_gemm=mode)
        bank = synth.make_fp4_bank(E, H, I, fmt, 31, dev)
        synth.load_bank(layer, bank)
        g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = layer.route(torch.rand((T, E), generator=g, device=dev))
        out = layer.forward_prefill(x, ids, w)
        again = layer.forward_prefill(x, ids, w)
        layer.check_errors()
        assert torch.equal(out, again), "prefill is not deterministic"
        outs[mode] = out
        if mode == "tcgen05":
            ref = tr.layer_forward(x, ids.long(), w, _fp4_dequant(bank, fmt, I))
            assert tr.rel_l2(out, ref) < TOL
        layer.close()
    assert tr.rel_l2(outs["tcgen05"], outs["skinny"]) < 2e-3


def test_prefill_tcgen05_skewed_mixed_tier(dev, pkg):
    """Zipf routing (some experts > 128 routes, some with one) over an NVFP4
    bank on tcgen05 plus an IQ2_XXS bank on the skinny kernels, sharing one
    combine."""
    from b200moe import synth, tiers

    H, I, E, K, T = 4096, 2048, 48, 8, 384
    tier, rank = tiers.zipf_tier(E, 30, seed=9)
    layer, dequant, _, _ = _make_layer(dev, H, I, E, K, 4, tier=tier, seed=9, max_prefill=T)
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.float16)
    ids, w = layer.route(synth.zipf_logits(T, rank, 2.0, 1.1, 9, dev))
    counts = torch.bincount(ids.reshape(-1).long(), minlength=E)
    assert counts.max() > 128 and (counts[counts > 0].min() < 16)
    out = layer.forward_prefill(x, ids, w)
    layer.check_errors()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()


# ------------------------------------------------------------------ pack loading
@pytest.mark.parametrize("gemm", ["tcgen05", "fp4"])
def test_pack_layer_load(dev, pkg, tmp_path, gemm):
    """Whole MXFP4 experts -> the reference's four TP-rank records -> a v2
    pack on disk -> load_pack_layer: the layer's output matches the fp32
    dequant of the original experts; an EP rank loads only its own experts."""
    from b200moe import moe, packs, tiers

    H, I, E, K, M = 1024, 512, 16, 4, 9
    geom = packs.PackGeometry(hidden=H, tp_inter=I // 4, w2_k=I // 4 + 32, tp_ranks=4, num_experts=E, num_layers=40)
    rng = np.random.default_rng(31)
    q13 = [mo.mxfp4_quantize(rng.normal(0, 0.02, (2 * I, H)).astype(np.float32)) for _ in range(E)]
    q2 = [mo.mxfp4_quantize(rng.normal(0, 0.02, (H, I)).astype(np.float32)) for _ in range(E)]
    full = (np.stack([c for c, _ in q13]), np.stack([s for _, s in q13]), np.stack([c for c, _ in q2]),
            np.stack([s for _, s in q2]))
    recs = packs.split_expert(*full, geom=geom)
    packs.write_id_order_pack(tmp_path, {(3, r): rec for r, rec in enumerate(recs)}, geom)
    tier = np.zeros(E, np.int8)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier,
                              fp4_format="mxfp4", device=dev, prefill_gemm=gemm)
    assert packs.load_pack_layer(layer, tmp_path, 3, geom, chunk=5) == E
    d = [torch.from_numpy(a).to(dev) for a in full]

    def dequant(e):
        return tr.mxfp4_decode(d[0][e], d[1][e]), tr.mxfp4_decode(d[2][e], d[3][e])

    g = torch.Generator(device=dev).manual_seed(31)
    x = torch.randn((M, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((M, E), generator=g, device=dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    assert tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant)) < TOL
    layer.close()
    owner = tiers.balanced_owners(tier, 2)
    part = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=1, max_tokens=64, tier=tier,
                             fp4_format="mxfp4", device=dev, prefill_gemm=gemm, rank=1, world=2, owner=owner)
    assert packs.load_pack_layer(part, tmp_path, 3, geom) == int((owner == 1).sum())
    part.close()


# ------------------------------------------------------------------ route counters
def test_route_stats_kernel(dev, pkg):
    """b200moe_route_stats against the reference's RouteStats counters (the
    golden run of 420 decode calls), bit for bit, eagerly and as graph replays."""
    from b200moe import stats

    tier, calls = gi.route_stats_inputs()
    z = np.load(GOLDEN / "route_stats.npz")
    marks = set(z["marks"].tolist())
    rs = stats.RouteStats(tier, dev)
    for i, ids in enumerate(calls):
        rs.count(torch.from_numpy(ids).to(dev))
        if i in marks:
            got = rs.read()
            for k in ("stat", "gap_hist", "recent", "routes"):
                np.testing.assert_array_equal(got[k], z[f"{k}_{i}"], err_msg=f"{k} after call {i}")
            np.testing.assert_array_equal(rs.last_round.cpu().numpy(), z[f"last_round_{i}"])
    rs.check_errors()
    # captured once, replayed: the counters keep counting (round = replays so far)
    rs2 = stats.RouteStats(tier, dev)
    c = mo.route_stats_new(384)
    ids = torch.from_numpy(calls[7]).to(dev)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            rs2.count(ids)
    torch.cuda.current_stream(dev).wait_stream(side)
    for _ in range(300):
        graph.replay()
        mo.route_stats_count(c, calls[7], (tier == 2).astype(np.uint8), (tier == 1).astype(np.uint8))
    torch.cuda.synchronize(dev)
    got = rs2.read()
    for k in ("stat", "gap_hist", "routes"):
        np.testing.assert_array_equal(got[k], c[k])
    del graph
    with pytest.raises(RuntimeError):
        rs2.count(torch.tensor([[3, 400]], dtype=torch.int32, device=dev))
        rs2.check_errors()


def test_layer_route_stats(dev, pkg):
    """A layer with its counters on: every decode forward adds its routes."""
    H, I, E, K, M = 1024, 512, 32, 4, 12
    layer, _, _, _ = _make_layer(dev, H, I, E, K, M, seed=4)
    st = layer.enable_route_stats()
    g = torch.Generator(device=dev).manual_seed(4)
    want = np.zeros(E, np.int64)
    for m in (M, 3):
        x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
        layer.forward(x, ids, w)
        want += np.bincount(ids.cpu().numpy().reshape(-1), minlength=E)
    got = st.read()
    np.testing.assert_array_equal(got["routes"], want)
    assert got["stat"].tolist()[:2] == [2, int(want.sum())] and got["stat"][2] == 0
    layer.check_errors()
    layer.close()


def test_back_to_back_calls_match_isolated_calls(dev, pkg):
    """The forward's launches overlap their predecessors' tails (programmatic
    dependent launch): a kernel may start while the one before it finishes and
    must wait before touching that kernel's memory.  Calls of every shape class
    on two block-scaled layers (FP4-only and mixed tier), queued back to back
    on one stream without synchronization, give the bits each call gives when
    run alone: 1 and 4 tokens (plan and planes in one launch, combine in the W2
    epilogue), 8 (combine in the epilogue), 32 (separate combine), a 600-token
    prefill (the tcgen05 GEMM), in an order that makes every pair of shapes
    neighbours."""
    from b200moe import tiers

    H, I, E, K = 2048, 1024, 64, 8
    a, _, _, _ = _make_layer(dev, H, I, E, K, 64, seed=41, max_prefill=600, gemm="fp4")
    b, _, _, _ = _make_layer(dev, H, I, E, K, 64, tier=tiers.zipf_tier(E, 40, seed=6)[0], seed=43, max_prefill=600,
                             gemm="fp4")
    try:
        g = torch.Generator(device=dev).manual_seed(410)
        calls = []
        for layer, m in ((a, 1), (b, 32), (a, 600), (b, 4), (a, 8), (b, 600), (a, 32), (b, 1), (a, 4), (b, 8)):
            x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
            ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
            calls.append((layer, x, ids, w, m > 64))
        torch.cuda.synchronize()

        def run(layer, x, ids, w, prefill):
            out = layer.forward_prefill(x, ids, w) if prefill else layer.forward(x, ids, w)
            return out.clone()

        alone = []
        for c in calls:
            alone.append(run(*c))
            torch.cuda.synchronize()
        queued = [run(*c) for c in calls]  # no synchronization between calls
        torch.cuda.synchronize()
        a.check_errors()
        b.check_errors()
        for i, (p, q) in enumerate(zip(alone, queued)):
            assert torch.equal(p, q), f"call {i} differs when queued behind the others"
    finally:
        a.close()
        b.close()


_PLAIN_LAUNCH_SCRIPT = r"""
import sys, numpy as np, torch
for sub in ("", "/tests", "/tests/golden"):
    sys.path.insert(0, sys.argv[1] + sub)
from __graft_entry__ import load_package
load_package()
from test_gpu_parity import _make_layer
dev = torch.device("cuda", 0)
layer, _, _, _ = _make_layer(dev, 2048, 1024, 64, 8, 64, seed=51, gemm="fp4")
g = torch.Generator(device=dev).manual_seed(510)
outs = []
for m in (1, 8, 64):
    x = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, 64), generator=g, device=dev))
    outs.append(layer.forward(x, ids, w).clone().cpu().numpy())
layer.check_errors()
np.savez(sys.argv[2], *outs)
"""


def test_plain_launches_give_the_same_bits(dev, pkg, tmp_path):
    """B200MOE_PDL=0 launches every forward kernel without programmatic stream
    serialization (read once per process): a child process run that way gives
    the bits of this process's programmatic launches, at 1, 8 and 64 tokens."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    out = tmp_path / "plain.npz"
    env = dict(os.environ, B200MOE_PDL="0")
    subprocess.run([sys.executable, "-c", _PLAIN_LAUNCH_SCRIPT, str(root), str(out)], env=env, check=True,
                   timeout=600)
    plain = np.load(out)
    layer, _, _, _ = _make_layer(dev, 2048, 1024, 64, 8, 64, seed=51, gemm="fp4")
    try:
        g = torch.Generator(device=dev).manual_seed(510)
        for i, m in enumerate((1, 8, 64)):
            x = torch.randn((m, 2048), generator=g, device=dev).to(torch.bfloat16)
            ids, w = layer.route(torch.randn((m, 64), generator=g, device=dev))
            got = layer.forward(x, ids, w).clone().cpu().numpy()
            assert np.array_equal(got.view(np.uint32), plain[f"arr_{i}"].view(np.uint32)), m
        layer.check_errors()
    finally:
        layer.close()
