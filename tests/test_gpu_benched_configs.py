"""GPU parity at the exact configurations bench.py times, through the C ABI,
against the plain fp32 dequant-then-matmul reference (tests/torch_ref.py):

- configs[1] on the block-scaled FP4 tensor path (the bench default): hidden
  4096, inter 2048, 384 NVFP4 experts, top-8, M = 1 / 8 / 32 / 64 with the
  bench's seeds; four E2M1 activation planes, so the bar is rel-L2 2e-3;
- configs[2] on the same path: 150 NVFP4 + 234 IQ2_XXS experts, M = 32;
- configs[3] on the default prefill path (the tcgen05 grouped GEMM over the
  block-scaled layout's weight units): T = 4096, 384 MXFP4 experts, a seeded
  sample of 256 tokens checked.

The reference's own acceptance rule is rel-L2 1e-2
(harness/benchmarks/nvfp4_8r/accept_p2.py:36); the FP4 path is held to 2e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_ref as tr

pytestmark = pytest.mark.gpu
H, I, E, K = 4096, 2048, 384, 8
TOL_FP4 = 2e-3
TOL_LAYER = 1e-2


@pytest.fixture(scope="module")
def dev(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    torch.cuda.set_device(d)
    return d


def fp4_dequant(bank, inter):
    def deq(j):
        if bank.fmt == "nvfp4":
            g = bank.globals[j]
            w13 = torch.cat([tr.nvfp4_decode(bank.w13_codes[j, :inter], bank.w13_scales[j, :inter], g[0]),
                             tr.nvfp4_decode(bank.w13_codes[j, inter:], bank.w13_scales[j, inter:], g[1])])
            return w13, tr.nvfp4_decode(bank.w2_codes[j], bank.w2_scales[j], g[2])
        return tr.mxfp4_decode(bank.w13_codes[j], bank.w13_scales[j]), tr.mxfp4_decode(bank.w2_codes[j],
                                                                                         bank.w2_scales[j])
    return deq


@pytest.fixture(scope="module")
def c1(dev):
    from b200moe import moe, synth

    bank = synth.make_fp4_bank(E, H, I, "nvfp4", 1000, dev)  # bench.py's configs[1] bank
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=np.zeros(E, np.int8),
                              device=dev, prefill_gemm="fp4")
    synth.load_bank(layer, bank)
    layer.check_errors()
    yield layer, fp4_dequant(bank, I)
    layer.close()
    del bank
    torch.cuda.empty_cache()


@pytest.mark.parametrize("m", [1, 8, 32, 64])
def test_c1_block_scaled_decode_at_bench_shape(dev, c1, m):
    layer, dequant = c1
    g = torch.Generator(device=dev).manual_seed(1000 + m)  # bench.py's inputs of this M
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    out = layer.forward(x, ids, w).clone()
    layer.check_errors()
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < TOL_FP4, err
    assert torch.equal(layer.forward(x, ids, w), out), "forward is not deterministic"


def test_c1_block_scaled_graph_replay_equals_eager(dev, c1):
    layer, _ = c1
    g = torch.Generator(device=dev).manual_seed(1064)
    x = torch.randn((64, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((64, E), generator=g, device=dev)
    eager = layer.forward(x, *layer.route(logits)).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward(x, *layer.route(logits))
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer.forward(x, *layer.route(logits))
    layer.out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    layer.check_errors()
    assert torch.equal(out, eager)


def test_c2_mixed_tier_at_bench_shape(dev, pkg):
    from gguf.quants import IQ2_XXS

    from b200moe import moe, synth, tiers

    tier, tier_rank = tiers.zipf_tier(E, 150, seed=2)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier, device=dev,
                              prefill_gemm="fp4")
    try:
        fp4 = synth.make_fp4_bank(150, H, I, "nvfp4", 2000, dev)
        synth.load_bank(layer, fp4)
        iq2 = synth.make_iq2_bank(E - 150, H, I, 2001, dev)
        layer.set_iq_tables()
        synth.load_bank(layer, iq2)
        layer.check_errors()
        IQ2_XXS.init_grid()
        grid = np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.int8)
        ksigns = np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
        fdeq = fp4_dequant(fp4, I)

        def deq(e):
            if layer.fp4_slot[e] >= 0:
                return fdeq(int(layer.fp4_slot[e]))
            s = int(layer.iq2_slot[e])
            return (torch.cat([tr.iq2xxs_decode(iq2.w1[s], grid, ksigns), tr.iq2xxs_decode(iq2.w3[s], grid, ksigns)]),
                    tr.iq2xxs_decode(iq2.w2[s], grid, ksigns))

        logits = synth.zipf_logits(32, tier_rank, 0.8, 1.1, 2032, dev)
        g = torch.Generator(device=dev).manual_seed(2032)
        x = torch.randn((32, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = layer.route(logits)
        out = layer.forward(x, ids, w).clone()
        layer.check_errors()
        hot = float(torch.from_numpy(layer.fp4_slot >= 0).to(dev)[ids.long()].float().mean())
        assert 0.5 < hot < 1.0  # both banks are on the path
        err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, deq))
        assert err < TOL_LAYER, err
    finally:
        layer.close()
        torch.cuda.empty_cache()


def test_c3_prefill_at_bench_shape(dev, pkg):
    from b200moe import moe, synth

    T = 4096
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=8, tier=np.zeros(E, np.int8),
                              fp4_format="mxfp4", device=dev, max_prefill_tokens=T, prefill_gemm="fp4")
    try:
        bank = synth.make_fp4_bank(E, H, I, "mxfp4", 3000, dev)  # bench.py's configs[3] bank and inputs
        synth.load_bank(layer, bank)
        layer.check_errors()
        g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = layer.route(torch.rand((T, E), generator=g, device=dev))
        out = layer.forward_prefill(x, ids, w)
        layer.check_errors()
        rows = torch.as_tensor(np.sort(np.random.default_rng(3).choice(T, 256, replace=False)), device=dev)
        ref = tr.layer_forward(x[rows], ids[rows].long(), w[rows], fp4_dequant(bank, I))
        err = tr.rel_l2(out[rows], ref)
        assert err < TOL_FP4, err
        again = layer.forward_prefill(x, ids, w)
        layer.check_errors()
        assert torch.equal(again, out), "prefill is not deterministic"
    finally:
        layer.close()
        torch.cuda.empty_cache()


def test_tensor_peak_microbenchmark(dev, pkg):
    """b200moe_mma_peak runs every MMA kind the kernels use and reports a
    throughput in the range of a B200 (the pool's cuBLAS bf16 burst is ~1.6
    PFLOP/s dense; FP8 about twice, FP4 about four times that)."""
    import ctypes

    from b200moe import _lib

    got = {}
    for kind in range(5):
        tf, ms = ctypes.c_float(), ctypes.c_float()
        _lib.check("b200moe_mma_peak", _lib.lib().b200moe_mma_peak(0, kind, 20000, ctypes.byref(tf),
                                                                   ctypes.byref(ms)))
        assert ms.value > 0
        got[kind] = tf.value
    assert 500 < got[0] < 3000, got
    assert got[1] > 1.3 * got[0] and got[2] > 1.3 * got[1], got
