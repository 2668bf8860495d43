"""The allocation-free decode forward (b200moe_forward_static) against b200moe_forward.

b200moe_forward_static exists for callers that may not allocate device memory
when they run a decode step (for example an engine that has given all free
HBM to its KV cache); it keeps its scratch in one array built into the library.
This file is collected last so that a failure here comes after every other
test has run; it also passes alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch

import torch_ref as tr

pytestmark = pytest.mark.gpu
TOL = 1e-2  # the layer tolerance every other parity test uses (rel-L2)


@pytest.fixture(scope="module", params=["tcgen05", "fp4"])
def layer(pkg, request):
    """Decode on the skinny GEMV ("tcgen05" layers) and on the block-scaled FP4
    tensor path ("fp4" layers, whose plane buffers are the layer's own)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from b200moe import moe, synth, tiers

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, I, E, K = 4096, 2048, 64, 8
    tier, _ = tiers.zipf_tier(E, 40, seed=11)  # both banks: 40 NVFP4 + 24 IQ2_XXS experts
    lay = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=32, tier=tier, device=dev,
                            prefill_gemm=request.param)
    synth.load_bank(lay, synth.make_fp4_bank(int((tier == tiers.HOT).sum()), H, I, "nvfp4", 11, dev))
    lay.set_iq2_tables()
    synth.load_bank(lay, synth.make_iq2_bank(int((tier == tiers.WARM).sum()), H, I, 12, dev))
    lay.check_errors()
    yield lay
    lay.close()


def test_static_forward_matches_forward_on_two_calls(layer):
    dev = layer.device
    g = torch.Generator(device=dev).manual_seed(123)
    # calls in a row, different shapes: 16 tokens (separate combine launch), 5 (combine in the W2 epilogue),
    # 2 (route plan and x planes in one launch on the block-scaled path)
    for m, dtype in ((16, torch.bfloat16), (5, torch.float16), (2, torch.bfloat16)):
        x = torch.randn((m, layer.hidden), generator=g, device=dev).to(dtype)
        ids, w = layer.route(torch.randn((m, layer.num_experts), generator=g, device=dev))
        out = torch.full((m, layer.hidden), float("nan"), dtype=torch.float32, device=dev)
        got = layer.forward_static(x, ids, w, out)
        want = layer.forward(x, ids, w).clone()
        layer.check_errors()
        assert got.data_ptr() == out.data_ptr()
        assert torch.isfinite(got).all()
        assert tr.rel_l2(got, want) < TOL
        assert torch.equal(got, want)  # same kernels, same order: bit-equal in practice


def test_static_forward_graph_replay(layer):
    """forward_static captured in a CUDA graph (its array's address is looked
    up when the layer is made, so no call has to come first outside a
    capture): every replay gives the eager call's bits."""
    dev = layer.device
    g = torch.Generator(device=dev).manual_seed(321)
    m = 8
    x = torch.randn((m, layer.hidden), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, layer.num_experts), generator=g, device=dev))
    eager = layer.forward_static(x, ids, w, torch.empty((m, layer.hidden), dtype=torch.float32, device=dev)).clone()
    layer.check_errors()
    out = torch.full((m, layer.hidden), float("nan"), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward_static(x, ids, w, out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer.forward_static(x, ids, w, out)
    for _ in range(3):
        out.fill_(float("nan"))
        graph.replay()
    torch.cuda.synchronize()
    layer.check_errors()
    assert torch.equal(out, eager)
    del graph


def test_static_forward_refuses_sizes_beyond_its_array(layer):
    from b200moe import _lib

    dev = layer.device
    m = 17  # above the array's 16-token limit
    x = torch.zeros((m, layer.hidden), dtype=torch.float16, device=dev)
    ids = torch.zeros((m, layer.top_k), dtype=torch.int32, device=dev)
    w = torch.zeros((m, layer.top_k), dtype=torch.float32, device=dev)
    out = torch.zeros((m, layer.hidden), dtype=torch.float32, device=dev)
    with pytest.raises(_lib.B200MoeError, match="B200MOE_ERR_RANGE"):
        layer.forward_static(x, ids, w, out)
    m = layer.max_tokens + 1  # above the layer's own decode limit, as b200moe_forward refuses it
    x = torch.zeros((m, layer.hidden), dtype=torch.float16, device=dev)
    ids = torch.zeros((m, layer.top_k), dtype=torch.int32, device=dev)
    w = torch.zeros((m, layer.top_k), dtype=torch.float32, device=dev)
    out = torch.zeros((m, layer.hidden), dtype=torch.float32, device=dev)
    with pytest.raises(_lib.B200MoeError, match="B200MOE_ERR_INVALID_ARG"):
        layer.forward_static(x, ids, w, out)


@pytest.mark.parametrize("gemm", ["tcgen05", "fp4"])
def test_static_forward_at_the_chunk_limit_with_iq2xs_and_iq1m(pkg, gemm):
    """512 experts held (the array's limit), 16 tokens x top-8 on 128 distinct
    experts (the most route chunks a call can make), IQ2_XS gate/up and IQ1_M
    down beside NVFP4: bit-equal to b200moe_forward with no kernel error."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from b200moe import moe, synth, tiers

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, I, E, K, M = 512, 256, 512, 8, 16
    tier = tiers.zipf_tier(E, 256, seed=5)[0]
    lay = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=16, tier=tier, device=dev,
                            prefill_gemm=gemm, iq_types=(17, 29))
    try:
        synth.load_bank(lay, synth.make_fp4_bank(int((tier == tiers.HOT).sum()), H, I, "nvfp4", 21, dev))
        synth.load_bank(lay, synth.make_iq2_bank(int((tier == tiers.WARM).sum()), H, I, 22, dev, iq_types=(17, 29)))
        lay.check_errors()
        g = torch.Generator(device=dev).manual_seed(7)
        ids = torch.randperm(E, generator=g, device=dev)[:M * K].to(torch.int32).reshape(M, K).contiguous()
        w = torch.rand((M, K), generator=g, device=dev)
        w = (w / w.sum(1, keepdim=True)).contiguous()
        for call in range(2):
            x = torch.randn((M, H), generator=g, device=dev).to(torch.bfloat16)
            out = torch.full((M, H), float("nan"), dtype=torch.float32, device=dev)
            got = lay.forward_static(x, ids, w, out)
            want = lay.forward(x, ids, w).clone()
            lay.check_errors()
            assert torch.isfinite(got).all()
            assert tr.rel_l2(got, want) < TOL
            assert torch.equal(got, want), f"call {call}"
    finally:
        lay.close()
