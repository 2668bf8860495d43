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
    lay = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=16, tier=tier, device=dev,
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
    for m, dtype in ((16, torch.bfloat16), (5, torch.float16)):  # two calls in a row, different shapes
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
