"""The fused two-launch decode of an FP4-only layer (csrc/decode.cu: W13 and W2,
each CTA planning the call and quantizing its chunk's rows itself, W2
combining each token's rows) against the chained six-launch path on the same
layer and inputs: the same output bits, on both FP4 formats, f16 and bf16
activations, 1 to 64 routes, experts with several chunks, routes without an
expert, CUDA graph replay; and against the fp32 dequant-then-matmul reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_ref as tr
from test_gpu_parity import _make_layer

pytestmark = pytest.mark.gpu
H, I, E = 2048, 1024, 64
TOL_FP4 = 2e-3


@pytest.fixture(scope="module")
def dev(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    torch.cuda.set_device(d)
    return d


@pytest.fixture(scope="module", params=["nvfp4", "mxfp4"])
def layer8(request, dev):
    layer, dequant, _, _ = _make_layer(dev, H, I, E, 8, 64, fmt=request.param, seed=31, gemm="fp4")
    yield layer, dequant
    layer.close()


def both_paths(layer, x, ids, w):
    layer.set_decode_fusion(64)
    fused = layer.forward(x, ids, w).clone()
    layer.check_errors()
    layer.set_decode_fusion(0)
    chained = layer.forward(x, ids, w).clone()
    layer.check_errors()
    return fused, chained


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_decode_equals_chained(dev, layer8, m, dtype):
    layer, dequant = layer8
    g = torch.Generator(device=dev).manual_seed(310 + m)
    x = torch.randn((m, H), generator=g, device=dev).to(dtype)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    fused, chained = both_paths(layer, x, ids, w)
    assert torch.equal(fused, chained)
    err = tr.rel_l2(fused, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < TOL_FP4, err
    layer.set_decode_fusion(64)
    assert torch.equal(layer.forward(x, ids, w), fused), "fused decode is not deterministic"
    layer.set_decode_fusion(0)


def test_fused_decode_popular_experts(dev, layer8):
    """Eight tokens on the same few experts: runs of 8 routes split into two
    chunks of four, so CTAs switch chunks inside their item range."""
    layer, dequant = layer8
    m = 8
    g = torch.Generator(device=dev).manual_seed(320)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    logits[:, 3] += 20.0
    logits[:, 7] += 18.0
    logits[:, 11] += 16.0
    ids, w = layer.route(logits)
    assert int((ids == 3).sum()) == m and int((ids == 7).sum()) == m
    fused, chained = both_paths(layer, x, ids, w)
    assert torch.equal(fused, chained)
    assert tr.rel_l2(fused, tr.layer_forward(x, ids.long(), w, dequant)) < TOL_FP4


@pytest.mark.parametrize("k,m", [(4, 16), (1, 64), (2, 1)])
def test_fused_decode_other_top_k(dev, pkg, k, m):
    layer, dequant, _, _ = _make_layer(dev, H, I, E, k, 64, fmt="nvfp4", seed=33, gemm="fp4")
    try:
        g = torch.Generator(device=dev).manual_seed(330 + k)
        x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
        fused, chained = both_paths(layer, x, ids, w)
        assert torch.equal(fused, chained)
        assert tr.rel_l2(fused, tr.layer_forward(x, ids.long(), w, dequant)) < TOL_FP4
    finally:
        layer.close()


def test_fused_decode_route_without_expert(dev, layer8):
    """An id outside [0, E) is refused with B200MOE_ERR_BOUNDS on both paths and
    contributes a zero row: the other routes' sums are the same bits."""
    from b200moe import _lib

    layer, _ = layer8
    m = 4
    g = torch.Generator(device=dev).manual_seed(340)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    ids = ids.clone()
    ids[1, 2] = -1
    ids[3, 0] = E + 5
    outs = []
    for fuse in (64, 0):
        layer.set_decode_fusion(fuse)
        outs.append(layer.forward(x, ids, w).clone())
        with pytest.raises(_lib.B200MoeError, match="BOUNDS"):
            layer.check_errors()
    layer.set_decode_fusion(0)
    assert torch.equal(outs[0], outs[1])
    # and the layer is clean afterwards: a valid call matches the chained path again
    ids2, w2 = layer.route(torch.randn((m, E), generator=g, device=dev))
    fused, chained = both_paths(layer, x, ids2, w2)
    assert torch.equal(fused, chained)


def test_fused_decode_graph_replay(dev, layer8):
    layer, _ = layer8
    layer.set_decode_fusion(64)
    m = 4
    g = torch.Generator(device=dev).manual_seed(350)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    eager = layer.forward(x, *layer.route(logits)).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward(x, *layer.route(logits))
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer.forward(x, *layer.route(logits))
    for _ in range(3):
        layer.out.zero_()
        graph.replay()
    torch.cuda.synchronize()
    layer.check_errors()
    assert torch.equal(out, eager)
    del graph
    layer.set_decode_fusion(0)


def test_fused_decode_perm_matches_plan(dev, layer8):
    """The W13 launch's CTA 0 stores the sorted order the chained route plan
    would (b200moe_debug_perm): stable by expert slot."""
    layer, _ = layer8
    m = 8
    g = torch.Generator(device=dev).manual_seed(360)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = layer.route(torch.randn((m, E), generator=g, device=dev))
    perms = []
    for fuse in (64, 0):
        layer.set_decode_fusion(fuse)
        layer.forward(x, ids, w)
        perms.append(layer.debug_perm(m * 8).cpu().numpy())
    layer.set_decode_fusion(0)
    assert np.array_equal(perms[0], perms[1])
    keys = layer.fp4_slot[ids.reshape(-1).cpu().numpy()]
    assert np.array_equal(perms[0], np.argsort(keys, kind="stable"))
