"""The route plan of large prefill calls (at least 4,096 routes), which runs on
one CTA per 1,024 routes plus a CTA for the chunk tables (csrc/route.cu): the
sorted order is exactly the stable argsort by expert key, as the one-CTA plan's
is (nvfp4_8r_native.py:806-822), for uniform, skewed and ragged route counts,
routes without an expert sorted last with B200MOE_ERR_BOUNDS reported; and the
layer output through that plan matches the fp32 dequant-then-matmul reference
on both prefill GEMMs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torch_ref as tr
from test_gpu_parity import _make_layer

pytestmark = pytest.mark.gpu
H, I, E, K = 256, 256, 384, 8
TOL = 1e-2


@pytest.fixture(scope="module")
def dev(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d = torch.device("cuda", 0)
    torch.cuda.set_device(d)
    return d


@pytest.fixture(scope="module", params=["tcgen05", "fp4-bs"])
def layer(request, dev):
    lay, dequant, _, _ = _make_layer(dev, H, I, E, K, 64, fmt="mxfp4", seed=41, max_prefill=1536,
                                     gemm=request.param)
    yield lay, dequant
    lay.close()


def stable_order(layer, ids: np.ndarray) -> np.ndarray:
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    keys = np.where(valid, layer.fp4_slot[np.clip(flat, 0, E - 1)], E)
    return np.argsort(keys, kind="stable")


@pytest.mark.parametrize("m,skew", [(512, False), (777, False), (1536, False), (1024, True)])
def test_wide_plan_is_the_stable_order(dev, layer, m, skew):
    lay, dequant = layer
    g = torch.Generator(device=dev).manual_seed(400 + m)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.float16)
    logits = torch.randn((m, E), generator=g, device=dev)
    if skew:  # a few experts take most routes: runs far longer than one CTA's 1,024
        logits[:, 5] += 30.0
        logits[:, 200] += 25.0
        logits[: m // 2, 17] += 20.0
    ids, w = lay.route(logits)
    out = lay.forward_prefill(x, ids, w)
    lay.check_errors()
    perm = lay.debug_perm(m * K).cpu().numpy()
    assert np.array_equal(perm, stable_order(lay, ids.cpu().numpy()))
    err = tr.rel_l2(out, tr.layer_forward(x, ids.long(), w, dequant))
    assert err < TOL, err


def test_wide_plan_routes_without_expert(dev, layer):
    from b200moe import _lib

    lay, dequant = layer
    m = 640
    g = torch.Generator(device=dev).manual_seed(450)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.float16)
    ids, w = lay.route(torch.randn((m, E), generator=g, device=dev))
    ids = ids.clone()
    ids[3, 1] = -1
    ids[600, 7] = E + 2
    ids[601, :] = -5  # every route of one token
    out = lay.forward_prefill(x, ids, w)
    with pytest.raises(_lib.B200MoeError, match="BOUNDS"):
        lay.check_errors()
    perm = lay.debug_perm(m * K).cpu().numpy()
    assert np.array_equal(perm, stable_order(lay, ids.cpu().numpy()))
    assert torch.count_nonzero(out[601]) == 0
    keep = torch.ones(m, dtype=torch.bool, device=dev)
    keep[[3, 600, 601]] = False
    ids_ok = ids.clone().long()
    w_ok = w.clone()
    bad = (ids_ok < 0) | (ids_ok >= E)
    ids_ok[bad] = 0
    w_ok[bad] = 0.0
    want = tr.layer_forward(x, ids_ok, w_ok, dequant)
    assert tr.rel_l2(out[keep], want[keep]) < TOL
    assert tr.rel_l2(out[[3, 600]], want[[3, 600]]) < TOL


def test_wide_plan_repeats_bit_exactly(dev, layer):
    lay, _ = layer
    m = 1200
    g = torch.Generator(device=dev).manual_seed(460)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.float16)
    ids, w = lay.route(torch.randn((m, E), generator=g, device=dev))
    a = lay.forward_prefill(x, ids, w)
    b = lay.forward_prefill(x, ids, w)
    lay.check_errors()
    assert torch.equal(a, b)
