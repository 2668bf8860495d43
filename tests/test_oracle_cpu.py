"""The C oracle against the numpy oracle and against the reference's own CPU
expert kernel (built from its source by ``oracle/Makefile``)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cpu_layer
from oracle import moe_oracle as mo


def _expert(rng, fmt, hidden, inter, scale=0.02):
    w13 = rng.normal(0, scale, (2 * inter, hidden)).astype(np.float32)
    w2 = rng.normal(0, scale, (hidden, inter)).astype(np.float32)
    if fmt == 0:
        c1, s1, g1 = mo.nvfp4_quantize(w13[:inter])
        c3, s3, g3 = mo.nvfp4_quantize(w13[inter:])
        c2, s2, g2 = mo.nvfp4_quantize(w2)
        ex = dict(fmt=0, w13c=np.concatenate([c1, c3]), w13s=np.concatenate([s1, s3]),
                  g13=np.array([g1, g3], np.float32), w2c=c2, w2s=s2, g2=g2)
        deq = (np.concatenate([mo.nvfp4_decode(c1, s1, g1), mo.nvfp4_decode(c3, s3, g3)]),
               mo.nvfp4_decode(c2, s2, g2))
    else:
        c13, s13 = mo.mxfp4_quantize(w13)
        c2, s2 = mo.mxfp4_quantize(w2)
        ex = dict(fmt=1, w13c=c13, w13s=s13, g13=np.ones(2, np.float32), w2c=c2, w2s=s2,
                  g2=np.float32(1))
        deq = (mo.mxfp4_decode(c13, s13), mo.mxfp4_decode(c2, s2))
    return ex, deq


@pytest.mark.parametrize("avx2", [False, True])
@pytest.mark.parametrize("fmt", [0, 1])
def test_c_oracle_matches_numpy_layer(fmt, avx2):
    """Both C forms (the scalar checker and the AVX2 timed baseline) against
    the numpy oracle in fp64; m = 21 routes per expert crosses the AVX2 form's
    8-row groups."""
    rng = np.random.default_rng(11 + fmt)
    hidden, inter, e, k, m = 256, 128, 6, 3, 43
    experts = [_expert(rng, fmt, hidden, inter) for _ in range(e)]
    x = rng.normal(0, 1, (m, hidden)).astype(np.float32)
    ids, w = mo.route(rng.normal(0, 1, (m, e)).astype(np.float32), k)
    cpu = cpu_layer.CpuMoe(hidden, inter, avx2=avx2)
    got = cpu.forward(x, ids, w, [ex for ex, _ in experts])
    want = mo.layer_forward(x, ids, w, lambda i: experts[i][1], dtype=np.float64)
    assert mo.rel_l2(got, want) < 1e-5
    # C dequant = numpy decode, bit for bit
    ex, deq = experts[0]
    g = ex["g13"][0] if fmt == 0 else 1.0
    d = cpu.dequant(fmt, ex["w13c"][:inter], ex["w13s"][:inter], g)
    assert np.array_equal(d.view(np.uint32), deq[0][:inter].view(np.uint32))


def test_c_oracle_matches_reference_cpu_kernel():
    if not cpu_layer.REF_LIB.exists():
        try:
            cpu_layer.build(ref=True)
        except Exception:
            pytest.skip("reference tree not present: the reference CPU kernel cannot be built here")
    ref = cpu_layer.RefCpuExpert()
    rng = np.random.default_rng(3)
    H, I = ref.HIDDEN, ref.INTER
    ex, deq = _expert(rng, 1, H, I)
    rec = ref.record(ex["w13c"], ex["w13s"], ex["w2c"], ex["w2s"])
    x = rng.normal(0, 1, (4, H)).astype(np.float32)
    rows = np.array([0, 2, 3], np.int32)
    w = np.array([0.5, 0.25, 0.125], np.float32)
    want = np.zeros((4, H), np.float32)
    ref.expert(rec, x, rows, w, want)
    for avx2 in (False, True):
        got = np.zeros((4, H), np.float32)
        cpu_layer.CpuMoe(H, I, avx2=avx2).expert(ex, x, rows, w, got)
        assert mo.rel_l2(got, want) < 1e-5


def test_threads_follow_the_affinity_not_omp_num_threads(monkeypatch):
    """torchrun sets OMP_NUM_THREADS=1; the CPU baseline still uses every core
    the process may run on."""
    import os

    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    assert cpu_layer.threads() == len(os.sched_getaffinity(0))
