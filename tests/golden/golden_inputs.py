"""Seeded inputs of the golden fixtures.

Shared by ``make_golden.py`` (which runs the reference on them once) and the
tests (which regenerate them and run the oracle or the CUDA path on them).
Everything here is deterministic numpy; nothing reads the reference tree.
"""

from __future__ import annotations

import numpy as np

ROUTE_PLAN_SEED = 20261201
SAMPLE_ROWS = np.array([0, 1, 17, 511, 1024, 2047, 2303], np.int64)


def _e4m3_finite_bytes(rng, shape):
    b = rng.integers(0, 256, size=shape, dtype=np.uint8)
    nan = (b & 127) == 127
    b[nan] = b[nan] & 0xF7  # 0x7F -> 0x77: finite
    return b


def nvfp4_decode_inputs():
    """One w1 projection at the reference checkpoint geometry (2304 x 5120):
    random E2M1 codes, random finite E4M3 scales, a fixed global."""
    rng = np.random.default_rng(101)
    rows, cols = 2304, 5120
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = _e4m3_finite_bytes(rng, (rows, cols // 16))
    return codes, scales, np.float32(3.0517578e-05)


def mxfp4_decode_inputs():
    """A raw MXFP4 record section (codes then E8M0) for accept_p1.packed_projection."""
    rng = np.random.default_rng(102)
    rows, cols = 576, 5120
    codes = rng.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
    scales = rng.integers(100, 140, size=rows * cols // 32, dtype=np.uint8)
    return np.concatenate([codes, scales]), rows, cols


def fold_inputs(foldable: bool):
    """A C0-shaped W13 projection [2816, 2048] in NVFP4.  Foldable: both
    16-halves of every 32-block share a power-of-two E4M3 scale, so the E8M0/32
    fold is exact.  Not foldable: one block pair gets scales 1.5 and 1.0."""
    rng = np.random.default_rng(103 if foldable else 104)
    rows, cols = 2816, 2048
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    # powers of two in E4M3: exponent field 1..14, mantissa 0 -> 2^(e-7)
    e = rng.integers(1, 15, size=(rows, cols // 32), dtype=np.uint8)
    bits = np.repeat((e << 3).astype(np.uint8), 2, axis=1)
    if not foldable:
        bits[5, 6] = (7 << 3) | 4  # 1.5
        bits[5, 7] = 7 << 3        # 1.0
        codes[5, 48:64] = 0x77     # every element of that 32-block is +-6 magnitude
    return codes, bits, np.float32(0.125)


def contribution_inputs():
    rng = np.random.default_rng(105)
    h, i = 96, 40
    w1 = rng.normal(0, 0.2, (i, h))
    w3 = rng.normal(0, 0.2, (i, h))
    w2 = rng.normal(0, 0.2, (h, i))
    x = rng.normal(0, 1, h).astype(np.float16)
    return w1, w3, w2, x, 0.37


SWIGLU_SPECIALS = np.array([0x0000, 0x8000, 0x7C00, 0xFC00, 0x7E00, 0x4900, 0xC900, 0x4901, 0xC901,
                            0x7BFF, 0xFBFF, 0x0001, 0x8001, 0x0400, 0x8400], np.uint16)


def swiglu_inputs():
    """y13 fp16 [48, 2 * 576]: normal values times 4 with the fp16 specials
    (+-0, +-inf, NaN, +-10, +-10.0078, +-65504, smallest subnormal and normal)
    in the first columns of gate and up, rolled per row."""
    rng = np.random.default_rng(106)
    s, inter = 48, 576
    y = (rng.standard_normal((s, 2 * inter)) * 4).astype(np.float16)
    sp = SWIGLU_SPECIALS.view(np.float16)
    for r in range(s):
        y[r, : sp.size] = sp
        y[r, inter: inter + sp.size] = np.roll(sp, r)
    return y


def iq2_inputs():
    """Random valid IQ2_XXS blocks [64 rows, 8 blocks, 66 bytes]."""
    rng = np.random.default_rng(107)
    rows, nb = 64, 8
    out = rng.integers(0, 256, size=(rows, nb, 66), dtype=np.uint8)
    d = (0.02 / 48.0) * rng.uniform(0.5, 1.5, size=(rows, nb))
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return out
