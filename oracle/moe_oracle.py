"""CPU oracle for the routed-expert MoE path.

TEST INFRASTRUCTURE ONLY.  This module is the checker, never the product: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  The product path lives in the
package's CUDA library and fails loudly when that library is missing.

It restates, in numpy, the arithmetic of the reference build
(ProprietaryLegal/Volta-Max-uPLIft-FP4-DeepSeek-V4.1-Flash-1017-NVFP4-8xV100-SXM2-PP2xTP4).
Paths below are relative to that project; each function names the lines it
follows.  ``EXP/`` = ``engine/src/vllm/model_executor/layers/fused_moe/experts/``,
``HB/`` = ``harness/benchmarks/nvfp4_8r/``.

Pinning (what ties this oracle to the reference):
- the NVFP4 / MXFP4 decode formulas, the NVFP4 -> MXFP4 fold, the route-plan
  chain and the slot maps are checked against golden vectors produced by
  importing the reference's own Python (``tests/golden/make_golden.py``);
- the IQ2_XXS decode is checked against gguf-py 0.19.0's ``dequantize``
  (the reference calls it at ``HB/make_t3_refs.py:61-64``);
- the NVFP4 and MXFP4 *quantizers* and the softmax/top-k gating have no
  counterpart in the reference (NVIDIA made the packs, the engine owns the
  router): they are this build's own definitions, checked only for round-trip
  consistency with the pinned decode formulas ("parity unpinned" for those two).
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# FP4 / FP8 element formats
# ---------------------------------------------------------------------------

#: E2M1 magnitudes by 3-bit code (HB/accept_p1.py:78, HB/build_packs.py MAG).
E2M1_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
#: Signed E2M1 values by 4-bit code, bit 3 = sign (HB/accept_p1.py:92-94).
E2M1_VALUES = np.concatenate([E2M1_MAG, -E2M1_MAG]).astype(np.float32)

NVFP4_BLOCK = 16
MXFP4_BLOCK = 32
IQ2_BLOCK = 256
IQ2_BLOCK_BYTES = 66
#: 6 * 448: the largest E2M1 magnitude times the largest finite E4M3 value.
NVFP4_GLOBAL_DIVISOR = np.float32(2688.0)


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    """E4M3FN byte -> float32: sign bit, bias 7, three fraction bits,
    subnormal step 2^-9 (HB/accept_p1.py:64-71).  0x7F / 0xFF (NaN) are refused."""
    bits = np.asarray(bits, np.uint8)
    if np.any((bits & 127) == 127):
        raise ValueError("NaN E4M3FN code")
    exp = ((bits >> 3) & 15).astype(np.int32)
    man = (bits & 7).astype(np.float32)
    mag = np.where(exp == 0, man * np.float32(2.0**-9), np.ldexp(1 + man / 8, exp - 7))
    return np.where(bits & 128, -mag, mag).astype(np.float32)


def e4m3_from_f32(x: np.ndarray) -> np.ndarray:
    """Non-negative float32 -> E4M3FN byte, round to nearest even, saturating
    at 448 (0x7E).  This build's own rounding rule (the reference ships no
    NVFP4 quantizer); the CUDA packer implements the same integer steps."""
    x = np.asarray(x, np.float32)
    if np.any(~np.isfinite(x)) or np.any(x < 0):
        raise ValueError("E4M3 scale input must be finite and non-negative")
    xd = x.astype(np.float64)
    _, ex = np.frexp(xd)
    e = np.maximum(ex.astype(np.int32) - 1, -6)  # floor(log2 x), subnormal floor -6
    quantum = np.ldexp(1.0, e - 3)
    q = np.rint(xd / quantum) * quantum  # exact: power-of-two quantum, half-even
    q = np.minimum(q, 448.0)
    # encode q (a representable E4M3 value) back to bits
    out = np.zeros(x.shape, np.uint8)
    nz = q > 0
    _, qe = np.frexp(q[nz])
    qe = qe.astype(np.int32) - 1
    sub = qe < -6
    man_sub = np.rint(np.ldexp(q[nz], 9)).astype(np.int32)
    man_norm = np.rint((np.ldexp(q[nz], -qe) - 1.0) * 8).astype(np.int32)
    enc = np.where(sub, man_sub, ((qe + 7) << 3) | man_norm)
    out[nz] = enc.astype(np.uint8)
    return out


def e2m1_code(t: np.ndarray) -> np.ndarray:
    """|t| (float32, >= 0) -> 3-bit E2M1 magnitude code, round to nearest with
    ties to the even code, saturating at 6.  Thresholds are the midpoints of
    E2M1_MAG; at a midpoint the even code (low bit 0) wins."""
    t = np.asarray(t, np.float32)
    c = ((t > 0.25).astype(np.uint8) + (t >= 0.75) + (t > 1.25) + (t >= 1.75)
         + (t > 2.5) + (t >= 3.5) + (t > 5.0))
    return c.astype(np.uint8)


def _nibbles(codes: np.ndarray) -> np.ndarray:
    """uint8 [..., K/2] -> uint8 [..., K]; the low nibble is the even element
    (HB/cpu_mxfp4_moe.c:1-3, HB/accept_p1.py:75-76)."""
    out = np.empty(codes.shape[:-1] + (codes.shape[-1] * 2,), np.uint8)
    out[..., 0::2] = codes & 15
    out[..., 1::2] = codes >> 4
    return out


def _pack_nibbles(nib: np.ndarray) -> np.ndarray:
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).astype(np.uint8)


# ---------------------------------------------------------------------------
# NVFP4 and MXFP4: decode (pinned) and quantize (this build's rule)
# ---------------------------------------------------------------------------

def nvfp4_decode(codes: np.ndarray, scales: np.ndarray, global_scale) -> np.ndarray:
    """NVFP4 projection -> float32 [R, K]: (E2M1 * E4M3 block scale) * global,
    FP32, in that order (HB/accept_p1.py:53-84)."""
    rows = codes.shape[0]
    k = codes.shape[1] * 2
    block = e4m3_to_f32(scales).reshape(rows, k // NVFP4_BLOCK)
    g = np.float32(global_scale)
    if not np.isfinite(g):
        raise ValueError("nonfinite NVFP4 global scale")
    values = E2M1_VALUES[_nibbles(codes)].reshape(rows, k // NVFP4_BLOCK, NVFP4_BLOCK)
    values = values * block[:, :, None]
    return (values * g).astype(np.float32).reshape(rows, k)


def mxfp4_decode(codes: np.ndarray, e8m0: np.ndarray) -> np.ndarray:
    """MXFP4 projection -> float32 [R, K]: E2M1 * 2^(e - 127), E8M0 255
    refused (HB/accept_p1.py:87-101)."""
    rows = codes.shape[0]
    k = codes.shape[1] * 2
    e8m0 = np.asarray(e8m0, np.uint8).reshape(rows, k // MXFP4_BLOCK)
    if np.any(e8m0 == 255):
        raise ValueError("invalid E8M0 pack scales")
    values = E2M1_VALUES[_nibbles(codes)].reshape(rows, k // MXFP4_BLOCK, MXFP4_BLOCK)
    return np.ldexp(values, e8m0.astype(np.int32)[:, :, None] - 127).astype(np.float32).reshape(rows, k)


def nvfp4_quantize(w: np.ndarray):
    """float32 [R, K] -> (codes uint8 [R, K/2], E4M3 scales uint8 [R, K/16],
    global float32).  This build's quantizer: global = amax / 2688 (amax over
    the projection; 1.0 when it is all zero); block scale = E4M3(RNE) of
    block_amax / (6 * global); element code = E2M1(RNE) of w / (scale * global),
    sign bit = w < 0.  All divisions are IEEE float32 round-to-nearest."""
    w = np.ascontiguousarray(w, np.float32)
    rows, k = w.shape
    if k % NVFP4_BLOCK:
        raise ValueError("K must be a multiple of 16")
    amax = np.float32(np.max(np.abs(w))) if w.size else np.float32(0)
    glob = np.float32(amax / NVFP4_GLOBAL_DIVISOR) if amax > 0 else np.float32(1.0)
    denom = np.float32(np.float32(6.0) * glob)
    blk = np.abs(w).reshape(rows, k // NVFP4_BLOCK, NVFP4_BLOCK).max(axis=2)
    sbits = e4m3_from_f32((blk / denom).astype(np.float32))
    qscale = (e4m3_to_f32(sbits) * glob).astype(np.float32)  # decode step per block
    safe = np.where(qscale > 0, qscale, np.float32(1.0)).astype(np.float32)
    t = (np.abs(w).reshape(rows, -1, NVFP4_BLOCK) / safe[:, :, None]).astype(np.float32)
    mag = np.where(qscale[:, :, None] > 0, e2m1_code(t), 0).astype(np.uint8)
    sign = (w.reshape(rows, -1, NVFP4_BLOCK) < 0).astype(np.uint8) << 3
    nib = (mag | sign).reshape(rows, k)
    return _pack_nibbles(nib), sbits, glob


def mxfp4_quantize(w: np.ndarray):
    """float32 [R, K] -> (codes uint8 [R, K/2], E8M0 uint8 [R, K/32]).  The
    block exponent is the smallest e with 6 * 2^e >= block_amax (the exponent
    choice of the reference's exact fold, HB/build_packs.py:131-136); element
    code = E2M1(RNE) of w / 2^e, sign bit = w < 0."""
    w = np.ascontiguousarray(w, np.float32)
    rows, k = w.shape
    if k % MXFP4_BLOCK:
        raise ValueError("K must be a multiple of 32")
    blk = np.abs(w).reshape(rows, k // MXFP4_BLOCK, MXFP4_BLOCK).max(axis=2)
    m, ex = np.frexp(blk.astype(np.float64))
    e = np.where(m <= 0.75, ex - 3, ex - 2).astype(np.int32)
    e = np.where(blk > 0, e, 0)
    if np.any((e < -127) | (e > 127)):
        raise ValueError("block exponent outside the E8M0 range")
    t = np.ldexp(np.abs(w).reshape(rows, -1, MXFP4_BLOCK), -e[:, :, None]).astype(np.float32)
    mag = e2m1_code(t)
    sign = (w.reshape(rows, -1, MXFP4_BLOCK) < 0).astype(np.uint8) << 3
    nib = (mag | sign).reshape(rows, k)
    return _pack_nibbles(nib), (e + 127).astype(np.uint8)


def fold_nvfp4_to_mxfp4(codes: np.ndarray, scales: np.ndarray, global_scale):
    """Exact NVFP4 -> MXFP4 (E8M0 per 32) or ValueError at the first loss.

    Same steps as the reference's offline fold (HB/build_packs.py:120-151):
    per 16-block the largest decoded magnitude, per 32-block the larger of
    its two halves, exponent = ceil(log2(max32 / 6)) (0 for an all-zero
    block), then every decoded value v of the block must equal
    E2M1_MAG[c] * 2^exponent for some code c, found by searching E2M1_MAG for
    v * 2^-exponent; the sign bit is carried over."""
    rows, half_k = codes.shape
    block = e4m3_to_f32(scales).reshape(rows, half_k * 2 // NVFP4_BLOCK)
    g = np.float32(global_scale)
    nib = _nibbles(codes).reshape(rows, -1, NVFP4_BLOCK)
    mag16 = E2M1_MAG[nib & 7].max(axis=2)
    max16 = ((mag16 * block) * g).astype(np.float32)
    max32 = max16.reshape(rows, -1, 2).max(axis=2)
    expo = np.zeros(max32.shape, np.int32)
    pos = max32 > 0
    expo[pos] = np.ceil(np.log2(max32[pos].astype(np.float64) / 6)).astype(np.int32)
    if np.any((expo < -127) | (expo > 127)):
        raise ValueError("exact E8M0 exponent is outside the finite range")
    expo16 = np.repeat(expo, 2, axis=1)
    # decoded magnitude of every code of every 16-block, in the decode's order
    value = ((E2M1_MAG[None, None, :] * block[:, :, None]) * g).astype(np.float32)
    target = np.ldexp(value, -expo16[:, :, None])
    mapped = np.clip(np.searchsorted(E2M1_MAG, target), 0, 7).astype(np.uint8)
    exact = np.ldexp(E2M1_MAG[mapped], expo16[:, :, None]) == value
    used_ok = np.take_along_axis(exact, (nib & 7).astype(np.int64), axis=2)
    if not used_ok.all():
        raise ValueError("NVFP4 block cannot fold exactly to MXFP4 E8M0/32")
    new_mag = np.take_along_axis(mapped, (nib & 7).astype(np.int64), axis=2)
    new_nib = (new_mag | (nib & 8)).reshape(rows, -1)
    return _pack_nibbles(new_nib), (expo + 127).astype(np.uint8)


# ---------------------------------------------------------------------------
# IQ2_XXS (ggml type 16): 66 bytes per 256 weights
# ---------------------------------------------------------------------------

def iq2xxs_tables():
    """(grid int8 [256, 8], ksigns uint8 [128]) from gguf-py 0.19.0 at run time.
    The codebook is ggml data; it is loaded, not written out here."""
    from gguf.quants import IQ2_XXS

    IQ2_XXS.init_grid()
    grid = np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.int8)
    ksigns = np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
    return grid, ksigns


def iq2xxs_decode(blocks: np.ndarray, grid: np.ndarray, ksigns: np.ndarray) -> np.ndarray:
    """IQ2_XXS blocks uint8 [R, K/256, 66] -> float32 [R, K].

    ggml's published decode (gguf-py 0.19.0 ``IQ2_XXS.dequantize_blocks``):
    d = fp16 bytes 0..1; per 32-value sub-block ib, word a = u32 at 2+8ib
    (four grid indices, one byte each), word b = u32 at 6+8ib (four 7-bit sign
    indices at bits 0,7,14,21 and a 4-bit scale at bits 28..31);
    db = d * (0.5 + scale) * 0.25; value[32ib + 8l + j] = db * grid[a.byte(l)][j]
    negated when bit j of ksigns[(b >> 7l) & 127] is set."""
    blocks = np.asarray(blocks, np.uint8)
    rows, nb, nbytes = blocks.shape
    if nbytes != IQ2_BLOCK_BYTES:
        raise ValueError("IQ2_XXS blocks are 66 bytes")
    d = blocks[..., :2].copy().view(np.float16).astype(np.float32).reshape(rows, nb)
    qs = blocks[..., 2:].copy().view(np.uint32).reshape(rows, nb, 8, 2)
    a, b = qs[..., 0], qs[..., 1]
    db = (d[..., None] * (np.float32(0.5) + (b >> 28).astype(np.float32))) * np.float32(0.25)
    gidx = np.ascontiguousarray(a).view(np.uint8).reshape(rows, nb, 8, 4)
    vals = grid[gidx].astype(np.float32)  # [R, nb, 8, 4, 8]
    sidx = (b[..., None] >> np.array([0, 7, 14, 21], np.uint32)) & 127
    sbyte = ksigns[sidx]  # [R, nb, 8, 4]
    neg = (sbyte[..., None] >> np.arange(8, dtype=np.uint8)) & 1
    sgn = np.where(neg == 1, np.float32(-1), np.float32(1))
    out = (db[..., None, None] * vals) * sgn
    return out.astype(np.float32).reshape(rows, nb * IQ2_BLOCK)


def iq2xxs_random_blocks(rng: np.random.Generator, rows: int, k: int, wscale: float) -> np.ndarray:
    """Seeded random *valid* IQ2_XXS blocks: every byte pattern of the 64 qs
    bytes is a legal block (any grid index, sign index and 4-bit scale); d is
    fp16 sized so the decoded weights have roughly ``wscale`` spread."""
    if k % IQ2_BLOCK:
        raise ValueError("K must be a multiple of 256")
    nb = k // IQ2_BLOCK
    out = rng.integers(0, 256, size=(rows, nb, IQ2_BLOCK_BYTES), dtype=np.uint8)
    d = (wscale / 48.0) * rng.uniform(0.75, 1.25, size=(rows, nb))
    out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return out


IQ2XS_BLOCK_BYTES = 74
IQ1M_BLOCK_BYTES = 56
IQ1M_DELTA = np.float32(0.125)


def iq_tables(ggml_type: int):
    """(grid int8 [n, 8], ksigns uint8 [128] or None) of GGML type 16 (IQ2_XXS),
    17 (IQ2_XS) or 29 (IQ1_M), from gguf-py 0.19.0 at run time (ggml data)."""
    from gguf.quants import IQ1_M, IQ2_XS, IQ2_XXS

    cls = {16: IQ2_XXS, 17: IQ2_XS, 29: IQ1_M}[ggml_type]
    cls.init_grid()
    grid = np.asarray(cls.grid, np.float32).reshape(-1, 8).astype(np.int8)
    ksigns = None if ggml_type == 29 else np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
    return grid, ksigns


def iq2xs_decode(blocks: np.ndarray, grid: np.ndarray, ksigns: np.ndarray) -> np.ndarray:
    """IQ2_XS blocks uint8 [R, K/256, 74] -> float32 [R, K].

    ggml's published decode (gguf-py 0.19.0 ``IQ2_XS.dequantize_blocks``):
    d = fp16 bytes 0..1, 32 u16 qs at 2..65, 8 scale bytes at 66..73; group
    g = 4ib + l of 8 values (sub-block ib, entry l) takes grid[qs[g] & 511],
    negated per bit j of ksigns[qs[g] >> 9]; its scale is
    db = d * (0.5 + s) * 0.25, s = low nibble of scale byte ib for l < 2, high
    nibble for l >= 2."""
    blocks = np.asarray(blocks, np.uint8)
    rows, nb, nbytes = blocks.shape
    if nbytes != IQ2XS_BLOCK_BYTES:
        raise ValueError("IQ2_XS blocks are 74 bytes")
    d = blocks[..., :2].copy().view(np.float16).astype(np.float32).reshape(rows, nb)
    qs = blocks[..., 2:66].copy().view(np.uint16).reshape(rows, nb, 32)
    sc = blocks[..., 66:74]
    s = np.stack([sc & 15, sc >> 4], axis=-1).reshape(rows, nb, 16).astype(np.float32)  # per 16 values
    db = (d[..., None] * (np.float32(0.5) + s)) * np.float32(0.25)
    vals = grid[(qs & 511).astype(np.int64)].astype(np.float32)  # [R, nb, 32, 8]
    neg = (ksigns[(qs >> 9).astype(np.int64)][..., None] >> np.arange(8, dtype=np.uint8)) & 1
    sgn = np.where(neg == 1, np.float32(-1), np.float32(1))
    out = (np.repeat(db, 2, axis=-1)[..., None] * vals) * sgn
    return out.astype(np.float32).reshape(rows, nb * IQ2_BLOCK)


def iq1m_decode(blocks: np.ndarray, grid: np.ndarray) -> np.ndarray:
    """IQ1_M blocks uint8 [R, K/256, 56] -> float32 [R, K].

    ggml's published decode (gguf-py 0.19.0 ``IQ1_M.dequantize_blocks``):
    qs bytes 0..31, qh bytes 32..47, four u16 scale words at 48..55.  d is the
    fp16 whose four nibbles are the words' top nibbles (word 0 lowest); the
    3-bit scale s of the 16-value half i is bits 3(i % 4).. of word i // 4,
    dl = d * (2s + 1).  Group g of 8 values takes nibble g % 2 of qh byte g // 2:
    bits 0..2 extend qs[g] to an 11-bit grid index, bit 3 makes delta -1/8
    (else +1/8); value = dl * (grid + delta)."""
    blocks = np.asarray(blocks, np.uint8)
    rows, nb, nbytes = blocks.shape
    if nbytes != IQ1M_BLOCK_BYTES:
        raise ValueError("IQ1_M blocks are 56 bytes")
    qs = blocks[..., :32].astype(np.int64)
    qh = blocks[..., 32:48]
    w = blocks[..., 48:56].copy().view(np.uint16).reshape(rows, nb, 4).astype(np.uint32)
    dbits = ((w[..., 0] >> 12) | ((w[..., 1] >> 8) & 0xF0) | ((w[..., 2] >> 4) & 0xF00) | (w[..., 3] & 0xF000))
    d = dbits.astype(np.uint16).view(np.float16).astype(np.float32)
    s = ((w[..., :, None] >> np.array([0, 3, 6, 9], np.uint32)) & 7).reshape(rows, nb, 16).astype(np.float32)
    dl = d[..., None] * (np.float32(2) * s + np.float32(1))  # [R, nb, 16]
    nib = np.stack([qh & 15, qh >> 4], axis=-1).reshape(rows, nb, 32)
    idx = qs | ((nib & 7).astype(np.int64) << 8)
    delta = np.where((nib & 8) == 0, IQ1M_DELTA, -IQ1M_DELTA).astype(np.float32)
    vals = grid[idx].astype(np.float32) + delta[..., None]  # [R, nb, 32, 8]
    out = np.repeat(dl, 2, axis=-1)[..., None] * vals
    return out.astype(np.float32).reshape(rows, nb * IQ2_BLOCK)


def iq_random_blocks(rng: np.random.Generator, ggml_type: int, rows: int, k: int, wscale: float) -> np.ndarray:
    """Seeded random valid blocks of IQ2_XXS (16), IQ2_XS (17) or IQ1_M (29):
    every pattern of the index, sign and scale bits is legal; the fp16 d is set
    so the decoded weights have roughly ``wscale`` spread."""
    if ggml_type == 16:
        return iq2xxs_random_blocks(rng, rows, k, wscale)
    if k % IQ2_BLOCK:
        raise ValueError("K must be a multiple of 256")
    nb = k // IQ2_BLOCK
    if ggml_type == 17:
        out = rng.integers(0, 256, size=(rows, nb, IQ2XS_BLOCK_BYTES), dtype=np.uint8)
        d = (wscale / 48.0) * rng.uniform(0.75, 1.25, size=(rows, nb))
        out[..., :2] = d.astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
        return out
    if ggml_type == 29:
        out = rng.integers(0, 256, size=(rows, nb, IQ1M_BLOCK_BYTES), dtype=np.uint8)
        d = ((wscale / 6.0) * rng.uniform(0.75, 1.25, size=(rows, nb))).astype(np.float16).view(np.uint16)
        w = out[..., 48:56].copy().view(np.uint16).reshape(rows, nb, 4) & np.uint16(0x0FFF)
        for i in range(4):  # d's nibble i in word i's top nibble
            w[..., i] |= ((d >> np.uint16(4 * i)) & np.uint16(15)) << np.uint16(12)
        out[..., 48:56] = w.view(np.uint8).reshape(rows, nb, 8)
        return out
    raise ValueError(f"GGML type {ggml_type} is not IQ2_XXS / IQ2_XS / IQ1_M")


def iq_decode(ggml_type: int, blocks: np.ndarray) -> np.ndarray:
    grid, ksigns = iq_tables(ggml_type)
    if ggml_type == 16:
        return iq2xxs_decode(blocks, grid, ksigns)
    if ggml_type == 17:
        return iq2xs_decode(blocks, grid, ksigns)
    return iq1m_decode(blocks, grid)


# ---------------------------------------------------------------------------
# Router gating (this build's definition; the engine's router is not in the mount)
# ---------------------------------------------------------------------------

def route(logits: np.ndarray, k: int):
    """Softmax top-k with renormalised weights.

    ids: the k largest logits per row, larger first, ties to the smaller
    expert id (softmax is monotone, so selecting on logits selects on
    probabilities).  weights: e_i = exp(l_i - l_max) in float64 for the
    selected experts, summed in rank order, w_i = float32(e_i / sum).  The
    full softmax denominator cancels in the renormalisation."""
    logits = np.asarray(logits, np.float32)
    t, e = logits.shape
    if not np.all(np.isfinite(logits)):
        raise ValueError("router logits must be finite")
    if not 1 <= k <= e:
        raise ValueError("bad top-k")
    order = np.lexsort((np.broadcast_to(np.arange(e), (t, e)), -logits.astype(np.float64)), axis=1)
    ids = order[:, :k].astype(np.int32)
    sel = np.take_along_axis(logits, ids, axis=1).astype(np.float64)
    ex = np.exp(sel - sel[:, :1])
    total = np.zeros(t, np.float64)
    for j in range(k):
        total = total + ex[:, j]
    return ids, (ex / total[:, None]).astype(np.float32)


# ---------------------------------------------------------------------------
# Route plan: the reference chain (EXP/nvfp4_8r_native.py:806-872)
# ---------------------------------------------------------------------------

def compact(keys: np.ndarray):
    """Stable sort of per-route keys into groups (EXP/nvfp4_8r_native.py:806-822):
    perm = stable argsort; a group starts where the sorted key changes;
    goff[g] = first sorted position of group g (n past the last group);
    gids[g] = the group's key (0 past the last group)."""
    keys = np.asarray(keys, np.int64).reshape(-1)
    n = keys.size
    perm = np.argsort(keys, kind="stable").astype(np.int32)
    sk = keys[perm]
    new_group = np.ones(n, bool)
    new_group[1:] = sk[1:] != sk[:-1]
    gidx = np.cumsum(new_group) - 1
    goff = np.full(n + 1, n, np.int64)
    starts = np.flatnonzero(new_group)
    goff[gidx[starts]] = starts
    gids = np.zeros(n, np.int64)
    gids[gidx[starts]] = sk[starts]
    return perm, gids, goff, sk, new_group


def groups_resident(ids: np.ndarray, hot_slot: np.ndarray):
    """One launch, every expert resident (EXP/nvfp4_8r_native.py:824-827)."""
    flat = hot_slot[np.asarray(ids).reshape(-1)].astype(np.int64)
    perm, gids, goff, _, _ = compact(flat)
    return [(perm, gids.astype(np.int32), goff.astype(np.int32))]


def groups_split(ids, hot_slot, cold_slot, n_hot: int):
    """HBM launch plus host launch (EXP/nvfp4_8r_native.py:829-843)."""
    flat = np.asarray(ids).reshape(-1)
    n = flat.size
    hot = hot_slot[flat].astype(np.int64)
    key = np.where(hot >= 0, hot, n_hot + cold_slot[flat].astype(np.int64))
    perm, gids, goff, sk, ng = compact(key)
    count_hot = int((key < n_hot).sum())
    groups_hot = int((ng & (sk < n_hot)).sum())
    gids_h = np.where(gids < n_hot, gids, 0).astype(np.int32)
    goff_h = np.minimum(goff, count_hot).astype(np.int32)
    idx = np.minimum(np.arange(n + 1) + groups_hot, n)
    goff_c = goff[idx].astype(np.int32)
    gids_c = np.maximum(gids[np.minimum(idx[:n], n - 1)] - n_hot, 0).astype(np.int32)
    return [(perm, gids_h, goff_h), (perm, gids_c, goff_c)]


def groups_tier(ids, hot_slot, host_slot, n_hot: int, n_cold: int, host_in_decode: bool):
    """Three-tier launches (EXP/nvfp4_8r_native.py:845-872): HOT slots first,
    HOST slots next, one sentinel key for every WARM route."""
    flat = np.asarray(ids).reshape(-1)
    n = flat.size
    hot = hot_slot[flat].astype(np.int64)
    host = host_slot[flat].astype(np.int64)
    key = np.where(hot >= 0, hot, np.where(host >= 0, n_hot + host, n_hot + n_cold))
    perm, gids, goff, sk, ng = compact(key)
    count_hot = int((key < n_hot).sum())
    out = [(perm, np.where(gids < n_hot, gids, 0).astype(np.int32),
            np.minimum(goff, count_hot).astype(np.int32))]
    if host_in_decode:
        count_native = int((key < n_hot + n_cold).sum())
        groups_hot = int((ng & (sk < n_hot)).sum())
        idx = np.minimum(np.arange(n + 1) + groups_hot, n)
        goff_c = np.minimum(goff[idx], count_native).astype(np.int32)
        gids_c = np.clip(gids[np.minimum(idx[:n], n - 1)] - n_hot, 0, n_cold - 1).astype(np.int32)
        out.append((perm, gids_c, goff_c))
    return out


def group_plan(ids, hot_slot, second_slot, n_hot: int, n_second: int, split: bool,
               host: bool, iq_slot=None):
    """The one-launch plan's definition (EXP/nvfp4_8r_group_plan.py:13-24):
    key = HOT slot, else n_hot + second slot, else the sentinel n_hot + n_second;
    rank[i] = #{key < key_i} + #{j < i, key_j == key_i}; perm[rank[i]] = i;
    HBM tables: gids_hot = key if < n_hot else 0, goff_hot = min(goff, #HOT);
    host tables rotated left by the HOT groups, goff_host = min(goff, #native),
    gids_host = clamp(gids - n_hot, 0, n_second - 1).  Returns a dict of int32
    arrays (perm, gids_hot, goff_hot[, gids_host, goff_host][, iq])."""
    flat = np.asarray(ids).reshape(-1)
    n = flat.size
    hot = hot_slot[flat].astype(np.int64)
    if split:
        sec = second_slot[flat].astype(np.int64)
        key = np.where(hot >= 0, hot, np.where(sec >= 0, n_hot + sec, n_hot + n_second))
    else:
        key = hot
    perm, gids, goff, sk, ng = compact(key)
    res = {"perm": perm}
    count_hot = int((key < n_hot).sum())
    res["gids_hot"] = np.where(gids < n_hot, gids, 0).astype(np.int32)
    res["goff_hot"] = np.minimum(goff, count_hot).astype(np.int32)
    if host:
        count_native = int((key < n_hot + n_second).sum())
        groups_hot = int((ng & (sk < n_hot)).sum())
        idx = np.minimum(np.arange(n + 1) + groups_hot, n)
        res["goff_host"] = np.minimum(goff[idx], count_native).astype(np.int32)
        res["gids_host"] = np.clip(gids[np.minimum(idx[:n], n - 1)] - n_hot, 0,
                                   n_second - 1).astype(np.int32)
    if iq_slot is not None:
        res["iq"] = iq_slot[flat].astype(np.int32)
    return res


# ---------------------------------------------------------------------------
# Tier map -> slot maps (EXP/nvfp4_8r_tiers.py:48-51,169-179)
# ---------------------------------------------------------------------------

HOT, WARM, HOST = 0, 1, 2


def slot_maps(tier: np.ndarray) -> dict:
    """int32 slot of each expert per bank, -1 where absent; slots are ranks in
    ascending expert id.  ``cold`` = every non-HOT expert, ``host`` = its HOST
    subset with the same slot numbers, ``iq`` = the WARM experts."""
    tier = np.asarray(tier, np.int8)
    if tier.ndim != 1 or np.any((tier < 0) | (tier > 2)):
        raise ValueError("a tier array is int8 [E] of HOT/WARM/HOST")

    def ranks(mask):
        out = np.full(tier.size, -1, np.int32)
        out[mask] = np.arange(int(mask.sum()), dtype=np.int32)
        return out

    cold = ranks(tier != HOT)
    return {"hot": ranks(tier == HOT), "cold": cold,
            "host": np.where(tier == HOST, cold, -1).astype(np.int32),
            "iq": ranks(tier == WARM)}


# ---------------------------------------------------------------------------
# Limited SwiGLU and the slot-order weighted reduce
# ---------------------------------------------------------------------------

SWIGLU_LIMIT = 10.0


def swiglu_chain(y13: np.ndarray, inter: int, limit: float = SWIGLU_LIMIT) -> np.ndarray:
    """fp16 y13 [S, 2I] (gate | up) -> fp16 [S, I]: g = min(f32(gate), limit),
    u = clamp(f32(up), -limit, limit), fp16(g / (1 + exp(-g)) * u), FP32
    round-to-nearest ops, NaN propagates (EXP/nvfp4_8r_native.py:937-939,
    EXP/nvfp4_8r_swiglu.py:84-110)."""
    y = np.asarray(y13, np.float16)
    g = y[:, :inter].astype(np.float32)
    u = y[:, inter:2 * inter].astype(np.float32)
    lim = np.float32(limit)
    g = np.where(g > lim, lim, g)
    u = np.where(u > lim, lim, u)
    u = np.where(u < -lim, -lim, u)
    with np.errstate(over="ignore", invalid="ignore"):
        act = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
        return (act * u).astype(np.float32).astype(np.float16)


def weighted_reduce(y2: np.ndarray, w: np.ndarray) -> np.ndarray:
    """out[t] = sum over slot 0..k-1 of f32(y2[k t + slot]) * w[t, slot], in
    slot order, FP32 (EXP/nvfp4_8r_iq_tail.py:106-120)."""
    w = np.asarray(w, np.float32)
    m, k = w.shape
    y = np.asarray(y2).astype(np.float32).reshape(m, k, -1)
    acc = np.zeros((m, y.shape[2]), np.float32)
    for s in range(k):
        acc = (acc + y[:, s, :] * w[:, s:s + 1]).astype(np.float32)
    return acc


# ---------------------------------------------------------------------------
# Whole layer: dequant-then-matmul (the reference's CPU path)
# ---------------------------------------------------------------------------

def expert_fp32(x_rows: np.ndarray, w13: np.ndarray, w2: np.ndarray, limit=SWIGLU_LIMIT) -> np.ndarray:
    """FP32 expert on dequantized weights: W2 (silu(min(W1 x, L)) * clamp(W3 x, +-L))."""
    inter = w2.shape[1]
    h = x_rows.astype(np.float32) @ w13.T.astype(np.float32)
    g = np.minimum(h[:, :inter], np.float32(limit))
    u = np.clip(h[:, inter:], -np.float32(limit), np.float32(limit))
    a = (g / (np.float32(1) + np.exp(-g))) * u
    return (a.astype(np.float32) @ w2.T.astype(np.float32)).astype(np.float32)


def contribution_fp64(w13: np.ndarray, w2: np.ndarray, x: np.ndarray, weight: float,
                      limit=SWIGLU_LIMIT) -> np.ndarray:
    """One routed slot in float64: weight * W2 (silu(min(W1 x, L)) * clamp(W3 x, +-L))
    (HB/make_p2_refs.py:52-59)."""
    inter = w2.shape[1]
    xf = np.asarray(x, np.float64)
    h = w13.astype(np.float64) @ xf
    g = np.minimum(h[:inter], limit)
    u = np.clip(h[inter:], -limit, limit)
    return weight * (w2.astype(np.float64) @ (g / (1.0 + np.exp(-g)) * u))


def layer_forward(x: np.ndarray, ids: np.ndarray, w: np.ndarray, dequant, limit=SWIGLU_LIMIT,
                  dtype=np.float32) -> np.ndarray:
    """out[t] = sum over slots of w[t,s] * expert_{ids[t,s]}(x[t]), slot order.
    ``dequant(e) -> (w13 [2I, H], w2 [H, I])`` float32.  dtype float32 follows
    the reference CPU torch path; float64 follows HB/make_p2_refs.py."""
    x = np.asarray(x, np.float32)
    ids = np.asarray(ids)
    m, k = ids.shape
    hdim = x.shape[1]
    contrib = np.zeros((m, k, hdim), dtype)
    for e in np.unique(ids):
        w13, w2 = dequant(int(e))
        rows, slots = np.nonzero(ids == e)
        if dtype == np.float64:
            for r, s in zip(rows, slots):
                contrib[r, s] = contribution_fp64(w13, w2, x[r], float(w[r, s]), limit)
        else:
            y = expert_fp32(x[rows], w13, w2, limit)
            contrib[rows, slots] = y * w[rows, slots][:, None]
    out = np.zeros((m, hdim), dtype)
    for s in range(k):
        out = out + contrib[:, s]
    return out


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a - b))


# ---------------------------------------------------------------------------
# decode route counters (EXP/nvfp4_8r_stats.py:41-110)
# ---------------------------------------------------------------------------

#: stat fields, gap-histogram edges and "recent" windows (EXP/nvfp4_8r_stats.py:45-50)
STAT_FIELDS = ("calls", "routes", "host_routes", "host_groups", "warm_routes")
GAP_EDGES = (1, 2, 4, 16, 64, 256)
RECENT = (4, 16, 64, 256)
NEVER = -(2**30)


def route_stats_new(num_experts: int) -> dict:
    """Zeroed counters of one layer: stat int64 [5], gap_hist int64 [7],
    routes int64 [E], last_round int32 [E + 1] (entry E takes the writes of
    non-HOST routes), as RouteStats.__init__ (EXP/nvfp4_8r_stats.py:68-79)."""
    return {"stat": np.zeros(len(STAT_FIELDS), np.int64), "gap_hist": np.zeros(len(GAP_EDGES) + 1, np.int64),
            "routes": np.zeros(num_experts, np.int64),
            "last_round": np.full(num_experts + 1, NEVER, np.int32)}


def route_stats_count(c: dict, ids: np.ndarray, is_host: np.ndarray, is_warm: np.ndarray) -> None:
    """One decode call's routes, in place (RouteStats.count,
    EXP/nvfp4_8r_stats.py:81-98): the round r = calls so far; each HOST route
    adds to the gap bucket of r - (its expert's last HOST round), buckets
    (<=1, 2, <=4, <=16, <=64, <=256, more or never); then the HOST experts'
    last round becomes r; routes per expert, HOST routes, distinct HOST experts
    of this call, WARM routes, routes and calls are counted."""
    flat = np.asarray(ids, np.int64).reshape(-1)
    E = c["routes"].size
    host = is_host[flat].astype(bool)
    slot = np.where(host, flat, E)
    r = int(c["stat"][0])
    gap = r - c["last_round"][slot].astype(np.int64)
    bucket = np.searchsorted(np.asarray(GAP_EDGES, np.int64), gap, side="left")
    np.add.at(c["gap_hist"], bucket[host], 1)
    c["last_round"][slot] = np.where(host, r, NEVER).astype(np.int32)
    np.add.at(c["routes"], flat, 1)
    c["stat"][2] += int(host.sum())
    c["stat"][3] += int((c["last_round"][:E] == r).sum())
    c["stat"][4] += int(is_warm[flat].astype(bool).sum())
    c["stat"][1] += flat.size
    c["stat"][0] += 1


def route_stats_recent(c: dict) -> np.ndarray:
    """Experts whose last HOST use is within each RECENT window (RouteStats.read)."""
    age = int(c["stat"][0]) - c["last_round"][:-1].astype(np.int64)
    return np.array([int((age <= g).sum()) for g in RECENT], np.int64)
