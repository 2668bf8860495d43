"""The NVFP4 / MXFP4 quantizers of ``moe_oracle.py`` written with stock torch
ops, so that large seeded expert banks can be packed on any device without
this build's CUDA library.

TEST INFRASTRUCTURE ONLY: bench.py's reference arm packs its experts with these
functions (that process must not load the product library), and
``tests/test_oracle_golden.py`` pins them bit for bit to ``moe_oracle.py``'s
``nvfp4_quantize`` / ``mxfp4_quantize`` (which the library's GPU quantizers
also match bit for bit).  The rules are the oracle's: all divisions IEEE
float32 round-to-nearest; E4M3 by round-half-even on the power-of-two quantum
of the value's binade, saturating at 448; E2M1 by the midpoint thresholds with
ties to the even code.
"""

from __future__ import annotations

import torch

NVFP4_GLOBAL_DIVISOR = 2688.0  # 6 * 448


def e2m1_code(t: torch.Tensor) -> torch.Tensor:
    """|t| (float32) -> 3-bit E2M1 magnitude code (moe_oracle.e2m1_code)."""
    c = ((t > 0.25).to(torch.uint8) + (t >= 0.75) + (t > 1.25) + (t >= 1.75)
         + (t > 2.5) + (t >= 3.5) + (t > 5.0))
    return c.to(torch.uint8)


def e4m3_from_f32(x: torch.Tensor) -> torch.Tensor:
    """Non-negative float32 -> E4M3FN byte (moe_oracle.e4m3_from_f32)."""
    xd = x.to(torch.float64)
    _, ex = torch.frexp(xd)
    e = torch.clamp(ex.to(torch.int32) - 1, min=-6)
    quantum = torch.ldexp(torch.ones_like(xd), (e - 3).to(torch.float64))
    q = torch.clamp(torch.round(xd / quantum) * quantum, max=448.0)
    _, qe = torch.frexp(q)
    qe = qe.to(torch.int32) - 1
    man_sub = torch.round(torch.ldexp(q, torch.full_like(q, 9.0))).to(torch.int32)
    man_norm = torch.round((torch.ldexp(q, (-qe).to(torch.float64)) - 1.0) * 8).to(torch.int32)
    enc = torch.where(qe < -6, man_sub, ((qe + 7) << 3) | man_norm)
    return torch.where(q > 0, enc, torch.zeros_like(enc)).to(torch.uint8)


def e4m3_to_f32(bits: torch.Tensor) -> torch.Tensor:
    b = bits.to(torch.int32)
    e = (b >> 3) & 15
    m = (b & 7).to(torch.float32)
    mag = torch.where(e == 0, m * 2.0**-9, torch.ldexp(1 + m / 8, (e - 7).to(torch.float32)))
    return torch.where((b & 128) != 0, -mag, mag)


def _pack(nib: torch.Tensor) -> torch.Tensor:
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)


def nvfp4_quantize(w: torch.Tensor):
    """float32 [R, K] -> (codes uint8 [R, K/2], E4M3 uint8 [R, K/16], global
    float32 0-d tensor) as moe_oracle.nvfp4_quantize."""
    w = w.to(torch.float32).contiguous()
    rows, k = w.shape
    a = w.abs()
    amax = a.max()
    glob = torch.where(amax > 0, amax / NVFP4_GLOBAL_DIVISOR, torch.ones_like(amax))
    denom = glob * 6.0
    blk = a.reshape(rows, k // 16, 16).amax(dim=2)
    sbits = e4m3_from_f32(blk / denom)
    qscale = e4m3_to_f32(sbits) * glob
    safe = torch.where(qscale > 0, qscale, torch.ones_like(qscale))
    t = a.reshape(rows, -1, 16) / safe[:, :, None]
    mag = torch.where(qscale[:, :, None] > 0, e2m1_code(t), torch.zeros_like(t, dtype=torch.uint8))
    sign = (w.reshape(rows, -1, 16) < 0).to(torch.uint8) << 3
    return _pack((mag | sign).reshape(rows, k)), sbits, glob


def mxfp4_quantize(w: torch.Tensor):
    """float32 [R, K] -> (codes uint8 [R, K/2], E8M0 uint8 [R, K/32]) as
    moe_oracle.mxfp4_quantize."""
    w = w.to(torch.float32).contiguous()
    rows, k = w.shape
    a = w.abs()
    blk = a.reshape(rows, k // 32, 32).amax(dim=2)
    m, ex = torch.frexp(blk.to(torch.float64))
    e = torch.where(m <= 0.75, ex - 3, ex - 2).to(torch.int32)
    e = torch.where(blk > 0, e, torch.zeros_like(e))
    if bool(((e < -127) | (e > 127)).any()):
        raise ValueError("block exponent outside the E8M0 range")
    t = torch.ldexp(a.reshape(rows, -1, 32).to(torch.float64), (-e[:, :, None]).to(torch.float64)).to(torch.float32)
    sign = (w.reshape(rows, -1, 32) < 0).to(torch.uint8) << 3
    return _pack((e2m1_code(t) | sign).reshape(rows, k)), (e + 127).to(torch.uint8)


def fp4_expert_bank(n: int, hidden: int, inter: int, fmt: str, seed: int, device, std: float = 0.02, pick=None):
    """The seeded experts of the product's synthetic banks (the same generator
    calls, so the same fp32 weights), packed here: a list of dicts in the C
    oracle's form (numpy arrays on the host), for the experts in ``pick``
    (default all ``n``)."""
    import numpy as np

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I = hidden, inter
    want = set(range(n)) if pick is None else {int(p) for p in pick}
    out = {}
    for e in range(max(want) + 1 if want else 0):
        w13 = torch.randn((2 * I, H), generator=g, device=device, dtype=torch.float32).mul_(std)
        w2 = torch.randn((H, I), generator=g, device=device, dtype=torch.float32).mul_(std)
        if e not in want:
            continue
        if fmt == "nvfp4":
            c1, s1, g1 = nvfp4_quantize(w13[:I])
            c3, s3, g3 = nvfp4_quantize(w13[I:])
            c2, s2, g2 = nvfp4_quantize(w2)
            out[e] = dict(fmt=0, w13c=torch.cat([c1, c3]).cpu().numpy(), w13s=torch.cat([s1, s3]).cpu().numpy(),
                          g13=np.array([float(g1), float(g3)], np.float32), w2c=c2.cpu().numpy(),
                          w2s=s2.cpu().numpy(), g2=float(g2))
        else:
            c13, s13 = mxfp4_quantize(w13)
            c2, s2 = mxfp4_quantize(w2)
            out[e] = dict(fmt=1, w13c=c13.cpu().numpy(), w13s=s13.cpu().numpy(), g13=np.ones(2, np.float32),
                          w2c=c2.cpu().numpy(), w2s=s2.cpu().numpy(), g2=1.0)
    return out
