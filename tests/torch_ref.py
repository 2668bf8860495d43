"""Plain PyTorch fp32 dequant-then-matmul reference (test infrastructure).

The same formulas as ``oracle/moe_oracle.py`` written with torch ops so the
large parity cases run on the GPU; ``test_torch_ref_matches_oracle`` pins it
to the numpy oracle bit for bit on the decode step and to 1e-6 on the layer.
"""

from __future__ import annotations

import numpy as np
import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _e4m3_table(device) -> torch.Tensor:
    b = torch.arange(256)
    e = (b >> 3) & 15
    m = (b & 7).float()
    mag = torch.where(e == 0, m * 2.0**-9, torch.ldexp(1 + m / 8, (e - 7).float()))
    return torch.where((b & 128) != 0, -mag, mag).to(torch.float32).to(device)


def nibbles(codes: torch.Tensor) -> torch.Tensor:
    c = codes.to(torch.int64)
    return torch.stack([c & 15, c >> 4], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)


def nvfp4_decode(codes, scales, glob) -> torch.Tensor:
    rows, k = codes.shape[0], codes.shape[1] * 2
    vals = E2M1.to(codes.device)[nibbles(codes)].reshape(rows, k // 16, 16)
    blk = _e4m3_table(codes.device)[scales.to(torch.int64)].reshape(rows, k // 16, 1)
    return ((vals * blk) * torch.as_tensor(glob, dtype=torch.float32, device=codes.device)).reshape(rows, k)


def mxfp4_decode(codes, e8m0) -> torch.Tensor:
    rows, k = codes.shape[0], codes.shape[1] * 2
    vals = E2M1.to(codes.device)[nibbles(codes)].reshape(rows, k // 32, 32)
    return torch.ldexp(vals, (e8m0.to(torch.int64) - 127).reshape(rows, k // 32, 1).float()).reshape(rows, k)


def iq2xxs_decode(blocks, grid: np.ndarray, ksigns: np.ndarray) -> torch.Tensor:
    dev = blocks.device
    rows, nb, _ = blocks.shape
    d = blocks[..., :2].contiguous().view(torch.float16).float().reshape(rows, nb)
    qs = blocks[..., 2:].contiguous().view(torch.int32).reshape(rows, nb, 8, 2).to(torch.int64) & 0xFFFFFFFF
    a, b = qs[..., 0], qs[..., 1]
    db = (d[..., None] * (0.5 + (b >> 28).float())) * 0.25
    gidx = torch.stack([(a >> (8 * l)) & 255 for l in range(4)], dim=-1)  # [R, nb, 8, 4]
    g = torch.as_tensor(grid, dtype=torch.float32, device=dev)[gidx]     # [R, nb, 8, 4, 8]
    sidx = torch.stack([(b >> (7 * l)) & 127 for l in range(4)], dim=-1)
    sb = torch.as_tensor(ksigns.astype(np.int64), device=dev)[sidx]
    neg = (sb[..., None] >> torch.arange(8, device=dev)) & 1
    sgn = torch.where(neg == 1, -1.0, 1.0)
    return ((db[..., None, None] * g) * sgn).reshape(rows, nb * 256)


def layer_forward(x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, dequant, limit: float = 10.0) -> torch.Tensor:
    """fp32: out[t] = sum over slots (slot order) of w * W2(silu(min(W1 x, L)) * clamp(W3 x, +-L))."""
    x = x.float()
    m, k = ids.shape
    contrib = torch.zeros((m, k, x.shape[1]), dtype=torch.float32, device=x.device)
    for e in torch.unique(ids).tolist():
        w13, w2 = dequant(int(e))
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        inter = w2.shape[1]
        h = x[rows] @ w13.T
        g = torch.clamp(h[:, :inter], max=limit)
        u = torch.clamp(h[:, inter:], -limit, limit)
        y = ((g / (1 + torch.exp(-g))) * u) @ w2.T
        contrib[rows, slots] = y * w[rows, slots][:, None]
    out = torch.zeros((m, x.shape[1]), dtype=torch.float32, device=x.device)
    for s in range(k):
        out = out + contrib[:, s]
    return out


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
