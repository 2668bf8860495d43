"""Seeded synthetic experts and inputs of the benchmark configurations.

There are no real checkpoints here: weights are drawn ~N(0, std) on the GPU
from a seeded generator and packed by the library's own quantizers; IQ2_XXS
experts are seeded random valid blocks (every byte pattern of a block's 64
code bytes is legal) with an fp16 super-block scale sized to the weight std.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import packing


@dataclass
class Fp4Bank:
    """Natural-layout packed experts (device tensors), the input of load_fp4."""

    fmt: str
    w13_codes: torch.Tensor   # [n, 2I, H/2]
    w13_scales: torch.Tensor  # [n, 2I, H/bs]
    w2_codes: torch.Tensor    # [n, H, I/2]
    w2_scales: torch.Tensor   # [n, H, I/bs]
    globals: torch.Tensor | None  # [n, 3] (NVFP4)

    @property
    def n(self) -> int:
        return self.w13_codes.shape[0]


@dataclass
class Iq2Bank:
    w1: torch.Tensor  # [n, I, H/256, block bytes of the gate/up type]
    w3: torch.Tensor
    w2: torch.Tensor  # [n, H, I/256, block bytes of the down type]

    @property
    def n(self) -> int:
        return self.w1.shape[0]


def make_fp4_bank(n: int, hidden: int, inter: int, fmt: str, seed: int, device, std: float = 0.02) -> Fp4Bank:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I = hidden, inter
    bs = 16 if fmt == "nvfp4" else 32
    u8 = dict(dtype=torch.uint8, device=device)
    bank = Fp4Bank(fmt, torch.empty((n, 2 * I, H // 2), **u8), torch.empty((n, 2 * I, H // bs), **u8),
                   torch.empty((n, H, I // 2), **u8), torch.empty((n, H, I // bs), **u8),
                   torch.empty((n, 3), dtype=torch.float32, device=device) if fmt == "nvfp4" else None)
    for e in range(n):
        w13 = torch.randn((2 * I, H), generator=g, device=device, dtype=torch.float32).mul_(std)
        w2 = torch.randn((H, I), generator=g, device=device, dtype=torch.float32).mul_(std)
        if fmt == "nvfp4":
            packing.quantize_nvfp4_into(w13[:I], bank.w13_codes[e, :I], bank.w13_scales[e, :I], bank.globals[e, 0:1])
            packing.quantize_nvfp4_into(w13[I:].contiguous(), bank.w13_codes[e, I:], bank.w13_scales[e, I:],
                                        bank.globals[e, 1:2])
            packing.quantize_nvfp4_into(w2, bank.w2_codes[e], bank.w2_scales[e], bank.globals[e, 2:3])
        else:
            c, s = packing.quantize_mxfp4(w13, check=False)
            bank.w13_codes[e].copy_(c)
            bank.w13_scales[e].copy_(s)
            c, s = packing.quantize_mxfp4(w2, check=False)
            bank.w2_codes[e].copy_(c)
            bank.w2_scales[e].copy_(s)
    return bank


IQ_BLOCK_BYTES = {16: 66, 17: 74, 29: 56}  # IQ2_XXS, IQ2_XS, IQ1_M


def _iq2_blocks(g, rows: int, k: int, n: int, std: float, device, ggml_type: int = 16) -> torch.Tensor:
    """Random valid ggml blocks: any index, sign and scale bits; d sized for ``std``."""
    nb, bb = k // 256, IQ_BLOCK_BYTES[ggml_type]
    b = torch.randint(0, 256, (n, rows, nb, bb), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    if ggml_type == 29:  # IQ1_M: d is the fp16 made of the four scale words' top nibbles
        d = ((std / 6.0) * (0.75 + 0.5 * torch.rand((n, rows, nb), generator=g, device=device)))
        dbits = d.to(torch.float16).view(torch.int16).to(torch.int32) & 0xFFFF
        w = b[..., 48:56].contiguous().view(torch.int16).to(torch.int32) & 0x0FFF
        w = w | (((dbits[..., None] >> torch.tensor([0, 4, 8, 12], device=device)) & 15) << 12)
        b[..., 48:56] = w.to(torch.int16).view(torch.uint8)
    else:
        d = (std / 48.0) * (0.75 + 0.5 * torch.rand((n, rows, nb), generator=g, device=device))
        b[..., :2] = d.to(torch.float16).view(torch.uint8).reshape(n, rows, nb, 2)
    return b


def make_iq2_bank(n: int, hidden: int, inter: int, seed: int, device, std: float = 0.02,
                  iq_types: tuple[int, int] = (16, 16)) -> Iq2Bank:
    """Seeded random IQ experts: gate/up of GGML type iq_types[0], down of iq_types[1]."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    t13, t2 = iq_types
    return Iq2Bank(_iq2_blocks(g, inter, hidden, n, std, device, t13), _iq2_blocks(g, inter, hidden, n, std, device, t13),
                   _iq2_blocks(g, hidden, inter, n, std, device, t2))


def load_bank(layer, bank, slot_begin: int = 0, step: int = 16) -> None:
    if isinstance(bank, Fp4Bank):
        for s in range(0, bank.n, step):
            e = min(bank.n, s + step)
            layer.load_fp4(slot_begin + s, bank.w13_codes[s:e], bank.w13_scales[s:e], bank.w2_codes[s:e],
                           bank.w2_scales[s:e], None if bank.globals is None else bank.globals[s:e])
    else:
        for s in range(0, bank.n, step):
            e = min(bank.n, s + step)
            layer.load_iq2(slot_begin + s, bank.w1[s:e].contiguous(), bank.w3[s:e].contiguous(),
                           bank.w2[s:e].contiguous())


def zipf_logits(tokens: int, rank, alpha: float, s: float, seed: int, device) -> torch.Tensor:
    """Router logits whose Gumbel-top-k sampling follows Zipf(s) popularity:
    alpha * log p(rank) + Gumbel(0, 1) noise, seeded."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    r = torch.as_tensor(rank, device=device, dtype=torch.float32)
    logp = -s * torch.log(r + 1.0)
    u = torch.rand((tokens, r.numel()), generator=g, device=device).clamp_(1e-12, 1 - 1e-7)
    return (alpha * logp)[None, :] - torch.log(-torch.log(u))


def load_local(layer, tier, fp4: Fp4Bank | None, iq2: Iq2Bank | None) -> None:
    """Load one rank's experts from banks that hold every expert of the layer:
    the bank of a format is indexed by the expert's rank among that format's
    experts (ascending id); the rank's experts, in local slot order, are
    gathered from it (any placement)."""
    import numpy as np
    import torch

    from . import tiers as tiersmod

    maps = tiersmod.slot_maps(tier)
    for fmt, bank, local, glob in (("fp4", fp4, layer.fp4_slot, maps.hot), ("iq2", iq2, layer.iq2_slot, maps.iq)):
        mine = np.flatnonzero(local >= 0)
        if mine.size == 0:
            continue
        mine = mine[np.argsort(local[mine])]
        if not np.array_equal(local[mine], np.arange(mine.size)):
            raise ValueError("local slots of a format must be 0..n-1")
        rows = glob[mine]
        run = int(rows[0])
        pick = (lambda t: t[run:run + rows.size]) if np.array_equal(rows, np.arange(run, run + rows.size)) else (
            lambda t: t.index_select(0, torch.as_tensor(rows, dtype=torch.int64, device=t.device)))
        if fmt == "fp4":
            layer.load_fp4(0, pick(bank.w13_codes).contiguous(), pick(bank.w13_scales).contiguous(),
                           pick(bank.w2_codes).contiguous(), pick(bank.w2_scales).contiguous(),
                           None if bank.globals is None else pick(bank.globals).contiguous())
        else:
            layer.load_iq2(0, pick(bank.w1).contiguous(), pick(bank.w3).contiguous(), pick(bank.w2).contiguous())
