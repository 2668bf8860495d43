"""The reference's expert pack directories -> this library's FP4 bank (host logic).

A pack holds one MXFP4 record per (layer, TP rank, expert) of the reference's
four-way tensor-parallel split (format and readers:
engine/src/vllm/model_executor/layers/fused_moe/experts/nvfp4_8r_native.py:59-75,176-250;
writer: harness/benchmarks/nvfp4_8r/build_packs.py:217-257).  At the
reference's sizes a record is 4,874,240 bytes:

  w1 codes [576][2560]   w1 E8M0 [576][160]    rows 576 r .. 576 r + 575 of W1 (rank r)
  w3 codes [576][2560]   w3 E8M0 [576][160]    the same rows of W3
  w2 codes [5120][320]   w2 E8M0 [5120][20]    K columns 576 r .. of W2, K padded
                                               576 -> 640 (zero codes, scale 127)

Codes hold the even element in the low nibble; E8M0 scales have bias 127 and
255 is refused.  Two directory formats, each described by ``manifest.json``:

  v1 ``nvfp4-8r-mxfp4-v1``: per (layer, rank) a ``-hot`` and a ``-cold`` file,
     the expert ids of each listed in the manifest;
  v2 ``nvfp4-8r-mxfp4-v2-id-order``: one file per (layer, rank), records in
     expert-id order.

A B200 holds whole experts, so the four rank slices of an expert are joined:
W1 rows of ranks 0..3, then W3 rows of ranks 0..3 (the layer's W13, gate rows
then up rows) and W2 with each rank's 576 K columns side by side, padding
dropped.  ``load_pack_layer`` streams a layer's FP4 experts, a chunk at a
time, into a ``B200NativeMoe`` created with ``fp4_format="mxfp4"``.  The IQ2
(WARM) experts come from GGUF blocks through ``B200NativeMoe.load_iq2``.
"""

from __future__ import annotations

import json
import os
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np

PACK_FORMAT = "nvfp4-8r-mxfp4-v1"
PACK_FORMAT_ID_ORDER = "nvfp4-8r-mxfp4-v2-id-order"
FILE_PATTERN = "L{layer:02d}-r{rank}.bin"


@dataclass(frozen=True)
class PackGeometry:
    """Record shapes of a pack: the reference's sizes by default."""

    hidden: int = 5120
    tp_inter: int = 576
    w2_k: int = 640  # W2's K per rank after padding
    tp_ranks: int = 4
    num_experts: int = 384
    num_layers: int = 40

    def __post_init__(self) -> None:
        if (self.hidden % 32 or self.tp_inter % 32 or self.w2_k % 32 or self.w2_k < self.tp_inter
                or min(self.tp_ranks, self.num_experts, self.num_layers) < 1):
            raise ValueError(f"invalid pack geometry {self}")

    @property
    def inter(self) -> int:
        return self.tp_ranks * self.tp_inter

    def parts(self) -> list[tuple[str, tuple[int, int]]]:
        """(name, [rows, bytes per row]) of a record's six parts, in file order."""
        H, Ip, K2 = self.hidden, self.tp_inter, self.w2_k
        return [("w1_codes", (Ip, H // 2)), ("w1_scales", (Ip, H // 32)),
                ("w3_codes", (Ip, H // 2)), ("w3_scales", (Ip, H // 32)),
                ("w2_codes", (H, K2 // 2)), ("w2_scales", (H, K2 // 32))]

    @property
    def expert_bytes(self) -> int:
        return sum(r * c for _, (r, c) in self.parts())


REFERENCE_GEOMETRY = PackGeometry()
assert REFERENCE_GEOMETRY.expert_bytes == 4_874_240


def _manifest(packs: Path) -> dict:
    path = Path(packs) / "manifest.json"
    if not path.is_file():
        raise ValueError(f"no pack manifest in {packs}")
    doc = json.loads(path.read_text())
    if not isinstance(doc, dict):
        raise ValueError(f"{path} is not a JSON object")
    return doc


def read_manifest(packs, geom: PackGeometry = REFERENCE_GEOMETRY) -> list:
    """The v1 manifest's per-layer, per-rank {"hot": ids, "cold": ids} lists."""
    doc = _manifest(packs)
    if doc.get("format") != PACK_FORMAT:
        raise ValueError(f"unknown pack format {doc.get('format')!r}")
    layers = doc.get("layers")
    if not isinstance(layers, list) or len(layers) != geom.num_layers or any(
            not isinstance(l, list) or len(l) != geom.tp_ranks for l in layers):
        raise ValueError(f"{packs}/manifest.json: 'layers' must list {geom.num_layers} layers x "
                         f"{geom.tp_ranks} ranks")
    return layers


def read_id_order_manifest(packs, geom: PackGeometry = REFERENCE_GEOMETRY) -> dict:
    """The v2 manifest, checked whole: exactly these keys (and an optional comment)."""
    doc = _manifest(packs)
    want = {"format": PACK_FORMAT_ID_ORDER, "num_layers": geom.num_layers, "tp_ranks": geom.tp_ranks,
            "num_experts": geom.num_experts, "expert_bytes": geom.expert_bytes, "file": FILE_PATTERN}
    got = {k: doc.get(k) for k in want}
    if got != want or set(doc) - set(want) - {"comment"}:
        raise ValueError(f"{packs}/manifest.json is not an {PACK_FORMAT_ID_ORDER} manifest: {got}")
    return doc


def check_packs(packs, geom: PackGeometry = REFERENCE_GEOMETRY) -> str:
    """The format of a pack directory (v1 or v2), its manifest validated."""
    fmt = _manifest(packs).get("format")
    if fmt == PACK_FORMAT_ID_ORDER:
        read_id_order_manifest(packs, geom)
    else:
        read_manifest(packs, geom)
    return fmt


def read_rank_experts(packs, layer: int, rank: int, geom: PackGeometry = REFERENCE_GEOMETRY) -> np.ndarray:
    """All expert records of one (layer, rank) as uint8 [E, expert_bytes],
    indexed by expert id.  A v2 file is memory-mapped read-only (records are
    read when used); a v1 pair is scattered by the manifest's ids, which must
    partition 0..E-1."""
    packs = Path(packs)
    E, B = geom.num_experts, geom.expert_bytes
    if not (0 <= layer < geom.num_layers and 0 <= rank < geom.tp_ranks):
        raise ValueError(f"no pack file for layer {layer} rank {rank}")
    if _manifest(packs).get("format") == PACK_FORMAT_ID_ORDER:
        read_id_order_manifest(packs, geom)
        path = packs / FILE_PATTERN.format(layer=layer, rank=rank)
        size = os.stat(path).st_size
        if size != E * B:
            raise ValueError(f"{path}: {size} bytes, want {E} x {B}")
        return np.memmap(path, dtype=np.uint8, mode="r", shape=(E, B))
    split = read_manifest(packs, geom)[layer][rank]
    if not isinstance(split, dict) or set(split) != {"hot", "cold"}:
        raise ValueError(f"L{layer} r{rank}: a v1 split is {{'hot': ids, 'cold': ids}}")
    ids = [e for temp in ("hot", "cold") for e in split[temp]]
    if any(type(e) is not int for e in ids) or sorted(ids) != list(range(E)):
        raise ValueError(f"L{layer} r{rank}: hot + cold is not a partition of {E}")
    out = np.empty((E, B), np.uint8)
    for temp in ("hot", "cold"):
        path = packs / f"L{layer:02d}-r{rank}-{temp}.bin"
        n = len(split[temp])
        size = os.stat(path).st_size
        if size != n * B:
            raise ValueError(f"{path}: {size} bytes for {n} experts")
        if n:
            out[np.asarray(split[temp], np.int64)] = np.fromfile(path, np.uint8).reshape(n, B)
    return out


def split_records(raw: np.ndarray, geom: PackGeometry = REFERENCE_GEOMETRY) -> tuple[np.ndarray, ...]:
    """Views of records uint8 [n, expert_bytes] as their six parts
    (w1 codes, w1 scales, w3 codes, w3 scales, w2 codes, w2 scales), each [n, rows, bytes]."""
    if raw.dtype != np.uint8 or raw.ndim != 2 or raw.shape[1] != geom.expert_bytes:
        raise ValueError(f"expert records must be uint8 [n, {geom.expert_bytes}]")
    n, o, out = raw.shape[0], 0, []
    for _, (rows, cols) in geom.parts():
        out.append(raw[:, o:o + rows * cols].reshape(n, rows, cols))
        o += rows * cols
    return tuple(out)


def join_experts(slices: Sequence[np.ndarray], geom: PackGeometry = REFERENCE_GEOMETRY):
    """Whole experts from their rank slices.

    ``slices[r]`` holds rank r's records of the same n experts (uint8 [n,
    expert_bytes]).  Returns (w13_codes [n, 2I, H/2], w13_scales [n, 2I, H/32],
    w2_codes [n, H, I/2], w2_scales [n, H, I/32]) in the layout
    ``B200NativeMoe.load_fp4`` takes for MXFP4, I = tp_ranks x tp_inter.
    Refuses W2 padding codes that are not zero (the reference's check,
    nvfp4_8r_native.py:277-278) and E8M0 scale 255."""
    if len(slices) != geom.tp_ranks:
        raise ValueError(f"an expert has {geom.tp_ranks} rank slices, got {len(slices)}")
    parts = [split_records(np.asarray(s), geom) for s in slices]
    n = parts[0][0].shape[0]
    if any(p[0].shape[0] != n for p in parts):
        raise ValueError("rank slices hold different numbers of experts")
    kc, ks = geom.tp_inter // 2, geom.tp_inter // 32
    for r, (_, _, _, _, w2c, _) in enumerate(parts):
        if w2c.shape[2] > kc and np.any(w2c[:, :, kc:]):
            raise ValueError(f"rank {r}: W2 K padding codes are not zero")
    w13c = np.concatenate([p[0] for p in parts] + [p[2] for p in parts], axis=1)
    w13s = np.concatenate([p[1] for p in parts] + [p[3] for p in parts], axis=1)
    w2c = np.concatenate([p[4][:, :, :kc] for p in parts], axis=2)
    w2s = np.concatenate([p[5][:, :, :ks] for p in parts], axis=2)
    if np.any(w13s == 255) or np.any(w2s == 255):
        raise ValueError("E8M0 scale 255 (NaN) in an expert record")
    return w13c, w13s, w2c, w2s


def split_expert(w13c: np.ndarray, w13s: np.ndarray, w2c: np.ndarray, w2s: np.ndarray,
                 geom: PackGeometry = REFERENCE_GEOMETRY) -> list[np.ndarray]:
    """The inverse of ``join_experts``: per rank, records uint8 [n,
    expert_bytes] with W2's K padded by zero codes and scale 127 (as the
    reference's pack builder writes them, build_packs.py:236-247)."""
    H, Ip, I = geom.hidden, geom.tp_inter, geom.inter
    n = w13c.shape[0]
    shapes = {"w13c": (n, 2 * I, H // 2), "w13s": (n, 2 * I, H // 32), "w2c": (n, H, I // 2),
              "w2s": (n, H, I // 32)}
    for name, a in (("w13c", w13c), ("w13s", w13s), ("w2c", w2c), ("w2s", w2s)):
        if a.dtype != np.uint8 or a.shape != shapes[name]:
            raise ValueError(f"{name} must be uint8 {shapes[name]}")
    out = []
    for r in range(geom.tp_ranks):
        rows = slice(r * Ip, (r + 1) * Ip)
        up = slice(I + r * Ip, I + (r + 1) * Ip)
        pc = np.zeros((n, H, geom.w2_k // 2), np.uint8)
        ps = np.full((n, H, geom.w2_k // 32), 127, np.uint8)
        pc[:, :, :Ip // 2] = w2c[:, :, r * Ip // 2:(r + 1) * Ip // 2]
        ps[:, :, :Ip // 32] = w2s[:, :, r * Ip // 32:(r + 1) * Ip // 32]
        pieces = (w13c[:, rows], w13s[:, rows], w13c[:, up], w13s[:, up], pc, ps)
        out.append(np.concatenate([p.reshape(n, -1) for p in pieces], axis=1))
    return out


def write_id_order_pack(packs, records: dict, geom: PackGeometry = REFERENCE_GEOMETRY,
                        comment: str | None = None) -> None:
    """Write a v2 pack: ``records[(layer, rank)]`` = uint8 [E, expert_bytes]
    in expert-id order.  The manifest is written last."""
    packs = Path(packs)
    packs.mkdir(parents=True, exist_ok=True)
    for (layer, rank), rec in records.items():
        rec = np.ascontiguousarray(rec, np.uint8)
        if rec.shape != (geom.num_experts, geom.expert_bytes):
            raise ValueError(f"L{layer} r{rank}: records must be uint8 [{geom.num_experts}, {geom.expert_bytes}]")
        rec.tofile(packs / FILE_PATTERN.format(layer=layer, rank=rank))
    doc = {"format": PACK_FORMAT_ID_ORDER, "num_layers": geom.num_layers, "tp_ranks": geom.tp_ranks,
           "num_experts": geom.num_experts, "expert_bytes": geom.expert_bytes, "file": FILE_PATTERN}
    if comment is not None:
        doc["comment"] = comment
    (packs / "manifest.json").write_text(json.dumps(doc, indent=1) + "\n")


def load_pack_layer(layer_obj, packs, layer: int, geom: PackGeometry = REFERENCE_GEOMETRY, chunk: int = 16) -> int:
    """Load one layer's FP4 (HOT) experts from a pack into ``layer_obj`` (a
    ``B200NativeMoe`` with ``fp4_format="mxfp4"`` and the pack's hidden,
    inter = tp_ranks x tp_inter and expert count).  Experts this GPU does not
    hold in its FP4 bank are skipped.  Reads ``chunk`` experts at a time from
    the four rank files, joins them on the host and copies them to the device
    through pinned memory.  Returns the number of experts loaded."""
    import torch

    if getattr(layer_obj, "fp4_format", None) != "mxfp4":
        raise ValueError("packs hold MXFP4 records: the layer needs fp4_format='mxfp4'")
    if (layer_obj.hidden, layer_obj.inter, layer_obj.num_experts) != (geom.hidden, geom.inter, geom.num_experts):
        raise ValueError(f"layer is {layer_obj.hidden} x {layer_obj.inter} with {layer_obj.num_experts} experts; "
                         f"the pack is {geom.hidden} x {geom.inter} with {geom.num_experts}")
    if chunk < 1:
        raise ValueError("chunk must be positive")
    check_packs(packs, geom)
    ranks = [read_rank_experts(packs, layer, r, geom) for r in range(geom.tp_ranks)]
    slot = np.asarray(layer_obj.fp4_slot)
    ids = np.nonzero(slot >= 0)[0]
    ids = ids[np.argsort(slot[ids], kind="stable")]
    if ids.size and not np.array_equal(slot[ids], np.arange(ids.size)):
        raise ValueError("the layer's FP4 slots are not 0..n-1")
    dev = layer_obj.device
    done = 0
    while done < ids.size:
        sel = ids[done:done + chunk]
        parts = join_experts([np.asarray(r[sel]) for r in ranks], geom)
        dst = [torch.from_numpy(np.ascontiguousarray(p)).pin_memory().to(dev, non_blocking=True) for p in parts]
        layer_obj.load_fp4(done, *dst)
        torch.cuda.current_stream(dev).synchronize()  # the pinned staging is freed next iteration
        done += sel.size
    return int(ids.size)
