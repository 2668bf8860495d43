"""Device-side packing and the reference-parity route plan (torch tensors in,
library kernels do the work).

- ``quantize_nvfp4`` / ``quantize_mxfp4``: fp32 weights -> packed FP4 (this
  build's RNE rule; the reference's packs came from NVIDIA);
- ``fold_nvfp4_to_mxfp4``: the exact E8M0/32 fold of
  harness/benchmarks/nvfp4_8r/build_packs.py:120-151 (refuses a lossy block);
- ``route_plan``: GroupPlanner.plan's tables (engine/.../experts/nvfp4_8r_group_plan.py:163-332).
"""

from __future__ import annotations

import torch

from . import _lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class PackError(ValueError):
    pass


def _err_buf(dev) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=dev)


def _raise_bits(where: str, err: torch.Tensor) -> None:
    bits = int(err.item())
    if bits:
        raise PackError(f"{where}: kernel error bits {bits:#x}")


def quantize_nvfp4(w: torch.Tensor):
    """fp32 [R, K] (CUDA) -> (codes uint8 [R, K/2], E4M3 scales uint8 [R, K/16], global fp32 [1])."""
    if w.dtype != torch.float32 or w.dim() != 2 or not w.is_contiguous() or not w.is_cuda:
        raise ValueError("w must be a contiguous fp32 [R, K] CUDA tensor")
    r, k = w.shape
    codes = torch.empty((r, k // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((r, k // 16), dtype=torch.uint8, device=w.device)
    glob = torch.empty(1, dtype=torch.float32, device=w.device)
    _lib.check("b200moe_quantize_nvfp4", _lib.lib().b200moe_quantize_nvfp4(
        _stream(), w.data_ptr(), r, k, codes.data_ptr(), scales.data_ptr(), glob.data_ptr()))
    return codes, scales, glob


def quantize_nvfp4_into(w: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, glob: torch.Tensor) -> None:
    """As ``quantize_nvfp4`` into caller-owned views (no allocation)."""
    r, k = w.shape
    _lib.check("b200moe_quantize_nvfp4", _lib.lib().b200moe_quantize_nvfp4(
        _stream(), w.data_ptr(), r, k, codes.data_ptr(), scales.data_ptr(), glob.data_ptr()))


def quantize_mxfp4(w: torch.Tensor, check: bool = True):
    """fp32 [R, K] (CUDA) -> (codes uint8 [R, K/2], E8M0 uint8 [R, K/32])."""
    if w.dtype != torch.float32 or w.dim() != 2 or not w.is_contiguous() or not w.is_cuda:
        raise ValueError("w must be a contiguous fp32 [R, K] CUDA tensor")
    r, k = w.shape
    codes = torch.empty((r, k // 2), dtype=torch.uint8, device=w.device)
    e8 = torch.empty((r, k // 32), dtype=torch.uint8, device=w.device)
    err = _err_buf(w.device)
    _lib.check("b200moe_quantize_mxfp4", _lib.lib().b200moe_quantize_mxfp4(
        _stream(), w.data_ptr(), r, k, codes.data_ptr(), e8.data_ptr(), err.data_ptr()))
    if check:
        _raise_bits("quantize_mxfp4", err)
    return codes, e8


def fold_nvfp4_to_mxfp4(codes: torch.Tensor, scales: torch.Tensor, glob: torch.Tensor):
    """Exact NVFP4 -> MXFP4 E8M0/32 fold on the GPU; PackError if a block cannot fold."""
    r, half_k = codes.shape
    k = half_k * 2
    oc = torch.empty_like(codes)
    oe = torch.empty((r, k // 32), dtype=torch.uint8, device=codes.device)
    err = _err_buf(codes.device)
    g = glob.reshape(1).to(torch.float32).contiguous()
    _lib.check("b200moe_fold_nvfp4_to_mxfp4", _lib.lib().b200moe_fold_nvfp4_to_mxfp4(
        _stream(), codes.data_ptr(), scales.data_ptr(), g.data_ptr(), r, k, oc.data_ptr(), oe.data_ptr(),
        err.data_ptr()))
    bits = int(err.item())
    if bits:
        raise PackError("NVFP4 block cannot fold exactly to MXFP4 E8M0/32" if bits & 8 else f"fold error {bits:#x}")
    return oc, oe


def route_plan(ids: torch.Tensor, hot_slot: torch.Tensor, second_slot: torch.Tensor | None = None,
               n_hot: int | None = None, n_second: int = 0, host: bool = False,
               iq_slot: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
    """The reference route plan in one launch.  ``second_slot`` None = every
    expert resident (one launch); else split keys (HOT, then second, then the
    WARM sentinel).  Returns perm, gids_hot, goff_hot (+ gids_host, goff_host,
    iq) as int32 tensors."""
    dev = ids.device
    flat = ids.reshape(-1).to(torch.int32).contiguous()
    n = flat.numel()
    split = second_slot is not None
    if n_hot is None:
        n_hot = int(hot_slot.numel()) if not split else int((hot_slot >= 0).sum())
    z = lambda m: torch.zeros(m, dtype=torch.int32, device=dev)  # noqa: E731
    out = {"perm": z(n), "gids_hot": z(n), "goff_hot": z(n + 1)}
    if host:
        out["gids_host"], out["goff_host"] = z(n), z(n + 1)
    if iq_slot is not None:
        out["iq"] = z(n)
    err = _err_buf(dev)
    _lib.check("b200moe_route_plan", _lib.lib().b200moe_route_plan(
        _stream(), flat.data_ptr(), n, int(hot_slot.numel()), hot_slot.data_ptr(),
        _lib.ptr(second_slot), n_hot, n_second if split else 1, int(split), int(host), _lib.ptr(iq_slot),
        out["perm"].data_ptr(), out["gids_hot"].data_ptr(), out["goff_hot"].data_ptr(),
        _lib.ptr(out.get("gids_host")), _lib.ptr(out.get("goff_host")), _lib.ptr(out.get("iq")), err.data_ptr()))
    _raise_bits("route_plan", err)
    return out
