"""ctypes binding of ``libb200moe.so`` (the C ABI of ``include/b200moe.h``).

The library is the only compute path: if it is missing or fails to load, every
entry point raises; there is no CPU or PyTorch fallback.  As the reference pins
its compiled kernel library by sha256 (engine/.../experts/nvfp4_8r_qpn_rb.py:37-41,
70-81), the loader refuses a library whose bytes differ from the digest the build
wrote beside it (``libb200moe.so.sha256``) or from ``B200MOE_LIB_SHA256`` when
that is set.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libb200moe.so"
PIN_PATH = HERE / "libb200moe.so.sha256"

P = ctypes.c_void_p
I32 = ctypes.c_int
F32 = ctypes.c_float

STATUS = {
    0: "B200MOE_OK",
    1: "B200MOE_ERR_INVALID_ARG",
    2: "B200MOE_ERR_DTYPE",
    3: "B200MOE_ERR_ALIGN",
    4: "B200MOE_ERR_CUDA",
    5: "B200MOE_ERR_BOUNDS",
    6: "B200MOE_ERR_TIMEOUT",
    7: "B200MOE_ERR_FORMAT",
    8: "B200MOE_ERR_RANGE",
    9: "B200MOE_ERR_NOMEM",
    10: "B200MOE_ERR_STATE",
}
F16, BF16, FP32 = 0, 1, 2
NVFP4, MXFP4, IQ2XXS = 0, 1, 2


class Config(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
                ("max_prefill_tokens", ctypes.c_int32), ("fp4_format", ctypes.c_int32),
                ("n_fp4", ctypes.c_int32), ("n_iq2", ctypes.c_int32), ("swiglu_limit", ctypes.c_float),
                ("prefill_gemm", ctypes.c_int32), ("iq_type13", ctypes.c_int32), ("iq_type2", ctypes.c_int32)]


# name -> (argtypes, restype); every symbol include/b200moe.h declares
SIGNATURES = {
    "b200moe_status_name": ([I32], ctypes.c_char_p),
    "b200moe_version": ([], ctypes.c_char_p),
    "b200moe_layer_create": ([ctypes.POINTER(Config), I32, ctypes.POINTER(P)], I32),
    "b200moe_layer_destroy": ([P], I32),
    "b200moe_set_slot_maps": ([P, P, P], I32),
    "b200moe_set_iq2_tables": ([P, P, P], I32),
    "b200moe_set_iq_grid": ([P, I32, P, I32, P], I32),
    "b200moe_load_fp4": ([P, P, I32, I32, P, P, P, P, P], I32),
    "b200moe_load_iq2": ([P, P, I32, I32, P, P, P], I32),
    "b200moe_route": ([P, P, P, P, P, I32], I32),
    "b200moe_forward": ([P, P, P, I32, P, P, P, I32], I32),
    "b200moe_forward_prefill": ([P, P, P, I32, P, P, P, I32], I32),
    "b200moe_forward_static": ([P, P, P, I32, P, P, P, I32], I32),
    "b200moe_check_errors": ([P, P, ctypes.POINTER(ctypes.c_uint32)], I32),
    "b200moe_set_debug_y13": ([P, P], I32),
    "b200moe_debug_perm": ([P, P, P, I32], I32),
    "b200moe_debug_inter": ([P, P, P, I32], I32),
    "b200moe_set_timing_events": ([P, P, I32], I32),
    "b200moe_set_split_k": ([P, I32, I32], I32),
    "b200moe_set_decode_fusion": ([P, I32], I32),
    "b200moe_route_plan": ([P, P, I32, I32, P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P], I32),
    "b200moe_quantize_nvfp4": ([P, P, I32, I32, P, P, P], I32),
    "b200moe_quantize_mxfp4": ([P, P, I32, I32, P, P, P], I32),
    "b200moe_fold_nvfp4_to_mxfp4": ([P, P, P, P, I32, I32, P, P, P], I32),
    "b200moe_gate": ([P, P, I32, I32, I32, P, P, P], I32),
    "b200moe_route_stats": ([P, P, I32, I32, P, P, P, P, P, P, P], I32),
    "b200moe_ep_workspace_bytes": ([I32, I32], ctypes.c_size_t),
    "b200moe_ep_dispatch": ([P, P, I32, P, I32, I32, I32, I32, P, I32, P, P, P, P, P, ctypes.c_size_t, P], I32),
    "b200moe_ep_combine": ([P, P, P, P, I32, I32, I32, P, P], I32),
    "b200moe_ep_create": ([I32, I32, I32, I32, I32, P], I32),
    "b200moe_ep_ipc_handle": ([P, P], I32),
    "b200moe_ep_connect": ([P, P], I32),
    "b200moe_ep_destroy": ([P], I32),
    "b200moe_ep_recv_buffers": ([P, P, P, P, P, P, P], I32),
    "b200moe_ep_push": ([P, P, P, I32, P, I32, I32, I32, P], I32),
    "b200moe_ep_return": ([P, P], I32),
    "b200moe_ep_forward": ([P, P, P, I32], I32),
    "b200moe_ep_combine_p2p": ([P, P, P, P, I32, I32, I32, P, P, P], I32),
    "b200moe_ep_check_errors": ([P, P, P], I32),
    "b200moe_ep_received": ([P, P, P, P, I32], I32),
    "b200moe_forward_rows": ([P, P, P, P, P, P, I32, P], I32),
    "b200moe_f32_to_f16": ([P, P, ctypes.c_int64, P], I32),
    "b200moe_mma_peak": ([I32, I32, I32, ctypes.POINTER(F32), ctypes.POINTER(F32)], I32),
}

_LIB: ctypes.CDLL | None = None


class B200MoeError(RuntimeError):
    """A non-zero status from the library; ``.status`` holds the code."""

    def __init__(self, where: str, status: int):
        self.status = status
        super().__init__(f"{where}: {STATUS.get(status, status)}")


def lib() -> ctypes.CDLL:
    """The loaded library (raises when it was not built: no fallback exists)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                               "(the CUDA library is the only implementation)")
        want = os.environ.get("B200MOE_LIB_SHA256") or (PIN_PATH.read_text().strip() if PIN_PATH.exists() else "")
        if want:
            got = hashlib.sha256(LIB_PATH.read_bytes()).hexdigest()
            if got != want:
                raise RuntimeError(f"{LIB_PATH} is sha256 {got}, the pin is {want}: rebuild with "
                                   "__graft_entry__.build()")
        dll = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(dll, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = dll
    return _LIB


def check(where: str, status: int) -> None:
    if status != 0:
        raise B200MoeError(where, status)


def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
