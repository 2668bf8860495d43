"""CPU tests: the C-ABI library loads and exports every symbol the header
declares; host-side logic (tier maps, EP placement, the plugin's argument
checks) matches the reference's definitions.  No compute call needs a GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200moe.h"


@pytest.fixture(scope="module")
def lib(pkg):
    from b200moe import _lib

    if not _lib.LIB_PATH.exists():
        import __graft_entry__

        __graft_entry__.build()
    return _lib.lib()


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200moe_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(lib, pkg):
    from b200moe import _lib

    syms = declared_symbols()
    assert len(syms) >= 18
    for name in syms:
        assert hasattr(lib, name), f"{name} declared in include/b200moe.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(syms)


def test_status_names_and_version(lib):
    assert lib.b200moe_status_name(0) == b"B200MOE_OK"
    assert lib.b200moe_status_name(5) == b"B200MOE_ERR_BOUNDS"
    assert b"sm_100a" in lib.b200moe_version()


def test_config_struct_layout(pkg):
    from b200moe import _lib

    assert ctypes.sizeof(_lib.Config) == 52
    text = HEADER.read_text()
    block = text[text.index("typedef struct {"):text.index("} b200moe_config;")]
    fields = re.findall(r"(?:int32_t|float)\s+(\w+);", block)
    assert fields == [f for f, _ in _lib.Config._fields_]


def test_create_refuses_bad_config_without_gpu(lib, pkg):
    from b200moe import _lib

    h = ctypes.c_void_p()
    bad = _lib.Config(300, 2048, 384, 8, 64, 0, 0, 384, 0, 10.0, 0)  # hidden not a multiple of 256
    assert lib.b200moe_layer_create(ctypes.byref(bad), 0, ctypes.byref(h)) == 1
    bad = _lib.Config(4096, 2048, 384, 8, 65, 0, 0, 384, 0, 10.0, 0)  # max_tokens > 64
    assert lib.b200moe_layer_create(ctypes.byref(bad), 0, ctypes.byref(h)) == 1
    bad = _lib.Config(4096, 2048, 384, 8, 64, 0, 0, 200, 184, 10.0, 0, 17, 18)  # GGML type 18 is no IQ type
    assert lib.b200moe_layer_create(ctypes.byref(bad), 0, ctypes.byref(h)) == 1


def test_slot_maps_match_reference_golden(pkg):
    from b200moe import tiers

    with np.load(ROOT / "tests" / "golden" / "route_plan.npz") as z:
        for j in range(24):
            m = tiers.slot_maps(z[f"tier{j}"])
            for name in ("hot", "cold", "host", "iq"):
                assert np.array_equal(getattr(m, name), z[f"map{j}_{name}"])


def test_local_maps_partition(pkg):
    from b200moe import tiers

    tier, rank = tiers.zipf_tier(384, 150, seed=2)
    assert (tier == tiers.HOT).sum() == 150 and np.all(tier[rank < 150] == tiers.HOT)
    for world in (1, 2, 4, 8):
        seen = np.zeros(384, int)
        for r in range(world):
            fp4, iq2 = tiers.local_maps(tier, r, world)
            own = (fp4 >= 0) | (iq2 >= 0)
            assert not np.any((fp4 >= 0) & (iq2 >= 0))
            seen += own
            assert np.array_equal(np.sort(fp4[fp4 >= 0]), np.arange((fp4 >= 0).sum()))
            ids = np.flatnonzero(own)
            assert ids.min() == tiers.owner_ranges(384, world)[r].start
        assert np.all(seen == 1)
    with pytest.raises(ValueError, match="HOST"):
        tiers.local_maps(np.full(384, tiers.HOST, np.int8), 0, 1)


def test_placement_digest(pkg):
    from b200moe import tiers

    t1, _ = tiers.zipf_tier(384, 150, seed=2)
    t2 = t1.copy()
    t2[0] ^= 1
    assert tiers.placement_digest(t1, 8) == tiers.placement_digest(t1.copy(), 8)
    assert tiers.placement_digest(t1, 8) != tiers.placement_digest(t2, 8)
    assert tiers.placement_digest(t1, 4) != tiers.placement_digest(t1, 8)


def test_library_missing_fails_loudly(pkg, monkeypatch, tmp_path):
    from b200moe import _lib

    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libb200moe.so")
    with pytest.raises(RuntimeError, match="only implementation"):
        _lib.lib()


def test_library_sha256_pin(pkg, lib, monkeypatch):
    """The loader refuses a library whose bytes differ from the pinned digest
    (the reference's own rule for its kernel library)."""
    import hashlib

    from b200moe import _lib

    assert _lib.PIN_PATH.read_text().strip() == hashlib.sha256(_lib.LIB_PATH.read_bytes()).hexdigest()
    saved = _lib._LIB
    try:
        _lib._LIB = None
        monkeypatch.setenv("B200MOE_LIB_SHA256", "0" * 64)
        with pytest.raises(RuntimeError):
            _lib.lib()
    finally:
        _lib._LIB = saved


def test_plugin_refusals_follow_the_reference_hook(pkg):
    """``B200NativeMoEMethod`` refuses what the reference hook refuses
    (engine/patches/gguf_moe.patch, ``apply``: anything but output-weighted
    SiLU; ``_apply_nvfp4_8r``: non-fp32 router weights), and accepts an
    ``expert_map`` only when its local experts are exactly the layer's."""
    import types

    import torch
    from b200moe import moe

    fake = types.SimpleNamespace(fp4_slot=np.array([0, 1, -1, -1], np.int32),
                                 iq2_slot=np.array([-1, -1, 0, -1], np.int32))
    method = moe.B200NativeMoEMethod(fake)
    x = torch.zeros((2, 8), dtype=torch.float16)
    w = torch.zeros((2, 2), dtype=torch.float32)
    layer = types.SimpleNamespace(activation="silu", apply_router_weight_on_input=False, expert_map=None)
    method._checks(layer, x, w)
    for act in ("swigluoai", "gelu", "silu_no_mul"):
        with pytest.raises(ValueError, match="SiLU"):
            method._checks(types.SimpleNamespace(activation=act, expert_map=None), x, w)
    try:
        from vllm.model_executor.layers.fused_moe.activation import MoEActivation
    except Exception:
        MoEActivation = None
    if MoEActivation is not None:
        method._checks(types.SimpleNamespace(activation=MoEActivation.SILU, expert_map=None), x, w)
        with pytest.raises(ValueError):
            method._checks(types.SimpleNamespace(activation=MoEActivation.SWIGLUOAI, expert_map=None), x, w)
    with pytest.raises(ValueError):
        method._checks(types.SimpleNamespace(activation="silu", apply_router_weight_on_input=True), x, w)
    with pytest.raises(RuntimeError, match="fp32"):
        method._checks(layer, x, w.half())
    ok = types.SimpleNamespace(activation="silu", expert_map=torch.tensor([0, 1, 2, -1], dtype=torch.int32))
    method._checks(ok, x, w)
    bad = types.SimpleNamespace(activation="silu", expert_map=torch.tensor([0, 1, -1, 2], dtype=torch.int32))
    with pytest.raises(RuntimeError, match="expert_map"):
        method._checks(bad, x, w)
