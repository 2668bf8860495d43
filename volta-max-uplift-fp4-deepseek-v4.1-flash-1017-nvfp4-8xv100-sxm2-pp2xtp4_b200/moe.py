"""The routed-expert MoE plugin on B200: the drop-in for the reference's
``NativeV41Moe`` (engine/.../experts/nvfp4_8r_native.py:609-1122) and the
quant-method hook ``_apply_nvfp4_8r`` (engine/patches/gguf_moe.patch:53-80).

PyTorch is used for device memory and the current stream only; every
computation runs in ``libb200moe.so`` (hand-written sm_100a kernels).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from . import tiers as tiersmod

SWIGLU_LIMIT = 10.0
IQ_BLOCK_BYTES = {16: 66, 17: 74, 29: 56}  # GGML type -> bytes per 256 weights (IQ2_XXS, IQ2_XS, IQ1_M)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _want(name: str, t: torch.Tensor, dtype, shape=None, device=None) -> None:
    if not isinstance(t, torch.Tensor) or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {dtype} tensor, got "
                         f"{getattr(t, 'dtype', type(t))} {tuple(getattr(t, 'shape', ()))}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, the layer on {device}")


class B200NativeMoe:
    """One routed-expert MoE layer on one B200.

    ``tier`` int8 [E]: HOT experts are FP4 (``fp4_format`` "nvfp4" or
    "mxfp4"), WARM experts IQ2_XXS.  ``rank`` / ``world`` select this GPU's
    experts under expert parallelism (contiguous id ranges, or ``owner``, int32
    [E] rank of each expert, e.g. ``tiers.balanced_owners``); with world 1
    every expert is local.  Buffers are fixed at construction (``max_tokens`` for the
    graph-capturable decode ``forward``, ``max_prefill_tokens`` for
    ``forward_prefill``); forward never allocates or syncs with the host.
    ``prefill_gemm`` picks the FP4 bank's kernels: "tcgen05" (forward_prefill
    on the tensor-core grouped GEMM over dequantized f16 tiles, 128-route
    tiles; decode on the skinny kernels), "skinny" (the skinny kernels for
    both) or "fp4" (hidden and inter multiples of 256: every FP4-bank launch,
    decode and prefill, on the block-scaled FP4 tensor cores,
    tcgen05.mma.kind::mxf4nvf4 with the format's own block scales (E4M3 per 16
    or E8M0 per 32), the activations as four E2M1 planes (~1e-4 relative);
    prefills of >= 4096 routes on the tcgen05 f16 GEMM over the same weight
    units: the fastest decode and prefill) or "fp4-bs" (every call on the
    block-scaled kernel, 32-route chunks for long prefills: slower there, kept
    for comparison).  IQ experts always use their int8
    kernel.
    """

    def __init__(self, *, hidden: int, inter: int, num_experts: int, top_k: int, max_tokens: int,
                 tier, fp4_format: str = "nvfp4", max_prefill_tokens: int = 0,
                 swiglu_limit: float = SWIGLU_LIMIT, device: torch.device | int | None = None,
                 rank: int = 0, world: int = 1, prefill_gemm: str = "tcgen05", owner=None,
                 iq_types: tuple[int, int] = (16, 16)):
        if fp4_format not in ("nvfp4", "mxfp4"):
            raise ValueError(f"fp4_format must be nvfp4 or mxfp4, got {fp4_format!r}")
        if prefill_gemm not in ("tcgen05", "skinny", "fp4", "fp4-bs"):
            raise ValueError(f"prefill_gemm must be tcgen05, skinny, fp4 or fp4-bs, got {prefill_gemm!r}")
        self.prefill_gemm = prefill_gemm
        if len(iq_types) != 2 or any(t not in IQ_BLOCK_BYTES for t in iq_types):
            raise ValueError(f"iq_types are GGML types (gate/up, down) of 16 IQ2_XXS, 17 IQ2_XS, 29 IQ1_M, "
                             f"got {iq_types!r}")
        self.iq_types = (int(iq_types[0]), int(iq_types[1]))
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           (device if isinstance(device, int) else device.index))
        if dev.index is None:
            raise ValueError("the layer needs an indexed CUDA device")
        self.device = dev
        tier = tiersmod.check_tier_array(tier, num_experts)
        fp4_map, iq2_map = tiersmod.local_maps(tier, rank, world, owner)
        self.tier = tier
        self.hidden, self.inter, self.num_experts, self.top_k = hidden, inter, num_experts, top_k
        self.max_tokens, self.max_prefill_tokens = max_tokens, max_prefill_tokens
        self.fp4_format = fp4_format
        self.n_fp4, self.n_iq2 = int((fp4_map >= 0).sum()), int((iq2_map >= 0).sum())
        self.fp4_slot, self.iq2_slot = fp4_map, iq2_map
        cfg = _lib.Config(hidden, inter, num_experts, top_k, max_tokens, max_prefill_tokens,
                          _lib.NVFP4 if fp4_format == "nvfp4" else _lib.MXFP4, self.n_fp4, self.n_iq2,
                          float(swiglu_limit), {"skinny": 0, "tcgen05": 1, "fp4": 2, "fp4-bs": 3}[prefill_gemm],
                          self.iq_types[0], self.iq_types[1])
        handle = ctypes.c_void_p()
        L = _lib.lib()
        _lib.check("b200moe_layer_create", L.b200moe_layer_create(ctypes.byref(cfg), dev.index, ctypes.byref(handle)))
        self._h = handle
        _lib.check("b200moe_set_slot_maps", L.b200moe_set_slot_maps(
            self._h, fp4_map.ctypes.data_as(ctypes.c_void_p), iq2_map.ctypes.data_as(ctypes.c_void_p)))
        self.out = torch.empty((max_tokens, hidden), dtype=torch.float32, device=dev)
        self._tables_set = False
        self.stats = None  # decode route counters (enable_route_stats)

    # -------------------------------------------------------------- weights
    def load_fp4(self, slot_begin: int, w13_codes, w13_scales, w2_codes, w2_scales, globals=None) -> None:
        """Load consecutive FP4 slots from natural-layout device arrays (see
        ``include/b200moe.h``: b200moe_load_fp4)."""
        n = w13_codes.shape[0]
        bs = 16 if self.fp4_format == "nvfp4" else 32
        H, I = self.hidden, self.inter
        _want("w13_codes", w13_codes, torch.uint8, (n, 2 * I, H // 2), self.device)
        _want("w13_scales", w13_scales, torch.uint8, (n, 2 * I, H // bs), self.device)
        _want("w2_codes", w2_codes, torch.uint8, (n, H, I // 2), self.device)
        _want("w2_scales", w2_scales, torch.uint8, (n, H, I // bs), self.device)
        if self.fp4_format == "nvfp4":
            _want("globals", globals, torch.float32, (n, 3), self.device)
        _lib.check("b200moe_load_fp4", _lib.lib().b200moe_load_fp4(
            self._h, _stream(), slot_begin, n, w13_codes.data_ptr(), w13_scales.data_ptr(), w2_codes.data_ptr(),
            w2_scales.data_ptr(), _lib.ptr(globals)))

    def load_iq2(self, slot_begin: int, w1, w3, w2) -> None:
        """Load consecutive IQ slots from ggml blocks (uint8 [n][rows][K/256][B]):
        W1 / W3 blocks of the gate/up type, W2 blocks of the down type
        (``iq_types``; B = 66 IQ2_XXS, 74 IQ2_XS, 56 IQ1_M)."""
        n = w1.shape[0]
        H, I = self.hidden, self.inter
        b13, b2 = IQ_BLOCK_BYTES[self.iq_types[0]], IQ_BLOCK_BYTES[self.iq_types[1]]
        _want("w1", w1, torch.uint8, (n, I, H // 256, b13), self.device)
        _want("w3", w3, torch.uint8, (n, I, H // 256, b13), self.device)
        _want("w2", w2, torch.uint8, (n, H, I // 256, b2), self.device)
        if not self._tables_set:
            self.set_iq_tables()
        _lib.check("b200moe_load_iq2", _lib.lib().b200moe_load_iq2(
            self._h, _stream(), slot_begin, n, w1.data_ptr(), w3.data_ptr(), w2.data_ptr()))

    def set_iq_tables(self) -> None:
        """The codebooks of the layer's IQ types (ggml data, loaded from gguf-py)."""
        for t in sorted(set(self.iq_types)):
            if t == 16:
                self.set_iq2_tables()
                continue
            from gguf.quants import IQ1_M, IQ2_XS, IQ2_XXS

            cls = IQ2_XS if t == 17 else IQ1_M
            cls.init_grid()
            grid = np.ascontiguousarray(np.asarray(cls.grid, np.float32).reshape(-1, 8).astype(np.int8))
            ksigns = None if t == 29 else np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
            _lib.check("b200moe_set_iq_grid", _lib.lib().b200moe_set_iq_grid(
                self._h, t, grid.ctypes.data_as(ctypes.c_void_p), grid.shape[0],
                None if ksigns is None else ksigns.ctypes.data_as(ctypes.c_void_p)))
        self._tables_set = True

    def set_iq2_tables(self, grid: np.ndarray | None = None, ksigns: np.ndarray | None = None) -> None:
        """The IQ2_XXS codebook (ggml data): loaded from gguf-py when not given."""
        if grid is None or ksigns is None:
            from gguf.quants import IQ2_XXS

            IQ2_XXS.init_grid()
            grid = np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.int8)
            ksigns = np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()
        grid = np.ascontiguousarray(grid, np.int8)
        ksigns = np.ascontiguousarray(ksigns, np.uint8)
        if grid.shape != (256, 8) or ksigns.shape != (128,):
            raise ValueError("IQ2_XXS tables are grid int8 [256, 8] and ksigns uint8 [128]")
        _lib.check("b200moe_set_iq2_tables", _lib.lib().b200moe_set_iq2_tables(
            self._h, grid.ctypes.data_as(ctypes.c_void_p), ksigns.ctypes.data_as(ctypes.c_void_p)))
        self._tables_set = set(self.iq_types) == {16}

    # -------------------------------------------------------------- forward
    def route(self, router_logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Softmax top-k gating: fp32 logits [T, E] -> (ids int32 [T, k], weights fp32 [T, k])."""
        t = router_logits.shape[0]
        _want("router_logits", router_logits, torch.float32, (t, self.num_experts), self.device)
        ids = torch.empty((t, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((t, self.top_k), dtype=torch.float32, device=self.device)
        _lib.check("b200moe_route", _lib.lib().b200moe_route(
            self._h, _stream(), router_logits.data_ptr(), ids.data_ptr(), w.data_ptr(), t))
        return ids, w

    def _check_io(self, x, topk_ids, topk_weights):
        m = x.size(0) if x.dim() == 2 else -1
        if x.dim() != 2 or x.shape[1] != self.hidden or x.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError(f"x must be fp16 or bf16 [M, {self.hidden}], got {x.dtype} {tuple(x.shape)}")
        _want("x", x, x.dtype, None, self.device)
        if topk_ids.shape != (m, self.top_k):
            raise ValueError(f"bad routing shape {tuple(topk_ids.shape)} for M={m}")
        _want("topk_ids", topk_ids, torch.int32, (m, self.top_k), self.device)
        _want("topk_weights", topk_weights, torch.float32, (m, self.top_k), self.device)
        return m, (_lib.F16 if x.dtype == torch.float16 else _lib.BF16)

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        """Decode: x [M, H] -> fp32 [M, H], a view of the layer's persistent
        buffer (as the reference's forward returns), 1 <= M <= max_tokens."""
        m, dt = self._check_io(x, topk_ids, topk_weights)
        if not 0 < m <= self.max_tokens:
            raise ValueError(f"bad routing shape {tuple(topk_ids.shape)} for M={m}")
        out = self.out[:m]
        if self.stats is not None:
            self.stats.count(topk_ids)
        _lib.check("b200moe_forward", _lib.lib().b200moe_forward(
            self._h, _stream(), x.data_ptr(), dt, topk_ids.data_ptr(), topk_weights.data_ptr(), out.data_ptr(), m))
        return out

    def enable_route_stats(self):
        """Count this layer's decode routes on the device from now on (one
        extra launch per ``forward``, captured with it in a graph); returns the
        ``stats.RouteStats`` (the reference's counters, off unless asked for)."""
        from .stats import RouteStats

        if self.stats is None:
            self.stats = RouteStats(self.tier, self.device)
        return self.stats

    def forward_prefill(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        """Any M up to max_prefill_tokens -> a new fp32 [M, H] tensor."""
        m, dt = self._check_io(x, topk_ids, topk_weights)
        if not 0 < m <= max(self.max_prefill_tokens, self.max_tokens):
            raise ValueError(f"{m} tokens, the layer holds {self.max_prefill_tokens}")
        out = torch.empty((m, self.hidden), dtype=torch.float32, device=self.device)
        _lib.check("b200moe_forward_prefill", _lib.lib().b200moe_forward_prefill(
            self._h, _stream(), x.data_ptr(), dt, topk_ids.data_ptr(), topk_weights.data_ptr(), out.data_ptr(), m))
        return out

    def forward_static(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                       out: torch.Tensor) -> torch.Tensor:
        """Decode forward that allocates nothing: its scratch is one array built
        into the library (M <= 16, top-k <= 8, hidden <= 4096, inter <= 2048,
        <= 512 experts on this GPU), for callers that may not allocate device
        memory at decode time.  Writes the caller's fp32 ``out`` [M, H].  Calls
        share that array, so they must not overlap on the GPU."""
        m, dt = self._check_io(x, topk_ids, topk_weights)
        _want("out", out, torch.float32, (m, self.hidden), self.device)
        _lib.check("b200moe_forward_static", _lib.lib().b200moe_forward_static(
            self._h, _stream(), x.data_ptr(), dt, topk_ids.data_ptr(), topk_weights.data_ptr(), out.data_ptr(), m))
        return out

    def check_errors(self) -> None:
        """Synchronize and raise if a kernel recorded an error since the last check."""
        bits = ctypes.c_uint32(0)
        _lib.check("b200moe_check_errors", _lib.lib().b200moe_check_errors(self._h, _stream(), ctypes.byref(bits)))

    def set_debug_y13(self, y13: torch.Tensor | None) -> None:
        _lib.check("b200moe_set_debug_y13", _lib.lib().b200moe_set_debug_y13(self._h, _lib.ptr(y13)))

    def debug_perm(self, n: int) -> torch.Tensor:
        """The route permutation of the last forward (int32 [n]: route index at each sorted position)."""
        out = torch.empty(n, dtype=torch.int32, device=self.device)
        _lib.check("b200moe_debug_perm", _lib.lib().b200moe_debug_perm(self._h, _stream(), out.data_ptr(), n))
        return out

    def set_split_k(self, ks_fp4: int = 0, ks_iq2: int = 0) -> None:
        """Fix the GEMV split-K per bank (1, 2, 4 or 8; 0 = chosen per launch).
        Layers with the same fixed split-K give bit-equal rows per route."""
        _lib.check("b200moe_set_split_k", _lib.lib().b200moe_set_split_k(self._h, int(ks_fp4), int(ks_iq2)))

    def set_decode_fusion(self, max_routes: int = 64) -> None:
        """Route-count limit (<= 64) of the fused two-launch decode of an FP4-only
        layer on the block-scaled path; 0 (the layer's default) runs every call
        on the chained launches, measured faster on B200.  Both give the same
        output bits."""
        _lib.check("b200moe_set_decode_fusion", _lib.lib().b200moe_set_decode_fusion(self._h, int(max_routes)))

    def set_timing_events(self, events) -> None:
        """Record torch.cuda.Event objects between the forward's launches (None: off)."""
        events = list(events or [])
        for e in events:
            e.record()  # torch creates the CUDA event lazily, at its first record
        self._timing_events = events  # keep them alive while the library holds their handles
        arr = (ctypes.c_void_p * max(1, len(events)))(*[e.cuda_event for e in events])
        _lib.check("b200moe_set_timing_events", _lib.lib().b200moe_set_timing_events(self._h, arr, len(events)))

    def debug_inter(self, rows: int) -> torch.Tensor:
        """SwiGLU output rows of the last forward (fp16 [rows, I], by sorted route position)."""
        out = torch.empty((rows, self.inter), dtype=torch.float16, device=self.device)
        _lib.check("b200moe_debug_inter", _lib.lib().b200moe_debug_inter(self._h, _stream(), out.data_ptr(), rows))
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().b200moe_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class B200NativeMoEMethod:
    """The quant-method hook: the counterpart of ``_apply_nvfp4_8r``
    (engine/patches/gguf_moe.patch:53-80).  M in 1..max_tokens goes to the
    graph-capturable ``forward``, anything larger to ``forward_prefill``; the
    result is cast to x's dtype.  ``apply_logits`` takes router logits instead
    of a routing (gating runs in the library)."""

    def __init__(self, moe: B200NativeMoe):
        self.native_moe = moe
        self._checked_map = None  # the expert_map tensor already checked against the layer's experts

    def _checks(self, layer, x, topk_weights) -> None:
        """The refusals of the reference hook (gguf_moe.patch, ``apply`` and
        ``_apply_nvfp4_8r``): output-weighted SiLU only, fp32 router weights.
        The reference refuses any ``expert_map`` (it holds every expert); this
        layer may hold a share of them (expert parallelism), so a map is
        accepted only when its local experts (entries >= 0) are exactly this
        layer's, checked once per map tensor."""
        act = getattr(layer, "activation", "silu")
        if getattr(layer, "apply_router_weight_on_input", False) or \
                str(getattr(act, "value", act)).lower() != "silu":
            raise ValueError("b200moe experts require output-weighted SiLU routing")
        if topk_weights.dtype != torch.float32 or x.dtype not in (torch.float16, torch.bfloat16):
            raise RuntimeError(f"b200moe needs fp16/bf16 x and fp32 weights, got {x.dtype}/{topk_weights.dtype}")
        emap = getattr(layer, "expert_map", None)
        if emap is not None and emap is not self._checked_map:
            moe = self.native_moe
            local = np.asarray(torch.as_tensor(emap).cpu()) >= 0
            mine = (moe.fp4_slot >= 0) | (moe.iq2_slot >= 0)
            if local.shape != mine.shape or not np.array_equal(local, mine):
                raise RuntimeError("layer.expert_map does not match the experts this layer holds "
                                   "(b200moe takes global ids; its local experts come from its owner map)")
            self._checked_map = emap

    def apply(self, layer, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
              shared_experts=None, shared_experts_input=None) -> torch.Tensor:
        self._checks(layer, x, topk_weights)
        moe = self.native_moe
        ids = topk_ids.to(torch.int32).contiguous()
        x = x.contiguous()
        w = topk_weights.contiguous()
        if 1 <= x.size(0) <= moe.max_tokens:
            return moe.forward(x, ids, w).to(x.dtype)
        return moe.forward_prefill(x, ids, w).to(x.dtype)

    def apply_logits(self, layer, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        ids, w = self.native_moe.route(router_logits.float().contiguous())
        return self.apply(layer, x, w, ids)
