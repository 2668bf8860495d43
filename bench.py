#!/usr/bin/env python
"""Benchmark of the routed-expert MoE layer on B200 (one JSON line on rank 0).

Workloads (all inputs seeded synthetic, weights
random-init and packed by the library's own quantizers):

``c1`` (default) configs[1], the decode layer the metric is quoted on: hidden
    4096, 384 routed experts, intermediate 2048, top-8 from router logits
    ~N(0,1), all experts NVFP4 (weights ~N(0,0.02)), bf16 activations ~N(0,1),
    M = 64 tokens per step (``--m`` picks 1, 8, 32 or 64).  At M >= 8 a step
    streams >= 0.8 GB of expert weights, far above the 126 MB L2; at M = 1 the
    8 routed experts (113 MB) would fit, so M = 1 rotates over 8 seeded
    routings, one per step (``config.l2``).
``c2`` configs[2], the mixed-tier decode layer at M = 32: a seeded Zipf(1.1)
    tier map puts the 150 most popular experts in NVFP4 and 234 in IQ2_XXS;
    router logits alpha * log p(rank) + Gumbel noise, alpha chosen from a grid
    so that about 80 % of routes reach the NVFP4 experts.
``c3`` configs[3], prefill: T = 4096 tokens (``--tokens 16384``), MXFP4
    experts, logits ~U(0,1).
``c4`` configs[4], a 40-layer stack of c2 layers, one decode batch of 256
    tokens for the whole box (strong scaling), residual adds between layers,
    experts sharded over the N GPUs (peer-memory exchange); one CUDA graph.

The default run (``python bench.py``) prints the configs[1] M = 64 line and,
under ``also``, the same measurements for configs[1] M = 1 / 8 / 32,
configs[2] and configs[3] T = 4096, so that one driver run measures every
single-GPU config (``--no-also`` skips them).

A step = gating (router logits -> top-8) + the layer forward, all on the GPU.
Decode steps replay one CUDA graph per step (the reference captures its
decode path the same way); ``--eager`` launches them one by one.

``value``    tokens/s of the whole job, inputs resident in HBM, CUDA events on
             the launching stream around exactly K steps, max over ranks.
``e2e``      the same through the public API with host buffers: each step
             copies x and the logits from pinned host memory and reads the
             output back, inside the timed region.
``parity``   the run's own output against a plain fp32 dequant-then-matmul
             reference (torch on the GPU, tests/torch_ref.py) on the same
             inputs, before the timed region: rel-L2 and the tolerance.  Under
             expert parallelism: bit-equality with the single-GPU layer.
``roofline`` the dominant launch: algorithmic bytes (routed distinct experts x
             the projection's packed bytes) or FLOPs (c3: 2 x routes x
             weights) over its event-timed duration, against
             MEASURED_PEAKS.json.
``cpu_baseline`` this build's AVX2 restatement of the reference's CPU expert
             kernel (oracle/cpu_moe.c, OpenMP on every core of the process's
             affinity) on the same routing.

``--impl reference`` times the reference's CPU expert path on the workload
(rank 0 only, without the product library; see ``run_reference``).

Multi-GPU (torchrun, N ranks, expert parallel over the library's NVLink
peer-memory exchange): the configs[1] decode batch of 64 tokens is split over
the N GPUs (64 / N tokens per GPU: strong scaling, the same work as the
N = 1 line), experts sharded by id; ``weak_scaling`` adds the 64-tokens-per-
GPU run.  ``c4`` runs the 40-layer stack instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, E, K_TOP = 4096, 2048, 384, 8
W13_BYTES = 2 * I * H // 2 + 2 * I * H // 16   # NVFP4 codes + E4M3 scales
W2_BYTES = H * I // 2 + H * I // 16
EXPERT_BYTES = W13_BYTES + W2_BYTES            # 14,155,776
MX_W13_BYTES = 2 * I * H // 2 + 2 * I * H // 32
MX_W2_BYTES = H * I // 2 + H * I // 32
IQ_W13_BYTES = 2 * I * H // 256 * 66           # 4,325,376
IQ_W2_BYTES = H * I // 256 * 66                # 2,162,688
C2_HOT, C2_HOT_SHARE = 150, 0.80
TOL_FP4 = 2e-3   # block-scaled FP4 path (four E2M1 activation planes) vs the fp32 dequant reference
TOL_LAYER = 1e-2  # the reference's layer rule (harness/benchmarks/nvfp4_8r/accept_p2.py:36)

# DRAM bytes per routed expert of the W13 launch, copied from the ncu captures
# of `python bench.py --profile` (dram__bytes_read.sum + dram__bytes_write.sum
# of that launch over its 289 distinct experts), kept with the capture's
# command in profiles/fp4_w13_c1_decode.md and profiles/gemv_w13_c1_decode.md.
NCU_W13_TRAFFIC_PER_EXPERT = {"fp4": 2.7447e9 / 289, "gemv": None}

DTYPE_FP4 = "e2m1x4 activations (E4M3 block scales) x nvfp4 weights, f32 accumulate"
DTYPE_GEMV = "f16 activations x nvfp4 weights dequantized to f16, f32 accumulate"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4"], default="c1")
    ap.add_argument("--layers", type=int, default=40, help="c4: layers in the stack")
    ap.add_argument("--batch", type=int, default=256, help="c4: decode tokens of the whole box per step")
    ap.add_argument("--m", type=int, default=None, choices=[1, 8, 32, 64],
                    help="decode tokens per step (c1 default 64, c2 default 32; multi-GPU: of the whole box)")
    ap.add_argument("--tokens", type=int, default=4096,
                    help="c3 prefill tokens (4096 or 16384 for configs[3]; other values with --experts for a "
                         "small ncu capture)")
    ap.add_argument("--eager", action="store_true", help="decode: launch each kernel instead of a graph replay")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="multi-GPU: the library's NVLink peer-memory exchange (default) or NCCL all-to-all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-also", action="store_true", help="default run: skip the other configs' sub-results")
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts (384 = configs[1]; fewer only for a small ncu capture)")
    ap.add_argument("--split-k", type=int, default=0,
                    help="fix the GEMV split-K (0 = chosen per call; set only to give a small ncu capture "
                         "the split-K of the full-size run)")
    ap.add_argument("--placement", choices=["range", "balanced"], default="range",
                    help="c4 over N > 1 GPUs: experts by id range, or tiers.balanced_owners on the expected routes")
    ap.add_argument("--iq-types", default="16,16",
                    help="c2: GGML types of the IQ experts' gate/up and down (16 IQ2_XXS, 17 IQ2_XS, 29 IQ1_M)")
    ap.add_argument("--gemm", choices=["fp4", "fp4-bs", "gemv"], default="fp4",
                    help="the FP4 bank on the block-scaled FP4 tensor path (tcgen05.mma kind::mxf4nvf4, default; "
                         "c3: the tcgen05 f16 GEMM over the same weight units), fp4-bs (c3: the block-scaled kernel "
                         "with 32-route chunks) or gemv (decode: the skinny GEMV; c3: the tcgen05 f16 GEMM over the "
                         "decode bank's units)")
    ap.add_argument("--profile", action="store_true",
                    help="warm-up + timed steps only (no per-launch, e2e or CPU passes): the ncu command")
    a = ap.parse_args()
    if a.m is None:
        a.m = 32 if a.workload == "c2" else 64
    return a


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def loaded_libraries() -> list[str]:
    """Shared objects of this repository mapped into this process."""
    try:
        maps = Path("/proc/self/maps").read_text().splitlines()
    except OSError:
        return []
    root = str(ROOT)
    return sorted({ln.split()[-1][len(root) + 1:] for ln in maps
                   if ln.split() and ln.split()[-1].startswith(root) and ".so" in ln.split()[-1]})


class Clocks:
    """SM clock and throttle reasons polled through NVML every 2 ms while the
    timed region runs (reading only; no setting is changed)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, device):
        import threading

        self.samples, self.bits, self.error = [], 0, None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            import torch

            props = torch.cuda.get_device_properties(device)
            try:
                bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report why
            self.error = f"nvml unavailable: {exc}"[:200]
            return
        self.stop_flag = threading.Event()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.bits |= int(get_reasons(self.h))
            except Exception as exc:
                self.error = str(exc)[:200]
                return
            self.stop_flag.wait(0.002)

    def stop(self) -> dict:
        if self.error and not self.samples:
            return {"error": self.error}
        self.stop_flag.set()
        self.t.join(timeout=2)
        if not self.samples:
            return {"error": self.error or "no samples"}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for b, n in self.REASONS.items() if self.bits & b),
                "samples": len(self.samples), "source": "nvml, polled every 2 ms during the timed region"}


# ------------------------------------------------------------------ tensor peaks
PEAK_KINDS = {0: ("kind::f16 (f16 x f16, N 256)", 100000), 1: ("kind::f8f6f4 (E4M3 x E4M3, N 256)", 100000),
              2: ("kind::mxf4nvf4 block16 (E2M1, UE4M3 per 16, N 128)", 200000),
              3: ("kind::mxf4nvf4 block32 (E2M1, UE8M0 per 32, N 128)", 200000),
              4: ("kind::f16 (f16 x f16, N 128)", 200000)}


_PEAKS: dict = {}


def tensor_peaks(dev) -> dict:
    """Dense tcgen05 throughput of this GPU per MMA kind (b200moe_mma_peak: one
    CTA per SM, back-to-back MMAs on shared-memory operands, ~30 ms each), with
    the SM clocks seen while they ran; measured once per process."""
    import ctypes

    from b200moe import _lib

    if _PEAKS:
        return _PEAKS
    out = _PEAKS
    clk = Clocks(dev)
    for kind, (name, iters) in PEAK_KINDS.items():
        tf, ms = ctypes.c_float(), ctypes.c_float()
        _lib.check("b200moe_mma_peak", _lib.lib().b200moe_mma_peak(dev.index, kind, iters, ctypes.byref(tf),
                                                                   ctypes.byref(ms)))
        out[name] = {"tflops": float(tf.value), "ms": float(ms.value)}
    out["clocks"] = clk.stop()
    out["how"] = ("tcgen05.mma, M 128, one CTA per SM (148), operands in shared memory, "
                  "csrc/peak.cu; dense FLOPs = 2 M N K per MMA")
    return out


# ------------------------------------------------------------------ parity
def torch_ref():
    sys.path.insert(0, str(ROOT / "tests"))
    import torch_ref as tr

    return tr


def fp4_dequant(bank, inter: int):
    """Slot -> (W13 fp32 [2I, H], W2 fp32 [H, I]) of a natural-layout FP4 bank,
    by the reference's decode formula (torch, on the bank's device)."""
    import torch

    tr = torch_ref()

    def deq(j: int):
        if bank.fmt == "nvfp4":
            g = bank.globals[j]
            w13 = torch.cat([tr.nvfp4_decode(bank.w13_codes[j, :inter], bank.w13_scales[j, :inter], g[0]),
                                tr.nvfp4_decode(bank.w13_codes[j, inter:], bank.w13_scales[j, inter:], g[1])])
            return w13, tr.nvfp4_decode(bank.w2_codes[j], bank.w2_scales[j], g[2])
        return tr.mxfp4_decode(bank.w13_codes[j], bank.w13_scales[j]), tr.mxfp4_decode(bank.w2_codes[j],
                                                                                         bank.w2_scales[j])
    return deq


def iq2xxs_dequant(bank):
    import torch
    from gguf.quants import IQ2_XXS

    tr = torch_ref()
    IQ2_XXS.init_grid()
    grid = np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.int8)
    ksigns = np.frombuffer(IQ2_XXS.ksigns, np.uint8).copy()

    def deq(j: int):
        w13 = torch.cat([tr.iq2xxs_decode(bank.w1[j], grid, ksigns), tr.iq2xxs_decode(bank.w3[j], grid, ksigns)])
        return w13, tr.iq2xxs_decode(bank.w2[j], grid, ksigns)
    return deq


def parity(out, x, ids, w, dequant, tol: float, rows=None, what: str = "") -> dict:
    """rel-L2 of the layer output against the fp32 dequant-then-matmul
    reference on the same inputs (``rows``: a sample of the tokens)."""
    import torch

    tr = torch_ref()
    sel = slice(None) if rows is None else torch.as_tensor(rows, device=x.device, dtype=torch.long)
    ref = tr.layer_forward(x[sel].float(), ids[sel], w[sel], dequant)
    err = tr.rel_l2(out[sel].float(), ref)
    n = x.shape[0] if rows is None else len(rows)
    return {"rel_l2": err, "tol": tol, "ok": bool(err < tol), "tokens_checked": int(n),
            "reference": "fp32 dequant-then-matmul (torch on the GPU, tests/torch_ref.py)" + (f"; {what}" if what else "")}


# ------------------------------------------------------------------ CPU legs
def fp4_expert(bank, j: int, fmt: int) -> dict:
    """One expert of a natural-layout FP4 bank as the C oracle takes it."""
    g = bank.globals[j].cpu().numpy() if bank.globals is not None else np.ones(3, np.float32)
    return dict(fmt=fmt, w13c=bank.w13_codes[j].cpu().numpy(), w13s=bank.w13_scales[j].cpu().numpy(),
                g13=g[:2].copy(), w2c=bank.w2_codes[j].cpu().numpy(), w2s=bank.w2_scales[j].cpu().numpy(),
                g2=float(g[2]))


def cpu_fp4_layer(experts_of, ids_np, w_np, x_np, tokens, sample_experts=None, reps=2) -> dict:
    """The AVX2 C port (OpenMP, every core of this process's affinity) on the
    layer of this routing: every routed expert, or a bounded sample of them
    scaled to the layer by routes."""
    from oracle import cpu_layer

    used = np.unique(ids_np[ids_np >= 0])
    pick = used if sample_experts is None else used[:sample_experts]
    experts = {int(e): experts_of(int(e)) for e in pick.tolist()}
    cpu = cpu_layer.CpuMoe(H, I, avx2=True)
    cpu.forward(x_np, ids_np, w_np, experts, only=pick)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu.forward(x_np, ids_np, w_np, experts, only=pick)
    dt = (time.perf_counter() - t0) / reps
    routes_all = int((ids_np >= 0).sum())
    routes_pick = int(np.isin(ids_np, pick).sum())
    layer_s = dt * routes_all / max(routes_pick, 1)
    what = "full layer" if sample_experts is None else f"{pick.size} of {used.size} routed experts " \
                                                       f"({routes_pick} of {routes_all} routes), scaled by routes"
    return {"value": tokens / layer_s, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
            "sample": f"{what}; {reps} timed runs, {dt * 1e3:.1f} ms each (oracle/cpu_moe.c oracle_expert_avx2)",
            "ms_per_layer": layer_s * 1e3}


def cpu_iq_part(iq_blocks_of, iq_ids, ids_np, x_np, iq_types, sample: int) -> tuple[float, str]:
    """Seconds per layer of the IQ experts on the host: ggml dequant (numpy
    restatement of gguf-py's) then fp32 matmuls, the reference's CPU route for
    them (harness/benchmarks/nvfp4_8r/make_t3_refs.py:58-72), on a bounded
    sample scaled by routes."""
    from oracle import moe_oracle as mo

    pick = iq_ids[:sample]
    t0 = time.perf_counter()
    for e in pick.tolist():
        b1, b3, b2 = iq_blocks_of(int(e))
        w13 = np.concatenate([mo.iq_decode(iq_types[0], b1), mo.iq_decode(iq_types[0], b3)])
        w2 = mo.iq_decode(iq_types[1], b2)
        rows = np.nonzero(ids_np == e)[0]
        mo.expert_fp32(x_np[rows], w13, w2)
    dt = time.perf_counter() - t0
    routes_pick = int(np.isin(ids_np, pick).sum())
    return dt * np.isin(ids_np, iq_ids).sum() / max(routes_pick, 1), f"{pick.size} of {iq_ids.size} IQ experts"


# ------------------------------------------------------------------ job
class Job:
    """Rank, device and the timing helpers shared by the workloads."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world > 1:
            from datetime import timedelta

            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        self.dev = torch.device("cuda", local)
        torch.cuda.set_device(self.dev)

    def maxall(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def allok(self, ok: bool) -> bool:
        return self.maxall(0.0 if ok else 1.0) == 0.0

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def timed(self, step, steps: int, clocks: bool = True) -> tuple[float, dict | None]:
        """ms per step over exactly `steps` steps (events on the current stream,
        barrier + synchronize on both sides, max over ranks) and the clocks."""
        import torch

        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = Clocks(self.dev) if (clocks and self.rank == 0) else None
        self.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        self.barrier()
        c = clk.stop() if clk else None
        return self.maxall(e0.elapsed_time(e1) / steps), c

    def finish(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


def graphed(step, use_graph: bool, warm: int):
    """Warm the step eagerly, then (decode) capture it in one CUDA graph."""
    import torch

    for _ in range(max(3, warm)):
        step()
    torch.cuda.synchronize()
    if not use_graph:
        return step, None
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # one more warm call on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return g.replay, g


def rotating(steps, use_graph: bool, warm: int):
    """One graph per step function; the returned step replays them in turn
    (a different routing per step keeps a small working set out of L2)."""
    runs, graphs = [], []
    for s in steps:
        r, g = graphed(s, use_graph, warm)
        runs.append(r)
        graphs.append(g)
    if len(runs) == 1:
        return runs[0], graphs
    state = {"i": 0}

    def run():
        runs[state["i"] % len(runs)]()
        state["i"] += 1
    return run, graphs


def per_launch(layer, steps_fns, steps: int, n_events: int) -> np.ndarray:
    """Mean duration (ms) between the layer's timing events (eager steps,
    rotating over ``steps_fns``)."""
    import torch

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_events)]
    layer.set_timing_events(evs)
    per = np.zeros(n_events - 1)
    for i in range(steps):
        steps_fns[i % len(steps_fns)]()
        torch.cuda.synchronize()
        per += [evs[j].elapsed_time(evs[j + 1]) for j in range(n_events - 1)]
    layer.set_timing_events(None)
    return per / steps


def e2e_decode(job, layer, xs, logits_list, m: int, steps: int, use_graph: bool) -> dict:
    """The public API with pinned host buffers: H2D of x and logits, gating,
    forward, D2H of the output, every step inside the timed region (rotating
    over the routings like the device-timed run)."""
    import torch

    fns = []
    keep = []
    for x, logits in zip(xs, logits_list):
        hx = x.cpu().pin_memory()
        hl = logits.cpu().pin_memory()
        hout = torch.empty((m, layer.hidden), dtype=torch.float32).pin_memory()
        dx, dl = torch.empty_like(x), torch.empty_like(logits)
        keep.append((hx, hl, hout, dx, dl))

        def step(hx=hx, hl=hl, hout=hout, dx=dx, dl=dl):
            dx.copy_(hx, non_blocking=True)
            dl.copy_(hl, non_blocking=True)
            hout.copy_(layer.forward(dx, *layer.route(dl)), non_blocking=True)
        fns.append(step)
    run, graphs = rotating(fns, use_graph, 2)
    ms, _ = job.timed(run, steps, clocks=False)
    layer.check_errors()
    del graphs
    hx, hl, hout = keep[0][:3]
    return {"value": job.world * m / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
            "d2h_bytes_per_step": int(hout.numel() * hout.element_size())}


def line_base(job, args, metric, value, ms, config, dtype, steps=None) -> dict:
    return {"metric": metric, "value": value, "unit": "tokens/s", "n_gpus": job.world,
            "steps": args.steps if steps is None else steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded; random-init experts)", "config": config}


# --------------------------------------------------------------------------- c1
def c1_inputs(m: int, n_exp: int, dev, rotations: int):
    """x bf16 [m, H] and logits [m, E] of configs[1] (seed 1000 + m), plus
    further seeded routings when the step rotates."""
    import torch

    xs, ls = [], []
    for r in range(rotations):
        g = torch.Generator(device=dev).manual_seed(1000 + m + 100003 * r)
        xs.append(torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16))
        ls.append(torch.randn((m, E), generator=g, device=dev)[:, :n_exp].contiguous())
    return xs, ls


def c1_layer(job, n_exp: int, f4: bool):
    from b200moe import moe, synth

    bank = synth.make_fp4_bank(n_exp, H, I, "nvfp4", 1000, job.dev)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=n_exp, top_k=K_TOP, max_tokens=64,
                              tier=np.zeros(n_exp, np.int8), device=job.dev, prefill_gemm="fp4" if f4 else "tcgen05")
    synth.load_bank(layer, bank)
    layer.check_errors()
    return layer, bank


def run_c1(job, m: int, layer=None, bank=None, main: bool = True) -> dict:
    """configs[1] decode at M = m on one GPU (the layer and bank may be shared
    with other M)."""
    import torch

    args, dev = job.args, job.dev
    use_graph = not args.eager
    f4 = args.gemm != "gemv"
    n_exp = args.experts
    rotations = 8 if m == 1 else 1
    own = layer is None
    if own:
        layer, bank = c1_layer(job, n_exp, f4)
    if args.split_k:
        layer.set_split_k(args.split_k, 0)
    xs, ls = c1_inputs(m, n_exp, dev, rotations)
    if args.profile:
        del bank
        torch.cuda.synchronize()
        for i in range(args.warmup + args.steps):
            layer.forward(xs[i % rotations], *layer.route(ls[i % rotations]))
        torch.cuda.synchronize()
        layer.check_errors()
        distinct = int(torch.unique(layer.route(ls[0])[0]).numel())
        layer.close()
        return {"profile_run": True, "experts": n_exp, "m": m, "distinct_experts": distinct,
                "w13_algorithmic_bytes": distinct * W13_BYTES, "w2_algorithmic_bytes": distinct * W2_BYTES}
    config = {"workload": f"configs[1] decode layer: hidden {H}, {n_exp} experts NVFP4, inter {I}, top-{K_TOP}, M={m}",
              "gemm": "block-scaled FP4 tensor path (tcgen05.mma kind::mxf4nvf4, E4M3 block scales in TMEM, "
                      "activations as four E2M1 planes)" if f4 else "skinny GEMV (mma.sync, weights dequantized "
                                                                     "in registers)",
              "tokens_per_step": m, "hidden": H, "inter": I, "experts": n_exp, "top_k": K_TOP, "format": "nvfp4",
              "l2": "inputs larger than L2 (>= 0.8 GB of expert weights streamed per step)" if m > 1 else
                    f"inputs larger than L2: {rotations} seeded routings replayed in turn, one per step "
                    "(8 x ~113 MB of experts, different experts from one step to the next)",
              "launch": "one CUDA graph replay per step" if use_graph else "eager launches",
              "parallelism": "single GPU"}
    if n_exp != E:
        config["workload"] += f" (ncu capture case: {n_exp} experts)"

    # parity on the first routing, before the timed region
    ids0, w0 = layer.route(ls[0])
    out0 = layer.forward(xs[0], ids0, w0).clone()
    layer.check_errors()
    par = parity(out0, xs[0], ids0, w0, fp4_dequant(bank, I), TOL_FP4 if f4 else TOL_LAYER)

    fns = [(lambda x=x, lg=lg: layer.forward(x, *layer.route(lg))) for x, lg in zip(xs, ls)]
    run, graphs = rotating(fns, use_graph, args.warmup)
    layer.check_errors()
    distinct = float(np.mean([torch.unique(layer.route(lg)[0]).numel() for lg in ls]))
    ms, clk = job.timed(run, args.steps)
    layer.check_errors()
    value = m / (ms / 1e3)
    del graphs

    if f4:  # start, convert (none for bf16 x), plan, x planes (made with the plan up to 32 routes), W13
        #     (+SwiGLU), SwiGLU planes, W2, combine (in the W2 epilogue up to 64 routes)
        fused_combine = m * K_TOP <= 64
        per = per_launch(layer, fns, args.steps, 7 if fused_combine else 8)
        t_w13_ms = float(per[3])
        names = ["convert", "plan", "x_planes", "w13", "swiglu_planes", "w2"] + ([] if fused_combine else ["combine"])
    else:  # convert, plan, W13, W2 (+SwiGLU or combine: fused up to 32 routes)
        sep = m * K_TOP > 32
        per = per_launch(layer, fns, args.steps, 6 if sep else 5)
        t_w13_ms = float(per[2])
        names = ["convert", "plan", "w13", "w2"] + (["combine"] if sep else [])
    pk = peaks()
    achieved = distinct * W13_BYTES / (t_w13_ms / 1e3) / 1e9
    layer_bytes = distinct * EXPERT_BYTES
    tpe = NCU_W13_TRAFFIC_PER_EXPERT["fp4" if f4 else "gemv"]
    traffic = tpe * distinct if (tpe and n_exp == E) else None
    e2e = e2e_decode(job, layer, xs, ls, m, args.steps, use_graph)

    cpu = None
    if main and job.rank == 0 and not args.no_cpu_baseline:
        ids_np, w_np = ids0.cpu().numpy(), w0.cpu().numpy()
        cpu = cpu_fp4_layer(lambda e: fp4_expert(bank, e, 0), ids_np, w_np, xs[0].float().cpu().numpy(), m)
    line = line_base(job, args, "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m, value, ms, config,
                     DTYPE_FP4 if f4 else DTYPE_GEMV)
    line.update({
        "parity": par,
        "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel" if f4 else "gemv_kernel") + " W13 (+SwiGLU)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)",
                     "traffic": traffic,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per routed expert of the "
                                       "W13 launch, copied from the capture in profiles/fp4_w13_c1_decode.md, "
                                       "times this run's distinct experts" if traffic else None,
                     "algorithmic_bytes_per_launch": distinct * W13_BYTES, "distinct_experts": distinct,
                     "launch_ms": t_w13_ms},
        "layer_roofline": {"bytes": layer_bytes, "ms": float(per.sum()),
                           "achieved_gbs": layer_bytes / (per.sum() / 1e3) / 1e9,
                           "frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                           # the whole timed step (gating included, one graph replay) against the same bytes
                           "gbs_over_step": layer_bytes / (ms / 1e3) / 1e9,
                           "frac_over_step": layer_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
                           "launch_ms": {k: float(v) for k, v in zip(names, per)}},
        "e2e": e2e,
        # fp4: gating, route plan, x planes (read bf16 x directly; with the plan up to 32 routes), W13 (+SwiGLU),
        # SwiGLU planes, W2, combine (fused into W2 up to 64 routes);
        # gemv: gating, bf16 copy, route plan, W13 (+SwiGLU), W2, combine (fused into W2 up to 32 routes)
        "gpu_launches": ((5 if m * K_TOP <= 32 else 6 if m * K_TOP <= 64 else 7) if f4 else
                         6 if m * K_TOP > 32 else 5) * args.steps,
        "cpu_baseline": cpu,
        "clocks": clk,
    })
    if own:
        layer.close()
    return line


# --------------------------------------------------------------------------- c2
def c2_alpha(route_fn, hot_mask: np.ndarray, tier_rank, m, dev):
    """Logits alpha * log p(rank) + Gumbel: alpha from a grid, the one whose
    routing sends closest to 80 % of routes to the NVFP4 experts."""
    from b200moe import synth

    best = None
    for alpha in np.round(np.arange(0.40, 1.21, 0.05), 2):
        logits = synth.zipf_logits(m, tier_rank, float(alpha), 1.1, 2000 + m, dev)
        ids = route_fn(logits)
        share = float(hot_mask[ids].mean())
        if best is None or abs(share - C2_HOT_SHARE) < abs(best[1] - C2_HOT_SHARE):
            best = (float(alpha), share, logits)
    return best


def run_c2(job, main: bool = True) -> dict:
    import torch

    from b200moe import moe, synth, tiers

    args, dev, m = job.args, job.dev, (job.args.m if main else 32)
    tier, tier_rank = tiers.zipf_tier(E, C2_HOT, seed=2)
    f4 = args.gemm != "gemv"
    iq_types = tuple(int(t) for t in args.iq_types.split(",")) if main else (16, 16)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=64, tier=tier, device=dev,
                              prefill_gemm="fp4" if f4 else "tcgen05", iq_types=iq_types)
    fp4 = synth.make_fp4_bank(C2_HOT, H, I, "nvfp4", 2000, dev)
    synth.load_bank(layer, fp4)
    iq2 = synth.make_iq2_bank(E - C2_HOT, H, I, 2001, dev, iq_types=iq_types)
    layer.set_iq_tables()
    synth.load_bank(layer, iq2)
    iq_w13_bytes = 2 * I * H // 256 * moe.IQ_BLOCK_BYTES[iq_types[0]]
    iq_w2_bytes = H * I // 256 * moe.IQ_BLOCK_BYTES[iq_types[1]]
    iq_name = {16: "IQ2_XXS", 17: "IQ2_XS", 29: "IQ1_M"}
    iq_desc = iq_name[iq_types[0]] if iq_types[0] == iq_types[1] else \
        f"{iq_name[iq_types[0]]} gate/up + {iq_name[iq_types[1]]} down"
    layer.check_errors()
    hot_mask = layer.fp4_slot >= 0
    alpha, share, logits = c2_alpha(lambda lg: layer.route(lg)[0].cpu().numpy(), hot_mask, tier_rank, m, dev)
    g = torch.Generator(device=dev).manual_seed(2032)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    if args.profile:
        del fp4, iq2
        torch.cuda.synchronize()
        for _ in range(args.warmup + args.steps):
            layer.forward(x, *layer.route(logits))
        torch.cuda.synchronize()
        layer.check_errors()
        layer.close()
        return {"profile_run": True, "workload": "c2", "alpha": alpha, "share": share}
    use_graph = not args.eager
    config = {"workload": f"configs[2] mixed-tier decode layer: hidden {H}, {C2_HOT} NVFP4 + {E - C2_HOT} {iq_desc} "
                          f"experts (Zipf 1.1 tier map, seed 2), inter {I}, top-{K_TOP}, M={m}",
              "tokens_per_step": m, "alpha": alpha, "hot_route_share": share,
              "l2": "inputs larger than L2 (expert weights streamed per step)",
              "launch": "one CUDA graph replay per step" if use_graph else "eager launches",
              "parallelism": "single GPU"}

    ids, w = layer.route(logits)
    out0 = layer.forward(x, ids, w).clone()
    layer.check_errors()
    par = None
    if iq_types == (16, 16):
        fdeq, ideq = fp4_dequant(fp4, I), iq2xxs_dequant(iq2)

        def deq(e):
            return fdeq(int(layer.fp4_slot[e])) if layer.fp4_slot[e] >= 0 else ideq(int(layer.iq2_slot[e]))
        par = parity(out0, x, ids, w, deq, TOL_LAYER, what="IQ2_XXS experts decoded as gguf-py does")

    def step():
        return layer.forward(x, *layer.route(logits))

    run, graph = graphed(step, use_graph, args.warmup)
    ids_np = ids.cpu().numpy()
    used = np.unique(ids_np)
    hot_used = used[layer.fp4_slot[used] >= 0]
    iq_used = used[layer.iq2_slot[used] >= 0]
    ms, clk = job.timed(run, args.steps)
    layer.check_errors()
    del graph
    if f4:  # start, convert, x int8 blocks, plan, x planes, W13 fp4, W13 iq2, SwiGLU planes, SwiGLU int8 blocks,
        #     W2 fp4, W2 iq2, combine
        per = per_launch(layer, [step], args.steps, 12)
        i13, i2, extra = (4, 5), (8, 9), {"x_planes": 3, "inter_planes": 6, "inter_int8": 7, "combine": 10}
    else:  # start, convert, x int8 blocks, plan, W13 fp4, W13 iq2, SwiGLU int8 blocks, W2 fp4, W2 iq2, combine
        sep = m * K_TOP > 32
        per = per_launch(layer, [step], args.steps, 10 if sep else 9)
        i13, i2, extra = (3, 4), (6, 7), dict({"inter_int8": 5}, **({"combine": 8} if sep else {}))
    pk = peaks()
    launches = {"w13_fp4": (per[i13[0]], hot_used.size * W13_BYTES),
                "w13_iq2": (per[i13[1]], iq_used.size * iq_w13_bytes),
                "w2_fp4": (per[i2[0]], hot_used.size * W2_BYTES), "w2_iq2": (per[i2[1]], iq_used.size * iq_w2_bytes)}
    dom = max(launches, key=lambda k: launches[k][0])
    t_dom, b_dom = launches[dom]
    achieved = b_dom / (t_dom / 1e3) / 1e9
    layer_bytes = hot_used.size * EXPERT_BYTES + iq_used.size * (iq_w13_bytes + iq_w2_bytes)
    e2e = e2e_decode(job, layer, [x], [logits], m, args.steps, use_graph)

    cpu = None
    if main and job.rank == 0 and not args.no_cpu_baseline:
        hot = cpu_fp4_layer(lambda e: fp4_expert(fp4, int(layer.fp4_slot[e]), 0),
                            np.where(np.isin(ids_np, hot_used), ids_np, -1), w.cpu().numpy(),
                            x.float().cpu().numpy(), m, reps=1)
        s = int
        iq_s, what = cpu_iq_part(lambda e: (iq2.w1[s(layer.iq2_slot[e])].cpu().numpy(),
                                            iq2.w3[s(layer.iq2_slot[e])].cpu().numpy(),
                                            iq2.w2[s(layer.iq2_slot[e])].cpu().numpy()),
                                 iq_used, ids_np, x.float().cpu().numpy(), iq_types, 6)
        total = hot["ms_per_layer"] / 1e3 + iq_s
        cpu = {"value": m / total, "unit": "tokens/s", "cores": hot["cores"], "kind": "port",
               "sample": f"NVFP4 experts: all {hot_used.size} through oracle/cpu_moe.c (AVX2); {what} "
                         "(numpy dequant + fp32 matmul), scaled by routes", "ms_per_layer": total * 1e3}
    line = line_base(job, args, "MoE-layer tokens/s (mixed-tier decode M=%d) & %% HBM roofline" % m,
                     m / (ms / 1e3), ms, config,
                     ("nvfp4 bank: " + DTYPE_FP4 if f4 else "nvfp4 bank: " + DTYPE_GEMV) +
                     "; IQ bank: two int8 activation planes x int8 codebook weights, s32 accumulate")
    line.update({
        "parity": par,
        "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel " if f4 and dom.endswith("fp4") else
                                               "gemv_kernel ") + dom, "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": None, "algorithmic_bytes_per_launch": b_dom,
                     "launch_ms": t_dom, "distinct_hot": int(hot_used.size), "distinct_iq2": int(iq_used.size)},
        "layer_roofline": {"bytes": layer_bytes, "ms": float(per.sum()),
                           "achieved_gbs": layer_bytes / (per.sum() / 1e3) / 1e9,
                           "frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                           "gbs_over_step": layer_bytes / (ms / 1e3) / 1e9,
                           "frac_over_step": layer_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
                           "launch_ms": {"convert": float(per[0]), "x_int8": float(per[1]), "plan": float(per[2]),
                                         **{k: float(per[v]) for k, v in extra.items()},
                                         **{k: float(v[0]) for k, v in launches.items()}}},
        "e2e": e2e,
        # gating, bf16 copy, x int8 blocks, plan, W13 x 2 banks, SwiGLU int8 blocks, W2 x 2 banks, combine
        # (fp4: + x planes, SwiGLU planes; the GEMV path fuses the combine up to 32 routes)
        "gpu_launches": (12 if f4 else 10 if m * K_TOP > 32 else 9) * args.steps,
        "cpu_baseline": cpu,
        "clocks": clk,
    })
    layer.close()
    return line


# --------------------------------------------------------------------------- c3
def run_c3(job, main: bool = True) -> dict:
    import torch

    from b200moe import moe, synth

    args, dev, T = job.args, job.dev, (job.args.tokens if main else 4096)
    E = args.experts if main else globals()["E"]  # fewer experts only for a small ncu capture
    mode = {"fp4": "fp4", "fp4-bs": "fp4-bs", "gemv": "tcgen05"}[args.gemm]
    bs = mode == "fp4-bs"  # every launch on the block-scaled kernel (32-route chunks)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=8,
                              tier=np.zeros(E, np.int8), fp4_format="mxfp4", device=dev, max_prefill_tokens=T,
                              prefill_gemm=mode)
    bank = synth.make_fp4_bank(E, H, I, "mxfp4", 3000, dev)
    synth.load_bank(layer, bank)
    layer.check_errors()
    g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.rand((T, E), generator=g, device=dev)
    if args.profile:
        del bank
        torch.cuda.synchronize()
        for _ in range(args.warmup + args.steps):
            layer.forward_prefill(x, *layer.route(logits))
        torch.cuda.synchronize()
        layer.check_errors()
        layer.close()
        return {"profile_run": True, "workload": "c3", "tokens": T}
    config = {"workload": f"configs[3] prefill layer: hidden {H}, {E} experts MXFP4, inter {I}, top-{K_TOP}, T={T}",
              "tokens_per_step": T, "format": "mxfp4",
              "gemm": ("block-scaled tcgen05 grouped GEMM (kind::mxf4nvf4.block32: E2M1 weights read as stored, "
                       "activations as four E2M1 planes with UE8M0 scales, 32 routes x 4 planes per MMA N, one "
                       "TMEM accumulator per item)" if bs else
                       "tcgen05 grouped GEMM (kind::f16, TMEM accumulators) on " +
                       ("the weight units of the block-scaled layout (one bulk copy per 256-K unit, per-row dequant)"
                        if mode == "fp4" else "the decode bank's units")),
              "l2": "inputs larger than L2 (all 384 experts, 5.1 GB, streamed per step)",
              "parallelism": "single GPU"}

    def step():
        return layer.forward_prefill(x, *layer.route(logits))

    ids, w = layer.route(logits)
    out0 = step()
    layer.check_errors()
    rows = np.sort(np.random.default_rng(3).choice(T, 256, replace=False))
    par = parity(out0, x, ids, w, fp4_dequant(bank, I), TOL_LAYER, rows=rows,
                 what="256 seeded tokens of the T-token call")
    for _ in range(max(3, args.warmup)):
        step()
    layer.check_errors()
    distinct = int(torch.unique(ids).numel())
    steps = max(3, args.steps // 10)
    ms, clk = job.timed(step, steps)
    layer.check_errors()
    if bs:  # start, convert, plan, x planes, W13, SwiGLU planes, W2, combine
        per = per_launch(layer, [step], steps, 8)
        names = ["convert", "plan", "x_planes", "w13", "swiglu_planes", "w2", "combine"]
        t13, t2 = float(per[3]), float(per[5])
    else:  # start, convert, plan, gather, W13, W2, combine
        per = per_launch(layer, [step], steps, 7)
        names = ["convert", "plan", "gather", "w13", "w2", "combine"]
        t13, t2 = float(per[3]), float(per[4])
    pk = peaks()
    tp = tensor_peaks(dev)
    fp4_peak = tp["kind::mxf4nvf4 block32 (E2M1, UE8M0 per 32, N 128)"]["tflops"]
    f16_peak = tp["kind::f16 (f16 x f16, N 256)"]["tflops"]
    mma_peak = fp4_peak if bs else f16_peak
    routes = T * K_TOP
    f13, f2 = 2.0 * routes * H * 2 * I, 2.0 * routes * I * H
    ach = f13 / (t13 / 1e3) / 1e12
    layer_flops = f13 + f2
    layer_bytes = distinct * (MX_W13_BYTES + MX_W2_BYTES)
    layer_ms = float(per.sum())
    bound_ms = max(layer_bytes / pk["hbm_gbs"] / 1e6, layer_flops / mma_peak / 1e9)

    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)
    hout = torch.empty((T, H), dtype=torch.float32).pin_memory()

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        hout.copy_(layer.forward_prefill(dx, *layer.route(dl)), non_blocking=True)

    e2e_step()
    e2e_ms, _ = job.timed(e2e_step, steps, clocks=False)

    cpu = None
    if main and job.rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_fp4_layer(lambda e: fp4_expert(bank, e, 1), ids.cpu().numpy(), w.cpu().numpy(),
                            x.float().cpu().numpy(), T, sample_experts=3, reps=1)
    line = line_base(job, args, "MoE-layer tokens/s (prefill T=%d) & %% tensor roofline" % T, T / (ms / 1e3), ms,
                     config, "e2m1x4 activations (UE8M0 block scales) x mxfp4 weights, f32 accumulate" if bs else
                     "f16 activations x mxfp4 weights dequantized to f16 on the SM, f32 accumulate", steps=steps)
    line.update({
        "parity": par,
        "roofline": {"bound": "tensor", "kernel": ("fp4_gemm_kernel (block-scaled, 32-route chunks)" if bs else
                                                   "tcgen05 grouped GEMM") + " W13 (+SwiGLU)",
                     "achieved": ach, "peak": mma_peak, "unit": "TFLOP/s", "frac": ach / mma_peak,
                     "peak_source": "this run's tcgen05 microbenchmark (b200moe_mma_peak) of the MMA kind the "
                                    "kernel issues: " + ("kind::mxf4nvf4 (dense FP4); the four activation planes "
                                                         "make the MMAs 4x the algorithmic FLOPs" if bs else
                                                         "kind::f16 (the MMAs run on dequantized weights)"),
                     "frac_of_measured_bf16_cublas": ach / pk["bf16_tflops"],
                     "frac_of_dense_fp4_peak": ach / fp4_peak,
                     "traffic": None, "algorithmic_flops_per_launch": f13, "launch_ms": t13},
        "layer_roofline": {"flops": layer_flops, "bytes": layer_bytes, "ms": layer_ms,
                           "tflops": layer_flops / (layer_ms / 1e3) / 1e12,
                           "tensor_frac": layer_flops / (layer_ms / 1e3) / 1e12 / mma_peak,
                           "hbm_frac": layer_bytes / (layer_ms / 1e3) / 1e9 / pk["hbm_gbs"],
                           "binding_bound_ms": bound_ms, "frac_of_binding_bound": bound_ms / layer_ms,
                           "binding_bound": "max(distinct expert bytes / measured HBM, FLOPs / measured peak of "
                                            "the MMA kind)",
                           "launch_ms": {k: float(v) for k, v in zip(names, per)}},
        "e2e": {"value": T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(hx.numel() * 2 + hl.numel() * 4),
                "d2h_bytes_per_step": int(hout.numel() * 4)},
        # block-scaled: gating, plan, x planes (read bf16 x), W13, SwiGLU planes, W2, combine;
        # f16 GEMM: gating, [bf16 copy], plan, row gather (converts bf16 itself), W13, W2, combine
        "gpu_launches": (7 if bs else 6 if mode == "fp4" else 7) * steps,
        "cpu_baseline": cpu,
        "clocks": clk,
    })
    layer.close()
    return line


def compact(line: dict) -> dict:
    """The figures of a sub-result worth keeping in the default run's line."""
    keep = ("metric", "value", "unit", "ms_per_step", "steps", "dtype", "config", "parity", "roofline",
            "layer_roofline", "e2e", "gpu_launches", "clocks")
    return {k: line[k] for k in keep if k in line}


def run_default(job) -> dict:
    """configs[1] M = 64, then (``also``) configs[1] M = 1 / 8 / 32,
    configs[2] and configs[3] T = 4096 on the same GPU."""
    import torch

    args = job.args
    f4 = args.gemm != "gemv"
    layer, bank = c1_layer(job, args.experts, f4)
    line = run_c1(job, 64, layer, bank, main=True)
    if args.no_also or args.experts != E:
        layer.close()
        return line
    line["tensor_peaks"] = tensor_peaks(job.dev)
    also = []
    for m in (1, 8, 32):
        also.append(compact(run_c1(job, m, layer, bank, main=False)))
    layer.close()
    del bank
    torch.cuda.empty_cache()
    also.append(compact(run_c2(job, main=False)))
    torch.cuda.empty_cache()
    also.append(compact(run_c3(job, main=False)))
    line["also"] = also
    return line


# --------------------------------------------------------------------------- c4
def run_c4(job) -> dict:
    import torch

    from b200moe import ep, moe, synth, tiers

    args, dev, rank, world = job.args, job.dev, job.rank, job.world
    n_layers, batch = args.layers, args.batch
    if batch % world:
        raise SystemExit(f"--batch {batch} must divide over {world} GPUs")
    T = batch // world
    peer = ep.PeerExchange(H, T * K_TOP, None, dev) if world > 1 else None
    layers = []
    # the routing bias of configs[2], chosen once on a whole-layer tier map
    tier0, trank0 = tiers.zipf_tier(E, C2_HOT, seed=4000)
    probe = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=min(T, 64),
                              max_prefill_tokens=T, tier=tier0, device=dev)
    alpha = c2_alpha(lambda lg: probe.route(lg)[0].cpu().numpy(), probe.fp4_slot >= 0, trank0, T, dev)[0]
    probe.close()
    for li in range(n_layers):
        tier, trank = tiers.zipf_tier(E, C2_HOT, seed=4000 + li)
        owner = None
        if world > 1 and args.placement == "balanced":  # expected routes ~ p(rank)^alpha of the Zipf(1.1) popularity
            expect = np.floor(1e9 * (trank + 1.0) ** (-1.1 * alpha)).astype(np.int64)
            owner = tiers.balanced_owners(tier, world, expect)
        if world == 1:
            lay = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=min(T, 64),
                                    max_prefill_tokens=T, tier=tier, device=dev,
                                    prefill_gemm="fp4" if args.gemm != "gemv" else "skinny")
            local = lay
        else:
            lay = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, tokens=T, tier=tier,
                                       device=dev, peer=peer, gemm="fp4" if args.gemm != "gemv" else "skinny",
                                       owner=owner)
            local = lay.layer
        n_hot, n_iq = int((local.fp4_slot >= 0).sum()), int((local.iq2_slot >= 0).sum())
        if n_hot:
            synth.load_bank(local, synth.make_fp4_bank(n_hot, H, I, "nvfp4", 4000 + 131 * li + rank, dev))
        local.set_iq2_tables()
        if n_iq:
            synth.load_bank(local, synth.make_iq2_bank(n_iq, H, I, 9000 + 131 * li + rank, dev))
        logits = synth.zipf_logits(T, trank, alpha, 1.1, 4000 + li + 7919 * rank, dev)
        layers.append((lay, logits))
        torch.cuda.empty_cache()
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    x0 = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    h = torch.empty((T, H), dtype=torch.float32, device=dev)
    xb = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    routes = [lay.route(lg) for lay, lg in layers]

    def single(lay, ids, w):  # world 1: the whole layer on this GPU
        return lay.forward(xb, ids, w) if T <= 64 else lay.forward_prefill(xb, ids, w)

    def step():
        h.copy_(x0)
        xb.copy_(x0)
        for (lay, _), (ids, w) in zip(layers, routes):
            if world == 1:
                h.add_(single(lay, ids, w))
            else:
                lay.forward(xb, ids, w, residual=h, out=h)
            xb.copy_(h)

    def step_with_gating():
        h.copy_(x0)
        xb.copy_(x0)
        for lay, lg in layers:
            ids, w = lay.route(lg)
            if world == 1:
                h.add_(single(lay, ids, w))
            else:
                lay.forward(xb, ids, w, residual=h, out=h)
            xb.copy_(h)

    run, graph = graphed(step_with_gating, not args.eager, args.warmup)
    for lay, _ in layers:
        lay.check_errors()
    steps = max(3, args.steps // 10)
    ms, clk = job.timed(run, steps)
    for lay, _ in layers:
        lay.check_errors()
    del graph
    value = batch / (ms / 1e3)

    # bytes this GPU streams per step (distinct local experts per layer) and exposed exchange time
    comm, local_bytes = 0.0, 0
    step()
    torch.cuda.synchronize()
    for (lay, _), (ids, w) in zip(layers, routes):
        local = lay if world == 1 else lay.layer
        if world == 1:
            used = np.unique(ids.cpu().numpy())
        else:
            lay.forward(xb, ids, w, residual=h, out=h)
            torch.cuda.synchronize()
            comm += lay.comm_ms()
            used = np.unique(lay.received())
        local_bytes += int((local.fp4_slot[used] >= 0).sum()) * EXPERT_BYTES + \
            int((local.iq2_slot[used] >= 0).sum()) * (IQ_W13_BYTES + IQ_W2_BYTES)
    comm_max = job.maxall(comm)
    # this library's launches per layer
    launches_per_step = 0
    fp4_path = args.gemm != "gemv"
    for lay, _ in layers:
        local = lay if world == 1 else lay.layer
        has_fp4, has_iq = bool((local.fp4_slot >= 0).any()), bool((local.iq2_slot >= 0).any())
        n = 1 + 1  # gating, route plan
        if world == 1:
            n += 1 if (has_iq or not fp4_path) else 0  # bf16 -> f16 copy of x (the FP4 planes read bf16 x)
            n += 1 if (fp4_path or T * K_TOP > 32) else 0  # the combine launch
        else:
            n += 3  # push, return, combine
        n += 2 if has_iq else 0  # int8 blocks of x and of the SwiGLU rows
        n += 2 if (fp4_path and has_fp4) else 0  # x planes, SwiGLU planes
        n += 2 * (int(has_fp4) + int(has_iq))  # W13 and W2 per bank
        launches_per_step += n
    pk = peaks()
    achieved = local_bytes / (ms / 1e3) / 1e9
    frac_min = -job.maxall(-achieved / pk["hbm_gbs"])

    hx = x0.cpu().pin_memory()
    hout = torch.empty((T, H), dtype=torch.float32).pin_memory()

    def e2e_step():
        x0.copy_(hx, non_blocking=True)
        step_with_gating()
        hout.copy_(h, non_blocking=True)

    run2, graph2 = graphed(e2e_step, not args.eager, 1)
    e2e_ms, _ = job.timed(run2, steps, clocks=False)
    del graph2
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # one layer on the host cores, scaled by the layer count
        lay0, _ = layers[0]
        ids0, w0 = routes[0]
        ids_np = ids0.cpu().numpy()
        used = np.unique(ids_np)
        hot_used, iq_used = used[lay0.fp4_slot[used] >= 0], used[lay0.iq2_slot[used] >= 0]
        hot0 = synth.make_fp4_bank(C2_HOT, H, I, "nvfp4", 4000, dev)
        iq0 = synth.make_iq2_bank(E - C2_HOT, H, I, 9000, dev)
        hot = cpu_fp4_layer(lambda e: fp4_expert(hot0, int(lay0.fp4_slot[e]), 0),
                            np.where(np.isin(ids_np, hot_used), ids_np, -1), w0.cpu().numpy(),
                            x0.float().cpu().numpy(), T, reps=1)
        s = int
        iq_s, what = cpu_iq_part(lambda e: (iq0.w1[s(lay0.iq2_slot[e])].cpu().numpy(),
                                            iq0.w3[s(lay0.iq2_slot[e])].cpu().numpy(),
                                            iq0.w2[s(lay0.iq2_slot[e])].cpu().numpy()),
                                 iq_used, ids_np, x0.float().cpu().numpy(), (16, 16), 6)
        total = (hot["ms_per_layer"] / 1e3 + iq_s) * n_layers
        cpu = {"value": batch / total, "unit": "tokens/s", "cores": hot["cores"], "kind": "port",
               "sample": f"one layer of the stack (NVFP4 experts through oracle/cpu_moe.c AVX2, {what} by numpy), "
                         f"time x {n_layers} layers", "ms_per_step": total * 1e3}
    line = None
    if rank == 0:
        config = {"workload": f"configs[4] {n_layers}-layer stack of configs[2] layers ({C2_HOT} NVFP4 + "
                              f"{E - C2_HOT} IQ2_XXS experts each), decode batch {batch} tokens per box, "
                              f"{T} per GPU, residual add between layers",
                  "layers": n_layers, "batch": batch, "tokens_per_gpu": T, "alpha": alpha,
                  "experts_per_gpu_per_layer": E // world,
                  "placement": ("experts by id range" if args.placement == "range" else
                                "tiers.balanced_owners on the expected routes") if world > 1 else "all experts",
                  "l2": "inputs larger than L2 (GBs of expert weights per step)",
                  "launch": "one CUDA graph replay per step" if not args.eager else "eager",
                  "parallelism": f"expert parallel x{world} (NVLink peer-memory exchange kernels)" if world > 1
                                 else "single GPU"}
        line = line_base(job, args, f"MoE-stack tokens/s ({n_layers} layers, decode batch {batch}) & % HBM roofline",
                         value, ms, config, "nvfp4 bank: " + (DTYPE_FP4 if args.gemm != "gemv" else DTYPE_GEMV) +
                         "; IQ bank: two int8 activation planes x int8 codebook weights", steps=steps)
        line["scaling"] = "strong"
        line.update({
            "roofline": {"bound": "hbm", "kernel": "all expert launches of the stack on rank 0 (whole step: " +
                         ("fp4_gemm_kernel for the NVFP4 bank, gemv_kernel for IQ2)" if args.gemm != "gemv" else
                          "gemv_kernel for both banks)"),
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "min_frac_over_ranks": frac_min,
                         "peak_source": pk["source"], "traffic": None, "algorithmic_bytes_per_step": local_bytes},
            "exposed_comm_ms": comm_max,
            "e2e": {"value": batch / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(hx.numel() * 2), "d2h_bytes_per_step": int(hout.numel() * 4)},
            "gpu_launches": launches_per_step * steps,
            "cpu_baseline": cpu,
            "clocks": clk,
        })
    for lay, _ in layers:
        lay.close()
    if peer is not None:
        peer.close()
    return line


# ------------------------------------------------------------- expert parallel
def run_expert_parallel(job) -> dict | None:
    """N ranks, expert parallel (see the module docstring): the box batch of
    configs[1] split over the ranks, then 64 tokens per rank."""
    import torch

    from b200moe import ep, moe, synth

    args, dev, rank, world = job.args, job.dev, job.rank, job.world
    m_box = args.m
    if m_box % world:
        raise SystemExit(f"--m {m_box} must divide over {world} GPUs")
    m_rank = m_box // world
    tier = np.zeros(E, np.int8)
    f4 = args.gemm != "gemv"
    layer = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, tokens=64, tier=tier, device=dev,
                                 exchange=args.exchange, gemm="fp4" if f4 else "skinny")
    n_local = int((layer.layer.fp4_slot >= 0).sum())
    synth.load_bank(layer.layer, synth.make_fp4_bank(n_local, H, I, "nvfp4", 1000 + rank, dev))
    # the single-GPU layer with every expert (each rank's bank from its own seed): the parity reference
    full = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=64, tier=tier, device=dev,
                             prefill_gemm="fp4" if f4 else "skinny")
    for r in range(world):
        synth.load_bank(full, synth.make_fp4_bank(n_local, H, I, "nvfp4", 1000 + r, dev), slot_begin=r * n_local)
        torch.cuda.empty_cache()
    if not f4:
        full.set_split_k(1, 1)
        layer.layer.set_split_k(1, 1)
    # strong: this rank's share of the configs[1] box batch; weak: 64 tokens of its own
    g = torch.Generator(device=dev).manual_seed(1000 + m_box)
    xb = torch.randn((m_box, H), generator=g, device=dev).to(torch.bfloat16)
    lb = torch.randn((m_box, E), generator=g, device=dev)
    x_s = xb[rank * m_rank:(rank + 1) * m_rank].contiguous()
    l_s = lb[rank * m_rank:(rank + 1) * m_rank].contiguous()
    g = torch.Generator(device=dev).manual_seed(1000 + 64 + 7919 * rank)
    x_w = torch.randn((64, H), generator=g, device=dev).to(torch.bfloat16)
    l_w = torch.randn((64, E), generator=g, device=dev)
    out = torch.empty((64, H), dtype=torch.float32, device=dev)

    def measure(x, logits, m, main):
        def step():
            ids, w = layer.route(logits)
            return layer.forward(x, ids, w, out=out[:m])

        # parity: bit-equal to the single-GPU layer on this rank's tokens
        ids, w = layer.route(logits)
        got = layer.forward(x, ids, w, out=out[:m]).clone()
        want = full.forward(x, ids, w).clone()
        layer.check_errors()
        full.check_errors()
        equal = bool(torch.equal(got, want))
        err = float((got.double() - want.double()).norm() / want.double().norm())
        all_equal = job.allok(equal)
        err_max = job.maxall(err)
        run, graph = graphed(step, args.exchange == "p2p" and not args.eager, args.warmup)
        layer.check_errors()
        ms, clk = job.timed(run, args.steps, clocks=main)
        layer.check_errors()
        del graph
        # exposed exchange and the local W13 launch (separate pass: these read events every step)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(7 if f4 else 5)]
        i13 = 3 if f4 else 2
        layer.layer.set_timing_events(evs)
        comm, w13_ms, used = 0.0, 0.0, 0
        n = max(5, args.steps // 4)
        for _ in range(n):
            step()
            torch.cuda.synchronize()
            comm += layer.comm_ms()  # push, the receive wait in the owner's plan launch, return, combine
            w13_ms += evs[i13].elapsed_time(evs[i13 + 1])
            used += layer.local_experts_used()
        layer.layer.set_timing_events(None)
        comm, w13_ms, used = comm / n, w13_ms / n, used / n
        pk = peaks()
        w13_gbs = used * W13_BYTES / (w13_ms / 1e3) / 1e9
        layer_gbs = used * EXPERT_BYTES / (ms / 1e3) / 1e9
        res = {"value": world * m / (ms / 1e3), "ms_per_step": ms, "tokens_per_gpu": m,
               "parity": {"bit_equal_to_single_gpu_layer": all_equal, "rel_l2_max_over_ranks": err_max,
                          "reference": "the single-GPU layer holding every expert (same seeds, same "
                                       + ("block-scaled FP4 path" if f4 else "GEMV path, split-K 1") +
                                       "), on each rank's own tokens"},
               "exposed_comm_ms": job.maxall(comm),
               "per_gpu": {"local_distinct_experts": used, "w13_launch_ms": w13_ms, "w13_gbs": w13_gbs,
                           "w13_frac": w13_gbs / pk["hbm_gbs"], "min_w13_frac_over_ranks":
                               -job.maxall(-w13_gbs / pk["hbm_gbs"]),
                           "layer_gbs_over_step": layer_gbs, "layer_frac_over_step": layer_gbs / pk["hbm_gbs"],
                           "min_layer_frac_over_ranks": -job.maxall(-layer_gbs / pk["hbm_gbs"])},
               "clocks": clk}
        return res, step

    strong, _ = measure(x_s, l_s, m_rank, True)
    weak, _ = measure(x_w, l_w, 64, False)

    # e2e of the strong run: pinned host x and logits in, output back, every step
    hx = x_s.cpu().pin_memory()
    hl = l_s.cpu().pin_memory()
    hout = torch.empty((m_rank, H), dtype=torch.float32).pin_memory()
    dx, dl = torch.empty_like(x_s), torch.empty_like(l_s)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        ids2, w2 = layer.route(dl)
        hout.copy_(layer.forward(dx, ids2, w2, out=out[:m_rank]), non_blocking=True)

    e2e_step()
    e2e_ms, _ = job.timed(e2e_step, args.steps, clocks=False)
    layer.check_errors()
    full.close()
    line = None
    if rank == 0:
        pk = peaks()
        config = {"workload": f"configs[1] decode layer: hidden {H}, {E} experts NVFP4, inter {I}, top-{K_TOP}, "
                              f"M={m_box} tokens per box, expert parallel over {world} GPUs ({m_rank} tokens per GPU)",
                  "tokens_per_step": m_box, "experts_per_gpu": n_local, "format": "nvfp4",
                  "l2": "inputs larger than L2 (expert weights streamed per step)",
                  "launch": "one CUDA graph replay per step" if args.exchange == "p2p" and not args.eager else
                            "eager" + (" (the exchange sizes come from a host read of the route counts)"
                                       if args.exchange == "nccl" else ""),
                  "parallelism": f"expert parallel x{world} ("
                                 + ("NVLink peer-memory exchange kernels" if args.exchange == "p2p" else
                                    "NCCL all-to-all") + ")"}
        line = line_base(job, args, "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m_box, strong["value"],
                         strong["ms_per_step"], config, DTYPE_FP4 if f4 else DTYPE_GEMV)
        line["scaling"] = "strong"
        pg = strong["per_gpu"]
        line.update({
            "parity": strong["parity"],
            "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel" if f4 else "gemv_kernel") +
                                                   " W13 (+SwiGLU) of rank 0's local experts",
                         "achieved": pg["w13_gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": pg["w13_frac"],
                         "min_frac_over_ranks": pg["min_w13_frac_over_ranks"], "peak_source": pk["source"],
                         "traffic": None, "algorithmic_bytes_per_launch": pg["local_distinct_experts"] * W13_BYTES,
                         "launch_ms": pg["w13_launch_ms"]},
            "per_gpu": pg,
            "exposed_comm_ms": strong["exposed_comm_ms"],
            "weak_scaling": dict(weak, note="64 tokens per GPU (the box batch grows with N); each GPU streams "
                                            "fewer distinct experts as N grows, so this curve is not a "
                                            "fixed-work scaling curve"),
            "e2e": {"value": world * m_rank / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
                    "d2h_bytes_per_step": int(hout.numel() * hout.element_size())},
            # p2p: gating; push; local plan (waits for every rank's push), W13, W2; return; combine
            # (fp4: + the two plane launches of the local run)
            "gpu_launches": (9 if f4 else 7) * args.steps,
            "cpu_baseline": None,
            "clocks": strong["clocks"],
        })
    layer.close()
    return line


# ------------------------------------------------------------ reference arm
def run_reference(args) -> None:
    """The reference's CPU expert path on the workload, rank 0 only (under
    torchrun the other ranks exit at once; no process group is made).

    The reference's own CPU kernel (harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c,
    AVX2 + OpenMP) is compiled from its source into oracle/_ref/ but has its
    shapes fixed at hidden 5120 / TP slice 576 and reads MXFP4 only, so it
    cannot run these configs; the timed value is this build's AVX2 restatement
    of that kernel with parametric shapes and NVFP4 (oracle/cpu_moe.c,
    ``oracle_expert_avx2``) on the workload's exact experts and routing, and
    the reference's kernel is timed beside it at its own shape, per expert
    slice and per weight byte (``reference_kernel``).  Nothing here loads the
    product library: experts are packed by oracle/torch_quant.py (bit-equal to
    the library's quantizers) from the same seeded weights, routing is the
    oracle's gating, and the GPU (when present) only draws the seeded
    weights with stock torch ops."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch

    from oracle import cpu_layer
    from oracle import moe_oracle as mo
    from oracle import torch_quant as tq

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))) if torch.cuda.is_available() \
        else torch.device("cpu")
    wl, n_exp = args.workload, args.experts
    budget_s = 60.0  # the timed region of the whole run stays about a minute
    iq_s, iq_what, iq_types = 0.0, "", (16, 16)
    if wl == "c3":
        T = args.tokens
        g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        logits = torch.rand((T, E), generator=g, device=dev)[:, :n_exp]
        tokens, fmt, seed, sample = T, "mxfp4", 3000, 3
        metric = "MoE-layer tokens/s (prefill T=%d) & %% tensor roofline" % T
        workload = f"configs[3] prefill layer: hidden {H}, {n_exp} experts MXFP4, inter {I}, top-{K_TOP}, T={T}"
        ids, w = mo.route(logits.cpu().numpy(), K_TOP)
        hot_ids = None
    elif wl in ("c2", "c4"):
        from b200moe import synth, tiers

        if wl == "c2":  # as run_c2: tier map seed 2, banks 2000 / 2001, logits seed 2000 + m, x seed 2032
            m, seed_t, seed, seed_iq = args.m, 2, 2000, 2001
        else:  # as run_c4's layer 0 at one GPU: tier map 4000, banks 4000 / 9000, logits 4000, x 4000
            m, seed_t, seed, seed_iq = args.batch, 4000, 4000, 9000
        tier, trank = tiers.zipf_tier(E, C2_HOT, seed=seed_t)
        hot_mask = tier == tiers.HOT
        alpha, share, logits = c2_alpha(lambda lg: mo.route(lg.cpu().numpy(), K_TOP)[0], hot_mask, trank, m, dev)
        if wl == "c4":
            logits = synth.zipf_logits(m, trank, alpha, 1.1, 4000, dev)
        g = torch.Generator(device=dev).manual_seed(2032 if wl == "c2" else 4000)
        x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = mo.route(logits.cpu().numpy(), K_TOP)
        tokens, fmt, sample = m, "nvfp4", None
        metric = ("MoE-layer tokens/s (mixed-tier decode M=%d) & %% HBM roofline" % m if wl == "c2" else
                  f"MoE-stack tokens/s ({args.layers} layers, decode batch {m}) & % HBM roofline")
        workload = (f"configs[2] mixed-tier decode layer: hidden {H}, {C2_HOT} NVFP4 + {E - C2_HOT} IQ2_XXS experts, "
                    f"inter {I}, top-{K_TOP}, M={m}" if wl == "c2" else
                    f"configs[4] {args.layers}-layer stack of configs[2] layers, decode batch {m} on one GPU (layer 0 "
                    f"timed, x {args.layers})")
        hot_ids = np.flatnonzero(hot_mask)
        slot = np.cumsum(hot_mask) - 1
        islot = np.cumsum(~hot_mask) - 1
        used = np.unique(ids)
        iq_used = used[~hot_mask[used]]
        iq2 = synth.make_iq2_bank(E - C2_HOT, H, I, seed_iq, dev)
        iq_s, iq_what = cpu_iq_part(lambda e: (iq2.w1[islot[e]].cpu().numpy(), iq2.w3[islot[e]].cpu().numpy(),
                                               iq2.w2[islot[e]].cpu().numpy()),
                                    iq_used, ids, x.float().cpu().numpy(), iq_types, 6)
        del iq2
        ids = np.where(hot_mask[ids], slot[ids], -1).astype(np.int32)  # NVFP4 routes, by bank slot
    else:
        m = args.m
        g = torch.Generator(device=dev).manual_seed(1000 + m)
        x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
        logits = torch.randn((m, E), generator=g, device=dev)[:, :n_exp]
        tokens, fmt, seed, sample = m, "nvfp4", 1000, None
        metric = "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m
        workload = f"configs[1] decode layer: hidden {H}, {n_exp} experts NVFP4, inter {I}, top-{K_TOP}, M={m}"
        ids, w = mo.route(logits.cpu().numpy(), K_TOP)
        hot_ids = None
    x_np = x.float().cpu().numpy()
    used = np.unique(ids[ids >= 0])
    n_bank = n_exp if hot_ids is None else hot_ids.size
    pick = used if sample is None else used[:sample]
    experts = tq.fp4_expert_bank(n_bank, H, I, fmt, seed, dev, pick=pick)
    cpu = cpu_layer.CpuMoe(H, I, avx2=True)
    routes_all = int((ids >= 0).sum())

    def layer_seconds(sel):
        t0 = time.perf_counter()
        cpu.forward(x_np, ids, w, experts, only=sel)
        dt = time.perf_counter() - t0
        return dt, dt * routes_all / max(int(np.isin(ids, sel).sum()), 1)

    # one untimed pass sizes the sample so that --steps K fit the budget
    warm_dt, _ = layer_seconds(pick)
    steps = max(1, args.steps)
    if warm_dt * steps > budget_s and pick.size > 1:
        keep = max(1, int(pick.size * budget_s / (warm_dt * steps)))
        pick = pick[:keep]
    for _ in range(max(0, args.warmup - 1)):
        layer_seconds(pick)
    times = [layer_seconds(pick)[1] for _ in range(steps)]
    fp4_s = float(np.mean(times))
    layer_s = fp4_s + iq_s
    if wl == "c4":
        layer_s *= args.layers
    v = tokens / layer_s
    what = (f"{pick.size} of {used.size} routed FP4 experts per step, scaled by routes" if pick.size < used.size
            else f"all {used.size} routed FP4 experts")
    if iq_what:
        what += f"; IQ2_XXS: {iq_what} (numpy dequant + fp32 matmul), scaled by routes"
    if wl == "c4":
        what += f"; one layer x {args.layers}"

    # the reference's own kernel at its fixed shape, beside the port at the same shape and rows
    refk = None
    rows_per_expert = max(1, int(round(routes_all / max(used.size, 1))))
    if cpu_layer.REF_LIB.exists():
        ref = cpu_layer.RefCpuExpert()
        rng = np.random.default_rng(5)
        rh, ri = ref.HIDDEN, ref.INTER
        w13 = rng.normal(0, 0.02, (2 * ri, rh)).astype(np.float32)
        w2 = rng.normal(0, 0.02, (rh, ri)).astype(np.float32)
        c13, s13 = mo.mxfp4_quantize(w13)
        c2, s2 = mo.mxfp4_quantize(w2)
        rec = ref.record(c13, s13, c2, s2)
        ex = dict(fmt=1, w13c=c13, w13s=s13, g13=np.ones(2, np.float32), w2c=c2, w2s=s2, g2=1.0)
        mm = min(rows_per_expert, 16)
        xr = rng.normal(0, 1, (mm, rh)).astype(np.float32)
        rws = np.arange(mm, dtype=np.int32)
        ww = np.ones(mm, np.float32)
        port = cpu_layer.CpuMoe(rh, ri, avx2=True)
        o = np.zeros((mm, rh), np.float32)

        def clock(fn, n=30):
            fn()
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            return (time.perf_counter() - t0) / n

        t_ref = clock(lambda: ref.expert(rec, xr, rws, ww, o))
        t_port = clock(lambda: port.expert(ex, xr, rws, ww, o))
        weights = 3 * rh * ri
        ours_weights = 3 * H * I
        refk = {"kernel": "harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c expert_slice, compiled from the reference's "
                          "source into oracle/_ref/ with its own flags",
                "shape": f"hidden {rh}, TP slice {ri}, MXFP4 record {rec.nbytes} B, {mm} rows (this workload's "
                         "routes per routed expert, at most the kernel's 16)",
                "us_per_expert_slice": t_ref * 1e6, "port_us_same_shape": t_port * 1e6,
                "port_over_reference_time": t_port / t_ref,
                "reference_gb_per_s_of_record": rec.nbytes / t_ref / 1e9,
                "layer_estimate_tokens_per_s": tokens / (layer_s * (t_ref / t_port)),
                "layer_estimate_note": f"the port's layer time scaled by the reference kernel's time over the port's "
                                       f"on the same slice ({weights:,} weights; this config's experts have "
                                       f"{ours_weights:,})",
                "published_us_per_expert": 2953.7,
                "published_source": "docs/measurements.md:1677 (the reference's host, V100 box)"}
    line = {"impl": "reference", "metric": metric, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": layer_s * 1e3, "higher_is_better": True,
            "scaling": "strong" if wl == "c4" else "weak", "vs_baseline": None,
            "dtype": "f32 (activations f32, weights decoded from nvfp4/mxfp4 codes, f32 accumulate)",
            "data": "synthetic (seeded; the same weights, inputs and routing as the product's run)",
            "config": {"workload": workload, "tokens_per_step": tokens},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
                             "sample": what},
            "reference_kernel": refk,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "libraries_loaded": loaded_libraries(),
            "note": "the reference's CPU expert path, restated with parametric shapes and NVFP4 (its own kernel "
                    "is fixed at 5120/576 MXFP4 and is timed beside it under reference_kernel); the reference's "
                    "GPU kernels are V100-only and not in its source tree"}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    job = Job(args)
    import __graft_entry__

    __graft_entry__.load_package()
    if args.workload == "c4":
        line = run_c4(job)
    elif job.world > 1:
        line = run_expert_parallel(job)
    elif args.workload == "c2":
        line = run_c2(job)
    elif args.workload == "c3":
        line = run_c3(job)
    elif args.m == 64 and not args.profile:
        line = run_default(job)
    else:
        line = run_c1(job, args.m)
    if job.rank == 0 and line is not None:
        if "profile_run" not in line:
            line["libraries_loaded"] = loaded_libraries()
        print(json.dumps(line), flush=True)
    job.finish()


if __name__ == "__main__":
    main()
