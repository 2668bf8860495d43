#!/usr/bin/env python
"""Benchmark of the routed-expert MoE layer on B200 (one JSON line on rank 0).

Workloads (all inputs seeded synthetic, weights
random-init and packed by the library's own quantizers):

``c1`` (default) configs[1], the decode layer the metric is quoted on: hidden
    4096, 384 routed experts, intermediate 2048, top-8 from router logits
    ~N(0,1), all experts NVFP4 (weights ~N(0,0.02)), bf16 activations ~N(0,1),
    M = 64 tokens per step (``--m`` picks 1, 8, 32 or 64).  At M = 64 a step
    streams ~4 GB of expert weights, far above the 126 MB L2, so no flush is
    needed (``config.l2``).
``c2`` configs[2], the mixed-tier decode layer at M = 32: a seeded Zipf(1.1)
    tier map puts the 150 most popular experts in NVFP4 and 234 in IQ2_XXS;
    router logits alpha * log p(rank) + Gumbel noise, alpha chosen on the
    device from a grid so that about 80 % of routes reach the NVFP4 experts.
``c3`` configs[3], prefill: T = 4096 tokens (``--tokens 16384``), MXFP4
    experts, logits ~U(0,1); the W13/W2 launches are the tcgen05 grouped GEMM.
``c4`` configs[4], a 40-layer stack of c2 layers (own seeded tier map and
    experts per layer), one decode batch of 256 tokens for the whole box
    (256 / N per GPU: strong scaling), Zipf routing, residual add between
    layers; experts sharded by id over the N GPUs (peer-memory exchange); the
    whole 40-layer step is one CUDA graph.  Reports box tokens/s and the
    exposed exchange time summed over the layers.

A step = gating (router logits -> top-8) + the layer forward, all on the GPU.
Decode steps (c1, c2) replay one CUDA graph per step (the reference captures
its decode path the same way); ``--eager`` launches them one by one.

``value``   tokens/s of the whole job, inputs resident in HBM, CUDA events on
            the launching stream around exactly K steps, max over ranks.
``e2e``     the same through the public API with host buffers: each step
            copies x and the logits from pinned host memory and reads the
            output back, inside the timed region.
``roofline`` the dominant launch: algorithmic bytes (routed distinct experts x
            the projection's packed bytes) or FLOPs (c3: 2 x routes x weights)
            over its event-timed duration, against MEASURED_PEAKS.json.
``cpu_baseline`` the C restatement of the reference's CPU expert kernel
            (oracle/cpu_moe.c, OpenMP on the host cores) on the same routing,
            whole layer or a bounded sample of experts scaled to the layer.

``--impl reference`` times that CPU implementation alone on the workload (the
reference's own GPU kernels are V100-only and are not in its source tree).

Multi-GPU (torchrun, N ranks): expert parallel on c1.  Rank r owns experts
[r*384/N, (r+1)*384/N); each rank is home to its own M = 64 tokens (weak
scaling: tokens per GPU fixed), gates them, dispatches every route to its
owner over NCCL all-to-all, runs its local experts on the routes it receives
and combines the returned rows in slot order.  ``value`` = N*M / (max over
ranks of the step time); ``exposed_comm_ms`` = the all-to-all time on the
critical path (counts + rows out, y2 back), from CUDA events.
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
                    help="decode tokens per step (c1 default 64, c2 default 32)")
    ap.add_argument("--tokens", type=int, default=4096, choices=[4096, 16384], help="c3 prefill tokens")
    ap.add_argument("--eager", action="store_true", help="decode: launch each kernel instead of a graph replay")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="multi-GPU: the library's NVLink peer-memory exchange (default) or NCCL all-to-all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts (384 = configs[1]; fewer only for a small ncu capture)")
    ap.add_argument("--split-k", type=int, default=0,
                    help="fix the GEMV split-K (0 = chosen per call; set only to give a small ncu capture "
                         "the split-K of the full-size run)")
    ap.add_argument("--placement", choices=["range", "balanced"], default="range",
                    help="c4 over N > 1 GPUs: experts by id range, or tiers.balanced_owners on the expected routes")
    ap.add_argument("--iq-types", default="16,16",
                    help="c2: GGML types of the IQ experts' gate/up and down (16 IQ2_XXS, 17 IQ2_XS, 29 IQ1_M)")
    ap.add_argument("--gemm", choices=["fp4", "gemv"], default="fp4",
                    help="c1, c2, c4: the FP4 bank on the block-scaled FP4 tensor path (tcgen05.mma "
                         "kind::mxf4nvf4, default) or on the skinny GEMV; c3: the tcgen05 prefill GEMM reading "
                         "the block-scaled layout's weight units (default) or the decode bank's units")
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


def measured_traffic(distinct: int, summary: str = "gemv_w13_c1_decode.md") -> dict | None:
    """DRAM bytes of one W13 launch from the committed ncu summary
    (dram__bytes_read.sum + dram__bytes_write.sum of this bench's W13 launch),
    scaled from the captured routing's distinct experts to this one's."""
    import re

    p = ROOT / "profiles" / summary
    if not p.exists():
        return None
    txt = p.read_text()
    m1 = re.search(r"^traffic_bytes_per_launch:\s*([0-9.e+]+)", txt, re.M)
    m2 = re.search(r"^captured_distinct_experts:\s*([0-9]+)", txt, re.M)
    if not (m1 and m2):
        return None
    b, d = float(m1.group(1)), int(m2.group(1))
    return {"bytes": b * distinct / d, "captured_bytes": b, "captured_distinct_experts": d,
            "source": f"profiles/{summary} (ncu dram__bytes_read.sum + dram__bytes_write.sum)"}


def fp4_expert(bank, j: int, fmt: int) -> dict:
    """One expert of a natural-layout FP4 bank as the C oracle takes it."""
    g = bank.globals[j].cpu().numpy() if bank.globals is not None else np.ones(3, np.float32)
    return dict(fmt=fmt, w13c=bank.w13_codes[j].cpu().numpy(), w13s=bank.w13_scales[j].cpu().numpy(),
                g13=g[:2].copy(), w2c=bank.w2_codes[j].cpu().numpy(), w2s=bank.w2_scales[j].cpu().numpy(),
                g2=float(g[2]))


def cpu_fp4_layer(experts_of, ids_np, w_np, x_np, tokens, sample_experts=None, reps=2) -> dict:
    """The C oracle (OpenMP, all host cores) on the layer of this routing: every
    routed expert, or a bounded sample of them scaled to the layer by routes."""
    from oracle import cpu_layer

    used = np.unique(ids_np[ids_np >= 0])
    pick = used if sample_experts is None else used[:sample_experts]
    experts = {int(e): experts_of(int(e)) for e in pick.tolist()}
    cpu = cpu_layer.CpuMoe(H, I)
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
            "sample": f"{what}; {reps} timed runs, {dt * 1e3:.1f} ms each", "ms_per_layer": layer_s * 1e3}


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


def per_launch(layer, step, steps: int, n_events: int) -> np.ndarray:
    """Mean duration (ms) between the layer's timing events (eager steps)."""
    import torch

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_events)]
    layer.set_timing_events(evs)
    per = np.zeros(n_events - 1)
    for _ in range(steps):
        step()
        torch.cuda.synchronize()
        per += [evs[i].elapsed_time(evs[i + 1]) for i in range(n_events - 1)]
    layer.set_timing_events(None)
    return per / steps


def e2e_decode(job, layer, x, logits, out_like, steps: int, use_graph: bool) -> tuple[float, dict]:
    """The public API with pinned host buffers: H2D of x and logits, gating,
    forward, D2H of the output, every step inside the timed region."""
    import torch

    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty(out_like.shape, dtype=out_like.dtype).pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)

    def step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        hout.copy_(layer.forward(dx, *layer.route(dl)), non_blocking=True)

    run, g = graphed(step, use_graph, 2)
    ms, _ = job.timed(run, steps, clocks=False)
    layer.check_errors()
    del g
    return ms, {"h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
                "d2h_bytes_per_step": int(hout.numel() * hout.element_size())}


def line_base(job, args, metric, value, ms, config, dtype="f16") -> dict:
    return {"metric": metric, "value": value, "unit": "tokens/s", "n_gpus": job.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded; random-init experts)", "config": config}


def profile_run(layer, step, args, info: dict) -> None:
    """The ncu command: eager warm-up and timed steps only, then one line."""
    import torch

    torch.cuda.synchronize()
    for _ in range(args.warmup + args.steps):
        step()
    torch.cuda.synchronize()
    layer.check_errors()
    layer.close()
    print(json.dumps(dict({"profile_run": True, "workload": args.workload}, **info)), flush=True)


# --------------------------------------------------------------------------- c1
def run_c1(job) -> None:
    import torch

    from b200moe import moe, synth

    args, dev, m = job.args, job.dev, job.args.m
    g = torch.Generator(device=dev).manual_seed(1000 + m)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    use_graph = not args.eager
    f4 = args.gemm == "fp4"
    config = {"workload": f"configs[1] decode layer: hidden {H}, {E} experts NVFP4, inter {I}, top-{K_TOP}, M={m}",
              "gemm": "block-scaled FP4 tensor path (tcgen05.mma kind::mxf4nvf4, E4M3 block scales in TMEM, "
                      "activations as four E2M1 planes)" if f4 else "skinny GEMV (mma.sync, weights dequantized "
                                                                     "in registers)",
              "tokens_per_step": m, "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "format": "nvfp4",
              "l2": "inputs larger than L2 (expert weights streamed per step)" if m >= 32 else
                    "inputs smaller than L2 at this M: weights may stay cached across steps",
              "launch": "one CUDA graph replay per step" if use_graph else "eager launches",
              "parallelism": "single GPU"}
    n_exp = args.experts
    if n_exp != E:
        config["workload"] += f" (ncu capture case: {n_exp} experts)"
        config["experts"] = n_exp
        logits = logits[:, :n_exp].contiguous()

    bank = synth.make_fp4_bank(n_exp, H, I, "nvfp4", 1000, dev)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=n_exp, top_k=K_TOP, max_tokens=64,
                              tier=np.zeros(n_exp, np.int8), device=dev, prefill_gemm="fp4" if f4 else "tcgen05")
    synth.load_bank(layer, bank)
    layer.check_errors()
    if args.split_k:
        layer.set_split_k(args.split_k, 0)
        config["split_k"] = args.split_k
    if args.profile:
        del bank
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            layer.forward(x, *layer.route(logits))
        for _ in range(args.steps):
            layer.forward(x, *layer.route(logits))
        torch.cuda.synchronize()
        layer.check_errors()
        distinct = int(torch.unique(layer.route(logits)[0]).numel())
        layer.close()
        print(json.dumps({"profile_run": True, "experts": n_exp, "m": m, "distinct_experts": distinct,
                          "w13_algorithmic_bytes": distinct * W13_BYTES,
                          "w2_algorithmic_bytes": distinct * W2_BYTES}), flush=True)
        return

    def step():
        return layer.forward(x, *layer.route(logits))

    run, graph = graphed(step, use_graph, args.warmup)
    layer.check_errors()
    ids, w = layer.route(logits)
    distinct = int(torch.unique(ids).numel())
    ms, clk = job.timed(run, args.steps)
    layer.check_errors()
    value = job.world * m / (ms / 1e3)
    del graph

    if f4:  # convert, plan, x planes, W13, SwiGLU planes, W2, combine
        per = per_launch(layer, step, args.steps, 8)
        t_w13_ms, t_w2_ms = float(per[3]), float(per[5])
        names = ["convert", "plan", "x_planes", "w13", "swiglu_planes", "w2", "combine"]
    else:  # convert, plan, W13, W2 (+SwiGLU or combine: fused up to 32 routes)
        sep = m * K_TOP > 32
        per = per_launch(layer, step, args.steps, 6 if sep else 5)
        t_w13_ms, t_w2_ms = float(per[2]), float(per[3])
        names = ["convert", "plan", "w13", "w2"] + (["combine"] if sep else [])
    pk = peaks()
    achieved = distinct * W13_BYTES / (t_w13_ms / 1e3) / 1e9
    layer_bytes = distinct * EXPERT_BYTES
    traffic = measured_traffic(distinct, "fp4_w13_c1_decode.md" if f4 else "gemv_w13_c1_decode.md") \
        if n_exp == E else None
    e2e_ms, e2e_bytes = e2e_decode(job, layer, x, logits, layer.out[:m], args.steps, use_graph)

    cpu = None
    if job.rank == 0 and job.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_fp4_layer(lambda e: fp4_expert(bank, e, 0), ids.cpu().numpy(), w.cpu().numpy(),
                            x.float().cpu().numpy(), m)
    if job.rank == 0:
        line = line_base(job, args, "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m, value, ms, config)
        line.update({
            "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel" if f4 else "gemv_kernel") + " W13 (+SwiGLU)",
                         "achieved": achieved,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": pk["source"], "traffic": traffic["bytes"] if traffic else None,
                         "traffic_detail": traffic,
                         "algorithmic_bytes_per_launch": distinct * W13_BYTES, "distinct_experts": distinct,
                         "launch_ms": t_w13_ms},
            "layer_roofline": {"bytes": layer_bytes, "ms": float(per.sum()),
                               "achieved_gbs": layer_bytes / (per.sum() / 1e3) / 1e9,
                               "frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                               "launch_ms": {k: float(v) for k, v in zip(names, per)}},
            "e2e": dict({"value": job.world * m / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms},
                        **e2e_bytes),
            # fp4: gating, route plan, x planes (read bf16 x directly), W13 (+SwiGLU), SwiGLU planes, W2, combine;
            # gemv: gating, bf16 copy, route plan, W13 (+SwiGLU), W2, combine (fused into W2 up to 32 routes)
            "gpu_launches": (7 if f4 else 6 if m * K_TOP > 32 else 5) * args.steps,
            "cpu_baseline": cpu,
            "clocks": clk,
        })
        print(json.dumps(line), flush=True)
    layer.close()


# --------------------------------------------------------------------------- c2
def c2_inputs(layer, tier_rank, m, dev):
    """Logits alpha * log p(rank) + Gumbel: alpha from a grid, the one whose
    routing sends closest to 80 % of routes to the NVFP4 experts."""
    import torch

    from b200moe import synth

    hot = torch.from_numpy(layer.fp4_slot >= 0).to(dev)
    best = None
    for alpha in np.round(np.arange(0.40, 1.21, 0.05), 2):
        logits = synth.zipf_logits(m, tier_rank, float(alpha), 1.1, 2000 + m, dev)
        ids, _ = layer.route(logits)
        share = float(hot[ids.long()].float().mean())
        if best is None or abs(share - C2_HOT_SHARE) < abs(best[1] - C2_HOT_SHARE):
            best = (float(alpha), share, logits)
    return best


def run_c2(job) -> None:
    import torch

    from b200moe import moe, synth, tiers

    args, dev, m = job.args, job.dev, job.args.m
    tier, tier_rank = tiers.zipf_tier(E, C2_HOT, seed=2)
    f4 = args.gemm == "fp4"
    iq_types = tuple(int(t) for t in args.iq_types.split(","))
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
    alpha, share, logits = c2_inputs(layer, tier_rank, m, dev)
    g = torch.Generator(device=dev).manual_seed(2032)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    if args.profile:
        del fp4, iq2
        profile_run(layer, lambda: layer.forward(x, *layer.route(logits)), args, {"alpha": alpha, "share": share})
        return
    use_graph = not args.eager
    config = {"workload": f"configs[2] mixed-tier decode layer: hidden {H}, {C2_HOT} NVFP4 + {E - C2_HOT} {iq_desc} "
                          f"experts (Zipf 1.1 tier map, seed 2), inter {I}, top-{K_TOP}, M={m}",
              "tokens_per_step": m, "alpha": alpha, "hot_route_share": share,
              "l2": "inputs larger than L2 (expert weights streamed per step)",
              "launch": "one CUDA graph replay per step" if use_graph else "eager launches",
              "parallelism": "single GPU"}

    def step():
        return layer.forward(x, *layer.route(logits))

    run, graph = graphed(step, use_graph, args.warmup)
    ids, w = layer.route(logits)
    ids_np = ids.cpu().numpy()
    used = np.unique(ids_np)
    hot_used = used[layer.fp4_slot[used] >= 0]
    iq_used = used[layer.iq2_slot[used] >= 0]
    ms, clk = job.timed(run, args.steps)
    layer.check_errors()
    del graph
    if f4:  # start, convert, x int8 blocks, plan, x planes, W13 fp4, W13 iq2, SwiGLU planes, SwiGLU int8 blocks,
        #     W2 fp4, W2 iq2, combine
        per = per_launch(layer, step, args.steps, 12)
        i13, i2, extra = (4, 5), (8, 9), {"x_planes": 3, "inter_planes": 6, "inter_int8": 7, "combine": 10}
    else:  # start, convert, x int8 blocks, plan, W13 fp4, W13 iq2, SwiGLU int8 blocks, W2 fp4, W2 iq2, combine
        sep = m * K_TOP > 32
        per = per_launch(layer, step, args.steps, 10 if sep else 9)
        i13, i2, extra = (3, 4), (6, 7), dict({"inter_int8": 5}, **({"combine": 8} if sep else {}))
    pk = peaks()
    launches = {"w13_fp4": (per[i13[0]], hot_used.size * W13_BYTES),
                "w13_iq2": (per[i13[1]], iq_used.size * iq_w13_bytes),
                "w2_fp4": (per[i2[0]], hot_used.size * W2_BYTES), "w2_iq2": (per[i2[1]], iq_used.size * iq_w2_bytes)}
    dom = max(launches, key=lambda k: launches[k][0])
    t_dom, b_dom = launches[dom]
    achieved = b_dom / (t_dom / 1e3) / 1e9
    layer_bytes = hot_used.size * EXPERT_BYTES + iq_used.size * (iq_w13_bytes + iq_w2_bytes)
    e2e_ms, e2e_bytes = e2e_decode(job, layer, x, logits, layer.out[:m], args.steps, use_graph)

    cpu = None
    if job.rank == 0 and job.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_c2(fp4, iq2, layer, ids_np, w.cpu().numpy(), x.float().cpu().numpy(), m, iq_types=iq_types)
    if job.rank == 0:
        line = line_base(job, args, "MoE-layer tokens/s (mixed-tier decode M=%d) & %% HBM roofline" % m,
                         job.world * m / (ms / 1e3), ms, config)
        line.update({
            "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel " if f4 and dom.endswith("fp4") else
                                                   "gemv_kernel ") + dom, "achieved": achieved,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": pk["source"], "traffic": None, "algorithmic_bytes_per_launch": b_dom,
                         "launch_ms": t_dom, "distinct_hot": int(hot_used.size), "distinct_iq2": int(iq_used.size)},
            "layer_roofline": {"bytes": layer_bytes, "ms": float(per.sum()),
                               "achieved_gbs": layer_bytes / (per.sum() / 1e3) / 1e9,
                               "frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                               "launch_ms": {"convert": float(per[0]), "x_int8": float(per[1]), "plan": float(per[2]),
                                             **{k: float(per[v]) for k, v in extra.items()},
                                             **{k: float(v[0]) for k, v in launches.items()}}},
            "e2e": dict({"value": job.world * m / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms},
                        **e2e_bytes),
            # gating, bf16 copy, x int8 blocks, plan, W13 x 2 banks, SwiGLU int8 blocks, W2 x 2 banks, combine
            # (fp4: + x planes, SwiGLU planes; the GEMV path fuses the combine up to 32 routes)
            "gpu_launches": (12 if f4 else 10 if m * K_TOP > 32 else 9) * args.steps,
            "cpu_baseline": cpu,
            "clocks": clk,
        })
        print(json.dumps(line), flush=True)
    layer.close()


def cpu_c2(fp4, iq2, layer, ids_np, w_np, x_np, m, sample_iq=6, iq_types=(16, 16)) -> dict:
    """CPU layer of the mixed tier: NVFP4 experts through the C oracle, IQ2
    experts as the reference's CPU path does them (gguf dequantize, then fp32
    matmuls; numpy restatement), on a bounded sample of IQ2 experts scaled by
    routes."""
    from oracle import cpu_layer
    from oracle import moe_oracle as mo

    used = np.unique(ids_np)
    hot_ids = used[layer.fp4_slot[used] >= 0]
    iq_ids = used[layer.iq2_slot[used] >= 0]
    hot = cpu_fp4_layer(lambda e: fp4_expert(fp4, int(layer.fp4_slot[e]), 0),
                        np.where(np.isin(ids_np, hot_ids), ids_np, -1), w_np, x_np, m, reps=1)
    hot_s = hot["ms_per_layer"] / 1e3
    pick = iq_ids[:sample_iq]
    t0 = time.perf_counter()
    for e in pick.tolist():
        s = int(layer.iq2_slot[e])
        w13 = np.concatenate([mo.iq_decode(iq_types[0], iq2.w1[s].cpu().numpy()),
                              mo.iq_decode(iq_types[0], iq2.w3[s].cpu().numpy())])
        w2 = mo.iq_decode(iq_types[1], iq2.w2[s].cpu().numpy())
        rows = np.nonzero(ids_np == e)[0]
        mo.expert_fp32(x_np[rows], w13, w2)
    dt = time.perf_counter() - t0
    routes_pick = int(np.isin(ids_np, pick).sum())
    iq_s = dt * np.isin(ids_np, iq_ids).sum() / max(routes_pick, 1)
    total = hot_s + iq_s
    return {"value": m / total, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
            "sample": f"NVFP4 experts: all {hot_ids.size} through oracle/cpu_moe.c; IQ2_XXS: {pick.size} of "
                      f"{iq_ids.size} experts (numpy dequant + matmul), scaled by routes", "ms_per_layer": total * 1e3}


# --------------------------------------------------------------------------- c3
def run_c3(job) -> None:
    import torch

    from b200moe import moe, synth

    args, dev, T = job.args, job.dev, job.args.tokens
    units = args.gemm == "fp4"  # the block-scaled layout's weight units also feed the tcgen05 prefill GEMM
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=8,
                              tier=np.zeros(E, np.int8), fp4_format="mxfp4", device=dev, max_prefill_tokens=T,
                              prefill_gemm="fp4" if units else "tcgen05")
    bank = synth.make_fp4_bank(E, H, I, "mxfp4", 3000, dev)
    synth.load_bank(layer, bank)
    layer.check_errors()
    g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.rand((T, E), generator=g, device=dev)
    if args.profile:
        del bank
        profile_run(layer, lambda: layer.forward_prefill(x, *layer.route(logits)), args, {"tokens": T})
        return
    config = {"workload": f"configs[3] prefill layer: hidden {H}, {E} experts MXFP4, inter {I}, top-{K_TOP}, T={T}",
              "tokens_per_step": T, "format": "mxfp4",
              "gemm": "tcgen05 grouped GEMM (kind::f16, TMEM accumulators) on " +
                      ("the weight units of the block-scaled layout (one bulk copy per 256-K unit, per-row dequant)"
                       if units else "the decode bank's units"),
              "l2": "inputs larger than L2 (all 384 experts, 5.1 GB, streamed per step)",
              "parallelism": "single GPU"}

    def step():
        return layer.forward_prefill(x, *layer.route(logits))

    for _ in range(max(3, args.warmup)):
        step()
    layer.check_errors()
    ids, w = layer.route(logits)
    distinct = int(torch.unique(ids).numel())
    steps = max(3, args.steps // 10)
    ms, clk = job.timed(step, steps)
    layer.check_errors()
    per = per_launch(layer, step, steps, 7)  # convert, plan, gather, W13, W2, combine
    pk = peaks()
    routes = T * K_TOP
    f13, f2 = 2.0 * routes * H * 2 * I, 2.0 * routes * I * H
    t13, t2 = float(per[3]), float(per[4])
    ach = f13 / (t13 / 1e3) / 1e12
    layer_flops = f13 + f2
    layer_bytes = distinct * (MX_W13_BYTES + MX_W2_BYTES)

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
    if job.rank == 0 and job.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_fp4_layer(lambda e: fp4_expert(bank, e, 1), ids.cpu().numpy(), w.cpu().numpy(),
                            x.float().cpu().numpy(), T, sample_experts=3, reps=1)
    if job.rank == 0:
        line = line_base(job, args, "MoE-layer tokens/s (prefill T=%d) & %% tensor roofline" % T,
                         job.world * T / (ms / 1e3), ms, config)
        line["steps"] = steps
        line.update({
            "roofline": {"bound": "tensor", "kernel": "tcgen05 grouped GEMM W13 (+SwiGLU)", "achieved": ach,
                         "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"],
                         "peak_source": pk["source"] + " bf16 dense (the MMAs are kind::f16 on dequantized weights)",
                         "traffic": None, "algorithmic_flops_per_launch": f13, "launch_ms": t13},
            "layer_roofline": {"flops": layer_flops, "bytes": layer_bytes, "ms": float(per.sum()),
                               "tflops": layer_flops / (per.sum() / 1e3) / 1e12,
                               "tensor_frac": layer_flops / (per.sum() / 1e3) / 1e12 / pk["bf16_tflops"],
                               "hbm_frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                               "launch_ms": {"convert": float(per[0]), "plan": float(per[1]),
                                             "gather": float(per[2]), "w13": t13, "w2": t2,
                                             "combine": float(per[5])}},
            "e2e": {"value": job.world * T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(hx.numel() * 2 + hl.numel() * 4),
                    "d2h_bytes_per_step": int(hout.numel() * 4)},
            # gating, [bf16 copy], plan, row gather (converts bf16 itself), W13, W2, combine
            "gpu_launches": (6 if units else 7) * steps,
            "cpu_baseline": cpu,
            "clocks": clk,
        })
        print(json.dumps(line), flush=True)
    layer.close()


# --------------------------------------------------------------------------- c4
def run_c4(job) -> None:
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
    alpha = c2_inputs(probe, trank0, T, dev)[0]
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
                                    prefill_gemm="fp4" if args.gemm == "fp4" else "skinny")
            local = lay
        else:
            lay = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, tokens=T, tier=tier,
                                       device=dev, peer=peer, gemm="fp4" if args.gemm == "fp4" else "skinny",
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

    def single(lay, ids, w):  # world 1: the whole layer on this GPU, fused combine
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
    # this library's launches per layer: gating; world 1: bf16 copy, x int8 blocks, plan, W13 and W2 per bank,
    # SwiGLU int8 blocks; world > 1 adds owner plan, push, receive, return, combine (no bf16 copy)
    launches_per_step = 0
    for lay, _ in layers:
        local = lay if world == 1 else lay.layer
        banks = int((local.fp4_slot >= 0).any()) + int((local.iq2_slot >= 0).any())
        launches_per_step += 1 + 2 * banks + (3 if world == 1 else 2) + (5 if world > 1 else 0)
        if world == 1 and (args.gemm == "fp4" or T * K_TOP > 32):  # the combine launch
            launches_per_step += 1
        if args.gemm == "fp4" and (local.fp4_slot >= 0).any():  # x and SwiGLU planes
            launches_per_step += 2
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
        hot0 = synth.make_fp4_bank(C2_HOT, H, I, "nvfp4", 4000, dev)
        iq0 = synth.make_iq2_bank(E - C2_HOT, H, I, 9000, dev)
        one = cpu_c2(hot0, iq0, lay0, ids0.cpu().numpy(), w0.cpu().numpy(), x0.float().cpu().numpy(), T)
        one["value"] /= n_layers
        one["sample"] = f"one layer of the stack ({one['sample']}), time x {n_layers} layers"
        cpu = one
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
                         value, ms, config)
        line["steps"] = steps
        line["scaling"] = "strong"
        line.update({
            "roofline": {"bound": "hbm", "kernel": "all expert launches of the stack on rank 0 (whole step: " +
                         ("fp4_gemm_kernel for the NVFP4 bank, gemv_kernel for IQ2)" if args.gemm == "fp4" else
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
        print(json.dumps(line), flush=True)
    for lay, _ in layers:
        lay.close()
    if peer is not None:
        peer.close()


# ------------------------------------------------------------- expert parallel
def run_expert_parallel(job) -> None:
    """N ranks, expert parallel over NCCL (see the module docstring)."""
    import torch

    from b200moe import ep, synth

    args, dev, rank, world, m = job.args, job.dev, job.rank, job.world, job.args.m
    tier = np.zeros(E, np.int8)
    f4 = args.gemm == "fp4"
    layer = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, tokens=m, tier=tier, device=dev,
                                 exchange=args.exchange, gemm="fp4" if f4 else "skinny")
    n_local = int((layer.layer.fp4_slot >= 0).sum())
    bank = synth.make_fp4_bank(n_local, H, I, "nvfp4", 1000 + rank, dev)
    synth.load_bank(layer.layer, bank)
    del bank
    # each rank is home to its own tokens
    g = torch.Generator(device=dev).manual_seed(1000 + m + 7919 * rank)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    out = torch.empty((m, H), dtype=torch.float32, device=dev)
    config = {"workload": f"configs[1] decode layer: hidden {H}, {E} experts NVFP4, inter {I}, top-{K_TOP}, M={m}, "
                          f"expert parallel over {world} GPUs, {m} tokens per GPU",
              "tokens_per_step": m * world, "experts_per_gpu": n_local, "format": "nvfp4",
              "l2": "inputs larger than L2 (expert weights streamed per step)",
              "launch": "one CUDA graph replay per step" if args.exchange == "p2p" and not args.eager else
                        "eager" + (" (the exchange sizes come from a host read of the route counts)"
                                   if args.exchange == "nccl" else ""),
              "parallelism": f"expert parallel x{world} ("
                             + ("NVLink peer-memory exchange kernels" if args.exchange == "p2p" else "NCCL all-to-all")
                             + ")"}

    def step():
        ids, w = layer.route(logits)
        return layer.forward(x, ids, w, out=out)

    run, graph = graphed(step, args.exchange == "p2p" and not args.eager, args.warmup)
    layer.check_errors()
    ms, clk = job.timed(run, args.steps)
    layer.check_errors()
    value = world * m / (ms / 1e3)
    del graph

    # exposed communication and the local W13 launch (separate pass: these read events every step)
    # local expert run: start, convert, plan, [x planes], W13, [SwiGLU planes], W2
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7 if f4 else 5)]
    i13 = 3 if f4 else 2
    layer.layer.set_timing_events(evs)
    comm, w13_ms, used = 0.0, 0.0, 0
    for _ in range(args.steps):
        step()
        torch.cuda.synchronize()
        comm += layer.comm_ms()
        w13_ms += evs[i13].elapsed_time(evs[i13 + 1])
        used += layer.local_experts_used()
    layer.layer.set_timing_events(None)
    comm, w13_ms, used = comm / args.steps, w13_ms / args.steps, used / args.steps
    comm_max = job.maxall(comm)
    pk = peaks()
    achieved = used * W13_BYTES / (w13_ms / 1e3) / 1e9
    frac_min = -job.maxall(-achieved / pk["hbm_gbs"])

    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty((m, H), dtype=torch.float32).pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        ids2, w2 = layer.route(dl)
        hout.copy_(layer.forward(dx, ids2, w2, out=out), non_blocking=True)

    e2e_step()
    e2e_ms, _ = job.timed(e2e_step, args.steps, clocks=False)
    layer.check_errors()
    if rank == 0:
        line = line_base(job, args, "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m, value, ms, config)
        line.update({
            "roofline": {"bound": "hbm", "kernel": ("fp4_gemm_kernel" if f4 else "gemv_kernel") +
                                                   " W13 (+SwiGLU) of rank 0's local experts",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "min_frac_over_ranks": frac_min,
                         "peak_source": pk["source"], "traffic": None,
                         "algorithmic_bytes_per_launch": used * W13_BYTES, "distinct_local_experts": used,
                         "launch_ms": w13_ms},
            "exposed_comm_ms": comm_max,
            "e2e": {"value": world * m / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
                    "d2h_bytes_per_step": int(hout.numel() * hout.element_size())},
            # p2p: gating; owner plan, push, receive; local plan, W13, W2; return; combine
            # nccl: gating; owner plan, row gather, metadata; local plan, W13, W2, f32->f16; combine
            # (fp4: + the two plane launches of the local run)
            "gpu_launches": (9 + (2 if f4 else 0)) * args.steps,
            "cpu_baseline": None,
            "clocks": clk,
        })
        print(json.dumps(line), flush=True)
    layer.close()


# ------------------------------------------------------------ reference arm
def run_reference(job) -> None:
    """The reference's CPU expert path (restated in C, oracle/cpu_moe.c) on the
    workload's routing, all host threads; rank 0 only."""
    import torch

    from b200moe import moe, synth

    args, dev = job.args, job.dev
    if job.rank != 0:
        return
    from oracle import cpu_layer

    wl = args.workload
    if wl == "c3":
        T = args.tokens
        tokens, fmt, bank = T, 1, synth.make_fp4_bank(E, H, I, "mxfp4", 3000, dev)
        g = torch.Generator(device=dev).manual_seed(3000 + T // 1024)
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        logits = torch.rand((T, E), generator=g, device=dev)
        sample = 3
        metric = "MoE-layer tokens/s (prefill T=%d) & %% tensor roofline" % T
        workload = f"configs[3] prefill layer: hidden {H}, {E} experts MXFP4, inter {I}, top-{K_TOP}, T={T}"
    else:
        m = args.m
        tokens, fmt, bank = m, 0, synth.make_fp4_bank(E, H, I, "nvfp4", 1000, dev)
        g = torch.Generator(device=dev).manual_seed(1000 + m)
        x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
        logits = torch.randn((m, E), generator=g, device=dev)
        sample = None
        metric = "MoE-layer tokens/s (decode M=%d) & %% HBM roofline" % m
        workload = f"configs[1] decode layer: hidden {H}, {E} experts NVFP4, inter {I}, top-{K_TOP}, M={m}"
        if wl == "c2":
            workload += " (the reference arm times the all-NVFP4 layer: the IQ2 path has no C restatement)"
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=64,
                              tier=np.zeros(E, np.int8), device=dev)
    ids, w = layer.route(logits)
    ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
    x_np = x.float().cpu().numpy()
    layer.close()
    used = np.unique(ids_np)
    pick = used if sample is None else used[:sample]
    experts = {int(e): fp4_expert(bank, int(e), fmt) for e in pick.tolist()}
    del bank
    cpu = cpu_layer.CpuMoe(H, I)
    steps = args.steps if sample is None else max(1, args.steps // 50)
    warm = args.warmup if sample is None else 1
    for _ in range(warm):
        cpu.forward(x_np, ids_np, w_np, experts, only=pick)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu.forward(x_np, ids_np, w_np, experts, only=pick)
    dt = (time.perf_counter() - t0) / steps
    layer_s = dt * ids_np.size / max(int(np.isin(ids_np, pick).sum()), 1)
    v = tokens / layer_s
    what = "full layer" if sample is None else f"{pick.size} of {used.size} routed experts, scaled by routes"
    line = {"impl": "reference", "metric": metric, "value": v, "unit": "tokens/s", "n_gpus": job.world,
            "steps": steps, "warmup": warm, "ms_per_step": layer_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
                             "sample": f"{what}, {used.size} routed experts per step"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's CPU expert path (harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c) restated in C "
                    "with parametric shapes (oracle/cpu_moe.c); its GPU kernels are V100-only and not in its "
                    "source tree"}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse()
    job = Job(args)
    import __graft_entry__

    __graft_entry__.load_package()
    if args.impl == "reference":
        run_reference(job)
    elif args.workload == "c4":
        run_c4(job)
    elif job.world > 1:
        run_expert_parallel(job)
    elif args.workload == "c2":
        run_c2(job)
    elif args.workload == "c3":
        run_c3(job)
    else:
        run_c1(job)
    job.finish()


if __name__ == "__main__":
    main()
