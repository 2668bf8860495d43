#!/usr/bin/env python
"""Benchmark of the routed-expert MoE layer on B200 (one JSON line on rank 0).

Workload (the decode layer the metric is quoted on):
hidden 4096, 384 routed experts, intermediate 2048, top-8 from router logits
~N(0,1), all experts NVFP4 (weights ~N(0,0.02), seeded, packed by the
library's own quantizer), bf16 activations ~N(0,1), M = 64 tokens per step
(``--m`` picks 1, 8, 32 or 64).  A step = gating (router logits -> top-8) +
the layer forward, all on the GPU.  At M = 64 a step streams ~4 GB of expert
weights, far above the 126 MB L2, so no flush is needed (``config.l2``).

``value``   tokens/s of the whole job, inputs resident in HBM, CUDA events on
            the launching stream around exactly K steps, max over ranks.
``e2e``     the same through the public API with host buffers: each step
            copies x and the logits from pinned host memory and reads the
            output back, inside the timed region.
``roofline`` the W13 launch (the largest kernel): algorithmic bytes = routed
            distinct experts x W13 NVFP4 bytes, over its event-timed duration,
            against MEASURED_PEAKS.json hbm_gbs.
``cpu_baseline`` the C restatement of the reference's CPU expert kernel
            (oracle/cpu_moe.c, OpenMP on all host cores) on the same layer.

``--impl reference`` times that CPU implementation alone on this workload (the
reference's own GPU kernels are V100-only and are not in its source tree).

Multi-GPU (torchrun, N ranks): expert parallel.  Rank r owns experts
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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=64, choices=[1, 8, 32, 64])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts (384 = configs[1]; fewer only for a small ncu capture)")
    ap.add_argument("--split-k", type=int, default=0,
                    help="fix the GEMV split-K (0 = chosen per launch; set only to give a small ncu capture "
                         "the split-K of the full-size run)")
    ap.add_argument("--profile", action="store_true",
                    help="warm-up + timed steps only (no per-launch, e2e or CPU passes): the ncu command")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


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


def measured_traffic(distinct: int) -> dict | None:
    """DRAM bytes of one W13 launch from the committed ncu summary
    (dram__bytes_read.sum + dram__bytes_write.sum of this bench's W13 launch),
    scaled from the captured routing's distinct experts to this one's."""
    import re

    p = ROOT / "profiles" / "gemv_w13_c1_decode.md"
    if not p.exists():
        return None
    txt = p.read_text()
    m1 = re.search(r"^traffic_bytes_per_launch:\s*([0-9.e+]+)", txt, re.M)
    m2 = re.search(r"^captured_distinct_experts:\s*([0-9]+)", txt, re.M)
    if not (m1 and m2):
        return None
    b, d = float(m1.group(1)), int(m2.group(1))
    return {"bytes": b * distinct / d, "captured_bytes": b, "captured_distinct_experts": d,
            "source": "profiles/gemv_w13_c1_decode.md (ncu dram__bytes_read.sum + dram__bytes_write.sum)"}


def cpu_layer_tokens_per_s(bank, ids_np, w_np, x_np, m, reps=2) -> dict:
    """The C oracle (OpenMP, all host cores) on the full layer of this routing."""
    from oracle import cpu_layer

    used = np.unique(ids_np)
    experts = {}
    for e in used.tolist():
        experts[e] = dict(fmt=0, w13c=bank.w13_codes[e].cpu().numpy(), w13s=bank.w13_scales[e].cpu().numpy(),
                          g13=bank.globals[e, :2].cpu().numpy(), w2c=bank.w2_codes[e].cpu().numpy(),
                          w2s=bank.w2_scales[e].cpu().numpy(), g2=float(bank.globals[e, 2]))
    cpu = cpu_layer.CpuMoe(H, I)
    cpu.forward(x_np, ids_np, w_np, experts)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu.forward(x_np, ids_np, w_np, experts)
    dt = (time.perf_counter() - t0) / reps
    return {"value": m / dt, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
            "sample": f"full layer at M={m} ({used.size} routed experts), {reps} timed runs, "
                      f"{dt * 1e3:.1f} ms per layer", "ms_per_layer": dt * 1e3}


def run_expert_parallel(args, dev, rank, world, x, logits, config, maxall) -> None:
    """N ranks, expert parallel over NCCL (see the module docstring)."""
    import torch
    import torch.distributed as dist

    from b200moe import ep, synth

    m = args.m
    tier = np.zeros(E, np.int8)
    layer = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, tokens=m, tier=tier, device=dev)
    n_local = int((layer.layer.fp4_slot >= 0).sum())
    bank = synth.make_fp4_bank(n_local, H, I, "nvfp4", 1000 + rank, dev)
    synth.load_bank(layer.layer, bank)
    del bank
    # each rank is home to its own tokens
    g = torch.Generator(device=dev).manual_seed(1000 + m + 7919 * rank)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    out = torch.empty((m, H), dtype=torch.float32, device=dev)
    config = dict(config, parallelism=f"expert parallel x{world} (NCCL all-to-all)", experts_per_gpu=n_local,
                  tokens_per_step=m * world)
    config["workload"] += f", expert parallel over {world} GPUs, {m} tokens per GPU"

    def step():
        ids, w = layer.route(logits)
        return layer.forward(x, ids, w, out=out)

    for _ in range(max(3, args.warmup)):
        step()
    layer.check_errors()

    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(dev) if rank == 0 else None
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = maxall(e0.elapsed_time(e1) / args.steps)
    layer.check_errors()
    value = world * m / (ms / 1e3)

    # exposed communication and the local W13 launch (separate pass: these read events every step)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    layer.layer.set_timing_events(evs)  # start, convert, plan, W13, W2 of the local expert run
    comm, w13_ms, used = 0.0, 0.0, 0
    for _ in range(args.steps):
        step()
        torch.cuda.synchronize()
        comm += layer.comm_ms()
        w13_ms += evs[2].elapsed_time(evs[3])
        used += layer.local_experts_used()
    layer.layer.set_timing_events(None)
    comm, w13_ms, used = comm / args.steps, w13_ms / args.steps, used / args.steps
    comm_max = maxall(comm)
    pk = peaks()
    achieved = used * W13_BYTES / (w13_ms / 1e3) / 1e9
    frac_min = -maxall(-achieved / pk["hbm_gbs"])

    # e2e through the public API with host buffers
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty((m, H), dtype=torch.float32).pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        ids2, w2 = layer.route(dl)
        hout.copy_(layer.forward(dx, ids2, w2, out=out), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = maxall(e0.elapsed_time(e1) / args.steps)
    layer.check_errors()
    if rank == 0:
        line = {
            "metric": "MoE-layer tokens/s (decode M=64) & % HBM roofline",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded; random-init NVFP4 experts)", "config": config,
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel W13 (+SwiGLU) of rank 0's local experts",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / pk["hbm_gbs"], "min_frac_over_ranks": frac_min,
                         "peak_source": pk["source"], "traffic": None,
                         "algorithmic_bytes_per_launch": used * W13_BYTES, "distinct_local_experts": used,
                         "launch_ms": w13_ms},
            "exposed_comm_ms": comm_max,
            "e2e": {"value": world * m / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
                    "d2h_bytes_per_step": int(hout.numel() * hout.element_size()), "ms_per_step": e2e_ms},
            # gating; dispatch plan, row gather, metadata; local convert, plan, W13, W2; f32->f16; combine
            "gpu_launches": 10 * args.steps,
            "cpu_baseline": None,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    args = parse()
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    m = args.m

    def maxall(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    import __graft_entry__

    __graft_entry__.load_package()
    from b200moe import moe, synth

    g = torch.Generator(device=dev).manual_seed(1000 + m)
    x = torch.randn((m, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((m, E), generator=g, device=dev)
    config = {"workload": f"configs[1] decode layer: hidden {H}, {E} experts NVFP4, inter {I}, top-{K_TOP}, M={m}",
              "tokens_per_step": m, "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "format": "nvfp4",
              "l2": "inputs larger than L2 (expert weights streamed per step)" if m >= 32 else
                    "inputs smaller than L2 at this M: weights may stay cached across steps",
              "parallelism": f"replicas x{world}" if world > 1 else "single GPU"}

    n_exp = args.experts
    if n_exp != E:
        config["workload"] += f" (ncu capture case: {n_exp} experts)"
        config["experts"] = n_exp
        logits = logits[:, :n_exp].contiguous()

    if args.impl == "reference":
        if rank == 0:
            bank = synth.make_fp4_bank(E, H, I, "nvfp4", 1000, dev)
            layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K_TOP, max_tokens=64,
                                      tier=np.zeros(E, np.int8), device=dev)
            ids, w = layer.route(logits)
            ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
            x_np = x.float().cpu().numpy()
            layer.close()
            from oracle import cpu_layer

            used = np.unique(ids_np)
            experts = {e: dict(fmt=0, w13c=bank.w13_codes[e].cpu().numpy(), w13s=bank.w13_scales[e].cpu().numpy(),
                               g13=bank.globals[e, :2].cpu().numpy(), w2c=bank.w2_codes[e].cpu().numpy(),
                               w2s=bank.w2_scales[e].cpu().numpy(), g2=float(bank.globals[e, 2]))
                       for e in used.tolist()}
            del bank
            cpu = cpu_layer.CpuMoe(H, I)
            for _ in range(args.warmup):
                cpu.forward(x_np, ids_np, w_np, experts)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                cpu.forward(x_np, ids_np, w_np, experts)
            dt = (time.perf_counter() - t0) / args.steps
            v = m / dt
            line = {"impl": "reference", "metric": "MoE-layer tokens/s (decode)", "value": v, "unit": "tokens/s",
                    "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                    "data": "synthetic", "config": config,
                    "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cpu_layer.threads(), "kind": "port",
                                     "sample": f"full layer at M={m}, {used.size} routed experts per step"},
                    "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    "note": "the reference's CPU expert path (harness/benchmarks/nvfp4_8r/cpu_mxfp4_moe.c) "
                            "restated in C with parametric shapes (oracle/cpu_moe.c); its GPU kernels are "
                            "V100-only and not in its source tree"}
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    if world > 1:
        run_expert_parallel(args, dev, rank, world, x, logits, config, maxall)
        return

    bank = synth.make_fp4_bank(n_exp, H, I, "nvfp4", 1000, dev)
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=n_exp, top_k=K_TOP, max_tokens=64,
                              tier=np.zeros(n_exp, np.int8), device=dev)
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
        ids, w = layer.route(logits)
        return layer.forward(x, ids, w), ids, w

    for _ in range(max(3, args.warmup)):
        step()
    layer.check_errors()
    ids, w = layer.route(logits)
    distinct = int(torch.unique(ids).numel())

    # ---- value: K steps, inputs resident, CUDA events on the current stream
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(dev) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = maxall(e0.elapsed_time(e1) / args.steps)
    layer.check_errors()
    value = world * m / (ms / 1e3)

    # ---- per-launch times (same steps, events between the forward's launches)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    layer.set_timing_events(evs)  # start, convert, plan, W13, W2
    per = np.zeros(4)
    for _ in range(args.steps):
        step()
        torch.cuda.synchronize()
        per += [evs[i].elapsed_time(evs[i + 1]) for i in range(4)]
    layer.set_timing_events(None)
    per /= args.steps
    t_w13_ms, t_w2_ms = float(per[2]), float(per[3])
    pk = peaks()
    achieved = distinct * W13_BYTES / (t_w13_ms / 1e3) / 1e9
    layer_bytes = distinct * EXPERT_BYTES
    traffic = measured_traffic(distinct)

    # ---- e2e through the public API, host buffers in pinned memory
    hx = x.cpu().pin_memory()
    hl = logits.cpu().pin_memory()
    hout = torch.empty((m, H), dtype=torch.float32).pin_memory()
    dx, dl = torch.empty_like(x), torch.empty_like(logits)
    for _ in range(2):
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        hout.copy_(layer.forward(dx, *layer.route(dl)), non_blocking=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(args.steps):
        dx.copy_(hx, non_blocking=True)
        dl.copy_(hl, non_blocking=True)
        ids2, w2 = layer.route(dl)
        hout.copy_(layer.forward(dx, ids2, w2), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = maxall(e0.elapsed_time(e1) / args.steps)
    layer.check_errors()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_layer_tokens_per_s(bank, ids.cpu().numpy(), w.cpu().numpy(), x.float().cpu().numpy(), m)

    launches_per_step = 5  # gating, bf16 copy, route plan, W13 (+SwiGLU), W2 (+combine)
    if rank == 0:
        line = {
            "metric": "MoE-layer tokens/s (decode M=64) & % HBM roofline",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded; random-init NVFP4 experts)", "config": config,
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel W13 (+SwiGLU)", "achieved": achieved,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": pk["source"], "traffic": traffic["bytes"] if traffic else None,
                         "traffic_detail": traffic,
                         "algorithmic_bytes_per_launch": distinct * W13_BYTES, "distinct_experts": distinct,
                         "launch_ms": t_w13_ms},
            "layer_roofline": {"bytes": layer_bytes, "ms": float(per.sum()),
                               "achieved_gbs": layer_bytes / (per.sum() / 1e3) / 1e9,
                               "frac": layer_bytes / (per.sum() / 1e3) / 1e9 / pk["hbm_gbs"],
                               "launch_ms": {"convert": float(per[0]), "plan": float(per[1]), "w13": t_w13_ms,
                                             "w2": t_w2_ms}},
            "e2e": {"value": world * m / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + hl.numel() * hl.element_size()),
                    "d2h_bytes_per_step": int(hout.numel() * hout.element_size()), "ms_per_step": e2e_ms},
            "gpu_launches": launches_per_step * args.steps,
            "cpu_baseline": cpu,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
