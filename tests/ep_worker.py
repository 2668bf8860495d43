"""One rank of the expert-parallel parity check (launched by torchrun from
tests/test_gpu_ep.py): every rank builds the same seeded experts, runs the
sharded layer on its own tokens and the full single-GPU layer on the same
tokens, and writes the relative L2 distance per case to a JSON file."""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from b200moe import ep, moe, synth, tiers  # noqa: E402


def main(out_path: str, exchange: str, gemm: str, placement: str) -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dev = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    H, I, E, K, T = 1024, 512, 64, 6, 48
    tier, pop_rank = tiers.zipf_tier(E, 40, seed=3)
    if placement.endswith("-fp4only"):  # every expert FP4: the owners' W2 stores y2 at home (fused return)
        tier = np.full(E, tiers.HOT, np.int8)
        placement = placement[: -len("-fp4only")]
    n_hot, n_iq = int((tier == tiers.HOT).sum()), int((tier == tiers.WARM).sum())
    fp4 = synth.make_fp4_bank(n_hot, H, I, "nvfp4", 11, dev)
    iq2 = synth.make_iq2_bank(n_iq, H, I, 12, dev)
    pg = "fp4" if gemm == "fp4" else "tcgen05"
    full = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier, device=dev,
                             prefill_gemm=pg)
    synth.load_bank(full, fp4)
    full.set_iq2_tables()
    synth.load_bank(full, iq2)
    # "balanced": experts dealt by expected routes (the zipf popularity), not by id range
    owner = None
    if placement == "balanced":
        owner = tiers.balanced_owners(tier, world, (1e6 / (pop_rank + 1.0) ** 1.1).astype(np.int64))
    sharded = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K, tokens=T, tier=tier, device=dev,
                                   exchange=exchange, gemm=gemm, owner=owner)
    exact = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K, tokens=T, tier=tier, device=dev,
                                 split_k=(2, 2), exchange=exchange, gemm=gemm, owner=owner)
    sharded.set_iq2_tables()
    synth.load_local(sharded.layer, tier, fp4, iq2)
    exact.set_iq2_tables()
    synth.load_local(exact.layer, tier, fp4, iq2)
    full2 = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier, device=dev,
                              prefill_gemm=pg)
    synth.load_bank(full2, fp4)
    full2.set_iq2_tables()
    synth.load_bank(full2, iq2)
    full2.set_split_k(2, 2)
    res = {}
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    cases = {"zipf": (T, synth.zipf_logits(T, pop_rank, 1.0, 1.1, 200 + rank, dev)),
             "ragged": (17 + 9 * rank, torch.randn((17 + 9 * rank, E), generator=g, device=dev)),
             # every route of every rank goes to rank 0's experts
             "one_owner": (T, torch.where(torch.from_numpy(sharded.owner_np == 0).to(dev), 5.0, -5.0).expand(T, E)
                           + 0.1 * torch.randn((T, E), generator=g, device=dev))}
    for name, (t, logits) in cases.items():
        x = torch.randn((t, H), generator=g, device=dev).to(torch.bfloat16)
        resid = torch.randn((t, H), generator=g, device=dev)
        ids, w = sharded.route(logits.contiguous())
        y = sharded.forward(x, ids, w, residual=resid)
        ref = full.forward_prefill(x, ids, w) if t > 64 else full.forward(x, ids, w).clone()
        sharded.check_errors()
        full.check_errors()
        d = (y - resid - ref).norm() / ref.norm()
        res[name] = float(d)
        res[name + "_comm_ms"] = sharded.comm_ms()
        got = sharded.received()
        res[name + "_routes_in"] = int(got.size)
        res[name + "_foreign_ids"] = int(((got < 0) | (got >= E) | (sharded.owner.cpu().numpy()[np.clip(got, 0, E - 1)] != rank)).sum())
        # fixed split-K on both sides: the sharded layer equals the single-GPU one bit for bit
        y_exact = exact.forward(x, ids, w)
        ref_exact = full2.forward(x, ids, w).clone()
        exact.check_errors()
        res[name + "_bitequal"] = bool(torch.equal(y_exact, ref_exact))
    dist.barrier()
    with open(f"{out_path}.{rank}", "w") as f:
        json.dump(res, f)
    sharded.close()
    exact.close()
    full.close()
    full2.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "p2p", sys.argv[3] if len(sys.argv) > 3 else "skinny",
         sys.argv[4] if len(sys.argv) > 4 else "range")
