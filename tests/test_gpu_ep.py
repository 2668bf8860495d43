"""Expert-parallel layer on the GPU: dispatch -> owner compute -> combine
against the full single-GPU layer on the same tokens (world 1 here; world 2
over NCCL through torchrun when the box has two GPUs)."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-3  # two fp16-y2 paths whose split-K sums differ in order


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("exchange,gemm", [("p2p", "skinny"), ("nccl", "skinny"), ("p2p", "fp4")])
def test_ep_world1_matches_layer(dev, pkg, exchange, gemm):
    from b200moe import ep, moe, synth, tiers

    H, I, E, K, T = 1024, 512, 64, 6, 48
    tier, pop_rank = tiers.zipf_tier(E, 40, seed=3)
    n_hot, n_iq = int((tier == tiers.HOT).sum()), int((tier == tiers.WARM).sum())
    fp4 = synth.make_fp4_bank(n_hot, H, I, "nvfp4", 11, dev)
    iq2 = synth.make_iq2_bank(n_iq, H, I, 12, dev)
    full = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier, device=dev,
                             prefill_gemm="fp4" if gemm == "fp4" else "tcgen05")
    synth.load_bank(full, fp4)
    full.set_iq2_tables()
    synth.load_bank(full, iq2)
    sharded = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K, tokens=T, tier=tier, device=dev,
                                   exchange=exchange, gemm=gemm)
    sharded.set_iq2_tables()
    synth.load_local(sharded.layer, tier, fp4, iq2)
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    logits = synth.zipf_logits(T, pop_rank, 1.0, 1.1, 6, dev)
    ids, w = sharded.route(logits)
    ids2, w2 = full.route(logits)
    assert torch.equal(ids, ids2) and torch.equal(w, w2)
    ref = full.forward(x, ids, w).clone()
    y = sharded.forward(x, ids, w)
    sharded.check_errors()
    assert float((y - ref).norm() / ref.norm()) < TOL
    resid = torch.randn((T, H), generator=g, device=dev)
    y_r = sharded.forward(x, ids, w, residual=resid)
    assert torch.equal(y_r, y + resid)
    assert sharded.received().size == T * K
    # a route without an expert: flagged, contributes nothing, the layer recovers
    bad = ids.clone()
    bad[3, 2] = E + 7
    y_b = sharded.forward(x, bad, w)
    from b200moe import _lib

    with pytest.raises(_lib.B200MoeError) as ei:
        sharded.check_errors()
    assert ei.value.status == 5
    w_b = w.clone()
    w_b[3, 2] = 0.0
    y_z = sharded.forward(x, ids, w_b)
    sharded.check_errors()
    assert float((y_b[3] - y_z[3]).norm() / y_z[3].norm()) < TOL
    assert torch.equal(sharded.forward(x, ids, w), y)
    if exchange == "p2p":  # the step holds no host sync: replay it from a CUDA graph
        out = torch.empty_like(y)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            sharded.forward(x, ids, w, out=out)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                sharded.forward(x, ids, w, out=out)
        torch.cuda.current_stream().wait_stream(s)
        out.zero_()
        g.replay()
        g.replay()
        sharded.check_errors()
        assert torch.equal(out, y)
        del g
    # same fixed split-K on both sides: bit-equal to the single-GPU layer
    full.set_split_k(2, 2)
    sharded.layer.set_split_k(2, 2)
    ref = full.forward(x, ids, w).clone()
    assert torch.equal(sharded.forward(x, ids, w), ref)
    with pytest.raises(_lib.B200MoeError):
        full.set_split_k(3, 0)
    sharded.close()
    full.close()


@pytest.mark.parametrize("exchange,gemm,placement", [("p2p", "skinny", "range"), ("nccl", "skinny", "range"),
                                                     ("p2p", "fp4", "range"), ("p2p", "fp4", "balanced"),
                                                     ("p2p", "fp4", "range-fp4only")])
def test_ep_two_gpus(tmp_path, exchange, gemm, placement):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "ep"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(Path(__file__).with_name("ep_worker.py")), str(out), exchange, gemm, placement]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    for rank in range(2):
        res = json.loads(Path(f"{out}.{rank}").read_text())
        for case in ("zipf", "ragged", "one_owner"):
            assert res[case] < TOL, (rank, case, res)
            assert res[case + "_bitequal"], (rank, case)
        for case in ("zipf", "ragged", "one_owner"):
            assert res[case + "_foreign_ids"] == 0, (rank, case)
        # every route goes to rank 0's experts: rank 1 receives none
        assert res["one_owner_routes_in"] == 0 if rank == 1 else res["one_owner_routes_in"] > 0
        assert res["zipf_comm_ms"] > 0


def test_ep_world1_fused_return_bit_equal(dev, pkg):
    """An all-FP4 block-scaled layer: the owner's W2 epilogue stores each y2
    row at its home (no return launch) and raises the return flag; the
    result is bit-equal to the single-GPU layer on the same path, step after
    step (the flags' epochs advance, the reservation counters reset)."""
    from b200moe import ep, moe, synth

    H, I, E, K, T = 1024, 512, 48, 8, 40
    tier = np.zeros(E, np.int8)
    bank = synth.make_fp4_bank(E, H, I, "nvfp4", 17, dev)
    full = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=K, max_tokens=64, tier=tier, device=dev,
                             prefill_gemm="fp4")
    synth.load_bank(full, bank)
    sharded = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K, tokens=T, tier=tier, device=dev,
                                   gemm="fp4")
    assert sharded.fused_return
    synth.load_bank(sharded.layer, bank)
    g = torch.Generator(device=dev).manual_seed(8)
    for step in range(3):
        x = torch.randn((T - 7 * step, H), generator=g, device=dev).to(torch.bfloat16)
        ids, w = sharded.route(torch.randn((x.shape[0], E), generator=g, device=dev))
        want = full.forward(x, ids, w).clone()
        got = sharded.forward(x, ids, w).clone()
        sharded.check_errors()
        full.check_errors()
        assert torch.equal(got, want), step
    sharded.close()
    full.close()


@pytest.mark.parametrize("gemm", ["skinny", "fp4"])
def test_rows_forward_device_count(dev, pkg, gemm):
    """The top-1 rows forward of expert parallelism with fewer valid rows than
    the launch bound (the count lives on the device): rows past the count are
    ignored even when an earlier call left their routes in other places."""
    from b200moe import _lib, moe, synth

    H, I, E, R = 1024, 512, 32, 96
    layer = moe.B200NativeMoe(hidden=H, inter=I, num_experts=E, top_k=1, max_tokens=64, max_prefill_tokens=R,
                              tier=np.zeros(E, np.int8), device=dev, prefill_gemm="fp4" if gemm == "fp4" else "skinny")
    synth.load_bank(layer, synth.make_fp4_bank(E, H, I, "nvfp4", 21, dev))
    layer.set_split_k(2, 0)
    g = torch.Generator(device=dev).manual_seed(22)
    rows = torch.randn((R, H), generator=g, device=dev).to(torch.float16)
    eids = torch.randint(0, E, (R,), generator=g, device=dev, dtype=torch.int32)
    y2 = torch.empty((R, H), dtype=torch.float16, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    L = _lib.lib()

    def run(n):
        cnt = torch.tensor([n], dtype=torch.int32, device=dev)
        rng = torch.tensor([0, n], dtype=torch.int32, device=dev)
        y2.fill_(float("nan"))
        _lib.check("b200moe_forward_rows", L.b200moe_forward_rows(
            layer._h, st, rows.data_ptr(), eids.data_ptr(), cnt.data_ptr(), rng.data_ptr(), R, y2.data_ptr()))
        layer.check_errors()
        return y2.clone()

    full = run(R)
    eids[R // 2:] = (eids[R // 2:] + 7) % E  # the stale half now belongs to other experts
    half = run(R // 2)
    assert torch.equal(half[:R // 2], full[:R // 2])
    assert torch.isnan(half[R // 2:].float()).all()  # nothing written past the count
    layer.close()


def test_ep_bounded_wait_times_out_and_recovers(dev, pkg):
    """A flag that nothing sets: a push without its return leaves the
    combine's return flag behind the step's epoch.  The combine's wait ends
    at its bound (2 s) with B200MOE_ERR_TIMEOUT, writes nothing, and the
    exchange keeps working: the next full step gives the same bits as before."""
    import time

    from b200moe import _lib, ep, synth

    H, I, E, K, T = 1024, 512, 32, 4, 16
    tier = np.zeros(E, np.int8)
    lay = ep.ExpertParallelMoe(hidden=H, inter=I, num_experts=E, top_k=K, tokens=T, tier=tier, device=dev)
    synth.load_bank(lay.layer, synth.make_fp4_bank(E, H, I, "nvfp4", 3, dev))
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    ids, w = lay.route(torch.randn((T, E), generator=g, device=dev))
    y0 = lay.forward(x, ids, w).clone()
    lay.check_errors()
    L, pe = _lib.lib(), lay._peer
    st = torch.cuda.current_stream(dev).cuda_stream
    _lib.check("push", L.b200moe_ep_push(pe.handle, st, x.data_ptr(), _lib.BF16, ids.data_ptr(), T, K, E,
                                         lay.owner.data_ptr()))
    out = torch.full((T, H), 7.0, dtype=torch.float32, device=dev)
    torch.cuda.synchronize(dev)
    t0 = time.monotonic()
    _lib.check("combine", L.b200moe_ep_combine_p2p(pe.handle, st, ids.data_ptr(), w.data_ptr(), T, K, E,
                                                   lay.owner.data_ptr(), None, out.data_ptr()))
    status = pe.check()
    waited = time.monotonic() - t0
    assert _lib.STATUS[status] == "B200MOE_ERR_TIMEOUT", status
    assert 1.5 < waited < 60, waited
    assert torch.all(out == 7.0)  # nothing written after the wait gave up
    assert pe.check() == 0  # the error word was cleared
    y1 = lay.forward(x, ids, w).clone()
    lay.check_errors()
    assert torch.equal(y0, y1)
    lay.close()
