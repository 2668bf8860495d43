"""Expert-parallel host logic on CPU ranks (gloo, world size 2): the placement
digest must agree on every rank (a rank that differs makes all ranks refuse),
and the per-rank route counts exchange gives each rank its transposed row."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, tier_flip: bool, q, owner_mode=None) -> None:
    import sys

    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import __graft_entry__

    __graft_entry__.load_package()
    from b200moe import ep, tiers

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tier, _ = tiers.zipf_tier(384, 150, seed=2)
        if tier_flip and rank == 1:
            tier = tier.copy()
            tier[7] ^= 1
        owner = None
        if owner_mode is not None:  # a placement by expected routes; "flip": rank 1 counted other routes
            counts = np.arange(384, dtype=np.int64)[::-1].copy()
            if owner_mode == "flip" and rank == 1:
                counts[[0, 1]] = counts[[1, 0]] + np.array([0, 5])
            owner = tiers.balanced_owners(tier, world, counts)
        try:
            ep.check_placement(tier, world, owner=owner)
            placement = "agree"
        except RuntimeError:
            placement = "refused"
        # routes of this rank: random ids; counts per owner rank
        rng = np.random.default_rng(100 + rank)
        ids = rng.integers(0, 384, (64, 8))
        owner = ep.owner_of_expert(384, world)
        counts = torch.from_numpy(np.bincount(owner[ids.reshape(-1)], minlength=world).astype(np.int32))
        send, recv = ep.exchange_counts(counts, world)
        q.put((rank, placement, send, recv, counts.tolist()))
    finally:
        dist.destroy_process_group()


def _run(tier_flip: bool, owner_mode=None):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tier_flip, q, owner_mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return {r: rest for r, *rest in out}


def test_placement_agrees_and_counts_transpose():
    res = _run(False)
    assert all(v[0] == "agree" for v in res.values())
    for r in range(2):
        _, send, recv, counts = res[r]
        assert send == counts
        assert recv == [res[s][3][r] for s in range(2)]


def test_placement_mismatch_refused_on_every_rank():
    res = _run(True)
    assert all(v[0] == "refused" for v in res.values())


def test_owner_map_is_part_of_the_placement():
    assert all(v[0] == "agree" for v in _run(False, "same").values())
    assert all(v[0] == "refused" for v in _run(False, "flip").values())


def test_owner_ranges_cover_all_experts():
    from __graft_entry__ import load_package

    load_package()
    from b200moe import ep

    for world in (1, 2, 4, 8):
        own = ep.owner_of_expert(384, world)
        assert np.all(np.diff(own) >= 0) and own[0] == 0 and own[-1] == world - 1
        assert np.bincount(own).tolist() == [384 // world] * world
    with pytest.raises(ValueError):
        ep.owner_of_expert(4, 8)
