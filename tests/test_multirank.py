"""Multi-rank host logic on CPU: world-size-2 gloo process groups.

Sequence sharding must cover every sequence once; the context-parallel
protocol (slice -> partial (m, l, O) -> all-gather -> rank-ordered
log-sum-exp merge) must equal attention over the whole sequence.  Partial
states here come from the oracle (CPU); on GPUs the same gather runs over
NCCL between ec_decode_attention_partial and ec_lse_combine.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import oracle as O
import ranks
import workloads as W

D = 128


@pytest.mark.parametrize("n,world", [(0, 2), (1, 2), (7, 2), (32, 8), (5, 8), (1048576, 8)])
def test_shard_covers_every_unit_once_in_rank_order(n, world):
    bounds = [ranks.shard(n, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a, b), (c, d) in zip(bounds, bounds[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_weighted_balances_ragged_lengths(world):
    """Config 2's ragged batch (lengths uniform in [512, 8192]): contiguous,
    rank-ordered blocks covering every sequence once, each rank's cached tokens
    within one sequence of the even share; equal lengths give `shard`'s blocks."""
    import random
    rng = random.Random(world)
    for n in (0, 1, 7, 64, 129):
        lens = [rng.randint(512, 8192) for _ in range(n)]
        blocks = [ranks.shard_weighted(lens, r, world) for r in range(world)]
        assert blocks[0][0] == 0 and blocks[-1][1] == n
        for (lo, hi), (lo2, _) in zip(blocks, blocks[1:]):
            assert lo <= hi == lo2
        if n:
            for lo, hi in blocks:
                assert sum(lens[lo:hi]) <= sum(lens) / world + max(lens)
        assert [ranks.shard_weighted([5] * n, r, world) for r in range(world)] == \
            [ranks.shard(n, r, world) for r in range(world)]


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        ranks.shard(10, 2, 2)
    with pytest.raises(ValueError):
        ranks.shard(10, 0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_worker(rank, world, port, L, seed, result_path):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(seed)          # same sequence on every rank
        kf = W.kv_rows(rng, L, 4, D)
        vf = W.kv_rows(rng, L, 4, D)
        q = W.queries(rng, 1, 16, D)[0]
        kq, ks = O.quantize_kv(kf, 4, D)
        vq, vs = O.quantize_kv(vf, 4, D)
        lo, hi = ranks.shard(L, rank, world)
        o, ml = O.decode_partial(kq[lo:hi], vq[lo:hi], ks[lo:hi], vs[lo:hi], q, 16, 4, D,
                                 W.softmax_scale(D))
        po, pml = ranks.gather_partials(torch.from_numpy(o), torch.from_numpy(ml))
        merged = O.lse_combine(po.numpy(), pml.numpy())
        if rank == 0:
            want = O.decode_attention(kq, vq, ks, vs, L, q, 16, 4, D, W.softmax_scale(D))
            err = float(np.abs(merged - want).max())
            tol = float((2e-3 + 1e-3 * np.abs(want)).min())
            np.save(result_path, np.array([err, tol, po.shape[0]]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L", [1, 777, 4096])
def test_context_parallel_protocol_gloo_world2(tmp_path, L):
    import torch.multiprocessing as mp
    world = 2
    out = str(tmp_path / "r.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_cp_worker, args=(r, world, port, L, L, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    err, tol, parts = np.load(out)
    assert parts == world
    assert err <= tol, (err, tol)
