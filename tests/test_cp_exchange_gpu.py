"""The fused context-parallel exchange + merge (ec_cp_exchange_combine over
peer memory): one rank, two ranks on two GPUs (skipped with fewer GPUs), and
the bounded wait running out when a rank never publishes (two processes on
one GPU, only one of which launches anything)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close

pytestmark = pytest.mark.gpu
D = 128
H, HKV = 16, 4


def _seq(L, seed):
    rng = np.random.default_rng(seed)
    kq, ks = O.quantize_kv(W.kv_rows(rng, L, HKV, D), HKV, D)
    vq, vs = O.quantize_kv(W.kv_rows(rng, L, HKV, D), HKV, D)
    q = W.queries(rng, 1, H, D)
    return kq, vq, ks, vs, q


def _partial(torch, eckv, kq, vq, ks, vs, q, dev):
    from _util import fill_batch
    bc = eckv.BatchCache([max(len(kq), 1)], num_kv_heads=HKV, device=dev)
    fill_batch(bc, [(kq, vq, ks, vs)])
    po = torch.empty((1, H, D), device=dev)
    pml = torch.empty((1, H, 2), device=dev)
    bc.decode_partial(torch.from_numpy(q).to(dev), po, pml, H, W.softmax_scale(D))
    return bc, po, pml


def test_single_rank_exchange_is_the_normalised_output(cuda):
    import torch
    import eckv
    import ranks
    kq, vq, ks, vs, q = _seq(3000, 1)
    bc, po, pml = _partial(torch, eckv, kq, vq, ks, vs, q, "cuda")
    cx = ranks.CPExchange(1, H)
    out = torch.empty((1, H, D), device="cuda")
    for _ in range(3):                                  # epochs 1..3, both parities
        cx.combine(po, pml, out)
    torch.cuda.synchronize()
    assert eckv.device_error() == 0
    want = O.decode_attention(kq, vq, ks, vs, 3000, q[0], H, HKV, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy()[0], want, "cp x1")
    cx.close()


def test_single_rank_device_epoch_replays_as_a_graph(cuda):
    """epoch 0: the epoch advances on the device, so the call captured once
    in a CUDA graph is correct on every replay (both parities); a comm then
    refuses a caller epoch."""
    import torch
    import eckv
    import ranks
    kq, vq, ks, vs, q = _seq(3000, 2)
    bc, po, pml = _partial(torch, eckv, kq, vq, ks, vs, q, "cuda")
    cx = ranks.CPExchange(1, H, device_epoch=True)
    out = torch.zeros((1, H, D), device="cuda")
    cx.combine(po, pml, out)                            # device epoch 1, eager
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=side):
        cx.combine(po, pml, out, torch.cuda.current_stream())
    want = O.decode_attention(kq, vq, ks, vs, 3000, q[0], H, HKV, D, W.softmax_scale(D))
    for _ in range(3):                                  # device epochs 2..4
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert eckv.device_error() == 0
        assert_attn_close(out.cpu().numpy()[0], want, "cp x1 graph")
    del g
    import ctypes
    rc = cx._lib.ec_cp_exchange_combine(cx._h, eckv._ptr(po), eckv._ptr(pml), ctypes.c_uint32(7),
                                        eckv._ptr(out), None)
    assert rc == eckv.EC_ERR_INVALID_ARGUMENT
    cx.close()


@pytest.mark.parametrize("L", [3000, 200000])
def test_single_rank_fused_decode_exchange(cuda, L):
    """ec_cp_decode_exchange on one rank: the decode kernel's split-K chunks
    (one chunk at 3,000 tokens, several hundred at 200,000) merged inside the
    exchange kernel give the oracle's output, step after step."""
    import torch
    import eckv
    import ranks
    from _util import fill_batch
    kq, vq, ks, vs, q = _seq(L, 11)
    bc = eckv.BatchCache([L], num_kv_heads=HKV)
    fill_batch(bc, [(kq, vq, ks, vs)])
    cx = ranks.CPExchange(1, H)
    out = torch.empty((1, H, D), device="cuda")
    want = O.decode_attention(kq, vq, ks, vs, L, q[0], H, HKV, D, W.softmax_scale(D))
    qd = torch.from_numpy(q).cuda()
    for step in range(3):
        out.fill_(7.0)
        cx.decode_exchange(bc, qd, out, H, W.softmax_scale(D))
        torch.cuda.synchronize()
        assert eckv.device_error() == 0 and bc.device_error() == 0
        assert_attn_close(out.cpu().numpy()[0], want, f"fused x1 L{L} step {step}")
    cx.close()


def test_single_rank_fused_step_replays_as_a_graph(cuda):
    import torch
    import eckv
    import ranks
    from _util import fill_batch
    L = 50000
    kq, vq, ks, vs, q = _seq(L, 12)
    bc = eckv.BatchCache([L], num_kv_heads=HKV)
    fill_batch(bc, [(kq, vq, ks, vs)])
    cx = ranks.CPExchange(1, H, device_epoch=True)
    out = torch.zeros((1, H, D), device="cuda")
    qd = torch.from_numpy(q).cuda()
    cx.decode_exchange(bc, qd, out, H, W.softmax_scale(D))      # workspace, epoch 1
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=side):
        cx.decode_exchange(bc, qd, out, H, W.softmax_scale(D), torch.cuda.current_stream())
    want = O.decode_attention(kq, vq, ks, vs, L, q[0], H, HKV, D, W.softmax_scale(D))
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert eckv.device_error() == 0
        assert_attn_close(out.cpu().numpy()[0], want, "fused x1 graph")
    del g
    cx.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank, world, port, L, result, same_gpu_timeout, graph=False, fused=False):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("oracle", "echo-core_b200", "tests"):
        sys.path.insert(0, os.path.join(root, sub))
    import datetime
    import torch
    import torch.distributed as dist
    import eckv
    import ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", 0 if same_gpu_timeout else rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        kq, vq, ks, vs, q = _seq(L, 7)
        lo, hi = ranks.shard(L, rank, world)
        bc, po, pml = _partial(torch, eckv, kq[lo:hi], vq[lo:hi], ks[lo:hi], vs[lo:hi], q, dev)
        cx = ranks.CPExchange(1, H, device_epoch=graph)
        out = torch.full((1, H, D), 9.0, device=dev)
        eckv.device_error()                              # clear
        if same_gpu_timeout:
            # rank 1 never publishes: rank 0's bounded wait runs out
            if rank == 0:
                cx.combine(po, pml, out)
                torch.cuda.synchronize()
                code = eckv.device_error()
                np.save(result, np.array([code, float(np.abs(out.cpu().numpy()).max())]))
            dist.barrier()
        elif fused:
            # decode + chunk merge + exchange in two launches per rank
            from _util import fill_batch
            sb = eckv.BatchCache([max(hi - lo, 1)], num_kv_heads=HKV, device=dev)
            fill_batch(sb, [(kq[lo:hi], vq[lo:hi], ks[lo:hi], vs[lo:hi])])
            qd = torch.from_numpy(q).to(dev)
            for _ in range(3):
                cx.decode_exchange(sb, qd, out, H, W.softmax_scale(D))
            torch.cuda.synchronize()
            assert sb.device_error() == 0
        elif graph:
            # every rank captures its step once and replays it: device epochs
            cx.combine(po, pml, out)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=side):
                cx.combine(po, pml, out, torch.cuda.current_stream())
            dist.barrier()
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            del g
        else:
            for _ in range(3):
                cx.combine(po, pml, out)
            torch.cuda.synchronize()
        if not same_gpu_timeout:
            if rank == 0:
                want = O.decode_attention(kq, vq, ks, vs, L, q[0], H, HKV, D, W.softmax_scale(D))
                got = out.cpu().numpy()[0]
                err = float(np.abs(got - want).max())
                ok = bool(np.all(np.abs(got - want) <= 2e-3 + 1e-3 * np.abs(want)))
                np.save(result, np.array([eckv.device_error(), err, float(ok)]))
        cx.close()
    finally:
        dist.destroy_process_group()


def _spawn(tmp_path, same_gpu_timeout, L=20000, world=2, graph=False, fused=False):
    import torch.multiprocessing as mp
    out = str(tmp_path / "r.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_rank_worker,
                      args=(r, world, port, L, out, same_gpu_timeout, graph, fused))
          for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(180)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    return np.load(out)


def test_two_ranks_on_two_gpus(cuda, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    code, err, ok = _spawn(tmp_path, False)
    assert code == 0 and ok == 1.0, (code, err)


def test_all_ranks_on_all_gpus(cuda, tmp_path):
    """One rank per visible GPU (3 to 8): every rank stores into every
    other rank's buffer; the merged output matches the oracle."""
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 3:
        pytest.skip("needs 3 or more GPUs")
    code, err, ok = _spawn(tmp_path, False, L=50000, world=world)
    assert code == 0 and ok == 1.0, (code, err)


def test_ranks_replay_captured_exchange(cuda, tmp_path):
    """Device epochs across ranks: each rank replays its captured exchange;
    one rank per visible GPU (2 to 8)."""
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    code, err, ok = _spawn(tmp_path, False, L=30000, world=world, graph=True)
    assert code == 0 and ok == 1.0, (code, err)


def test_missing_rank_times_out_with_an_error_status(cuda, tmp_path):
    import eckv
    code, amax = _spawn(tmp_path, True, L=2000)
    assert code == eckv.DEVERR_TIMEOUT
    assert amax == 0.0


def test_ranks_fused_decode_exchange(cuda, tmp_path):
    """ec_cp_decode_exchange across ranks, one per visible GPU (2 to 8): each
    rank decodes its contiguous slice; chunk merge, exchange and rank merge
    run in one kernel; the merged output matches the oracle."""
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    code, err, ok = _spawn(tmp_path, False, L=60000, world=world, fused=True)
    assert code == 0 and ok == 1.0, (code, err)
