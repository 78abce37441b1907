"""The allocation-free decode entry point, ec_decode_attention_noalloc.

It serves callers that cannot allocate device memory when they run decode
(code where cudaMalloc is off limits, or a runtime whose memory was fixed at
start-up): the split-K workspace comes from a 16 MiB array built into the
library instead of from the caller.  This test calls it through the C ABI and
checks that two calls in a row give the same output as ec_decode_attention
with a caller-provided workspace, within the attention tolerance the other
tests use.  It lives in a file pytest collects last, so a run that stops at
the first failure has already run everything else.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close, fill_batch

pytestmark = pytest.mark.gpu

D = 128


def _seqs(rng, lens, mode=O.SCALE_PER_HEAD):
    seqs = []
    ns = 4 if mode == O.SCALE_PER_HEAD else 1
    for L in lens:
        if L == 0:
            seqs.append((np.zeros((0, 4 * D), np.int8), np.zeros((0, 4 * D), np.int8),
                         np.zeros((0, ns), np.float32), np.zeros((0, ns), np.float32)))
            continue
        kq, ks = O.quantize_kv(W.kv_rows(rng, L, 4, D), 4, D, mode)
        vq, vs = O.quantize_kv(W.kv_rows(rng, L, 4, D), 4, D, mode)
        seqs.append((kq, vq, ks, vs))
    return seqs


def _make_batch(torch, eckv, lens, seed, mode=O.SCALE_PER_HEAD, seqs_out=None):
    rng = np.random.default_rng(seed)
    seqs = _seqs(rng, lens, mode)
    bc = eckv.BatchCache([max(L, 1) for L in lens], num_kv_heads=4, scale_mode=mode)
    fill_batch(bc, seqs)
    q = torch.from_numpy(W.queries(rng, len(lens), 16, D)).cuda()
    if seqs_out is not None:
        seqs_out.extend(seqs)
    return bc, q


def _noalloc(eckv, torch, bc, q, out):
    d = bc.desc()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return eckv.lib().ec_decode_attention_noalloc(
        ctypes.byref(d), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(out.data_ptr()), 16,
        ctypes.c_float(W.softmax_scale(D)), stream)


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    import torch
    import eckv
    # ragged lengths long enough that decode splits and uses its scratch
    lens = [9000, 1, 4096, 0, 20000, 777, 15000, 3333]
    bc, q = _make_batch(torch, eckv, lens, 21)
    want = torch.empty((len(lens), 16, D), device="cuda")
    bc.decode(q, want, 16, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert eckv.lib().ec_decode_workspace_size(bc.num_seqs, 16, D, bc.max_seq_len) > 0
    ref = want.cpu().numpy()
    for call in range(2):
        out = torch.full((len(lens), 16, D), float("nan"), device="cuda")
        rc = _noalloc(eckv, torch, bc, q, out)
        assert rc == eckv.EC_OK, eckv.lib().ec_last_error()
        torch.cuda.synchronize()
        assert bc.device_error() == 0
        assert_attn_close(out.cpu().numpy(), ref, f"no-alloc call {call}")


def _workspace_result(torch, bc, q):
    want = torch.empty((bc.num_seqs, 16, D), device="cuda")
    bc.decode(q, want, 16, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    return want.cpu().numpy()


def _noalloc_result(torch, eckv, bc, q):
    out = torch.full((bc.num_seqs, 16, D), float("nan"), device="cuda")
    rc = _noalloc(eckv, torch, bc, q, out)
    assert rc == eckv.EC_OK, eckv.lib().ec_last_error()
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    return out.cpu().numpy()


def test_noalloc_row_scales_match_workspace_entry_point(cuda):
    """ROW scales (one scale per token row, the reference's KVCache::append
    layout) through the no-alloc path, split so the scratch is used."""
    import torch
    import eckv
    bc, q = _make_batch(torch, eckv, [6000, 130, 11000], 22, mode=O.SCALE_ROW)
    assert bc.workspace(16)[1] > 0
    assert_attn_close(_noalloc_result(torch, eckv, bc, q), _workspace_result(torch, bc, q), "row")


def test_noalloc_paged_batch_without_offsets_matches_oracle(cuda):
    """A paged batch built the documented way (seq_offset NULL, shuffled pages
    of one pool) decoded by the no-alloc path, against the CPU oracle."""
    import torch
    import eckv
    rng = np.random.default_rng(23)
    lens = [3000, 0, 777, 5000]
    seqs = _seqs(rng, lens)
    bc = eckv.PagedBatchCache(len(lens), num_pages=80, page_tokens=128, max_pages=48,
                              shuffle_seed=9)
    for s, (k, v, ks, vs) in enumerate(seqs):
        L = k.shape[0]
        bc.reserve(s, max(L, 1))
        if L:
            slots = torch.tensor([bc.slot(s, t) for t in range(L)], dtype=torch.long, device="cuda")
            bc.keys[slots] = torch.from_numpy(k).cuda()
            bc.values[slots] = torch.from_numpy(v).cuda()
            idx = (slots[:, None] * 4 + torch.arange(4, device="cuda")).reshape(-1)
            bc.key_scales[idx] = torch.from_numpy(ks.reshape(-1)).cuda()
            bc.val_scales[idx] = torch.from_numpy(vs.reshape(-1)).cuda()
    bc.length.copy_(torch.tensor(lens, dtype=torch.int32))
    assert bc.desc().seq_offset is None
    assert bc.workspace(16)[1] > 0
    qn = W.queries(rng, len(lens), 16, D)
    q = torch.from_numpy(qn).cuda()
    for call in range(2):
        got = _noalloc_result(torch, eckv, bc, q)
        for s, L in enumerate(lens):
            if L == 0:
                assert not got[s].any()
                continue
            want = O.decode_attention(*seqs[s], L, qn[s], 16, 4, D, W.softmax_scale(D))
            assert_attn_close(got[s], want, f"paged no-alloc call {call} seq {s}")


def test_noalloc_scratch_reused_across_split_plans(cuda):
    """Calls with different split-K plans share the one array: a widely split
    batch, then a lightly split one, then the first again, each equal to the
    workspace entry point's result."""
    import torch
    import eckv
    big = _make_batch(torch, eckv, [30000, 25000], 24)
    small = _make_batch(torch, eckv, [2000] * 40, 25)
    assert big[0].workspace(16)[1] > 0 and small[0].workspace(16)[1] > 0
    for bc, q in (big, small, big):
        assert_attn_close(_noalloc_result(torch, eckv, bc, q), _workspace_result(torch, bc, q),
                          f"{bc.num_seqs} sequences")


def test_noalloc_rejects_batches_beyond_its_fixed_scratch(cuda):
    import torch
    import eckv
    # 4096 sequences of up to 1M tokens would need far more than 16 MiB of
    # split-K scratch; the call must refuse before touching any buffer.
    bc, q = _make_batch(torch, eckv, [64], 3)
    d = bc.desc()
    d.num_seqs = 4096
    d.max_seq_len = 1 << 20
    out = torch.empty((1, 16, D), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = eckv.lib().ec_decode_attention_noalloc(
        ctypes.byref(d), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(out.data_ptr()), 16,
        ctypes.c_float(0.1), stream)
    assert rc == eckv.EC_ERR_WORKSPACE
    assert b"16777216-byte array" in eckv.lib().ec_last_error()
