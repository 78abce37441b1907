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


def _make_batch(torch, eckv, lens, seed):
    rng = np.random.default_rng(seed)
    seqs = []
    for L in lens:
        if L == 0:
            seqs.append((np.zeros((0, 4 * D), np.int8), np.zeros((0, 4 * D), np.int8),
                         np.zeros((0, 4), np.float32), np.zeros((0, 4), np.float32)))
            continue
        kq, ks = O.quantize_kv(W.kv_rows(rng, L, 4, D), 4, D)
        vq, vs = O.quantize_kv(W.kv_rows(rng, L, 4, D), 4, D)
        seqs.append((kq, vq, ks, vs))
    bc = eckv.BatchCache([max(L, 1) for L in lens], num_kv_heads=4)
    fill_batch(bc, seqs)
    q = torch.from_numpy(W.queries(rng, len(lens), 16, D)).cuda()
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
