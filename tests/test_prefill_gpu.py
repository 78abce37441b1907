"""Chunked-prefill attention on the tcgen05 tensor cores against the oracle.

The oracle for a chunk is the reference's decode loop run per query row with
a causal length (the reference feeds prompts one token at a time,
src/main.cpp:404-405).  Queries are bf16-cast on load, so the oracle is fed
the same bf16-rounded queries; the tolerance is the attention bar of the other
tests (max-abs 2e-3, |err| <= 2e-3 + 1e-3*|ref|).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close, fill_batch

pytestmark = pytest.mark.gpu

D = 128


def _bf16_round(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).bfloat16().float().numpy()


def _case(torch, eckv, pasts, n_new, H, hkv, seed, mode=0, rows=None, qmul=None, raw_q=False):
    """Builds caches of `pasts` tokens, appends n_new tokens per sequence on
    the GPU, runs prefill; returns GPU output and the oracle check rows
    (oracle fed the bf16-cast queries, or the raw fp32 ones with raw_q)."""
    rng = np.random.default_rng(seed)
    seqs, k_new, v_new = [], [], []
    for p in pasts:
        kf = W.kv_rows(rng, p + n_new, hkv, D)
        vf = W.kv_rows(rng, p + n_new, hkv, D)
        seqs.append((kf, vf))
    bc = eckv.BatchCache([p + n_new for p in pasts], num_kv_heads=hkv, scale_mode=mode)
    filled = []
    for (kf, vf), p in zip(seqs, pasts):
        if p:
            kq, ks = O.quantize_kv(kf[:p], hkv, D, mode)
            vq, vs = O.quantize_kv(vf[:p], hkv, D, mode)
        else:
            ns = hkv if mode == 0 else 1
            kq = vq = np.zeros((0, hkv * D), np.int8)
            ks = vs = np.zeros((0, ns) if mode == 0 else (0,), np.float32)
        filled.append((kq, vq, ks, vs))
    fill_batch(bc, filled)
    kn = np.stack([kf[p:] for (kf, vf), p in zip(seqs, pasts)])
    vn = np.stack([vf[p:] for (kf, vf), p in zip(seqs, pasts)])
    bc.append(torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda(), n_new)
    q = W.queries(rng, len(pasts) * n_new, H, D).reshape(len(pasts), n_new, H, D)
    if qmul is not None:
        q = (q * np.asarray(qmul, np.float32).reshape(1, -1, 1, 1)).astype(np.float32)
    out = torch.full((len(pasts), n_new, H, D), float("nan"), device="cuda")
    bc.prefill(torch.from_numpy(q).cuda(), out, n_new, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    got = out.cpu().numpy()
    qb = q if raw_q else _bf16_round(q)
    checks = []
    for s, ((kf, vf), p) in enumerate(zip(seqs, pasts)):
        kq, ks = O.quantize_kv(kf, hkv, D, mode)
        vq, vs = O.quantize_kv(vf, hkv, D, mode)
        for i in (rows if rows is not None else range(n_new)):
            want = O.decode_attention(kq, vq, ks, vs, p + i + 1, qb[s, i], H, hkv, D,
                                      W.softmax_scale(D), mode)
            checks.append((got[s, i], want, f"seq {s} row {i}"))
    return checks


def test_prefill_small_ragged_unaligned(cuda):
    """Pasts not multiples of the 128-token tile, a chunk that ends mid block."""
    import torch
    import eckv
    for got, want, what in _case(torch, eckv, [300, 1000, 0], 200, 16, 4, 1):
        assert_attn_close(got, want, what)


def test_prefill_config5_shape_rows(cuda):
    """Config 5's shapes (8192 cached + 4096 appended, 16 Q / 4 KV heads) on
    two sequences; rows checked at both ends of the chunk and at block edges."""
    import torch
    import eckv
    rows = [0, 1, 2, 127, 128, 129, 1000, 2047, 2048, 4000, 4094, 4095]
    for got, want, what in _case(torch, eckv, [8192, 8192], 4096, 16, 4, 4, rows=rows):
        assert_attn_close(got, want, what)


@pytest.mark.parametrize("n_new", [1, 2, 127, 129])
def test_prefill_chunk_lengths(cuda, n_new):
    """Degenerate and block-edge chunk lengths (one token is a decode step)."""
    import torch
    import eckv
    for got, want, what in _case(torch, eckv, [0, 130, 511], n_new, 16, 4, 40 + n_new):
        assert_attn_close(got, want, what)


@pytest.mark.parametrize("H,hkv", [(8, 8), (32, 8), (4, 1), (16, 2), (12, 4), (6, 2)])
def test_prefill_gqa_groupings(cuda, H, hkv):
    import torch
    import eckv
    for got, want, what in _case(torch, eckv, [129, 40], 130, H, hkv, H + hkv):
        assert_attn_close(got, want, what)


def test_prefill_row_scales(cuda):
    import torch
    import eckv
    for got, want, what in _case(torch, eckv, [77, 256], 64, 16, 4, 9, mode=1):
        assert_attn_close(got, want, what)


def test_prefill_bad_table_flagged(cuda):
    import torch
    import eckv
    bc = eckv.BatchCache([64, 64], num_kv_heads=4)
    bc.length.copy_(torch.tensor([64, 10], dtype=torch.int32))   # 10 < n_new: past < 0
    q = torch.randn(2, 32, 16, D, device="cuda")
    out = torch.zeros(2, 32, 16, D, device="cuda")
    bc.prefill(q, out, 32, 16, 0.1)
    torch.cuda.synchronize()
    assert bc.device_error() == eckv.DEVERR_BAD_TABLE
    assert not out[1].cpu().numpy().any()


@pytest.mark.parametrize("scale", [1e-3, 40.0])
def test_prefill_query_magnitudes(cuda, scale):
    """Queries far from unit scale (the f16 staging of Q uses one power-of-two
    scale per CTA): tiny queries give near-uniform attention, large ones a
    near-one-hot softmax."""
    import torch
    import eckv
    for got, want, what in _case(torch, eckv, [200, 37], 150, 16, 4, 11,
                                 qmul=np.full(150, scale)):
        assert_attn_close(got, want, what)


def test_prefill_mixed_row_magnitudes(cuda):
    """Rows of one 128-row block differ by 10^5 in magnitude: the CTA-wide
    scale comes from the largest row, the small rows keep their precision."""
    import torch
    import eckv
    qmul = np.where(np.arange(128) % 3 == 0, 30.0, 3e-4)
    for got, want, what in _case(torch, eckv, [300], 128, 8, 2, 12, qmul=qmul):
        assert_attn_close(got, want, what)


def test_prefill_error_against_raw_fp32_queries(cuda):
    """The contract casts queries to bf16 on load; against an oracle fed the
    raw fp32 queries the difference is that cast's (about 2^-9 relative per
    query element), reported here beside the bf16-query error."""
    import torch
    import eckv
    rows = [0, 5, 63, 64, 500, 1023]
    cb = _case(torch, eckv, [1024, 64], 1024, 16, 4, 21, rows=rows)
    cr = _case(torch, eckv, [1024, 64], 1024, 16, 4, 21, rows=rows, raw_q=True)
    eb = max(float(np.abs(g - w).max()) for g, w, _ in cb)
    er = max(float(np.abs(g - w).max()) for g, w, _ in cr)
    print(f"prefill max-abs error: {eb:.2e} vs bf16-cast queries, {er:.2e} vs raw fp32 queries")
    for got, want, what in cb:
        assert_attn_close(got, want, what)
    assert er < 0.1, er


def _value_range_case(torch, eckv, past, n_new, vmod, seed):
    """Prefill with V values modified by vmod(v_past, v_new) before
    quantization; returns (got, want, vmax) for every row against the
    oracle's decode loop over the row's causal prefix with the bf16-cast
    query; vmax[row, head] = 127 x the largest v-scale of that head's KV head
    over the row's causal range (the largest |v| it attends over)."""
    rng = np.random.default_rng(seed)
    H, hkv = 16, 4
    kp, vp = W.kv_rows(rng, past, hkv, D), W.kv_rows(rng, past, hkv, D)
    kn, vn = W.kv_rows(rng, n_new, hkv, D), W.kv_rows(rng, n_new, hkv, D)
    vp, vn = vmod(vp, vn)
    bc = eckv.BatchCache([past + n_new], num_kv_heads=hkv)
    if past:
        kq, ks = O.quantize_kv(kp, hkv, D)
        vq, vs = O.quantize_kv(vp, hkv, D)
        fill_batch(bc, [(kq, vq, ks, vs)])
    bc.append(torch.from_numpy(kn[None]).cuda(), torch.from_numpy(vn[None]).cuda(), n_new)
    q = W.queries(rng, n_new, H, D)[None]
    out = torch.empty((1, n_new, H, D), device="cuda")
    bc.prefill(torch.from_numpy(q).cuda(), out, n_new, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    K = np.concatenate([kp, kn]) if past else kn
    V = np.concatenate([vp, vn]) if past else vn
    kq, ks = O.quantize_kv(K, hkv, D)
    vq, vs = O.quantize_kv(V, hkv, D)
    qb = _bf16_round(q)[0]
    got = out.cpu().numpy()[0]
    want = np.stack([O.decode_attention(kq, vq, ks, vs, past + i + 1, qb[i], H, hkv, D,
                                        W.softmax_scale(D)) for i in range(n_new)])
    vpre = 127.0 * np.maximum.accumulate(vs.astype(np.float64), axis=0)[past:]   # [row][kv head]
    vmax = vpre[:, np.arange(H) % hkv]
    return got, want, vmax


def _assert_scaled_close(got, want, vmax, what):
    """The attention bar on data whose values reach 1e6: per (row, head),
    |err| <= 2e-3 + 1e-5 * max|ref| + 2^-24 * vmax, vmax the largest |v| in
    the row's causal range.  A fixed 2e-3 absolute bar is below fp32
    resolution at such magnitudes.  The last term is the kernel's
    precision statement: p' = p * v_scale * 2^-E is carried as an f16 pair
    under the row's own power of two E (set by that largest v-scale), so a
    token's p' keeps an absolute resolution of 2^-25 * 2^E, which in output
    units is about 2^-31 of vmax per token -- below 2^-24 of vmax summed over
    these rows (fp32's own resolution of the largest value the row attends
    over).  Rows whose values stay O(1) are still held to about 2e-3."""
    assert np.isfinite(got).all(), what
    err = np.abs(got - want).max(axis=-1)
    scale = np.abs(want).max(axis=-1)
    bad = err > 2e-3 + 1e-5 * scale + 2.0 ** -24 * vmax
    assert not bad.any(), (what, float(err.max()), float(scale.max()), int(bad.sum()))


def test_prefill_large_v_scales_in_range(cuda):
    """v-scales far above the f16 range of p = softmax weight (|v| in the
    hundreds of thousands, in the first tile, in a later tile and inside the
    diagonal band, so that rows of one CTA have different exponents): each
    row's power of two on p' * v_scale covers them and the rows match the
    oracle (outputs reach 5e5)."""
    import torch
    import eckv

    def big(vp, vn):
        vn = vn.copy()
        vn[10] *= 20000.0          # tile 0 of the chunk (past 0)
        vn[300] *= 3.0e5           # first met in tile 2: the exponent rises mid-row
        vn[301:310] *= 1.0e3
        return vp, vn
    got, want, vmax = _value_range_case(torch, eckv, 0, 384, big, 61)
    _assert_scaled_close(got, want, vmax, "large v")
    got, want, vmax = _value_range_case(torch, eckv, 200, 140, lambda vp, vn: (vp * 4.0e4, vn), 62)
    _assert_scaled_close(got, want, vmax, "large v in the cached part")
    # one token near 1e30 (a v-scale near 2^94): finite, and the rows match
    got, want, vmax = _value_range_case(
        torch, eckv, 0, 200, lambda vp, vn: (vp, vn * np.where(np.arange(200) == 5, 1.0e30, 1.0)[:, None]
                                             .astype(np.float32)), 64)
    _assert_scaled_close(got, want, vmax, "v near 1e30")


def test_prefill_tiny_v_scales_keep_relative_precision(cuda):
    """|v| around 1e-4: p' sits far below f16's normal range without the
    power of two; with it the rows keep their relative precision."""
    import torch
    import eckv
    got, want, _ = _value_range_case(torch, eckv, 130, 200,
                                     lambda vp, vn: (vp * 1.0e-4, vn * 1.0e-4), 63)
    err = float(np.abs(got - want).max())
    assert err <= 1e-3 * float(np.abs(want).max()), err
