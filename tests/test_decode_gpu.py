"""Split-K decode attention on the GPU against the oracle's fp32 output
(max-abs 2e-3 / rel 1e-3), including the reference's golden outputs, the
BASELINE shapes, GQA groupings, ROW scales, ragged and empty sequences, and
context-parallel partials merged by the log-sum-exp combine."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close, fill_batch

pytestmark = pytest.mark.gpu

D = 128


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _make_seq(rng, L, hkv, mode=O.SCALE_PER_HEAD):
    if L == 0:
        ns = hkv if mode == O.SCALE_PER_HEAD else 1
        z8, zs = np.zeros((0, hkv * D), np.int8), np.zeros((0, ns), np.float32)
        return z8, z8, zs, zs
    kq, ks = O.quantize_kv(W.kv_rows(rng, L, hkv, D), hkv, D, mode)
    vq, vs = O.quantize_kv(W.kv_rows(rng, L, hkv, D), hkv, D, mode)
    return kq, vq, ks, vs


def _run_batch(torch, eckv, seqs, q, H, hkv, mode=0, caps=None, scale=None):
    caps = caps or [max(s[0].shape[0], 1) for s in seqs]
    bc = eckv.BatchCache(caps, num_kv_heads=hkv, scale_mode=mode)
    fill_batch(bc, seqs)
    out = torch.empty((len(seqs), H, D), dtype=torch.float32, device="cuda")
    bc.decode(_dev(torch, q), out, H, W.softmax_scale(D) if scale is None else scale)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    return out.cpu().numpy(), bc


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_decode_matches_reference_golden(cuda, golden, tag):
    import torch
    import eckv
    g = golden("attention.npz")
    seq = (g[f"{tag}_keys"], g[f"{tag}_values"], g[f"{tag}_kscales"], g[f"{tag}_vscales"])
    got, _ = _run_batch(torch, eckv, [seq], g[f"{tag}_q"][None], 16, 4)
    assert_attn_close(got[0], g[f"{tag}_out"], tag)


def test_config1_single_sequence_4096(cuda):
    """batch 1, ctx 4096, 16 Q / 4 KV heads, seed 0."""
    import torch
    import eckv
    cfg = W.config(1)
    rng = np.random.default_rng(cfg.seed)
    seq = _make_seq(rng, 4096, 4)
    q = W.queries(rng, 1, 16, D)
    got, _ = _run_batch(torch, eckv, [seq], q, 16, 4)
    want = O.decode_attention(*seq, 4096, q[0], 16, 4, D, W.softmax_scale(D))
    assert_attn_close(got[0], want, "cfg1")


def test_config2_ragged_batch_append_then_decode(cuda):
    """64 sequences, ctx U[512, 8192], append one token per
    sequence (quantize-on-append on the GPU), then decode; seed 1."""
    import torch
    import eckv
    cfg = W.config(2)
    rng = np.random.default_rng(cfg.seed)
    seqs = [_make_seq(rng, L, 4) for L in cfg.ctx]
    k_new = W.kv_rows(rng, 64, 4, D)
    v_new = W.kv_rows(rng, 64, 4, D)
    q = W.queries(rng, 64, 16, D)
    bc = eckv.BatchCache([L + 1 for L in cfg.ctx], num_kv_heads=4)
    fill_batch(bc, seqs)
    bc.append(_dev(torch, k_new), _dev(torch, v_new), 1)
    out = torch.empty((64, 16, D), dtype=torch.float32, device="cuda")
    bc.decode(_dev(torch, q), out, 16, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    got = out.cpu().numpy()
    for s in range(64):
        kq, vq, ks, vs = seqs[s]
        nk, nks = O.quantize_kv(k_new[s:s + 1], 4, D)
        nv, nvs = O.quantize_kv(v_new[s:s + 1], 4, D)
        K = np.concatenate([kq, nk]); V = np.concatenate([vq, nv])
        KS = np.concatenate([ks, nks]); VS = np.concatenate([vs, nvs])
        want = O.decode_attention(K, V, KS, VS, cfg.ctx[s] + 1, q[s], 16, 4, D, W.softmax_scale(D))
        assert_attn_close(got[s], want, f"seq {s}")


@pytest.mark.parametrize("H,hkv", [
    (16, 4), (8, 4), (4, 4), (32, 8), (16, 8), (8, 8),
    # every num_kv_heads the append covers, query groups up to 32
    (8, 1), (16, 2), (32, 4), (64, 8), (1, 1), (2, 1), (4, 2), (2, 2), (12, 4), (6, 2),
    (24, 4), (16, 1), (48, 8), (32, 1), (40, 2), (20, 4)])
def test_gqa_groupings(cuda, H, hkv):
    import torch
    import eckv
    rng = np.random.default_rng(H * 100 + hkv)
    lens = [1, 31, 32, 33, 200, 1000]
    seqs = [_make_seq(rng, L, hkv) for L in lens]
    q = W.queries(rng, len(lens), H, D)
    got, _ = _run_batch(torch, eckv, seqs, q, H, hkv)
    for s, L in enumerate(lens):
        want = O.decode_attention(*seqs[s], L, q[s], H, hkv, D, W.softmax_scale(D))
        assert_attn_close(got[s], want, f"H{H} hkv{hkv} L{L}")


@pytest.mark.parametrize("H,hkv", [(16, 4), (8, 1), (16, 2), (64, 8), (32, 4)])
def test_row_scale_mode(cuda, H, hkv):
    import torch
    import eckv
    rng = np.random.default_rng(42 + H + hkv)
    lens = [7, 130, 515, 3001]
    seqs = [_make_seq(rng, L, hkv, O.SCALE_ROW) for L in lens]
    q = W.queries(rng, len(lens), H, D)
    got, _ = _run_batch(torch, eckv, seqs, q, H, hkv, mode=eckv.SCALE_ROW)
    for s, L in enumerate(lens):
        want = O.decode_attention(*seqs[s], L, q[s], H, hkv, D, W.softmax_scale(D), O.SCALE_ROW)
        assert_attn_close(got[s], want, f"row H{H} hkv{hkv} L{L}")


@pytest.mark.parametrize("H,hkv", [(8, 1), (16, 2), (32, 4)])
def test_small_kv_head_counts_long_ragged(cuda, H, hkv):
    """One and two KV heads (4-byte scale copies) and split head blocks over
    long ragged sequences at unaligned slab offsets, split-K included."""
    import torch
    import eckv
    rng = np.random.default_rng(H * 3 + hkv)
    lens = [20001, 4097, 1, 9999, 0, 15000]
    seqs = [_make_seq(rng, L, hkv) for L in lens]
    q = W.queries(rng, len(lens), H, D)
    got, bc = _run_batch(torch, eckv, seqs, q, H, hkv, caps=[max(L, 3) for L in lens])
    assert bc.workspace(H)[1] > 0
    for s, L in enumerate(lens):
        if L == 0:
            assert not got[s].any()
            continue
        want = O.decode_attention(*seqs[s], L, q[s], H, hkv, D, W.softmax_scale(D))
        assert_attn_close(got[s], want, f"H{H} hkv{hkv} L{L}")


@pytest.mark.parametrize("H,hkv", [(8, 1), (16, 2)])
def test_kvcache_object_small_kv_head_counts(cuda, H, hkv):
    """The KVCache object's attention with one and two KV heads."""
    import torch
    import eckv
    rng = np.random.default_rng(H + 100 * hkv)
    L = 777
    k = W.kv_rows(rng, L, hkv, D)
    v = W.kv_rows(rng, L, hkv, D)
    q = W.queries(rng, 1, H, D)[0]
    c = eckv.KVCache(num_heads=H, num_kv_heads=hkv, head_dim=D, num_layers=1, max_seq_len=1024)
    kd, vd = _dev(torch, k), _dev(torch, v)
    for t in range(L):
        c.append(0, kd[t], vd[t])
    out = torch.empty(H * D, dtype=torch.float32, device="cuda")
    c.attention(0, _dev(torch, q), out, W.softmax_scale(D))
    torch.cuda.synchronize()
    kq, ks = O.quantize_kv(k, hkv, D)
    vq, vs = O.quantize_kv(v, hkv, D)
    want = O.decode_attention(kq, vq, ks, vs, L, q, H, hkv, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy().reshape(H, D), want, f"kvcache H{H} hkv{hkv}")
    c.close()


def test_empty_and_single_token_sequences(cuda):
    """A sequence with no cached token yields zeros (src/inference.cpp:328-331)."""
    import torch
    import eckv
    rng = np.random.default_rng(7)
    e = (np.zeros((0, 512), np.int8), np.zeros((0, 512), np.int8), np.zeros(0, np.float32),
         np.zeros(0, np.float32))
    seqs = [e, _make_seq(rng, 1, 4), e, _make_seq(rng, 3000, 4)]
    q = W.queries(rng, 4, 16, D)
    got, _ = _run_batch(torch, eckv, seqs, q, 16, 4, caps=[4, 4, 4, 3000])
    assert not got[0].any() and not got[2].any()
    for s in (1, 3):
        L = seqs[s][0].shape[0]
        want = O.decode_attention(*seqs[s], L, q[s], 16, 4, D, W.softmax_scale(D))
        assert_attn_close(got[s], want, f"L{L}")


def test_all_empty_batch_direct_path(cuda):
    import torch
    import eckv
    bc = eckv.BatchCache([8, 8], num_kv_heads=4)
    q = torch.randn(2, 16, D, device="cuda")
    out = torch.full((2, 16, D), 7.0, device="cuda")
    bc.decode(q, out, 16, 0.1)
    torch.cuda.synchronize()
    assert not out.cpu().numpy().any()


def test_kvcache_object_append_then_attention(cuda):
    """The KVCache object path: append through the GPU quantizer one token at a
    time (the reference's per-token loop), then attention over layer 1's own
    length, against the oracle fed the same fp32 projections."""
    import torch
    import eckv
    rng = np.random.default_rng(11)
    L = 300
    k = W.kv_rows(rng, L, 4, D)
    v = W.kv_rows(rng, L, 4, D)
    q = W.queries(rng, 1, 16, D)[0]
    c = eckv.KVCache(num_heads=16, num_kv_heads=4, head_dim=D, num_layers=2, max_seq_len=512)
    kd, vd = _dev(torch, k), _dev(torch, v)
    for t in range(L):
        c.append(1, kd[t], vd[t])
    out = torch.empty(16 * D, dtype=torch.float32, device="cuda")
    c.attention(1, _dev(torch, q), out, W.softmax_scale(D))
    torch.cuda.synchronize()
    kq, ks = O.quantize_kv(k, 4, D)
    vq, vs = O.quantize_kv(v, 4, D)
    want = O.decode_attention(kq, vq, ks, vs, L, q, 16, 4, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy().reshape(16, D), want, "kvcache object")
    out0 = torch.ones(16 * D, dtype=torch.float32, device="cuda")
    c.attention(0, _dev(torch, q), out0, W.softmax_scale(D))  # layer 0 is empty
    torch.cuda.synchronize()
    assert not out0.cpu().numpy().any()
    c.close()


@pytest.mark.parametrize("parts", [2, 3, 4])
def test_context_parallel_partials_and_lse_combine(cuda, parts):
    """One long sequence split contiguously across `parts` shards: partial
    (m, l, O) per shard, merged by ec_lse_combine, equals the whole."""
    import torch
    import eckv
    rng = np.random.default_rng(parts)
    L = 20000
    kq, vq, ks, vs = _make_seq(rng, L, 4)
    q = W.queries(rng, 1, 16, D)
    bounds = np.linspace(0, L, parts + 1).astype(int)
    po = torch.empty((parts, 1, 16, D), dtype=torch.float32, device="cuda")
    pml = torch.empty((parts, 1, 16, 2), dtype=torch.float32, device="cuda")
    qd = _dev(torch, q)
    for p in range(parts):
        a, b = bounds[p], bounds[p + 1]
        bc = eckv.BatchCache([b - a], num_kv_heads=4)
        fill_batch(bc, [(kq[a:b], vq[a:b], ks[a:b], vs[a:b])])
        bc.decode_partial(qd, po[p], pml[p], 16, W.softmax_scale(D))
    out = torch.empty((1, 16, D), dtype=torch.float32, device="cuda")
    eckv.lse_combine(po, pml, parts, 1, 16, D, out)
    torch.cuda.synchronize()
    want = O.decode_attention(kq, vq, ks, vs, L, q[0], 16, 4, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy()[0], want, f"cp{parts}")


@pytest.mark.parametrize("nseq,H,hkv,dh", [
    (2, 16, 4, 128),     # 32 (sequence, head) pairs: the merge splits each pair's dims over 8 CTAs
    (6, 16, 4, 128),     # 96 pairs: 4 CTAs a pair
    (12, 16, 4, 128),    # 192 pairs: 2 CTAs a pair
    (24, 16, 4, 128),    # 384 pairs: one 128-thread CTA a pair
    (2, 8, 2, 256),      # head_dim 256, 16 pairs: 8 CTAs a pair of 32 dims each
    (20, 16, 4, 256),    # head_dim 256, 320 pairs: one 256-thread CTA a pair
    (40, 16, 4, 128),    # 40 sequences: the stream-K plan, its pieces merged by 128-thread CTAs
    (40, 16, 4, 256),    # stream-K at head_dim 256
])
def test_split_k_merge_layouts(cuda, nseq, H, hkv, dh):
    """Every CTA layout of the split-K merge (dims split 8/4/2/1 ways by the
    batch's pair count, 128 or 256 threads) over chunked plans of several
    chunks a sequence and over stream-K pieces: normalised output and the
    partial (m, l, O) form, against the oracle."""
    import torch
    import eckv
    rng = np.random.default_rng(1000 + nseq * 10 + dh)
    lens = [int(x) for x in rng.integers(2000, 9000, nseq)]
    seqs = []
    for L in lens:
        kq, ks = O.quantize_kv(W.kv_rows(rng, L, hkv, dh), hkv, dh)
        vq, vs = O.quantize_kv(W.kv_rows(rng, L, hkv, dh), hkv, dh)
        seqs.append((kq, vq, ks, vs))
    q = W.queries(rng, nseq, H, dh)
    bc = eckv.BatchCache(lens, num_kv_heads=hkv, head_dim=dh)
    fill_batch(bc, seqs)
    assert bc.workspace(H)[1] > 0, "a split plan"
    sc = W.softmax_scale(dh)
    qd = _dev(torch, q)
    out = torch.empty((nseq, H, dh), device="cuda")
    bc.decode(qd, out, H, sc)
    po = torch.empty((nseq, H, dh), device="cuda")
    pml = torch.empty((nseq, H, 2), device="cuda")
    bc.decode_partial(qd, po, pml, H, sc)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    got = out.cpu().numpy()
    part = po.cpu().numpy() / pml.cpu().numpy()[..., 1:2]
    for s in range(nseq):
        want = O.decode_attention(*seqs[s], lens[s], q[s], H, hkv, dh, sc)
        assert_attn_close(got[s], want, f"seq {s}")
        assert_attn_close(part[s], want, f"partial seq {s}")


def test_bad_length_table_is_flagged_not_read(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(5)
    seqs = [_make_seq(rng, 40, 4), _make_seq(rng, 40, 4)]
    bc = eckv.BatchCache([40, 40], num_kv_heads=4)
    fill_batch(bc, seqs)
    bc.length.copy_(torch.tensor([40, 41], dtype=torch.int32))  # 41 > capacity 40
    out = torch.zeros((2, 16, D), device="cuda")
    q = W.queries(rng, 2, 16, D)
    bc.decode(_dev(torch, q), out, 16, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == eckv.DEVERR_BAD_TABLE
    want = O.decode_attention(*seqs[0], 40, q[0], 16, 4, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy()[0], want, "good sequence still decoded")


def test_repeated_calls_are_deterministic(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(8)
    seqs = [_make_seq(rng, L, 4) for L in (5000, 70, 9000)]
    q = W.queries(rng, 3, 16, D)
    a, bc = _run_batch(torch, eckv, seqs, q, 16, 4)
    out = torch.empty((3, 16, D), dtype=torch.float32, device="cuda")
    for _ in range(3):
        bc.decode(_dev(torch, q), out, 16, W.softmax_scale(D))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), a)


def test_ragged_batch_plan_from_token_hint(cuda):
    """A host estimate of the batch's cached tokens (ec_kv_batch.total_tokens_hint)
    steers only the split-K plan (the stream-K grid's size, or the chunk size
    of a chunked plan): the ragged batch of config 2 decodes to the oracle's
    results with and without it."""
    import ctypes
    import torch
    import eckv
    rng = np.random.default_rng(12)
    lens = [int(x) for x in rng.integers(512, 8193, 64)]
    seqs = [_make_seq(rng, L, 4) for L in lens]
    q = _dev(torch, W.queries(rng, 64, 16, D))
    bc = eckv.BatchCache(lens, num_kv_heads=4)
    fill_batch(bc, seqs)
    sc = W.softmax_scale(D)
    outs = []
    for hint in (0, sum(lens)):
        bc.tokens_hint = hint
        d = bc.desc()
        outs.append((eckv.lib().ec_decode_workspace_size_batch(ctypes.byref(d), 16), torch.empty((64, 16, D), device="cuda")))
        bc.decode(q, outs[-1][1], 16, sc)
        torch.cuda.synchronize()
        assert bc.device_error() == 0
    qn = q.cpu().numpy()
    for s in range(0, 64, 7):
        want = O.decode_attention(*seqs[s], lens[s], qn[s], 16, 4, D, sc)
        for _, out in outs:
            assert_attn_close(out.cpu().numpy()[s], want, f"seq {s}")


def test_layer_steps_replayed_as_a_graph(cuda):
    """Append-then-decode over two layers captured once in a CUDA graph and
    replayed: the append, decode and split-K merge kernels follow each other
    with programmatic dependent launch, and every replay must see the token
    the previous kernel appended and the partials it wrote."""
    import torch
    import eckv
    rng = np.random.default_rng(21)
    lens = [int(x) for x in rng.integers(300, 3001, 12)]
    sc = W.softmax_scale(D)
    layers = []
    for _ in range(2):
        seqs = [list(_make_seq(rng, L, 4)) for L in lens]
        bc = eckv.BatchCache([L + 4 for L in lens], num_kv_heads=4)
        fill_batch(bc, [tuple(s) for s in seqs])
        layers.append((bc, seqs))
    k_buf = [torch.empty((12, 4 * D), device="cuda") for _ in layers]
    v_buf = [torch.empty((12, 4 * D), device="cuda") for _ in layers]
    q_buf = [torch.empty((12, 16, D), device="cuda") for _ in layers]
    o_buf = [torch.empty((12, 16, D), device="cuda") for _ in layers]
    for (bc, _), q, o in zip(layers, q_buf, o_buf):
        q.zero_()
        bc.decode(q, o, 16, sc)      # workspace and one-time set-up outside the capture
    torch.cuda.synchronize()
    assert any(bc.workspace(16)[1] > 0 for bc, _ in layers)   # the plan splits
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (bc, _), k, v, q, o in zip(layers, k_buf, v_buf, q_buf, o_buf):
            bc.append(k, v, 1)
            bc.decode(q, o, 16, sc)
    for step in range(3):
        news = []
        for l in range(2):
            kn, vn = W.kv_rows(rng, 12, 4, D), W.kv_rows(rng, 12, 4, D)
            qn = W.queries(rng, 12, 16, D)
            k_buf[l].copy_(_dev(torch, kn)); v_buf[l].copy_(_dev(torch, vn))
            q_buf[l].copy_(_dev(torch, qn))
            news.append((kn, vn, qn))
        g.replay()
        torch.cuda.synchronize()
        for l, ((bc, seqs), (kn, vn, qn)) in enumerate(zip(layers, news)):
            assert bc.device_error() == 0
            got = o_buf[l].cpu().numpy()
            for s in range(12):
                nk, nks = O.quantize_kv(kn[s:s + 1], 4, D)
                nv, nvs = O.quantize_kv(vn[s:s + 1], 4, D)
                kq, vq, ks, vs = seqs[s]
                seqs[s] = [np.concatenate([kq, nk]), np.concatenate([vq, nv]),
                           np.concatenate([ks, nks]), np.concatenate([vs, nvs])]
                L = lens[s] + step + 1
                want = O.decode_attention(*seqs[s], L, qn[s], 16, 4, D, sc)
                assert_attn_close(got[s], want, f"replay {step} layer {l} seq {s}")
    del g
