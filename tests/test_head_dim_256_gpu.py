"""head_dim 256 (the size the reference's target model family uses for its
full-attention layers): quantize-on-append, decode attention, context-split
partials, the KVCache object and the fused norm + RoPE append, against the
oracle at head_dim 256 (src/inference.cpp:302-305 is generic in head_dim)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close, fill_batch

pytestmark = pytest.mark.gpu
D = 256


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _seq(rng, L, hkv, mode=O.SCALE_PER_HEAD):
    if L == 0:
        ns = hkv if mode == O.SCALE_PER_HEAD else 1
        z8, zs = np.zeros((0, hkv * D), np.int8), np.zeros((0, ns), np.float32)
        return z8, z8, zs, zs
    kq, ks = O.quantize_kv(W.kv_rows(rng, L, hkv, D), hkv, D, mode)
    vq, vs = O.quantize_kv(W.kv_rows(rng, L, hkv, D), hkv, D, mode)
    return kq, vq, ks, vs


@pytest.mark.parametrize("hkv,mode", [(1, 0), (2, 0), (4, 0), (8, 0), (2, 1), (4, 1)])
def test_append_bit_exact(cuda, hkv, mode):
    import torch
    import eckv
    rng = np.random.default_rng(70 + hkv + 10 * mode)
    pasts, n_new = [0, 5, 300], 7
    bc = eckv.BatchCache([p + n_new for p in pasts], num_kv_heads=hkv, head_dim=D,
                         scale_mode=mode)
    bc.length.copy_(torch.tensor(pasts, dtype=torch.int32))
    k = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    v = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    k[1, 2] *= 1e-38           # a subnormal-scale row takes the exact path
    bc.append(_dev(torch, k), _dev(torch, v), n_new)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    keys, vals = bc.keys.cpu().numpy(), bc.values.cpu().numpy()
    ks, vs = bc.key_scales.cpu().numpy(), bc.val_scales.cpu().numpy()
    ns = hkv if mode == 0 else 1
    for s, p in enumerate(pasts):
        off = int(bc.offsets_host[s]) + p
        kq, kscale = O.quantize_kv(k[s], hkv, D, mode)
        vq, vscale = O.quantize_kv(v[s], hkv, D, mode)
        assert np.array_equal(keys[off:off + n_new], kq)
        assert np.array_equal(vals[off:off + n_new], vq)
        assert np.array_equal(ks[off * ns:(off + n_new) * ns].view(np.uint32),
                              kscale.reshape(-1).view(np.uint32))
        assert np.array_equal(vs[off * ns:(off + n_new) * ns].view(np.uint32),
                              vscale.reshape(-1).view(np.uint32))
    assert bc.length.cpu().tolist() == [p + n_new for p in pasts]


@pytest.mark.parametrize("H,hkv", [(8, 2), (16, 4), (4, 1), (1, 1), (32, 4), (64, 8), (16, 1),
                                   (32, 1), (12, 2), (8, 8)])
def test_decode_groupings(cuda, H, hkv):
    import torch
    import eckv
    rng = np.random.default_rng(H * 10 + hkv + 256)
    lens = [1, 31, 33, 1000, 6001, 0]
    seqs = [_seq(rng, L, hkv) for L in lens]
    q = W.queries(rng, len(lens), H, D)
    bc = eckv.BatchCache([max(L, 1) for L in lens], num_kv_heads=hkv, head_dim=D)
    fill_batch(bc, seqs)
    out = torch.empty((len(lens), H, D), device="cuda")
    bc.decode(_dev(torch, q), out, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    assert bc.workspace(H)[1] > 0
    got = out.cpu().numpy()
    for s, L in enumerate(lens):
        if L == 0:
            assert not got[s].any()
            continue
        want = O.decode_attention(*seqs[s], L, q[s], H, hkv, D, W.softmax_scale(D))
        assert_attn_close(got[s], want, f"H{H} hkv{hkv} L{L}")


def test_decode_row_scales(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(257)
    H, hkv, lens = 16, 4, [9, 700, 4000]
    seqs = [_seq(rng, L, hkv, O.SCALE_ROW) for L in lens]
    q = W.queries(rng, len(lens), H, D)
    bc = eckv.BatchCache(lens, num_kv_heads=hkv, head_dim=D, scale_mode=eckv.SCALE_ROW)
    fill_batch(bc, seqs)
    out = torch.empty((len(lens), H, D), device="cuda")
    bc.decode(_dev(torch, q), out, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    for s, L in enumerate(lens):
        want = O.decode_attention(*seqs[s], L, q[s], H, hkv, D, W.softmax_scale(D), O.SCALE_ROW)
        assert_attn_close(out.cpu().numpy()[s], want, f"row L{L}")


def test_context_split_partials_and_combine(cuda):
    """One 30,000-token sequence split into 3 shards: partial states at
    head_dim 256 merged by ec_lse_combine equal the whole."""
    import torch
    import eckv
    rng = np.random.default_rng(258)
    H, hkv, L, parts = 8, 2, 30000, 3
    kq, vq, ks, vs = _seq(rng, L, hkv)
    q = W.queries(rng, 1, H, D)
    bounds = np.linspace(0, L, parts + 1).astype(int)
    po = torch.empty((parts, 1, H, D), device="cuda")
    pml = torch.empty((parts, 1, H, 2), device="cuda")
    for p in range(parts):
        a, b = bounds[p], bounds[p + 1]
        bc = eckv.BatchCache([b - a], num_kv_heads=hkv, head_dim=D)
        fill_batch(bc, [(kq[a:b], vq[a:b], ks[a:b], vs[a:b])])
        bc.decode_partial(_dev(torch, q), po[p], pml[p], H, W.softmax_scale(D))
    out = torch.empty((1, H, D), device="cuda")
    eckv.lse_combine(po, pml, parts, 1, H, D, out)
    torch.cuda.synchronize()
    want = O.decode_attention(kq, vq, ks, vs, L, q[0], H, hkv, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy()[0], want, "cp3 d256")


def test_kvcache_object(cuda):
    """The KVCache object at head_dim 256: per-token append through the GPU
    quantizer, then attention over the layer, against the oracle."""
    import torch
    import eckv
    rng = np.random.default_rng(259)
    H, hkv, L = 8, 2, 500
    k, v = W.kv_rows(rng, L, hkv, D), W.kv_rows(rng, L, hkv, D)
    q = W.queries(rng, 1, H, D)[0]
    c = eckv.KVCache(num_heads=H, num_kv_heads=hkv, head_dim=D, num_layers=1, max_seq_len=600)
    kd, vd = _dev(torch, k), _dev(torch, v)
    for t in range(L):
        c.append(0, kd[t], vd[t])
    out = torch.empty(H * D, device="cuda")
    c.attention(0, _dev(torch, q), out, W.softmax_scale(D))
    torch.cuda.synchronize()
    kq, ks = O.quantize_kv(k, hkv, D)
    vq, vs = O.quantize_kv(v, hkv, D)
    want = O.decode_attention(kq, vq, ks, vs, L, q, H, hkv, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy().reshape(H, D), want, "kvcache d256")
    c.close()


def test_norm_rope_append_and_query_rows_bit_exact(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(260)
    hkv, H, pasts, n_new = 2, 8, [0, 1000], 5
    bc = eckv.BatchCache([p + n_new for p in pasts], num_kv_heads=hkv, head_dim=D)
    bc.length.copy_(torch.tensor(pasts, dtype=torch.int32))
    k = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    v = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    w = (1.0 + 0.2 * rng.standard_normal(D)).astype(np.float16)
    wd = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    bc.append_rope(_dev(torch, k), _dev(torch, v), n_new, rope_base=10000.0, norm_weight=wd)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    keys, ks = bc.keys.cpu().numpy(), bc.key_scales.cpu().numpy()
    for s, p in enumerate(pasts):
        off = int(bc.offsets_host[s]) + p
        x = np.stack([O.norm_rope(k[s, i].reshape(hkv, D), p + i, 10000.0, w.astype(np.float32))
                      for i in range(n_new)]).reshape(n_new, -1)
        kq, kscale = O.quantize_kv(x, hkv, D)
        assert np.array_equal(keys[off:off + n_new], kq)
        assert np.array_equal(ks[off * hkv:(off + n_new) * hkv].view(np.uint32),
                              kscale.reshape(-1).view(np.uint32))
    qrows = W.queries(rng, 3, H, D)
    pos = np.array([0, 17, 500000], np.int32)
    qd = _dev(torch, qrows.copy())
    eckv.rope_rows(qd, 3, H, torch.from_numpy(pos).cuda(), 10000.0, wd, head_dim=D)
    torch.cuda.synchronize()
    got = qd.cpu().numpy()
    for r in range(3):
        want = O.norm_rope(qrows[r], int(pos[r]), 10000.0, w.astype(np.float32))
        assert np.array_equal(got[r].view(np.uint32), want.view(np.uint32)), r
