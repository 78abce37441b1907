"""Paged KV layout (ec_kv_batch.page_table): sequences hold shuffled pages of
one pool.  Append, decode and prefill over the paged batch give exactly the
contiguous layout's results (same arithmetic on the same bytes, read through
the page table); sequences grow page by page past any initial size; a page
id outside the pool is flagged, not dereferenced."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close, fill_batch

pytestmark = pytest.mark.gpu
D, H, HKV = 128, 16, 4


def _fill_paged(torch, bc, seqs):
    for s, (k, v, ks, vs) in enumerate(seqs):
        L = k.shape[0]
        bc.reserve(s, L)
        if L:
            slots = torch.tensor([bc.slot(s, t) for t in range(L)], dtype=torch.long,
                                 device=bc.keys.device)
            bc.keys[slots] = torch.from_numpy(np.ascontiguousarray(k)).to(bc.keys.device)
            bc.values[slots] = torch.from_numpy(np.ascontiguousarray(v)).to(bc.keys.device)
            ks_idx = (slots[:, None] * HKV + torch.arange(HKV, device=slots.device)).reshape(-1)
            bc.key_scales[ks_idx] = torch.from_numpy(ks.reshape(-1)).to(bc.keys.device)
            bc.val_scales[ks_idx] = torch.from_numpy(vs.reshape(-1)).to(bc.keys.device)
    bc.length.copy_(torch.tensor([s[0].shape[0] for s in seqs], dtype=torch.int32))
    torch.cuda.synchronize()


def _seqs(rng, lens):
    out = []
    for L in lens:
        if L == 0:
            z8 = np.zeros((0, HKV * D), np.int8)
            zs = np.zeros((0, HKV), np.float32)
            out.append((z8, z8, zs, zs))
            continue
        kq, ks = O.quantize_kv(W.kv_rows(rng, L, HKV, D), HKV, D)
        vq, vs = O.quantize_kv(W.kv_rows(rng, L, HKV, D), HKV, D)
        out.append((kq, vq, ks, vs))
    return out


def test_paged_equals_contiguous(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(31)
    lens, n_new = [700, 0, 1300, 255], 130
    seqs = _seqs(rng, lens)
    # same max_seq_len (16 pages x 128) so that both get the same split-K plan
    cont = eckv.BatchCache([L + n_new for L in lens], num_kv_heads=HKV, max_seq_len=16 * 128)
    fill_batch(cont, seqs)
    paged = eckv.PagedBatchCache(len(lens), num_pages=40, page_tokens=128, max_pages=16,
                                 shuffle_seed=5)
    _fill_paged(torch, paged, seqs)
    for s, L in enumerate(lens):
        paged.reserve(s, L + n_new)
    kn = torch.from_numpy(np.stack([W.kv_rows(rng, n_new, HKV, D) for _ in lens])).cuda()
    vn = torch.from_numpy(np.stack([W.kv_rows(rng, n_new, HKV, D) for _ in lens])).cuda()
    cont.append(kn, vn, n_new)
    paged.append(kn, vn, n_new)
    # prefill of the appended chunk
    q = torch.from_numpy(W.queries(rng, len(lens) * n_new, H, D).reshape(len(lens), n_new, H, D)).cuda()
    oc = torch.empty_like(q)
    op = torch.empty_like(q)
    cont.prefill(q, oc, n_new, H, W.softmax_scale(D))
    paged.prefill(q, op, n_new, H, W.softmax_scale(D))
    # decode of one more step
    qd = torch.from_numpy(W.queries(rng, len(lens), H, D)).cuda()
    dc = torch.empty((len(lens), H, D), device="cuda")
    dp = torch.empty_like(dc)
    cont.decode(qd, dc, H, W.softmax_scale(D))
    paged.decode(qd, dp, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert cont.device_error() == 0 and paged.device_error() == 0
    assert torch.equal(cont.length, paged.length)
    for s, L in enumerate(lens):
        off = int(cont.offsets_host[s])
        slots = [paged.slot(s, t) for t in range(L + n_new)]
        assert torch.equal(cont.keys[off:off + L + n_new].cpu(), paged.keys[slots].cpu())
        assert torch.equal(cont.values[off:off + L + n_new].cpu(), paged.values[slots].cpu())
    assert torch.equal(oc, op)
    assert torch.equal(dc, dp)


def test_paged_sequence_grows_page_by_page(cuda):
    """Token-at-a-time growth over many pages (128 tokens each), as the
    reference's engine appends, then decode against the oracle."""
    import torch
    import eckv
    rng = np.random.default_rng(32)
    T = 700
    kf, vf = W.kv_rows(rng, T, HKV, D), W.kv_rows(rng, T, HKV, D)
    bc = eckv.PagedBatchCache(1, num_pages=8, page_tokens=128, shuffle_seed=9)
    kd, vd = torch.from_numpy(kf).cuda(), torch.from_numpy(vf).cuda()
    for t in range(T):
        bc.reserve(0, t + 1)
        bc.append(kd[t:t + 1].view(1, 1, -1), vd[t:t + 1].view(1, 1, -1), 1)
    q = W.queries(rng, 1, H, D)
    out = torch.empty((1, H, D), device="cuda")
    bc.decode(torch.from_numpy(q).cuda(), out, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    assert len(bc.pages[0]) == 6
    kq, ks = O.quantize_kv(kf, HKV, D)
    vq, vs = O.quantize_kv(vf, HKV, D)
    want = O.decode_attention(kq, vq, ks, vs, T, q[0], H, HKV, D, W.softmax_scale(D))
    assert_attn_close(out.cpu().numpy()[0], want, "paged growth")


def test_paged_bad_page_is_flagged(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(33)
    bc = eckv.PagedBatchCache(2, num_pages=4, page_tokens=128)
    _fill_paged(torch, bc, _seqs(rng, [100, 100]))
    bc.page_table[1, 0] = 1 << 20                   # far outside the 4-page pool
    out = torch.zeros((2, H, D), device="cuda")
    bc.decode(torch.randn(2, H, D, device="cuda"), out, H, 0.1)
    torch.cuda.synchronize()
    assert bc.device_error() == eckv.DEVERR_BAD_TABLE


def test_released_pages_serve_a_new_sequence(cuda):
    """A finished sequence's pages go back to the pool and the sequence that
    takes its slot appends into them; attention sees only its own tokens,
    while the other sequence keeps growing past the reuse."""
    import torch
    import eckv
    rng = np.random.default_rng(34)
    bc = eckv.PagedBatchCache(2, num_pages=8, page_tokens=128, shuffle_seed=4)

    def rows(n):
        return W.kv_rows(rng, n, HKV, D)

    k1 = np.stack([rows(256), rows(256)])
    v1 = np.stack([rows(256), rows(256)])
    bc.reserve(0, 256)
    bc.reserve(1, 256)
    bc.append(torch.from_numpy(k1).cuda(), torch.from_numpy(v1).cuda(), 256)
    torch.cuda.synchronize()
    old0 = list(bc.pages[0])
    bc.release(0)
    k2 = np.stack([rows(384), rows(384)])
    v2 = np.stack([rows(384), rows(384)])
    bc.reserve(0, 384)
    bc.reserve(1, 256 + 384)
    assert set(bc.pages[0]) & set(old0)             # the released pages are reused
    bc.append(torch.from_numpy(k2).cuda(), torch.from_numpy(v2).cuda(), 384)
    q = W.queries(rng, 2, H, D)
    out = torch.empty((2, H, D), device="cuda")
    bc.decode(torch.from_numpy(q).cuda(), out, H, W.softmax_scale(D))
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    assert bc.length.cpu().tolist() == [384, 640]
    for s, (kf, vf) in enumerate([(k2[0], v2[0]), (np.concatenate([k1[1], k2[1]]),
                                                   np.concatenate([v1[1], v2[1]]))]):
        kq, ks = O.quantize_kv(kf, HKV, D)
        vq, vs = O.quantize_kv(vf, HKV, D)
        want = O.decode_attention(kq, vq, ks, vs, len(kf), q[s], H, HKV, D, W.softmax_scale(D))
        assert_attn_close(out.cpu().numpy()[s], want, f"sequence {s} after the reuse")
