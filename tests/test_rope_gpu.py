"""Head norm + RoPE on K fused into the append (echo-core-zig
src/inference/engine.zig:466-532, 544-559) and the same on Q rows, against the
oracle restatement (oracle/ec_oracle.c oracle_norm_rope).  The kernels follow
the restatement's operation order exactly -- the sum of squares in dimension
order, each product and sum rounded on its own, cos and sin as the fp32
rounding of the double-precision values -- so codes, scales and rotated rows
are compared bit for bit.  The restatement itself is not pinned to a Zig
output (no Zig toolchain here)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W

pytestmark = pytest.mark.gpu
D = 128


def _weights(rng):
    return (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float16)


def test_append_rope_matches_oracle(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(21)
    pasts, n_new, hkv = [0, 100, 5000], 3, 4
    bc = eckv.BatchCache([p + n_new for p in pasts], num_kv_heads=hkv)
    bc.length.copy_(torch.tensor(pasts, dtype=torch.int32))
    k = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    v = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    w = _weights(rng)
    wd = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    bc.append_rope(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), n_new,
                   rope_base=10000.0, norm_weight=wd)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    keys, vals = bc.keys.cpu().numpy(), bc.values.cpu().numpy()
    ks, vs = bc.key_scales.cpu().numpy(), bc.val_scales.cpu().numpy()
    for s, p in enumerate(pasts):
        off = int(bc.offsets_host[s])
        for i in range(n_new):
            x = O.norm_rope(k[s, i].reshape(hkv, D), p + i, 10000.0, w.astype(np.float32))
            kq, kscale = O.quantize_kv(x.reshape(1, -1), hkv, D)
            assert np.array_equal(keys[off + p + i], kq[0]), f"K codes seq {s} token {i}"
            assert np.array_equal(ks[(off + p + i) * hkv:(off + p + i + 1) * hkv].view(np.uint32),
                                  kscale[0].view(np.uint32)), f"K scales seq {s} token {i}"
            vq, vscale = O.quantize_kv(v[s, i].reshape(1, -1), hkv, D)
            assert np.array_equal(vals[off + p + i], vq[0])
            assert np.array_equal(vs[(off + p + i) * hkv:(off + p + i + 1) * hkv], vscale[0])


@pytest.mark.parametrize("hkv,mode", [(1, 0), (2, 0), (8, 0), (4, 1)])
def test_append_rope_bit_exact_many_positions(cuda, hkv, mode):
    """Codes and scales bit-exact over many tokens at positions up to 2^20
    (large angles), every KV-head count, ROW scales; norm weights of both
    signs and magnitudes."""
    import torch
    import eckv
    rng = np.random.default_rng(31 + hkv + 10 * mode)
    pasts, n_new = [0, 77, 4095, 1048000], 64
    bc = eckv.BatchCache([p + n_new for p in pasts], num_kv_heads=hkv, scale_mode=mode)
    bc.length.copy_(torch.tensor(pasts, dtype=torch.int32))
    k = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    v = np.stack([W.kv_rows(rng, n_new, hkv, D) for _ in pasts])
    w = (rng.standard_normal(D) * 2.0).astype(np.float16)
    wd = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    bc.append_rope(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), n_new,
                   rope_base=10000.0, norm_weight=wd)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    keys, ks = bc.keys.cpu().numpy(), bc.key_scales.cpu().numpy()
    ns = hkv if mode == 0 else 1
    for s, p in enumerate(pasts):
        off = int(bc.offsets_host[s])
        x = np.stack([O.norm_rope(k[s, i].reshape(hkv, D), p + i, 10000.0, w.astype(np.float32))
                      for i in range(n_new)]).reshape(n_new, -1)
        kq, kscale = O.quantize_kv(x, hkv, D, mode)
        assert np.array_equal(keys[off + p:off + p + n_new], kq), f"K codes seq {s}"
        assert np.array_equal(ks[(off + p) * ns:(off + p + n_new) * ns].view(np.uint32),
                              kscale.reshape(-1).view(np.uint32)), f"K scales seq {s}"


def test_append_rope_without_rotation_or_norm_is_plain_append(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(22)
    k = torch.from_numpy(W.kv_rows(rng, 10, 4, D)).cuda().view(2, 5, -1)
    v = torch.from_numpy(W.kv_rows(rng, 10, 4, D)).cuda().view(2, 5, -1)
    a = eckv.BatchCache([8, 8], num_kv_heads=4)
    b = eckv.BatchCache([8, 8], num_kv_heads=4)
    a.append(k, v, 5)
    b.append_rope(k, v, 5, rope_base=0.0, norm_weight=None)
    torch.cuda.synchronize()
    assert torch.equal(a.keys, b.keys) and torch.equal(a.key_scales, b.key_scales)
    assert torch.equal(a.length, b.length)


@pytest.mark.parametrize("norm", [False, True])
def test_rope_rows_on_queries(cuda, norm):
    import torch
    import eckv
    rng = np.random.default_rng(23 + norm)
    rows, H = 6, 16
    q = W.queries(rng, rows, H, D)
    pos = np.array([0, 1, 7, 1000, 65535, 1048575], np.int32)
    w = _weights(rng) if norm else None
    qd = torch.from_numpy(q.copy()).cuda()
    wd = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda() if norm else None
    eckv.rope_rows(qd, rows, H, torch.from_numpy(pos).cuda(), 10000.0, wd)
    torch.cuda.synchronize()
    got = qd.cpu().numpy()
    for r in range(rows):
        want = O.norm_rope(q[r].reshape(H, D), int(pos[r]), 10000.0,
                           None if w is None else w.astype(np.float32))
        assert np.array_equal(got[r].reshape(H, D).view(np.uint32), want.view(np.uint32)), r
