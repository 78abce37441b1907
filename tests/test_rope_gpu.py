"""Head norm + RoPE on K fused into the append (echo-core-zig
src/inference/engine.zig:466-532, 544-559) and the same on Q rows, against the
oracle restatement.  The sines and cosines come from different libraries
(CUDA double-precision sincos rounded to fp32 on the GPU, glibc cosf/sinf in
the oracle), so rotated values may differ in the last bit: rotated fp32 rows
are compared to 4 ulp-scale, and int8 codes may differ by 1 where a value
sits on a rounding edge (bounded fraction).  V and the unrotated path are
bit-exact."""
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
    mism, total = 0, 0
    for s, p in enumerate(pasts):
        off = int(bc.offsets_host[s])
        for i in range(n_new):
            x = O.norm_rope(k[s, i].reshape(hkv, D), p + i, 10000.0, w.astype(np.float32))
            kq, kscale = O.quantize_kv(x.reshape(1, -1), hkv, D)
            got = keys[off + p + i].astype(np.int32)
            d = np.abs(got - kq[0].astype(np.int32))
            assert d.max() <= 1
            mism += int((d > 0).sum())
            total += d.size
            np.testing.assert_allclose(ks[(off + p + i) * hkv:(off + p + i + 1) * hkv], kscale[0],
                                       rtol=4e-7 * 8, atol=0)
            vq, vscale = O.quantize_kv(v[s, i].reshape(1, -1), hkv, D)
            assert np.array_equal(vals[off + p + i], vq[0])
            assert np.array_equal(vs[(off + p + i) * hkv:(off + p + i + 1) * hkv], vscale[0])
    assert mism <= max(2, total // 1000), (mism, total)


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
        np.testing.assert_allclose(got[r].reshape(H, D), want, rtol=0, atol=4e-6 * max(1.0, np.abs(want).max()))
