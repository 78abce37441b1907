"""Cache snapshots (persistence): snapshot -> restore into a fresh cache gives
the same bytes and the same attention; mismatched or damaged images are
refused without touching the cache."""
from __future__ import annotations

import numpy as np
import pytest

import workloads as W

pytestmark = pytest.mark.gpu
D = 128


def _filled(torch, eckv, quant, mode, lens, seed):
    rng = np.random.default_rng(seed)
    c = eckv.KVCache(num_heads=16, num_kv_heads=4, head_dim=D, num_layers=len(lens),
                     max_seq_len=64, use_kv_quantization=quant, scale_mode=mode)
    for l, n in enumerate(lens):
        k = torch.from_numpy(W.kv_rows(rng, n, 4, D)).cuda()
        v = torch.from_numpy(W.kv_rows(rng, n, 4, D)).cuda()
        for t in range(n):
            c.append(l, k[t], v[t])
    return c


def _attend(torch, c, layers, q):
    outs = []
    for l in range(layers):
        o = torch.empty((16, D), device="cuda")
        c.attention(l, q, o, W.softmax_scale(D))
        outs.append(o)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("quant,mode", [(True, 0), (True, 1), (False, 0)])
def test_snapshot_roundtrip(cuda, quant, mode):
    import torch
    import eckv
    lens = [17, 0, 63]
    a = _filled(torch, eckv, quant, mode, lens, 3)
    img = a.snapshot()
    b = eckv.KVCache(num_heads=16, num_kv_heads=4, head_dim=D, num_layers=3, max_seq_len=64,
                     use_kv_quantization=quant, scale_mode=mode)
    b.restore(img)
    for l in range(3):
        assert b.layer(l).seq_len == lens[l]
    assert b.snapshot() == img                         # byte-identical contents
    q = torch.randn(16, D, device="cuda")
    for x, y in zip(_attend(torch, a, 3, q), _attend(torch, b, 3, q)):
        assert np.array_equal(x, y)
    a.close()
    b.close()


def test_snapshot_refuses_mismatch_and_damage(cuda):
    import torch
    import eckv
    a = _filled(torch, eckv, True, 0, [5, 5], 4)
    img = a.snapshot()
    other = eckv.KVCache(num_heads=16, num_kv_heads=4, head_dim=D, num_layers=3, max_seq_len=64)
    with pytest.raises(eckv.ECError):
        other.restore(img)                             # different layer count
    same = _filled(torch, eckv, True, 0, [2, 2], 5)
    before = same.snapshot()
    with pytest.raises(eckv.ECError):
        same.restore(img[:-1])                         # truncated
    bad = bytearray(img)
    bad[0] ^= 0xFF
    with pytest.raises(eckv.ECError):
        same.restore(bytes(bad))                       # wrong magic
    assert same.snapshot() == before                   # nothing changed
    for c in (a, other, same):
        c.close()
