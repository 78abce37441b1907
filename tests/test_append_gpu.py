"""Quantize-on-append on the GPU, bit-exact against the oracle and the
reference's golden bytes (codes memcmp-equal, scales equal as fp32 bits)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import bits, d2h

pytestmark = pytest.mark.gpu


def _dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda") if dtype is None else t.to("cuda", dtype)


@pytest.mark.parametrize("n", [4, 7, 8, 9, 16, 31, 128, 133, 512])
def test_quantize_rows_matches_reference_golden(cuda, golden, n):
    import torch
    import eckv
    g = golden("quantize.npz")
    x = g[f"x_{n}"]
    xin = _dev(torch, x)
    q = torch.empty(x.shape, dtype=torch.int8, device="cuda")
    s = torch.empty(x.shape[0], dtype=torch.float32, device="cuda")
    eckv.quantize_per_token_symmetric(xin, q, s, x.shape[0], n)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), g[f"q_{n}"])
    assert np.array_equal(bits(s.cpu().numpy()), bits(g[f"s_{n}"]))


@pytest.mark.parametrize("rows,n", [(1, 1), (3, 5), (1000, 128), (257, 512), (64, 1000), (5, 8191)])
def test_quantize_rows_random(cuda, rows, n):
    import torch
    import eckv
    rng = np.random.default_rng(rows * 31 + n)
    x = (rng.standard_normal((rows, n)) * rng.uniform(0.01, 50, (rows, 1))).astype(np.float32)
    x[rows // 2] = 0.0
    # exact ties x*inv == k + 0.5 appear when x is a half-integer multiple of scale
    wq, ws = O.quantize_per_token_symmetric(x, rows, n)
    q = torch.empty((rows, n), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    eckv.quantize_per_token_symmetric(_dev(torch, x), q, s, rows, n)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(-1), wq)
    assert np.array_equal(bits(s.cpu().numpy()), bits(ws))


@pytest.mark.parametrize("n", [7, 128, 133, 512])
def test_quantize_rows_extreme_magnitudes(cuda, n):
    """Subnormal absmaxes make the scale subnormal and its reciprocal inf:
    the codes then follow x86's out-of-range conversion (-128 body, -127 tail),
    as the reference computes them."""
    import torch
    import eckv
    from test_oracle import extreme_rows
    x = extreme_rows(np.random.default_rng(n + 5), n)
    rows = x.shape[0]
    wq, ws = O.quantize_per_token_symmetric(x, rows, n)
    q = torch.empty((rows, n), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.float32, device="cuda")
    eckv.quantize_per_token_symmetric(_dev(torch, x), q, s, rows, n)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(-1), wq)
    assert np.array_equal(bits(s.cpu().numpy()), bits(ws))


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
def test_batch_append_extreme_magnitudes(cuda, mode, hkv):
    """Append of tokens whose heads span zero, subnormal and huge absmaxes
    (each head of each token drawn at its own magnitude), bit-exact."""
    import torch
    import eckv
    from test_oracle import EXTREME_ROW_SCALES
    rng = np.random.default_rng(100 + 10 * hkv + mode)
    n_tok = 24
    mags = rng.choice(EXTREME_ROW_SCALES, (2, n_tok, hkv, 1))
    kv = (rng.standard_normal((2, n_tok, hkv, 128)) * mags).astype(np.float32)
    kv[:, 0] = 0.0
    k = kv[0].reshape(1, n_tok, hkv * 128)
    v = kv[1].reshape(1, n_tok, hkv * 128)
    bc = eckv.BatchCache([n_tok], num_kv_heads=hkv, head_dim=128, scale_mode=mode)
    bc.append(_dev(torch, k), _dev(torch, v), n_tok)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    off = bc.offsets_host[0]
    for t, (src, codes, scales) in enumerate(((k, bc.keys, bc.key_scales), (v, bc.values, bc.val_scales))):
        wq, ws = O.quantize_kv(src[0], hkv, 128, mode)
        ns = hkv if mode == 0 else 1
        assert np.array_equal(codes.cpu().numpy()[off:off + n_tok], wq), ("kv"[t], hkv, mode)
        assert np.array_equal(bits(scales.cpu().numpy()[off * ns:(off + n_tok) * ns]),
                              bits(ws.reshape(-1)))


def _batch_case(torch, eckv, mode, hkv, caps, lens, n_new, seed):
    rng = np.random.default_rng(seed)
    bc = eckv.BatchCache(caps, num_kv_heads=hkv, head_dim=128, scale_mode=mode)
    bc.length.copy_(torch.tensor(lens, dtype=torch.int32))
    k = W.kv_rows(rng, len(caps) * n_new, hkv, 128).reshape(len(caps), n_new, hkv * 128)
    v = W.kv_rows(rng, len(caps) * n_new, hkv, 128).reshape(len(caps), n_new, hkv * 128)
    bc.append(_dev(torch, k), _dev(torch, v), n_new)
    torch.cuda.synchronize()
    return bc, k, v


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
def test_batch_append_bit_exact(cuda, mode, hkv):
    import torch
    import eckv
    caps = [5, 9, 3, 16, 1]
    lens = [0, 4, 1, 15, 0]
    bc, k, v = _batch_case(torch, eckv, mode, hkv, caps, lens, 1, 10 + hkv + mode)
    assert bc.device_error() == 0
    assert bc.length.cpu().tolist() == [l + 1 for l in lens]
    keys = bc.keys.cpu().numpy()
    vals = bc.values.cpu().numpy()
    ks = bc.key_scales.cpu().numpy()
    vs = bc.val_scales.cpu().numpy()
    ns = hkv if mode == 0 else 1
    for s, (off, L) in enumerate(zip(bc.offsets_host, lens)):
        slot = off + L
        wk, wks = O.quantize_kv(k[s], hkv, 128, mode)
        wv, wvs = O.quantize_kv(v[s], hkv, 128, mode)
        assert np.array_equal(keys[slot], wk[0]) and np.array_equal(vals[slot], wv[0])
        assert np.array_equal(bits(ks[slot * ns:(slot + 1) * ns]), bits(wks.reshape(-1)))
        assert np.array_equal(bits(vs[slot * ns:(slot + 1) * ns]), bits(wvs.reshape(-1)))


def test_batch_append_chunk_of_tokens(cuda):
    """Prefill-style append: 37 tokens per sequence in one call."""
    import torch
    import eckv
    caps, lens, n_new = [100, 64, 37], [10, 27, 0], 37
    bc, k, v = _batch_case(torch, eckv, 0, 4, caps, lens, n_new, 77)
    assert bc.device_error() == 0
    assert bc.length.cpu().tolist() == [l + n_new for l in lens]
    keys = bc.keys.cpu().numpy()
    ks = bc.key_scales.cpu().numpy()
    for s, (off, L) in enumerate(zip(bc.offsets_host, lens)):
        wk, wks = O.quantize_kv(k[s], 4, 128)
        assert np.array_equal(keys[off + L:off + L + n_new], wk)
        assert np.array_equal(bits(ks[(off + L) * 4:(off + L + n_new) * 4]), bits(wks.reshape(-1)))


def test_batch_append_overflow_flags_and_skips(cuda):
    import torch
    import eckv
    caps, lens = [4, 4], [4, 2]
    bc, k, v = _batch_case(torch, eckv, 0, 4, caps, lens, 1, 5)
    assert bc.device_error() == eckv.DEVERR_OVERFLOW
    assert bc.length.cpu().tolist() == [4, 3]      # full sequence untouched, other appended
    assert not bc.keys.cpu().numpy()[:4].any()     # nothing written into the full slab
    assert bc.device_error() == 0                  # reading clears the word


def test_batch_append_bad_table_flags_and_skips(cuda):
    """A length table corrupted on the host is caught on the device."""
    import torch
    import eckv
    bc = eckv.BatchCache([8, 8], num_kv_heads=4)
    bc.offset.copy_(torch.tensor([0, 12], dtype=torch.int32))  # 12 + 8 > 16 slots
    k = torch.randn(2, 512, device="cuda")
    bc.append(k, k, 1)
    torch.cuda.synchronize()
    assert bc.device_error() == eckv.DEVERR_BAD_TABLE
    assert bc.length.cpu().tolist() == [1, 0]
    assert not bc.keys.cpu().numpy()[8:].any()


def test_kvcache_object_reproduces_reference_selftest(cuda, golden):
    """src/kv_cache.cpp:158-251 with the GPU cache in ROW mode (the literal
    KVCache::append): bytes equal to what the reference wrote."""
    import torch
    import eckv
    g = golden("kvcache_row.npz")
    c = eckv.KVCache(num_heads=8, num_kv_heads=4, head_dim=8, num_layers=2, max_seq_len=16,
                     scale_mode=eckv.SCALE_ROW)
    for t in range(5):
        c.append(0, _dev(torch, g["k"][t]), _dev(torch, g["v"][t]))
    torch.cuda.synchronize()
    assert c.seq_len() == 5
    L0 = c.layer(0)
    assert L0.keys_int8 and L0.values_int8 and not L0.keys_fp32
    keys = d2h(L0.keys_int8, (5, 32), np.int8)
    scales = d2h(L0.key_scales, (5,), np.float32)
    assert np.array_equal(keys, g["keys"])
    assert np.array_equal(bits(scales), bits(g["key_scales"]))
    c.reset()
    assert c.seq_len() == 0
    c.append(1, _dev(torch, np.ones(32, np.float32)), _dev(torch, np.full(32, 2.0, np.float32)))
    assert c.layer(1).seq_len == 1 and c.seq_len() == 0
    for _ in range(15):
        c.append(1, _dev(torch, np.ones(32, np.float32)), _dev(torch, np.ones(32, np.float32)))
    with pytest.raises(eckv.ECError) as e:
        c.append(1, _dev(torch, np.ones(32, np.float32)), _dev(torch, np.ones(32, np.float32)))
    assert e.value.status == eckv.EC_ERR_CAPACITY
    c.close()


def test_fp32_mode_is_a_plain_copy(cuda):
    """src/kv_cache.cpp:253-300: fp32 mode stores the projections verbatim."""
    import torch
    import eckv
    c = eckv.KVCache(num_heads=8, num_kv_heads=4, head_dim=8, num_layers=2, max_seq_len=16,
                     use_kv_quantization=False)
    rows = [np.arange(32, dtype=np.float32) + t * 10 for t in range(5)]
    for r in rows:
        c.append(0, _dev(torch, r), _dev(torch, r * 10))
    torch.cuda.synchronize()
    L0 = c.layer(0)
    assert L0.keys_fp32 and not L0.keys_int8
    got = d2h(L0.keys_fp32, (5, 32), np.float32)
    assert np.array_equal(got, np.stack(rows))
    c.close()


def test_fused_dequant_dot(cuda):
    import torch
    import eckv
    rng = np.random.default_rng(3)
    for dim, L in ((4, 3), (16, 2), (128, 1000), (33, 17)):
        k = rng.integers(-127, 128, (L, dim)).astype(np.int8)
        s = rng.random(L).astype(np.float32)
        q = rng.standard_normal(dim).astype(np.float32)
        out = torch.empty(L, dtype=torch.float32, device="cuda")
        eckv.fused_dequant_dot_int8(_dev(torch, q), _dev(torch, k), _dev(torch, s), out, dim, L)
        want = O.fused_dequant_dot_int8(q, k, s, dim, L)
        # fp32 sums in a different order: bound the error by the terms' magnitude
        mag = (np.abs(k.astype(np.float32)) * s[:, None] * np.abs(q)[None, :]).sum(1)
        assert np.all(np.abs(out.cpu().numpy() - want) <= 1e-6 * mag * np.sqrt(dim) + 1e-6)
