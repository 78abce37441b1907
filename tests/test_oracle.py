"""The CPU oracle (oracle/ec_oracle.c) pinned against the reference.

Three layers of pinning, all CPU-only:
  1. the reference's own known-answer tests, restated
     (src/kernels/quant.cpp:403-521, src/kv_cache.cpp:158-300);
  2. golden fixtures produced by the reference's compiled code
     (tests/golden/make_golden.py) -- bit-exact;
  3. when oracle/_ref is built here, fresh seeded cases run through the
     reference itself -- bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------- 1. reference KATs
def test_quant_test1_known_answer():
    # src/kernels/quant.cpp:403-432: {1,2,3,4} -> scale 4/127 (+-1e-6), error < scale/2
    x = np.array([1, 2, 3, 4], np.float32)
    q, s = O.quantize_per_token_symmetric(x, 1, 4)
    assert abs(s[0] - 4.0 / 127.0) < 1e-6
    err = np.abs(q.astype(np.float32) * s[0] - x).max()
    assert err < s[0] * 0.5 + 1e-6


def test_quant_test2_fused_dot_known_answer():
    # src/kernels/quant.cpp:434-486: 3x4 keys, fused dot within 1e-4 of dequantised dot
    q = np.array([1, 2, 3, 4], np.float32)
    keys = np.array([[1, 0, -1, 0.5], [0, 1, 0, 0], [2, 2, 2, 2]], np.float32)
    k8, ks = O.quantize_per_token_symmetric(keys, 3, 4)
    k8 = k8.reshape(3, 4)
    got = O.fused_dequant_dot_int8(q, k8, ks, 4, 3)
    want = (k8.astype(np.float32) * ks[:, None]) @ q
    assert np.abs(got - want).max() < 1e-4


def test_quant_test3_dim16_known_answer():
    # src/kernels/quant.cpp:488-521: dim 16, error < scale*8 + 1
    q = np.arange(1, 17, dtype=np.float32)
    keys = np.stack([np.arange(1, 17), np.arange(16, 0, -1)]).astype(np.float32)
    k8, ks = O.quantize_per_token_symmetric(keys, 2, 16)
    got = O.fused_dequant_dot_int8(q, k8.reshape(2, 16), ks, 16, 2)
    exact = keys @ q
    assert np.all(np.abs(got - exact) < ks * 8 + 1)


def test_kvcache_test1_row_semantics(golden):
    # src/kv_cache.cpp:158-251: 5 tokens, 4 heads x 8; dequant error of token 0
    # < scale; fused dot over the 32-wide row with key_scales[t] within 1e-3.
    g = golden("kvcache_row.npz")
    hkv, d = 4, 8
    keys = np.zeros((16, hkv * d), np.int8)
    vals = np.zeros((16, hkv * d), np.int8)
    ks = np.zeros(16 * hkv, np.float32)
    vs = np.zeros(16 * hkv, np.float32)
    for t in range(5):
        kk, ksc = O.quantize_kv(g["k"][t:t + 1], hkv, d, O.SCALE_ROW)
        vv, vsc = O.quantize_kv(g["v"][t:t + 1], hkv, d, O.SCALE_ROW)
        keys[t], vals[t], ks[t], vs[t] = kk[0], vv[0], ksc[0], vsc[0]
    assert np.array_equal(keys[:5], g["keys"]) and np.array_equal(vals[:5], g["values"])
    assert np.array_equal(bits(ks[:5]), bits(g["key_scales"][:5]))
    assert np.array_equal(bits(vs[:5]), bits(g["val_scales"][:5]))
    err = np.abs(keys[0].astype(np.float32) * ks[0] - g["k"][0]).max()
    assert err < ks[0] + 1e-4
    scores = O.fused_dequant_dot_int8(np.ones(32, np.float32), keys[:5], ks[:5], 32, 5)
    want = (keys[:5].astype(np.float32) * ks[:5, None]).sum(1)
    assert np.abs(scores - want).max() < 1e-3


# ------------------------------------------------------ 2. golden fixtures
@pytest.mark.parametrize("n", [4, 7, 8, 9, 16, 31, 128, 133, 512])
def test_quantize_matches_golden(golden, n):
    g = golden("quantize.npz")
    x = g[f"x_{n}"]
    q, s = O.quantize_per_token_symmetric(x, x.shape[0], n)
    assert np.array_equal(q.reshape(x.shape), g[f"q_{n}"])
    assert np.array_equal(bits(s), bits(g[f"s_{n}"]))


def test_quantize_test1_golden(golden):
    g = golden("quantize.npz")
    q, s = O.quantize_per_token_symmetric(g["x_test1"], 1, 4)
    assert np.array_equal(q.reshape(1, 4), g["q_test1"]) and np.array_equal(bits(s), bits(g["s_test1"]))


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_decode_attention_matches_golden(golden, tag):
    g = golden("attention.npz")
    L = int(g[f"{tag}_len"][0])
    out = O.decode_attention(g[f"{tag}_keys"], g[f"{tag}_values"], g[f"{tag}_kscales"],
                             g[f"{tag}_vscales"], L, g[f"{tag}_q"], 16, 4, 128, W.softmax_scale(128))
    assert np.array_equal(bits(out), bits(g[f"{tag}_out"]))


def test_prefill_is_decode_per_row():
    rng = np.random.default_rng(5)
    H, hkv, d, past, n = 8, 4, 128, 9, 6
    kq, ks = O.quantize_kv(W.kv_rows(rng, past + n, hkv, d), hkv, d)
    vq, vs = O.quantize_kv(W.kv_rows(rng, past + n, hkv, d), hkv, d)
    q = W.queries(rng, n, H, d)
    out = O.prefill_attention(kq, vq, ks, vs, past, n, q, H, hkv, d, 0.1)
    for i in range(n):
        row = O.decode_attention(kq, vq, ks, vs, past + i + 1, q[i], H, hkv, d, 0.1)
        assert np.array_equal(bits(out[i]), bits(row))


def test_empty_cache_gives_zeros():
    out = O.decode_attention(np.zeros((1, 512), np.int8), np.zeros((1, 512), np.int8),
                             np.ones(4, np.float32), np.ones(4, np.float32), 0,
                             np.ones(16 * 128, np.float32), 16, 4, 128, 0.1)
    assert not out.any()


# ------------------------------------- 3. the reference itself, when built
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built here")


@needs_ref
@pytest.mark.parametrize("n", [1, 5, 8, 13, 64, 128, 250, 512, 1000])
def test_quantize_matches_reference_build(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((17, n)) * 4).astype(np.float32)
    x[3] = 0.0
    a = O.quantize_per_token_symmetric(x, 17, n)
    b = O.ref_quantize_per_token_symmetric(x, 17, n)
    assert np.array_equal(a[0], b[0]) and np.array_equal(bits(a[1]), bits(b[1]))


# row magnitudes from an all-zero row through subnormal absmaxes (whose scale
# is subnormal and whose reciprocal overflows to inf) to near FLT_MAX / 127
EXTREME_ROW_SCALES = [0.0, 1e-45, 1e-44, 1e-41, 1e-39, 1e-37, 2e-37, 5e-37, 1.5e-36, 3e-36, 1e-30, 1.0,
                      1e30, 1e37]


def extreme_rows(rng, n, reps=2):
    rows = []
    for s in EXTREME_ROW_SCALES:
        for _ in range(reps):
            rows.append(rng.standard_normal(n) * s)
    x = np.array(rows, dtype=np.float64).astype(np.float32)
    x[1, : n // 2] = 0.0
    return x


@needs_ref
@pytest.mark.parametrize("n", [7, 128, 133, 512])
def test_quantize_extreme_magnitudes_match_reference_build(n):
    x = extreme_rows(np.random.default_rng(n + 5), n)
    rows = x.shape[0]
    a = O.quantize_per_token_symmetric(x, rows, n)
    b = O.ref_quantize_per_token_symmetric(x, rows, n)
    assert np.array_equal(a[0], b[0]) and np.array_equal(bits(a[1]), bits(b[1]))


@needs_ref
@pytest.mark.parametrize("dim", [4, 16, 33, 128])
def test_fused_dot_matches_reference_build(dim):
    rng = np.random.default_rng(dim)
    k = rng.integers(-127, 128, (9, dim)).astype(np.int8)
    s = rng.random(9).astype(np.float32)
    q = rng.standard_normal(dim).astype(np.float32)
    assert np.array_equal(bits(O.fused_dequant_dot_int8(q, k, s, dim, 9)),
                          bits(O.ref_fused_dequant_dot_int8(q, k, s, dim, 9)))


@needs_ref
def test_kvcache_append_matches_reference_build():
    hkv, d, n = 4, 128, 7
    rng = np.random.default_rng(9)
    k = W.kv_rows(rng, n, hkv, d)
    v = W.kv_rows(rng, n, hkv, d)
    c = O.RefKVCache(hkv, d, 1, 8, quant=True)
    for t in range(n):
        c.append(0, k[t], v[t])
    kq, vq, ks, vs = c.layer_arrays(0)
    mk, mks = O.quantize_kv(k, hkv, d, O.SCALE_ROW)
    assert np.array_equal(kq[:n], mk) and np.array_equal(bits(ks[:n]), bits(mks))
    assert c.seq_len() == n
    c.reset()
    assert c.seq_len() == 0


@needs_ref
@pytest.mark.parametrize("L,H", [(1, 16), (2, 16), (129, 16), (700, 16), (50, 8), (50, 4)])
def test_decode_attention_matches_reference_build(L, H):
    hkv, d = 4, 128
    rng = np.random.default_rng(L * 7 + H)
    kq, ks = O.quantize_kv(W.kv_rows(rng, L, hkv, d), hkv, d)
    vq, vs = O.quantize_kv(W.kv_rows(rng, L, hkv, d), hkv, d)
    q = W.queries(rng, 1, H, d)[0]
    r = O.RefAttention(H, hkv, d, L + 1)
    want = r.run(kq, vq, ks, vs, L, q)
    r.close()
    got = O.decode_attention(kq, vq, ks, vs, L, q, H, hkv, d, W.softmax_scale(d))
    assert np.array_equal(bits(got), bits(want))


@needs_ref
@pytest.mark.parametrize("L,H", [(1, 16), (700, 16), (4096, 16), (50, 8)])
def test_reference_attention_without_projections_is_the_same_loop(L, H):
    """The reference arm of the bench times InferenceEngine::attention through
    the reference's own weight-absent branch (no Q/K/V/O matvecs).  Step after
    step over the same loaded cache it gives the restatement's output bit for
    bit, as the identity-projection path does."""
    hkv, d = 4, 128
    rng = np.random.default_rng(L + 3 * H)
    kq, ks = O.quantize_kv(W.kv_rows(rng, L, hkv, d), hkv, d)
    vq, vs = O.quantize_kv(W.kv_rows(rng, L, hkv, d), hkv, d)
    r = O.RefAttention(H, hkv, d, L + 1, projections=False)
    r.load(kq, vq, ks, vs, L)
    for _ in range(3):
        q = W.queries(rng, 1, H, d)[0]
        got = r.step(q).reshape(H, d)
        want = O.decode_attention(kq, vq, ks, vs, L, q, H, hkv, d, W.softmax_scale(d))
        assert np.array_equal(bits(got), bits(want))
    r.close()


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_decode_attention_f32_matches_golden(golden, tag):
    """FP32 cache mode (src/inference.cpp:346-358, 386-393): the restatement
    reproduces the reference's bytes."""
    g = golden("attention_f32.npz")
    H, hkv, L = (int(x) for x in g[f"{tag}_shape"])
    out = O.decode_attention_f32(g[f"{tag}_keys"], g[f"{tag}_values"], L, g[f"{tag}_q"], H, hkv,
                                 128, W.softmax_scale(128))
    assert np.array_equal(bits(out), bits(g[f"{tag}_out"]))


@needs_ref
@pytest.mark.parametrize("L,H,hkv", [(1, 16, 4), (77, 16, 4), (300, 8, 8), (40, 32, 4)])
def test_decode_attention_f32_matches_reference_build(L, H, hkv):
    rng = np.random.default_rng(L + H + hkv)
    k = W.kv_rows(rng, L, hkv, 128)
    v = W.kv_rows(rng, L, hkv, 128)
    q = W.queries(rng, 1, H, 128)[0]
    r = O.RefAttentionF32(H, hkv, 128, L + 1)
    want = r.run(k, v, L, q)
    r.close()
    got = O.decode_attention_f32(k, v, L, q, H, hkv, 128, W.softmax_scale(128))
    assert np.array_equal(bits(got), bits(want))
