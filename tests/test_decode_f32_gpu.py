"""Decode attention over the fp32 cache mode (use_kv_quantization = false) on
the GPU against the oracle restatement of src/inference.cpp:346-358, 386-393,
which is pinned to the reference build (tests/test_oracle.py).  Tokens enter
through the cache object's own append (src/kv_cache.cpp:106-110: fp32 copy)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close

pytestmark = pytest.mark.gpu
D = 128


def _run(torch, eckv, H, hkv, L, seed, max_seq=None):
    rng = np.random.default_rng(seed)
    k = W.kv_rows(rng, L, hkv, D)
    v = W.kv_rows(rng, L, hkv, D)
    q = W.queries(rng, 1, H, D)[0]
    c = eckv.KVCache(num_heads=H, num_kv_heads=hkv, head_dim=D, num_layers=2,
                     max_seq_len=max_seq or L + 1, use_kv_quantization=False)
    kd = torch.from_numpy(k).cuda()
    vd = torch.from_numpy(v).cuda()
    for t in range(L):
        c.append(1, kd[t], vd[t])
    out = torch.full((H, D), float("nan"), device="cuda")
    c.attention(1, torch.from_numpy(q).cuda(), out, W.softmax_scale(D))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    c.close()
    want = O.decode_attention_f32(k, v, L, q, H, hkv, D, W.softmax_scale(D))
    return got, want


@pytest.mark.parametrize("H,hkv", [(16, 4), (8, 8), (32, 4), (16, 2), (4, 4), (64, 8)])
def test_f32_cache_attention_groups(cuda, H, hkv):
    import torch
    import eckv
    got, want = _run(torch, eckv, H, hkv, 300, H * 10 + hkv)
    assert_attn_close(got, want, f"H{H} hkv{hkv}")


@pytest.mark.parametrize("L", [1, 2, 31, 32, 33, 127, 128, 129, 1000])
def test_f32_cache_attention_lengths(cuda, L):
    import torch
    import eckv
    got, want = _run(torch, eckv, 16, 4, L, L)
    assert_attn_close(got, want, f"L{L}")


def test_f32_cache_attention_long(cuda):
    """Many split-K chunks (20000 tokens: 157 chunks of 128)."""
    import torch
    import eckv
    got, want = _run(torch, eckv, 16, 4, 20000, 3)
    assert_attn_close(got, want, "L20000")


def test_f32_cache_empty_layer_gives_zeros(cuda):
    import torch
    import eckv
    c = eckv.KVCache(num_heads=16, num_kv_heads=4, head_dim=D, num_layers=1, max_seq_len=8,
                     use_kv_quantization=False)
    out = torch.full((16, D), 7.0, device="cuda")
    c.attention(0, torch.randn(16, D, device="cuda"), out, 0.1)
    torch.cuda.synchronize()
    assert not out.cpu().numpy().any()
    c.close()


def test_f32_golden_on_gpu(cuda, golden):
    """The reference's own fp32-mode outputs (tests/golden/attention_f32.npz)."""
    import torch
    import eckv
    g = golden("attention_f32.npz")
    for tag in "abc":
        H, hkv, L = (int(x) for x in g[f"{tag}_shape"])
        c = eckv.KVCache(num_heads=H, num_kv_heads=hkv, head_dim=D, num_layers=1,
                         max_seq_len=L + 1, use_kv_quantization=False)
        kd = torch.from_numpy(np.ascontiguousarray(g[f"{tag}_keys"])).cuda()
        vd = torch.from_numpy(np.ascontiguousarray(g[f"{tag}_values"])).cuda()
        for t in range(L):
            c.append(0, kd[t], vd[t])
        out = torch.empty((H, D), device="cuda")
        c.attention(0, torch.from_numpy(g[f"{tag}_q"]).cuda(), out, W.softmax_scale(D))
        torch.cuda.synchronize()
        assert_attn_close(out.cpu().numpy(), g[f"{tag}_out"], f"golden {tag}")
        c.close()
