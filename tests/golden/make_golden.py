"""Regenerates the golden fixtures in this directory from the reference itself.

Runs echo-core's own compiled code (oracle/_ref/libecref.so, built by
``make -C oracle REF=<reference checkout>``) on seeded inputs and stores
inputs and outputs as compressed .npz files.  The parity tests then pin both
the C restatement (oracle/) and the CUDA kernels to these bytes without
needing the reference at test time.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "echo-core_b200"))

import oracle as O  # noqa: E402
import workloads as W  # noqa: E402


def quant_golden():
    """quantize_per_token_symmetric over row lengths that hit the 8-wide body,
    the scalar tail and both, plus an all-zero row, exact .5 ties and the
    reference's own Test 1 input (src/kernels/quant.cpp:405)."""
    rng = np.random.default_rng(100)
    cases = {}
    for n in (4, 7, 8, 9, 16, 31, 128, 133, 512):
        x = (rng.standard_normal((6, n)) * rng.uniform(0.1, 20, (6, 1))).astype(np.float32)
        x[2] = 0.0
        if n >= 8:
            x[3, : n // 2] = (np.arange(n // 2, dtype=np.float32) - n // 4) * 0.5
        q, s = O.ref_quantize_per_token_symmetric(x, x.shape[0], n)
        cases[f"x_{n}"] = x
        cases[f"q_{n}"] = q.reshape(x.shape)
        cases[f"s_{n}"] = s
    x = np.array([[1.0, 2.0, 3.0, 4.0]], np.float32)
    q, s = O.ref_quantize_per_token_symmetric(x, 1, 4)
    cases["x_test1"], cases["q_test1"], cases["s_test1"] = x, q.reshape(1, 4), s
    np.savez_compressed(os.path.join(HERE, "quantize.npz"), **cases)


def kvcache_golden():
    """KVCache::append in the reference's own int8 (ROW) and fp32 modes with
    the inputs of its self-test (src/kv_cache.cpp:134-172): 4 KV heads,
    head_dim 8, 5 tokens, k = t*10+i, v = t*100+i, layer 0."""
    hkv, d, n = 4, 8, 5
    k = np.array([[t * 10 + i for i in range(hkv * d)] for t in range(n)], np.float32)
    v = np.array([[t * 100 + i for i in range(hkv * d)] for t in range(n)], np.float32)
    c = O.RefKVCache(hkv, d, 2, 16, quant=True)
    for t in range(n):
        c.append(0, k[t], v[t])
    kq, vq, ks, vs = c.layer_arrays(0)
    np.savez_compressed(os.path.join(HERE, "kvcache_row.npz"), k=k, v=v, keys=kq[:n], values=vq[:n],
                        key_scales=ks[:n], val_scales=vs[:n], seq_len=np.array([c.seq_len()]))
    c.close()


def attention_golden():
    """InferenceEngine::attention (src/inference.cpp:321-406) run by the
    reference on per-head int8 caches built with its own quantizer."""
    H, hkv, d = 16, 4, 128
    out = {}
    for tag, L, seed in (("a", 1, 0), ("b", 37, 1), ("c", 300, 2)):
        rng = np.random.default_rng(200 + seed)
        kf = W.kv_rows(rng, L, hkv, d)
        vf = W.kv_rows(rng, L, hkv, d)
        kq, ks = O.quantize_kv(kf, hkv, d)
        vq, vs = O.quantize_kv(vf, hkv, d)
        q = W.queries(rng, 1, H, d)[0]
        r = O.RefAttention(H, hkv, d, L + 1)
        o = r.run(kq, vq, ks, vs, L, q)
        r.close()
        out.update({f"{tag}_keys": kq, f"{tag}_values": vq,
                    f"{tag}_kscales": ks, f"{tag}_vscales": vs, f"{tag}_q": q, f"{tag}_out": o,
                    f"{tag}_len": np.array([L])})
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)


def attention_f32_golden():
    """The same loop in its FP32 cache mode (use_kv_quantization = false,
    src/inference.cpp:346-358, 386-393), run by the reference."""
    out = {}
    for tag, H, hkv, L, seed in (("a", 16, 4, 1, 0), ("b", 16, 4, 23, 1), ("c", 8, 2, 9, 2)):
        rng = np.random.default_rng(300 + seed)
        k = W.kv_rows(rng, L, hkv, 128)
        v = W.kv_rows(rng, L, hkv, 128)
        q = W.queries(rng, 1, H, 128)[0]
        r = O.RefAttentionF32(H, hkv, 128, L + 1)
        o = r.run(k, v, L, q)
        r.close()
        out.update({f"{tag}_keys": k, f"{tag}_values": v, f"{tag}_q": q, f"{tag}_out": o,
                    f"{tag}_shape": np.array([H, hkv, L])})
    np.savez_compressed(os.path.join(HERE, "attention_f32.npz"), **out)


if __name__ == "__main__":
    if not O.ref_available():
        sys.exit("oracle/_ref/libecref.so is not built")
    quant_golden()
    kvcache_golden()
    attention_golden()
    attention_f32_golden()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
