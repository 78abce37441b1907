"""ctypes front end of the CPU checkers (TEST INFRASTRUCTURE ONLY).

Loads ``liboracle.so`` (the C restatement in ec_oracle.c) and, when it has
been built, ``_ref/libecref.so`` (the reference's own compiled sources behind
ref_shim.cpp).  Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` import this module.  The shipped library never does.

All arrays are numpy, C-contiguous, float32 / int8.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libecref.so")

SCALE_PER_HEAD = 0
SCALE_ROW = 1

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u32 = ctypes.c_uint32


def _p(a: np.ndarray, ty):
    return a.ctypes.data_as(ty)


def build_oracle() -> None:
    """Compile liboracle.so if it is missing (gcc only, a second or two)."""
    if not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        build_oracle()
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_quantize_per_token_symmetric.argtypes = [_f32p, _i8p, _f32p, _u32, _u32]
        L.oracle_fused_dequant_dot_int8.argtypes = [_f32p, _i8p, _f32p, _f32p, _u32, _u32]
        L.oracle_kv_append_token.argtypes = [_i8p, _i8p, _f32p, _f32p, _u32, _f32p, _f32p, _u32,
                                             _u32, ctypes.c_int]
        L.oracle_decode_attention.argtypes = [_i8p, _i8p, _f32p, _f32p, _u32, _f32p, _f32p, _u32,
                                              _u32, _u32, ctypes.c_float, ctypes.c_int, _f32p]
        L.oracle_decode_attention_f32.argtypes = [_f32p, _f32p, _u32, _f32p, _f32p, _u32, _u32,
                                                  _u32, ctypes.c_float, _f32p]
        L.oracle_norm_rope.argtypes = [_f32p, _u32, _u32, _u32, _f32p, ctypes.c_float]
        L.oracle_prefill_attention.argtypes = [_i8p, _i8p, _f32p, _f32p, _u32, _u32, _f32p, _f32p,
                                               _u32, _u32, _u32, ctypes.c_float, ctypes.c_int, _f32p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own code (oracle/_ref).  Raises if it was not built."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_SO} not built (make -C oracle REF=<reference checkout>)")
        L = ctypes.CDLL(REF_SO)
        vp = ctypes.c_void_p
        L.ref_quantize_per_token_symmetric.argtypes = [_f32p, _i8p, _f32p, _u32, _u32]
        L.ref_fused_dequant_dot_int8.argtypes = [_f32p, _i8p, _f32p, _f32p, _u32, _u32]
        L.ref_kvcache_create.argtypes = [_u32, _u32, _u32, _u32, ctypes.c_int]
        L.ref_kvcache_create.restype = vp
        L.ref_kvcache_destroy.argtypes = [vp]
        L.ref_kvcache_append.argtypes = [vp, _u32, _f32p, _f32p]
        L.ref_kvcache_seq_len.argtypes = [vp]
        L.ref_kvcache_seq_len.restype = _u32
        L.ref_kvcache_layer_seq_len.argtypes = [vp, _u32]
        L.ref_kvcache_layer_seq_len.restype = _u32
        L.ref_kvcache_reset.argtypes = [vp]
        L.ref_kvcache_layer_ptrs.argtypes = [vp, _u32, ctypes.POINTER(vp)]
        L.ref_attn_create.argtypes = [_u32, _u32, _u32, _u32]
        L.ref_attn_create.restype = vp
        L.ref_attn_destroy.argtypes = [vp]
        L.ref_attn_run.argtypes = [vp, _u32, _i8p, _i8p, _f32p, _f32p, _f32p, _f32p]
        L.ref_attn_run.restype = ctypes.c_int
        L.ref_attn_load.argtypes = [vp, _u32, _i8p, _i8p, _f32p, _f32p]
        L.ref_attn_load.restype = ctypes.c_int
        L.ref_attn_step.argtypes = [vp, _u32, _f32p, _f32p]
        L.ref_attn_step.restype = ctypes.c_int
        L.ref_attn_create_noproj.argtypes = [_u32, _u32, _u32, _u32]
        L.ref_attn_create_noproj.restype = vp
        L.ref_attn_step_noproj.argtypes = [vp, _u32, _f32p, _f32p]
        L.ref_attn_step_noproj.restype = ctypes.c_int
        L.ref_attn_f32_create.argtypes = [_u32, _u32, _u32, _u32]
        L.ref_attn_f32_create.restype = vp
        L.ref_attn_f32_run.argtypes = [vp, _u32, _f32p, _f32p, _f32p, _f32p]
        L.ref_attn_f32_run.restype = ctypes.c_int
        _ref = L
    return _ref


# ---------------------------------------------------------------- restatement
def quantize_per_token_symmetric(x: np.ndarray, num_tokens: int, num_elements: int):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size == num_tokens * num_elements
    q = np.zeros(x.size, np.int8)
    s = np.zeros(num_tokens, np.float32)
    lib().oracle_quantize_per_token_symmetric(_p(x, _f32p), _p(q, _i8p), _p(s, _f32p),
                                              num_tokens, num_elements)
    return q, s


def fused_dequant_dot_int8(query, key_cache, scales, dim, seq_len):
    query = np.ascontiguousarray(query, np.float32)
    key_cache = np.ascontiguousarray(key_cache, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    out = np.zeros(seq_len, np.float32)
    lib().oracle_fused_dequant_dot_int8(_p(query, _f32p), _p(key_cache, _i8p), _p(scales, _f32p),
                                        _p(out, _f32p), dim, seq_len)
    return out


def quantize_kv(x: np.ndarray, num_kv_heads: int, head_dim: int, mode: int = SCALE_PER_HEAD):
    """Quantize a [tokens, num_kv_heads*head_dim] block the way KVCache::append
    does one token at a time.  Returns (codes [tokens, Hkv*d] int8, scales
    [tokens, Hkv] (PER_HEAD) or [tokens] (ROW))."""
    x = np.ascontiguousarray(x, np.float32)
    ntok = x.shape[0]
    if mode == SCALE_ROW:
        q, s = quantize_per_token_symmetric(x, ntok, num_kv_heads * head_dim)
        return q.reshape(ntok, -1), s
    q, s = quantize_per_token_symmetric(x, ntok * num_kv_heads, head_dim)
    return q.reshape(ntok, -1), s.reshape(ntok, num_kv_heads)


def decode_attention(keys, values, kscales, vscales, kv_len, q, num_heads, num_kv_heads,
                     head_dim, softmax_scale, mode=SCALE_PER_HEAD):
    keys = np.ascontiguousarray(keys, np.int8)
    values = np.ascontiguousarray(values, np.int8)
    kscales = np.ascontiguousarray(kscales, np.float32)
    vscales = np.ascontiguousarray(vscales, np.float32)
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    out = np.zeros(num_heads * head_dim, np.float32)
    scratch = np.zeros(max(kv_len, 1), np.float32)
    lib().oracle_decode_attention(_p(keys, _i8p), _p(values, _i8p), _p(kscales, _f32p),
                                  _p(vscales, _f32p), kv_len, _p(q, _f32p), _p(out, _f32p),
                                  num_heads, num_kv_heads, head_dim, ctypes.c_float(softmax_scale),
                                  mode, _p(scratch, _f32p))
    return out.reshape(num_heads, head_dim)


def decode_attention_f32(keys, values, kv_len, q, num_heads, num_kv_heads, head_dim,
                         softmax_scale):
    """FP32 cache mode (use_kv_quantization = false) of the decode loop:
    keys / values [kv_len, num_kv_heads*head_dim] fp32."""
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    out = np.zeros(num_heads * head_dim, np.float32)
    scratch = np.zeros(max(kv_len, 1), np.float32)
    lib().oracle_decode_attention_f32(_p(keys, _f32p), _p(values, _f32p), kv_len, _p(q, _f32p),
                                      _p(out, _f32p), num_heads, num_kv_heads, head_dim,
                                      ctypes.c_float(softmax_scale), _p(scratch, _f32p))
    return out.reshape(num_heads, head_dim)


def norm_rope(x, pos, rope_base=10000.0, norm_w=None):
    """echo-core-zig's per-head RMS norm (fp32 values of the fp16 weight, or
    None) then RoPE at position pos, on x [num_heads, 128]; returns a copy."""
    x = np.array(x, np.float32, copy=True, order="C")
    H, d = x.shape
    w = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
    lib().oracle_norm_rope(_p(x, _f32p), H, d, pos, _p(w, _f32p) if w is not None else None,
                           ctypes.c_float(rope_base))
    return x


def prefill_attention(keys, values, kscales, vscales, past_len, n_new, q, num_heads,
                      num_kv_heads, head_dim, softmax_scale, mode=SCALE_PER_HEAD):
    keys = np.ascontiguousarray(keys, np.int8)
    values = np.ascontiguousarray(values, np.int8)
    kscales = np.ascontiguousarray(kscales, np.float32)
    vscales = np.ascontiguousarray(vscales, np.float32)
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    out = np.zeros(n_new * num_heads * head_dim, np.float32)
    scratch = np.zeros(past_len + n_new, np.float32)
    lib().oracle_prefill_attention(_p(keys, _i8p), _p(values, _i8p), _p(kscales, _f32p),
                                   _p(vscales, _f32p), past_len, n_new, _p(q, _f32p),
                                   _p(out, _f32p), num_heads, num_kv_heads, head_dim,
                                   ctypes.c_float(softmax_scale), mode, _p(scratch, _f32p))
    return out.reshape(n_new, num_heads, head_dim)



def decode_partial(keys, values, kscales, vscales, q, num_heads, num_kv_heads, head_dim,
                   softmax_scale, mode=SCALE_PER_HEAD):
    """Unnormalised partial decode state of one sequence slice, in float64:
    per query head h, m = max_t s_t*log2(e), l = sum_t 2^(s_t*log2(e) - m),
    o = sum_t 2^(s_t*log2(e) - m) * v_t, with s_t = softmax_scale * q_h . k_t
    over the dequantised codes (query head h reads KV head h % num_kv_heads,
    src/inference.cpp:335).  An empty slice gives m = -inf, l = 0, o = 0.
    Restates the state ec_decode_attention_partial exchanges between ranks;
    the reference itself has no such state (it keeps one sequence on one
    device)."""
    keys = np.asarray(keys, np.int8).reshape(-1, num_kv_heads, head_dim).astype(np.float64)
    values = np.asarray(values, np.int8).reshape(-1, num_kv_heads, head_dim).astype(np.float64)
    n = keys.shape[0]
    if mode == SCALE_ROW:
        ks = np.repeat(np.asarray(kscales, np.float64).reshape(n, 1), num_kv_heads, 1)
        vs = np.repeat(np.asarray(vscales, np.float64).reshape(n, 1), num_kv_heads, 1)
    else:
        ks = np.asarray(kscales, np.float64).reshape(n, num_kv_heads)
        vs = np.asarray(vscales, np.float64).reshape(n, num_kv_heads)
    q = np.asarray(q, np.float64).reshape(num_heads, head_dim)
    o = np.zeros((num_heads, head_dim))
    ml = np.zeros((num_heads, 2))
    for h in range(num_heads):
        g = h % num_kv_heads
        if n == 0:
            ml[h] = (-np.inf, 0.0)
            continue
        s = softmax_scale * (keys[:, g, :] @ q[h]) * ks[:, g] * np.log2(np.e)
        m = s.max()
        p = np.exp2(s - m)
        ml[h] = (m, p.sum())
        o[h] = (p * vs[:, g]) @ values[:, g, :]
    return o, ml


def lse_combine(part_o, part_ml):
    """Merges stacked partial states [parts][heads][dim], [parts][heads][2]
    (rank order) into the normalised output [heads][dim]."""
    part_o = np.asarray(part_o, np.float64)
    part_ml = np.asarray(part_ml, np.float64)
    m = part_ml[..., 0].max(axis=0)
    w = np.where(np.isfinite(part_ml[..., 0]), np.exp2(part_ml[..., 0] - m), 0.0)
    l = (part_ml[..., 1] * w).sum(axis=0)
    o = (part_o * w[..., None]).sum(axis=0)
    return o / l[:, None]

# -------------------------------------------------------- the reference itself
def ref_quantize_per_token_symmetric(x, num_tokens, num_elements):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    q = np.zeros(x.size, np.int8)
    s = np.zeros(num_tokens, np.float32)
    ref().ref_quantize_per_token_symmetric(_p(x, _f32p), _p(q, _i8p), _p(s, _f32p),
                                           num_tokens, num_elements)
    return q, s


def ref_fused_dequant_dot_int8(query, key_cache, scales, dim, seq_len):
    query = np.ascontiguousarray(query, np.float32)
    key_cache = np.ascontiguousarray(key_cache, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    out = np.zeros(seq_len, np.float32)
    ref().ref_fused_dequant_dot_int8(_p(query, _f32p), _p(key_cache, _i8p), _p(scales, _f32p),
                                     _p(out, _f32p), dim, seq_len)
    return out


class RefKVCache:
    """The reference's KVCache (src/kv_cache.cpp), host memory."""

    def __init__(self, num_kv_heads, head_dim, num_layers, max_seq_len, quant=True):
        self.h = ref().ref_kvcache_create(num_kv_heads, head_dim, num_layers, max_seq_len,
                                          int(quant))
        self.hkv, self.d, self.max_seq = num_kv_heads, head_dim, max_seq_len
        self.quant = quant

    def close(self):
        if self.h:
            ref().ref_kvcache_destroy(self.h)
            self.h = None

    __del__ = close

    def append(self, layer, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        ref().ref_kvcache_append(self.h, layer, _p(k, _f32p), _p(v, _f32p))

    def seq_len(self):
        return ref().ref_kvcache_seq_len(self.h)

    def layer_seq_len(self, layer):
        return ref().ref_kvcache_layer_seq_len(self.h, layer)

    def reset(self):
        ref().ref_kvcache_reset(self.h)

    def layer_arrays(self, layer):
        """Copies of the layer's int8 codes [max_seq, Hkv*d] and both scale
        buffers [max_seq*Hkv] (int8 mode), or fp32 K/V (fp32 mode)."""
        ptrs = (ctypes.c_void_p * 6)()
        ref().ref_kvcache_layer_ptrs(self.h, layer, ptrs)
        row = self.hkv * self.d
        n = self.max_seq
        if self.quant:
            k = np.ctypeslib.as_array(ctypes.cast(ptrs[0], _i8p), (n * row,)).copy()
            v = np.ctypeslib.as_array(ctypes.cast(ptrs[1], _i8p), (n * row,)).copy()
            ks = np.ctypeslib.as_array(ctypes.cast(ptrs[2], _f32p), (n * self.hkv,)).copy()
            vs = np.ctypeslib.as_array(ctypes.cast(ptrs[3], _f32p), (n * self.hkv,)).copy()
            return k.reshape(n, row), v.reshape(n, row), ks, vs
        k = np.ctypeslib.as_array(ctypes.cast(ptrs[4], _f32p), (n * row,)).copy()
        v = np.ctypeslib.as_array(ctypes.cast(ptrs[5], _f32p), (n * row,)).copy()
        return k.reshape(n, row), v.reshape(n, row)


class RefAttentionF32:
    """The reference's attention loop in its FP32 cache mode
    (src/inference.cpp:346-358, 386-393)."""

    def __init__(self, num_heads, num_kv_heads, head_dim, max_seq_len):
        self.h = ref().ref_attn_f32_create(num_heads, num_kv_heads, head_dim, max_seq_len)
        self.H, self.d = num_heads, head_dim

    def close(self):
        if self.h:
            ref().ref_attn_destroy(self.h)
            self.h = None

    __del__ = close

    def run(self, keys, values, kv_len, q):
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        out = np.zeros(self.H * self.d, np.float32)
        if ref().ref_attn_f32_run(self.h, kv_len, _p(keys, _f32p), _p(values, _f32p),
                                  _p(q, _f32p), _p(out, _f32p)) != 0:
            raise ValueError("kv_len must be below the engine's max_seq_len")
        return out.reshape(self.H, self.d)


class RefAttention:
    """The reference's InferenceEngine::attention loop (src/inference.cpp:321-406).

    projections=True runs it as the reference does, with fp16 identity Q and O
    weight matvecs around the loop (:313-319, :410-411); projections=False
    takes the reference's weight-absent branch, so step() times the attention
    loop and the append alone (run() needs the projections)."""

    def __init__(self, num_heads, num_kv_heads, head_dim, max_seq_len, projections=True):
        create = ref().ref_attn_create if projections else ref().ref_attn_create_noproj
        self.h = create(num_heads, num_kv_heads, head_dim, max_seq_len)
        self.projections = projections
        self.H, self.hkv, self.d = num_heads, num_kv_heads, head_dim

    def close(self):
        if self.h:
            ref().ref_attn_destroy(self.h)
            self.h = None

    __del__ = close

    def run(self, keys, values, kscales, vscales, kv_len, q):
        keys = np.ascontiguousarray(keys, np.int8)
        values = np.ascontiguousarray(values, np.int8)
        kscales = np.ascontiguousarray(kscales, np.float32)
        vscales = np.ascontiguousarray(vscales, np.float32)
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        out = np.zeros(self.H * self.d, np.float32)
        rc = ref().ref_attn_run(self.h, kv_len, _p(keys, _i8p), _p(values, _i8p),
                                _p(kscales, _f32p), _p(vscales, _f32p), _p(q, _f32p),
                                _p(out, _f32p))
        if rc != 0:
            raise ValueError("kv_len must be below the engine's max_seq_len")
        return out.reshape(self.H, self.d)

    def load(self, keys, values, kscales, vscales, kv_len):
        """Copies a cache in once; step() then attends to it repeatedly."""
        self._keep = [np.ascontiguousarray(keys, np.int8), np.ascontiguousarray(values, np.int8),
                      np.ascontiguousarray(kscales, np.float32),
                      np.ascontiguousarray(vscales, np.float32)]
        k, v, ks, vs = self._keep
        if ref().ref_attn_load(self.h, kv_len, _p(k, _i8p), _p(v, _i8p), _p(ks, _f32p),
                               _p(vs, _f32p)) != 0:
            raise ValueError("kv_len must be below the engine's max_seq_len")
        self.kv_len = kv_len

    def step(self, q, out=None):
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        if out is None:
            out = np.zeros(self.H * self.d, np.float32)
        fn = ref().ref_attn_step if self.projections else ref().ref_attn_step_noproj
        fn(self.h, self.kv_len, _p(q, _f32p), _p(out, _f32p))
        return out
