"""Helpers shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np

ATOL = 2e-3   # attention output tolerance against the oracle's fp32 output:
RTOL = 1e-3   # |gpu - oracle| <= ATOL + RTOL*|oracle| and max|gpu - oracle| <= ATOL


def assert_attn_close(got, want, what=""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    diff = np.abs(got - want)
    mx = float(diff.max()) if diff.size else 0.0
    ok = diff <= ATOL + RTOL * np.abs(want)
    assert mx <= ATOL and ok.all(), (
        f"{what}: max abs err {mx:.3e}, worst rel "
        f"{float((diff / np.maximum(np.abs(want), 1e-6)).max()):.3e}")
    return mx


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def fill_batch(bc, seqs):
    """Writes per-sequence (keys [L,row] int8, values, kscales, vscales) into
    a BatchCache's slabs and sets the length table."""
    import torch
    lens = []
    for s, (k, v, ks, vs) in enumerate(seqs):
        off = int(bc.offsets_host[s])
        L = k.shape[0]
        ns = ks.size // max(L, 1) if L else 0
        if L:
            bc.keys[off:off + L] = torch.from_numpy(np.ascontiguousarray(k)).to(bc.keys.device)
            bc.values[off:off + L] = torch.from_numpy(np.ascontiguousarray(v)).to(bc.keys.device)
            bc.key_scales[off * ns:(off + L) * ns] = torch.from_numpy(ks.reshape(-1)).to(bc.keys.device)
            bc.val_scales[off * ns:(off + L) * ns] = torch.from_numpy(vs.reshape(-1)).to(bc.keys.device)
        lens.append(L)
    bc.length.copy_(torch.tensor(lens, dtype=torch.int32))
    torch.cuda.synchronize()


def d2h(ptr: int, shape, dtype):
    """Copies device memory at a raw pointer (e.g. a KVCacheLayer field) to a
    new numpy array."""
    from cuda.bindings import runtime as rt
    out = np.empty(shape, dtype)
    (err,) = rt.cudaMemcpy(out.ctypes.data, int(ptr), out.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess, err
    return out


def h2d(ptr: int, arr):
    from cuda.bindings import runtime as rt
    arr = np.ascontiguousarray(arr)
    (err,) = rt.cudaMemcpy(int(ptr), arr.ctypes.data, arr.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert err == rt.cudaError_t.cudaSuccess, err
