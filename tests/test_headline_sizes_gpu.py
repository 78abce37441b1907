"""Parity at the BASELINE configs' own sizes, every sequence against the oracle.

The other GPU tests exercise the kernels at reduced sizes; these run the
shapes the bench measures:

* config 3: one layer of 128 sequences x 32,768 cached tokens, built with the
  bench's own capacities, grid bound and token hint (so the same split-K
  plan), one token appended per sequence by ec_kv_batch_append, then decode;
  every sequence is compared with the oracle's decode loop
  (src/inference.cpp:321-392) over the same codes plus the appended token;
* config 4: one 1,048,576-token sequence, decoded whole by
  ec_decode_attention and as 8 contiguous context shards through
  ec_decode_attention_partial + ec_lse_combine (what 8 ranks compute);
* config 5: all 32 sequences (8192 cached + 4096 appended tokens), each with
  a sample of query rows checked against the decode loop over that row's
  causal prefix, with bf16-cast queries.

Tolerance: max-abs 2e-3 and |err| <= 2e-3 + 1e-3 |ref| (tests/_util.py).
The K/V codes come from the oracle's quantizer (bit-exact with the
reference's, tests/test_oracle.py); the tokens appended on the GPU are
checked byte for byte against the oracle's codes.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O
import workloads as W
from _util import assert_attn_close

pytestmark = pytest.mark.gpu

D, H, HKV = 128, 16, 4


def _quantized(rng, n):
    kq, ks = O.quantize_kv(W.kv_rows(rng, n, HKV, D), HKV, D)
    vq, vs = O.quantize_kv(W.kv_rows(rng, n, HKV, D), HKV, D)
    return kq, vq, ks, vs


def _upload(torch, bc, off, kq, vq, ks, vs):
    n = kq.shape[0]
    bc.keys[off:off + n].copy_(torch.from_numpy(kq), non_blocking=False)
    bc.values[off:off + n].copy_(torch.from_numpy(vq), non_blocking=False)
    bc.key_scales[off * HKV:(off + n) * HKV].copy_(torch.from_numpy(ks.reshape(-1)))
    bc.val_scales[off * HKV:(off + n) * HKV].copy_(torch.from_numpy(vs.reshape(-1)))


def _plan_chunks(eckv, bc, num_heads=H):
    d = bc.desc()
    ws = eckv.lib().ec_decode_workspace_size_batch(ctypes.byref(d), num_heads)
    return ws // (bc.num_seqs * num_heads * (D + 2) * 4) if ws else 1


def test_config3_one_layer_128x32k_bench_plan(cuda):
    """Config 3 at size (seed 2): 128 x 32,768 tokens, the bench's plan."""
    import torch
    import eckv
    cfg = W.config(3)
    lens = cfg.ctx
    caps, max_len, hint = W.decode_bench_batch(lens)
    bc = eckv.BatchCache(caps, num_kv_heads=HKV, max_seq_len=max_len)
    bc.tokens_hint = hint
    nchunks = _plan_chunks(eckv, bc)
    assert nchunks > 1, "the bench's plan splits every sequence"
    rng = np.random.default_rng(cfg.seed)
    q = W.queries(rng, len(lens), H, D)
    k_new = W.kv_rows(rng, len(lens), HKV, D)
    v_new = W.kv_rows(rng, len(lens), HKV, D)
    sc = W.softmax_scale(D)
    want = np.empty((len(lens), H, D), np.float32)
    new_codes = []
    for s, L in enumerate(lens):
        kq, vq, ks, vs = _quantized(rng, L)
        _upload(torch, bc, int(bc.offsets_host[s]), kq, vq, ks, vs)
        nk, nks = O.quantize_kv(k_new[s:s + 1], HKV, D)
        nv, nvs = O.quantize_kv(v_new[s:s + 1], HKV, D)
        new_codes.append((nk, nv, nks, nvs))
        want[s] = O.decode_attention(np.concatenate([kq, nk]), np.concatenate([vq, nv]),
                                     np.concatenate([ks, nks]), np.concatenate([vs, nvs]),
                                     L + 1, q[s], H, HKV, D, sc)
    bc.length.copy_(torch.tensor(lens, dtype=torch.int32))
    bc.append(torch.from_numpy(k_new).cuda(), torch.from_numpy(v_new).cuda(), 1)
    out = torch.empty((len(lens), H, D), device="cuda")
    bc.decode(torch.from_numpy(q).cuda(), out, H, sc)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    assert bc.length.cpu().tolist() == [L + 1 for L in lens]
    got = out.cpu().numpy()
    worst = 0.0
    for s, L in enumerate(lens):
        off = int(bc.offsets_host[s]) + L
        nk, nv, nks, nvs = new_codes[s]
        assert np.array_equal(bc.keys[off].cpu().numpy(), nk[0]), f"appended K codes, seq {s}"
        assert np.array_equal(bc.values[off].cpu().numpy(), nv[0]), f"appended V codes, seq {s}"
        worst = max(worst, assert_attn_close(got[s], want[s], f"cfg3 seq {s} ({nchunks} chunks)"))
    print(f"config 3 at size: {len(lens)} sequences, {nchunks}-chunk plan, max-abs err {worst:.2e}")


def test_config4_one_sequence_1m_whole_and_8_shards(cuda):
    """Config 4 at size (seed 3): one 1,048,576-token sequence, decoded whole
    and as 8 contiguous shards merged by the log-sum-exp combine."""
    import torch
    import eckv
    cfg = W.config(4)
    L = cfg.ctx[0]
    rng = np.random.default_rng(cfg.seed)
    bc = eckv.BatchCache([L], num_kv_heads=HKV)
    K = np.empty((L, HKV * D), np.int8)
    V = np.empty((L, HKV * D), np.int8)
    KS = np.empty((L, HKV), np.float32)
    VS = np.empty((L, HKV), np.float32)
    step = 1 << 16
    for t in range(0, L, step):
        kq, vq, ks, vs = _quantized(rng, step)
        K[t:t + step], V[t:t + step], KS[t:t + step], VS[t:t + step] = kq, vq, ks, vs
        _upload(torch, bc, t, kq, vq, ks, vs)
    bc.length.copy_(torch.tensor([L], dtype=torch.int32))
    q = W.queries(rng, 1, H, D)
    sc = W.softmax_scale(D)
    want = O.decode_attention(K, V, KS, VS, L, q[0], H, HKV, D, sc)
    qd = torch.from_numpy(q).cuda()

    out = torch.empty((1, H, D), device="cuda")
    bc.decode(qd, out, H, sc)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    err_whole = assert_attn_close(out.cpu().numpy()[0], want, "cfg4 whole")

    # 8 shards of the same slab: one batch entry per shard (offset lo, length
    # hi - lo), each entry decoded to its partial state as one rank would
    parts = 8
    bounds = [L * r // parts for r in range(parts + 1)]
    offs = torch.tensor(bounds[:-1], dtype=torch.int32, device="cuda")
    lens = torch.tensor([bounds[r + 1] - bounds[r] for r in range(parts)], dtype=torch.int32,
                        device="cuda")
    d = eckv.KVBatch(keys=bc.keys.data_ptr(), values=bc.values.data_ptr(),
                     key_scales=bc.key_scales.data_ptr(), val_scales=bc.val_scales.data_ptr(),
                     seq_offset=offs.data_ptr(), seq_capacity=lens.data_ptr(),
                     seq_len=lens.data_ptr(), error_word=bc.err.data_ptr(),
                     total_slots=bc.total_slots, num_seqs=parts, num_kv_heads=HKV, head_dim=D,
                     scale_mode=0, max_seq_len=L // parts)
    ws_bytes = eckv.lib().ec_decode_workspace_size_batch(ctypes.byref(d), H)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    qrep = qd.expand(parts, H, D).contiguous()
    po = torch.empty((parts, 1, H, D), device="cuda")
    pml = torch.empty((parts, 1, H, 2), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    eckv.check(eckv.lib().ec_decode_attention_partial(
        ctypes.byref(d), ctypes.c_void_p(qrep.data_ptr()), ctypes.c_void_p(po.data_ptr()),
        ctypes.c_void_p(pml.data_ptr()), H, ctypes.c_float(sc), ctypes.c_void_p(ws.data_ptr()),
        ws.numel(), stream))
    out8 = torch.empty((1, H, D), device="cuda")
    eckv.lse_combine(po, pml, parts, 1, H, D, out8)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    err_shards = assert_attn_close(out8.cpu().numpy()[0], want, "cfg4 8 shards")
    print(f"config 4 at size: max-abs err {err_whole:.2e} whole, {err_shards:.2e} over 8 shards")


def test_config5_all_32_sequences_row_sample(cuda):
    """Config 5 at size (seed 4): 32 sequences append a 4096-token chunk
    (quantize-on-append on the GPU) onto 8192 cached tokens, then chunked
    prefill; 8 query rows of every sequence checked, block edges included."""
    import torch
    import eckv
    cfg = W.config(5)
    past, n_new, nseq = cfg.ctx[0], cfg.new_tokens, cfg.num_seqs
    rng = np.random.default_rng(cfg.seed)
    bc = eckv.BatchCache([past + n_new] * nseq, num_kv_heads=HKV)
    q = W.queries(rng, nseq * n_new, H, D).reshape(nseq, n_new, H, D)
    qb = torch.from_numpy(q).bfloat16().float().numpy()
    sc = W.softmax_scale(D)
    out = torch.empty((nseq, n_new, H, D), device="cuda")
    checks = []
    kn_all = np.empty((nseq, n_new, HKV * D), np.float32)
    vn_all = np.empty((nseq, n_new, HKV * D), np.float32)
    seqs = []
    for s in range(nseq):
        kq, vq, ks, vs = _quantized(rng, past)
        _upload(torch, bc, int(bc.offsets_host[s]), kq, vq, ks, vs)
        kn_all[s] = W.kv_rows(rng, n_new, HKV, D)
        vn_all[s] = W.kv_rows(rng, n_new, HKV, D)
        seqs.append((kq, vq, ks, vs))
    bc.length.copy_(torch.tensor([past] * nseq, dtype=torch.int32))
    bc.append(torch.from_numpy(kn_all).cuda(), torch.from_numpy(vn_all).cuda(), n_new)
    bc.prefill(torch.from_numpy(q).cuda(), out, n_new, H, sc)
    torch.cuda.synchronize()
    assert bc.device_error() == 0
    got = out.cpu().numpy()
    fixed = [0, 127, 128, 2047, 4095]
    worst = 0.0
    for s in range(nseq):
        kq, vq, ks, vs = seqs[s]
        nk, nks = O.quantize_kv(kn_all[s], HKV, D)
        nv, nvs = O.quantize_kv(vn_all[s], HKV, D)
        off = int(bc.offsets_host[s]) + past
        assert np.array_equal(bc.keys[off:off + n_new].cpu().numpy(), nk), f"K codes, seq {s}"
        assert np.array_equal(bc.values[off:off + n_new].cpu().numpy(), nv), f"V codes, seq {s}"
        K, V = np.concatenate([kq, nk]), np.concatenate([vq, nv])
        KS, VS = np.concatenate([ks, nks]), np.concatenate([vs, nvs])
        rows = fixed + [int(r) for r in rng.integers(0, n_new, 3)]
        for i in rows:
            want = O.decode_attention(K, V, KS, VS, past + i + 1, qb[s, i], H, HKV, D, sc)
            worst = max(worst, assert_attn_close(got[s, i], want, f"cfg5 seq {s} row {i}"))
    print(f"config 5 at size: {nseq} sequences x 8 rows, max-abs err {worst:.2e}")
