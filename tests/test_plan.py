"""The split-K plan, read through the workspace size the library asks for
(ec_decode_workspace_size_batch is host arithmetic: no GPU needed, and with
no device the library plans for the B200's 148 SMs).

* 32 to 1024 sequences, ragged or not, take the stream-K grid: one wave of
  the resident slots (148 SMs x 2 CTAs for 4 KV heads at head_dim 128), a
  partial row per (CTA, sequence) piece and the tile prefix;
* fewer than 32 or more than 1024 sequences take the chunked grid: a
  partial row per (sequence, chunk).
"""
from __future__ import annotations

import ctypes

import pytest

import eckv
import workloads as W

H, HKV, D = 16, 4, 128


def _ws(lens, num_heads=H, hkv=HKV, head_dim=D, hint=None):
    n = len(lens)
    fake = 0x1000                      # never dereferenced: planning reads sizes only
    d = eckv.KVBatch(keys=fake, values=fake, key_scales=fake, val_scales=fake, seq_offset=fake,
                     seq_capacity=fake, seq_len=fake, error_word=fake,
                     total_slots=sum(lens), num_seqs=n, num_kv_heads=hkv, head_dim=head_dim,
                     scale_mode=0, max_seq_len=max(lens),
                     total_tokens_hint=sum(lens) if hint is None else hint)
    return eckv.lib().ec_decode_workspace_size_batch(ctypes.byref(d), num_heads)


def _stream_bytes(ctas, n, num_heads=H, head_dim=D):
    return (ctas + n) * num_heads * (head_dim + 2) * 4 + ((n + 1) * 4 + 15) // 16 * 16


@pytest.mark.parametrize("n", [32, 128, 1024])
def test_uniform_batches_take_stream_k(n):
    assert _ws([32768] * n) == _stream_bytes(296, n)


def test_ragged_config2_batch_takes_stream_k():
    lens = W.config(2).ctx
    assert _ws(lens) == _stream_bytes(296, len(lens))


def test_stream_k_grid_shrinks_to_the_tile_count():
    # 40 sequences of 32 tokens: 40 tiles, so 40 CTAs
    assert _ws([32] * 40) == _stream_bytes(40, 40)


@pytest.mark.parametrize("n", [1, 16, 31, 1025])
def test_other_batch_sizes_take_the_chunked_grid(n):
    ws = _ws([32768] * n)
    row = n * H * (D + 2) * 4
    assert ws % row == 0
    chunks = ws // row
    assert 2 <= chunks <= 1024


def test_single_long_sequence_fills_the_resident_slots():
    # one 1M-token sequence: about one chunk per resident slot (296)
    chunks = _ws([1 << 20]) // (H * (D + 2) * 4)
    assert 256 <= chunks <= 296


def test_head_dim_256_stream_k_rows():
    n = 64
    ws = _ws([8192] * n, head_dim=256)
    prefix = ((n + 1) * 4 + 15) // 16 * 16
    rows = (ws - prefix) // (H * 258 * 4)
    assert (ws - prefix) % (H * 258 * 4) == 0
    assert n < rows <= n + 1024
