"""Seeded synthetic inputs for the INT8 KV-cache path.

The reference quotes no dataset for this path; every workload is synthetic:
fp32 K/V drawn N(0,1) with four fixed outlier channels per KV head scaled x8
(channels 0, 31, 64 and 127 of each 128-wide head), fp32 Q drawn N(0,1).
Generation is numpy ``default_rng(seed)``, so CPU checks and GPU runs see
the same bytes.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

OUTLIER_CHANNELS = (0, 31, 64, 127)
OUTLIER_FACTOR = 8.0


def kv_rows(rng: np.random.Generator, ntok: int, num_kv_heads: int, head_dim: int,
            outliers: bool = True) -> np.ndarray:
    """[ntok, num_kv_heads*head_dim] fp32 K or V projections."""
    x = rng.standard_normal((ntok, num_kv_heads, head_dim), dtype=np.float32)
    if outliers:
        ch = [c for c in OUTLIER_CHANNELS if c < head_dim]
        x[:, :, ch] *= np.float32(OUTLIER_FACTOR)
    return x.reshape(ntok, num_kv_heads * head_dim)


def queries(rng: np.random.Generator, n: int, num_heads: int, head_dim: int) -> np.ndarray:
    return rng.standard_normal((n, num_heads, head_dim), dtype=np.float32)


def softmax_scale(head_dim: int) -> float:
    """1/sqrt(head_dim) rounded to fp32 the way src/inference.cpp:322 computes it."""
    return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))


@dataclass
class Config:
    name: str
    num_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 128
    seed: int = 0
    num_layers: int = 1
    num_seqs: int = 1
    ctx: list = field(default_factory=list)     # per-sequence cached length before the step
    new_tokens: int = 1                         # tokens appended per sequence in the step


def config(idx: int) -> Config:
    """The five BASELINE configs (1-based index)."""
    if idx == 1:
        return Config("cfg1_single_decode_4k", seed=0, num_seqs=1, ctx=[4096], new_tokens=0)
    if idx == 2:
        rng = np.random.default_rng(1)
        ctx = rng.integers(512, 8192, size=64, endpoint=True).tolist()
        return Config("cfg2_ragged_batch64", seed=1, num_seqs=64, ctx=ctx, new_tokens=1)
    if idx == 3:
        return Config("cfg3_decode_8layers_128x32k", seed=2, num_layers=8, num_seqs=128,
                      ctx=[32768] * 128, new_tokens=1)
    if idx == 4:
        return Config("cfg4_long_context_1m", seed=3, num_seqs=1, ctx=[1048576], new_tokens=0)
    if idx == 5:
        return Config("cfg5_chunked_prefill_32x4k_on_8k", seed=4, num_seqs=32, ctx=[8192] * 32,
                      new_tokens=4096)
    raise ValueError(idx)


# bytes of one cached token of one layer: K and V codes plus their fp32 scales
def kv_bytes_per_token(num_kv_heads: int = 4, head_dim: int = 128) -> int:
    return 2 * num_kv_heads * head_dim + 2 * num_kv_heads * 4


def decode_bench_batch(lens, warmup: int = 3, steps: int = 20, new_tokens: int = 1):
    """Capacities, max_seq_len and split-K token hint of the per-layer batch the
    decode bench builds over cached lengths `lens` for `warmup` untimed and
    `steps` timed steps of `new_tokens` appended tokens each.  The parity test
    at the headline size builds its batch from the same numbers, so it runs the
    bench's own split-K plan."""
    cap_extra = (warmup + steps + 1) * new_tokens + 1
    caps = [int(L) + cap_extra for L in lens]
    max_seq_len = max(int(L) for L in lens) + cap_extra
    hint = int(sum(int(L) for L in lens)) + len(lens) * (warmup + 1 + steps // 2) * new_tokens
    return caps, max_seq_len, hint
