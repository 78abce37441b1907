"""Host-side multi-rank plumbing of the INT8 KV-cache path (one process per GPU).

The reference serves one sequence in one process (src/main.cpp); it has no
multi-GPU path.  Two ways of spreading the path over ranks follow from its
data layout and need no new arithmetic:

* sequence sharding (decode, prefill): whole sequences are independent, so a
  batch is split into contiguous runs of sequences, one run per rank, with no
  data-path collective (``shard``);
* context parallelism (one long sequence): the sequence's cached tokens are
  split contiguously; every rank computes the unnormalised partial state
  (m, l, O) of its slice with ``ec_decode_attention_partial``, the states are
  all-gathered (``gather_partials``) and every rank merges them, in rank
  order, with ``ec_lse_combine``.  That all-gather is the only exchange.

Process groups come from ``torch.distributed`` (NCCL on GPUs, gloo for the
CPU tests of this module); nothing here computes attention.
"""
from __future__ import annotations


def shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) share of n units for `rank` of `world`.

    Shares differ by at most one unit, cover [0, n) exactly once and are in
    rank order, so rank r's slice of a sequence precedes rank r+1's (the order
    ``ec_lse_combine`` merges partial states in)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n < 0:
        raise ValueError(f"negative unit count {n}")
    return rank * n // world, (rank + 1) * n // world


def gather_partials(part_o, part_ml, group=None):
    """All-gathers this rank's partial decode state.

    part_o [num_seqs][num_heads][head_dim] and part_ml [num_seqs][num_heads][2]
    (the layout of ec_decode_attention_partial) become
    [world][num_seqs][num_heads][head_dim] and [world][num_seqs][num_heads][2],
    stacked in rank order.  Every rank must call this with tensors of the same
    shape, dtype and device; a rank that never calls it leaves the others to
    the process group's timeout."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    # one collective: (O, m, l) packed per rank, split again after the gather
    no = part_o.numel()
    flat = torch.cat([part_o.reshape(-1), part_ml.reshape(-1)])
    out = torch.empty((world, flat.numel()), dtype=flat.dtype, device=flat.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), flat, group=group)
    out_o = out[:, :no].reshape((world,) + tuple(part_o.shape))
    out_ml = out[:, no:].reshape((world,) + tuple(part_ml.shape))
    return out_o, out_ml
