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
  ``CPExchange`` does the exchange and the merge in one kernel instead: each
  rank stores its partial straight into every rank's receive buffer over
  NVLink (CUDA IPC peer mappings) and merges once all have arrived.

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


def shard_weighted(weights, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [lo, hi) block of units for `rank`, balanced by weight.

    For ragged batches the weight of a sequence is its cached-token count, so
    every rank streams about the same KV bytes.  Boundary r is the last unit
    index whose prefix sum does not exceed r/world of the total; blocks are rank-ordered,
    cover every unit exactly once, and a rank's sum exceeds total/world by at
    most one unit's weight.  Equal weights give the same blocks as `shard`.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    w = [float(x) for x in weights]
    if any(x < 0 for x in w):
        raise ValueError("negative weight")
    n = len(w)
    total = sum(w)
    if total <= 0:
        return shard(n, rank, world)

    def boundary(r):
        if r <= 0:
            return 0
        if r >= world:
            return n
        target = total * r / world
        acc, best = 0.0, 0
        for i in range(n):
            acc += w[i]
            if acc > target * (1 + 1e-12):
                break
            best = i + 1
        return best

    lo, hi = boundary(rank), boundary(rank + 1)
    return lo, max(lo, hi)


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


class CPExchange:
    """The context-parallel exchange and merge in one kernel over NVLink peer
    memory (ec_cp_exchange_combine), in place of ``gather_partials`` plus
    ``ec_lse_combine``.

    Construction is collective: every rank creates its receive buffer and the
    ranks swap CUDA IPC handles over the process group (any backend; the
    handles are 64 bytes of host data).  ``combine`` is called by every rank
    once per step, in the same order; ``close`` is collective too, so that no
    rank frees its buffer while a peer may still store into it."""

    def __init__(self, num_seqs: int, num_heads: int, group=None, device_epoch: bool = False):
        import ctypes
        import torch.distributed as dist
        import eckv
        self._lib = eckv.lib()
        self._group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        handle = (ctypes.c_char * 64)()
        self._h = ctypes.c_void_p()
        eckv.check(self._lib.ec_cp_comm_create(self.world, self.rank, num_seqs, num_heads,
                                               ctypes.byref(self._h), handle))
        if self.world > 1:
            got = [None] * self.world
            dist.all_gather_object(got, bytes(handle), group=group)
            blob = b"".join(got)
            eckv.check(self._lib.ec_cp_comm_open(self._h, ctypes.create_string_buffer(blob, len(blob))))
        self.epoch = 0
        # device_epoch: the epoch lives on the GPU and advances in stream
        # order, so combine() can be captured into a CUDA graph and replayed
        self.device_epoch = device_epoch

    def combine(self, part_o, part_ml, out, stream=None) -> None:
        import ctypes
        import eckv
        self.epoch += 1
        eckv.check(self._lib.ec_cp_exchange_combine(
            self._h, eckv._ptr(part_o), eckv._ptr(part_ml),
            ctypes.c_uint32(0 if self.device_epoch else self.epoch), eckv._ptr(out),
            eckv._stream(stream)))

    def decode_exchange(self, batch, q, out, num_heads: int, softmax_scale: float,
                        stream=None) -> None:
        """One context-parallel decode step in two launches
        (ec_cp_decode_exchange): decode of this rank's slice held in `batch`
        (a BatchCache of this comm's sequences) with the split-K chunk merge,
        the exchange and the rank merge done by one kernel."""
        import ctypes
        import torch
        import eckv
        self.epoch += 1
        d = batch.desc()
        need = self._lib.ec_cp_decode_workspace_size(ctypes.byref(d), num_heads)
        ws = getattr(self, "_ws", None)
        if ws is None or ws.numel() < need:
            ws = self._ws = torch.empty(max(need, 16), dtype=torch.uint8, device=batch.keys.device)
        eckv.check(self._lib.ec_cp_decode_exchange(
            self._h, ctypes.byref(d), eckv._ptr(q), num_heads, ctypes.c_float(softmax_scale),
            eckv._ptr(ws), ws.numel(), ctypes.c_uint32(0 if self.device_epoch else self.epoch),
            eckv._ptr(out), eckv._stream(stream)))

    def close(self) -> None:
        if not getattr(self, "_h", None) or not self._h.value:
            return
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self._group)
        self._lib.ec_cp_comm_destroy(self._h)
        self._h = None
