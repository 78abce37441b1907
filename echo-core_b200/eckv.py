"""Python binding of libeckv.so (the C ABI in include/ec_kv.h), via ctypes.

Mirrors the reference's interface for the INT8 KV-cache path:
  * ``quantize_per_token_symmetric`` / ``fused_dequant_dot_int8``
    (include/kernels/quant.h:8-26 of echo-core),
  * ``KVCache`` with ``layer / append / seq_len / reset``
    (include/kv_cache.h:21-48) plus ``attention`` (the KV part of
    InferenceEngine::attention, src/inference.cpp:321-406),
  * ``BatchCache``: the batched ragged layout (per-sequence slabs and an
    int32 offset / capacity / length table) with ``append``, ``decode``,
    ``decode_partial`` and ``lse_combine``.

Device memory and streams come from PyTorch (plumbing only); every
computation runs in libeckv.so.  There is no fallback: importing this module
without the built library raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeckv.so")

EC_OK = 0
EC_ERR_INVALID_ARGUMENT = 1
EC_ERR_MISALIGNED = 2
EC_ERR_CAPACITY = 3
EC_ERR_UNSUPPORTED = 4
EC_ERR_CUDA = 5
EC_ERR_WORKSPACE = 6
EC_ERR_DEVICE_CHECK = 7

SCALE_PER_HEAD = 0
SCALE_ROW = 1

DEVERR_NONE = 0
DEVERR_BAD_TABLE = 1
DEVERR_OVERFLOW = 2
DEVERR_TIMEOUT = 3
DEVERR_RANGE = 4

# Every symbol include/ec_kv.h declares.
EXPORTS = (
    "ec_abi_version", "ec_status_string", "ec_last_error", "ec_device_error",
    "ec_quantize_per_token_symmetric", "ec_fused_dequant_dot_int8",
    "ec_kv_cache_create", "ec_kv_cache_destroy", "ec_kv_cache_layer", "ec_kv_cache_append",
    "ec_kv_cache_seq_len", "ec_kv_cache_reset", "ec_kv_cache_attention",
    "ec_kv_batch_append", "ec_decode_workspace_size", "ec_decode_workspace_size_batch",
    "ec_decode_attention",
    "ec_decode_attention_partial", "ec_lse_combine", "ec_prefill_attention",
    "ec_decode_attention_noalloc", "ec_kv_cache_step", "ec_kv_cache_step_host",
    "ec_kv_cache_snapshot_size", "ec_kv_cache_snapshot", "ec_kv_cache_restore",
    "ec_kv_batch_append_rope", "ec_rope_rows",
    "ec_cp_comm_create", "ec_cp_comm_open", "ec_cp_exchange_combine", "ec_cp_comm_destroy",
    "ec_cp_decode_workspace_size", "ec_cp_decode_exchange",
)


class ECError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[ec status {status}] {msg}")
        self.status = status


class ModelConfig(ctypes.Structure):
    """ec_model_config: field-for-field ModelConfig (include/config.h:6-24)."""
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "hidden_dim", "num_heads", "num_kv_heads", "head_dim", "num_layers",
        "ffn_hidden_dim", "max_seq_len")] + [
        ("ffn_type", ctypes.c_int32), ("norm_type", ctypes.c_int32),
        ("pos_encoding", ctypes.c_int32), ("use_kv_quantization", ctypes.c_bool)]


class KVLayer(ctypes.Structure):
    """ec_kv_layer: KVCacheLayer (include/kv_cache.h:7-18), device pointers."""
    _fields_ = [("keys_int8", ctypes.c_void_p), ("values_int8", ctypes.c_void_p),
                ("key_scales", ctypes.c_void_p), ("val_scales", ctypes.c_void_p),
                ("keys_fp32", ctypes.c_void_p), ("values_fp32", ctypes.c_void_p),
                ("seq_len", ctypes.c_uint32),
                ("_align64", ctypes.c_uint8 * 8)]   # KVCacheLayer is alignas(64): 64 bytes


class RopeDesc(ctypes.Structure):
    """ec_rope_desc: rope_base (<= 0: no rotation), fp16 [128] norm weight or NULL."""
    _fields_ = [("rope_base", ctypes.c_float), ("norm_weight", ctypes.c_void_p)]


def rope_rows(x, rows: int, num_heads: int, positions=None, rope_base: float = 10000.0,
              norm_weight=None, stream=None, head_dim: int = 128) -> None:
    """In-place per-head RMS norm and RoPE of query rows (ec_rope_rows)."""
    d = RopeDesc(rope_base, _ptr(norm_weight) if norm_weight is not None else None)
    check(lib().ec_rope_rows(_ptr(x), rows, num_heads, head_dim,
                             _ptr(positions) if positions is not None else None,
                             ctypes.byref(d), _stream(stream)))


class KVBatch(ctypes.Structure):
    _fields_ = [("keys", ctypes.c_void_p), ("values", ctypes.c_void_p),
                ("key_scales", ctypes.c_void_p), ("val_scales", ctypes.c_void_p),
                ("seq_offset", ctypes.c_void_p), ("seq_capacity", ctypes.c_void_p),
                ("seq_len", ctypes.c_void_p), ("error_word", ctypes.c_void_p),
                ("total_slots", ctypes.c_uint64), ("num_seqs", ctypes.c_uint32),
                ("num_kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("scale_mode", ctypes.c_int32), ("max_seq_len", ctypes.c_uint32),
                ("page_table", ctypes.c_void_p), ("page_tokens", ctypes.c_uint32),
                ("max_pages", ctypes.c_uint32), ("total_tokens_hint", ctypes.c_uint64)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libeckv.so; raises if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `make -C echo-core_b200` "
                              "or __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        vp, u32, i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int
        f = ctypes.c_float
        sig = {
            "ec_abi_version": ([], i32),
            "ec_status_string": ([i32], ctypes.c_char_p),
            "ec_last_error": ([], ctypes.c_char_p),
            "ec_device_error": ([vp, vp, ctypes.POINTER(ctypes.c_int32)], i32),
            "ec_quantize_per_token_symmetric": ([vp, vp, vp, u32, u32, vp], i32),
            "ec_fused_dequant_dot_int8": ([vp, vp, vp, vp, u32, u32, vp], i32),
            "ec_kv_cache_create": ([ctypes.POINTER(ModelConfig), i32, ctypes.POINTER(vp)], i32),
            "ec_kv_cache_destroy": ([vp], None),
            "ec_kv_cache_layer": ([vp, u32, ctypes.POINTER(KVLayer)], i32),
            "ec_kv_cache_append": ([vp, u32, vp, vp, vp], i32),
            "ec_kv_cache_seq_len": ([vp], u32),
            "ec_kv_cache_reset": ([vp], i32),
            "ec_kv_cache_attention": ([vp, u32, vp, vp, f, vp], i32),
            "ec_kv_batch_append": ([ctypes.POINTER(KVBatch), vp, vp, u32, vp], i32),
            "ec_decode_workspace_size": ([u32, u32, u32, u32], ctypes.c_size_t),
            "ec_decode_workspace_size_batch": ([ctypes.POINTER(KVBatch), u32], ctypes.c_size_t),
            "ec_decode_attention": ([ctypes.POINTER(KVBatch), vp, vp, u32, f, vp, ctypes.c_size_t,
                                     vp], i32),
            "ec_decode_attention_partial": ([ctypes.POINTER(KVBatch), vp, vp, vp, u32, f, vp,
                                             ctypes.c_size_t, vp], i32),
            "ec_lse_combine": ([vp, vp, u32, u32, u32, u32, vp, vp], i32),
            "ec_prefill_attention": ([ctypes.POINTER(KVBatch), vp, vp, u32, u32, f, vp], i32),
            "ec_decode_attention_noalloc": ([ctypes.POINTER(KVBatch), vp, vp, u32, f, vp], i32),
            "ec_cp_decode_workspace_size": ([ctypes.POINTER(KVBatch), u32], ctypes.c_size_t),
            "ec_cp_decode_exchange": ([vp, ctypes.POINTER(KVBatch), vp, u32, f, vp, ctypes.c_size_t,
                                       ctypes.c_uint32, vp, vp], i32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != EC_OK:
        raise ECError(status, lib().ec_last_error().decode())


def _torch():
    import torch
    return torch


def _stream(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def device_error(err_word=None, stream=None) -> int:
    """Reads and clears a device error word (library word when None)."""
    code = ctypes.c_int32(0)
    check(lib().ec_device_error(_ptr(err_word), _stream(stream), ctypes.byref(code)))
    return code.value


# ------------------------------------------------------------------ kernels
def quantize_per_token_symmetric(inp, out, scales, num_tokens: int, num_elements: int,
                                 stream=None) -> None:
    """include/kernels/quant.h:8-14 on device tensors (fp32 in, int8 / fp32 out)."""
    check(lib().ec_quantize_per_token_symmetric(_ptr(inp), _ptr(out), _ptr(scales), num_tokens,
                                                num_elements, _stream(stream)))


def fused_dequant_dot_int8(query, key_cache, scales, scores, dim: int, seq_len: int,
                           stream=None) -> None:
    """include/kernels/quant.h:19-26 on device tensors."""
    check(lib().ec_fused_dequant_dot_int8(_ptr(query), _ptr(key_cache), _ptr(scales),
                                          _ptr(scores), dim, seq_len, _stream(stream)))


# ------------------------------------------------------------------ KVCache
class KVCache:
    """The reference's KVCache (include/kv_cache.h:21-48) with HBM storage."""

    def __init__(self, *, num_heads: int, num_kv_heads: int, head_dim: int, num_layers: int,
                 max_seq_len: int, use_kv_quantization: bool = True,
                 scale_mode: int = SCALE_PER_HEAD):
        cfg = ModelConfig(vocab_size=0, hidden_dim=num_heads * head_dim, num_heads=num_heads,
                          num_kv_heads=num_kv_heads, head_dim=head_dim, num_layers=num_layers,
                          ffn_hidden_dim=0, max_seq_len=max_seq_len, ffn_type=0, norm_type=0,
                          pos_encoding=0, use_kv_quantization=use_kv_quantization)
        h = ctypes.c_void_p()
        check(lib().ec_kv_cache_create(ctypes.byref(cfg), scale_mode, ctypes.byref(h)))
        self._h = h
        self.config = cfg
        self.scale_mode = scale_mode

    def close(self):
        if getattr(self, "_h", None) and self._h.value:
            lib().ec_kv_cache_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def layer(self, idx: int) -> KVLayer:
        out = KVLayer()
        check(lib().ec_kv_cache_layer(self._h, idx, ctypes.byref(out)))
        return out

    def append(self, idx: int, k_proj, v_proj, stream=None) -> None:
        check(lib().ec_kv_cache_append(self._h, idx, _ptr(k_proj), _ptr(v_proj), _stream(stream)))

    def seq_len(self) -> int:
        return lib().ec_kv_cache_seq_len(self._h)

    def reset(self) -> None:
        check(lib().ec_kv_cache_reset(self._h))

    def attention(self, idx: int, q, out, softmax_scale: float, stream=None) -> None:
        check(lib().ec_kv_cache_attention(self._h, idx, _ptr(q), _ptr(out),
                                          ctypes.c_float(softmax_scale), _stream(stream)))

    def snapshot(self) -> bytes:
        """Host image of the cache's contents (ec_kv_cache_snapshot)."""
        L = lib()
        L.ec_kv_cache_snapshot_size.restype = ctypes.c_size_t
        n = L.ec_kv_cache_snapshot_size(self._h)
        buf = ctypes.create_string_buffer(n)
        check(L.ec_kv_cache_snapshot(self._h, buf, ctypes.c_size_t(n)))
        return buf.raw

    def restore(self, image: bytes) -> None:
        """Replaces the cache's contents with a snapshot (ec_kv_cache_restore)."""
        buf = ctypes.create_string_buffer(bytes(image), len(image))
        check(lib().ec_kv_cache_restore(self._h, buf, ctypes.c_size_t(len(image))))


# ---------------------------------------------------------------- BatchCache
class BatchCache:
    """Ragged batch of per-sequence int8 slabs in one set of device buffers.

    Sequence s owns slots [offset[s], offset[s] + capacity[s]); the table
    (offset, capacity, length) is int32 on the device.
    """

    def __init__(self, capacities, *, num_kv_heads=4, head_dim=128, scale_mode=SCALE_PER_HEAD,
                 device="cuda", align_slots=1, max_seq_len=None):
        torch = _torch()
        caps = np.asarray(capacities, dtype=np.int64)
        padded = ((caps + align_slots - 1) // align_slots) * align_slots
        offs = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.int64)
        total = int(padded.sum())
        if total >= 2 ** 31:
            raise ValueError("slot offsets must fit int32")
        self.num_seqs = len(caps)
        self.hkv, self.d = num_kv_heads, head_dim
        self.scale_mode = scale_mode
        self.total_slots = total
        row = num_kv_heads * head_dim
        ns = num_kv_heads if scale_mode == SCALE_PER_HEAD else 1
        self.keys = torch.zeros((total, row), dtype=torch.int8, device=device)
        self.values = torch.zeros((total, row), dtype=torch.int8, device=device)
        self.key_scales = torch.zeros((total * ns,), dtype=torch.float32, device=device)
        self.val_scales = torch.zeros((total * ns,), dtype=torch.float32, device=device)
        self.offset = torch.tensor(offs, dtype=torch.int32, device=device)
        self.capacity = torch.tensor(caps, dtype=torch.int32, device=device)
        self.length = torch.zeros(self.num_seqs, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.offsets_host = offs
        self.capacities_host = caps
        self.max_seq_len = int(caps.max()) if max_seq_len is None else int(max_seq_len)
        self._ws = None
        # host estimate of the cached tokens at decode (0: unknown); steers the split-K plan
        self.tokens_hint = 0

    def desc(self) -> KVBatch:
        return KVBatch(keys=self.keys.data_ptr(), values=self.values.data_ptr(),
                       key_scales=self.key_scales.data_ptr(), val_scales=self.val_scales.data_ptr(),
                       seq_offset=self.offset.data_ptr(), seq_capacity=self.capacity.data_ptr(),
                       seq_len=self.length.data_ptr(), error_word=self.err.data_ptr(),
                       total_slots=self.total_slots, num_seqs=self.num_seqs,
                       num_kv_heads=self.hkv, head_dim=self.d, scale_mode=self.scale_mode,
                       max_seq_len=self.max_seq_len, total_tokens_hint=self.tokens_hint)

    def workspace(self, num_heads: int):
        torch = _torch()
        d = self.desc()
        need = lib().ec_decode_workspace_size_batch(ctypes.byref(d), num_heads)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 16), dtype=torch.uint8, device=self.keys.device)
        return self._ws, need

    def append(self, k, v, tokens_per_seq: int, stream=None) -> None:
        d = self.desc()
        check(lib().ec_kv_batch_append(ctypes.byref(d), _ptr(k), _ptr(v), tokens_per_seq,
                                       _stream(stream)))

    def append_rope(self, k, v, tokens_per_seq: int, rope_base: float = 10000.0,
                    norm_weight=None, stream=None) -> None:
        """append() with K normed and rotated at its cache position
        (ec_kv_batch_append_rope)."""
        d = self.desc()
        r = RopeDesc(rope_base, _ptr(norm_weight) if norm_weight is not None else None)
        check(lib().ec_kv_batch_append_rope(ctypes.byref(d), _ptr(k), _ptr(v), tokens_per_seq,
                                            ctypes.byref(r), _stream(stream)))

    def decode(self, q, out, num_heads: int, softmax_scale: float, stream=None) -> None:
        d = self.desc()
        ws, need = self.workspace(num_heads)
        check(lib().ec_decode_attention(ctypes.byref(d), _ptr(q), _ptr(out), num_heads,
                                        ctypes.c_float(softmax_scale), _ptr(ws), ws.numel(),
                                        _stream(stream)))

    def decode_partial(self, q, part_o, part_ml, num_heads: int, softmax_scale: float,
                       stream=None) -> None:
        d = self.desc()
        ws, need = self.workspace(num_heads)
        check(lib().ec_decode_attention_partial(ctypes.byref(d), _ptr(q), _ptr(part_o),
                                                _ptr(part_ml), num_heads,
                                                ctypes.c_float(softmax_scale), _ptr(ws),
                                                ws.numel(), _stream(stream)))

    def prefill(self, q, out, n_new: int, num_heads: int, softmax_scale: float,
                stream=None) -> None:
        """Causal attention of the last n_new cached tokens of every sequence
        (q [num_seqs][n_new][num_heads][128] fp32, bf16-cast on load)."""
        d = self.desc()
        check(lib().ec_prefill_attention(ctypes.byref(d), _ptr(q), _ptr(out), n_new, num_heads,
                                         ctypes.c_float(softmax_scale), _stream(stream)))

    def device_error(self, stream=None) -> int:
        return device_error(self.err, stream)


def lse_combine(part_o, part_ml, num_parts: int, num_seqs: int, num_heads: int, head_dim: int,
                out, stream=None) -> None:
    check(lib().ec_lse_combine(_ptr(part_o), _ptr(part_ml), num_parts, num_seqs, num_heads,
                               head_dim, _ptr(out), _stream(stream)))


# ----------------------------------------------------------- PagedBatchCache
class PagedBatchCache(BatchCache):
    """A batch whose sequences hold pages of ``page_tokens`` slots from one
    pool (ec_kv_batch.page_table) instead of fixed slabs: a sequence grows by
    ``reserve``-ing more pages, up to ``max_pages`` of them.  The host keeps
    the free list and each sequence's page list; the device holds the page
    table and the capacity / length table the kernels read."""

    def __init__(self, num_seqs, *, num_pages, page_tokens=256, max_pages=None, num_kv_heads=4,
                 head_dim=128, scale_mode=SCALE_PER_HEAD, device="cuda", shuffle_seed=None):
        torch = _torch()
        if page_tokens < 128 or page_tokens & (page_tokens - 1):
            raise ValueError("page_tokens must be a power of two >= 128")
        self.num_seqs = int(num_seqs)
        self.hkv, self.d = num_kv_heads, head_dim
        self.scale_mode = scale_mode
        self.page_tokens = int(page_tokens)
        self.max_pages = int(max_pages or num_pages)
        self.total_slots = int(num_pages) * self.page_tokens
        if self.total_slots >= 2 ** 31:
            raise ValueError("the pool's slots must fit int32")
        row = num_kv_heads * head_dim
        ns = num_kv_heads if scale_mode == SCALE_PER_HEAD else 1
        self.keys = torch.zeros((self.total_slots, row), dtype=torch.int8, device=device)
        self.values = torch.zeros((self.total_slots, row), dtype=torch.int8, device=device)
        self.key_scales = torch.zeros((self.total_slots * ns,), dtype=torch.float32, device=device)
        self.val_scales = torch.zeros((self.total_slots * ns,), dtype=torch.float32, device=device)
        self.page_table = torch.full((self.num_seqs, self.max_pages), -1, dtype=torch.int32,
                                     device=device)
        self.offset = None
        self.capacity = torch.zeros(self.num_seqs, dtype=torch.int32, device=device)
        self.length = torch.zeros(self.num_seqs, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        order = np.arange(num_pages)
        if shuffle_seed is not None:
            np.random.default_rng(shuffle_seed).shuffle(order)
        self.free = list(order[::-1])          # pop() hands out pages in `order`
        self.pages = [[] for _ in range(self.num_seqs)]
        self.max_seq_len = self.max_pages * self.page_tokens
        self._ws = None
        # host estimate of the cached tokens at decode (0: unknown); steers the split-K plan
        self.tokens_hint = 0

    def slot(self, seq: int, t: int) -> int:
        """Pool slot of token t of sequence seq."""
        return int(self.pages[seq][t // self.page_tokens]) * self.page_tokens + t % self.page_tokens

    def reserve(self, seq: int, tokens: int) -> None:
        """Gives sequence seq pages for at least `tokens` tokens."""
        torch = _torch()
        need = -(-int(tokens) // self.page_tokens)
        if need > self.max_pages:
            raise ValueError(f"{tokens} tokens exceed max_pages * page_tokens")
        grew = False
        while len(self.pages[seq]) < need:
            if not self.free:
                raise MemoryError("page pool exhausted")
            self.pages[seq].append(self.free.pop())
            grew = True
        if grew:
            row = self.pages[seq] + [-1] * (self.max_pages - len(self.pages[seq]))
            self.page_table[seq].copy_(torch.tensor(row, dtype=torch.int32))
            self.capacity[seq] = len(self.pages[seq]) * self.page_tokens

    def release(self, seq: int) -> None:
        """Returns sequence seq's pages to the pool (a finished sequence) and
        empties its row, capacity and length.  Call it only once no launch
        that reads the sequence is still in flight."""
        torch = _torch()
        self.free.extend(reversed(self.pages[seq]))
        self.pages[seq] = []
        self.page_table[seq].copy_(torch.full((self.max_pages,), -1, dtype=torch.int32))
        self.capacity[seq] = 0
        self.length[seq] = 0

    def desc(self) -> KVBatch:
        return KVBatch(keys=self.keys.data_ptr(), values=self.values.data_ptr(),
                       key_scales=self.key_scales.data_ptr(), val_scales=self.val_scales.data_ptr(),
                       seq_offset=None, seq_capacity=self.capacity.data_ptr(),
                       seq_len=self.length.data_ptr(), error_word=self.err.data_ptr(),
                       total_slots=self.total_slots, num_seqs=self.num_seqs,
                       num_kv_heads=self.hkv, head_dim=self.d, scale_mode=self.scale_mode,
                       max_seq_len=self.max_seq_len, page_table=self.page_table.data_ptr(),
                       page_tokens=self.page_tokens, max_pages=self.max_pages,
                       total_tokens_hint=self.tokens_hint)
