"""The C-ABI library loads, exports every symbol include/ec_kv.h declares, and
its structs have the layout the bindings assume.  CPU only: no call here
launches a kernel or touches a CUDA device."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ec_kv.h")


@pytest.fixture(scope="module")
def L():
    import eckv
    if not os.path.exists(eckv.LIB_PATH):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "echo-core_b200")], check=True)
    return eckv.lib()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"EC_API\s+[\w\s\*]+?\b(ec_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    import eckv
    assert declared_symbols() == sorted(eckv.EXPORTS)


def test_every_declared_symbol_is_exported(L):
    out = subprocess.run(["nm", "-D", "--defined-only", L._name], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (ec_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    for s in declared_symbols():
        assert hasattr(L, s)


def test_version_and_status_strings(L):
    import eckv
    assert L.ec_abi_version() == 4
    assert L.ec_status_string(eckv.EC_ERR_CAPACITY) == b"cache capacity exceeded"
    assert L.ec_status_string(12345) == b"unknown status"


def test_argument_validation_fails_before_any_device_work(L):
    import eckv
    null = ctypes.c_void_p(0)
    rc = L.ec_quantize_per_token_symmetric(null, null, null, 4, 8, null)
    assert rc == eckv.EC_ERR_INVALID_ARGUMENT
    assert b"null" in L.ec_last_error()
    # zero tokens is a valid no-op
    assert L.ec_quantize_per_token_symmetric(null, null, null, 0, 8, null) == eckv.EC_OK
    assert L.ec_kv_batch_append(None, null, null, 1, null) == eckv.EC_ERR_INVALID_ARGUMENT
    b = eckv.KVBatch(keys=16, values=16, key_scales=16, val_scales=16, seq_offset=16,
                     seq_capacity=16, seq_len=16, total_slots=1, num_seqs=1, num_kv_heads=4,
                     head_dim=64, scale_mode=0, max_seq_len=1)
    rc = L.ec_decode_attention(ctypes.byref(b), ctypes.c_void_p(16), ctypes.c_void_p(16), 16,
                               ctypes.c_float(0.1), null, 0, null)
    assert rc == eckv.EC_ERR_UNSUPPORTED
    b.head_dim, b.keys = 128, 17
    rc = L.ec_decode_attention(ctypes.byref(b), ctypes.c_void_p(16), ctypes.c_void_p(16), 16,
                               ctypes.c_float(0.1), null, 0, null)
    assert rc == eckv.EC_ERR_MISALIGNED
    b.keys, b.scale_mode = 16, 7
    assert L.ec_kv_batch_append(ctypes.byref(b), ctypes.c_void_p(16), ctypes.c_void_p(16), 1,
                                null) == eckv.EC_ERR_INVALID_ARGUMENT
    cfg = eckv.ModelConfig(num_heads=16, num_kv_heads=0, head_dim=128, num_layers=1,
                           max_seq_len=8, use_kv_quantization=True)
    h = ctypes.c_void_p()
    assert L.ec_kv_cache_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == eckv.EC_ERR_INVALID_ARGUMENT
    assert L.ec_kv_cache_create(ctypes.byref(cfg), 9, ctypes.byref(h)) == eckv.EC_ERR_INVALID_ARGUMENT


def test_struct_layouts_match_the_c_header(tmp_path):
    """Compile a probe against ec_kv.h and compare sizeof/offsetof with ctypes."""
    import eckv
    src = tmp_path / "probe.c"
    fields = {
        "ec_model_config": [f[0] for f in eckv.ModelConfig._fields_],
        "ec_kv_layer": [f[0] for f in eckv.KVLayer._fields_ if not f[0].startswith("_")],
        "ec_kv_batch": [f[0] for f in eckv.KVBatch._fields_],
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "ec_kv.h"', "int main(void){"]
    for st, fs in fields.items():
        lines.append(f'printf("{st} size %zu\\n", sizeof({st}));')
        for f in fs:
            lines.append(f'printf("{st} {f} %zu\\n", offsetof({st}, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o",
                    str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n"):
        if line:
            st, f, v = line.split()
            got[(st, f)] = int(v)
    for st, cls in (("ec_model_config", eckv.ModelConfig), ("ec_kv_layer", eckv.KVLayer),
                    ("ec_kv_batch", eckv.KVBatch)):
        assert got[(st, "size")] == ctypes.sizeof(cls), st
        for f in fields[st]:
            assert got[(st, f)] == getattr(cls, f).offset, (st, f)


def test_model_config_mirrors_reference_layout():
    """ModelConfig (include/config.h:6-24): eight uint32, three int-sized enum
    classes, one bool -> 48 bytes with the bool at offset 44."""
    import eckv
    assert ctypes.sizeof(eckv.ModelConfig) == 48
    assert eckv.ModelConfig.use_kv_quantization.offset == 44


@pytest.mark.parametrize("page_tokens,max_pages,total_slots", [
    (96, 4, 96 * 4),       # not a power of two
    (16, 4, 64),           # below 128: a 32-token decode tile would cross pages
    (256, 0, 1024),        # no page-table row
    (256, 4, 1000),        # pool not a whole number of pages
    (1 << 25, 4, 1 << 25),  # beyond the page-size limit
])
def test_noalloc_refuses_bad_paged_batches_like_the_main_entry_point(L, page_tokens, max_pages,
                                                                     total_slots):
    """ec_decode_attention_noalloc validates a batch with the same code as
    ec_decode_attention: a paged descriptor whose page_tokens / max_pages /
    total_slots the kernels cannot address is refused on the host, before
    any device call, by both entry points.  A valid paged descriptor (with
    seq_offset NULL, as the header allows) passes the batch check and only
    then meets the device."""
    import eckv
    null = ctypes.c_void_p(0)
    b = eckv.KVBatch(keys=256, values=256, key_scales=256, val_scales=256, seq_offset=None,
                     seq_capacity=256, seq_len=256, total_slots=total_slots, num_seqs=1,
                     num_kv_heads=4, head_dim=128, scale_mode=0, max_seq_len=page_tokens,
                     page_table=256, page_tokens=page_tokens, max_pages=max_pages)
    q = ctypes.c_void_p(256)
    rc_main = L.ec_decode_attention(ctypes.byref(b), q, q, 16, ctypes.c_float(0.1), q, 1 << 20, null)
    msg_main = L.ec_last_error()
    rc = L.ec_decode_attention_noalloc(ctypes.byref(b), q, q, 16, ctypes.c_float(0.1), null)
    assert rc == rc_main == eckv.EC_ERR_INVALID_ARGUMENT, (rc, rc_main)
    assert L.ec_last_error().split(b":", 1)[1] == msg_main.split(b":", 1)[1]


def test_noalloc_takes_the_main_entry_points_null_argument_checks(L):
    import eckv
    null = ctypes.c_void_p(0)
    assert L.ec_decode_attention_noalloc(None, null, null, 16, ctypes.c_float(0.1),
                                         null) == eckv.EC_ERR_INVALID_ARGUMENT
    b = eckv.KVBatch(keys=256, values=256, key_scales=256, val_scales=256, seq_offset=None,
                     seq_capacity=256, seq_len=256, total_slots=1024, num_seqs=1,
                     num_kv_heads=4, head_dim=128, scale_mode=0, max_seq_len=512)
    # neither seq_offset nor a page table
    assert L.ec_decode_attention_noalloc(ctypes.byref(b), ctypes.c_void_p(256), ctypes.c_void_p(256),
                                         16, ctypes.c_float(0.1), null) == eckv.EC_ERR_INVALID_ARGUMENT
    b.seq_offset = 256
    b.head_dim = 64
    assert L.ec_decode_attention_noalloc(ctypes.byref(b), ctypes.c_void_p(256), ctypes.c_void_p(256),
                                         16, ctypes.c_float(0.1), null) == eckv.EC_ERR_UNSUPPORTED


def test_kv_layer_has_the_reference_alignment(tmp_path):
    """KVCacheLayer is alignas(64) (include/kv_cache.h:7): ec_kv_layer keeps
    that size and alignment in C and C++, and the binding's struct is 64 bytes."""
    import eckv
    assert ctypes.sizeof(eckv.KVLayer) == 64
    src = tmp_path / "align.c"
    src.write_text('#include "ec_kv.h"\n'
                   '_Static_assert(sizeof(ec_kv_layer) == 64, "size");\n'
                   '_Static_assert(_Alignof(ec_kv_layer) == 64, "align");\n'
                   'int main(void) { return 0; }\n')
    subprocess.run(["gcc", "-std=c11", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                    str(src)], check=True)


def test_reference_layer_call_site_compiles_against_the_wrapper(tmp_path):
    """The reference engine's own call site, `KVCacheLayer& cache_layer =
    kv_cache_->layer(layer_idx);` (src/inference.cpp:331), and its
    `layer(0).seq_len` read (src/kv_cache.cpp:115-118) compile unchanged
    against ec::gpu::KVCache, with a KVCacheLayer laid out as the
    reference declares it (include/kv_cache.h:7-18)."""
    src = tmp_path / "site.cpp"
    src.write_text(r"""
#include <cstdint>
#include <memory>
#include "ec_kv_cache.hpp"
struct alignas(64) KVCacheLayer {
    int8_t* keys_int8; int8_t* values_int8; float* key_scales; float* val_scales;
    float* keys_fp32; float* values_fp32; uint32_t seq_len;
};
using KVCache = ec::gpu::KVCache;
uint32_t site(std::unique_ptr<KVCache>& kv_cache_, uint32_t layer_idx) {
    KVCacheLayer& cache_layer = kv_cache_->layer(layer_idx);
    const KVCache& c = *kv_cache_;
    const KVCacheLayer& l0 = c.layer(0);
    return cache_layer.seq_len + l0.seq_len + kv_cache_->layer(0).seq_len;
}
""")
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-I",
                    os.path.join(ROOT, "include"), str(src)], check=True)
