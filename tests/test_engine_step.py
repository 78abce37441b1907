"""The InferenceEngine integration path in C++: ec::gpu::KVCache::step_host
(include/ec_kv_cache.hpp) driven token by token and layer by layer the way
InferenceEngine::forward drives attention (src/inference.cpp:301-415), against
the oracle (tests/cpp/engine_step.cpp)."""
from __future__ import annotations

import os
import subprocess

import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "echo-core_b200")


def _build(tmp_path) -> str:
    O.lib()   # builds oracle/liboracle.so when missing
    exe = str(tmp_path / "engine_step")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "engine_step.cpp"), "-o", exe,
           "-L", LIB_DIR, "-leckv", "-L", os.path.dirname(O.ORACLE_SO), "-loracle",
           f"-Wl,-rpath,{LIB_DIR}", f"-Wl,-rpath,{os.path.dirname(O.ORACLE_SO)}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_engine_step_program_compiles_and_links(tmp_path):
    """The C++ wrapper compiles against the reference's ModelConfig layout and
    links to libeckv.so (no GPU needed)."""
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_engine_step_matches_oracle(tmp_path, cuda):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "engine_step ok" in r.stdout
