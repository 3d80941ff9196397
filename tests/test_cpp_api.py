"""The C++ host API (include/turboquant.hpp, the reference's namespace
turboquant of lib/turboquant.h): CPU checks that the library exports every
declared C++ entry point and that the C++ mirror of the reference's
tests/test_sdpa_int4.cpp builds; on a GPU, that program's parity checks pass."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HPP = os.path.join(ROOT, "include", "turboquant.hpp")


def declared_cpp_functions():
    txt = open(HPP).read()
    names = set(re.findall(r"TQ_CXX_API\s+[\w:<>\s\*&]+?\b(\w+)\s*\(", txt))
    return names


def test_library_exports_cpp_api():
    from gemma4metal_b200.turboquant import LIB_PATH
    names = declared_cpp_functions()
    assert {"quantize", "dequantize", "sdpa_int4", "set_metallib_path", "sdpa_int4_partial",
            "lse_merge", "polar_quantize", "polar_dequantize", "polar_quantize_packed",
            "polar_dequantize_packed", "polar_dequantize_packed_fast", "compressed_sdpa",
            "polar_dequantize_fast", "compressed_score"} <= names
    out = subprocess.run(["nm", "-DC", "--defined-only", LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    for n in names:
        assert re.search(r" T turboquant::" + n + r"\(", out), f"turboquant::{n} not exported"
    for member in ("turboquant::array::array(", "turboquant::array::to_host(",
                   "turboquant::KVCache::append(", "turboquant::KVCache::sdpa("):
        assert member in out, member


def test_cpp_mirror_test_builds():
    from gemma4metal_b200 import build as b
    exes = b.build_cpp_tests()
    assert any(e.endswith("test_sdpa_int4_cpp") for e in exes)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test_sdpa_int4", "test_polar"])
def test_cpp_programs_pass(name):
    """tests/cpp/test_sdpa_int4.cpp mirrors the reference's tests/test_sdpa_int4.cpp;
    tests/cpp/test_polar.cpp exercises the reference's PolarQuant entry points."""
    from gemma4metal_b200 import build as b
    exe = b.cpp_test_binary(name)
    if not os.path.exists(exe):
        b.build_cpp_tests()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and r.stdout.strip().endswith("PASS")


@pytest.mark.gpu
def test_cpp_kv_cache_file_round_trip(tmp_path):
    """The engine's kv_cache.safetensors written by the Python store (a
    global layer of 1001 tokens and a sliding layer of window 950 that has
    seen 1500 tokens) loads through turboquant::load_kv_cache, decodes, and
    comes back out of turboquant::save_kv_cache as the same file, byte for
    byte (engine/gemma4_multilayer.cpp:113-144)."""
    import torch

    import gemma4metal_b200.turboquant as tq
    from gemma4metal_b200 import build as b
    from gemma4metal_b200.kvstore import save_kv_cache
    g = torch.Generator(device="cuda").manual_seed(5)
    glob = tq.KVCache(1, 16, 128, 1004)
    glob.append(torch.randn(1, 16, 1001, 128, device="cuda", generator=g).half(),
                torch.randn(1, 16, 1001, 128, device="cuda", generator=g).half())
    ring = tq.RingKVCache(16, 128, 950)
    for _ in range(3):
        ring.append(torch.randn(1, 16, 500, 128, device="cuda", generator=g).half(),
                    torch.randn(1, 16, 500, 128, device="cuda", generator=g).half())
    src, dst = tmp_path / "engine.safetensors", tmp_path / "cpp.safetensors"
    save_kv_cache(str(src), {0: glob, 3: ring}, cache_offset=1501)
    exe = b.cpp_test_binary("test_kvstore")
    if not os.path.exists(exe):
        b.build_cpp_tests()
    r = subprocess.run([exe, str(src), str(dst)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0 and r.stdout.strip().endswith("PASS"), r.stdout + r.stderr
    assert src.read_bytes() == dst.read_bytes()
