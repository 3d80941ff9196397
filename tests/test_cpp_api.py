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
