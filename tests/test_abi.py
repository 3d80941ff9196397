"""CPU checks of the drop-in boundary: the shared library loads, exports every
symbol that include/*.h declares, validates arguments on the host (no GPU
needed for a rejected call), and the C++ header compiles."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for f in os.listdir(INC):
        if f.endswith(".h"):
            txt = open(os.path.join(INC, f)).read()
            names |= set(re.findall(r"TQ_API\s+[\w\s\*]+?\b(tq_\w+)\s*\(", txt))
    return names


def test_library_exports_every_declared_symbol():
    from gemma4metal_b200.turboquant import LIB_PATH, load_library
    L = load_library()
    syms = declared_symbols()
    assert len(syms) >= 12
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (tq_\w+)", out))
    missing = syms - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for s in syms:
        getattr(L, s)


def test_version_and_noop_metallib():
    import gemma4metal_b200.turboquant as tq
    assert "sm_100a" in tq.version()
    tq.set_metallib_path("/nonexistent/turboquant.metallib")


def test_host_validation_rejects_bad_arguments():
    from gemma4metal_b200.turboquant import load_library
    L = load_library()
    P = ctypes.c_void_p
    fake = P(0x1000)  # never dereferenced: validation fails first
    # head_dim 96 unsupported
    rc = L.tq_sdpa_int4(fake, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16, 96,
                        10, 12, None, fake, 1, None, 0, None)
    assert rc == 2 and b"head_dim" in L.tq_last_error()
    # gqa 3 unsupported
    rc = L.tq_sdpa_int4(fake, 1, fake, fake, fake, fake, fake, fake, 1, 3, 1.0, 0, 1, 16, 128,
                        10, 12, None, fake, 1, None, 0, None)
    assert rc == 2 and b"gqa" in L.tq_last_error()
    # n_tokens > capacity
    rc = L.tq_sdpa_int4(fake, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16, 128,
                        20, 12, None, fake, 1, None, 0, None)
    assert rc == 1 and b"capacity" in L.tq_last_error()
    # capacity not a multiple of 4
    rc = L.tq_sdpa_int4(fake, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16, 128,
                        10, 10, None, fake, 1, None, 0, None)
    assert rc == 1 and b"multiple of 4" in L.tq_last_error()
    # null pointer
    rc = L.tq_sdpa_int4(None, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16, 128,
                        10, 12, None, fake, 1, None, 0, None)
    assert rc == 1
    # misaligned cache pointer
    rc = L.tq_sdpa_int4(fake, 1, P(0x1004), fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16,
                        128, 10, 12, None, fake, 1, None, 0, None)
    assert rc == 1 and b"aligned" in L.tq_last_error()
    # append past the capacity
    rc = L.tq_quantize_append(fake, fake, 1, 1, 16, 128, 2, fake, fake, fake, fake, fake, fake,
                              1, 8, 7, None, None)
    assert rc == 1 and b"capacity" in L.tq_last_error()
    # merge with too many parts
    rc = L.tq_lse_merge(fake, 65, 1, 8, 128, fake, 0, None)
    assert rc == 1
    # quantize head_dim not a multiple of 64
    rc = L.tq_quantize(fake, 0, 4, 100, fake, fake, fake, 1, None)
    assert rc == 1


def test_cpp_header_compiles():
    src = os.path.join(ROOT, "tests", "cpp", "test_sdpa_int4.cpp")
    if not os.path.exists(src):
        pytest.skip("C++ mirror test not present")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I" + INC,
                        "-I/usr/local/cuda/include", src], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_decode_step_host_validation():
    """tq_decode_step_* reject bad arguments before touching the GPU."""
    from gemma4metal_b200.turboquant import load_library
    L = load_library()
    fake = ctypes.c_void_p(0x1000)
    h = ctypes.c_void_p()
    # head_dim 96 unsupported
    rc = L.tq_decode_step_create(1, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16,
                                 96, 64, 1, ctypes.byref(h))
    assert rc == 2 and b"head_dim" in L.tq_last_error() and not h.value
    # capacity not a multiple of 4
    rc = L.tq_decode_step_create(1, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16,
                                 128, 62, 1, ctypes.byref(h))
    assert rc == 1 and b"sizes" in L.tq_last_error()
    # null cache pointer, bad scale dtype
    rc = L.tq_decode_step_create(1, 1, None, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1, 16,
                                 128, 64, 1, ctypes.byref(h))
    assert rc == 1 and b"null" in L.tq_last_error()
    rc = L.tq_decode_step_create(1, 1, fake, fake, fake, fake, fake, fake, 2, 2, 1.0, 0, 1, 16,
                                 128, 64, 1, ctypes.byref(h))
    assert rc == 1 and b"dtype" in L.tq_last_error()
    # null step object
    n = (ctypes.c_int32 * 1)(5)
    assert L.tq_decode_step_run(None, None, None, None, n, None) == 1
    slot = (ctypes.c_int32 * 1)(4)
    assert L.tq_decode_step_run_at(None, None, None, None, n, slot, None) == 1
    assert L.tq_decode_step_run_at(None, None, None, None, n, None, None) == 1
    # the per-sequence-slot step needs its slot array
    rc = L.tq_sdpa_int4_append_slots(fake, 1, fake, fake, 1, fake, fake, fake, fake, fake, fake,
                                     1, 2, 1.0, 0, 1, 16, 128, 10, 12, None, None, fake, 1, None,
                                     0, None)
    assert rc == 1 and b"slots" in L.tq_last_error()
    assert L.tq_decode_step_buffers(None, None, None, None, None) == 1
    assert L.tq_decode_step_destroy(None) == 0


def test_noalloc_and_workspace_size_reject_unsupported_head_dim():
    """head_dim 0 or far above 512 must come back as an error code, not reach
    the split planner (which divides by head_dim)."""
    from gemma4metal_b200.turboquant import load_library
    L = load_library()
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.tq_sdpa_int4_noalloc.argtypes = [P, I, P, P, P, P, P, P, I, I, F, I, I, I, I, I, I, P, P, I,
                                       P]
    L.tq_sdpa_int4_workspace_size.restype = ctypes.c_size_t
    L.tq_sdpa_int4_workspace_size.argtypes = [I, I, I, I, I, I]
    fake = P(0x1000)  # never dereferenced: validation fails first
    for hd in (0, 96, 16384):
        assert L.tq_sdpa_int4_workspace_size(1, 32, 16, hd, 1024, 0) == 0
        rc = L.tq_sdpa_int4_noalloc(fake, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 1,
                                    16, hd, 1024, 1024, None, fake, 1, None)
        assert rc == 2 and b"head_dim" in L.tq_last_error(), (hd, rc)
    rc = L.tq_sdpa_int4_noalloc(fake, 1, fake, fake, fake, fake, fake, fake, 1, 3, 1.0, 0, 1, 16,
                                128, 1024, 1024, None, fake, 1, None)
    assert rc == 2 and b"gqa" in L.tq_last_error()
    rc = L.tq_sdpa_int4_noalloc(fake, 1, fake, fake, fake, fake, fake, fake, 1, 2, 1.0, 0, 0, 16,
                                128, 1024, 1024, None, fake, 1, None)
    assert rc == 1
