"""The C ABI on a machine without a GPU: the library loads, exports every
symbol include/b2a.h declares, and its host-only logic and argument checks
behave as the reference's do."""
import ctypes
import os
import re

import numpy as np
import pytest

import b2a
from b2a import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "b2a.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2a_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers exactly the header
    assert sorted(_lib.SIGNATURES) == names


def test_abi_version():
    assert _lib.load().b2a_abi_version() == 1


def test_kv_head_for_is_blocked():
    assert [b2a.kvHeadFor(h, 14, 2) for h in range(14)] == [0] * 7 + [1] * 7
    assert _lib.load().b2a_kv_head_for(0, 14, 3) == -1


def test_rope_frequencies_match_oracle(oracle):
    for hd, theta in ((64, 1e6), (8, 10000), (128, 5e5)):
        assert np.array_equal(b2a.ropeFrequencies(hd, theta), oracle.rope_frequencies(hd, theta))


def test_rope_tables_match_oracle(oracle, golden):
    t = b2a.ropeTables(64, 1e6, 40)
    assert t["half"] == 32
    assert np.array_equal(t["cos"], golden["rope_cos_64_1e6_40"])
    assert np.array_equal(t["sin"], golden["rope_sin_64_1e6_40"])


def test_capacity_error_matches_reference_before_any_device_work():
    lib = _lib.load()
    h = ctypes.c_void_p()
    st = lib.b2a_kvcache_create(None, 2, 2, 64, 0, 1, 1, ctypes.byref(h))
    assert st == _lib.B2A_ERANGE
    assert _lib.last_error() == "cache capacity must be a positive integer, got 0"
    with pytest.raises(b2a.RangeError, match="positive integer"):
        _lib.check(lib.b2a_kvcache_create(None, 2, 2, 64, -1, 1, 1, ctypes.byref(h)))


def test_init_without_gpu_fails_cleanly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    lib = _lib.load()
    h = ctypes.c_void_p()
    st = lib.b2a_init(0, ctypes.byref(h))
    assert st == _lib.B2A_ENODEV
    assert "no CUDA device" in _lib.last_error() or "out of range" in _lib.last_error()


def test_status_names():
    lib = _lib.load()
    assert lib.b2a_status_name(2) == b"B2A_ERANGE"
    assert lib.b2a_status_name(3) == b"B2A_EBUSY"


def test_noalloc_scratch_size_matches_header():
    import re
    with open(os.path.join(ROOT, "include", "b2a.h")) as f:
        m = re.search(r"#define B2A_NOALLOC_SCRATCH_BYTES \(([0-9 *]+)\)", f.read())
    assert m is not None
    n = 1
    for part in m.group(1).split("*"):
        n *= int(part)
    assert n == _lib.B2A_NOALLOC_SCRATCH_BYTES


def test_napi_addon_compiles_against_the_header(tmp_path):
    """addon/b2a_napi.c (the Node-API binding; runtime-unverified: no Node here)
    compiles warning-free against include/b2a.h and exports the module entry."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    src = os.path.join(ROOT, "addon", "b2a_napi.c")
    obj = str(tmp_path / "napi.o")
    subprocess.run([gcc, "-c", "-O2", "-std=c11", "-Wall", "-Wextra", "-Werror", "-fPIC", "-fvisibility=hidden",
                    "-I", os.path.join(ROOT, "include"), src, "-o", obj], check=True)
    syms = subprocess.run(["nm", obj], check=True, capture_output=True, text=True).stdout
    assert " T napi_register_module_v1" in syms
    # every libb2a entry the addon calls is one include/b2a.h declares
    called = set(re.findall(r"\b(b2a_[a-z_0-9]+)\s*\(", open(src).read()))
    assert called and called <= set(declared_symbols()), called - set(declared_symbols())
