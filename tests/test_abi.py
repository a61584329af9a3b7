"""CPU tests of the C ABI: the library loads, exports every symbol that
include/kyro_spec.h declares, and rejects bad arguments on the host before
touching a GPU."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kyro_spec.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(kyro_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    from kyro_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_declarations_match_binding_list():
    from kyro_b200._lib import EXPORTS
    assert header_functions() == sorted(EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    from kyro_b200._lib import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (kyro_\w+)$", out, re.M))
    for name in header_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None
    # nothing beyond the C ABI leaks out under a kyro_ name
    assert exported == set(header_functions())


def test_version_and_strings(lib):
    assert lib.kyro_version() == 1
    assert lib.kyro_status_string(0) == b"ok"
    assert b"workspace" in lib.kyro_status_string(8)
    names = lib.kyro_kernel_names().decode().split(";")
    assert "verify_attention_kernel" in names and "accept_stats_kernel" in names


def test_null_context_is_rejected(lib):
    from kyro_b200._lib import AcceptParams, AttnParams, KVParams, last_error
    p = AcceptParams(8, 4, 32000, 0, 1.0, 0, 0, 0)
    st = lib.kyro_spec_accept(None, C.byref(p), None, None, None, None, None, None, None, None, 0)
    assert st == 1 and "kyro_ctx" in last_error()
    a = AttnParams(1, 6, 32, 8, 128, 16, 8, 16, 0.0, 0)
    assert lib.kyro_verify_attention(None, C.byref(a), *([None] * 8), 0) == 1
    k = KVParams(1, 16, 8, 16)
    assert lib.kyro_kv_commit(None, C.byref(k), 6, None, None, None, None, None, None) == 1


def test_workspace_sizes(lib):
    from kyro_b200._lib import AcceptParams, AttnParams, SampleParams
    p = AcceptParams(64, 5, 128256, 0, 1.0, 0, 0, 0)
    stoch = lib.kyro_spec_accept_workspace_size(C.byref(p))
    nchunks = -(-128256 // 512)
    assert stoch >= 64 * 11 * nchunks * 16
    p.mode = 1
    assert lib.kyro_spec_accept_workspace_size(C.byref(p)) < stoch
    s = SampleParams(8, 4, 32000, 1.0, 0, 0, 0, 0)
    assert lib.kyro_sample_workspace_size(C.byref(s)) > 0
    a = AttnParams(64, 6, 32, 8, 128, 16, 257, 16384, 0.0, 0)
    assert lib.kyro_verify_attention_workspace_size(C.byref(a)) > 0
    a.head_dim = 96  # unsupported: size query reports 0
    assert lib.kyro_verify_attention_workspace_size(C.byref(a)) == 0


def test_context_create_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from kyro_b200._lib import last_error
    h = C.c_void_p()
    st = lib.kyro_ctx_create(0, None, C.byref(h))
    assert st in (2, 1) and not h.value
    assert last_error()


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from kyro_b200 import _lib
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError, match="no CPU fallback"):
        _lib.load()
