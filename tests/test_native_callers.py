"""The C ABI from native callers, without ctypes.

- The Rust -sys crate (rust/kyro-spec-sys/src/lib.rs) declares exactly the
  functions, argument counts and parameter structs of include/kyro_spec.h.
  Rust is not in this image, so the crate is checked against the header
  textually here; this is the binding a Kyro maintainer adds under
  worker.rs.
- A C++ program (tests/cpp/accept_harness.cpp) built against the header and
  linked with libkyro_spec.so: on CPU it checks the host-side error path; on
  a GPU it runs one acceptance call and must match the oracle bit for bit.
"""
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kyro_spec.h")
RUST = os.path.join(ROOT, "rust", "kyro-spec-sys", "src", "lib.rs")
HARNESS = os.path.join(ROOT, "tests", "cpp", "accept_harness.cpp")
BUILD = os.path.join(ROOT, "tests", "cpp", "_build")


def _split_args(s):
    depth, parts, cur = 0, [], ""
    for ch in s:
        if ch == "(":
            depth += 1
        elif ch == ")":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    if cur.strip():
        parts.append(cur)
    return [p.strip() for p in parts if p.strip() and p.strip() != "void"]


def header_signatures():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    sigs = {}
    for m in re.finditer(r"^\w[\w\s\*]*?\b(kyro_\w+)\s*\((.*?)\)\s*;", text, re.M | re.S):
        sigs[m.group(1)] = len(_split_args(m.group(2)))
    return sigs


def _balanced(text, start):
    """The text between the parenthesis at text[start] and its match."""
    depth = 0
    for i in range(start, len(text)):
        if text[i] == "(":
            depth += 1
        elif text[i] == ")":
            depth -= 1
            if depth == 0:
                return text[start + 1:i]
    raise ValueError("unbalanced")


def rust_signatures():
    text = open(RUST).read()
    sigs = {}
    for m in re.finditer(r"pub fn (kyro_\w+)\s*\(", text):
        sigs[m.group(1)] = len(_split_args(_balanced(text, m.end() - 1)))
    return sigs


def header_structs():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"typedef struct (kyro_\w+) \{(.*?)\}", text, re.S):
        out[m.group(1)] = re.findall(r"(\w+)\s*;", m.group(2))
    return out


def rust_structs():
    text = open(RUST).read()
    out = {}
    for m in re.finditer(r"pub struct (kyro_\w+) \{(.*?)\}", text, re.S):
        out[m.group(1)] = re.findall(r"pub (\w+)\s*:", m.group(2))
    return out


def test_rust_sys_crate_mirrors_the_header():
    h, r = header_signatures(), rust_signatures()
    assert sorted(h) == sorted(r)
    for name in h:
        assert h[name] == r[name], (name, h[name], r[name])
    hs, rs = header_structs(), rust_structs()
    for name, fields in hs.items():
        assert rs.get(name) == fields, (name, fields, rs.get(name))


def _build_harness():
    os.makedirs(BUILD, exist_ok=True)
    from kyro_b200 import build
    lib = build.build()
    exe = os.path.join(BUILD, "accept_harness")
    libdir = os.path.dirname(lib)
    if not os.path.exists(exe) or os.path.getmtime(exe) < max(os.path.getmtime(HARNESS),
                                                               os.path.getmtime(lib)):
        subprocess.run([build.nvcc(), "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                        HARNESS, "-o", exe, "-L" + libdir, "-lkyro_spec", "-lcudart",
                        "-Xlinker", "-rpath=" + libdir], check=True)
    return exe


def test_cpp_harness_error_path_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    exe = _build_harness()
    r = subprocess.run([exe, "--no-gpu"], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert "no-gpu ok" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("B,k,V,mode,T", [(8, 4, 32000, 0, 1.0), (5, 5, 128256, 0, 0.7),
                                          (4, 3, 32000, 2, 1.0)])
def test_cpp_harness_accept_matches_oracle(oracle, tmp_path, B, k, V, mode, T):
    exe = _build_harness()
    rng = np.random.default_rng(B + k)
    tgt = (rng.standard_normal((B, k + 1, V), dtype=np.float32) * np.float32(3.0))
    drf = (tgt[:, :k] + rng.standard_normal((B, k, V), dtype=np.float32)).astype(np.float32)
    drafts = oracle.sample_tokens(drf, T, seed=7)[0] if k else np.zeros((B, 0), np.int32)
    seed, step = 11, 3
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        f.write(np.array([B, k, V, mode], dtype=np.int32).tobytes())
        f.write(np.array([T], dtype=np.float32).tobytes())
        f.write(np.array([step], dtype=np.uint32).tobytes())
        f.write(np.array([seed], dtype=np.uint64).tobytes())
        f.write(tgt.tobytes())
        f.write(drf.tobytes())
        f.write(np.ascontiguousarray(drafts, dtype=np.int32).tobytes())
    out = tmp_path / "out.bin"
    r = subprocess.run([exe, str(inp), str(out)], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stderr)
    raw = np.fromfile(out, dtype=np.int32)
    acc, raw = raw[:B], raw[B:]
    toks, raw = raw[:B * (k + 1)].reshape(B, k + 1), raw[B * (k + 1):]
    num, raw = raw[:B], raw[B:]
    probs = raw[:B * k * 2].view(np.float32).reshape(B, k, 2)
    status = int(raw[B * k * 2])
    ref = oracle.spec_accept(tgt, drf if mode == 0 else None, drafts, mode=mode, temperature=T,
                             seed=seed, step=step, nthreads=os.cpu_count() or 1)
    assert status == 0
    assert np.array_equal(acc, ref[0])
    assert np.array_equal(toks, ref[1])
    assert np.array_equal(num, ref[2])
    if mode == 0:
        assert np.array_equal(probs, ref[3])
