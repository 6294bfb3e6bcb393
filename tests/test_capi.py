"""CPU-side checks of the C ABI: the library loads (no GPU needed to load
it) and exports exactly what include/*.h declares; the Python bindings
declare the same set."""
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(rnn_[a-z0-9_]+)\s*\(", text):
            syms.add(m.group(1))
    return syms


@pytest.fixture(scope="module")
def lib():
    from rustnn_b200 import _lib

    if not os.path.exists(_lib.LIB_PATH):
        from rustnn_b200 import build

        build.build()
    return _lib.lib()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {"rnn_gemm_dev", "rnn_conv2d_fwd_dev", "rnn_resnet_train_step"} <= syms
    assert len(syms) > 40


def test_library_exports_every_declared_symbol(lib):
    from rustnn_b200 import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for s in declared_symbols():
        assert hasattr(lib, s)


def test_python_bindings_cover_header():
    from rustnn_b200 import _lib

    bound = set(_lib.SIGS) | {"rnn_last_error"}
    assert declared_symbols() <= bound, sorted(declared_symbols() - bound)


def test_errors_are_reported_without_gpu(lib):
    """A null context is rejected on the host before any CUDA call."""
    import ctypes as C

    code = lib.rnn_gemm_dev(None, 1, 1, 1, None, 0, None, 0, None, 0)
    assert code == -1
    assert b"context" in lib.rnn_last_error()
    del C


def _header_arity():
    out = {}
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for m in re.finditer(r"\b(rnn_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
            args = " ".join(m.group(2).split())
            out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_rust_sys_crate_binds_every_entry_point():
    """rust/rnn-b200-sys (the -sys crate a Rust host links; no cargo in this
    image, so it is checked against the header as text): one extern "C"
    item per declared function, with the same number of parameters."""
    src = open(os.path.join(ROOT, "rust", "rnn-b200-sys", "src", "lib.rs")).read()
    rust = {}
    for m in re.finditer(r"pub fn (rnn_[a-z0-9_]+)\(([^)]*)\)", src):
        args = m.group(2).strip()
        rust[m.group(1)] = 0 if not args else args.count(":")
    hdr = _header_arity()
    assert set(hdr) == set(rust), (sorted(set(hdr) - set(rust)), sorted(set(rust) - set(hdr)))
    bad = {k: (hdr[k], rust[k]) for k in hdr if hdr[k] != rust[k]}
    assert not bad, bad
