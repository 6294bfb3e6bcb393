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
