"""The checkpoint format (csrc/ckpt.cu) on the host: the reference's own
checkpoint tests (ckpt.rs:252-369) run against rnn_ckpt_write / rnn_ckpt_read,
the FNV-1a hash against the published FNV-1a 64 test vectors, and the bytes
against the restatement in oracle/ckpt.py."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import ckpt as K


@pytest.fixture(scope="module")
def L():
    from rustnn_b200 import _lib

    return _lib


def lib_hash(L, kind: bytes, values):
    v = np.ascontiguousarray(values, dtype=np.uint64)
    return L.lib().rnn_ckpt_config_hash(kind, len(kind), C.c_void_p(v.ctypes.data if v.size else 0), v.size)


def fake(fill):
    """ckpt.rs:272-287: parameters of 6 and 4 values, a buffer of 3."""
    p0 = np.array([fill + j for j in range(6)], np.float32)
    p1 = np.array([fill + 10 + j for j in range(4)], np.float32)
    buf = np.full(3, fill * 2.0, np.float32)
    return np.concatenate([p0, p1, buf]), 3


def write(L, path, payload, tensors, h):
    return L.lib().rnn_ckpt_write(str(path).encode(), tensors, h, C.c_void_p(payload.ctypes.data), payload.size)


def read(L, path, n, tensors, h):
    out = np.zeros(n, np.float32)
    rc = L.lib().rnn_ckpt_read(str(path).encode(), tensors, h, C.c_void_p(out.ctypes.data), n)
    return rc, out


def test_fnv1a_vectors(L):
    """FNV-1a 64 of "", "a" and "foobar" (the published test vectors)."""
    assert K.fnv1a(b"") == 0xCBF29CE484222325
    assert K.fnv1a(b"a") == 0xAF63DC4C8601EC8C
    assert K.fnv1a(b"foobar") == 0x85944171F73967E8
    assert lib_hash(L, b"", []) == 0xCBF29CE484222325
    assert lib_hash(L, b"foobar", []) == 0x85944171F73967E8
    for kind, vals in [(b"resnet", [9, 64, 100]), (b"rustvit", [1, 2**40, 2**64 - 1]), (b"x", [])]:
        assert lib_hash(L, kind, vals) == K.config_hash(kind, vals)
    assert lib_hash(L, b"resnet", [9, 64, 100]) == K.resnet_hash(9, 64, 100)


def test_round_trip(L, tmp_path):
    """ckpt.rs:310-326 (round_trip_preserva_tudo): the bytes are the
    restated format's."""
    path = tmp_path / "roundtrip.bin"
    payload, tensors = fake(1.5)
    assert write(L, path, payload, tensors, 0xABCD) == 0
    rc, got = read(L, path, payload.size, tensors, 0xABCD)
    assert rc == 0 and np.array_equal(got, payload)
    data = path.read_bytes()
    assert data.startswith(K.MAGIC)
    assert data == K.encode(tensors, 0xABCD, payload)
    assert not os.path.exists(str(path) + ".tmp")


def test_refuses_other_config(L, tmp_path):
    """ckpt.rs:328-338 (recusa_configuracao_diferente)."""
    path = tmp_path / "config.bin"
    payload, tensors = fake(1.0)
    assert write(L, path, payload, tensors, 0x1111) == 0
    rc, _ = read(L, path, payload.size, tensors, 0x2222)
    assert rc == -1 and "incompatible" in L.lib().rnn_last_error().decode()


def test_refuses_other_tensor_count(L, tmp_path):
    path = tmp_path / "tensors.bin"
    payload, tensors = fake(1.0)
    assert write(L, path, payload, tensors, 5) == 0
    rc, _ = read(L, path, payload.size, tensors + 1, 5)
    assert rc == -1 and "tensors" in L.lib().rnn_last_error().decode()


def test_refuses_truncated(L, tmp_path):
    """ckpt.rs:340-348 (recusa_arquivo_truncado)."""
    path = tmp_path / "trunc.bin"
    payload, tensors = fake(1.0)
    assert write(L, path, payload, tensors, 7) == 0
    data = path.read_bytes()
    path.write_bytes(data[:-8])
    rc, _ = read(L, path, payload.size, tensors, 7)
    assert rc != 0
    path.write_bytes(data[:10])  # inside the header
    rc, _ = read(L, path, payload.size, tensors, 7)
    assert rc != 0


def test_accepts_legacy_without_header(L, tmp_path):
    """ckpt.rs:350-364 (aceita_legado_sem_cabecalho)."""
    path = tmp_path / "legacy.bin"
    payload, tensors = fake(3.0)
    assert write(L, path, payload, tensors, 42) == 0
    path.write_bytes(path.read_bytes()[K.HEADER_LEN:])
    rc, got = read(L, path, payload.size, tensors, 42)
    assert rc == 0 and np.array_equal(got, payload)


def test_failed_save_keeps_previous(L, tmp_path):
    """ckpt.rs:366-379 (save_nao_destroi_o_anterior_ao_falhar)."""
    path = tmp_path / "atomic.bin"
    payload, tensors = fake(5.0)
    assert write(L, path, payload, tensors, 1) == 0
    good = path.read_bytes()
    bad = path / "not-a-directory"
    payload9, _ = fake(9.0)
    assert write(L, bad, payload9, tensors, 1) == -6  # RNN_ERR_IO
    assert path.read_bytes() == good
    assert not os.path.exists(str(bad) + ".tmp")


def test_missing_file(L, tmp_path):
    rc, _ = read(L, tmp_path / "absent.bin", 4, 1, 0)
    assert rc == -6
