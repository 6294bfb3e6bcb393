"""Restatement of the reference's checkpoint format (TEST INFRASTRUCTURE ONLY).

ckpt.rs:8-189: the magic "RUSTNN\\0", the tensor count (u32), the scalar
count (u64) and the configuration hash (u64), little endian, then the
little-endian f32 payload; config_hash is FNV-1a over the kind's bytes and
each value's 8 little-endian bytes (ckpt.rs:83-96).
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = b"RUSTNN\0"
HEADER_LEN = len(MAGIC) + 4 + 8 + 8
FNV_OFFSET = 0xCBF29CE484222325
FNV_PRIME = 0x00000100000001B3
M64 = 2**64 - 1


def fnv1a(data: bytes, h: int = FNV_OFFSET) -> int:
    for b in data:
        h = ((h ^ b) * FNV_PRIME) & M64
    return h


def config_hash(kind: bytes, values) -> int:
    """ckpt.rs:83-96."""
    h = fnv1a(kind)
    for v in values:
        h = fnv1a(struct.pack("<Q", int(v) & M64), h)
    return h


def resnet_hash(depth_n, width, nclass) -> int:
    """model.rs:220-229."""
    return config_hash(b"resnet", [depth_n, width, nclass])


def rustvit_hash(cfg: dict, nclass, ncoarse, use_exits, parent) -> int:
    """vit.rs:780-801; cfg holds the Cfg fields (droppath as f32 bits)."""
    dp_bits = struct.unpack("<I", struct.pack("<f", float(np.float32(cfg["droppath"]))))[0]
    fields = [cfg["width"], cfg["cmid"], cfg["dim"], cfg["heads"], cfg["depth3"], cfg["dim4"], cfg["heads4"],
              cfg["depth4"], dp_bits, cfg["img"], nclass, ncoarse, int(use_exits), len(cfg["mem_at"])]
    fields += list(cfg["mem_at"]) + [len(parent)] + [int(p) for p in parent]
    return config_hash(b"rustvit", fields)


def encode(tensors: int, chash: int, payload) -> bytes:
    """write_checkpoint's bytes (ckpt.rs:99-128)."""
    payload = np.ascontiguousarray(payload, dtype="<f4").ravel()
    return MAGIC + struct.pack("<IQQ", tensors, payload.size, chash) + payload.tobytes()


def decode(data: bytes):
    """(tensors, scalars, hash, payload) of a headed checkpoint."""
    assert data.startswith(MAGIC)
    tensors, scalars, chash = struct.unpack_from("<IQQ", data, len(MAGIC))
    return tensors, scalars, chash, np.frombuffer(data[HEADER_LEN:], dtype="<f4").copy()
