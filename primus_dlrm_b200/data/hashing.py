"""Cross-feature hashing (``primus_dlrm/data/hashing.py``).

Wire format (a contract: trained cross tables depend on it): xxhash64 with
``seed = salt`` over the little-endian int64 concatenation of the keys,
modulo the table size.  ``cross_hash_nway([a, b], ...) ==
cross_hash_int64(a, b, ...)`` by construction.

The per-pair host hash uses the ``xxhash`` C library; ``xxh64_np`` is a
vectorised numpy restatement of the published XXH64 algorithm (Yann Collet,
xxHash specification) for whole arrays of fixed-width keys, used by the
batch path and checked against the library in the tests.
"""
from __future__ import annotations

import struct

import numpy as np

try:
    import xxhash as _xx
except ImportError:  # pragma: no cover
    _xx = None

__all__ = ["cross_hash_int64", "cross_hash_nway", "cross_hash_batch", "xxh64_np"]

_P1 = np.uint64(0x9E3779B185EBCA87)
_P2 = np.uint64(0xC2B2AE3D27D4EB4F)
_P3 = np.uint64(0x165667B19E3779F9)
_P4 = np.uint64(0x85EBCA77C2B2AE63)
_P5 = np.uint64(0x27D4EB2F165667C5)


def _rotl(x: np.ndarray, r: int) -> np.ndarray:
    return (x << np.uint64(r)) | (x >> np.uint64(64 - r))


def _round(acc: np.ndarray, lane: np.ndarray) -> np.ndarray:
    acc = acc + lane * _P2
    acc = _rotl(acc, 31)
    return acc * _P1


def _merge(acc: np.ndarray, v: np.ndarray) -> np.ndarray:
    acc = acc ^ _round(np.zeros_like(v), v)
    return acc * _P1 + _P4


def xxh64_np(words: np.ndarray, seed: int = 0) -> np.ndarray:
    """XXH64 of each row of ``words`` ([N, n] uint64, little-endian 8-byte lanes)."""
    words = np.ascontiguousarray(words, dtype=np.uint64)
    n_rows, n = words.shape
    length = np.uint64(8 * n)
    seed = np.uint64(seed & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        i = 0
        if n >= 4:
            v1 = np.full(n_rows, seed + _P1 + _P2, dtype=np.uint64)
            v2 = np.full(n_rows, seed + _P2, dtype=np.uint64)
            v3 = np.full(n_rows, seed, dtype=np.uint64)
            v4 = np.full(n_rows, seed - _P1, dtype=np.uint64)
            while i + 4 <= n:
                v1 = _round(v1, words[:, i])
                v2 = _round(v2, words[:, i + 1])
                v3 = _round(v3, words[:, i + 2])
                v4 = _round(v4, words[:, i + 3])
                i += 4
            h = _rotl(v1, 1) + _rotl(v2, 7) + _rotl(v3, 12) + _rotl(v4, 18)
            h = _merge(h, v1)
            h = _merge(h, v2)
            h = _merge(h, v3)
            h = _merge(h, v4)
        else:
            h = np.full(n_rows, seed + _P5, dtype=np.uint64)
        h = h + length
        while i < n:
            k = _round(np.zeros(n_rows, dtype=np.uint64), words[:, i])
            h = h ^ k
            h = _rotl(h, 27) * _P1 + _P4
            i += 1
        h = h ^ (h >> np.uint64(33))
        h = h * _P2
        h = h ^ (h >> np.uint64(29))
        h = h * _P3
        h = h ^ (h >> np.uint64(32))
    return h


def cross_hash_nway(keys: list[int], table_size: int, salt: int = 0) -> int:
    """xxhash64(seed=salt) of ``struct.pack('<{n}q', *keys)`` mod ``table_size``."""
    n = len(keys)
    assert n >= 2, f"cross_hash_nway needs >=2 keys, got {n}"
    data = struct.pack(f"<{n}q", *(int(k) for k in keys))
    if _xx is not None:
        return _xx.xxh64(data, seed=salt).intdigest() % table_size
    w = np.frombuffer(data, dtype="<u8").reshape(1, n)
    return int(xxh64_np(w, salt)[0]) % table_size


def cross_hash_int64(feat_a: int, feat_b: int, table_size: int, salt: int = 0) -> int:
    return cross_hash_nway([feat_a, feat_b], table_size, salt)


def cross_hash_batch(arr_a, arr_b, table_size: int, salt: int = 0) -> np.ndarray:
    """Vectorised 2-way hash over int64 arrays (scalar operands broadcast)."""
    a = np.asarray(arr_a, dtype=np.int64).ravel()
    b = np.asarray(arr_b, dtype=np.int64).ravel()
    if b.shape[0] == 1 and a.shape[0] != 1:
        b = np.broadcast_to(b, a.shape)
    elif a.shape[0] == 1 and b.shape[0] != 1:
        a = np.broadcast_to(a, b.shape)
    assert a.shape == b.shape, f"cross_hash_batch shape mismatch: {a.shape} vs {b.shape}"
    words = np.stack([a.astype("<i8").view("<u8"), b.astype("<i8").view("<u8")], axis=1)
    return (xxh64_np(words, salt) % np.uint64(table_size)).astype(np.int64)
