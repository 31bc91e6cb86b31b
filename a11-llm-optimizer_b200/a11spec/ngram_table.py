"""The hashed trigram table on disk.

The reference names "N-gram spec tables" (README.md) but defines no format,
so this is the format of this library, little-endian:

    offset  size  field
    0       8     magic b"A11NGRAM"
    8       4     version (uint32) = 1
    12      4     log2_buckets (uint32)
    16      4     slots (uint32)
    20      4     reserved (uint32) = 0
    24      ...   int32 [2^log2_buckets][slots][2]: (token, count); count <= 0 = empty slot

A bucket is a11s_ngram_bucket(prev, last, log2_buckets): the SplitMix64
finaliser of the token pair, top log2_buckets bits. a11s_ngram_expand reads
the table, a11s_ngram_update learns into it.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = b"A11NGRAM"
VERSION = 1
_HEADER = struct.Struct("<8sIIII")


def save(path: str, table: np.ndarray, log2_buckets: int) -> None:
    table = np.ascontiguousarray(table, dtype="<i4")
    if table.ndim != 3 or table.shape[0] != 1 << log2_buckets or table.shape[2] != 2:
        raise ValueError(f"table shape {table.shape} is not [2^{log2_buckets}, slots, 2]")
    with open(path, "wb") as f:
        f.write(_HEADER.pack(MAGIC, VERSION, log2_buckets, table.shape[1], 0))
        f.write(table.tobytes())


def load(path: str):
    """Returns (table int32 [2^k, slots, 2], log2_buckets)."""
    with open(path, "rb") as f:
        head = f.read(_HEADER.size)
        if len(head) != _HEADER.size:
            raise ValueError(f"{path}: truncated header")
        magic, version, log2_buckets, slots, _ = _HEADER.unpack(head)
        if magic != MAGIC:
            raise ValueError(f"{path}: not an n-gram table (magic {magic!r})")
        if version != VERSION:
            raise ValueError(f"{path}: version {version}, this library reads {VERSION}")
        if not 1 <= log2_buckets <= 30 or not 1 <= slots <= 32:
            raise ValueError(f"{path}: log2_buckets {log2_buckets} / slots {slots} out of range")
        n = (1 << log2_buckets) * slots * 2
        data = np.frombuffer(f.read(4 * n), dtype="<i4")
        if data.size != n:
            raise ValueError(f"{path}: {data.size} entries, expected {n}")
    return data.reshape(1 << log2_buckets, slots, 2).astype(np.int32), log2_buckets


def empty(log2_buckets: int, slots: int = 8) -> np.ndarray:
    """A table with every slot empty (token -1, count 0)."""
    t = np.zeros((1 << log2_buckets, slots, 2), np.int32)
    t[:, :, 0] = -1
    return t
