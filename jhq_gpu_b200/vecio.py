"""Readers (and writers, for tests and data preparation) of the vector file
formats the reference's demos load, so that an index can be built from the
same files:

  .fvecs  per vector: int32 dim, then dim float32   (common/fvecs_io.cuh:8-57)
  .ivecs  per vector: int32 dim, then dim int32     (ground-truth ids)
  .bvecs  per vector: int32 dim, then dim uint8     (common/bvecs_io.cuh:13-88)
  .i8bin  header int32 npts, int32 dim, then npts*dim int8 (common/spacev_io.cuh:23-70)

Readers memory-map the file and return float32 rows (int32 for .ivecs) for a
row range, so a 100M-row file can be added to an index block by block. They
raise ValueError on a malformed file (ragged dims, truncated data).
"""
from __future__ import annotations

import os
from typing import Iterator, Tuple

import numpy as np

_REC = {".fvecs": (np.float32, 4), ".ivecs": (np.int32, 4), ".bvecs": (np.uint8, 1)}


def _vecs_layout(path: str) -> Tuple[np.dtype, int, int, int]:
    ext = os.path.splitext(path)[1].lower()
    if ext not in _REC:
        raise ValueError(f"{path}: not a .fvecs/.ivecs/.bvecs file")
    dt, esz = _REC[ext]
    size = os.path.getsize(path)
    if size < 4:
        raise ValueError(f"{path}: empty or truncated")
    d = int(np.fromfile(path, dtype=np.int32, count=1)[0])
    if d <= 0:
        raise ValueError(f"{path}: bad dimension {d}")
    rec = 4 + d * esz
    if size % rec:
        raise ValueError(f"{path}: size {size} is not a multiple of the record size {rec}")
    return np.dtype(dt), d, rec, size // rec


def vecs_shape(path: str) -> Tuple[int, int]:
    """(rows, dim) of a .fvecs/.ivecs/.bvecs file."""
    _, d, _, n = _vecs_layout(path)
    return n, d


def read_vecs(path: str, start: int = 0, count: int = -1) -> np.ndarray:
    """Rows [start, start+count) of a .fvecs/.ivecs/.bvecs file: float32 rows
    (.fvecs, .bvecs) or int32 rows (.ivecs)."""
    dt, d, rec, n = _vecs_layout(path)
    start = max(0, start)
    end = n if count < 0 else min(n, start + count)
    if end <= start:
        return np.zeros((0, d), np.int32 if dt == np.int32 else np.float32)
    raw = np.memmap(path, dtype=np.uint8, mode="r", offset=start * rec,
                    shape=((end - start) * rec,)).reshape(end - start, rec)
    dims = raw[:, :4].copy().view(np.int32).ravel()
    if (dims != d).any():
        raise ValueError(f"{path}: ragged vectors (dims {sorted(set(dims.tolist()))[:4]})")
    body = np.ascontiguousarray(raw[:, 4:]).view(dt).reshape(end - start, d)
    return body.astype(np.int32 if dt == np.int32 else np.float32)


def write_vecs(path: str, rows: np.ndarray) -> None:
    ext = os.path.splitext(path)[1].lower()
    dt = _REC[ext][0]
    rows = np.asarray(rows)
    n, d = rows.shape
    out = np.empty((n, 4 + d * np.dtype(dt).itemsize), np.uint8)
    out[:, :4] = np.full((n, 1), d, np.int32).view(np.uint8)
    out[:, 4:] = np.ascontiguousarray(rows.astype(dt)).view(np.uint8).reshape(n, -1)
    out.tofile(path)


def i8bin_shape(path: str) -> Tuple[int, int]:
    hdr = np.fromfile(path, dtype=np.int32, count=2)
    if hdr.size < 2 or hdr[0] < 0 or hdr[1] <= 0:
        raise ValueError(f"{path}: bad .i8bin header")
    n, d = int(hdr[0]), int(hdr[1])
    if os.path.getsize(path) < 8 + n * d:
        raise ValueError(f"{path}: truncated (header says {n} x {d})")
    return n, d


def read_i8bin(path: str, start: int = 0, count: int = -1, pad_to: int = 0) -> np.ndarray:
    """Rows [start, start+count) of a .i8bin file as float32, zero-padded to
    pad_to columns when pad_to > dim (C4: D=100 -> 104)."""
    n, d = i8bin_shape(path)
    start = max(0, start)
    end = n if count < 0 else min(n, start + count)
    w = max(d, pad_to)
    if end <= start:
        return np.zeros((0, w), np.float32)
    raw = np.memmap(path, dtype=np.int8, mode="r", offset=8 + start * d, shape=(end - start, d))
    out = np.zeros((end - start, w), np.float32)
    out[:, :d] = raw
    return out


def write_i8bin(path: str, rows: np.ndarray) -> None:
    rows = np.asarray(rows)
    n, d = rows.shape
    with open(path, "wb") as f:
        np.array([n, d], np.int32).tofile(f)
        np.ascontiguousarray(rows.astype(np.int8)).tofile(f)


def iter_rows(path: str, block: int = 1 << 20, pad_to: int = 0) -> Iterator[np.ndarray]:
    """Float32 row blocks of any of the four formats, for block-wise add()."""
    if path.lower().endswith(".i8bin"):
        n, _ = i8bin_shape(path)
        for s in range(0, n, block):
            yield read_i8bin(path, s, block, pad_to)
    else:
        n, _ = vecs_shape(path)
        for s in range(0, n, block):
            yield read_vecs(path, s, block).astype(np.float32)
