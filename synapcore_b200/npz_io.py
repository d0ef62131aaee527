"""Parallel reader for the prefix cache's `.npz` blocks.

`np.savez` writes an uncompressed ("stored") zip of `.npy` members; the
reference reloads each block with `np.load` (native/native_engine.py:2270-2280),
whose zip layer parses and CRC-checks every member under the interpreter
lock. `read_npz_many` reads whole files with one `read` each, checks every
member's CRC-32 (zlib releases the interpreter lock on large buffers) and
maps the arrays straight out of the file bytes, on a small thread pool. Any
file that is not a plain stored zip of version 1/2 `.npy` members (deflated
members, zip64, Fortran order, object arrays) goes through `np.load`. A CRC
mismatch raises `zipfile.BadZipFile`, as `np.load` would.
"""
from __future__ import annotations

import io
import os
import struct
import threading
import zipfile
import zlib
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Union

import numpy as np

PathLike = Union[str, Path]

_EOCD = b"PK\x05\x06"
_CDIR = b"PK\x01\x02"
_LOCAL = b"PK\x03\x04"

_pool: Optional[ThreadPoolExecutor] = None
_pool_lock = threading.Lock()


def _executor() -> ThreadPoolExecutor:
    global _pool
    with _pool_lock:
        if _pool is None:
            _pool = ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1)),
                                       thread_name_prefix="sckv-npz")
        return _pool


def _np_load(path: PathLike) -> Dict[str, np.ndarray]:
    with np.load(path) as data:
        return {name: data[name] for name in data.files}


def _parse_npy(buf: memoryview, start: int, size: int) -> Optional[np.ndarray]:
    fp = io.BytesIO(buf[start:start + min(size, 4096)])
    try:
        major, _ = np.lib.format.read_magic(fp)
        if major == 1:
            shape, fortran, dtype = np.lib.format.read_array_header_1_0(fp)
        elif major == 2:
            shape, fortran, dtype = np.lib.format.read_array_header_2_0(fp)
        else:
            return None
    except ValueError:
        return None
    if fortran or dtype.hasobject:
        return None
    count = int(np.prod(shape, dtype=np.int64))
    off = start + fp.tell()
    if off + count * dtype.itemsize > start + size:
        return None
    return np.frombuffer(buf, dtype=dtype, count=count, offset=off).reshape(shape)


def read_npz(path: PathLike) -> Dict[str, np.ndarray]:
    """All arrays of one `.npz` (read-only views of the file's bytes)."""
    with open(path, "rb") as f:
        raw = f.read()
    buf = memoryview(raw)
    end = raw.rfind(_EOCD, max(0, len(raw) - 65558))
    if end < 0 or end + 22 > len(raw):
        return _np_load(path)
    n_entries, cd_size, cd_off = struct.unpack_from("<HII", raw, end + 10)
    if cd_off == 0xFFFFFFFF or n_entries == 0xFFFF:
        return _np_load(path)
    out: Dict[str, np.ndarray] = {}
    pos = cd_off
    for _ in range(n_entries):
        if raw[pos:pos + 4] != _CDIR:
            return _np_load(path)
        (method, crc, csize, usize, nlen, elen, clen) = struct.unpack_from("<H4xIIIHHH", raw, pos + 10)
        (local_off,) = struct.unpack_from("<I", raw, pos + 42)
        name = raw[pos + 46:pos + 46 + nlen].decode("utf-8")
        pos += 46 + nlen + elen + clen
        if method != 0 or csize != usize or 0xFFFFFFFF in (csize, usize, local_off):
            return _np_load(path)
        if raw[local_off:local_off + 4] != _LOCAL:
            return _np_load(path)
        lnlen, lelen = struct.unpack_from("<HH", raw, local_off + 26)
        start = local_off + 30 + lnlen + lelen
        if start + usize > len(raw):
            raise zipfile.BadZipFile(f"truncated member {name!r} in {path}")
        if zlib.crc32(buf[start:start + usize]) != crc:
            raise zipfile.BadZipFile(f"Bad CRC-32 for file {name!r} in {path}")
        arr = _parse_npy(buf, start, usize)
        if arr is None:
            return _np_load(path)
        out[name[:-4] if name.endswith(".npy") else name] = arr
    return out


def parallel_for(fn, n: int) -> None:
    """fn(i) for i in range(n) on the shared thread pool (for large array
    copies, which run without the interpreter lock)."""
    if n <= 1:
        for i in range(n):
            fn(i)
        return
    for _ in _executor().map(fn, range(n)):
        pass


def read_npz_many(paths: Sequence[PathLike]) -> List[Dict[str, np.ndarray]]:
    """read_npz over many files on the shared thread pool, results in order."""
    if len(paths) <= 1:
        return [read_npz(p) for p in paths]
    return list(_executor().map(read_npz, paths))
