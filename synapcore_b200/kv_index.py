"""KV prefix hash table: the bridge half of the prefix cache.

`KVPrefixIndex` exposes the two calls NativeKVPrefixCache makes on its
bridge — ``kv_lookup`` and ``kv_insert`` (native/native_engine.py:1714-1752)
— plus the ``kv_evictions_issued`` counter, backed by the C++ table in
libsckv (sckv_kv_lookup / sckv_kv_insert). The 1024 x 80-byte slot array is
caller memory: a private bytearray by default, or any writable buffer such
as the KV region of an index file mapping, so the table persists exactly
where the reference's did (OFFSET_KV_HASH_TBL of merkle_tree.idx,
native/native_engine.py:1279).
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

from . import _native as N

KV_SLOTS = 1024
KV_SLOT_BYTES = 80
KV_TABLE_BYTES = KV_SLOTS * KV_SLOT_BYTES
# Byte offset of the KV table inside a reference index file (merkle_tree.idx):
# 256 (header) + 2048*32 (XOR tree) + 1024*64 (experts) + 50304*40 (tokens).
OFFSET_KV_HASH_TBL = 256 + 2048 * 32 + 1024 * 64 + 50304 * 40


class KVPrefixIndex:
    """Drop-in for the KV side of NativeMmapIndexBridge."""

    def __init__(self, buffer=None, offset: int = 0):
        if buffer is None:
            buffer = bytearray(KV_TABLE_BYTES)
            offset = 0
        mv = memoryview(buffer)
        if mv.readonly:
            raise ValueError("KV table buffer must be writable")
        if len(mv) - offset < KV_TABLE_BYTES:
            raise ValueError(f"KV table needs {KV_TABLE_BYTES} bytes at offset {offset}")
        self._buffer = buffer
        self._cbuf = (ctypes.c_char * KV_TABLE_BYTES).from_buffer(buffer, offset)
        self._ptr = ctypes.addressof(self._cbuf)
        self.idx_lock = threading.RLock()
        self._evictions = ctypes.c_uint64(0)
        self._lib = N.lib()

    @property
    def kv_evictions_issued(self) -> int:
        return int(self._evictions.value)

    @kv_evictions_issued.setter
    def kv_evictions_issued(self, v: int) -> None:
        self._evictions.value = int(v)

    def table_bytes(self) -> bytes:
        return ctypes.string_at(self._ptr, KV_TABLE_BYTES)

    def kv_lookup(self, prefix_hash_bytes: bytes) -> bool:
        h = bytes(prefix_hash_bytes)
        if len(h) != 32:
            return False
        with self.idx_lock:
            return bool(self._lib.sckv_kv_lookup(self._ptr, h, None))

    def kv_lookup_token_end(self, prefix_hash_bytes: bytes) -> Optional[int]:
        h = bytes(prefix_hash_bytes)
        if len(h) != 32:
            return None
        out = ctypes.c_uint32(0)
        with self.idx_lock:
            if self._lib.sckv_kv_lookup(self._ptr, h, ctypes.byref(out)):
                return int(out.value)
        return None

    def kv_insert(self, prefix_hash_bytes: bytes, parent_hash_bytes: bytes, token_end: int,
                  timestamp: float) -> Optional[str]:
        """Returns the evicted prefix hash (hex) when the probe window was
        full, else None — the reference bridge's contract."""
        h, p = bytes(prefix_hash_bytes), bytes(parent_hash_bytes)
        if len(h) != 32 or len(p) != 32:
            raise ValueError("prefix and parent hashes must be 32 bytes")
        ev = ctypes.create_string_buffer(32)
        with self.idx_lock:
            rc = self._lib.sckv_kv_insert(self._ptr, h, p, int(token_end) & 0xFFFFFFFF, float(timestamp), ev,
                                          ctypes.byref(self._evictions))
        if rc == 1:
            return None
        if rc == 2:
            return ev.raw.hex()
        if rc == 3:
            # window full with no timestamp below +inf (e.g. all NaN): the
            # home slot was overwritten, and the reference bridge names no
            # evicted hash (native/native_engine.py:1747-1752)
            return None
        N.check(rc, "sckv_kv_insert")
        return None

    def close(self) -> None:
        # release the exported buffer view
        self._cbuf = None
