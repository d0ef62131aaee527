"""The C++ KV prefix hash table (host code in libsckv) against the
reference's known answers: the --verify-kv-eviction self-test
(native/synapcore_native.mm:1365-1414: 100 colliding inserts -> 36 evicted,
0/36 old kept, 64/64 new kept) and tests/test_reliability.py::test_06
(260-block chain, 70-way collision), compared byte for byte with tables the
reference's own Python twin produced (tests/golden)."""
import hashlib
import json
import mmap
import struct
from pathlib import Path

import pytest

from oracle.kv_oracle import KVTableOracle, chain_prefix_hash
from synapcore_b200.kv_index import KV_TABLE_BYTES, OFFSET_KV_HASH_TBL, KVPrefixIndex

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


def test_collision_eviction_kat():
    g = GOLD["kv_table_kat"]
    idx = KVPrefixIndex()
    hashes, evicted = [], []
    for i in range(100):
        h = bytearray(32)
        struct.pack_into("<I", h, 0, 77 | ((i + 1) << 10))
        h[4] = i & 0xFF
        hashes.append(bytes(h))
        evicted.append(idx.kv_insert(bytes(h), b"\x00" * 32, (i + 1) * 16, 1000.0 + i))
    assert idx.kv_evictions_issued == 36
    assert sum(idx.kv_lookup(h) for h in hashes[:36]) == 0
    assert sum(idx.kv_lookup(h) for h in hashes[36:]) == 64
    assert evicted == g["evicted_hashes"]
    assert hashlib.sha256(idx.table_bytes()).hexdigest() == g["table_sha256"]


def test_long_context_chain_and_bucket_collisions():
    g = GOLD["kv_table_long_context"]
    idx = KVPrefixIndex()
    prev = GOLD["prefix_cache_t4"]["seed_root"]
    chain = []
    for bi in range(260):
        cur = chain_prefix_hash(prev, [((bi * 16) + t) % 50000 for t in range(16)])
        idx.kv_insert(bytes.fromhex(cur), bytes.fromhex(prev), (bi + 1) * 16, 5000.0 + bi * 0.001)
        chain.append(cur)
        prev = cur
    assert [idx.kv_lookup(bytes.fromhex(h)) for h in chain[-128:]] == g["recent_found"]
    evs = [idx.kv_insert(struct.pack("<I", 42) + struct.pack("<I", c + 1) + b"\x11" * 24, b"\x00" * 32,
                         (c + 1) * 16, 1000.0 + c) for c in range(70)]
    assert evs == g["collision_evicted"]
    assert idx.kv_lookup(struct.pack("<I", 42) + struct.pack("<I", 70) + b"\x11" * 24)
    assert not idx.kv_lookup(struct.pack("<I", 42) + struct.pack("<I", 1) + b"\x11" * 24)
    assert hashlib.sha256(idx.table_bytes()).hexdigest() == g["table_sha256"]


def test_random_ops_match_python_twin():
    import random

    rnd = random.Random(5)
    idx, twin = KVPrefixIndex(), KVTableOracle()
    keys = [bytes(rnd.getrandbits(8) for _ in range(32)) for _ in range(3000)]
    # force dense buckets: half the keys share 8 home slots
    for i in range(0, 3000, 2):
        keys[i] = struct.pack("<I", (i % 8) * 128) + keys[i][4:]
    for i, k in enumerate(keys):
        ts = float(rnd.randint(0, 500))
        assert idx.kv_insert(k, keys[i - 1], i, ts) == twin.insert(k, keys[i - 1], i, ts)
        if i % 7 == 0:
            probe = keys[rnd.randrange(0, i + 1)]
            assert idx.kv_lookup(probe) == twin.lookup(probe)
            assert idx.kv_lookup_token_end(probe) == (None if not twin.lookup(probe) else idx.kv_lookup_token_end(probe))
    assert idx.table_bytes() == bytes(twin.table)
    assert idx.kv_evictions_issued == twin.evictions


def test_table_lives_in_caller_memory(tmp_path):
    """The table can sit at the reference's offset inside an index file
    mapping, and what it writes persists across reopen."""
    path = tmp_path / "merkle_tree.idx"
    path.write_bytes(b"\x00" * (OFFSET_KV_HASH_TBL + KV_TABLE_BYTES))
    h = hashlib.sha256(b"persist").digest()
    with open(path, "r+b") as f:
        mm = mmap.mmap(f.fileno(), 0)
        idx = KVPrefixIndex(mm, OFFSET_KV_HASH_TBL)
        assert idx.kv_insert(h, b"\x01" * 32, 48, 7.0) is None
        idx.close()
        del idx
        mm.flush()
        mm.close()
    with open(path, "r+b") as f:
        mm = mmap.mmap(f.fileno(), 0)
        idx2 = KVPrefixIndex(mm, OFFSET_KV_HASH_TBL)
        assert idx2.kv_lookup(h) and idx2.kv_lookup_token_end(h) == 48
        idx2.close()
        del idx2
        mm.close()


def test_bad_hash_length_rejected():
    idx = KVPrefixIndex()
    with pytest.raises(ValueError):
        idx.kv_insert(b"\x00" * 31, b"\x00" * 32, 1, 0.0)
    assert idx.kv_lookup(b"short") is False


def test_short_hash_token_end_lookup_is_a_miss():
    idx = KVPrefixIndex()
    h = hashlib.sha256(b"x").digest()
    assert idx.kv_insert(h, b"\x00" * 32, 16, 1.0) is None
    assert idx.kv_lookup_token_end(h) == 16
    assert idx.kv_lookup_token_end(h[:4]) is None
    assert idx.kv_lookup_token_end(b"") is None


@pytest.mark.parametrize("case", ["nan", "inf", "mixed"])
def test_window_without_comparable_timestamps_matches_reference(case):
    """A full probe window whose created_at values are all NaN / +inf: the
    reference bridge overwrites the home slot, counts the eviction and names
    no evicted hash; later inserts with finite stamps evict normally."""
    g = GOLD["kv_table_unordered_timestamps"][case]
    idx, twin = KVPrefixIndex(), KVTableOracle()
    rets = []
    for c in range(64):
        h = struct.pack("<I", 300 | ((c + 1) << 10)) + bytes([c]) + b"\x22" * 27
        ts = {"nan": float("nan"), "inf": float("inf")}.get(case, float("nan") if c % 3 else float("inf"))
        rets.append(idx.kv_insert(h, b"\x00" * 32, (c + 1) * 16, ts))
        assert twin.insert(h, b"\x00" * 32, (c + 1) * 16, ts) == rets[-1]
    for c in range(3):
        h = struct.pack("<I", 300 | ((c + 100) << 10)) + b"\x33" * 28
        rets.append(idx.kv_insert(h, b"\x01" * 32, 7 + c, 50.0 + c))
        assert twin.insert(h, b"\x01" * 32, 7 + c, 50.0 + c) == rets[-1]
    assert rets == g["returns"]
    assert idx.kv_evictions_issued == g["evictions"] == twin.evictions
    assert hashlib.sha256(idx.table_bytes()).hexdigest() == g["table_sha256"]
    assert idx.table_bytes() == bytes(twin.table)
