"""The drop-in PagedKVArena / NativeKVPrefixCache on the GPU against the
reference's own tests (tests/test_p1_2_paged_kv_cache.py T1, T3, T4), with
every observable compared to what the reference produced (tests/golden):
returned page ids, tables, counters, and SHA-256 of the gathered bytes."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "golden.json").read_text())


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_t1_arena_lru_eviction_and_contiguous_gather(cuda_device):
    from synapcore_b200 import PagedKVArena

    g = GOLD["arena_t1"]
    arena = PagedKVArena(max_pages=8, num_layers=16, num_kv_heads=16, head_dim=128, quant_mode="fp16")
    rng = np.random.default_rng(101)
    written, log, pages = [], [], []
    for i in range(12):
        h = f"{i + 1:064x}"
        k = rng.standard_normal((16, 1, 16, 16, 128)).astype(np.float16)
        v = rng.standard_normal((16, 1, 16, 16, 128)).astype(np.float16)
        written.append(h)
        pages.append((k, v))
        log.append(["write", h, arena.write_page_fp16(h, k, v)])
        if i >= 2:
            log.append(["lookup", written[0], arena.lookup_page_id(written[0])])
            log.append(["lookup", written[1], arena.lookup_page_id(written[1])])
    assert len(arena.page_table) == 8 and arena.page_evictions == 4
    for idx in range(6):
        log.append(["lookup", written[idx], arena.lookup_page_id(written[idx])])
    surv = [0, 1, 6, 7, 8, 9, 10, 11]
    pids = [arena.lookup_page_id(written[i]) for i in surv]
    kc, vc = arena.gather_contiguous_kv_numpy(pids)
    assert log == g["log"]
    assert pids == g["survivor_pids"]
    assert arena.page_table == g["page_table"] and arena.page_last_used == g["page_last_used"]
    assert list(arena.free_pages) == g["free_pages"]
    assert (arena.step_clock, arena.page_hits, arena.page_misses) == (g["step_clock"], g["page_hits"],
                                                                      g["page_misses"])
    assert list(kc.shape) == g["gather_shape"] == [16, 1, 16, 128, 128]
    assert sha(kc) == g["gather_k_sha256"] and sha(vc) == g["gather_v_sha256"]
    k_ref = np.concatenate([pages[i][0] for i in surv], axis=3)
    assert float(np.max(np.abs(kc - k_ref))) == 0.0
    # device views are laid out like the reference's numpy pool
    assert tuple(arena.k_pool_fp16.shape) == (8, 16, 1, 16, 16, 128)
    np.testing.assert_array_equal(arena.k_pool_fp16[pids[2]].cpu().numpy(), pages[6][0])
    arena.clear()
    assert arena.k_pool_fp16 is None and len(arena.free_pages) == 8


def test_t3_int8_quantized_kv_memory_and_precision(cuda_device):
    from synapcore_b200 import PagedKVArena

    g = GOLD["int8_t3"]
    a16 = PagedKVArena(max_pages=16, quant_mode="fp16")
    a8 = PagedKVArena(max_pages=16, quant_mode="int8")
    assert a16.bytes_per_page == 2097152 and a8.bytes_per_page == 1064960
    rng = np.random.default_rng(2026)
    k = (rng.standard_normal((16, 1, 16, 16, 128)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((16, 1, 16, 16, 128)) * 0.5).astype(np.float16)
    pid = a8.write_page_fp16("a" * 64, k, v)
    kd, vd = a8.read_page_fp16(pid)
    # stored codes and scales are the reference quantiser's, bit for bit
    assert sha(a8.k_pool_q[pid].cpu().numpy()) == g["k_pool_q_sha256"]
    assert sha(a8.k_scale[pid].cpu().numpy()) == g["k_scale_sha256"]
    assert sha(kd) == g["k_deq_sha256"] and sha(vd) == g["v_deq_sha256"]
    kf, kdf = k.astype(np.float32).reshape(-1), kd.astype(np.float32).reshape(-1)
    cos = float(np.dot(kf, kdf) / (np.linalg.norm(kf) * np.linalg.norm(kdf)))
    assert cos > 0.9999 and abs(cos - g["cosine"]) < 1e-9
    assert float(np.mean(np.abs(kf - kdf))) < 0.005
    a16.clear()
    a8.clear()


def test_int8_small_rows_bit_exact(cuda_device):
    """Quantisation of rows incl. an all-zero row (scale floor 1e-7)."""
    from synapcore_b200 import PagedKVArena

    arr = np.load(Path(__file__).resolve().parent / "golden" / "golden_arrays.npz")
    x = arr["int8_small_x"]  # [2, 1, 3, 16, 128]
    a8 = PagedKVArena(max_pages=2, num_layers=2, num_kv_heads=3, head_dim=128, quant_mode="int8")
    pid = a8.write_page_fp16("b" * 64, x, x)
    kq, ks, _, _ = a8.read_page_quantized(pid)
    np.testing.assert_array_equal(kq, arr["int8_small_q"])
    np.testing.assert_array_equal(ks.view(np.uint16), arr["int8_small_s"].view(np.uint16))
    kd, _ = a8.read_page_fp16(pid)
    np.testing.assert_array_equal(kd.view(np.uint16), arr["int8_small_deq"].view(np.uint16))
    # write_page_quantized into an fp16 arena dequantises like the reference
    a16 = PagedKVArena(max_pages=2, num_layers=2, num_kv_heads=3, head_dim=128, quant_mode="fp16")
    pid = a16.write_page_quantized("c" * 64, arr["int8_small_q"], arr["int8_small_s"], arr["int8_small_q"],
                                   arr["int8_small_s"])
    kd16, _ = a16.read_page_fp16(pid)
    np.testing.assert_array_equal(kd16.view(np.uint16), arr["int8_small_deq"].view(np.uint16))


def test_t4_prefix_cache_arena_hits_disk_reload_and_budget(cuda_device, tmp_path):
    from synapcore_b200 import KVPrefixIndex, NativeKVPrefixCache

    g = GOLD["prefix_cache_t4"]
    bridge = KVPrefixIndex()
    cache = NativeKVPrefixCache(tmp_path, bridge, device="cpu", num_layers=16, num_kv_heads=16, head_dim=128,
                                max_pages=4, max_disk_blocks=3, quant_mode="int8", timestamp_fn=lambda: 0.0)
    rng = np.random.default_rng(77)
    tokens = list(range(100, 165))
    k = (rng.standard_normal((16, 1, 16, 65, 128)) * 0.4).astype(np.float16)
    v = (rng.standard_normal((16, 1, 16, 65, 128)) * 0.4).astype(np.float16)
    seed = g["seed_root"]
    assert cache.save_prefix_blocks_numpy(tokens, k, v, seed) == 4
    assert cache.disk_blocks_evicted == 1
    assert sorted(p.name for p in cache.kv_dir.iterdir()) == g["after_first_save"]["files"]
    short = tokens[:49]
    cache.save_prefix_blocks_numpy(short, k[:, :, :, :49], v[:, :, :, :49], seed)
    before = cache.blocks_loaded_from_arena
    m1, k1, v1 = cache.match_longest_prefix_numpy(short, seed)
    assert m1 == 48 and cache.blocks_loaded_from_arena - before == 3
    assert k1.shape == (16, 1, 16, 48, 128)
    assert sha(k1) == g["k_restored_sha256"] and sha(v1) == g["v_restored_sha256"]
    cache.arena.page_table.clear()
    cache.arena.reverse_page_table.clear()
    cache.arena.free_pages.clear()
    cache.arena.free_pages.extend(range(cache.arena.max_pages))
    m2, k2, v2 = cache.match_longest_prefix_numpy(short, seed)
    assert m2 == 48 and float(np.max(np.abs(k1.astype(np.float32) - k2.astype(np.float32)))) == 0.0
    assert sha(k2) == g["k_disk_sha256"] and sha(v2) == g["v_disk_sha256"]
    assert (cache.blocks_loaded_from_disk, cache.blocks_loaded_from_arena, cache.blocks_saved_to_disk,
            cache.tokens_skipped) == (g["blocks_loaded_from_disk"], g["blocks_loaded_from_arena"],
                                      g["blocks_saved_to_disk"], g["tokens_skipped"])
    assert cache.get_paged_kv_stats() == g["stats"]
    assert sorted(p.name for p in cache.kv_dir.iterdir()) == g["files_end"]
    assert hashlib.sha256(bridge.table_bytes()).hexdigest() == g["kv_table_sha256"]
    # the int8 blocks on disk hold exactly the reference quantiser's codes
    for f in cache.kv_dir.iterdir():
        with np.load(f) as d:
            assert set(d.files) == {"kq", "ks", "vq", "vs"}
            assert d["kq"].dtype == np.int8 and d["ks"].dtype == np.float16
            assert d["kq"].shape == (16, 1, 16, 16, 128) and d["ks"].shape == (16, 1, 16, 16, 1)


def test_fp16_prefix_cache_matches_reference_semantics(cuda_device, tmp_path):
    """fp16 mode against the oracle restatement of the reference prefix cache.
    With 3 arena pages and a 5-block prefix, matching reloads evicted blocks
    from disk and the LRU reuses pages already in the match list — the
    reference returns those overwritten pages too, and so must the drop-in.
    With enough pages the match returns exactly the saved K/V."""
    from oracle.kv_oracle import ArenaOracle, KVTableOracle, PrefixCacheOracle
    from synapcore_b200 import NativeKVPrefixCache

    rng = np.random.default_rng(3)
    toks = list(range(7, 7 + 81))
    k = rng.standard_normal((2, 1, 4, 81, 128)).astype(np.float16)
    v = rng.standard_normal((2, 1, 4, 81, 128)).astype(np.float16)
    for max_pages in (3, 8):
        cache = NativeKVPrefixCache(tmp_path / f"d{max_pages}", None, num_layers=2, num_kv_heads=4, head_dim=128,
                                    max_pages=max_pages, max_disk_blocks=8, quant_mode="fp16",
                                    timestamp_fn=lambda: 1.0)
        ora = PrefixCacheOracle(tmp_path / f"o{max_pages}" / "kv_cache_blocks",
                                ArenaOracle(max_pages, 2, 4, 128, "fp16"), KVTableOracle(), max_disk_blocks=8)
        assert cache.save_prefix_blocks_numpy(toks, k, v, "ab" * 32) == 5
        assert ora.save(toks, k, v, "ab" * 32, timestamp=lambda: 1.0) == 5
        n, kd, vd = cache.match_longest_prefix(toks, "ab" * 32)
        n_o, k_o, v_o = ora.match(toks, "ab" * 32)
        assert n == n_o == 80
        np.testing.assert_array_equal(kd.cpu().numpy(), k_o)
        np.testing.assert_array_equal(vd.cpu().numpy(), v_o)
        assert cache.arena.page_table == ora.arena.page_table
        assert list(cache.arena.free_pages) == list(ora.arena.free_pages)
        assert (cache.blocks_loaded_from_disk, cache.blocks_loaded_from_arena) == (ora.blocks_loaded_from_disk,
                                                                                 ora.blocks_loaded_from_arena)
        assert cache.bridge.table_bytes() == bytes(ora.table.table)
        if max_pages == 8:
            np.testing.assert_array_equal(kd.cpu().numpy(), k[:, :, :, :80])
            np.testing.assert_array_equal(vd.cpu().numpy(), v[:, :, :, :80])


def test_int8_prefix_cache_reload_matches_reference_semantics(cuda_device, tmp_path):
    """int8 mode: blocks reloaded from disk in one staged write per match,
    against the oracle's one-write-per-block walk. With 3 arena pages the
    walk's own allocations evict pages it already listed."""
    from oracle.kv_oracle import ArenaOracle, KVTableOracle, PrefixCacheOracle
    from synapcore_b200 import NativeKVPrefixCache

    rng = np.random.default_rng(11)
    toks = list(range(3, 3 + 97))
    k = (rng.standard_normal((2, 1, 4, 97, 128)) * 0.7).astype(np.float16)
    v = (rng.standard_normal((2, 1, 4, 97, 128)) * 0.7).astype(np.float16)
    for max_pages in (3, 8):
        cache = NativeKVPrefixCache(tmp_path / f"d{max_pages}", None, num_layers=2, num_kv_heads=4, head_dim=128,
                                    max_pages=max_pages, max_disk_blocks=8, quant_mode="int8",
                                    timestamp_fn=lambda: 2.0)
        ora = PrefixCacheOracle(tmp_path / f"o{max_pages}" / "kv_cache_blocks",
                                ArenaOracle(max_pages, 2, 4, 128, "int8"), KVTableOracle(), max_disk_blocks=8)
        assert cache.save_prefix_blocks_numpy(toks, k, v, "cd" * 32) == 6
        assert ora.save(toks, k, v, "cd" * 32, timestamp=lambda: 2.0) == 6
        # drop the arena's tables so every block comes back from disk
        for a in (cache.arena, ora.arena):
            a.page_table.clear()
            a.reverse_page_table.clear()
            a.page_last_used.clear()
            a.free_pages.clear()
            a.free_pages.extend(range(a.max_pages))
        n, kd, vd = cache.match_longest_prefix(toks, "cd" * 32)
        n_o, k_o, v_o = ora.match(toks, "cd" * 32)
        assert n == n_o == 96
        np.testing.assert_array_equal(kd.cpu().numpy(), k_o)
        np.testing.assert_array_equal(vd.cpu().numpy(), v_o)
        assert cache.arena.page_table == ora.arena.page_table
        assert cache.arena.page_last_used == ora.arena.page_last_used
        assert list(cache.arena.free_pages) == list(ora.arena.free_pages)
        assert cache.blocks_loaded_from_disk == ora.blocks_loaded_from_disk == 6


def test_fp16_cache_reloads_int8_blocks_as_dequantised_pages(cuda_device, tmp_path):
    """An fp16 cache over a store written in int8 mode stores
    fp16(q * f32(scale)) for each reloaded block, as the reference's
    write_page_quantized does in fp16 mode."""
    from oracle.kv_oracle import dequantize_kv_int8
    from synapcore_b200 import NativeKVPrefixCache

    rng = np.random.default_rng(12)
    toks = list(range(50, 50 + 65))
    k = rng.standard_normal((2, 1, 4, 65, 128)).astype(np.float16)
    v = rng.standard_normal((2, 1, 4, 65, 128)).astype(np.float16)
    writer = NativeKVPrefixCache(tmp_path, None, num_layers=2, num_kv_heads=4, head_dim=128, max_pages=8,
                                 max_disk_blocks=8, quant_mode="int8", timestamp_fn=lambda: 0.0)
    assert writer.save_prefix_blocks_numpy(toks, k, v, "ef" * 32) == 4
    reader = NativeKVPrefixCache(tmp_path, None, num_layers=2, num_kv_heads=4, head_dim=128, max_pages=8,
                                 max_disk_blocks=8, quant_mode="fp16", timestamp_fn=lambda: 0.0)
    n, kd, vd = reader.match_longest_prefix(toks, "ef" * 32)
    assert n == 64 and reader.blocks_loaded_from_disk == 4
    from synapcore_b200.prefix_cache import chain_merkle_prefix_hash

    prev, want_k, want_v = "ef" * 32, [], []
    for b in range(4):
        cur = chain_merkle_prefix_hash(prev, toks[16 * b:16 * (b + 1)])
        with np.load(reader.kv_dir / f"{cur[:32]}_np.npz") as d:
            want_k.append(dequantize_kv_int8(d["kq"], d["ks"]))
            want_v.append(dequantize_kv_int8(d["vq"], d["vs"]))
        prev = cur
    np.testing.assert_array_equal(kd.cpu().numpy(), np.concatenate(want_k, axis=3))
    np.testing.assert_array_equal(vd.cpu().numpy(), np.concatenate(want_v, axis=3))
