#!/usr/bin/env python3
"""Generate golden fixtures by running the reference's own Python code.

    python tests/golden/make_golden.py --reference <reference checkout>
    (or set SCKV_REFERENCE_DIR)

Imports the reference's PagedKVArena, NativeKVPrefixCache, int8 KV
quantisation, prefix-chain hash, KV hash-table twin, ModularAttentionEngine
and FP8 LUT from the reference checkout (read-only), replays the scenarios of
its own tests (tests/test_p1_2_paged_kv_cache.py T1-T4, the C++ self-test
--verify-kv-eviction at native/synapcore_native.mm:1365-1414,
tests/test_reliability.py::test_06) plus decode-SDPA cases, and writes the
observed outputs to tests/golden/. Large arrays are recorded as SHA-256
digests of their bytes (inputs are regenerated from the same seeds by the
tests); small ones are stored in golden_arrays.npz.

Only this script reads the reference; the fixtures it writes are what the
tests use, so they run anywhere.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import struct
import sys
import tempfile
import threading
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def stand_in_bridge(ne):
    """NativeMmapIndexBridge without a store: a zeroed index image in memory,
    using the reference's own kv_lookup / kv_insert methods."""
    b = ne.NativeMmapIndexBridge.__new__(ne.NativeMmapIndexBridge)
    b.idx_mmap = bytearray(ne.TOTAL_IDX_BYTES)
    b.idx_lock = threading.RLock()
    b.kv_evictions_issued = 0
    return b


GOLDEN_SEED_ROOT = hashlib.sha256(b"synapcore-b200 golden seed root").hexdigest()


def arena_t1(ne):
    """tests/test_p1_2_paged_kv_cache.py:51-99 replayed, recording every return."""
    arena = ne.PagedKVArena(max_pages=8, num_layers=16, num_kv_heads=16, head_dim=128, quant_mode="fp16")
    rng = np.random.default_rng(101)
    written, log = [], []
    for i in range(12):
        h = f"{i + 1:064x}"
        k = rng.standard_normal((16, 1, 16, 16, 128)).astype(np.float16)
        v = rng.standard_normal((16, 1, 16, 16, 128)).astype(np.float16)
        written.append(h)
        log.append(["write", h, arena.write_page_fp16(h, k, v)])
        if i >= 2:
            log.append(["lookup", written[0], arena.lookup_page_id(written[0])])
            log.append(["lookup", written[1], arena.lookup_page_id(written[1])])
    for idx in (0, 1, 2, 3, 4, 5):
        log.append(["lookup", written[idx], arena.lookup_page_id(written[idx])])
    surv = [0, 1, 6, 7, 8, 9, 10, 11]
    pids = [arena.lookup_page_id(written[i]) for i in surv]
    kc, vc = arena.gather_contiguous_kv_numpy(pids)
    return {
        "log": log,
        "survivor_pids": pids,
        "page_table": dict(arena.page_table),
        "page_last_used": dict(arena.page_last_used),
        "free_pages": list(arena.free_pages),
        "step_clock": arena.step_clock,
        "page_hits": arena.page_hits,
        "page_misses": arena.page_misses,
        "page_evictions": arena.page_evictions,
        "gather_shape": list(kc.shape),
        "gather_k_sha256": sha(kc),
        "gather_v_sha256": sha(vc),
    }


def int8_t3(ne, arrays):
    """tests/test_p1_2_paged_kv_cache.py:117-147."""
    a16 = ne.PagedKVArena(max_pages=16, quant_mode="fp16")
    a8 = ne.PagedKVArena(max_pages=16, quant_mode="int8")
    rng = np.random.default_rng(2026)
    k = (rng.standard_normal((16, 1, 16, 16, 128)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((16, 1, 16, 16, 128)) * 0.5).astype(np.float16)
    pid = a8.write_page_fp16("a" * 64, k, v)
    kd, vd = a8.read_page_fp16(pid)
    kq, ks = ne.quantize_kv_int8_numpy(k)
    kf, kdf = k.astype(np.float32).reshape(-1), kd.astype(np.float32).reshape(-1)
    small = (np.random.default_rng(7).standard_normal((2, 1, 3, 16, 128)) * 3).astype(np.float16)
    small[0, 0, 0, 0] = 0  # all-zero row -> scale floor 1e-7
    sq, ss = ne.quantize_kv_int8_numpy(small)
    arrays["int8_small_x"] = small
    arrays["int8_small_q"] = sq
    arrays["int8_small_s"] = ss
    arrays["int8_small_deq"] = ne.dequantize_kv_int8_numpy(sq, ss)
    return {
        "bytes_per_page_fp16": a16.bytes_per_page,
        "bytes_per_page_int8": a8.bytes_per_page,
        "kq_sha256": sha(kq),
        "ks_sha256": sha(ks),
        "k_pool_q_sha256": sha(a8.k_pool_q[pid]),
        "k_scale_sha256": sha(a8.k_scale[pid]),
        "k_deq_sha256": sha(kd),
        "v_deq_sha256": sha(vd),
        "cosine": float(np.dot(kf, kdf) / (np.linalg.norm(kf) * np.linalg.norm(kdf))),
        "mean_abs_err": float(np.mean(np.abs(kf - kdf))),
    }


def prefix_cache_t4(ne):
    """tests/test_p1_2_paged_kv_cache.py:149-222 with a stand-in bridge.
    save_prefix_blocks_numpy stamps hash-table slots with time.time()
    (native/native_engine.py:2231); a fixed clock (0.0) is substituted inside
    the reference module so the table bytes are reproducible."""
    import types
    import time as _time

    ne.time = types.SimpleNamespace(time=lambda: 0.0, perf_counter=_time.perf_counter)
    tmp = Path(tempfile.mkdtemp(prefix="sckv_golden_"))
    try:
        bridge = stand_in_bridge(ne)
        cache = ne.NativeKVPrefixCache(tmp, bridge, device="cpu", num_layers=16, num_kv_heads=16, head_dim=128,
                                       max_pages=4, max_disk_blocks=3, quant_mode="int8")
        rng = np.random.default_rng(77)
        tokens = list(range(100, 165))
        k = (rng.standard_normal((16, 1, 16, 65, 128)) * 0.4).astype(np.float16)
        v = (rng.standard_normal((16, 1, 16, 65, 128)) * 0.4).astype(np.float16)
        seed = GOLDEN_SEED_ROOT
        saved = cache.save_prefix_blocks_numpy(tokens, k, v, seed)
        after_save = {"saved_pages": saved, "disk_blocks_evicted": cache.disk_blocks_evicted,
                      "files": sorted(p.name for p in cache.kv_dir.iterdir())}
        short = tokens[:49]
        cache.save_prefix_blocks_numpy(short, k[:, :, :, :49], v[:, :, :, :49], seed)
        hits0 = cache.blocks_loaded_from_arena
        m1, k1, v1 = cache.match_longest_prefix_numpy(short, seed)
        arena_hits = cache.blocks_loaded_from_arena - hits0
        cache.arena.page_table.clear()
        cache.arena.reverse_page_table.clear()
        cache.arena.free_pages.clear()
        cache.arena.free_pages.extend(range(cache.arena.max_pages))
        m2, k2, v2 = cache.match_longest_prefix_numpy(short, seed)
        stats = cache.get_paged_kv_stats()
        return {
            "seed_root": seed,
            "after_first_save": after_save,
            "matched_arena": m1,
            "arena_hits": arena_hits,
            "k_restored_shape": list(k1.shape),
            "k_restored_sha256": sha(k1),
            "v_restored_sha256": sha(v1),
            "matched_disk": m2,
            "k_disk_sha256": sha(k2),
            "v_disk_sha256": sha(v2),
            "blocks_loaded_from_disk": cache.blocks_loaded_from_disk,
            "blocks_loaded_from_arena": cache.blocks_loaded_from_arena,
            "blocks_saved_to_disk": cache.blocks_saved_to_disk,
            "tokens_skipped": cache.tokens_skipped,
            "stats": stats,
            "files_end": sorted(p.name for p in cache.kv_dir.iterdir()),
            "kv_table_sha256": hashlib.sha256(bytes(bridge.idx_mmap[ne.OFFSET_KV_HASH_TBL:])).hexdigest(),
        }
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
        ne.time = _time


def kv_table_kat(ne):
    """--verify-kv-eviction (native/synapcore_native.mm:1365-1414) through the
    Python twin (native/native_engine.py:1714-1752)."""
    b = stand_in_bridge(ne)
    parent = b"\x00" * 32
    hashes, evicted, rcs = [], [], []
    for i in range(100):
        h = bytearray(32)
        struct.pack_into("<I", h, 0, 77 | ((i + 1) << 10))
        h[4] = i & 0xFF
        h = bytes(h)
        hashes.append(h)
        ev = b.kv_insert(h, parent, (i + 1) * 16, 1000.0 + i)
        evicted.append(ev)
    old_found = sum(b.kv_lookup(h) for h in hashes[:36])
    new_found = sum(b.kv_lookup(h) for h in hashes[36:])
    return {
        "evictions": b.kv_evictions_issued,
        "old_found": old_found,
        "new_found": new_found,
        "evicted_hashes": evicted,
        "table_sha256": hashlib.sha256(bytes(b.idx_mmap[ne.OFFSET_KV_HASH_TBL:])).hexdigest(),
    }


def kv_table_long_context(ne):
    """tests/test_reliability.py:213-259 with fixed timestamps (the test uses time.time())."""
    b = stand_in_bridge(ne)
    prev = GOLDEN_SEED_ROOT
    chain = []
    for bi in range(260):
        toks = [((bi * 16) + t) % 50000 for t in range(16)]
        cur = ne.chain_merkle_prefix_hash(prev, toks)
        b.kv_insert(bytes.fromhex(cur), bytes.fromhex(prev), (bi + 1) * 16, 5000.0 + bi * 0.001)
        chain.append(cur)
        prev = cur
    recent_found = [bool(b.kv_lookup(bytes.fromhex(h))) for h in chain[-128:]]
    evs = []
    for c in range(70):
        h = struct.pack("<I", 42) + struct.pack("<I", c + 1) + b"\x11" * 24
        evs.append(b.kv_insert(h, b"\x00" * 32, (c + 1) * 16, 1000.0 + c))
    newest = struct.pack("<I", 42) + struct.pack("<I", 70) + b"\x11" * 24
    oldest = struct.pack("<I", 42) + struct.pack("<I", 1) + b"\x11" * 24
    return {
        "chain_first": chain[0],
        "chain_last": chain[-1],
        "recent_found": recent_found,
        "collision_evicted": evs,
        "newest_found": bool(b.kv_lookup(newest)),
        "oldest_found": bool(b.kv_lookup(oldest)),
        "evictions": b.kv_evictions_issued,
        "table_sha256": hashlib.sha256(bytes(b.idx_mmap[ne.OFFSET_KV_HASH_TBL:])).hexdigest(),
    }


def kv_table_unordered_timestamps(ne):
    """Probe windows whose created_at values compare false (NaN) or never
    below +inf: the Python twin overwrites the home slot, counts an eviction
    and names no evicted hash (native/native_engine.py:1741-1752)."""
    out = {}
    for name, ts_fill in (("nan", float("nan")), ("inf", float("inf")), ("mixed", None)):
        b = stand_in_bridge(ne)
        rets = []
        for c in range(64):
            h = struct.pack("<I", 300 | ((c + 1) << 10)) + bytes([c]) + b"\x22" * 27
            ts = ts_fill if ts_fill is not None else (float("nan") if c % 3 else float("inf"))
            rets.append(b.kv_insert(h, b"\x00" * 32, (c + 1) * 16, ts))
        for c in range(3):
            h = struct.pack("<I", 300 | ((c + 100) << 10)) + b"\x33" * 28
            rets.append(b.kv_insert(h, b"\x01" * 32, 7 + c, 50.0 + c))
        out[name] = {
            "returns": rets,
            "evictions": b.kv_evictions_issued,
            "table_sha256": hashlib.sha256(bytes(b.idx_mmap[ne.OFFSET_KV_HASH_TBL:])).hexdigest(),
        }
    return out


def arena_alloc_streams(ne, arrays):
    """PagedKVArena's page-id bookkeeping (native/native_engine.py:297-337)
    over long seeded operation streams: writes of new keys (FIFO free list,
    then LRU victims), rewrites of live keys (a touch), lookups that hit and
    miss (the clock ticks on both), and evict_prefix_hash of live and absent
    keys. Every returned page id / bool is recorded with the final counters,
    free-list order and clocks, so a page-id-keyed allocator can be replayed
    against it op for op."""
    streams = []
    for seed, max_pages, n_ops in ((11, 40, 1500), (12, 97, 2500), (13, 300, 4000)):
        rng = np.random.default_rng(seed)
        arena = ne.PagedKVArena(max_pages=max_pages, num_layers=1, num_kv_heads=1, head_dim=8, quant_mode="fp16")
        page = np.zeros((1, 1, 1, 16, 8), np.float16)
        next_key = 0
        seen = []
        ops = []
        for _ in range(n_ops):
            r = rng.random()
            live = [int(h, 16) for h in arena.page_table.keys()]
            if r < 0.45 or not seen:
                if rng.random() < 0.1 and seen:
                    key = seen[int(rng.integers(0, len(seen)))]  # live or evicted earlier
                else:
                    key = next_key
                    next_key += 1
                    seen.append(key)
                ops.append((0, key, int(arena.write_page_fp16(f"{key:064x}", page, page))))
            elif r < 0.8:
                if rng.random() < 0.6 and live:
                    key = live[int(rng.integers(0, len(live)))]
                elif rng.random() < 0.5:
                    key = seen[int(rng.integers(0, len(seen)))]
                else:
                    key = 10**9 + int(rng.integers(0, 10**6))  # never written
                pid = arena.lookup_page_id(f"{key:064x}")
                ops.append((1, key, -1 if pid is None else int(pid)))
            else:
                if rng.random() < 0.8 and live:
                    key = live[int(rng.integers(0, len(live)))]
                else:
                    key = seen[int(rng.integers(0, len(seen)))]
                ops.append((2, key, int(bool(arena.evict_prefix_hash(f"{key:064x}")))))
        arrays[f"arena_stream_{seed}_ops"] = np.asarray(ops, np.int64)
        streams.append({
            "seed": seed,
            "max_pages": max_pages,
            "ops": f"arena_stream_{seed}_ops",
            "step_clock": arena.step_clock,
            "page_hits": arena.page_hits,
            "page_misses": arena.page_misses,
            "page_evictions": arena.page_evictions,
            "free_pages": list(map(int, arena.free_pages)),
            "last_used_by_page": {str(arena.page_table[h]): int(c) for h, c in arena.page_last_used.items()},
        })
    return streams


def sdpa_cases(ad, arrays):
    """Decode SDPA through ModularAttentionEngine.forward_numpy
    (models/adapters.py:1148-1231) with identity q/o projections, zero k/v
    projections and pos_offset 0 (RoPE angle 0): output = SDPA of q over the
    cached K/V followed by one all-zero token."""
    out = []
    for name, hq, hkv, T, seed in (("mha", 4, 4, 37, 1), ("gqa4", 8, 2, 70, 2), ("mqa", 4, 1, 16, 3),
                                   ("gqa8_long", 16, 2, 301, 4)):
        d = 128
        hidden = hq * d
        cfg = {"model_type": "mixtral", "num_hidden_layers": 1, "num_experts": 8, "num_experts_per_tok": 2,
               "hidden_size": hidden, "intermediate_size": hidden * 2, "num_attention_heads": hq,
               "num_key_value_heads": hkv, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 10000.0}
        eng = ad.ModularAttentionEngine(ad.MixtralAdapter(cfg).spec)
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((1, 1, hidden)).astype(np.float32)
        pk = rng.standard_normal((1, hkv, T, d)).astype(np.float16)
        pv = rng.standard_normal((1, hkv, T, d)).astype(np.float16)
        qw = np.eye(hidden, dtype=np.float16)
        kw = np.zeros((hkv * d, hidden), np.float16)
        ow = np.eye(hidden, dtype=np.float16)
        kk, vv = [pk.copy()], [pv.copy()]
        y = eng.forward_numpy(x, qw, kw, kw, ow, kv_cache_k=kk, kv_cache_v=vv, layer_idx=0, pos_offset=0)
        arrays[f"sdpa_{name}_q"] = x.reshape(hq, d)
        arrays[f"sdpa_{name}_k"] = pk[0]
        arrays[f"sdpa_{name}_v"] = pv[0]
        arrays[f"sdpa_{name}_out"] = y.reshape(hq, d)
        arrays[f"sdpa_{name}_kfull"] = kk[0][0]
        out.append({"name": name, "hq": hq, "hkv": hkv, "T": T, "appended_tokens": int(kk[0].shape[2] - T)})
    return out


def qk_rope_cases(ad, arrays):
    """QK-norm + RoPE as forward_numpy composes them (models/adapters.py:
    1171-1195), through the reference engine's own rmsnorm_f32 and
    apply_rope_f32: per-head norm (Qwen3 style), whole-projection norm
    (OLMoE style), and no norm with a RoPE scaling factor."""
    out = []
    for name, hq, hkv, T, pos, theta, scaling, norm, seed in (
            ("perhead", 8, 2, 5, 37, 1000000.0, 1.0, "head", 11),
            ("fullwidth", 4, 4, 3, 4090, 10000.0, 1.0, "full", 12),
            ("nonorm_scaled", 4, 1, 4, 20000, 500000.0, 2.0, None, 13)):
        d = 128
        hidden = hq * d
        cfg = {"model_type": "mixtral", "num_hidden_layers": 1, "num_experts": 8, "num_experts_per_tok": 2,
               "hidden_size": hidden, "intermediate_size": hidden * 2, "num_attention_heads": hq,
               "num_key_value_heads": hkv, "vocab_size": 32000, "rms_norm_eps": 1e-6, "rope_theta": theta}
        eng = ad.ModularAttentionEngine(ad.MixtralAdapter(cfg).spec)
        eng.rope_scaling_factor = scaling
        rng = np.random.default_rng(seed)
        q = rng.standard_normal((1, T, hq * d)).astype(np.float32) * 3
        k = rng.standard_normal((1, T, hkv * d)).astype(np.float32) * 3
        if norm == "head":
            qw = rng.uniform(0.5, 1.5, d).astype(np.float16)
            kw = rng.uniform(0.5, 1.5, d).astype(np.float16)
            qn = eng.rmsnorm_f32(q.reshape(1, T, hq, d), qw).reshape(1, T, hq * d)
            kn = eng.rmsnorm_f32(k.reshape(1, T, hkv, d), kw).reshape(1, T, hkv * d)
        elif norm == "full":
            qw = rng.uniform(0.5, 1.5, hq * d).astype(np.float16)
            kw = rng.uniform(0.5, 1.5, hkv * d).astype(np.float16)
            qn, kn = eng.rmsnorm_f32(q, qw), eng.rmsnorm_f32(k, kw)
        else:
            qw = kw = None
            qn, kn = q, k
        qr = eng.apply_rope_f32(qn.reshape(1, T, hq, d).transpose(0, 2, 1, 3), pos_offset=pos)
        kr = eng.apply_rope_f32(kn.reshape(1, T, hkv, d).transpose(0, 2, 1, 3), pos_offset=pos)
        arrays[f"rope_{name}_q"] = q.reshape(T, hq, d)
        arrays[f"rope_{name}_k"] = k.reshape(T, hkv, d)
        if qw is not None:
            arrays[f"rope_{name}_qw"] = qw
            arrays[f"rope_{name}_kw"] = kw
        arrays[f"rope_{name}_inv_freq"] = eng.rope_inv_freq
        arrays[f"rope_{name}_q_rot"] = qr[0].transpose(1, 0, 2)
        arrays[f"rope_{name}_k_cache"] = kr[0].transpose(1, 0, 2).astype(np.float16)
        out.append({"name": name, "hq": hq, "hkv": hkv, "T": T, "pos": pos, "theta": theta, "scaling": scaling,
                    "norm": norm, "eps": 1e-6})
    return out


def attention_layer_cases(ad, arrays):
    """A whole attention layer through ModularAttentionEngine.forward_numpy
    (models/adapters.py:1148-1231): q/k/v projections with random fp16
    weights, QK-norm (per head, whole width, or none) with the adapter's
    eps, RoPE from the cached prefix's length, the fp16 cache concat, causal
    SDPA (none for one token) and o_proj. Records the layer output and the
    cache entries the call appended; the inputs come from seeds
    (attn_layer_inputs.py, which the tests use too) and are recorded as
    digests."""
    sys.path.insert(0, str(OUT))
    from attn_layer_inputs import ATTN_LAYER_CASES, attn_layer_inputs  # noqa: E402

    adapters = {"qwen2_moe": ad.QwenMoEAdapter, "olmoe": ad.OLMoEAdapter, "mixtral": ad.MixtralAdapter}
    out = []
    for name, kind, hq, hkv, prefix, T, norm, theta, seed in ATTN_LAYER_CASES:
        d = 128
        hidden = hq * d
        cfg = {"model_type": kind, "num_hidden_layers": 1, "num_experts": 8, "num_experts_per_tok": 2,
               "hidden_size": hidden, "intermediate_size": hidden * 2, "moe_intermediate_size": hidden * 2,
               "num_attention_heads": hq, "num_key_value_heads": hkv, "vocab_size": 32000,
               "rms_norm_eps": 1e-6, "rope_theta": theta, "use_qk_norm": norm is not None}
        eng = ad.ModularAttentionEngine(adapters[kind](cfg).spec)
        inp = attn_layer_inputs(hq, hkv, prefix, T, norm, seed)
        kk = [inp["pk"][None].copy() if prefix else None]
        vv = [inp["pv"][None].copy() if prefix else None]
        y = eng.forward_numpy(inp["x"][None], inp["wq"], inp["wk"], inp["wv"], inp["wo"], q_norm_w_fp16=inp["qn"],
                              k_norm_w_fp16=inp["kn"], kv_cache_k=kk, kv_cache_v=vv, layer_idx=0,
                              pos_offset=prefix)
        arrays[f"attn_layer_{name}_out"] = y[0].astype(np.float32)
        arrays[f"attn_layer_{name}_k_new"] = kk[0][0][:, prefix:]
        arrays[f"attn_layer_{name}_v_new"] = vv[0][0][:, prefix:]
        out.append({"name": name, "adapter": kind, "hq": hq, "hkv": hkv, "prefix": prefix, "T": T, "norm": norm,
                    "theta": theta, "seed": seed, "eps": float(eng.rms_eps),
                    "has_qk_norm": bool(eng.has_qk_norm), "scale": float(eng.scale),
                    "inputs_sha256": {k: sha(v) for k, v in inp.items() if v is not None}})
    return out


def _stub_engine(ne, ad, w, c, tmp):
    """A stub of the reference engine carrying the seeded weights of
    tests/stub_model.py: real ModularAttentionEngine attention, real
    NativeKVPrefixCache (stand-in bridge), one routed expert."""
    import types

    cfg = {"model_type": "olmoe", "num_hidden_layers": c["num_layers"], "num_experts": 1, "num_experts_per_tok": 1,
           "hidden_size": c["hidden"], "intermediate_size": c["inter"], "num_attention_heads": c["hq"],
           "num_key_value_heads": c["hkv"], "vocab_size": c["vocab"], "rms_norm_eps": c["rms_eps"],
           "rope_theta": c["rope_theta"], "eos_token_id": 50279}
    eng = types.SimpleNamespace()
    eng.config = cfg
    eng.num_layers = c["num_layers"]
    eng.hidden_size = c["hidden"]
    eng.rms_eps = c["rms_eps"]
    eng.top_k = 1
    eng.enable_merkle_kv = True
    eng.active_merkle_root = GOLDEN_SEED_ROOT
    eng.adapter = ad.OLMoEAdapter(cfg)
    eng.attention_engine = ad.ModularAttentionEngine(eng.adapter.spec)
    eng.kv_prefix_cache = ne.NativeKVPrefixCache(tmp, stand_in_bridge(ne), device="cpu",
                                                 num_layers=c["num_layers"], num_kv_heads=c["hkv"],
                                                 head_dim=c["head_dim"], max_pages=64, quant_mode="fp16")
    eng.emb_np_view = w["emb"]
    eng.lm_head_w_int8_view = w["lm_w_int8"]
    eng.lm_head_s_fp16_view = w["lm_s_fp16"]
    eng.core_np_views = {k: v for k, v in w.items() if k.startswith("model.")}
    eng.live_routing_buffer = types.SimpleNamespace(record_numpy_layer=lambda l, idx: None)
    eng._rmsnorm_numpy = types.MethodType(ne.NativeMerkleMoEEngine._rmsnorm_numpy, eng)
    eng.forward_attention_layer_numpy = types.MethodType(ne.NativeMerkleMoEEngine.forward_attention_layer_numpy,
                                                         eng)
    eng.load_or_get_expert_entry = lambda l, e, is_prefetch=False: types.SimpleNamespace(
        gate_w=w[f"model.layers.{l}.expert.gate"], up_w=w[f"model.layers.{l}.expert.up"],
        down_w=w[f"model.layers.{l}.expert.down"])
    return eng


def scheduler_runs(ne, ad, arrays):
    """The reference ContinuousBatchScheduler (engine/scheduler.py) over the
    stub engine. Runs the six requests batched (max_batch_size 4), isolated,
    and batched over the first layer only (max_layers=1)."""
    import time as _time
    import types

    sys.path.insert(0, str(OUT.parent))
    from stub_model import CFG, make_weights, prompts  # noqa: E402
    from engine import scheduler as sch  # noqa: E402

    w = make_weights()
    ne.time = types.SimpleNamespace(time=lambda: 0.0, perf_counter=_time.perf_counter)
    ps = prompts()
    out = {"prompts": ps}
    try:
        for mode, mbs, max_layers in (("batched", 4, None), ("isolated", 1, None), ("batched_1layer", 4, 1)):
            tmp = Path(tempfile.mkdtemp(prefix="sckv_sched_"))
            eng = _stub_engine(ne, ad, w, CFG, tmp)
            s_ = sch.ContinuousBatchScheduler(eng, max_batch_size=mbs)
            for i, pr in enumerate(ps):
                s_.submit_request(f"req_{i}", pr, max_new_tokens=5, stop_token_ids=set())
            steps = s_.run_until_complete_numpy(max_layers=max_layers)
            done = s_.completed_requests
            out[mode] = {
                "generated": {k: list(map(int, v.generated_ids)) for k, v in done.items()},
                "prefix_skipped": {k: int(v.kv_prefix_skipped) for k, v in done.items()},
                "tokens_skipped": int(eng.kv_prefix_cache.tokens_skipped),
                "blocks_loaded_from_arena": int(eng.kv_prefix_cache.blocks_loaded_from_arena),
                "steps": len(steps),
                "batch_sizes": [int(st["batch_size"]) for st in steps],
                "unique_expert_dispatches": int(s_.total_unique_expert_dispatches),
                "naive_expert_dispatches": int(s_.total_naive_expert_dispatches),
            }
            for k, v in done.items():
                arrays[f"sched_{mode}_{k}_logits"] = v.last_logits.astype(np.float32)
            shutil.rmtree(tmp, ignore_errors=True)
    finally:
        ne.time = _time
    return out


def scheduler_benchmark(ne, ad):
    """The body of benchmark_continuous_batch_scheduler
    (engine/scheduler.py:391-481) over the stub engine (the benchmark itself
    builds a NativeMerkleMoEEngine from a model store this checkout does not
    ship): the reference's prompts, each request alone with max_batch_size=1,
    then all four together; one engine shared by all runs, as there."""
    import time as _time
    import types

    sys.path.insert(0, str(OUT.parent))
    from stub_model import BENCH_CFG, make_weights  # noqa: E402
    from engine import scheduler as sch  # noqa: E402

    w = make_weights(cfg=BENCH_CFG)
    ne.time = types.SimpleNamespace(time=lambda: 0.0, perf_counter=_time.perf_counter)
    tmp = Path(tempfile.mkdtemp(prefix="sckv_bench_"))
    try:
        eng = _stub_engine(ne, ad, w, BENCH_CFG, tmp)
        num_requests, max_new_tokens, max_layers = 4, 3, 2
        shared_prefix = [1, 512, 1024, 2048, 4096, 8192, 12, 34, 56, 78, 90, 111, 222, 333, 444, 555]
        prompts = [shared_prefix + [100 + r, 200 + r] for r in range(num_requests)]
        seq_tokens, seq_logits = {}, {}
        for r, p_ids in enumerate(prompts):
            single = sch.ContinuousBatchScheduler(eng, max_batch_size=1)
            single.submit_request(f"req_{r}", p_ids, max_new_tokens=max_new_tokens, stop_token_ids=set())
            single.run_until_complete_numpy(max_layers=max_layers)
            d = single.completed_requests[f"req_{r}"]
            seq_tokens[f"req_{r}"] = list(map(int, d.generated_ids))
            seq_logits[f"req_{r}"] = d.last_logits.copy()
        batch = sch.ContinuousBatchScheduler(eng, max_batch_size=num_requests)
        for r, p_ids in enumerate(prompts):
            batch.submit_request(f"req_{r}", p_ids, max_new_tokens=max_new_tokens, stop_token_ids=set())
        steps = batch.run_until_complete_numpy(max_layers=max_layers)
        err = max(float(np.max(np.abs(batch.completed_requests[k].last_logits - seq_logits[k]))) for k in seq_logits)
        uniq, naive = batch.total_unique_expert_dispatches, batch.total_naive_expert_dispatches
        return {
            "seq_tokens": seq_tokens,
            "batch_tokens": {k: list(map(int, v.generated_ids)) for k, v in batch.completed_requests.items()},
            "total_requests_completed": len(batch.completed_requests),
            "total_tokens_generated": int(batch.total_tokens_generated),
            "max_concurrent_batch_size": max(int(st["batch_size"]) for st in steps),
            "total_batch_steps": len(steps),
            "total_unique_expert_dispatches": int(uniq),
            "total_naive_expert_dispatches": int(naive),
            "cross_request_expert_sharing_pct": round(100.0 * (1.0 - uniq / max(1, naive)), 2),
            "paged_kv_prefix_tokens_skipped": int(eng.kv_prefix_cache.tokens_skipped),
            "numerical_parity_max_abs_err": round(err, 8),
        }
    finally:
        ne.time = _time
        shutil.rmtree(tmp, ignore_errors=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SCKV_REFERENCE_DIR"),
                    help="path of the reference checkout (default: $SCKV_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or SCKV_REFERENCE_DIR) is required")
    sys.path.insert(0, args.reference)
    from native import native_engine as ne  # noqa: E402
    from models import adapters as ad  # noqa: E402

    arrays = {}
    golden = {
        "generator": "tests/golden/make_golden.py (reference code run in-process)",
        "arena_t1": arena_t1(ne),
        "int8_t3": int8_t3(ne, arrays),
        "prefix_cache_t4": prefix_cache_t4(ne),
        "kv_table_kat": kv_table_kat(ne),
        "kv_table_long_context": kv_table_long_context(ne),
        "kv_table_unordered_timestamps": kv_table_unordered_timestamps(ne),
        "arena_alloc_streams": arena_alloc_streams(ne, arrays),
        "sdpa": sdpa_cases(ad, arrays),
        "scheduler": scheduler_runs(ne, ad, arrays),
        "scheduler_benchmark": scheduler_benchmark(ne, ad),
        "qk_rope": qk_rope_cases(ad, arrays),
        "attention_layer": attention_layer_cases(ad, arrays),
        "chain_hash": [ne.chain_merkle_prefix_hash(GOLDEN_SEED_ROOT, list(range(16))),
                       ne.chain_merkle_prefix_hash("00" * 32, [0] * 16),
                       ne.chain_merkle_prefix_hash("ff" * 32, [4294967295] * 16)],
    }
    arrays["fp8_lut"] = ad.fp8_e4m3_bytes_to_fp32(np.arange(256, dtype=np.uint8))
    (OUT / "golden.json").write_text(json.dumps(golden, indent=1, sort_keys=True))
    np.savez_compressed(OUT / "golden_arrays.npz", **arrays)
    print("wrote", OUT / "golden.json", OUT / "golden_arrays.npz")


if __name__ == "__main__":
    main()
