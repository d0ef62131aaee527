"""Kernel 5: the on-device allocator against the oracle's restatement of
PagedKVArena's bookkeeping (native/native_engine.py:289-337): FIFO free
ring, step clock, LRU victims, explicit frees to the ring tail — bit-exact
page-id sequences over random operation mixes, plus the decode-step
reservation and pool-exhaustion status."""
import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS, AllocatorOracle

pytestmark = pytest.mark.gpu


def _pool(dev, P):
    from synapcore_b200.pool import KVPool

    return KVPool(1, 1, 128, P, "fp16", device=dev)


def _compare(pool, ora):
    """Counters agree; the ring order and LRU order are checked by draining."""
    st = pool.alloc_state()
    assert st["free"] == len(ora.ring)
    assert st["clock"] == ora.clock
    assert st["evictions"] == ora.evictions
    assert st["allocated"] == int(ora.allocated.sum())
    return st


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_op_mix_matches_reference_allocation_order(cuda_device, seed):
    rng = np.random.default_rng(seed)
    P = int(rng.integers(40, 300))
    pool = _pool(cuda_device, P)
    ora = AllocatorOracle(P)
    for step in range(120):
        op = rng.choice(["alloc", "alloc", "touch", "free", "evict", "pin"])
        if op == "alloc":
            live = int(ora.allocated.sum())
            cand = int(np.count_nonzero(ora.allocated & (ora.pin == 0)))
            n = int(rng.integers(1, max(2, min(P // 3, len(ora.ring) + cand) + 1)))
            if n > len(ora.ring) + cand:
                continue
            pin = bool(rng.random() < 0.2)
            ids, vic = pool.alloc_pages(n, pin=pin)
            e_ids, e_vic = ora.alloc(n, pin=pin)
            assert ids.cpu().tolist() == e_ids, (step, op)
            assert vic.cpu().tolist() == e_vic
        elif op == "touch":
            n = int(rng.integers(1, 20))
            ids = rng.integers(-1, P, size=n).tolist()
            pool.touch_pages(torch.tensor(ids, dtype=torch.int32))
            ora.touch(ids)
        elif op == "free":
            alive = np.nonzero(ora.allocated)[0]
            if alive.size == 0:
                continue
            n = int(rng.integers(1, min(alive.size, 30) + 1))
            ids = rng.choice(alive, size=n, replace=False).tolist()
            ids = ids + ids[: n // 3]  # repeats are skipped
            rng.shuffle(ids)
            pool.free_pages(torch.tensor(ids, dtype=torch.int32))
            ora.free(ids)
        elif op == "evict":
            n = int(rng.integers(1, 12))
            got = pool.evict_lru(n).cpu().tolist()
            assert got == ora.evict_lru(n), step
        else:
            alive = np.nonzero(ora.allocated)[0]
            if alive.size == 0:
                continue
            ids = rng.choice(alive, size=min(5, alive.size), replace=False).tolist()
            delta = 1 if rng.random() < 0.6 else -1
            ok = [i for i in ids if ora.pin[i] + delta >= 0]
            if not ok:
                continue
            pool.pin_pages(torch.tensor(ok, dtype=torch.int32), delta)
            ora.pin_pages(ok, delta)
        _compare(pool, ora)
    assert pool.status()[0] == 0
    # drain: allocating everything left reproduces the ring order and LRU order
    cand = int(np.count_nonzero(ora.allocated & (ora.pin == 0)))
    n = len(ora.ring) + cand
    if n:
        ids, _ = pool.alloc_pages(n)
        assert ids.cpu().tolist() == ora.alloc(n)[0]
    pool.close()


def test_large_batch_eviction_crosses_sort_rounds(cuda_device):
    """More victims than one selection round (4096) in a single call."""
    P = 10000
    pool = _pool(cuda_device, P)
    ora = AllocatorOracle(P)
    ids, _ = pool.alloc_pages(P)
    assert ids.cpu().tolist() == ora.alloc(P)[0]
    rng = np.random.default_rng(9)
    touch = rng.permutation(P)[:7000].tolist()
    pool.touch_pages(torch.tensor(touch, dtype=torch.int32))
    ora.touch(touch)
    ids, vic = pool.alloc_pages(9000)
    e_ids, e_vic = ora.alloc(9000)
    assert ids.cpu().tolist() == e_ids and vic.cpu().tolist() == e_vic
    got = pool.evict_lru(5000).cpu().tolist()
    assert got == ora.evict_lru(5000)
    _compare(pool, ora)
    pool.close()


def test_pool_exhaustion_reports_status_not_fault(cuda_device):
    from synapcore_b200 import SCKVPoolExhausted

    pool = _pool(cuda_device, 16)
    ids, _ = pool.alloc_pages(16, pin=True)
    out, _ = pool.alloc_pages(4)
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [-1] * 4
    with pytest.raises(SCKVPoolExhausted):
        pool.raise_on_status()
    assert pool.status()[0] == 0  # cleared by raise_on_status
    st = pool.alloc_state()
    assert st["allocated"] == 16 and st["free"] == 0
    pool.close()


def test_reserve_decode_matches_sequential_allocation(cuda_device):
    rng = np.random.default_rng(4)
    P, B, max_blocks = 400, 37, 24
    pool = _pool(cuda_device, P)
    ora = AllocatorOracle(P)
    ctx = rng.integers(0, 300, size=B).astype(np.int32)
    ctx[::5] = (ctx[::5] // PAGE_TOKENS) * PAGE_TOKENS  # many sequences at a page boundary
    bt = np.full((B, max_blocks), -1, np.int32)
    bt_d = torch.from_numpy(bt.copy()).to(cuda_device)
    ctx_d = torch.from_numpy(ctx.copy()).to(cuda_device)
    for step in range(40):
        pool.reserve_decode(bt_d, ctx_d)
        ora.reserve_decode(bt, ctx)
        if step % 9 == 4:
            # some sequences finish: free their pages
            done = rng.choice(B, size=3, replace=False)
            for b in done:
                n = (int(ctx[b]) + PAGE_TOKENS - 1) // PAGE_TOKENS
                ids = bt[b, :n].tolist()
                pool.free_pages(torch.tensor(ids, dtype=torch.int32))
                ora.free(ids)
                bt[b] = -1
                ctx[b] = 0
            bt_d.copy_(torch.from_numpy(bt))
            ctx_d.copy_(torch.from_numpy(ctx))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bt_d.cpu().numpy(), bt)
    np.testing.assert_array_equal(ctx_d.cpu().numpy(), ctx)
    assert pool.status()[0] == 0
    _compare(pool, ora)
    pool.close()


def test_reserve_decode_bounds_error_changes_nothing(cuda_device):
    pool = _pool(cuda_device, 64)
    bt = torch.full((2, 2), -1, dtype=torch.int32, device=cuda_device)
    ctx = torch.tensor([32, 3], dtype=torch.int32, device=cuda_device)  # seq 0 is at its block limit
    pool.reserve_decode(bt, ctx)
    torch.cuda.synchronize()
    code, detail, kernel, _ = pool.status()
    assert code == -3 and detail == 0
    assert ctx.cpu().tolist() == [32, 3] and bt.cpu().tolist() == [[-1, -1], [-1, -1]]
    pool.clear_status()
    pool.close()


class _DeviceAllocator:
    """The device allocator (kernel 5) behind the replay interface."""

    def __init__(self, pool):
        self.pool = pool

    def alloc(self, n):
        ids, vic = self.pool.alloc_pages(n)
        return ids.cpu().tolist(), vic.cpu().tolist()

    def touch(self, ids):
        self.pool.touch_pages(torch.tensor(ids, dtype=torch.int32))

    def free(self, ids):
        self.pool.free_pages(torch.tensor(ids, dtype=torch.int32))


@pytest.mark.parametrize("idx", [0, 1, 2])
@pytest.mark.parametrize("batch", [False, True])
def test_device_allocator_replays_reference_arena_streams(cuda_device, idx, batch):
    """Kernel 5 reproduces, page id for page id, the reference PagedKVArena's
    allocations, LRU victims, clock, eviction count, free-list order and LRU
    order over long operation streams recorded from the reference itself
    (tests/golden arena_alloc_streams), issued one operation per call and in
    batched calls (n allocations in one launch = n reference allocations)."""
    import json
    from pathlib import Path

    from arena_replay import check_final_state, replay

    gold_dir = Path(__file__).resolve().parent / "golden"
    st = json.loads((gold_dir / "golden.json").read_text())["arena_alloc_streams"][idx]
    ops = np.load(gold_dir / "golden_arrays.npz")[st["ops"]]
    pool = _pool(cuda_device, st["max_pages"])
    dev = _DeviceAllocator(pool)
    counters = replay(ops, dev, batch=batch)
    state = pool.alloc_state()
    assert state["free"] == len(st["free_pages"])
    assert pool.status()[0] == 0
    check_final_state(dev, st, counters, state["clock"], state["evictions"])
    pool.close()


def test_evict_to_watermark_matches_oracle(cuda_device):
    """sckv_evict_to_watermark decides the eviction count on the device:
    after it at most `limit` pages are allocated (or every unpinned page is
    gone), victims in LRU order, the same as the oracle's restatement."""
    rng = np.random.default_rng(17)
    P = 300
    pool = _pool(cuda_device, P)
    ora = AllocatorOracle(P)
    cnt = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for step in range(60):
        n = int(rng.integers(1, 40))
        cand = int(np.count_nonzero(ora.allocated & (ora.pin == 0)))
        if n <= len(ora.ring) + cand:
            pin = bool(rng.random() < 0.3)
            ids, _ = pool.alloc_pages(n, pin=pin)
            assert ids.cpu().tolist() == ora.alloc(n, pin=pin)[0]
        if rng.random() < 0.4:
            t = rng.integers(0, P, size=10).tolist()
            pool.touch_pages(torch.tensor(t, dtype=torch.int32))
            ora.touch(t)
        if rng.random() < 0.2:
            pinned = np.nonzero(ora.allocated & (ora.pin > 0))[0]
            if pinned.size:
                ids = rng.choice(pinned, size=min(5, pinned.size), replace=False).tolist()
                pool.release_pages(torch.tensor(ids, dtype=torch.int32), keep_cached=True)
                for i in ids:
                    ora.pin[i] -= 1
        limit = int(rng.integers(P // 4, P))
        pool.evict_to_watermark(limit, out_count=cnt)
        exp = ora.evict_to_watermark(limit)
        assert int(cnt.item()) == exp, step
        _compare(pool, ora)
        alloc = int(ora.allocated.sum())
        assert alloc <= limit or not np.any(ora.allocated & (ora.pin == 0))
    assert pool.status()[0] == 0
    pool.close()


def test_paged_cache_watermark_policy(cuda_device):
    """PagedKVCache(evict_watermark=f): finished sequences kept cached are
    evicted LRU first once more than f of the pool is allocated; live
    sequences' pages are never touched."""
    from synapcore_b200.paged_cache import PagedKVCache

    c = PagedKVCache(1, 1, 128, max_pages=100, max_seqs=16, max_blocks_per_seq=16, device=cuda_device,
                     evict_watermark=0.5)
    kv = torch.zeros((1, 160, 1, 128), dtype=torch.float16, device=cuda_device)
    for i in range(8):  # 8 x 10 pages
        c.add_sequence(i)
        c.append_prefill(i, kv, kv)
    c.remove_sequences([0, 1, 2, 3], keep_cached=True)  # 40 cached pages, 40 live
    st = c.pool.alloc_state()
    assert st["allocated"] == 80
    c.enforce_watermark()
    assert c.pool.alloc_state()["allocated"] == 50  # 30 oldest cached pages evicted
    c.enforce_watermark()
    assert c.pool.alloc_state()["allocated"] == 50
    c.remove_sequences([4, 5, 6, 7])  # freed outright
    assert c.pool.alloc_state()["allocated"] == 10
    c.check()
