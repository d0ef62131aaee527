"""Replay of PagedKVArena operation streams recorded from the reference.

tests/golden/make_golden.py drives the reference PagedKVArena
(native/native_engine.py:297-337) through seeded streams of page writes,
lookups and evict_prefix_hash calls and records every returned page id.
`replay` runs the same stream through a page-id-keyed allocator (the
oracle's AllocatorOracle, or the device allocator behind a small adapter)
with the prefix-hash -> page-id map kept here on the host, the way
synapcore_b200.arena keeps it:

  write of a live key    -> touch([pid])        (clock+1, LRU refresh)
  write of a new key     -> alloc(1)            (ring head, else LRU victim)
  lookup hit / miss      -> touch([pid]) / touch([-1])  (the clock ticks on both)
  evict_prefix_hash      -> free([pid])         (ring tail), absent key: nothing

With batch=True, consecutive operations of one kind go out as one call
(runs of writes of keys not live at the run's start as one alloc(n), lookups
as one touch, evictions as one free), which checks that a batched device call
equals the same number of sequential reference operations.
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import numpy as np

WRITE, LOOKUP, EVICT = 0, 1, 2


def replay(ops: np.ndarray, alloc, batch: bool = False) -> Dict[str, int]:
    """Runs `ops` (rows kind, key, expected result) through `alloc`, which has
    alloc(n) -> (ids, victims), touch(ids), free(ids); asserts every result.
    Returns the host-side counters (hits, misses, live page -> key map)."""
    ops = [tuple(int(x) for x in row) for row in np.asarray(ops)]
    key_to_pid: Dict[int, int] = {}
    pid_to_key: Dict[int, int] = {}
    hits = misses = 0
    i, n = 0, len(ops)
    while i < n:
        kind, key, res = ops[i]
        if kind == WRITE and key in key_to_pid:
            pid = key_to_pid[key]
            alloc.touch([pid])
            assert pid == res, (i, "rewrite of a live key", pid, res)
            i += 1
        elif kind == WRITE:
            run: List[Tuple[int, int, int]] = [ops[i]]
            j = i + 1
            if batch:
                keys = {key}
                while j < n and ops[j][0] == WRITE and ops[j][1] not in key_to_pid and ops[j][1] not in keys:
                    keys.add(ops[j][1])
                    run.append(ops[j])
                    j += 1
            ids, victims = alloc.alloc(len(run))
            for (_, k2, r2), pid, vic in zip(run, ids, victims):
                if vic >= 0:
                    old = pid_to_key.pop(vic)
                    del key_to_pid[old]
                assert pid == r2, (i, "allocation", pid, r2)
                key_to_pid[k2] = pid
                pid_to_key[pid] = k2
            i = j
        elif kind == LOOKUP:
            run_ids: List[int] = []
            j = i
            while j < n and ops[j][0] == LOOKUP and (batch or j == i):
                _, k2, r2 = ops[j]
                pid = key_to_pid.get(k2, -1)
                if pid >= 0:
                    hits += 1
                else:
                    misses += 1
                assert pid == r2, (j, "lookup", pid, r2)
                run_ids.append(pid)
                j += 1
            alloc.touch(run_ids)
            i = j
        else:
            run_ids = []
            j = i
            while j < n and ops[j][0] == EVICT and (batch or j == i):
                _, k2, r2 = ops[j]
                pid = key_to_pid.pop(k2, -1)
                if pid >= 0:
                    del pid_to_key[pid]
                    run_ids.append(pid)
                assert int(pid >= 0) == r2, (j, "evict", pid, r2)
                j += 1
            if run_ids:
                alloc.free(run_ids)
            i = j
    return {"hits": hits, "misses": misses, "live": len(key_to_pid)}


def check_final_state(alloc, stream: dict, counters: Dict[str, int], clock: int, evictions: int) -> None:
    """Counters equal the reference arena's; draining the allocator then
    yields the reference's free-list order followed by its live pages in LRU
    order (smallest last-used clock first)."""
    assert counters["hits"] == stream["page_hits"]
    assert counters["misses"] == stream["page_misses"]
    assert clock == stream["step_clock"]
    assert evictions == stream["page_evictions"]
    free = list(stream["free_pages"])
    lru = [int(p) for p, _ in sorted(stream["last_used_by_page"].items(), key=lambda kv: kv[1])]
    assert counters["live"] == len(lru)
    if free:
        ids, victims = alloc.alloc(len(free))
        assert list(ids) == free and all(v < 0 for v in victims)
    if lru:
        ids, victims = alloc.alloc(len(lru))
        assert list(victims) == lru and list(ids) == lru


class OracleAllocator:
    """AllocatorOracle behind the replay interface."""

    def __init__(self, ora):
        self.ora = ora

    def alloc(self, n: int) -> Tuple[Sequence[int], Sequence[int]]:
        return self.ora.alloc(n)

    def touch(self, ids: Sequence[int]) -> None:
        self.ora.touch(ids)

    def free(self, ids: Sequence[int]) -> None:
        self.ora.free(ids)
