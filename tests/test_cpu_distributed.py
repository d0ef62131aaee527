"""Multi-process host logic on CPU: two `gloo` ranks.

* sequence sharding deals every sequence to exactly one rank;
* KV-head sharding: each rank computes attention for its kv heads only (the
  oracle SDPA stands in for the GPU kernel here), and the all-gather
  reassembles exactly the single-process result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from synapcore_b200.distributed import (HeadShardedOutput, head_range, query_head_range, shard_of,
                                        shard_sequences)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, k, v, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.kv_oracle import sdpa_decode

        B, hq, D = q.shape
        hkv = k.shape[1]
        kvr = head_range(hkv, world, rank)
        qr = query_head_range(hq, hkv, world, rank)
        local = np.stack([sdpa_decode(q[b, qr.start:qr.stop], k[b, kvr.start:kvr.stop], v[b, kvr.start:kvr.stop])
                          for b in range(B)])
        full = HeadShardedOutput(world).gather(torch.from_numpy(local))
        # sequence sharding: every id lands on exactly one rank
        mine = shard_sequences(list(range(37)), world, rank)
        counts = torch.tensor([len(mine)], dtype=torch.int64)
        dist.all_reduce(counts)
        if rank == 0:
            np.savez(out_path, full=full.numpy(), total=counts.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_head_sharded_attention_gather_matches_single_process(tmp_path):
    from oracle.kv_oracle import sdpa_decode

    rng = np.random.default_rng(0)
    B, hq, hkv, T, D = 3, 8, 4, 40, 128
    q = rng.standard_normal((B, hq, D)).astype(np.float32)
    k = rng.standard_normal((B, hkv, T, D)).astype(np.float16)
    v = rng.standard_normal((B, hkv, T, D)).astype(np.float16)
    out = tmp_path / "r0.npz"
    mp.start_processes(_worker, args=(2, _free_port(), q, k, v, str(out)), nprocs=2, join=True,
                       start_method="spawn")
    res = np.load(out)
    ref = np.stack([sdpa_decode(q[b], k[b], v[b]) for b in range(B)])
    np.testing.assert_array_equal(res["full"], ref)
    assert int(res["total"][0]) == 37


def test_shard_helpers():
    assert [shard_of(i, 4) for i in range(6)] == [0, 1, 2, 3, 0, 1]
    ids = list(range(10))
    parts = [shard_sequences(ids, 3, r) for r in range(3)]
    assert sorted(sum(parts, [])) == ids
    assert list(head_range(8, 4, 2)) == [4, 5]
    assert list(query_head_range(32, 8, 4, 1)) == list(range(8, 16))
    with pytest.raises(ValueError):
        head_range(6, 4, 0)
