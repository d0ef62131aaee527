"""Batched PagedKVCache calls (one launch for several new sequences) equal
the per-sequence calls bit for bit: append + causal prefill attention of
newly admitted prompts (one of them sharing a prefix), and releasing several
finished sequences at once."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(dev, kv="fp16"):
    from synapcore_b200.paged_cache import PagedKVCache

    return PagedKVCache(2, 4, 128, max_pages=128, max_seqs=8, max_blocks_per_seq=24, kv_dtype=kv, device=dev)


@pytest.mark.parametrize("kv", ["fp16", "bf16", "fp8_e4m3"])
def test_batched_prefill_equals_per_sequence(cuda_device, kv):
    rng = np.random.default_rng(3)
    L, hkv, hq, D = 2, 4, 16, 128
    dt = torch.float16 if kv == "fp16" else torch.bfloat16
    T = [37, 100, 16, 65]
    tot = sum(T)
    k = torch.from_numpy(rng.standard_normal((L, tot, hkv, D)).astype(np.float32)).to(dt).to(cuda_device)
    v = torch.from_numpy(rng.standard_normal((L, tot, hkv, D)).astype(np.float32)).to(dt).to(cuda_device)
    q = torch.from_numpy(rng.standard_normal((L, tot, hq, D)).astype(np.float32)).to(dt).to(cuda_device)
    pre = torch.from_numpy(rng.standard_normal((L, 32, hkv, D)).astype(np.float32)).to(dt).to(cuda_device)
    cu = np.concatenate([[0], np.cumsum(T)]).tolist()

    outs = []
    for batched in (False, True):
        c = _cache(cuda_device, kv)
        c.add_sequence("p")
        c.append_prefill("p", pre, pre)
        prefix = c.page_ids("p")
        ids = ["a", "b", "c", "d"]
        for sid in ids:
            c.add_sequence(sid)
        c.share_prefix("b", prefix)  # "b" continues the 32-token prefix
        starts = [c.length(s) for s in ids]
        res = torch.empty((L, tot, hq, D), dtype=torch.float32, device=cuda_device)
        if batched:
            c.append_prefill_batch(ids, k, v, cu)
            cu_d = torch.tensor(cu, dtype=torch.int32, device=cuda_device)
            st_d = torch.tensor(starts, dtype=torch.int32, device=cuda_device)
            for l in range(L):
                res[l] = c.prefill_attention_batch(l, ids, q[l], cu_d, st_d, out_dtype=torch.float32)
        else:
            for i, sid in enumerate(ids):
                c.append_prefill(sid, k[:, cu[i]:cu[i + 1]], v[:, cu[i]:cu[i + 1]])
            for l in range(L):
                for i, sid in enumerate(ids):
                    res[l, cu[i]:cu[i + 1]] = c.prefill_attention(l, sid, q[l, cu[i]:cu[i + 1]], starts[i],
                                                                  out_dtype=torch.float32)
        torch.cuda.synchronize()
        c.check()
        kk, vv = zip(*[c.gather(s) for s in ids])
        outs.append((res.cpu(), [x.cpu() for x in kk], [x.cpu() for x in vv], [c.length(s) for s in ids]))
        c.pool.close()
    (r0, k0, v0, n0), (r1, k1, v1, n1) = outs
    assert n0 == n1
    assert torch.equal(r0, r1)
    for a, b in zip(k0 + v0, k1 + v1):
        assert torch.equal(a, b)


def test_remove_sequences_equals_sequential_removal(cuda_device):
    rng = np.random.default_rng(4)
    states = []
    for batched in (False, True):
        c = _cache(cuda_device)
        for i, T in enumerate([20, 50, 33, 16, 90]):
            c.add_sequence(i)
            x = torch.from_numpy(rng.standard_normal((2, T, 4, 128)).astype(np.float16)).to(cuda_device)
            c.append_prefill(i, x, x)
        c.fork(1, 9)
        gone = [3, 1, 0]
        if batched:
            c.remove_sequences(gone, keep_cached=True)
        else:
            for s in gone:
                c.remove_sequence(s, keep_cached=True)
        torch.cuda.synchronize()
        c.check()
        st = c.pool.alloc_state()
        pins = c.pool.alloc_region  # raw allocator region (ring, clocks, pins, states)
        states.append((st, list(c.seq_at), [c.page_ids(s) for s in c.seq_at], pins.cpu().clone()))
        c.pool.close()
        rng = np.random.default_rng(4)
    a, b = states
    assert a[0] == b[0] and a[1] == b[1] and a[2] == b[2]
    assert torch.equal(a[3], b[3])
