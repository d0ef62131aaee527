"""Limits of the paging and attention kernels: sequences that fill their
block table to the last slot, the last page id of the pool, the largest
head group the kernels build (G = 16), long split-K contexts with an exact
multiple of the split size, and the append of a token into the final slot
of a full table. Results against the oracle (bit-exact for pages,
2e-3 relative for attention)."""
import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS, PagedPoolOracle

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _rel(o, r):
    return float(np.max(np.abs(o - r)) / max(np.max(np.abs(r)), 1e-30))


@pytest.mark.parametrize("kv_dtype,hq,hkv,qdt", [("fp16", 16, 16, torch.float16), ("fp16", 32, 2, torch.float16),
                                                 ("bf16", 32, 2, torch.bfloat16), ("fp8_e4m3", 64, 4, torch.bfloat16)])
def test_full_block_tables_and_last_page(cuda_device, kv_dtype, hq, hkv, qdt):
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(3)
    D, P, L = 128, 96, 1
    mb = 24  # 384 tokens per sequence at most
    pool = KVPool(L, hkv, D, P, kv_dtype, device=cuda_device)
    ora = PagedPoolOracle(L, hkv, D, P, kv_dtype)
    # sequence 0 ends on the pool's last page id and fills its table exactly;
    # sequence 1 fills all but one slot of its last page
    perm = rng.permutation(P - 1)  # disjoint pages; sequence 0 also gets page P - 1
    bt = np.stack([np.concatenate([perm[:mb - 1], [P - 1]]), perm[mb - 1:2 * mb - 1]]).astype(np.int32)
    ctx = [mb * PAGE_TOKENS, mb * PAGE_TOKENS - 1]
    n_tok = sum(ctx)
    src_t = torch.float16 if kv_dtype == "fp16" else torch.bfloat16
    k = torch.from_numpy(rng.standard_normal((L, n_tok, hkv, D)).astype(np.float32)).to(src_t)
    v = torch.from_numpy(rng.standard_normal((L, n_tok, hkv, D)).astype(np.float32)).to(src_t)
    cu = np.array([0, ctx[0], n_tok], np.int32)
    start = np.zeros(2, np.int32)
    pool.append(k.to(cuda_device), v.to(cuda_device), torch.from_numpy(cu).to(cuda_device),
                torch.from_numpy(start).to(cuda_device), torch.from_numpy(bt).to(cuda_device))
    ora.append(0, k.float().numpy(), v.float().numpy(), cu, start, bt)
    q = torch.from_numpy(rng.standard_normal((2, hq, D)).astype(np.float32)).to(qdt)
    for chunk in (0, mb, 8):  # auto split, one split, three splits of exactly 8 pages
        out = pool.decode_attn(0, q.to(cuda_device), torch.from_numpy(bt).to(cuda_device),
                               torch.tensor(ctx, dtype=torch.int32, device=cuda_device), out_dtype=torch.float32,
                               chunk_pages=chunk)
        torch.cuda.synchronize()
        pool.raise_on_status()
        ref = ora.decode(0, q.float().numpy(), bt, np.array(ctx))
        for b in range(2):
            assert _rel(out.cpu().numpy()[b], ref[b]) <= TOL, (chunk, b)
    # pages bit for bit (raw codes for quantised pools)
    raw = pool.data.cpu().numpy()
    page_bytes = ora.data[0, 0].nbytes
    for b in range(2):
        for j in range(mb):
            pg = int(bt[b, j])
            np.testing.assert_array_equal(raw[pg * page_bytes:(pg + 1) * page_bytes],
                                          ora.data[0, pg].view(np.uint8).ravel())
    # the table is full: one more token is a reported bounds error, not a write
    before = pool.pool_view().clone()
    one = torch.zeros((1, 1, hkv, D), dtype=src_t, device=cuda_device)
    pool.append(one, one, torch.tensor([0, 1], dtype=torch.int32, device=cuda_device),
                torch.tensor([mb * PAGE_TOKENS], dtype=torch.int32, device=cuda_device),
                torch.from_numpy(bt[:1]).to(cuda_device))
    torch.cuda.synchronize()
    code = pool.status()[0]
    pool.clear_status()
    assert code != 0
    assert torch.equal(before, pool.pool_view())


def test_prefill_fills_block_table_to_the_last_slot(cuda_device):
    from oracle.kv_oracle import sdpa_prefill
    from synapcore_b200.paged_cache import PagedKVCache

    rng = np.random.default_rng(8)
    L, hkv, hq, D, mb = 1, 2, 32, 128, 12
    cache = PagedKVCache(L, hkv, D, max_pages=mb, max_seqs=1, max_blocks_per_seq=mb, device=cuda_device)
    cache.add_sequence("s")
    T = mb * PAGE_TOKENS  # every page of the pool, every slot of the table
    k = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
    v = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
    cache.append_prefill("s", k, v)
    q = rng.standard_normal((T, hq, D)).astype(np.float32)
    got = cache.prefill_attention(0, "s", torch.from_numpy(q).half().to(cuda_device), 0, out_dtype=torch.float32)
    kd, vd = cache.gather("s")
    ref = sdpa_prefill(torch.from_numpy(q).half().float().numpy(), kd[0].cpu().numpy(), vd[0].cpu().numpy(), 0)
    assert _rel(got.cpu().numpy(), ref) <= TOL
    assert sorted(cache.page_ids("s")) == list(range(mb))
    cache.check()


def test_bounded_wait_runs_out_reports_timeout_and_context_survives(cuda_device):
    """A kernel whose barrier nothing completes gives up after its limit and
    reports SCKV_ERR_TIMEOUT through the status word; the context keeps
    working (a decode afterwards matches the oracle)."""
    import time

    import numpy as np
    import torch

    from oracle.kv_oracle import PagedPoolOracle
    from synapcore_b200 import _native as N
    from synapcore_b200.pool import KVPool

    pool = KVPool(1, 2, 128, 8, "fp16", device=cuda_device)
    t0 = time.perf_counter()
    pool.selftest_wait_timeout(20000)  # 20 ms
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    code, detail, kernel, count = pool.status()
    assert code == N.SCKV_ERR_TIMEOUT and detail == -1 and count == 1
    assert 0.015 <= dt < 2.0
    with pytest.raises(N.SCKVError):
        pool.raise_on_status()
    pool.clear_status()
    assert pool.status()[0] == 0
    rng = np.random.default_rng(0)
    k = rng.standard_normal((8, 1, 2, 16, 128)).astype(np.float16)
    v = rng.standard_normal((8, 1, 2, 16, 128)).astype(np.float16)
    ids = np.arange(8, dtype=np.int32)
    pool.write_pages(torch.from_numpy(ids).to(cuda_device), torch.from_numpy(k).to(cuda_device),
                     torch.from_numpy(v).to(cuda_device))
    ora = PagedPoolOracle(1, 2, 128, 8, "fp16")
    ora.write_pages(ids, k.astype(np.float32), v.astype(np.float32))
    q = rng.standard_normal((1, 8, 128)).astype(np.float16)
    bt = ids.reshape(1, 8)
    out = pool.decode_attn(0, torch.from_numpy(q).to(cuda_device), torch.from_numpy(bt).to(cuda_device),
                           torch.tensor([100], dtype=torch.int32, device=cuda_device), out_dtype=torch.float32)
    ref = ora.decode(0, q.astype(np.float32), bt, np.array([100]))
    assert float(np.max(np.abs(out.cpu().numpy() - ref)) / np.max(np.abs(ref))) <= 2e-3
    pool.close()
