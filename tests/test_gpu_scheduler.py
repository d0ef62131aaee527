"""Sequence-level paged cache and the continuous-batching scheduler on the GPU.

The scheduler test runs the same seeded stub model as the reference run in
tests/golden (the reference ContinuousBatchScheduler over a stub engine):
generated tokens must match exactly, prefix reuse must skip the same tokens,
and final logits must agree to attention tolerance (the only numerical
difference is fp32 accumulation order in attention and the projections).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS

pytestmark = pytest.mark.gpu

GOLD_DIR = Path(__file__).resolve().parent / "golden"
GOLD = json.loads((GOLD_DIR / "golden.json").read_text())
ARR = np.load(GOLD_DIR / "golden_arrays.npz")


def _cache(dev, layers=2, hkv=2, pages=256, seqs=8, blocks=16, kv="fp16"):
    from synapcore_b200.paged_cache import PagedKVCache

    return PagedKVCache(layers, hkv, 128, pages, seqs, blocks, kv_dtype=kv, device=dev)


def test_prefill_decode_append_fork_and_release(cuda_device):
    rng = np.random.default_rng(0)
    c = _cache(cuda_device)
    L, H, D = 2, 2, 128
    lens = [37, 16, 5]
    exp_k, exp_v = {}, {}
    for i, n in enumerate(lens):
        c.add_sequence(i)
        k = rng.standard_normal((L, n, H, D)).astype(np.float16)
        v = rng.standard_normal((L, n, H, D)).astype(np.float16)
        exp_k[i], exp_v[i] = k, v
        c.append_prefill(i, torch.from_numpy(k).to(cuda_device), torch.from_numpy(v).to(cuda_device))
    for _ in range(3):  # three decode steps for every row
        c.decode_reserve(3)
        kn = rng.standard_normal((L, 3, H, D)).astype(np.float16)
        vn = rng.standard_normal((L, 3, H, D)).astype(np.float16)
        for l in range(L):
            c.decode_append(l, torch.from_numpy(kn[l]).to(cuda_device), torch.from_numpy(vn[l]).to(cuda_device), 3)
        for i in range(3):
            exp_k[i] = np.concatenate([exp_k[i], kn[:, i:i + 1]], axis=1)
            exp_v[i] = np.concatenate([exp_v[i], vn[:, i:i + 1]], axis=1)
    torch.cuda.synchronize()
    c.check()
    assert c.lengths == [40, 19, 8]
    for i in range(3):
        gk, gv = c.gather(i)  # [L, H, T, D]
        np.testing.assert_array_equal(gk.cpu().numpy(), exp_k[i].transpose(0, 2, 1, 3))
        np.testing.assert_array_equal(gv.cpu().numpy(), exp_v[i].transpose(0, 2, 1, 3))
    # copy-on-write fork: same contents, shared full pages, private tail page
    c.fork(0, "f")
    k0, v0 = c.gather(0)
    kf, vf = c.gather("f")
    assert torch.equal(k0, kf) and torch.equal(v0, vf)
    p_src, p_dst = c.page_ids(0), c.page_ids("f")
    n_full = 40 // PAGE_TOKENS
    assert p_src[:n_full] == p_dst[:n_full] and p_src[n_full] != p_dst[n_full]
    c.move_to_row("f", 0)  # the sequence to extend must be in the decode rows
    c.decode_reserve(1)
    for l in range(L):
        c.decode_append(l, torch.ones((1, H, D), dtype=torch.float16, device=cuda_device),
                        torch.ones((1, H, D), dtype=torch.float16, device=cuda_device), 1)
    k0b, _ = c.gather(0)
    assert torch.equal(k0b, k0), "appending to the fork changed the source"
    kfb, _ = c.gather("f")
    assert torch.equal(kfb[:, :, :40], k0) and bool(torch.all(kfb[:, :, 40] == 1))
    # release: shared pages survive until their last holder lets go
    st0 = c.pool.alloc_state()
    c.remove_sequence("f")
    st1 = c.pool.alloc_state()
    assert st0["allocated"] - st1["allocated"] == 1  # only the fork's private tail page
    for sid in (0, 1, 2):
        c.remove_sequence(sid)
    assert c.pool.alloc_state()["allocated"] == 0
    c.check()


def test_decode_attention_rows_match_isolated(cuda_device):
    """Batched decode over compact rows gives bit-identical results to each
    sequence alone (fixed split size)."""
    rng = np.random.default_rng(1)
    c = _cache(cuda_device, hkv=2, blocks=32)
    lens = [300, 17, 64, 129]
    for i, n in enumerate(lens):
        c.add_sequence(i)
        k = torch.from_numpy(rng.standard_normal((2, n, 2, 128)).astype(np.float16)).to(cuda_device)
        c.append_prefill(i, k, k * 0.5)
    q = torch.from_numpy(rng.standard_normal((4, 8, 128)).astype(np.float32)).to(cuda_device)
    batched = c.decode_attention(1, q, 4, out_dtype=torch.float32)  # rows 0..3 = sequences 0..3
    for i in range(4):
        c.move_to_row(i, 0)
        alone = c.decode_attention(1, q[i:i + 1], 1, out_dtype=torch.float32)
        assert torch.equal(alone[0], batched[i])
    c.check()


def _run_scheduler(dev, max_batch):
    from stub_model import TorchStubModel, make_weights, prompts
    from synapcore_b200.paged_cache import PagedKVCache
    from synapcore_b200.scheduler import ContinuousBatchScheduler, PrefixPageIndex

    model = TorchStubModel(make_weights(), dev)
    cache = PagedKVCache(2, 2, 128, max_pages=256, max_seqs=8, max_blocks_per_seq=16, device=dev)
    index = PrefixPageIndex(cache, GOLD["prefix_cache_t4"]["seed_root"])
    s = ContinuousBatchScheduler(model, cache, max_batch_size=max_batch, prefix_index=index)
    for i, p in enumerate(prompts()):
        s.submit_request(f"req_{i}", p, max_new_tokens=5, stop_token_ids=set())
    steps = s.run_until_complete()
    cache.check()
    return s, steps, index, cache


@pytest.mark.parametrize("mode,max_batch", [("batched", 4), ("isolated", 1)])
def test_scheduler_matches_reference_scheduler(cuda_device, mode, max_batch):
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    g = GOLD["scheduler"][mode]
    s, steps, index, cache = _run_scheduler(cuda_device, max_batch)
    done = s.completed_requests
    assert {k: v.generated_ids for k, v in done.items()} == g["generated"]
    assert {k: v.kv_prefix_skipped for k, v in done.items()} == g["prefix_skipped"]
    assert index.tokens_skipped == g["tokens_skipped"] == 128
    assert [st["batch_size"] for st in steps] == g["batch_sizes"]
    for k, v in done.items():
        ref = ARR[f"sched_{mode}_{k}_logits"]
        got = v.last_logits.float().cpu().numpy()
        assert np.max(np.abs(got - ref)) <= 2e-3 * np.max(np.abs(ref)), k
    # only the prefix index still holds pages once every request is done
    assert cache.n_live == 0
    assert cache.pool.alloc_state()["allocated"] == len(index.pages)
    m = s.metrics()
    assert m["total_requests_completed"] == 6 and m["total_tokens_generated"] == 30
