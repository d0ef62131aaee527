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


def _run_scheduler(dev, max_batch, capture=False):
    from stub_model import TorchStubModel, make_weights, prompts
    from synapcore_b200.paged_cache import PagedKVCache
    from synapcore_b200.scheduler import ContinuousBatchScheduler, PrefixPageIndex

    model = TorchStubModel(make_weights(), dev)
    cache = PagedKVCache(2, 2, 128, max_pages=256, max_seqs=8, max_blocks_per_seq=16, device=dev)
    index = PrefixPageIndex(cache, GOLD["prefix_cache_t4"]["seed_root"])
    s = ContinuousBatchScheduler(model, cache, max_batch_size=max_batch, prefix_index=index,
                                 capture_decode=capture)
    for i, p in enumerate(prompts()):
        s.submit_request(f"req_{i}", p, max_new_tokens=5, stop_token_ids=set())
    steps = s.run_until_complete()
    cache.check()
    return s, steps, index, cache


@pytest.mark.parametrize("mode,max_batch,capture", [("batched", 4, False), ("isolated", 1, False),
                                                    ("batched", 4, True), ("isolated", 1, True)])
def test_scheduler_matches_reference_scheduler(cuda_device, mode, max_batch, capture):
    """capture=True replays the decode steps from CUDA graphs (one per batch
    size): the same goldens hold."""
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    g = GOLD["scheduler"][mode]
    s, steps, index, cache = _run_scheduler(cuda_device, max_batch, capture)
    if capture:
        assert s._decode_graphs  # the decode steps did replay graphs
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


def _engine_scheduler_run(dev, mode, max_batch, max_layers=None):
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from stub_model import StubEngine, make_weights, prompts
    from synapcore_b200.scheduler import ContinuousBatchScheduler

    eng = StubEngine(make_weights(), GOLD["prefix_cache_t4"]["seed_root"])
    s = ContinuousBatchScheduler(eng, max_batch, device=dev)  # the reference's call, positional batch size
    for i, p in enumerate(prompts()):
        s.submit_request(f"req_{i}", p, max_new_tokens=5, stop_token_ids=set())
    steps = s.run_until_complete_numpy(max_layers=max_layers)
    s.cache.check()
    return s, steps


@pytest.mark.parametrize("mode,max_batch,max_layers", [("batched", 4, None), ("isolated", 1, None),
                                                       ("batched_1layer", 4, 1)])
def test_engine_built_scheduler_matches_reference_scheduler(cuda_device, mode, max_batch, max_layers):
    """ContinuousBatchScheduler(engine, max_batch_size) with a reference-style
    engine object (tests/stub_model.StubEngine over the stub weights): the
    reference scheduler's generated tokens, prefix skips and batch sizes, and
    its final logits (host numpy, as in the reference) to attention
    tolerance; `max_layers` runs the first layers only, with the prefix keys
    the reference derives for a shortened run (engine/scheduler.py:139-143)."""
    g = GOLD["scheduler"][mode]
    s, steps = _engine_scheduler_run(cuda_device, mode, max_batch, max_layers)
    done = s.completed_requests
    assert {k: v.generated_ids for k, v in done.items()} == g["generated"]
    assert {k: v.kv_prefix_skipped for k, v in done.items()} == g["prefix_skipped"]
    assert s.prefix_index.tokens_skipped == g["tokens_skipped"]
    assert [st["batch_size"] for st in steps] == g["batch_sizes"]
    assert s.total_naive_expert_dispatches == g["naive_expert_dispatches"]
    for k, v in done.items():
        assert isinstance(v.last_logits, np.ndarray)
        ref = ARR[f"sched_{mode}_{k}_logits"]
        assert np.max(np.abs(v.last_logits - ref)) <= 2e-3 * np.max(np.abs(ref)), k
    assert s.cache.n_live == 0


def test_engine_schedulers_share_cache_and_prefix_index(cuda_device):
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from stub_model import StubEngine, make_weights, prompts
    from synapcore_b200.scheduler import ContinuousBatchScheduler

    eng = StubEngine(make_weights(), GOLD["prefix_cache_t4"]["seed_root"])
    a = ContinuousBatchScheduler(eng, max_batch_size=1, device=cuda_device)
    a.submit_request("x", prompts()[0], max_new_tokens=2, stop_token_ids=set())
    a.run_until_complete_numpy()
    b = ContinuousBatchScheduler(eng, max_batch_size=2, device=cuda_device)
    assert b.cache is a.cache and b.prefix_index is a.prefix_index
    b.submit_request("y", prompts()[1], max_new_tokens=2, stop_token_ids=set())
    b.run_until_complete_numpy()
    assert b.completed_requests["y"].kv_prefix_skipped == 32  # blocks cached by the other scheduler


def test_benchmark_continuous_batch_scheduler_reference_assertions(cuda_device):
    """benchmark_continuous_batch_scheduler with the reference test's
    arguments (tests/test_p2_merkle_cow_and_scheduler.py:239-261) over the
    stub engine: the reference test's assertions hold, and the tokens, prefix
    skips and dispatch counts equal the reference scheduler's own run of the
    same benchmark body (tests/golden scheduler_benchmark). Prefill here is
    batched (one forward for a step's admitted requests), so fewer unique
    expert loads happen than in the reference's one-request-at-a-time
    prefill; the naive count is the same."""
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from stub_model import BENCH_CFG, StubEngine, make_weights
    from synapcore_b200.scheduler import benchmark_continuous_batch_scheduler

    g = GOLD["scheduler_benchmark"]
    eng = StubEngine(make_weights(cfg=BENCH_CFG), GOLD["prefix_cache_t4"]["seed_root"], cfg=BENCH_CFG)
    m = benchmark_continuous_batch_scheduler(None, num_requests=4, max_new_tokens=3, max_layers=2, engine=eng,
                                             device=cuda_device)
    assert m["total_requests_completed"] == 4
    assert m["total_tokens_generated"] == 12
    assert m["max_concurrent_batch_size"] == 4
    assert m["numerical_parity_max_abs_err"] <= 1e-5
    assert m["cross_request_expert_sharing_pct"] > 10.0
    assert m["paged_kv_prefix_tokens_skipped"] >= 48
    assert m["paged_kv_prefix_tokens_skipped"] == g["paged_kv_prefix_tokens_skipped"]
    assert m["total_batch_steps"] == g["total_batch_steps"]
    assert m["total_naive_expert_dispatches"] == g["total_naive_expert_dispatches"]
    assert m["total_unique_expert_dispatches"] <= g["total_unique_expert_dispatches"]
    s = eng._sckv_paged_state
    assert s.cache.n_live == 0
    print("scheduler benchmark:", m)
