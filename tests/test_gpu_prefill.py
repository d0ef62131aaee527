"""Tensor-core causal prefill attention against the oracle's causal SDPA
(models/adapters.py:1209-1229, mask :1218-1224): each new token at position
start+t sees the cached tokens at positions <= start+t.

Tolerance as for decode: max|o - o_ref| / max|o_ref| <= 2e-3 per sequence
(fp32 accumulation); FP8 pools are compared with the dequantised pages.
"""
import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS, PagedPoolOracle

pytestmark = pytest.mark.gpu

TOL = 2e-3
# rounding the output to 16 bits adds at most half an ulp of the element
OUT_ROUNDING = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


def _rel_err(o, r):
    return float(np.max(np.abs(o - r)) / max(np.max(np.abs(r)), 1e-30))


def _case(dev, kv_dtype, hq, hkv, T, start, pool_pages=160, layers=2, seed=3, nan_tail=False):
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(seed)
    D = 128
    pool = KVPool(layers, hkv, D, pool_pages, kv_dtype, device=dev)
    ora = PagedPoolOracle(layers, hkv, D, pool_pages, kv_dtype)
    k = rng.standard_normal((pool_pages, layers, hkv, PAGE_TOKENS, D)).astype(np.float32)
    v = rng.standard_normal((pool_pages, layers, hkv, PAGE_TOKENS, D)).astype(np.float32)
    if kv_dtype == "fp8_e4m3":
        f = rng.uniform(0.5, 4.0, size=(pool_pages, layers, hkv, 1, 1)).astype(np.float32)
        k *= f
        v *= f
    B = len(T)
    ctx = [s + t for s, t in zip(start, T)]
    mb = max(1, max((c + PAGE_TOKENS - 1) // PAGE_TOKENS for c in ctx))
    perm = rng.permutation(pool_pages)[:B * mb].reshape(B, mb).astype(np.int32)
    if nan_tail:
        # slots past each sequence's end hold NaN: the kernel must never let them in
        for b in range(B):
            last, used = divmod(ctx[b], PAGE_TOKENS)
            if used:
                k[perm[b, last], :, :, used:] = np.nan
                v[perm[b, last], :, :, used:] = np.nan
    src_t = torch.float16 if kv_dtype in ("fp16", "int8") else torch.bfloat16
    k_t, v_t = torch.from_numpy(k).to(src_t), torch.from_numpy(v).to(src_t)
    ids = np.arange(pool_pages, dtype=np.int32)
    pool.write_pages(torch.from_numpy(ids).to(dev), k_t.to(dev), v_t.to(dev))
    ora.write_pages(ids, k_t.float().numpy(), v_t.float().numpy())
    cu = np.concatenate([[0], np.cumsum(T)]).astype(np.int32)
    q = rng.standard_normal((int(cu[-1]), hq, D)).astype(np.float32)
    return pool, ora, perm, cu, np.array(start, np.int32), q


def _check(pool, ora, bt, cu, start, q_t, out_dtype=torch.float32):
    dev = pool.device
    qv = q_t.float().numpy()
    for layer in range(pool.num_layers):
        out = pool.prefill_attn(layer, q_t.to(dev), torch.from_numpy(cu).to(dev), torch.from_numpy(start).to(dev),
                                torch.from_numpy(bt).to(dev), out_dtype=out_dtype)
        torch.cuda.synchronize()
        pool.raise_on_status()
        got = out.float().cpu().numpy()
        ref = ora.prefill(layer, qv, cu, start, bt)
        assert np.all(np.isfinite(got))
        for b in range(len(cu) - 1):
            t0, t1 = cu[b], cu[b + 1]
            if t1 > t0:
                err = _rel_err(got[t0:t1], ref[t0:t1])
                assert err <= TOL + OUT_ROUNDING[out_dtype] / 2, (layer, b, err)


@pytest.mark.parametrize("kv_dtype,hq,hkv,qdt", [
    ("fp16", 8, 8, torch.float16),      # MHA (G=1)
    ("fp16", 16, 8, torch.float16),     # G=2
    ("fp16", 16, 4, torch.float32),     # G=4
    ("fp16", 32, 4, torch.bfloat16),    # G=8
    ("fp16", 32, 2, torch.float16),     # G=16
    ("bf16", 16, 4, torch.bfloat16),
    ("bf16", 32, 2, torch.bfloat16),
    ("fp8_e4m3", 32, 4, torch.bfloat16),
    ("fp8_e4m3", 16, 2, torch.float16),
    ("fp8_e4m3", 8, 8, torch.float32),
    ("int8", 16, 4, torch.float16),
    ("int8", 32, 8, torch.bfloat16),
    ("int8", 8, 8, torch.float32),
    ("int8", 32, 2, torch.float16),
])
def test_prefill_matches_oracle(cuda_device, kv_dtype, hq, hkv, qdt):
    T = [1, 5, 64, 130, 17, 16, 33]
    start = [0, 30, 0, 100, 16, 7, 0]
    pool, ora, bt, cu, st, q = _case(cuda_device, kv_dtype, hq, hkv, T, start)
    _check(pool, ora, bt, cu, st, torch.from_numpy(q).to(qdt))


@pytest.mark.parametrize("kv_dtype", ["fp16", "bf16"])
def test_prefill_never_reads_past_context(cuda_device, kv_dtype):
    T = [3, 20, 77]
    start = [0, 9, 40]
    pool, ora, bt, cu, st, q = _case(cuda_device, kv_dtype, 16, 4, T, start, nan_tail=True)
    qdt = torch.bfloat16 if kv_dtype == "bf16" else torch.float16
    _check(pool, ora, bt, cu, st, torch.from_numpy(q).to(qdt), out_dtype=qdt)


def test_prefill_long_prompt_and_zero_length_sequences(cuda_device):
    T = [0, 700, 0, 2]
    start = [5, 0, 0, 600]
    pool, ora, bt, cu, st, q = _case(cuda_device, "fp16", 16, 4, T, start, pool_pages=200, layers=1)
    _check(pool, ora, bt, cu, st, torch.from_numpy(q).to(torch.float16))


def test_prefill_unsupported_and_bounds(cuda_device):
    from synapcore_b200 import _native as N
    from synapcore_b200.pool import KVPool

    # three q heads per kv head: not a power of two
    pool = KVPool(1, 4, 128, 16, "int8", device=cuda_device)
    q3 = torch.zeros(4, 12, 128, dtype=torch.float16, device=cuda_device)
    cu = torch.tensor([0, 4], dtype=torch.int32, device=cuda_device)
    st = torch.tensor([0], dtype=torch.int32, device=cuda_device)
    bt = torch.zeros(1, 2, dtype=torch.int32, device=cuda_device)
    with pytest.raises(N.SCKVError) as e:
        pool.prefill_attn(0, q3, cu, st, bt)
    assert e.value.code == N.SCKV_ERR_UNSUPPORTED
    q = torch.zeros(4, 8, 128, dtype=torch.float16, device=cuda_device)
    # a sequence that would run past its block table is reported, not read
    pool = KVPool(1, 4, 128, 16, "fp16", device=cuda_device)
    st_bad = torch.tensor([30], dtype=torch.int32, device=cuda_device)
    pool.prefill_attn(0, q, cu, st_bad, bt)
    torch.cuda.synchronize()
    assert pool.status()[0] == N.SCKV_ERR_BOUNDS
    pool.clear_status()


def test_paged_cache_prefill_uses_tensor_core_kernel_and_matches_decode_path(cuda_device):
    """PagedKVCache.prefill_attention (tensor-core kernel) equals the same
    causal attention computed token by token by the decode kernel."""
    from synapcore_b200.paged_cache import PagedKVCache

    rng = np.random.default_rng(5)
    L, hkv, hq, D = 2, 4, 16, 128
    cache = PagedKVCache(L, hkv, D, max_pages=64, max_seqs=4, max_blocks_per_seq=16, device=cuda_device)
    cache.add_sequence("a")
    T0, T1 = 37, 21
    for T in (T0, T1):
        start = cache.length("a")
        k = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
        v = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
        cache.append_prefill("a", k, v)
        q = torch.from_numpy(rng.standard_normal((T, hq, D)).astype(np.float16)).to(cuda_device)
        for layer in range(L):
            got = cache.prefill_attention(layer, "a", q, start, out_dtype=torch.float32)
            r = cache.row_of["a"]
            bt = cache.block_table[r:r + 1].expand(T, cache.max_blocks)
            ctx = torch.arange(start + 1, start + T + 1, dtype=torch.int32, device=cuda_device)
            ref = cache.pool.decode_attn(layer, q, bt, ctx, out_dtype=torch.float32, max_blocks=cache.max_blocks)
            torch.cuda.synchronize()
            assert _rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= TOL
    cache.check()


def test_paged_cache_int8_prefill_and_decode_match_oracle(cuda_device):
    """int8 pools (the arena's quant mode, per-token fp16 scales) attend
    through the SIMT decode kernel; the reference attends over the fp16
    dequantisation fp16(code * scale) of the same pages."""
    from oracle.kv_oracle import sdpa_decode, sdpa_prefill
    from synapcore_b200.paged_cache import PagedKVCache

    rng = np.random.default_rng(9)
    L, hkv, hq, D, T = 2, 4, 16, 128, 45
    cache = PagedKVCache(L, hkv, D, max_pages=32, max_seqs=2, max_blocks_per_seq=8, kv_dtype="int8",
                         device=cuda_device)
    cache.add_sequence(7)
    k = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
    v = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(cuda_device)
    cache.append_prefill(7, k, v)
    kd, vd = cache.gather(7)  # [L, Hkv, T, D] fp16 dequantised on the device
    kd, vd = kd.cpu().numpy(), vd.cpu().numpy()
    q = rng.standard_normal((T, hq, D)).astype(np.float32)
    for layer in range(L):
        got = cache.prefill_attention(layer, 7, torch.from_numpy(q).to(cuda_device), 0, out_dtype=torch.float32)
        ref = sdpa_prefill(q, kd[layer], vd[layer], 0)
        assert _rel_err(got.cpu().numpy(), ref) <= TOL
    cache.decode_reserve(1)
    kn = torch.from_numpy(rng.standard_normal((1, hkv, D)).astype(np.float16)).to(cuda_device)
    for layer in range(L):
        cache.decode_append(layer, kn, kn, 1)
    kd, vd = cache.gather(7)
    kd, vd = kd.cpu().numpy(), vd.cpu().numpy()
    qd = rng.standard_normal((1, hq, D)).astype(np.float32)
    for layer in range(L):
        got = cache.decode_attention(layer, torch.from_numpy(qd).to(cuda_device), 1, out_dtype=torch.float32)
        ref = sdpa_decode(qd[0], kd[layer], vd[layer])
        assert _rel_err(got.cpu().numpy()[0], ref) <= TOL
    cache.check()


@pytest.mark.parametrize("kv,hq,hkv", [("fp16", 8, 8), ("fp16", 16, 4), ("bf16", 16, 4), ("bf16", 32, 2)])
def test_tensor_memory_kernel_rescales_and_matches_mma_kernel(cuda_device, kv, hq, hkv, monkeypatch):
    """Keys grow in magnitude along the sequence, so the running max moves
    by more than 2^8 several times and the tensor-memory kernel must rescale
    its O accumulator in TMEM. Its output matches the oracle and the
    mma.sync kernel (SCKV_PREFILL_KERNEL=mma) within the tolerance."""
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(12)
    D, P = 128, 64
    T, start = [300, 77], [50, 0]
    ctx = [s + t for s, t in zip(start, T)]
    pool = KVPool(1, hkv, D, P, kv, device=cuda_device)
    ora = PagedPoolOracle(1, hkv, D, P, kv)
    growth = (1.0 + np.arange(P * PAGE_TOKENS, dtype=np.float32) / 40.0).reshape(P, 1, 1, PAGE_TOKENS, 1)
    k = (rng.standard_normal((P, 1, hkv, PAGE_TOKENS, D)).astype(np.float32) * growth)
    v = rng.standard_normal((P, 1, hkv, PAGE_TOKENS, D)).astype(np.float32)
    src_t = torch.float16 if kv == "fp16" else torch.bfloat16
    k_t, v_t = torch.from_numpy(k).to(src_t), torch.from_numpy(v).to(src_t)
    ids = np.arange(P, dtype=np.int32)
    pool.write_pages(torch.from_numpy(ids).to(cuda_device), k_t.to(cuda_device), v_t.to(cuda_device))
    ora.write_pages(ids, k_t.float().numpy(), v_t.float().numpy())
    mb = (max(ctx) + PAGE_TOKENS - 1) // PAGE_TOKENS
    bt = np.stack([np.arange(mb, dtype=np.int32), np.arange(mb, 2 * mb, dtype=np.int32)])  # page i = tokens 16i..
    cu = np.array([0, T[0], T[0] + T[1]], np.int32)
    st = np.array(start, np.int32)
    qdt = torch.float16 if kv == "fp16" else torch.bfloat16
    q_t = torch.from_numpy(rng.standard_normal((sum(T), hq, D)).astype(np.float32)).to(qdt)
    ref = ora.prefill(0, q_t.float().numpy(), cu, st, bt)
    outs = {}
    for which in ("tc", "mma"):
        if which == "mma":
            monkeypatch.setenv("SCKV_PREFILL_KERNEL", "mma")
        else:
            monkeypatch.delenv("SCKV_PREFILL_KERNEL", raising=False)
        o = pool.prefill_attn(0, q_t.to(cuda_device), torch.from_numpy(cu).to(cuda_device),
                              torch.from_numpy(st).to(cuda_device), torch.from_numpy(bt).to(cuda_device),
                              out_dtype=torch.float32)
        torch.cuda.synchronize()
        pool.raise_on_status()
        outs[which] = o.cpu().numpy()
    for which, got in outs.items():
        for b in range(2):
            err = _rel_err(got[cu[b]:cu[b + 1]], ref[cu[b]:cu[b + 1]])
            assert err <= TOL, (which, b, err)
    assert _rel_err(outs["tc"], outs["mma"]) <= TOL


def test_prefill_launches_on_two_streams_share_one_pool(cuda_device):
    """Each launch claims work items from its own counter: concurrent prefills
    of one pool on two streams both cover every item."""
    T = [300, 5, 260, 64, 190]
    start = [0, 40, 16, 0, 33]
    pool, ora, bt, cu, st, q = _case(cuda_device, "fp16", 16, 4, T, start, pool_pages=200, layers=2)
    dev = pool.device
    q_t = torch.from_numpy(q).to(torch.float16).to(dev)
    cu_t, st_t, bt_t = (torch.from_numpy(a).to(dev) for a in (cu, st, bt))
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    torch.cuda.synchronize()
    outs = []
    for rep in range(8):
        for layer, s in ((0, s1), (1, s2)):
            with torch.cuda.stream(s):
                outs.append((layer, pool.prefill_attn(layer, q_t, cu_t, st_t, bt_t, stream=s)))
    torch.cuda.synchronize()
    pool.raise_on_status()
    refs = {layer: ora.prefill(layer, q_t.float().cpu().numpy(), cu, st, bt) for layer in (0, 1)}
    for layer, out in outs:
        got = out.float().cpu().numpy()
        assert _rel_err(got, refs[layer]) <= TOL, layer


@pytest.mark.parametrize("kv_dtype", ["fp8_e4m3", "int8"])
def test_one_byte_pools_prefill_long_prompts_with_prefix(cuda_device, kv_dtype):
    """One-byte pools on the tensor-memory kernel: codes staged by TMA and
    decoded into the f16 rings; prompts long enough that every producer
    warp cycles its staging slots and the 3-slot rings many times, behind a
    cached prefix (start > 0) and with ragged ends."""
    T = [700, 1, 333]
    start = [64, 500, 0]
    pool, ora, bt, cu, st, q = _case(cuda_device, kv_dtype, 32, 8, T, start, pool_pages=200, layers=1)
    _check(pool, ora, bt, cu, st, torch.from_numpy(q).to(torch.bfloat16))
