"""Decode with the new token's K/V append fused into the attention launch
(sckv_decode_attn_append) against the two-call path it replaces: sckv_append
at position ctx - 1, then sckv_decode_attn (the KV-cache concat and SDPA of
one decode step of ModularAttentionEngine.forward_numpy,
models/adapters.py:1194-1229).

The fused call must leave the pool bit-identical to the append and return
bit-identical outputs (same kernel, same split); the result is also checked
against the oracle's SDPA over its own appended pages (tolerance 2e-3 of
max|o_ref|, fp32 accumulation, as the decode tests).
"""
import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS

from test_gpu_decode import _make_case, _rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _private_table(ctx, pool_pages, rng):
    """Block table whose read pages (the first ceil(ctx / 16) of each row)
    are distinct across sequences: the page a sequence appends into is read
    by no other sequence of the call, as copy-on-write keeps it in use."""
    n_pages = [(c + PAGE_TOKENS - 1) // PAGE_TOKENS for c in ctx]
    max_blocks = max(n_pages)
    perm = rng.permutation(pool_pages)
    assert sum(n_pages) <= pool_pages
    bt = rng.integers(0, pool_pages, size=(len(ctx), max_blocks)).astype(np.int32)
    off = 0
    for b, n in enumerate(n_pages):
        bt[b, :n] = perm[off:off + n]
        off += n
    return bt


def _clone(pool, cuda_device):
    from synapcore_b200.pool import KVPool

    twin = KVPool(pool.num_layers, pool.num_kv_heads, pool.head_dim, pool.max_pages, pool.kv_dtype,
                  device=cuda_device)
    twin.data.copy_(pool.data)
    if pool.scale_view() is not None:
        twin.scale_view().copy_(pool.scale_view())
    return twin


@pytest.mark.parametrize("kv_dtype,hq,hkv,qdt,src_dt", [
    ("fp16", 16, 16, torch.float16, torch.float16),    # CUDA-core kernel, same type
    ("fp16", 16, 16, torch.float16, torch.float32),    # fp32 rows rounded on the way in
    ("bf16", 8, 8, torch.float32, torch.bfloat16),     # CUDA-core kernel, bf16 pool
    ("fp16", 8, 2, torch.float16, torch.bfloat16),     # tensor-core kernel, bf16 rows into an fp16 pool
    ("bf16", 32, 8, torch.bfloat16, torch.bfloat16),   # tensor-core kernel, Qwen3-style GQA
    ("bf16", 32, 8, torch.bfloat16, torch.float32),
    ("int8", 16, 16, torch.float16, torch.float16),    # one-byte pools: append, then decode
    ("int8", 32, 8, torch.bfloat16, torch.float32),
    ("fp8_e4m3", 32, 8, torch.bfloat16, torch.bfloat16),
])
@pytest.mark.parametrize("chunk_pages", [0, 3])
def test_decode_append_matches_two_calls(cuda_device, kv_dtype, hq, hkv, qdt, src_dt, chunk_pages):
    ctx = [1, 16, 17, 100, 333, 1024, 513, 32, 2]
    pool, ora, _, q = _make_case(cuda_device, kv_dtype, hq, hkv, ctx, pool_pages=220, seed=5)
    twin = _clone(pool, cuda_device)
    rng = np.random.default_rng(17)
    bt = _private_table(ctx, 220, rng)
    B, D = len(ctx), 128
    bt_d = torch.from_numpy(bt).to(cuda_device)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    cu = torch.arange(B + 1, dtype=torch.int32, device=cuda_device)
    q_t = torch.from_numpy(q).to(qdt).to(cuda_device)
    for layer in range(pool.num_layers):
        k_new = torch.from_numpy(rng.standard_normal((B, hkv, D)).astype(np.float32)).to(src_dt).to(cuda_device)
        v_new = torch.from_numpy(rng.standard_normal((B, hkv, D)).astype(np.float32)).to(src_dt).to(cuda_device)
        pool.append(k_new, v_new, cu, ctx_d - 1, bt_d, layer0=layer)
        ref = pool.decode_attn(layer, q_t, bt_d, ctx_d, out_dtype=torch.float32, chunk_pages=chunk_pages)
        got = twin.decode_attn_append(layer, q_t, k_new, v_new, bt_d, ctx_d, out_dtype=torch.float32,
                                      chunk_pages=chunk_pages)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"layer {layer}: fused output differs from append + decode"
        assert torch.equal(twin.data, pool.data), f"layer {layer}: pool pages differ"
        if pool.scale_view() is not None:
            assert torch.equal(twin.scale_view(), pool.scale_view())
        # the oracle: same rows appended through its own quantisation, then its SDPA
        kn = k_new.float().cpu().numpy()[None]
        vn = v_new.float().cpu().numpy()[None]
        ora.append(layer, kn, vn, np.arange(B + 1, dtype=np.int32), np.array(ctx, np.int32) - 1, bt)
        o_ref = ora.decode(layer, q_t.float().cpu().numpy(), bt, np.array(ctx))
        o = got.cpu().numpy()
        for b in range(B):
            assert _rel_err(o[b], o_ref[b]) <= TOL, (layer, b, ctx[b], _rel_err(o[b], o_ref[b]))
    assert pool.status()[0] == 0 and twin.status()[0] == 0


def test_decode_append_stores_only_the_new_rows(cuda_device):
    """Every byte outside the appended rows is untouched, and the new rows
    hold exactly the rounded inputs (fp32 -> fp16, RN)."""
    ctx = [5, 16, 48, 49]
    pool, _, _, q = _make_case(cuda_device, "fp16", 16, 16, ctx, pool_pages=40, seed=3)
    before = pool.pool_view().clone()  # [L, P, 2, H, 16, D]
    B, D = len(ctx), 128
    rng = np.random.default_rng(9)
    bt = _private_table(ctx, 40, rng)
    k_new = torch.from_numpy(rng.standard_normal((B, 16, D)).astype(np.float32)).to(cuda_device)
    v_new = torch.from_numpy(rng.standard_normal((B, 16, D)).astype(np.float32)).to(cuda_device)
    bt_d = torch.from_numpy(bt).to(cuda_device)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    layer = 1
    pool.decode_attn_append(layer, torch.from_numpy(q).half().to(cuda_device), k_new, v_new, bt_d, ctx_d)
    torch.cuda.synchronize()
    after = pool.pool_view()
    expect = before.clone()
    for b, c in enumerate(ctx):
        page = int(bt[b, (c - 1) // PAGE_TOKENS])
        row = (c - 1) % PAGE_TOKENS
        expect[layer, page, 0, :, row] = k_new[b].half()
        expect[layer, page, 1, :, row] = v_new[b].half()
    assert torch.equal(after, expect)


def test_decode_append_rejects_bad_rows(cuda_device):
    from synapcore_b200.pool import KVPool

    pool = KVPool(1, 2, 128, 8, "fp16", device=cuda_device)
    bt = torch.zeros((2, 2), dtype=torch.int32, device=cuda_device)
    ctx = torch.tensor([3, 4], dtype=torch.int32, device=cuda_device)
    q = torch.zeros((2, 4, 128), dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError):
        pool.decode_attn_append(0, q, torch.zeros((2, 1, 128), device=cuda_device),
                                torch.zeros((2, 1, 128), device=cuda_device), bt, ctx)
    with pytest.raises(TypeError):
        pool.decode_attn_append(0, q, torch.zeros((2, 2, 128), device=cuda_device),
                                torch.zeros((2, 2, 128), dtype=torch.float16, device=cuda_device), bt, ctx)


@pytest.mark.parametrize("kv_dtype,hq,hkv", [("fp16", 16, 16), ("bf16", 32, 8)])
def test_decode_append_bad_page_matches_two_calls(cuda_device, kv_dtype, hq, hkv):
    """A sequence whose last block holds an out-of-range page id: the bounds
    checks report SCKV_ERR_BOUNDS, its row is stored nowhere, page 0 is read
    in its place — and the fused call still equals append + decode bit for
    bit, outputs and pool bytes (the other sequences are untouched by it)."""
    from synapcore_b200 import _native as N

    ctx = [40, 17, 100, 64]
    P = 60
    pool, _, _, q = _make_case(cuda_device, kv_dtype, hq, hkv, ctx, pool_pages=P, seed=21)
    twin = _clone(pool, cuda_device)
    rng = np.random.default_rng(4)
    bt = _private_table(ctx, P, rng)
    bad = 1
    bt[bad, (ctx[bad] - 1) // PAGE_TOKENS] = P + 5  # out of range
    B, D = len(ctx), 128
    qdt = torch.bfloat16 if kv_dtype == "bf16" else torch.float16
    bt_d = torch.from_numpy(bt).to(cuda_device)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
    cu = torch.arange(B + 1, dtype=torch.int32, device=cuda_device)
    q_t = torch.from_numpy(q).to(qdt).to(cuda_device)
    k_new = torch.from_numpy(rng.standard_normal((B, hkv, D)).astype(np.float32)).to(qdt).to(cuda_device)
    v_new = torch.from_numpy(rng.standard_normal((B, hkv, D)).astype(np.float32)).to(qdt).to(cuda_device)
    layer = 0
    # the calls return at once; the kernels' bounds checks record the bad id
    pool.append(k_new, v_new, cu, ctx_d - 1, bt_d, layer0=layer)
    out = pool.decode_attn(layer, q_t, bt_d, ctx_d, out_dtype=torch.float32)
    got = twin.decode_attn_append(layer, q_t, k_new, v_new, bt_d, ctx_d, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert pool.status()[0] == N.SCKV_ERR_BOUNDS
    assert twin.status()[0] == N.SCKV_ERR_BOUNDS
    assert torch.equal(got, out)
    assert torch.equal(twin.data, pool.data)
    pool.clear_status()
    twin.clear_status()
