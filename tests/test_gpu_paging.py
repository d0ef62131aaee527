"""Kernel 1 (append) and kernel 2 (gather, CoW copy) parity against the oracle.

Bit-exact comparisons on the append+gather workload of the OLMoE attention
shape: 1 layer, 16 KV heads, head_dim 128, 16-token pages, 4 sequences of
lengths {37, 128, 255, 512}, K/V ~ N(0, 1) from a seed.
"""
import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS, PagedPoolOracle, bf16_bits_to_f32

pytestmark = pytest.mark.gpu

LENS = [37, 128, 255, 512]
H, D = 16, 128


def _setup(kv_dtype, seed=7, layers=1, pool_pages=160):
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(seed)
    n_pages = [(n + PAGE_TOKENS - 1) // PAGE_TOKENS for n in LENS]
    perm = rng.permutation(pool_pages)[: sum(n_pages)]
    max_blocks = max(n_pages)
    bt = np.full((len(LENS), max_blocks), -1, np.int32)
    o = 0
    for b, n in enumerate(n_pages):
        bt[b, :n] = perm[o:o + n]
        o += n
    pool = KVPool(layers, H, D, pool_pages, kv_dtype, device="cuda:0")
    ora = PagedPoolOracle(layers, H, D, pool_pages, kv_dtype)
    return rng, pool, ora, bt


def _src(rng, n_tok, layers, dtype):
    x = rng.standard_normal((layers, n_tok, H, D)).astype(np.float32)
    if dtype == torch.float16:
        x = x.astype(np.float16).astype(np.float32)
    elif dtype == torch.bfloat16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    return x


def _pool_np(pool):
    v = pool.pool_view()
    if pool.kv_dtype == "bf16":
        return v.view(torch.int16).cpu().numpy().view(np.uint16)
    return v.cpu().numpy()


@pytest.mark.parametrize("kv_dtype,src_dtype", [
    ("fp16", torch.float16), ("bf16", torch.bfloat16), ("fp16", torch.float32),
    ("int8", torch.float16), ("fp8_e4m3", torch.bfloat16), ("fp8_e4m3", torch.float16)])
@pytest.mark.parametrize("mode", ["bulk", "token_by_token", "chunks"])
def test_append_then_gather_bit_exact(cuda_device, kv_dtype, src_dtype, mode):
    rng, pool, ora, bt = _setup(kv_dtype)
    layers = 1
    total = sum(LENS)
    k = _src(rng, total, layers, src_dtype)
    v = _src(rng, total, layers, src_dtype)
    offs = np.concatenate([[0], np.cumsum(LENS)])
    bt_d = torch.from_numpy(bt).to(cuda_device)

    def do_append(pieces):
        # pieces: list of (b, start, n) appended in one call each
        for call in pieces:
            rows, cu, sp = [], [0], []
            for b, s, n in call:
                rows.append(np.arange(offs[b] + s, offs[b] + s + n))
                cu.append(cu[-1] + n)
                sp.append(s)
            rows = np.concatenate(rows)
            kk, vv = k[:, rows], v[:, rows]
            cu_a, sp_a = np.array(cu, np.int32), np.array(sp, np.int32)
            # the oracle wants per-sequence block table rows in call order
            bt_call = np.stack([bt[b] for b, _, _ in call])
            ora.append(0, kk, vv, cu_a, sp_a, bt_call)
            pool.append(torch.from_numpy(kk).to(cuda_device, src_dtype), torch.from_numpy(vv).to(cuda_device, src_dtype),
                        torch.from_numpy(cu_a).to(cuda_device), torch.from_numpy(sp_a).to(cuda_device),
                        torch.from_numpy(bt_call).to(cuda_device))

    if mode == "bulk":
        do_append([[(b, 0, n) for b, n in enumerate(LENS)]])
    elif mode == "token_by_token":
        # decode-style: one token per live sequence per call
        calls = []
        for t in range(max(LENS)):
            calls.append([(b, t, 1) for b, n in enumerate(LENS) if t < n])
        # keep the test quick: first 20 steps one token at a time, rest bulk
        head = calls[:20]
        tail = [[(b, 20, n - 20) for b, n in enumerate(LENS) if n > 20]]
        do_append(head + tail)
    else:
        rs = np.random.default_rng(3)
        calls = []
        pos = [0] * len(LENS)
        while any(p < n for p, n in zip(pos, LENS)):
            call = []
            for b, n in enumerate(LENS):
                if pos[b] < n:
                    step = int(min(n - pos[b], rs.integers(1, 40)))
                    call.append((b, pos[b], step))
                    pos[b] += step
            calls.append(call)
        do_append(calls)
    torch.cuda.synchronize()
    assert pool.status()[0] == 0

    # raw pool state bit-exact (codes and scales)
    got = _pool_np(pool)
    np.testing.assert_array_equal(got, ora.data)
    if kv_dtype in ("int8", "fp8_e4m3"):
        sv = pool.scale_view().cpu().numpy()
        np.testing.assert_array_equal(sv.view(np.uint8), ora.scales.view(np.uint8))

    # gather per sequence, compare with oracle gather (bit-exact in f32)
    for b, n in enumerate(LENS):
        n_pages = (n + PAGE_TOKENS - 1) // PAGE_TOKENS
        ids = torch.from_numpy(bt[b, :n_pages].copy()).to(cuda_device)
        gk, gv = pool.gather(ids, n, out_dtype=torch.float32)
        ok, ov = ora.gather(0, 1, bt[b, :n_pages], n)
        np.testing.assert_array_equal(gk.cpu().numpy(), ok)
        np.testing.assert_array_equal(gv.cpu().numpy(), ov)
        if kv_dtype in ("fp16", "bf16"):
            # lossless pools return exactly what was appended
            src_k = k[0, offs[b]:offs[b] + n].transpose(1, 0, 2)
            if kv_dtype == "fp16":
                src_k = src_k.astype(np.float16).astype(np.float32)
            else:
                src_k = torch.from_numpy(np.ascontiguousarray(src_k)).to(torch.bfloat16).float().numpy()
            np.testing.assert_array_equal(gk[0].cpu().numpy(), src_k)
    pool.close()


@pytest.mark.parametrize("kv_dtype", ["fp16", "int8", "fp8_e4m3"])
def test_copy_pages_cow(cuda_device, kv_dtype):
    rng, pool, ora, bt = _setup(kv_dtype, layers=2, pool_pages=64)
    n = 12
    ids = rng.permutation(64)[:2 * n].astype(np.int32)
    src_ids, dst_ids = ids[:n], ids[n:]
    ks = rng.standard_normal((n, 2, H, PAGE_TOKENS, D)).astype(np.float16)
    vs = rng.standard_normal((n, 2, H, PAGE_TOKENS, D)).astype(np.float16)
    pool.write_pages(torch.from_numpy(src_ids).to(cuda_device), torch.from_numpy(ks).to(cuda_device),
                     torch.from_numpy(vs).to(cuda_device))
    ora.write_pages(src_ids, ks.astype(np.float32), vs.astype(np.float32))
    pool.copy_pages(torch.from_numpy(src_ids).to(cuda_device), torch.from_numpy(dst_ids).to(cuda_device))
    ora.copy_pages(src_ids, dst_ids)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_pool_np(pool), ora.data)
    if kv_dtype != "fp16":
        np.testing.assert_array_equal(pool.scale_view().cpu().numpy().view(np.uint8), ora.scales.view(np.uint8))
    pool.close()
