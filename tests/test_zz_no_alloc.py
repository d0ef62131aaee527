"""The no-allocation decode entry point, called through the C ABI.

sckv_decode_attn_noalloc serves callers that cannot allocate device memory
(a host whose HBM is owned up front by another allocator, or a binding that
only holds the pool handle): its split-K partials live in a fixed device
array inside the library instead of a caller-provided workspace. This test
checks it against the allocating entry point, sckv_decode_attn, on two calls
in a row (the shared array keeps the previous call's contents, which must
not matter), that an oversized request is refused before any launch (after
the usual argument checks), and that an unsplit request, which needs no
scratch, is never refused.
It lives in its own file, collected last, and builds all of its own state so
it passes alone in a fresh process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3  # decode tolerance used by the other attention tests


def _rel_err(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _pool_with_pages(dev, layers, hkv, pages, seed):
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(seed)
    pool = KVPool(layers, hkv, 128, pages, "fp16", device=dev)
    k = torch.from_numpy(rng.standard_normal((pages, layers, hkv, 16, 128)).astype(np.float16)).to(dev)
    v = torch.from_numpy(rng.standard_normal((pages, layers, hkv, 16, 128)).astype(np.float16)).to(dev)
    pool.write_pages(torch.arange(pages, dtype=torch.int32, device=dev), k, v)
    return pool, rng


def _call_allocating(lib, pool, layer, q, bt, max_blocks, ctx, out, chunk):
    from synapcore_b200 import _native as N

    B, hq, _ = q.shape
    need = lib.sckv_decode_workspace_bytes(pool.handle, B, hq, max_blocks, chunk)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    rc = lib.sckv_decode_attn(pool.handle, layer, q.data_ptr(), N.DTYPE_F16, hq, bt.data_ptr(), bt.stride(0),
                              max_blocks, ctx.data_ptr(), B, ctypes.c_float(128 ** -0.5), out.data_ptr(),
                              N.DTYPE_F32, ws.data_ptr(), ws.numel(), chunk,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == N.SCKV_OK


def _call_noalloc(lib, pool, layer, q, bt, max_blocks, ctx, out, chunk):
    from synapcore_b200 import _native as N

    B, hq, _ = q.shape
    return lib.sckv_decode_attn_noalloc(pool.handle, layer, q.data_ptr(), N.DTYPE_F16, hq, bt.data_ptr(),
                                        bt.stride(0), max_blocks, ctx.data_ptr(), B, ctypes.c_float(128 ** -0.5),
                                        out.data_ptr(), N.DTYPE_F32, chunk,
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_decode_matches_allocating_entry_point(cuda_device):
    from synapcore_b200 import _native as N

    lib = N.load()
    dev = cuda_device
    pool, rng = _pool_with_pages(dev, layers=2, hkv=4, pages=96, seed=42)
    hq, max_blocks = 16, 40
    # two different request shapes; each is run twice in a row
    cases = [([3, 70, 640, 17, 255, 16], 0), ([500, 1, 333], 4)]
    for ctx_list, chunk in cases:
        B = len(ctx_list)
        bt = torch.from_numpy(np.stack([rng.choice(96, size=max_blocks, replace=False) for _ in range(B)])
                              .astype(np.int32)).to(dev)
        ctx = torch.tensor(ctx_list, dtype=torch.int32, device=dev)
        q = torch.from_numpy(rng.standard_normal((B, hq, 128)).astype(np.float16)).to(dev)
        for layer in range(2):
            ref = torch.empty((B, hq, 128), dtype=torch.float32, device=dev)
            _call_allocating(lib, pool, layer, q, bt, max_blocks, ctx, ref, chunk)
            for _ in range(2):
                out = torch.full((B, hq, 128), float("nan"), dtype=torch.float32, device=dev)
                assert _call_noalloc(lib, pool, layer, q, bt, max_blocks, ctx, out, chunk) == N.SCKV_OK
                torch.cuda.synchronize()
                assert pool.status()[0] == N.SCKV_OK
                got, exp = out.cpu().numpy(), ref.cpu().numpy()
                for b in range(B):
                    assert _rel_err(got[b], exp[b]) <= TOL
    pool.close()


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device):
    from synapcore_b200 import _native as N

    lib = N.load()
    dev = cuda_device
    pool, rng = _pool_with_pages(dev, layers=1, hkv=4, pages=16, seed=3)
    hq, B, max_blocks = 16, 8, 4096
    # chunk_pages=1 over 4096 blocks needs 8*16*4096*520 bytes of partials,
    # far above the fixed 4 MiB; the block table is a full [B, 4096] of valid
    # ids so even a launch would stay in bounds.
    bt = torch.zeros((B, max_blocks), dtype=torch.int32, device=dev)
    ctx = torch.full((B,), 20, dtype=torch.int32, device=dev)
    q = torch.zeros((B, hq, 128), dtype=torch.float16, device=dev)
    out = torch.zeros((B, hq, 128), dtype=torch.float32, device=dev)
    assert _call_noalloc(lib, pool, 0, q, bt, max_blocks, ctx, out, 1) == N.SCKV_ERR_SCRATCH_LIMIT
    # an invalid call is reported as such even when it is also oversized, so
    # a caller that falls back to the allocating entry point on the scratch
    # limit is not misled
    assert _call_noalloc(lib, pool, 1, q, bt, max_blocks, ctx, out, 1) == N.SCKV_ERR_INVALID_ARG
    torch.cuda.synchronize()
    assert pool.status()[0] == N.SCKV_OK
    assert N.status_string(N.SCKV_ERR_SCRATCH_LIMIT) == "request exceeds the fixed no-allocation scratch"
    pool.close()


def test_noalloc_unsplit_large_batch_needs_no_scratch(cuda_device):
    """An unsplit launch writes its output directly and uses none of the
    fixed array, so a batch whose partials would not fit (512 sequences x 32
    query heads, GQA 32/8) still runs at one split, and its result matches
    the oracle's SDPA over the same pages."""
    from oracle.kv_oracle import sdpa_decode
    from synapcore_b200 import _native as N

    lib = N.load()
    dev = cuda_device
    pool, rng = _pool_with_pages(dev, layers=1, hkv=8, pages=64, seed=7)
    hq, B, max_blocks = 32, 512, 4
    bt_np = np.stack([rng.choice(64, size=max_blocks, replace=False) for _ in range(B)]).astype(np.int32)
    ctx_np = rng.integers(1, max_blocks * 16 + 1, size=B).astype(np.int32)
    bt = torch.from_numpy(bt_np).to(dev)
    ctx = torch.from_numpy(ctx_np).to(dev)
    q = torch.from_numpy(rng.standard_normal((B, hq, 128)).astype(np.float16)).to(dev)
    # 512 * 32 * 2 splits * 520 bytes = 17 MB of partials: refused when split
    assert lib.sckv_decode_workspace_bytes(pool.handle, B, hq, max_blocks, 2) > N.NOALLOC_SCRATCH_BYTES
    assert _call_noalloc(lib, pool, 0, q, bt, max_blocks, ctx, torch.empty((B, hq, 128), dtype=torch.float32,
                                                                          device=dev), 2) == N.SCKV_ERR_SCRATCH_LIMIT
    assert lib.sckv_decode_workspace_bytes(pool.handle, B, hq, max_blocks, max_blocks) == 0
    k_all = pool.pool_view()[0, :, 0].float().cpu().numpy()  # [pages, hkv, 16, 128]
    v_all = pool.pool_view()[0, :, 1].float().cpu().numpy()
    q_np = q.float().cpu().numpy()
    for chunk in (max_blocks, 0):  # explicit single split, and the default pick widened to fit
        for _ in range(2):
            out = torch.full((B, hq, 128), float("nan"), dtype=torch.float32, device=dev)
            assert _call_noalloc(lib, pool, 0, q, bt, max_blocks, ctx, out, chunk) == N.SCKV_OK
            torch.cuda.synchronize()
            assert pool.status()[0] == N.SCKV_OK
            got = out.cpu().numpy()
            for b in range(0, B, 37):
                n = int(ctx_np[b])
                pages = bt_np[b, : (n + 15) // 16]
                kk = np.concatenate([k_all[p] for p in pages], axis=1)[:, :n]
                vv = np.concatenate([v_all[p] for p in pages], axis=1)[:, :n]
                exp = sdpa_decode(q_np[b], kk, vv)
                assert _rel_err(got[b], exp) <= TOL
    pool.close()
