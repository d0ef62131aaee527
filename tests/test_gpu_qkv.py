"""Fused projections + QK-norm + RoPE + append (sckv_qkv_append) against the
oracle's restatement of forward_numpy (models/adapters.py:1167-1207): fp32
x @ W^T, then qk_norm_rope, K / V rounded once to the pool's type.

Tolerance: the tensor cores sum the hidden dim in their own order (fp32
accumulation; an fp32 x enters as a 16-bit hi + lo pair, ~2^-22 relative),
so the projections differ from numpy's fp32 matmul by sum-order rounding.
q is checked at 1e-4 of its row's largest value; K and V at one 16-bit ulp
plus the same 1e-4 of the row maximum (a value near a rounding boundary can
round the other way). Indexing or layout mistakes show up as O(1) errors.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu

D = 128
TOL = 1e-4


def _ulp16(x, dt):
    if dt == torch.float16:
        e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14)))
        return 2.0 ** (e - 10)
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -126)))
    return 2.0 ** (e - 7)


def _rows_close(got, ref, extra=0.0):
    scale = np.max(np.abs(ref), axis=-1, keepdims=True)
    assert np.all(np.abs(got - ref) <= TOL * scale + extra + 1e-30), float(np.max(np.abs(got - ref) / (scale + 1e-30)))


def _run_case(dev, kv_dtype, wdt, x_kind, hq, hkv, hidden, Ts, starts, norm, q_out_dtype=torch.float32, seed=0):
    from synapcore_b200.pool import KVPool

    rng = np.random.default_rng(seed)
    n = sum(Ts)
    x = rng.standard_normal((n, hidden)).astype(np.float32)
    sc = 1.0 / np.sqrt(hidden)
    wq = (rng.standard_normal((hq * D, hidden)) * sc).astype(np.float32)
    wk = (rng.standard_normal((hkv * D, hidden)) * sc).astype(np.float32)
    wv = (rng.standard_normal((hkv * D, hidden)) * sc).astype(np.float32)
    if norm == "head":
        qw, kw = rng.uniform(0.5, 1.5, D).astype(np.float16), rng.uniform(0.5, 1.5, D).astype(np.float16)
    elif norm == "full":
        qw, kw = (rng.uniform(0.5, 1.5, hq * D).astype(np.float16),
                  rng.uniform(0.5, 1.5, hkv * D).astype(np.float16))
    else:
        qw = kw = None
    # weights and a 16-bit x in the MMA type; the oracle sees the same values
    wq_t, wk_t, wv_t = (torch.from_numpy(w).to(wdt) for w in (wq, wk, wv))
    wq32, wk32, wv32 = (w.float().numpy() for w in (wq_t, wk_t, wv_t))
    x_t = torch.from_numpy(x) if x_kind == "f32" else torch.from_numpy(x).to(wdt)
    x32 = x_t.float().numpy()
    inv = O.rope_inv_freq(1000000.0, D)

    cu = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int32)
    mb = max((s + t + 15) // 16 for s, t in zip(starts, Ts))
    P = len(Ts) * mb + 3
    pool = KVPool(2, hkv, D, P, kv_dtype, device=dev)
    bt = rng.permutation(P)[:len(Ts) * mb].reshape(len(Ts), mb).astype(np.int32)
    layer = 1
    q_out = pool.qkv_append(layer, x_t.to(dev), wq_t.to(dev), wk_t.to(dev), wv_t.to(dev),
                            torch.from_numpy(cu).to(dev), torch.from_numpy(np.array(starts, np.int32)).to(dev),
                            torch.from_numpy(bt).to(dev), torch.from_numpy(inv).to(dev), rope_scaling=1.0,
                            q_norm_w=None if qw is None else torch.from_numpy(qw).to(dev),
                            k_norm_w=None if kw is None else torch.from_numpy(kw).to(dev), eps=1e-6,
                            q_out_dtype=q_out_dtype)
    torch.cuda.synchronize()
    pool.raise_on_status()
    got_q = q_out.float().cpu().numpy()
    view = pool.pool_view()[layer]  # [P, 2, H, 16, D]
    dt = torch.float16 if kv_dtype == "fp16" else torch.bfloat16
    q_all, k_all, v_all = O.qkv_project(x32, wq32, wk32, wv32, hq, hkv)
    for b, (s, t) in enumerate(zip(starts, Ts)):
        if t == 0:
            continue
        sl = slice(cu[b], cu[b + 1])
        qr, _ = O.qk_norm_rope(q_all[sl], k_all[sl], qw, kw, 1e-6, inv, 1.0, s)
        rnd = 0.0 if q_out_dtype == torch.float32 else np.abs(qr) * (2.0 ** -8)
        _rows_close(got_q[sl], qr, rnd)
        kf = k_all[sl].reshape(1, t, hkv * D)
        if kw is not None:
            kf = (O.rmsnorm_f32(kf.reshape(1, t, hkv, D), kw, 1e-6).reshape(1, t, hkv * D) if kw.size == D
                  else O.rmsnorm_f32(kf, kw, 1e-6))
        k32 = O.apply_rope_f32(kf.reshape(1, t, hkv, D).transpose(0, 2, 1, 3), inv, s, 1.0)[0].transpose(1, 0, 2)
        pos = np.arange(s, s + t)
        pages = torch.from_numpy(bt[b, pos // 16]).long()
        slots = torch.from_numpy(pos % 16).long()
        got_k = view[pages, 0, :, slots].float().cpu().numpy()
        got_v = view[pages, 1, :, slots].float().cpu().numpy()
        for got, ref in ((got_k, k32), (got_v, v_all[sl])):
            ref_r = torch.from_numpy(np.ascontiguousarray(ref)).to(dt).float().numpy()
            _rows_close(got, ref_r, _ulp16(ref_r, dt))
    return pool


@pytest.mark.parametrize("kv_dtype,wdt,x_kind,norm,hq,hkv,hidden", [
    ("fp16", torch.float16, "f32", "head", 8, 2, 520),     # fp32 x as hi + lo; hidden % 64 != 0; 2-way split
    ("fp16", torch.float16, "16", None, 4, 4, 256),        # MHA, f16 x, no norm
    ("bf16", torch.bfloat16, "16", "head", 16, 4, 384),
    ("bf16", torch.bfloat16, "f32", None, 8, 1, 128),      # MQA
    ("fp16", torch.float16, "f32", "full", 8, 2, 256),     # whole-width norm: unfused route
    ("bf16", torch.bfloat16, "f32", "head", 4, 2, 2048),   # few tiles: hidden split 8 ways + finishing launch
])
def test_qkv_append_matches_oracle(cuda_device, kv_dtype, wdt, x_kind, norm, hq, hkv, hidden):
    Ts, starts = [5, 130, 1, 0, 77], [0, 16, 300, 4, 9]   # 213 tokens: two token tiles, the second partial
    _run_case(cuda_device, kv_dtype, wdt, x_kind, hq, hkv, hidden, Ts, starts, norm)


@pytest.mark.parametrize("wdt,x_kind", [(torch.bfloat16, "16"), (torch.float16, "f32")])
def test_qkv_append_two_heads_per_tile_with_odd_head_counts(cuda_device, wdt, x_kind):
    """1,600 tokens give enough tiles for two heads per CTA (N = 256); odd
    head counts leave the last group one head short."""
    kv = "bf16" if wdt == torch.bfloat16 else "fp16"
    _run_case(cuda_device, kv, wdt, x_kind, 15, 3, 192, [700, 900], [3, 40], "head", seed=9)


@pytest.mark.parametrize("q_out_dtype", [torch.float16, torch.bfloat16])
def test_qkv_append_16bit_q_out(cuda_device, q_out_dtype):
    _run_case(cuda_device, "fp16", torch.float16, "f32", 8, 2, 256, [40, 3], [7, 0], "head", q_out_dtype, seed=4)


def test_qkv_append_reports_bad_pages_and_rejects_unsupported(cuda_device):
    from synapcore_b200 import _native as N
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    hidden, hq, hkv = 128, 2, 1
    x = torch.randn(4, hidden, device=dev, dtype=torch.float16)
    w = [torch.randn(h * D, hidden, device=dev, dtype=torch.float16) * 0.05 for h in (hq, hkv, hkv)]
    cu = torch.tensor([0, 4], dtype=torch.int32, device=dev)
    st = torch.tensor([14], dtype=torch.int32, device=dev)
    inv = torch.from_numpy(O.rope_inv_freq(10000.0, D)).to(dev)
    pool = KVPool(1, hkv, D, 4, "fp16", device=dev)
    bt = torch.tensor([[2, 9]], dtype=torch.int32, device=dev)  # page 9 does not exist
    pool.qkv_append(0, x, *w, cu, st, bt, inv)
    torch.cuda.synchronize()
    code, detail, _, _ = pool.status()
    assert code == N.SCKV_ERR_BOUNDS and detail == 9
    pool.clear_status()
    d64 = KVPool(1, hkv, 64, 4, "fp16", device=dev)  # head_dim 128 only
    w64 = [torch.randn(h * 64, hidden, device=dev, dtype=torch.float16) * 0.05 for h in (hq, hkv, hkv)]
    with pytest.raises(N.SCKVError) as e:
        d64.qkv_append(0, x, *w64, cu, st, bt[:, :1], inv[:32])
    assert e.value.code == N.SCKV_ERR_UNSUPPORTED
    xb = torch.randn(4, 100, device=dev, dtype=torch.float16)  # hidden % 8 != 0
    wb = [torch.randn(h * D, 100, device=dev, dtype=torch.float16) for h in (hq, hkv, hkv)]
    with pytest.raises(N.SCKVError) as e:
        pool.qkv_append(0, xb, *wb, cu, st, bt, inv)
    assert e.value.code == N.SCKV_ERR_UNSUPPORTED


@pytest.mark.parametrize("hidden,Ts", [(256, [40, 3, 0, 90]), (2048, [5, 1, 9])])  # unsplit; split + finishing kernel
def test_qkv_append_int8_pool_quantises_rows_as_the_arena(cuda_device, hidden, Ts):
    """int8 pools: every new K / V row is stored as the arena's int8 mode
    stores its fp16 pages (quantize_kv_int8: per-row scale max|x|/127,
    round-half-even codes). The fp16 row may differ from numpy's by one ulp
    (projection sum order), so codes are checked through their dequantised
    values: within one quantisation step of the oracle's."""
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    rng = np.random.default_rng(31)
    hq, hkv = 8, 2
    n = sum(Ts)
    x = rng.standard_normal((n, hidden)).astype(np.float32)
    sc = 1.0 / np.sqrt(hidden)
    w = [(rng.standard_normal((h * D, hidden)) * sc).astype(np.float16) for h in (hq, hkv, hkv)]
    qw, kw = rng.uniform(0.5, 1.5, D).astype(np.float16), rng.uniform(0.5, 1.5, D).astype(np.float16)
    starts = [3, 17, 0, 40][:len(Ts)]
    inv = O.rope_inv_freq(10000.0, D)
    cu = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int32)
    mb = max((s + t + 15) // 16 for s, t in zip(starts, Ts))
    P = len(Ts) * mb + 2
    pool = KVPool(1, hkv, D, P, "int8", device=dev)
    bt = rng.permutation(P)[:len(Ts) * mb].reshape(len(Ts), mb).astype(np.int32)
    pool.qkv_append(0, torch.from_numpy(x).to(dev), *(torch.from_numpy(a).to(dev) for a in w),
                    torch.from_numpy(cu).to(dev), torch.from_numpy(np.array(starts, np.int32)).to(dev),
                    torch.from_numpy(bt).to(dev), torch.from_numpy(inv).to(dev), q_norm_w=torch.from_numpy(qw).to(dev),
                    k_norm_w=torch.from_numpy(kw).to(dev), eps=1e-6)
    torch.cuda.synchronize()
    pool.raise_on_status()
    codes = pool.pool_view()[0].cpu().numpy()      # [P, 2, H, 16, D] int8
    scales = pool.scale_view()[0].cpu().numpy()    # [P, 2, H, 16] fp16
    q_all, k_all, v_all = O.qkv_project(x, *(a.astype(np.float32) for a in w), hq, hkv)
    for b, (s0, t) in enumerate(zip(starts, Ts)):
        if t == 0:
            continue
        sl = slice(cu[b], cu[b + 1])
        _, k16 = O.qk_norm_rope(q_all[sl], k_all[sl], qw, kw, 1e-6, inv, 1.0, s0)   # [t, Hkv, D] fp16
        v16 = v_all[sl].astype(np.float16)
        pos = np.arange(s0, s0 + t)
        for kv, ref16 in ((0, k16), (1, v16)):
            rq, rs = O.quantize_kv_int8(ref16)
            ref = O.dequantize_kv_int8(rq, rs).astype(np.float32)
            gq = codes[bt[b, pos // 16], kv, :, pos % 16]          # [t, Hkv, D]
            gs = scales[bt[b, pos // 16], kv, :, pos % 16]         # [t, Hkv]
            got = O.dequantize_kv_int8(gq, gs[..., None]).astype(np.float32)
            step = rs.astype(np.float32)
            assert np.all(np.abs(got - ref) <= 1.01 * step + 2e-3 * np.abs(ref)), (b, kv)
            assert np.all(np.abs(gs.astype(np.float32) - rs[..., 0].astype(np.float32))
                          <= 2e-3 * rs[..., 0].astype(np.float32) + 1e-7)


def test_qkv_append_fp8_pool_through_the_fp8_append(cuda_device):
    """FP8 pools: the projection stages the new K / V rows in fp16 and the
    FP8 append stores them (per-page-head scale max|x| / 448, grown and
    re-encoded as later tokens of a page arrive). Two calls, the second
    filling pages the first left partial, against the oracle's FP8 pool fed
    the oracle's fp16 rows. A row one fp16 ulp off can move an e4m3 code by
    one step (2^-3 relative) and a page scale slightly, hence the bound."""
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    rng = np.random.default_rng(41)
    hq, hkv, hidden = 8, 2, 512
    sc = 1.0 / np.sqrt(hidden)
    w = [(rng.standard_normal((h * D, hidden)) * sc).astype(np.float16) for h in (hq, hkv, hkv)]
    qw, kw = rng.uniform(0.5, 1.5, D).astype(np.float16), rng.uniform(0.5, 1.5, D).astype(np.float16)
    inv = O.rope_inv_freq(10000.0, D)
    mb, P = 4, 16
    bt = rng.permutation(P)[:3 * mb].reshape(3, mb).astype(np.int32)
    pool = KVPool(1, hkv, D, P, "fp8_e4m3", device=dev)
    ora = O.PagedPoolOracle(1, hkv, D, P, "fp8_e4m3")
    lens = [0, 0, 0]
    for Ts in ([5, 20, 1], [7, 30, 16]):
        n = sum(Ts)
        x = rng.standard_normal((n, hidden)).astype(np.float32)
        cu = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int32)
        st = np.array(lens, np.int32)
        pool.qkv_append(0, torch.from_numpy(x).to(dev), *(torch.from_numpy(a).to(dev) for a in w),
                        torch.from_numpy(cu).to(dev), torch.from_numpy(st).to(dev), torch.from_numpy(bt).to(dev),
                        torch.from_numpy(inv).to(dev), q_norm_w=torch.from_numpy(qw).to(dev),
                        k_norm_w=torch.from_numpy(kw).to(dev), eps=1e-6)
        q_all, k_all, v_all = O.qkv_project(x, *(a.astype(np.float32) for a in w), hq, hkv)
        k16 = np.zeros((n, hkv, D), np.float16)
        for b in range(3):
            sl = slice(cu[b], cu[b + 1])
            if Ts[b]:
                _, k16[sl] = O.qk_norm_rope(q_all[sl], k_all[sl], qw, kw, 1e-6, inv, 1.0, lens[b])
        v16 = v_all.astype(np.float16)
        ora.append(0, k16.astype(np.float32)[None], v16.astype(np.float32)[None], cu, st, bt)
        lens = [a + b for a, b in zip(lens, Ts)]
    torch.cuda.synchronize()
    pool.raise_on_status()
    codes = pool.pool_view()[0].cpu().numpy()
    scales = pool.scale_view()[0].cpu().numpy()
    for b in range(3):
        for page in bt[b, :(lens[b] + 15) // 16]:
            for kv in range(2):
                ref = ora.values(0, page, kv)
                got = O.fp8_decode(codes[page, kv]) * scales[page, kv][:, None, None]
                pmax = np.max(np.abs(ref), axis=(1, 2), keepdims=True)
                assert np.all(np.abs(got - ref) <= 0.07 * np.abs(ref) + 0.01 * pmax), (b, page, kv)
