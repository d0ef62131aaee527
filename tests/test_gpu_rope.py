"""Fused QK-norm + RoPE + append (sckv_append_rope) against the reference's
composition (models/adapters.py:1171-1207): the golden vectors made by the
reference engine, and the oracle on larger varlen batches.

Tolerances: the kernel computes in fp32 with IEEE operations in the
reference's order; cos / sin of the angle come from CUDA's sincosf, numpy's
from its own float32 routines, and the norm's sum runs in another order, so
the rotated q may differ by a few float32 ulps (checked at 4e-6 relative to
the row's largest value) and the cached K by at most one 16-bit ulp (a value
near a rounding boundary can round the other way). V is copied bit for bit.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu

GOLD_DIR = Path(__file__).resolve().parent / "golden"
GOLD = json.loads((GOLD_DIR / "golden.json").read_text())
ARR = np.load(GOLD_DIR / "golden_arrays.npz")


def _ulp16(x: np.ndarray, dt) -> np.ndarray:
    if dt == torch.float16:
        e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14)))
        return 2.0 ** (e - 10)
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -126)))
    return 2.0 ** (e - 7)


def _check_q(got, ref):
    scale = np.max(np.abs(ref), axis=-1, keepdims=True)
    assert np.all(np.abs(got - ref) <= 4e-6 * scale + 1e-30)


def _run(dev, kv_dtype, hq, hkv, Ts, starts, q_np, k_np, v_np, qw, kw, eps, inv, scaling, q_out_dtype=torch.float32):
    from synapcore_b200.pool import KVPool

    D = 128
    cu = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int32)
    mb = max((s + t + 15) // 16 for s, t in zip(starts, Ts))
    pool = KVPool(1, hkv, D, len(Ts) * mb, kv_dtype, device=dev)
    bt = np.arange(len(Ts) * mb, dtype=np.int32).reshape(len(Ts), mb)
    q_out = pool.append_rope(
        0, torch.from_numpy(q_np).to(dev), torch.from_numpy(k_np).to(dev),
        torch.from_numpy(v_np).to(dev), torch.from_numpy(cu).to(dev),
        torch.from_numpy(np.array(starts, np.int32)).to(dev), torch.from_numpy(bt).to(dev),
        torch.from_numpy(inv).to(dev), rope_scaling=scaling,
        q_norm_w=None if qw is None else torch.from_numpy(qw).to(dev),
        k_norm_w=None if kw is None else torch.from_numpy(kw).to(dev), eps=eps, q_out_dtype=q_out_dtype)
    torch.cuda.synchronize()
    pool.raise_on_status()
    view = pool.pool_view()[0]  # [P, 2, H, 16, D]
    ks, vs = [], []
    for b, (s, t) in enumerate(zip(starts, Ts)):
        pos = np.arange(s, s + t)
        pages = bt[b, pos // 16]
        ks.append(view[torch.from_numpy(pages).long(), 0, :, torch.from_numpy(pos % 16).long()].float().cpu().numpy())
        vs.append(view[torch.from_numpy(pages).long(), 1, :, torch.from_numpy(pos % 16).long()].cpu())
    return q_out.float().cpu().numpy(), ks, vs, cu


@pytest.mark.parametrize("case", [c["name"] for c in GOLD["qk_rope"]])
def test_fused_rope_matches_reference_golden(cuda_device, case):
    g = next(c for c in GOLD["qk_rope"] if c["name"] == case)
    q, k = ARR[f"rope_{case}_q"], ARR[f"rope_{case}_k"]
    qw = ARR[f"rope_{case}_qw"] if g["norm"] else None
    kw = ARR[f"rope_{case}_kw"] if g["norm"] else None
    v = np.random.default_rng(0).standard_normal(k.shape).astype(np.float32)
    qo, ks, vs, _ = _run(cuda_device, "fp16", g["hq"], g["hkv"], [g["T"]], [g["pos"]], q, k, v, qw, kw,
                         g["eps"], ARR[f"rope_{case}_inv_freq"], g["scaling"])
    _check_q(qo, ARR[f"rope_{case}_q_rot"])
    ref_k = ARR[f"rope_{case}_k_cache"].astype(np.float32)
    assert np.all(np.abs(ks[0] - ref_k) <= _ulp16(ref_k, torch.float16))
    assert torch.equal(vs[0], torch.from_numpy(v).half())


@pytest.mark.parametrize("kv_dtype,norm", [("fp16", "head"), ("fp16", "full"), ("bf16", "head"), ("bf16", None)])
def test_fused_rope_varlen_batch_matches_oracle(cuda_device, kv_dtype, norm):
    rng = np.random.default_rng(5)
    hq, hkv, D = 16, 4, 128
    Ts, starts = [3, 17, 1, 40], [0, 30, 511, 100]
    n = sum(Ts)
    q = rng.standard_normal((n, hq, D)).astype(np.float32) * 2
    k = rng.standard_normal((n, hkv, D)).astype(np.float32) * 2
    v = rng.standard_normal((n, hkv, D)).astype(np.float32)
    if norm == "head":
        qw, kw = rng.uniform(0.5, 1.5, D).astype(np.float16), rng.uniform(0.5, 1.5, D).astype(np.float16)
    elif norm == "full":
        qw, kw = (rng.uniform(0.5, 1.5, hq * D).astype(np.float16),
                  rng.uniform(0.5, 1.5, hkv * D).astype(np.float16))
    else:
        qw = kw = None
    inv = O.rope_inv_freq(1000000.0, D)
    qo, ks, vs, cu = _run(cuda_device, kv_dtype, hq, hkv, Ts, starts, q, k, v, qw, kw, 1e-6, inv, 1.0)
    dt = torch.float16 if kv_dtype == "fp16" else torch.bfloat16
    for b, (s, t) in enumerate(zip(starts, Ts)):
        qs, ksrc = q[cu[b]:cu[b + 1]], k[cu[b]:cu[b + 1]]
        qr, _ = O.qk_norm_rope(qs, ksrc, qw, kw, 1e-6, inv, 1.0, s)
        _check_q(qo[cu[b]:cu[b + 1]], qr)
        # K rotated in fp32 by the oracle's steps, rounded once to the pool's type
        kf = ksrc.reshape(1, t, hkv * D)
        if kw is not None:
            kf = (O.rmsnorm_f32(kf.reshape(1, t, hkv, D), kw, 1e-6).reshape(1, t, hkv * D) if kw.size == D
                  else O.rmsnorm_f32(kf, kw, 1e-6))
        kr32 = O.apply_rope_f32(kf.reshape(1, t, hkv, D).transpose(0, 2, 1, 3), inv, s, 1.0)[0].transpose(1, 0, 2)
        kref = torch.from_numpy(np.ascontiguousarray(kr32)).to(dt).float().numpy()
        assert np.all(np.abs(ks[b] - kref) <= _ulp16(kref, dt)), b
        assert torch.equal(vs[b], torch.from_numpy(v[cu[b]:cu[b + 1]]).to(dt)), b


@pytest.mark.parametrize("case", [c["name"] for c in GOLD["qk_rope"]])
def test_fused_rope_on_int8_pool_quantises_as_the_arena(cuda_device, case):
    """int8 pools: the rotated K row and the V row are stored as the arena's
    int8 mode stores fp16 pages (quantize_kv_int8 of the fp16 values). The
    reference golden K rows are the fp16 cache values; the kernel's fp16 K
    may sit one ulp away, so codes are compared through their dequantised
    values, within one quantisation step; V (fp16 input, copied) exactly."""
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    g = next(c for c in GOLD["qk_rope"] if c["name"] == case)
    q, k = ARR[f"rope_{case}_q"], ARR[f"rope_{case}_k"]
    qw = ARR[f"rope_{case}_qw"] if g["norm"] else None
    kw = ARR[f"rope_{case}_kw"] if g["norm"] else None
    v16 = np.random.default_rng(0).standard_normal(k.shape).astype(np.float16)
    v = v16.astype(np.float32)  # k's dtype; fp16-representable values
    T, hq, hkv, s0 = g["T"], g["hq"], g["hkv"], g["pos"]
    mb = (s0 + T + 15) // 16
    pool = KVPool(1, hkv, 128, mb, "int8", device=dev)
    bt = np.arange(mb, dtype=np.int32).reshape(1, mb)
    pool.append_rope(0, torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev),
                     torch.tensor([0, T], dtype=torch.int32, device=dev),
                     torch.tensor([s0], dtype=torch.int32, device=dev), torch.from_numpy(bt).to(dev),
                     torch.from_numpy(ARR[f"rope_{case}_inv_freq"]).to(dev), rope_scaling=g["scaling"],
                     q_norm_w=None if qw is None else torch.from_numpy(qw).to(dev),
                     k_norm_w=None if kw is None else torch.from_numpy(kw).to(dev), eps=g["eps"])
    torch.cuda.synchronize()
    pool.raise_on_status()
    pos = np.arange(s0, s0 + T)
    codes = pool.pool_view()[0].cpu().numpy()[bt[0, pos // 16], :, :, pos % 16]   # [T, 2, H, D]
    scales = pool.scale_view()[0].cpu().numpy()[bt[0, pos // 16], :, :, pos % 16]  # [T, 2, H]
    for kv, ref16 in ((0, ARR[f"rope_{case}_k_cache"]), (1, v16)):
        rq, rs = O.quantize_kv_int8(ref16)
        got = O.dequantize_kv_int8(codes[:, kv], scales[:, kv][..., None]).astype(np.float32)
        ref = O.dequantize_kv_int8(rq, rs).astype(np.float32)
        if kv == 1:
            np.testing.assert_array_equal(codes[:, kv], rq)
            np.testing.assert_array_equal(scales[:, kv], rs[..., 0])
        else:
            assert np.all(np.abs(got - ref) <= 1.01 * rs.astype(np.float32) + 2e-3 * np.abs(ref))
