"""Decode attention parity at the benchmarked configurations' real shapes.

Each case builds the benchmark's own state (bench.build_state: the same pool
type, head counts, batch, contexts, random block-table permutation and pool
size), so the kernel variant and the default split-K chunk are exactly those
the benchmark times, runs the benchmark's step (append + decode for every
layer), and compares sampled sequences with the oracle SDPA
(models/adapters.py:1209-1229) over the same pages, dequantised by the
oracle:

  olmoe        fp16 MHA 16/16, 64 x 4,096, 16 layers (layers 0 and 15 checked)
  qwen3-fp8    FP8-e4m3 GQA 32/8, bf16 q, 128 x 16,384 (two sequences
               re-appended with K/V ~ N(0,1) * U[0.5,4] per head, two with the
               benchmark's random codes)
  qwen3-long   bf16 GQA 32/8, 64 sequences ~U[8192, 32768] with contexts
               8,192 / 20,000 / 32,768 among them, three growing steps
  qwen3-int8   the arena's int8 mode on the tensor-core kernel, 128 x 16,384

Tolerance (fp32 accumulation): max|o - o_ref| / max|o_ref| <= 2e-3 per
sequence. The benchmark stores 16-bit outputs; the comparison uses an fp32
output of the same launch shape, and the 16-bit outputs are checked against
it to within their own rounding.
"""
import gc

import numpy as np
import pytest
import torch

from oracle.kv_oracle import PAGE_TOKENS, dequantize_kv_int8, fp8_decode, sdpa_decode

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _rel_err(o, r):
    return float(np.max(np.abs(o - r)) / max(np.max(np.abs(r)), 1e-30))


def _bench():
    import bench

    return bench


def _seq_kv(pool, layer, bt_row, ctx):
    """K, V of one sequence in `layer` as float32 [H, ctx, D], dequantised
    with the oracle's functions from the raw page bytes."""
    n = (ctx + PAGE_TOKENS - 1) // PAGE_TOKENS
    ids = torch.as_tensor(np.asarray(bt_row[:n], np.int64), device=pool.device)
    raw = pool.pool_view()[layer].index_select(0, ids)  # [n, 2, H, 16, D]
    if pool.kv_dtype in ("fp16", "bf16"):
        vals = raw.float().cpu().numpy()
    elif pool.kv_dtype == "int8":
        sc = pool.scale_view()[layer].index_select(0, ids).cpu().numpy()  # [n, 2, H, 16] fp16
        vals = dequantize_kv_int8(raw.cpu().numpy(), sc[..., None]).astype(np.float32)
    else:
        sc = pool.scale_view()[layer].index_select(0, ids).cpu().numpy()  # [n, 2, H] fp32
        vals = fp8_decode(raw.cpu().numpy()) * sc[:, :, :, None, None]
    H, D = vals.shape[2], vals.shape[4]
    k = vals[:, 0].transpose(1, 0, 2, 3).reshape(H, n * PAGE_TOKENS, D)[:, :ctx]
    v = vals[:, 1].transpose(1, 0, 2, 3).reshape(H, n * PAGE_TOKENS, D)[:, :ctx]
    return np.ascontiguousarray(k), np.ascontiguousarray(v)


def _expected_splits(pool, B, max_blocks):
    """The library's default split (pick_chunk in csrc/sckv_decode.cu)."""
    sms = torch.cuda.get_device_properties(pool.device).multi_processor_count
    units = B * pool.num_kv_heads
    splits = max(1, (16 * sms * 3 + units - 1) // units)
    chunk = min(max(16, (max_blocks + splits - 1) // splits), max_blocks)
    return (max_blocks + chunk - 1) // chunk


def _check_layer(w, s, layer, seqs, out16=None):
    """fp32-output decode of `layer` with the benchmark's launch shape and
    default split, compared per sampled sequence with the oracle."""
    pool, bt = s["pool"], s["bt"]
    # a growing workload's step advances the contexts after its decode: check
    # the contexts that step attended over
    ctx = s["ctx"] - 1 if s["grow"] else s["ctx"]
    B, hq = w["batch"], w["hq"]
    mb = s["max_blocks"]
    splits = _expected_splits(pool, B, mb)
    assert splits > 1
    assert pool.decode_workspace_bytes(B, hq, mb) == B * hq * splits * (128 + 2) * 4
    q = s["q"][layer]
    out = pool.decode_attn(layer % s["n_phys"], q, bt, ctx, out_dtype=torch.float32)
    torch.cuda.synchronize()
    pool.raise_on_status()
    got = out.cpu().numpy()
    assert np.all(np.isfinite(got))
    if out16 is not None:
        o16 = out16.float().cpu().numpy()
        eps = 2.0 ** -8 if out16.dtype == torch.bfloat16 else 2.0 ** -10
        assert np.all(np.abs(o16 - got) <= eps * np.abs(got) + 1e-6)
    bt_h = bt.cpu().numpy()
    ctx_h = ctx.cpu().numpy()
    qv = q.float().cpu().numpy()
    errs = {}
    for b in seqs:
        k, v = _seq_kv(pool, layer % s["n_phys"], bt_h[b], int(ctx_h[b]))
        ref = sdpa_decode(qv[b], k, v)
        errs[b] = _rel_err(got[b], ref)
        assert errs[b] <= TOL, (layer, b, int(ctx_h[b]), errs[b])
    return errs


def _free(s):
    s["pool"].close()
    s.clear()
    gc.collect()
    torch.cuda.empty_cache()


def test_olmoe_decode_config_parity(cuda_device):
    """fp16 MHA 16/16, 64 sequences x 4,096 over a random permutation of the
    18,750-page pool, all 16 layers (the headline workload, as benchmarked)."""
    B = _bench()
    w = dict(B.WORKLOADS["olmoe"])
    s = B.build_state(w, 0)
    B.run_step(w, s)
    torch.cuda.synchronize()
    s["pool"].raise_on_status()
    for layer in (0, 15):
        errs = _check_layer(w, s, layer, seqs=[0, 21, 42, 63], out16=s["out"][layer])
        print(f"olmoe layer {layer}: max rel err {max(errs.values()):.2e}")
    _free(s)


def test_qwen3_fp8_decode_config_parity(cuda_device):
    """FP8-e4m3 GQA 32/8 with bf16 queries, 128 x 16,384 (default split of the
    benchmark). Sequences 5 and 77 are re-appended through the FP8 append
    with K/V ~ N(0,1) * U[0.5,4] per head; the stated FP8 bound is checked
    on their pages: every dequantised element within 2^-4 x its page-head
    max of the bf16 value it encodes."""
    B = _bench()
    w = dict(B.WORKLOADS["qwen3-fp8"], layers=3)
    s = B.build_state(w, 0)
    pool, dev = s["pool"], s["pool"].device
    ctx_h = s["ctx"].cpu().numpy()
    real = [5, 77]
    T = int(ctx_h[real[0]])
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    layer = 2
    src = {}
    for kv in ("k", "v"):
        f = torch.empty((1, w["hkv"], 1), device=dev).uniform_(0.5, 4.0, generator=g)
        src[kv] = (torch.randn((len(real) * T, w["hkv"], 128), generator=g, device=dev) * f).to(torch.bfloat16)
    cu = torch.tensor([0, T, 2 * T], dtype=torch.int32, device=dev)
    start = torch.zeros(2, dtype=torch.int32, device=dev)
    bt_real = s["bt"][real].contiguous()
    pool.append(src["k"], src["v"], cu, start, bt_real, layer0=layer)
    torch.cuda.synchronize()
    pool.raise_on_status()
    B.run_step(w, s)  # the benchmark's step: one appended token per sequence, then decode
    torch.cuda.synchronize()
    pool.raise_on_status()
    errs = _check_layer(w, s, layer, seqs=real + [0, 127], out16=s["out"][layer])
    print(f"qwen3-fp8 layer {layer}: max rel err {max(errs.values()):.2e}")
    # bound on the codes of the re-appended pages (the step rewrote slot T-1)
    bt_h = s["bt"].cpu().numpy()
    for i, b in enumerate(real):
        k8, v8 = _seq_kv(pool, layer, bt_h[b], T - 1)
        for x8, kv in ((k8, "k"), (v8, "v")):
            xb = src[kv][i * T: i * T + T - 1].float().cpu().numpy().transpose(1, 0, 2)  # [H, T-1, D]
            n_full = (T - 1) // PAGE_TOKENS * PAGE_TOKENS
            xb_p = xb[:, :n_full].reshape(w["hkv"], -1, PAGE_TOKENS, 128)
            x8_p = x8[:, :n_full].reshape(w["hkv"], -1, PAGE_TOKENS, 128)
            amax = np.max(np.abs(xb_p), axis=(2, 3), keepdims=True)
            assert np.all(np.abs(x8_p - xb_p) <= amax * 2.0 ** -4 + 1e-12)
    _free(s)


def test_qwen3_long_bf16_decode_config_parity(cuda_device):
    """bf16 GQA 32/8 with bf16 queries, 64 sequences ~U[8192, 32768] (three
    of them at 8,192, 20,000 and 32,768), contexts growing one token per step
    over three benchmark steps; parity checked after every step."""
    B = _bench()
    w = dict(B.WORKLOADS["qwen3-long"], layers=2)
    ctx0 = B.seq_contexts(w, 0)
    ctx0[:3] = [8192, 20000, 32768]
    s = B.build_state(w, 0, grow_steps=3, ctx0=ctx0)
    for step in range(3):
        B.run_step(w, s)
        torch.cuda.synchronize()
        s["pool"].raise_on_status()
        for layer in range(2):
            errs = _check_layer(w, s, layer, seqs=[0, 1, 2, 40], out16=s["out"][layer])
        print(f"qwen3-long step {step}: max rel err {max(errs.values()):.2e}")
    assert s["ctx"].cpu().tolist()[:3] == [8192 + 1 + 3, 20000 + 1 + 3, 32768 + 1 + 3]
    _free(s)


def test_qwen3_int8_decode_config_parity(cuda_device):
    """The arena's int8 mode (per-token fp16 scales) on the tensor-core
    kernel at 128 x 16,384 with bf16 queries: 1,024 pages per sequence, so the
    per-page K-offset correction and the V-scale reference moves run many
    times per item."""
    B = _bench()
    w = dict(B.WORKLOADS["qwen3-int8"], layers=2)
    s = B.build_state(w, 0)
    B.run_step(w, s)
    torch.cuda.synchronize()
    s["pool"].raise_on_status()
    errs = _check_layer(w, s, 1, seqs=[0, 63, 127], out16=s["out"][1])
    print(f"qwen3-int8: max rel err {max(errs.values()):.2e}")
    _free(s)
