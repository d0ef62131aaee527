"""A whole attention layer on the device (PagedAttentionLayer: sckv_qkv_append,
sckv_prefill_attn / sckv_decode_attn, sckv_o_proj) against the reference
engine's forward_numpy outputs recorded in tests/golden, and against the
oracle's composition of the same steps over batches of sequences; plus the
output projection alone (sckv_o_proj) against an fp64 matmul.

Tolerances: layer outputs within 2e-3 of the output's largest value (the
attention bar: fp32 accumulation, fp32 queries rounded to the pool's type
inside the attention kernels); appended K / V within one 16-bit ulp plus
1e-4 of the row maximum (projection sum order); o_proj within 2e-5 of the
row's largest magnitude (fp32 accumulation over in_features; an fp32 input
enters as hi + lo, ~2^-22 relative), plus half an ulp for 16-bit outputs.
"""
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O

pytestmark = pytest.mark.gpu

D = 128
GOLD_DIR = Path(__file__).resolve().parent / "golden"
GOLD = json.loads((GOLD_DIR / "golden.json").read_text())
ARR = np.load(GOLD_DIR / "golden_arrays.npz")
ATTN_TOL = 2e-3


def _ulp16(x):
    e = np.floor(np.log2(np.maximum(np.abs(x), 2.0 ** -14)))
    return 2.0 ** (e - 10)


def _dev(a, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(dev) if dt is None else t.to(dev, dt)


def _rel_err(got, ref):
    return float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))


@pytest.mark.parametrize("case", [c["name"] for c in GOLD["attention_layer"]])
def test_layer_matches_reference_engine(cuda_device, case):
    """Each recorded forward_numpy call (GQA prompt after a cached prefix with
    per-head QK-norm; MHA decode with whole-width norms; MQA prompt with an
    empty cache) replayed through PagedAttentionLayer."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache

    sys.path.insert(0, str(GOLD_DIR))
    from attn_layer_inputs import attn_layer_inputs

    dev = cuda_device
    g = next(c for c in GOLD["attention_layer"] if c["name"] == case)
    hq, hkv, prefix, T = g["hq"], g["hkv"], g["prefix"], g["T"]
    inp = attn_layer_inputs(hq, hkv, prefix, T, g["norm"], g["seed"])
    cache = PagedKVCache(1, hkv, D, max_pages=64, max_seqs=2, max_blocks_per_seq=32, kv_dtype="fp16", device=dev)
    cache.add_sequence("s")
    if prefix:
        cache.append_prefill("s", _dev(inp["pk"].transpose(1, 0, 2), dev), _dev(inp["pv"].transpose(1, 0, 2), dev))
    layer = PagedAttentionLayer(cache, hq, rope_theta=g["theta"], rms_eps=g["eps"])
    w = [_dev(inp[k], dev) for k in ("wq", "wk", "wv", "wo")]
    qn = None if inp["qn"] is None else _dev(inp["qn"], dev)
    kn = None if inp["kn"] is None else _dev(inp["kn"], dev)
    x = _dev(inp["x"], dev)
    if T == 1 and prefix:
        out = layer.decode(0, x, 1, *w, q_norm_w=qn, k_norm_w=kn)
    else:
        out = layer.prefill(0, "s", x, *w, q_norm_w=qn, k_norm_w=kn)
    torch.cuda.synchronize()
    cache.pool.raise_on_status()
    ref = ARR[f"attn_layer_{case}_out"]
    got = out.cpu().numpy()
    assert got.shape == ref.shape
    assert _rel_err(got, ref) <= ATTN_TOL, _rel_err(got, ref)
    assert cache.length("s") == prefix + T
    kc, vc = cache.gather("s")
    for got_kv, ref_kv in ((kc[0, :, prefix:], ARR[f"attn_layer_{case}_k_new"]),
                           (vc[0, :, prefix:], ARR[f"attn_layer_{case}_v_new"])):
        r = ref_kv.astype(np.float32)
        gk = got_kv.float().cpu().numpy()
        assert np.all(np.abs(gk - r) <= _ulp16(r) + 1e-4 * np.max(np.abs(r), axis=-1, keepdims=True))
    if prefix:
        # the cached prefix is untouched
        np.testing.assert_array_equal(kc[0, :, :prefix].cpu().numpy(), inp["pk"])


def test_layer_batched_prompts_then_decode_steps_match_oracle(cuda_device):
    """Qwen3-style GQA 16/4 with per-head QK-norm, two layers, six sequences:
    prompts of ragged lengths through prefill, then three decode steps for
    all rows at once; every output against the oracle's forward_numpy
    composition over that sequence's own history."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache

    dev = cuda_device
    hq, hkv, L = 16, 4, 2
    hidden = hq * D
    eps, theta = 1e-6, 1000000.0
    rng = np.random.default_rng(5)
    sd = 1.0 / np.sqrt(hidden)
    W = [[(rng.standard_normal(s) * sd).astype(np.float16)
          for s in ((hq * D, hidden), (hkv * D, hidden), (hkv * D, hidden), (hidden, hq * D))] for _ in range(L)]
    NW = [[rng.uniform(0.5, 1.5, D).astype(np.float16) for _ in range(2)] for _ in range(L)]
    Wd = [[_dev(w, dev) for w in ws] for ws in W]
    NWd = [[_dev(w, dev) for w in ws] for ws in NW]
    cache = PagedKVCache(L, hkv, D, max_pages=256, max_seqs=8, max_blocks_per_seq=32, kv_dtype="fp16", device=dev)
    layer = PagedAttentionLayer(cache, hq, rope_theta=theta, rms_eps=eps)
    prompts = [5, 40, 130, 300, 16, 1]
    hist_k = [[None] * L for _ in prompts]
    hist_v = [[None] * L for _ in prompts]
    worst = 0.0
    for b, T in enumerate(prompts):
        cache.add_sequence(b)
        for l in range(L):
            x = rng.standard_normal((T, hidden)).astype(np.float32)
            out = layer.prefill(l, b, _dev(x, dev), *Wd[l], q_norm_w=NWd[l][0], k_norm_w=NWd[l][1])
            ref, hist_k[b][l], hist_v[b][l] = O.attention_layer(x, *W[l], hq, hkv, hist_k[b][l], hist_v[b][l],
                                                                NW[l][0], NW[l][1], eps, theta)
            e = _rel_err(out.cpu().numpy(), ref)
            worst = max(worst, e)
            assert e <= ATTN_TOL, (b, l, e)
    n = len(prompts)
    for step in range(3):
        for l in range(L):
            x = rng.standard_normal((n, hidden)).astype(np.float32)
            out = layer.decode(l, _dev(x, dev), n, *Wd[l], q_norm_w=NWd[l][0], k_norm_w=NWd[l][1]).cpu().numpy()
            for b in range(n):
                ref, hist_k[b][l], hist_v[b][l] = O.attention_layer(x[b:b + 1], *W[l], hq, hkv, hist_k[b][l],
                                                                    hist_v[b][l], NW[l][0], NW[l][1], eps, theta)
                e = _rel_err(out[b:b + 1], ref)
                worst = max(worst, e)
                assert e <= ATTN_TOL, (step, l, b, e)
    torch.cuda.synchronize()
    cache.pool.raise_on_status()
    for b, T in enumerate(prompts):
        assert cache.length(b) == T + 3
    print("worst relative error", worst)


def test_layer_prompt_batch_matches_oracle(cuda_device):
    """Several prompts (one of them empty) through one prefill_batch call per
    layer, then a decode step: every output against the oracle's
    forward_numpy composition over that sequence's own history."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache

    dev = cuda_device
    hq, hkv, L = 8, 2, 2
    hidden = hq * D
    eps, theta = 1e-6, 10000.0
    rng = np.random.default_rng(17)
    sd = 1.0 / np.sqrt(hidden)
    W = [[(rng.standard_normal(sh) * sd).astype(np.float16)
          for sh in ((hq * D, hidden), (hkv * D, hidden), (hkv * D, hidden), (hidden, hq * D))] for _ in range(L)]
    NW = [[rng.uniform(0.5, 1.5, D).astype(np.float16) for _ in range(2)] for _ in range(L)]
    Wd = [[_dev(w, dev) for w in ws] for ws in W]
    NWd = [[_dev(w, dev) for w in ws] for ws in NW]
    cache = PagedKVCache(L, hkv, D, max_pages=128, max_seqs=8, max_blocks_per_seq=32, kv_dtype="fp16", device=dev)
    layer = PagedAttentionLayer(cache, hq, rope_theta=theta, rms_eps=eps)
    prompts = [70, 0, 200, 17]
    cu = np.concatenate([[0], np.cumsum(prompts)]).tolist()
    for b in range(len(prompts)):
        cache.add_sequence(b)
    hist_k = [[None] * L for _ in prompts]
    hist_v = [[None] * L for _ in prompts]
    for l in range(L):
        x = rng.standard_normal((cu[-1], hidden)).astype(np.float32)
        out = layer.prefill_batch(l, range(len(prompts)), _dev(x, dev), cu, *Wd[l], q_norm_w=NWd[l][0],
                                  k_norm_w=NWd[l][1]).cpu().numpy()
        for b, T in enumerate(prompts):
            if T == 0:
                continue
            ref, hist_k[b][l], hist_v[b][l] = O.attention_layer(x[cu[b]:cu[b + 1]], *W[l], hq, hkv, hist_k[b][l],
                                                                hist_v[b][l], NW[l][0], NW[l][1], eps, theta)
            assert _rel_err(out[cu[b]:cu[b + 1]], ref) <= ATTN_TOL, (l, b)
    for b, T in enumerate(prompts):
        assert cache.length(b) == T
    # the empty prompt's sequence decodes from position 0
    n = len(prompts)
    for l in range(L):
        x = rng.standard_normal((n, hidden)).astype(np.float32)
        out = layer.decode(l, _dev(x, dev), n, *Wd[l], q_norm_w=NWd[l][0], k_norm_w=NWd[l][1]).cpu().numpy()
        for b in range(n):
            ref, hist_k[b][l], hist_v[b][l] = O.attention_layer(x[b:b + 1], *W[l], hq, hkv, hist_k[b][l],
                                                                hist_v[b][l], NW[l][0], NW[l][1], eps, theta)
            assert _rel_err(out[b:b + 1], ref) <= ATTN_TOL, (l, b)
    torch.cuda.synchronize()
    cache.pool.raise_on_status()


@pytest.mark.parametrize("norm", ["head", "full"])
def test_layer_on_int8_pool_matches_oracle(cuda_device, norm):
    """The arena's int8 mode under a whole layer: new K / V rows quantised by
    the fused projection epilogue (quantize_kv_int8), attention over the
    dequantised pages, against the oracle's composition with the same int8
    round trip of the cache. A prompt, then two decode steps (the second
    crossing into a fresh page for one sequence)."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache

    dev = cuda_device
    hq, hkv = 8, 2
    hidden = hq * D
    eps, theta = 1e-6, 10000.0
    rng = np.random.default_rng(23)
    sd = 1.0 / np.sqrt(hidden)
    W = [(rng.standard_normal(sh) * sd).astype(np.float16)
         for sh in ((hq * D, hidden), (hkv * D, hidden), (hkv * D, hidden), (hidden, hq * D))]
    # per-head norm weights (fused projection), or whole-width ones (the
    # unfused route: fp32 projections, then append_rope)
    NW = [rng.uniform(0.5, 1.5, D if norm == "head" else h * D).astype(np.float16) for h in (hq, hkv)]
    Wd = [_dev(w, dev) for w in W]
    NWd = [_dev(w, dev) for w in NW]
    cache = PagedKVCache(1, hkv, D, max_pages=64, max_seqs=4, max_blocks_per_seq=16, kv_dtype="int8", device=dev)
    layer = PagedAttentionLayer(cache, hq, rope_theta=theta, rms_eps=eps)
    prompts = [47, 15]
    hk = [None, None]
    hv = [None, None]
    for b, T in enumerate(prompts):
        cache.add_sequence(b)
        x = rng.standard_normal((T, hidden)).astype(np.float32)
        out = layer.prefill(0, b, _dev(x, dev), *Wd, q_norm_w=NWd[0], k_norm_w=NWd[1]).cpu().numpy()
        ref, hk[b], hv[b] = O.attention_layer(x, *W, hq, hkv, hk[b], hv[b], NW[0], NW[1], eps, theta, int8_cache=True)
        assert _rel_err(out, ref) <= ATTN_TOL, b
    for step in range(2):
        x = rng.standard_normal((2, hidden)).astype(np.float32)
        out = layer.decode(0, _dev(x, dev), 2, *Wd, q_norm_w=NWd[0], k_norm_w=NWd[1]).cpu().numpy()
        for b in range(2):
            ref, hk[b], hv[b] = O.attention_layer(x[b:b + 1], *W, hq, hkv, hk[b], hv[b], NW[0], NW[1], eps, theta,
                                                  int8_cache=True)
            assert _rel_err(out[b:b + 1], ref) <= ATTN_TOL, (step, b)
    torch.cuda.synchronize()
    cache.pool.raise_on_status()


def test_layer_on_fp8_pool_matches_oracle_over_its_pages(cuda_device):
    """FP8 pools under a whole layer (rows staged, then the FP8 append): a
    prompt then a decode step; each output against the oracle's causal SDPA
    and o_proj over the K / V the pool actually holds (decoded from its
    pages), with the oracle's own rotated q. How the rows are encoded is
    checked against the oracle's FP8 pool in test_gpu_qkv.py."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache

    dev = cuda_device
    hq, hkv = 8, 2
    hidden = hq * D
    eps, theta = 1e-6, 10000.0
    rng = np.random.default_rng(29)
    sd = 1.0 / np.sqrt(hidden)
    W = [(rng.standard_normal(sh) * sd).astype(np.float16)
         for sh in ((hq * D, hidden), (hkv * D, hidden), (hkv * D, hidden), (hidden, hq * D))]
    NW = [rng.uniform(0.5, 1.5, D).astype(np.float16) for _ in range(2)]
    cache = PagedKVCache(1, hkv, D, max_pages=32, max_seqs=2, max_blocks_per_seq=8, kv_dtype="fp8_e4m3",
                         device=dev)
    layer = PagedAttentionLayer(cache, hq, rope_theta=theta, rms_eps=eps)
    cache.add_sequence("s")
    inv = O.rope_inv_freq(theta, D)
    start = 0
    for T in (37, 1):
        x = rng.standard_normal((T, hidden)).astype(np.float32)
        xd = _dev(x, dev)
        wd = [_dev(w, dev) for w in W]
        if T > 1:
            out = layer.prefill(0, "s", xd, *wd, q_norm_w=_dev(NW[0], dev), k_norm_w=_dev(NW[1], dev))
        else:
            out = layer.decode(0, xd, 1, *wd, q_norm_w=_dev(NW[0], dev), k_norm_w=_dev(NW[1], dev))
        torch.cuda.synchronize()
        cache.pool.raise_on_status()
        n = start + T
        pages = cache.page_ids("s")
        codes = cache.pool.pool_view()[0].cpu().numpy()
        scales = cache.pool.scale_view()[0].cpu().numpy()
        kv = np.stack([np.concatenate([O.fp8_decode(codes[pg, i]) * scales[pg, i][:, None, None] for pg in pages],
                                      axis=1)[:, :n] for i in range(2)])        # [2, Hkv, n, D]
        q, k, _ = O.qkv_project(x, *(w.astype(np.float32) for w in W[:3]), hq, hkv)
        qr, _ = O.qk_norm_rope(q, k, NW[0], NW[1], eps, inv, 1.0, start)
        ref = O.o_project(O.sdpa_prefill(qr, kv[0], kv[1], start), W[3])
        assert _rel_err(out.cpu().numpy(), ref) <= ATTN_TOL, T
        start = n


@pytest.mark.parametrize("n_tok,fin,fout,x_kind,wdt,out_dtype", [
    (1, 512, 1024, "f32", torch.float16, torch.float32),        # decode size: split over in_features
    (128, 4096, 4096, "f32", torch.float16, torch.float32),     # Qwen3-8B decode batch, 4-way split
    (300, 1024, 512, "16", torch.float16, torch.float32),       # two token tiles, the second partial
    (77, 2048, 2048, "16", torch.bfloat16, torch.bfloat16),     # bf16, 16-bit output
    (200, 520, 256, "f32", torch.bfloat16, torch.float16),      # in_features % 64 != 0
    (1300, 4096, 4096, "f32", torch.float16, torch.float32),    # enough tiles for two output tiles per CTA
])
def test_o_proj_matches_fp64(cuda_device, n_tok, fin, fout, x_kind, wdt, out_dtype):
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    rng = np.random.default_rng(n_tok + fin)
    x = rng.standard_normal((n_tok, fin)).astype(np.float32)
    w = torch.from_numpy((rng.standard_normal((fout, fin)) / np.sqrt(fin)).astype(np.float32)).to(wdt)
    x_t = torch.from_numpy(x) if x_kind == "f32" else torch.from_numpy(x).to(wdt)
    ref = x_t.double().numpy() @ w.double().numpy().T
    pool = KVPool(1, 1, D, 4, "fp16", device=dev)
    out = pool.o_proj(x_t.to(dev), w.to(dev), out_dtype=out_dtype)
    torch.cuda.synchronize()
    pool.raise_on_status()
    got = out.double().cpu().numpy()
    row = np.max(np.abs(ref), axis=-1, keepdims=True)
    rnd = 0.0
    if out_dtype != torch.float32:
        rnd = np.abs(ref) * (2.0 ** -8 if out_dtype == torch.bfloat16 else 2.0 ** -11)
    assert np.all(np.abs(got - ref) <= 2e-5 * row + rnd), float(np.max(np.abs(got - ref) / row))


def test_o_proj_rejects_unsupported_shapes(cuda_device):
    from synapcore_b200 import _native as N
    from synapcore_b200.pool import KVPool

    dev = cuda_device
    pool = KVPool(1, 1, D, 4, "fp16", device=dev)
    x = torch.randn(4, 256, device=dev, dtype=torch.float16)
    with pytest.raises(N.SCKVError) as e:
        pool.o_proj(x, torch.randn(100, 256, device=dev, dtype=torch.float16))  # out_features % 128
    assert e.value.code == N.SCKV_ERR_UNSUPPORTED
    with pytest.raises(N.SCKVError) as e:
        pool.o_proj(torch.randn(4, 100, device=dev, dtype=torch.float16),
                    torch.randn(128, 100, device=dev, dtype=torch.float16))  # in_features % 8
    assert e.value.code == N.SCKV_ERR_UNSUPPORTED
    with pytest.raises(TypeError):
        pool.o_proj(x, torch.randn(128, 256, device=dev, dtype=torch.bfloat16))  # f16 x, bf16 weights
    # empty batch: nothing launched, empty result
    assert pool.o_proj(x[:0], torch.randn(128, 256, device=dev, dtype=torch.float16)).shape == (0, 128)
