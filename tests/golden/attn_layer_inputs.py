"""Seeded inputs of the attention-layer golden cases, shared by
make_golden.py (which runs them through the reference's
ModularAttentionEngine.forward_numpy) and the tests (which regenerate them
and compare against the recorded outputs)."""
from __future__ import annotations

import numpy as np

ATTN_LAYER_CASES = (
    # name, adapter, hq, hkv, prefix tokens, new tokens, qk-norm weights, rope theta, seed
    ("qwen_gqa_prefill", "qwen2_moe", 8, 2, 37, 20, "head", 1000000.0, 21),
    ("olmoe_mha_decode", "olmoe", 4, 4, 300, 1, "full", 10000.0, 22),
    ("mixtral_mqa_prompt", "mixtral", 4, 1, 0, 33, None, 10000.0, 23),
)


def attn_layer_inputs(hq, hkv, prefix, T, norm, seed):
    """Seeded inputs of one attention-layer case (the tests regenerate them
    with the same calls): x ~ N(0, 1); fp16 weights ~ N(0, 1/hidden); norm
    weights ~ U[0.5, 1.5]; a cached prefix of `prefix` fp16 tokens."""
    d = 128
    hidden = hq * d
    rng = np.random.default_rng(seed)
    sd = 1.0 / np.sqrt(hidden)
    x = rng.standard_normal((T, hidden)).astype(np.float32)
    wq = (rng.standard_normal((hq * d, hidden)) * sd).astype(np.float16)
    wk = (rng.standard_normal((hkv * d, hidden)) * sd).astype(np.float16)
    wv = (rng.standard_normal((hkv * d, hidden)) * sd).astype(np.float16)
    wo = (rng.standard_normal((hidden, hq * d)) * sd).astype(np.float16)
    qn = kn = None
    if norm == "head":
        qn = rng.uniform(0.5, 1.5, d).astype(np.float16)
        kn = rng.uniform(0.5, 1.5, d).astype(np.float16)
    elif norm == "full":
        qn = rng.uniform(0.5, 1.5, hq * d).astype(np.float16)
        kn = rng.uniform(0.5, 1.5, hkv * d).astype(np.float16)
    pk = rng.standard_normal((hkv, prefix, d)).astype(np.float16) if prefix else None
    pv = rng.standard_normal((hkv, prefix, d)).astype(np.float16) if prefix else None
    return {"x": x, "wq": wq, "wk": wk, "wv": wv, "wo": wo, "qn": qn, "kn": kn, "pk": pk, "pv": pv}
