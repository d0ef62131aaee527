"""A tiny seeded decoder used to drive both schedulers — TEST INFRASTRUCTURE.

`make_weights` builds the weights once (numpy, seeded). The reference side
(tests/golden/make_golden.py) wraps them in a stub of the reference engine
and runs the reference ContinuousBatchScheduler; the B200 side wraps the same
weights in `TorchStubModel` (the `PagedDecoderModel` protocol) and runs
synapcore_b200's scheduler over the paged GPU cache. The model math outside
attention restates the reference engine for this stub: RMSNorm
(native/native_engine.py:2927-2930), q/k/v projections with full-width
QK-norm and rotate-half RoPE (models/adapters.py:1125-1193), one routed
SwiGLU expert with the fp16 round trips of engine/scheduler.py:227-297, and
the int8 LM head (engine/scheduler.py:299-309).
"""
from __future__ import annotations

import numpy as np

CFG = dict(num_layers=2, hidden=512, hq=4, hkv=2, head_dim=128, inter=256, vocab=512, rms_eps=1e-5,
           rope_theta=10000.0)
# the reference scheduler benchmark's prompts use token ids up to 8192
BENCH_CFG = dict(CFG, vocab=8448)


def make_weights(seed: int = 1234, cfg=CFG):
    rng = np.random.default_rng(seed)
    H, hq, hkv, D = cfg["hidden"], cfg["hq"], cfg["hkv"], cfg["head_dim"]
    kvd = hkv * D
    f16 = lambda a: a.astype(np.float16)  # noqa: E731
    w = {"emb": f16(rng.standard_normal((cfg["vocab"], H)) * 0.5)}
    for l in range(cfg["num_layers"]):
        p = f"model.layers.{l}"
        w[f"{p}.input_layernorm.weight"] = f16(1.0 + 0.1 * rng.standard_normal(H))
        w[f"{p}.post_attention_layernorm.weight"] = f16(1.0 + 0.1 * rng.standard_normal(H))
        w[f"{p}.self_attn.q_proj.weight"] = f16(rng.standard_normal((H, H)) * (1.5 / np.sqrt(H)))
        w[f"{p}.self_attn.k_proj.weight"] = f16(rng.standard_normal((kvd, H)) * (1.5 / np.sqrt(H)))
        w[f"{p}.self_attn.v_proj.weight"] = f16(rng.standard_normal((kvd, H)) * (1.0 / np.sqrt(H)))
        w[f"{p}.self_attn.o_proj.weight"] = f16(rng.standard_normal((H, H)) * (1.0 / np.sqrt(H)))
        w[f"{p}.self_attn.q_norm.weight"] = f16(1.0 + 0.1 * rng.standard_normal(H))
        w[f"{p}.self_attn.k_norm.weight"] = f16(1.0 + 0.1 * rng.standard_normal(kvd))
        w[f"{p}.mlp.gate.weight"] = f16(rng.standard_normal((1, H)) * 0.02)
        w[f"{p}.expert.gate"] = f16(rng.standard_normal((cfg["inter"], H)) * (1.0 / np.sqrt(H)))
        w[f"{p}.expert.up"] = f16(rng.standard_normal((cfg["inter"], H)) * (1.0 / np.sqrt(H)))
        w[f"{p}.expert.down"] = f16(rng.standard_normal((H, cfg["inter"])) * (1.0 / np.sqrt(cfg["inter"])))
    w["model.norm.weight"] = f16(1.0 + 0.1 * rng.standard_normal(H))
    lm = rng.standard_normal((cfg["vocab"], H))
    s = np.maximum(np.max(np.abs(lm), axis=1, keepdims=True) / 127.0, 1e-7).astype(np.float16)
    w["lm_w_int8"] = np.clip(np.rint(lm / s.astype(np.float64)), -127, 127).astype(np.int8)
    w["lm_s_fp16"] = s
    return w


def prompts():
    """Four requests sharing a 33-token prefix (two full 16-token blocks), one
    short request with no cacheable block, and one longer prompt."""
    rng = np.random.default_rng(7)
    prefix = [int(x) for x in rng.integers(1, 500, size=33)]
    out = [prefix + [100 + i, 200 + i, 300 + i][: i + 1] for i in range(4)]
    out.append([5, 6, 7, 8, 9])
    out.append(prefix + [int(x) for x in rng.integers(1, 500, size=20)])
    return out


class TorchStubModel:
    """`PagedDecoderModel` over torch tensors on one GPU."""

    def __init__(self, w, device, cfg=CFG):
        import torch

        self.t = torch
        self.cfg = cfg
        self.num_layers = cfg["num_layers"]
        self.dev = device
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
        self.emb = T(w["emb"])
        self.layers = []
        for l in range(self.num_layers):
            p = f"model.layers.{l}"
            self.layers.append({k: T(w[f"{p}.{k}"]).float() for k in (
                "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                "self_attn.q_norm.weight", "self_attn.k_norm.weight", "expert.gate", "expert.up", "expert.down")})
        self.final_norm = T(w["model.norm.weight"]).float()
        self.lm_w = T(w["lm_w_int8"]).float()
        self.lm_s = T(w["lm_s_fp16"]).float()[:, 0]
        D = cfg["head_dim"]
        self.inv_freq = 1.0 / (cfg["rope_theta"] ** (torch.arange(0, D, 2, dtype=torch.float32, device=device) / D))

    def _rms(self, x, w):
        var = (x * x).mean(dim=-1, keepdim=True)
        return x * (1.0 / self.t.sqrt(var + self.cfg["rms_eps"])) * w

    def _rope(self, x, positions):
        # x [T, H, D]; rotate-half with angles = position * inv_freq
        ang = positions.to(self.t.float32)[:, None] * self.inv_freq[None, :]
        cos, sin = self.t.cos(ang)[:, None, :], self.t.sin(ang)[:, None, :]
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        return self.t.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    def embed(self, token_ids):
        return self.emb[token_ids].float()

    def attn_in(self, layer, h, positions):
        L = self.layers[layer]
        c = self.cfg
        x = self._rms(h, L["input_layernorm.weight"])
        q = x @ L["self_attn.q_proj.weight"].T
        k = x @ L["self_attn.k_proj.weight"].T
        v = x @ L["self_attn.v_proj.weight"].T
        q = self._rms(q, L["self_attn.q_norm.weight"])
        k = self._rms(k, L["self_attn.k_norm.weight"])
        T = h.shape[0]
        q = self._rope(q.view(T, c["hq"], c["head_dim"]), positions)
        k = self._rope(k.view(T, c["hkv"], c["head_dim"]), positions)
        v = v.view(T, c["hkv"], c["head_dim"])
        # the reference caches K/V as fp16 and attends with fp32 queries
        return q.contiguous(), k.to(self.t.float16).contiguous(), v.to(self.t.float16).contiguous()

    def attn_out(self, layer, h, attn):
        return h + attn.reshape(h.shape[0], -1).float() @ self.layers[layer]["self_attn.o_proj.weight"].T

    def mlp(self, layer, h):
        L = self.layers[layer]
        x = self._rms(h, L["post_attention_layernorm.weight"]).to(self.t.float16).float()
        g = x @ L["expert.gate"].T
        u = x @ L["expert.up"].T
        act = (g / (1.0 + self.t.exp(-g))) * u
        out = (act @ L["expert.down"].T) * 1.0  # one expert, router score 1.0
        return h + out.to(self.t.float16).float()

    def logits(self, h_last):
        x = self._rms(h_last, self.final_norm)
        return (x @ self.lm_w.T) * self.lm_s[None, :]


class StubEngine:
    """The reference engine's scheduler-facing surface (engine/scheduler.py:
    119-309) over the same seeded weights, for driving synapcore_b200's
    ContinuousBatchScheduler(engine, max_batch_size) the way the reference
    scheduler is driven in tests/golden/make_golden.py. Router: the reference
    adapter's softmax top-k (models/adapters.py:244-260) over one expert;
    attention parameters as ModularAttentionEngine derives them for this
    OLMoE-style config (models/adapters.py:1105-1127)."""

    def __init__(self, w, seed_root_hex: str, cfg=CFG):
        import types

        self.config = {"model_type": "olmoe", "num_hidden_layers": cfg["num_layers"], "hidden_size": cfg["hidden"],
                       "num_attention_heads": cfg["hq"], "num_key_value_heads": cfg["hkv"],
                       "vocab_size": cfg["vocab"], "rms_norm_eps": cfg["rms_eps"], "rope_theta": cfg["rope_theta"],
                       "eos_token_id": 50279}
        self.num_layers = cfg["num_layers"]
        self.hidden_size = cfg["hidden"]
        self.rms_eps = cfg["rms_eps"]
        self.top_k = 1
        self.enable_merkle_kv = True
        self.active_merkle_root = seed_root_hex
        self.emb_np_view = w["emb"]
        self.lm_head_w_int8_view = w["lm_w_int8"]
        self.lm_head_s_fp16_view = w["lm_s_fp16"]
        self.core_np_views = {k: v for k, v in w.items() if k.startswith("model.")}
        self._w = w
        d = cfg["head_dim"]
        self.attention_engine = types.SimpleNamespace(
            num_heads=cfg["hq"], num_kv_heads=cfg["hkv"], head_dim=d, rms_eps=cfg["rms_eps"],
            rope_scaling_factor=1.0, has_qk_norm=True, scale=float(d) ** -0.5,
            rope_inv_freq=1.0 / (cfg["rope_theta"] ** (np.arange(0, d, 2, dtype=np.float32) / float(d))))
        self.adapter = types.SimpleNamespace(route_tokens_numpy=self._route)
        self.live_routing_buffer = types.SimpleNamespace(record_numpy_layer=lambda l, idx: None)
        self.closed = False

    def _route(self, x_flat_f32, router_w_fp16):
        logits = x_flat_f32 @ router_w_fp16.astype(np.float32).T
        p = np.exp(logits - np.max(logits, axis=-1, keepdims=True))
        p = p / np.sum(p, axis=-1, keepdims=True)
        idx = np.argpartition(-p, kth=self.top_k - 1, axis=-1)[:, :self.top_k].astype(np.int32)
        return idx, np.take_along_axis(p, idx, axis=-1)

    def load_or_get_expert_entry(self, layer, e, is_prefetch=False):
        import types

        p = f"model.layers.{layer}"
        return types.SimpleNamespace(gate_w=self._w[f"{p}.expert.gate"], up_w=self._w[f"{p}.expert.up"],
                                     down_w=self._w[f"{p}.expert.down"])

    def close(self):
        self.closed = True
