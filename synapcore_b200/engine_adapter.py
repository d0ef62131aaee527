"""The reference engine's model surface as a `PagedDecoderModel`.

`ContinuousBatchScheduler(engine, max_batch_size)` in the reference
(engine/scheduler.py:94-99) drives a NativeMerkleMoEEngine through a small
surface (engine/scheduler.py:119-309): `config`, `num_layers`,
`hidden_size`, `rms_eps`, `top_k`, `emb_np_view`, `core_np_views` (norm,
projection, QK-norm and router weights), `attention_engine`
(ModularAttentionEngine: heads, head_dim, RoPE, QK-norm eps),
`adapter.route_tokens_numpy`, `load_or_get_expert_entry`,
`lm_head_w_int8_view` / `lm_head_s_fp16_view`, plus `enable_merkle_kv` and
`active_merkle_root` for the prefix cache. `EngineModel` reads exactly that
surface and computes everything around attention on the GPU, so the paged
KV cache and its kernels take the place of the per-request NumPy arrays
while the engine object stays the caller's.

Arithmetic follows the reference engine: RMSNorm as `_rmsnorm_numpy`
(native/native_engine.py:2927-2930), projections x @ W^T with the fp16
weights widened, QK-norm over the whole projection or per head as the norm
weight's length says, rotate-half RoPE at position / rope_scaling_factor
(models/adapters.py:1129-1193), K/V rounded to fp16 for the cache
(:1197-1198), o_proj (:1231); the post-attention norm rounded to fp16, one
router call per token (engine/scheduler.py:254-262), top-k SwiGLU experts
summed in router order, the expert sum rounded to fp16 (:281-297); the final
norm and the int8 LM head (:299-309). `compute_dtype` (default float64) is
the type of those products: float64 keeps every token's result independent
of how many tokens share a launch, so a batched run reproduces an isolated
one the way the reference's own parity check expects.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np
import torch


def _attention_spec(engine) -> Dict[str, float]:
    """Heads, head_dim, RoPE and QK-norm parameters of the engine's attention."""
    ae = getattr(engine, "attention_engine", None)
    cfg = dict(getattr(engine, "config", {}) or {})
    if ae is not None:
        return {
            "num_heads": int(ae.num_heads), "num_kv_heads": int(ae.num_kv_heads), "head_dim": int(ae.head_dim),
            "rms_eps": float(ae.rms_eps), "rope_scaling": float(ae.rope_scaling_factor),
            "has_qk_norm": bool(ae.has_qk_norm), "scale": float(ae.scale),
            "inv_freq": np.asarray(ae.rope_inv_freq, np.float32),
        }
    hq = int(cfg["num_attention_heads"])
    hkv = int(cfg.get("num_key_value_heads", hq))
    d = int(cfg.get("head_dim", int(cfg["hidden_size"]) // hq))
    theta = float(cfg.get("rope_theta", 10000.0))
    return {
        "num_heads": hq, "num_kv_heads": hkv, "head_dim": d, "rms_eps": float(cfg.get("rms_norm_eps", 1e-5)),
        "rope_scaling": 1.0, "has_qk_norm": True, "scale": float(d) ** -0.5,
        "inv_freq": (1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float32) / float(d)))).astype(np.float32),
    }


class EngineModel:
    """`PagedDecoderModel` over a reference-style engine object (see module doc)."""

    def __init__(self, engine, device: torch.device, compute_dtype: torch.dtype = torch.float64):
        self.engine = engine
        self.device = torch.device(device)
        self.cd = compute_dtype
        self.num_layers = int(engine.num_layers)
        self.hidden = int(engine.hidden_size)
        self.rms_eps = float(getattr(engine, "rms_eps", 1e-5))
        self.top_k = int(getattr(engine, "top_k", 1))
        spec = _attention_spec(engine)
        self.num_heads, self.num_kv_heads, self.head_dim = spec["num_heads"], spec["num_kv_heads"], spec["head_dim"]
        self.attn_eps = spec["rms_eps"]
        self.rope_scaling = spec["rope_scaling"]
        self.has_qk_norm = spec["has_qk_norm"]
        self.attn_scale = spec["scale"]
        self.inv_freq = torch.from_numpy(spec["inv_freq"]).to(self.device)
        self._w: Dict[str, torch.Tensor] = {}
        self._experts: Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
        self._lm = None
        # the reference's expert-sharing counters (engine/scheduler.py:246-270)
        self.unique_expert_dispatches = 0
        self.naive_expert_dispatches = 0

    # ----------------------------------------------------------- weights
    def _weight(self, name: str):
        w = self._w.get(name)
        if w is None:
            src = self.engine.core_np_views.get(name)
            if src is None:
                return None
            w = torch.from_numpy(np.ascontiguousarray(src)).to(self.device).to(self.cd)
            self._w[name] = w
        return w

    def _expert(self, layer: int, e: int):
        key = (layer, e)
        t = self._experts.get(key)
        if t is None:
            ent = self.engine.load_or_get_expert_entry(layer, e, is_prefetch=False)
            t = tuple(torch.from_numpy(np.ascontiguousarray(a)).to(self.device).to(self.cd)
                      for a in (ent.gate_w, ent.up_w, ent.down_w))
            self._experts[key] = t
        return t

    def _rms(self, x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        var = (x * x).mean(dim=-1, keepdim=True)
        return x * (1.0 / torch.sqrt(var + eps)) * w

    def _rope(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        # x [T, H, D]; angles in fp32 as the reference computes them
        pos = positions.to(torch.float32)[:, None] / self.rope_scaling
        ang = pos * self.inv_freq[None, :]
        cos = torch.cos(ang).to(self.cd)[:, None, :]
        sin = torch.sin(ang).to(self.cd)[:, None, :]
        half = self.head_dim // 2
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    # ------------------------------------------------- PagedDecoderModel
    def embed(self, token_ids: torch.Tensor) -> torch.Tensor:
        ids = token_ids.cpu().numpy()
        rows = np.asarray(self.engine.emb_np_view[ids], np.float32)
        return torch.from_numpy(rows).to(self.device).to(self.cd)

    def attn_in(self, layer: int, h: torch.Tensor, positions: torch.Tensor):
        p = f"model.layers.{layer}"
        ap = f"{p}.self_attn"
        x = self._rms(h, self._weight(f"{p}.input_layernorm.weight"), self.rms_eps)
        q = x @ self._weight(f"{ap}.q_proj.weight").T
        k = x @ self._weight(f"{ap}.k_proj.weight").T
        v = x @ self._weight(f"{ap}.v_proj.weight").T
        T = h.shape[0]
        hq, hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        qn, kn = self._weight(f"{ap}.q_norm.weight"), self._weight(f"{ap}.k_norm.weight")
        if self.has_qk_norm and qn is not None and kn is not None:
            if qn.shape[-1] == q.shape[-1]:
                q = self._rms(q, qn, self.attn_eps)
            else:
                q = self._rms(q.view(T, hq, d), qn, self.attn_eps).reshape(T, hq * d)
            if kn.shape[-1] == k.shape[-1]:
                k = self._rms(k, kn, self.attn_eps)
            else:
                k = self._rms(k.view(T, hkv, d), kn, self.attn_eps).reshape(T, hkv * d)
        q = self._rope(q.view(T, hq, d), positions)
        k = self._rope(k.view(T, hkv, d), positions)
        v = v.view(T, hkv, d)
        return (q.to(torch.float32).contiguous(), k.to(torch.float16).contiguous(),
                v.to(torch.float16).contiguous())

    def attn_out(self, layer: int, h: torch.Tensor, attn: torch.Tensor) -> torch.Tensor:
        w_o = self._weight(f"model.layers.{layer}.self_attn.o_proj.weight")
        return h + attn.reshape(h.shape[0], -1).to(self.cd) @ w_o.T

    def mlp(self, layer: int, h: torch.Tensor) -> torch.Tensor:
        p = f"model.layers.{layer}"
        x = self._rms(h, self._weight(f"{p}.post_attention_layernorm.weight"), self.rms_eps)
        x = x.to(torch.float16).to(self.cd)
        # routing on the host, one call per token as the reference does
        x_np = x.to(torch.float32).cpu().numpy()
        router_w = self.engine.core_np_views[f"{p}.mlp.gate.weight"]
        n_tok = x_np.shape[0]
        idx = np.empty((n_tok, self.top_k), np.int64)
        sc = np.empty((n_tok, self.top_k), np.float32)
        for t in range(n_tok):
            ti, ts = self.engine.adapter.route_tokens_numpy(x_np[t:t + 1], router_w)
            idx[t], sc[t] = ti[0], ts[0]
        rec = getattr(getattr(self.engine, "live_routing_buffer", None), "record_numpy_layer", None)
        if rec is not None:
            rec(layer, idx)
        experts = sorted(set(int(e) for e in idx.reshape(-1)))
        self.naive_expert_dispatches += n_tok * self.top_k
        self.unique_expert_dispatches += len(experts)
        out = torch.zeros_like(x)
        idx_d = torch.from_numpy(idx).to(self.device)
        sc_d = torch.from_numpy(sc).to(self.device).to(self.cd)
        for k_i in range(self.top_k):
            contrib = torch.zeros_like(x)
            for e in experts:
                rows = (idx_d[:, k_i] == e).nonzero().flatten()
                if rows.numel() == 0:
                    continue
                g_w, u_w, d_w = self._expert(layer, e)
                xr = x[rows]
                g = xr @ g_w.T
                u = xr @ u_w.T
                act = (g / (1.0 + torch.exp(-g))) * u
                contrib[rows] = act @ d_w.T
            out = out + sc_d[:, k_i:k_i + 1] * contrib
        return h + out.to(torch.float16).to(self.cd)

    def logits(self, h_last: torch.Tensor) -> torch.Tensor:
        if self._lm is None:
            w = torch.from_numpy(np.ascontiguousarray(self.engine.lm_head_w_int8_view)).to(self.device).to(self.cd)
            s = np.asarray(self.engine.lm_head_s_fp16_view)
            s = torch.from_numpy(np.ascontiguousarray(s.reshape(s.shape[0], -1)[:, 0])).to(self.device).to(self.cd)
            self._lm = (w, s)
        w, s = self._lm
        x = self._rms(h_last, self._weight("model.norm.weight"), self.rms_eps)
        return ((x @ w.T) * s[None, :]).to(torch.float32)
