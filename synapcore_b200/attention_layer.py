"""A whole attention layer over the paged cache: the device form of
ModularAttentionEngine.forward_numpy (models/adapters.py:1148-1231).

The reference runs, per request and layer: q/k/v = x @ W^T with fp16
weights (:1167-1169), optional QK-norm (:1171-1185), RoPE from the
request's position (:1191-1192), the fp16 KV concat (:1194-1207), causal
SDPA in fp32 (:1209-1229) and o_proj (:1231). Here a decode call covers
every row of a batch and a prefill call one prompt, in three steps:

- `sckv_qkv_append`: projections, per-head QK-norm, RoPE and the K/V page
  append fused in one tcgen05 kernel (whole-width norms take the unfused
  route inside `KVPool.qkv_append`); q comes back rotated, in fp32;
- `sckv_prefill_attn` (prompts) or `sckv_decode_attn` (one token per
  sequence) over the sequences' pages, fp32 output;
- `sckv_o_proj`: the output projection on the tensor cores, the fp32
  attention output entering as a 16-bit hi + lo pair so the products keep
  fp32 accuracy.

Every pool type works: fp16 / bf16 rows are stored by the fused epilogue,
int8 rows quantised there as the arena quantises its fp16 pages, and FP8
rows (whose page scale spans 16 tokens) staged in fp16 and stored by the
FP8 append launch that follows. Whole-width QK-norm weights (OLMoE style)
take the unfused route, which serves 16-bit and int8 pools. Page bookkeeping follows
`PagedKVCache`: pages for a prompt are reserved
when layer 0 runs and the sequence's length advances after the last layer;
a decode step reserves its token's pages on the device at layer 0.
"""
from __future__ import annotations

from typing import Hashable, Optional, Sequence

import torch

from .paged_cache import PagedKVCache
from .pool import rope_inv_freq, to_device


class PagedAttentionLayer:
    def __init__(self, cache: PagedKVCache, num_q_heads: int, rope_theta: float = 10000.0,
                 rope_scaling: float = 1.0, rms_eps: float = 1e-6, scale: Optional[float] = None):
        if num_q_heads % cache.num_kv_heads != 0:
            raise ValueError("num_q_heads must be a multiple of the cache's kv heads "
                             "(models/adapters.py:1107-1111)")
        self.cache = cache
        self.pool = cache.pool
        self.num_q_heads = int(num_q_heads)
        self.rope_scaling = float(rope_scaling)
        self.rms_eps = float(rms_eps)
        self.scale = float(cache.head_dim) ** -0.5 if scale is None else float(scale)  # :1121
        self.inv_freq = rope_inv_freq(rope_theta, cache.head_dim, cache.device)

    def prefill(self, layer: int, seq_id: Hashable, x: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor,
                w_v: torch.Tensor, w_o: torch.Tensor, q_norm_w: Optional[torch.Tensor] = None,
                k_norm_w: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """x [T, hidden] (the normed layer input; fp32 as in the reference,
        or the weights' 16-bit type) of T new tokens of one sequence at
        positions length..length+T-1 -> the layer output [T, hidden_out]."""
        c = self.cache
        r = c.row_of[seq_id]
        T = x.shape[0]
        start = c.lengths[r]
        if layer == 0:
            c._grow(r, T)
        meta = to_device([0, T, start], torch.int32, c.device)
        q = self.pool.qkv_append(layer, x, w_q, w_k, w_v, meta[:2], meta[2:], c.block_table[r:r + 1],
                                 self.inv_freq, self.rope_scaling, q_norm_w, k_norm_w, self.rms_eps,
                                 q_out_dtype=torch.float32, max_blocks=c.max_blocks)
        attn = c.prefill_attention(layer, seq_id, q, start, scale=self.scale, out_dtype=torch.float32)
        out = self.pool.o_proj(attn, w_o, out_dtype=out_dtype)
        if layer == c.num_layers - 1:
            c.lengths[r] += T
            c.ctx_lens[r] = c.lengths[r]
        return out

    def prefill_batch(self, layer: int, seq_ids: Sequence[Hashable], x: torch.Tensor, cu_tokens: Sequence[int],
                      w_q: torch.Tensor, w_k: torch.Tensor, w_v: torch.Tensor, w_o: torch.Tensor,
                      q_norm_w: Optional[torch.Tensor] = None, k_norm_w: Optional[torch.Tensor] = None,
                      out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Prompts of several sequences in one set of launches (the
        scheduler's admitted prompts of a step): sequence i's new tokens are
        rows cu_tokens[i] .. cu_tokens[i+1]-1 of x [total, hidden] (host
        offsets), at positions length..length+T_i-1. The sequences must sit on
        consecutive cache rows (e.g. added one after another). Returns the
        layer output [total, hidden_out]."""
        c = self.cache
        seq_ids = list(seq_ids)
        n = len(seq_ids)
        cu = [int(v) for v in cu_tokens]
        if len(cu) != n + 1 or cu[0] != 0 or any(b < a for a, b in zip(cu, cu[1:])):
            raise ValueError("cu_tokens must be n+1 non-decreasing offsets from 0")
        if x.shape[0] < cu[-1]:
            raise ValueError("x has fewer rows than cu_tokens[-1]")
        r0 = c._consecutive_rows(seq_ids)
        T = [cu[i + 1] - cu[i] for i in range(n)]
        starts = [c.lengths[r0 + i] for i in range(n)]
        if layer == 0:
            c._grow_rows(r0, T)
        meta = to_device(cu + starts, torch.int32, c.device)
        cu_d, st_d = meta[:n + 1], meta[n + 1:]
        bt = c.block_table[r0:r0 + n]
        q = self.pool.qkv_append(layer, x[:cu[-1]], w_q, w_k, w_v, cu_d, st_d, bt, self.inv_freq, self.rope_scaling,
                                 q_norm_w, k_norm_w, self.rms_eps, q_out_dtype=torch.float32,
                                 max_blocks=c.max_blocks)
        attn = c.prefill_attention_batch(layer, seq_ids, q, cu_d, st_d, scale=self.scale, out_dtype=torch.float32)
        out = self.pool.o_proj(attn, w_o, out_dtype=out_dtype)
        if layer == c.num_layers - 1:
            for i in range(n):
                c.lengths[r0 + i] += T[i]
            c.ctx_lens[r0:r0 + n].copy_(to_device(c.lengths[r0:r0 + n], torch.int32, c.device))
        return out

    def decode(self, layer: int, x: torch.Tensor, n_rows: int, w_q: torch.Tensor, w_k: torch.Tensor,
               w_v: torch.Tensor, w_o: torch.Tensor, q_norm_w: Optional[torch.Tensor] = None,
               k_norm_w: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """One new token for each of rows 0..n_rows-1: x [n_rows, hidden] ->
        the layer output [n_rows, hidden_out]. Layer 0 reserves the tokens'
        pages (on the device) and advances the lengths."""
        c = self.cache
        if layer == 0:
            c.decode_reserve(n_rows)
        start = c.ctx_lens[:n_rows] - 1
        q = self.pool.qkv_append(layer, x, w_q, w_k, w_v, c._arange[:n_rows + 1], start, c.block_table[:n_rows],
                                 self.inv_freq, self.rope_scaling, q_norm_w, k_norm_w, self.rms_eps,
                                 q_out_dtype=torch.float32, max_blocks=c.max_blocks)
        attn = c.decode_attention(layer, q, n_rows, scale=self.scale, out_dtype=torch.float32)
        return self.pool.o_proj(attn, w_o, out_dtype=out_dtype)
