"""CPU oracle for the paged KV-cache path — TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the reference algorithms the B200 library
replaces. Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import it, and only as the checker (or the timed CPU
baseline); the product path in ``synapcore_b200`` never calls it.

Pinning: every function here is checked against fixtures produced by the
reference itself (tests/golden/make_golden.py imports the reference's own
modules and records their outputs) — see tests/test_oracle_golden.py.

Reference citations are ``path:line`` inside the synapcore project.
"""
from __future__ import annotations

import collections
import hashlib
import struct
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import numpy as np

PAGE_TOKENS = 16  # PagedKVArena.PAGE_TOKENS, native/native_engine.py:230
BLOCK_SIZE = 16   # NativeKVPrefixCache.BLOCK_SIZE, native/native_engine.py:2130


# --------------------------------------------------------------------------
# INT8 KV quantisation — native/native_engine.py:207-221
# --------------------------------------------------------------------------
def quantize_kv_int8(x_fp16: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Symmetric int8 along the last axis; fp32 scale max(max|x|/127, 1e-7),
    round-half-even, clip to +-127; scale stored as fp16 (:207-216)."""
    x = x_fp16.astype(np.float32)
    m = np.max(np.abs(x), axis=-1, keepdims=True)
    s = np.maximum(m / np.float32(127.0), np.float32(1e-7)).astype(np.float32)
    q = np.clip(np.rint(x / s), -127.0, 127.0).astype(np.int8)
    return q, s.astype(np.float16)


def dequantize_kv_int8(q: np.ndarray, s_fp16: np.ndarray) -> np.ndarray:
    """fp16(f32(q) * f32(scale)) (:219-221)."""
    return (q.astype(np.float32) * s_fp16.astype(np.float32)).astype(np.float16)


# --------------------------------------------------------------------------
# Prefix-chain hash — native/native_engine.py:778-782
# --------------------------------------------------------------------------
def chain_prefix_hash(prev_hash_hex: str, token_block: Sequence[int]) -> str:
    h = hashlib.sha256()
    h.update(bytes.fromhex(prev_hash_hex))
    h.update(struct.pack(f"<{len(token_block)}I", *[int(t) for t in token_block]))
    return h.digest().hex()


# --------------------------------------------------------------------------
# FP8 e4m3 — decode LUT of models/adapters.py:692-722; encode = IEEE-style
# round-to-nearest-even onto the e4m3fn grid with saturation at +-448.
# --------------------------------------------------------------------------
def _fp8_lut() -> np.ndarray:
    lut = np.zeros(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if (b & 0x80) else 1.0
        e = (b >> 3) & 0x0F
        m = b & 0x07
        if e == 0:
            v = sign * (2.0 ** -6) * (m / 8.0)
        elif e == 15 and m == 7:
            v = 0.0  # NaN byte mapped to 0 as in the reference LUT
        else:
            v = sign * (2.0 ** (e - 7)) * (1.0 + m / 8.0)
        lut[b] = np.float32(v)
    return lut


FP8_LUT = _fp8_lut()
FP8_MAX = np.float32(448.0)


def fp8_decode(codes: np.ndarray) -> np.ndarray:
    return FP8_LUT[np.asarray(codes, dtype=np.uint8)]


def fp8_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn byte, round half to even, saturating to +-448."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    out = np.zeros(a.shape, dtype=np.uint8)
    sub = a < 2.0 ** -6
    # subnormals (and zero): units of 2^-9, code == unit count (8 -> min normal)
    q_sub = np.rint(a[sub] / 2.0 ** -9).astype(np.int64)
    out[sub] = q_sub.astype(np.uint8)
    nrm = ~sub
    if np.any(nrm):
        an = a[nrm]
        mant, ex = np.frexp(an)          # an = mant * 2^ex, mant in [0.5, 1)
        e = ex - 1                        # an = (2*mant) * 2^e, 2*mant in [1, 2)
        q = np.rint((2.0 * mant - 1.0) * 8.0).astype(np.int64)
        carry = q == 8
        e = e + carry
        q = np.where(carry, 0, q)
        code = ((e + 7) << 3) | q
        out[nrm] = np.minimum(code, 0x7E).astype(np.uint8)
    return out | sign


def fp8_page_scale(x: np.ndarray) -> np.float32:
    """Per-page-head fp32 scale max|x| / 448 (0 for an all-zero page)."""
    return np.float32(np.max(np.abs(np.asarray(x, dtype=np.float32)))) / FP8_MAX


# --------------------------------------------------------------------------
# Reference decode SDPA — models/adapters.py:1209-1229 (seq_len == 1, no mask)
# --------------------------------------------------------------------------
def sdpa_decode(q_f32: np.ndarray, k_f16: np.ndarray, v_f16: np.ndarray, scale: Optional[float] = None) -> np.ndarray:
    """q [Hq, D] fp32; k, v [Hkv, T, D] (fp16, or fp32 already dequantised).
    K/V upcast to fp32, GQA repeat along heads (:1211-1215), scores
    (q @ k^T) * D^-0.5 (:1121, :1217), max-subtracted softmax (:1226-1228),
    P @ V (:1229). Returns [Hq, D] fp32."""
    hq, d = q_f32.shape
    hkv = k_f16.shape[0]
    g = hq // hkv
    scale = float(d) ** -0.5 if scale is None else scale
    k = k_f16.astype(np.float32)
    v = v_f16.astype(np.float32)
    if g > 1:
        k = np.repeat(k, g, axis=0)
        v = np.repeat(v, g, axis=0)
    q = q_f32.astype(np.float32)[:, None, :]                 # [Hq, 1, D]
    scores = (q @ k.transpose(0, 2, 1)) * np.float32(scale)  # [Hq, 1, T]
    smax = np.max(scores, axis=-1, keepdims=True)
    p = np.exp(scores - smax)
    p = p / np.sum(p, axis=-1, keepdims=True)
    return (p @ v)[:, 0, :]


def rope_inv_freq(theta: float, head_dim: int) -> np.ndarray:
    """models/adapters.py:1123-1127 (float32)."""
    return 1.0 / (float(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / float(head_dim)))


def rmsnorm_f32(x_f32: np.ndarray, weight_fp16: np.ndarray, eps: float) -> np.ndarray:
    """models/adapters.py:1129-1132: x / sqrt(mean(x^2) + eps) * w over the last axis."""
    var = np.mean(x_f32 * x_f32, axis=-1, keepdims=True)
    normed = x_f32 * (1.0 / np.sqrt(var + eps))
    return normed * weight_fp16.astype(np.float32)


def apply_rope_f32(x_bhld: np.ndarray, inv_freq: np.ndarray, pos_offset: int, scaling: float) -> np.ndarray:
    """models/adapters.py:1134-1146: rotate the two halves of the head dim by
    angle (pos / scaling) * inv_freq[i]."""
    seq_len = x_bhld.shape[2]
    positions = np.arange(pos_offset, pos_offset + seq_len, dtype=np.float32)[:, None] / scaling
    angles = positions * inv_freq[None, :]
    cos = np.cos(angles)[None, None, :, :]
    sin = np.sin(angles)[None, None, :, :]
    half = x_bhld.shape[-1] // 2
    x1, x2 = x_bhld[..., :half], x_bhld[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


def qk_norm_rope(q: np.ndarray, k: np.ndarray, q_w: Optional[np.ndarray], k_w: Optional[np.ndarray], eps: float,
                 inv_freq: np.ndarray, scaling: float, pos_offset: int) -> Tuple[np.ndarray, np.ndarray]:
    """The attention-input steps of forward_numpy (models/adapters.py:1171-1195)
    for one sequence: q [T, Hq, D], k [T, Hkv, D] float32 straight from the
    projections; optional QK-norm (weights of D = per head, else over the
    whole projection), RoPE from position pos_offset. Returns (q rotated,
    float32 [T, Hq, D]; k rotated as stored in the cache, float16 [T, Hkv, D])."""
    T, hq, d = q.shape
    hkv = k.shape[1]
    qf = q.reshape(1, T, hq * d).astype(np.float32)
    kf = k.reshape(1, T, hkv * d).astype(np.float32)
    if q_w is not None and k_w is not None:
        if q_w.shape[-1] == hq * d:
            qf = rmsnorm_f32(qf, q_w, eps)
        else:
            qf = rmsnorm_f32(qf.reshape(1, T, hq, d), q_w, eps).reshape(1, T, hq * d)
        if k_w.shape[-1] == hkv * d:
            kf = rmsnorm_f32(kf, k_w, eps)
        else:
            kf = rmsnorm_f32(kf.reshape(1, T, hkv, d), k_w, eps).reshape(1, T, hkv * d)
    qb = qf.reshape(1, T, hq, d).transpose(0, 2, 1, 3)
    kb = kf.reshape(1, T, hkv, d).transpose(0, 2, 1, 3)
    qr = apply_rope_f32(qb, inv_freq, pos_offset, scaling)
    kr = apply_rope_f32(kb, inv_freq, pos_offset, scaling)
    return qr[0].transpose(1, 0, 2), kr[0].transpose(1, 0, 2).astype(np.float16)


def qkv_project(x_f32: np.ndarray, w_q: np.ndarray, w_k: np.ndarray, w_v: np.ndarray, hq: int, hkv: int
                ) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The projections of forward_numpy (models/adapters.py:1167-1169):
    x [T, hidden] float32 times each fp16 weight [out, hidden] widened to
    float32 and transposed. Returns q [T, Hq, D], k and v [T, Hkv, D] float32."""
    x = x_f32.astype(np.float32)
    q = x @ w_q.astype(np.float32).T
    k = x @ w_k.astype(np.float32).T
    v = x @ w_v.astype(np.float32).T
    T = x.shape[0]
    return q.reshape(T, hq, -1), k.reshape(T, hkv, -1), v.reshape(T, hkv, -1)


def sdpa_prefill(q_f32: np.ndarray, k: np.ndarray, v: np.ndarray, start: int,
                 scale: Optional[float] = None) -> np.ndarray:
    """Causal prompt pass (models/adapters.py:1209-1229 with the -1e9 mask of
    :1218-1224): query t at position start+t sees keys 0..start+t. The -1e9
    mask makes masked probabilities exactly 0 in fp32, so each row is the
    decode SDPA over its visible prefix. q [T, Hq, D]; k, v [Hkv, ctx, D]."""
    return np.stack([sdpa_decode(q_f32[t], k[:, :start + t + 1], v[:, :start + t + 1], scale)
                     for t in range(q_f32.shape[0])])


def o_project(attn_f32: np.ndarray, w_o: np.ndarray) -> np.ndarray:
    """The output projection of forward_numpy (models/adapters.py:1231):
    attn [T, Hq*D] (or [T, Hq, D]) float32 times the fp16 weight
    [hidden, Hq*D] widened to float32 and transposed. Returns [T, hidden]."""
    a = attn_f32.reshape(attn_f32.shape[0], -1).astype(np.float32)
    return a @ w_o.astype(np.float32).T


def attention_layer(x_f32: np.ndarray, w_q: np.ndarray, w_k: np.ndarray, w_v: np.ndarray, w_o: np.ndarray,
                    hq: int, hkv: int, prev_k: Optional[np.ndarray], prev_v: Optional[np.ndarray],
                    q_w: Optional[np.ndarray] = None, k_w: Optional[np.ndarray] = None, eps: float = 1e-6,
                    theta: float = 10000.0, scaling: float = 1.0, scale: Optional[float] = None,
                    int8_cache: bool = False) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """ModularAttentionEngine.forward_numpy (models/adapters.py:1148-1231) for
    one sequence, composed from the steps above: projections (:1167-1169),
    QK-norm + RoPE from position len(prev) (:1171-1192), the fp16 cache
    concat (:1194-1207), causal SDPA (:1209-1229, no mask for one token) and
    o_proj (:1231). x [T, hidden]; prev_k / prev_v [Hkv, P, D] fp16 or None.
    int8_cache: the new K / V rows go through the arena's int8 mode (quantised
    per row as quantize_kv_int8, read back as dequantize_kv_int8,
    native/native_engine.py:207-221) before the attention reads them.
    Returns (out [T, hidden] float32, k_full, v_full [Hkv, P + T, D] fp16)."""
    T = x_f32.shape[0]
    q, k, v = qkv_project(x_f32, w_q, w_k, w_v, hq, hkv)
    d = q.shape[-1]
    start = 0 if prev_k is None else prev_k.shape[1]
    qr, kc = qk_norm_rope(q, k, q_w, k_w, eps, rope_inv_freq(theta, d), scaling, start)
    k_new = kc.transpose(1, 0, 2)
    v_new = v.astype(np.float16).transpose(1, 0, 2)
    if int8_cache:
        k_new = dequantize_kv_int8(*quantize_kv_int8(k_new))
        v_new = dequantize_kv_int8(*quantize_kv_int8(v_new))
    k_full = k_new if prev_k is None else np.concatenate([prev_k, k_new], axis=1)
    v_full = v_new if prev_v is None else np.concatenate([prev_v, v_new], axis=1)
    attn = sdpa_prefill(qr, k_full, v_full, start, scale)
    return o_project(attn, w_o), k_full, v_full


# --------------------------------------------------------------------------
# PagedKVArena restatement — native/native_engine.py:224-432
# --------------------------------------------------------------------------
class ArenaOracle:
    """Host pool + bookkeeping exactly as PagedKVArena (:232-432)."""

    def __init__(self, max_pages: int = 64, num_layers: int = 16, num_kv_heads: int = 16, head_dim: int = 128,
                 quant_mode: str = "fp16"):
        if quant_mode not in ("fp16", "int8"):
            raise ValueError(quant_mode)
        self.max_pages = max(1, int(max_pages))
        self.num_layers, self.num_kv_heads, self.head_dim = int(num_layers), int(num_kv_heads), int(head_dim)
        self.quant_mode = quant_mode
        shape = (self.max_pages, self.num_layers, 1, self.num_kv_heads, PAGE_TOKENS, self.head_dim)
        sshape = shape[:-1] + (1,)
        if quant_mode == "int8":
            self.k_q = np.zeros(shape, np.int8); self.v_q = np.zeros(shape, np.int8)
            self.k_s = np.ones(sshape, np.float16); self.v_s = np.ones(sshape, np.float16)
            self.bytes_per_page = (2 * self.num_layers * self.num_kv_heads * PAGE_TOKENS * self.head_dim
                                   + 2 * self.num_layers * self.num_kv_heads * PAGE_TOKENS * 2)
        else:
            self.k = np.zeros(shape, np.float16); self.v = np.zeros(shape, np.float16)
            self.bytes_per_page = 2 * self.num_layers * self.num_kv_heads * PAGE_TOKENS * self.head_dim * 2
        self.free_pages: Deque[int] = collections.deque(range(self.max_pages))
        self.page_table: Dict[str, int] = {}
        self.reverse_page_table: Dict[int, str] = {}
        self.page_last_used: Dict[str, int] = {}
        self.step_clock = 0
        self.page_hits = self.page_misses = self.page_evictions = 0

    def lookup_page_id(self, h: str) -> Optional[int]:  # :297-305
        self.step_clock += 1
        if h in self.page_table:
            self.page_hits += 1
            self.page_last_used[h] = self.step_clock
            return self.page_table[h]
        self.page_misses += 1
        return None

    def evict_prefix_hash(self, h: str) -> bool:  # :307-316
        pid = self.page_table.pop(h, None)
        if pid is None:
            return False
        self.reverse_page_table.pop(pid, None)
        self.page_last_used.pop(h, None)
        self.free_pages.append(pid)
        self.page_evictions += 1
        return True

    def allocate(self, h: str) -> int:  # _allocate_page_slot_unlocked :318-337
        if h in self.page_table:
            self.step_clock += 1
            self.page_last_used[h] = self.step_clock
            return self.page_table[h]
        if self.free_pages:
            pid = self.free_pages.popleft()
        else:
            victim = min(self.page_table.keys(), key=lambda x: self.page_last_used.get(x, 0))
            pid = self.page_table.pop(victim)
            self.reverse_page_table.pop(pid, None)
            self.page_last_used.pop(victim, None)
            self.page_evictions += 1
        self.step_clock += 1
        self.page_table[h] = pid
        self.reverse_page_table[pid] = h
        self.page_last_used[h] = self.step_clock
        return pid

    def write_page_fp16(self, h: str, k: np.ndarray, v: np.ndarray) -> int:  # :339-359
        pid = self.allocate(h)
        if self.quant_mode == "int8":
            kq, ks = quantize_kv_int8(k); vq, vs = quantize_kv_int8(v)
            self.k_q[pid], self.v_q[pid], self.k_s[pid], self.v_s[pid] = kq, vq, ks, vs
        else:
            self.k[pid], self.v[pid] = k, v
        return pid

    def write_page_quantized(self, h, kq, ks, vq, vs) -> int:  # :361-386
        pid = self.allocate(h)
        if self.quant_mode == "int8":
            self.k_q[pid], self.k_s[pid], self.v_q[pid], self.v_s[pid] = kq, ks, vq, vs
        else:
            self.k[pid] = dequantize_kv_int8(kq, ks)
            self.v[pid] = dequantize_kv_int8(vq, vs)
        return pid

    def read_page_fp16(self, pid: int) -> Tuple[np.ndarray, np.ndarray]:  # :388-401
        if self.quant_mode == "int8":
            return dequantize_kv_int8(self.k_q[pid], self.k_s[pid]), dequantize_kv_int8(self.v_q[pid], self.v_s[pid])
        return self.k[pid], self.v[pid]

    def gather_contiguous_kv_numpy(self, page_ids: List[int]) -> Tuple[np.ndarray, np.ndarray]:  # :403-419
        n = len(page_ids)
        shape = (self.num_layers, 1, self.num_kv_heads, n * PAGE_TOKENS, self.head_dim)
        kc = np.empty(shape, np.float16); vc = np.empty(shape, np.float16)
        for i, pid in enumerate(page_ids):
            k, v = self.read_page_fp16(pid)
            kc[:, :, :, i * PAGE_TOKENS:(i + 1) * PAGE_TOKENS] = k
            vc[:, :, :, i * PAGE_TOKENS:(i + 1) * PAGE_TOKENS] = v
        return kc, vc


# --------------------------------------------------------------------------
# Device-allocator restatement: FIFO ring + LRU clock with pins.
# Same bookkeeping as ArenaOracle.allocate / lookup_page_id /
# evict_prefix_hash, keyed by page id instead of prefix hash.
# --------------------------------------------------------------------------
class AllocatorOracle:
    def __init__(self, max_pages: int):
        self.P = int(max_pages)
        self.ring: Deque[int] = collections.deque(range(self.P))
        self.last_used = np.zeros(self.P, np.int64)
        self.pin = np.zeros(self.P, np.int64)
        self.allocated = np.zeros(self.P, bool)
        self.clock = 0
        self.evictions = 0

    def _victim(self) -> Optional[int]:
        cand = np.nonzero(self.allocated & (self.pin == 0))[0]
        if cand.size == 0:
            return None
        return int(cand[np.argmin(self.last_used[cand])])

    def alloc(self, n: int, pin: bool = False) -> Tuple[List[int], List[int]]:
        """n successive allocations for new keys (native_engine.py:318-337)."""
        # the device call checks capacity up front
        cand = int(np.count_nonzero(self.allocated & (self.pin == 0)))
        if n > len(self.ring) + cand:
            raise MemoryError("pool exhausted")
        ids, victims = [], []
        for _ in range(n):
            if self.ring:
                pid = self.ring.popleft(); vic = -1
                self.allocated[pid] = True
            else:
                pid = self._victim(); vic = pid
                self.evictions += 1
            self.clock += 1
            self.last_used[pid] = self.clock
            self.pin[pid] = 1 if pin else 0
            ids.append(pid); victims.append(vic)
        return ids, victims

    def free(self, ids: Sequence[int]) -> None:
        """evict_prefix_hash (:307-316): ring tail, repeats / free ids skipped."""
        for pid in ids:
            pid = int(pid)
            if pid < 0 or pid >= self.P or not self.allocated[pid]:
                continue
            self.allocated[pid] = False
            self.pin[pid] = 0
            self.last_used[pid] = 0
            self.ring.append(pid)
            self.evictions += 1

    def touch(self, ids: Sequence[int]) -> None:
        """lookup_page_id (:297-305): clock per entry, -1 = miss."""
        for pid in ids:
            self.clock += 1
            pid = int(pid)
            if 0 <= pid < self.P and self.allocated[pid]:
                self.last_used[pid] = self.clock

    def pin_pages(self, ids: Sequence[int], delta: int) -> None:
        for pid in ids:
            self.pin[int(pid)] += delta

    def release(self, ids: Sequence[int], keep_cached: bool = False) -> None:
        """Drop one pin per page; pin 0 -> ring tail (or stay cached)."""
        for pid in ids:
            pid = int(pid)
            if pid < 0 or pid >= self.P or not self.allocated[pid]:
                continue
            self.pin[pid] -= 1
            if self.pin[pid] == 0 and not keep_cached:
                self.allocated[pid] = False
                self.last_used[pid] = 0
                self.ring.append(pid)

    def evict_lru(self, n: int) -> List[int]:
        out = []
        for _ in range(n):
            v = self._victim()
            if v is None:
                break
            self.allocated[v] = False
            self.last_used[v] = 0
            self.ring.append(v)
            self.evictions += 1
            out.append(v)
        return out + [-1] * (n - len(out))

    def evict_to_watermark(self, max_allocated: int) -> int:
        """LRU evictions until at most max_allocated pages are allocated (or
        no unpinned page is left); the serving policy of the device pool
        (no reference counterpart: the arena evicts only when its free list
        is empty, native/native_engine.py:324-331)."""
        over = int(self.allocated.sum()) - int(max_allocated)
        if over <= 0:
            return 0
        return sum(1 for v in self.evict_lru(over) if v >= 0)

    def reserve_decode(self, block_table: np.ndarray, ctx_lens: np.ndarray) -> None:
        need = [b for b in range(len(ctx_lens)) if ctx_lens[b] % PAGE_TOKENS == 0]
        ids, _ = self.alloc(len(need), pin=True)
        for b, pid in zip(need, ids):
            block_table[b, ctx_lens[b] // PAGE_TOKENS] = pid
        ctx_lens += 1


# --------------------------------------------------------------------------
# Block-table paged cache restatement (the device layout, on the host).
# pool[layer][page][kv][head][slot][dim]
# --------------------------------------------------------------------------
class PagedPoolOracle:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_pages: int, dtype: str = "fp16"):
        self.L, self.H, self.D, self.P = num_layers, num_kv_heads, head_dim, max_pages
        self.dtype = dtype
        shape = (num_layers, max_pages, 2, num_kv_heads, PAGE_TOKENS, head_dim)
        if dtype == "fp16":
            self.data = np.zeros(shape, np.float16)
        elif dtype == "bf16":
            self.data = np.zeros(shape, np.uint16)  # raw bf16 bits
        elif dtype == "int8":
            self.data = np.zeros(shape, np.int8)
            self.scales = np.zeros(shape[:-1], np.float16)
        elif dtype == "fp8_e4m3":
            self.data = np.zeros(shape, np.uint8)
            self.scales = np.zeros(shape[:4], np.float32)
        else:
            raise ValueError(dtype)

    # ---- append: scatter token rows through the block table (kernel 1)
    def append(self, layer0: int, k_new: np.ndarray, v_new: np.ndarray, cu: np.ndarray, start_pos: np.ndarray,
               block_table: np.ndarray) -> None:
        """k_new/v_new [n_layers][n_tokens][H][D] float32 values (already the
        source dtype's values). Token t of sequence b sits at start_pos[b] + (t - cu[b])."""
        nl = k_new.shape[0]
        for b in range(len(cu) - 1):
            t0, t1 = int(cu[b]), int(cu[b + 1])
            if t1 == t0:
                continue
            for l in range(nl):
                for kv, src in ((0, k_new), (1, v_new)):
                    if self.dtype == "fp8_e4m3":
                        t = t0
                        while t < t1:
                            pos = int(start_pos[b]) + (t - t0)
                            slot0 = pos % PAGE_TOKENS
                            n_new = min(t1 - t, PAGE_TOKENS - slot0)
                            page = int(block_table[b, pos // PAGE_TOKENS])
                            for h in range(self.H):
                                self._fp8_update(layer0 + l, page, kv, h, slot0, src[l, t:t + n_new, h, :])
                            t += n_new
                    else:
                        for t in range(t0, t1):
                            pos = int(start_pos[b]) + (t - t0)
                            page = int(block_table[b, pos // PAGE_TOKENS])
                            self._write_row(layer0 + l, page, kv, pos % PAGE_TOKENS, src[l, t])

    def _write_row(self, layer, page, kv, slot, rows_hd: np.ndarray) -> None:
        x = np.asarray(rows_hd, np.float32)  # [H, D]
        if self.dtype == "fp16":
            self.data[layer, page, kv, :, slot] = x.astype(np.float16)
        elif self.dtype == "bf16":
            self.data[layer, page, kv, :, slot] = f32_to_bf16_bits(x)
        elif self.dtype == "int8":
            q, s = quantize_kv_int8(x)  # per head row
            self.data[layer, page, kv, :, slot] = q
            self.scales[layer, page, kv, :, slot] = s[:, 0]

    def _fp8_update(self, layer, page, kv, h, slot0, x_new: np.ndarray) -> None:
        """Per-page-head scale growth with re-encode of earlier slots."""
        x_new = np.asarray(x_new, np.float32)
        s_old = np.float32(0.0) if slot0 == 0 else self.scales[layer, page, kv, h]
        m = np.float32(np.max(np.abs(x_new))) if x_new.size else np.float32(0.0)
        s_new = np.maximum(s_old, m / FP8_MAX).astype(np.float32)
        blk = self.data[layer, page, kv, h]
        if s_new > s_old and slot0 > 0:
            old = fp8_decode(blk[:slot0]) * s_old
            blk[:slot0] = fp8_encode((old / s_new).astype(np.float32))
        if s_new > 0:
            blk[slot0:slot0 + x_new.shape[0]] = fp8_encode((x_new / s_new).astype(np.float32))
        else:
            blk[slot0:slot0 + x_new.shape[0]] = 0
        self.scales[layer, page, kv, h] = s_new

    # ---- whole-page write [n][L][H][16][D]
    def write_pages(self, ids: Sequence[int], k_src: np.ndarray, v_src: np.ndarray) -> None:
        for i, page in enumerate(ids):
            for kv, src in ((0, k_src), (1, v_src)):
                for l in range(self.L):
                    if self.dtype == "fp8_e4m3":
                        for h in range(self.H):
                            self._fp8_update(l, page, kv, h, 0, src[i, l, h])
                    else:
                        for slot in range(PAGE_TOKENS):
                            self._write_row(l, page, kv, slot, src[i, l, :, slot, :])

    # ---- values of a page-head as float32 (dequantised)
    def values(self, layer, page, kv) -> np.ndarray:
        raw = self.data[layer, page, kv]
        if self.dtype == "fp16":
            return raw.astype(np.float32)
        if self.dtype == "bf16":
            return bf16_bits_to_f32(raw)
        if self.dtype == "int8":
            return dequantize_kv_int8(raw, self.scales[layer, page, kv][..., None]).astype(np.float32)
        return fp8_decode(raw) * self.scales[layer, page, kv][:, None, None]

    # ---- gather (kernel 2): [n_layers][H][n_tokens][D] float32
    def gather(self, layer0: int, n_layers: int, ids: Sequence[int], n_tokens: int) -> Tuple[np.ndarray, np.ndarray]:
        out = np.zeros((2, n_layers, self.H, n_tokens, self.D), np.float32)
        n_pages = (n_tokens + PAGE_TOKENS - 1) // PAGE_TOKENS
        for kv in range(2):
            for l in range(n_layers):
                for i in range(n_pages):
                    t0 = i * PAGE_TOKENS
                    t1 = min(n_tokens, t0 + PAGE_TOKENS)
                    vals = self.values(layer0 + l, int(ids[i]), kv)
                    out[kv, l, :, t0:t1] = vals[:, : t1 - t0]
        return out[0], out[1]

    def copy_pages(self, src: Sequence[int], dst: Sequence[int]) -> None:
        for s, d in zip(src, dst):
            self.data[:, d] = self.data[:, s]
            if hasattr(self, "scales"):
                self.scales[:, d] = self.scales[:, s]

    # ---- paged decode attention over block tables (kernels 3+4)
    def prefill(self, layer: int, q: np.ndarray, cu_q: Sequence[int], start_pos: Sequence[int],
                block_table: np.ndarray, scale: Optional[float] = None) -> np.ndarray:
        """q [n_tokens][Hq][D] float32 values; sequence b owns rows
        cu_q[b]..cu_q[b+1]-1 at positions start_pos[b]+i -> causal SDPA
        (sdpa_prefill) over the gathered pages, [n_tokens][Hq][D] float32."""
        out = np.zeros(q.shape, np.float32)
        for b in range(len(cu_q) - 1):
            t0, t1, st = int(cu_q[b]), int(cu_q[b + 1]), int(start_pos[b])
            if t1 == t0:
                continue
            ctx = st + t1 - t0
            n_pages = (ctx + PAGE_TOKENS - 1) // PAGE_TOKENS
            k, v = self.gather(layer, 1, block_table[b, :n_pages], ctx)
            out[t0:t1] = sdpa_prefill(q[t0:t1].astype(np.float32), k[0], v[0], st, scale)
        return out

    def decode(self, layer: int, q: np.ndarray, block_table: np.ndarray, ctx_lens: np.ndarray,
               scale: Optional[float] = None) -> np.ndarray:
        """q [B][Hq][D] float32 values -> [B][Hq][D] float32 via sdpa_decode
        on the gathered contiguous K/V of each sequence."""
        B, hq, d = q.shape
        out = np.zeros((B, hq, d), np.float32)
        for b in range(B):
            ctx = int(ctx_lens[b])
            if ctx == 0:
                continue
            n_pages = (ctx + PAGE_TOKENS - 1) // PAGE_TOKENS
            k, v = self.gather(layer, 1, block_table[b, :n_pages], ctx)
            out[b] = sdpa_decode(q[b].astype(np.float32), k[0], v[0], scale)
        return out


# --------------------------------------------------------------------------
# bf16 helpers (round to nearest even, as torch / CUDA do)
# --------------------------------------------------------------------------
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# --------------------------------------------------------------------------
# KV prefix hash table — Python twin native/native_engine.py:1714-1752,
# C++ native/synapcore_native.mm:716-780. Slot struct "<32s32sIId"
# (native_engine.py:1284), 1024 slots, 64 probes.
# --------------------------------------------------------------------------
_KV_SLOT = struct.Struct("<32s32sIId")
KV_TABLE_BYTES = 1024 * 80


class KVTableOracle:
    def __init__(self, table: Optional[bytearray] = None):
        self.table = table if table is not None else bytearray(KV_TABLE_BYTES)
        self.evictions = 0

    def lookup(self, h: bytes) -> bool:
        slot = struct.unpack_from("<I", h, 0)[0] & 1023
        for probe in range(64):
            pos = ((slot + probe) & 1023) * 80
            p_hash, _, occ, _, _ = _KV_SLOT.unpack_from(self.table, pos)
            if occ == 0:
                return False
            if p_hash == h:
                return True
        return False

    def insert(self, h: bytes, parent: bytes, token_end: int, ts: float) -> Optional[str]:
        slot = struct.unpack_from("<I", h, 0)[0] & 1023
        oldest_pos = slot * 80
        oldest_ts = float("inf")
        oldest_hash = b""
        for probe in range(64):
            pos = ((slot + probe) & 1023) * 80
            p_hash, _, occ, _, created = _KV_SLOT.unpack_from(self.table, pos)
            if occ == 0 or p_hash == h:
                _KV_SLOT.pack_into(self.table, pos, h, parent, 1, int(token_end), float(ts))
                return None
            if created < oldest_ts:
                oldest_ts, oldest_pos, oldest_hash = created, pos, bytes(p_hash)
        _KV_SLOT.pack_into(self.table, oldest_pos, h, parent, 1, int(token_end), float(ts))
        self.evictions += 1
        return oldest_hash.hex() if oldest_hash else None


# --------------------------------------------------------------------------
# NativeKVPrefixCache restatement (numpy path) — native/native_engine.py:2125-2435
# --------------------------------------------------------------------------
class PrefixCacheOracle:
    """save_prefix_blocks_numpy (:2202-2246) / match_longest_prefix_numpy
    (:2248-2291) over ArenaOracle, a KVTableOracle and .npz files in kv_dir."""

    def __init__(self, kv_dir, arena: ArenaOracle, table: KVTableOracle, max_disk_blocks: int = 512):
        from pathlib import Path

        self.kv_dir = Path(kv_dir)
        self.kv_dir.mkdir(parents=True, exist_ok=True)
        self.arena, self.table = arena, table
        self.max_disk_blocks = max(1, int(max_disk_blocks))
        self.quant_mode = arena.quant_mode
        self.disk_lru: "collections.OrderedDict[str, object]" = collections.OrderedDict()
        self.blocks_loaded_from_disk = self.blocks_loaded_from_arena = 0
        self.blocks_saved_to_disk = self.disk_blocks_evicted = self.tokens_skipped = 0

    def _evict_disk_block_by_hash(self, h: str) -> None:  # :2173-2187
        self.arena.evict_prefix_hash(h)
        p = self.disk_lru.pop(h, None)
        for cand in (p, self.kv_dir / f"{h[:32]}_mlx.safetensors", self.kv_dir / f"{h[:32]}_mlx_int8.safetensors",
                     self.kv_dir / f"{h[:32]}_np.npz"):
            if cand is not None and cand.exists():
                cand.unlink()
                self.disk_blocks_evicted += 1

    def _enforce_disk_budget(self, h: str, path) -> None:  # :2189-2200
        self.disk_lru[h] = path
        self.disk_lru.move_to_end(h)
        while len(self.disk_lru) > self.max_disk_blocks:
            oh, op = self.disk_lru.popitem(last=False)
            self.arena.evict_prefix_hash(oh)
            if op.exists():
                op.unlink()
                self.disk_blocks_evicted += 1

    def save(self, token_ids, k_seq, v_seq, seed_root_hex: str, timestamp=lambda: 0.0) -> int:
        n_full = max(0, len(token_ids) - 1) // BLOCK_SIZE
        prev, saved = seed_root_hex, 0
        for bi in range(n_full):
            s, e = bi * BLOCK_SIZE, (bi + 1) * BLOCK_SIZE
            cur = chain_prefix_hash(prev, token_ids[s:e])
            kp, vp = k_seq[:, :, :, s:e, :], v_seq[:, :, :, s:e, :]
            self.arena.write_page_fp16(cur, kp, vp)
            ev = self.table.insert(bytes.fromhex(cur), bytes.fromhex(prev), e, timestamp())
            if ev is not None and ev != cur:
                self._evict_disk_block_by_hash(ev)
            path = self.kv_dir / f"{cur[:32]}_np.npz"
            if not path.exists():
                if self.quant_mode == "int8":
                    kq, ks = quantize_kv_int8(kp)
                    vq, vs = quantize_kv_int8(vp)
                    np.savez(path, kq=kq, ks=ks, vq=vq, vs=vs)
                else:
                    np.savez(path, k=kp, v=vp)
                self._enforce_disk_budget(cur, path)
                self.blocks_saved_to_disk += 1
            prev = cur
            saved += 1
        return saved

    def match(self, token_ids, seed_root_hex: str):
        n_full = max(0, len(token_ids) - 1) // BLOCK_SIZE
        if n_full == 0:
            return 0, None, None
        prev, pids = seed_root_hex, []
        for bi in range(n_full):
            cur = chain_prefix_hash(prev, token_ids[bi * BLOCK_SIZE:(bi + 1) * BLOCK_SIZE])
            pid = self.arena.lookup_page_id(cur)
            if pid is not None:
                pids.append(pid)
                self.blocks_loaded_from_arena += 1
                prev = cur
                continue
            found = self.table.lookup(bytes.fromhex(cur))
            path = self.kv_dir / f"{cur[:32]}_np.npz"
            if (found or path.exists()) and path.exists():
                with np.load(path) as data:
                    if "kq" in data:
                        pid = self.arena.write_page_quantized(cur, data["kq"], data["ks"], data["vq"], data["vs"])
                    else:
                        pid = self.arena.write_page_fp16(cur, data["k"], data["v"])
                pids.append(pid)
                self.blocks_loaded_from_disk += 1
                prev = cur
            else:
                break
        if not pids:
            return 0, None, None
        kc, vc = self.arena.gather_contiguous_kv_numpy(pids)
        n = len(pids) * BLOCK_SIZE
        self.tokens_skipped += n
        return n, kc, vc
