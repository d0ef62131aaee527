"""Device page pool: torch-owned HBM regions driven through the libsckv C ABI.

`KVPool` owns three device regions (page data, quantisation scales, allocator
state) allocated by torch and handed to the library with `sckv_pool_wrap`.
All methods take device tensors and launch on the current torch stream;
nothing here synchronises except the explicit status / state readers.

Layout: data[layer][page][K|V][kv_head][16][head_dim]; a page id names the
same 16-token slot in every layer, as the reference's all-layer page does
(native/native_engine.py:250-257).
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch

from . import _native as N

PAGE_TOKENS = 16

DTYPE_CODES = {
    "fp16": N.DTYPE_F16,
    "bf16": N.DTYPE_BF16,
    "int8": N.DTYPE_INT8,
    "fp8_e4m3": N.DTYPE_FP8_E4M3,
}
TORCH_POOL_DTYPE = {
    "fp16": torch.float16,
    "bf16": torch.bfloat16,
    "int8": torch.int8,
    "fp8_e4m3": torch.uint8,
}
_TORCH_TO_CODE = {torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16, torch.float32: N.DTYPE_F32}


def torch_dtype_code(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported tensor dtype {dt}; expected float16, bfloat16 or float32") from None


def rope_inv_freq(theta: float, head_dim: int, device: Optional[torch.device] = None) -> torch.Tensor:
    """1 / theta^(2i / head_dim), i < head_dim / 2, computed in float32 exactly as
    ModularAttentionEngine.__init__ does (models/adapters.py:1123-1127)."""
    import numpy as np

    inv = 1.0 / (float(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / float(head_dim)))
    return torch.from_numpy(np.asarray(inv, dtype=np.float32)).to(device if device is not None else "cpu")


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, device: torch.device, dtype: Optional[torch.dtype] = None,
          min_numel: int = 0, contiguous: bool = True) -> None:
    """Reject tensors the kernels would read out of bounds or misinterpret."""
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, the pool is on {device}")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.numel() < min_numel:
        raise ValueError(f"{name} has {t.numel()} elements, needs at least {min_numel}")


def to_device(values, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Host values -> a device tensor through pinned memory, without a stream
    synchronisation. (A copy from pageable host memory makes CUDA wait for
    the stream's earlier work before it starts, so the host stops feeding
    the GPU; the pinned copy is queued behind that work instead and the
    caching host allocator keeps the buffer alive until it ran.)"""
    t = values if isinstance(values, torch.Tensor) else torch.as_tensor(values, dtype=dtype)
    t = t.to(dtype=dtype).contiguous()
    if t.device.type == "cuda":
        return t.to(device)
    return t.pin_memory().to(device, non_blocking=True)


def _dev_i32(x, device) -> torch.Tensor:
    if isinstance(x, torch.Tensor) and x.device.type == "cuda":
        return x.to(device=device, dtype=torch.int32).contiguous()
    return to_device(x, torch.int32, device)


class KVPool:
    """One page pool on one GPU."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_pages: int,
                 kv_dtype: str = "fp16", device: Optional[torch.device] = None):
        if kv_dtype not in DTYPE_CODES:
            raise ValueError(f"kv_dtype must be one of {sorted(DTYPE_CODES)}, got {kv_dtype!r}")
        self.lib = N.lib()
        dev = torch.device(device if device is not None else "cuda")
        if dev.type != "cuda":
            raise ValueError("KVPool lives in GPU memory; pass a cuda device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.num_layers, self.num_kv_heads, self.head_dim = int(num_layers), int(num_kv_heads), int(head_dim)
        self.max_pages = int(max_pages)
        self.kv_dtype = kv_dtype
        self.code = DTYPE_CODES[kv_dtype]
        data_b, scale_b, alloc_b = N.required_bytes(self.num_layers, self.num_kv_heads, self.head_dim, PAGE_TOKENS,
                                                    self.max_pages, self.code)
        with torch.cuda.device(self.device):
            self.data = torch.zeros(data_b, dtype=torch.uint8, device=self.device)
            self.scales = torch.zeros(max(scale_b, 16), dtype=torch.uint8, device=self.device) if scale_b else None
            self.alloc_region = torch.zeros(alloc_b, dtype=torch.uint8, device=self.device)
            h = ctypes.c_void_p()
            N.check(self.lib.sckv_pool_wrap(self.num_layers, self.num_kv_heads, self.head_dim, PAGE_TOKENS,
                                            self.max_pages, self.code, self.device.index, self.data.data_ptr(),
                                            _ptr(self.scales), self.alloc_region.data_ptr(), ctypes.byref(h)),
                    "sckv_pool_wrap")
            self.handle = h
            self.alloc_reset()
        self._workspace: Optional[torch.Tensor] = None

    # ------------------------------------------------------------------ views
    @property
    def bytes_per_page(self) -> int:
        """Bytes one page id occupies across all layers (data + scales)."""
        el = 2 if self.kv_dtype in ("fp16", "bf16") else 1
        b = 2 * self.num_layers * self.num_kv_heads * PAGE_TOKENS * self.head_dim * el
        if self.kv_dtype == "int8":
            b += 2 * self.num_layers * self.num_kv_heads * PAGE_TOKENS * 2
        elif self.kv_dtype == "fp8_e4m3":
            b += 2 * self.num_layers * self.num_kv_heads * 4
        return b

    def pool_view(self) -> torch.Tensor:
        """[L, P, 2, H, 16, D] view of the page data (pool element type)."""
        shape = (self.num_layers, self.max_pages, 2, self.num_kv_heads, PAGE_TOKENS, self.head_dim)
        return self.data.view(TORCH_POOL_DTYPE[self.kv_dtype]).view(shape)

    def scale_view(self) -> Optional[torch.Tensor]:
        if self.kv_dtype == "int8":
            n = self.num_layers * self.max_pages * 2 * self.num_kv_heads * PAGE_TOKENS
            return self.scales[: n * 2].view(torch.float16).view(
                self.num_layers, self.max_pages, 2, self.num_kv_heads, PAGE_TOKENS)
        if self.kv_dtype == "fp8_e4m3":
            n = self.num_layers * self.max_pages * 2 * self.num_kv_heads
            return self.scales[: n * 4].view(torch.float32).view(self.num_layers, self.max_pages, 2,
                                                                  self.num_kv_heads)
        return None

    # ---------------------------------------------------------------- kernel 1
    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, cu_tokens: torch.Tensor, start_pos: torch.Tensor,
               block_table: torch.Tensor, layer0: int = 0, max_blocks: Optional[int] = None,
               stream: Optional[torch.cuda.Stream] = None) -> None:
        """k_new, v_new: [n_layers, n_tokens, H, D] (or [n_tokens, H, D] for one layer)."""
        if k_new.dim() == 3:
            k_new, v_new = k_new.unsqueeze(0), v_new.unsqueeze(0)
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
        nl, nt = k_new.shape[0], k_new.shape[1]
        n_seqs = cu_tokens.numel() - 1
        bt = block_table if block_table.dim() == 2 else block_table.view(1, -1)
        mb = bt.shape[1] if max_blocks is None else int(max_blocks)
        if tuple(k_new.shape[2:]) != (self.num_kv_heads, self.head_dim) or k_new.shape != v_new.shape:
            raise ValueError(f"k_new/v_new must be [n_layers, n_tokens, {self.num_kv_heads}, {self.head_dim}]")
        if layer0 < 0 or layer0 + nl > self.num_layers:
            raise ValueError("append layers out of range")
        _need(k_new, "k_new", self.device)
        _need(v_new, "v_new", self.device)
        _need(cu_tokens, "cu_tokens", self.device, torch.int32, 1)
        _need(start_pos, "start_pos", self.device, torch.int32, n_seqs)
        _need(bt, "block_table", self.device, torch.int32, contiguous=False)
        if bt.dim() != 2 or bt.shape[0] < n_seqs or mb > bt.shape[1] or bt.stride(1) != 1:
            raise ValueError("block_table must be [>= n_seqs, >= max_blocks] with unit column stride")
        N.check(self.lib.sckv_append(self.handle, layer0, nl, k_new.data_ptr(), v_new.data_ptr(),
                                     torch_dtype_code(k_new.dtype), n_seqs, nt, cu_tokens.data_ptr(),
                                     start_pos.data_ptr(), bt.data_ptr(), bt.stride(0), mb, _stream_ptr(stream)),
                "sckv_append")

    def append_rope(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                    cu_tokens: torch.Tensor, start_pos: torch.Tensor, block_table: torch.Tensor,
                    inv_freq: torch.Tensor, rope_scaling: float = 1.0, q_norm_w: Optional[torch.Tensor] = None,
                    k_norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6, q_out: Optional[torch.Tensor] = None,
                    q_out_dtype: Optional[torch.dtype] = None, max_blocks: Optional[int] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """QK-norm (optional) + RoPE + append for one layer in one launch.
        q [n_tokens, Hq, D], k_new / v_new [n_tokens, Hkv, D] straight from the
        projections; returns the rotated q (q_out)."""
        q, k_new, v_new = q.contiguous(), k_new.contiguous(), v_new.contiguous()
        nt, hq, d = q.shape
        n_seqs = cu_tokens.numel() - 1
        bt = block_table if block_table.dim() == 2 else block_table.view(1, -1)
        mb = bt.shape[1] if max_blocks is None else int(max_blocks)
        if d != self.head_dim or tuple(k_new.shape) != (nt, self.num_kv_heads, d) or k_new.shape != v_new.shape:
            raise ValueError("q must be [n_tokens, Hq, D] and k_new / v_new [n_tokens, Hkv, D]")
        if k_new.dtype != v_new.dtype:
            raise TypeError("k_new and v_new must have the same dtype")
        if not 0 <= layer < self.num_layers:
            raise ValueError("layer out of range")
        for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new)):
            _need(t, name, self.device)
        _need(inv_freq, "inv_freq", self.device, torch.float32, d // 2)
        _need(cu_tokens, "cu_tokens", self.device, torch.int32, 1)
        _need(start_pos, "start_pos", self.device, torch.int32, n_seqs)
        _need(bt, "block_table", self.device, torch.int32, contiguous=False)
        if bt.dim() != 2 or bt.shape[0] < n_seqs or mb > bt.shape[1] or bt.stride(1) != 1:
            raise ValueError("block_table must be [>= n_seqs, >= max_blocks] with unit column stride")
        weights = []
        for name, w in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w)):
            if w is None:
                weights.append((None, 0))
                continue
            _need(w, name, self.device, torch.float16)
            weights.append((w, w.numel()))
        if q_out is None:
            q_out = torch.empty((nt, hq, d), dtype=q_out_dtype or q.dtype, device=self.device)
        else:
            _need(q_out, "q_out", self.device)
            if tuple(q_out.shape) != (nt, hq, d):
                raise ValueError("q_out must have q's shape")
        (qw, qn), (kw, kn) = weights
        N.check(self.lib.sckv_append_rope(self.handle, layer, q.data_ptr(), q_out.data_ptr(), hq,
                                          torch_dtype_code(q.dtype), torch_dtype_code(q_out.dtype), k_new.data_ptr(),
                                          v_new.data_ptr(), torch_dtype_code(k_new.dtype), _ptr(qw), qn, _ptr(kw), kn,
                                          float(eps), inv_freq.data_ptr(), float(rope_scaling), n_seqs, nt,
                                          cu_tokens.data_ptr(), start_pos.data_ptr(), bt.data_ptr(), bt.stride(0), mb,
                                          _stream_ptr(stream)),
                "sckv_append_rope")
        return q_out

    def qkv_append(self, layer: int, x: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor, w_v: torch.Tensor,
                   cu_tokens: torch.Tensor, start_pos: torch.Tensor, block_table: torch.Tensor,
                   inv_freq: torch.Tensor, rope_scaling: float = 1.0, q_norm_w: Optional[torch.Tensor] = None,
                   k_norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6, q_out: Optional[torch.Tensor] = None,
                   q_out_dtype: torch.dtype = torch.float32, max_blocks: Optional[int] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """q/k/v projections of x [n_tokens, hidden] with row-major weights
        (w_q [Hq*D, hidden], w_k / w_v [Hkv*D, hidden], float16 or bfloat16),
        optional per-head QK-norm, RoPE, and the K/V append for one layer, in
        one tensor-core launch; returns the rotated q [n_tokens, Hq, D].
        An fp32 x is split into hi + lo parts of the weights' type, so the
        products keep fp32 accuracy; a 16-bit x must have the weights' type.
        Pools: f16 / bf16 rows are stored directly, int8 rows quantised as
        the arena quantises its fp16 pages, FP8 rows staged in fp16 and
        stored by the FP8 append (one more launch). Whole-width norms
        (weights of Hq*D / Hkv*D elements) need every head of a token in one
        place and take the unfused route (16-bit and int8 pools): the
        projections as fp32 matmuls, then append_rope."""
        nt, hidden = x.shape
        wdt = w_q.dtype
        if wdt not in (torch.float16, torch.bfloat16) or w_k.dtype != wdt or w_v.dtype != wdt:
            raise TypeError("w_q, w_k, w_v must share one dtype, float16 or bfloat16")
        d = self.head_dim
        if w_q.dim() != 2 or w_q.shape[1] != hidden or w_q.shape[0] % d != 0:
            raise ValueError("w_q must be [Hq*D, hidden]")
        hq = w_q.shape[0] // d
        hkv = self.num_kv_heads
        for name, w in (("w_k", w_k), ("w_v", w_v)):
            if tuple(w.shape) != (hkv * d, hidden):
                raise ValueError(f"{name} must be [Hkv*D, hidden]")
        full_width = any(w is not None and w.numel() != d for w in (q_norm_w, k_norm_w))
        if full_width:
            xf = x.float()
            q = (xf @ w_q.float().T).view(nt, hq, d)
            k = (xf @ w_k.float().T).view(nt, hkv, d)
            v = (xf @ w_v.float().T).view(nt, hkv, d)
            return self.append_rope(layer, q, k, v, cu_tokens, start_pos, block_table, inv_freq, rope_scaling,
                                    q_norm_w, k_norm_w, eps, q_out, q_out_dtype, max_blocks, stream)
        x = x.contiguous()
        w_q, w_k, w_v = w_q.contiguous(), w_k.contiguous(), w_v.contiguous()
        n_seqs = cu_tokens.numel() - 1
        bt = block_table if block_table.dim() == 2 else block_table.view(1, -1)
        mb = bt.shape[1] if max_blocks is None else int(max_blocks)
        if not 0 <= layer < self.num_layers:
            raise ValueError("layer out of range")
        for name, t in (("x", x), ("w_q", w_q), ("w_k", w_k), ("w_v", w_v)):
            _need(t, name, self.device)
        _need(inv_freq, "inv_freq", self.device, torch.float32, d // 2)
        _need(cu_tokens, "cu_tokens", self.device, torch.int32, 1)
        _need(start_pos, "start_pos", self.device, torch.int32, n_seqs)
        _need(bt, "block_table", self.device, torch.int32, contiguous=False)
        if bt.dim() != 2 or bt.shape[0] < n_seqs or mb > bt.shape[1] or bt.stride(1) != 1:
            raise ValueError("block_table must be [>= n_seqs, >= max_blocks] with unit column stride")
        norms = []
        for name, w in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w)):
            if w is None:
                norms.append((None, 0))
            else:
                _need(w, name, self.device, torch.float16)
                norms.append((w, w.numel()))
        x_lo = None
        if x.dtype == torch.float32:
            hi = torch.empty((nt, hidden), dtype=wdt, device=self.device)
            x_lo = torch.empty_like(hi)
            N.check(self.lib.sckv_split_hi_lo(x.data_ptr(), x.numel(), hi.data_ptr(), x_lo.data_ptr(),
                                              torch_dtype_code(wdt), _stream_ptr(stream)), "sckv_split_hi_lo")
            x = hi
        elif x.dtype != wdt:
            raise TypeError("a 16-bit x must have the weights' dtype")
        if q_out is None:
            q_out = torch.empty((nt, hq, d), dtype=q_out_dtype, device=self.device)
        else:
            _need(q_out, "q_out", self.device)
            if tuple(q_out.shape) != (nt, hq, d):
                raise ValueError("q_out must be [n_tokens, Hq, D]")
        ws_bytes = int(self.lib.sckv_qkv_workspace_bytes(self.handle, nt, hq, hidden))
        ws = torch.empty(max(16, ws_bytes) // 4 + 4, dtype=torch.float32, device=self.device)
        (qw, qn), (kw, kn) = norms
        N.check(self.lib.sckv_qkv_append(self.handle, layer, x.data_ptr(), _ptr(x_lo), torch_dtype_code(x.dtype), nt,
                                         hidden, w_q.data_ptr(), w_k.data_ptr(), w_v.data_ptr(), hq, _ptr(qw), qn,
                                         _ptr(kw), kn, float(eps), inv_freq.data_ptr(), float(rope_scaling), n_seqs,
                                         cu_tokens.data_ptr(), start_pos.data_ptr(), bt.data_ptr(), bt.stride(0), mb,
                                         q_out.data_ptr(), torch_dtype_code(q_out.dtype), ws.data_ptr(),
                                         ws.numel() * 4, _stream_ptr(stream)),
                "sckv_qkv_append")
        if stream is not None:
            # temporaries freed on return stay reserved until `stream` is past them
            for t in (ws, x_lo, x if x_lo is not None else None):
                if t is not None:
                    t.record_stream(stream)
        return q_out

    def o_proj(self, x: torch.Tensor, w_o: torch.Tensor, out: Optional[torch.Tensor] = None,
               out_dtype: torch.dtype = torch.float32, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Output projection after attention, x [n_tokens, in_features] @
        w_o^T with w_o [out_features, in_features] (float16 or bfloat16),
        on the tensor cores; returns [n_tokens, out_features] in out_dtype.
        An fp32 x (the attention output) is split into hi + lo parts of the
        weights' type, as in qkv_append; a 16-bit x must have the weights'
        type. Needs out_features % 128 == 0 and in_features % 8 == 0."""
        if x.dim() == 3:
            x = x.reshape(x.shape[0], -1)
        x = x.contiguous()
        w_o = w_o.contiguous()
        nt, fin = x.shape
        wdt = w_o.dtype
        if wdt not in (torch.float16, torch.bfloat16):
            raise TypeError("w_o must be float16 or bfloat16")
        if w_o.dim() != 2 or w_o.shape[1] != fin:
            raise ValueError("w_o must be [out_features, in_features]")
        fout = w_o.shape[0]
        _need(x, "x", self.device)
        _need(w_o, "w_o", self.device)
        if out is None:
            out = torch.empty((nt, fout), dtype=out_dtype, device=self.device)
        else:
            _need(out, "out", self.device)
            if tuple(out.shape) != (nt, fout):
                raise ValueError("out must be [n_tokens, out_features]")
        x_lo = None
        if x.dtype == torch.float32:
            hi = torch.empty((nt, fin), dtype=wdt, device=self.device)
            x_lo = torch.empty_like(hi)
            N.check(self.lib.sckv_split_hi_lo(x.data_ptr(), x.numel(), hi.data_ptr(), x_lo.data_ptr(),
                                              torch_dtype_code(wdt), _stream_ptr(stream)), "sckv_split_hi_lo")
            x = hi
        elif x.dtype != wdt:
            raise TypeError("a 16-bit x must have the weights' dtype")
        ws_bytes = int(self.lib.sckv_o_proj_workspace_bytes(self.handle, nt, fin, fout))
        ws = torch.empty(max(16, ws_bytes) // 4 + 4, dtype=torch.float32, device=self.device)
        N.check(self.lib.sckv_o_proj(self.handle, x.data_ptr(), _ptr(x_lo), torch_dtype_code(x.dtype), nt, fin,
                                     w_o.data_ptr(), fout, out.data_ptr(), torch_dtype_code(out.dtype), ws.data_ptr(),
                                     ws.numel() * 4, _stream_ptr(stream)),
                "sckv_o_proj")
        if stream is not None:
            for t in (ws, x_lo, x if x_lo is not None else None):
                if t is not None:
                    t.record_stream(stream)
        return out

    def write_pages(self, page_ids: torch.Tensor, k_src: torch.Tensor, v_src: torch.Tensor,
                    stream: Optional[torch.cuda.Stream] = None) -> None:
        """k_src, v_src: [n, L, H, 16, D] float16 / bfloat16 / float32."""
        k_src, v_src = k_src.contiguous(), v_src.contiguous()
        n = page_ids.numel()
        shape = (n, self.num_layers, self.num_kv_heads, PAGE_TOKENS, self.head_dim)
        if tuple(k_src.shape) != shape or tuple(v_src.shape) != shape:
            raise ValueError(f"k_src/v_src must be {list(shape)}")
        _need(page_ids, "page_ids", self.device, torch.int32)
        _need(k_src, "k_src", self.device)
        _need(v_src, "v_src", self.device)
        N.check(self.lib.sckv_write_pages(self.handle, page_ids.data_ptr(), page_ids.numel(), k_src.data_ptr(),
                                          v_src.data_ptr(), torch_dtype_code(k_src.dtype), _stream_ptr(stream)),
                "sckv_write_pages")

    def write_pages_quantized(self, page_ids: torch.Tensor, kq: torch.Tensor, ks: torch.Tensor, vq: torch.Tensor,
                              vs: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> None:
        """kq/vq int8 [n, L, H, 16, D]; ks/vs float16 [n, L, H, 16]."""
        kq, ks, vq, vs = (t.contiguous() for t in (kq, ks, vq, vs))
        n = page_ids.numel()
        qs = (n, self.num_layers, self.num_kv_heads, PAGE_TOKENS, self.head_dim)
        if tuple(kq.shape) != qs or tuple(vq.shape) != qs or tuple(ks.shape) != qs[:-1] or tuple(vs.shape) != qs[:-1]:
            raise ValueError("quantized page shapes do not match the pool")
        _need(page_ids, "page_ids", self.device, torch.int32)
        for t, name, dt in ((kq, "kq", torch.int8), (vq, "vq", torch.int8), (ks, "ks", torch.float16),
                            (vs, "vs", torch.float16)):
            _need(t, name, self.device, dt)
        N.check(self.lib.sckv_write_pages_quantized(self.handle, page_ids.data_ptr(), page_ids.numel(),
                                                    kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
                                                    _stream_ptr(stream)),
                "sckv_write_pages_quantized")

    # ---------------------------------------------------------------- kernel 2
    def gather(self, page_ids: torch.Tensor, n_tokens: Optional[int] = None, layer0: int = 0,
               n_layers: Optional[int] = None, out_dtype: torch.dtype = torch.float16,
               out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
               stream: Optional[torch.cuda.Stream] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Contiguous [n_layers, H, n_tokens, D] K and V of the listed pages."""
        n_pages = page_ids.numel()
        nt = n_pages * PAGE_TOKENS if n_tokens is None else int(n_tokens)
        nl = self.num_layers - layer0 if n_layers is None else int(n_layers)
        shape = (nl, self.num_kv_heads, nt, self.head_dim)
        _need(page_ids, "page_ids", self.device, torch.int32)
        if nt > n_pages * PAGE_TOKENS or layer0 < 0 or layer0 + nl > self.num_layers:
            raise ValueError("gather range out of bounds")
        if out is not None:
            for t in out:
                _need(t, "out", self.device)
                if tuple(t.shape) != shape:
                    raise ValueError(f"gather outputs must be {list(shape)}")
        if out is None:
            ok = torch.empty(shape, dtype=out_dtype, device=self.device)
            ov = torch.empty(shape, dtype=out_dtype, device=self.device)
        else:
            ok, ov = out
        N.check(self.lib.sckv_gather(self.handle, layer0, nl, page_ids.data_ptr(), n_pages, nt, ok.data_ptr(),
                                     ov.data_ptr(), torch_dtype_code(ok.dtype), _stream_ptr(stream)),
                "sckv_gather")
        return ok, ov

    def copy_pages(self, src_ids: torch.Tensor, dst_ids: torch.Tensor,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
        _need(src_ids, "src_ids", self.device, torch.int32)
        _need(dst_ids, "dst_ids", self.device, torch.int32, src_ids.numel())
        N.check(self.lib.sckv_copy_pages(self.handle, src_ids.data_ptr(), dst_ids.data_ptr(), src_ids.numel(),
                                         _stream_ptr(stream)), "sckv_copy_pages")

    # -------------------------------------------------------------- kernels 3+4
    def decode_workspace_bytes(self, n_seqs: int, num_q_heads: int, max_blocks: int, chunk_pages: int = 0) -> int:
        return int(self.lib.sckv_decode_workspace_bytes(self.handle, n_seqs, num_q_heads, max_blocks, chunk_pages))

    def _decode_args(self, layer, q, block_table, ctx_lens, scale, out, out_dtype, max_blocks, chunk_pages,
                     workspace):
        """Checks shared by the decode entry points; returns (q, B, hq, mb,
        scale, out, workspace)."""
        q = q.contiguous()
        B, hq, d = q.shape
        mb = block_table.shape[1] if max_blocks is None else int(max_blocks)
        if d != self.head_dim or hq % self.num_kv_heads != 0:
            raise ValueError(f"q must be [B, k*{self.num_kv_heads}, {self.head_dim}]")
        if not 0 <= layer < self.num_layers:
            raise ValueError("layer out of range")
        _need(q, "q", self.device)
        _need(ctx_lens, "ctx_lens", self.device, torch.int32, B)
        _need(block_table, "block_table", self.device, torch.int32, contiguous=False)
        if block_table.dim() != 2 or block_table.stride(1) != 1 or mb > block_table.shape[1]:
            raise ValueError("block_table must be 2-D with unit column stride and >= max_blocks columns")
        if block_table.stride(0) != 0 and block_table.shape[0] < B:
            raise ValueError("block_table has fewer rows than sequences")
        if scale is None:
            scale = float(d) ** -0.5
        if out is None:
            out = torch.empty((B, hq, d), dtype=out_dtype or q.dtype, device=self.device)
        else:
            _need(out, "out", self.device, min_numel=B * hq * d)
            if tuple(out.shape) != (B, hq, d):
                raise ValueError("out must have q's shape")
        need = self.decode_workspace_bytes(B, hq, mb, chunk_pages)
        if workspace is not None:
            _need(workspace, "workspace", self.device, min_numel=need)
        if workspace is None:
            if self._workspace is None or self._workspace.numel() < need:
                self._workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=self.device)
            workspace = self._workspace
        return q, B, hq, mb, float(scale), out, workspace

    def decode_attn(self, layer: int, q: torch.Tensor, block_table: torch.Tensor, ctx_lens: torch.Tensor,
                    scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                    out_dtype: Optional[torch.dtype] = None, max_blocks: Optional[int] = None,
                    chunk_pages: int = 0, workspace: Optional[torch.Tensor] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """q [B, Hq, D] -> out [B, Hq, D]: softmax(scale q K^T) V over each
        sequence's first ctx_lens[b] tokens of `layer`."""
        q, B, hq, mb, scale, out, workspace = self._decode_args(layer, q, block_table, ctx_lens, scale, out,
                                                                out_dtype, max_blocks, chunk_pages, workspace)
        N.check(self.lib.sckv_decode_attn(self.handle, layer, q.data_ptr(), torch_dtype_code(q.dtype), hq,
                                          block_table.data_ptr(), block_table.stride(0), mb, ctx_lens.data_ptr(), B,
                                          scale, out.data_ptr(), torch_dtype_code(out.dtype),
                                          workspace.data_ptr(), workspace.numel(), chunk_pages, _stream_ptr(stream)),
                "sckv_decode_attn")
        return out

    def decode_attn_append(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                           block_table: torch.Tensor, ctx_lens: torch.Tensor, scale: Optional[float] = None,
                           out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                           max_blocks: Optional[int] = None, chunk_pages: int = 0,
                           workspace: Optional[torch.Tensor] = None,
                           stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """One decode step of `layer`: the new token's k_new / v_new [B, Hkv, D]
        go to position ctx_lens[b] - 1 of each sequence, then q [B, Hq, D]
        attends over ctx_lens[b] tokens. 16-bit pools do both in the decode
        launch (sckv_decode_attn_append); one-byte pools, whose rows are
        quantised against their page or token scale, run sckv_append then
        sckv_decode_attn."""
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
        q, B, hq, mb, scale, out, workspace = self._decode_args(layer, q, block_table, ctx_lens, scale, out,
                                                                out_dtype, max_blocks, chunk_pages, workspace)
        if tuple(k_new.shape) != (B, self.num_kv_heads, self.head_dim) or k_new.shape != v_new.shape:
            raise ValueError(f"k_new/v_new must be [B, {self.num_kv_heads}, {self.head_dim}]")
        if k_new.dtype != v_new.dtype:
            raise TypeError("k_new and v_new must have the same dtype")
        _need(k_new, "k_new", self.device)
        _need(v_new, "v_new", self.device)
        if self.kv_dtype not in ("fp16", "bf16"):
            cu = torch.arange(B + 1, dtype=torch.int32, device=self.device)
            self.append(k_new, v_new, cu, ctx_lens - 1, block_table, layer0=layer, max_blocks=mb, stream=stream)
            return self.decode_attn(layer, q, block_table, ctx_lens, scale=scale, out=out, max_blocks=mb,
                                    chunk_pages=chunk_pages, workspace=workspace, stream=stream)
        N.check(self.lib.sckv_decode_attn_append(self.handle, layer, q.data_ptr(), torch_dtype_code(q.dtype), hq,
                                                 k_new.data_ptr(), v_new.data_ptr(), torch_dtype_code(k_new.dtype),
                                                 block_table.data_ptr(), block_table.stride(0), mb,
                                                 ctx_lens.data_ptr(), B, scale, out.data_ptr(),
                                                 torch_dtype_code(out.dtype), workspace.data_ptr(),
                                                 workspace.numel(), chunk_pages, _stream_ptr(stream)),
                "sckv_decode_attn_append")
        return out

    def prefill_attn(self, layer: int, q: torch.Tensor, cu_q: torch.Tensor, start_pos: torch.Tensor,
                     block_table: torch.Tensor, scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     out_dtype: Optional[torch.dtype] = None, max_blocks: Optional[int] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Causal attention of new query tokens q [n_tokens, Hq, D] (sequence b
        owns rows cu_q[b]..cu_q[b+1]-1 at positions start_pos[b]+i) over their
        sequences' pages. Raises SCKVError(SCKV_ERR_UNSUPPORTED) for pool /
        head combinations the tensor-core kernel does not build."""
        q = q.contiguous()
        n_tok, hq, d = q.shape
        n_seqs = cu_q.numel() - 1
        mb = block_table.shape[1] if max_blocks is None else int(max_blocks)
        if d != self.head_dim or hq % self.num_kv_heads != 0:
            raise ValueError(f"q must be [n_tokens, k*{self.num_kv_heads}, {self.head_dim}]")
        if not 0 <= layer < self.num_layers:
            raise ValueError("layer out of range")
        _need(q, "q", self.device)
        _need(cu_q, "cu_q", self.device, torch.int32, 2)
        _need(start_pos, "start_pos", self.device, torch.int32, n_seqs)
        _need(block_table, "block_table", self.device, torch.int32, contiguous=False)
        if block_table.dim() != 2 or block_table.stride(1) != 1 or block_table.shape[0] < n_seqs or \
                mb > block_table.shape[1] or block_table.stride(0) < mb:
            raise ValueError("block_table must be [>= n_seqs, >= max_blocks] rows with unit column stride")
        if scale is None:
            scale = float(d) ** -0.5
        if out is None:
            out = torch.empty((n_tok, hq, d), dtype=out_dtype or q.dtype, device=self.device)
        else:
            _need(out, "out", self.device)
            if tuple(out.shape) != (n_tok, hq, d):
                raise ValueError("out must have q's shape")
        N.check(self.lib.sckv_prefill_attn(self.handle, layer, q.data_ptr(), torch_dtype_code(q.dtype), hq, n_seqs,
                                           n_tok, cu_q.data_ptr(), start_pos.data_ptr(), block_table.data_ptr(),
                                           block_table.stride(0), mb, float(scale), out.data_ptr(),
                                           torch_dtype_code(out.dtype), _stream_ptr(stream)),
                "sckv_prefill_attn")
        return out

    # ---------------------------------------------------------------- kernel 5
    def alloc_reset(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        N.check(self.lib.sckv_alloc_reset(self.handle, _stream_ptr(stream)), "sckv_alloc_reset")

    def alloc_pages(self, n: int, pin: bool = False, stream: Optional[torch.cuda.Stream] = None
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
        ids = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        vic = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        N.check(self.lib.sckv_alloc_pages(self.handle, n, 1 if pin else 0, ids.data_ptr(), vic.data_ptr(),
                                          _stream_ptr(stream)), "sckv_alloc_pages")
        return ids[:n], vic[:n]

    def free_pages(self, ids: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> None:
        ids = _dev_i32(ids, self.device)
        N.check(self.lib.sckv_free_pages(self.handle, ids.data_ptr(), ids.numel(), _stream_ptr(stream)),
                "sckv_free_pages")

    def touch_pages(self, ids: torch.Tensor, stream: Optional[torch.cuda.Stream] = None) -> None:
        ids = _dev_i32(ids, self.device)
        N.check(self.lib.sckv_touch_pages(self.handle, ids.data_ptr(), ids.numel(), _stream_ptr(stream)),
                "sckv_touch_pages")

    def pin_pages(self, ids: torch.Tensor, delta: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        ids = _dev_i32(ids, self.device)
        N.check(self.lib.sckv_pin_pages(self.handle, ids.data_ptr(), ids.numel(), int(delta), _stream_ptr(stream)),
                "sckv_pin_pages")

    def release_pages(self, ids: torch.Tensor, keep_cached: bool = False,
                      stream: Optional[torch.cuda.Stream] = None) -> None:
        ids = _dev_i32(ids, self.device)
        N.check(self.lib.sckv_release_pages(self.handle, ids.data_ptr(), ids.numel(), 1 if keep_cached else 0,
                                            _stream_ptr(stream)), "sckv_release_pages")

    def evict_lru(self, n: int, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        out = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        N.check(self.lib.sckv_evict_lru(self.handle, n, out.data_ptr(), _stream_ptr(stream)), "sckv_evict_lru")
        return out[:n]

    def evict_to_watermark(self, max_allocated: int, out_count: Optional[torch.Tensor] = None,
                           stream: Optional[torch.cuda.Stream] = None) -> None:
        """Evict LRU unpinned pages until at most max_allocated are allocated
        (decided on the device; out_count, an int32 device tensor, receives
        how many were evicted)."""
        if out_count is not None:
            _need(out_count, "out_count", self.device, torch.int32, 1)
        N.check(self.lib.sckv_evict_to_watermark(self.handle, int(max_allocated), _ptr(out_count),
                                                 _stream_ptr(stream)), "sckv_evict_to_watermark")

    def reserve_decode(self, block_table: torch.Tensor, ctx_lens: torch.Tensor, n_seqs: Optional[int] = None,
                       max_blocks: Optional[int] = None, stream: Optional[torch.cuda.Stream] = None) -> None:
        n = ctx_lens.numel() if n_seqs is None else int(n_seqs)
        mb = block_table.shape[1] if max_blocks is None else int(max_blocks)
        _need(ctx_lens, "ctx_lens", self.device, torch.int32, n)
        _need(block_table, "block_table", self.device, torch.int32, contiguous=False)
        if block_table.dim() != 2 or block_table.stride(1) != 1 or block_table.shape[0] < n or \
                mb > block_table.shape[1]:
            raise ValueError("block_table must be [>= n_seqs, >= max_blocks] with unit column stride")
        N.check(self.lib.sckv_reserve_decode(self.handle, block_table.data_ptr(), block_table.stride(0), mb,
                                             ctx_lens.data_ptr(), n, _stream_ptr(stream)), "sckv_reserve_decode")

    def alloc_state(self, stream: Optional[torch.cuda.Stream] = None) -> Dict[str, int]:
        arr = (ctypes.c_int64 * 5)()
        N.check(self.lib.sckv_alloc_state(self.handle, arr, _stream_ptr(stream)), "sckv_alloc_state")
        head, tail, clock, ev, alloc = (int(x) for x in arr)
        return {"head": head, "tail": tail, "free": tail - head, "clock": clock, "evictions": ev,
                "allocated": alloc}

    # ------------------------------------------------------------ status word
    def status(self, stream: Optional[torch.cuda.Stream] = None) -> Tuple[int, int, int, int]:
        arr = (ctypes.c_int32 * 4)()
        N.check(self.lib.sckv_get_status(self.handle, arr, _stream_ptr(stream)), "sckv_get_status")
        return int(arr[0]), int(arr[1]), int(arr[2]), int(arr[3])

    def selftest_wait_timeout(self, limit_us: int = 20000, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Launch a kernel whose bounded wait runs out (nothing completes its
        barrier): afterwards status() reads SCKV_ERR_TIMEOUT, detail -1."""
        N.check(self.lib.sckv_selftest_wait_timeout(self.handle, int(limit_us), _stream_ptr(stream)),
                "sckv_selftest_wait_timeout")

    def clear_status(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        N.check(self.lib.sckv_clear_status(self.handle, _stream_ptr(stream)), "sckv_clear_status")

    def raise_on_status(self) -> None:
        code, detail, kernel, count = self.status()
        if code != N.SCKV_OK:
            self.clear_status()
            err = N.SCKVPoolExhausted if code == N.SCKV_ERR_POOL_EXHAUSTED else (
                N.SCKVBoundsError if code == N.SCKV_ERR_BOUNDS else N.SCKVError)
            e = err(code, f"device status (kernel {kernel}, detail {detail}, {count} errors)")
            raise e

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.sckv_pool_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
