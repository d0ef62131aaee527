"""Drop-in PagedKVArena with its page pool in GPU memory.

Same constructor, attributes and methods as the reference arena
(native/native_engine.py:224-432): 16-token pages keyed by prefix hash,
`page_table` / `reverse_page_table` / `page_last_used` dicts, a FIFO
`free_pages` deque, a `step_clock` that ticks on every allocation and lookup,
and LRU victim choice (smallest last-used clock) when the free list is empty.
The bookkeeping stays on the host because callers hold and mutate these
containers directly (the reference's own tests clear and refill
`free_pages`); the page bytes live in a `KVPool` on the GPU and every copy,
int8 quantisation and dequantisation runs in the libsckv kernels.

Differences callers can see:
  * pool views (`k_pool_fp16`, `k_pool_q`, `k_scale`, ...) are torch CUDA
    tensors shaped like the reference's numpy pools [P, L, 1, H, 16, D];
  * `read_page_fp16` returns host numpy copies (the reference returns views
    of its numpy pool in fp16 mode); `read_page_device` returns device views;
  * `gather_contiguous_kv` returns device tensors; the `_numpy` form copies
    the result to the host as the reference's name promises.
"""
from __future__ import annotations

import collections
import threading
from typing import Deque, Dict, List, Optional, Tuple, Union

import numpy as np
import torch

from .npz_io import parallel_for
from .pool import KVPool, PAGE_TOKENS

ArrayLike = Union[np.ndarray, torch.Tensor]


def _to_device(x: ArrayLike, device: torch.device, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        t = x.to(device=device)
    else:
        t = torch.from_numpy(np.ascontiguousarray(x)).to(device)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


class PagedKVArena:
    """Fixed pool of 16-token pages (all layers, all KV heads) on one GPU."""

    PAGE_TOKENS: int = PAGE_TOKENS

    def __init__(self, max_pages: int = 64, num_layers: int = 16, num_kv_heads: int = 16, head_dim: int = 128,
                 quant_mode: str = "fp16", device: Optional[Union[str, torch.device]] = None):
        if quant_mode not in ("fp16", "int8"):
            raise ValueError(f"Unsupported kv_quant_mode={quant_mode!r}; expected 'fp16' or 'int8'")
        self.max_pages: int = max(1, int(max_pages))
        self.num_layers: int = int(num_layers)
        self.num_kv_heads: int = int(num_kv_heads)
        self.head_dim: int = int(head_dim)
        self.quant_mode: str = quant_mode
        self.lock = threading.RLock()
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type != "cuda" or dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.pool: Optional[KVPool] = KVPool(self.num_layers, self.num_kv_heads, self.head_dim, self.max_pages,
                                             quant_mode, device=dev)
        # reference byte accounting (native/native_engine.py:271-283)
        L, H, D, T = self.num_layers, self.num_kv_heads, self.head_dim, self.PAGE_TOKENS
        if quant_mode == "int8":
            self.bytes_per_page: int = 2 * L * H * T * D * 1 + 2 * L * H * T * 2
        else:
            self.bytes_per_page = 2 * L * H * T * D * 2
        self._bind_views()
        self.free_pages: Deque[int] = collections.deque(range(self.max_pages))
        self.page_table: Dict[str, int] = {}
        self.reverse_page_table: Dict[int, str] = {}
        self.page_last_used: Dict[str, int] = {}
        self.step_clock: int = 0
        self.page_hits: int = 0
        self.page_misses: int = 0
        self.page_evictions: int = 0

    # ---------------------------------------------------------------- views
    def _bind_views(self) -> None:
        v = self.pool.pool_view()  # [L, P, 2, H, 16, D]
        k_view = v[:, :, 0].permute(1, 0, 2, 3, 4).unsqueeze(2)  # [P, L, 1, H, 16, D]
        v_view = v[:, :, 1].permute(1, 0, 2, 3, 4).unsqueeze(2)
        if self.quant_mode == "int8":
            s = self.pool.scale_view()  # [L, P, 2, H, 16]
            self.k_pool_q, self.v_pool_q = k_view, v_view
            self.k_scale = s[:, :, 0].permute(1, 0, 2, 3).unsqueeze(2).unsqueeze(-1)
            self.v_scale = s[:, :, 1].permute(1, 0, 2, 3).unsqueeze(2).unsqueeze(-1)
            self.k_pool_fp16 = self.v_pool_fp16 = None
        else:
            self.k_pool_fp16, self.v_pool_fp16 = k_view, v_view
            self.k_pool_q = self.v_pool_q = self.k_scale = self.v_scale = None

    def _ids(self, ids: List[int]) -> torch.Tensor:
        return torch.tensor(ids, dtype=torch.int32, device=self.device)

    # ----------------------------------------------------------- bookkeeping
    def lookup_page_id(self, prefix_hash_hex: str) -> Optional[int]:
        """native/native_engine.py:297-305."""
        with self.lock:
            self.step_clock += 1
            if prefix_hash_hex in self.page_table:
                self.page_hits += 1
                self.page_last_used[prefix_hash_hex] = self.step_clock
                return self.page_table[prefix_hash_hex]
            self.page_misses += 1
            return None

    def evict_prefix_hash(self, prefix_hash_hex: str) -> bool:
        """native/native_engine.py:307-316."""
        with self.lock:
            page_id = self.page_table.pop(prefix_hash_hex, None)
            if page_id is None:
                return False
            self.reverse_page_table.pop(page_id, None)
            self.page_last_used.pop(prefix_hash_hex, None)
            self.free_pages.append(page_id)
            self.page_evictions += 1
            return True

    def _allocate_page_slot_unlocked(self, prefix_hash_hex: str) -> int:
        """native/native_engine.py:318-337: existing key -> touch; else FIFO
        free list; else evict the least recently used key."""
        if prefix_hash_hex in self.page_table:
            self.step_clock += 1
            self.page_last_used[prefix_hash_hex] = self.step_clock
            return self.page_table[prefix_hash_hex]
        if self.free_pages:
            page_id = self.free_pages.popleft()
        else:
            victim = min(self.page_table.keys(), key=lambda h: self.page_last_used.get(h, 0))
            page_id = self.page_table.pop(victim)
            self.reverse_page_table.pop(page_id, None)
            self.page_last_used.pop(victim, None)
            self.page_evictions += 1
        self.step_clock += 1
        self.page_table[prefix_hash_hex] = page_id
        self.reverse_page_table[page_id] = prefix_hash_hex
        self.page_last_used[prefix_hash_hex] = self.step_clock
        return page_id

    # ----------------------------------------------------------------- writes
    def _check_pool(self) -> KVPool:
        if self.pool is None:
            raise AssertionError("arena pools were released by clear()")
        return self.pool

    def write_page_fp16(self, prefix_hash_hex: str, k_page: ArrayLike, v_page: ArrayLike) -> int:
        """Allocate (or touch) the page for this key and store K/V
        [L, 1, H, 16, D] fp16 — quantised to int8 in int8 mode
        (native/native_engine.py:339-359)."""
        with self.lock:
            pool = self._check_pool()
            page_id = self._allocate_page_slot_unlocked(prefix_hash_hex)
            shape = (1, self.num_layers, self.num_kv_heads, self.PAGE_TOKENS, self.head_dim)
            k = _to_device(k_page, self.device, torch.float16).reshape(shape)
            v = _to_device(v_page, self.device, torch.float16).reshape(shape)
            pool.write_pages(self._ids([page_id]), k, v)
            return page_id

    def write_pages_fp16(self, prefix_hashes: List[str], k_pages: ArrayLike, v_pages: ArrayLike) -> List[int]:
        """Batched write_page_fp16: allocations happen in list order exactly
        as n single calls; the page bytes move in one launch. k_pages/v_pages
        are [n, L, 1, H, 16, D] (or [n, L, H, 16, D])."""
        with self.lock:
            pool = self._check_pool()
            ids = [self._allocate_page_slot_unlocked(h) for h in prefix_hashes]
            n = len(ids)
            if n == 0:
                return ids
            shape = (n, self.num_layers, self.num_kv_heads, self.PAGE_TOKENS, self.head_dim)
            k = _to_device(k_pages, self.device, torch.float16).reshape(shape)
            v = _to_device(v_pages, self.device, torch.float16).reshape(shape)
            # a page id reused within the batch keeps its last write
            last = {}
            for i, pid in enumerate(ids):
                last[pid] = i
            sel = sorted(last.values())
            if len(sel) != n:
                k, v = k[sel], v[sel]
            pool.write_pages(self._ids([ids[i] for i in sel]), k, v)
            return ids

    def reserve_page(self, prefix_hash_hex: str) -> int:
        """The allocation step of write_page_fp16 alone (same clock, free-list
        and LRU effects); the caller writes the page bytes later."""
        with self.lock:
            self._check_pool()
            return self._allocate_page_slot_unlocked(prefix_hash_hex)

    def write_loaded_pages(self, entries: List[Tuple[int, Dict[str, np.ndarray]]]) -> None:
        """Write pages reloaded from `.npz` blocks, in list order, with one
        pinned host -> device copy per array kind and one write launch per
        kind. Each entry is (page_id, arrays) with arrays either {k, v}
        ([L, 1, H, 16, D] fp16) or {kq, ks, vq, vs} (int8 codes and fp16
        scales). A page id listed twice keeps its last entry, as writing the
        entries one by one would."""
        last: Dict[int, int] = {}
        for i, (pid, _) in enumerate(entries):
            last[int(pid)] = i
        plain = [entries[i] for i in sorted(last.values()) if "kq" not in entries[i][1]]
        quant = [entries[i] for i in sorted(last.values()) if "kq" in entries[i][1]]
        L, H, T, D = self.num_layers, self.num_kv_heads, self.PAGE_TOKENS, self.head_dim
        with self.lock:
            pool = self._check_pool()
            if plain:
                k = self._stage([a["k"] for _, a in plain], (L, H, T, D), torch.float16)
                v = self._stage([a["v"] for _, a in plain], (L, H, T, D), torch.float16)
                pool.write_pages(self._ids([p for p, _ in plain]), k, v)
            if quant:
                kq = self._stage([a["kq"] for _, a in quant], (L, H, T, D), torch.int8)
                vq = self._stage([a["vq"] for _, a in quant], (L, H, T, D), torch.int8)
                ks = self._stage([a["ks"] for _, a in quant], (L, H, T), torch.float16)
                vs = self._stage([a["vs"] for _, a in quant], (L, H, T), torch.float16)
                pool.write_pages_quantized(self._ids([p for p, _ in quant]), kq, ks, vq, vs)

    def _stage(self, arrays: List[np.ndarray], shape: Tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        """Stack host arrays into one pinned buffer and start its copy to the
        device (the pinned block is not reused before the copy completes)."""
        host = torch.empty((len(arrays),) + shape, dtype=dtype, pin_memory=True)
        h = host.numpy()

        def fill(i: int) -> None:
            h[i] = np.asarray(arrays[i]).reshape(shape)

        parallel_for(fill, len(arrays))
        return host.to(self.device, non_blocking=True)

    def write_page_quantized(self, prefix_hash_hex: str, kq: ArrayLike, ks: ArrayLike, vq: ArrayLike,
                             vs: ArrayLike) -> int:
        """native/native_engine.py:361-386: int8 mode stores codes + fp16
        scales; fp16 mode stores fp16(q * f32(scale))."""
        with self.lock:
            pool = self._check_pool()
            page_id = self._allocate_page_slot_unlocked(prefix_hash_hex)
            L, H, T, D = self.num_layers, self.num_kv_heads, self.PAGE_TOKENS, self.head_dim
            kq_t = _to_device(kq, self.device, torch.int8).reshape(1, L, H, T, D)
            vq_t = _to_device(vq, self.device, torch.int8).reshape(1, L, H, T, D)
            ks_t = _to_device(ks, self.device, torch.float16).reshape(1, L, H, T)
            vs_t = _to_device(vs, self.device, torch.float16).reshape(1, L, H, T)
            pool.write_pages_quantized(self._ids([page_id]), kq_t, ks_t, vq_t, vs_t)
            return page_id

    # ------------------------------------------------------------------ reads
    def read_page_device(self, page_id: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """[L, 1, H, 16, D] fp16 device tensors (dequantised in int8 mode)."""
        with self.lock:
            pool = self._check_pool()
            k, v = pool.gather(self._ids([page_id]), out_dtype=torch.float16)
            return k.unsqueeze(1), v.unsqueeze(1)

    def read_page_fp16(self, page_id: int) -> Tuple[np.ndarray, np.ndarray]:
        """native/native_engine.py:388-401 (host copies)."""
        k, v = self.read_page_device(page_id)
        return k.cpu().numpy(), v.cpu().numpy()

    def read_page_quantized(self, page_id: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        """int8 mode: the stored codes and fp16 scales of one page
        ([L,1,H,16,D] int8, [L,1,H,16,1] fp16 each for K and V)."""
        if self.quant_mode != "int8":
            raise ValueError("read_page_quantized needs quant_mode='int8'")
        with self.lock:
            self._check_pool()
            return (self.k_pool_q[page_id].cpu().numpy(), self.k_scale[page_id].cpu().numpy(),
                    self.v_pool_q[page_id].cpu().numpy(), self.v_scale[page_id].cpu().numpy())

    def gather_contiguous_kv(self, page_ids: List[int], out_dtype: torch.dtype = torch.float16
                             ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Pages in list order -> contiguous [L, 1, H, n*16, D] device tensors."""
        with self.lock:
            pool = self._check_pool()
            if len(page_ids) == 0:
                shape = (self.num_layers, 1, self.num_kv_heads, 0, self.head_dim)
                return (torch.empty(shape, dtype=out_dtype, device=self.device),
                        torch.empty(shape, dtype=out_dtype, device=self.device))
            k, v = pool.gather(self._ids([int(p) for p in page_ids]), out_dtype=out_dtype)
            return k.unsqueeze(1), v.unsqueeze(1)

    def gather_contiguous_kv_numpy(self, page_ids: List[int]) -> Tuple[np.ndarray, np.ndarray]:
        """native/native_engine.py:403-419."""
        k, v = self.gather_contiguous_kv(page_ids)
        return k.cpu().numpy(), v.cpu().numpy()

    def clear(self) -> None:
        """native/native_engine.py:421-432: reset the tables and drop the pools."""
        with self.lock:
            self.page_table.clear()
            self.reverse_page_table.clear()
            self.page_last_used.clear()
            self.free_pages = collections.deque(range(self.max_pages))
            if self.pool is not None:
                self.pool.close()
            self.pool = None
            self.k_pool_fp16 = self.v_pool_fp16 = None
            self.k_pool_q = self.v_pool_q = self.k_scale = self.v_scale = None
