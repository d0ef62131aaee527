"""Drop-in NativeKVPrefixCache over the GPU arena.

Behaviour follows native/native_engine.py:2125-2435 (NumPy path):
16-token prefix blocks chained by SHA-256 from a seed root, pages written
into the arena and registered in the KV hash table, one `.npz` per block on
disk (keys k, v — or kq, ks, vq, vs in int8 mode) under an LRU disk budget,
and longest-prefix matching that takes arena hits first and reloads evicted
blocks from disk. A match allocates reloaded pages during its walk (the
reference's bookkeeping order), then reads their block files in parallel and
moves them to the device in one pinned copy and one write launch per block
kind. The page bytes live on the GPU; the int8 codes saved to
disk are read back from the device quantiser, so they are the codes the
reference's quantize_kv_int8_numpy would produce.

The MLX variants (match_longest_prefix_mlx / save_prefix_blocks_mlx) are
Apple-only; `match_longest_prefix` returns device tensors instead.
"""
from __future__ import annotations

import collections
import hashlib
import struct
import time
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple, TypedDict, Union

import numpy as np
import torch

from .arena import PagedKVArena
from .kv_index import KVPrefixIndex
from .npz_io import read_npz_many


class PagedKVStats(TypedDict):
    quant_mode: str
    page_tokens: int
    max_pages: int
    allocated_pages: int
    free_pages: int
    bytes_per_page: int
    arena_allocated_mb: float
    arena_active_mb: float
    page_hits: int
    page_misses: int
    page_evictions: int
    kv_hash_evictions: int
    disk_blocks_evicted: int


def chain_merkle_prefix_hash(prev_hash_hex: str, token_block: Sequence[int]) -> str:
    """sha256(bytes(prev) || u32le tokens) as hex (native/native_engine.py:778-782)."""
    h = hashlib.sha256()
    h.update(bytes.fromhex(prev_hash_hex))
    h.update(struct.pack(f"<{len(token_block)}I", *[int(t) for t in token_block]))
    return h.digest().hex()


class NativeKVPrefixCache:
    """Paged 16-token prefix KV cache backed by a GPU PagedKVArena."""

    BLOCK_SIZE: int = 16

    def __init__(self, store_dir: Union[str, Path], bridge: Optional[object] = None, device: str = "cuda",
                 num_layers: int = 16, num_kv_heads: int = 16, head_dim: int = 128, max_pages: int = 64,
                 max_disk_blocks: int = 512, quant_mode: str = "fp16", timestamp_fn=time.time):
        self.store_dir = Path(store_dir)
        self.kv_dir = self.store_dir / "kv_cache_blocks"
        self.kv_dir.mkdir(parents=True, exist_ok=True)
        self.bridge = bridge if bridge is not None else KVPrefixIndex()
        self.device = device
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.max_disk_blocks = max(1, int(max_disk_blocks))
        self.quant_mode = quant_mode
        torch_dev = device if isinstance(device, torch.device) or str(device).startswith("cuda") else None
        self.arena = PagedKVArena(max_pages=max_pages, num_layers=num_layers, num_kv_heads=num_kv_heads,
                                  head_dim=head_dim, quant_mode=quant_mode, device=torch_dev)
        self.disk_lru: "collections.OrderedDict[str, Path]" = collections.OrderedDict()
        self.blocks_loaded_from_disk = 0
        self.blocks_loaded_from_arena = 0
        self.blocks_saved_to_disk = 0
        self.disk_blocks_evicted = 0
        self.tokens_skipped = 0
        self._now = timestamp_fn

    # ---------------------------------------------------------------- disk
    def _npz_path(self, h: str) -> Path:
        return self.kv_dir / f"{h[:32]}_np.npz"

    def _evict_disk_block_by_hash(self, h: str) -> None:
        """native/native_engine.py:2173-2187."""
        self.arena.evict_prefix_hash(h)
        p = self.disk_lru.pop(h, None)
        for cand in (p, self.kv_dir / f"{h[:32]}_mlx.safetensors", self.kv_dir / f"{h[:32]}_mlx_int8.safetensors",
                     self._npz_path(h)):
            if cand is not None and cand.exists():
                try:
                    cand.unlink()
                    self.disk_blocks_evicted += 1
                except OSError:
                    pass

    def _enforce_disk_budget(self, h: str, path: Path) -> None:
        """native/native_engine.py:2189-2200."""
        self.disk_lru[h] = path
        self.disk_lru.move_to_end(h)
        while len(self.disk_lru) > self.max_disk_blocks:
            oh, op = self.disk_lru.popitem(last=False)
            self.arena.evict_prefix_hash(oh)
            if op.exists():
                try:
                    op.unlink()
                    self.disk_blocks_evicted += 1
                except OSError:
                    pass

    # ---------------------------------------------------------------- save
    def save_prefix_blocks_numpy(self, token_ids: List[int], k_seq_np, v_seq_np, seed_root_hex: str) -> int:
        """native/native_engine.py:2202-2246. k_seq/v_seq: [L, 1, H, T, D]
        fp16 (numpy or torch)."""
        n_full = max(0, len(token_ids) - 1) // self.BLOCK_SIZE
        if n_full == 0:
            return 0
        k_host = k_seq_np if isinstance(k_seq_np, np.ndarray) else k_seq_np.detach().cpu().numpy()
        v_host = v_seq_np if isinstance(v_seq_np, np.ndarray) else v_seq_np.detach().cpu().numpy()
        prev = seed_root_hex
        saved = 0
        for bi in range(n_full):
            s, e = bi * self.BLOCK_SIZE, (bi + 1) * self.BLOCK_SIZE
            cur = chain_merkle_prefix_hash(prev, token_ids[s:e])
            kp = k_host[:, :, :, s:e, :]
            vp = v_host[:, :, :, s:e, :]
            pid = self.arena.write_page_fp16(cur, kp, vp)
            ev = self.bridge.kv_insert(bytes.fromhex(cur), bytes.fromhex(prev), e, self._now())
            if ev is not None and ev != cur:
                self._evict_disk_block_by_hash(ev)
            path = self._npz_path(cur)
            if not path.exists():
                if self.quant_mode == "int8":
                    # codes and scales exactly as stored by the device quantiser
                    kq, ks, vq, vs = self.arena.read_page_quantized(pid)
                    np.savez(path, kq=kq, ks=ks, vq=vq, vs=vs)
                else:
                    np.savez(path, k=np.ascontiguousarray(kp, dtype=np.float16),
                             v=np.ascontiguousarray(vp, dtype=np.float16))
                self._enforce_disk_budget(cur, path)
                self.blocks_saved_to_disk += 1
            prev = cur
            saved += 1
        return saved

    # ---------------------------------------------------------------- match
    def _match_page_ids(self, token_ids: List[int], seed_root_hex: str) -> List[int]:
        n_full = max(0, len(token_ids) - 1) // self.BLOCK_SIZE
        prev = seed_root_hex
        pids: List[int] = []
        staged: List[Tuple[int, Path]] = []
        for bi in range(n_full):
            cur = chain_merkle_prefix_hash(prev, token_ids[bi * self.BLOCK_SIZE:(bi + 1) * self.BLOCK_SIZE])
            pid = self.arena.lookup_page_id(cur)
            if pid is not None:
                pids.append(pid)
                self.blocks_loaded_from_arena += 1
                prev = cur
                continue
            found = self.bridge.kv_lookup(bytes.fromhex(cur))
            path = self._npz_path(cur)
            if (found or path.exists()) and path.exists():
                # the page is allocated now (same clock / LRU / free-list
                # order as a write per block); the block files are read in
                # parallel after the walk and written in one staged copy
                pid = self.arena.reserve_page(cur)
                staged.append((pid, path))
                pids.append(pid)
                self.blocks_loaded_from_disk += 1
                prev = cur
            else:
                break
        if staged:
            arrays = read_npz_many([path for _, path in staged])
            self.arena.write_loaded_pages([(pid, a) for (pid, _), a in zip(staged, arrays)])
        return pids

    def match_longest_prefix(self, token_ids: List[int], seed_root_hex: str
                             ) -> Tuple[int, Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Longest cached prefix as device tensors [L, 1, H, 16n, D] fp16."""
        pids = self._match_page_ids(token_ids, seed_root_hex)
        if not pids:
            return 0, None, None
        k, v = self.arena.gather_contiguous_kv(pids)
        n = len(pids) * self.BLOCK_SIZE
        self.tokens_skipped += n
        return n, k, v

    def match_longest_prefix_page_ids(self, token_ids: List[int], seed_root_hex: str) -> List[int]:
        """Matched page ids in prefix order (no gather): the block-table form
        of a prefix hit, for callers that attend over the pages in place."""
        pids = self._match_page_ids(token_ids, seed_root_hex)
        self.tokens_skipped += len(pids) * self.BLOCK_SIZE
        return pids

    def match_longest_prefix_numpy(self, token_ids: List[int], seed_root_hex: str
                                   ) -> Tuple[int, Optional[np.ndarray], Optional[np.ndarray]]:
        """native/native_engine.py:2248-2291."""
        n, k, v = self.match_longest_prefix(token_ids, seed_root_hex)
        if n == 0:
            return 0, None, None
        return n, k.cpu().numpy(), v.cpu().numpy()

    # ---------------------------------------------------------------- stats
    def get_paged_kv_stats(self) -> PagedKVStats:
        """native/native_engine.py:2415-2435."""
        with self.arena.lock:
            alloc = len(self.arena.page_table)
            free = len(self.arena.free_pages)
            return {
                "quant_mode": self.arena.quant_mode,
                "page_tokens": self.arena.PAGE_TOKENS,
                "max_pages": self.arena.max_pages,
                "allocated_pages": alloc,
                "free_pages": free,
                "bytes_per_page": self.arena.bytes_per_page,
                "arena_allocated_mb": round(self.arena.max_pages * self.arena.bytes_per_page / (1024.0 * 1024.0), 2),
                "arena_active_mb": round(alloc * self.arena.bytes_per_page / (1024.0 * 1024.0), 2),
                "page_hits": self.arena.page_hits,
                "page_misses": self.arena.page_misses,
                "page_evictions": self.arena.page_evictions,
                "kv_hash_evictions": int(getattr(self.bridge, "kv_evictions_issued", 0)),
                "disk_blocks_evicted": self.disk_blocks_evicted,
            }
