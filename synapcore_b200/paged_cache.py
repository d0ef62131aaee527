"""Per-sequence paged KV cache on one GPU: block tables over a KVPool.

This is the B200 form of the scheduler's per-request KV state. The reference
keeps one contiguous `[1, Hkv, T, D]` array per request and layer, grown by
`np.concatenate` on every token (models/adapters.py:1194-1207), and gives a
forked request an eager copy of a matched prefix (engine/scheduler.py:150-152).
Here every sequence owns a row of a device block table; pages come from the
pool's on-device allocator; a decode step reserves its new pages on the GPU
(`sckv_reserve_decode`) without a host round trip; a prefix shared by several
sequences is the same physical pages (pin count = number of holders), and a
fork copies only the partially filled last page (copy-on-write).

Rows are kept compact: live sequences occupy rows 0..n_live-1, so a decode
batch is a contiguous slice. Removing a sequence moves the last row into its
place. Host state is only the per-row token counts (deterministic, no device
reads on the decode path).
"""
from __future__ import annotations

from typing import Dict, Hashable, List, Optional, Sequence, Tuple

import torch

from . import _native as N
from .pool import KVPool, PAGE_TOKENS, to_device


def _ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


class PagedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_pages: int, max_seqs: int,
                 max_blocks_per_seq: int, kv_dtype: str = "fp16", device: Optional[torch.device] = None,
                 chunk_pages: int = 32, evict_watermark: Optional[float] = None):
        """evict_watermark: None keeps the arena's policy — pages released
        with keep_cached stay allocated and are taken back, least recently
        used first, only when an allocation finds the free ring empty
        (native/native_engine.py:324-331). A fraction f in (0, 1] adds the
        serving policy "evict at f full": enforce_watermark() evicts cached
        pages, LRU first, until at most f * max_pages are allocated."""
        if evict_watermark is not None and not 0.0 < float(evict_watermark) <= 1.0:
            raise ValueError("evict_watermark must be in (0, 1]")
        self.evict_watermark = None if evict_watermark is None else float(evict_watermark)
        self.pool = KVPool(num_layers, num_kv_heads, head_dim, max_pages, kv_dtype, device=device)
        self.device = self.pool.device
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.max_seqs, self.max_blocks = int(max_seqs), int(max_blocks_per_seq)
        # A fixed split size keeps every sequence's attention result independent
        # of which other sequences share the batch.
        self.chunk_pages = int(chunk_pages)
        self.block_table = torch.full((self.max_seqs, self.max_blocks), -1, dtype=torch.int32, device=self.device)
        self.ctx_lens = torch.zeros(self.max_seqs, dtype=torch.int32, device=self.device)
        self.lengths: List[int] = []           # tokens per live row
        self.row_of: Dict[Hashable, int] = {}  # sequence id -> row
        self.seq_at: List[Hashable] = []       # row -> sequence id
        self._arange = torch.arange(self.max_seqs + 1, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ rows
    @property
    def n_live(self) -> int:
        return len(self.seq_at)

    def add_sequence(self, seq_id: Hashable) -> int:
        if seq_id in self.row_of:
            raise KeyError(f"sequence {seq_id!r} already exists")
        if self.n_live >= self.max_seqs:
            raise RuntimeError("PagedKVCache: all sequence rows are in use")
        r = self.n_live
        self.row_of[seq_id] = r
        self.seq_at.append(seq_id)
        self.lengths.append(0)
        self.block_table[r].fill_(-1)
        self.ctx_lens[r] = 0
        return r

    def length(self, seq_id: Hashable) -> int:
        return self.lengths[self.row_of[seq_id]]

    def _pages_of(self, r: int) -> int:
        return _ceil_div(self.lengths[r], PAGE_TOKENS)

    def remove_sequence(self, seq_id: Hashable, keep_cached: bool = False) -> None:
        """Drop the sequence's pins on its pages (shared pages survive for their
        other holders) and compact the rows."""
        r = self.row_of.pop(seq_id)
        n = self._pages_of(r)
        if n:
            self.pool.release_pages(self.block_table[r, :n], keep_cached=keep_cached)
        last = self.n_live - 1
        if r != last:
            self.block_table[r].copy_(self.block_table[last])
            self.ctx_lens[r] = self.ctx_lens[last]
            moved = self.seq_at[last]
            self.seq_at[r] = moved
            self.lengths[r] = self.lengths[last]
            self.row_of[moved] = r
        self.seq_at.pop()
        self.lengths.pop()
        self.block_table[last].fill_(-1)
        self.ctx_lens[last] = 0

    def remove_sequences(self, seq_ids: Sequence[Hashable], keep_cached: bool = False) -> None:
        """remove_sequence for several sequences with one release launch (the
        pins of all their pages are dropped together, in the order given)."""
        seq_ids = list(seq_ids)
        if not seq_ids:
            return
        if len(set(seq_ids)) != len(seq_ids):
            raise ValueError("duplicate sequence ids")
        parts = []
        for sid in seq_ids:
            r = self.row_of[sid]
            n = self._pages_of(r)
            if n:
                parts.append(self.block_table[r, :n])
        if parts:
            self.pool.release_pages(torch.cat(parts), keep_cached=keep_cached)
        for sid in seq_ids:
            r = self.row_of[sid]
            self.lengths[r] = 0  # pages already released
            self.remove_sequence(sid)

    def move_to_row(self, seq_id: Hashable, row: int) -> None:
        """Swap two live rows (used to keep decode-phase sequences first)."""
        r = self.row_of[seq_id]
        if r == row:
            return
        other = self.seq_at[row]
        tmp_bt = self.block_table[row].clone()
        self.block_table[row].copy_(self.block_table[r])
        self.block_table[r].copy_(tmp_bt)
        tmp_len = self.ctx_lens[row].clone()
        self.ctx_lens[row] = self.ctx_lens[r]
        self.ctx_lens[r] = tmp_len
        self.seq_at[row], self.seq_at[r] = seq_id, other
        self.lengths[row], self.lengths[r] = self.lengths[r], self.lengths[row]
        self.row_of[seq_id], self.row_of[other] = row, r

    # ------------------------------------------------------------- eviction
    def enforce_watermark(self, out_count: Optional[torch.Tensor] = None) -> None:
        """With an evict_watermark, evict cached (unpinned) pages in LRU order
        until at most watermark * max_pages pages are allocated; decided on
        the device (one launch, no host read). Pages held by live sequences
        or a prefix index (pinned) are never evicted. No-op without one."""
        if self.evict_watermark is None:
            return
        limit = int(self.evict_watermark * self.pool.max_pages)
        self.pool.evict_to_watermark(limit, out_count=out_count)

    # -------------------------------------------------------------- prefill
    def _grow(self, r: int, n_new: int) -> None:
        """Allocate (pinned) pages so row r can hold n_new more tokens."""
        have = self._pages_of(r)
        need = _ceil_div(self.lengths[r] + n_new, PAGE_TOKENS)
        if need > self.max_blocks:
            raise ValueError(f"sequence would need {need} blocks > max_blocks_per_seq={self.max_blocks}")
        if need > have:
            ids, _ = self.pool.alloc_pages(need - have, pin=True)
            self.block_table[r, have:need].copy_(ids)

    def append_prefill(self, seq_id: Hashable, k: torch.Tensor, v: torch.Tensor, layer0: int = 0) -> None:
        """Append T tokens of one sequence: k, v [n_layers, T, Hkv, D] (or
        [T, Hkv, D] for one layer, layer0). Pages are reserved on the first
        layer written (layer0 == 0 or n_layers == all) and the length advances
        once the last layer is written."""
        if k.dim() == 3:
            k, v = k.unsqueeze(0), v.unsqueeze(0)
        r = self.row_of[seq_id]
        nl, T = k.shape[0], k.shape[1]
        if layer0 == 0:
            self._grow(r, T)
        cu = self._arange[:2].clone()
        cu[1] = T
        start = torch.full((1,), self.lengths[r], dtype=torch.int32, device=self.device)
        self.pool.append(k, v, cu, start, self.block_table[r:r + 1], layer0=layer0)
        if layer0 + nl == self.num_layers:
            self.lengths[r] += T
            self.ctx_lens[r] = self.lengths[r]

    def _consecutive_rows(self, seq_ids: Sequence[Hashable]) -> int:
        rows = [self.row_of[s] for s in seq_ids]
        r0 = rows[0]
        if rows != list(range(r0, r0 + len(rows))):
            raise ValueError("sequences must occupy consecutive rows in the given order "
                             "(sequences added one after another do)")
        return r0

    def _grow_rows(self, r0: int, n_new: Sequence[int]) -> None:
        """Pinned pages for rows r0.. so each can hold n_new[i] more tokens:
        one allocation launch and one block-table scatter for all rows."""
        rows, cols = [], []
        for i, t in enumerate(n_new):
            r = r0 + i
            have = self._pages_of(r)
            need = _ceil_div(self.lengths[r] + int(t), PAGE_TOKENS)
            if need > self.max_blocks:
                raise ValueError(f"sequence would need {need} blocks > max_blocks_per_seq={self.max_blocks}")
            rows.extend([r] * (need - have))
            cols.extend(range(have, need))
        if rows:
            ids, _ = self.pool.alloc_pages(len(rows), pin=True)
            idx = to_device([rows, cols], torch.int64, self.device)
            self.block_table[idx[0], idx[1]] = ids

    def append_prefill_batch(self, seq_ids: Sequence[Hashable], k: torch.Tensor, v: torch.Tensor,
                             cu_tokens: Sequence[int]) -> None:
        """Append several sequences' new tokens with one allocation and one
        append launch: sequence i gets rows cu_tokens[i]..cu_tokens[i+1]-1 of
        k, v [num_layers, total, Hkv, D]. The sequences must sit on
        consecutive rows (e.g. added one after another)."""
        seq_ids = list(seq_ids)
        n = len(seq_ids)
        cu = [int(c) for c in cu_tokens]
        if len(cu) != n + 1 or cu[0] != 0 or any(b < a for a, b in zip(cu, cu[1:])):
            raise ValueError("cu_tokens must be n+1 non-decreasing offsets from 0")
        if k.dim() != 4 or k.shape[0] != self.num_layers or k.shape[1] < cu[-1]:
            raise ValueError("k, v must be [num_layers, >= total tokens, Hkv, D]")
        r0 = self._consecutive_rows(seq_ids)
        T = [cu[i + 1] - cu[i] for i in range(n)]
        self._grow_rows(r0, T)
        meta = to_device(cu + [self.lengths[r0 + i] for i in range(n)], torch.int32, self.device)
        self.pool.append(k[:, :cu[-1]], v[:, :cu[-1]], meta[:n + 1], meta[n + 1:], self.block_table[r0:r0 + n],
                         layer0=0, max_blocks=self.max_blocks)
        for i in range(n):
            self.lengths[r0 + i] += T[i]
        self.ctx_lens[r0:r0 + n].copy_(to_device(self.lengths[r0:r0 + n], torch.int32, self.device))

    def begin_prefill_batch(self, seq_ids: Sequence[Hashable], n_new: Sequence[int],
                            shared: Optional[Sequence[Sequence[tuple]]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Set up the prompt pass of several new, empty sequences on
        consecutive rows (added one after another), to be run layer by layer
        with `append_layer_batch` + `prefill_attention_batch` and closed with
        `end_prefill_batch`.

        n_new[i]: tokens sequence i computes in this pass.
        shared[i] (optional): its leading full blocks, taken from elsewhere
        instead of computed, each ("page", page_id) — a page another holder
        keeps (a prefix index) — or ("row", j, b) — block b of the j-th
        sequence of this same batch (j < i), which this pass allocates and
        whose append runs before any attention reads it.

        One allocation launch covers every sequence's own pages; shared pages
        get one more pin per new holder. Returns the device int32 cu_tokens
        [n + 1] and start_pos [n] of the pass."""
        seq_ids = list(seq_ids)
        n = len(seq_ids)
        shared = [list(s) for s in shared] if shared is not None else [[] for _ in range(n)]
        if len(shared) != n or len(n_new) != n:
            raise ValueError("one n_new and one shared list per sequence")
        r0 = self._consecutive_rows(seq_ids)
        page_rc, page_ids, dst_rc, src_rc = [], [], [], []
        for i, blocks in enumerate(shared):
            r = r0 + i
            if self.lengths[r] != 0:
                raise ValueError("begin_prefill_batch needs empty sequences")
            for b, src in enumerate(blocks):
                if src[0] == "page":
                    page_rc.append((r, b))
                    page_ids.append(int(src[1]))
                elif src[0] == "row" and 0 <= int(src[1]) < i:
                    dst_rc.append((r, b))
                    src_rc.append((r0 + int(src[1]), int(src[2])))
                else:
                    raise ValueError(f"bad shared block source {src!r}")
            self.lengths[r] = len(blocks) * PAGE_TOKENS
        if page_ids:
            t = to_device([[r for r, _ in page_rc], [c for _, c in page_rc], page_ids], torch.int64, self.device)
            self.block_table[t[0], t[1]] = t[2].to(torch.int32)
        self._grow_rows(r0, [int(t) for t in n_new])
        if dst_rc:
            t = to_device([[r for r, _ in dst_rc], [c for _, c in dst_rc], [r for r, _ in src_rc],
                           [c for _, c in src_rc]], torch.int64, self.device)
            self.block_table[t[0], t[1]] = self.block_table[t[2], t[3]]
        held = page_rc + dst_rc
        if held:
            t = to_device([[r for r, _ in held], [c for _, c in held]], torch.int64, self.device)
            self.pool.pin_pages(self.block_table[t[0], t[1]], +1)
        cu = [0]
        for t in n_new:
            cu.append(cu[-1] + int(t))
        meta = to_device(cu + [self.lengths[r0 + i] for i in range(n)], torch.int32, self.device)
        return meta[:n + 1], meta[n + 1:]

    def append_layer_batch(self, layer: int, seq_ids: Sequence[Hashable], k: torch.Tensor, v: torch.Tensor,
                           cu_tokens: torch.Tensor, start_pos: torch.Tensor) -> None:
        """One layer's K/V of a pass set up by begin_prefill_batch:
        k, v [total, Hkv, D]."""
        r0 = self._consecutive_rows(seq_ids)
        n = len(seq_ids)
        self.pool.append(k, v, cu_tokens, start_pos, self.block_table[r0:r0 + n], layer0=layer,
                         max_blocks=self.max_blocks)

    def end_prefill_batch(self, seq_ids: Sequence[Hashable], n_new: Sequence[int]) -> None:
        """Advance the lengths once every layer of the pass has been written."""
        r0 = self._consecutive_rows(seq_ids)
        n = len(seq_ids)
        for i in range(n):
            self.lengths[r0 + i] += int(n_new[i])
        self.ctx_lens[r0:r0 + n].copy_(to_device(self.lengths[r0:r0 + n], torch.int32, self.device))

    def prefill_attention_batch(self, layer: int, seq_ids: Sequence[Hashable], q: torch.Tensor,
                                cu_q: torch.Tensor, start_pos: torch.Tensor, scale: Optional[float] = None,
                                out: Optional[torch.Tensor] = None,
                                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """Causal attention of several sequences' new tokens in one launch:
        q [total, Hq, D], rows cu_q[i]..cu_q[i+1]-1 of sequence i at positions
        start_pos[i]+t (device int32 tensors, appended already). Sequences on
        consecutive rows."""
        seq_ids = list(seq_ids)
        r0 = self._consecutive_rows(seq_ids)
        n = len(seq_ids)
        try:
            return self.pool.prefill_attn(layer, q, cu_q, start_pos, self.block_table[r0:r0 + n], scale=scale,
                                          out=out, out_dtype=out_dtype, max_blocks=self.max_blocks)
        except N.SCKVError as e:
            if e.code != N.SCKV_ERR_UNSUPPORTED:
                raise
        # pools / head groupings the tensor-core kernel does not build: one
        # sequence at a time through the decode kernel (reads the offsets back)
        cu = cu_q.tolist()
        st = start_pos.tolist()
        res = out if out is not None else torch.empty(q.shape, dtype=out_dtype or q.dtype, device=self.device)
        for i, sid in enumerate(seq_ids):
            if cu[i + 1] > cu[i]:
                res[cu[i]:cu[i + 1]] = self.prefill_attention(layer, sid, q[cu[i]:cu[i + 1]], st[i], scale=scale,
                                                              out_dtype=res.dtype)
        return res

    def prefill_attention(self, layer: int, seq_id: Hashable, q: torch.Tensor, start: int,
                          scale: Optional[float] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """Causal attention of T new query tokens at positions start..start+T-1
        (already appended) over the sequence's pages: token t sees positions
        <= start+t. q [T, Hq, D] -> [T, Hq, D]."""
        r = self.row_of[seq_id]
        T = q.shape[0]
        meta = to_device([0, T, start], torch.int32, self.device)
        cu, st = meta[:2], meta[2:]
        try:
            return self.pool.prefill_attn(layer, q, cu, st, self.block_table[r:r + 1], scale=scale,
                                          out_dtype=out_dtype, max_blocks=self.max_blocks)
        except N.SCKVError as e:
            if e.code != N.SCKV_ERR_UNSUPPORTED:
                raise
        # combinations the tensor-core prefill kernel does not build
        # (non-power-of-two groups, head_dim != 128): token t is a decode query of length
        # start+t+1 over the same row (block-table stride 0)
        bt = self.block_table[r:r + 1].expand(T, self.max_blocks)
        ctx = torch.arange(start + 1, start + T + 1, dtype=torch.int32, device=self.device)
        return self.pool.decode_attn(layer, q, bt, ctx, scale=scale, out_dtype=out_dtype,
                                     max_blocks=self.max_blocks, chunk_pages=self.chunk_pages)

    # --------------------------------------------------------------- decode
    def decode_reserve(self, n_rows: int) -> None:
        """One new token for rows 0..n_rows-1: pages for those crossing a page
        boundary are allocated on the device, lengths advance by one."""
        self.pool.reserve_decode(self.block_table, self.ctx_lens, n_seqs=n_rows, max_blocks=self.max_blocks)
        for r in range(n_rows):
            self.lengths[r] += 1

    def decode_append(self, layer: int, k: torch.Tensor, v: torch.Tensor, n_rows: int) -> None:
        """k, v [n_rows, Hkv, D]: the token reserved by decode_reserve."""
        start = self.ctx_lens[:n_rows] - 1
        self.pool.append(k, v, self._arange[:n_rows + 1], start, self.block_table[:n_rows], layer0=layer,
                         max_blocks=self.max_blocks)

    def decode_attention(self, layer: int, q: torch.Tensor, n_rows: int, scale: Optional[float] = None,
                         out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None
                         ) -> torch.Tensor:
        return self.pool.decode_attn(layer, q, self.block_table[:n_rows], self.ctx_lens[:n_rows], scale=scale,
                                     out=out, out_dtype=out_dtype, max_blocks=self.max_blocks,
                                     chunk_pages=self.chunk_pages)

    def decode_append_attention(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_rows: int,
                                scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                                out_dtype: Optional[torch.dtype] = None,
                                workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
        """decode_append then decode_attention for rows 0..n_rows-1; 16-bit
        pools do both in one launch (sckv_decode_attn_append)."""
        return self.pool.decode_attn_append(layer, q, k, v, self.block_table[:n_rows], self.ctx_lens[:n_rows],
                                            scale=scale, out=out, out_dtype=out_dtype, max_blocks=self.max_blocks,
                                            chunk_pages=self.chunk_pages, workspace=workspace)

    # ------------------------------------------------------ sharing / fork
    def share_prefix(self, seq_id: Hashable, page_ids: Sequence[int]) -> None:
        """Start an empty sequence with full prefix pages held elsewhere (a
        prefix-cache hit): its block table points at them and pins them."""
        r = self.row_of[seq_id]
        if self.lengths[r] != 0:
            raise ValueError("share_prefix needs an empty sequence")
        n = len(page_ids)
        if n == 0:
            return
        ids = to_device(list(page_ids), torch.int32, self.device)
        self.block_table[r, :n].copy_(ids)
        self.pool.pin_pages(ids, +1)
        self.lengths[r] = n * PAGE_TOKENS
        self.ctx_lens[r] = self.lengths[r]

    def fork(self, src_id: Hashable, dst_id: Hashable) -> int:
        """Copy-on-write fork: full pages are shared (pinned once more), the
        partially filled last page is copied to a fresh page."""
        rs = self.row_of[src_id]
        rd = self.add_sequence(dst_id)
        n_tok = self.lengths[rs]
        n_full = n_tok // PAGE_TOKENS
        if n_full:
            self.block_table[rd, :n_full].copy_(self.block_table[rs, :n_full])
            self.pool.pin_pages(self.block_table[rd, :n_full], +1)
        if n_tok % PAGE_TOKENS:
            ids, _ = self.pool.alloc_pages(1, pin=True)
            self.pool.copy_pages(self.block_table[rs, n_full:n_full + 1], ids)
            self.block_table[rd, n_full:n_full + 1].copy_(ids)
        self.lengths[rd] = n_tok
        self.ctx_lens[rd] = n_tok
        return rd

    def page_ids(self, seq_id: Hashable) -> List[int]:
        r = self.row_of[seq_id]
        return self.block_table[r, :self._pages_of(r)].tolist()

    # --------------------------------------------------------------- gather
    def gather(self, seq_id: Hashable, out_dtype: torch.dtype = torch.float16) -> Tuple[torch.Tensor, torch.Tensor]:
        """Contiguous [L, Hkv, T, D] K and V of one sequence (all layers)."""
        r = self.row_of[seq_id]
        n = self._pages_of(r)
        return self.pool.gather(self.block_table[r, :n], self.lengths[r], out_dtype=out_dtype)

    def check(self) -> None:
        """Raise if any kernel recorded an error in the device status word."""
        self.pool.raise_on_status()


class DecodeStepGraph:
    """One decode step of a `PagedKVCache` over rows 0..n_rows-1, captured
    once in a CUDA graph and replayed: page reservation on the device
    allocator, then for every layer the new token's K/V append and the
    decode attention (one launch plus the split combine for 16-bit pools,
    sckv_decode_attn_append; one-byte pools append first), all issued by
    one call.

    The step reads its inputs from static buffers `q` [L, n, Hq, D] and `k`,
    `v` [L, n, Hkv, D] and writes `out` [L, n, Hq, D]; fill them (copy or
    compute into them) before each `replay()`. Block tables and lengths are
    read on the device at replay time, so sequences joining, leaving or
    moving between rows keep the graph valid as long as rows 0..n_rows-1 are
    the decode batch; another batch size needs another graph.
    """

    def __init__(self, cache: PagedKVCache, n_rows: int, q_dtype: torch.dtype = torch.float16,
                 out_dtype: Optional[torch.dtype] = None, num_q_heads: Optional[int] = None,
                 scale: Optional[float] = None):
        if not 0 < n_rows <= cache.n_live:
            raise ValueError("n_rows must be between 1 and the number of live sequences")
        self.cache, self.n_rows = cache, int(n_rows)
        L, hkv, d = cache.num_layers, cache.num_kv_heads, cache.head_dim
        hq = hkv if num_q_heads is None else int(num_q_heads)
        src_dt = torch.bfloat16 if cache.pool.kv_dtype == "bf16" else torch.float16
        dev = cache.device
        self.q = torch.zeros((L, n_rows, hq, d), dtype=q_dtype, device=dev)
        self.k = torch.zeros((L, n_rows, hkv, d), dtype=src_dt, device=dev)
        self.v = torch.zeros((L, n_rows, hkv, d), dtype=src_dt, device=dev)
        self.out = torch.empty((L, n_rows, hq, d), dtype=out_dtype or q_dtype, device=dev)
        pool = cache.pool
        self._ws = torch.empty(max(16, pool.decode_workspace_bytes(n_rows, hq, cache.max_blocks, cache.chunk_pages)),
                               dtype=torch.uint8, device=dev)
        self._scale = scale
        # one eager attention (it only reads the pool) sets up the kernels'
        # launch attributes and tensor maps outside the capture
        pool.decode_attn(0, self.q[0], cache.block_table[:n_rows], cache.ctx_lens[:n_rows], scale=scale,
                         out=self.out[0], max_blocks=cache.max_blocks, chunk_pages=cache.chunk_pages,
                         workspace=self._ws)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()

    def _step(self) -> None:
        c, n = self.cache, self.n_rows
        pool = c.pool
        pool.reserve_decode(c.block_table, c.ctx_lens, n_seqs=n, max_blocks=c.max_blocks)
        for layer in range(c.num_layers):
            c.decode_append_attention(layer, self.q[layer], self.k[layer], self.v[layer], n, scale=self._scale,
                                      out=self.out[layer], workspace=self._ws)

    def replay(self) -> torch.Tensor:
        """Run the captured step on the current stream; returns `out`."""
        if self.cache.n_live < self.n_rows:
            raise RuntimeError("fewer live sequences than the captured batch")
        self.graph.replay()
        for r in range(self.n_rows):
            self.cache.lengths[r] += 1
        return self.out
