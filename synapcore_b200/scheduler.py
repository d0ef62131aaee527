"""Continuous-batching scheduler over the paged GPU KV cache.

Request lifecycle and step semantics follow ContinuousBatchScheduler
(engine/scheduler.py:88-388): FIFO admission up to `max_batch_size`
(:132-135); a newly admitted request is prefilled on its own — longest cached
prefix first, then the remaining prompt tokens — and emits its first token
(:137-189); requests prefilled in earlier steps decode one token each as one
batch (:311-380); a request finishes on a stop token or `max_new_tokens`.

What changes is the KV side. The reference keeps per-request contiguous
arrays, copies a matched prefix into them (:150-152) and runs attention
request by request (:229-244). Here every request is a row of a
`PagedKVCache`: a prefix hit shares the cached pages in place (pins, no
copy), new tokens are scattered into pages by the append kernel, and each
layer's decode attention is one launch for the whole batch over the block
tables, with the decode step's new pages reserved on the device.

Everything outside attention (embeddings, projections, norms, MLP / MoE,
LM head) belongs to the model, supplied through `PagedDecoderModel`.
"""
from __future__ import annotations

import collections
import hashlib
import struct
import time
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Protocol, Sequence, Set, TypedDict

import torch

from .paged_cache import PAGE_TOKENS, PagedKVCache
from .pool import to_device


class PagedDecoderModel(Protocol):
    """The model around attention. Tensors live on the cache's device."""

    num_layers: int

    def embed(self, token_ids: torch.Tensor) -> torch.Tensor:
        """[T] int64 -> hidden states [T, hidden]."""

    def attn_in(self, layer: int, h: torch.Tensor, positions: torch.Tensor):
        """Hidden states -> (q [T, Hq, D], k [T, Hkv, D], v [T, Hkv, D]) for
        tokens at `positions` (norm, projections, RoPE)."""

    def attn_out(self, layer: int, h: torch.Tensor, attn: torch.Tensor) -> torch.Tensor:
        """Residual update from the attention output attn [T, Hq, D]."""

    def mlp(self, layer: int, h: torch.Tensor) -> torch.Tensor:
        """The rest of the layer (post-attention norm, MLP / MoE, residual)."""

    def logits(self, h_last: torch.Tensor) -> torch.Tensor:
        """[B, hidden] -> [B, vocab]."""


class BatchStepResult(TypedDict):
    step_idx: int
    batch_size: int
    active_request_ids: List[str]
    emitted_tokens: Dict[str, int]
    completed_request_ids: List[str]
    decode_batch_size: int
    step_latency_ms: float


class BatchSchedulerMetrics(TypedDict):
    total_requests_completed: int
    total_tokens_generated: int
    max_concurrent_batch_size: int
    total_batch_steps: int
    paged_kv_pages_allocated: int
    paged_kv_prefix_tokens_skipped: int
    batched_total_ms: float
    throughput_tok_per_s: float


@dataclass
class BatchRequestState:
    """Per-request state (engine/scheduler.py:67-85); the KV lives in the cache."""

    request_id: str
    prompt_ids: List[int]
    max_new_tokens: int
    stop_token_ids: Set[int] = field(default_factory=lambda: {0, 50278, 50279})
    generated_ids: List[int] = field(default_factory=list)
    pos_offset: int = 0
    prefill_done: bool = False
    is_finished: bool = False
    kv_prefix_skipped: int = 0
    last_logits: Optional[torch.Tensor] = None


def chain_hash(prev_hex: str, block: Sequence[int]) -> str:
    """sha256(prev hash bytes || u32le tokens) (native/native_engine.py:778-782)."""
    h = hashlib.sha256()
    h.update(bytes.fromhex(prev_hex))
    h.update(struct.pack(f"<{len(block)}I", *[int(t) for t in block]))
    return h.digest().hex()


class PrefixPageIndex:
    """Prefix-chain hash -> page id for pages of the paged cache.

    Same keys and matching rule as NativeKVPrefixCache (16-token blocks
    chained from a seed root, the last prompt token never cached,
    native/native_engine.py:2202-2291), but a hit is the physical page itself:
    the index holds one pin on every page it lists, and a sequence that reuses
    a prefix pins the same pages. Beyond `max_entries` the least recently used
    entry drops its pin (the page is freed once no sequence holds it)."""

    def __init__(self, cache: PagedKVCache, seed_root_hex: str, max_entries: int = 1 << 20):
        self.cache = cache
        self.seed_root_hex = seed_root_hex
        self.max_entries = int(max_entries)
        self.pages: "collections.OrderedDict[str, int]" = collections.OrderedDict()
        self.hits = 0
        self.misses = 0
        self.tokens_skipped = 0

    def match(self, token_ids: Sequence[int]) -> List[int]:
        n_full = max(0, len(token_ids) - 1) // PAGE_TOKENS
        prev, out = self.seed_root_hex, []
        for b in range(n_full):
            cur = chain_hash(prev, token_ids[b * PAGE_TOKENS:(b + 1) * PAGE_TOKENS])
            pid = self.pages.get(cur)
            if pid is None:
                self.misses += 1
                break
            self.pages.move_to_end(cur)
            self.hits += 1
            out.append(pid)
            prev = cur
        self.tokens_skipped += len(out) * PAGE_TOKENS
        return out

    def register(self, token_ids: Sequence[int], page_ids: Sequence[int]) -> int:
        """List the full prompt blocks of a prefilled sequence; returns how
        many new entries were added (each pins its page)."""
        n_full = min(max(0, len(token_ids) - 1) // PAGE_TOKENS, len(page_ids))
        prev, new = self.seed_root_hex, []
        for b in range(n_full):
            cur = chain_hash(prev, token_ids[b * PAGE_TOKENS:(b + 1) * PAGE_TOKENS])
            if cur in self.pages:
                self.pages.move_to_end(cur)
            else:
                self.pages[cur] = int(page_ids[b])
                new.append(int(page_ids[b]))
            prev = cur
        if new:
            self.cache.pool.pin_pages(torch.tensor(new, dtype=torch.int32), +1)
        self._trim()
        return len(new)

    def _trim(self) -> None:
        drop = []
        while len(self.pages) > self.max_entries:
            _, pid = self.pages.popitem(last=False)
            drop.append(pid)
        if drop:
            self.cache.pool.release_pages(torch.tensor(drop, dtype=torch.int32))

    def evict(self, n: int) -> int:
        """Drop the n least recently used entries."""
        drop = []
        while self.pages and len(drop) < n:
            _, pid = self.pages.popitem(last=False)
            drop.append(pid)
        if drop:
            self.cache.pool.release_pages(torch.tensor(drop, dtype=torch.int32))
        return len(drop)


class ContinuousBatchScheduler:
    """FIFO admission, per-request prefill, batched paged decode."""

    def __init__(self, model: PagedDecoderModel, cache: PagedKVCache, max_batch_size: int = 8,
                 prefix_index: Optional[PrefixPageIndex] = None, eos_token_id: int = 50279,
                 attn_scale: Optional[float] = None):
        self.model = model
        self.cache = cache
        self.max_batch_size = max(1, int(max_batch_size))
        self.prefix_index = prefix_index
        self.eos_token_id = int(eos_token_id)
        self.attn_scale = attn_scale
        self.waiting_queue: Deque[BatchRequestState] = collections.deque()
        self.active_requests: Dict[str, BatchRequestState] = collections.OrderedDict()
        self.completed_requests: Dict[str, BatchRequestState] = collections.OrderedDict()
        self.step_counter = 0
        self.total_tokens_generated = 0
        self.max_concurrent = 0
        self.elapsed_ms = 0.0
        self.device = cache.device

    # ----------------------------------------------------------- requests
    def submit_request(self, request_id: str, prompt_ids: List[int], max_new_tokens: int = 16,
                       stop_token_ids: Optional[Set[int]] = None) -> BatchRequestState:
        """engine/scheduler.py:110-128."""
        if not prompt_ids:
            raise ValueError(f"Request {request_id!r} must have at least 1 prompt token")
        stops = stop_token_ids if stop_token_ids is not None else {self.eos_token_id, 0, 50278}
        st = BatchRequestState(request_id=str(request_id), prompt_ids=list(prompt_ids),
                               max_new_tokens=max(1, int(max_new_tokens)), stop_token_ids=stops)
        self.waiting_queue.append(st)
        return st

    def _admit(self) -> None:
        while self.waiting_queue and len(self.active_requests) < self.max_batch_size:
            req = self.waiting_queue.popleft()
            self.active_requests[req.request_id] = req

    # ------------------------------------------------------------- forward
    def _layers(self, h: torch.Tensor, positions: torch.Tensor, attend) -> torch.Tensor:
        for l in range(self.model.num_layers):
            q, k, v = self.model.attn_in(l, h, positions)
            attn = attend(l, q, k, v)
            h = self.model.attn_out(l, h, attn)
            h = self.model.mlp(l, h)
        return h

    def _emit(self, req: BatchRequestState, logits_row: torch.Tensor, tok: int) -> None:
        req.last_logits = logits_row
        req.generated_ids.append(tok)
        self.total_tokens_generated += 1
        if tok in req.stop_token_ids or len(req.generated_ids) >= req.max_new_tokens:
            req.is_finished = True

    def _prefill(self, req: BatchRequestState) -> int:
        cache = self.cache
        rid = req.request_id
        cache.add_sequence(rid)
        matched = 0
        if self.prefix_index is not None:
            pages = self.prefix_index.match(req.prompt_ids)
            if pages:
                cache.share_prefix(rid, pages)
                matched = len(pages) * PAGE_TOKENS
                req.kv_prefix_skipped = matched
        rem = req.prompt_ids[matched:]
        toks = to_device(rem, torch.int64, self.device)
        positions = torch.arange(matched, matched + len(rem), dtype=torch.int64, device=self.device)

        def attend(l, q, k, v):
            cache.append_prefill(rid, k, v, layer0=l)
            return cache.prefill_attention(l, rid, q, matched, scale=self.attn_scale, out_dtype=torch.float32)

        h = self._layers(self.model.embed(toks), positions, attend)
        logits = self.model.logits(h[-1:])
        tok = int(torch.argmax(logits[0]).item())
        if self.prefix_index is not None:
            self.prefix_index.register(req.prompt_ids, cache.page_ids(rid))
        req.pos_offset = len(req.prompt_ids)
        req.prefill_done = True
        self._emit(req, logits[0], tok)
        return tok

    def _decode(self, reqs: List[BatchRequestState]) -> List[int]:
        cache = self.cache
        B = len(reqs)
        for r, req in enumerate(reqs):
            cache.move_to_row(req.request_id, r)
        toks = to_device([req.generated_ids[-1] for req in reqs], torch.int64, self.device)
        positions = to_device([req.pos_offset for req in reqs], torch.int64, self.device)
        cache.decode_reserve(B)

        def attend(l, q, k, v):
            cache.decode_append(l, k, v, B)
            return cache.decode_attention(l, q, B, scale=self.attn_scale, out_dtype=torch.float32)

        h = self._layers(self.model.embed(toks), positions, attend)
        logits = self.model.logits(h)
        out = torch.argmax(logits, dim=-1).tolist()
        for r, req in enumerate(reqs):
            req.pos_offset += 1
            self._emit(req, logits[r], int(out[r]))
        return out

    # --------------------------------------------------------------- steps
    def step_batch(self) -> Optional[BatchStepResult]:
        """engine/scheduler.py:311-380, with the decode batch in one launch per layer."""
        self._admit()
        if not self.active_requests:
            return None
        t0 = time.perf_counter()
        self.step_counter += 1
        emitted: Dict[str, int] = {}
        completed: List[str] = []
        active_ids = list(self.active_requests.keys())
        decode_reqs = [self.active_requests[i] for i in active_ids if self.active_requests[i].prefill_done]
        new_reqs = [self.active_requests[i] for i in active_ids if not self.active_requests[i].prefill_done]
        for req in new_reqs:
            emitted[req.request_id] = self._prefill(req)
            if req.is_finished:
                completed.append(req.request_id)
        if decode_reqs:
            toks = self._decode(decode_reqs)
            for req, tok in zip(decode_reqs, toks):
                emitted[req.request_id] = int(tok)
                if req.is_finished:
                    completed.append(req.request_id)
        for cid in completed:
            done = self.active_requests.pop(cid, None)
            if done is not None:
                self.cache.remove_sequence(cid)
                self.completed_requests[cid] = done
        self.max_concurrent = max(self.max_concurrent, len(active_ids))
        ms = (time.perf_counter() - t0) * 1000.0
        self.elapsed_ms += ms
        return {
            "step_idx": self.step_counter,
            "batch_size": len(active_ids),
            "active_request_ids": active_ids,
            "emitted_tokens": emitted,
            "completed_request_ids": completed,
            "decode_batch_size": len(decode_reqs),
            "step_latency_ms": round(ms, 3),
        }

    def run_until_complete(self) -> List[BatchStepResult]:
        steps = []
        while self.waiting_queue or self.active_requests:
            r = self.step_batch()
            if r is not None:
                steps.append(r)
        return steps

    # reference-compatible names (engine/scheduler.py:311, 382)
    step_batch_numpy = step_batch
    run_until_complete_numpy = run_until_complete

    def metrics(self) -> BatchSchedulerMetrics:
        st = self.cache.pool.alloc_state()
        return {
            "total_requests_completed": len(self.completed_requests),
            "total_tokens_generated": self.total_tokens_generated,
            "max_concurrent_batch_size": self.max_concurrent,
            "total_batch_steps": self.step_counter,
            "paged_kv_pages_allocated": st["allocated"],
            "paged_kv_prefix_tokens_skipped": self.prefix_index.tokens_skipped if self.prefix_index else 0,
            "batched_total_ms": round(self.elapsed_ms, 3),
            "throughput_tok_per_s": round(1000.0 * self.total_tokens_generated / max(1e-3, self.elapsed_ms), 2),
        }
