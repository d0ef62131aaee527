"""Continuous-batching scheduler over the paged GPU KV cache.

Request lifecycle and step semantics follow ContinuousBatchScheduler
(engine/scheduler.py:88-388): FIFO admission up to `max_batch_size`
(:132-135); a newly admitted request is prefilled — longest cached prefix
first, then the remaining prompt tokens — and emits its first token
(:137-189); requests prefilled in earlier steps decode one token each as one
batch (:311-380); a request finishes on a stop token or `max_new_tokens`.
The reference prefills a step's admitted requests one after another; here
they go out together (one launch per layer), with prefix matches decided in
the reference's order so the same tokens are skipped.

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
    unique_experts_loaded_across_layers: int
    naive_expert_calls_without_sharing: int
    expert_dedup_savings_pct: float
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
    entry drops its pin (the page is freed once no sequence holds it).
    `seed_root_hex` may be overridden per call (the reference scheduler seeds
    runs over fewer layers differently, engine/scheduler.py:139-143)."""

    def __init__(self, cache: PagedKVCache, seed_root_hex: str, max_entries: int = 1 << 20):
        self.cache = cache
        self.seed_root_hex = seed_root_hex
        self.max_entries = int(max_entries)
        self.pages: "collections.OrderedDict[str, int]" = collections.OrderedDict()
        self.hits = 0
        self.misses = 0
        self.tokens_skipped = 0

    def chain(self, token_ids: Sequence[int], seed_root_hex: Optional[str] = None) -> List[str]:
        """Chain hashes of the cacheable full blocks ((len - 1) // 16 of them)."""
        n_full = max(0, len(token_ids) - 1) // PAGE_TOKENS
        prev, out = seed_root_hex or self.seed_root_hex, []
        for b in range(n_full):
            prev = chain_hash(prev, token_ids[b * PAGE_TOKENS:(b + 1) * PAGE_TOKENS])
            out.append(prev)
        return out

    def get(self, h: str) -> Optional[int]:
        """Page of one chain hash (refreshes its LRU position), or None."""
        pid = self.pages.get(h)
        if pid is not None:
            self.pages.move_to_end(h)
        return pid

    def match(self, token_ids: Sequence[int], seed_root_hex: Optional[str] = None) -> List[int]:
        out = []
        for h in self.chain(token_ids, seed_root_hex):
            pid = self.get(h)
            if pid is None:
                self.misses += 1
                break
            self.hits += 1
            out.append(pid)
        self.tokens_skipped += len(out) * PAGE_TOKENS
        return out

    def register(self, token_ids: Sequence[int], page_ids: Sequence[int],
                 seed_root_hex: Optional[str] = None) -> int:
        """List the full prompt blocks of a prefilled sequence; returns how
        many new entries were added (each pins its page)."""
        return self.register_many([(token_ids, page_ids)], seed_root_hex)

    def register_many(self, items, seed_root_hex: Optional[str] = None) -> int:
        """register() for several (token_ids, page_ids) pairs with one pin launch."""
        new = []
        for token_ids, page_ids in items:
            hashes = self.chain(token_ids, seed_root_hex)[:len(page_ids)]
            for b, cur in enumerate(hashes):
                if cur in self.pages:
                    self.pages.move_to_end(cur)
                else:
                    self.pages[cur] = int(page_ids[b])
                    new.append(int(page_ids[b]))
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


def _is_engine(obj) -> bool:
    """A reference-style engine object (NativeMerkleMoEEngine's surface)."""
    return hasattr(obj, "core_np_views") and hasattr(obj, "emb_np_view")


class _EngineState:
    """What schedulers built on one engine share: the model adapter, the
    paged cache and the prefix index (the reference's schedulers share the
    engine's kv_prefix_cache the same way, engine/scheduler.py:145-179)."""

    def __init__(self, engine, max_seqs: int, max_context: int, max_pages: int, device, compute_dtype):
        from .engine_adapter import EngineModel

        self.model = EngineModel(engine, device, compute_dtype)
        m = self.model
        self.cache = PagedKVCache(m.num_layers, m.num_kv_heads, m.head_dim, max_pages, max_seqs,
                                  -(-int(max_context) // PAGE_TOKENS), "fp16", device=device)
        root = str(getattr(engine, "active_merkle_root", "00" * 32))
        self.index = PrefixPageIndex(self.cache, root) if getattr(engine, "enable_merkle_kv", True) else None


def _engine_state(engine, max_batch_size: int, max_context: int, max_pages: Optional[int], device,
                  compute_dtype) -> _EngineState:
    """The state shared by schedulers on `engine`, kept on the engine object
    itself so it lives exactly as long as the engine."""
    st = getattr(engine, "_sckv_paged_state", None)
    if st is not None and st.cache.max_seqs >= max_batch_size:
        return st
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    rows = max(64, int(max_batch_size))
    blocks = -(-int(max_context) // PAGE_TOKENS)
    if max_pages is None:
        from .engine_adapter import _attention_spec

        spec = _attention_spec(engine)
        page_bytes = 2 * int(engine.num_layers) * spec["num_kv_heads"] * PAGE_TOKENS * spec["head_dim"] * 2
        max_pages = max(256, min(rows * blocks, (8 << 30) // page_bytes))
    st = _EngineState(engine, rows, max_context, int(max_pages), dev, compute_dtype)
    setattr(engine, "_sckv_paged_state", st)
    return st


class ContinuousBatchScheduler:
    """FIFO admission, batched prefill of each step's admitted requests,
    batched paged decode.

    Two ways to build one:
      ContinuousBatchScheduler(model, cache, max_batch_size, prefix_index)
        — a `PagedDecoderModel` over a `PagedKVCache` you own;
      ContinuousBatchScheduler(engine, max_batch_size)
        — the reference's call (engine/scheduler.py:94-99): `engine` is a
        reference-style engine object (NativeMerkleMoEEngine's surface, see
        engine_adapter); the model adapter, a paged fp16 cache and a prefix
        index seeded from `engine.active_merkle_root` are created on first
        use (stored on the engine as `_sckv_paged_state`) and shared by every
        scheduler built on the same engine, as the reference's schedulers
        share the engine's prefix cache. Keyword options: max_context (tokens
        per sequence, default 4096), max_pages (default: at most 8 GiB of
        pages), device, compute_dtype (engine_adapter.EngineModel). In this
        mode `last_logits` are host numpy arrays, as in the reference.

    capture_decode=True replays each decode step from a CUDA graph, one per
    (batch size, layers), for models whose step is device work only (torch
    ops with no host reads; the reference-engine adapter routes experts on
    the host and cannot be captured). The first step at a batch size runs
    eagerly and is then captured; later ones copy their token ids and
    positions into the graph's inputs and replay it. Row moves and page
    reservation stay outside the graph."""

    def __init__(self, model, cache=None, max_batch_size: int = 8,
                 prefix_index: Optional[PrefixPageIndex] = None, eos_token_id: Optional[int] = None,
                 attn_scale: Optional[float] = None, *, max_context: int = 4096, max_pages: Optional[int] = None,
                 device=None, compute_dtype: torch.dtype = torch.float64, keep_finished_cached: bool = False,
                 capture_decode: bool = False):
        if isinstance(cache, int) and not isinstance(cache, bool):
            max_batch_size, cache = cache, None  # ContinuousBatchScheduler(engine, 4)
        self.engine = None
        if _is_engine(model):
            self.engine = model
            st = _engine_state(model, max_batch_size, max_context, max_pages, device, compute_dtype)
            model, cache = st.model, st.cache
            if prefix_index is None:
                prefix_index = st.index
            if eos_token_id is None:
                eos_token_id = int(dict(getattr(self.engine, "config", {}) or {}).get("eos_token_id", 50279))
            if attn_scale is None:
                attn_scale = st.model.attn_scale
        if cache is None:
            raise ValueError("a PagedKVCache is needed unless the first argument is an engine")
        self.model = model
        self.cache = cache
        self.max_batch_size = max(1, int(max_batch_size))
        self.prefix_index = prefix_index
        self.eos_token_id = 50279 if eos_token_id is None else int(eos_token_id)
        self.attn_scale = attn_scale
        # finished requests' pages: freed (the reference drops its per-request
        # arrays) or kept cached for LRU reuse under the cache's eviction policy
        self.keep_finished_cached = bool(keep_finished_cached)
        self.waiting_queue: Deque[BatchRequestState] = collections.deque()
        self.active_requests: Dict[str, BatchRequestState] = collections.OrderedDict()
        self.completed_requests: Dict[str, BatchRequestState] = collections.OrderedDict()
        self.step_counter = 0
        self.total_tokens_generated = 0
        self.max_concurrent = 0
        self.elapsed_ms = 0.0
        self.device = cache.device
        self._dispatch0 = self._dispatch_counts()
        if capture_decode and self.engine is not None:
            raise ValueError("capture_decode needs a model whose decode step is device work only")
        self.capture_decode = bool(capture_decode)
        # (batch size, layers) -> (graph, token ids, positions, logits, next ids)
        self._decode_graphs: Dict[tuple, tuple] = {}

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

    # --------------------------------------------------- expert counters
    def _dispatch_counts(self):
        return (int(getattr(self.model, "unique_expert_dispatches", 0)),
                int(getattr(self.model, "naive_expert_dispatches", 0)))

    @property
    def total_unique_expert_dispatches(self) -> int:
        """Unique experts loaded per layer and forward, summed (the reference's
        cross-request sharing counter, engine/scheduler.py:266-270); 0 for
        models without routed experts."""
        return self._dispatch_counts()[0] - self._dispatch0[0]

    @property
    def total_naive_expert_dispatches(self) -> int:
        return self._dispatch_counts()[1] - self._dispatch0[1]

    # ------------------------------------------------------------- forward
    def _n_layers(self, max_layers: Optional[int]) -> int:
        L = self.model.num_layers
        return L if max_layers is None else max(1, min(int(max_layers), L))

    def _seed_root(self, n_layers: int) -> Optional[str]:
        """engine/scheduler.py:139-143: runs over fewer layers than the model
        has key their blocks from a root that names the layer count."""
        if self.prefix_index is None:
            return None
        root = self.prefix_index.seed_root_hex
        return root if n_layers == self.model.num_layers else f"{root[:56]}{n_layers:08x}"

    def _layers(self, h: torch.Tensor, positions: torch.Tensor, attend, n_layers: int) -> torch.Tensor:
        for l in range(n_layers):
            q, k, v = self.model.attn_in(l, h, positions)
            attn = attend(l, q, k, v)
            h = self.model.attn_out(l, h, attn)
            h = self.model.mlp(l, h)
        return h

    def _emit(self, req: BatchRequestState, logits_row, tok: int) -> None:
        req.last_logits = logits_row
        req.generated_ids.append(tok)
        self.total_tokens_generated += 1
        if tok in req.stop_token_ids or len(req.generated_ids) >= req.max_new_tokens:
            req.is_finished = True

    def _prefill_batch(self, reqs: List[BatchRequestState], n_layers: int) -> List[int]:
        """Prompt passes of a step's admitted requests, one launch per layer
        for all of them. Prefix matching keeps the reference's order
        (engine/scheduler.py:145-179): request i may reuse the full blocks that
        requests before it in the same step will have cached, which here
        means sharing their pages, written by this same pass's append before
        any attention reads them."""
        cache, index = self.cache, self.prefix_index
        seed = self._seed_root(n_layers)
        ids = [req.request_id for req in reqs]
        for rid in ids:
            cache.add_sequence(rid)
        pending: Dict[str, tuple] = {}  # chain hash -> block source, for blocks this batch computes
        shared, chains, n_new = [], [], []
        for i, req in enumerate(reqs):
            hashes = index.chain(req.prompt_ids, seed) if index is not None else []
            src = []
            for h in hashes:
                pid = index.get(h)
                if pid is not None:
                    src.append(("page", pid))
                elif h in pending:
                    src.append(pending[h])
                else:
                    index.misses += 1
                    break
            if index is not None:
                index.hits += len(src)
                index.tokens_skipped += len(src) * PAGE_TOKENS
            for b in range(len(src), len(hashes)):
                if hashes[b] not in pending:
                    pending[hashes[b]] = ("row", i, b)
            req.kv_prefix_skipped = len(src) * PAGE_TOKENS
            shared.append(src)
            chains.append(hashes)
            n_new.append(len(req.prompt_ids) - req.kv_prefix_skipped)
        cu_d, st_d = cache.begin_prefill_batch(ids, n_new, shared)
        toks, pos = [], []
        for req, t in zip(reqs, n_new):
            m = req.kv_prefix_skipped
            toks.extend(req.prompt_ids[m:])
            pos.extend(range(m, m + t))
        meta = to_device([toks, pos], torch.int64, self.device)

        def attend(l, q, k, v):
            cache.append_layer_batch(l, ids, k, v, cu_d, st_d)
            return cache.prefill_attention_batch(l, ids, q, cu_d, st_d, scale=self.attn_scale,
                                                 out_dtype=torch.float32)

        h = self._layers(self.model.embed(meta[0]), meta[1], attend, n_layers)
        cache.end_prefill_batch(ids, n_new)
        last = to_device([sum(n_new[:i + 1]) - 1 for i in range(len(reqs))], torch.int64, self.device)
        logits = self.model.logits(h[last])
        # one device-to-host read: the first tokens and the new rows' page ids
        r0 = cache.row_of[ids[0]]
        nb = max(1, max(-(-len(req.prompt_ids) // PAGE_TOKENS) for req in reqs))
        host = torch.cat([torch.argmax(logits, dim=-1).to(torch.int32),
                          cache.block_table[r0:r0 + len(reqs), :nb].reshape(-1)]).cpu()
        toks_out = host[:len(reqs)].tolist()
        if index is not None:
            bt = host[len(reqs):].view(len(reqs), nb).tolist()
            index.register_many([(req.prompt_ids, bt[i][:len(chains[i])]) for i, req in enumerate(reqs)], seed)
        logits_host = logits.cpu().numpy() if self.engine is not None else None
        for i, req in enumerate(reqs):
            req.pos_offset = len(req.prompt_ids)
            req.prefill_done = True
            self._emit(req, logits_host[i] if logits_host is not None else logits[i], int(toks_out[i]))
        return toks_out

    def _decode(self, reqs: List[BatchRequestState], n_layers: int) -> List[int]:
        cache = self.cache
        B = len(reqs)
        for r, req in enumerate(reqs):
            cache.move_to_row(req.request_id, r)
        meta = to_device([[req.generated_ids[-1] for req in reqs], [req.pos_offset for req in reqs]], torch.int64,
                         self.device)
        cache.decode_reserve(B)

        def attend(l, q, k, v):
            return cache.decode_append_attention(l, q, k, v, B, scale=self.attn_scale, out_dtype=torch.float32)

        def step(ids, pos):
            logits = self.model.logits(self._layers(self.model.embed(ids), pos, attend, n_layers))
            return logits, torch.argmax(logits, dim=-1)

        key = (B, n_layers)
        g = self._decode_graphs.get(key) if self.capture_decode else None
        if g is not None:
            graph, ids_buf, pos_buf, logits, nxt = g
            ids_buf.copy_(meta[0])
            pos_buf.copy_(meta[1])
            graph.replay()
            logits = logits.clone()  # the graph's output buffer is rewritten by the next replay
        else:
            logits, nxt = step(meta[0], meta[1])
            if self.capture_decode:
                # this step ran eagerly (kernels and workspaces are set up);
                # capture the same step for the next ones at this batch size.
                # Nothing runs during capture.
                ids_buf, pos_buf = meta[0].clone(), meta[1].clone()
                torch.cuda.synchronize(self.device)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    g_logits, g_nxt = step(ids_buf, pos_buf)
                self._decode_graphs[key] = (graph, ids_buf, pos_buf, g_logits, g_nxt)
        out = nxt.tolist()
        logits_host = logits.cpu().numpy() if self.engine is not None else None
        for r, req in enumerate(reqs):
            req.pos_offset += 1
            self._emit(req, logits_host[r] if logits_host is not None else logits[r], int(out[r]))
        return out

    # --------------------------------------------------------------- steps
    def step_batch(self, max_layers: Optional[int] = None) -> Optional[BatchStepResult]:
        """engine/scheduler.py:311-380: admitted requests prefill (here as one
        batch), earlier ones decode one token each as one batch; `max_layers`
        runs only the first layers, as the reference's parameter does."""
        self._admit()
        if not self.active_requests:
            return None
        self.cache.enforce_watermark()
        n_layers = self._n_layers(max_layers)
        t0 = time.perf_counter()
        self.step_counter += 1
        d0 = self._dispatch_counts()
        emitted: Dict[str, int] = {}
        completed: List[str] = []
        active_ids = list(self.active_requests.keys())
        decode_reqs = [self.active_requests[i] for i in active_ids if self.active_requests[i].prefill_done]
        new_reqs = [self.active_requests[i] for i in active_ids if not self.active_requests[i].prefill_done]
        if new_reqs:
            toks = self._prefill_batch(new_reqs, n_layers)
            for req, tok in zip(new_reqs, toks):
                emitted[req.request_id] = int(tok)
                if req.is_finished:
                    completed.append(req.request_id)
        d1 = self._dispatch_counts()
        if decode_reqs:
            toks = self._decode(decode_reqs, n_layers)
            for req, tok in zip(decode_reqs, toks):
                emitted[req.request_id] = int(tok)
                if req.is_finished:
                    completed.append(req.request_id)
        d2 = self._dispatch_counts()
        done = [cid for cid in completed if cid in self.active_requests]
        if done:
            self.cache.remove_sequences(done, keep_cached=self.keep_finished_cached)
        for cid in done:
            self.completed_requests[cid] = self.active_requests.pop(cid)
        self.max_concurrent = max(self.max_concurrent, len(active_ids))
        ms = (time.perf_counter() - t0) * 1000.0
        self.elapsed_ms += ms
        uniq, naive = d2[0] - d1[0], d2[1] - d1[1]  # the decode batch's (engine/scheduler.py:361-366)
        del d0
        return {
            "step_idx": self.step_counter,
            "batch_size": len(active_ids),
            "active_request_ids": active_ids,
            "emitted_tokens": emitted,
            "completed_request_ids": completed,
            "decode_batch_size": len(decode_reqs),
            "unique_experts_loaded_across_layers": uniq,
            "naive_expert_calls_without_sharing": naive,
            "expert_dedup_savings_pct": round(100.0 * (1.0 - uniq / max(1, naive)), 2) if naive > 0 else 0.0,
            "step_latency_ms": round(ms, 3),
        }

    def run_until_complete(self, max_layers: Optional[int] = None) -> List[BatchStepResult]:
        steps = []
        while self.waiting_queue or self.active_requests:
            r = self.step_batch(max_layers=max_layers)
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


def benchmark_continuous_batch_scheduler(store_dir: object = None, num_requests: int = 4, max_new_tokens: int = 3,
                                         max_layers: int = 2, engine=None, device=None) -> Dict[str, object]:
    """engine/scheduler.py:391-481 over the paged GPU cache: the same prompts
    (a shared 16-token prefix + two tokens per request), run one request at a
    time with max_batch_size=1, then all together with max_batch_size =
    num_requests; generated tokens must be equal and the final logits'
    largest difference is reported. Returns the reference's metric keys.

    `engine`: a reference-style engine object. Without one, the host
    application's NativeMerkleMoEEngine is built from `store_dir` with the
    reference benchmark's arguments (this needs the reference package
    importable, as it is inside the application this replaces) and closed
    afterwards."""
    import numpy as np

    own = engine is None
    if own:
        from pathlib import Path

        from native.native_engine import NativeMerkleMoEEngine  # the host application's engine

        engine = NativeMerkleMoEEngine(Path(str(store_dir)), expert_cache_size=64, max_cache_ram_mb=768.0,
                                       on_demand_streaming=False, enable_lookahead=False, enable_merkle_kv=True,
                                       verify_merkle_on_load=False, device="cpu")
    try:
        shared_prefix = [1, 512, 1024, 2048, 4096, 8192, 12, 34, 56, 78, 90, 111, 222, 333, 444, 555]
        prompts = [shared_prefix + [100 + r, 200 + r] for r in range(num_requests)]
        t_seq0 = time.perf_counter()
        seq_tokens, seq_logits = {}, {}
        for r, p_ids in enumerate(prompts):
            rid = f"req_{r}"
            single = ContinuousBatchScheduler(engine, max_batch_size=1, device=device)
            single.submit_request(rid, p_ids, max_new_tokens=max_new_tokens, stop_token_ids=set())
            single.run_until_complete_numpy(max_layers=max_layers)
            done = single.completed_requests[rid]
            seq_tokens[rid] = list(done.generated_ids)
            seq_logits[rid] = np.asarray(done.last_logits, np.float32).copy()
        seq_ms = (time.perf_counter() - t_seq0) * 1000.0

        t_bat0 = time.perf_counter()
        batch = ContinuousBatchScheduler(engine, max_batch_size=num_requests, device=device)
        for r, p_ids in enumerate(prompts):
            batch.submit_request(f"req_{r}", p_ids, max_new_tokens=max_new_tokens, stop_token_ids=set())
        steps = batch.run_until_complete_numpy(max_layers=max_layers)
        torch.cuda.synchronize(batch.device)
        bat_ms = (time.perf_counter() - t_bat0) * 1000.0

        max_abs_err = 0.0
        for r in range(num_requests):
            rid = f"req_{r}"
            done_b = batch.completed_requests[rid]
            if done_b.generated_ids != seq_tokens[rid]:
                raise AssertionError(f"Token parity mismatch for {rid}: batched={done_b.generated_ids} "
                                     f"vs seq={seq_tokens[rid]}")
            diff = float(np.max(np.abs(np.asarray(done_b.last_logits, np.float32) - seq_logits[rid])))
            max_abs_err = max(max_abs_err, diff)
        uniq, naive = batch.total_unique_expert_dispatches, batch.total_naive_expert_dispatches
        total = batch.total_tokens_generated
        idx = batch.prefix_index
        return {
            "total_requests_completed": len(batch.completed_requests),
            "total_tokens_generated": total,
            "max_concurrent_batch_size": max((s["batch_size"] for s in steps), default=0),
            "total_batch_steps": len(steps),
            "total_unique_expert_dispatches": uniq,
            "total_naive_expert_dispatches": naive,
            "cross_request_expert_sharing_pct": round(100.0 * (1.0 - uniq / max(1, naive)), 2) if naive else 0.0,
            "paged_kv_pages_allocated": batch.cache.pool.alloc_state()["allocated"],
            "paged_kv_prefix_tokens_skipped": idx.tokens_skipped if idx is not None else 0,
            "batched_total_ms": round(bat_ms, 3),
            "sequential_total_ms": round(seq_ms, 3),
            "throughput_tok_per_s": round(1000.0 * total / max(1e-3, bat_ms), 2),
            "numerical_parity_max_abs_err": round(max_abs_err, 8),
        }
    finally:
        if own:
            engine.close()
