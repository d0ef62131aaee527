"""Multi-GPU layouts for the paged KV path (one process per GPU).

Sequence sharding (the default): sequences are dealt round-robin by id, each
rank owns its own pool, allocator and block tables, and decode attention
needs no communication — the aggregate is just the sum over ranks.

KV-head sharding (optional): every rank holds all sequences but only kv heads
[r*Hkv/n, (r+1)*Hkv/n) and the query heads that read them; after each
layer's attention every rank needs the full [B, Hq, D] output. Two ways:
`HeadShardedExchange` (the default in bench.py) has the decode kernel's
epilogue store every output element straight into every rank's full-head
buffer over NVLink (CUDA IPC mappings, plain stores) and flag the layer done
on every rank, so there is no separate collective; `HeadShardedOutput` is the
NCCL all-gather of the per-rank [B, Hq/n, D] outputs into a local buffer.
Neither reads another GPU's memory with TMA or multicast.

The reference has no multi-process code; these layouts are the B200 side's
way of scaling one box (8 GPUs).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch


def shard_of(seq_id: int, world: int) -> int:
    """Rank that owns sequence `seq_id` under round-robin sequence sharding."""
    return int(seq_id) % int(world)


def shard_sequences(seq_ids: Sequence[int], world: int, rank: int) -> List[int]:
    """The sequences rank `rank` owns, in their original order."""
    return [s for s in seq_ids if shard_of(s, world) == rank]


def head_range(num_kv_heads: int, world: int, rank: int) -> range:
    """kv heads owned by `rank` in KV-head-sharded mode (contiguous, equal)."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} kv heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return range(rank * per, (rank + 1) * per)


def query_head_range(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> range:
    """Query heads that read the kv heads of `rank` (q head h reads kv head h // G)."""
    g = num_q_heads // num_kv_heads
    kv = head_range(num_kv_heads, world, rank)
    return range(kv.start * g, kv.stop * g)


class HeadShardedOutput:
    """All-gather of per-rank attention outputs in KV-head-sharded mode.

    `gather(local)` takes this rank's [B, Hq/n, D] output and returns the full
    [B, Hq, D] in head order, using all_gather_into_tensor into a
    preallocated buffer (rank-major [n, B, Hq/n, D], then a local transpose)."""

    def __init__(self, world: int, group: Optional["torch.distributed.ProcessGroup"] = None):
        self.world = int(world)
        self.group = group
        self._buf: Optional[torch.Tensor] = None

    def gather(self, local: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        local = local.contiguous()
        B, hq_local, D = local.shape
        shape = (self.world * B, hq_local, D)  # rank-major
        if self._buf is None or tuple(self._buf.shape) != shape or self._buf.dtype != local.dtype \
                or self._buf.device != local.device:
            self._buf = torch.empty(shape, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(self._buf, local, group=self.group)
        return self._buf.view(self.world, B, hq_local, D).permute(1, 0, 2, 3).reshape(B, self.world * hq_local, D)


class HeadShardedExchange:
    """KV-head-sharded decode whose output exchange is fused into the kernel.

    Every rank owns an exchange buffer [layers, max_seqs, Hq, D] (out_dtype)
    in its own memory; the ranks swap CUDA IPC handles once through `group`
    and map each other's buffers. `decode(layer, q_local, ...)` runs this
    rank's heads with sckv_decode_attn_exchange, which writes the rank's
    slice of every output row into every rank's buffer and then raises this
    rank's flag for the call's epoch on every rank; `wait(epoch)` queues a
    bounded device wait for all ranks' flags, after which `output(layer, B)`
    holds the full [B, Hq, D] result. Epochs grow by one per call and are
    identical on all ranks: pass them explicitly, or pass 0 to both calls to
    let each rank's device counter supply them (then a whole step can be
    captured in a CUDA graph and replayed). `k_new` / `v_new` [B, Hkv/world,
    D] append the step's new token in the same launch (16-bit pools). A
    layer's slice is rewritten in the next step as soon as the writer has
    waited for every rank's signal of the following layer, so each rank must
    read layer l's output before it signals layer l + 1 (a model's next
    layer consumes it anyway); a caller that reads only after a whole step
    (e.g. a replayed graph with no consumer inside) holds the other ranks at
    a barrier until it has read."""

    def __init__(self, pool, world: int, rank: int, layers: int, max_seqs: int, num_q_heads_total: int,
                 out_dtype: torch.dtype = torch.float32, group: Optional["torch.distributed.ProcessGroup"] = None):
        import ctypes

        import torch.distributed as dist

        from . import _native as N
        from .pool import torch_dtype_code

        self.N, self.lib, self.pool = N, N.lib(), pool
        self.world, self.rank = int(world), int(rank)
        self.layers, self.max_seqs, self.hq_total = int(layers), int(max_seqs), int(num_q_heads_total)
        if self.hq_total % self.world:
            raise ValueError("query heads must split evenly over the ranks")
        self.out_dtype = out_dtype
        self.code = torch_dtype_code(out_dtype)
        self.esize = torch.empty((), dtype=out_dtype).element_size()
        self.slice_elems = self.max_seqs * self.hq_total * pool.head_dim
        h = ctypes.c_void_p()
        N.check(self.lib.sckv_exchange_create(pool.device.index, self.world, self.rank,
                                              self.layers * self.slice_elems * self.esize, ctypes.byref(h)),
                "sckv_exchange_create")
        self.handle = h
        mine = (ctypes.c_uint8 * 128)()
        N.check(self.lib.sckv_exchange_ipc_handles(self.handle, mine), "sckv_exchange_ipc_handles")
        allh = [None] * self.world
        dist.all_gather_object(allh, bytes(mine), group=group)
        for r, hb in enumerate(allh):
            if r != self.rank:
                buf = (ctypes.c_uint8 * 128).from_buffer_copy(hb)
                N.check(self.lib.sckv_exchange_open_peer(self.handle, r, buf), "sckv_exchange_open_peer")
        ptr = int(self.lib.sckv_exchange_buffer(self.handle))
        self._view = _device_view(ptr, self.layers * self.slice_elems, out_dtype, pool.device)
        self._ws: Optional[torch.Tensor] = None

    def decode(self, layer: int, q: torch.Tensor, block_table: torch.Tensor, ctx_lens: torch.Tensor, epoch: int = 0,
               phys_layer: Optional[int] = None, scale: Optional[float] = None, chunk_pages: int = 0,
               k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None) -> None:
        from .pool import _stream_ptr, torch_dtype_code

        q = q.contiguous()
        B, hq, d = q.shape
        if B > self.max_seqs or hq * self.world != self.hq_total:
            raise ValueError("q must be [<= max_seqs, Hq / world, D]")
        k_ptr = v_ptr = None
        src_code = 0
        if (k_new is None) != (v_new is None):
            raise ValueError("pass both k_new and v_new, or neither")
        if k_new is not None:
            k_new, v_new = k_new.contiguous(), v_new.contiguous()
            if tuple(k_new.shape) != (B, self.pool.num_kv_heads, d) or k_new.shape != v_new.shape:
                raise ValueError(f"k_new/v_new must be [B, {self.pool.num_kv_heads}, {d}]")
            if k_new.dtype != v_new.dtype:
                raise TypeError("k_new and v_new must have the same dtype")
            k_ptr, v_ptr, src_code = k_new.data_ptr(), v_new.data_ptr(), torch_dtype_code(k_new.dtype)
        mb = block_table.shape[1]
        need = self.pool.decode_workspace_bytes(B, hq, mb, chunk_pages)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 16), dtype=torch.uint8, device=self.pool.device)
        scale = float(d) ** -0.5 if scale is None else float(scale)
        pl = layer if phys_layer is None else phys_layer
        self.N.check(self.lib.sckv_decode_attn_exchange(
            self.pool.handle, self.handle, pl, q.data_ptr(), torch_dtype_code(q.dtype), hq, k_ptr, v_ptr, src_code,
            block_table.data_ptr(), block_table.stride(0), mb, ctx_lens.data_ptr(), B, scale, self.code,
            layer * self.slice_elems, self.hq_total, int(epoch), self._ws.data_ptr(), self._ws.numel(), chunk_pages,
            _stream_ptr(stream)), "sckv_decode_attn_exchange")

    def wait(self, epoch: int = 0, limit_us: int = 0, stream: Optional[torch.cuda.Stream] = None) -> None:
        from .pool import _stream_ptr

        self.N.check(self.lib.sckv_exchange_wait(self.handle, int(epoch), int(limit_us), _stream_ptr(stream)),
                     "sckv_exchange_wait")

    def output(self, layer: int, n_seqs: int) -> torch.Tensor:
        """The full [n_seqs, Hq, D] output of `layer` (valid after wait)."""
        d = self.pool.head_dim
        base = layer * self.slice_elems
        return self._view[base: base + n_seqs * self.hq_total * d].view(n_seqs, self.hq_total, d)

    def status(self, clear: bool = False):
        import ctypes

        arr = (ctypes.c_int32 * 4)()
        self.N.check(self.lib.sckv_exchange_status(self.handle, arr, 1 if clear else 0, None), "sckv_exchange_status")
        return tuple(int(x) for x in arr)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            self.lib.sckv_exchange_destroy(self.handle)
            self.handle = None


def _device_view(ptr: int, numel: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A tensor over device memory the library owns (no copy, no ownership)."""
    esize = torch.empty((), dtype=dtype).element_size()

    class _Mem:
        __cuda_array_interface__ = {
            "shape": (numel * esize,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None,
        }

    return torch.as_tensor(_Mem(), device=device).view(dtype)
