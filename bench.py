#!/usr/bin/env python3
"""Paged decode-attention benchmark (B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (synthetic, seeded):
  olmoe       16 layers x 16 KV heads (MHA), head_dim 128, fp16, 16-token pages,
              64 sequences x context 4096 per GPU, one query token per
              sequence, block tables a random permutation of a pool of 18,750
              all-layer pages (= 300,000 layer-pages of 128 KiB).
  qwen3-fp8   36 layers, 32 query / 8 KV heads, head_dim 128, FP8-e4m3 KV with
              per-page fp32 scales, bf16 queries, 128 sequences x context 16384.
  qwen3-long  36 layers, 32 / 8 heads, bf16 KV and queries, 64 sequences per
              GPU with contexts ~U[8192, 32768] that grow by one token per
              step; 100 GB of physical layers per GPU, logical layer l reads
              physical layer l mod Lp (the full KV of 512 such sequences,
              ~1.55 TB, exceeds the box).
  *-small     profiling-sized variants (2 layers, a few hundred MB).

A step = for every layer: append one new K/V token per sequence (scatter
through the block table), then paged decode attention for every sequence.
Fixed-context workloads keep the context (the new token rewrites slot
ctx-1); growing ones append at slot ctx and attend over ctx+1 tokens.

One JSON line on rank 0. `value` = KV GB/s over all ranks (algorithmic bytes
of attention + append per step / step time, inputs resident in HBM). `e2e`
= the same metric through the pool's public calls with inputs copied from
pinned host memory each step and outputs read back. `roofline` = the decode
attention op's algorithmic bytes per launch / its average CUDA-event time.
Under torchrun each rank owns its own pool and sequences (sequence sharding,
no collective on the data path; weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

if "--impl" in sys.argv and "reference" in sys.argv:
    _n = str(os.cpu_count() or 1)
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ.setdefault(_v, _n)

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PAGE = 16
WORKLOADS = {
    "olmoe": dict(model="OLMoE-1B-7B attention", layers=16, hq=16, hkv=16, d=128, kv="fp16", qdt=torch.float16,
                  batch=64, ctx=4096, pool_pages=18750),
    "qwen3-fp8": dict(model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128, kv="fp8_e4m3",
                      qdt=torch.bfloat16, batch=128, ctx=16384, pool_pages=128 * 1024 + 512),
    # profiling-sized variants: same per-launch structure, 2 layers, a few hundred MB
    "olmoe-small": dict(model="OLMoE-1B-7B attention", layers=2, hq=16, hkv=16, d=128, kv="fp16",
                        qdt=torch.float16, batch=8, ctx=4096, pool_pages=2200),
    "qwen3-fp8-small": dict(model="Qwen3-8B attention", layers=2, hq=32, hkv=8, d=128, kv="fp8_e4m3",
                            qdt=torch.bfloat16, batch=16, ctx=16384, pool_pages=16 * 1024 + 64),
    # the OLMoE decode (16 layers, 64 x 4,096 tokens) with the reference
    # arena's int8 mode, and with FP8 pages
    "olmoe-int8": dict(model="OLMoE-1B-7B attention", layers=16, hq=16, hkv=16, d=128, kv="int8",
                       qdt=torch.float16, batch=64, ctx=4096, pool_pages=18750),
    "olmoe-fp8": dict(model="OLMoE-1B-7B attention", layers=16, hq=16, hkv=16, d=128, kv="fp8_e4m3",
                      qdt=torch.float16, batch=64, ctx=4096, pool_pages=18750),
    # the Qwen3-8B decode (36 layers, 128 x 16,384 tokens) with the reference
    # arena's int8 mode (per-token fp16 scales)
    "qwen3-int8": dict(model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128, kv="int8",
                       qdt=torch.bfloat16, batch=128, ctx=16384, pool_pages=128 * 1024 + 512),
    "qwen3-int8-1l": dict(model="Qwen3-8B attention", layers=1, hq=32, hkv=8, d=128, kv="int8",
                          qdt=torch.bfloat16, batch=128, ctx=16384, pool_pages=128 * 1024 + 512),
    # one layer of the full config-4 launch (4.3 GB), for whole-launch captures
    "qwen3-fp8-1l": dict(model="Qwen3-8B attention", layers=1, hq=32, hkv=8, d=128, kv="fp8_e4m3",
                         qdt=torch.bfloat16, batch=128, ctx=16384, pool_pages=128 * 1024 + 512),
    # long-context scale-out: 64 sequences per GPU, context ~U[8192, 32768],
    # every step appends one token per sequence (contexts grow). bf16 KV of
    # 512 such sequences is ~1.55 TB, above one 8-GPU box, so each GPU keeps
    # `pool_gb` of physical layers and logical layer l reads layer l mod Lp
    # (every launch still streams its own >> L2 bytes from HBM).
    "qwen3-long": dict(model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128, kv="bf16", qdt=torch.bfloat16,
                       batch=64, ctx=(8192, 32768), grow=True, pool_gb=100.0),
    "qwen3-long-small": dict(model="Qwen3-8B attention", layers=2, hq=32, hkv=8, d=128, kv="bf16",
                             qdt=torch.bfloat16, batch=8, ctx=(8192, 32768), grow=True, pool_gb=4.0),
    # continuous-batching mix: 256 live sequences (~U[16, 8192] tokens, a
    # quarter of them forked from one shared 1024-token prefix); every step
    # retires 8 sequences (pages kept cached), admits 8 prompts ~U[64, 2048]
    # (a quarter forked from the prefix) with causal prefill attention, and
    # decodes one token for every live sequence; LRU eviction keeps pool
    # occupancy at or below 90 %.
    "olmoe-mix": dict(kind="mix", model="OLMoE-1B-7B attention", layers=16, hq=16, hkv=16, d=128, kv="fp16",
                      qdt=torch.float16, batch=256, ctx=(16, 8192), new_per_step=8, prompt=(64, 2048),
                      fork_frac=0.25, prefix=1024, pool_pages=72000, evict_at=0.9),
    "olmoe-mix-small": dict(kind="mix", model="OLMoE-1B-7B attention", layers=2, hq=16, hkv=16, d=128,
                            kv="fp16", qdt=torch.float16, batch=32, ctx=(16, 8192), new_per_step=8,
                            prompt=(64, 2048), fork_frac=0.25, prefix=1024, pool_pages=9000, evict_at=0.9),
    # the paging kernels at OLMoE scale (the append + gather of sequences of
    # 37 / 128 / 255 / 512 tokens, sized up):
    # per step append 64 sequences x 64 new tokens into all 16 layers, gather
    # 256 random all-layer pages into contiguous K/V, copy 256 pages (CoW)
    "olmoe-paging": dict(kind="paging", model="OLMoE-1B-7B attention", layers=16, hkv=16, d=128, kv="fp16",
                         batch=64, new_tokens=64, gather_pages=256, copy_pages=256, pool_pages=8192),
    # the same launches on a 2 GB pool, for profiler captures
    "olmoe-paging-small": dict(kind="paging", model="OLMoE-1B-7B attention", layers=16, hkv=16, d=128,
                               kv="fp16", batch=64, new_tokens=64, gather_pages=256, copy_pages=128,
                               pool_pages=1024),
    # prompt passes alone: causal prefill attention over whole prompts whose
    # K/V are already in the pages (one sckv_prefill_attn per layer)
    "qwen3-prefill": dict(kind="prefill", model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128,
                          kv="bf16", qdt=torch.bfloat16, batch=16, prompt=2048),
    "qwen3-fp8-prefill": dict(kind="prefill", model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128,
                              kv="fp8_e4m3", qdt=torch.bfloat16, batch=16, prompt=2048),
    "qwen3-int8-prefill": dict(kind="prefill", model="Qwen3-8B attention", layers=36, hq=32, hkv=8, d=128,
                               kv="int8", qdt=torch.bfloat16, batch=16, prompt=2048),
    # the attention input either side of the cache: q/k/v projections of
    # the hidden states (bf16 activations and weights), per-head QK-norm,
    # RoPE and the K/V append, fused in one launch per layer (sckv_qkv_append)
    "qwen3-qkv": dict(kind="qkv", model="Qwen3-8B attention", layers=36, hidden=4096, hq=32, hkv=8, d=128,
                      kv="bf16", batch=128, tokens_per_seq=1, ctx=16384),
    "qwen3-qkv-prefill": dict(kind="qkv", model="Qwen3-8B attention", layers=36, hidden=4096, hq=32, hkv=8, d=128,
                              kv="bf16", batch=8, tokens_per_seq=1024, ctx=0),
    # the whole attention layer at the Qwen3-8B FP8 decode shape (128 x 16,384 tokens),
    # through PagedAttentionLayer.decode: fused q/k/v projection + QK-norm +
    # RoPE (rows staged, FP8 append), decode attention over 16,384 tokens,
    # o_proj; fp32 normed input x and fp16 weights as the reference engine
    "qwen3-fp8-layer": dict(kind="layer", model="Qwen3-8B attention", layers=36, hidden=4096, hq=32, hkv=8, d=128,
                            kv="fp8_e4m3", batch=128, ctx=16384),
    # the other side: o_proj of the fp32 attention output with fp16 weights
    # (models/adapters.py:1231), one sckv_o_proj per layer
    "qwen3-oproj": dict(kind="oproj", model="Qwen3-8B attention", layers=36, hidden=4096, hq=32, hkv=8, d=128,
                        kv="fp16", batch=128, tokens_per_seq=1, ctx=0),
    "qwen3-oproj-prefill": dict(kind="oproj", model="Qwen3-8B attention", layers=36, hidden=4096, hq=32, hkv=8,
                                d=128, kv="fp16", batch=8, tokens_per_seq=1024, ctx=0),
}


def kv_bytes_per_elem(kv: str) -> int:
    return 2 if kv in ("fp16", "bf16") else 1


def attn_bytes_per_launch(w, ctx=None) -> int:
    """Algorithmic bytes one decode-attention launch must move: every
    sequence's K and V (plus FP8 page scales and block-table entries) once,
    its query row in and its output row out. `ctx` = per-sequence context
    lengths (default: the workload's uniform context)."""
    hkv, hq, d = w["hkv"], w["hq"], w["d"]
    c = np.full(w["batch"], w["ctx"], np.int64) if ctx is None else np.asarray(ctx, np.int64)
    pages = (c + PAGE - 1) // PAGE
    b = kv_bytes_per_elem(w["kv"])
    kv = int(c.sum()) * hkv * d * 2 * b
    scales = 0
    if w["kv"] == "fp8_e4m3":
        scales = int(pages.sum()) * hkv * 2 * 4          # one fp32 scale per (page, head, K|V)
    elif w["kv"] == "int8":
        scales = int(c.sum()) * hkv * 2 * 2             # one fp16 scale per (token, head, K|V)
    bt = int(pages.sum()) * 4
    qo = len(c) * hq * d * 2 * 2
    return kv + scales + bt + qo


def append_bytes_per_launch(w) -> int:
    B, hkv, d = w["batch"], w["hkv"], w["d"]
    src = B * hkv * d * 2 * 2          # read K and V rows (16-bit source)
    dst = B * hkv * d * 2 * kv_bytes_per_elem(w["kv"])
    return src + dst


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        mhz, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not mhz:
            return None
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(mhz)}


# ----------------------------------------------------------------------------- helpers
def measured_peak_gbs():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(workload: str, part: str = ""):
    """DRAM bytes (read + write) per launch of the dominant kernel from the
    committed ncu summaries: a `traffic_bytes_per_launch[<workload>]:` (or
    `[<workload>:<part>]`) line in any profiles/*.md, else the plain
    `traffic_bytes_per_launch:` line of profiles/decode_attn_<workload>.md."""
    key = f"{workload}:{part}" if part else workload
    pat = re.compile(r"traffic_bytes_per_launch\[" + re.escape(key) + r"\]:\s*([0-9.eE+]+)")
    for f in sorted((REPO / "profiles").glob("*.md")):
        m = pat.search(f.read_text())
        if m:
            return float(m.group(1))
    f = REPO / "profiles" / f"decode_attn_{workload}.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        # NCCL's own messages (e.g. its version banner) go to stderr so that
        # stdout carries only the JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device(f"cuda:{local}"))
    elif torch.cuda.is_available():  # the reference arm runs on host cores and needs no GPU
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- our arm
def local_workload(w, world: int, layout: str):
    """Per-rank slice of the workload: the same sequences with Hkv/N kv heads
    (and their query heads) under KV-head sharding; the full workload under
    sequence sharding (each rank its own sequences)."""
    if layout != "heads" or world == 1:
        return dict(w)
    if w["hkv"] % world:
        raise SystemExit(f"--layout heads needs {w['hkv']} kv heads divisible by {world}")
    lw = dict(w)
    lw["hkv"] = w["hkv"] // world
    lw["hq"] = w["hq"] // world
    return lw


def ctx_desc(w) -> str:
    if isinstance(w["ctx"], tuple):
        g = " growing 1/step" if w.get("grow") else ""
        return f"~U[{w['ctx'][0]},{w['ctx'][1]}]{g}"
    return str(w["ctx"])


def mean_ctx(w) -> int:
    return int(np.mean(w["ctx"])) if isinstance(w["ctx"], tuple) else int(w["ctx"])


def seq_contexts(w, rank: int) -> np.ndarray:
    """Per-sequence starting context lengths (uniform or ~U[lo, hi], seeded per rank)."""
    if isinstance(w["ctx"], tuple):
        lo, hi = w["ctx"]
        return np.random.default_rng(100 + rank).integers(lo, hi + 1, size=w["batch"]).astype(np.int64)
    return np.full(w["batch"], w["ctx"], np.int64)


def build_state(w, rank: int, grow_steps: int = 0, ctx0=None):
    """Pool, block tables and per-layer inputs of one rank.

    Fixed-context workloads: the step's new token rewrites slot ctx-1, so
    every step moves the same bytes. Growing workloads (`grow`): the new
    token goes to slot ctx and contexts advance by one per step; block tables
    have room for `grow_steps` more tokens and `reset()` rewinds them.
    `ctx0` (optional, one int per sequence) replaces the seeded starting
    contexts."""
    from synapcore_b200.pool import KVPool

    dev = torch.device("cuda", torch.cuda.current_device())
    L, hq, hkv, d, B = w["layers"], w["hq"], w["hkv"], w["d"], w["batch"]
    grow = bool(w.get("grow"))
    ctx0 = seq_contexts(w, rank) if ctx0 is None else np.asarray(ctx0, np.int64)
    if ctx0.shape != (B,):
        raise ValueError(f"ctx0 must hold {B} contexts")
    cap = ctx0 + (grow_steps + 1 if grow else 0)
    n_blocks = (cap + PAGE - 1) // PAGE
    max_blocks = int(n_blocks.max())
    if "pool_pages" in w:
        pool_pages = int(w["pool_pages"])
        n_phys = L
    else:
        pool_pages = int(n_blocks.sum()) + 64
        layer_bytes = pool_pages * 2 * hkv * PAGE * d * kv_bytes_per_elem(w["kv"])
        n_phys = max(1, min(L, int(w["pool_gb"] * 1e9 // layer_bytes)))
    pool = KVPool(n_phys, hkv, d, pool_pages, w["kv"], device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    view = pool.pool_view()
    if w["kv"] == "fp8_e4m3":
        # random e4m3 codes (no NaN bytes 0x7f / 0xff) and per-page-head scales U[0.5,4]/448*4
        for l in range(n_phys):
            for c0 in range(0, pool_pages, 8192):
                blk = view[l, c0:c0 + 8192]
                codes = torch.randint(0, 0x7F, blk.shape, dtype=torch.uint8, device=dev, generator=g)
                codes |= torch.randint(0, 2, blk.shape, dtype=torch.uint8, device=dev, generator=g) << 7
                blk.copy_(codes)
                del codes
        pool.scale_view().uniform_(0.5 / 448 * 4, 4.0 / 448 * 4, generator=g)
    elif w["kv"] == "int8":
        # codes U{-127..127} and per-(token, head) fp16 scales ~ max|x| / 127 of N(0,1)*U[0.5,4] rows
        for l in range(n_phys):
            for c0 in range(0, pool_pages, 8192):
                blk = view[l, c0:c0 + 8192]
                blk.copy_(torch.randint(-127, 128, blk.shape, dtype=torch.int8, device=dev, generator=g))
        sv = pool.scale_view()
        for l in range(n_phys):
            sv[l].uniform_(1.5 / 127, 12.0 / 127, generator=g)
    else:
        for l in range(n_phys):
            for c0 in range(0, pool_pages, 8192):
                view[l, c0:c0 + 8192].normal_(generator=g)
    rng = np.random.default_rng(rank)
    perm = rng.permutation(pool_pages)[: int(n_blocks.sum())].astype(np.int32)
    bt_h = np.zeros((B, max_blocks), np.int32)
    off = 0
    for b in range(B):
        bt_h[b, : n_blocks[b]] = perm[off: off + n_blocks[b]]
        off += n_blocks[b]
    bt = torch.from_numpy(bt_h).to(dev)
    # attention context after the step's append, and the append slot
    ctx_attn0 = ctx0 + 1 if grow else ctx0
    ctx = torch.from_numpy(ctx_attn0.astype(np.int32)).to(dev)
    start = torch.from_numpy((ctx_attn0 - 1).astype(np.int32)).to(dev)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    q = torch.randn((L, B, hq, d), generator=g, device=dev).to(w["qdt"])
    src_dt = torch.float16 if w["kv"] == "fp16" else torch.bfloat16
    kn = torch.randn((L, B, hkv, d), generator=g, device=dev).to(src_dt)
    vn = torch.randn((L, B, hkv, d), generator=g, device=dev).to(src_dt)
    out = torch.empty((L, B, hq, d), dtype=w["qdt"], device=dev)
    ws = torch.empty(pool.decode_workspace_bytes(B, hq, max_blocks), dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    st = dict(pool=pool, bt=bt, ctx=ctx, cu=cu, start=start, q=q, kn=kn, vn=vn, out=out, ws=ws,
              n_phys=n_phys, grow=grow, ctx0=ctx0, ctx_host=ctx_attn0.copy(), max_blocks=max_blocks,
              pool_pages=pool_pages)
    return st


def reset_contexts(s):
    """Rewind growing contexts to their starting lengths."""
    if s["grow"]:
        s["ctx"].copy_(torch.from_numpy((s["ctx0"] + 1).astype(np.int32)))
        s["start"].copy_(torch.from_numpy(s["ctx0"].astype(np.int32)))
        s["ctx_host"] = s["ctx0"] + 1


def step_bytes(w, s) -> int:
    """Algorithmic bytes of the next step (attention at the current contexts + appends)."""
    return w["layers"] * (attn_bytes_per_launch(w, s["ctx_host"]) + append_bytes_per_launch(w))


def advance(s):
    if s["grow"]:
        s["ctx"] += 1
        s["start"] += 1
        s["ctx_host"] = s["ctx_host"] + 1


def exchange_layer(s, l, pl, q, out_full=None, k_new=None, v_new=None):
    """KV-head-sharded layer with the exchange fused into the decode: this
    rank's heads go straight into every rank's full-head buffer, then a
    device wait for every rank's flag of this (step, layer). Epochs come from
    each rank's device counter (the same sequence of calls on every rank), so
    the step can also be replayed from a CUDA graph."""
    ex = s["exchange"]
    ex.decode(l, q, s["bt"], s["ctx"], 0, phys_layer=pl, k_new=k_new, v_new=v_new)
    ex.wait(0)
    if out_full is not None:
        out_full.copy_(ex.output(l, q.shape[0]))


def fused_append(w, s) -> bool:
    """16-bit pools store the new token's K/V inside the decode launch
    (sckv_decode_attn_append, or the exchange decode); one-byte pools run
    the append kernel first."""
    return w["kv"] in ("fp16", "bf16")


def layer_calls(w, s, l, q, k, v, out, out_full=None, events=None):
    """One layer of the decode step through the public calls; `events` (a
    list) gets a CUDA event on each side of the attention launch."""
    pool = s["pool"]
    pl = l % s["n_phys"]
    fused = fused_append(w, s)
    if not fused:
        pool.append(k, v, s["cu"], s["start"], s["bt"], layer0=pl)
    if events is not None:
        events.append(torch.cuda.Event(enable_timing=True))
        events[-1].record()
    if "exchange" in s:
        exchange_layer(s, l, pl, q, out_full=out_full, k_new=k if fused else None, v_new=v if fused else None)
    elif fused:
        pool.decode_attn_append(pl, q, k, v, s["bt"], s["ctx"], out=out, workspace=s["ws"])
    else:
        pool.decode_attn(pl, q, s["bt"], s["ctx"], out=out, workspace=s["ws"])
    if events is not None:
        events.append(torch.cuda.Event(enable_timing=True))
        events[-1].record()
    if "gather" in s and out_full is not None:
        out_full.copy_(s["gather"].gather(out))


def run_step(w, s, attn_events=None):
    if "graph" in s and attn_events is None:
        # the whole step captured once (KV-head-sharded exchange layout)
        s["graph"].replay()
        advance(s)
        return
    for l in range(w["layers"]):
        layer_calls(w, s, l, s["q"][l], s["kn"][l], s["vn"][l], s["out"][l],
                    out_full=s["full"][l] if "gather" in s else None, events=attn_events)
    advance(s)


def bench_ours(args, w_full, world, rank, local):
    w = local_workload(w_full, world, args.layout)
    s = build_state(w, rank, grow_steps=max(args.steps, args.warmup))
    pool = s["pool"]
    if args.layout == "heads" and world > 1 and args.exchange == "nccl":
        from synapcore_b200.distributed import HeadShardedOutput

        s["gather"] = HeadShardedOutput(world)
        s["full"] = torch.empty((w["layers"], w["batch"], w_full["hq"], w["d"]), dtype=w["qdt"], device="cuda")
    elif args.layout == "heads" and world > 1:
        from synapcore_b200.distributed import HeadShardedExchange

        s["exchange"] = HeadShardedExchange(pool, world, rank, w["layers"], w["batch"], w_full["hq"], w["qdt"])
        s["full"] = torch.empty((w["layers"], w["batch"], w_full["hq"], w["d"]), dtype=w["qdt"], device="cuda")
    for _ in range(args.warmup):
        run_step(w, s)
    torch.cuda.synchronize()
    pool.raise_on_status()
    if "exchange" in s:
        # 16 small layer launches per rank and step: replay the step from a
        # CUDA graph (captured on every rank, nothing runs during capture)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for l in range(w["layers"]):
                layer_calls(w, s, l, s["q"][l], s["kn"][l], s["vn"][l], s["out"][l])
        s["graph"] = g
    reset_contexts(s)
    total_bytes = 0
    launch_bytes = []

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    fused = fused_append(w, s)
    for _ in range(args.steps):
        total_bytes += step_bytes(w, s)
        launch_bytes.append(attn_bytes_per_launch(w, s["ctx_host"]) + (append_bytes_per_launch(w) if fused else 0))
        run_step(w, s)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    pool.raise_on_status()
    # per-launch attention times for the roofline: a second pass over the
    # same contexts with CUDA events around each attention launch (kept out
    # of the timed loop above)
    reset_contexts(s)
    attn_ev = []
    for _ in range(args.steps):
        run_step(w, s, attn_ev)
    torch.cuda.synchronize()
    attn_ms = [attn_ev[i].elapsed_time(attn_ev[i + 1]) for i in range(0, len(attn_ev), 2)]
    attn_avg_ms = max_over_ranks(float(np.mean(attn_ms)), world)
    pool.raise_on_status()

    # ---- e2e through the public calls, host buffers in pinned memory. Like a
    # serving loop, step i+1's inputs are copied in on a copy stream while
    # step i computes, and step i's outputs are copied out while step i+1
    # computes (two device buffers each); every step still moves its own
    # inputs and reads back its own result inside the timed region.
    L = w["layers"]
    res_t = s["full"] if ("gather" in s or "exchange" in s) else s["out"]
    h_q = s["q"].cpu().pin_memory()
    h_k = s["kn"].cpu().pin_memory()
    h_v = s["vn"].cpu().pin_memory()
    h_out = [torch.empty(res_t.shape, dtype=res_t.dtype).pin_memory() for _ in range(2)]
    d_in = [(torch.empty_like(s["q"]), torch.empty_like(s["kn"]), torch.empty_like(s["vn"])) for _ in range(2)]
    d_res = [res_t, torch.empty_like(res_t)]
    d_out = [s["out"], torch.empty_like(s["out"])] if "gather" in s else d_res
    comp = torch.cuda.current_stream()
    cstream = torch.cuda.Stream()
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in_ready", "in_free", "out_ready", "out_done")}

    def copy_in(i):
        b = i % 2
        with torch.cuda.stream(cstream):
            if i >= 2:
                cstream.wait_event(ev["in_free"][b])
            for h, d in zip((h_q, h_k, h_v), d_in[b]):
                d.copy_(h, non_blocking=True)
            ev["in_ready"][b].record(cstream)

    def compute(i):
        b = i % 2
        comp.wait_event(ev["in_ready"][b])
        if i >= 2:
            comp.wait_event(ev["out_done"][b])
        d_q, d_k, d_v = d_in[b]
        for l in range(L):
            layer_calls(w, s, l, d_q[l], d_k[l], d_v[l], d_out[b][l],
                        out_full=d_res[b][l] if ("gather" in s or "exchange" in s) else None)
        ev["in_free"][b].record(comp)
        ev["out_ready"][b].record(comp)
        advance(s)

    def copy_out(i):
        b = i % 2
        with torch.cuda.stream(cstream):
            cstream.wait_event(ev["out_ready"][b])
            h_out[b].copy_(d_res[b], non_blocking=True)
            ev["out_done"][b].record(cstream)

    def e2e_run(n):
        copy_in(0)
        for i in range(n):
            if i + 1 < n:
                copy_in(i + 1)
            compute(i)
            copy_out(i)
        comp.wait_event(ev["out_done"][(n - 1) % 2])

    reset_contexts(s)
    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize()
    reset_contexts(s)
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    cstream.wait_stream(comp)
    e2e_run(args.steps)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    h2d = h_q.numel() * h_q.element_size() + 2 * h_k.numel() * h_k.element_size()
    d2h = h_out[0].numel() * h_out[0].element_size()
    pool.raise_on_status()

    ms_step = ms_total / args.steps
    # the e2e pass replays the same context sequence, so it moves the same bytes
    value = world * total_bytes / (ms_total * 1e-3) / 1e9
    e2e_value = world * total_bytes / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    avg_launch_bytes = float(np.mean(launch_bytes))
    achieved = avg_launch_bytes / (attn_avg_ms * 1e-3) / 1e9
    traffic = profiled_traffic(args.workload)
    # a split launch (non-zero workspace) adds the combine kernel
    split = pool.decode_workspace_bytes(w["batch"], w["hq"], s["bt"].shape[1]) > 0
    # the exchange adds its signal and wait kernels
    launches_per_layer = (1 if fused else 2) + (1 if split else 0) + (2 if "exchange" in s else 0)
    res = {
        "metric": "paged decode-attn KV GB/s (% HBM peak) and decode tok/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if (args.layout == "heads" and world > 1) else "weak",
        "vs_baseline": None,
        "dtype": w["kv"],
        "data": "synthetic (seeded N(0,1) KV pages, random block-table permutation)",
        "tok_per_s": round((w["batch"] if (args.layout == "heads" and world > 1) else world * w["batch"])
                           / (ms_step * 1e-3), 1),
        "pct_hbm_peak": round(100.0 * value / world / peak, 2),
        "config": {
            "workload": f"{args.workload}: paged decode attention, {w_full['model']} shape {w_full['layers']}L x "
                        f"{w_full['hq']}q/{w_full['hkv']}kv heads x d{w_full['d']}, {w_full['kv']} KV, page 16, "
                        f"batch {w_full['batch']}" + ("" if (args.layout == "heads" and world > 1) else "/GPU")
                        + f", context {ctx_desc(w_full)}, pool {s['pool_pages']} pages x {s['n_phys']} layers"
                        + (f" (logical layer l reads physical layer l mod {s['n_phys']})"
                           if s["n_phys"] < w["layers"] else "")
                        + ("; the one-token K/V append runs inside the decode launch" if fused
                           else "; one append launch then one decode launch per layer"),
            "global_batch": w["batch"] if (args.layout == "heads" and world > 1) else world * w["batch"],
            "seq_len": ctx_desc(w_full),
            "parallelism": ((f"kv-head-sharded x{world} (NCCL all-gather of outputs per layer)"
                             if args.exchange == "nccl" else
                             f"kv-head-sharded x{world} (outputs stored into every rank's buffer by the "
                             f"decode kernel over NVLink, one flag wait per layer)")
                            if (args.layout == "heads" and world > 1)
                            else f"sequence-sharded x{world} (independent pools)"),
            "l2": "inputs larger than L2 (KV per layer launch >> 126 MB)",
        },
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": int(args.steps * L * launches_per_layer),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": ("decode_mma_kernel" if (w["hq"] // w["hkv"] >= 2 or kv_bytes_per_elem(w["kv"]) == 1)
                                else "decode_kernel")
                               + (" with the fused append" if fused else "")
                               + (" (+combine)" if split else "") + " per layer launch",
                     "bytes_per_launch": int(avg_launch_bytes), "avg_launch_ms": round(attn_avg_ms, 4)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_seconds)
        rc = reference_code_baseline(w, budget_s=min(5.0, args.cpu_seconds))
        if rc is not None:
            res["cpu_baseline"]["reference_code"] = rc
    if "exchange" in s:
        # every rank's writes into this rank's buffer ended before its last
        # wait; the barrier keeps all ranks' mappings alive until all are done
        torch.cuda.synchronize()
        s.pop("graph", None)  # the captured step refers to the exchange's buffers
        barrier(world)
        st = s["exchange"].status()
        if st[0] != 0:
            raise RuntimeError(f"exchange status {st}")
        s["exchange"].close()
    pool.close()
    return res


# ----------------------------------------------------------------------------- paging kernels
def bench_paging(args, w, world, rank, local):
    """One step = one append of `new_tokens` per sequence into every layer
    (sckv_append), one gather of `gather_pages` random pages into contiguous
    K / V (sckv_gather) and one copy of `copy_pages` pages (sckv_copy_pages)."""
    from synapcore_b200 import _native as N
    from synapcore_b200.pool import KVPool

    dev = torch.device("cuda", local)
    L, H, d, B, T, P = w["layers"], w["hkv"], w["d"], w["batch"], w["new_tokens"], w["pool_pages"]
    eb = kv_bytes_per_elem(w["kv"])
    pool = KVPool(L, H, d, P, w["kv"], device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    view = pool.pool_view()
    for l in range(L):
        view[l].normal_(generator=g)
    mb = (T + PAGE - 1) // PAGE
    perm = torch.randperm(P, generator=g, device=dev).to(torch.int32)
    bt = perm[: B * mb].view(B, mb).contiguous()
    cu = torch.arange(0, B * T + 1, T, dtype=torch.int32, device=dev)
    start = torch.zeros(B, dtype=torch.int32, device=dev)
    kn = torch.randn(L, B * T, H, d, device=dev, generator=g).half()
    vn = torch.randn(L, B * T, H, d, device=dev, generator=g).half()
    gids = perm[B * mb: B * mb + w["gather_pages"]].contiguous()
    c0 = B * mb + w["gather_pages"]
    src = perm[c0: c0 + w["copy_pages"]].contiguous()
    dst = perm[c0 + w["copy_pages"]: c0 + 2 * w["copy_pages"]].contiguous()
    nt = w["gather_pages"] * PAGE
    gk = torch.empty(L, H, nt, d, dtype=torch.float16, device=dev)
    gv = torch.empty_like(gk)
    page_bytes = 2 * L * H * PAGE * d * eb
    bytes_append = L * B * T * H * d * 2 * (2 + eb) + B * mb * 4  # read fp16 source, write pool, block table
    bytes_gather = w["gather_pages"] * page_bytes + L * H * nt * d * 2 * 2
    bytes_copy = 2 * w["copy_pages"] * page_bytes
    kernels = [("append", bytes_append), ("gather", bytes_gather), ("copy", bytes_copy)]

    def step(ev=None):
        def mark():
            if ev is not None:
                ev.append(torch.cuda.Event(enable_timing=True))
                ev[-1].record()
        mark()
        pool.append(kn, vn, cu, start, bt)
        mark()
        pool.gather(gids, out=(gk, gv))
        mark()
        pool.copy_pages(src, dst)
        mark()

    n0 = N.launch_count()
    step()
    launches_per_step = N.launch_count() - n0
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    pool.raise_on_status()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    per = {k: [] for k, _ in kernels}
    for _ in range(args.steps):
        ev = []
        step(ev)
        torch.cuda.synchronize()
        for i, (k, _) in enumerate(kernels):
            per[k].append(ev[i].elapsed_time(ev[i + 1]))
    pool.raise_on_status()
    peak, peak_kind = measured_peak_gbs()
    sub = {}
    for k, b in kernels:
        ms = max_over_ranks(float(np.mean(per[k])), world)
        sub[k] = {"bytes_per_launch": int(b), "avg_launch_ms": round(ms, 4),
                  "achieved": round(b / (ms * 1e-3) / 1e9, 1), "frac": round(b / (ms * 1e-3) / 1e9 / peak, 4)}

    # e2e: new K/V rows from pinned host memory each step, gathered K/V read back
    h_k, h_v = kn.cpu().pin_memory(), vn.cpu().pin_memory()
    h_gk = torch.empty(gk.shape, dtype=gk.dtype).pin_memory()
    h_gv = torch.empty(gv.shape, dtype=gv.dtype).pin_memory()
    d_k, d_v = torch.empty_like(kn), torch.empty_like(vn)
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        d_k.copy_(h_k, non_blocking=True)
        d_v.copy_(h_v, non_blocking=True)
        pool.append(d_k, d_v, cu, start, bt)
        pool.gather(gids, out=(gk, gv))
        pool.copy_pages(src, dst)
        h_gk.copy_(gk, non_blocking=True)
        h_gv.copy_(gv, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    pool.raise_on_status()

    step_bytes_all = sum(b for _, b in kernels)
    value = world * step_bytes_all / (ms_total * 1e-3 / args.steps) / 1e9
    e2e_value = world * step_bytes_all / (e2e_ms * 1e-3 / args.steps) / 1e9
    top = max(sub, key=lambda k: sub[k]["avg_launch_ms"])
    res = {
        "metric": "paging kernels GB/s (append + gather + CoW page copy)",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_total / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w["kv"],
        "data": "synthetic (seeded N(0,1) pages and new rows, random page ids)",
        "config": {
            "workload": f"{args.workload}: {w['model']} {L} layers x {H} kv heads x d{d}, {w['kv']} pages of 16 "
                        f"tokens; per step append {B} x {T} tokens into all layers, gather {w['gather_pages']} "
                        f"pages, copy {w['copy_pages']} pages; pool {P} pages",
            "global_batch": world * B, "seq_len": T, "parallelism": f"sequence-sharded x{world}",
            "l2": "each kernel moves >= 1 GB per launch (>> L2)",
        },
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(2 * h_k.numel() * 2), "d2h_bytes_per_step": int(2 * h_gk.numel() * 2)},
        "gpu_launches": int(launches_per_step * args.steps),
        "roofline": {"bound": "hbm", "achieved": sub[top]["achieved"], "peak": peak, "unit": "GB/s",
                     "frac": sub[top]["frac"], "traffic": profiled_traffic(args.workload, top),
                     "peak_kind": peak_kind,
                     "kernel": f"{top} (the step's longest launch)", "bytes_per_launch": sub[top]["bytes_per_launch"],
                     "avg_launch_ms": sub[top]["avg_launch_ms"]},
        "kernels": sub,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_gather(w, budget_s=args.cpu_seconds)
    pool.close()
    return res


def cpu_baseline_gather(w, budget_s: float = 15.0):
    """The reference's page-by-page NumPy gather (oracle restatement of
    gather_contiguous_kv_numpy, native/native_engine.py:403-419) of 32 pages."""
    from oracle.kv_oracle import ArenaOracle

    L, H, d = w["layers"], w["hkv"], w["d"]
    n = 32
    ar = ArenaOracle(n, L, H, d, "fp16")
    rng = np.random.default_rng(0)
    ar.k[:] = rng.standard_normal(ar.k.shape).astype(np.float16)
    ar.v[:] = rng.standard_normal(ar.v.shape).astype(np.float16)
    ids = list(rng.permutation(n))
    reps, t0 = 0, time.perf_counter()
    while True:
        ar.gather_contiguous_kv_numpy(ids)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    page_bytes = 2 * L * H * PAGE * d * 2
    gbs = reps * 2 * n * page_bytes / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
            or (os.cpu_count() or 1), "kind": "port",
            "sample": f"gather of {n} fp16 pages ({n * page_bytes / 1e6:.0f} MB), {reps} reps in {el:.1f}s"}


# ----------------------------------------------------------------------------- prompt passes
def prefill_flops(w) -> int:
    """Causal attention flops of one layer over the step's prompts: query t
    of a T-token prompt sees t + 1 keys (2 matmuls x 2 flops per MAC)."""
    T = w["prompt"]
    return w["batch"] * 4 * w["hq"] * w["d"] * (T * (T + 1) // 2)


def bench_prefill(args, w, world, rank, local):
    """One step = sckv_prefill_attn for every layer over `batch` prompts of
    `prompt` tokens whose K/V already fill their pages."""
    from synapcore_b200.pool import KVPool

    dev = torch.device("cuda", local)
    L, hq, hkv, d, B, T = w["layers"], w["hq"], w["hkv"], w["d"], w["batch"], w["prompt"]
    mb = (T + PAGE - 1) // PAGE
    P = B * mb
    pool = KVPool(L, hkv, d, P, w["kv"], device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    view = pool.pool_view()
    for l in range(L):
        if w["kv"] == "fp8_e4m3":
            codes = torch.randint(0, 0x7F, view[l].shape, dtype=torch.uint8, device=dev, generator=g)
            codes |= torch.randint(0, 2, view[l].shape, dtype=torch.uint8, device=dev, generator=g) << 7
            view[l].copy_(codes)
        elif w["kv"] == "int8":
            view[l].copy_(torch.randint(-127, 128, view[l].shape, dtype=torch.int8, device=dev, generator=g))
        else:
            view[l].normal_(generator=g)
    if w["kv"] == "fp8_e4m3":
        pool.scale_view().uniform_(0.5 / 448 * 4, 4.0 / 448 * 4, generator=g)
    elif w["kv"] == "int8":
        pool.scale_view().uniform_(1.5 / 127, 12.0 / 127, generator=g)
    perm = torch.randperm(P, generator=g, device=dev).to(torch.int32)
    bt = perm.view(B, mb)
    cu = torch.arange(0, B * T + 1, T, dtype=torch.int32, device=dev)
    start = torch.zeros(B, dtype=torch.int32, device=dev)
    # one query tensor serves every layer (268 MB >> L2 at the default size)
    q = torch.randn(B * T, hq, d, device=dev, generator=g).to(w["qdt"])
    out = torch.empty_like(q)

    def step(qs, outs, ev=None):
        for l in range(L):
            if ev is not None:
                ev.append(torch.cuda.Event(enable_timing=True))
                ev[-1].record()
            pool.prefill_attn(l, qs, cu, start, bt, out=outs)
            if ev is not None:
                ev.append(torch.cuda.Event(enable_timing=True))
                ev[-1].record()

    from synapcore_b200 import _native as N

    n0 = N.launch_count()
    step(q, out)
    launches_per_step = N.launch_count() - n0
    for _ in range(args.warmup):
        step(q, out)
    torch.cuda.synchronize()
    pool.raise_on_status()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step(q, out)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    ev = []
    step(q, out, ev)
    torch.cuda.synchronize()
    launch_ms = max_over_ranks(float(np.mean([ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)])), world)
    pool.raise_on_status()

    # e2e: each step copies the queries in from pinned host memory and reads
    # the last layer's output back
    h_q = q.cpu().pin_memory()
    h_o = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_q = torch.empty_like(q)
    step(d_q, out)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    f0.record()
    for _ in range(args.steps):
        d_q.copy_(h_q, non_blocking=True)
        step(d_q, out)
        h_o.copy_(out, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    pool.raise_on_status()

    flops = prefill_flops(w)
    peak, peak_kind = 1590.0, "fallback"
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        try:
            peak, peak_kind = float(json.loads(pk.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    value = world * L * flops / (ms_total * 1e-3 / args.steps) / 1e12
    e2e_value = world * L * flops / (e2e_ms * 1e-3 / args.steps) / 1e12
    achieved = flops / (launch_ms * 1e-3) / 1e12
    res = {
        "metric": "causal prefill attention TFLOP/s (counting the causal half)",
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_total / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w["kv"],
        "data": "synthetic (seeded codes / N(0,1) KV pages, random block-table permutation, N(0,1) queries)",
        "tok_per_s": round(world * B * T / (ms_total * 1e-3 / args.steps), 1),
        "config": {
            "workload": f"{args.workload}: {w['model']} {L} layers, {hq}q/{hkv}kv heads x d{d}, {w['kv']} KV, "
                        f"{B} prompts x {T} tokens per GPU, one sckv_prefill_attn per layer",
            "global_batch": world * B, "seq_len": T, "parallelism": f"sequence-sharded x{world}",
            "l2": "each layer's K/V (%.2f GB) read by every head group; > L2 for 16-bit pools"
                  % (B * T * hkv * d * 2 * kv_bytes_per_elem(w["kv"]) / 1e9),
        },
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": int(h_q.numel() * 2),
                "d2h_bytes_per_step": int(h_o.numel() * 2)},
        "gpu_launches": int(launches_per_step * args.steps),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args.workload),
                     "peak_kind": peak_kind,
                     "kernel": "prefill_tc_kernel (tcgen05) per layer launch", "flops_per_launch": int(flops),
                     "avg_launch_ms": round(launch_ms, 4)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_prefill(w, budget_s=args.cpu_seconds)
    pool.close()
    return res


# ----------------------------------------------------------------------------- fused attention input
def qkv_flops(w, n_tok: int) -> int:
    if w["kind"] == "oproj":
        return 2 * n_tok * w["hq"] * w["d"] * w["hidden"]
    return 2 * n_tok * w["hidden"] * (w["hq"] + 2 * w["hkv"]) * w["d"]


def qkv_bytes(w, n_tok: int) -> int:
    """Algorithmic bytes of one layer launch: weights + x read, q_out + K/V
    rows written (bf16); for o_proj the fp16 weights, the fp32 attention
    output read and the fp32 result written."""
    if w["kind"] == "oproj":
        fin = w["hq"] * w["d"]
        return 2 * fin * w["hidden"] + 4 * n_tok * fin + 4 * n_tok * w["hidden"]
    hd = (w["hq"] + 2 * w["hkv"]) * w["d"]
    return 2 * (hd * w["hidden"] + n_tok * w["hidden"] + n_tok * hd)


def bench_layer(args, w, world, rank, local):
    """One step = PagedAttentionLayer.decode for every layer: one new token
    for each of `batch` sequences whose contexts start at `ctx` (seeded FP8
    pages) and grow by one per step."""
    from synapcore_b200 import PagedAttentionLayer, PagedKVCache
    from synapcore_b200 import _native as N

    dev = torch.device("cuda", local)
    L, H, hq, d, hidden, B, ctx0 = w["layers"], w["hkv"], w["hq"], w["d"], w["hidden"], w["batch"], w["ctx"]
    steps_total = args.warmup + 2 * args.steps + 2
    blocks = (ctx0 + steps_total + PAGE - 1) // PAGE
    cache = PagedKVCache(L, H, d, max_pages=B * blocks + 64, max_seqs=B, max_blocks_per_seq=blocks, kv_dtype=w["kv"],
                         device=dev)
    # synthetic contexts: every sequence holds ctx0 tokens of seeded pages
    for b in range(B):
        cache.add_sequence(b)
    cache._grow_rows(0, [ctx0] * B)
    for b in range(B):
        cache.lengths[b] = ctx0
    cache.ctx_lens[:B].fill_(ctx0)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    view = cache.pool.pool_view()
    for l in range(L):
        for c0 in range(0, view.shape[1], 8192):
            blk = view[l, c0:c0 + 8192]
            codes = torch.randint(0, 0x7F, blk.shape, dtype=torch.uint8, device=dev, generator=g)
            codes |= torch.randint(0, 2, blk.shape, dtype=torch.uint8, device=dev, generator=g) << 7
            blk.copy_(codes)
            del codes
    cache.pool.scale_view().uniform_(0.5 / 448 * 4, 4.0 / 448 * 4, generator=g)
    layer = PagedAttentionLayer(cache, hq, rope_theta=1e6, rms_eps=1e-6)
    sc = hidden ** -0.5
    wts = [[(torch.randn(r, c, device=dev, generator=g) * sc).half()
            for r, c in ((hq * d, hidden), (H * d, hidden), (H * d, hidden), (hidden, hq * d))] for _ in range(L)]
    qn = torch.rand(d, device=dev, generator=g).add_(0.5).half()
    kn = torch.rand(d, device=dev, generator=g).add_(0.5).half()
    x = torch.randn(L, B, hidden, device=dev, generator=g)
    out = torch.empty(B, hidden, device=dev)

    def step():
        for l in range(L):
            o = layer.decode(l, x[l], B, *wts[l], q_norm_w=qn, k_norm_w=kn)
        out.copy_(o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    cache.pool.raise_on_status()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    n0 = N.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    launches = N.launch_count() - n0
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    cache.pool.raise_on_status()
    # e2e: each step's normed inputs come from pinned host memory and the
    # last layer's output goes back
    h_x = x.cpu().pin_memory()
    h_o = torch.empty(B, hidden).pin_memory()
    barrier(world)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x.copy_(h_x, non_blocking=True)
        step()
        h_o.copy_(out, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world) / args.steps
    # algorithmic bytes per step: K/V codes + page scales read, weights and
    # activations, the new rows
    ctx_mid = ctx0 + args.warmup + args.steps // 2
    kv_b = B * ctx_mid * H * d * 2 + B * ((ctx_mid + PAGE - 1) // PAGE) * H * 2 * 4
    w_b = 2 * ((hq + 2 * H) * d * hidden + hidden * hq * d)
    act_b = B * (hidden * 4 + hq * d * 4 * 2 + hidden * 4)
    per_layer = kv_b + w_b + act_b
    peak, peak_kind = measured_peak_gbs()
    achieved = per_layer / (ms * 1e-3 / L) / 1e9
    res = {
        "metric": "whole attention layer decode tok/s (projections, FP8 paged attention, o_proj)",
        "value": round(world * B / (ms * 1e-3), 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8 KV, fp16 weights, fp32 activations",
        "data": "synthetic (seeded e4m3 pages and U[0.5,4]-scaled page scales, N(0,1) inputs, N(0,1/hidden) weights)",
        "kv_gb_per_s": round(world * L * per_layer / (ms * 1e-3) / 1e9, 1),
        "config": {"workload": f"{args.workload}: {w['model']} {L} layers, hidden {hidden}, {hq}q/{H}kv heads x d{d}, "
                               f"FP8 pool, {B} sequences from {ctx0} tokens, one token each per step through "
                               f"PagedAttentionLayer.decode",
                   "global_batch": world * B, "seq_len": ctx0, "parallelism": f"sequence-sharded x{world}",
                   "l2": "each layer's K/V (%.1f GB) >> L2" % (kv_b / 1e9)},
        "e2e": {"value": round(world * B / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": int(h_x.numel() * 4), "d2h_bytes_per_step": int(h_o.numel() * 4)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "one layer's launches (projection, finish, FP8 append, reserve, decode attention, "
                               "combine, split, o_proj), step time / layers",
                     "bytes_per_launch": int(per_layer), "avg_launch_ms": round(ms / L, 4)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_layer(w, budget_s=args.cpu_seconds)
    return res


def cpu_baseline_layer(w, budget_s: float = 15.0):
    """The reference's forward_numpy for one layer and one decode token of a
    sequence with `ctx` cached tokens (oracle composition of
    models/adapters.py:1148-1231), repeated for ~budget_s; tok/s of the full
    model step extrapolated (/ layers)."""
    from oracle.kv_oracle import attention_layer

    rng = np.random.default_rng(0)
    hidden, hq, H, d, ctx = w["hidden"], w["hq"], w["hkv"], w["d"], w["ctx"]
    sc = hidden ** -0.5
    wts = [(rng.standard_normal(sh) * sc).astype(np.float16)
           for sh in ((hq * d, hidden), (H * d, hidden), (H * d, hidden), (hidden, hq * d))]
    qn = kn = np.ones(d, np.float16)
    pk = rng.standard_normal((H, ctx, d)).astype(np.float16)
    pv = rng.standard_normal((H, ctx, d)).astype(np.float16)
    x = rng.standard_normal((1, hidden)).astype(np.float32)
    reps, t0 = 0, time.perf_counter()
    while True:
        attention_layer(x, *wts, hq, H, pk, pv, qn, kn, 1e-6, 1e6)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    return {"value": round(reps / el / w["layers"], 4), "unit": "tok/s",
            "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0) or (os.cpu_count() or 1), "kind": "port",
            "sample": f"1 layer x 1 sequence x ctx {ctx} (fp16 cache), {reps} reps in {el:.1f}s; "
                      f"tok/s = layer calls per second / {w['layers']} layers"}


def bench_qkv(args, w, world, rank, local):
    """One step = sckv_qkv_append for every layer over the step's tokens
    (decode: one token per sequence; prefill: whole prompts)."""
    from synapcore_b200.pool import KVPool, rope_inv_freq

    dev = torch.device("cuda", local)
    L, H, hq, d, hidden = w["layers"], w["hkv"], w["hq"], w["d"], w["hidden"]
    B, tps = w["batch"], w["tokens_per_seq"]
    n_tok = B * tps
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    scale = hidden ** -0.5
    oproj = w["kind"] == "oproj"
    ctx0 = w["ctx"]
    if oproj:
        # fp32 attention outputs (as the reference's attn_out) and fp16 weights
        fin = hq * d
        wo = [torch.randn(hidden, fin, device=dev, generator=g).mul_(fin ** -0.5).half() for _ in range(L)]
        x = torch.randn(L, n_tok, fin, device=dev, generator=g)
        q_out = torch.empty(L, n_tok, hidden, dtype=torch.float32, device=dev)
        pool = KVPool(1, H, d, 4, w["kv"], device=dev)

        def step(xs, outs):
            for l in range(L):
                pool.o_proj(xs[l], wo[l], out=outs[l])
    else:
        wq = [torch.randn(hq * d, hidden, device=dev, generator=g).mul_(scale).to(torch.bfloat16) for _ in range(L)]
        wk = [torch.randn(H * d, hidden, device=dev, generator=g).mul_(scale).to(torch.bfloat16) for _ in range(L)]
        wv = [torch.randn(H * d, hidden, device=dev, generator=g).mul_(scale).to(torch.bfloat16) for _ in range(L)]
        qn = torch.rand(d, device=dev, generator=g).add_(0.5).half()
        kn = torch.rand(d, device=dev, generator=g).add_(0.5).half()
        x = torch.randn(L, n_tok, hidden, device=dev, generator=g).to(torch.bfloat16)
        mb = (ctx0 + tps + PAGE - 1) // PAGE
        # only the pages the new tokens land in exist; earlier blocks are never touched
        b0 = ctx0 // PAGE
        nb = mb - b0
        pool = KVPool(L, H, d, B * nb, w["kv"], device=dev)
        bt = torch.zeros(B, mb, dtype=torch.int32, device=dev)
        bt[:, b0:] = torch.arange(B * nb, dtype=torch.int32, device=dev).view(B, nb)
        cu = torch.arange(0, n_tok + 1, tps, dtype=torch.int32, device=dev)
        start = torch.full((B,), ctx0, dtype=torch.int32, device=dev)
        inv = rope_inv_freq(1e6, d, dev)
        q_out = torch.empty(L, n_tok, hq, d, dtype=torch.bfloat16, device=dev)

        def step(xs, outs):
            for l in range(L):
                pool.qkv_append(l, xs[l], wq[l], wk[l], wv[l], cu, start, bt, inv, q_norm_w=qn, k_norm_w=kn,
                                q_out=outs[l])

    # a step is launch-bound at decode sizes (host work per call ~ the
    # kernel's time), so each step is replayed from a CUDA graph, as a
    # serving loop would; one graph per input / output buffer pair
    comp = torch.cuda.current_stream()
    d_x = [x, torch.empty_like(x)]
    d_q = [q_out, torch.empty_like(q_out)]
    d_x[1].copy_(x)
    from synapcore_b200 import _native as N

    n0 = N.launch_count()
    step(x, q_out)
    launches_per_step = N.launch_count() - n0  # rope table + projection (+ split-K finish) per layer
    graphs = []
    cap = torch.cuda.Stream()
    for b in range(2):
        cap.wait_stream(comp)
        with torch.cuda.stream(cap):
            step(d_x[b], d_q[b])
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=cap):
            step(d_x[b], d_q[b])
        graphs.append(gph)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graphs[0].replay()
    torch.cuda.synchronize()
    pool.raise_on_status()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graphs[0].replay()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    launch_ms = ms_total / args.steps / L  # rope table + projection kernel of one layer
    pool.raise_on_status()

    # e2e: each step copies its hidden states in from pinned host memory and
    # reads the rotated q back (double-buffered across steps, as a serving loop would)
    h_x = x.cpu().pin_memory()
    h_q = [torch.empty(q_out.shape, dtype=q_out.dtype).pin_memory() for _ in range(2)]
    cstream = torch.cuda.Stream()
    evs = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in_ready", "in_free", "out_ready", "out_done")}

    def e2e_run(n):
        def copy_in(i):
            b = i % 2
            with torch.cuda.stream(cstream):
                if i >= 2:
                    cstream.wait_event(evs["in_free"][b])
                d_x[b].copy_(h_x, non_blocking=True)
                evs["in_ready"][b].record(cstream)
        copy_in(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                copy_in(i + 1)
            comp.wait_event(evs["in_ready"][b])
            if i >= 2:
                comp.wait_event(evs["out_done"][b])
            graphs[b].replay()
            evs["in_free"][b].record(comp)
            evs["out_ready"][b].record(comp)
            with torch.cuda.stream(cstream):
                cstream.wait_event(evs["out_ready"][b])
                h_q[b].copy_(d_q[b], non_blocking=True)
                evs["out_done"][b].record(cstream)
        comp.wait_event(evs["out_done"][(n - 1) % 2])

    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    cstream.wait_stream(comp)
    e2e_run(args.steps)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    pool.raise_on_status()
    del graphs
    launches = launches_per_step * args.steps

    prefill = tps > 1
    ms_step = ms_total / args.steps
    flops, nbytes = qkv_flops(w, n_tok), qkv_bytes(w, n_tok)
    if prefill:
        unit, per_launch, peak, peak_kind = "TFLOP/s", flops / 1e12, 1590.0, "fallback"
        pk = REPO / "MEASURED_PEAKS.json"
        if pk.exists():
            try:
                peak, peak_kind = float(json.loads(pk.read_text())["bf16_tflops"]), "measured"
            except Exception:
                pass
    else:
        unit, per_launch = "GB/s", nbytes / 1e9
        peak, peak_kind = measured_peak_gbs()
    value = world * L * per_launch / (ms_total * 1e-3 / args.steps)
    e2e_value = world * L * per_launch / (e2e_ms * 1e-3 / args.steps)
    achieved = per_launch / (launch_ms * 1e-3)
    res = {
        "metric": (("attention output projection (o_proj) " if oproj else
                    "fused q/k/v projection + QK-norm + RoPE + KV append ") +
                   ("TFLOP/s" if prefill else "GB/s (weights + activations)")),
        "value": round(value, 2),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 x fp16 (hi + lo)" if oproj else "bf16",
        "data": ("synthetic (seeded N(0,1) fp32 attention outputs, N(0,1/in) fp16 weights)" if oproj else
                 "synthetic (seeded N(0,1) hidden states, N(0,1/hidden) weights)"),
        "tok_per_s": round(world * n_tok / (ms_step * 1e-3), 1),
        "config": {
            "workload": (f"{args.workload}: {w['model']} {L} layers, o_proj [{hq * d} -> {hidden}] fp16 weights, "
                         f"fp32 attention output of {B} sequences x {tps} token(s) per step, one sckv_o_proj per "
                         f"layer (fp32 result)" if oproj else
                         f"{args.workload}: {w['model']} {L} layers, hidden {hidden}, {hq}q/{H}kv heads x d{d}, "
                         f"per-head QK-norm, RoPE, bf16 pool; {B} sequences x {tps} new token(s) at position "
                         f"{ctx0} per step, one sckv_qkv_append per layer"),
            "global_batch": world * n_tok,
            "seq_len": tps,
            "parallelism": f"sequence-sharded x{world}",
            "l2": "weights of all layers (%.1f GB) >> L2; each layer's weights are read once per step"
                  % (L * 2 * (hq * d * hidden if oproj else (hq + 2 * H) * d * hidden) / 1e9),
        },
        "e2e": {"value": round(e2e_value, 2), "unit": unit,
                "h2d_bytes_per_step": int(h_x.numel() * h_x.element_size()),
                "d2h_bytes_per_step": int(h_q[0].numel() * h_q[0].element_size())},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor" if prefill else "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": unit, "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args.workload),
                     "peak_kind": peak_kind,
                     "kernel": ("split_hi_lo_kernel + qkv_append_kernel (plain mode) (+ qkv_finish_kernel when "
                                "in_features is split) per layer (CUDA-graph replay, step time / layers)" if oproj
                                else "qkv_append_kernel + rope_table_kernel (+ qkv_finish_kernel when the hidden "
                                     "dim is split) per layer (CUDA-graph replay, step time / layers)"),
                     ("flops_per_launch" if prefill else "bytes_per_launch"): int(flops if prefill else nbytes),
                     "avg_launch_ms": round(launch_ms, 4)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_qkv(w, prefill, budget_s=args.cpu_seconds)
    pool.close()
    return res


def cpu_baseline_qkv(w, prefill: bool, budget_s: float = 15.0):
    """The reference's NumPy projections + QK-norm + RoPE (oracle restatement of
    models/adapters.py:1167-1194) on one layer x 32 tokens, repeated for ~budget_s."""
    from oracle.kv_oracle import o_project, qk_norm_rope, qkv_project, rope_inv_freq

    rng = np.random.default_rng(0)
    n, hidden, hq, H, d = 32, w["hidden"], w["hq"], w["hkv"], w["d"]
    if w["kind"] == "oproj":
        # the reference's o_proj (models/adapters.py:1231): fp32 attn_out @ fp16 weights widened to fp32
        a = rng.standard_normal((n, hq * d)).astype(np.float32)
        wo = (rng.standard_normal((hidden, hq * d)) * (hq * d) ** -0.5).astype(np.float16)
        reps, t0 = 0, time.perf_counter()
        while True:
            o_project(a, wo)
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s or reps >= 1000:
                break
        if prefill:
            val, unit = reps * qkv_flops(w, n) / el / 1e12, "TFLOP/s"
        else:
            val, unit = reps * qkv_bytes(w, n) / el / 1e9, "GB/s"
        return {"value": round(val, 5), "unit": unit, "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
                or (os.cpu_count() or 1), "kind": "port",
                "sample": f"1 layer x {n} tokens (fp32 attention output, fp16 weights), {reps} reps in {el:.1f}s"}
    x = rng.standard_normal((n, hidden)).astype(np.float32)
    wq = (rng.standard_normal((hq * d, hidden)) * hidden ** -0.5).astype(np.float16)
    wk = (rng.standard_normal((H * d, hidden)) * hidden ** -0.5).astype(np.float16)
    wv = (rng.standard_normal((H * d, hidden)) * hidden ** -0.5).astype(np.float16)
    qw, kw = np.ones(d, np.float16), np.ones(d, np.float16)
    inv = rope_inv_freq(1e6, d)
    reps, t0 = 0, time.perf_counter()
    while True:
        q, k, v = qkv_project(x, wq, wk, wv, hq, H)
        qk_norm_rope(q, k, qw, kw, 1e-6, inv, 1.0, w["ctx"])
        v.astype(np.float16)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    if prefill:
        val, unit = reps * qkv_flops(w, n) / el / 1e12, "TFLOP/s"
    else:
        val, unit = reps * qkv_bytes(w, n) / el / 1e9, "GB/s"
    return {"value": round(val, 5), "unit": unit, "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
            or (os.cpu_count() or 1), "kind": "port",
            "sample": f"1 layer x {n} tokens (fp32 x, fp16 weights), {reps} reps in {el:.1f}s"}


# ----------------------------------------------------------------------------- continuous-batching mix
class MixState:
    """A PagedKVCache driven like a serving loop, with exact host-side
    accounting of the pool (ring / cached / pinned pages) so the 90 % eviction
    policy needs no device read on the step path."""

    def __init__(self, w, rank: int, max_steps: int):
        from synapcore_b200.paged_cache import PagedKVCache
        from synapcore_b200.pool import to_device

        self.to_device = to_device

        self.w = w
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.rng = np.random.default_rng(300 + rank)
        L, hq, hkv, d = w["layers"], w["hq"], w["hkv"], w["d"]
        self.L = L
        lo, hi = w["ctx"]
        self.max_new = w["new_per_step"] * w["prompt"][1]
        max_blocks = (hi + w["prompt"][1] + max_steps + 2 * PAGE) // PAGE + 1
        self.max_rows = w["batch"] + w["new_per_step"] + 1
        self.P = int(w["pool_pages"])
        # retired sequences keep their pages cached; the cache evicts them LRU
        # first whenever more than evict_at of the pool is allocated
        self.cache = PagedKVCache(L, hkv, d, self.P, self.max_rows, max_blocks, w["kv"], device=dev,
                                  evict_watermark=w["evict_at"])
        g = torch.Generator(device=dev)
        g.manual_seed(4321 + rank)
        self.src_k = torch.randn((L, hi, hkv, d), generator=g, device=dev).to(w["qdt"])
        self.src_v = torch.randn((L, hi, hkv, d), generator=g, device=dev).to(w["qdt"])
        # a step's prompt inputs, flat so that [L, tot, ...] views are contiguous
        self.pre_k = torch.randn(L * self.max_new * hkv * d, generator=g, device=dev).to(w["qdt"])
        self.pre_v = torch.randn(L * self.max_new * hkv * d, generator=g, device=dev).to(w["qdt"])
        self.pre_q = torch.randn(L * self.max_new * hq * d, generator=g, device=dev).to(w["qdt"])
        self.out_pre = torch.empty((self.max_new, hq, d), dtype=w["qdt"], device=dev)
        self.q_dec = torch.randn((L, self.max_rows, hq, d), generator=g, device=dev).to(w["qdt"])
        self.k_dec = torch.randn((L, self.max_rows, hkv, d), generator=g, device=dev).to(w["qdt"])
        self.v_dec = torch.randn((L, self.max_rows, hkv, d), generator=g, device=dev).to(w["qdt"])
        self.out_dec = torch.empty((self.max_rows, hq, d), dtype=w["qdt"], device=dev)
        self.forked = set()
        self.next_id = 0
        c = self.cache
        # the shared prefix: written once, held by one extra pin
        npre = w["prefix"]
        c.add_sequence("prefix")
        c.append_prefill("prefix", self.src_k[:, :npre], self.src_v[:, :npre])
        self.prefix_pages = c.page_ids("prefix")
        c.pool.pin_pages(torch.tensor(self.prefix_pages, dtype=torch.int32, device=dev), +1)
        c.remove_sequence("prefix")
        n_fork = int(round(w["batch"] * w["fork_frac"]))
        forks = set(self.rng.choice(w["batch"], size=n_fork, replace=False).tolist())
        for i in range(w["batch"]):
            sid = self._new_id()
            c.add_sequence(sid)
            if i in forks:
                c.share_prefix(sid, self.prefix_pages)
                self.forked.add(sid)
                own = int(self.rng.integers(lo, hi - npre + 1))
            else:
                own = int(self.rng.integers(lo, hi + 1))
            c.append_prefill(sid, self.src_k[:, :own], self.src_v[:, :own])
        torch.cuda.synchronize()
        self.check_accounting()
        self.events = []

    def _new_id(self):
        self.next_id += 1
        return self.next_id

    def check_accounting(self):
        """The allocator recorded no error (an exhausted pool would show here)."""
        self.cache.check()

    def step(self, timing=None, io=None):
        """One serving step; returns (algorithmic bytes, decode tokens, prefill tokens, launch bytes)."""
        w, c, L = self.w, self.cache, self.L
        hkv, hq, d = w["hkv"], w["hq"], w["d"]
        eb = kv_bytes_per_elem(w["kv"])
        # 1. retire sequences (their pages stay cached for prefix reuse)
        live = list(c.seq_at)
        gone = [live[i] for i in self.rng.choice(len(live), size=w["new_per_step"], replace=False)]
        for sid in gone:
            self.forked.discard(sid)
        c.remove_sequences(gone, keep_cached=True)
        # 2. eviction policy: the cache evicts LRU cached pages on the device
        #    until at most evict_at of the pool is allocated
        c.enforce_watermark()
        # 3. admit new prompts: forks share the prefix pages, all prefill causally
        plo, phi = w["prompt"]
        new_ids, T, starts = [], [], []
        for _ in range(w["new_per_step"]):
            sid = self._new_id()
            c.add_sequence(sid)
            if self.rng.random() < w["fork_frac"]:
                c.share_prefix(sid, self.prefix_pages)
                self.forked.add(sid)
            t = int(self.rng.integers(plo, phi + 1))
            new_ids.append(sid)
            T.append(t)
            starts.append(c.length(sid))
        cu = np.concatenate([[0], np.cumsum(T)]).astype(np.int64)
        tot = int(cu[-1])
        if io is not None:
            io["pre_in"](tot)
        pk = self.pre_k[:L * tot * hkv * d].view(L, tot, hkv, d)
        pv = self.pre_v[:L * tot * hkv * d].view(L, tot, hkv, d)
        pq = self.pre_q[:L * tot * hq * d].view(L, tot, hq, d)
        c.append_prefill_batch(new_ids, pk, pv, cu.tolist())
        meta = self.to_device(np.concatenate([cu, starts]).astype(np.int32), torch.int32, self.dev)
        cu_d, st_d = meta[:len(T) + 1], meta[len(T) + 1:]
        for l in range(L):
            if timing is not None:
                timing["pre"].append(torch.cuda.Event(enable_timing=True))
                timing["pre"][-1].record()
            c.prefill_attention_batch(l, new_ids, pq[l], cu_d, st_d, out=self.out_pre[:tot])
            if timing is not None:
                timing["pre"].append(torch.cuda.Event(enable_timing=True))
                timing["pre"][-1].record()
        # 4. decode one token for every live sequence
        n = c.n_live
        if io is not None:
            io["dec_in"](n)
        c.decode_reserve(n)
        fused = w["kv"] in ("fp16", "bf16")  # the append runs inside the decode launch
        for l in range(L):
            if not fused:
                c.decode_append(l, self.k_dec[l, :n], self.v_dec[l, :n], n)
            if timing is not None:
                timing["dec"].append(torch.cuda.Event(enable_timing=True))
                timing["dec"][-1].record()
            if fused:
                c.decode_append_attention(l, self.q_dec[l, :n], self.k_dec[l, :n], self.v_dec[l, :n], n,
                                          out=self.out_dec[:n])
            else:
                c.decode_attention(l, self.q_dec[l, :n], n, out=self.out_dec[:n])
            if timing is not None:
                timing["dec"].append(torch.cuda.Event(enable_timing=True))
                timing["dec"][-1].record()
        if io is not None:
            io["out"](n, tot)
        # algorithmic bytes
        ctx = np.asarray(c.lengths[:n], np.int64)
        dec = int(ctx.sum()) * hkv * d * 2 * eb + int(((ctx + PAGE - 1) // PAGE).sum()) * 4 + n * hq * d * 2 * 2
        app_tok = hkv * d * 2 * (2 + eb)          # read the new K/V row, write it into its page
        pre_ctx = np.asarray(starts, np.int64) + np.asarray(T, np.int64)
        pre = int(pre_ctx.sum()) * hkv * d * 2 * eb + tot * hq * d * 2 * 2
        total = L * (dec + pre + (n + tot) * app_tok)
        pre_flops = L * 4 * hq * d * int(sum(t * s + t * (t + 1) // 2 for t, s in zip(T, starts)))
        if fused:
            dec += n * app_tok  # the timed decode launch also stores the new rows
        return total, n, tot, dec, pre, pre_flops


def bench_mix(args, w, world, rank, local):
    from synapcore_b200 import _native as N

    total_steps = args.warmup + 2 * args.steps + max(1, args.warmup)
    st = MixState(w, rank, total_steps)
    for _ in range(args.warmup):
        st.step()
    torch.cuda.synchronize()
    st.cache.check()
    st.check_accounting()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    timing = {"pre": [], "dec": []}
    barrier(world)
    torch.cuda.synchronize()
    l0 = N.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tot_bytes = dec_tok = pre_tok = 0
    dec_bytes, pre_bytes, pre_flops = [], [], []
    e0.record()
    for _ in range(args.steps):
        b, n, t, db, pb, pf = st.step(timing)
        tot_bytes += b
        dec_tok += n
        pre_tok += t
        dec_bytes.append(db)
        pre_bytes.append(pb)
        pre_flops.append(pf)
    e1.record()
    torch.cuda.synchronize()
    launches = N.launch_count() - l0
    barrier(world)
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    dec_ms = [timing["dec"][i].elapsed_time(timing["dec"][i + 1]) for i in range(0, len(timing["dec"]), 2)]
    pre_ms = [timing["pre"][i].elapsed_time(timing["pre"][i + 1]) for i in range(0, len(timing["pre"]), 2)]
    st.cache.check()
    st.check_accounting()

    # ---- e2e: the step's new K/V and queries copied from pinned host memory,
    # the last layer's outputs read back
    L, hq, hkv, d = w["layers"], w["hq"], w["hkv"], w["d"]
    h_pre = [(x.cpu().pin_memory(), x, per) for x, per in ((st.pre_k, hkv * d), (st.pre_v, hkv * d),
                                                          (st.pre_q, hq * d))]
    h_dec = [(x.cpu().pin_memory(), x) for x in (st.q_dec, st.k_dec, st.v_dec)]
    h_out_dec = torch.empty_like(st.out_dec, device="cpu").pin_memory()
    h_out_pre = torch.empty_like(st.out_pre, device="cpu").pin_memory()
    moved = {"h2d": 0, "d2h": 0}

    def pre_in(tot):
        for h, dd, per in h_pre:
            m = L * tot * per
            dd[:m].copy_(h[:m], non_blocking=True)
            moved["h2d"] += m * h.element_size()

    def dec_in(n):
        for h, dd in h_dec:
            for l in range(L):
                dd[l, :n].copy_(h[l, :n], non_blocking=True)
            moved["h2d"] += L * h[0, :n].numel() * h.element_size()

    def out(n, tot):
        h_out_dec[:n].copy_(st.out_dec[:n], non_blocking=True)
        h_out_pre[:tot].copy_(st.out_pre[:tot], non_blocking=True)
        moved["d2h"] += (n + tot) * hq * d * h_out_dec.element_size()

    io = {"pre_in": pre_in, "dec_in": dec_in, "out": out}
    for _ in range(max(1, args.warmup)):
        st.step(io=io)
    torch.cuda.synchronize()
    moved = {"h2d": 0, "d2h": 0}
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_bytes = 0
    f0.record()
    for _ in range(args.steps):
        e2e_bytes += st.step(io=io)[0]
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
    st.cache.check()
    st.check_accounting()

    peak, peak_kind = measured_peak_gbs()
    ms_step = ms_total / args.steps
    value = world * tot_bytes / (ms_total * 1e-3) / 1e9
    dec_avg_ms = max_over_ranks(float(np.mean(dec_ms)), world)
    pre_avg_ms = max_over_ranks(float(np.mean(pre_ms)), world)
    dec_launch_bytes = float(np.mean(dec_bytes))
    achieved = dec_launch_bytes / (dec_avg_ms * 1e-3) / 1e9
    tflops = float(np.mean(pre_flops)) / L / (pre_avg_ms * 1e-3) / 1e12
    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    tc_peak = float(peaks.get("bf16_tflops", 1590.0))
    res = {
        "metric": "paged decode-attn KV GB/s (% HBM peak) and decode tok/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w["kv"],
        "data": "synthetic (seeded N(0,1) K/V/Q, random prompt lengths, retirements and forks)",
        "tok_per_s": round(world * dec_tok / (ms_total * 1e-3), 1),
        "prefill_tok_per_s": round(world * pre_tok / (ms_total * 1e-3), 1),
        "pct_hbm_peak": round(100.0 * value / world / peak, 2),
        "config": {
            "workload": f"{args.workload}: continuous batching, {w['model']} shape {w['layers']}L x "
                        f"{w['hq']}q/{w['hkv']}kv heads x d{w['d']}, {w['kv']} KV, page 16; {w['batch']} live "
                        f"sequences/GPU ~U{list(w['ctx'])}, {int(w['fork_frac'] * 100)}% forked from a shared "
                        f"{w['prefix']}-token prefix; per step retire {w['new_per_step']}, admit "
                        f"{w['new_per_step']} prompts ~U{list(w['prompt'])} (causal prefill), decode all; "
                        f"LRU eviction above {int(w['evict_at'] * 100)}% of a {w['pool_pages']}-page pool",
            "global_batch": world * w["batch"],
            "seq_len": ctx_desc(w),
            "parallelism": f"sequence-sharded x{world} (independent pools)",
            "l2": "inputs larger than L2 (KV per decode launch >> 126 MB)",
        },
        "e2e": {"value": round(world * e2e_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(moved["h2d"] / args.steps),
                "d2h_bytes_per_step": int(moved["d2h"] / args.steps)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args.workload),
                     "peak_kind": peak_kind,
                     "kernel": ("decode_kernel with the fused append" if w["kv"] in ("fp16", "bf16") else
                                "decode_mma_kernel") + " (+combine) per layer launch",
                     "bytes_per_launch": int(dec_launch_bytes), "avg_launch_ms": round(dec_avg_ms, 4)},
        "prefill_roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                             "frac": round(tflops / tc_peak, 4),
                             "kernel": "prefill_tc_kernel (tcgen05) per layer launch",
                             "flops_per_launch": int(np.mean(pre_flops) / L), "avg_launch_ms": round(pre_avg_ms, 4)},
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(w, budget_s=args.cpu_seconds)
    st.cache.pool.close()
    return res


# ----------------------------------------------------------------------------- CPU (reference) arm
def cpu_sample(w, n_seqs: int, ctx: int, seed: int = 0):
    """A bounded slice of the workload on the host: one layer x n_seqs."""
    rng = np.random.default_rng(seed)
    hq, hkv, d = w["hq"], w["hkv"], w["d"]
    q = rng.standard_normal((n_seqs, hq, d)).astype(np.float32)
    k = rng.standard_normal((n_seqs, hkv, ctx, d)).astype(np.float16)
    v = rng.standard_normal((n_seqs, hkv, ctx, d)).astype(np.float16)
    return q, k, v


def cpu_baseline(w, budget_s: float = 15.0):
    """The reference's NumPy decode SDPA (oracle port of models/adapters.py:1209-1229)
    on one layer x 8 sequences at the workload's context, repeated for ~budget_s."""
    from oracle.kv_oracle import sdpa_decode

    n_seqs = 8
    T = mean_ctx(w)
    q, k, v = cpu_sample(w, n_seqs, T)
    if w["kv"] == "fp8_e4m3":
        from oracle.kv_oracle import fp8_decode, fp8_encode

        s = (np.abs(k.astype(np.float32)).max(axis=(2, 3), keepdims=True) / 448).astype(np.float32)
        kc = fp8_encode(k.astype(np.float32) / s)
        vc = fp8_encode(v.astype(np.float32) / s)
    per_call_bytes = n_seqs * T * w["hkv"] * w["d"] * 2 * kv_bytes_per_elem(w["kv"])
    reps, t0 = 0, time.perf_counter()
    while True:
        for b in range(n_seqs):
            if w["kv"] == "fp8_e4m3":
                kk = fp8_decode(kc[b]) * s[b]
                vv = fp8_decode(vc[b]) * s[b]
                sdpa_decode(q[b], kk, vv)
            else:
                sdpa_decode(q[b], k[b], v[b])
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    gbs = reps * per_call_bytes / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
            or (os.cpu_count() or 1), "kind": "port",
            "sample": f"1 layer x {n_seqs} seqs x ctx {T} ({w['kv']} KV), {reps} reps in {el:.1f}s; "
                      f"tok/s extrapolated to the full step = "
                      f"{w['batch'] * gbs * 1e9 / (w['layers'] * attn_bytes_per_launch(w, [T] * w['batch'])):.3f}"}


def reference_code_baseline(w, budget_s: float = 5.0):
    """The reference's own decode code, when an installed copy is importable
    from baseline/_ref: ModularAttentionEngine.forward_numpy
    (models/adapters.py:1148-1231) for one token of one sequence and one layer
    at the workload's context, its fp16 cache growing by np.concatenate as in
    the reference. The call includes the reference's q/k/v/o projections,
    which the device metric does not count, so this is reported beside the
    SDPA-only port, not in its place. None when no copy is installed."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "models" / "adapters.py").exists():
        return None
    sys.path.insert(0, str(ref))
    try:
        from models import adapters as ad
    except Exception as e:  # the installed copy does not import here
        return {"unavailable": f"baseline/_ref does not import: {type(e).__name__}: {e}"[:200]}
    finally:
        sys.path.remove(str(ref))
    hq, hkv, d = w["hq"], w["hkv"], w["d"]
    hidden = hq * d
    T = mean_ctx(w)
    cfg = {"model_type": "olmoe", "num_hidden_layers": 1, "num_experts": 8, "num_experts_per_tok": 2,
           "hidden_size": hidden, "intermediate_size": hidden * 2, "num_attention_heads": hq,
           "num_key_value_heads": hkv, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 10000.0}
    eng = ad.ModularAttentionEngine(ad.OLMoEAdapter(cfg).spec)
    rng = np.random.default_rng(0)
    wq = (rng.standard_normal((hidden, hidden)) * 0.02).astype(np.float16)
    wk = (rng.standard_normal((hkv * d, hidden)) * 0.02).astype(np.float16)
    wv = (rng.standard_normal((hkv * d, hidden)) * 0.02).astype(np.float16)
    wo = (rng.standard_normal((hidden, hidden)) * 0.02).astype(np.float16)
    kk = [rng.standard_normal((1, hkv, T, d)).astype(np.float16)]
    vv = [rng.standard_normal((1, hkv, T, d)).astype(np.float16)]
    x = rng.standard_normal((1, 1, hidden)).astype(np.float32)
    calls, nbytes, t0 = 0, 0, time.perf_counter()
    while True:
        ctx = kk[0].shape[2] + 1
        eng.forward_numpy(x, wq, wk, wv, wo, kv_cache_k=kk, kv_cache_v=vv, layer_idx=0, pos_offset=ctx - 1)
        calls += 1
        nbytes += ctx * hkv * d * 2 * 2
        el = time.perf_counter() - t0
        if el >= budget_s or calls >= 2000:
            break
    gbs = nbytes / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "reference",
            "sample": f"forward_numpy, 1 layer x 1 seq x ctx {T} (fp16 cache; includes its q/k/v/o "
                      f"projections and concatenate append), {calls} calls in {el:.1f}s"}


def cpu_baseline_prefill(w, budget_s: float = 15.0):
    """The reference's NumPy causal prompt pass (oracle restatement of
    models/adapters.py:1209-1229 with its -1e9 mask) on one layer of one
    256-token prompt, repeated for ~budget_s."""
    from oracle.kv_oracle import sdpa_prefill

    rng = np.random.default_rng(0)
    T, hq, hkv, d = 256, w["hq"], w["hkv"], w["d"]
    q = rng.standard_normal((T, hq, d)).astype(np.float32)
    k = rng.standard_normal((hkv, T, d)).astype(np.float16)
    v = rng.standard_normal((hkv, T, d)).astype(np.float16)
    reps, t0 = 0, time.perf_counter()
    while True:
        sdpa_prefill(q, k, v, 0)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    tflops = reps * 4 * hq * d * (T * (T + 1) // 2) / el / 1e12
    return {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": int(os.environ.get("OMP_NUM_THREADS", "0") or 0)
            or (os.cpu_count() or 1), "kind": "port",
            "sample": f"1 layer x one {T}-token prompt, {reps} reps in {el:.1f}s"}


def bench_reference(args, w, world, rank):
    if rank != 0:
        return None
    steps = []
    kind = w.get("kind")
    qkv = kind in ("qkv", "oproj")
    budget = args.cpu_seconds / max(1, args.steps)
    for i in range(args.warmup + args.steps):
        if qkv:
            r = cpu_baseline_qkv(w, w["tokens_per_seq"] > 1, budget_s=budget)
        elif kind == "prefill":
            r = cpu_baseline_prefill(w, budget_s=budget)
        elif kind == "paging":
            r = cpu_baseline_gather(w, budget_s=budget)
        elif kind == "layer":
            r = cpu_baseline_layer(w, budget_s=budget)
        else:
            r = cpu_baseline(w, budget_s=budget)
        if i >= args.warmup:
            steps.append(r["value"])
    val = float(np.mean(steps))
    cores = os.cpu_count() or 1
    if kind == "layer":
        return {"metric": "whole attention layer decode tok/s (projections, FP8 paged attention, o_proj)",
                "impl": "reference", "value": round(val, 6), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
                "config": {"workload": f"{args.workload}: reference NumPy forward_numpy on a bounded host sample",
                           "parallelism": "host cores"},
                "cpu_baseline": {"value": round(val, 6), "unit": "tok/s", "cores": cores, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(val, 6), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if kind in ("prefill", "paging"):
        return {"metric": ("causal prefill attention TFLOP/s (counting the causal half)" if kind == "prefill"
                           else "paging kernels GB/s (append + gather + CoW page copy)"),
                "impl": "reference", "value": round(val, 6), "unit": r["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": w["kv"], "data": "synthetic (seeded)",
                "config": {"workload": f"{args.workload}: reference NumPy path on a bounded host sample",
                           "parallelism": "host cores"},
                "cpu_baseline": {"value": round(val, 6), "unit": r["unit"], "cores": cores, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(val, 6), "unit": r["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if qkv:
        return {"metric": (("attention output projection (o_proj) " if kind == "oproj" else
                            "fused q/k/v projection + QK-norm + RoPE + KV append ") +
                           ("TFLOP/s" if w["tokens_per_seq"] > 1 else "GB/s (weights + activations)")),
                "impl": "reference", "value": round(val, 5), "unit": r["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
                "config": {"workload": f"{args.workload}: reference NumPy "
                                       f"{'o_proj' if kind == 'oproj' else 'projections + QK-norm + RoPE'} on a "
                                       f"bounded host sample", "parallelism": "host cores"},
                "cpu_baseline": {"value": round(val, 5), "unit": r["unit"], "cores": cores, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(val, 5), "unit": r["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return {
        "metric": "paged decode-attn KV GB/s (% HBM peak) and decode tok/s",
        "impl": "reference",
        "value": round(val, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w["kv"],
        "data": "synthetic (seeded)",
        "config": {"workload": f"{args.workload}: reference NumPy decode SDPA on a bounded host sample",
                   "global_batch": w["batch"], "seq_len": ctx_desc(w), "parallelism": "host cores"},
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"per step: 1 layer x 8 seqs x ctx {mean_ctx(w)}, ~{args.cpu_seconds / max(1, args.steps):.1f}s"},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_code": reference_code_baseline(w, budget_s=min(5.0, args.cpu_seconds)),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="olmoe")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layout", choices=["seq", "heads"], default="seq",
                    help="multi-GPU layout: sequence sharding (default) or KV-head sharding")
    ap.add_argument("--exchange", choices=["nvlink", "nccl"], default="nvlink",
                    help="KV-head sharding's output exchange: fused into the decode over NVLink peer stores "
                         "(default) or a separate NCCL all-gather")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    # stdout carries exactly the one JSON line: anything a library prints on
    # file descriptor 1 (e.g. NCCL's version banner when a communicator
    # comes up) goes to stderr, and the line is written to the saved stdout
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            res = bench_reference(args, w, world, rank)
        elif w.get("kind") == "mix":
            res = bench_mix(args, w, world, rank, local)
        elif w.get("kind") in ("qkv", "oproj"):
            res = bench_qkv(args, w, world, rank, local)
        elif w.get("kind") == "layer":
            res = bench_layer(args, w, world, rank, local)
        elif w.get("kind") == "prefill":
            res = bench_prefill(args, w, world, rank, local)
        elif w.get("kind") == "paging":
            res = bench_paging(args, w, world, rank, local)
        else:
            res = bench_ours(args, w, world, rank, local)
        if rank == 0 and res is not None:
            sys.stdout.flush()
            os.write(json_fd, (json.dumps(res) + "\n").encode())
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
