"""Two-GPU runs (skipped with fewer than 2 GPUs): KV-head-sharded decode
attention with the NCCL all-gather equals the single-GPU result, and
sequence-sharded pools run independently on each GPU."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=0):
    rng = np.random.default_rng(seed)
    L, hq, hkv, D, P = 2, 16, 4, 128, 96
    ctx = [37, 200, 513, 16]
    k = rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)
    v = rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)
    mb = max((c + 15) // 16 for c in ctx)
    bt = np.stack([rng.choice(P, size=mb, replace=False) for _ in ctx]).astype(np.int32)
    q = rng.standard_normal((len(ctx), hq, D)).astype(np.float16)
    return L, hq, hkv, D, P, ctx, k, v, bt, q


def _worker(rank, world, port, out_path):
    import torch.distributed as dist

    from synapcore_b200.distributed import HeadShardedOutput, head_range, query_head_range
    from synapcore_b200.pool import KVPool

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        L, hq, hkv, D, P, ctx, k, v, bt, q = _case()
        kvr = head_range(hkv, world, rank)
        qr = query_head_range(hq, hkv, world, rank)
        pool = KVPool(L, len(kvr), D, P, "fp16", device=dev)
        ids = torch.arange(P, dtype=torch.int32, device=dev)
        pool.write_pages(ids, torch.from_numpy(np.ascontiguousarray(k[:, :, kvr.start:kvr.stop])).to(dev),
                         torch.from_numpy(np.ascontiguousarray(v[:, :, kvr.start:kvr.stop])).to(dev))
        bt_d = torch.from_numpy(bt).to(dev)
        ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
        q_d = torch.from_numpy(np.ascontiguousarray(q[:, qr.start:qr.stop])).to(dev)
        gather = HeadShardedOutput(world)
        outs = []
        for layer in range(L):
            local = pool.decode_attn(layer, q_d, bt_d, ctx_d, out_dtype=torch.float32)
            outs.append(gather.gather(local))
        torch.cuda.synchronize()
        pool.raise_on_status()
        if rank == 0:
            np.save(out_path, torch.stack(outs).cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_head_sharded_decode_equals_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from synapcore_b200.pool import KVPool

    out = tmp_path / "sharded.npy"
    mp.start_processes(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True, start_method="spawn")
    sharded = np.load(out)
    L, hq, hkv, D, P, ctx, k, v, bt, q = _case()
    dev = torch.device("cuda", 0)
    pool = KVPool(L, hkv, D, P, "fp16", device=dev)
    pool.write_pages(torch.arange(P, dtype=torch.int32, device=dev), torch.from_numpy(k).to(dev),
                     torch.from_numpy(v).to(dev))
    bt_d = torch.from_numpy(bt).to(dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    for layer in range(L):
        full = pool.decode_attn(layer, torch.from_numpy(q).to(dev), bt_d, ctx_d, out_dtype=torch.float32)
        ref = full.cpu().numpy()
        got = sharded[layer]
        assert np.max(np.abs(got - ref)) <= 2e-3 * np.max(np.abs(ref))


def _exchange_worker(rank, world, port, out_path, steps=3, graph=False):
    """KV-head-sharded decode with the exchange fused into the kernel: every
    rank runs its heads, waits for every rank's flag, and rank 0 records the
    full output of each (step, layer). graph=True captures one step with
    device-counter epochs in a CUDA graph and replays it per step."""
    import torch.distributed as dist

    from synapcore_b200.distributed import HeadShardedExchange, head_range, query_head_range
    from synapcore_b200.pool import KVPool

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ex = None
    try:
        L, hq, hkv, D, P, ctx, k, v, bt, q = _case()
        kvr = head_range(hkv, world, rank)
        qr = query_head_range(hq, hkv, world, rank)
        pool = KVPool(L, len(kvr), D, P, "fp16", device=dev)
        ids = torch.arange(P, dtype=torch.int32, device=dev)
        pool.write_pages(ids, torch.from_numpy(np.ascontiguousarray(k[:, :, kvr.start:kvr.stop])).to(dev),
                         torch.from_numpy(np.ascontiguousarray(v[:, :, kvr.start:kvr.stop])).to(dev))
        bt_d = torch.from_numpy(bt).to(dev)
        ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
        ex = HeadShardedExchange(pool, world, rank, L, len(ctx), hq, torch.float32)
        outs = []
        q_loc = torch.from_numpy(np.ascontiguousarray(q[:, qr.start:qr.stop])).to(dev)
        q_d = q_loc.clone()
        g = None
        if graph:
            # every rank makes the same eager call first (launch set-up outside
            # the capture), then captures the step
            ex.decode(0, q_d, bt_d, ctx_d, 0)
            ex.wait(0)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for layer in range(L):
                    ex.decode(layer, q_d, bt_d, ctx_d, 0)
                    ex.wait(0)
        for step in range(steps):
            # each step scales q differently, so a stale slice would show
            q_d.copy_(q_loc * (1.0 + 0.25 * step))
            if g is not None:
                g.replay()
                for layer in range(L):
                    outs.append(ex.output(layer, len(ctx)).clone())
                # the whole step is read after its last signal: keep the other
                # rank's next step from rewriting the slices until then
                torch.cuda.synchronize()
                dist.barrier()
                continue
            for layer in range(L):
                epoch = step * L + layer + 1
                ex.decode(layer, q_d, bt_d, ctx_d, epoch)
                ex.wait(epoch)
                outs.append(ex.output(layer, len(ctx)).clone())
        torch.cuda.synchronize()
        pool.raise_on_status()
        assert ex.status()[0] == 0
        if rank == 0:
            np.save(out_path, torch.stack(outs).cpu().numpy())
        del g
        dist.barrier()
    finally:
        if ex is not None:
            torch.cuda.synchronize()
            dist.barrier()
            ex.close()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("graph", [False, True])
def test_head_sharded_exchange_equals_single_gpu(tmp_path, graph):
    """Two ranks, fused NVLink exchange (explicit epochs, or device-counter
    epochs in a replayed CUDA graph): every (step, layer) output equals the
    single-GPU decode of all heads."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from synapcore_b200.pool import KVPool

    out = tmp_path / "exchange.npy"
    steps = 3
    mp.start_processes(_exchange_worker, args=(2, _free_port(), str(out), steps, graph), nprocs=2, join=True,
                       start_method="spawn")
    got_all = np.load(out)
    L, hq, hkv, D, P, ctx, k, v, bt, q = _case()
    dev = torch.device("cuda", 0)
    pool = KVPool(L, hkv, D, P, "fp16", device=dev)
    pool.write_pages(torch.arange(P, dtype=torch.int32, device=dev), torch.from_numpy(k).to(dev),
                     torch.from_numpy(v).to(dev))
    bt_d = torch.from_numpy(bt).to(dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    i = 0
    for step in range(steps):
        qs = (torch.from_numpy(q) * (1.0 + 0.25 * step)).to(dev)
        for layer in range(L):
            ref = pool.decode_attn(layer, qs, bt_d, ctx_d, out_dtype=torch.float32).cpu().numpy()
            assert np.max(np.abs(got_all[i] - ref)) <= 2e-3 * np.max(np.abs(ref)), (step, layer)
            i += 1


def test_exchange_single_rank_and_bounded_wait(cuda_device):
    """One rank (its own buffer is the only target): the exchange decode
    equals sckv_decode_attn bit for bit in fp32, for MHA and GQA pools; a wait
    for an epoch nobody signals gives up after its limit, records
    SCKV_ERR_TIMEOUT (detail = the late rank) and leaves the context usable."""
    import torch.distributed as dist

    from synapcore_b200 import _native as N
    from synapcore_b200.distributed import HeadShardedExchange
    from synapcore_b200.pool import KVPool

    own_group = not dist.is_initialized()
    if own_group:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        for hq, hkv in ((16, 16), (16, 4)):
            L, D, P = 2, 128, 96
            rng = np.random.default_rng(3)
            ctx = [37, 700, 513, 16, 1]
            mb = max((c + 15) // 16 for c in ctx)
            bt = torch.from_numpy(np.stack([rng.choice(P, size=mb, replace=False) for _ in ctx]).astype(np.int32))
            pool = KVPool(L, hkv, D, P, "fp16", device=cuda_device)
            kv = torch.from_numpy(rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)).to(cuda_device)
            pool.write_pages(torch.arange(P, dtype=torch.int32, device=cuda_device), kv, kv * 0.5)
            bt_d = bt.to(cuda_device)
            ctx_d = torch.tensor(ctx, dtype=torch.int32, device=cuda_device)
            q = torch.from_numpy(rng.standard_normal((len(ctx), hq, D)).astype(np.float16)).to(cuda_device)
            ex = HeadShardedExchange(pool, 1, 0, L, 8, hq, torch.float32)
            for layer in range(L):
                ex.decode(layer, q, bt_d, ctx_d, epoch=layer + 1)
                ex.wait(layer + 1)
                ref = pool.decode_attn(layer, q, bt_d, ctx_d, out_dtype=torch.float32)
                torch.cuda.synchronize()
                assert torch.equal(ex.output(layer, len(ctx)), ref)
            assert ex.status()[0] == 0
            ex.wait(99, limit_us=20000)  # nothing will ever signal epoch 99
            torch.cuda.synchronize()
            code, detail, kernel, _ = ex.status(clear=True)
            assert code == N.SCKV_ERR_TIMEOUT and detail == 0
            assert ex.status()[0] == 0
            pool.raise_on_status()
            # the context still works
            again = pool.decode_attn(0, q, bt_d, ctx_d, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.isfinite(again).all()
            ex.close()
            pool.close()
    finally:
        if own_group:
            dist.destroy_process_group()


def test_exchange_device_epochs_in_a_graph_with_fused_append(cuda_device):
    """One rank: a step of two layers (exchange decode with the new token's
    K/V appended in the same launch, then the wait), both taking their epochs
    from the device counter, captured once in a CUDA graph and replayed
    twice. Every replay equals sckv_append + sckv_decode_attn bit for bit,
    pool bytes included."""
    import torch.distributed as dist

    from synapcore_b200.distributed import HeadShardedExchange
    from synapcore_b200.pool import KVPool

    own_group = not dist.is_initialized()
    if own_group:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
        dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        L, hq, hkv, D, P = 2, 16, 4, 128, 120
        rng = np.random.default_rng(8)
        ctx0 = np.array([37, 700, 513, 16, 1, 255], np.int64)
        n_pages = (ctx0 + 2 + 15) // 16  # room for the two replayed tokens
        mb = int(n_pages.max())
        perm = rng.permutation(P)
        bt = np.zeros((len(ctx0), mb), np.int32)
        off = 0
        for b, n in enumerate(n_pages):  # private pages: nothing appended is read by another sequence
            bt[b, :n] = perm[off:off + n]
            off += n
        kv = torch.from_numpy(rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)).to(cuda_device)
        ref_pool = KVPool(L, hkv, D, P, "fp16", device=cuda_device)
        pool = KVPool(L, hkv, D, P, "fp16", device=cuda_device)
        for p_ in (ref_pool, pool):
            p_.write_pages(torch.arange(P, dtype=torch.int32, device=cuda_device), kv, kv * 0.5)
        bt_d = torch.from_numpy(bt).to(cuda_device)
        ctx_d = torch.tensor(ctx0 + 1, dtype=torch.int32, device=cuda_device)
        cu = torch.arange(len(ctx0) + 1, dtype=torch.int32, device=cuda_device)
        q = torch.from_numpy(rng.standard_normal((L, len(ctx0), hq, D)).astype(np.float16)).to(cuda_device)
        k_new = torch.from_numpy(rng.standard_normal((L, len(ctx0), hkv, D)).astype(np.float16)).to(cuda_device)
        v_new = torch.from_numpy(rng.standard_normal((L, len(ctx0), hkv, D)).astype(np.float16)).to(cuda_device)
        ex = HeadShardedExchange(pool, 1, 0, L, 8, hq, torch.float32)
        # one eager call sets up launch attributes outside the capture (it only reads the pool)
        ex.decode(0, q[0], bt_d, ctx_d, 0)
        ex.wait(0)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for layer in range(L):
                ex.decode(layer, q[layer], bt_d, ctx_d, 0, k_new=k_new[layer], v_new=v_new[layer])
                ex.wait(0)
        for step in range(2):
            g.replay()
            for layer in range(L):
                ref_pool.append(k_new[layer], v_new[layer], cu, ctx_d - 1, bt_d, layer0=layer)
                ref = ref_pool.decode_attn(layer, q[layer], bt_d, ctx_d, out_dtype=torch.float32)
                torch.cuda.synchronize()
                assert torch.equal(ex.output(layer, len(ctx0)), ref), (step, layer)
            assert torch.equal(pool.data, ref_pool.data), step
            ctx_d += 1  # the next step's token
        assert ex.status()[0] == 0
        pool.raise_on_status()
        del g
        ex.close()
        pool.close()
        ref_pool.close()
    finally:
        if own_group:
            dist.destroy_process_group()


def _append_case(seed=5, steps=3):
    """A pool case whose sequences own their pages (a page being appended into
    is read by no other sequence), plus each step's new K/V rows."""
    rng = np.random.default_rng(seed)
    L, hq, hkv, D, P = 2, 16, 4, 128, 96
    ctx0 = [37, 200, 130, 15]
    mb = max((c + steps + 15) // 16 for c in ctx0)
    k = rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)
    v = rng.standard_normal((P, L, hkv, 16, D)).astype(np.float16)
    bt = rng.permutation(P)[:len(ctx0) * mb].reshape(len(ctx0), mb).astype(np.int32)
    q = rng.standard_normal((len(ctx0), hq, D)).astype(np.float16)
    kn = rng.standard_normal((steps, L, len(ctx0), hkv, D)).astype(np.float16)
    vn = rng.standard_normal((steps, L, len(ctx0), hkv, D)).astype(np.float16)
    return L, hq, hkv, D, P, ctx0, k, v, bt, q, kn, vn


def _exchange_append_worker(rank, world, port, out_path, steps):
    """The KV-head-sharded step as the bench runs it: every layer's exchange
    decode appends the step's new token (this rank's kv heads) in the same
    launch, epochs come from the device counter, and the whole step is one
    replayed CUDA graph. Rank 0 records every (step, layer) output."""
    import torch.distributed as dist

    from synapcore_b200.distributed import HeadShardedExchange, head_range, query_head_range
    from synapcore_b200.pool import KVPool

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ex = None
    g = None
    try:
        L, hq, hkv, D, P, ctx0, k, v, bt, q, kn, vn = _append_case(steps=steps)
        kvr = head_range(hkv, world, rank)
        qr = query_head_range(hq, hkv, world, rank)
        pool = KVPool(L, len(kvr), D, P, "fp16", device=dev)
        pool.write_pages(torch.arange(P, dtype=torch.int32, device=dev),
                         torch.from_numpy(np.ascontiguousarray(k[:, :, kvr.start:kvr.stop])).to(dev),
                         torch.from_numpy(np.ascontiguousarray(v[:, :, kvr.start:kvr.stop])).to(dev))
        bt_d = torch.from_numpy(bt).to(dev)
        ctx_d = torch.tensor(ctx0, dtype=torch.int32, device=dev) + 1  # step 0's token sits at ctx0
        q_d = torch.from_numpy(np.ascontiguousarray(q[:, qr.start:qr.stop])).to(dev)
        k_d = torch.zeros((L, len(ctx0), len(kvr), D), dtype=torch.float16, device=dev)
        v_d = torch.zeros_like(k_d)
        ex = HeadShardedExchange(pool, world, rank, L, len(ctx0), hq, torch.float32)
        outs = []
        for step in range(steps):
            k_d.copy_(torch.from_numpy(np.ascontiguousarray(kn[step, :, :, kvr.start:kvr.stop])))
            v_d.copy_(torch.from_numpy(np.ascontiguousarray(vn[step, :, :, kvr.start:kvr.stop])))
            if g is None:
                # step 0 runs eagerly (launch set-up), then the step is captured
                for layer in range(L):
                    ex.decode(layer, q_d, bt_d, ctx_d, 0, k_new=k_d[layer], v_new=v_d[layer])
                    ex.wait(0)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for layer in range(L):
                        ex.decode(layer, q_d, bt_d, ctx_d, 0, k_new=k_d[layer], v_new=v_d[layer])
                        ex.wait(0)
            else:
                g.replay()
            for layer in range(L):
                outs.append(ex.output(layer, len(ctx0)).clone())
            torch.cuda.synchronize()
            dist.barrier()  # every rank has read this step before any rank starts the next
            ctx_d += 1
        pool.raise_on_status()
        assert ex.status()[0] == 0
        if rank == 0:
            np.save(out_path, torch.stack(outs).cpu().numpy())
        del g
        dist.barrier()
    finally:
        if ex is not None:
            torch.cuda.synchronize()
            dist.barrier()
            ex.close()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_head_sharded_graph_step_with_fused_append_equals_single_gpu(tmp_path):
    """Two ranks replaying the KV-head-sharded decode step with the new
    token's append fused into each layer's exchange decode: every (step,
    layer) output equals sckv_append + sckv_decode_attn of all heads on one
    GPU."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from synapcore_b200.pool import KVPool

    out = tmp_path / "exchange_append.npy"
    steps = 3
    mp.start_processes(_exchange_append_worker, args=(2, _free_port(), str(out), steps), nprocs=2, join=True,
                       start_method="spawn")
    got_all = np.load(out)
    L, hq, hkv, D, P, ctx0, k, v, bt, q, kn, vn = _append_case(steps=steps)
    dev = torch.device("cuda", 0)
    pool = KVPool(L, hkv, D, P, "fp16", device=dev)
    pool.write_pages(torch.arange(P, dtype=torch.int32, device=dev), torch.from_numpy(k).to(dev),
                     torch.from_numpy(v).to(dev))
    bt_d = torch.from_numpy(bt).to(dev)
    q_d = torch.from_numpy(q).to(dev)
    B = len(ctx0)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    i = 0
    for step in range(steps):
        ctx_d = torch.tensor([c + step + 1 for c in ctx0], dtype=torch.int32, device=dev)
        for layer in range(L):
            pool.append(torch.from_numpy(kn[step, layer]).to(dev), torch.from_numpy(vn[step, layer]).to(dev), cu,
                        ctx_d - 1, bt_d, layer0=layer)
            ref = pool.decode_attn(layer, q_d, bt_d, ctx_d, out_dtype=torch.float32).cpu().numpy()
            assert np.max(np.abs(got_all[i] - ref)) <= 2e-3 * np.max(np.abs(ref)), (step, layer)
            i += 1
    pool.raise_on_status()
