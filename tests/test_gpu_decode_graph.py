"""A decode step captured in a CUDA graph (DecodeStepGraph) produces the
same pages, block tables, allocator state and attention outputs, bit for
bit, as the same step run eagerly, over several steps that cross page
boundaries."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cache(dev, lengths, seed):
    from synapcore_b200.paged_cache import PagedKVCache

    rng = np.random.default_rng(seed)
    L, hkv, D = 2, 4, 128
    c = PagedKVCache(L, hkv, D, max_pages=256, max_seqs=8, max_blocks_per_seq=32, device=dev)
    for i, T in enumerate(lengths):
        c.add_sequence(i)
        x = torch.from_numpy(rng.standard_normal((L, T, hkv, D)).astype(np.float16)).to(dev)
        c.append_prefill(i, x, x * 0.5)
    return c


@pytest.mark.parametrize("hq", [4, 16])
def test_graph_replay_equals_eager_steps(cuda_device, hq):
    from synapcore_b200.paged_cache import DecodeStepGraph

    lengths = [15, 16, 47, 100, 1]
    eager, graphed = _cache(cuda_device, lengths, 1), _cache(cuda_device, lengths, 1)
    g = DecodeStepGraph(graphed, n_rows=len(lengths), num_q_heads=hq)
    rng = np.random.default_rng(2)
    L, n, hkv, D = 2, len(lengths), 4, 128
    for step in range(20):
        q = torch.from_numpy(rng.standard_normal((L, n, hq, D)).astype(np.float16)).to(cuda_device)
        k = torch.from_numpy(rng.standard_normal((L, n, hkv, D)).astype(np.float16)).to(cuda_device)
        v = torch.from_numpy(rng.standard_normal((L, n, hkv, D)).astype(np.float16)).to(cuda_device)
        eager.decode_reserve(n)
        ref = []
        for layer in range(L):
            eager.decode_append(layer, k[layer], v[layer], n)
            ref.append(eager.decode_attention(layer, q[layer], n))
        g.q.copy_(q)
        g.k.copy_(k)
        g.v.copy_(v)
        out = g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, torch.stack(ref)), step
    assert eager.lengths == graphed.lengths
    assert torch.equal(eager.block_table, graphed.block_table)
    assert torch.equal(eager.ctx_lens, graphed.ctx_lens)
    assert eager.pool.alloc_state() == graphed.pool.alloc_state()
    for s in range(n):
        ke, ve = eager.gather(s)
        kg, vg = graphed.gather(s)
        assert torch.equal(ke, kg) and torch.equal(ve, vg)
    eager.check()
    graphed.check()
