"""Synthetic graph and neighbour sampler (the inputs of the benchmarks),
checked on CPU against an explicit CSC of the same graph."""
import numpy as np
import torch

from GIDS.synthetic import (NeighborSampler, SyntheticGraph, edge_key, hop_seed, seed_batches, unique_first,
                            zipf_truncation)


def test_zipf_truncation_reaches_mean():
    for alpha, mean in [(1.1, 15), (1.2, 15), (1.0, 8), (1.1, 10)]:
        K = zipf_truncation(alpha, mean)
        k = np.arange(1, K + 1, dtype=np.float64)
        w = k ** -alpha
        assert (k * w).sum() / w.sum() >= mean
        k = k[:-1]
        w = w[:-1]
        assert (k * w).sum() / w.sum() < mean


def test_graph_degrees_and_determinism():
    g = SyntheticGraph(50000, 15, 1.1, seed=3)
    ip, ind = g.materialize()
    assert abs(ind.numel() / g.N - 15) < 0.2  # Poisson(15) in-degrees
    out = torch.bincount(ind, minlength=g.N).double()
    assert abs(out.mean().item() - 15) < 0.2
    assert out.max().item() > 5 * 15  # heavy-tailed sources
    ip2, ind2 = SyntheticGraph(50000, 15, 1.1, seed=3).materialize()
    assert torch.equal(ip, ip2) and torch.equal(ind, ind2)
    ip3, ind3 = SyntheticGraph(50000, 15, 1.1, seed=4).materialize()
    assert not torch.equal(ind, ind3)


def test_unique_first():
    x = torch.tensor([5, 3, 5, 9, 3, 1, 9])
    assert unique_first(x).tolist() == [5, 3, 9, 1]


def test_sampler_semantics_against_csc():
    g = SyntheticGraph(20000, 15, 1.1, seed=0)
    ip, ind = g.materialize()
    s = NeighborSampler(g, [10, 5], seed=7)
    seeds = seed_batches(g.N, 300, 1, 7)[0]
    frontier = unique_first(seeds)
    sh = hop_seed(7, 0, 0)
    dst, src = s.sample_neighbors(frontier, 5, sh)
    for v in frontier[:200].tolist():
        nb = ind[ip[v]:ip[v + 1]]
        got = src[dst == v]
        assert got.numel() == min(5, nb.numel())
        # the in-edges of smallest key, in key order
        j = torch.arange(nb.numel())
        keys = edge_key(sh, torch.full_like(j, v), j)
        assert torch.equal(got, nb[torch.argsort(keys)[:5]])
    inp, sd = s.sample(seeds)
    assert torch.equal(inp[:seeds.numel()], unique_first(seeds))  # seeds first
    assert torch.unique(inp).numel() == inp.numel()


def test_sampler_is_seeded():
    g = SyntheticGraph(10000, 15, 1.1, seed=0)
    a = NeighborSampler(g, [15, 10, 5], seed=1000).sample(seed_batches(g.N, 64, 1, 1000)[0])[0]
    b = NeighborSampler(g, [15, 10, 5], seed=1000).sample(seed_batches(g.N, 64, 1, 1000)[0])[0]
    c = NeighborSampler(g, [15, 10, 5], seed=1001).sample(seed_batches(g.N, 64, 1, 1001)[0])[0]
    assert torch.equal(a, b) and not torch.equal(a, c)


def test_zipf_seeds_are_skewed():
    s = seed_batches(100000, 4000, 1, 3, zipf_alpha=1.0)[0]
    assert s.numel() == 4000 and torch.unique(s).numel() == 4000


def test_bench_batch_stream_is_the_batch_list():
    """bench.py's lazy sampler stream yields the same minibatches as its list
    form (the timed steps and the loader measurement draw from the same law)."""
    import bench

    cfg = dict(bench.CONFIGS["c1"], nodes=20000, batch=64)
    lst, _ = bench.make_batches(cfg, 3, 0, "cpu")
    lazy = list(bench.batch_stream(cfg, 3, 0, "cpu"))
    assert len(lst) == len(lazy) == 3
    for a, b in zip(lst, lazy):
        assert torch.equal(a, b)
    other = list(bench.batch_stream(cfg, 1, 1, "cpu"))[0]
    assert not torch.equal(other, lst[0])


def test_hop_seeds_and_edge_keys_are_fixed_integers():
    """Known answers: the key functions are plain 64-bit integer arithmetic
    (the CUDA sampler and any device reproduce them)."""
    from GIDS.synthetic import mix64

    # the first output of SplitMix64 seeded with 0 (published test value)
    assert mix64(0) == 0 and mix64(0x9E3779B97F4A7C15) == 0xE220A8397B1DCDAF
    sh = hop_seed(1000, 0, 0)
    assert -(1 << 63) <= sh < (1 << 63)
    k = edge_key(sh, torch.tensor([5, 5, 6]), torch.tensor([0, 1, 0]))
    assert (k >= 0).all() and (k & ((1 << 24) - 1)).tolist() == [0, 1, 0]
    assert hop_seed(1000, 0, 1) != sh and hop_seed(1000, 1, 0) != sh and hop_seed(1001, 0, 0) != sh


def test_sampler_calls_draw_fresh_minibatches():
    g = SyntheticGraph(10000, 15, 1.1, seed=0)
    s = NeighborSampler(g, [10, 5], seed=3)
    sd = seed_batches(g.N, 64, 1, 3)[0]
    a = s.sample(sd)[0]
    b = s.sample(sd)[0]  # same seeds, next call: other edges
    assert not torch.equal(a, b) and torch.equal(a[:64], b[:64])


def test_chunked_csc_equals_one_chunk():
    g = SyntheticGraph(30000, 15, 1.1, seed=2)
    ip, ind = g.materialize()
    ip2, ind2 = g.materialize(torch.int32, chunk_rows=7000)
    assert torch.equal(ip, ip2) and ind2.dtype == torch.int32 and torch.equal(ind, ind2.long())


def test_relation_csc_has_its_own_destinations():
    """A heterograph relation's CSC spans the destination type, whose size
    differs from the source type's."""
    g = SyntheticGraph(5000, 8, 1.0, seed=3)
    ip, ind = g.materialize(torch.int32, n_dst=3000, chunk_rows=1000)
    assert ip.numel() == 3001 and int(ip[-1]) == ind.numel()
    v = torch.arange(3000)
    assert torch.equal(ip[1:] - ip[:-1], g.in_degree(v))
    rows = torch.repeat_interleave(v, ip[1:] - ip[:-1])
    j = torch.arange(ind.numel()) - torch.repeat_interleave(ip[:-1], ip[1:] - ip[:-1])
    assert torch.equal(ind.long(), g.in_neighbor(rows, j)) and int(ind.max()) < 5000
