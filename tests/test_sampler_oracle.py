"""The oracle's sampler and pin-list PageRank (oracle/sampler_oracle.c), on
CPU: the sampler against the torch restatement in GIDS/synthetic.py over the
explicit CSC of the same graph, and the float32 PageRank against the
reference's compute_pagerank (evaluation/page_rank_node_list_gen.py:126-134)
written out line by line with float32 torch tensors."""
import numpy as np
import torch

from GIDS.synthetic import NeighborSampler, SyntheticGraph, edge_key, hop_seed, seed_batches
from oracle import oracle


def test_key_functions_agree_with_torch(built):
    for seed, call, hop in [(1000, 0, 0), (1007, 3, 2), (2**40 + 5, 17, 1)]:
        assert oracle.hop_seed(seed, call, hop) == hop_seed(seed, call, hop) & (2**64 - 1)
    sh = hop_seed(1000, 0, 1)
    v = torch.tensor([0, 5, 99999, 2**33])
    j = torch.tensor([0, 7, 31, 12345])
    ks = edge_key(sh, v, j).tolist()
    assert ks == [oracle.edge_key(sh, int(a), int(b)) for a, b in zip(v, j)]


def test_oracle_sampler_equals_torch_sampler(built):
    g = SyntheticGraph(40000, 15, 1.1, seed=0)
    ip, ind = g.materialize()
    for fanouts, seed in [([15, 10, 5], 1000), ([10, 10], 7), ([20], 3)]:
        s = NeighborSampler(g, fanouts, seed=seed)
        for call, sd in enumerate(seed_batches(g.N, 256, 3, seed)):
            want = s.sample(sd)[0].numpy()
            got = oracle.sample(ip.numpy(), ind.numpy().astype(np.int32), fanouts, sd.numpy(), seed, call)
            assert np.array_equal(got, want), (fanouts, call)


def test_oracle_sampler_duplicate_seeds_and_high_degree(built):
    # node 0 has 100 in-edges (more than one warp's worth), node 1 none
    n = 300
    rng = np.random.default_rng(0)
    deg = rng.integers(0, 6, size=n)
    deg[0], deg[1] = 100, 0
    ip = np.zeros(n + 1, dtype=np.int64)
    ip[1:] = np.cumsum(deg)
    ind = rng.integers(0, n, size=int(ip[-1])).astype(np.int64)
    seeds = np.array([0, 1, 0, 5, 1, 7])
    got = oracle.sample(ip, ind, [4, 8], seeds, 11)
    assert list(got[:4]) == [0, 1, 5, 7]
    assert len(set(got.tolist())) == len(got)
    # hop 0 (fanout 8) keeps node 0's 8 in-edges of smallest key, in key order
    sh = oracle.hop_seed(11, 0, 0)
    keys = [oracle.edge_key(sh, 0, j) for j in range(100)]
    kept = ind[ip[0] + np.argsort(keys)[:8]]
    firsts = [x for x in dict.fromkeys(kept.tolist()) if x not in (0, 1, 5, 7)]
    assert list(got[4:4 + len(firsts)]) == firsts


def reference_pagerank_f32(ip: np.ndarray, ind: np.ndarray, K: int = 20, DAMP: float = 0.85) -> np.ndarray:
    """compute_pagerank (page_rank_node_list_gen.py:126-134) line by line on
    float32 torch tensors; DGL's update_all(copy_u, sum) as a sequential sum
    over each node's in-edges in CSC order; a zero in-degree contributes 0."""
    N = len(ip) - 1
    pv = torch.ones(N) / N
    degrees = torch.from_numpy(np.diff(ip)).type(torch.float32)
    for _ in range(K):
        pv = torch.where(degrees > 0, pv / degrees, torch.zeros(()))
        m = pv.numpy()
        new = np.empty(N, dtype=np.float32)
        for v in range(N):
            s = np.float32(0.0)
            for e in range(ip[v], ip[v + 1]):
                s = np.float32(s + m[ind[e]])
            new[v] = s
        pv = (1 - DAMP) / N + DAMP * torch.from_numpy(new)
    return pv.numpy()


def test_oracle_pagerank_equals_reference_in_float32(built):
    g = SyntheticGraph(1500, 15, 1.2, seed=1)
    ip, ind = g.materialize()
    ip, ind = ip.numpy(), ind.numpy()
    want = reference_pagerank_f32(ip, ind, K=6)
    got = oracle.pagerank_f32(ip, ind.astype(np.int32), iters=6)
    assert got.dtype == np.float32 and got.view(np.uint32).tobytes() == want.view(np.uint32).tobytes()


def test_oracle_topk_order(built):
    pv = np.array([0.1, 0.5, 0.5, 0.2, 0.5, 0.05], dtype=np.float32)
    assert oracle.topk_desc(pv, 4).tolist() == [1, 2, 4, 3]
    g = SyntheticGraph(3000, 15, 1.2, seed=4)
    ip, ind = g.materialize()
    pv = oracle.pagerank_f32(ip.numpy(), ind.numpy(), iters=20)
    top = oracle.topk_desc(pv, 30)
    order = np.lexsort((np.arange(len(pv)), -pv.astype(np.float64)))
    assert top.tolist() == order[:30].tolist()
