"""Seeded synthetic graphs and a multi-layer neighbour sampler.

The reference feeds fetch_feature with node ids from DGL's
MultiLayerNeighborSampler over IGB/OGB graphs (homogenous_train.py:201-203,
dataloader.py). Neither DGL nor the datasets exist on the build or GPU
machines, so the benchmarks draw ids from this module instead.

Graph model (CSC, defined by hash functions so that a 100M-node graph needs
no edge list): every node u has an out-degree weight d_u drawn from a Zipf(alpha)
law truncated to [1, K], with K chosen so that the mean is ``mean_degree``;
every node v has Poisson(mean_degree) in-edges whose sources are drawn with
probability proportional to d_u ("neighbours chosen uniformly" among edge
ends). Neighbour j of v is a pure function of (seed, v, j), so the graph is
fixed by its seed; ``materialize`` builds the explicit CSC for small graphs.

Sampler (MultiLayerNeighborSampler semantics): for fanouts [f_0, ..., f_L-1],
hop h (from the seeds outward) takes min(f_{L-1-h}, in_degree) distinct
in-edges of every node of the current frontier; the next frontier is the
current node set plus the new sources in order of first appearance, and the
last node set is ``input_nodes`` (seeds first).

Every random choice is a pure function of integers (counter-based SplitMix64
hashes), not of a random generator's stream, so a minibatch is the same on
the CPU, on any GPU and in the CUDA sampler kernel of this package: the
in-edges a node keeps at a hop are the ones with the smallest
``edge_key(hop_seed(seed, call, hop), v, j)``, listed in increasing key order.
"""
from __future__ import annotations

import math

import numpy as np
import torch

_M1 = np.int64(np.uint64(0xBF58476D1CE4E5B9).astype(np.int64))
_M2 = np.int64(np.uint64(0x94D049BB133111EB).astype(np.int64))
_G = np.int64(np.uint64(0x9E3779B97F4A7C15).astype(np.int64))


def _i64(v: int) -> int:
    """Python int wrapped to a signed 64-bit value."""
    v &= (1 << 64) - 1
    return v - (1 << 64) if v >= (1 << 63) else v


def _srl(z: torch.Tensor, k: int) -> torch.Tensor:
    return (z >> k) & ((1 << (64 - k)) - 1)


def _mix(z: torch.Tensor) -> torch.Tensor:
    z = (z ^ _srl(z, 30)) * int(_M1)
    z = (z ^ _srl(z, 27)) * int(_M2)
    return z ^ _srl(z, 31)


def _uniform(z: torch.Tensor) -> torch.Tensor:
    """uniform [0, 1) float64 from 53 hash bits"""
    return _srl(_mix(z), 11).to(torch.float64) * (2.0 ** -53)


_MASK64 = (1 << 64) - 1
EDGE_INDEX_BITS = 24  # an edge key keeps j in its low bits: in-degrees below 2^24


def mix64(x: int) -> int:
    """SplitMix64 finalizer (Steele, Lea, Flood 2014) on a Python int."""
    x &= _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def hop_seed(seed: int, call: int, hop: int) -> int:
    """Key seed (a signed 64-bit value) of hop ``hop`` of the ``call``-th
    minibatch a sampler of seed ``seed`` draws."""
    return _i64(mix64(seed * 0x9E3779B97F4A7C15 + call * 0xD1B54A32D192ED03 + hop * 0x8CB92BA72F3D8DD7 +
                      0x632BE59BD9B4E019))


def edge_key(seed_h: int, v: torch.Tensor, j: torch.Tensor) -> torch.Tensor:
    """Selection key of in-edge j of node v at a hop of seed ``seed_h``: 39
    hash bits above the edge index j (24 bits), so the keys of one node are
    distinct and nonnegative, and sorting them needs no tie rule."""
    z = _mix(v * int(_G) + int(seed_h))
    z = _mix(z + (j + 1) * int(_M2))
    return (_srl(z, 1 + EDGE_INDEX_BITS) << EDGE_INDEX_BITS) | j


def zipf_truncation(alpha: float, mean: float) -> int:
    """Smallest K with E[d] >= mean for P(d = k) ~ k^-alpha on [1, K]."""

    def m(K):
        k = np.arange(1, K + 1, dtype=np.float64)
        w = k ** -alpha
        return float((k * w).sum() / w.sum())

    if mean <= 1.0:
        return 1
    hi = 2
    while m(hi) < mean:  # the mean grows with K: double, then bisect
        hi *= 2
        if hi > (1 << 26):
            raise ValueError("mean degree not reachable with this alpha")
    lo = hi // 2
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if m(mid) >= mean:
            hi = mid
        else:
            lo = mid
    return hi


class SyntheticGraph:
    def __init__(self, num_nodes: int, mean_degree: float = 15.0, alpha: float = 1.1, seed: int = 0,
                 device="cpu"):
        self.N = int(num_nodes)
        self.mean = float(mean_degree)
        self.alpha = float(alpha)
        self.seed = int(seed)
        self.device = torch.device(device)
        self.K = zipf_truncation(self.alpha, self.mean)
        k = np.arange(1, self.K + 1, dtype=np.float64)
        w = k ** -self.alpha
        self._deg_cdf = torch.tensor(np.cumsum(w / w.sum()), dtype=torch.float64, device=self.device)
        # Poisson(mean) in-degree table, capped where the tail is below 1e-12
        kmax = int(self.mean + 12 * math.sqrt(self.mean) + 20)
        pmf = [math.exp(-self.mean)]
        for i in range(1, kmax + 1):
            pmf.append(pmf[-1] * self.mean / i)
        self.max_in_degree = kmax
        self._in_cdf = torch.tensor(np.cumsum(pmf) / np.sum(pmf), dtype=torch.float64, device=self.device)
        # out-degree class of every node, nodes grouped by class
        d = self.out_degree(torch.arange(self.N, device=self.device))
        self._order = torch.argsort(d, stable=True)
        counts = torch.bincount(d - 1, minlength=self.K)
        self._class_count = counts
        self._class_off = torch.cumsum(counts, 0) - counts
        mass = counts.to(torch.float64) * torch.arange(1, self.K + 1, device=self.device, dtype=torch.float64)
        self._class_cdf = torch.cumsum(mass / mass.sum(), 0)
        del d

    def _h(self, salt: int, x: torch.Tensor) -> torch.Tensor:
        return x * int(_G) + _i64((self.seed * 1_000_003 + salt) * int(_M1))

    def out_degree(self, u: torch.Tensor) -> torch.Tensor:
        x = _uniform(self._h(1, u))
        return torch.searchsorted(self._deg_cdf, x, right=True).clamp_(max=self.K - 1) + 1

    def in_degree(self, v: torch.Tensor) -> torch.Tensor:
        x = _uniform(self._h(2, v))
        return torch.searchsorted(self._in_cdf, x, right=True).clamp_(max=self.max_in_degree)

    def in_neighbor(self, v: torch.Tensor, j: torch.Tensor) -> torch.Tensor:
        """Source of in-edge j of v (j < in_degree(v))."""
        e = v * (self.max_in_degree + 1) + j
        c = torch.searchsorted(self._class_cdf, _uniform(self._h(3, e)), right=True).clamp_(max=self.K - 1)
        cnt = self._class_count[c]
        off = (_uniform(self._h(4, e)) * cnt.to(torch.float64)).to(torch.int64).clamp_(min=0)
        off = torch.minimum(off, (cnt - 1).clamp(min=0))
        return self._order[self._class_off[c] + off]

    def materialize(self, index_dtype=torch.int64, chunk_rows: int = 1 << 22, n_dst: int | None = None):
        """Explicit CSC (indptr int64 [n_dst+1], indices [E] of index_dtype) of
        the graph: indices[indptr[v] + j] = in_neighbor(v, j), built chunk by
        chunk of destination rows. n_dst (default N) is the number of
        destinations: a heterograph relation's destinations are another node
        type than its sources."""
        dev = self.device
        nd = self.N if n_dst is None else int(n_dst)
        deg = self.in_degree(torch.arange(nd, device=dev))
        indptr = torch.zeros(nd + 1, dtype=torch.int64, device=dev)
        torch.cumsum(deg, 0, out=indptr[1:])
        indices = torch.empty(int(indptr[-1]), dtype=index_dtype, device=dev)
        for lo in range(0, nd, chunk_rows):
            hi = min(nd, lo + chunk_rows)
            d = deg[lo:hi]
            rows = torch.repeat_interleave(torch.arange(lo, hi, device=dev), d)
            j = torch.arange(rows.numel(), device=dev) - torch.repeat_interleave(indptr[lo:hi] - indptr[lo], d)
            indices[int(indptr[lo]):int(indptr[hi])] = self.in_neighbor(rows, j).to(index_dtype)
        return indptr, indices


def unique_first(x: torch.Tensor) -> torch.Tensor:
    """Unique values of x in order of first appearance."""
    if x.numel() == 0:
        return x
    u, inv = torch.unique(x, return_inverse=True)
    first = torch.full((u.numel(),), x.numel(), dtype=torch.int64, device=x.device)
    first.scatter_reduce_(0, inv, torch.arange(x.numel(), device=x.device), reduce="amin")
    return u[torch.argsort(first)]


class NeighborSampler:
    """Seeded stand-in for dgl.dataloading.MultiLayerNeighborSampler(fanouts).

    The ``call``-th ``sample`` draws hop ``h`` with key seed
    ``hop_seed(seed, call, h)``; each node of the frontier keeps its
    min(fanout, in_degree) in-edges of smallest ``edge_key``."""

    def __init__(self, graph: SyntheticGraph, fanouts, seed: int = 1000):
        self.g = graph
        self.fanouts = [int(f) for f in fanouts]
        self.seed = int(seed)
        self.calls = 0

    def sample_neighbors(self, frontier: torch.Tensor, fanout: int, seed_h: int):
        """(dst, src) pairs: the min(fanout, deg) in-edges of smallest key per
        frontier node, dst-major, keys increasing."""
        g = self.g
        if frontier.numel() == 0:
            return frontier, frontier
        deg = g.in_degree(frontier)
        D = int(deg.max().item())
        if D == 0:
            e = frontier[:0]
            return e, e
        if D >= (1 << EDGE_INDEX_BITS):
            raise ValueError("in-degree too large for the edge key")
        pos = torch.arange(D, device=frontier.device)
        keys = edge_key(seed_h, frontier[:, None], pos[None, :])
        keys.masked_fill_(pos[None, :] >= deg[:, None], torch.iinfo(torch.int64).max)
        take = min(fanout, D)
        # keys are distinct within a row: the k smallest, in order, are well defined
        j = torch.topk(keys, take, dim=1, largest=False, sorted=True).indices
        valid = torch.arange(take, device=frontier.device)[None, :] < torch.clamp(deg, max=fanout)[:, None]
        dst = frontier[:, None].expand(-1, take)[valid]
        jj = j[valid]
        return dst, g.in_neighbor(dst, jj)

    def sample(self, seeds: torch.Tensor):
        """input_nodes (seeds first, then new sources by first appearance), seeds."""
        call = self.calls
        self.calls += 1
        nodes = unique_first(seeds.to(self.g.device))
        for hop, f in enumerate(reversed(self.fanouts)):
            _, src = self.sample_neighbors(nodes, f, hop_seed(self.seed, call, hop))
            new = unique_first(src)
            new = new[~torch.isin(new, nodes)]
            nodes = torch.cat([nodes, new])
        return nodes, seeds


def seed_batches(num_nodes: int, batch_size: int, n_batches: int, seed: int, device="cpu", zipf_alpha=None):
    """Batches of distinct seed nodes: uniform over [0, N) or, with zipf_alpha,
    Zipf over node ids (ranks scattered over the id space by a hash). Drawn
    on the CPU from a counter-based hash of (seed, draw index), so the batches
    do not depend on the device they are moved to."""
    a = None if zipf_alpha is None else float(zipf_alpha)
    base = _i64(mix64(int(seed) * 0xA0761D6478BD642F + 0xE7037ED1A0B428DB))
    counter = [0]

    def draw(m):
        k = torch.arange(counter[0], counter[0] + m, dtype=torch.int64)
        counter[0] += m
        z = _mix(k * int(_G) + base)
        if a is None:
            return _srl(z, 1) % num_nodes
        u = _srl(z, 11).to(torch.float64) * (2.0 ** -53)
        if abs(a - 1.0) < 1e-9:
            r = torch.exp(u * math.log(num_nodes))
        else:
            r = (1 + u * (num_nodes ** (1 - a) - 1)) ** (1 / (1 - a))
        rank = r.to(torch.int64).clamp_(0, num_nodes - 1)
        return _srl(_mix(rank * int(_G) + 77), 1) % num_nodes

    out = []
    batch_size = min(batch_size, num_nodes)
    for _ in range(n_batches):
        s = unique_first(draw(batch_size * 2))
        for _ in range(64):  # skewed laws repeat ids: keep drawing until the batch is full
            if s.numel() >= batch_size:
                break
            more = draw(batch_size * 4)
            s = unique_first(torch.cat([s, more]))
        out.append(s[:batch_size].to(device))
    return out


class HeteroSyntheticGraph:
    """Heterograph of several node types; every relation (src type, dst type)
    is a SyntheticGraph over the source type: Poisson(mean) in-edges per
    destination node, sources drawn proportionally to truncated-Zipf weights."""

    def __init__(self, type_sizes: dict, relations, mean_degree: float = 8.0, alpha: float = 1.0, seed: int = 0,
                 device="cpu"):
        self.type_sizes = dict(type_sizes)
        self.relations = [tuple(r) for r in relations]
        self.device = torch.device(device)
        self.rel = {}
        for i, (src, dst) in enumerate(self.relations):
            self.rel[(src, dst)] = SyntheticGraph(self.type_sizes[src], mean_degree, alpha, seed=seed * 100 + i + 1,
                                                  device=device)

    def offsets(self) -> dict:
        """heterograph_map: first global node id of each type (types laid out in order)."""
        out, acc = {}, 0
        for t, n in self.type_sizes.items():
            out[t] = acc
            acc += n
        return out


class HeteroNeighborSampler:
    """Seeded stand-in for DGL's MultiLayerNeighborSampler on a heterograph:
    every hop samples min(fanout, in_degree) in-edges per frontier node along
    every relation whose destination type the node has."""

    def __init__(self, graph: HeteroSyntheticGraph, fanouts, seed: int = 1000):
        self.g = graph
        self.fanouts = [int(f) for f in fanouts]
        self.samplers = {r: NeighborSampler(g, [1], seed=seed + 7 * i) for i, (r, g) in enumerate(graph.rel.items())}
        self.calls = 0

    def sample(self, seeds: dict):
        """{type: input node ids (type-local ids, seeds first)}, seeds."""
        dev = self.g.device
        call = self.calls
        self.calls += 1
        nodes = {t: torch.zeros(0, dtype=torch.int64, device=dev) for t in self.g.type_sizes}
        for t, s in seeds.items():
            nodes[t] = unique_first(s.to(dev))
        for hop, f in enumerate(reversed(self.fanouts)):
            new = {t: [] for t in nodes}
            for (src, dst), smp in self.samplers.items():
                if nodes[dst].numel() == 0:
                    continue
                _, nb = smp.sample_neighbors(nodes[dst], f, hop_seed(smp.seed, call, hop))
                new[src].append(nb)
            for t, parts in new.items():
                if not parts:
                    continue
                cand = unique_first(torch.cat(parts))
                cand = cand[~torch.isin(cand, nodes[t])]
                nodes[t] = torch.cat([nodes[t], cand])
        return nodes, seeds
