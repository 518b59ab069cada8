"""GPU neighbour sampler and pin-list PageRank: the producers of the node ids
fetch_feature gathers and of the constant CPU buffer's pin list.

* ``GPUNeighborSampler`` stands in for the DGL MultiLayerNeighborSampler that
  feeds the reference's loader (GIDS_Setup/GIDS/GIDS.py:178-201,
  evaluation/homogenous_train.py:201-203): hand-written kernels over a CSC
  graph in HBM, no host synchronisation between hops, and minibatches
  bit-identical to ``GIDS.synthetic.NeighborSampler`` (same counter-hashed
  edge choice) on any device.
* ``pagerank_pin_list`` is compute_pagerank + top-k of
  evaluation/page_rank_node_list_gen.py:126-134, 282-285, in float32 on the
  GPU (the reference's dtype), producing the ``pin_file`` node list.

* ``out_degree`` / ``hot_rows`` rank nodes by how often neighbour sampling can
  reach them (their out-degree: the in-edges they are the source of), the
  rank of a static GPU-cache hot set (``GIDS.pin_cache`` with
  ``cache_admission="static"``), as degree-ranked GPU feature caches do.

All run in the library behind ``BAM_Feature_Store`` (imported on first use).
"""
from __future__ import annotations

import torch


def _store_module():
    from .GIDS import _feature_store_module

    return _feature_store_module()


def _check_csc(indptr: torch.Tensor, indices: torch.Tensor):
    if not (indptr.is_cuda and indices.is_cuda and indptr.device == indices.device):
        raise ValueError("indptr and indices must be CUDA tensors on one device")
    if indptr.dtype != torch.int64 or indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("indptr must be int64 and indices int32 or int64")
    if not (indptr.is_contiguous() and indices.is_contiguous()):
        raise ValueError("indptr and indices must be contiguous")


class GPUNeighborSampler:
    """MultiLayerNeighborSampler(fanouts) on the GPU over a CSC graph
    (in-edges of v: ``indices[indptr[v]:indptr[v+1]]``). The graph tensors
    are kept referenced. ``sample(seeds)`` returns ``(input_nodes, seeds)``:
    the seeds without duplicates, then every hop's new sources in order of
    first appearance, as an int64 tensor on the graph's device."""

    def __init__(self, indptr: torch.Tensor, indices: torch.Tensor, fanouts, seed: int = 1000,
                 max_seeds: int = 4096):
        _check_csc(indptr, indices)
        self.indptr, self.indices = indptr, indices
        self.device = indptr.device
        self.fanouts = [int(f) for f in fanouts]
        self.seed = int(seed)
        self.max_seeds = int(max_seeds)
        self.num_nodes = indptr.numel() - 1
        with torch.cuda.device(self.device):
            self._s = _store_module().GIDS_Sampler(self.device.index, indptr.data_ptr(), indices.data_ptr(),
                                                   indices.element_size(), self.num_nodes, self.fanouts,
                                                   self.max_seeds, self.seed)
        self.capacity = self._s.capacity()
        self.calls = 0

    def sample(self, seeds: torch.Tensor):
        seeds = seeds.to(self.device, torch.int64).contiguous()
        if seeds.numel() > self.max_seeds:
            raise ValueError(f"{seeds.numel()} seeds, the sampler was made for {self.max_seeds}")
        out = torch.empty(self.capacity, dtype=torch.int64, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        n = self._s.sample(seeds.data_ptr(), seeds.numel(), out.data_ptr(), out.numel(), 0, self.calls, stream)
        self.calls += 1
        return out[:n], seeds


def pagerank(indptr: torch.Tensor, indices: torch.Tensor, iters: int = 20, damping: float = 0.85,
             with_keys: bool = False):
    """float32 PageRank vector (and, with_keys, the top-k order keys) of the
    CSC graph; nodes without in-edges contribute 0."""
    _check_csc(indptr, indices)
    n = indptr.numel() - 1
    pv = torch.empty(n, dtype=torch.float32, device=indptr.device)
    keys = torch.empty(n, dtype=torch.int64, device=indptr.device) if with_keys else None
    stream = torch.cuda.current_stream(indptr.device).cuda_stream
    _store_module().pagerank(indptr.device.index, indptr.data_ptr(), indices.data_ptr(), indices.element_size(), n,
                             int(iters), float(damping), pv.data_ptr(), keys.data_ptr() if with_keys else 0, stream)
    return (pv, keys) if with_keys else pv


def pagerank_pin_list(indptr: torch.Tensor, indices: torch.Tensor, fraction: float = 0.01, damping: float = 0.85,
                      iters: int = 20) -> torch.Tensor:
    """pin_file node ids: the top ``fraction`` of nodes by float32 PageRank,
    value descending, node id ascending (int64, on the graph's device)."""
    _, keys = pagerank(indptr, indices, iters, damping, with_keys=True)
    k = max(1, int((indptr.numel() - 1) * fraction))
    # the keys are distinct and nonnegative: their k smallest are one order
    top = torch.topk(keys, k, largest=False, sorted=True).values
    return top & 0xFFFFFFFF


def out_degree(indices: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """int32 [num_nodes]: how many in-edges of the CSC graph each node is the source of."""
    if not indices.is_cuda or indices.dtype not in (torch.int32, torch.int64) or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int32 or int64 CUDA tensor")
    counts = torch.empty(num_nodes, dtype=torch.int32, device=indices.device)
    stream = torch.cuda.current_stream(indices.device).cuda_stream
    _store_module().out_degree(indices.device.index, indices.data_ptr(), indices.element_size(), indices.numel(),
                               num_nodes, counts.data_ptr(), stream)
    return counts


def top_rows(counts: torch.Tensor, k: int) -> torch.Tensor:
    """The k nodes of largest count (counts < 2^32 per node, fewer than 2^32
    nodes), count descending then node id ascending (int64)."""
    n = counts.numel()
    keys = ((0xFFFFFFFF - counts.to(torch.int64)) << 32) | torch.arange(n, device=counts.device)
    k = max(0, min(int(k), n))
    # the keys are distinct and nonnegative: their k smallest are one order
    return torch.topk(keys, k, largest=False, sorted=True).values & 0xFFFFFFFF


def hot_rows(indices: torch.Tensor, num_nodes: int, k: int) -> torch.Tensor:
    """The k nodes of highest out-degree, degree descending then node id
    ascending (int64, on the graph's device)."""
    return top_rows(out_degree(indices, num_nodes), k)
