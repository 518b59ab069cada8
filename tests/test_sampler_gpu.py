"""GPU neighbour sampler and float32 pin-list PageRank (csrc/sampler.cu),
bit for bit against the oracle (oracle/sampler_oracle.c) and the torch
sampler, through the C ABI and the Python classes: several graphs, int32 and
int64 sources, nodes with more in-edges than a warp, nodes without any,
duplicate seeds, consecutive calls, the device-side count, and bad input."""
import ctypes

import numpy as np
import pytest
import torch

import gids_abi
from gids_abi import check
from oracle import oracle

pytestmark = pytest.mark.gpu


def synth_csc(n, mean, alpha, seed, dtype=torch.int32):
    from GIDS.synthetic import SyntheticGraph

    ip, ind = SyntheticGraph(n, mean, alpha, seed=seed).materialize(dtype)
    return ip.numpy(), ind.numpy()


def hub_csc(n=5000, seed=0, dtype=np.int64):
    """Random CSC where every 50th node has 33-300 in-edges and every 7th none."""
    rng = np.random.default_rng(seed)
    deg = rng.integers(0, 12, size=n)
    deg[::50] = rng.integers(33, 300, size=deg[::50].shape)
    deg[::7] = 0
    ip = np.zeros(n + 1, dtype=np.int64)
    ip[1:] = np.cumsum(deg)
    return ip, rng.integers(0, n, size=int(ip[-1])).astype(dtype)


class AbiSampler:
    def __init__(self, ip, ind, fanouts, max_seeds, seed):
        self.ip = torch.as_tensor(ip).cuda()
        self.ind = torch.as_tensor(ind).cuda()
        f = (ctypes.c_int * len(fanouts))(*fanouts)
        self.s = ctypes.c_void_p()
        check(gids_abi.lib().gids_sampler_create(ctypes.byref(self.s), 0, self.ip.data_ptr(), self.ind.data_ptr(),
                                                 self.ind.element_size(), len(ip) - 1, f, len(fanouts), max_seeds,
                                                 seed))
        cap = ctypes.c_uint64()
        check(gids_abi.lib().gids_sampler_capacity(self.s, ctypes.byref(cap)))
        self.cap = cap.value

    def sample(self, seeds, call=-1, device_count=False):
        d = torch.as_tensor(seeds, dtype=torch.int64).cuda()
        out = torch.full((self.cap,), -9, dtype=torch.int64, device="cuda")
        if device_count:
            cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
            check(gids_abi.lib().gids_sampler_sample(self.s, d.data_ptr(), len(seeds), out.data_ptr(), self.cap,
                                                     cnt.data_ptr(), None, call, None))
            n = int(cnt.item())
        else:
            hc = ctypes.c_uint64()
            check(gids_abi.lib().gids_sampler_sample(self.s, d.data_ptr(), len(seeds), out.data_ptr(), self.cap,
                                                     None, ctypes.byref(hc), call, None))
            n = hc.value
        return out[:n].cpu().numpy()

    def close(self):
        gids_abi.lib().gids_sampler_destroy(self.s)


@pytest.mark.parametrize("fanouts", [[15, 10, 5], [10, 10], [32], [1, 2, 3]])
def test_sampler_equals_oracle_synthetic(built, fanouts):
    ip, ind = synth_csc(60000, 15, 1.1, seed=0)
    s = AbiSampler(ip, ind, fanouts, 512, 1000)
    rng = np.random.default_rng(len(fanouts))
    try:
        for call in range(3):
            seeds = rng.integers(0, len(ip) - 1, size=512)
            got = s.sample(seeds)  # the sampler's own call counter: 0, 1, 2
            assert np.array_equal(got, oracle.sample(ip, ind, fanouts, seeds, 1000, call)), call
    finally:
        s.close()


@pytest.mark.parametrize("dtype", [np.int64, np.int32])
def test_sampler_hubs_empty_nodes_duplicate_seeds(built, dtype):
    ip, ind = hub_csc(dtype=dtype)
    s = AbiSampler(ip, ind, [20, 32, 7], 800, 5)
    rng = np.random.default_rng(1)
    try:
        for call in (0, 4, 9):
            seeds = np.concatenate([np.arange(0, 5000, 50)[:60], rng.integers(0, 5000, size=300)])
            seeds = np.concatenate([seeds, seeds[:100]])  # duplicates
            got = s.sample(seeds, call=call, device_count=(call == 4))
            assert np.array_equal(got, oracle.sample(ip, ind, [20, 32, 7], seeds, 5, call)), call
        assert len(s.sample(np.zeros(0, dtype=np.int64))) == 0
    finally:
        s.close()


def test_sampler_rejects_bad_input(built):
    ip, ind = hub_csc(n=500)
    s = AbiSampler(ip, ind, [5], 16, 1)
    L = gids_abi.lib()
    try:
        d = torch.tensor([3, 700], dtype=torch.int64, device="cuda")  # 700: not a node
        out = torch.empty(s.cap, dtype=torch.int64, device="cuda")
        hc = ctypes.c_uint64()
        assert L.gids_sampler_sample(s.s, d.data_ptr(), 2, out.data_ptr(), s.cap, None, ctypes.byref(hc), 0,
                                     None) == gids_abi.GIDS_E_RANGE
        assert L.gids_sampler_sample(s.s, d.data_ptr(), 2, out.data_ptr(), 1, None, ctypes.byref(hc), 0,
                                     None) == gids_abi.GIDS_E_INVAL  # output below capacity
        big = torch.zeros(17, dtype=torch.int64, device="cuda")
        assert L.gids_sampler_sample(s.s, big.data_ptr(), 17, out.data_ptr(), s.cap, None, ctypes.byref(hc), 0,
                                     None) == gids_abi.GIDS_E_INVAL  # more seeds than max_seeds
        f = (ctypes.c_int * 1)(33)
        bad = ctypes.c_void_p()
        ipd = torch.as_tensor(ip).cuda()
        indd = torch.as_tensor(ind).cuda()
        assert L.gids_sampler_create(ctypes.byref(bad), 0, ipd.data_ptr(), indd.data_ptr(), 8, len(ip) - 1, f, 1,
                                     16, 1) == gids_abi.GIDS_E_UNSUPPORTED  # fanout above 32
    finally:
        s.close()


def test_python_sampler_equals_torch_sampler(built):
    from GIDS.sampler import GPUNeighborSampler
    from GIDS.synthetic import NeighborSampler, SyntheticGraph, seed_batches

    g = SyntheticGraph(300000, 15, 1.1, seed=0, device="cuda")
    ip, ind = g.materialize(torch.int32)
    gs = GPUNeighborSampler(ip, ind, [15, 10, 5], seed=1000, max_seeds=1024)
    ts = NeighborSampler(g, [15, 10, 5], seed=1000)
    for sd in seed_batches(g.N, 1024, 4, 1000, device="cuda"):
        a = gs.sample(sd)[0]
        b = ts.sample(sd)[0]
        assert torch.equal(a, b)


@pytest.mark.parametrize("graph", ["synthetic_i32", "hubs_i64"])
def test_pagerank_equals_oracle(built, graph):
    from GIDS.sampler import pagerank, pagerank_pin_list

    if graph == "synthetic_i32":
        ip, ind = synth_csc(40000, 15, 1.2, seed=1)
    else:
        ip, ind = hub_csc(n=8000, seed=3)  # every 7th node has no in-edges
    want = oracle.pagerank_f32(ip, ind, iters=20, damping=0.85)
    ipd, indd = torch.as_tensor(ip).cuda(), torch.as_tensor(ind).cuda()
    got = pagerank(ipd, indd, iters=20, damping=0.85).cpu().numpy()
    assert got.view(np.uint32).tobytes() == want.view(np.uint32).tobytes()
    k = int((len(ip) - 1) * 0.01)
    pins = pagerank_pin_list(ipd, indd, 0.01).cpu().numpy()
    assert pins.tolist() == oracle.topk_desc(want, k).tolist()
