"""Host-side policy of GIDS.fetch_feature (GIDS.py:791-1058) on CPU: window
buffering, the Storage Access Accumulator, heterograph key offsets and the
constant-CPU-buffer setup, against a fake store that gathers with the oracle."""
import ctypes

import numpy as np
import pytest
import torch

import sys

import GIDS
from oracle import oracle

gmod = sys.modules["GIDS.GIDS"]  # the module (the package attribute GIDS.GIDS is the class)


class FakeControllers:
    def __init__(self):
        self.calls = []

    def init_GIDS_controllers(self, n, qd, nq, lst):
        self.calls.append(("init", n, qd, nq, list(lst)))

    def set_emulation(self, cap, pattern):
        self.calls.append(("emulation", cap, pattern))


class FakeStore:
    """Records calls and gathers from a numpy table (CPU pointers)."""

    table = None  # set by the test

    def __init__(self):
        self.calls = []
        self.cpu_pins = None
        self.cpu_count = 0

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)

        def rec(*a):
            self.calls.append((name,) + a)

        return rec

    @staticmethod
    def _ids(ptr, n):
        return np.ctypeslib.as_array((ctypes.c_int64 * n).from_address(ptr)).copy() if n else np.zeros(0, np.int64)

    def _gather(self, out_ptr, idx_ptr, n, dim, key_off):
        ids = self._ids(idx_ptr, n)
        res = oracle.gather(self.table, ids, dim=dim, key_off=key_off)
        if n:
            dst = np.ctypeslib.as_array((ctypes.c_float * (n * dim)).from_address(out_ptr))
            dst[:] = res.reshape(-1)
        if self.cpu_pins is not None:
            self.cpu_count += int(np.isin(ids + key_off, self.cpu_pins).sum())

    def read_feature(self, out, idx, n, dim, cache_dim, key_off, stream=0):
        self.calls.append(("read_feature", n))
        self._gather(out, idx, n, dim, key_off)

    def read_feature_hetero(self, k, outs, idxs, ns, dim, cache_dim, keys, stream=0):
        self.calls.append(("read_feature_hetero", k, list(ns), list(keys)))
        for o, i, n, kk in zip(outs, idxs, ns, keys):
            self._gather(o, i, n, dim, kk)

    read_feature_merged_hetero = read_feature_hetero

    def read_feature_merged(self, k, outs, idxs, ns, dim, cache_dim, stream=0):
        self.calls.append(("read_feature_merged", k, list(ns)))
        for o, i, n in zip(outs, idxs, ns):
            self._gather(o, i, n, dim, 0)

    def set_window_buffering(self, ptr, n, off, stream=0):
        self.calls.append(("wb", tuple(self._ids(ptr, n)), off))

    def prefetch(self, ptr, n, dim, cache_dim, key_off, stream=0):
        self.calls.append(("prefetch", tuple(self._ids(ptr, n)), dim, cache_dim, key_off))

    def set_cpu_buffer(self, ptr, num):
        self.cpu_pins = self._ids(ptr, num)
        self.calls.append(("set_cpu_buffer", num))

    def get_cpu_access_count(self):
        return self.cpu_count

    def flush_cpu_access_count(self):
        self.cpu_count = 0


@pytest.fixture
def fake(monkeypatch):
    import types

    fake_mod = types.SimpleNamespace(BAM_Feature_Store_float=FakeStore, BAM_Feature_Store_long=FakeStore,
                                     GIDS_Controllers=FakeControllers)
    monkeypatch.setattr(gmod, "_feature_store_module", lambda: fake_mod)
    monkeypatch.setattr(gmod, "_current_stream_handle", lambda d: 0)
    FakeStore.table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 1000, 64)

    def make(**kw):
        g = GIDS.GIDS(page_size=4096, cache_dim=64, num_ele=1000 * 64, **kw)
        g.device = torch.device("cpu")
        return g

    return make


def batches(n, size, seed=0, rows=1000):
    rng = np.random.default_rng(seed)
    return [[torch.as_tensor(rng.integers(0, rows, size=size)), f"seeds{i}", f"blocks{i}"] for i in range(n)]


def test_constructor_forwards_reference_arguments(fake):
    g = fake(off=3 * 4096 * 2 + 1, num_ssd=2, ssd_list=[5, 6], cache_size=7)
    # GIDS.py:583 -- byte offset to first page per SSD
    assert g.off == int(np.ceil(np.ceil((3 * 4096 * 2 + 1) / 4096) / 2))
    assert g.GIDS_controller.calls[0] == ("init", 2, 1024, 128, [5, 6])
    names = [c[0] for c in g.BAM_FS.calls]
    assert names[:5] == ["set_device", "init_controllers", "set_row_layout", "set_cache_policy", "set_synchronous"]
    assert ("set_cache_policy", True, 3) in g.BAM_FS.calls
    assert g.BAM_FS.calls[1][2:] == (4096, g.off, 7, 1000 * 64, 2)


def test_constructor_forwards_extensions(fake):
    g = fake(cache_admission=False, cache_ref_max=1, gather_blocks=148, cache_line=512)
    calls = g.BAM_FS.calls
    assert ("set_cache_line", 512) in calls
    assert ("set_cache_policy", False, 1) in calls
    assert ("set_gather_blocks", 148) in calls
    names = [c[0] for c in calls]
    # the cache line is fixed before the store is built; the policy and grid cap after
    assert names.index("set_cache_line") < names.index("init_controllers") < names.index("set_cache_policy")
    g2 = fake()
    assert "set_gather_blocks" not in [c[0] for c in g2.BAM_FS.calls]  # 0 keeps the resident maximum


def test_bench_arms_name_the_same_workload():
    import argparse

    import bench

    for name, cfg in bench.CONFIGS.items():
        w = bench.workload_name(argparse.Namespace(config=name), cfg)
        assert w.startswith(f"{name}: {cfg['nodes']} nodes") and f"batch {cfg['batch']}" in w
        assert f"in {cfg['line'] or cfg['page']} B lines" in w
    assert set(bench.POLICIES) >= {"admit2", "clock"} and bench.POLICIES["clock"] == (False, 1)


def test_default_path(fake):
    g = fake()
    bs = batches(3, 50)
    it = iter([list(b) for b in bs])
    for b in bs:
        out = g.fetch_feature(64, it, "cpu")
        assert out[1] == b[1] and out[2] == b[2]
        assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, b[0].numpy()))
    assert [c[0] for c in g.BAM_FS.calls].count("read_feature") == 3


def test_tuple_batches_get_features_appended(fake):
    g = fake()
    b = batches(1, 10)[0]
    out = g.fetch_feature(32, iter([tuple(b)]), "cpu")
    assert isinstance(out, tuple) and len(out) == 4
    assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, b[0].numpy(), dim=32))


def test_window_buffering_marks_ahead(fake):
    g = fake(window_buffer=True, wb_size=3)
    bs = batches(8, 20)
    it = iter([list(b) for b in bs])
    out = g.fetch_feature(64, it, "cpu")
    wb = [c for c in g.BAM_FS.calls if c[0] == "wb"]
    # fill_wb pulls wb_size batches and marks them, then the next batch is marked too (GIDS.py:816-833)
    assert [c[1] for c in wb] == [tuple(b[0].numpy()) for b in bs[:4]]
    assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, bs[0][0].numpy()))
    for i in range(1, 4):
        out = g.fetch_feature(64, it, "cpu")
        assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, bs[i][0].numpy()))
    wb = [c for c in g.BAM_FS.calls if c[0] == "wb"]
    assert len(wb) == 7 and wb[-1][1] == tuple(bs[6][0].numpy())


def test_window_buffer_prefetch_follows_each_mark(fake):
    g = fake(window_buffer=True, wb_size=2, wb_prefetch=True)
    bs = batches(5, 20)
    it = iter([list(b) for b in bs])
    for i in range(2):
        out = g.fetch_feature(48, it, "cpu")
        assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, bs[i][0].numpy(), dim=48))
    ev = [c for c in g.BAM_FS.calls if c[0] in ("wb", "prefetch", "read_feature")]
    # every batch entering the window is marked, then prefetched with the gathers' columns
    marks = [c for c in ev if c[0] == "wb"]
    pref = [c for c in ev if c[0] == "prefetch"]
    assert [c[1] for c in pref] == [c[1] for c in marks] == [tuple(b[0].numpy()) for b in bs[:4]]
    assert all(c[2:] == (48, 64, 0) for c in pref)
    assert [c[0] for c in ev[:4]] == ["wb", "prefetch", "wb", "prefetch"]
    # without the flag nothing is prefetched
    g2 = fake(window_buffer=True, wb_size=2)
    g2.fetch_feature(64, iter([list(b) for b in bs]), "cpu")
    assert not [c for c in g2.BAM_FS.calls if c[0] == "prefetch"]


def test_replicated_rows_map_to_their_cache_lines(fake):
    g = fake()  # float32 x 64 columns: 256-byte rows, 4 KB lines
    assert g._row_lines(torch.tensor([0, 15, 16, 100, 16])).tolist() == [0, 1, 6]
    g.cache_dim = 768  # 3072-byte rows straddle 4 KB lines
    assert g._row_lines(torch.tensor([1, 0, 3])).tolist() == [0, 1, 2]  # row 3 is bytes 9216-12287: line 2
    assert g._row_lines(torch.tensor([2])).tolist() == [1, 2]
    with pytest.raises(RuntimeError):
        g.replicate_rows(torch.tensor([1]))  # one rank: no sharded cache to replicate in


def test_replica_model_trades_nvlink_for_host_reads():
    import bench

    ranked = 8000
    refs = 1.0 / np.arange(1, ranked + 1)  # Zipf-like reference counts, hottest first
    cum = np.concatenate([[0.0], np.cumsum(refs)])
    total = float(cum[-1]) * 1.004  # 0.4 % of the references go to rows beyond the ranked ones
    # 8 GPUs of 1000 rows each hold all 8000 ranked rows unreplicated: NVLink-bound
    r8, rate8 = bench.replica_model(cum, total, 1000, 8, 737.0, 25.0)
    r0 = bench.replica_model(cum, total, 1000, 8, 737.0, 25.0)  # deterministic
    assert (r8, rate8) == r0 and r8 > 0
    # the rate at R = r8 beats the rate without replicas (all 8000 rows sharded)
    cached = cum[-1] / total
    rate_no = 1.0 / max(cached * 7 / 8 / (0.86 * 737.0), (1 - cached) / (0.92 * 25.0))
    assert rate8 > rate_no
    # a slow host link makes host reads dear: fewer rows replicated
    r_slow, _ = bench.replica_model(cum, total, 1000, 8, 737.0, 2.0)
    assert r_slow < r8
    # 2 GPUs of 1000 rows: 6000 ranked rows are read from the host already; replicating adds more: none
    r2, _ = bench.replica_model(cum, total, 1000, 2, 737.0, 25.0)
    assert r2 == 0
    # everything cached: replicate until the rows pushed out to the host cost what NVLink saves
    cum_all = np.concatenate([[0.0], np.cumsum(refs[:2000])])
    r_all, rate_all = bench.replica_model(cum_all, float(cum_all[-1]), 1000, 2, 737.0, 25.0)
    assert 0 < r_all < 1000 and rate_all > 0.86 * 737.0 / 0.5  # unreplicated: half the bytes remote


def test_choose_replicas_end_to_end_on_cpu(monkeypatch):
    """The bench's replica choice over pre-sampled minibatches (torch sampler on
    the CPU, reference counts by bincount instead of the CUDA counting kernel):
    'auto' returns rank 0's model choice, a number is clamped, 'off' is 0."""
    import types

    import bench
    from GIDS import sampler as gs

    monkeypatch.setattr(gs, "out_degree", lambda ids, n: torch.bincount(ids, minlength=n).to(torch.int32))
    cfg = dict(bench.CONFIGS["c2"], nodes=20000, batch=64, torch_sampler=True)
    _, ind = bench.graph_csc(cfg, "cpu")
    hot = gs.top_rows(torch.bincount(ind.to(torch.int64), minlength=cfg["nodes"]).to(torch.int32), 8 * 1500)

    class OneRank:
        rank, world = 0, 1

        def max(self, v):
            return v

    store = types.SimpleNamespace(geometry=lambda: {"cache_slots": 1500})
    g = types.SimpleNamespace(BAM_FS=store, world=8)
    args = types.SimpleNamespace(replicate="auto")
    r = bench.choose_replicas(args, cfg, g, hot, "cpu", OneRank(), 1, 737.0, 25.0)
    assert 0 <= r <= 1500
    args.replicate = "100000"
    assert bench.choose_replicas(args, cfg, g, hot, "cpu", OneRank(), 1, 737.0, 25.0) == 1500
    args.replicate = "off"
    assert bench.choose_replicas(args, cfg, g, hot, "cpu", OneRank(), 1, 737.0, 25.0) == 0


def test_accumulator_merges_until_threshold(fake):
    g = fake(accumulator_flag=True)
    g.set_required_storage_access(bw=1.0, l_ssd=10, l_system=5, num_ssd=1, p=0.5)
    # GIDS.py:785
    assert g.required_accesses == pytest.approx(0.5 * 1.0 * 1024 / 4096 * 15 * 1 / 0.5)
    g.required_accesses = 95  # three batches of 40 ids are needed to exceed it
    bs = batches(9, 40)
    it = iter([list(b) for b in bs])
    for i in range(6):
        out = g.fetch_feature(64, it, "cpu")
        assert np.array_equal(out[-1].numpy(), oracle.gather(FakeStore.table, bs[i][0].numpy()))
    merged = [c for c in g.BAM_FS.calls if c[0] == "read_feature_merged"]
    assert [c[1] for c in merged] == [3, 3]


def test_accumulator_counts_cpu_buffer_hits(fake):
    g = fake(accumulator_flag=True)
    g.required_accesses = 50
    g.set_cpu_buffer(torch.arange(1000), 500)
    bs = batches(6, 40)
    it = iter([list(b) for b in bs])
    g.fetch_feature(64, it, "cpu")
    merged = [c for c in g.BAM_FS.calls if c[0] == "read_feature_merged"]
    assert merged[0][1] == 2
    pins = np.arange(500)
    hits = sum(int(np.isin(b[0].numpy(), pins).sum()) for b in bs[:2])
    assert g.prev_cpu_access == hits // 2  # GIDS.py:980-982


def test_heterograph_key_offsets_and_empty_types(fake):
    hmap = {"paper": 0, "author": 400, "fos": 900}
    g = fake(heterograph=True, heterograph_map=hmap)
    rng = np.random.default_rng(3)
    b = [{"paper": torch.as_tensor(rng.integers(0, 400, 30)), "author": torch.as_tensor(rng.integers(0, 500, 20)),
          "fos": torch.zeros(0, dtype=torch.int64)}, "s", "bl"]
    out = g.fetch_feature(64, iter([b]), "cpu")
    feats = out[-1]
    assert feats["fos"].shape == (0, 64)
    for k in ("paper", "author"):
        exp = oracle.gather(FakeStore.table, b[0][k].numpy(), key_off=hmap[k])
        assert np.array_equal(feats[k].numpy(), exp)
    het = [c for c in g.BAM_FS.calls if c[0] == "read_feature_hetero"]
    assert len(het) == 1 and het[0][1] == 2 and het[0][3] == [0, 400]


def test_heterograph_window_buffering_skips_empty(fake):
    hmap = {"a": 0, "b": 500}
    g = fake(heterograph=True, heterograph_map=hmap, window_buffer=True, wb_size=1)
    b1 = [{"a": torch.tensor([1, 2]), "b": torch.zeros(0, dtype=torch.int64)}]
    b2 = [{"a": torch.tensor([3]), "b": torch.tensor([4])}]
    g.fetch_feature(64, iter([b1, b2]), "cpu")
    wb = [c for c in g.BAM_FS.calls if c[0] == "wb"]
    assert wb == [("wb", (1, 2), 0), ("wb", (3,), 0), ("wb", (4,), 500)]
    g = fake(heterograph=True, heterograph_map=hmap, window_buffer=True, wb_size=1, wb_prefetch=True)
    g.fetch_feature(64, iter([b1, b2]), "cpu")
    pf = [c for c in g.BAM_FS.calls if c[0] == "prefetch"]
    assert pf == [("prefetch", (1, 2), 64, 64, 0), ("prefetch", (3,), 64, 64, 0), ("prefetch", (4,), 64, 64, 500)]


def test_out_of_scope_methods_raise(fake):
    g = fake()
    for m in (lambda: g.init_graph_GIDS(4096, 0, 1, 1, 1), g.get_offset_array, g.get_array_ptr):
        with pytest.raises(NotImplementedError):
            m()


def test_store_tensor_passes_rows(fake):
    g = fake()
    t = torch.zeros((5, 1024))
    g.store_tensor(t, 0)
    assert ("store_tensor", t.data_ptr(), 5, 0) in g.BAM_FS.calls
