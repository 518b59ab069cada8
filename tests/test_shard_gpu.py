"""Page cache sharded by page id (page p owned by rank p % world).

* one process, one GPU: two stores (ranks 0 and 1) share their shards and
  gather one after the other (never concurrently on one GPU); every fill,
  hit and eviction of a page happens in its owner's shard;
* one process per GPU (2 GPUs, skipped otherwise): the shards are mapped
  through CUDA IPC handles exchanged over torch.distributed (gloo), and every
  rank gathers both its own and the other rank's ids, bit-exact against the
  oracle, with hits read from the peer's HBM.
"""
import ctypes
import os
import tempfile

import numpy as np
import pytest
import torch

import gids_abi
from gids_abi import check
from oracle import oracle

pytestmark = pytest.mark.gpu


def bits_equal(a: torch.Tensor, b: np.ndarray) -> bool:
    return a.detach().cpu().numpy().tobytes() == np.ascontiguousarray(b).tobytes()


class Shared:
    """Controllers + `world` stores on one device, shards shared in-process."""

    def __init__(self, table, world, page=4096, cache_mb=1, num_ssd=2, device=0, line=0, admission=True, replicas=0):
        L = gids_abi.lib()
        self.c = ctypes.c_void_p()
        check(L.gids_ctrls_create(ctypes.byref(self.c)))
        lst = (ctypes.c_int32 * num_ssd)(*range(num_ssd))
        check(L.gids_ctrls_init(self.c, num_ssd, 1024, 128, lst))
        check(L.gids_ctrls_bind(self.c, num_ssd, page, 0, table.nbytes))
        check(L.gids_ctrls_write(self.c, table.ctypes.data, table.nbytes, 0))
        self.s = []
        for r in range(world):
            s = ctypes.c_void_p()
            check(L.gids_store_create(ctypes.byref(s), table.dtype.itemsize, device))
            check(L.gids_store_set_sharding(s, world, r))
            if line:
                check(L.gids_store_set_cache_line(s, line))
            if replicas:
                check(L.gids_store_set_replicas(s, replicas))
            check(L.gids_store_init_controllers(s, self.c, page, 0, cache_mb, table.size, num_ssd))
            check(L.gids_store_set_cache_policy(s, 1 if admission else 0, 3))
            self.s.append(s)
        arr = (ctypes.c_void_p * world)(*self.s)
        check(L.gids_store_share_shards(arr, world))

    def gather(self, r, ids, dim, cdim):
        d = torch.as_tensor(ids, dtype=torch.int64).cuda()
        out = torch.empty((len(ids), dim), device="cuda", dtype=torch.float32)
        rc = gids_abi.lib().gids_read_feature(self.s[r], out.data_ptr(), d.data_ptr(), len(ids), dim, cdim, 0, None)
        torch.cuda.synchronize()
        check(rc)
        return out

    def stats(self, r):
        v = (ctypes.c_uint64 * gids_abi.N_STATS)()
        check(gids_abi.lib().gids_get_stats(self.s[r], v, gids_abi.N_STATS))
        return dict(zip(gids_abi.STAT_NAMES, list(v)))

    def close(self):
        L = gids_abi.lib()
        for s in self.s:
            check(L.gids_store_destroy(s))
        check(L.gids_ctrls_destroy(self.c))


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    yield


def test_gather_refused_before_peers_attached():
    L = gids_abi.lib()
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 100, 256)
    c = ctypes.c_void_p()
    check(L.gids_ctrls_create(ctypes.byref(c)))
    lst = (ctypes.c_int32 * 1)(0)
    check(L.gids_ctrls_init(c, 1, 1024, 128, lst))
    s = ctypes.c_void_p()
    check(L.gids_store_create(ctypes.byref(s), 4, 0))
    check(L.gids_store_set_sharding(s, 2, 0))
    check(L.gids_store_init_controllers(s, c, 4096, 0, 1, t.size, 1))
    d = torch.arange(4, dtype=torch.int64, device="cuda")
    out = torch.empty((4, 256), device="cuda")
    assert L.gids_read_feature(s, out.data_ptr(), d.data_ptr(), 4, 256, 256, 0, None) == gids_abi.GIDS_E_STATE
    h = ctypes.create_string_buffer(64)
    check(L.gids_store_ipc_handle(s, h, 64))
    # the shard a peer maps through CUDA IPC is a whole number of 2 MB pages
    # (an odd-sized one is mapped with small pages and read at a third of the link)
    g = (ctypes.c_uint64 * 8)()
    check(L.gids_store_geometry(s, g, 8))
    assert g[7] > 0 and g[7] % (2 << 20) == 0
    check(L.gids_store_destroy(s))
    check(L.gids_ctrls_destroy(c))


@pytest.mark.parametrize("world", [2, 3])
def test_in_process_shards_one_gpu(world):
    rows, cdim = 12000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 21, rows, cdim)
    sh = Shared(t, world, cache_mb=64, admission=False)  # 16384 slots per shard: nothing is evicted
    rng = np.random.default_rng(world)
    try:
        ids = rng.integers(0, rows, size=5000)
        out = sh.gather(0, ids, cdim, cdim)
        assert bits_equal(out, oracle.gather(t, ids))
        st0 = sh.stats(0)
        assert st0["bytes_peer"] > 0 and st0["read_io"] > 0 and st0["evictions"] == 0
        # the same ids from every other rank: the pages sit in their owners' shards
        for r in range(1, world):
            out = sh.gather(r, ids, cdim, cdim)
            assert bits_equal(out, oracle.gather(t, ids))
            st = sh.stats(r)
            assert st["miss"] == 0 and st["bypass"] == 0 and st["hit"] == st["access"]
            assert st["bytes_peer"] > 0
    finally:
        sh.close()


@pytest.mark.parametrize("world", [2, 3])
def test_in_process_shards_prefetch(world):
    """A prefetch by one rank fills the owners' shards; every rank's gather then hits."""
    rows, cdim = 6000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 27, rows, cdim)
    sh = Shared(t, world, cache_mb=64, admission=False)
    L = gids_abi.lib()
    try:
        ids = np.random.default_rng(world + 10).integers(0, rows, size=3000)
        d = torch.as_tensor(ids, dtype=torch.int64).cuda()
        check(L.gids_reset_stats(sh.s[0]))
        check(L.gids_prefetch(sh.s[0], ctypes.c_void_p(d.data_ptr()), len(ids), cdim, cdim, 0, None))
        torch.cuda.synchronize()
        st = sh.stats(0)
        assert st["rows"] == 0 and st["read_io"] == len(np.unique(ids))  # every distinct line, in its owner's shard
        for r in range(world):
            check(L.gids_reset_stats(sh.s[r]))
            out = sh.gather(r, ids, cdim, cdim)
            assert bits_equal(out, oracle.gather(t, ids))
            st = sh.stats(r)
            assert st["miss"] == 0 and st["bypass"] == 0 and st["hit"] == st["access"]
    finally:
        sh.close()


def _replicate(sh, lines):
    arr = np.ascontiguousarray(np.asarray(lines, dtype=np.uint64))
    for s in sh.s:
        check(gids_abi.lib().gids_store_set_replicated_lines(s, arr.ctypes.data, len(arr)))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_in_process_shards_replicated_lines(world):
    """Replicated lines live in every rank's own shard: their hits are local,
    each rank fills its own copy, and every gather stays bit-exact."""
    rows, cdim = 6000, 1024  # 4 KB rows: row i is line i
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 29, rows, cdim)
    sh = Shared(t, world, cache_mb=64, admission=False, replicas=1000)
    rng = np.random.default_rng(world + 20)
    L = gids_abi.lib()
    try:
        rep_lines = np.sort(rng.choice(rows, size=700, replace=False))
        _replicate(sh, rep_lines)
        ids = np.concatenate([rep_lines, rng.choice(rep_lines, size=1300)])
        rng.shuffle(ids)
        for r in range(world):  # every rank fills its own copies, then hits them
            check(L.gids_reset_stats(sh.s[r]))
            assert bits_equal(sh.gather(r, ids, cdim, cdim), oracle.gather(t, ids))
            st = sh.stats(r)
            assert st["bytes_peer"] == 0 and st["read_io"] == len(np.unique(ids)) and st["bypass"] == 0
            check(L.gids_reset_stats(sh.s[r]))
            assert bits_equal(sh.gather(r, ids[::-1].copy(), cdim, cdim), oracle.gather(t, ids[::-1]))
            st = sh.stats(r)
            assert st["hit"] == st["access"] and st["bytes_peer"] == 0
        # the other lines stay sharded by page id: hits on them come from the owners
        other = np.setdiff1d(np.arange(rows), rep_lines)
        ids2 = rng.choice(other, size=3000)
        mixed = np.concatenate([ids2, rng.choice(rep_lines, size=500)])
        rng.shuffle(mixed)
        for r in range(world):
            check(L.gids_reset_stats(sh.s[r]))
            assert bits_equal(sh.gather(r, mixed, cdim, cdim), oracle.gather(t, mixed))
        st = sh.stats(world - 1)  # by now every line is resident: a sharded hit off-rank is a peer read
        assert st["hit"] == st["access"] and st["bytes_peer"] > 0
        # the replica entries follow the owned ones: a set larger than reserved, or unsorted, is refused
        big = np.arange(1001, dtype=np.uint64)
        assert L.gids_store_set_replicated_lines(sh.s[0], big.ctypes.data, len(big)) == gids_abi.GIDS_E_RANGE
        bad = np.array([5, 3], dtype=np.uint64)
        assert L.gids_store_set_replicated_lines(sh.s[0], bad.ctypes.data, 2) == gids_abi.GIDS_E_INVAL
    finally:
        sh.close()


def test_replicated_lines_pinned_under_static_policy():
    """Pins of replicated rows pin each rank's own copy; the static policy then
    holds them locally on every rank."""
    rows, cdim, world = 4000, 1024, 2
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 30, rows, cdim)
    sh = Shared(t, world, cache_mb=8, admission=False, replicas=256)  # 2048 slots per shard
    L = gids_abi.lib()
    try:
        hot = np.arange(100, 356)  # 256 rows, replicated
        _replicate(sh, hot)
        d = torch.as_tensor(hot, dtype=torch.int64).cuda()
        for r in range(world):
            check(L.gids_store_set_cache_policy(sh.s[r], 2, 3))
            check(L.gids_store_pin_rows(sh.s[r], ctypes.c_void_p(d.data_ptr()), len(hot), 0, 0, None))
        torch.cuda.synchronize()
        for r in range(world):
            sh.gather(r, hot, cdim, cdim)  # fills the pinned copies
            check(L.gids_reset_stats(sh.s[r]))
            out = sh.gather(r, np.concatenate([hot, np.arange(2000, 2100)]), cdim, cdim)
            assert bits_equal(out, oracle.gather(t, np.concatenate([hot, np.arange(2000, 2100)])))
            st = sh.stats(r)
            assert st["hit"] == 256 and st["bypass"] == 100 and st["bytes_peer"] == 0
    finally:
        sh.close()


def test_replicated_rows_straddling_small_lines():
    """fp16 rows of 1536 bytes over 512-byte lines: a replicated row's three lines
    are all local; rows sharing a line with a replicated row stay exact."""
    rows, cdim, world = 5000, 768, 2
    t = oracle.synth_table(oracle.KIND_F16_NORMAL, 31, rows, cdim)
    sh = Shared(t, world, cache_mb=16, line=512, admission=False, replicas=4000)
    L = gids_abi.lib()
    try:
        rng = np.random.default_rng(33)
        rep_rows = np.sort(rng.choice(rows, size=900, replace=False))
        stride = cdim * 2
        lines = np.unique(np.concatenate([(rep_rows * stride + k * 512) // 512 for k in range(3)]))
        _replicate(sh, lines)
        for r in range(world):
            d = torch.as_tensor(rep_rows, dtype=torch.int64).cuda()
            out = torch.empty((len(rep_rows), cdim), device="cuda", dtype=torch.float16)
            check(L.gids_reset_stats(sh.s[r]))
            check(L.gids_read_feature(sh.s[r], out.data_ptr(), d.data_ptr(), len(rep_rows), cdim, cdim, 0, None))
            torch.cuda.synchronize()
            assert bits_equal(out, oracle.gather(t, rep_rows))
            assert sh.stats(r)["bytes_peer"] == 0
            mixed = rng.integers(0, rows, size=3000)
            dm = torch.as_tensor(mixed, dtype=torch.int64).cuda()
            out = torch.empty((len(mixed), cdim), device="cuda", dtype=torch.float16)
            check(L.gids_read_feature(sh.s[r], out.data_ptr(), dm.data_ptr(), len(mixed), cdim, cdim, 0, None))
            torch.cuda.synchronize()
            assert bits_equal(out, oracle.gather(t, mixed))
    finally:
        sh.close()


def test_replicas_need_a_sharded_cache():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 100, 256)
    s = gids_abi.Store(4, 4096, t.size, 1)
    try:
        one = np.array([1], dtype=np.uint64)
        assert gids_abi.lib().gids_store_set_replicated_lines(s.s, one.ctypes.data, 1) == gids_abi.GIDS_E_STATE
    finally:
        s.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_in_process_shards_churn(world):
    rows, cdim = 12000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 23, rows, cdim)
    sh = Shared(t, world, cache_mb=1)  # 256 slots per shard
    rng = np.random.default_rng(10 + world)
    try:
        for k in range(8):
            ids = rng.integers(0, rows, size=7000)
            out = sh.gather(k % world, ids, cdim, cdim)
            assert bits_equal(out, oracle.gather(t, ids))
        tot = [sh.stats(r) for r in range(world)]
        assert sum(s["evictions"] for s in tot) > 0
        assert all(s["access"] == s["hit"] + s["miss"] + s["bypass"] for s in tot)
    finally:
        sh.close()


def test_in_process_shards_with_small_lines():
    rows, cdim = 30000, 128  # 512-byte rows, 512-byte cache lines, 4 KB stripe pages
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 24, rows, cdim)
    sh = Shared(t, 2, cache_mb=1, line=512)
    rng = np.random.default_rng(24)
    try:
        for k in range(4):
            ids = rng.integers(0, rows, size=9000)
            out = sh.gather(k % 2, ids, cdim, cdim)
            assert bits_equal(out, oracle.gather(t, ids))
    finally:
        sh.close()


def test_in_process_shards_window_buffering():
    rows, cdim = 8000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 22, rows, cdim)
    sh = Shared(t, 2, cache_mb=2)
    L = gids_abi.lib()
    rng = np.random.default_rng(5)
    try:
        b = [torch.as_tensor(rng.integers(0, rows, size=400)).cuda() for _ in range(4)]
        for x in b:
            check(L.gids_set_window_buffering(sh.s[0], ctypes.c_void_p(x.data_ptr()), len(x), 0, 0, None))
        for x in b:
            out = sh.gather(0, x.cpu().numpy(), cdim, cdim)
            assert bits_equal(out, oracle.gather(t, x.cpu().numpy()))
        flood = rng.integers(0, rows, size=6000)
        out = sh.gather(1, flood, cdim, cdim)
        assert bits_equal(out, oracle.gather(t, flood))
    finally:
        sh.close()


# ------------------------------------------------------------- two processes
def _rank_main(rank, world, port, pattern, rows, cdim, q):
    try:
        import sys

        here = os.path.dirname(os.path.abspath(__file__))
        repo = os.path.dirname(here)
        for p in (repo, os.path.join(repo, "gids-study_b200"), here):
            sys.path.insert(0, p)
        import datetime

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        torch.cuda.set_device(rank)
        import GIDS
        from oracle import oracle as orc

        t = orc.synth_table(orc.KIND_F32_UNIFORM, 31, rows, cdim)
        if rank == 0:
            import BAM_Feature_Store

            c = BAM_Feature_Store.GIDS_Controllers()
            c.init_GIDS_controllers(2, 1024, 128, [0, 1])
            c.set_emulation(0, pattern)
            c.bind(2, 4096, 0, t.nbytes)
            c.write(t.ctypes.data, t.nbytes, 0)
            del c
        dist.barrier()
        g = GIDS.GIDS(page_size=4096, cache_dim=cdim, num_ele=t.size, num_ssd=2, cache_size=16, ctrl_idx=rank,
                      ssd_path=pattern, synchronous=True, shard_cache=True)
        assert g.world == world and g.rank == rank
        rng = [np.random.default_rng(100 + r) for r in range(world)]
        ids = [rng[r].integers(0, rows, size=4000) for r in range(world)]
        for step in range(3):
            mine = ids[rank] if step != 1 else ids[(rank + 1) % world]
            out = g.fetch_feature(cdim, iter([[torch.as_tensor(mine)]]), g.gids_device)[-1]
            torch.cuda.synchronize()
            ok = out.cpu().numpy().tobytes() == orc.gather(t, mine).tobytes()
            if not ok:
                raise AssertionError(f"rank {rank} step {step}: gathered rows differ")
            dist.barrier()
        st = g.get_stats()
        g.close()
        dist.destroy_process_group()
        q.put((rank, "ok", int(st["bytes_peer"]), int(st["hit"])))
    except Exception as e:  # reported to the parent
        q.put((rank, f"error: {type(e).__name__}: {e}", 0, 0))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_processes_two_gpus_ipc_shards():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    d = tempfile.mkdtemp(dir="/dev/shm" if os.path.isdir("/dev/shm") else None)
    pattern = os.path.join(d, "ssd{}")
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, pattern, 20000, 1024, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, msg, peer, hit = q.get(timeout=240)
            res[r] = (msg, peer, hit)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
        for f in os.listdir(d):
            os.unlink(os.path.join(d, f))
        os.rmdir(d)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    assert res[0][1] > 0 and res[1][1] > 0  # hits served from the peer GPU's shard
