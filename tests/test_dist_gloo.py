"""Multi-rank host logic on CPU (gloo, world size 2): the bench's
max/sum/gather-over-ranks timing helpers, per-rank sampler seeds, and the CUDA IPC
handle exchange of a sharded GIDS (with a fake store recording what it got)."""
import os
import sys

import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _worker(rank, world, port, q):
    try:
        for p in (REPO, os.path.join(REPO, "gids-study_b200"), HERE):
            sys.path.insert(0, p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                          LOCAL_RANK=str(rank))
        import bench

        d = bench.Dist()
        d.init("gloo")
        t_max = d.max(1.0 + rank)
        s_sum = d.sum(10.0 * (rank + 1))
        per_rank = d.gather(0.5 + rank)
        d.barrier()

        # sharded GIDS handle exchange with a fake store
        import torch

        import GIDS  # noqa: F401

        gmod = sys.modules["GIDS.GIDS"]

        class FakeCtrl:
            def init_GIDS_controllers(self, *a):
                pass

            def set_emulation(self, *a):
                pass

        class FakeStore:
            def __init__(self):
                self.calls = []

            def __getattr__(self, name):
                def rec(*a):
                    self.calls.append((name,) + a)

                return rec

            def ipc_handle(self):
                return bytes([rank]) * 64

            def open_peers(self, handles):
                self.calls.append(("open_peers", list(handles)))

            def geometry(self):
                return {"shard_bytes": 1 << 21}

        import types

        gmod._feature_store_module = lambda: types.SimpleNamespace(BAM_Feature_Store_float=FakeStore,
                                                                   GIDS_Controllers=FakeCtrl)
        g = gmod.GIDS(page_size=4096, cache_dim=64, num_ele=1000 * 64, shard_cache=True, replicas=100)
        n_rep = g.replicate_rows(torch.tensor([0, 16, 17, 5]))  # 256-byte rows: lines 0 and 1
        names = [c[0] for c in g.BAM_FS.calls]
        opened = [c for c in g.BAM_FS.calls if c[0] == "open_peers"][0][1]
        rep_call = [c for c in g.BAM_FS.calls if c[0] == "set_replicated_lines"][0]
        q.put((rank, t_max, s_sum, bench.sampler_seed(rank), g.world, g.rank, names, opened, per_rank,
               (n_rep, rep_call[2], ("set_replicas", 100) in g.BAM_FS.calls)))
        d.close()
    except Exception as e:
        q.put((rank, "error", repr(e)))


def test_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r = q.get(timeout=180)
            out[r[0]] = r
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert out[r][1] != "error", out[r]
        _, t_max, s_sum, seed, world, grank, names, opened, per_rank, reps = out[r]
        assert t_max == 2.0 and s_sum == 30.0  # max and sum over both ranks
        assert per_rank == [0.5, 1.5]  # every rank's value, in rank order
        assert seed == 1000 + r
        assert (world, grank) == (2, r)
        # sharding is set before init_controllers; handles arrive in rank order
        assert names.index("set_sharding") < names.index("init_controllers") < names.index("open_peers")
        assert opened == [bytes([0]) * 64, bytes([1]) * 64]
        # replicas are reserved before the shard exists; two distinct lines are replicated
        assert names.index("set_sharding") < names.index("set_replicas") < names.index("init_controllers")
        assert reps == (2, 2, True)
