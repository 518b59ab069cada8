"""GIDS.fetch_feature on the GPU through the real store: the policy branches of
the reference's fetch_feature (GIDS_Setup/GIDS/GIDS.py:791-1058) -- window
buffering, the Storage Access Accumulator, heterograph key offsets, the
constant CPU buffer, and their combinations -- each gathered batch checked bit
for bit against the oracle, and handed out in the order the iterator produced
the batches."""
import numpy as np
import pytest
import torch

import GIDS
from oracle import oracle

pytestmark = pytest.mark.gpu

ROWS, CDIM = 6000, 256  # 1 KB rows: four rows per 4 KB page


@pytest.fixture(scope="module")
def table(built):
    return oracle.synth_table(oracle.KIND_F32_UNIFORM, 51, ROWS, CDIM)


def make_gids(t, dtype=torch.float32, cache_mb=1, **kw):
    g = GIDS.GIDS(page_size=4096, cache_dim=t.shape[1], num_ele=t.size, num_ssd=3, cache_size=cache_mb, ctrl_idx=0,
                  dtype=dtype, **kw)
    g.BAM_FS.write_range(t.ctypes.data, t.nbytes, 0)
    return g


def homo_batches(n, size, seed, rows=ROWS):
    rng = np.random.default_rng(seed)
    return [[torch.as_tensor(rng.integers(0, rows, size=size)), f"seeds{i}", f"blocks{i}"] for i in range(n)]


def bits(x: torch.Tensor) -> bytes:
    return x.detach().cpu().contiguous().numpy().view(np.uint8).tobytes()


def check_homo(t, got_batches, want_batches, dim):
    assert len(got_batches) == len(want_batches)
    for got, want in zip(got_batches, want_batches):
        assert got[1] == want[1]  # the same batch, in order
        feat = got[-1]
        assert feat.shape == (len(want[0]), dim)
        assert bits(feat) == oracle.gather(t, want[0].numpy(), dim=dim).tobytes(), want[1]


def run(g, batches, n, dim):
    it = iter([list(b) for b in batches])
    out = [g.fetch_feature(dim, it, g.device) for _ in range(n)]
    torch.cuda.synchronize()
    return out


def test_plain_fetch_matches_oracle(table):
    g = make_gids(table)
    bs = homo_batches(5, 3000, 1)
    check_homo(table, run(g, bs, 5, CDIM), bs, CDIM)
    st = g.get_stats()
    assert st["rows"] == 5 * 3000 and st["launches"] == 5
    g.close()


def test_window_buffering_fetch(table):
    # a 256-slot cache, a window of 3 batches marked ahead, more lines than slots
    g = make_gids(table, window_buffer=True, wb_size=3)
    bs = homo_batches(9, 2500, 2)
    got = run(g, bs, 6, 200)  # column subset; 3 batches stay queued in the window
    check_homo(table, got, bs[:6], 200)
    assert len(g.window_buffer) == 3
    # abandon the window (its marks are taken back) and start a fresh iterator
    g.drop_window_buffer()
    assert g.window_buffer == [] and not g.wb_init
    fresh = homo_batches(7, 2500, 3)  # the refilled window reads 3 batches ahead
    check_homo(table, run(g, fresh, 4, CDIM), fresh[:4], CDIM)
    g.close()


def test_accumulator_merges_batches_into_one_launch(table):
    g = make_gids(table, accumulator_flag=True)
    g.required_accesses = 2.5 * 1000  # about three 1000-row batches per merged launch
    bs = homo_batches(12, 1000, 4)  # the accumulator pulls batches ahead of the ones it hands out
    got = run(g, bs, 9, CDIM)
    check_homo(table, got, bs[:9], CDIM)
    st = g.get_stats()
    assert st["rows"] == 9000 and st["launches"] == 3
    g.close()


def test_accumulator_with_window_buffering(table):
    g = make_gids(table, accumulator_flag=True, window_buffer=True, wb_size=2)
    g.required_accesses = 1.5 * 1200
    bs = homo_batches(10, 1200, 5)
    got = run(g, bs, 7, CDIM)
    check_homo(table, got, bs[:7], CDIM)
    g.close()


TYPES = {"paper": 3000, "author": 2000, "fos": 1000}


def hetero_batches(n, seed, empty_type=None):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        d = {}
        for k, (t, size) in enumerate(TYPES.items()):
            m = 0 if t == empty_type else 400 + 150 * k
            d[t] = torch.as_tensor(rng.integers(0, size, size=m))
        out.append([d, f"seeds{i}", f"blocks{i}"])
    return out


def hmap():
    m, acc = {}, 0
    for t, size in TYPES.items():
        m[t] = acc
        acc += size
    return m


def check_hetero(t, got_batches, want_batches, dim):
    offs = hmap()
    for got, want in zip(got_batches, want_batches):
        assert got[1] == want[1]
        feats = got[-1]
        assert set(feats) == set(want[0])
        for ty, ids in want[0].items():
            assert feats[ty].shape == (len(ids), dim)
            assert bits(feats[ty]) == oracle.gather(t, ids.numpy(), dim=dim, key_off=offs[ty]).tobytes(), (want[1], ty)


def test_heterograph_fetch(table):
    g = make_gids(table, heterograph=True, heterograph_map=hmap())
    bs = hetero_batches(4, 6, empty_type="fos")
    got = run(g, bs, 4, CDIM)
    check_hetero(table, got, bs, CDIM)
    assert g.get_stats()["launches"] == 4  # one launch per batch, whatever the number of types
    g.close()


def test_heterograph_accumulator_and_window(table):
    g = make_gids(table, heterograph=True, heterograph_map=hmap(), accumulator_flag=True, window_buffer=True,
                  wb_size=2)
    g.required_accesses = 1.5 * sum(400 + 150 * k for k in range(3))
    bs = hetero_batches(9, 7)
    got = run(g, bs, 6, 128)
    check_hetero(table, got, bs[:6], 128)
    g.close()


def test_constant_cpu_buffer_through_gids(table):
    g = make_gids(table)
    pins = np.random.default_rng(8).permutation(ROWS)[:700]
    g.cpu_backing_buffer(CDIM, len(pins))
    g.set_cpu_buffer(torch.as_tensor(pins), len(pins))
    bs = homo_batches(4, 3000, 9)
    check_homo(table, run(g, bs, 4, CDIM), bs, CDIM)
    n_pinned = sum(int(np.isin(b[0].numpy(), pins).sum()) for b in bs)
    assert g.BAM_FS.get_cpu_access_count() == n_pinned > 0
    g.close()


def test_half_precision_rows_straddle_pages(built):
    t = oracle.synth_table(oracle.KIND_F16_BYTESUM, 52, 5000, 768)  # 1536-byte rows
    g = make_gids(t, dtype=torch.float16, window_buffer=True, wb_size=2)
    bs = homo_batches(6, 2000, 10, rows=5000)
    got = run(g, bs, 4, 768)
    check_homo(t, got, bs[:4], 768)
    g.close()


def test_sampler_draws_the_same_minibatches_on_cpu_and_gpu(built):
    from GIDS.synthetic import NeighborSampler, SyntheticGraph, seed_batches

    out = {}
    for dev in ("cpu", "cuda"):
        g = SyntheticGraph(200000, 15, 1.1, seed=0, device=dev)
        s = NeighborSampler(g, [15, 10, 5], seed=1000)
        out[dev] = [s.sample(b)[0].cpu() for b in seed_batches(g.N, 512, 3, 1000, device=dev)]
    for a, b in zip(out["cpu"], out["cuda"]):
        assert torch.equal(a, b)


def test_static_hot_set_through_gids(table):
    from GIDS.sampler import hot_rows

    g = make_gids(table, cache_admission="static")  # 1 MB cache: 256 lines of 4 KB (4 rows each)
    rng = np.random.default_rng(12)
    src = torch.as_tensor(rng.zipf(1.2, size=100000) % ROWS).cuda()  # sources of some graph's edges
    hot = hot_rows(src, ROWS, 200)  # at most 200 lines: every pinned line gets a slot
    g.pin_cache(hot)
    st0 = g.get_stats()
    bs = homo_batches(3, 3000, 13)
    check_homo(table, run(g, bs, 3, CDIM), bs, CDIM)
    st = g.get_stats()
    hits = st["hit"] - st0["hit"]
    hot_set = set(hot.cpu().numpy().tolist())
    n_hot_refs = sum(int(np.isin(b[0].numpy(), list(hot_set)).sum()) for b in bs)
    assert st["read_io"] == st0["read_io"] and hits >= n_hot_refs > 0  # nothing new inserted, pinned rows hit
    g.close()
