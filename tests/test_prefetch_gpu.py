"""Window-buffer prefetch (gids_prefetch): the gather without an output. The
rows' missing lines that the gather would insert (every line while the cache
fills; once it is full, lines pinned for a later batch or missed before in the
admission window; under the static policy, permanently pinned lines) are read
from the backing store into the cache ahead of the gather, and nothing is
copied out. Lines the gather would read through are left to it, and the
prefetch sets no admission bit. A later gather of the rows finds the inserted
lines resident and stays bit-exact. A prefetch counts only the lines it
inserted."""
import ctypes

import numpy as np
import pytest
import torch

import gids_abi
from gids_abi import Store, check
from oracle import oracle

pytestmark = pytest.mark.gpu

ROWS, CDIM = 3000, 1024  # 4 KB rows: row i is cache line i


@pytest.fixture(scope="module")
def table(built):
    return oracle.synth_table(oracle.KIND_F32_UNIFORM, 43, ROWS, CDIM)


def make(t, cache_mb, **kw):
    s = Store(t.dtype.itemsize, 4096, t.size, cache_mb, num_ssd=2, **kw)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    return s


def gather(s, t, ids, dim=None, cdim=None):
    cdim = cdim or t.shape[1]
    dim = dim or cdim
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    out = torch.empty((len(ids), dim), dtype=torch.float32 if t.dtype == np.float32 else torch.float16, device="cuda")
    s.reset_stats()
    check(s.read_feature(out.data_ptr(), d.data_ptr(), len(ids), dim, cdim))
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == oracle.gather(t, ids, dim=dim).tobytes()
    return s.stats()


def prefetch(s, ids, dim, cdim, key_off=0):
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    s.reset_stats()
    check(gids_abi.lib().gids_prefetch(s.s, ctypes.c_void_p(d.data_ptr()), len(ids), dim, cdim, key_off, None))
    torch.cuda.synchronize()
    return s.stats()


def full_cache(t):
    """256 slots filled by one launch: admission applies from the next launch"""
    s = make(t, 1)
    st = gather(s, t, np.arange(ROWS - 256, ROWS))
    assert st["miss"] == 256
    return s


def test_prefetch_inserts_what_the_gather_would_insert(table):
    s = full_cache(table)
    ids = np.arange(0, 300, 6)  # 50 lines never seen: the gather of a full cache reads them through
    st = prefetch(s, ids, CDIM, CDIM)
    assert (st["prefetched"], st["read_io"], st["evictions"]) == (0, 0, 0)
    st = gather(s, table, ids)  # the prefetch set no admission bit: still read through, bits set now
    assert (st["bypass"], st["miss"]) == (50, 0)
    st = prefetch(s, ids, CDIM, CDIM)  # missed before in this window: the gather would insert them
    assert (st["prefetched"], st["read_io"]) == (50, 50)
    assert (st["rows"], st["access"], st["hit"], st["miss"], st["bypass"]) == (0, 0, 0, 0, 0)
    st = gather(s, table, ids[::-1].copy())
    assert (st["hit"], st["miss"], st["bypass"], st["read_io"]) == (50, 0, 0, 0)
    # a second prefetch of resident lines inserts nothing
    assert prefetch(s, ids, CDIM, CDIM)["prefetched"] == 0
    # duplicates in one prefetch are fetched once
    dup = np.repeat(np.arange(1000, 1010), 7)
    assert gather(s, table, np.arange(1000, 1010))["bypass"] == 10
    assert prefetch(s, dup, CDIM, CDIM)["prefetched"] == 10
    assert gather(s, table, dup)["hit"] == 70
    s.close()


def test_prefetch_inserts_lines_pinned_for_a_later_batch(table):
    s = full_cache(table)
    ids = np.arange(400, 440)
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    L = gids_abi.lib()
    for _ in range(2):  # two batches of the window read these rows
        check(L.gids_set_window_buffering(s.s, ctypes.c_void_p(d.data_ptr()), len(ids), 0, 0, None))
    torch.cuda.synchronize()
    assert prefetch(s, ids, CDIM, CDIM)["prefetched"] == 40  # pins beyond this batch's own: inserted
    for _ in range(2):  # each gather consumes one pin per row and finds the lines resident
        assert gather(s, table, ids)["hit"] == 40
    s.close()


def test_prefetch_skips_bad_ids_and_reports_nothing(table):
    s = make(table, 1)  # an empty cache: every line the prefetch touches is inserted
    ids = np.array([5, ROWS + 7, 9, -3, 11])
    st = prefetch(s, ids, CDIM, CDIM)
    assert st["prefetched"] == 3 and st["bad_ids"] == 0
    # no error was left behind for the next call
    st = gather(s, table, np.array([5, 9, 11]))
    assert st["hit"] == 3
    s.close()


def test_prefetch_under_static_policy_fetches_only_pinned_lines(table):
    s = make(table, 1)
    s.set_policy(2, 3)
    hot = np.arange(0, 100)
    d = torch.as_tensor(hot, dtype=torch.int64).cuda()
    check(gids_abi.lib().gids_store_pin_rows(s.s, ctypes.c_void_p(d.data_ptr()), len(hot), 0, 0, None))
    torch.cuda.synchronize()
    st = prefetch(s, np.arange(0, 200), CDIM, CDIM)  # 100 pinned, 100 not
    assert st["prefetched"] == 100
    st = gather(s, table, np.arange(0, 200))
    assert (st["hit"], st["bypass"], st["miss"]) == (100, 100, 0)
    s.close()


def test_prefetch_rows_straddling_small_lines(built):
    # fp16 rows of 768 columns (1536 B) over 512-byte lines: a row spans 3 or 4 lines
    rows, cdim = 4000, 768
    t = oracle.synth_table(oracle.KIND_F16_NORMAL, 44, rows, cdim)
    s = make(t, 1, cache_line=512)
    ids = np.random.default_rng(3).integers(0, rows, 300)
    st = prefetch(s, ids, cdim, cdim)
    assert st["prefetched"] > 0 and st["prefetched"] == st["read_io"]
    st = gather(s, t, ids)
    assert st["miss"] == 0 and st["bypass"] == 0 and st["hit"] == st["access"]
    # a prefetch of the first 100 columns fetches only the lines those columns touch
    s2 = make(t, 1, cache_line=512)
    ids2 = np.arange(0, 400, 2)
    st = prefetch(s2, ids2, 100, cdim)
    assert st["prefetched"] == len(np.unique(ids2 * cdim * 2 // 512))
    assert gather(s2, t, ids2, dim=100)["hit"] == len(ids2)
    s.close()
    s2.close()


def test_gids_window_buffer_prefetch(built):
    import GIDS

    rows, cdim = 6000, 256
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 45, rows, cdim)
    g = GIDS.GIDS(page_size=4096, cache_dim=cdim, num_ele=rows * cdim, cache_size=16, window_buffer=True,
                  wb_size=2, wb_prefetch=True, synchronous=True)
    try:
        g.BAM_FS.write_range(t.ctypes.data, t.nbytes, 0)
        rng = np.random.default_rng(4)
        bs = [[torch.as_tensor(rng.integers(0, rows, 400))] for _ in range(6)]
        it = iter(bs)
        g.BAM_FS.reset_stats()
        for i in range(4):
            out = g.fetch_feature(cdim, it, "cuda")
            assert out[-1].cpu().numpy().tobytes() == oracle.gather(t, bs[i][0].numpy()).tobytes()
        st = g.BAM_FS.get_stats()
        # every line the gathers needed had been prefetched when its batch entered the window
        assert st["prefetched"] > 0 and st["miss"] == 0 and st["bypass"] == 0
    finally:
        g.close()
