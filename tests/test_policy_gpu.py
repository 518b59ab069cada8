"""Cache replacement policy: once the cache is full, a line's first miss
within a window of twice the cache's slots reads the backing store directly
and its second miss inserts it (admission); an empty cache admits every miss;
the window ages; lines that window buffering pinned for later batches are
inserted at once; the clock counter ceiling is bounded. The policy changes
hit ratios only: every gather stays bit-exact."""
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
    return oracle.synth_table(oracle.KIND_F32_UNIFORM, 41, ROWS, CDIM)


def make(t, cache_mb):
    s = Store(4, 4096, t.size, cache_mb, num_ssd=2)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    return s


def run(s, t, ids):
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    out = torch.empty((len(ids), CDIM), device="cuda")
    s.reset_stats()
    check(s.read_feature(out.data_ptr(), d.data_ptr(), len(ids), CDIM, CDIM))
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == oracle.gather(t, ids).tobytes()
    st = s.stats()
    assert st["access"] == st["hit"] + st["miss"] + st["bypass"]
    return st


def filled(t):
    """A 256-slot cache (1 MB of 4 KB lines) that one launch over 256 lines has
    filled: eight warps took the clock's first 8 x 32 slots, the hand has gone
    round, so admission applies from the next launch. 256 of the 512-reference
    admission window are used."""
    s = make(t, 1)
    st = run(s, t, np.arange(ROWS - 256, ROWS))
    assert (st["miss"], st["bypass"], st["evictions"]) == (256, 0, 0)  # an empty cache inserts every miss
    return s


def test_first_miss_bypasses_second_miss_inserts(table):
    s = filled(table)
    b = np.arange(0, 150, 3)  # 50 lines
    st = run(s, table, b)
    assert (st["bypass"], st["miss"], st["read_io"]) == (50, 0, 0)
    st = run(s, table, b)  # 356 references: still inside the window
    assert (st["bypass"], st["miss"], st["read_io"]) == (0, 50, 50)
    st = run(s, table, b[::-1].copy())
    assert st["hit"] == 50
    # with admission off every miss inserts, as in the reference
    s.set_policy(False, 1)
    c = np.arange(1000, 1050)
    st = run(s, table, c)
    assert (st["bypass"], st["miss"]) == (0, 50)
    s.close()


def test_admission_window_ages(table):
    s = filled(table)
    a = np.arange(0, 100)
    assert run(s, table, a)["bypass"] == 100  # 356 references
    flood = np.arange(1000, 1200)  # 556 > 512: the bits are cleared before this launch
    assert run(s, table, flood)["bypass"] == 200
    st = run(s, table, a)  # a's bits went with the clear
    assert st["bypass"] == 100 and st["miss"] == 0
    # flush_cache empties the cache, forgets the bits and restarts the clock:
    # every miss inserts again
    check(gids_abi.lib().gids_flush_cache(s.s))
    st = run(s, table, a)
    assert (st["miss"], st["bypass"]) == (100, 0)
    s.close()


def test_window_buffer_pins_admit_at_once(table):
    s = filled(table)
    L = gids_abi.lib()
    ids = np.arange(500, 600)
    d = torch.as_tensor(ids).cuda()
    for _ in range(2):  # this batch and a later one in the window
        check(L.gids_set_window_buffering(s.s, ctypes.c_void_p(d.data_ptr()), len(ids), 0, 0, None))
    st = run(s, table, ids)
    assert (st["miss"], st["bypass"]) == (len(ids), 0)
    st = run(s, table, ids)
    assert st["hit"] == len(ids)
    # pins of this batch alone do not admit
    other = np.arange(800, 850)
    d2 = torch.as_tensor(other).cuda()
    check(L.gids_set_window_buffering(s.s, ctypes.c_void_p(d2.data_ptr()), len(other), 0, 0, None))
    st = run(s, table, other)
    assert (st["miss"], st["bypass"]) == (0, len(other))
    s.close()


@pytest.mark.parametrize("admission,ref_max", [(False, 1), (True, 1), (False, 3), (True, 3), (True, 255)])
def test_every_policy_is_exact_under_churn(table, admission, ref_max):
    s = make(table, 1)
    s.set_policy(admission, ref_max)
    rng = np.random.default_rng(ref_max + 7 * admission)
    hot = rng.integers(0, ROWS, size=200)
    ev = 0
    for _ in range(6):
        ids = np.concatenate([rng.choice(hot, size=3000), rng.integers(0, ROWS, size=3000)])
        rng.shuffle(ids)
        ev += run(s, table, ids)["evictions"]
    assert ev > 0
    s.close()


def test_policy_arguments(table):
    s = make(table, 1)
    L = gids_abi.lib()
    assert L.gids_store_set_cache_policy(s.s, 1, 0) == gids_abi.GIDS_E_INVAL
    assert L.gids_store_set_cache_policy(s.s, 1, 256) == gids_abi.GIDS_E_INVAL
    check(L.gids_store_set_cache_policy(s.s, 0, 2))
    s.close()


def _mark(s, ids, times=1, unset=False):
    L = gids_abi.lib()
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    f = L.gids_unset_window_buffering if unset else L.gids_set_window_buffering
    for _ in range(times):
        check(f(s.s, ctypes.c_void_p(d.data_ptr()), len(ids), 0, 0, None))
    torch.cuda.synchronize()


def test_abandoned_window_no_longer_blocks_eviction(table):
    # a 256-slot cache whose every line is pinned by a window that is marked
    # but never gathered: a miss finds no victim and reads through
    s = make(table, 1)
    s.set_policy(False, 1)  # insert every miss (the reference's rule), second-chance clock
    a = np.arange(0, 256)
    _mark(s, a, times=2)  # this batch, and a later batch that will be abandoned
    assert run(s, table, a)["miss"] == 256  # fills every slot, consumes one pin of each line
    st = run(s, table, np.arange(1000, 1256))
    assert (st["evictions"], st["bypass"], st["miss"]) == (0, 256, 0)
    # the abandoned window's marks are taken back: its lines can go
    _mark(s, a, unset=True)
    _mark(s, a, unset=True)  # saturates at zero
    st = run(s, table, np.arange(2000, 2256))
    assert (st["evictions"], st["miss"], st["bypass"]) == (256, 256, 0)
    s.close()


def test_flush_cache_drops_window_pins(table):
    s = make(table, 1)
    s.set_policy(False, 1)
    a = np.arange(0, 256)
    _mark(s, a, times=3)
    assert run(s, table, a)["miss"] == 256  # 2 pins left on each line
    check(gids_abi.lib().gids_flush_cache(s.s))  # drops the lines and their pins
    assert run(s, table, a)["miss"] == 256  # refilled; pins would now be 1 without the flush's clear
    st = run(s, table, np.arange(2000, 2256))
    assert (st["evictions"], st["miss"], st["bypass"]) == (256, 256, 0)
    s.close()


def _pin(s, ids, unpin=False):
    L = gids_abi.lib()
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    f = L.gids_store_unpin_rows if unpin else L.gids_store_pin_rows
    check(f(s.s, ctypes.c_void_p(d.data_ptr()), len(ids), 0, 0, None))
    torch.cuda.synchronize()


def test_static_policy_holds_only_pinned_lines(table):
    s = make(table, 1)  # 256 slots
    s.set_policy(2, 3)
    hot = np.arange(0, 200)
    _pin(s, hot)
    st = run(s, table, hot)
    assert (st["miss"], st["read_io"], st["bypass"]) == (200, 200, 0)  # inserted on first touch
    st = run(s, table, np.arange(1000, 1200))
    assert (st["bypass"], st["miss"], st["evictions"]) == (200, 0, 0)  # unpinned rows read through
    st = run(s, table, hot[::-1].copy())
    assert st["hit"] == 200
    # unpinned lines become evictable again once the policy inserts misses
    _pin(s, hot[:100], unpin=True)
    s.set_policy(0, 1)
    st = run(s, table, np.arange(2000, 2156))  # the 56 free slots, then evictions of the unpinned lines
    assert st["miss"] == 156 and st["bypass"] == 0 and st["evictions"] == 100
    assert run(s, table, hot[100:])["hit"] == 100  # still pinned, never evicted
    s.close()


def test_permanent_pins_survive_window_consumption_and_flush_drops_them(table):
    s = make(table, 1)
    s.set_policy(0, 1)  # insert every miss: only the pins protect lines
    hot = np.arange(0, 128)
    _pin(s, hot)
    _mark(s, hot, times=2)  # window marks on pinned lines are consumed by gathers, the pin bit stays
    assert run(s, table, hot)["miss"] == 128
    run(s, table, hot)
    for k in range(4):  # churn through the other 128 slots many times over
        run(s, table, np.arange(1000 + 400 * k, 1400 + 400 * k))
    assert run(s, table, hot)["hit"] == 128
    check(gids_abi.lib().gids_flush_cache(s.s))  # drops the lines and every pin
    assert run(s, table, hot)["miss"] == 128
    st = run(s, table, np.arange(2000, 2256))
    assert st["evictions"] > 0
    s.close()


def test_out_degree_and_hot_rows(built):
    from GIDS.sampler import hot_rows, out_degree

    rng = np.random.default_rng(5)
    n = 50000
    for dt in (np.int32, np.int64):
        ind = rng.zipf(1.3, size=400000) % n
        ind = ind.astype(dt)
        d = torch.as_tensor(ind).cuda()
        got = out_degree(d, n).cpu().numpy()
        want = np.bincount(ind.astype(np.int64), minlength=n)
        assert np.array_equal(got, want)
        top = hot_rows(d, n, 777).cpu().numpy()
        order = np.lexsort((np.arange(n), -want))
        assert top.tolist() == order[:777].tolist()
    L = gids_abi.lib()
    bad = torch.tensor([1, 2, n + 5], dtype=torch.int64, device="cuda")
    cnt = torch.empty(n, dtype=torch.int32, device="cuda")
    assert L.gids_out_degree(0, bad.data_ptr(), 8, 3, n, cnt.data_ptr(), None) == gids_abi.GIDS_E_RANGE
