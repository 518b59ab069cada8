"""Failures made on the host, never by faulting the GPU: a cache line whose
filler never finishes (the bounded wait gives up and the gather reads the
backing store), a pin list with bad node ids, and a store used out of order.
Every case must leave the store usable and the gathered rows exact."""
import ctypes

import numpy as np
import pytest
import torch

import gids_abi
from gids_abi import Store, check
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    yield


def _gather(s, ids, dim, cdim):
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    out = torch.empty((len(ids), dim), device="cuda")
    rc = gids_abi.lib().gids_read_feature(s.s, out.data_ptr(), d.data_ptr(), len(ids), dim, cdim, 0, None)
    torch.cuda.synchronize()
    return rc, out.cpu().numpy()


@pytest.mark.parametrize("line", [0, 512])
def test_bounded_wait_on_a_line_nobody_fills(line):
    rows, cdim = 2000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 51, rows, cdim)
    s = Store(4, 4096, t.size, 16, num_ssd=2, cache_line=line)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    L = gids_abi.lib()
    try:
        check(L.gids_store_set_wait_limit(s.s, 200))
        stuck = 5 * (4096 // (line or 4096))  # the first line of row 5
        check(L.gids_store_debug_mark_busy(s.s, stuck))
        ids = np.array([5, 6, 5, 100, 1999, 5])
        for _ in range(2):  # the line stays stuck: every gather waits, gives up, bypasses
            rc, out = _gather(s, ids, cdim, cdim)
            check(rc)
            assert out.tobytes() == oracle.gather(t, ids).tobytes()
        st = s.stats()
        assert st["wait_timeouts"] >= 2 and st["bypass"] >= 2
        assert st["access"] == st["hit"] + st["miss"] + st["bypass"]
        # rows on other lines are cached as usual
        rc, out = _gather(s, np.array([6, 100]), cdim, cdim)
        check(rc)
        assert out.tobytes() == oracle.gather(t, np.array([6, 100])).tobytes()
        # flush_cache clears the stuck state
        check(L.gids_flush_cache(s.s))
        s.reset_stats()
        rc, out = _gather(s, np.array([5, 5]), cdim, cdim)
        check(rc)
        assert s.stats()["wait_timeouts"] == 0
        assert L.gids_store_debug_mark_busy(s.s, 10**12) == gids_abi.GIDS_E_RANGE
    finally:
        s.close()


def test_bad_pin_lists_are_rejected():
    rows, cdim = 1000, 256
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 52, rows, cdim)
    s = Store(4, 4096, t.size, 8, num_ssd=1)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    L = gids_abi.lib()
    try:
        check(L.gids_cpu_backing_buffer(s.s, cdim, 10))
        neg = np.array([3, -1, 4], dtype=np.int64)
        assert L.gids_set_cpu_buffer_host(s.s, neg.ctypes.data, 3) == gids_abi.GIDS_E_RANGE
        big = np.array([3, rows + 5], dtype=np.int64)
        check(L.gids_store_set_row_layout(s.s, cdim))
        assert L.gids_set_cpu_buffer_host(s.s, big.ctypes.data, 2) == gids_abi.GIDS_E_RANGE
        too_many = np.arange(11, dtype=np.int64)
        assert L.gids_set_cpu_buffer_host(s.s, too_many.ctypes.data, 11) == gids_abi.GIDS_E_INVAL
        # a valid list afterwards works and the gathers are exact
        ok = np.array([7, 3, 900], dtype=np.int64)
        check(L.gids_set_cpu_buffer_host(s.s, ok.ctypes.data, 3))
        ids = np.array([3, 4, 900, 7, 7])
        rc, out = _gather(s, ids, cdim, cdim)
        check(rc)
        assert out.tobytes() == oracle.gather(t, ids).tobytes()
        cnt = ctypes.c_uint32()
        check(L.gids_get_cpu_access_count(s.s, ctypes.byref(cnt)))
        assert cnt.value == 4
    finally:
        s.close()


def test_calls_out_of_order():
    L = gids_abi.lib()
    st = ctypes.c_void_p()
    check(L.gids_store_create(ctypes.byref(st), 4, 0))
    d = torch.arange(2, dtype=torch.int64, device="cuda")
    out = torch.empty((2, 8), device="cuda")
    assert L.gids_read_feature(st, out.data_ptr(), d.data_ptr(), 2, 8, 8, 0, None) == gids_abi.GIDS_E_STATE
    assert L.gids_cpu_backing_buffer(st, 8, 2) == gids_abi.GIDS_E_STATE
    assert L.gids_flush_cache(st) == gids_abi.GIDS_E_STATE
    check(L.gids_store_destroy(st))
    assert L.gids_store_create(ctypes.byref(st), 3, 0) == gids_abi.GIDS_E_INVAL  # element size
    assert L.gids_store_create(ctypes.byref(st), 4, 99) == gids_abi.GIDS_E_INVAL  # no such device
