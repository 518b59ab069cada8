"""gids_read_feature_noalloc: the gather for callers that cannot allocate GPU
memory (their device memory belongs to another allocator with a hard budget,
so a cudaMalloc would fail or take memory promised elsewhere). Its page cache
lives in the library's static device array instead of the store's HBM.

Checked through the C ABI against gids_read_feature on the same store and node
ids, on two calls in a row, bit for bit (the tolerance of every gather test
here), and against the oracle. This file is collected last on purpose.
"""
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


def _pair(s, ids, dim, cdim, dtype, key_off=0):
    L = gids_abi.lib()
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    ref = torch.full((len(ids), dim), -3, dtype=dtype, device="cuda")
    got = torch.full((len(ids), dim), -5, dtype=dtype, device="cuda")
    check(L.gids_read_feature(s.s, ref.data_ptr(), d.data_ptr(), len(ids), dim, cdim, key_off, None))
    check(L.gids_read_feature_noalloc(s.s, got.data_ptr(), d.data_ptr(), len(ids), dim, cdim, key_off, None))
    torch.cuda.synchronize()
    return ref.cpu().numpy(), got.cpu().numpy()


def test_noalloc_equals_read_feature_two_calls():
    rows, cdim = 20000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 41, rows, cdim)
    s = Store(4, 4096, t.size, 4, num_ssd=4)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    rng = np.random.default_rng(41)
    try:
        for call in range(2):
            ids = rng.integers(0, rows, size=9000)
            ids[:100] = ids[100:200]  # pages shared by several rows of one call
            ref, got = _pair(s, ids, cdim, cdim, torch.float32)
            assert got.tobytes() == ref.tobytes(), f"call {call}"
            assert got.tobytes() == oracle.gather(t, ids).tobytes()
    finally:
        s.close()


def test_noalloc_straddling_rows_and_cpu_buffer():
    rows, cdim = 6000, 768  # fp16, 1536-byte rows straddle 4 KB pages
    t = oracle.synth_table(oracle.KIND_F16_BYTESUM, 42, rows, cdim)
    s = Store(2, 4096, t.size, 2, num_ssd=3)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    L = gids_abi.lib()
    check(L.gids_cpu_backing_buffer(s.s, cdim, 300))
    pins = np.random.default_rng(1).permutation(rows)[:300].astype(np.int64)
    check(L.gids_set_cpu_buffer_host(s.s, pins.ctypes.data, len(pins)))
    rng = np.random.default_rng(42)
    try:
        for call in range(2):
            ids = rng.integers(0, rows - 7, size=4000)
            ref, got = _pair(s, ids, 700, cdim, torch.float16, key_off=7)
            assert got.tobytes() == ref.tobytes(), f"call {call}"
            assert got.tobytes() == oracle.gather(t, ids, dim=700, key_off=7).tobytes()
    finally:
        s.close()


def test_noalloc_with_small_cache_lines():
    rows, cdim = 30000, 128  # 512-byte rows in 512-byte lines of 4 KB pages
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 43, rows, cdim)
    s = Store(4, 4096, t.size, 1, num_ssd=2, cache_line=512)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    rng = np.random.default_rng(43)
    try:
        for call in range(2):
            ids = rng.integers(0, rows, size=7000)
            ref, got = _pair(s, ids, cdim, cdim, torch.float32)
            assert got.tobytes() == ref.tobytes(), f"call {call}"
            assert got.tobytes() == oracle.gather(t, ids).tobytes()
    finally:
        s.close()


def test_noalloc_rejects_a_page_table_beyond_the_scratch():
    page, cdim = 4096, 1024
    pages = 8 << 20  # 8M pages: a 64 MiB page table, the scratch holds 32 MiB
    s = Store(4, page, pages * cdim, 1, num_ssd=2, capacity=(4 << 20))  # small emulated SSDs, wrapped
    L = gids_abi.lib()
    try:
        d = torch.arange(4, dtype=torch.int64, device="cuda")
        out = torch.empty((4, cdim), device="cuda")
        rc = L.gids_read_feature_noalloc(s.s, out.data_ptr(), d.data_ptr(), 4, cdim, cdim, 0, None)
        assert rc == gids_abi.GIDS_E_RANGE
        buf = ctypes.create_string_buffer(512)
        L.gids_last_error(buf, 512)
        assert b"no-allocation scratch" in buf.value
        check(L.gids_read_feature(s.s, out.data_ptr(), d.data_ptr(), 4, cdim, cdim, 0, None))  # store unaffected
    finally:
        s.close()


def test_noalloc_leaves_free_memory_unchanged_and_counts_rows():
    rows, cdim = 12000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 44, rows, cdim)
    s = Store(4, 4096, t.size, 4, num_ssd=2)
    s.write_range(t.ctypes.data, t.nbytes, 0)
    L = gids_abi.lib()
    ids = np.random.default_rng(44).integers(0, rows, size=5000)
    d = torch.as_tensor(ids, dtype=torch.int64).cuda()
    out = torch.empty((len(ids), cdim), device="cuda")
    try:
        # the first call on the device loads the static array (CUDA loads it lazily)
        check(L.gids_read_feature_noalloc(s.s, out.data_ptr(), d.data_ptr(), len(ids), cdim, cdim, 0, None))
        torch.cuda.synchronize()
        s.reset_stats()
        free0 = torch.cuda.mem_get_info()[0]
        check(L.gids_read_feature_noalloc(s.s, out.data_ptr(), d.data_ptr(), len(ids), cdim, cdim, 0, None))
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        assert free1 == free0, f"free device memory moved by {free0 - free1} bytes"
        assert out.cpu().numpy().tobytes() == oracle.gather(t, ids).tobytes()
        st = s.stats()  # the call's counters are added to the store's
        assert st["rows"] == len(ids) and st["access"] == len(ids)
        assert st["hit"] + st["miss"] + st["bypass"] == st["access"] and st["read_io"] > 0
    finally:
        s.close()
