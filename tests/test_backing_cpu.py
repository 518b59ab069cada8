"""Emulated SSDs on the host, no GPU: the striped layout on the device files
equals the oracle's stripe image (page_cache_backup.h:626-652, STRIPE), reads
and writes go through the stripe map, capacity limits wrap, and the synthetic
fill equals the oracle's generator."""
import ctypes

import numpy as np
import pytest

import gids_abi
from gids_abi import check
from oracle import oracle


def controllers(n, pattern=None, capacity=0, ssd_list=None):
    L = gids_abi.lib()
    c = ctypes.c_void_p()
    check(L.gids_ctrls_create(ctypes.byref(c)))
    lst = (ctypes.c_int32 * n)(*(ssd_list or list(range(n))))
    check(L.gids_ctrls_init(c, n, 1024, 128, lst))
    if pattern or capacity:
        check(L.gids_ctrls_set_emulation(c, capacity, (pattern or "").encode()))
    return c


def geometry(c):
    g = (ctypes.c_uint64 * 4)()
    check(gids_abi.lib().gids_ctrls_geometry(c, g, 4))
    return list(g)


@pytest.mark.parametrize("n,page,off", [(1, 4096, 0), (3, 512, 2), (4, 4096, 5), (2, 1024, 0)])
def test_device_files_match_stripe_image(built, tmp_path, n, page, off):
    L = gids_abi.lib()
    pattern = str(tmp_path / "ssd{}.img")
    ssd_list = [7, 3, 9, 1][:n]
    c = controllers(n, pattern=pattern, ssd_list=ssd_list)
    try:
        logical = np.random.default_rng(n).integers(0, 256, size=37 * page + 100, dtype=np.uint8)
        check(L.gids_ctrls_bind(c, n, page, off, logical.nbytes))
        rp, wrap, ssd_bytes, nb = geometry(c)
        assert rp == -(-logical.nbytes // page) and wrap == rp and nb == n
        check(L.gids_ctrls_write(c, logical.ctypes.data, logical.nbytes, 0))
        back = np.zeros_like(logical)
        check(L.gids_ctrls_read(c, back.ctypes.data, back.nbytes, 0))
        assert np.array_equal(back, logical)
    finally:
        check(L.gids_ctrls_destroy(c))
    exp = oracle.stripe_image(logical, page, n, off, ssd_bytes)
    for i, k in enumerate(ssd_list):
        data = np.fromfile(pattern.replace("{}", str(k)), dtype=np.uint8)
        assert data.nbytes == ssd_bytes
        assert np.array_equal(data, exp[i]), f"SSD {k} (stripe {i}) differs"


def test_files_persist_across_controllers(built, tmp_path):
    L = gids_abi.lib()
    pattern = str(tmp_path / "dev{}")
    page = 512
    data = np.arange(page * 10 // 4, dtype=np.uint32).view(np.uint8)
    c = controllers(2, pattern=pattern)
    check(L.gids_ctrls_bind(c, 2, page, 1, data.nbytes))
    check(L.gids_ctrls_write(c, data.ctypes.data, data.nbytes, 0))
    check(L.gids_ctrls_destroy(c))
    c = controllers(2, pattern=pattern)
    check(L.gids_ctrls_bind(c, 2, page, 1, data.nbytes))
    back = np.zeros_like(data)
    check(L.gids_ctrls_read(c, back.ctypes.data, back.nbytes, 0))
    check(L.gids_ctrls_destroy(c))
    assert np.array_equal(back, data)


def test_unaligned_io_and_bounds(built):
    L = gids_abi.lib()
    c = controllers(3)
    page = 512
    try:
        check(L.gids_ctrls_bind(c, 3, page, 0, 20 * page))
        buf = np.random.default_rng(1).integers(0, 256, size=3 * page + 77, dtype=np.uint8)
        check(L.gids_ctrls_write(c, buf.ctypes.data, buf.nbytes, 333))
        back = np.zeros_like(buf)
        check(L.gids_ctrls_read(c, back.ctypes.data, back.nbytes, 333))
        assert np.array_equal(back, buf)
        assert L.gids_ctrls_write(c, buf.ctypes.data, 10, 20 * page - 5) == gids_abi.GIDS_E_RANGE
        # rebinding with another geometry is refused; the same geometry is reused
        assert L.gids_ctrls_bind(c, 3, 1024, 0, 20 * page) == gids_abi.GIDS_E_STATE
        check(L.gids_ctrls_bind(c, 3, page, 0, 20 * page))
    finally:
        check(L.gids_ctrls_destroy(c))


def test_capacity_wraps(built):
    L = gids_abi.lib()
    page, n, off = 512, 4, 2
    c = controllers(n, capacity=(off + 5) * page)  # 5 data pages per SSD -> 20 pages held
    try:
        check(L.gids_ctrls_bind(c, n, page, off, 100 * page))
        rp, wrap, ssd_bytes, _ = geometry(c)
        assert (rp, wrap, ssd_bytes) == (100, 20, (off + 5) * page)
        a = np.full(page, 7, dtype=np.uint8)
        check(L.gids_ctrls_write(c, a.ctypes.data, page, 3 * page))
        b = np.zeros(page, dtype=np.uint8)
        check(L.gids_ctrls_read(c, b.ctypes.data, page, (3 + 20 * 4) * page))  # page 83 = page 3 mod 20
        assert np.array_equal(a, b)
    finally:
        check(L.gids_ctrls_destroy(c))


@pytest.mark.parametrize("kind", [oracle.KIND_F32_UNIFORM, oracle.KIND_F16_BYTESUM, oracle.KIND_I64_RAW,
                                  oracle.KIND_F16_NORMAL])
def test_synthetic_fill_matches_oracle(built, kind):
    L = gids_abi.lib()
    page, n = 4096, 3
    eb = {1: 4, 2: 2, 3: 8, 4: 2}[kind]
    rows, cdim = 300, 512
    nbytes = rows * cdim * eb
    c = controllers(n, capacity=(1 + 20) * page)  # wraps after 60 pages
    try:
        check(L.gids_ctrls_bind(c, n, page, 1, nbytes))
        wrap = geometry(c)[1]
        check(L.gids_ctrls_fill_synthetic(c, kind, 99, 4))
        back = np.zeros(nbytes, dtype=np.uint8)
        check(L.gids_ctrls_read(c, back.ctypes.data, nbytes, 0))
    finally:
        check(L.gids_ctrls_destroy(c))
    got = back.view(oracle.KIND_DTYPE[kind]).reshape(rows, cdim)
    exp = oracle.gather_synth(kind, 99, rows, cdim, cdim, np.arange(rows), wrap_elems=wrap * page // eb)
    assert got.tobytes() == exp.tobytes()


def test_unopenable_emulated_ssd_is_an_io_error(built, tmp_path):
    L = gids_abi.lib()
    c = controllers(2, pattern=str(tmp_path / "no_such_dir" / "ssd{}"))
    try:
        assert L.gids_ctrls_bind(c, 2, 4096, 0, 1 << 20) == gids_abi.GIDS_E_IO
        buf = ctypes.create_string_buffer(512)
        L.gids_last_error(buf, 512)
        assert b"cannot open emulated SSD" in buf.value
        # unbound controllers refuse I/O
        x = np.zeros(16, dtype=np.uint8)
        assert L.gids_ctrls_write(c, x.ctypes.data, 16, 0) == gids_abi.GIDS_E_STATE
    finally:
        check(L.gids_ctrls_destroy(c))
