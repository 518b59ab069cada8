"""GPU parity of the gather through the C ABI: bit-exact against the oracle
(the reference's mmap index_select restated) on seeded inputs, over every
path of the page cache (hit, fill, eviction, bypass, wait), the constant CPU
buffer, window buffering, heterograph key offsets, multi-tuple launches,
rows straddling pages, element types, bad ids and empty inputs."""
import ctypes
import os

import numpy as np
import pytest
import torch

import gids_abi
from gids_abi import Store, check
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "gather_golden.npz")
NP2T = {np.dtype(np.float32): torch.float32, np.dtype(np.float16): torch.float16, np.dtype(np.int64): torch.int64}


def bits_equal(a: torch.Tensor, b: np.ndarray) -> bool:
    a = a.detach().cpu().contiguous().numpy()
    return a.shape == b.shape and a.view(np.uint8).tobytes() == np.ascontiguousarray(b).view(np.uint8).tobytes()


def make_store(table: np.ndarray, page_size=4096, cache_mb=64, num_ssd=2, read_off=0, **kw) -> Store:
    """Store holding `table` row-major at offset 0 (kw: capacity, pattern, cache_line, ...)."""
    s = Store(table.dtype.itemsize, page_size, table.size, cache_mb, num_ssd=num_ssd, read_off_pages=read_off, **kw)
    s.write_range(table.ctypes.data, table.nbytes, 0)
    return s


def gather(s: Store, ids: np.ndarray, dim: int, cache_dim: int, dtype, key_off=0, out=None):
    d_ids = torch.as_tensor(ids, dtype=torch.int64).cuda()
    if out is None:
        out = torch.full((len(ids), dim), -7, dtype=dtype, device="cuda")
    rc = s.read_feature(out.data_ptr(), d_ids.data_ptr(), len(ids), dim, cache_dim, key_off)
    torch.cuda.synchronize()
    return rc, out


@pytest.fixture(scope="module", autouse=True)
def _built(built):
    torch.cuda.init()
    yield


@pytest.fixture(scope="module")
def golden():
    z = np.load(GOLDEN)
    cases = {}
    for key in z.files:
        if "/" in key:
            name, field = key.split("/", 1)
            cases.setdefault(name, {})[field] = z[key]
    return cases


def table_of(c):
    if int(c["kind"]) == 0:
        return c["table"]
    return oracle.synth_table(int(c["kind"]), int(c["seed"]), int(c["rows"]), int(c["cache_dim"]))


@pytest.mark.parametrize("name", ["homo_f32_d1024", "homo_f16_d768", "homo_f32_d128", "subset_d200_of_1024",
                                  "long_d512", "special_f32", "empty"])
def test_golden_cases(golden, name):
    c = golden[name]
    t = table_of(c)
    s = make_store(t)
    for _ in range(2):  # cold (fills) then warm (hits)
        rc, out = gather(s, c["ids"], int(c["dim"]), int(c["cache_dim"]), NP2T[t.dtype], int(c["key_off"]))
        check(rc)
        assert bits_equal(out, c["out"])
    s.close()


def test_golden_hetero_one_launch(golden):
    names = ["hetero_t0", "hetero_t1", "hetero_t2", "hetero_t3"]
    t = table_of(golden[names[0]])
    s = make_store(t, num_ssd=4)
    ids = [torch.as_tensor(golden[n]["ids"]).cuda() for n in names]
    outs = [torch.empty((len(i), 256), dtype=torch.float32, device="cuda") for i in ids]
    check(s.read_multi([o.data_ptr() for o in outs], [i.data_ptr() for i in ids], [len(i) for i in ids], 256, 256,
                       [int(golden[n]["key_off"]) for n in names]))
    torch.cuda.synchronize()
    for n, o in zip(names, outs):
        assert bits_equal(o, golden[n]["out"])
    assert s.stats()["launches"] == 1
    s.close()


GEOMETRIES = [
    # page, ssds, read_off, cache_mb, rows, cache_dim, dim, dtype
    (4096, 1, 0, 8, 3000, 1024, 1024, np.float32),
    (4096, 4, 5, 8, 3000, 1024, 1000, np.float32),
    (512, 3, 2, 1, 5000, 128, 128, np.float32),
    (8192, 2, 0, 16, 2000, 1024, 512, np.float32),
    (4096, 3, 1, 4, 6000, 768, 768, np.float16),   # 1536-byte rows straddle pages
    (4096, 2, 0, 4, 4000, 300, 300, np.float32),   # 1200-byte rows, 16-byte aligned stride
    (4096, 2, 0, 4, 4000, 33, 31, np.float32),     # 132-byte stride: 4-byte vectors
    (1024, 5, 3, 2, 3000, 6000, 5000, np.float16), # rows span many pages
    (4096, 2, 0, 8, 2000, 512, 512, np.int64),
]


@pytest.mark.parametrize("page,ssds,off,cache_mb,rows,cdim,dim,dt", GEOMETRIES)
def test_geometries(page, ssds, off, cache_mb, rows, cdim, dim, dt):
    kind = {np.float32: oracle.KIND_F32_UNIFORM, np.float16: oracle.KIND_F16_BYTESUM, np.int64: oracle.KIND_I64_RAW}[dt]
    t = oracle.synth_table(kind, 11, rows, cdim)
    s = make_store(t, page_size=page, cache_mb=cache_mb, num_ssd=ssds, read_off=off)
    rng = np.random.default_rng(rows + cdim)
    for rep in range(3):
        ids = rng.integers(0, rows, size=2500)
        rc, out = gather(s, ids, dim, cdim, NP2T[np.dtype(dt)])
        check(rc)
        assert bits_equal(out, oracle.gather(t, ids, dim=dim))
    st = s.stats()
    assert st["access"] == st["hit"] + st["miss"] + st["bypass"]
    assert st["rows"] == 3 * 2500 and st["bad_ids"] == 0 and st["wait_timeouts"] == 0
    s.close()


LINE_GEOMETRIES = [
    # page, cache line, ssds, cache_mb, rows, cache_dim, dim, dtype
    (4096, 512, 4, 2, 20000, 128, 128, np.float32),    # config-5 rows: one 512 B line each
    (4096, 512, 4, 2, 6000, 768, 768, np.float16),     # config-4 rows: three lines each
    (4096, 1024, 3, 2, 6000, 768, 700, np.float16),    # rows straddle 1 KB lines
    (8192, 2048, 2, 4, 4000, 1024, 1024, np.float32),  # 4 KB rows over 2 KB lines
    (4096, 512, 2, 1, 5000, 33, 31, np.float32),       # 4-byte vectors
]


@pytest.mark.parametrize("page,line,ssds,cache_mb,rows,cdim,dim,dt", LINE_GEOMETRIES)
def test_cache_lines_smaller_than_pages(page, line, ssds, cache_mb, rows, cdim, dim, dt):
    kind = {np.float32: oracle.KIND_F32_UNIFORM, np.float16: oracle.KIND_F16_BYTESUM}[dt]
    t = oracle.synth_table(kind, 17, rows, cdim)
    s = make_store(t, page_size=page, cache_mb=cache_mb, num_ssd=ssds, cache_line=line)
    g = s.geometry()
    assert g["cache_line"] == line and g["cache_slots"] == cache_mb * (1 << 20) // line
    rng = np.random.default_rng(line + rows)
    for _ in range(3):
        ids = rng.integers(0, rows, size=4000)
        rc, out = gather(s, ids, dim, cdim, NP2T[np.dtype(dt)])
        check(rc)
        assert bits_equal(out, oracle.gather(t, ids, dim=dim))
    st = s.stats()
    assert st["access"] == st["hit"] + st["miss"] + st["bypass"] and st["wait_timeouts"] == 0
    # a missed row moves only its lines: fills x line bytes stays within (rows' lines) x line bytes
    assert st["read_io"] * line <= st["access"] * line
    s.close()


def test_cache_line_arguments():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 100, 256)
    L = gids_abi.lib()
    for bad in (256, 3000, 8192):  # below 512, not a power of two, above the page
        c = ctypes.c_void_p()
        check(L.gids_ctrls_create(ctypes.byref(c)))
        lst = (ctypes.c_int32 * 1)(0)
        check(L.gids_ctrls_init(c, 1, 1024, 128, lst))
        st = ctypes.c_void_p()
        check(L.gids_store_create(ctypes.byref(st), 4, 0))
        rc = L.gids_store_set_cache_line(st, bad)
        if rc == gids_abi.GIDS_OK:
            rc = L.gids_store_init_controllers(st, c, 4096, 0, 1, t.size, 1)
        assert rc == gids_abi.GIDS_E_INVAL, bad
        check(L.gids_store_destroy(st))
        check(L.gids_ctrls_destroy(c))


def test_small_cache_evicts_and_stays_exact():
    rows, cdim = 20000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 3, rows, cdim)
    s = make_store(t, cache_mb=1, num_ssd=4)  # 256 slots of 4 KB for 80 MB of rows
    assert s.geometry()["cache_slots"] == 256
    rng = np.random.default_rng(0)
    for _ in range(4):
        ids = rng.integers(0, rows, size=9000)
        rc, out = gather(s, ids, cdim, cdim, torch.float32)
        check(rc)
        assert bits_equal(out, oracle.gather(t, ids))
    st = s.stats()
    assert st["evictions"] > 0 and st["read_io"] > 0
    assert st["access"] == st["hit"] + st["miss"] + st["bypass"]
    s.close()


def test_hot_rows_hit_after_warmup():
    rows, cdim = 4000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 5, rows, cdim)
    s = make_store(t, cache_mb=64)  # everything fits
    s.set_policy(False, 1)  # insert on the first miss, as the reference does
    ids = np.arange(rows)
    check(gather(s, ids, cdim, cdim, torch.float32)[0])
    s.reset_stats()
    rc, out = gather(s, ids[::-1].copy(), cdim, cdim, torch.float32)
    check(rc)
    st = s.stats()
    assert st["hit"] == rows and st["miss"] == 0 and st["bypass"] == 0
    assert st["bytes_hit"] == rows * cdim * 4
    assert bits_equal(out, t[::-1])
    s.close()


def test_no_cache_bypasses():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 8, 3000, 256)
    s = make_store(t, cache_mb=0)
    ids = np.random.default_rng(1).integers(0, 3000, size=4000)
    rc, out = gather(s, ids, 256, 256, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(t, ids))
    st = s.stats()
    assert st["bypass"] == st["access"] > 0 and st["hit"] == 0
    s.close()


def test_contended_duplicate_pages():
    rows, cdim = 5000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 2, rows, cdim)
    s = make_store(t, cache_mb=1)
    rng = np.random.default_rng(3)
    hot = rng.integers(0, rows, size=64)
    ids = rng.choice(hot, size=200000)
    rc, out = gather(s, ids, cdim, cdim, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(t, ids))
    st = s.stats()
    assert st["access"] == st["hit"] + st["miss"] + st["bypass"]
    s.close()


def test_cpu_buffer_seq_then_pinned():
    rows, cdim = 6000, 512
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 4, rows, cdim)
    s = make_store(t, cache_mb=2)
    L = gids_abi.lib()
    check(L.gids_cpu_backing_buffer(s.s, cdim, 700))
    rng = np.random.default_rng(4)
    ids = rng.integers(0, rows, size=5000)
    # seq mode: rows [0, 700) are in the buffer (gids_kernel.cu:132-141)
    rc, out = gather(s, ids, cdim, cdim, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(t, ids))
    cnt = ctypes.c_uint32()
    check(L.gids_get_cpu_access_count(s.s, ctypes.byref(cnt)))
    assert cnt.value == int((ids < 700).sum())
    check(L.gids_flush_cpu_access_count(s.s))
    s.reset_stats()
    # pinned list from a device array (set_cpu_buffer), with duplicates and unsorted
    pins = rng.permutation(rows)[:650]
    pins = np.concatenate([pins, pins[:10]])
    d_pins = torch.as_tensor(pins).cuda()
    check(L.gids_set_cpu_buffer(s.s, ctypes.c_void_p(d_pins.data_ptr()), len(pins)))
    for dim in (cdim, 100):
        rc, out = gather(s, ids, dim, cdim, torch.float32)
        check(rc)
        assert bits_equal(out, oracle.gather(t, ids, dim=dim))
    check(L.gids_get_cpu_access_count(s.s, ctypes.byref(cnt)))
    assert cnt.value == 2 * int(np.isin(ids, pins).sum())
    assert s.stats()["bytes_cpu"] == int(np.isin(ids, pins).sum()) * (cdim + 100) * 4
    s.close()


def test_cpu_buffer_rejects_wider_rows():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 4, 100, 64)
    s = make_store(t)
    check(gids_abi.lib().gids_cpu_backing_buffer(s.s, 32, 10))
    rc, _ = gather(s, np.arange(5), 64, 64, torch.float32)
    assert rc == gids_abi.GIDS_E_INVAL
    s.close()


def test_window_buffering_marks_and_releases():
    rows, cdim = 8000, 1024
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 6, rows, cdim)
    s = make_store(t, cache_mb=2)  # 512 slots
    L = gids_abi.lib()
    rng = np.random.default_rng(6)
    batches = [rng.integers(0, rows, size=300) for _ in range(6)]
    d = [torch.as_tensor(b).cuda() for b in batches]
    for b in d[:3]:  # mark a window of three upcoming batches
        check(L.gids_set_window_buffering(s.s, ctypes.c_void_p(b.data_ptr()), len(b), 0, 0, None))
    for i, b in enumerate(batches):
        if i + 3 < len(d):
            check(L.gids_set_window_buffering(s.s, ctypes.c_void_p(d[i + 3].data_ptr()), len(d[i + 3]), 0, 0, None))
        rc, out = gather(s, b, cdim, cdim, torch.float32)
        check(rc)
        assert bits_equal(out, oracle.gather(t, b))
    # all marks consumed: a flood of fresh rows can evict everything
    s.reset_stats()
    flood = rng.integers(0, rows, size=6000)
    rc, out = gather(s, flood, cdim, cdim, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(t, flood))
    assert s.stats()["evictions"] > 0
    s.close()


def test_more_tuples_than_one_launch_holds():
    rows, cdim = 3000, 128
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 7, rows, cdim)
    s = make_store(t, cache_mb=4, num_ssd=3)
    rng = np.random.default_rng(7)
    k = 70
    ids = [rng.integers(0, rows - 50, size=int(rng.integers(0, 200))) for _ in range(k)]
    offs = [int(rng.integers(0, 50)) for _ in range(k)]
    d_ids = [torch.as_tensor(i, dtype=torch.int64).cuda() for i in ids]
    outs = [torch.empty((len(i), cdim), device="cuda") for i in ids]
    check(s.read_multi([o.data_ptr() for o in outs], [i.data_ptr() for i in d_ids], [len(i) for i in ids], cdim,
                       cdim, offs))
    torch.cuda.synchronize()
    for i, o, off in zip(ids, outs, offs):
        assert bits_equal(o, oracle.gather(t, i, key_off=off))
    s.close()


def test_bad_ids_give_error_and_zero_rows():
    rows, cdim = 1000, 256
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, rows, cdim)
    s = make_store(t)
    ids = np.array([3, -1, rows - 1, rows, 2**40, 7], dtype=np.int64)
    rc, out = gather(s, ids, cdim, cdim, torch.float32)
    assert rc == gids_abi.GIDS_E_RANGE
    good = np.array([0, 2, 5])
    assert bits_equal(out[good], oracle.gather(t, ids[good]))
    assert torch.count_nonzero(out[[1, 3, 4]]) == 0
    assert s.stats()["bad_ids"] == 3
    # key_off pushing a valid id out of range is caught too
    rc, _ = gather(s, np.array([rows - 2]), cdim, cdim, torch.float32, key_off=5)
    assert rc == gids_abi.GIDS_E_RANGE
    # the error does not stick
    rc, out = gather(s, np.array([1, 2]), cdim, cdim, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(t, np.array([1, 2])))
    s.close()


def test_empty_and_misaligned_output():
    rows, cdim = 500, 64
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 9, rows, cdim)
    s = make_store(t)
    check(gather(s, np.zeros(0, dtype=np.int64), cdim, cdim, torch.float32)[0])
    ids = np.random.default_rng(9).integers(0, rows, size=300)
    base = torch.zeros(len(ids) * cdim + 1, device="cuda")
    out = base[1:].view(len(ids), cdim)  # 4-byte aligned, not 16
    rc, out = gather(s, ids, cdim, cdim, torch.float32, out=out)
    check(rc)
    assert bits_equal(out, oracle.gather(t, ids))
    s.close()


def test_argument_errors():
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 9, 100, 64)
    s = make_store(t)
    rc, _ = gather(s, np.arange(3), 65, 64, torch.float32)  # dim > cache_dim
    assert rc == gids_abi.GIDS_E_INVAL
    rc, _ = gather(s, np.arange(3), 0, 64, torch.float32)
    assert rc == gids_abi.GIDS_E_INVAL
    s.close()


def test_synthetic_fill_with_wrap():
    page, cdim, rows, n_ssd = 4096, 1024, 40000, 4
    num_ele = rows * cdim
    cap = (2 + 1000) * page  # 1000 data pages per SSD -> wrap after 4000 pages
    s = Store(4, page, num_ele, 8, num_ssd=n_ssd, read_off_pages=2, capacity=cap)
    g = s.geometry()
    assert g["wrap_pages"] == 4000 and g["range_pages"] == rows
    check(gids_abi.lib().gids_fill_synthetic(s.s, oracle.KIND_F32_UNIFORM, 42, 0))
    ids = np.random.default_rng(10).integers(0, rows, size=5000)
    rc, out = gather(s, ids, cdim, cdim, torch.float32)
    check(rc)
    exp = oracle.gather_synth(oracle.KIND_F32_UNIFORM, 42, rows, cdim, cdim, ids, wrap_elems=4000 * page // 4)
    assert bits_equal(out, exp)
    s.close()


def test_async_on_torch_stream():
    rows, cdim = 5000, 512
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 12, rows, cdim)
    s = make_store(t, cache_mb=4)
    check(gids_abi.lib().gids_store_set_synchronous(s.s, 0))
    st = torch.cuda.Stream()
    ids = np.random.default_rng(12).integers(0, rows, size=20000)
    with torch.cuda.stream(st):
        d_ids = torch.as_tensor(ids).cuda(non_blocking=True)
        out = torch.empty((len(ids), cdim), device="cuda")
        check(s.read_feature(out.data_ptr(), d_ids.data_ptr(), len(ids), cdim, cdim, 0, ctypes.c_void_p(st.cuda_stream)))
        out2 = out * 1.0  # stream-ordered consumer
    st.synchronize()
    assert bits_equal(out2, oracle.gather(t, ids))
    check(gids_abi.lib().gids_store_synchronize(s.s))
    s.close()


def test_store_tensor_reference_semantics():
    # gids_kernel.cu:378-389: range[r*dim + i] = src[r*dim + i + offset/sizeof(T)], dim = page_size/sizeof(T)
    page = 4096
    per = page // 4
    src = oracle.synth_table(oracle.KIND_F32_UNIFORM, 13, 40, per)
    s = Store(4, page, 64 * per, 4, num_ssd=2)
    d_src = torch.as_tensor(src).cuda()
    off_elems = 3
    check(gids_abi.lib().gids_store_tensor(s.s, ctypes.c_void_p(d_src.data_ptr()), 30, off_elems * 4))
    exp = src.reshape(-1)[off_elems:off_elems + 30 * per].reshape(30, per)
    ids = np.arange(30)
    rc, out = gather(s, ids, per, per, torch.float32)
    check(rc)
    assert bits_equal(out, exp)
    back = np.empty(30 * per, dtype=np.float32)
    check(gids_abi.lib().gids_read_range_host(s.s, back.ctypes.data, back.nbytes, 0))
    assert np.array_equal(back.view(np.uint32), exp.reshape(-1).view(np.uint32))
    s.close()


def test_rewrite_invalidates_cache():
    rows, cdim = 2000, 1024
    a = oracle.synth_table(oracle.KIND_F32_UNIFORM, 14, rows, cdim)
    b = oracle.synth_table(oracle.KIND_F32_UNIFORM, 15, rows, cdim)
    s = make_store(a, cache_mb=16)
    ids = np.random.default_rng(14).integers(0, rows, size=3000)
    check(gather(s, ids, cdim, cdim, torch.float32)[0])
    s.write_range(b.ctypes.data, b.nbytes, 0)
    rc, out = gather(s, ids, cdim, cdim, torch.float32)
    check(rc)
    assert bits_equal(out, oracle.gather(b, ids))
    s.close()


def test_host_read_probe(built):
    """The host-link probe reads random lines of the backing store and rejects
    read sizes it cannot issue."""
    t = oracle.synth_table(oracle.KIND_F32_UNIFORM, 61, 20000, 128)  # 512-byte rows
    s = make_store(t, num_ssd=2, cache_line=512)
    L = gids_abi.lib()
    v = ctypes.c_double()
    check(L.gids_store_host_read_gbs(s.s, 512, 64 << 20, ctypes.byref(v)))
    assert v.value > 0.5
    assert L.gids_store_host_read_gbs(s.s, 1024, 1 << 20, ctypes.byref(v)) == gids_abi.GIDS_E_INVAL  # > line
    assert L.gids_store_host_read_gbs(s.s, 768, 1 << 20, ctypes.byref(v)) == gids_abi.GIDS_E_INVAL
    s.close()
