"""The C ABI library loads and exports every declared symbol; the Python
modules expose the reference's names. CPU only (no compute calls)."""
import ctypes
import inspect
import os
import subprocess
import sys

import pytest

import gids_abi

# pybind methods of BAM_Feature_Store_float/_long in the reference (gids_nvme.cu:830-891)
REFERENCE_STORE_METHODS = [
    "init_controllers", "read_feature", "read_feature_hetero", "read_feature_merged_hetero", "read_feature_merged",
    "set_window_buffering", "cpu_backing_buffer", "set_cpu_buffer", "flush_cache", "store_tensor", "read_tensor",
    "get_array_ptr", "get_offset_array", "set_offsets", "get_cpu_access_count", "flush_cpu_access_count",
    "print_stats",
]
# GIDS class methods (GIDS.py:636-1128)
REFERENCE_GIDS_METHODS = [
    "init_graph_GIDS", "get_offset_array", "get_array_ptr", "cpu_backing_buffer", "set_cpu_buffer",
    "window_buffering", "fill_wb", "set_required_storage_access", "fetch_feature", "print_stats", "store_tensor",
    "store_mmap_tensor", "read_tensor", "flush_cache",
]


def test_library_exports_header(built):
    declared = gids_abi.header_symbols()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", gids_abi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if l.strip())
    # exactly the declared entry points; the statically linked CUDA runtime stays hidden
    assert exported == declared
    L = gids_abi.lib()
    for name in declared:
        assert hasattr(L, name)


def test_strings_and_errors_without_compute(built):
    L = gids_abi.lib()
    assert b"sm_100a" in L.gids_version()
    assert L.gids_strerror(gids_abi.GIDS_E_RANGE) == b"node id out of range"
    # null arguments are rejected with a message, never a crash
    rc = L.gids_ctrls_create(None)
    assert rc == gids_abi.GIDS_E_INVAL
    buf = ctypes.create_string_buffer(256)
    assert L.gids_last_error(buf, 256) > 0 and b"null" in buf.value
    rc = L.gids_read_feature(None, None, None, 0, 1, 1, 0, None)
    assert rc == gids_abi.GIDS_E_INVAL


def test_controllers_validate_arguments(built):
    L = gids_abi.lib()
    c = ctypes.c_void_p()
    gids_abi.check(L.gids_ctrls_create(ctypes.byref(c)))
    try:
        lst = (ctypes.c_int32 * 33)(*range(33))
        assert L.gids_ctrls_init(c, 33, 1024, 128, lst) == gids_abi.GIDS_E_INVAL
        assert L.gids_ctrls_init(c, 0, 1024, 128, lst) == gids_abi.GIDS_E_INVAL
        assert L.gids_ctrls_init(c, 4, 1024, 128, lst) == gids_abi.GIDS_OK
        assert L.gids_ctrls_set_emulation(c, 1 << 30, b"") == gids_abi.GIDS_OK
    finally:
        gids_abi.check(L.gids_ctrls_destroy(c))


def test_pybind_module_surface(built):
    import BAM_Feature_Store as B

    for cls in (B.BAM_Feature_Store_float, B.BAM_Feature_Store_long, B.BAM_Feature_Store_half,
                B.BAM_Feature_Store_bfloat16):
        for m in REFERENCE_STORE_METHODS:
            assert hasattr(cls, m), (cls, m)
    assert hasattr(B.GIDS_Controllers, "init_GIDS_controllers")
    c = B.GIDS_Controllers()
    c.init_GIDS_controllers(4, 1024, 128, [3, 1, 2, 0])
    assert c.n_ctrls == 4
    s = B.BAM_Feature_Store_float()
    with pytest.raises(RuntimeError):
        s.read_feature(0, 0, 0, 1, 1, 0)  # before init_controllers
    # every method that releases the GIL raises its error as a Python exception
    # (a method that released it twice would abort the interpreter instead)
    for call in (lambda: s.prefetch(0, 0, 1, 1, 0, 0), lambda: s.set_window_buffering(0, 0, 0, 0),
                 lambda: s.unset_window_buffering(0, 0, 0, 0), lambda: s.pin_rows(0, 0, 0, 0),
                 lambda: s.read_feature_hetero(0, [], [], [], 1, 1, [], 0)):
        with pytest.raises(RuntimeError):
            call()


def test_gids_surface(built):
    import GIDS

    sig = inspect.signature(GIDS.GIDS.__init__)
    defaults = {k: v.default for k, v in sig.parameters.items() if k != "self"}
    # GIDS.py:510-517
    expect = dict(page_size=4096, off=0, cache_dim=1024, num_ele=300 * 1000 * 1000 * 1024, num_ssd=1, ssd_list=None,
                  cache_size=10, ctrl_idx=0, window_buffer=False, wb_size=8, accumulator_flag=False, long_type=False,
                  heterograph=False, heterograph_map=None)
    for k, v in expect.items():
        assert defaults[k] == v, k
    for m in REFERENCE_GIDS_METHODS:
        assert hasattr(GIDS.GIDS, m), m
    params = list(inspect.signature(GIDS.GIDS_DGLDataLoader).parameters)
    assert params[:6] == ["graph", "indices", "graph_sampler", "batch_size", "dim", "GIDS"]


def test_package_import_maps_no_library():
    """Importing GIDS, its synthetic graphs and the bench loads none of the
    compiled libraries (the bench's reference arm must run the reference's CPU
    gather with nothing of this library mapped); constructing a GIDS does."""
    code = ("import sys; sys.path[:0] = [%r, %r]; import GIDS, GIDS.synthetic, bench; "
            "maps = open('/proc/self/maps').read(); "
            "print('libgids_b200' in maps, 'BAM_Feature_Store' in maps)") % (
        os.path.dirname(os.path.dirname(gids_abi.LIB_PATH)), os.path.dirname(os.path.dirname(os.path.dirname(
            gids_abi.LIB_PATH))))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["False", "False"]
