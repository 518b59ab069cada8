"""ctypes binding of libgids_b200.so for the tests (the C ABI of include/gids_b200.h)."""
from __future__ import annotations

import ctypes
import os

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(REPO, "gids-study_b200", "lib", "libgids_b200.so")
HEADER = os.path.join(REPO, "include", "gids_b200.h")

GIDS_OK = 0
GIDS_E_INVAL = -1
GIDS_E_CUDA = -2
GIDS_E_STATE = -4
GIDS_E_RANGE = -5
GIDS_E_IO = -6
GIDS_E_UNSUPPORTED = -7
STAT_NAMES = ["access", "hit", "miss", "read_io", "bypass", "cpu_rows", "rows", "wait_timeouts", "bad_ids",
              "bytes_hit", "bytes_miss", "bytes_bypass", "bytes_cpu", "evictions", "launches", "bytes_peer",
              "ns_lookup", "ns_fill_wait", "ns_copy", "ns_release", "prefetched"]
N_STATS = 21

_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB_PATH)
        vp, u32, u64, i32, i64 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_int64
        P = ctypes.POINTER
        sig = {
            "gids_last_error": (i32, [ctypes.c_char_p, ctypes.c_size_t]),
            "gids_strerror": (ctypes.c_char_p, [i32]),
            "gids_version": (ctypes.c_char_p, []),
            "gids_current_device": (i32, [P(i32)]),
            "gids_ctrls_create": (i32, [P(vp)]),
            "gids_ctrls_init": (i32, [vp, u32, u64, u64, P(ctypes.c_int32)]),
            "gids_ctrls_set_emulation": (i32, [vp, u64, ctypes.c_char_p]),
            "gids_ctrls_destroy": (i32, [vp]),
            "gids_ctrls_bind": (i32, [vp, u32, u32, u64, u64]),
            "gids_ctrls_write": (i32, [vp, vp, u64, u64]),
            "gids_ctrls_read": (i32, [vp, vp, u64, u64]),
            "gids_ctrls_fill_synthetic": (i32, [vp, i32, u64, i32]),
            "gids_ctrls_geometry": (i32, [vp, P(u64), i32]),
            "gids_store_create": (i32, [P(vp), u32, i32]),
            "gids_store_init_controllers": (i32, [vp, vp, u32, u64, u64, u64, u64]),
            "gids_store_destroy": (i32, [vp]),
            "gids_store_set_synchronous": (i32, [vp, i32]),
            "gids_store_set_row_layout": (i32, [vp, u32]),
            "gids_read_feature": (i32, [vp, vp, vp, i64, i32, i32, u64, vp]),
            "gids_read_feature_multi": (i32, [vp, i32, P(vp), P(vp), P(u64), i32, i32, P(u64), vp]),
            "gids_read_feature_noalloc": (i32, [vp, vp, vp, i64, i32, i32, u64, vp]),
            "gids_prefetch": (i32, [vp, vp, i64, i32, i32, u64, vp]),
            "gids_store_set_replicas": (i32, [vp, u64]),
            "gids_store_set_replicated_lines": (i32, [vp, vp, u64]),
            "gids_set_window_buffering": (i32, [vp, vp, i64, i64, u32, vp]),
            "gids_unset_window_buffering": (i32, [vp, vp, i64, i64, u32, vp]),
            "gids_store_pin_rows": (i32, [vp, vp, i64, i64, u32, vp]),
            "gids_store_unpin_rows": (i32, [vp, vp, i64, i64, u32, vp]),
            "gids_out_degree": (i32, [i32, vp, i32, u64, u64, vp, vp]),
            "gids_cpu_backing_buffer": (i32, [vp, u64, u64]),
            "gids_set_cpu_buffer": (i32, [vp, vp, i32]),
            "gids_set_cpu_buffer_host": (i32, [vp, vp, i64]),
            "gids_get_cpu_access_count": (i32, [vp, P(u32)]),
            "gids_flush_cpu_access_count": (i32, [vp]),
            "gids_get_stats": (i32, [vp, P(u64), i32]),
            "gids_reset_stats": (i32, [vp]),
            "gids_print_stats": (i32, [vp]),
            "gids_get_kernel_time_ms": (i32, [vp, P(ctypes.c_double)]),
            "gids_store_synchronize": (i32, [vp]),
            "gids_store_tensor": (i32, [vp, vp, u64, u64]),
            "gids_write_range": (i32, [vp, vp, u64, u64]),
            "gids_flush_cache": (i32, [vp]),
            "gids_read_range_host": (i32, [vp, vp, u64, u64]),
            "gids_fill_synthetic": (i32, [vp, i32, u64, i32]),
            "gids_store_geometry": (i32, [vp, P(u64), i32]),
            "gids_store_set_sharding": (i32, [vp, i32, i32]),
            "gids_store_set_cache_line": (i32, [vp, u32]),
            "gids_store_set_wait_limit": (i32, [vp, u32]),
            "gids_store_set_cache_policy": (i32, [vp, i32, u32]),
            "gids_store_set_gather_blocks": (i32, [vp, u32]),
            "gids_store_debug_mark_busy": (i32, [vp, u64]),
            "gids_store_ipc_handle": (i32, [vp, vp, ctypes.c_size_t]),
            "gids_store_open_peers": (i32, [vp, vp, i32]),
            "gids_store_share_shards": (i32, [P(vp), i32]),
            "gids_store_peer_copy_gbs": (i32, [vp, i32, u64, P(ctypes.c_double)]),
            "gids_store_host_read_gbs": (i32, [vp, u32, u64, P(ctypes.c_double)]),
            "gids_sampler_create": (i32, [P(vp), i32, vp, vp, i32, u64, P(i32), i32, u64, u64]),
            "gids_sampler_capacity": (i32, [vp, P(u64)]),
            "gids_sampler_sample": (i32, [vp, vp, u64, vp, u64, vp, P(u64), i64, vp]),
            "gids_sampler_destroy": (i32, [vp]),
            "gids_pagerank": (i32, [i32, vp, vp, i32, u64, i32, ctypes.c_double, vp, vp, vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def header_symbols() -> list[str]:
    import re

    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^GIDS_API\s+[\w\s\*]*?\b(gids_\w+)\s*\(", txt, flags=re.M)))


class GidsError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{code}: {msg}")
        self.code = code


def check(rc):
    if rc != GIDS_OK:
        buf = ctypes.create_string_buffer(1024)
        lib().gids_last_error(buf, 1024)
        raise GidsError(rc, buf.value.decode())


class Store:
    """Thin owner of a gids_store_t + gids_ctrls_t pair."""

    def __init__(self, elem_bytes, page_size, num_ele, cache_mb, num_ssd=1, ssd_list=None, read_off_pages=0,
                 capacity=0, pattern=None, device=0, synchronous=True, world=1, rank=0, cache_line=0):
        L = lib()
        self.c = ctypes.c_void_p()
        check(L.gids_ctrls_create(ctypes.byref(self.c)))
        lst = (ctypes.c_int32 * num_ssd)(*(ssd_list or list(range(num_ssd))))
        check(L.gids_ctrls_init(self.c, num_ssd, 1024, 128, lst))
        if capacity or pattern:
            check(L.gids_ctrls_set_emulation(self.c, capacity, (pattern or "").encode()))
        self.s = ctypes.c_void_p()
        check(L.gids_store_create(ctypes.byref(self.s), elem_bytes, device))
        if world > 1:
            check(L.gids_store_set_sharding(self.s, world, rank))
        if cache_line:
            check(L.gids_store_set_cache_line(self.s, cache_line))
        check(L.gids_store_init_controllers(self.s, self.c, page_size, read_off_pages, cache_mb, num_ele, num_ssd))
        check(L.gids_store_set_synchronous(self.s, 1 if synchronous else 0))
        self.elem_bytes = elem_bytes
        self.page_size = page_size

    def close(self):
        if self.s:
            lib().gids_store_destroy(self.s)
            self.s = None
        if self.c:
            lib().gids_ctrls_destroy(self.c)
            self.c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def write_range(self, ptr, nbytes, off):
        check(lib().gids_write_range(self.s, ptr, nbytes, off))

    def read_feature(self, out_ptr, idx_ptr, n, dim, cache_dim, key_off=0, stream=None):
        return lib().gids_read_feature(self.s, out_ptr, idx_ptr, n, dim, cache_dim, key_off, stream)

    def read_multi(self, outs, idxs, ns, dim, cache_dim, key_offs=None, stream=None):
        k = len(outs)
        O = (ctypes.c_void_p * k)(*outs)
        I = (ctypes.c_void_p * k)(*idxs)
        N = (ctypes.c_uint64 * k)(*ns)
        K = (ctypes.c_uint64 * k)(*key_offs) if key_offs is not None else None
        return lib().gids_read_feature_multi(self.s, k, O, I, N, dim, cache_dim, K, stream)

    def stats(self):
        v = (ctypes.c_uint64 * N_STATS)()
        check(lib().gids_get_stats(self.s, v, N_STATS))
        return dict(zip(STAT_NAMES, list(v)[:len(STAT_NAMES)]))

    def reset_stats(self):
        check(lib().gids_reset_stats(self.s))

    def set_policy(self, admission, ref_max):
        mode = (1 if admission else 0) if isinstance(admission, bool) else int(admission)
        check(lib().gids_store_set_cache_policy(self.s, mode, ref_max))

    def geometry(self):
        v = (ctypes.c_uint64 * 8)()
        check(lib().gids_store_geometry(self.s, v, 8))
        return dict(zip(["range_pages", "wrap_pages", "ssd_bytes", "cache_slots", "page_size", "num_ssd",
                         "cache_line", "shard_bytes"], list(v)))
