"""CPU oracle for the GIDS feature gather and its inputs (test infrastructure only).

Only tests/, the smoke entry point and the bench's CPU-baseline leg import this
module; the product never does. It wraps the plain-C restatement in
gids_oracle.c (built by oracle/Makefile into oracle/_build/) and restates the
reference's mmap baseline gather in numpy/torch:

* evaluation/dataloader.py:166-169 -- features are a row-major np.memmap
  ``[N, dim]`` wrapped with ``torch.from_numpy``;
* evaluation/homogenous_train_baseline.py:244 -- DGL's ``blocks[0].srcdata['feat']``
  on a CPU tensor, i.e. ``torch.index_select(feat, 0, input_nodes)``;
* gids_module/gids_kernel.cu:68-84 -- GIDS reads row ``idx + key_off`` with
  source stride ``cache_dim`` and keeps the first ``dim`` columns;
* GIDS_Setup/GIDS/GIDS.py:989-1034 -- heterographs gather each node type
  with ``key_off = heterograph_map[ntype]`` (node-ID units).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libgids_oracle.so")

KIND_F32_UNIFORM = 1
KIND_F16_BYTESUM = 2
KIND_I64_RAW = 3
KIND_F16_NORMAL = 4
KIND_DTYPE = {KIND_F32_UNIFORM: np.float32, KIND_F16_BYTESUM: np.float16, KIND_I64_RAW: np.int64,
              KIND_F16_NORMAL: np.float16}

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u64, i64, u32, i32, vp = ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p
        L.go_synth_u64.restype = u64
        L.go_synth_u64.argtypes = [u64, u64]
        L.go_synth_fill.restype = i32
        L.go_synth_fill.argtypes = [i32, u64, u64, u64, vp, i32]
        L.go_gather.restype = i32
        L.go_gather.argtypes = [vp, u64, u32, u32, u32, vp, i64, u64, vp, i32]
        L.go_gather_synth.restype = i32
        L.go_gather_synth.argtypes = [i32, u64, u64, u64, u32, u32, vp, i64, u64, vp, i32]
        L.go_stripe_locate.restype = None
        L.go_stripe_locate.argtypes = [u64, u64, u64, u64, ctypes.POINTER(u64), ctypes.POINTER(u64)]
        L.go_stripe_image.restype = i32
        L.go_stripe_image.argtypes = [vp, u64, u32, u64, u64, ctypes.POINTER(vp), u64]
        L.go_hop_seed.restype = u64
        L.go_hop_seed.argtypes = [u64, u64, u64]
        L.go_edge_key.restype = u64
        L.go_edge_key.argtypes = [u64, u64, u64]
        L.go_sample.restype = i64
        L.go_sample.argtypes = [vp, vp, i32, u64, vp, i32, vp, u64, u64, u64, vp, u64]
        L.go_pagerank_f32.restype = i32
        L.go_pagerank_f32.argtypes = [vp, vp, i32, u64, i32, ctypes.c_double, vp]
        L.go_topk_desc.restype = i32
        L.go_topk_desc.argtypes = [vp, u64, u64, vp]
        _lib = L
    return _lib


def threads() -> int:
    return max(1, os.cpu_count() or 1)


def synth_u64(seed: int, e: int) -> int:
    return lib().go_synth_u64(seed, e)


def synth_table(kind: int, seed: int, rows: int, cache_dim: int, first_row: int = 0) -> np.ndarray:
    """Row-major synthetic table ``[rows, cache_dim]``: element (r, c) is the
    synthetic element ``(first_row + r) * cache_dim + c``."""
    out = np.empty((rows, cache_dim), dtype=KIND_DTYPE[kind])
    rc = lib().go_synth_fill(kind, seed, first_row * cache_dim, rows * cache_dim, out.ctypes.data, threads())
    assert rc == 0
    return out


def synth_fill_into(kind: int, seed: int, first_elem: int, arr: np.ndarray) -> None:
    """Fill a contiguous array (e.g. an np.memmap) with synthetic elements starting at first_elem."""
    assert arr.flags.c_contiguous and arr.dtype == KIND_DTYPE[kind]
    rc = lib().go_synth_fill(kind, seed, first_elem, arr.size, arr.ctypes.data, threads())
    assert rc == 0


def gather(table: np.ndarray, ids: np.ndarray, dim: int | None = None, key_off: int = 0) -> np.ndarray:
    """C restatement of read_feature_kernel over a row-major table (gids_kernel.cu:68-84)."""
    assert table.ndim == 2 and table.flags.c_contiguous
    cache_dim = table.shape[1]
    dim = cache_dim if dim is None else dim
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((ids.shape[0], dim), dtype=table.dtype)
    rc = lib().go_gather(table.ctypes.data, table.shape[0], table.dtype.itemsize, cache_dim, dim,
                         ids.ctypes.data, ids.shape[0], key_off, out.ctypes.data, threads())
    if rc == -2:
        raise IndexError("node id out of range")
    assert rc == 0
    return out


def gather_synth(kind: int, seed: int, table_rows: int, cache_dim: int, dim: int, ids: np.ndarray,
                 key_off: int = 0, wrap_elems: int = 0) -> np.ndarray:
    """Expected gather of the synthetic table without materialising it."""
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((ids.shape[0], dim), dtype=KIND_DTYPE[kind])
    rc = lib().go_gather_synth(kind, seed, wrap_elems, table_rows, cache_dim, dim, ids.ctypes.data,
                               ids.shape[0], key_off, out.ctypes.data, threads())
    if rc == -2:
        raise IndexError("node id out of range")
    assert rc == 0
    return out


def stripe_locate(page: int, n_ctrls: int, page_start: int, wrap_pages: int = 0) -> tuple[int, int]:
    c, p = ctypes.c_uint64(), ctypes.c_uint64()
    lib().go_stripe_locate(page, n_ctrls, page_start, wrap_pages, ctypes.byref(c), ctypes.byref(p))
    return c.value, p.value


def stripe_image(logical: np.ndarray, page_size: int, n_ctrls: int, page_start: int, dev_bytes: int) -> list[np.ndarray]:
    """Per-device byte images of a striped store holding ``logical`` (bytes)."""
    logical = np.ascontiguousarray(logical).view(np.uint8).reshape(-1)
    devs = [np.zeros(dev_bytes, dtype=np.uint8) for _ in range(n_ctrls)]
    ptrs = (ctypes.c_void_p * n_ctrls)(*[d.ctypes.data for d in devs])
    rc = lib().go_stripe_image(logical.ctypes.data, logical.size, page_size, n_ctrls, page_start, ptrs, dev_bytes)
    assert rc == 0, rc
    return devs


# ------------------------------------------------------------------ sampler and pin list
def hop_seed(seed: int, call: int, hop: int) -> int:
    return lib().go_hop_seed(seed & (2**64 - 1), call, hop)


def edge_key(seed_h: int, v: int, j: int) -> int:
    return lib().go_edge_key(seed_h & (2**64 - 1), v, j)


def _csc(indptr, indices):
    indptr = np.ascontiguousarray(indptr, dtype=np.int64)
    indices = np.ascontiguousarray(indices)
    assert indices.dtype in (np.int32, np.int64)
    return indptr, indices, indices.dtype.itemsize


def sample(indptr, indices, fanouts, seeds, seed: int, call: int = 0) -> np.ndarray:
    """Restated MultiLayerNeighborSampler with counter-hashed edge choice
    (sampler_oracle.c): the input nodes of one minibatch, seeds first."""
    indptr, indices, ib = _csc(indptr, indices)
    n = indptr.shape[0] - 1
    f = np.ascontiguousarray(fanouts, dtype=np.int32)
    seeds = np.ascontiguousarray(seeds, dtype=np.int64)
    cap = max(1, n)
    out = np.empty(cap, dtype=np.int64)
    rc = lib().go_sample(indptr.ctypes.data, indices.ctypes.data, ib, n, f.ctypes.data, len(f), seeds.ctypes.data,
                         len(seeds), seed & (2**64 - 1), call, out.ctypes.data, cap)
    if rc == -2:
        raise IndexError("seed outside the graph")
    assert rc >= 0, rc
    return out[:rc].copy()


def pagerank_f32(indptr, indices, iters: int = 20, damping: float = 0.85) -> np.ndarray:
    """compute_pagerank (page_rank_node_list_gen.py:126-134) restated in float32 (sampler_oracle.c)."""
    indptr, indices, ib = _csc(indptr, indices)
    n = indptr.shape[0] - 1
    pv = np.empty(n, dtype=np.float32)
    rc = lib().go_pagerank_f32(indptr.ctypes.data, indices.ctypes.data, ib, n, iters, damping, pv.ctypes.data)
    assert rc == 0, rc
    return pv


def topk_desc(pv: np.ndarray, k: int) -> np.ndarray:
    """Node ids of the k largest values, value descending then id ascending."""
    pv = np.ascontiguousarray(pv, dtype=np.float32)
    out = np.empty(k, dtype=np.int64)
    assert lib().go_topk_desc(pv.ctypes.data, pv.shape[0], k, out.ctypes.data) == 0
    return out


# ------------------------------------------------------------------ mmap baseline
def open_memmap_table(path: str, dtype, rows: int, dim: int) -> np.memmap:
    """Reference idiom (evaluation/dataloader.py:166-169): read-only row-major memmap."""
    return np.memmap(path, dtype=dtype, mode="r", shape=(rows, dim))


def mmap_index_select(feat_np: np.ndarray, ids, dim: int | None = None, key_off: int = 0):
    """Reference baseline gather: ``torch.index_select(torch.from_numpy(memmap), 0, ids)``
    (homogenous_train_baseline.py:244 through DGL's CPU srcdata gather), with
    the GIDS row offset and column slice applied (gids_kernel.cu:68-84)."""
    import warnings

    import torch

    with warnings.catch_warnings():  # read-only memmap, as in the reference
        warnings.simplefilter("ignore", UserWarning)
        t = torch.from_numpy(feat_np) if not isinstance(feat_np, torch.Tensor) else feat_np
    ids_t = torch.as_tensor(ids, dtype=torch.int64)
    if key_off:
        ids_t = ids_t + key_off
    out = torch.index_select(t, 0, ids_t)
    if dim is not None and dim != out.shape[1]:
        out = out[:, :dim].contiguous()
    return out
