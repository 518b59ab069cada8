"""Generate the golden gather fixtures from the reference's own CPU data path.

Run in a container that has the reference checkout (it is read, never written):

    python tests/golden/make_golden.py /path/to/reference

The reference's mmap baseline is the parity target for the GIDS gather:
features come from ``IGB260M.paper_feat`` (evaluation/dataloader.py:148-181),
a read-only ``np.load(..., mmap_mode='r')`` / ``np.memmap`` of a row-major
``[N, dim]`` table, wrapped with ``torch.from_numpy`` (dataloader.py:257) and
gathered by DGL as ``blocks[0].srcdata['feat']`` (homogenous_train_baseline.py:244),
which on a CPU tensor is ``torch.index_select(feat, 0, input_nodes)``.

This script imports the reference's ``dataloader`` module (with a stub ``dgl``,
which is not installed here and is not used by ``paper_feat``), writes small
synthetic ``node_feat.npy`` files, loads them through ``IGB260M.paper_feat``
and gathers with ``torch.index_select``. GIDS-specific parameters follow
gids_kernel.cu:68-84 (row ``idx + key_off``, source stride ``cache_dim``,
first ``dim`` columns) and GIDS.py:989-1034 (per-ntype ``key_off``).

Each fixture stores the inputs needed to rebuild the table (generator kind and
seed, or the explicit table when it holds special values), the node ids and
the expected output. The fixtures are small (< 1 MB in total).
"""
from __future__ import annotations

import importlib.util
import os
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import oracle  # noqa: E402


def load_reference_dataloader(ref_root: str):
    # dgl is imported at module scope by dataloader.py but paper_feat does not use it.
    dgl = types.ModuleType("dgl")
    dgl_data = types.ModuleType("dgl.data")

    class DGLDataset:  # minimal base class so the module body executes
        def __init__(self, *a, **k):
            pass

    dgl_data.DGLDataset = DGLDataset
    dgl.data = dgl_data
    sys.modules.setdefault("dgl", dgl)
    sys.modules.setdefault("dgl.data", dgl_data)
    path = os.path.join(ref_root, "evaluation", "dataloader.py")
    spec = importlib.util.spec_from_file_location("gids_ref_dataloader", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_gather(dl, table: np.ndarray, ids: np.ndarray, key_off: int, dim: int) -> np.ndarray:
    """Write `table` as node_feat.npy, load it through IGB260M.paper_feat (OGB
    branch: np.load(path, mmap_mode='r')), gather with torch.index_select."""
    with tempfile.TemporaryDirectory() as d:
        np.save(os.path.join(d, "node_feat.npy"), table)
        ds = dl.IGB260M(root=d, size="experimental", in_memory=0, uva_graph=0, classes=19, synthetic=0,
                        emb_size=table.shape[1], data="OGB")
        feat = ds.paper_feat
        assert isinstance(feat, np.memmap), type(feat)
        t = torch.from_numpy(feat)
        out = torch.index_select(t, 0, torch.from_numpy(ids.astype(np.int64)) + key_off)
        out = out[:, :dim].contiguous().numpy().copy()
        del t, feat
    return out


def special_table(rows: int, cols: int) -> np.ndarray:
    """fp32 table holding NaN payloads, signed zeros, infinities and denormals."""
    rng = np.random.default_rng(7)
    bits = rng.integers(0, 2**32, size=(rows, cols), dtype=np.uint64).astype(np.uint32)
    specials = np.array([0x7FC00001, 0x7F800001, 0xFFC12345, 0x80000000, 0x00000000, 0x7F800000, 0xFF800000,
                         0x00000001, 0x807FFFFF], dtype=np.uint32)
    bits[:, : len(specials)] = specials
    return bits.view(np.float32)


def main(ref_root: str) -> None:
    dl = load_reference_dataloader(ref_root)
    rng = np.random.default_rng(2024)
    cases = {}

    # 1. config-1 shape (fp32, dim 1024, one 4 KB row per page), small N
    rows, cdim = 2048, 1024
    table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, rows, cdim)
    ids = rng.integers(0, rows, size=96).astype(np.int64)
    ids[:4] = [0, rows - 1, 5, 5]  # ends of the table and a duplicate
    cases["homo_f32_d1024"] = dict(kind=oracle.KIND_F32_UNIFORM, seed=1, rows=rows, cache_dim=cdim, dim=cdim,
                                   key_off=0, ids=ids, out=reference_gather(dl, table, ids, 0, cdim))

    # 2. heterograph: four node types laid out contiguously, per-type key offsets
    type_rows = {"t0": 400, "t1": 300, "t2": 50, "t3": 10}
    offs, acc = {}, 0
    for k, v in type_rows.items():
        offs[k] = acc
        acc += v
    table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, acc, 256)
    for k, v in type_rows.items():
        ids = rng.integers(0, v, size=40).astype(np.int64)
        cases[f"hetero_{k}"] = dict(kind=oracle.KIND_F32_UNIFORM, seed=1, rows=acc, cache_dim=256, dim=256,
                                    key_off=offs[k], ids=ids, out=reference_gather(dl, table, ids, offs[k], 256))

    # 3. config-4 shape: fp16 rows of 1536 B that straddle 4 KB pages
    rows, cdim = 600, 768
    table = oracle.synth_table(oracle.KIND_F16_BYTESUM, 1, rows, cdim)
    ids = rng.integers(0, rows, size=64).astype(np.int64)
    cases["homo_f16_d768"] = dict(kind=oracle.KIND_F16_BYTESUM, seed=1, rows=rows, cache_dim=cdim, dim=cdim,
                                  key_off=0, ids=ids, out=reference_gather(dl, table, ids, 0, cdim))

    # 4. config-5 shape: fp32 dim 128 (512 B rows, 8 rows per page)
    rows, cdim = 4096, 128
    table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, rows, cdim)
    ids = rng.integers(0, rows, size=256).astype(np.int64)
    cases["homo_f32_d128"] = dict(kind=oracle.KIND_F32_UNIFORM, seed=1, rows=rows, cache_dim=cdim, dim=cdim,
                                  key_off=0, ids=ids, out=reference_gather(dl, table, ids, 0, cdim))

    # 5. dim < cache_dim (column subset) and a nonzero key_off on a homogeneous call
    rows, cdim, dim = 1000, 1024, 200
    table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 3, rows, cdim)
    ids = rng.integers(0, rows - 17, size=50).astype(np.int64)
    cases["subset_d200_of_1024"] = dict(kind=oracle.KIND_F32_UNIFORM, seed=3, rows=rows, cache_dim=cdim, dim=dim,
                                        key_off=17, ids=ids, out=reference_gather(dl, table, ids, 17, dim))

    # 6. long_type store (int64 features)
    rows, cdim = 300, 512
    table = oracle.synth_table(oracle.KIND_I64_RAW, 5, rows, cdim)
    ids = rng.integers(0, rows, size=32).astype(np.int64)
    cases["long_d512"] = dict(kind=oracle.KIND_I64_RAW, seed=5, rows=rows, cache_dim=cdim, dim=cdim, key_off=0,
                              ids=ids, out=reference_gather(dl, table, ids, 0, cdim))

    # 7. special fp32 bit patterns (explicit table stored in the fixture)
    rows, cdim = 64, 64
    table = special_table(rows, cdim)
    ids = rng.integers(0, rows, size=48).astype(np.int64)
    cases["special_f32"] = dict(kind=0, seed=0, rows=rows, cache_dim=cdim, dim=cdim, key_off=0, ids=ids,
                                out=reference_gather(dl, table, ids, 0, cdim), table=table)

    # 8. empty minibatch
    table = oracle.synth_table(oracle.KIND_F32_UNIFORM, 1, 16, 1024)
    ids = np.zeros(0, dtype=np.int64)
    cases["empty"] = dict(kind=oracle.KIND_F32_UNIFORM, seed=1, rows=16, cache_dim=1024, dim=1024, key_off=0,
                          ids=ids, out=reference_gather(dl, table, ids, 0, 1024))

    # generator pins: a few raw stream values
    pins = np.array([[s, e, oracle.synth_u64(s, e)] for s in (0, 1, 12345) for e in (0, 1, 2, 10**9, 2**40)],
                    dtype=np.uint64)

    dest = os.path.join(HERE, "gather_golden.npz")
    flat = {"synth_pins": pins}
    for name, c in cases.items():
        for k, v in c.items():
            flat[f"{name}/{k}"] = np.asarray(v)
    np.savez_compressed(dest, **flat)
    print(f"wrote {dest}: {len(cases)} cases, {os.path.getsize(dest)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
