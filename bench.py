"""Benchmark of the GIDS minibatch feature gather on B200.

One step = one minibatch: the gather of the input-node features of one
sampled minibatch (GIDS.fetch_feature's gather; the sampler is excluded, as
in the reference's metric). Default workload: config 2 of the reference's
benchmark table -- 100M-node homogeneous graph, fp32 x 1024 features
(409.6 GB range), 4 KB pages striped over 4 emulated SSDs (ssd_list
[0,1,2,3]), 40 GB GPU page cache, 3-layer fanout [15,10,5], batch 4096
uniform seeds. Data is synthetic: features from the seeded generator, node
ids from the seeded synthetic graph and sampler (GIDS/synthetic.py).

The emulated SSDs hold `--phys-gb` GB of pages (default 64); logical page p
is stored where page p mod (that many pages) is, so the 409.6 GB range, the
cache behaviour and the host-link traffic are those of the full config while
host RAM holds a fraction of it (the box has 196 GB of RAM).

Timed regions (after --warmup steps, each bracketed by a barrier and a
device synchronize, max over ranks):
  value: K gathers with the node ids already in HBM (kernel path);
  e2e:   K calls of GIDS.fetch_feature with the ids in pinned host memory
         (H2D copy of the ids, gather, D2H read of one output element).
A config-2 step reads about 13 GB, far larger than the 126 MB L2, so no
flush is needed between steps (the line's config.l2 states the size).

Multi-GPU (torchrun): one process per GPU, each an independent
data-parallel trainer with its own sampler seed (1000 + rank). The ranks'
page caches form one cache sharded by page id (page p on rank p % N; hits on
other ranks' pages are NVLink peer loads, misses fill the owner's slot);
the emulated SSDs are one shared-memory copy mapped by every rank. Only
setup (CUDA IPC handles), barriers and the max-over-ranks timing use
torch.distributed.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "gids-study_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

# policy: the default cache policy of the config (see POLICIES): the homogeneous graphs without window
# buffering hold a static hot set (the rows of highest out-degree); the heterograph (no CSC here) and the
# window-buffered config 4 keep the dynamic policy
BASE = dict(cpu_pin_frac=0.0, wb=0, phys_gb=64.0, line=0, hetero=None, policy="static")
C3_TYPES = {"t0": 40_000_000, "t1": 30_000_000, "t2": 5_000_000, "t3": 1_000_000}
C3_RELATIONS = [("t0", "t0"), ("t1", "t0"), ("t2", "t0"), ("t3", "t0"), ("t0", "t1"), ("t1", "t2")]
CONFIGS = {
    # nodes, mean degree, zipf alpha of the out-degree, feature dim/dtype, page size, emulated SSDs,
    # cache MB per GPU, fanouts, seed batch, seed law (None = uniform), pinned fraction, WB depth
    "c1": dict(BASE, nodes=1_000_000, mean_deg=15, alpha=1.1, dim=1024, dtype="float32", page=4096, ssds=1,
               cache_mb=4096, fanouts=[10, 5], batch=1024, seed_zipf=None),
    "c2": dict(BASE, nodes=100_000_000, mean_deg=15, alpha=1.1, dim=1024, dtype="float32", page=4096, ssds=4,
               cache_mb=40 * 1024, fanouts=[15, 10, 5], batch=4096, seed_zipf=None),
    "c3": dict(BASE, nodes=sum(C3_TYPES.values()), mean_deg=8, alpha=1.0, dim=1024, dtype="float32", page=4096,
               ssds=4, cache_mb=40 * 1024, fanouts=[15, 10], batch=1024, seed_zipf=None,
               hetero=dict(types=C3_TYPES, relations=C3_RELATIONS, seed_type="t0"), policy="admit2"),
    "c4": dict(BASE, nodes=50_000_000, mean_deg=15, alpha=1.2, dim=768, dtype="float16", page=4096, ssds=4,
               cache_mb=8 * 1024, fanouts=[10, 10], batch=2048, seed_zipf=1.0, cpu_pin_frac=0.01, wb=8,
               phys_gb=80.0, line=512, policy="admit2"),
    "c5": dict(BASE, nodes=500_000_000, mean_deg=10, alpha=1.1, dim=128, dtype="float32", page=4096, ssds=8,
               cache_mb=20 * 1024, fanouts=[20, 15, 10], batch=8192, seed_zipf=None, line=512),
}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per gathered row of gather_kernel, from one
# ncu --set full capture of a small case of the same config and policy, after the same cache warm-up
# (config 2, static hot set: 4M nodes, 2 GB cache, batch 512 -> 2.467 GB over 366,742 rows at 50 %
# hits; the full run has 45 %); a full launch's traffic is this times its rows. Other configs and
# policies report null.
TRAFFIC_PER_ROW = {("c2", "static"): 2.4666e9 / 366742}
# synthetic feature streams: fp32 uniform[-1, 1) (configs 1-3, 5), fp16 normal(0, 1) (config 4)
KIND = {"float32": 1, "float16": 4}
METRIC = "feature-gather GB/s (gathered rows x row bytes / gather time), all GPUs"
DATA = "synthetic (seeded features, seeded synthetic graph + neighbour sampler; DGL and IGB absent)"
TDTYPE = {"float32": torch.float32, "float16": torch.float16}
ESIZE = {"float32": 4, "float16": 2}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ distributed
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl", device=None):
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kw = dict(backend=backend, timeout=datetime.timedelta(seconds=300))
            if backend == "nccl" and device is not None:
                kw["device_id"] = device
            dist.init_process_group(**kw)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            if self.pg.get_backend() == "nccl":
                self.pg.barrier(device_ids=[self.local])
            else:
                self.pg.barrier()

    def max(self, v: float) -> float:
        if self.pg is None:
            return v
        dev = torch.device("cuda", self.local) if self.pg.get_backend() == "nccl" else torch.device("cpu")
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if self.pg is None:
            return v
        dev = torch.device("cuda", self.local) if self.pg.get_backend() == "nccl" else torch.device("cpu")
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def gather(self, v: float) -> list:
        """v of every rank, in rank order"""
        if self.pg is None:
            return [v]
        dev = torch.device("cuda", self.local) if self.pg.get_backend() == "nccl" else torch.device("cpu")
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [float(x.item()) for x in out]

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def sampler_seed(rank: int) -> int:
    return 1000 + rank


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ workload
_CSC = {}


def graph_csc(cfg, device):
    """Explicit CSC of the config's synthetic graph on `device` (int32
    sources), built once per process."""
    from GIDS.synthetic import SyntheticGraph

    key = (cfg["nodes"], cfg["mean_deg"], cfg["alpha"], str(device))
    if key not in _CSC:
        g = SyntheticGraph(cfg["nodes"], cfg["mean_deg"], cfg["alpha"], seed=0, device=device)
        idx_dtype = torch.int32 if cfg["nodes"] < 2**31 else torch.int64
        _CSC[key] = g.materialize(idx_dtype)
        del g
    return _CSC[key]


def use_gpu_sampler(cfg, device) -> bool:
    """Homogeneous graphs on a GPU draw their minibatches with the CUDA
    sampler (bit-identical to the torch sampler: tests/test_sampler_gpu.py);
    heterographs and CPU runs use the torch sampler."""
    return str(device) != "cpu" and not cfg["hetero"] and not cfg.get("torch_sampler")


def batch_stream(cfg, n_batches, rank, device):
    """Input-node ids of n_batches minibatches from the seeded graph and
    sampler, produced lazily (one neighbour-sampling pass per next())."""
    from GIDS.synthetic import NeighborSampler, SyntheticGraph, seed_batches

    if cfg["hetero"]:
        from GIDS.synthetic import HeteroNeighborSampler, HeteroSyntheticGraph

        h = cfg["hetero"]
        hg = HeteroSyntheticGraph(h["types"], h["relations"], cfg["mean_deg"], cfg["alpha"], seed=0, device=device)
        hs = HeteroNeighborSampler(hg, cfg["fanouts"], seed=sampler_seed(rank))
        for sd in seed_batches(h["types"][h["seed_type"]], cfg["batch"], n_batches, sampler_seed(rank), device=device):
            yield hs.sample({h["seed_type"]: sd})[0]
        return
    if use_gpu_sampler(cfg, device):
        from GIDS.sampler import GPUNeighborSampler

        indptr, indices = graph_csc(cfg, device)
        s = GPUNeighborSampler(indptr, indices, cfg["fanouts"], seed=sampler_seed(rank), max_seeds=cfg["batch"])
    else:
        g = SyntheticGraph(cfg["nodes"], cfg["mean_deg"], cfg["alpha"], seed=0, device=device)
        s = NeighborSampler(g, cfg["fanouts"], seed=sampler_seed(rank))
    for sd in seed_batches(cfg["nodes"], cfg["batch"], n_batches, sampler_seed(rank), device=device,
                           zipf_alpha=cfg["seed_zipf"]):
        yield s.sample(sd)[0]


class SideStreamBatches:
    """Iterator of [input_nodes] whose sampling runs on `side`; the consumer's
    stream waits for each batch with an event, so a batch is sampled while
    the consumer's previous work (the gather) is still running."""

    def __init__(self, gen, side, main):
        self.gen, self.side, self.main = gen, side, main

    def __iter__(self):
        return self

    def __next__(self):
        with torch.cuda.stream(self.side):
            b = next(self.gen)
            ev = torch.cuda.Event()
            ev.record(self.side)
        self.main.wait_event(ev)
        for t in (b.values() if isinstance(b, dict) else [b]):
            t.record_stream(self.main)
        return [b]


def time_sampler(cfg, n, rank, device, side):
    """Milliseconds per minibatch of the neighbour sampler alone, on `side`."""
    gen = batch_stream(cfg, n + 1, rank, device)
    with torch.cuda.stream(side):
        next(gen)  # graph setup and first-call costs stay out of the figure
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            next(gen)
        torch.cuda.synchronize()
    return (time.perf_counter() - t0) / n * 1e3


def make_batches(cfg, n_batches, rank, device, with_pins=False):
    """Input-node ids of n_batches minibatches from the seeded graph and
    sampler, and (with_pins) the PageRank pin list of the constant CPU buffer
    (the float32 GPU PageRank of the graph's CSC)."""
    t0 = time.time()
    pins = None
    if with_pins and cfg["cpu_pin_frac"] > 0 and not cfg["hetero"]:
        from GIDS.sampler import pagerank_pin_list

        indptr, indices = graph_csc(cfg, device)
        pins = pagerank_pin_list(indptr, indices, cfg["cpu_pin_frac"])
    out = list(batch_stream(cfg, n_batches, rank, device))
    if device != "cpu":
        torch.cuda.synchronize()
    if with_pins:
        return out, pins, time.time() - t0
    return out, time.time() - t0


# per-phase gather timers of a diagnosis build (stats names)
PHASES = ("ns_lookup", "ns_fill_wait", "ns_copy", "ns_release")

# untimed cache warm-up, in cache-sizes of line references
CACHE_WARMUP_CACHES = 12

# cache replacement policies: (admission on the second miss, clock counter ceiling)
POLICIES = {"admit2": (True, 3), "clock": (False, 1), "admit2_sc": (True, 1), "clock3": (False, 3),
            "static": ("static", 3)}


def host_link_peak_gbs(device, dist=None) -> float:
    """Pinned host -> device copy bandwidth (GB/s), best of 4 x 1 GiB. With
    several ranks, all ranks copy at the same time (a barrier before each
    copy), which is the link bandwidth one GPU gets while the others also read
    host memory."""
    n = 1 << 30
    h = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(n, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(4):
        if dist is not None:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        d.copy_(h, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, n / 1e9 / (a.elapsed_time(b) / 1e3))
    del h, d
    return best


def measured_hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s"


# ------------------------------------------------------------------ CPU baseline
def memmap_rows(cfg, file_gb: float) -> tuple[int, str]:
    """Rows of the CPU-baseline memmap and how ids map onto it. file_gb = 0:
    the bytes the GPU arm's emulated SSDs physically hold (the whole range when
    they hold it), capped at 40 % of host RAM; when that is the SSDs' wrap
    period, row r of the memmap holds exactly what the GPU arm reads for every
    id = r mod rows, so both arms gather the same bytes."""
    row_bytes = cfg["dim"] * ESIZE[cfg["dtype"]]
    logical, physical, wrap = backing_geometry(cfg)
    try:
        ram = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError):
        ram = 64 << 30
    want = int(file_gb * 1e9) if file_gb > 0 else physical
    want = min(want, int(0.4 * ram))
    rows = max(1, min(cfg["nodes"], want // row_bytes))
    same = (wrap == 0 and rows == cfg["nodes"]) or (wrap and rows * cfg["dim"] == wrap)
    return rows, ("the same bytes as the GPU arm (its emulated SSDs' wrap period)" if same
                  else f"ids mod {rows} rows (not the GPU arm's wrap period)")


def _flat_ids(cfg, ids):
    if isinstance(ids, dict):  # heterograph: type-local ids + the type's offset
        offs, acc = {}, 0
        for t, n in cfg["hetero"]["types"].items():
            offs[t] = acc
            acc += n
        return np.concatenate([v.cpu().numpy() + offs[k] for k, v in ids.items()])
    return ids.cpu().numpy()


def cpu_mmap_gather(cfg, ids_list, seconds_budget, path_dir="/dev/shm", file_gb=0.0, warmup_ids=(), h2d=True):
    """The reference's mmap baseline gather (torch.index_select on a np.memmap,
    evaluation/dataloader.py:166-169 + homogenous_train_baseline.py:244),
    timed on the host cores on a bounded sample of the same minibatches, with
    the OS page cache warm (the file in /dev/shm). With h2d, the reference's
    copy of each gathered minibatch to the GPU (homogenous_train_baseline.py:253)
    is timed after it and reported separately."""
    from oracle import oracle

    dim, dt = cfg["dim"], cfg["dtype"]
    row_bytes = dim * ESIZE[dt]
    rows, mapping = memmap_rows(cfg, file_gb)
    path = os.path.join(path_dir if os.path.isdir(path_dir) else "/tmp", f"gids_b200_mmap_{os.getpid()}.bin")
    t0 = time.perf_counter()
    mm = np.memmap(path, dtype=np.dtype(dt), mode="w+", shape=(rows, dim))
    oracle.synth_fill_into(KIND[dt], 1, 0, mm.reshape(-1))
    mm.flush()
    del mm
    t_fill = time.perf_counter() - t0
    feat = oracle.open_memmap_table(path, np.dtype(dt), rows, dim)
    try:
        for ids in warmup_ids:
            oracle.mmap_index_select(feat, torch.as_tensor(_flat_ids(cfg, ids) % rows))
        done_rows, t_total, n_batches = 0, 0.0, 0
        t_h2d, h2d_note = 0.0, None
        for ids in ids_list:
            ids_m = torch.as_tensor(_flat_ids(cfg, ids) % rows)
            t0 = time.perf_counter()
            out = oracle.mmap_index_select(feat, ids_m)
            t_total += time.perf_counter() - t0
            if h2d and h2d_note is None and torch.cuda.is_available():
                try:
                    torch.cuda.synchronize()
                    t1 = time.perf_counter()
                    dev_out = out.to("cuda")
                    torch.cuda.synchronize()
                    t_h2d += time.perf_counter() - t1
                    del dev_out
                except Exception as e:  # the baseline's own number stands without it
                    h2d_note = f"H2D copy not timed: {type(e).__name__}"
            done_rows += out.shape[0]
            n_batches += 1
            del out
            if t_total >= seconds_budget:
                break
    finally:
        del feat
        os.unlink(path)
    gbs = done_rows * row_bytes / 1e9 / t_total
    extra = {}
    if t_h2d > 0 and h2d_note is None:
        extra = dict(h2d_gbs=round(done_rows * row_bytes / 1e9 / t_h2d, 2),
                     with_h2d_gbs=round(done_rows * row_bytes / 1e9 / (t_total + t_h2d), 2),
                     h2d_note="pageable tensor.to('cuda') of each gathered minibatch, as the reference does")
    elif h2d_note is not None:
        extra = dict(h2d_note=h2d_note)
    return dict(value=gbs, unit="GB/s", cores=torch.get_num_threads(), kind="port", **extra,
                minibatches_per_s=n_batches / t_total, seconds=t_total, steps=n_batches, fill_s=round(t_fill, 1),
                sample=f"{n_batches} minibatches ({done_rows} rows of {row_bytes} B) gathered by torch.index_select "
                       f"from a {rows * row_bytes / 1e9:.1f} GB np.memmap in {path_dir}, page cache warm; "
                       f"{mapping}")


def cpu_mmap_gather_cold(cfg, ids, seconds_budget=15.0, file_gb=4.0):
    """The same gather from a memmap whose pages are not in the OS page cache:
    a file on the local disk, written, synced and dropped from the cache
    (posix_fadvise DONTNEED) before a bounded sample of one minibatch's ids is
    gathered in chunks. The reference's loader reads its feature file this way
    when the file is larger than host RAM."""
    import tempfile

    from oracle import oracle

    dim, dt = cfg["dim"], cfg["dtype"]
    row_bytes = dim * ESIZE[dt]
    d = tempfile.gettempdir()
    try:
        st = os.statvfs(d)
        free = st.f_bavail * st.f_frsize
    except OSError:
        free = 0
    rows = max(1, min(cfg["nodes"], int(min(file_gb * 1e9, 0.3 * free)) // row_bytes))
    if rows * row_bytes < 1e9:
        return {"note": f"no room for a cold-cache file in {d}"}
    path = os.path.join(d, f"gids_b200_cold_{os.getpid()}.bin")
    try:
        mm = np.memmap(path, dtype=np.dtype(dt), mode="w+", shape=(rows, dim))
        oracle.synth_fill_into(KIND[dt], 1, 0, mm.reshape(-1))
        mm.flush()
        del mm
        fd = os.open(path, os.O_RDONLY)
        try:
            os.fsync(fd)
            os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
        finally:
            os.close(fd)
        feat = oracle.open_memmap_table(path, np.dtype(dt), rows, dim)
        ids_m = torch.as_tensor(_flat_ids(cfg, ids) % rows)
        done, t_total = 0, 0.0
        for lo in range(0, ids_m.numel(), 16384):
            part = ids_m[lo:lo + 16384]
            t0 = time.perf_counter()
            out = oracle.mmap_index_select(feat, part)
            t_total += time.perf_counter() - t0
            done += out.shape[0]
            del out
            if t_total >= seconds_budget:
                break
        del feat
    finally:
        if os.path.exists(path):
            os.unlink(path)
    return {"value": round(done * row_bytes / 1e9 / t_total, 3), "unit": "GB/s", "rows": done,
            "sample": f"first {done} ids of one minibatch gathered by torch.index_select from a "
                      f"{rows * row_bytes / 1e9:.1f} GB np.memmap on the local disk ({d}) after fsync + "
                      f"posix_fadvise(DONTNEED)"}


# ------------------------------------------------------------------ parity
def parity_check(cfg, ids, feat, hmap, n_rows: int, seed: int = 0) -> dict:
    """Compares n_rows gathered rows per node type (a seeded random subset,
    always with the first and the last row) bit for bit with the oracle's
    restatement of the reference gather over the same synthetic table."""
    from oracle import oracle

    dim, dt = cfg["dim"], cfg["dtype"]
    _, _, wrap = backing_geometry(cfg)
    rng = np.random.default_rng(seed)
    if isinstance(feat, dict):
        items = [(k, ids[k], feat[k], hmap[k]) for k in feat]
    else:
        items = [(None, ids, feat, 0)]
    checked, bad = 0, 0
    for _, idv, out, key_off in items:
        n = int(idv.numel())
        if n == 0:
            continue
        m = min(n, n_rows)
        pick = np.unique(np.concatenate([[0, n - 1], rng.choice(n, size=m, replace=False)]))
        pt = torch.as_tensor(pick, device=out.device)
        got = out.index_select(0, pt).cpu().numpy()
        want = oracle.gather_synth(KIND[dt], 1, cfg["nodes"], dim, dim, idv.index_select(0, pt.to(idv.device)).cpu()
                                   .numpy(), key_off=key_off, wrap_elems=wrap)
        same = np.all(got.view(np.uint8).reshape(len(pick), -1) == want.view(np.uint8).reshape(len(pick), -1), axis=1)
        bad += int((~same).sum())
        checked += len(pick)
    return {"rows_checked": checked, "ok": bad == 0, "mismatched_rows": bad}


# ------------------------------------------------------------------ our arm
def replica_reservation(args, cfg, sharded: bool) -> int:
    """Cache lines each shard reserves for replicated rows: up to all of its slots."""
    if not sharded or args.replicate == "off" or cfg["hetero"]:
        return 0
    line = cfg["line"] or cfg["page"]
    return (cfg["cache_mb"] << 20) // line


def replica_model(cum, total: float, per_rank: int, world: int, bw_nvlink: float,
                  bw_host: float) -> tuple[int, float]:
    """Rows to replicate and the modelled per-GPU gather rate (GB/s). cum[i] =
    references to the i hottest rows (cum[0] = 0, len = rows ranked + 1); each
    GPU holds `per_rank` rows: the R replicated ones and its share of the next
    world x (per_rank - R), sharded by page id. A reference to a replicated row
    or to a row of the own shard reads HBM, to another shard NVLink, to an
    uncached row the host link; per gathered byte the time is the larger of
    f_remote / BW_NVLink and f_host / BW_host, with the link rates at the
    fractions of their peaks the gather reaches (NVLink 0.86, host link 0.92,
    measured). HBM is left out: replication moves no HBM traffic (every cached
    byte is read from some GPU's HBM either way), and on 2 GPUs a model capped
    by an HBM term stopped short of the measured best. The smallest R within
    0.1 % of the best rate wins."""
    n = len(cum) - 1
    best, best_r = 0.0, 0
    for r in range(0, per_rank + 1, max(1, per_rank // 64)):
        a, end = min(r, n), min(r + world * (per_rank - r), n)
        rep_f = float(cum[a]) / total
        shard_f = (float(cum[end]) - float(cum[a])) / total
        remote, host = shard_f * (world - 1) / world, max(0.0, 1.0 - rep_f - shard_f)
        rate = 1.0 / max(remote / (0.86 * bw_nvlink), host / (0.92 * bw_host), 1e-9)
        if rate > best * 1.001:
            best, best_r = rate, r
    return best_r, best


def choose_replicas(args, cfg, g, hot, device, dist, lpr, bw_nvlink, bw_host) -> int:
    """How many of the hottest rows every rank holds (a prefix of `hot`, the rows
    in out-degree order). 'auto': replica_model's choice, with the reference
    counts of 16 minibatches pre-sampled with other seeds and the live link
    peaks. Every rank uses rank 0's choice."""
    if args.replicate == "off":
        return 0
    per_rank = int(g.BAM_FS.geometry()["cache_slots"]) // lpr
    if args.replicate != "auto":
        return int(dist.max(float(min(int(args.replicate), per_rank, hot.numel()))))
    from GIDS.sampler import out_degree

    counts = torch.zeros(cfg["nodes"], dtype=torch.int32, device=device)
    for b in batch_stream(cfg, 16, dist.rank + 104729, device):
        counts += out_degree(b.contiguous(), cfg["nodes"])
    total = float(counts.sum(dtype=torch.int64))
    cum = torch.cat([torch.zeros(1, dtype=torch.float64, device=device),
                     counts[hot].to(torch.float64).cumsum(0)]).cpu()
    del counts
    best_r, best = replica_model(cum.numpy(), total, per_rank, g.world, bw_nvlink, bw_host)
    log(f"[rank {dist.rank}] replicas: model picks {best_r} rows ({best:.0f} GB/s per GPU modelled)")
    return int(dist.max(float(best_r))) if dist.rank == 0 else int(dist.max(0.0))


def run_ours(args, cfg, dist: Dist):
    import GIDS

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    dt, dim, page = cfg["dtype"], cfg["dim"], cfg["page"]
    esize = ESIZE[dt]
    row_bytes = dim * esize
    num_ele = cfg["nodes"] * dim
    range_bytes = num_ele * esize
    phys = min(int(cfg["phys_gb"] * 1e9), range_bytes)
    per_ssd = (phys // cfg["ssds"]) // page * page
    shared = dist.world > 1 or args.shared_backing
    hmap = None
    if cfg["hetero"]:
        hmap, acc = {}, 0
        for t, n in cfg["hetero"]["types"].items():
            hmap[t] = acc
            acc += n
    pattern = f"/dev/shm/gids_b200_bench_{os.environ.get('MASTER_PORT', 'x')}_ssd{{}}" if shared else None

    t0 = time.time()
    t_fill = 0.0
    if shared:
        # rank 0 writes the shared emulated SSDs once; every rank then maps them
        if dist.rank == 0:
            import BAM_Feature_Store

            c = BAM_Feature_Store.GIDS_Controllers()
            c.init_GIDS_controllers(cfg["ssds"], 1024, 128, list(range(cfg["ssds"])))
            c.set_emulation(per_ssd if phys < range_bytes else 0, pattern)
            c.bind(cfg["ssds"], page, 0, range_bytes)
            tf = time.time()
            c.fill_synthetic(KIND[dt], 1, 0)
            t_fill = time.time() - tf
            del c
        dist.barrier()
    g = GIDS.GIDS(page_size=page, off=0, cache_dim=dim, num_ele=num_ele, num_ssd=cfg["ssds"],
                  ssd_list=list(range(cfg["ssds"])), cache_size=cfg["cache_mb"], ctrl_idx=dist.local,
                  dtype=TDTYPE[dt], ssd_capacity=per_ssd if phys < range_bytes else 0, ssd_path=pattern,
                  synchronous=False, shard_cache=shared and not args.no_shard, window_buffer=cfg["wb"] > 0,
                  wb_size=max(1, cfg["wb"]), cache_line=cfg["line"] or None,
                  heterograph=cfg["hetero"] is not None, heterograph_map=hmap,
                  cache_admission=POLICIES[args.policy][0], cache_ref_max=POLICIES[args.policy][1],
                  gather_blocks=args.gather_blocks, wb_prefetch=args.wb_prefetch and cfg["wb"] > 0,
                  replicas=replica_reservation(args, cfg, shared and not args.no_shard))
    t_store = time.time() - t0
    if not shared:
        t0 = time.time()
        g.BAM_FS.fill_synthetic(KIND[dt], 1, 0)
        t_fill = time.time() - t0
    geo = g.BAM_FS.geometry()
    line = geo.get("cache_line", page)
    log(f"[rank {dist.rank}] store ready: {geo} (alloc {t_store:.1f}s, fill {t_fill:.1f}s)")

    wb = cfg["wb"]
    # each timed loop consumes `steps` batches; window buffering reads wb batches ahead
    n_batches = args.warmup + 2 * (args.steps + wb)
    batches, pins, t_sample = make_batches(cfg, n_batches, dist.rank, device, with_pins=True)

    def nrows(b):
        return sum(int(v.numel()) for v in b.values()) if isinstance(b, dict) else int(b.numel())

    def pin(b):
        return {k: v.cpu().pin_memory() for k, v in b.items()} if isinstance(b, dict) else b.cpu().pin_memory()

    sizes = [nrows(b) for b in batches]
    log(f"[rank {dist.rank}] sampled {n_batches} minibatches in {t_sample:.1f}s, input nodes mean "
        f"{np.mean(sizes):.0f}")
    if pins is not None:
        g.cpu_backing_buffer(dim, int(pins.numel()))
        g.set_cpu_buffer(pins, int(pins.numel()))
        log(f"[rank {dist.rank}] constant CPU buffer: {pins.numel()} pinned rows (PageRank top "
            f"{cfg['cpu_pin_frac']:.0%})")
    # link peaks, measured before the static hot set (the replica choice uses them) and reused by the roofline
    host_peak = host_link_peak_gbs(device, dist)
    nvlink_peak = None
    if g.world > 1:
        # every rank copies 1 GiB from the next rank's shard at the same time
        dist.barrier()
        nvlink_peak = g.BAM_FS.peer_copy_gbs((dist.rank + 1) % g.world, 1 << 30)
        dist.barrier()
    n_static = 0
    n_replicated = 0
    t_static = 0.0
    if args.policy == "static":
        # the static hot set: the rows neighbour sampling reaches most often (highest out-degree), as many
        # as the cache's lines hold (every rank's shard when sharded), pinned and filled in once
        from GIDS.sampler import hot_rows, out_degree, top_rows

        t0 = time.time()
        lpr = -(-row_bytes // line) + (0 if row_bytes % line == 0 else 1)
        k = geo["cache_slots"] * g.world // lpr
        if cfg["hetero"]:
            # a node's out-degree summed over the relations it is a source of, in global ids
            # (the types laid out one after another, heterograph_map)
            from GIDS.synthetic import HeteroSyntheticGraph

            h = cfg["hetero"]
            hg = HeteroSyntheticGraph(h["types"], h["relations"], cfg["mean_deg"], cfg["alpha"], seed=0,
                                      device=device)
            counts = torch.zeros(cfg["nodes"], dtype=torch.int32, device=device)
            for (src, dst), rg in hg.rel.items():
                _, ind = rg.materialize(torch.int32, n_dst=h["types"][dst])
                lo = hmap[src]
                counts[lo:lo + h["types"][src]] += out_degree(ind, h["types"][src])
                del ind
            hot = top_rows(counts, k)
            del hg, counts
        else:
            _, indices = graph_csc(cfg, device)
            hot = hot_rows(indices, cfg["nodes"], k)
        if g.world > 1:
            # replicated rows (the hottest R, held by every rank) take R of each rank's slots; the next
            # W x (slots - R) rows are sharded by page id, each rank pinning the rows its shard owns
            n_replicated = 0 if cfg["hetero"] else choose_replicas(args, cfg, g, hot, device, dist, lpr,
                                                                   nvlink_peak, host_peak)
            per_rank = geo["cache_slots"] // lpr
            rest = hot[n_replicated:n_replicated + g.world * (per_rank - n_replicated)]
            rest = rest[((rest * row_bytes) // line) % g.world == g.rank]
            if n_replicated:
                g.replicate_rows(hot[:n_replicated])  # flushes this rank's shard
            dist.barrier()  # no rank gathers from a shard another rank is still flushing
            hot = torch.cat([hot[:n_replicated], rest])
        g.pin_cache(hot)  # global row ids (heterograph: no type offset)
        n_static = int(dist.sum(hot.numel()))
        del hot
        torch.cuda.synchronize()
        t_static = time.time() - t0
        log(f"[rank {dist.rank}] static hot set: {n_static} rows of highest out-degree pinned in {t_static:.1f}s")
    host_batches = [pin(b) for b in batches]
    stream = torch.cuda.current_stream(device)
    bam = g.BAM_FS
    # generators: a batch list (and the features appended to it) lives only until the step ends
    dev_it = ([b] for b in batches[:args.warmup + args.steps + wb])

    # cache warm-up: minibatches from other sampler seeds, untimed, so that the
    # timed steps see the page cache of a job that has been training for a while
    # (admission fills the cache with lines that recur, which takes several
    # cache-sizes of line references); then the W warm-up steps
    refs_per_batch = float(np.mean(sizes)) * -(-row_bytes // line)
    n_cw = args.cache_warmup
    if n_cw < 0:
        n_cw = int(min(60, math.ceil(CACHE_WARMUP_CACHES * geo["cache_slots"] / max(1.0, refs_per_batch))))
    t0 = time.time()
    wbf = g.window_buffering_flag
    g.window_buffering_flag = False  # the warm-up leaves no window pins behind
    done, k = 0, 0
    while done < n_cw:
        m = min(8, n_cw - done)
        k += 1
        wbatches, _ = make_batches(cfg, m, dist.rank + 7919 * k, device)
        wit = ([b] for b in wbatches)
        for _ in range(m):
            g.fetch_feature(dim, wit, device)
        done += m
        del wbatches, wit
    torch.cuda.synchronize()
    g.window_buffering_flag = wbf
    t_cw = time.time() - t0
    log(f"[rank {dist.rank}] cache warm-up: {n_cw} minibatches in {t_cw:.1f}s")
    last = None
    for i in range(args.warmup):
        last = g.fetch_feature(dim, dev_it, device)  # held like the timed loop's last step
    # the caching allocator of a job that has been training holds blocks for its largest
    # minibatch: two outputs of the largest timed minibatch (the timed loop holds the last
    # step's features while the next step allocates), so no timed step waits on cudaMalloc
    big = max(nrows(b) for b in batches[args.warmup:])
    spare = [torch.empty((big, dim), dtype=TDTYPE[dt], device=device) for _ in range(2)]
    del spare
    torch.cuda.synchronize()
    bam.reset_stats()

    hbm_peak, hbm_src = measured_hbm_peak()
    # the link at the cache's own access size: random line reads from the emulated SSDs
    line_b = int(geo.get("cache_line", page))
    host_rand = bam.host_read_gbs(min(line_b, 4096), 4 << 30)

    # ---- timed region 1: node ids resident in HBM
    clocks = ClockSampler(dist.local)
    clocks.start()
    dev_ids = batches[args.warmup:args.warmup + args.steps]
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("gids_timed_value")
    ev0.record(stream)
    for _ in dev_ids:
        last = g.fetch_feature(dim, dev_it, device)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    dist.barrier()
    t_val = ev0.elapsed_time(ev1) / 1e3
    clk = clocks.stop()
    st = bam.get_stats()
    k_ms = bam.kernel_time_ms()
    launches = st["launches"]
    rows_val = st["rows"]
    # bit-exact spot check of the last timed minibatch (ids in HBM) against the oracle
    parity = [parity_check(cfg, last[0], last[-1], hmap, args.parity_rows, seed=dist.rank)]
    del last

    # ---- timed region 2: end to end through GIDS.fetch_feature, ids in pinned host memory
    g.drop_window_buffer()  # a fresh iterator starts a fresh window; the old one's marks are taken back
    first = args.warmup + args.steps + wb
    e2e_batches = host_batches[first:first + args.steps]
    it = ([b] for b in host_batches[first:])
    if wb:  # the window of a fresh epoch is filled before the timed steps
        g.fill_wb(it, wb)
        g.wb_init = True
    torch.cuda.synchronize()
    bam.reset_stats()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    torch.cuda.nvtx.range_push("gids_timed_e2e")
    e0.record(stream)
    checks = 0.0
    for i in range(len(e2e_batches)):
        batch = g.fetch_feature(dim, it, device)
        feat = batch[-1]
        if isinstance(feat, dict):
            feat = feat[max(feat, key=lambda k: feat[k].shape[0])]
        checks += float(feat[-1, -1].item())  # D2H read of the step's result
        del feat  # the step is done with its features, as a training step would be
        if i + 1 < len(e2e_batches):
            del batch
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - w0
    dist.barrier()
    t_e2e = e0.elapsed_time(e1) / 1e3
    st_e2e = bam.get_stats()
    rows_e2e = st_e2e["rows"]
    # and of the last end-to-end minibatch (ids from pinned host memory)
    parity.append(parity_check(cfg, batch[0], batch[-1], hmap, args.parity_rows, seed=100 + dist.rank))
    del batch

    # ---- loader: the sampler on a side stream overlapped with the gather, fresh
    #      minibatches (other sampler seeds); wall time with the device idle at both ends
    loader = None
    if not args.no_loader:
        side = torch.cuda.Stream(device)
        sample_ms = time_sampler(cfg, args.steps, dist.rank + 3571, device, side)
        g.drop_window_buffer()
        lit = SideStreamBatches(batch_stream(cfg, args.steps + wb, dist.rank + 3571, device), side, stream)
        if wb:
            g.fill_wb(lit, wb)
            g.wb_init = True
        torch.cuda.synchronize()
        bam.reset_stats()
        dist.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(args.steps):
            g.fetch_feature(dim, lit, device)
        torch.cuda.synchronize()
        t_loader = time.perf_counter() - w0
        dist.barrier()
        st_l = bam.get_stats()
        t_loader_max = dist.max(t_loader)
        loader = {"minibatches_per_s": round(dist.sum(args.steps) / t_loader_max, 3),
                  "gathered_gbs": round(dist.sum(st_l["rows"]) * row_bytes / 1e9 / t_loader_max, 3),
                  "sampler_ms_per_minibatch": round(sample_ms, 2),
                  "gather_ms_per_minibatch": None,
                  "note": "wall time of fetch_feature over a lazy sampler whose neighbour sampling runs on a "
                          "second CUDA stream while the previous minibatch's gather runs"}

    # ---- aggregate over ranks
    rank_ms = [round(x / max(1, len(dev_ids)) * 1e3, 3) for x in dist.gather(t_val)]
    t_val_max = dist.max(t_val)
    t_e2e_max = dist.max(t_e2e)
    rows_val_all = dist.sum(rows_val)
    rows_e2e_all = dist.sum(rows_e2e)
    steps_all = dist.sum(len(dev_ids))

    # ---- mixed roofline of the gather kernel (per launch averages, this rank)
    n_launch = max(1, launches)
    t_launch = k_ms / 1e3 / n_launch
    rows_l = st["rows"] / n_launch
    # host bytes: rows read through or filled by the gathers, constant-CPU-buffer rows, and the
    # lines window-buffer prefetch launches read into the cache
    r_host = (st["bytes_miss"] + st["bytes_bypass"] + st["bytes_cpu"] + st.get("prefetched", 0) * line) / n_launch
    r_hbm_src = st["bytes_hit"] / n_launch
    alg_hbm = r_hbm_src + rows_l * row_bytes + 8 * rows_l  # source reads of hits + output writes + ids
    r_peer = st.get("bytes_peer", 0) / n_launch  # hit bytes read from other ranks' shards over NVLink
    terms = {"hbm": (alg_hbm, hbm_peak), "host_link": (r_host, host_peak)}
    if nvlink_peak:
        terms["nvlink"] = (r_peer, nvlink_peak)
    bound = max(terms, key=lambda k: terms[k][0] / terms[k][1])
    t_star = terms[bound][0] / (terms[bound][1] * 1e9)
    achieved, peak, unit_peak = terms[bound][0] / t_launch / 1e9, terms[bound][1], "GB/s"
    acc = max(1, st["access"])
    roofline = {
        "bound": bound, "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": unit_peak,
        "frac": round(t_star / t_launch, 4),
        "traffic": (int(TRAFFIC_PER_ROW[(args.config, args.policy)] * rows_l)
                    if (args.config, args.policy) in TRAFFIC_PER_ROW and not args.nodes and dist.world == 1 else None),
        "peak_source": {"hbm": hbm_src + " (of measured)",
                        "host_link": "pinned host->device copy measured live in this run, all ranks copying at "
                                     "once (of measured)",
                        "nvlink": "device-to-device copy of 1 GiB from the next rank's shard, all ranks copying "
                                  "at once, measured live in this run (of measured)"}[bound],
        "model": "T* = max((R*(n_hit + n) + 8n)/BW_hbm, R*(n_cpu + n_miss + n_bypass)/BW_host, R*n_peer/BW_nvlink); "
                 "frac = T*/T_launch",
        "t_launch_ms": round(t_launch * 1e3, 3), "t_star_ms": round(t_star * 1e3, 3),
        "nvlink": {"alg_bytes_per_launch": int(r_peer), "achieved_gbs": round(r_peer / t_launch / 1e9, 1),
                   "peak_gbs": round(nvlink_peak, 1),
                   "peak_method": "cudaMemcpyAsync of 1 GiB from rank+1's shard, every rank at once, best of 3"}
        if nvlink_peak else None,
        "hbm": {"alg_bytes_per_launch": int(alg_hbm), "achieved_gbs": round(alg_hbm / t_launch / 1e9, 1),
                "peak_gbs": hbm_peak},
        "host_link": {"alg_bytes_per_launch": int(r_host), "achieved_gbs": round(r_host / t_launch / 1e9, 2),
                      "peak_gbs": round(host_peak, 2),
                      "random_read_gbs": round(host_rand, 2),
                      "random_read_method": f"random {min(line_b, 4096)}-byte reads from the start of cache lines of "
                                            "the emulated SSDs, 4 GiB, best of 3 (gids_store_host_read_gbs)",
                      "frac_of_random_read": round(r_host / t_launch / 1e9 / host_rand, 4) if host_rand else None},
        "mix": {"hit": round(st["hit"] / acc, 4), "miss": round(st["miss"] / acc, 4),
                "bypass": round(st["bypass"] / acc, 4), "cpu_rows": st["cpu_rows"],
                "peer_bytes_frac": round(st.get("bytes_peer", 0) / max(1, st["rows"] * row_bytes), 4)},
        "counters_per_launch": {k: round(st.get(k, 0) / n_launch, 1)
                                for k in ("access", "hit", "miss", "read_io", "bypass", "wait_timeouts", "evictions")},
        # only a library built with GIDS_PHASE_TIMERS=1 counts these (share of warp time per phase)
        "phase_share": ({k: round(st[k] / max(1, sum(st.get(x, 0) for x in PHASES)), 4) for k in PHASES}
                        if sum(st.get(x, 0) for x in PHASES) else None),
    }
    gb_val = rows_val_all * row_bytes / 1e9
    value = gb_val / t_val_max
    if loader is not None:
        loader["gather_ms_per_minibatch"] = round(t_val_max / len(dev_ids) * 1e3, 2)
    e2e_value = rows_e2e_all * row_bytes / 1e9 / t_e2e_max
    result = {
        "metric": METRIC,
        "value": round(value, 3), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t_val_max / len(dev_ids) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": {"float32": "f32", "float16": "f16"}[dt],
        "data": DATA,
        "minibatches_per_s": round(steps_all / t_val_max, 3),
        "config": workload_config(args, cfg, dist.world),
        "settings": {"trainers": f"{dist.world} independent data-parallel trainers" +
                                 (", page cache sharded by page id over NVLink" if g.world > 1 else ""),
                     "wrap_pages": geo["wrap_pages"],
                     "bytes_per_step_min": int(min(sizes) * row_bytes),
                     "input_nodes_per_step": round(rows_val / max(1, len(dev_ids)), 1),
                     "constant_cpu_buffer_rows": int(pins.numel()) if pins is not None else 0,
                     "window_buffer_depth": wb,
                     "cache_policy": args.policy,
                     "static_hot_rows": n_static or None,
                     "replicated_rows": n_replicated or None,
                     "cache_warmup_minibatches": n_cw,
                     "rank_ms_per_step": rank_ms,
                     "gather_grid_cap": args.gather_blocks or None,
                     "window_buffer_prefetch": bool(args.wb_prefetch and cfg["wb"] > 0)},
        "parity": {"rows_checked": int(dist.sum(sum(p["rows_checked"] for p in parity))),
                   "ok": bool(dist.sum(0.0 if all(p["ok"] for p in parity) else 1.0) == 0.0),
                   "against": "oracle.gather_synth: the reference's gather restated over the same synthetic "
                              "table (bit-exact)",
                   "minibatches": "the last timed step (ids in HBM) and the last e2e step (ids from host), "
                                  "every rank"},
        "roofline": roofline,
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "api": "GIDS.fetch_feature",
                "h2d_bytes_per_step": int(np.mean([nrows(b) * 8 for b in e2e_batches])),
                "d2h_bytes_per_step": esize, "wall_s": round(wall_e2e, 3),
                "minibatches_per_s": round(dist.sum(len(e2e_batches)) / t_e2e_max, 3),
                "mix": {"hit": round(st_e2e["hit"] / max(1, st_e2e["access"]), 4)}},
        "loader": loader,
        "gpu_launches": int(launches) + (len(dev_ids) if wb else 0),
        "clocks": clk,
        "setup_s": {"store": round(t_store, 1), "fill": round(t_fill, 1), "sampling": round(t_sample, 1),
                    "static_hot_set": round(t_static, 1),
                    "cache_warmup": round(t_cw, 1)},
    }
    torch.cuda.synchronize()
    g.close()
    return result, batches


def backing_geometry(cfg):
    """(logical range bytes, bytes the emulated SSDs physically hold, wrap period
    in elements or 0): the SSDs hold phys_gb of pages and logical page p is
    stored where page p mod (their page count) is."""
    esize, page = ESIZE[cfg["dtype"]], cfg["page"]
    range_bytes = cfg["nodes"] * cfg["dim"] * esize
    phys = min(int(cfg["phys_gb"] * 1e9), range_bytes)
    if phys >= range_bytes:
        return range_bytes, range_bytes, 0
    per_ssd = (phys // cfg["ssds"]) // page * page
    wrap_pages = per_ssd // page * cfg["ssds"]
    return range_bytes, wrap_pages * page, wrap_pages * page // esize


def workload_config(args, cfg, world: int) -> dict:
    """The JSON line's `config`, identical in both arms: what is gathered, not how."""
    logical, physical, _ = backing_geometry(cfg)
    return {"workload": workload_name(args, cfg),
            "global_batch": cfg["batch"] * world,
            "parallelism": f"dp{world}",
            "backing_store": {"logical_bytes": logical, "physical_bytes": physical},
            "node_ids": "seeded synthetic graph + counter-hashed neighbour sampler: both arms gather the same "
                        "minibatches",
            "l2": "no flush: every step gathers millions of rows (GBs), far larger than the 126 MB L2"}


def workload_name(args, cfg) -> str:
    """The workload as both arms name it in their JSON line."""
    dt, dim, page = cfg["dtype"], cfg["dim"], cfg["page"]
    range_gb = cfg["nodes"] * dim * ESIZE[dt] / 1e9
    return (f"{args.config}: {cfg['nodes']} nodes, {dt} x {dim} ({range_gb:.1f} GB range), {page} B pages over "
            f"{cfg['ssds']} emulated SSDs, {cfg['cache_mb'] // 1024} GB cache/GPU in {cfg['line'] or page} B lines, "
            f"fanout {cfg['fanouts']}, batch {cfg['batch']}")


def run_reference(args, cfg, dist: Dist):
    """The reference's CPU implementation of the path -- the mmap baseline
    gather -- on the host cores, over the same minibatches as our arm (the
    sampler is drawn on the CPU; its counter-hashed choices make the node ids
    identical to the GPU arm's). Nothing of the product is loaded: the
    synthetic graph and sampler are plain torch, and the gather runs through
    the oracle's restatement of the reference idiom."""
    if dist.rank != 0:
        return None
    n = args.warmup + args.steps
    t0 = time.time()
    batches, _ = make_batches(cfg, n, 0, "cpu")
    t_sample = time.time() - t0
    dt, dim = cfg["dtype"], cfg["dim"]
    # each step is one whole minibatch gathered by torch.index_select from the memmap
    res = cpu_mmap_gather(cfg, batches[args.warmup:], 1e9, file_gb=args.cpu_file_gb,
                          warmup_ids=batches[:args.warmup])
    cold = cpu_mmap_gather_cold(cfg, batches[args.warmup]) if not args.no_cold else None
    v = res["value"]
    return {
        "impl": "reference", "metric": METRIC,
        "value": round(v, 3), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(res["seconds"] / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {"float32": "f32", "float16": "f16"}[dt], "data": DATA,
        "minibatches_per_s": round(res["minibatches_per_s"], 3),
        "config": workload_config(args, cfg, dist.world),
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": res["cores"], "kind": "port",
                         "sample": res["sample"],
                         **{k: res[k] for k in ("h2d_gbs", "with_h2d_gbs", "h2d_note") if k in res},
                         "cold_page_cache": cold},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": {"sampling_cpu": round(t_sample, 1), "memmap_fill": res["fill_s"]},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--phys-gb", type=float, default=0.0, help="GB of pages the emulated SSDs hold (0: the config's)")
    ap.add_argument("--cpu-file-gb", type=float, default=0.0,
                    help="size of the CPU-baseline memmap (0: the bytes the emulated SSDs hold, <= 40%% of RAM)")
    ap.add_argument("--no-cold", action="store_true", help="reference arm: skip the cold-page-cache sample")
    ap.add_argument("--parity-rows", type=int, default=4096,
                    help="gathered rows per checked minibatch compared bit for bit with the oracle")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--nodes", type=int, default=0, help="override the node count (small profiling cases)")
    ap.add_argument("--cache-mb", type=int, default=0, help="override the cache size")
    ap.add_argument("--batch", type=int, default=0, help="override the seed batch size (small profiling cases)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--no-shard", action="store_true", help="N>1: independent caches instead of one sharded cache")
    ap.add_argument("--cache-line", type=int, default=-1, help="cache line bytes (0 = the page; -1 = the config's)")
    ap.add_argument("--no-loader", action="store_true", help="skip the loader (sampler overlapped) measurement")
    ap.add_argument("--shared-backing", action="store_true",
                    help="back the emulated SSDs with shared /dev/shm files even on one GPU (as N>1 runs do)")
    ap.add_argument("--gather-blocks", type=int, default=0, help="cap on the gather kernel's grid (0: all resident)")
    ap.add_argument("--replicate", default="auto",
                    help="N>1, static policy: rows every rank holds locally besides its shard -- 'off', 'auto' "
                         "(the count the link model favours) or a row count")
    ap.add_argument("--wb-prefetch", action="store_true",
                    help="window-buffered configs: fetch each batch's lines into the cache as it enters the window")
    ap.add_argument("--cache-warmup", type=int, default=-1,
                    help="untimed minibatches (other sampler seeds) gathered before the warm-up steps; -1: "
                         "enough for about 12 cache-sizes of line references, at most 60")
    ap.add_argument("--torch-sampler", action="store_true",
                    help="draw minibatches with the torch sampler instead of the CUDA sampler (same ids)")
    ap.add_argument("--policy", default="", choices=[""] + sorted(POLICIES),
                    help="cache replacement (default: the config's): admit2 = insert on the second miss + 2-bit "
                         "clock; clock = insert "
                         "every miss + second-chance clock (the reference's insertion rule); static = the cache "
                         "holds the rows of highest out-degree, pinned, and reads every other row through")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3")
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.nodes:
        cfg["nodes"] = args.nodes
    if args.cache_mb:
        cfg["cache_mb"] = args.cache_mb
    if args.batch:
        cfg["batch"] = args.batch
    if args.phys_gb:
        cfg["phys_gb"] = args.phys_gb
    if args.cache_line >= 0:
        cfg["line"] = args.cache_line
    cfg["torch_sampler"] = args.torch_sampler
    if not args.policy:
        args.policy = cfg["policy"]

    dist = Dist()
    if args.impl == "reference":
        dist.init("gloo")
        res = run_reference(args, cfg, dist)
        if res is not None:
            print(json.dumps(res), flush=True)
        dist.close()
        return

    dist.init("nccl", torch.device("cuda", dist.local))
    exit_code = 0
    try:
        res, batches = run_ours(args, cfg, dist)
        if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_mmap_gather(cfg, batches, args.cpu_seconds, file_gb=args.cpu_file_gb)
        if dist.rank == 0:
            print(json.dumps(res), flush=True)
        dist.barrier()
        if not res["parity"]["ok"]:
            log(f"[rank {dist.rank}] PARITY FAILURE: gathered rows differ from the oracle: {res['parity']}")
            exit_code = 1
    finally:
        if (dist.world > 1 or args.shared_backing) and dist.rank == 0:  # the shared emulated SSD files
            import glob

            for f in glob.glob(f"/dev/shm/gids_b200_bench_{os.environ.get('MASTER_PORT', 'x')}_ssd*"):
                os.unlink(f)
        dist.close()
    if exit_code:
        sys.exit(exit_code)


if __name__ == "__main__":
    main()
