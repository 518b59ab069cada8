"""GIDS Python API on the B200 feature store.

Drop-in for GIDS_Setup/GIDS/GIDS.py of the reference: the ``GIDS`` class keeps
its constructor keywords, its methods and the semantics of ``fetch_feature``
(window buffering, Storage Access Accumulator, heterograph key offsets), and
``GIDS_DGLDataLoader`` keeps its signature. Feature gathers run in the CUDA
library behind the ``BAM_Feature_Store`` module; nothing here touches feature
data on the CPU.

Differences from the reference, all of which leave the gathered values
unchanged:
* the output tensor has the store's element type (the reference always
  allocates float32, GIDS.py:908,961,1017,1046, which is wrong for
  ``long_type``) and is allocated with ``torch.empty`` (every element is
  written by the gather);
* gathers are stream-ordered on the current torch stream instead of ending in
  a device-wide synchronize (pass ``synchronous=True`` for the old behaviour);
* the store lives on ``cuda:ctrl_idx`` (the reference hard-wires device 0,
  bam_nvme.h:135,293);
* a heterograph type with an empty id list is skipped (the reference's
  ``next`` there is a no-op, GIDS.py:717-719).
"""
from __future__ import annotations

import math
import time

import torch

# feature element type -> BAM_Feature_Store class name
_STORE_CLASSES = {
    torch.float32: "BAM_Feature_Store_float",
    torch.int64: "BAM_Feature_Store_long",
    torch.float16: "BAM_Feature_Store_half",
    torch.bfloat16: "BAM_Feature_Store_bfloat16",
}


def _feature_store_module():
    """The compiled BAM_Feature_Store module, imported on first use so that
    importing this package maps no library (ImportError if it is not built:
    there is no CPU fallback)."""
    import BAM_Feature_Store

    return BAM_Feature_Store


def _admission_mode(v) -> int:
    """cache_admission -> the store's admission mode (0 every miss, 1 second miss, 2 pinned rows only)."""
    if isinstance(v, str):
        if v != "static":
            raise ValueError(f"cache_admission must be True, False or 'static', not {v!r}")
        return 2
    return 1 if v else 0


def _current_stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _as_index(v, device) -> torch.Tensor:
    t = v if isinstance(v, torch.Tensor) else torch.as_tensor(v)
    if t.dtype != torch.int64:
        t = t.to(torch.int64)
    return t.to(device, non_blocking=True).contiguous()


def _with_features(batch, feat):
    """Append the gathered features to a sampler batch (GIDS.py:1029-1034, 1053-1058)."""
    if isinstance(batch, tuple):
        return (*batch, feat)
    batch.append(feat)
    return batch


class GIDS:
    """Feature fetcher over the GPU page cache (GIDS.py:490-1128).

    Constructor keywords and defaults follow GIDS.py:510-517. Keyword-only
    extensions: ``dtype`` (feature element type; default float32, int64 with
    ``long_type``), ``ssd_capacity`` (bytes held per emulated SSD, 0 = the
    whole stripe; smaller values wrap), ``ssd_path`` (file pattern such as
    ``/dev/shm/gids_ssd{}`` for emulated SSDs shared across processes),
    ``synchronous``, and ``shard_cache``: with torch.distributed initialised
    (one process per GPU), the ranks' page caches form one cache sharded by
    page id (page p lives on rank p % world) and hits on other ranks' pages
    are read over NVLink. Every rank must construct its GIDS collectively
    with the same geometry, and call ``close()`` collectively. ``cache_line``
    (bytes, a power of two in [512, page_size]; default the page) sets the
    unit the GPU cache holds and fetches, so that rows much smaller than a
    page do not pull whole pages over the host link. ``cache_admission``
    (default True) inserts a line on its second miss within a window of twice
    the cache's slots, so lines touched once do not evict lines touched often;
    False inserts every miss (the reference's rule); ``"static"`` makes the
    cache hold only the rows pinned with ``pin_cache`` (a hot set chosen from
    the graph, for example by ``GIDS.sampler.hot_rows``) and read every other
    row through;
    ``cache_ref_max`` (default 3) is the clock counter ceiling (1 = the
    second-chance clock). Neither changes what is gathered. ``gather_blocks``
    caps the gather kernel's grid (0: every block the GPU holds at once), so a
    gather bound by the host link leaves SMs to kernels on other streams.
    ``replicas`` (with ``shard_cache``; default 0) reserves room in every
    shard for that many replicated cache lines: ``replicate_rows`` then makes
    rows held by every rank in its own shard (their hits are local instead of
    NVLink reads), while the other rows stay sharded by page id.
    ``wb_prefetch`` (with ``window_buffer``; default False) also fetches into
    the cache, as each batch enters the window, the lines of it that its
    gather would insert (a prefetch launch on the current stream that copies
    nothing out), so that the gather, ``wb_size`` batches later, finds them
    resident; the reference's window buffering only protects marked pages
    from eviction.
    """

    def __init__(self, page_size=4096, off=0, cache_dim=1024, num_ele=300 * 1000 * 1000 * 1024, num_ssd=1,
                 ssd_list=None, cache_size=10, ctrl_idx=0, window_buffer=False, wb_size=8, accumulator_flag=False,
                 long_type=False, heterograph=False, heterograph_map=None, *, dtype=None, ssd_capacity=0,
                 ssd_path=None, synchronous=False, shard_cache=False, process_group=None, cache_line=None,
                 cache_admission=True, cache_ref_max=3, gather_blocks=0, wb_prefetch=False, replicas=0):
        if dtype is None:
            dtype = torch.int64 if long_type else torch.float32
        if dtype not in _STORE_CLASSES:
            raise ValueError(f"unsupported feature dtype {dtype}")
        self.dtype = dtype
        BAM_Feature_Store = _feature_store_module()
        self.BAM_FS = getattr(BAM_Feature_Store, _STORE_CLASSES[dtype])()

        self.accumulator_flag = accumulator_flag
        self.required_accesses = 0
        self.prev_cpu_access = 0
        self.return_torch_buffer = []
        self.index_list = []

        self.window_buffering_flag = window_buffer
        self.window_buffer = []
        self.wb_init = False
        self.wb_size = wb_size
        self.wb_prefetch = wb_prefetch
        self._wb_dim = cache_dim  # columns the gathers read: the prefetch fetches those rows' lines

        self.page_size = page_size
        # byte offset -> first page on every SSD (GIDS.py:583)
        self.off = math.ceil(math.ceil(off / page_size) / num_ssd)
        self.num_ele = num_ele
        self.cache_size = cache_size
        self.heterograph = heterograph
        self.heterograph_map = heterograph_map
        self.graph_GIDS = None
        self.cache_dim = cache_dim
        self.gids_device = "cuda:" + str(ctrl_idx)
        self.device = torch.device(self.gids_device)

        self.GIDS_controller = BAM_Feature_Store.GIDS_Controllers()
        if ssd_list is None:
            print("SSD are not assigned")
            self.ssd_list = [i for i in range(num_ssd)]
        else:
            self.ssd_list = ssd_list
        print("ssd list: ", ssd_list)
        self.GIDS_controller.init_GIDS_controllers(num_ssd, 1024, 128, self.ssd_list)
        if ssd_capacity or ssd_path:
            self.GIDS_controller.set_emulation(int(ssd_capacity or 0), ssd_path or "")

        self.BAM_FS.set_device(ctrl_idx)
        if cache_line:
            self.BAM_FS.set_cache_line(int(cache_line))
        self._pg = None
        self.world, self.rank = 1, 0
        if shard_cache:
            import torch.distributed as dist

            if dist.is_available() and dist.is_initialized():
                self._pg = process_group
                self.world = dist.get_world_size(process_group)
                self.rank = dist.get_rank(process_group)
            if self.world > 1:
                self.BAM_FS.set_sharding(self.world, self.rank)
                if replicas:
                    self.BAM_FS.set_replicas(int(replicas))
        self.cache_line = int(cache_line or page_size)
        self.BAM_FS.init_controllers(self.GIDS_controller, page_size, self.off, cache_size, num_ele, num_ssd)
        if self.world > 1:
            self._attach_peer_shards()
        self.BAM_FS.set_row_layout(cache_dim)
        self.BAM_FS.set_cache_policy(_admission_mode(cache_admission), int(cache_ref_max))
        if gather_blocks:
            self.BAM_FS.set_gather_blocks(int(gather_blocks))
        self.BAM_FS.set_synchronous(bool(synchronous))
        self.synchronous = bool(synchronous)

        self.GIDS_time = 0.0
        self.WB_time = 0.0

    def _attach_peer_shards(self):
        """Exchange the shards' CUDA IPC handles and map every peer's shard."""
        import torch.distributed as dist

        mine = (self.BAM_FS.ipc_handle(), int(self.BAM_FS.geometry().get("shard_bytes", 0)))
        got = [None] * self.world
        dist.all_gather_object(got, mine, group=self._pg)
        # a peer's shard is addressed by this rank's layout: the ranks' shards must be alike
        if len({b for _, b in got}) != 1:
            raise RuntimeError(f"sharded cache: the ranks' shards differ in size ({[b for _, b in got]}); "
                               "every rank needs the same geometry, cache line and replicas")
        self.BAM_FS.open_peers([h for h, _ in got])
        dist.barrier(group=self._pg)

    def close(self):
        """Release the store. With a sharded cache this is collective: no rank
        frees its shard while another may still read it."""
        if getattr(self, "BAM_FS", None) is None:
            return
        self.BAM_FS.synchronize()
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self._pg)
        self.BAM_FS = None

    # ------------------------------------------------------------ out of scope
    def init_graph_GIDS(self, page_size, off, cache_size, num_ele, num_ssd):
        """Graph-structure-on-SSD sampling (GIDS.py:636-650) is not implemented."""
        raise NotImplementedError("graph-structure sampling from storage is not part of this library")

    def get_offset_array(self):
        raise NotImplementedError("graph-structure sampling from storage is not part of this library")

    def get_array_ptr(self):
        raise NotImplementedError("graph-structure sampling from storage is not part of this library")

    # ------------------------------------------------------ constant CPU buffer
    def cpu_backing_buffer(self, dim, length):
        """Allocate the pinned constant CPU buffer (GIDS.py:667-678)."""
        self.BAM_FS.cpu_backing_buffer(dim, length)

    def set_cpu_buffer(self, ten, N):
        """Pin the first N node ids of ``ten`` (a pin_file list, GIDS.py:680-699)."""
        topk_ten = torch.as_tensor(ten)[:N]
        topk_len = len(topk_ten)
        d_ten = topk_ten.to(torch.int64).to(self.device).contiguous()
        self.BAM_FS.set_cpu_buffer(d_ten.data_ptr(), topk_len)

    # ------------------------------------------------------- window buffering
    def window_buffering(self, batch):
        """Protect the pages of an upcoming batch from eviction (GIDS.py:702-748)."""
        s_time = time.time()
        stream = _current_stream_handle(self.device)
        if self.heterograph:
            for key, value in batch[0].items():
                if len(value) == 0:
                    continue
                input_tensor = _as_index(value, self.device)
                key_off = 0
                if self.heterograph_map is not None:
                    if key in self.heterograph_map:
                        key_off = self.heterograph_map[key]
                    else:
                        print("Cannot find key: ", key, " in the heterograph map!")
                self.BAM_FS.set_window_buffering(input_tensor.data_ptr(), len(input_tensor), int(key_off), stream)
                self._prefetch(input_tensor, int(key_off), stream)
        else:
            input_tensor = _as_index(batch[0], self.device)
            self.BAM_FS.set_window_buffering(input_tensor.data_ptr(), len(input_tensor), 0, stream)
            self._prefetch(input_tensor, 0, stream)
        self.WB_time += time.time() - s_time

    def _prefetch(self, ids, key_off, stream):
        """Window-buffer prefetch (extension): bring the lines of rows ``ids`` into the cache."""
        if self.wb_prefetch and len(ids):
            self.BAM_FS.prefetch(ids.data_ptr(), len(ids), self._wb_dim, self.cache_dim, key_off, stream)

    def fill_wb(self, it, num):
        """Pull ``num`` batches ahead and mark them (GIDS.py:752-769)."""
        for _ in range(num):
            batch = next(it)
            self.window_buffer.append(batch)
            self.window_buffering(batch)

    def drop_window_buffer(self):
        """Abandon the queued window (extension): the marks of every batch still
        in it are taken back, so its pages no longer resist eviction, and the
        next ``fetch_feature`` refills the window from its own iterator. The
        reference has no counterpart; its marks of an abandoned window stay."""
        if self.window_buffering_flag:
            stream = _current_stream_handle(self.device)
            # the accumulator has already gathered (and unpinned) the first
            # len(return_torch_buffer) batches of the window
            for batch in self.window_buffer[len(self.return_torch_buffer):]:
                for key, value in self._batch_ids(batch):
                    if len(value) == 0:
                        continue
                    t = _as_index(value, self.device)
                    self.BAM_FS.unset_window_buffering(t.data_ptr(), len(t), key, stream)
        self.window_buffer.clear()
        self.return_torch_buffer.clear()
        self.wb_init = False

    def _batch_ids(self, batch):
        """(key offset, ids) of every node type of a batch."""
        if self.heterograph:
            return [(self._key_off(k), v) for k, v in batch[0].items()]
        return [(0, batch[0])]

    # ---------------------------------------------------------- replicated rows
    def _row_lines(self, node_ids, key=None):
        """Cache lines touched by rows ``node_ids`` (of type ``key``), sorted, unique (int64 CPU)."""
        ids = torch.as_tensor(node_ids).to(torch.int64).cpu() + (self._key_off(key) if key is not None else 0)
        esize = torch.empty(0, dtype=self.dtype).element_size()
        stride = self.cache_dim * esize
        first = (ids * stride) // self.cache_line
        last = (ids * stride + stride - 1) // self.cache_line
        span = int((last - first).max()) + 1 if len(ids) else 1
        lines = torch.cat([first + k for k in range(span)]) if len(ids) else first
        if span > 1:
            lines = lines[lines <= torch.cat([last] * span)]
        return torch.unique(lines)

    def replicate_rows(self, node_ids, key=None):
        """Make the cache lines of rows ``node_ids`` replicated (extension): every
        rank holds them in its own shard, so their hits read local HBM instead
        of a peer's over NVLink; every other line stays sharded by page id.
        Collective in effect: every rank replicates the same rows, and no rank
        gathers until all have (a barrier), since it flushes this rank's shard
        (call it before ``pin_cache``).
        At most ``replicas`` lines (the constructor's reservation)."""
        if self.world <= 1:
            raise RuntimeError("replicated rows need a sharded cache (shard_cache=True on several ranks)")
        lines = self._row_lines(node_ids, key).contiguous()
        self.BAM_FS.set_replicated_lines(lines.data_ptr(), len(lines))
        return len(lines)

    # ---------------------------------------------------------- static hot set
    def pin_cache(self, node_ids, key=None, prefill=True, chunk_rows=1 << 18):
        """Pin the GPU-cache lines of rows ``node_ids`` (of node type ``key`` in
        a heterograph) for good (extension): they are inserted on their first
        miss and never evicted; with ``cache_admission="static"`` they are the
        only rows the cache holds. ``prefill`` gathers them once so that they
        are resident before the next minibatch. Pin at most as many lines as
        the cache has slots; ``flush_cache`` drops the pins."""
        ids = _as_index(node_ids, self.device)
        key_off = self._key_off(key) if key is not None else 0
        stream = _current_stream_handle(self.device)
        self.BAM_FS.pin_rows(ids.data_ptr(), len(ids), key_off, stream)
        if prefill and len(ids):
            n = min(chunk_rows, len(ids))
            scratch = torch.empty((n, self.cache_dim), dtype=self.dtype, device=self.device)
            for lo in range(0, len(ids), chunk_rows):
                part = ids[lo:lo + chunk_rows]
                self.BAM_FS.read_feature(scratch.data_ptr(), part.data_ptr(), len(part), self.cache_dim,
                                         self.cache_dim, key_off, stream)
            torch.cuda.current_stream(self.device).synchronize()
            del scratch

    def unpin_cache(self, node_ids, key=None):
        """Clear the permanent pins of rows ``node_ids`` (extension)."""
        ids = _as_index(node_ids, self.device)
        key_off = self._key_off(key) if key is not None else 0
        self.BAM_FS.unpin_rows(ids.data_ptr(), len(ids), key_off, _current_stream_handle(self.device))

    # ----------------------------------------------- storage access accumulator
    def set_required_storage_access(self, bw, l_ssd, l_system, num_ssd, p):
        """Accesses needed to keep the SSDs at fraction p of peak (GIDS.py:773-788)."""
        accesses = (p * bw * 1024 / self.page_size * (l_ssd + l_system) * num_ssd) / (1 - p)
        self.required_accesses = accesses
        print("Number of required storage accesses: ", accesses)

    # ------------------------------------------------------------ the gather
    def _new_out(self, n, dim):
        return torch.empty((n, dim), dtype=self.dtype, device=self.device)

    def _key_off(self, key):
        if self.heterograph_map is not None:
            if key in self.heterograph_map:
                return int(self.heterograph_map[key])
            print("Cannot find key: ", key, " in the heterograph map!")
        return 0

    def fetch_feature(self, dim, it, device):
        """Next batch from ``it`` with its gathered features appended (GIDS.py:791-1058)."""
        GIDS_time_start = time.time()
        stream = _current_stream_handle(self.device)
        self._wb_dim = dim

        if self.window_buffering_flag and not self.wb_init:
            self.fill_wb(it, self.wb_size)
            self.wb_init = True

        next_batch = next(it)
        self.window_buffer.append(next_batch)
        if self.window_buffering_flag:
            self.window_buffering(next_batch)

        if self.accumulator_flag:
            return self._fetch_accumulated(dim, it, stream, GIDS_time_start)

        batch = self.window_buffer.pop(0)
        if self.heterograph:
            ret_ten, outs, idxs, ns, keys = {}, [], [], [], []
            for key, v in batch[0].items():
                if len(v) == 0:
                    ret_ten[key] = self._new_out(0, dim)
                    continue
                g_index = _as_index(v, self.device)
                out = self._new_out(len(g_index), dim)
                ret_ten[key] = out
                outs.append(out.data_ptr())
                idxs.append(g_index.data_ptr())
                ns.append(len(g_index))
                keys.append(self._key_off(key))
            self.BAM_FS.read_feature_hetero(len(outs), outs, idxs, ns, dim, self.cache_dim, keys, stream)
            self.GIDS_time += time.time() - GIDS_time_start
            return _with_features(batch, ret_ten)

        index = _as_index(batch[0], self.device)
        out = self._new_out(len(index), dim)
        self.BAM_FS.read_feature(out.data_ptr(), index.data_ptr(), len(index), dim, self.cache_dim, 0, stream)
        self.GIDS_time += time.time() - GIDS_time_start
        return _with_features(batch, out)

    def _fetch_accumulated(self, dim, it, stream, t0):
        """Storage Access Accumulator (GIDS.py:836-984): gather enough queued
        batches in one launch to keep the storage busy, hand them out one per call."""
        if len(self.return_torch_buffer) != 0:
            return_ten = self.return_torch_buffer.pop(0)
            return_batch = self.window_buffer.pop(0)
            self.GIDS_time += time.time() - t0
            return _with_features(return_batch, return_ten)

        def n_access(b):
            if self.heterograph:
                return sum(len(v) for v in b[0].values())
            return len(b[0])

        buffer_size = len(self.window_buffer)
        current_access = 0
        num_iter = 0
        required_accesses = self.required_accesses
        while True:
            if num_iter >= buffer_size:
                batch = next(it)
                self.window_buffer.append(batch)
                if self.window_buffering_flag:
                    self.window_buffering(batch)
            else:
                batch = self.window_buffer[num_iter]
            current_access += n_access(batch)
            num_iter += 1
            required_accesses += self.prev_cpu_access
            if current_access > required_accesses:
                break

        outs, idxs, ns, keys = [], [], [], []
        keep_alive = []
        for i in range(num_iter):
            batch = self.window_buffer[i]
            if self.heterograph:
                ret_ten = {}
                for k, v in batch[0].items():
                    if len(v) == 0:
                        ret_ten[k] = self._new_out(0, dim)
                        continue
                    g_index = _as_index(v, self.device)
                    keep_alive.append(g_index)
                    out = self._new_out(len(g_index), dim)
                    ret_ten[k] = out
                    outs.append(out.data_ptr())
                    idxs.append(g_index.data_ptr())
                    ns.append(len(g_index))
                    keys.append(self._key_off(k))
                self.return_torch_buffer.append(ret_ten)
            else:
                g_index = _as_index(batch[0], self.device)
                keep_alive.append(g_index)
                out = self._new_out(len(g_index), dim)
                outs.append(out.data_ptr())
                idxs.append(g_index.data_ptr())
                ns.append(len(g_index))
                keys.append(0)
                self.return_torch_buffer.append(out)
        if self.heterograph:
            self.BAM_FS.read_feature_merged_hetero(len(outs), outs, idxs, ns, dim, self.cache_dim, keys, stream)
        else:
            self.BAM_FS.read_feature_merged(len(outs), outs, idxs, ns, dim, self.cache_dim, stream)
        del keep_alive  # stream-ordered: safe to release once the launch is queued

        return_ten = self.return_torch_buffer.pop(0)
        return_b = self.window_buffer.pop(0)
        self.GIDS_time += time.time() - t0
        cpu_access_count = self.BAM_FS.get_cpu_access_count()
        self.prev_cpu_access = int(cpu_access_count / num_iter)
        self.BAM_FS.flush_cpu_access_count()
        return _with_features(return_b, return_ten)

    # ---------------------------------------------------------------- stats
    def print_stats(self):
        """Print and reset timers and cache counters (GIDS.py:1062-1080)."""
        print("GIDS time: ", self.GIDS_time)
        print("WB time: ", self.WB_time)
        self.WB_time = 0.0
        self.GIDS_time = 0.0
        self.BAM_FS.print_stats()

    def get_stats(self):
        """Cumulative cache counters as a dict (extension)."""
        return self.BAM_FS.get_stats()

    # --------------------------------------------------------- backing store
    def store_tensor(self, in_ten, offset):
        """Write rows to the backing store (GIDS.py:1083-1093 -> gids_nvme.cu:616-663)."""
        t = in_ten.contiguous()
        self.BAM_FS.store_tensor(t.data_ptr(), len(t), offset)

    def store_mmap_tensor(self, in_ten, offset):
        """Same from a numpy (memmap) array (GIDS.py:1095-1116)."""
        import numpy as np

        y = np.ascontiguousarray(in_ten)
        self.BAM_FS.store_tensor(y.ctypes.data, len(y), offset)

    def read_tensor(self, num, offset):
        """Print ``num`` elements from element ``offset`` (GIDS.py:1118-1122)."""
        self.BAM_FS.read_tensor(num, offset)

    def flush_cache(self):
        """Drop resident pages (GIDS.py:1124-1128)."""
        self.BAM_FS.flush_cache()


# --------------------------------------------------------------------- loader
class _PrefetchingIter:
    """Iterator that appends gathered features to each sampled batch (GIDS.py:204-258)."""

    def __init__(self, dataloader, dataloader_it, GIDS_Loader=None):
        self.dataloader_it = dataloader_it
        self.dataloader = dataloader
        self.graph_sampler = getattr(dataloader, "graph_sampler", None)
        self.GIDS_Loader = GIDS_Loader

    def __iter__(self):
        return self

    def __next__(self):
        return self.GIDS_Loader.fetch_feature(self.dataloader.dim, self.dataloader_it, self.GIDS_Loader.gids_device)


def GIDS_DGLDataLoader(graph, indices, graph_sampler, batch_size, dim, GIDS, device=None, use_ddp=False,
                       ddp_seed=0, drop_last=False, shuffle=False, use_alternate_streams=None, **kwargs):
    """DGL DataLoader whose iterator appends GIDS-gathered features
    (GIDS.py:262-488). Needs dgl; it is imported here, so the rest of the
    package works without it."""
    from ._dgl_loader import make_dgl_loader

    return make_dgl_loader(graph, indices, graph_sampler, batch_size, dim, GIDS, device=device, use_ddp=use_ddp,
                           ddp_seed=ddp_seed, drop_last=drop_last, shuffle=shuffle,
                           use_alternate_streams=use_alternate_streams, **kwargs)
