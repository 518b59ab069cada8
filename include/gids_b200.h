/*
 * gids_b200.h -- C ABI of the B200 GIDS feature-gather library (libgids_b200.so).
 *
 * The reference exposes this path to Python through the pybind11 module
 * BAM_Feature_Store (gids_module/gids_nvme.cu:823-893), whose methods take raw
 * uint64 device addresses. Every entry point below replaces one of those
 * methods (or the host code behind it) and is cited next to its declaration.
 * All entry points:
 *   - take plain pointers and sizes (no torch or pybind types);
 *   - return GIDS_OK (0) or a negative GIDS_E* code, with a message readable
 *     through gids_last_error() on the calling thread;
 *   - never abort the process.
 * Streams are passed as `void*` holding a cudaStream_t (NULL = legacy default
 * stream). Gathers are asynchronous on that stream unless the store is in
 * synchronous mode (gids_store_set_synchronous), which is the default and
 * matches the reference: the output is complete when the call returns.
 *
 * Element types: the store copies rows as bytes; elem_bytes is 2 (fp16/bf16),
 * 4 (fp32, the reference's BAM_Feature_Store_float) or 8 (int64, the
 * reference's BAM_Feature_Store_long).
 */
#ifndef GIDS_B200_H
#define GIDS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GIDS_API __attribute__((visibility("default")))
#else
#define GIDS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ error codes */
#define GIDS_OK 0
#define GIDS_E_INVAL (-1)      /* bad argument (null pointer, size, alignment) */
#define GIDS_E_CUDA (-2)       /* a CUDA runtime call failed */
#define GIDS_E_NOMEM (-3)      /* host or device allocation failed */
#define GIDS_E_STATE (-4)      /* call out of order (e.g. gather before init) */
#define GIDS_E_RANGE (-5)      /* a node id addressed a row outside the store */
#define GIDS_E_IO (-6)         /* emulated-SSD file could not be opened/mapped */
#define GIDS_E_UNSUPPORTED (-7)

#define GIDS_MAX_SSD 32
#define GIDS_MAX_TUPLES 64

typedef struct gids_ctrls gids_ctrls_t; /* emulated SSD controllers */
typedef struct gids_store gids_store_t; /* one feature store (cache + CPU buffer) */

/* Message of the last failed call on this thread (empty if none). Returns the
 * message length. */
GIDS_API int gids_last_error(char *buf, size_t len);
GIDS_API const char *gids_strerror(int code);
/* Library version string and the compiled GPU architecture. */
GIDS_API const char *gids_version(void);
/* The calling thread's current CUDA device (the reference hard-wires device
 * 0, bam_nvme.h:135,293; a store here lives on the device it is created on). */
GIDS_API int gids_current_device(int *out);

/* --------------------------------------------------------- controllers --
 * Replaces GIDS_Controllers::init_GIDS_controllers (gids_nvme.cu:93-107),
 * which opens /dev/libnvm{ssd_list[i]} for i < n_ctrls with the given queue
 * depth and queue count. Here each entry of ssd_list names an emulated SSD: a
 * page-addressed region of host memory that the GPU reads zero-copy. q_depth
 * and n_queues are recorded (there is no NVMe queue to size).
 * If path_pattern is non-empty (gids_ctrls_set_emulation) the SSD of id k is
 * the file path_pattern with "{}" replaced by k, mapped shared, so that its
 * contents persist across processes like a device; otherwise it is anonymous
 * memory owned by the process. */
GIDS_API int gids_ctrls_create(gids_ctrls_t **out);
GIDS_API int gids_ctrls_init(gids_ctrls_t *c, uint32_t n_ctrls, uint64_t q_depth, uint64_t n_queues, const int32_t *ssd_list);
/* Emulation knobs (no reference counterpart; the reference's SSDs are real
 * devices): capacity_bytes_per_ssd = 0 sizes each SSD to hold its stripe of
 * the range; a smaller capacity makes the SSD wrap (logical page p is stored
 * where page p mod (n_ctrls * data_pages_per_ssd) is). */
GIDS_API int gids_ctrls_set_emulation(gids_ctrls_t *c, uint64_t capacity_bytes_per_ssd, const char *path_pattern);
GIDS_API int gids_ctrls_destroy(gids_ctrls_t *c);
/* Backing-store access without a GPU cache (no reference counterpart; the
 * reference writes its SSDs with tensor_write.py / nvm-readwrite_stripe-bench):
 * bind sizes and maps the first num_ssd SSDs for a range of range_bytes with
 * the given page size and first page read_off_pages (what
 * gids_store_init_controllers does; a later store with the same geometry
 * reuses the binding); write/read move host bytes through the stripe map;
 * fill_synthetic writes the synthetic stream of gids_fill_synthetic. No GPU
 * is needed until a store uses the controllers. */
GIDS_API int gids_ctrls_bind(gids_ctrls_t *c, uint32_t num_ssd, uint32_t page_size, uint64_t read_off_pages,
                             uint64_t range_bytes);
GIDS_API int gids_ctrls_write(gids_ctrls_t *c, const void *src, uint64_t nbytes, uint64_t offset_bytes);
GIDS_API int gids_ctrls_read(gids_ctrls_t *c, void *dst, uint64_t nbytes, uint64_t offset_bytes);
GIDS_API int gids_ctrls_fill_synthetic(gids_ctrls_t *c, int kind, uint64_t seed, int threads);
/* [0]=pages in the range, [1]=pages physically held, [2]=bytes per SSD, [3]=SSDs bound */
GIDS_API int gids_ctrls_geometry(gids_ctrls_t *c, uint64_t *out, int count);

/* --------------------------------------------------------------- store --
 * Replaces BAM_Feature_Store<T>'s default constructor (gids_nvme.cu:812-815,
 * pybind :830/:857) plus init_controllers (gids_nvme.cu:166-221):
 *   page_size      bytes per cache page / SSD page (power of two, >= 512)
 *   read_off_pages first page of the range on every SSD (GIDS.py:583 passes
 *                  ceil(ceil(off / page_size) / num_ssd))
 *   cache_size_mb  GPU page-cache size in MiB (n_slots = MiB * 2^20 / page_size)
 *   num_ele        elements in the range (bounds of every gather)
 *   num_ssd        SSDs the range is striped over (first num_ssd of ssd_list) */
GIDS_API int gids_store_create(gids_store_t **out, uint32_t elem_bytes, int device);
GIDS_API int gids_store_init_controllers(gids_store_t *s, gids_ctrls_t *c, uint32_t page_size, uint64_t read_off_pages,
                                uint64_t cache_size_mb, uint64_t num_ele, uint64_t num_ssd);
GIDS_API int gids_store_destroy(gids_store_t *s);
/* 1 (default) = every gather synchronizes its stream before returning, like
 * the reference (gids_nvme.cu:335,348); 0 = stream-ordered, asynchronous. */
GIDS_API int gids_store_set_synchronous(gids_store_t *s, int synchronous);
/* Cache line (no reference counterpart; the reference caches whole pages):
 * the unit of the GPU cache's page table, slots and fills, a power of two in
 * [512, page_size] (0 = the page, the default). The stripe layout of the
 * backing store keeps page_size. Smaller lines keep rows much smaller than a
 * page from pulling whole pages over the host link. Call before
 * gids_store_init_controllers. */
GIDS_API int gids_store_set_cache_line(gids_store_t *s, uint32_t bytes);
/* Replacement policy (no reference counterpart; the reference inserts every
 * missed page and evicts with a clock that has no reference bits,
 * page_cache_backup.h:2107-2256). admission = 1 (default): a line is inserted
 * on its second miss within a window of 2 x (cache slots) line references;
 * its first miss reads the backing store directly, so lines touched once do
 * not evict lines touched often. admission = 0: every miss is inserted (the
 * reference's rule). admission = 2 (static cache): only lines with a
 * permanent pin (gids_store_pin_rows) are inserted, on their first reference,
 * and every other line is read through -- a cache that holds a chosen hot set
 * (for example the rows of highest out-degree, gids_out_degree). ref_max
 * (default 3): a hit adds a chance up to ref_max and the clock hand spends one
 * per pass (1 = second chance). Results do not depend on the policy; only hit
 * ratios do. */
GIDS_API int gids_store_set_cache_policy(gids_store_t *s, int admission, uint32_t ref_max);
/* Largest grid of one gather launch, in blocks of 256 threads (no reference
 * counterpart). 0 (default): every block the GPU can hold at once (2 per SM).
 * A gather bound by the host link keeps the link busy with fewer blocks and
 * leaves SMs to kernels on other streams (a sampler, the training step). */
GIDS_API int gids_store_set_gather_blocks(gids_store_t *s, uint32_t max_blocks);
/* Bounded waits (no reference counterpart; the reference spins forever,
 * page_cache_backup.h:1389-1401): a gather polls a line that another warp or
 * GPU is filling at most `polls` times (exponential back-off, 32 ns to 2 us),
 * then reads the line from the backing store instead and counts a
 * GIDS_STAT_WAIT_TIMEOUT. Default 65536 polls. */
GIDS_API int gids_store_set_wait_limit(gids_store_t *s, uint32_t polls);
/* Failure injection for tests: marks cache line `line` as being filled by a
 * filler that never finishes (BUSY, no slot). The next gathers that need the
 * line wait for it up to the wait limit, then bypass the cache. The store
 * must be idle; the line must belong to the calling rank's shard. */
GIDS_API int gids_store_debug_mark_busy(gids_store_t *s, uint64_t line);
/* Source row stride (elements) used to fill the constant CPU buffer before
 * the first gather tells it (the reference assumes one row per page,
 * gids_nvme.cu:173,704). */
GIDS_API int gids_store_set_row_layout(gids_store_t *s, uint32_t cache_dim);

/* ------------------------------------------------------ sharded cache --
 * No reference counterpart (the reference caches on one GPU). W stores, one
 * per GPU, share one page cache: page p is owned by rank p % W, whose HBM
 * holds its page-table entry and, when resident, its data; every GPU looks
 * pages up in the owner's shard and reads hits over NVLink, and a miss fills
 * the owner's slot. Call gids_store_set_sharding before
 * gids_store_init_controllers (all ranks with the same geometry), then either
 *   - one process per GPU: exchange the 64-byte gids_store_ipc_handle of
 *     every rank (e.g. an all-gather) and call gids_store_open_peers on
 *     each rank with the handles in rank order; or
 *   - one process for all GPUs: gids_store_share_shards(stores, W).
 * Gathers fail with GIDS_E_STATE until the peers are attached. A rank's
 * shard must outlive every gather of every rank (destroy after a barrier);
 * flush_cache and writes drop only the calling rank's shard. */
GIDS_API int gids_store_set_sharding(gids_store_t *s, int world, int rank);
/* Replicated lines (no reference counterpart): in a sharded cache, lines
 * that every rank holds in its own shard instead of only their owner's, so
 * that hits on them are local rather than NVLink reads. set_replicas reserves
 * page-table entries for up to max_lines of them (before init_controllers,
 * the same on every rank; < 2^32). set_replicated_lines makes `lines` (a host
 * array of cache-line ids, strictly increasing, at most max_lines) the
 * replicated set of the calling rank and flushes that rank's shard; every rank
 * must set the same lines before gathering. Pins (gids_store_pin_rows) of a
 * replicated line pin this rank's copy. */
GIDS_API int gids_store_set_replicas(gids_store_t *s, uint64_t max_lines);
GIDS_API int gids_store_set_replicated_lines(gids_store_t *s, const uint64_t *lines, uint64_t n);
GIDS_API int gids_store_ipc_handle(gids_store_t *s, void *out, size_t len);
GIDS_API int gids_store_open_peers(gids_store_t *s, const void *handles, int world);
GIDS_API int gids_store_share_shards(gids_store_t *const *stores, int n);
/* Link bandwidth of an attached sharded cache (no reference counterpart; a
 * measurement aid): copies `bytes` (rounded down to 4 KB, at most one shard)
 * from rank `peer`'s shard into this GPU with cudaMemcpyAsync and returns the
 * best of three timed copies in GB/s. Run it on every rank at once for the
 * bandwidth a rank gets while the others also use their links. */
GIDS_API int gids_store_peer_copy_gbs(gids_store_t *s, int peer, uint64_t bytes, double *out);
/* Host-link bandwidth at the gather's own access size (no reference
 * counterpart; a measurement aid): total_bytes of random reads of read_bytes
 * (512, 1024, 2048 or 4096, at most one cache line) from the start of cache
 * lines of the bound backing store, eight 16-byte loads in flight per lane as
 * in the gather; returns the best of three launches in GB/s. Small random
 * host reads reach less than a bulk copy; this is their ceiling. */
GIDS_API int gids_store_host_read_gbs(gids_store_t *s, uint32_t read_bytes, uint64_t total_bytes, double *out);

/* -------------------------------------------------------------- gathers --
 * gids_read_feature replaces BAM_Feature_Store<T>::read_feature
 * (gids_nvme.cu:324-364; kernels gids_kernel.cu:60-86 and :111-175):
 *   out[i*dim + t] = range[(idx[i] + key_off) * cache_dim + t], t < dim,
 * for i < n. `out` and `idx` are device pointers on the store's GPU; idx is
 * int64. Rows pinned in the constant CPU buffer are read from it. A node id
 * whose row leaves the range gives GIDS_E_RANGE and a zero row. GIDS_E_CUDA
 * with "TMA bulk copy ... wait limit" reports a bulk load of cached lines that
 * did not complete in time; the rows were then copied another way and are
 * complete. */
GIDS_API int gids_read_feature(gids_store_t *s, void *out, const int64_t *idx, int64_t n, int dim, int cache_dim,
                      uint64_t key_off, void *stream);
/* Replaces read_feature_hetero / read_feature_merged_hetero
 * (gids_nvme.cu:382-445, :531-593) and, with key_offs == NULL,
 * read_feature_merged (:456-518): k (out, idx, n, key_off) tuples gathered by
 * ONE launch (the reference creates k streams and k launches). */
GIDS_API int gids_read_feature_multi(gids_store_t *s, int k, void *const *outs, const int64_t *const *idxs,
                            const uint64_t *ns, int dim, int cache_dim, const uint64_t *key_offs, void *stream);

/* No counterpart in the reference. The same gather as gids_read_feature, for
 * callers that cannot allocate GPU memory -- for example a process whose
 * device memory belongs to another allocator with a hard budget (a serving
 * runtime, or a framework caching allocator that reserved the GPU), where a
 * cudaMalloc fails or takes memory promised elsewhere. It allocates nothing:
 * the page cache its kernel uses (page table, slots, counters) lives in a
 * 32 MiB static device array, held on each GPU until the process exits; the
 * store's own cache is neither read nor written. The store must already be
 * initialised (by a caller that could allocate).
 * CUDA loads the array lazily: the first call on a device makes the 32 MiB
 * resident (and looks its address up), so make that call early, before the
 * other allocator reserves the device, and before any stream capture; later
 * calls leave the device's free memory unchanged.
 * Each call starts from an empty cache (it clears the page table, tags and
 * counters on its stream), so pages shared by rows of one call are fetched
 * once and nothing carries over between calls. Its rows, hits and misses are
 * added to the store's counters (gids_get_stats, gids_get_cpu_access_count).
 * All calls on a device share the array: calls that overlap on the GPU race.
 * A store whose range needs more than about 4M pages of page table gets
 * GIDS_E_RANGE. */
GIDS_API int gids_read_feature_noalloc(gids_store_t *s, void *out, const int64_t *idx, int64_t n, int dim,
                                       int cache_dim, uint64_t key_off, void *stream);

/* ---------------------------------------------------- window buffering --
 * Replaces set_window_buffering (gids_nvme.cu:242-249; kernel
 * gids_kernel.cu:246-256): marks the pages of the rows (idx[i] + hash_off)
 * of an upcoming minibatch so that they are not evicted before that
 * minibatch is gathered. Rows map to pages by bytes (the reference treats a
 * node id as a page id). row_stride_elems = 0 uses the store's row layout. */
GIDS_API int gids_set_window_buffering(gids_store_t *s, const int64_t *idx, int64_t n, int64_t hash_off,
                              uint32_t row_stride_elems, void *stream);
/* Takes back the marks gids_set_window_buffering made for the same rows (one
 * pin per row and page, saturating at 0): call it for a marked minibatch that
 * will not be gathered (an abandoned window), whose pins would otherwise keep
 * its pages from being evicted for good. No reference counterpart: the
 * reference never releases a window it does not gather
 * (page_cache_backup.h:1185-1195, 1265-1272). flush_cache and the writers drop
 * every pin of the calling rank's shard. */
GIDS_API int gids_unset_window_buffering(gids_store_t *s, const int64_t *idx, int64_t n, int64_t hash_off,
                                         uint32_t row_stride_elems, void *stream);
/* Window-buffer prefetch (no reference counterpart: the reference's window
 * buffering only protects marked pages from eviction,
 * page_cache_backup.h:1265-1272). The gather of gids_read_feature for rows
 * (idx[i] + key_off), dim / cache_dim as there, without an output: the rows'
 * cache lines are looked up, and every missing line that the gather would
 * insert is read from the backing store into a slot now, so a later gather of
 * the rows finds it resident. The rule is the gather's: every line while the
 * cache fills; once it is full, lines pinned for a later batch (more window
 * pins than this call's references) or missed before in the admission window;
 * with admission = 2, permanently pinned lines. The prefetch sets no admission
 * bit, and lines the gather would read through are left to it, so the cache
 * ends up holding what it would hold without the prefetch. Nothing is copied out, no
 * window-buffer pin is consumed (call it after gids_set_window_buffering for
 * the same rows, so the lines stay until their gather), bad ids and rows of
 * the constant CPU buffer are skipped. Stream-ordered on `stream`; lines it
 * inserts count in GIDS_STAT_PREFETCHED and GIDS_STAT_READ_IO, nothing else. */
GIDS_API int gids_prefetch(gids_store_t *s, const int64_t *idx, int64_t n, int dim, int cache_dim, uint64_t key_off,
                           void *stream);
/* Permanent pins (no reference counterpart; the reference keeps its hot set
 * in the constant CPU buffer instead, gids_cpu_backing_buffer): the cache
 * lines of rows (idx[i] + hash_off) (device int64 array; rows map to lines by
 * bytes as above) are never evicted once resident and are inserted on their
 * first miss whatever the admission rule; with admission = 2 they are the only
 * lines the cache holds. Pin at most as many lines as the cache has slots
 * (with a sharded cache, per owning shard); lines beyond that are read
 * through. unpin clears the pins; flush_cache clears every pin of the shard.
 * Gathering the pinned rows once fills them in. */
GIDS_API int gids_store_pin_rows(gids_store_t *s, const int64_t *idx, int64_t n, int64_t hash_off,
                                 uint32_t row_stride_elems, void *stream);
GIDS_API int gids_store_unpin_rows(gids_store_t *s, const int64_t *idx, int64_t n, int64_t hash_off,
                                   uint32_t row_stride_elems, void *stream);

/* --------------------------------------------------- constant CPU buffer --
 * cpu_backing_buffer (gids_nvme.cu:123-139): allocate a pinned, GPU-mapped
 * host buffer of len rows x dim elements. Until set_cpu_buffer is called,
 * rows [0, len) are the pinned set (the reference's seq mode,
 * gids_kernel.cu:132-141). */
GIDS_API int gids_cpu_backing_buffer(gids_store_t *s, uint64_t dim, uint64_t len);
/* set_cpu_buffer (gids_nvme.cu:694-711; kernels gids_kernel.cu:191-228):
 * pin the rows named by the first num entries of the int64 device array idx
 * (a pin_file prefix) and fill the buffer from the backing store. */
GIDS_API int gids_set_cpu_buffer(gids_store_t *s, const int64_t *idx, int num);
/* Same, with a host array (no reference counterpart; used by host callers). */
GIDS_API int gids_set_cpu_buffer_host(gids_store_t *s, const int64_t *idx, int64_t num);

/* ---------------------------------------------------------- statistics --
 * get_cpu_access_count / flush_cpu_access_count (gids_nvme.cu:779-794) and
 * the page-cache counters printed by print_stats (gids_nvme.cu:261-300,
 * page_cache_backup.h:974-977, 2046-2073). */
GIDS_API int gids_get_cpu_access_count(gids_store_t *s, uint32_t *out);
GIDS_API int gids_flush_cpu_access_count(gids_store_t *s);

#define GIDS_STAT_ACCESS 0       /* page references (reference access_cnt) */
#define GIDS_STAT_HIT 1          /* page references served by a resident page */
#define GIDS_STAT_MISS 2         /* page references that waited for a fill */
#define GIDS_STAT_READ_IO 3      /* pages filled from the backing store */
#define GIDS_STAT_BYPASS 4       /* page references read straight from the backing store */
#define GIDS_STAT_CPU_ROWS 5     /* rows served by the constant CPU buffer */
#define GIDS_STAT_ROWS 6         /* rows gathered */
#define GIDS_STAT_WAIT_TIMEOUT 7 /* bounded waits that gave up (then bypassed) */
#define GIDS_STAT_BAD_IDS 8      /* node ids outside the range (zero rows) */
#define GIDS_STAT_BYTES_HIT 9    /* output bytes copied from resident pages */
#define GIDS_STAT_BYTES_MISS 10  /* output bytes copied from pages filled in this call */
#define GIDS_STAT_BYTES_BYPASS 11
#define GIDS_STAT_BYTES_CPU 12
#define GIDS_STAT_EVICTIONS 13
#define GIDS_STAT_LAUNCHES 14    /* gather kernels launched */
#define GIDS_STAT_BYTES_PEER 15  /* output bytes copied from another GPU's shard (NVLink) */
/* Per-phase time of the gather, summed over warps in nanoseconds: lookup,
 * fills and waits, copy, release. Counted only by a library built with
 * GIDS_PHASE_TIMERS=1 (a diagnosis build); 0 otherwise. */
#define GIDS_STAT_NS_LOOKUP 16
#define GIDS_STAT_NS_FILL 17
#define GIDS_STAT_NS_COPY 18
#define GIDS_STAT_NS_RELEASE 19
#define GIDS_STAT_PREFETCHED 20  /* lines inserted by gids_prefetch (also counted in READ_IO) */
#define GIDS_STAT_COUNT 21
/* Copies the cumulative counters (synchronizes the store's last stream). */
GIDS_API int gids_get_stats(gids_store_t *s, uint64_t *out, int count);
GIDS_API int gids_reset_stats(gids_store_t *s);
/* print_stats (gids_nvme.cu:279-300): prints and resets the counters and the
 * accumulated gather time. */
GIDS_API int gids_print_stats(gids_store_t *s);
/* Accumulated device time of gathers since the last print/reset, in ms. */
GIDS_API int gids_get_kernel_time_ms(gids_store_t *s, double *out);
GIDS_API int gids_store_synchronize(gids_store_t *s);

/* ------------------------------------------------------- backing store --
 * store_tensor (gids_nvme.cu:616-663; kernel gids_kernel.cu:378-389): row r
 * < num_rows of the range, one page of elements (page_size / elem_bytes) per
 * row as in the reference (gids_nvme.cu:173), receives the elements that
 * start offset_bytes / elem_bytes elements into `src` (device or host
 * pointer) -- the reference applies the offset to the source and always
 * writes from element 0 of the range. The write goes through the stripe map
 * to the emulated SSDs; resident copies are then dropped so that gathers see
 * the new data (the reference flushes its dirty pages, flush_cache,
 * gids_nvme.cu:673-677). */
GIDS_API int gids_store_tensor(gids_store_t *s, const void *src, uint64_t num_rows, uint64_t offset_bytes);
/* General striped writer: nbytes from src (device or host pointer) to the
 * range at byte offset_bytes; resident copies are dropped. No reference
 * counterpart (the reference writes whole pages from row 0 only). */
GIDS_API int gids_write_range(gids_store_t *s, const void *src, uint64_t nbytes, uint64_t offset_bytes);
/* flush_cache (gids_nvme.cu:673-677): the cache holds no dirty pages here,
 * so this drops every resident page and every window-buffer pin (of the
 * calling rank's shard when the cache is sharded). */
GIDS_API int gids_flush_cache(gids_store_t *s);
/* Host-side read of the range through the stripe map (no reference
 * counterpart; the reference's read_tensor prints elements from a GPU
 * thread, gids_nvme.cu:764-770). */
GIDS_API int gids_read_range_host(gids_store_t *s, void *dst, uint64_t nbytes, uint64_t offset_bytes);
/* Fill the whole backing store with the synthetic feature stream `kind`
 * (1 = fp32 uniform[-1,1), 2 = fp16 byte-sum, 3 = int64 raw, 4 = fp16
 * normal(0,1) by Box-Muller) of `seed`:
 * element e of the range holds element (e mod wrap) of the stream, where
 * wrap covers the pages the SSDs physically hold. Uses `threads` host threads
 * (0 = all). No reference counterpart: the reference's SSDs are filled by
 * tensor_write.py / nvm-readwrite_stripe-bench before training. */
GIDS_API int gids_fill_synthetic(gids_store_t *s, int kind, uint64_t seed, int threads);
/* Geometry of the bound backing store: [0]=pages in the range, [1]=pages
 * physically held (wrap period), [2]=bytes per SSD, [3]=cache slots,
 * [4]=page size, [5]=number of SSDs, [6]=cache line size, [7]=bytes of this
 * store's cache allocation on its GPU (page table, slots and their metadata:
 * one allocation, a whole number of 2 MB pages). */
GIDS_API int gids_store_geometry(gids_store_t *s, uint64_t *out, int count);

/* ------------------------------------------------------------- sampler --
 * The minibatches fed to fetch_feature: replaces the DGL
 * MultiLayerNeighborSampler that feeds the reference's loader
 * (GIDS_Setup/GIDS/GIDS.py:178-201, evaluation/homogenous_train.py:201-203)
 * with a GPU sampler over a CSC graph held on the sampler's GPU: indptr is
 * int64 [num_nodes + 1], indices int32 or int64 (index_bytes 4 or 8) [edges];
 * in-edges of v are indices[indptr[v] .. indptr[v+1]). Both arrays must
 * outlive the sampler. fanouts[0..n_layers) as in DGL (fanouts[0] is the
 * layer nearest the input; hops run from the last fanout to the first), each
 * in [1, 32]. Each hop keeps, for every node of the current set, the
 * min(fanout, in-degree) in-edges of smallest counter-hashed key (a function
 * of seed, call index, hop, node and edge index), and appends the new sources
 * in order of first appearance; the result (seeds first, duplicates removed)
 * is the minibatch's input_nodes, bit-identical to the torch restatement in
 * GIDS/synthetic.py on any device. max_seeds bounds the seeds of one call.
 * gids_sampler_capacity: the output capacity a call needs (nodes).
 * gids_sampler_sample: runs on `stream` without a host synchronisation;
 * count_dev (device uint64, may be NULL) receives the node count; count_host
 * (may be NULL) makes the call wait and return it there. call < 0 uses the
 * sampler's own call counter (0, 1, 2, ...); a seed outside the graph gives
 * GIDS_E_RANGE (with count_host). */
typedef struct gids_sampler gids_sampler_t;
GIDS_API int gids_sampler_create(gids_sampler_t **out, int device, const int64_t *indptr, const void *indices,
                                 int index_bytes, uint64_t num_nodes, const int *fanouts, int n_layers,
                                 uint64_t max_seeds, uint64_t seed);
GIDS_API int gids_sampler_capacity(gids_sampler_t *s, uint64_t *out);
GIDS_API int gids_sampler_sample(gids_sampler_t *s, const int64_t *seeds, uint64_t n_seeds, int64_t *out_nodes,
                                 uint64_t out_cap, uint64_t *count_dev, uint64_t *count_host, int64_t call,
                                 void *stream);
GIDS_API int gids_sampler_destroy(gids_sampler_t *s);

/* The pin list of the constant CPU buffer: compute_pagerank of
 * evaluation/page_rank_node_list_gen.py:126-134 on the GPU, in float32 --
 * pv = 1/N; `iters` times: pv = pv / in_degree; pv[v] = sum of pv[u] over the
 * in-edges u -> v (in CSC order, one float32 add at a time); pv = (1-d)/N +
 * d * pv -- into pv[num_nodes] (device). Nodes without in-edges contribute 0
 * (the reference divides by zero there). With order_keys (device uint64
 * [num_nodes], may be NULL), also writes one key per node whose ascending
 * order is pv descending, node id ascending: the pin_file is the node ids
 * (key & 0xffffffff) of the k smallest keys (page_rank_node_list_gen.py:282-285
 * takes torch.topk of pv). */
GIDS_API int gids_pagerank(int device, const int64_t *indptr, const void *indices, int index_bytes, uint64_t num_nodes,
                           int iters, double damping, float *pv, uint64_t *order_keys, void *stream);

/* Out-degree of every node of a CSC graph (no reference counterpart; the rank
 * of a static hot set for gids_store_pin_rows): counts[v] (device uint32
 * [num_nodes]) = the number of in-edges whose source is v, i.e. how often
 * neighbour sampling can reach v. Waits for `stream`; a source outside the
 * graph gives GIDS_E_RANGE. */
GIDS_API int gids_out_degree(int device, const void *indices, int index_bytes, uint64_t num_edges, uint64_t num_nodes,
                             uint32_t *counts, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GIDS_B200_H */
