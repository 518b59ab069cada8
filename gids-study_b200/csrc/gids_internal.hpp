// Internal declarations shared by the device code (gather.cu), the store
// (store.cu), the emulated SSDs (backing.cpp) and the C ABI (abi.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "gids_b200.h"

#ifndef GIDS_MAX_WORLD
#define GIDS_MAX_WORLD 8
#endif

namespace gids {

// ------------------------------------------------------------------ errors
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
void set_last_error(const std::string& msg);
void clear_last_error();

#define GIDS_CUDA(call)                                                                                 \
  do {                                                                                                  \
    cudaError_t e_ = (call);                                                                            \
    if (e_ != cudaSuccess)                                                                              \
      throw ::gids::Error(GIDS_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_) + " (" +     \
                                           __FILE__ + ":" + std::to_string(__LINE__) + ")");           \
  } while (0)
#define GIDS_CHECK(cond, code, msg)                     \
  do {                                                  \
    if (!(cond)) throw ::gids::Error((code), (msg));    \
  } while (0)

// RAII guard: switch to the store's device for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) GIDS_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// -------------------------------------------------------- page state word
// One 64-bit word per page of the range (the page table). It plays the role
// of the reference's data_page_t state word (page_cache_backup.h:104-117,
// 143-152): a reference count in the low bits, BUSY while a fill is in
// flight, VALID once the page is resident, and the cache slot that holds the
// page in the high 32 bits.
constexpr uint64_t ST_REF_MASK = (1ull << 24) - 1;
constexpr uint64_t ST_BUSY = 1ull << 24;
constexpr uint64_t ST_VALID = 1ull << 25;
constexpr int ST_SLOT_SHIFT = 32;
constexpr uint64_t SLOT_EMPTY = ~0ull;

// Pin word of a line (DevShard::wb): the low 31 bits count window-buffer
// marks (batches queued to gather the line), the top bit is a permanent pin
// (gids_store_pin_rows). A line with a nonzero word is never evicted.
constexpr unsigned int WB_PERMANENT = 0x80000000u;
constexpr unsigned int WB_COUNT_MASK = 0x7FFFFFFFu;
enum : uint32_t { WB_MARK = 0, WB_UNMARK = 1, WB_PIN = 2, WB_UNPIN = 3 };

// Per-segment source classes used by the gather kernel and its counters.
enum : int { CLS_NONE = 0, CLS_HIT = 1, CLS_OWN = 2, CLS_WAIT = 3, CLS_WAITED = 4, CLS_BYPASS = 5 };

// ---------------------------------------------------- device-side views
// One shard of the page cache: the page table of the pages a rank owns
// (page p is owned by rank p % world, at local index p / world) and that
// rank's slots. Pointers are valid in the calling process: local memory, or
// a peer's memory mapped through CUDA IPC or peer access.
struct DevShard {
  unsigned long long* state;      // [n_pages_local] page table
  unsigned long long* slot_page;  // [n_slots] local page index held by each slot (SLOT_EMPTY if none)
  unsigned char* slot_ref;        // [n_slots] clock counter (chances left before eviction)
  unsigned int* wb;               // [n_pages_local] pin words (window marks + permanent bit), or nullptr
  char* slots;                    // [n_slots * page_size] resident pages
  unsigned long long* clock;      // clock hand
  unsigned long long* seen;       // [n_pages_local / 64 + 1] admission bits, or nullptr (admit every miss)
};

// The cache works in lines: a line is the unit of the page table, of a slot
// and of a fill. It divides the stripe page of the backing store (by default
// it is the page, as in the reference; smaller lines stop small rows from
// pulling whole pages over the host link).
struct DevCache {
  DevShard sh[GIDS_MAX_WORLD];
  uint64_t n_slots;  // slots per shard
  uint64_t n_pages;  // lines of the whole range
  uint32_t page_shift;  // log2(line size)
  uint32_t page_size;   // line size in bytes
  uint32_t world;  // ranks sharing the cache (1 = unsharded)
  uint32_t rank;
  uint32_t ref_max;  // clock counter ceiling: 1 = second chance, >1 = frequency clock
  uint32_t pinned_only;  // 1: only permanently pinned lines are inserted; the rest read through
  uint32_t wb_marks;     // 1: window buffering has marked lines since the pins were last cleared
  // Replicated lines (sharded caches): a line whose bit is set is held by
  // every rank, in its own shard, at page-table entry n_local + (its rank
  // among the set bits); every other line is owned by rank line % world.
  const unsigned long long* rep_bits;  // [rep_words] one bit per line, or nullptr
  const unsigned int* rep_rank;        // [rep_words] set bits in the words before
  uint64_t rep_words;
  uint64_t n_local;  // page-table entries of the lines a shard owns; replicas follow
};

// Shard and page-table entry of cache line p: its owner's shard at p / world,
// or, for a replicated line, this rank's own shard after the owned entries.
#ifdef __CUDACC__
struct LineHome {
  uint32_t owner;
  uint64_t entry;
};
__device__ __forceinline__ LineHome line_home(const DevCache& c, uint64_t p) {
  LineHome h{(uint32_t)(p % c.world), p / c.world};
  if (c.rep_bits) {
    const uint64_t w = p >> 6;
    if (w < c.rep_words) {
      const unsigned long long bits = __ldg(c.rep_bits + w);
      if ((bits >> (p & 63)) & 1ull) {
        h.owner = c.rank;
        h.entry = c.n_local + (uint64_t)__ldg(c.rep_rank + w) + (uint64_t)__popcll(bits & ((1ull << (p & 63)) - 1ull));
      }
    }
  }
  return h;
}
#endif

struct DevBacking {
  const char* ssd[GIDS_MAX_SSD];  // device addresses of the mapped SSD regions
  uint32_t n_ssd;
  uint64_t page_start;  // first page of the range on every SSD
  uint64_t wrap_pages;  // pages physically held (== n_pages when the SSDs hold the whole range)
  uint32_t page_shift;  // log2(stripe page size)
  uint32_t lpp_shift;   // log2(cache lines per stripe page)
};

struct DevCpuBuf {
  int mode;  // 0 = none, 1 = rows [0, seq_len) (seq mode), 2 = bitmap
  uint64_t seq_len;
  const unsigned long long* bits;  // [nwords] membership bitmap over rows
  const unsigned int* rank;        // [nwords] pinned rows before each word
  uint64_t nwords;
  const char* buf;  // device address of the mapped pinned buffer
  uint64_t stride;  // bytes between buffer rows
  uint32_t row_bytes;  // bytes held per buffer row
};

struct GatherTuple {
  const int64_t* idx;
  char* out;
  uint64_t n;
  uint64_t key_off;
  uint64_t chunk_begin;  // first chunk of this tuple in the launch
};

struct GatherArgs {
  DevCache c;
  DevBacking b;
  DevCpuBuf cpu;
  unsigned long long* stats;  // [GIDS_STAT_COUNT]
  int* host_err;              // mapped pinned host word, set to 1 on a bad id
  uint64_t src_stride;        // bytes between rows of the range (cache_dim * elem_bytes)
  uint64_t n_rows;            // rows that lie completely inside the range
  uint32_t row_bytes;         // bytes gathered per row (dim * elem_bytes)
  uint32_t seg_shift;         // log2(page segments per row lane group)
  uint32_t spin_limit;        // bounded wait for another warp's fill
  uint32_t sweep_limit;       // bounded clock sweep (rounds of 32 candidates)
  int k;
  uint64_t total_chunks;
  GatherTuple t[GIDS_MAX_TUPLES];
};

struct WbArgs {
  unsigned int* wb[GIDS_MAX_WORLD];  // pin counters of every shard
  uint32_t world;
  DevCache home;  // line -> (shard, entry) when sharded (line_home); only its rep/rank/world fields are used
  const int64_t* idx;
  uint64_t n;
  int64_t off;
  uint64_t stride;  // bytes per row of the range
  uint64_t row_bytes;
  uint64_t n_rows;
  uint32_t page_shift;
  uint32_t mode;  // WB_MARK, WB_UNMARK, WB_PIN or WB_UNPIN, per (row, page)
};

// Launchers (gather.cu). sys = the cache is shared with other GPUs, so
// state-word atomics and fences use system scope.
void launch_gather(const GatherArgs& a, int vec, bool sys, int grid, cudaStream_t st, bool prefetch = false);
void launch_wb_mark(const WbArgs& a, cudaStream_t st);
void launch_host_probe(const DevBacking& b, uint64_t n_lines, uint32_t line_shift, uint32_t read_bytes,
                       uint64_t reads, void* dst, uint64_t dst_bytes, uint64_t seed, cudaStream_t st);
int gather_blocks_per_sm(int vec, bool sys);
constexpr int GATHER_THREADS = 256;

// Neighbour sampler and pin-list PageRank (sampler.cu).
struct Sampler;
Sampler* sampler_create(int device, const int64_t* indptr, const void* indices, int index_bytes, uint64_t n_nodes,
                        const int* fanouts, int n_layers, uint64_t max_seeds, uint64_t seed);
void sampler_destroy(Sampler* s);
uint64_t sampler_capacity(const Sampler* s);
void sampler_sample(Sampler* s, const int64_t* seeds, uint64_t n_seeds, int64_t* out_nodes, uint64_t out_cap,
                    uint64_t* count_dev, uint64_t* host_count, int64_t call, cudaStream_t st);
void pagerank(int device, const int64_t* indptr, const void* indices, int index_bytes, uint64_t n, int iters,
              double damping, float* pv, uint64_t* keys, cudaStream_t st);
void out_degree(int device, const void* indices, int index_bytes, uint64_t n_edges, uint64_t n, uint32_t* counts,
                cudaStream_t st);

// ------------------------------------------------------- emulated SSDs
struct SsdRegion {
  char* host = nullptr;
  char* dev = nullptr;  // device address of the mapped region
  uint64_t bytes = 0;
  int fd = -1;
  bool registered = false;
  std::string path;
};

class Controllers {
 public:
  ~Controllers();
  void init(uint32_t n, uint64_t q_depth, uint64_t n_queues, const int32_t* ssd_list);
  void set_emulation(uint64_t capacity_per_ssd, const char* pattern);
  // Size and map the first n_ssd SSDs for a range of range_pages pages with
  // page_size bytes, starting at page_start on each SSD. Returns the wrap
  // period in pages.
  uint64_t bind(uint32_t n_ssd, uint32_t page_size, uint64_t page_start, uint64_t range_pages);
  void register_with_cuda();
  std::vector<SsdRegion> ssd;
  std::vector<int32_t> ssd_list;
  uint32_t n_ctrls = 0;
  uint64_t q_depth = 0, n_queues = 0;
  uint64_t capacity_per_ssd = 0;
  std::string pattern;
  uint32_t page_size = 0;
  uint64_t page_start = 0, range_pages = 0, wrap_pages = 0;
  uint32_t n_bound = 0;
  bool bound = false;
};

// Striped host I/O over the bound SSDs (backing.cpp). Offsets are bytes of
// the logical range.
void backing_write(Controllers& c, const void* src, uint64_t nbytes, uint64_t off);
void backing_read(const Controllers& c, void* dst, uint64_t nbytes, uint64_t off);
void backing_fill_synthetic(Controllers& c, int kind, uint64_t seed, int threads);
int synth_elem_bytes(int kind);
// Host pointer of logical page p (after wrap).
const char* backing_page_host(const Controllers& c, uint64_t p);

// Pinned, GPU-mapped host allocation (mmap + transparent huge pages +
// cudaHostRegister), which pins far faster than cudaHostAlloc at tens of GB.
struct PinnedHost {
  char* host = nullptr;
  char* dev = nullptr;
  uint64_t bytes = 0;
  void alloc(uint64_t bytes, int threads);
  void release();
  ~PinnedHost() { release(); }
};
void parallel_for(uint64_t n, int threads, const std::function<void(uint64_t, uint64_t)>& fn);

// ---------------------------------------------------------------- store
class Store {
 public:
  Store(uint32_t elem_bytes, int device);
  ~Store();
  void init_controllers(Controllers* c, uint32_t page_size, uint64_t read_off_pages, uint64_t cache_mb,
                        uint64_t num_ele, uint64_t num_ssd);
  // prefetch: outs are ignored (null tuples): the rows' lines are brought into
  // the cache and nothing is copied out (window-buffer prefetch)
  void read_multi(int k, void* const* outs, const int64_t* const* idxs, const uint64_t* ns, int dim,
                  int cache_dim, const uint64_t* key_offs, cudaStream_t st, bool prefetch = false);
  // mode WB_MARK: mark the rows' lines (one pin per row and line); WB_UNMARK:
  // take those marks back (a window that will not be gathered); WB_PIN /
  // WB_UNPIN: set / clear the lines' permanent pins
  void window_buffering(const int64_t* idx, int64_t n, int64_t off, uint32_t stride_elems, cudaStream_t st,
                        uint32_t mode = WB_MARK);
  void clear_window_pins();
  void cpu_backing_buffer(uint64_t dim, uint64_t len);
  void set_cpu_buffer(const int64_t* host_idx, int64_t num);
  void set_row_layout(uint32_t cache_dim);
  void set_cache_line(uint32_t bytes);
  void debug_mark_busy(uint64_t line);
  uint32_t wait_limit = 1u << 16;  // polls of a BUSY line before giving up and bypassing
  // replacement policy: admission (a line is inserted on its second miss
  // within a window of 2 x n_slots line references) and clock counter ceiling
  int admission = 1;  // 0: insert every miss, 1: insert on the second miss, 2: pinned lines only
  uint32_t ref_max = 3;
  uint64_t refs_since_seen_reset = 0;
  // window buffering has marked lines since the pins were last cleared: until
  // then a gather has no window pins to consume and skips reading them
  bool wb_marked = false;
  void set_policy(int admit, uint32_t ref_ceiling);
  void set_gather_blocks(uint32_t n);
  // gather with the page cache in the library's static no-allocation scratch (noalloc.cu)
  void read_noalloc(void* out, const int64_t* idx, int64_t n, int dim, int cache_dim, uint64_t key_off,
                    cudaStream_t st);
  void store_tensor(const void* src, uint64_t num_rows, uint64_t offset_bytes);
  void write_range(const void* src, uint64_t nbytes, uint64_t off);
  void flush_cache();
  void get_stats(uint64_t* out, int count);
  void reset_stats();
  void print_stats();
  double kernel_time_ms();
  void synchronize();
  uint32_t cpu_access_count();
  void flush_cpu_access_count();

  uint32_t elem_bytes;
  int device;
  bool synchronous = true;
  Controllers* ctrls = nullptr;
  bool initialized = false;
  uint32_t page_size = 0, page_shift = 0;   // stripe page of the backing store
  uint32_t line_size = 0, line_shift = 0;   // cache line (divides the page)
  uint32_t line_request = 0;                // set_cache_line before init; 0 = the page
  uint64_t read_off_pages = 0, num_ele = 0, range_bytes = 0, n_pages = 0, n_slots = 0;
  uint64_t n_lines = 0, n_lines_local = 0;
  // replicated lines (sharded caches): page-table entries reserved after the
  // owned ones (set_replicas, before init_controllers; the same on every
  // rank), the lines now replicated, and their bitmap and rank words
  uint64_t n_rep_max = 0, n_rep = 0, rep_words = 0;
  unsigned long long* d_rep_bits = nullptr;
  unsigned int* d_rep_rank = nullptr;
  uint64_t n_entries_local() const { return n_lines_local + n_rep_max; }
  void set_replicas(uint64_t max_lines);
  // host array of cache-line ids, strictly increasing; flushes this rank's shard
  void set_replicated_lines(const uint64_t* lines, uint64_t n);
  uint32_t row_layout = 0;  // source row stride (elements) for CPU-buffer fills / WB; 0 = unknown

  // sharding (page p is owned by rank p % world)
  uint32_t world = 1, rank = 0;
  bool shards_ready = true;           // false until peers are attached (world > 1)
  DevShard shards[GIDS_MAX_WORLD] = {};
  std::vector<void*> ipc_opened;      // peer shard bases opened through CUDA IPC
  void set_sharding(uint32_t world, uint32_t rank);
  void ipc_handle(void* out64);
  void open_peers(const void* handles, uint32_t n);
  static void share_in_process(Store* const* stores, uint32_t n);
  // bandwidth of a device-to-device copy of `bytes` from rank `peer`'s shard
  // into this GPU (GB/s, best of three): the link term of the roofline
  double peer_copy_gbs(uint32_t peer, uint64_t bytes);
  // host-link bandwidth of random reads of `read_bytes` from the start of
  // cache lines of the backing store (GB/s, best of three launches)
  double host_read_gbs(uint32_t read_bytes, uint64_t total_bytes);

  // device allocations (this rank's shard lives in one allocation, d_shard)
  char* d_shard = nullptr;
  uint64_t shard_bytes = 0;
  unsigned long long* d_state = nullptr;
  unsigned long long* d_slot_page = nullptr;
  unsigned char* d_slot_ref = nullptr;
  unsigned int* d_wb = nullptr;
  char* d_slots = nullptr;
  unsigned long long* d_clock = nullptr;
  unsigned long long* d_stats = nullptr;
  int* h_err = nullptr;  // mapped pinned host word
  int* d_err = nullptr;

  // constant CPU buffer
  PinnedHost cpu_buf;
  uint64_t cpu_dim = 0, cpu_len = 0;
  int cpu_mode = 0;
  std::vector<int64_t> cpu_rows;  // sorted pinned rows (bitmap mode)
  unsigned long long* d_cpu_bits = nullptr;
  unsigned int* d_cpu_rank = nullptr;
  uint64_t cpu_nwords = 0;
  uint32_t cpu_filled_stride = 0;  // source stride (elements) the buffer was filled with; 0 = not filled
  void fill_cpu_buffer(uint32_t src_stride_elems);

  // counters and timing
  uint64_t stat_base_cpu = 0;  // CPU-row counter at the last flush_cpu_access_count
  uint32_t cpu_access_host = 0;
  cudaStream_t last_stream = nullptr;
  struct EvPair {
    cudaEvent_t a, b;
  };
  std::vector<EvPair> ev_pending, ev_free;
  double kernel_ms = 0.0;
  uint64_t total_access = 0;
  uint64_t launches = 0;
  void fold_events(bool wait);
  int grid_blocks[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  uint32_t max_blocks = 0;  // cap on a gather's grid (0: the resident maximum)
  std::mutex mu;

 private:
  void free_all();
  DevCache dev_cache() const;
  DevBacking dev_backing() const;
  DevCpuBuf dev_cpu() const;
  void check_async_error();
};

}  // namespace gids

// The Store behind a C handle (abi.cpp).
gids::Store* gids_store_of(gids_store_t* s);
