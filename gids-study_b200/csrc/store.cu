// Host side of one feature store: the page cache in HBM, the constant CPU
// buffer, window buffering, counters and launches. Mirrors the members of the
// reference's BAM_Feature_Store<T> (gids_module/include/bam_nvme.h:230-613,
// gids_module/gids_nvme.cu:123-806).
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <thread>

#include "gids_internal.hpp"

namespace gids {

namespace {
// NVTX range for the duration of a host call (visible in Nsight traces)
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

uint32_t log2_exact(uint64_t v) {
  uint32_t s = 0;
  while ((1ull << s) < v) s++;
  return s;
}
uint64_t gcd64(uint64_t a, uint64_t b) {
  while (b) {
    uint64_t t = a % b;
    a = b;
    b = t;
  }
  return a;
}
int host_threads() {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}
}  // namespace

Store::Store(uint32_t eb, int dev) : elem_bytes(eb), device(dev) {
  GIDS_CHECK(eb == 2 || eb == 4 || eb == 8, GIDS_E_INVAL, "elem_bytes must be 2, 4 or 8");
  int n = 0;
  GIDS_CUDA(cudaGetDeviceCount(&n));
  GIDS_CHECK(dev >= 0 && dev < n, GIDS_E_INVAL, "device " + std::to_string(dev) + " not present");
  DeviceGuard g(device);
  GIDS_CUDA(cudaMalloc(&d_stats, GIDS_STAT_COUNT * sizeof(unsigned long long)));
  GIDS_CUDA(cudaMemset(d_stats, 0, GIDS_STAT_COUNT * sizeof(unsigned long long)));
  GIDS_CUDA(cudaMalloc(&d_clock, sizeof(unsigned long long)));
  GIDS_CUDA(cudaMemset(d_clock, 0, sizeof(unsigned long long)));
  GIDS_CUDA(cudaHostAlloc(&h_err, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
  *h_err = 0;
  GIDS_CUDA(cudaHostGetDevicePointer(&d_err, h_err, 0));
}

Store::~Store() {
  try {
    DeviceGuard g(device);
    cudaDeviceSynchronize();
    free_all();
    for (auto& e : ev_pending) {
      cudaEventDestroy(e.a);
      cudaEventDestroy(e.b);
    }
    for (auto& e : ev_free) {
      cudaEventDestroy(e.a);
      cudaEventDestroy(e.b);
    }
    if (d_stats) cudaFree(d_stats);
    if (d_clock) cudaFree(d_clock);
    if (h_err) cudaFreeHost(h_err);
  } catch (...) {
  }
}

void Store::free_all() {
  auto f = [](auto*& p) {
    if (p) cudaFree((void*)p);
    p = nullptr;
  };
  for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
  ipc_opened.clear();
  if (world == 1) f(d_wb);  // sharded stores keep the pins inside the shard allocation
  if (d_shard) cudaFree(d_shard);
  d_shard = nullptr;
  d_state = nullptr;
  d_slot_page = nullptr;
  d_slot_ref = nullptr;
  d_wb = nullptr;
  d_slots = nullptr;
  f(d_cpu_bits);
  f(d_cpu_rank);
  f(d_rep_bits);
  f(d_rep_rank);
  n_rep = rep_words = 0;
  cpu_buf.release();
}

namespace {
// Byte layout of one shard allocation; identical on every rank so that a
// peer's shard can be addressed from its base pointer alone.
struct ShardLayout {
  uint64_t state, slot_page, slot_ref, wb, clock, seen, seen_bytes, slots, total;
  ShardLayout(uint64_t n_local, uint64_t n_slots, uint32_t page_size, bool with_wb) {
    auto up = [](uint64_t v, uint64_t a) { return (v + a - 1) / a * a; };
    state = 0;
    slot_page = up(state + n_local * 8, 256);
    slot_ref = up(slot_page + n_slots * 8, 256);
    wb = up(slot_ref + n_slots, 256);
    clock = up(wb + (with_wb ? n_local * 4 : 0), 256);
    seen = up(clock + 8, 256);
    seen_bytes = (n_local / 64 + 1) * 8;
    slots = up(seen + seen_bytes, page_size > 4096 ? page_size : 4096);
    // a whole number of 2 MB pages: a peer process maps a CUDA-IPC allocation
    // whose size is not a multiple of 2 MB with small pages, and its random
    // 4 KB reads of the shard then run at a third of the link (B200, measured:
    // 235-390 GB/s against 783 GB/s for the same allocation rounded up)
    total = up(slots + n_slots * (uint64_t)page_size, 2ull << 20);
  }
  DevShard at(char* base, bool with_wb) const {
    DevShard d{};
    d.state = (unsigned long long*)(base + state);
    d.slot_page = (unsigned long long*)(base + slot_page);
    d.slot_ref = (unsigned char*)(base + slot_ref);
    d.wb = with_wb ? (unsigned int*)(base + wb) : nullptr;
    d.clock = (unsigned long long*)(base + clock);
    d.seen = (unsigned long long*)(base + seen);
    d.slots = base + slots;
    return d;
  }
};
}  // namespace

void Store::set_replicas(uint64_t max_lines) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(!initialized, GIDS_E_STATE, "set_replicas after init_controllers");
  GIDS_CHECK(max_lines < (1ull << 32), GIDS_E_INVAL, "at most 2^32 - 1 replicated lines");
  n_rep_max = max_lines;
}

// The lines every rank holds in its own shard: a bitmap over the range's lines
// and, per 64-bit word, the number of set bits before it (built on the host,
// once; the kernels find a line's entry with one word load and a popcount).
// The replica entries are cleared with the rest of this rank's shard, so that
// no slot stays tagged with an entry that now means another line.
void Store::set_replicated_lines(const uint64_t* lines, uint64_t n) {
  GIDS_CHECK(initialized, GIDS_E_STATE, "set_replicated_lines before init_controllers");
  GIDS_CHECK(world > 1, GIDS_E_STATE, "replicated lines need a sharded cache");
  GIDS_CHECK(n <= n_rep_max, GIDS_E_RANGE, "more replicated lines than set_replicas reserved");
  GIDS_CHECK(n == 0 || lines, GIDS_E_INVAL, "null line array");
  for (uint64_t i = 0; i < n; i++) {
    GIDS_CHECK(lines[i] < n_lines, GIDS_E_RANGE, "replicated line outside the range");
    GIDS_CHECK(i == 0 || lines[i] > lines[i - 1], GIDS_E_INVAL, "replicated lines must be strictly increasing");
  }
  flush_cache();
  std::lock_guard<std::mutex> lk(mu);
  DeviceGuard g(device);
  if (d_rep_bits) GIDS_CUDA(cudaFree(d_rep_bits));
  if (d_rep_rank) GIDS_CUDA(cudaFree(d_rep_rank));
  d_rep_bits = nullptr;
  d_rep_rank = nullptr;
  n_rep = rep_words = 0;
  if (!n) return;
  const uint64_t words = (lines[n - 1] >> 6) + 1;
  std::vector<unsigned long long> bits(words, 0ull);
  std::vector<unsigned int> rank_words(words, 0u);
  for (uint64_t i = 0; i < n; i++) bits[lines[i] >> 6] |= 1ull << (lines[i] & 63);
  uint64_t before = 0;
  for (uint64_t w = 0; w < words; w++) {
    rank_words[w] = (unsigned int)before;
    before += (uint64_t)__builtin_popcountll(bits[w]);
  }
  GIDS_CUDA(cudaMalloc(&d_rep_bits, words * sizeof(unsigned long long)));
  GIDS_CUDA(cudaMalloc(&d_rep_rank, words * sizeof(unsigned int)));
  GIDS_CUDA(cudaMemcpy(d_rep_bits, bits.data(), words * sizeof(unsigned long long), cudaMemcpyHostToDevice));
  GIDS_CUDA(cudaMemcpy(d_rep_rank, rank_words.data(), words * sizeof(unsigned int), cudaMemcpyHostToDevice));
  n_rep = n;
  rep_words = words;
}

void Store::set_sharding(uint32_t w, uint32_t r) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(!initialized, GIDS_E_STATE, "set_sharding after init_controllers");
  GIDS_CHECK(w >= 1 && w <= GIDS_MAX_WORLD && r < w, GIDS_E_INVAL, "need 1 <= world <= 8 and rank < world");
  world = w;
  rank = r;
}

void Store::ipc_handle(void* out64) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized && d_shard, GIDS_E_STATE, "no shard allocated yet");
  DeviceGuard g(device);
  cudaIpcMemHandle_t h;
  GIDS_CUDA(cudaIpcGetMemHandle(&h, d_shard));
  memcpy(out64, &h, sizeof(h));
}

void Store::open_peers(const void* handles, uint32_t n) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "open_peers before init_controllers");
  GIDS_CHECK(n == world, GIDS_E_INVAL, "need one handle per rank");
  DeviceGuard g(device);
  const ShardLayout L(n_entries_local(), n_slots, line_size, world > 1);
  const cudaIpcMemHandle_t* h = (const cudaIpcMemHandle_t*)handles;
  for (uint32_t r = 0; r < world; r++) {
    if (r == rank) continue;
    void* p = nullptr;
    GIDS_CUDA(cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess));
    ipc_opened.push_back(p);
    shards[r] = L.at((char*)p, world > 1);
  }
  shards_ready = true;
}

void Store::share_in_process(Store* const* stores, uint32_t n) {
  GIDS_CHECK(n >= 1 && n <= GIDS_MAX_WORLD, GIDS_E_INVAL, "1..8 stores");
  for (uint32_t i = 0; i < n; i++) {
    Store* s = stores[i];
    GIDS_CHECK(s && s->initialized, GIDS_E_STATE, "every store must be initialised");
    GIDS_CHECK(s->world == n && s->rank == i, GIDS_E_INVAL, "store i must have world n and rank i");
    GIDS_CHECK(s->n_lines == stores[0]->n_lines && s->n_slots == stores[0]->n_slots &&
                   s->line_size == stores[0]->line_size && s->n_rep_max == stores[0]->n_rep_max,
               GIDS_E_INVAL, "stores differ in geometry");
  }
  for (uint32_t i = 0; i < n; i++)
    for (uint32_t j = 0; j < n; j++) {
      const int di = stores[i]->device, dj = stores[j]->device;
      if (di == dj) continue;
      DeviceGuard g(di);
      cudaError_t e = cudaDeviceEnablePeerAccess(dj, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else {
        GIDS_CUDA(e);
      }
    }
  for (uint32_t i = 0; i < n; i++) {
    std::lock_guard<std::mutex> lk(stores[i]->mu);
    for (uint32_t j = 0; j < n; j++) stores[i]->shards[j] = stores[j]->shards[j];
    stores[i]->shards_ready = true;
  }
}

void Store::init_controllers(Controllers* c, uint32_t ps, uint64_t read_off_pages_, uint64_t cache_mb, uint64_t ne,
                             uint64_t num_ssd) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(c, GIDS_E_INVAL, "controllers are null");
  GIDS_CHECK(!initialized, GIDS_E_STATE, "init_controllers called twice");
  GIDS_CHECK(ps >= 512 && (ps & (ps - 1)) == 0, GIDS_E_INVAL, "page_size must be a power of two >= 512");
  GIDS_CHECK(ne > 0, GIDS_E_INVAL, "num_ele must be > 0");
  GIDS_CHECK(num_ssd >= 1 && num_ssd <= c->n_ctrls && num_ssd <= GIDS_MAX_SSD, GIDS_E_INVAL,
             "num_ssd must be in [1, controllers initialised]");
  DeviceGuard g(device);
  page_size = ps;
  page_shift = log2_exact(ps);
  read_off_pages = read_off_pages_;
  num_ele = ne;
  range_bytes = ne * elem_bytes;
  n_pages = (range_bytes + ps - 1) / ps;
  line_size = line_request ? line_request : ps;
  GIDS_CHECK(line_size >= 512 && (line_size & (line_size - 1)) == 0 && line_size <= ps, GIDS_E_INVAL,
             "cache line must be a power of two in [512, page_size]");
  line_shift = log2_exact(line_size);
  n_lines = (range_bytes + line_size - 1) / line_size;
  n_slots = cache_mb * (1ull << 20) / line_size;
  GIDS_CHECK(n_slots < (1ull << 32) - 1, GIDS_E_INVAL, "cache too large for 32-bit slot numbers");

  c->bind((uint32_t)num_ssd, ps, read_off_pages, n_pages);
  c->register_with_cuda();
  ctrls = c;

  // this rank's shard: page table of the pages it owns (p % world == rank),
  // slots, clock and (when sharded) window-buffer pins, in one allocation
  n_lines_local = (n_lines + world - 1) / world;
  if (world == 1) n_rep_max = 0;  // replicas only make sense in a sharded cache
  const bool with_wb = world > 1;
  const ShardLayout L(n_entries_local(), n_slots, line_size, with_wb);
  shard_bytes = L.total;
  GIDS_CUDA(cudaMalloc(&d_shard, shard_bytes));
  const DevShard mine = L.at(d_shard, with_wb);
  d_state = mine.state;
  d_slot_page = mine.slot_page;
  d_slot_ref = mine.slot_ref;
  d_slots = mine.slots;
  if (with_wb) d_wb = mine.wb;
  GIDS_CUDA(cudaMemset(d_shard, 0, L.slot_page));
  GIDS_CUDA(cudaMemset(d_shard + L.slot_page, 0xFF, n_slots * 8));
  GIDS_CUDA(cudaMemset(d_shard + L.slot_ref, 0, L.slots - L.slot_ref));
  shards[rank] = mine;
  shards_ready = world == 1;
  int sms = 0;
  GIDS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const int vecs[4] = {16, 8, 4, 2};
  for (int sy = 0; sy < 2; sy++)
    for (int i = 0; i < 4; i++) grid_blocks[sy][i] = std::max(1, gather_blocks_per_sm(vecs[i], sy == 1)) * sms;
  GIDS_CUDA(cudaDeviceSynchronize());
  initialized = true;
}

DevCache Store::dev_cache() const {
  DevCache c{};
  for (uint32_t r = 0; r < world; r++) c.sh[r] = shards[r];
  if (world == 1) c.sh[0].wb = d_wb;  // allocated on first use
  c.n_slots = n_slots;
  c.n_pages = n_lines;
  c.page_shift = line_shift;
  c.page_size = line_size;
  c.world = world;
  c.rank = rank;
  c.ref_max = ref_max;
  c.pinned_only = admission == 2 ? 1u : 0u;
  c.wb_marks = wb_marked ? 1u : 0u;
  c.n_local = n_lines_local;
  if (n_rep) {
    c.rep_bits = d_rep_bits;
    c.rep_rank = d_rep_rank;
    c.rep_words = rep_words;
  }
  if (admission != 1)
    for (uint32_t r = 0; r < world; r++) c.sh[r].seen = nullptr;
  return c;
}

DevBacking Store::dev_backing() const {
  DevBacking b{};
  for (uint32_t i = 0; i < ctrls->n_bound; i++) b.ssd[i] = ctrls->ssd[i].dev;
  b.n_ssd = ctrls->n_bound;
  b.page_start = ctrls->page_start;
  b.wrap_pages = ctrls->wrap_pages;
  b.page_shift = page_shift;
  b.lpp_shift = page_shift - line_shift;
  return b;
}

DevCpuBuf Store::dev_cpu() const {
  DevCpuBuf d{};
  d.mode = cpu_filled_stride ? cpu_mode : 0;
  d.seq_len = cpu_len;
  d.bits = d_cpu_bits;
  d.rank = d_cpu_rank;
  d.nwords = cpu_nwords;
  d.buf = cpu_buf.dev;
  d.stride = cpu_buf.bytes && cpu_len ? cpu_buf.bytes / cpu_len : 0;
  d.row_bytes = (uint32_t)(cpu_dim * elem_bytes);
  return d;
}

void Store::check_async_error() {
  const int e = h_err ? *reinterpret_cast<volatile int*>(h_err) : 0;
  if (e) {
    *reinterpret_cast<volatile int*>(h_err) = 0;
    if (e == 2)  // the gathered rows are complete: the kernel copied them again without the TMA
      throw Error(GIDS_E_CUDA, "a TMA bulk copy of the gather did not complete within its wait limit");
    throw Error(GIDS_E_RANGE, "a node id addressed a row outside the feature range (its output row is zero)");
  }
}

void Store::fold_events(bool wait) {
  size_t keep = 0;
  for (size_t i = 0; i < ev_pending.size(); i++) {
    auto& e = ev_pending[i];
    cudaError_t q = wait ? cudaEventSynchronize(e.b) : cudaEventQuery(e.b);
    if (q == cudaSuccess) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, e.a, e.b) == cudaSuccess) kernel_ms += ms;
      ev_free.push_back(e);
    } else {
      if (q != cudaErrorNotReady) GIDS_CUDA(q);
      ev_pending[keep++] = e;
    }
  }
  ev_pending.resize(keep);
}

void Store::debug_mark_busy(uint64_t line) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "debug_mark_busy before init_controllers");
  GIDS_CHECK(line < n_lines, GIDS_E_RANGE, "line outside the range");
  GIDS_CHECK(world == 1 || line % world == rank, GIDS_E_INVAL, "the line is owned by another rank's shard");
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  const unsigned long long busy = ST_BUSY;  // BUSY, no references, not VALID, no slot
  GIDS_CUDA(cudaMemcpy(d_state + (world == 1 ? line : line / world), &busy, sizeof(busy), cudaMemcpyHostToDevice));
}

void Store::set_policy(int admit, uint32_t ref_ceiling) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(ref_ceiling >= 1 && ref_ceiling <= 255, GIDS_E_INVAL, "clock counter ceiling must be in [1, 255]");
  GIDS_CHECK(admit >= 0 && admit <= 2, GIDS_E_INVAL, "admission must be 0, 1 or 2");
  admission = admit;
  ref_max = ref_ceiling;
}

void Store::set_gather_blocks(uint32_t n) {
  std::lock_guard<std::mutex> lk(mu);
  max_blocks = n;
}

void Store::set_cache_line(uint32_t bytes) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(!initialized, GIDS_E_STATE, "set_cache_line after init_controllers");
  GIDS_CHECK(bytes == 0 || (bytes >= 512 && (bytes & (bytes - 1)) == 0), GIDS_E_INVAL,
             "cache line must be 0 (the page) or a power of two >= 512");
  line_request = bytes;
}

void Store::set_row_layout(uint32_t cache_dim) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(cache_dim > 0, GIDS_E_INVAL, "cache_dim must be > 0");
  row_layout = cache_dim;
  if (initialized && cpu_mode && cpu_filled_stride != cache_dim) fill_cpu_buffer(cache_dim);
}

void Store::read_multi(int k, void* const* outs, const int64_t* const* idxs, const uint64_t* ns, int dim,
                       int cache_dim, const uint64_t* key_offs, cudaStream_t st, bool prefetch) {
  std::lock_guard<std::mutex> lk(mu);
  NvtxRange nv(prefetch ? "gids.prefetch" : "gids.read_feature");
  GIDS_CHECK(initialized, GIDS_E_STATE, "read_feature before init_controllers");
  GIDS_CHECK(shards_ready, GIDS_E_STATE, "sharded cache: peer shards not attached yet");
  GIDS_CHECK(k >= 0, GIDS_E_INVAL, "k must be >= 0");
  GIDS_CHECK(dim > 0 && cache_dim > 0 && dim <= cache_dim, GIDS_E_INVAL, "need 0 < dim <= cache_dim");
  DeviceGuard g(device);
  check_async_error();
  fold_events(false);
  const uint64_t row_bytes = (uint64_t)dim * elem_bytes;
  const uint64_t src_stride = (uint64_t)cache_dim * elem_bytes;
  GIDS_CHECK(row_bytes < (1ull << 31), GIDS_E_INVAL, "row too large");
  if (cpu_mode) {
    GIDS_CHECK((uint64_t)dim <= cpu_dim, GIDS_E_INVAL,
               "dim exceeds the constant CPU buffer's row width (cpu_backing_buffer dim)");
    if (cpu_filled_stride != (uint32_t)cache_dim) fill_cpu_buffer((uint32_t)cache_dim);
  }
  if (!row_layout) row_layout = (uint32_t)cache_dim;

  // lanes per row: cache lines one row can touch, rounded up to a power of two
  const uint64_t gst = gcd64(src_stride, line_size);
  const uint64_t max_pages = (line_size - gst + row_bytes - 1) / line_size + 1;
  uint32_t seg_shift = 0;
  while ((1ull << seg_shift) < max_pages) seg_shift++;
  GIDS_CHECK(seg_shift <= 5, GIDS_E_UNSUPPORTED, "a row may span more than 32 cache lines; use larger lines");
  const uint64_t rpc = 32ull >> seg_shift;

  // vector width: every address and length of the copy must be a multiple
  int vec = 16;
  auto fits = [&](uint64_t v) { return v % vec == 0; };
  while (vec > 2 && !(fits(row_bytes) && fits(src_stride))) vec >>= 1;
  for (int i = 0; i < k && !prefetch; i++)
    while (vec > 2 && (uint64_t)(uintptr_t)outs[i] % vec) vec >>= 1;
  GIDS_CHECK(row_bytes % vec == 0 && src_stride % vec == 0, GIDS_E_INVAL, "rows must be 2-byte aligned");
  for (int i = 0; i < k; i++) {
    GIDS_CHECK(ns[i] == 0 || ((prefetch || outs[i]) && idxs[i]), GIDS_E_INVAL, "null output or index pointer");
    GIDS_CHECK((uintptr_t)idxs[i] % 8 == 0 || ns[i] == 0, GIDS_E_INVAL, "index array must be 8-byte aligned");
    GIDS_CHECK(prefetch || (uintptr_t)outs[i] % vec == 0 || ns[i] == 0, GIDS_E_INVAL, "output not aligned");
  }

  GatherArgs a;
  memset(&a, 0, sizeof(a));
  a.c = dev_cache();
  a.b = dev_backing();
  a.cpu = dev_cpu();
  a.stats = d_stats;
  a.host_err = d_err;
  a.src_stride = src_stride;
  a.n_rows = range_bytes >= row_bytes ? (range_bytes - row_bytes) / src_stride + 1 : 0;
  a.row_bytes = (uint32_t)row_bytes;
  a.seg_shift = seg_shift;
  a.spin_limit = wait_limit;
  a.sweep_limit = 64;
  uint64_t rows_total = 0;
  if (admission == 1 && n_slots && !prefetch) {
    // age the admission bits: clear this shard's after 2 x n_slots line references
    uint64_t refs = 0;
    for (int i = 0; i < k; i++) refs += ns[i] * max_pages;
    refs_since_seen_reset += refs;
    if (refs_since_seen_reset > 2 * n_slots) {
      const ShardLayout Ls(n_entries_local(), n_slots, line_size, world > 1);
      GIDS_CUDA(cudaMemsetAsync(d_shard + Ls.seen, 0, Ls.seen_bytes, st));
      refs_since_seen_reset = refs;
    }
  }
  for (int base = 0; base < k || (k == 0 && base == 0); base += GIDS_MAX_TUPLES) {
    const int kk = std::min(GIDS_MAX_TUPLES, k - base);
    uint64_t chunks = 0;
    int used = 0;
    for (int i = 0; i < kk; i++) {
      const uint64_t n = ns[base + i];
      if (!n) continue;
      GatherTuple& t = a.t[used++];
      t.idx = idxs[base + i];
      t.out = prefetch ? nullptr : (char*)outs[base + i];  // no output: the kernel only fills
      t.n = n;
      t.key_off = key_offs ? key_offs[base + i] : 0;
      t.chunk_begin = chunks;
      chunks += (n + rpc - 1) / rpc;
      rows_total += n;
    }
    if (!chunks) {
      if (k == 0) break;
      continue;
    }
    a.k = used;
    a.total_chunks = chunks;
    const int vi = prefetch ? 1 : vec == 16 ? 0 : vec == 8 ? 1 : vec == 4 ? 2 : 3;  // prefetch: the 8-byte kernel's grid
    const uint64_t want_blocks = (chunks + (GATHER_THREADS / 32) - 1) / (GATHER_THREADS / 32);
    uint64_t cap = (uint64_t)grid_blocks[world > 1 ? 1 : 0][vi];
    if (max_blocks) cap = std::min<uint64_t>(cap, max_blocks);
    const int grid = (int)std::min<uint64_t>(want_blocks, cap);
    EvPair ev;
    if (!ev_free.empty()) {
      ev = ev_free.back();
      ev_free.pop_back();
    } else {
      GIDS_CUDA(cudaEventCreate(&ev.a));
      GIDS_CUDA(cudaEventCreate(&ev.b));
    }
    GIDS_CUDA(cudaEventRecord(ev.a, st));
    launch_gather(a, vec, world > 1, grid, st, prefetch);
    launches++;
    GIDS_CUDA(cudaEventRecord(ev.b, st));
    ev_pending.push_back(ev);
    if (k == 0) break;
  }
  if (!prefetch) total_access += rows_total;
  last_stream = st;
  if (synchronous) {
    GIDS_CUDA(cudaStreamSynchronize(st));
    fold_events(true);
    check_async_error();
  }
}

void Store::window_buffering(const int64_t* idx, int64_t n, int64_t off, uint32_t stride_elems, cudaStream_t st,
                             uint32_t mode) {
  std::lock_guard<std::mutex> lk(mu);
  NvtxRange nv(mode == WB_MARK ? "gids.window_buffering" : mode == WB_UNMARK ? "gids.window_unmark" : "gids.pin");
  GIDS_CHECK(initialized, GIDS_E_STATE, "set_window_buffering before init_controllers");
  GIDS_CHECK(n >= 0, GIDS_E_INVAL, "n must be >= 0");
  if (n == 0) return;
  GIDS_CHECK(idx, GIDS_E_INVAL, "null index pointer");
  GIDS_CHECK(shards_ready, GIDS_E_STATE, "sharded cache: peer shards not attached yet");
  DeviceGuard g(device);
  if (!d_wb) {
    if (mode == WB_UNMARK || mode == WB_UNPIN) return;  // nothing was ever marked
    GIDS_CUDA(cudaMalloc(&d_wb, n_lines * sizeof(unsigned int)));
    GIDS_CUDA(cudaMemset(d_wb, 0, n_lines * sizeof(unsigned int)));
  }
  // rows map to pages by bytes; without a known layout, one row per page
  // (the reference's assumption, gids_kernel.cu:251-252)
  uint32_t se = stride_elems ? stride_elems : row_layout ? row_layout : page_size / elem_bytes;
  WbArgs w{};
  w.world = world;
  w.home = dev_cache();
  for (uint32_t r = 0; r < world; r++) w.wb[r] = world == 1 ? d_wb : shards[r].wb;
  w.idx = idx;
  w.n = (uint64_t)n;
  w.off = off;
  w.stride = (uint64_t)se * elem_bytes;
  w.row_bytes = w.stride;
  w.n_rows = range_bytes >= w.row_bytes ? (range_bytes - w.row_bytes) / w.stride + 1 : 0;
  w.page_shift = line_shift;
  w.mode = mode;
  if (mode == WB_MARK) wb_marked = true;  // gathers launched from now on consume window pins
  launch_wb_mark(w, st);
  last_stream = st;
  if (synchronous) GIDS_CUDA(cudaStreamSynchronize(st));
}

void Store::cpu_backing_buffer(uint64_t dim, uint64_t len) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "cpu_backing_buffer before init_controllers");
  GIDS_CHECK(dim > 0, GIDS_E_INVAL, "dim must be > 0");
  DeviceGuard g(device);
  cudaDeviceSynchronize();
  cpu_buf.release();
  const uint64_t stride = (dim * elem_bytes + 15) / 16 * 16;
  cpu_dim = dim;
  cpu_len = len;
  cpu_rows.clear();
  cpu_mode = len ? 1 : 0;  // seq mode until set_cpu_buffer
  cpu_filled_stride = 0;
  if (len) cpu_buf.alloc(stride * len, host_threads());
  if (cpu_mode && row_layout) fill_cpu_buffer(row_layout);
}

void Store::set_cpu_buffer(const int64_t* idx, int64_t num) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "set_cpu_buffer before init_controllers");
  GIDS_CHECK(cpu_buf.bytes || num == 0, GIDS_E_STATE, "set_cpu_buffer before cpu_backing_buffer");
  GIDS_CHECK(num >= 0 && (uint64_t)num <= cpu_len, GIDS_E_INVAL, "more pinned rows than the CPU buffer holds");
  GIDS_CHECK(num == 0 || idx, GIDS_E_INVAL, "null index pointer");
  DeviceGuard g(device);
  cudaDeviceSynchronize();
  std::vector<int64_t> rows(idx, idx + num);
  std::sort(rows.begin(), rows.end());
  rows.erase(std::unique(rows.begin(), rows.end()), rows.end());
  GIDS_CHECK(rows.empty() || rows.front() >= 0, GIDS_E_RANGE, "negative node id in the pin list");
  cpu_rows = std::move(rows);
  // membership bitmap over rows [0, max pinned row], and the rank of each word
  cpu_nwords = cpu_rows.empty() ? 0 : (uint64_t)(cpu_rows.back() >> 6) + 1;
  std::vector<unsigned long long> bits(cpu_nwords, 0ull);
  std::vector<unsigned int> rank(cpu_nwords, 0u);
  for (int64_t r : cpu_rows) bits[r >> 6] |= 1ull << (r & 63);
  unsigned int acc = 0;
  for (uint64_t w = 0; w < cpu_nwords; w++) {
    rank[w] = acc;
    acc += (unsigned int)__builtin_popcountll(bits[w]);
  }
  if (d_cpu_bits) cudaFree(d_cpu_bits);
  if (d_cpu_rank) cudaFree(d_cpu_rank);
  d_cpu_bits = nullptr;
  d_cpu_rank = nullptr;
  if (cpu_nwords) {
    GIDS_CUDA(cudaMalloc(&d_cpu_bits, cpu_nwords * sizeof(unsigned long long)));
    GIDS_CUDA(cudaMalloc(&d_cpu_rank, cpu_nwords * sizeof(unsigned int)));
    GIDS_CUDA(cudaMemcpy(d_cpu_bits, bits.data(), cpu_nwords * 8, cudaMemcpyHostToDevice));
    GIDS_CUDA(cudaMemcpy(d_cpu_rank, rank.data(), cpu_nwords * 4, cudaMemcpyHostToDevice));
  }
  cpu_mode = 2;
  cpu_filled_stride = 0;
  if (row_layout) fill_cpu_buffer(row_layout);
}

// Copies the pinned rows from the backing store into the CPU buffer (host
// threads; the buffer and the emulated SSDs are both host memory). The
// reference fills through the GPU cache with one block per row
// (set_cpu_buffer_data_kernel, gids_kernel.cu:216-228).
void Store::fill_cpu_buffer(uint32_t src_stride_elems) {
  const uint64_t stride = cpu_len ? cpu_buf.bytes / cpu_len : 0;
  const uint64_t src_stride = (uint64_t)src_stride_elems * elem_bytes;
  const uint64_t row_bytes = cpu_dim * elem_bytes;
  const uint64_t n_rows = range_bytes >= row_bytes ? (range_bytes - row_bytes) / src_stride + 1 : 0;
  const uint64_t count = cpu_mode == 1 ? cpu_len : cpu_rows.size();
  if (cpu_mode == 2 && !cpu_rows.empty())
    GIDS_CHECK((uint64_t)cpu_rows.back() < n_rows, GIDS_E_RANGE, "pinned node id outside the feature range");
  const uint64_t lim = cpu_mode == 1 ? std::min<uint64_t>(count, n_rows) : count;
  parallel_for(lim, host_threads(), [&](uint64_t lo, uint64_t hi) {
    for (uint64_t k = lo; k < hi; k++) {
      const uint64_t r = cpu_mode == 1 ? k : (uint64_t)cpu_rows[k];
      backing_read(*ctrls, cpu_buf.host + k * stride, row_bytes, r * src_stride);
    }
  });
  if (cpu_mode == 1 && lim < cpu_len) cpu_len = lim;  // seq rows past the range are never pinned
  cpu_filled_stride = src_stride_elems;
}

void Store::store_tensor(const void* src, uint64_t num_rows, uint64_t offset_bytes) {
  // gids_nvme.cu:616-663 + gids_kernel.cu:378-389: row r (of page_size /
  // elem_bytes elements) of the range gets elements [r*dim + off, (r+1)*dim +
  // off) of src, off = offset_bytes / elem_bytes.
  const uint64_t dim = page_size / elem_bytes;
  const uint64_t nbytes = num_rows * dim * elem_bytes;
  const uint64_t src_off = offset_bytes / elem_bytes * elem_bytes;
  write_range((const char*)src + src_off, nbytes, 0);
}

void Store::write_range(const void* src, uint64_t nbytes, uint64_t off) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "write before init_controllers");
  GIDS_CHECK(off + nbytes <= (uint64_t)n_pages * page_size, GIDS_E_RANGE, "write past the end of the range");
  if (!nbytes) return;
  GIDS_CHECK(src, GIDS_E_INVAL, "null source");
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  cudaPointerAttributes attr{};
  GIDS_CUDA(cudaPointerGetAttributes(&attr, src));
  if (attr.type == cudaMemoryTypeDevice) {
    // stage device data through a pinned bounce buffer
    const uint64_t chunk = 256ull << 20;
    char* bounce = nullptr;
    GIDS_CUDA(cudaMallocHost(&bounce, std::min(chunk, nbytes)));
    try {
      for (uint64_t done = 0; done < nbytes; done += chunk) {
        const uint64_t len = std::min(chunk, nbytes - done);
        GIDS_CUDA(cudaMemcpy(bounce, (const char*)src + done, len, cudaMemcpyDeviceToHost));
        backing_write(*ctrls, bounce, len, off + done);
      }
    } catch (...) {
      cudaFreeHost(bounce);
      throw;
    }
    cudaFreeHost(bounce);
  } else {
    backing_write(*ctrls, src, nbytes, off);
  }
  // the cache and the CPU buffer may hold stale copies of the written pages
  // (a sharded cache drops this rank's shard; every rank has to flush)
  GIDS_CUDA(cudaMemset(d_state, 0, n_entries_local() * sizeof(unsigned long long)));
  if (n_slots) {
    GIDS_CUDA(cudaMemset(d_slot_page, 0xFF, n_slots * sizeof(unsigned long long)));
    GIDS_CUDA(cudaMemset(d_slot_ref, 0, n_slots));
  }
  clear_window_pins();
  if (cpu_mode && cpu_filled_stride) fill_cpu_buffer(cpu_filled_stride);
  GIDS_CUDA(cudaDeviceSynchronize());
}

// Drops every window-buffer pin of this rank's shard (the whole range when
// unsharded). A marked window that is never gathered would otherwise keep
// its lines from being evicted for good.
void Store::clear_window_pins() {
  if (d_wb) GIDS_CUDA(cudaMemset(d_wb, 0, (world == 1 ? n_lines : n_entries_local()) * sizeof(unsigned int)));
  wb_marked = false;
}

void Store::flush_cache() {
  // The cache never holds dirty pages (writes go straight to the backing
  // store), so flushing only has to drop every resident page, and with them
  // every window-buffer pin. A sharded cache drops this rank's shard: all
  // ranks flush, with no gather in flight.
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "flush_cache before init_controllers");
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  GIDS_CUDA(cudaMemset(d_state, 0, n_entries_local() * sizeof(unsigned long long)));
  if (n_slots) {
    GIDS_CUDA(cudaMemset(d_slot_page, 0xFF, n_slots * sizeof(unsigned long long)));
    GIDS_CUDA(cudaMemset(d_slot_ref, 0, n_slots));
  }
  // and forget which lines missed once; the clock restarts, so the empty
  // cache admits every miss again
  const ShardLayout L(n_entries_local(), n_slots, line_size, world > 1);
  GIDS_CUDA(cudaMemset(d_shard + L.seen, 0, L.seen_bytes));
  GIDS_CUDA(cudaMemset(d_shard + L.clock, 0, 8));
  clear_window_pins();
  refs_since_seen_reset = 0;
  GIDS_CUDA(cudaDeviceSynchronize());
}

double Store::peer_copy_gbs(uint32_t peer, uint64_t bytes) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized && world > 1 && shards_ready, GIDS_E_STATE, "needs an attached sharded cache");
  GIDS_CHECK(peer < world && peer != rank, GIDS_E_INVAL, "peer must be another rank of the cache");
  const uint64_t have = shard_bytes & ~4095ull;
  bytes = std::min<uint64_t>(bytes & ~4095ull, have);
  GIDS_CHECK(bytes > 0, GIDS_E_INVAL, "nothing to copy");
  DeviceGuard g(device);
  // the peer's whole shard allocation: its base is the peer's page table
  const char* src = reinterpret_cast<const char*>(shards[peer].state);
  char* dst = nullptr;
  cudaStream_t st = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  double best = 0.0;
  GIDS_CUDA(cudaMalloc(&dst, bytes));
  try {
    GIDS_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    GIDS_CUDA(cudaEventCreate(&a));
    GIDS_CUDA(cudaEventCreate(&b));
    for (int rep = 0; rep < 4; rep++) {  // the first is a warm-up
      GIDS_CUDA(cudaEventRecord(a, st));
      GIDS_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st));
      GIDS_CUDA(cudaEventRecord(b, st));
      GIDS_CUDA(cudaEventSynchronize(b));
      float ms = 0.f;
      GIDS_CUDA(cudaEventElapsedTime(&ms, a, b));
      if (rep && ms > 0.f) best = std::max(best, (double)bytes / 1e9 / (ms / 1e3));
    }
  } catch (...) {
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (st) cudaStreamDestroy(st);
    cudaFree(dst);
    throw;
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaStreamDestroy(st);
  cudaFree(dst);
  return best;
}

double Store::host_read_gbs(uint32_t read_bytes, uint64_t total_bytes) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "host_read_gbs before init_controllers");
  GIDS_CHECK(read_bytes >= 512 && read_bytes <= 4096 && 4096 % read_bytes == 0 && read_bytes <= line_size,
             GIDS_E_INVAL, "read size must be 512, 1024, 2048 or 4096 bytes and at most one cache line");
  DeviceGuard g(device);
  const uint64_t dst_bytes = 256ull << 20;
  const uint64_t reads = std::max<uint64_t>(1, total_bytes / read_bytes);
  // lines that lie in the physically held pages
  const uint64_t lines = std::min<uint64_t>(n_lines, ctrls->wrap_pages << (page_shift - line_shift));
  char* dst = nullptr;
  cudaEvent_t a = nullptr, b = nullptr;
  double best = 0.0;
  GIDS_CUDA(cudaMalloc(&dst, dst_bytes));
  try {
    GIDS_CUDA(cudaEventCreate(&a));
    GIDS_CUDA(cudaEventCreate(&b));
    for (int rep = 0; rep < 4; rep++) {  // the first is a warm-up
      GIDS_CUDA(cudaEventRecord(a, 0));
      launch_host_probe(dev_backing(), lines, line_shift, read_bytes, reads, dst, dst_bytes, 1234567ull * (rep + 1),
                        0);
      GIDS_CUDA(cudaEventRecord(b, 0));
      GIDS_CUDA(cudaEventSynchronize(b));
      float ms = 0.f;
      GIDS_CUDA(cudaEventElapsedTime(&ms, a, b));
      if (rep && ms > 0.f) best = std::max(best, (double)(reads * read_bytes) / 1e9 / (ms / 1e3));
    }
  } catch (...) {
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    cudaFree(dst);
    throw;
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaFree(dst);
  return best;
}

void Store::synchronize() {
  std::lock_guard<std::mutex> lk(mu);
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  fold_events(true);
  check_async_error();
}

void Store::get_stats(uint64_t* out, int count) {
  std::lock_guard<std::mutex> lk(mu);
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  unsigned long long h[GIDS_STAT_COUNT];
  GIDS_CUDA(cudaMemcpy(h, d_stats, sizeof(h), cudaMemcpyDeviceToHost));
  h[GIDS_STAT_LAUNCHES] = launches;
  for (int i = 0; i < count && i < GIDS_STAT_COUNT; i++) out[i] = h[i];
}

void Store::reset_stats() {
  std::lock_guard<std::mutex> lk(mu);
  DeviceGuard g(device);
  GIDS_CUDA(cudaDeviceSynchronize());
  GIDS_CUDA(cudaMemset(d_stats, 0, GIDS_STAT_COUNT * sizeof(unsigned long long)));
  fold_events(true);
  kernel_ms = 0.0;
  total_access = 0;
  launches = 0;
  stat_base_cpu = 0;
}

double Store::kernel_time_ms() {
  std::lock_guard<std::mutex> lk(mu);
  DeviceGuard g(device);
  fold_events(true);
  return kernel_ms;
}

uint32_t Store::cpu_access_count() {
  uint64_t s[GIDS_STAT_COUNT];
  get_stats(s, GIDS_STAT_COUNT);
  return (uint32_t)(s[GIDS_STAT_CPU_ROWS] - stat_base_cpu);
}

void Store::flush_cpu_access_count() {
  uint64_t s[GIDS_STAT_COUNT];
  get_stats(s, GIDS_STAT_COUNT);
  stat_base_cpu = s[GIDS_STAT_CPU_ROWS];
}

void Store::print_stats() {
  uint64_t s[GIDS_STAT_COUNT];
  get_stats(s, GIDS_STAT_COUNT);
  const double ms = kernel_time_ms();
  const double hr = s[GIDS_STAT_ACCESS] ? (double)s[GIDS_STAT_HIT] / (double)s[GIDS_STAT_ACCESS] : 0.0;
  printf("print stats: access %" PRIu64 " hit %" PRIu64 " miss %" PRIu64 " read_io %" PRIu64 " bypass %" PRIu64
         " evictions %" PRIu64 " hit_rate %.4f\n",
         s[GIDS_STAT_ACCESS], s[GIDS_STAT_HIT], s[GIDS_STAT_MISS], s[GIDS_STAT_READ_IO], s[GIDS_STAT_BYPASS],
         s[GIDS_STAT_EVICTIONS], hr);
  printf("cpu buffer rows: %" PRIu64 "  rows: %" PRIu64 "  wait timeouts: %" PRIu64 "  bad ids: %" PRIu64 "\n",
         s[GIDS_STAT_CPU_ROWS], s[GIDS_STAT_ROWS], s[GIDS_STAT_WAIT_TIMEOUT], s[GIDS_STAT_BAD_IDS]);
  printf("Kernel Time: \t %f\n", ms);
  printf("Total Access: \t %" PRIu64 "\n", total_access);
  fflush(stdout);
  reset_stats();
}

}  // namespace gids
