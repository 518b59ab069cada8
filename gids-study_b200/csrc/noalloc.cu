// gids_read_feature_noalloc: the feature gather without any device allocation.
//
// Some callers cannot call cudaMalloc: a process whose GPU memory is owned by
// another allocator with a hard budget (a serving runtime or a framework's
// caching allocator that reserved the device up front), where a cudaMalloc
// fails or takes memory the pool has promised elsewhere. This entry point
// gathers exactly what gids_read_feature gathers, from the same store's
// backing store and constant CPU buffer, but the page cache its kernel works
// in (page table, slot tags, clock bits, resident pages, counters) lives in
// the file-scope array below instead of the store's HBM allocations, which it
// neither reads nor writes.
//
// Properties a caller relies on:
//  * the array is kNoallocScratchBytes (32 MiB) on every GPU where it has
//    been loaded, held until the process exits. CUDA loads a module's device
//    arrays lazily, so the first call on a device is the one that makes the
//    32 MiB resident (the driver reserves it while loading the module): make
//    that first call early -- before another allocator reserves the rest of
//    the device -- and before any stream capture. It also looks the array's
//    device address up (cudaGetSymbolAddress, with that device current) and
//    keeps it. Later calls allocate nothing;
//  * its counters (rows, hits, misses, CPU-buffer rows, ...) are added to the
//    store's statistics after each call by one small stream-ordered kernel,
//    so gids_get_stats and gids_get_cpu_access_count include its rows;
//  * every call starts from an empty cache: it clears the counters, the clock
//    and the page table of the store's range on its stream before the launch,
//    so a page fetched by several rows of one call crosses the host link once,
//    and nothing carries over between calls (the array keeps the last call's
//    contents until the next call clears them);
//  * the array is shared by all calls on a device: calls that overlap on the
//    GPU (different streams, or an asynchronous store called again before the
//    previous call finished) race on it;
//  * a store whose page table does not fit (more than about 4M cache lines) is
//    rejected with GIDS_E_RANGE before anything is launched;
//  * no cudaMalloc, cudaFree or other allocating call is made.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "gids_internal.hpp"

namespace gids {
namespace {

constexpr uint64_t kNoallocScratchBytes = 32ull << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_addr_mu;
char* g_addr[64] = {};  // device address of g_noalloc_scratch per device

char* scratch_address(int device) {
  GIDS_CHECK(device >= 0 && device < 64, GIDS_E_INVAL, "device index out of range");
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[device]) {
    DeviceGuard g(device);
    void* p = nullptr;
    // host code must not take &g_noalloc_scratch: that is a host-side stand-in
    GIDS_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_addr[device] = (char*)p;
  }
  return g_addr[device];
}

uint64_t up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Adds the per-call counters kept in the scratch to the store's counters.
__global__ void add_counters_kernel(unsigned long long* __restrict__ dst, const unsigned long long* __restrict__ src,
                                    int n) {
  const int i = threadIdx.x;
  if (i < n && src[i]) atomicAdd(dst + i, src[i]);
}

}  // namespace

void Store::read_noalloc(void* out, const int64_t* idx, int64_t n, int dim, int cache_dim, uint64_t key_off,
                         cudaStream_t st) {
  std::lock_guard<std::mutex> lk(mu);
  GIDS_CHECK(initialized, GIDS_E_STATE, "read before init_controllers");
  GIDS_CHECK(n >= 0, GIDS_E_INVAL, "n must be >= 0");
  GIDS_CHECK(dim > 0 && cache_dim > 0 && dim <= cache_dim, GIDS_E_INVAL, "need 0 < dim <= cache_dim");
  GIDS_CHECK(n == 0 || (out && idx), GIDS_E_INVAL, "null output or index pointer");
  // layout of the scratch: counters | clock | page table | slot tags | clock bits | slots
  const uint64_t off_stats = 0, off_clock = 256, off_state = 512;
  const uint64_t off_tags = up(off_state + n_lines * 8, 256);
  GIDS_CHECK(off_tags <= kNoallocScratchBytes, GIDS_E_RANGE,
             "gids_read_feature_noalloc: the range has " + std::to_string(n_lines) +
                 " cache lines; its page table does not fit the " + std::to_string(kNoallocScratchBytes >> 20) +
                 " MiB no-allocation scratch (at most " + std::to_string((kNoallocScratchBytes - 512) / 8) +
                 " lines)");
  DeviceGuard g(device);
  check_async_error();
  char* base = scratch_address(device);
  const uint64_t room = kNoallocScratchBytes - off_tags;
  // slot tags (8 B) + clock bit (1 B) + page bytes per slot, pages 4 KB-aligned
  uint64_t ns = room / (line_size + 9);
  while (ns && up(off_tags + ns * 8, 256) + up(ns, 256) > kNoallocScratchBytes) ns--;
  uint64_t off_ref = up(off_tags + ns * 8, 256);
  uint64_t off_slots = up(off_ref + ns, 4096);
  while (ns && off_slots + ns * (uint64_t)line_size > kNoallocScratchBytes) {
    ns--;
    off_ref = up(off_tags + ns * 8, 256);
    off_slots = up(off_ref + ns, 4096);
  }

  const uint64_t row_bytes = (uint64_t)dim * elem_bytes;
  const uint64_t src_stride = (uint64_t)cache_dim * elem_bytes;
  if (cpu_mode) {
    GIDS_CHECK((uint64_t)dim <= cpu_dim, GIDS_E_INVAL,
               "dim exceeds the constant CPU buffer's row width (cpu_backing_buffer dim)");
    if (cpu_filled_stride != (uint32_t)cache_dim) fill_cpu_buffer((uint32_t)cache_dim);
  }
  uint64_t gst = src_stride, b = line_size;
  while (b) {
    const uint64_t t = gst % b;
    gst = b;
    b = t;
  }
  const uint64_t max_pages = (line_size - gst + row_bytes - 1) / line_size + 1;
  uint32_t seg_shift = 0;
  while ((1ull << seg_shift) < max_pages) seg_shift++;
  GIDS_CHECK(seg_shift <= 5, GIDS_E_UNSUPPORTED, "a row may span more than 32 cache lines; use larger lines");
  int vec = 16;
  while (vec > 2 && (row_bytes % vec || src_stride % vec || (uint64_t)(uintptr_t)out % vec)) vec >>= 1;
  GIDS_CHECK(row_bytes % vec == 0 && src_stride % vec == 0, GIDS_E_INVAL, "rows must be 2-byte aligned");
  GIDS_CHECK(n == 0 || (uintptr_t)idx % 8 == 0, GIDS_E_INVAL, "index array must be 8-byte aligned");
  if (n == 0) return;

  // clear what must start at zero (INVALID pages, no counts, clock at 0) and
  // mark every slot empty; the slot bytes need no clearing
  GIDS_CUDA(cudaMemsetAsync(base + off_stats, 0, 512, st));
  GIDS_CUDA(cudaMemsetAsync(base + off_state, 0, n_lines * 8, st));
  if (ns) {
    GIDS_CUDA(cudaMemsetAsync(base + off_tags, 0xFF, ns * 8, st));
    GIDS_CUDA(cudaMemsetAsync(base + off_ref, 0, ns, st));
  }

  GatherArgs a;
  memset(&a, 0, sizeof(a));
  a.c.sh[0].state = (unsigned long long*)(base + off_state);
  a.c.sh[0].slot_page = (unsigned long long*)(base + off_tags);
  a.c.sh[0].slot_ref = (unsigned char*)(base + off_ref);
  a.c.sh[0].wb = nullptr;
  a.c.sh[0].slots = base + off_slots;
  a.c.sh[0].clock = (unsigned long long*)(base + off_clock);
  a.c.n_slots = ns;
  a.c.n_pages = n_lines;
  a.c.page_shift = line_shift;
  a.c.page_size = line_size;
  a.c.world = 1;
  a.c.rank = 0;
  a.c.ref_max = 1;  // per-call cache: second-chance clock, every miss admitted (seen = nullptr)
  a.b = dev_backing();
  a.cpu = dev_cpu();
  a.stats = (unsigned long long*)(base + off_stats);
  a.host_err = d_err;
  a.src_stride = src_stride;
  a.n_rows = range_bytes >= row_bytes ? (range_bytes - row_bytes) / src_stride + 1 : 0;
  a.row_bytes = (uint32_t)row_bytes;
  a.seg_shift = seg_shift;
  a.spin_limit = wait_limit;
  a.sweep_limit = 64;
  a.k = 1;
  a.t[0].idx = idx;
  a.t[0].out = (char*)out;
  a.t[0].n = (uint64_t)n;
  a.t[0].key_off = key_off;
  a.t[0].chunk_begin = 0;
  const uint64_t rpc = 32ull >> seg_shift;
  a.total_chunks = ((uint64_t)n + rpc - 1) / rpc;
  const int vi = vec == 16 ? 0 : vec == 8 ? 1 : vec == 4 ? 2 : 3;
  const uint64_t want_blocks = (a.total_chunks + (GATHER_THREADS / 32) - 1) / (GATHER_THREADS / 32);
  const int grid = (int)std::min<uint64_t>(want_blocks, (uint64_t)grid_blocks[0][vi]);
  launch_gather(a, vec, false, grid, st);
  static_assert(GIDS_STAT_COUNT <= 32, "one warp adds the counters");
  add_counters_kernel<<<1, 32, 0, st>>>(d_stats, a.stats, GIDS_STAT_COUNT);
  GIDS_CUDA(cudaGetLastError());
  launches++;
  total_access += (uint64_t)n;
  last_stream = st;
  if (synchronous) {
    GIDS_CUDA(cudaStreamSynchronize(st));
    check_async_error();
  }
}

}  // namespace gids

extern "C" int gids_read_feature_noalloc(gids_store_t* s, void* out, const int64_t* idx, int64_t n, int dim,
                                         int cache_dim, uint64_t key_off, void* stream) {
  try {
    GIDS_CHECK(s != nullptr, GIDS_E_INVAL, "s is null");
    gids_store_of(s)->read_noalloc(out, idx, n, dim, cache_dim, key_off, (cudaStream_t)stream);
    gids::clear_last_error();
    return GIDS_OK;
  } catch (const gids::Error& e) {
    gids::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    gids::set_last_error(e.what());
    return GIDS_E_INVAL;
  } catch (...) {
    gids::set_last_error("unknown error");
    return GIDS_E_INVAL;
  }
}
