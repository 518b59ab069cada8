// Emulated SSDs: the backing store of the feature range.
//
// The reference reads features from NVMe SSDs opened through libnvm
// (GIDS_Controllers, gids_nvme.cu:93-107) with pages striped over the SSDs
// in ssd_list order (page_cache_backup.h:626-652, STRIPE). Here every SSD is a
// page-addressed region of host memory, pinned and mapped into the GPU's
// address space, so a cache miss is a zero-copy read over the host link.
// Regions come from mmap with transparent huge pages and are pinned with
// cudaHostRegister (about ten times faster to pin than cudaHostAlloc at tens
// of GB). With a path pattern, an SSD is a shared file mapping, so its
// contents outlive the process and can be shared by one process per GPU.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

#include "gids_internal.hpp"

namespace gids {

void parallel_for(uint64_t n, int threads, const std::function<void(uint64_t, uint64_t)>& fn) {
  if (n == 0) return;
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > n) threads = (int)n;
  if (threads == 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  th.reserve(threads);
  for (int t = 0; t < threads; t++) {
    const uint64_t lo = n / threads * t, hi = t == threads - 1 ? n : n / threads * (t + 1);
    th.emplace_back([&fn, lo, hi]() { fn(lo, hi); });
  }
  for (auto& x : th) x.join();
}

namespace {
int hw_threads() {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

bool cuda_device_present() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

// Spread a mapping's pages over all online NUMA nodes (MPOL_INTERLEAVE via
// the raw mbind syscall; best effort, nothing to do on a single-node host),
// so that GPUs attached to different sockets share the memory bandwidth of
// all sockets when they read the backing store.
void interleave_numa(void* p, uint64_t bytes) {
  FILE* f = fopen("/sys/devices/system/node/online", "r");
  if (!f) return;
  char buf[256] = {0};
  const size_t n = fread(buf, 1, sizeof(buf) - 1, f);
  fclose(f);
  if (!n) return;
  unsigned long mask[16] = {0};
  int count = 0;
  for (char* tok = strtok(buf, ",\n"); tok; tok = strtok(nullptr, ",\n")) {
    int a = -1, b = -1;
    if (sscanf(tok, "%d-%d", &a, &b) == 2) {
    } else if (sscanf(tok, "%d", &a) == 1) {
      b = a;
    } else {
      continue;
    }
    for (int i = a; i <= b && i >= 0 && i < 1024; i++) {
      mask[i / 64] |= 1ul << (i % 64);
      count++;
    }
  }
  if (count < 2) return;
  constexpr int kMpolInterleave = 3;
  syscall(SYS_mbind, p, bytes, kMpolInterleave, mask, 1024ul, 0u);
}

// Touch every page so that the region is backed (and huge pages are formed)
// before it is pinned. Anonymous memory is zeroed; file memory is only read.
void prefault(char* p, uint64_t bytes, bool write_zero, int threads) {
  const uint64_t step = 1ull << 21;
  const uint64_t n = (bytes + step - 1) / step;
  parallel_for(n, threads, [&](uint64_t lo, uint64_t hi) {
    for (uint64_t i = lo; i < hi; i++) {
      const uint64_t a = i * step, len = std::min(step, bytes - a);
      if (write_zero) {
        memset(p + a, 0, len);
      } else {
        volatile char s = 0;
        for (uint64_t o = 0; o < len; o += 4096) s ^= p[a + o];
        (void)s;
      }
    }
  });
}
}  // namespace

// ------------------------------------------------------------ PinnedHost
void PinnedHost::alloc(uint64_t nbytes, int threads) {
  release();
  if (!nbytes) return;
  void* p = mmap(nullptr, nbytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
  GIDS_CHECK(p != MAP_FAILED, GIDS_E_NOMEM, "mmap of " + std::to_string(nbytes) + " bytes failed");
  madvise(p, nbytes, MADV_HUGEPAGE);
  interleave_numa(p, nbytes);
  host = (char*)p;
  bytes = nbytes;
  prefault(host, bytes, true, threads);
  cudaError_t e = cudaHostRegister(host, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) {
    munmap(host, bytes);
    host = nullptr;
    bytes = 0;
    throw Error(GIDS_E_CUDA, std::string("cudaHostRegister: ") + cudaGetErrorString(e));
  }
  void* d = nullptr;
  GIDS_CUDA(cudaHostGetDevicePointer(&d, host, 0));
  dev = (char*)d;
}

void PinnedHost::release() {
  if (host) {
    cudaHostUnregister(host);
    munmap(host, bytes);
  }
  host = dev = nullptr;
  bytes = 0;
}

// ------------------------------------------------------------ Controllers
Controllers::~Controllers() {
  for (auto& s : ssd) {
    if (!s.host) continue;
    if (s.registered) cudaHostUnregister(s.host);
    munmap(s.host, s.bytes);
    if (s.fd >= 0) close(s.fd);
  }
}

void Controllers::init(uint32_t n, uint64_t qd, uint64_t nq, const int32_t* list) {
  GIDS_CHECK(!bound, GIDS_E_STATE, "controllers already bound to a store");
  GIDS_CHECK(n >= 1 && n <= GIDS_MAX_SSD, GIDS_E_INVAL, "n_ctrls must be in [1, 32]");
  n_ctrls = n;
  q_depth = qd;
  n_queues = nq;
  ssd_list.assign(n, 0);
  for (uint32_t i = 0; i < n; i++) ssd_list[i] = list ? list[i] : (int32_t)i;
}

void Controllers::set_emulation(uint64_t cap, const char* pat) {
  GIDS_CHECK(!bound, GIDS_E_STATE, "set_emulation after the controllers were bound");
  capacity_per_ssd = cap;
  pattern = pat ? pat : "";
}

uint64_t Controllers::bind(uint32_t n, uint32_t ps, uint64_t start, uint64_t pages) {
  if (bound) {  // reuse a binding made with the same geometry
    GIDS_CHECK(n == n_bound && ps == page_size && start == page_start && pages == range_pages, GIDS_E_STATE,
               "controllers already bound with a different geometry");
    return wrap_pages;
  }
  GIDS_CHECK(n_ctrls >= n, GIDS_E_STATE, "init_GIDS_controllers first");
  page_size = ps;
  page_start = start;
  range_pages = pages;
  n_bound = n;
  const uint64_t need = start + (pages + n - 1) / n;  // pages per SSD
  uint64_t cap_pages = need;
  wrap_pages = pages;
  if (capacity_per_ssd) {
    cap_pages = capacity_per_ssd / ps;
    GIDS_CHECK(cap_pages > start, GIDS_E_INVAL, "SSD capacity does not reach past read_off");
    if (cap_pages < need) wrap_pages = (cap_pages - start) * n;  // multiple of n: SSD of page p stays p % n
    else cap_pages = need;
  }
  if (wrap_pages == 0) wrap_pages = 1;
  const uint64_t bytes = cap_pages * (uint64_t)ps;
  ssd.assign(n, SsdRegion{});
  const int threads = hw_threads();
  try {
  for (uint32_t i = 0; i < n; i++) {
    SsdRegion& s = ssd[i];
    s.bytes = bytes;
    if (!pattern.empty()) {
      std::string path = pattern;
      const size_t at = path.find("{}");
      const std::string id = std::to_string(ssd_list[i]);
      if (at != std::string::npos) path.replace(at, 2, id);
      else path += id;
      s.path = path;
      s.fd = open(path.c_str(), O_RDWR | O_CREAT, 0644);
      GIDS_CHECK(s.fd >= 0, GIDS_E_IO, "cannot open emulated SSD " + path);
      struct stat stt{};
      fstat(s.fd, &stt);
      if ((uint64_t)stt.st_size < bytes)
        GIDS_CHECK(ftruncate(s.fd, (off_t)bytes) == 0, GIDS_E_IO, "cannot size emulated SSD " + path);
      void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, s.fd, 0);
      GIDS_CHECK(p != MAP_FAILED, GIDS_E_IO, "cannot map emulated SSD " + path);
      s.host = (char*)p;
      madvise(p, bytes, MADV_HUGEPAGE);
      interleave_numa(p, bytes);
      prefault(s.host, bytes, false, threads);
    } else {
      void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
      GIDS_CHECK(p != MAP_FAILED, GIDS_E_NOMEM, "cannot allocate emulated SSD of " + std::to_string(bytes) + " bytes");
      s.host = (char*)p;
      madvise(p, bytes, MADV_HUGEPAGE);
      interleave_numa(p, bytes);
      prefault(s.host, bytes, true, threads);
    }
  }
  } catch (...) {  // release what was mapped before the failure
    for (auto& r : ssd) {
      if (r.host) munmap(r.host, r.bytes);
      if (r.fd >= 0) close(r.fd);
    }
    ssd.clear();
    throw;
  }
  bound = true;
  return wrap_pages;
}

void Controllers::register_with_cuda() {
  if (!cuda_device_present()) return;
  for (auto& s : ssd) {
    if (s.registered || !s.host) continue;
    GIDS_CUDA(cudaHostRegister(s.host, s.bytes, cudaHostRegisterMapped | cudaHostRegisterPortable));
    void* d = nullptr;
    GIDS_CUDA(cudaHostGetDevicePointer(&d, s.host, 0));
    s.dev = (char*)d;
    s.registered = true;
  }
}

// ------------------------------------------------------------ striped I/O
const char* backing_page_host(const Controllers& c, uint64_t p) {
  const uint64_t q = p % c.wrap_pages;
  const uint64_t k = q % c.n_bound;
  const uint64_t dp = c.page_start + q / c.n_bound;
  return c.ssd[k].host + dp * c.page_size;
}

namespace {
template <typename F>
void for_pages(const Controllers& c, uint64_t nbytes, uint64_t off, int threads, F&& f) {
  GIDS_CHECK(c.bound, GIDS_E_STATE, "backing store not bound");
  if (!nbytes) return;
  const uint64_t ps = c.page_size;
  const uint64_t p0 = off / ps, p1 = (off + nbytes - 1) / ps;
  parallel_for(p1 - p0 + 1, nbytes >= (64ull << 20) ? threads : 1, [&](uint64_t lo, uint64_t hi) {
    for (uint64_t i = lo; i < hi; i++) {
      const uint64_t p = p0 + i;
      const uint64_t a = std::max(off, p * ps), b = std::min(off + nbytes, (p + 1) * ps);
      f(p, a - p * ps, a - off, b - a);
    }
  });
}
}  // namespace

void backing_write(Controllers& c, const void* src, uint64_t nbytes, uint64_t off) {
  const char* s = (const char*)src;
  for_pages(c, nbytes, off, hw_threads(), [&](uint64_t p, uint64_t in_page, uint64_t src_off, uint64_t len) {
    memcpy(const_cast<char*>(backing_page_host(c, p)) + in_page, s + src_off, len);
  });
}

void backing_read(const Controllers& c, void* dst, uint64_t nbytes, uint64_t off) {
  char* d = (char*)dst;
  for_pages(c, nbytes, off, hw_threads(), [&](uint64_t p, uint64_t in_page, uint64_t dst_off, uint64_t len) {
    memcpy(d + dst_off, backing_page_host(c, p) + in_page, len);
  });
}

// ------------------------------------------------------ synthetic content
// Element e of stream `seed` is the e-th output of SplitMix64 (Steele, Lea,
// Flood, OOPSLA 2014) seeded with `seed`, mapped to the element type with
// integer arithmetic only, so every value is exact:
//   kind 1, fp32: top 24 bits k, value k * 2^-23 - 1 (uniform on [-1, 1));
//   kind 2, fp16: m = (sum of the 8 bytes) - 1020, value m * 2^-8
//                 (bell-shaped, mean 0, sd about 0.82, exact in fp16);
//   kind 3, int64: the raw 64-bit output;
//   kind 4, fp16: normal(0, 1) by the Box-Muller transform (Box and Muller,
//                 Ann. Math. Statist. 1958) of the two 32-bit halves,
//                 u1 = (hi + 1) 2^-32 in (0, 1], u2 = lo 2^-32 in [0, 1):
//                 sqrt(-2 ln u1) cos(2 pi u2) in double, rounded to fp16 by
//                 the compiler's _Float16 conversion (round to nearest even).
//                 The host's libm computes it, here and in the oracle alike.
namespace {
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ULL;
inline uint64_t sm_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
inline uint64_t synth_u64(uint64_t seed, uint64_t e) { return sm_mix(seed + (e + 1) * kGolden); }
inline uint32_t synth_f32(uint64_t h) {
  const float v = (float)(uint32_t)(h >> 40) * (1.0f / 8388608.0f) - 1.0f;
  uint32_t b;
  memcpy(&b, &v, 4);
  return b;
}
inline uint16_t synth_f16(uint64_t h) {
  int32_t s = 0;
  for (int i = 0; i < 8; i++) s += (int32_t)((h >> (8 * i)) & 0xFF);
  const int32_t m = s - 1020;
  if (m == 0) return 0;
  const uint16_t sign = m < 0 ? 0x8000 : 0;
  const uint32_t a = (uint32_t)(m < 0 ? -m : m);
  const int e = 31 - __builtin_clz(a);
  return (uint16_t)(sign | ((uint16_t)(e + 7) << 10) | (uint16_t)((a << (10 - e)) & 0x3FF));
}
inline uint16_t synth_f16_normal(uint64_t h) {
  const double u1 = ((double)(h >> 32) + 1.0) * 0x1p-32;
  const double u2 = (double)(h & 0xFFFFFFFFull) * 0x1p-32;
  const _Float16 v = (_Float16)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
  uint16_t b;
  memcpy(&b, &v, 2);
  return b;
}
}  // namespace

int synth_elem_bytes(int kind) { return kind == 1 ? 4 : (kind == 2 || kind == 4) ? 2 : kind == 3 ? 8 : 0; }

void backing_fill_synthetic(Controllers& c, int kind, uint64_t seed, int threads) {
  const int eb = synth_elem_bytes(kind);
  GIDS_CHECK(eb, GIDS_E_INVAL, "unknown synthetic kind");
  GIDS_CHECK(c.bound, GIDS_E_STATE, "backing store not bound");
  if (threads <= 0) threads = hw_threads();
  const uint64_t per_page = c.page_size / eb;
  // physical page q (q < wrap_pages) holds logical page q
  parallel_for(c.wrap_pages, threads, [&](uint64_t lo, uint64_t hi) {
    for (uint64_t q = lo; q < hi; q++) {
      char* dst = const_cast<char*>(backing_page_host(c, q));
      const uint64_t e0 = q * per_page;
      if (kind == 1) {
        uint32_t* d = (uint32_t*)dst;
        for (uint64_t i = 0; i < per_page; i++) d[i] = synth_f32(synth_u64(seed, e0 + i));
      } else if (kind == 2) {
        uint16_t* d = (uint16_t*)dst;
        for (uint64_t i = 0; i < per_page; i++) d[i] = synth_f16(synth_u64(seed, e0 + i));
      } else if (kind == 4) {
        uint16_t* d = (uint16_t*)dst;
        for (uint64_t i = 0; i < per_page; i++) d[i] = synth_f16_normal(synth_u64(seed, e0 + i));
      } else {
        uint64_t* d = (uint64_t*)dst;
        for (uint64_t i = 0; i < per_page; i++) d[i] = synth_u64(seed, e0 + i);
      }
    }
  });
}

}  // namespace gids
