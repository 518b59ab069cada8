// Feature-gather kernels for sm_100a.
//
// One kernel serves every read entry point of the reference's
// BAM_Feature_Store (read_feature, read_feature_hetero, read_feature_merged,
// read_feature_merged_hetero; gids_nvme.cu:324-593) and both of its kernels
// (read_feature_kernel and read_feature_kernel_with_cpu_backing_memory,
// gids_kernel.cu:60-175):
//
//   out_t[i, 0:dim] = range[(idx_t[i] + key_off_t) * cache_dim + (0:dim)]
//
// Work is split into chunks of 32 lanes. A chunk covers 32 >> seg_shift rows
// and each row gets (1 << seg_shift) lanes, one per page the row can touch,
// so the lookups of a whole chunk run in parallel instead of one dependent
// chain per row. Per chunk a warp:
//   1. loads the node ids, checks them against the range, and looks rows up in
//      the constant CPU buffer (bitmap + rank, in L2);
//   2. deduplicates page references inside the warp (__match_any_sync, the
//      reference's coalesce_page, page_cache_backup.h:1514-1550) and lets one
//      leader per page take `count` references on the page-table word;
//   3. fills the pages it won (BUSY) from the emulated SSDs after a warp-wide
//      clock sweep for victim slots (as many candidates per atomic on the
//      hand as it has pages to place), and publishes them VALID; once the
//      cache is full, a page's first miss in the admission window is read
//      straight from the backing store instead of being inserted;
//   4. waits, with a bound, for pages another warp is filling; a wait that
//      runs out, or a fill that found no slot, reads the page straight from
//      the backing store (always correct: the store is read-only here);
//   5. copies the chunk's segments: slot-sourced ones through a TMA ring in
//      shared memory (16-byte kernels), the rest with vector loads/stores,
//      eight vectors in flight per lane; then drops its page references.
// The state-word protocol follows range_d_t::acquire_page/release_page
// (page_cache_backup.h:1278-1403, 1166-1229) with a 64-bit word that also
// holds the slot; eviction follows find_slot (:2107-2256) with a clock
// counter per slot (chances left) and every spin bounded.
#include <cuda_runtime.h>

#include <mutex>

#include "gids_internal.hpp"

namespace gids {
namespace {

// ------------------------------------------------------------ scoped atomics
// SYS = false: the cache is private to this GPU (gpu scope).
// SYS = true:  shards live on several GPUs and are read and filled over
//              NVLink, so every state-word operation uses system scope.
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_add_acquire(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.acquire.sys.global.add.u64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.acquire.gpu.global.add.u64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_or_acquire(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.acquire.sys.global.or.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.acquire.gpu.global.or.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_or_relaxed(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.relaxed.sys.global.or.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.relaxed.gpu.global.or.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ void atom_and_relaxed(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.relaxed.sys.global.and.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.relaxed.gpu.global.and.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  (void)r;
}
template <bool SYS>
__device__ __forceinline__ void red_add_release(unsigned long long* p, unsigned long long v) {
  if (SYS)
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
  else
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_add_relaxed(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.relaxed.sys.global.add.u64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.relaxed.gpu.global.add.u64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_cas_acq_rel(unsigned long long* p, unsigned long long cmp,
                                                               unsigned long long val) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.acq_rel.sys.global.cas.b64 %0, [%1], %2, %3;" : "=l"(r) : "l"(p), "l"(cmp), "l"(val) : "memory");
  else
    asm volatile("atom.acq_rel.gpu.global.cas.b64 %0, [%1], %2, %3;" : "=l"(r) : "l"(p), "l"(cmp), "l"(val) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long atom_exch_relaxed(unsigned long long* p, unsigned long long v) {
  unsigned long long r;
  if (SYS)
    asm volatile("atom.relaxed.sys.global.exch.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  else
    asm volatile("atom.relaxed.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(r) : "l"(p), "l"(v) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
  unsigned long long r;
  if (SYS)
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  else
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
  unsigned long long r;
  if (SYS)
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int* p) {
  unsigned int r;
  if (SYS)
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
template <bool SYS>
__device__ __forceinline__ unsigned int atom_cas_u32(unsigned int* p, unsigned int cmp, unsigned int val) {
  unsigned int r;
  if (SYS)
    asm volatile("atom.relaxed.sys.global.cas.b32 %0, [%1], %2, %3;" : "=r"(r) : "l"(p), "r"(cmp), "r"(val) : "memory");
  else
    asm volatile("atom.relaxed.gpu.global.cas.b32 %0, [%1], %2, %3;" : "=r"(r) : "l"(p), "r"(cmp), "r"(val) : "memory");
  return r;
}

// ------------------------------------------------------------ vector copies
template <int VEC>
struct VecT;
template <>
struct VecT<16> {
  using T = int4;
};
template <>
struct VecT<8> {
  using T = int2;
};
template <>
struct VecT<4> {
  using T = int;
};
template <>
struct VecT<2> {
  using T = short;
};

struct SegDesc {
  const char* src;  // nullptr: write zeros
  char* dst;
  uint32_t len;
  uint32_t pad;
};

constexpr int WARPS = GATHER_THREADS / 32;
constexpr int INFLIGHT = 8;  // vectors in flight per lane

// Copies the first nseg segments of sd with the whole warp. Control flow is
// warp-uniform: every lane walks the same (segment, block) cursor.
template <int VEC>
__device__ __forceinline__ void copy_segments(const SegDesc* sd, int nseg, int lane) {
  using V = typename VecT<VEC>::T;
  int j = 0;
  uint32_t m = 0;
  while (j < nseg) {
    V v[INFLIGHT];
    char* dp[INFLIGHT];
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++) {
      dp[q] = nullptr;
      if (j < nseg) {
        const uint32_t len = sd[j].len;
        const uint32_t off = (m * 32u + (uint32_t)lane) * VEC;
        if (off < len) {
          const char* s = sd[j].src;
          dp[q] = sd[j].dst + off;
          if (s)
            v[q] = __ldcg(reinterpret_cast<const V*>(s + off));
          else
            v[q] = V{};
        }
        m++;
        if (m * 32u * VEC >= len) {
          m = 0;
          j++;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++)
      if (dp[q]) __stcs(reinterpret_cast<V*>(dp[q]), v[q]);
  }
}

// ------------------------------------------------------------ TMA bulk copies
// Segments whose source is a cache slot (a hit, or a line another warp filled)
// are moved HBM -> shared -> output by the tensor memory accelerator rather
// than through registers: one lane per warp issues `cp.async.bulk` loads into
// the warp's ring of TMA_STAGES shared-memory stages (completion counted in
// bytes on each stage's mbarrier) and bulk stores from each completed stage to
// the output rows. Bytes in flight are then bounded by shared memory instead
// of the registers the lookups and fills already need. Only the 16-byte-vector
// kernels use it (bulk copies need 16-byte aligned addresses and sizes).
constexpr int TMA_STAGES = 3;
constexpr uint32_t TMA_STAGE_BYTES = 4096;
constexpr uint32_t TMA_WAIT_LIMIT = 1u << 22;  // mbarrier polls before a stage is given up

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long* b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, uint32_t parity) {
  uint32_t ok = 0;
  for (uint32_t it = 0; it < TMA_WAIT_LIMIT && !ok; it++)
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_load(char* sdst, const char* gsrc, uint32_t bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(sdst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store(char* gdst, const char* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}

// One warp's pipeline over n segments, run by one lane, its state in shared
// memory: stage k of the ring holds the k-th 4 KB of the segments'
// concatenation (pieces of several small segments share a stage). issue()
// starts the loads of the first stages; drain() completes every stage in
// order, stores it to the output, and refills it.
struct TmaPipe {
  const SegDesc* sd;
  char* ring;
  unsigned long long* bar;
  int n, jp, jc, issued, done;
  uint32_t op, oc;
  uint32_t sb[TMA_STAGES];
  uint32_t phase;  // parity of each stage's next completion
  uint32_t pend;   // stages whose loads were given up on and have not completed since
  int live;        // cleared for good if a stage ever fails to complete

  __device__ __forceinline__ bool pack(int s) {
    if (jp >= n) return false;
    uint32_t fill = 0;
    int j = jp;
    uint32_t o = op;
    while (j < n && fill < TMA_STAGE_BYTES) {
      const uint32_t take = min(sd[j].len - o, TMA_STAGE_BYTES - fill);
      fill += take;
      o += take;
      if (o == sd[j].len) {
        j++;
        o = 0;
      }
    }
    sb[s] = fill;
    mbar_expect_tx(bar + s, fill);
    char* const dst = ring + (size_t)s * TMA_STAGE_BYTES;
    fill = 0;
    while (jp < n && fill < TMA_STAGE_BYTES) {
      const uint32_t take = min(sd[jp].len - op, TMA_STAGE_BYTES - fill);
      bulk_load(dst + fill, sd[jp].src + op, take, bar + s);
      fill += take;
      op += take;
      if (op == sd[jp].len) {
        jp++;
        op = 0;
      }
    }
    return true;
  }
  __device__ __forceinline__ void issue(const SegDesc* segs, int count, char* r, unsigned long long* b) {
    sd = segs;
    n = count;
    ring = r;
    bar = b;
    jp = jc = issued = done = 0;
    op = oc = 0;
    // the previous chunk's bulk stores may still be reading the ring
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    // the slots were written through the generic proxy (fills, made visible by
    // the acquire on their page-table words); order them before the bulk reads
    asm volatile("fence.proxy.async.global;" ::: "memory");
    for (int s = 0; s < TMA_STAGES && pack(s); s++) issued++;
  }
  // Waits (bounded) for the bulk loads of every stage that was issued but
  // not completed; true when none is left in flight. After a stage wait gave
  // up, this decides whether the ring's shared memory and the slots the loads
  // read can be let go (see the give-up path in the kernel).
  __device__ __forceinline__ bool quiesce() {
    // at most TMA_STAGES stages are in flight, each on its own mbarrier; the
    // ones still outstanding are kept in `pend` across calls
    if (done < issued) {
      for (int k = done; k < issued; k++) pend |= 1u << (k % TMA_STAGES);
      done = issued;
    }
    for (int s = 0; s < TMA_STAGES; s++) {
      if (!((pend >> s) & 1u)) continue;
      bool ok = false;
      for (int rep = 0; rep < 4 && !ok; rep++) ok = mbar_wait(bar + s, (phase >> s) & 1u);
      if (ok) {
        phase ^= 1u << s;
        pend &= ~(1u << s);
      }
    }
    return pend == 0;
  }
  // false: a stage did not complete within the limit (the caller copies the
  // segments again another way)
  __device__ __forceinline__ bool drain() {
    while (done < issued) {
      const int s = done % TMA_STAGES;
      if (!mbar_wait(bar + s, (phase >> s) & 1u)) return false;
      phase ^= 1u << s;
      const char* const src = ring + (size_t)s * TMA_STAGE_BYTES;
      uint32_t used = 0;
      while (used < sb[s]) {
        const uint32_t take = min(sd[jc].len - oc, sb[s] - used);
        bulk_store(sd[jc].dst + oc, src + used, take);
        used += take;
        oc += take;
        if (oc == sd[jc].len) {
          jc++;
          oc = 0;
        }
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      done++;
      if (jp < n) {
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // the stage has been read out
        if (pack(s)) issued++;
      }
    }
    return true;
  }
};

// Whole-page fill from the backing store into a cache slot (16-byte vectors;
// pages are >= 512 B, power-of-two sized, and page-aligned on both sides).
// With FWD, the segments of the rows in `mem` (lanes whose rows read this
// page: in-page offset `ip`, length `ln`, output `dp`, all 16-byte aligned)
// are stored to the output from the same registers ("fill-forward"), so the
// copy phase does not read the slot back.
template <bool FWD>
__device__ __forceinline__ void fill_page(const char* __restrict__ src, char* __restrict__ dst, uint32_t page_size,
                                          int lane, unsigned mem, uint32_t ip, uint32_t ln, char* dp) {
  for (uint32_t base = 0; base < page_size; base += 32u * 16u * INFLIGHT) {
    int4 v[INFLIGHT];
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++) {
      const uint32_t off = base + ((uint32_t)q * 32u + (uint32_t)lane) * 16u;
      if (off < page_size) v[q] = __ldcg(reinterpret_cast<const int4*>(src + off));
    }
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++) {
      const uint32_t off = base + ((uint32_t)q * 32u + (uint32_t)lane) * 16u;
      if (off < page_size) __stcg(reinterpret_cast<int4*>(dst + off), v[q]);
    }
    if (FWD) {
      unsigned mm = mem;
      while (mm) {
        const int j = __ffs(mm) - 1;
        mm &= mm - 1;
        const uint32_t jip = __shfl_sync(0xffffffffu, ip, j);
        const uint32_t jln = __shfl_sync(0xffffffffu, ln, j);
        char* const jdp = reinterpret_cast<char*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dp), j));
#pragma unroll
        for (int q = 0; q < INFLIGHT; q++) {
          const uint32_t off = base + ((uint32_t)q * 32u + (uint32_t)lane) * 16u;
          if (off >= jip && off < jip + jln) __stcs(reinterpret_cast<int4*>(jdp + (off - jip)), v[q]);
        }
      }
    }
  }
}

// Address of cache line l on the emulated SSDs: its stripe page p (after the
// wrap) lives on SSD p % n at device page page_start + p / n
// (page_cache_backup.h:626-652, STRIPE); the line sits at its offset in p.
__device__ __forceinline__ const char* backing_addr(const DevBacking& b, uint64_t l, uint32_t line_shift) {
  const uint64_t p = l >> b.lpp_shift;
  const uint64_t q = p % b.wrap_pages;
  const uint32_t c = (uint32_t)(q % b.n_ssd);
  const uint64_t dp = b.page_start + q / b.n_ssd;
  return b.ssd[c] + (dp << b.page_shift) + ((l & ((1ull << b.lpp_shift) - 1ull)) << line_shift);
}

// Saturating decrement of the window-buffer part of a line's pin word (the
// permanent-pin bit is kept). The CAS loop runs until it lands or the count
// reads 0: every failed CAS means another thread changed the word, so the
// loop is bounded by the contention on this one word, and no pin is left
// behind when it is contended.
template <bool SYS>
__device__ __forceinline__ void wb_consume(unsigned int* w, unsigned int cnt) {
  unsigned int v = ld_relaxed_u32<SYS>(w);
  while (v & WB_COUNT_MASK) {
    const unsigned int c = v & WB_COUNT_MASK;
    const unsigned int nv = (v & WB_PERMANENT) | (c > cnt ? c - cnt : 0u);
    const unsigned int r = atom_cas_u32<SYS>(w, v, nv);
    if (r == v) break;
    v = r;
  }
}

enum {
  K_ROWS, K_CPU, K_BAD, K_ACCESS, K_HIT, K_MISS, K_BYPASS, K_READIO, K_TIMEOUT,
  K_BHIT, K_BMISS, K_BBYP, K_BCPU, K_EVICT, K_BPEER, K_PREFETCH,
#ifdef GIDS_PHASE_TIMERS
  K_TLOOK, K_TFILL, K_TCOPY, K_TREL,
#endif
  K_N
};
__constant__ int kStatMap[K_N] = {GIDS_STAT_ROWS,       GIDS_STAT_CPU_ROWS,     GIDS_STAT_BAD_IDS,
                                  GIDS_STAT_ACCESS,     GIDS_STAT_HIT,          GIDS_STAT_MISS,
                                  GIDS_STAT_BYPASS,     GIDS_STAT_READ_IO,      GIDS_STAT_WAIT_TIMEOUT,
                                  GIDS_STAT_BYTES_HIT,  GIDS_STAT_BYTES_MISS,   GIDS_STAT_BYTES_BYPASS,
                                  GIDS_STAT_BYTES_CPU,  GIDS_STAT_EVICTIONS,    GIDS_STAT_BYTES_PEER,
                                  GIDS_STAT_PREFETCHED,
#ifdef GIDS_PHASE_TIMERS
                                  GIDS_STAT_NS_LOOKUP,  GIDS_STAT_NS_FILL,      GIDS_STAT_NS_COPY,
                                  GIDS_STAT_NS_RELEASE,
#endif
};

#ifdef GIDS_PHASE_TIMERS
// Build option for diagnosis (build.py with GIDS_PHASE_TIMERS=1): lane 0 of
// every warp adds the nanoseconds (globaltimer) each chunk spends in the
// lookup, fill-and-wait, copy and release phases to four extra counters. The
// default build compiles none of it.
__device__ __forceinline__ unsigned long long phase_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define GIDS_PHASE_MARK(v) const unsigned long long v = phase_clock()
#else
#define GIDS_PHASE_MARK(v)
#endif

// PF: a prefetch launch (window-buffer prefetch): the tuples have no output;
// the rows' lines are brought into the cache and nothing is copied out. It is
// a separate instantiation so that the gather itself carries none of it.
template <int VEC, bool SYS, bool PF = false>
__global__ void __launch_bounds__(GATHER_THREADS, 2) gather_kernel(const __grid_constant__ GatherArgs a) {
  __shared__ SegDesc seg_sh[WARPS][32];
  __shared__ unsigned long long cnt_sh[WARPS][K_N];  // warp-private counters
  __shared__ unsigned char fill_lane[WARPS][8];      // owner lanes of one fill batch
  __shared__ unsigned char gate_sh[GIDS_MAX_WORLD];   // shard filters first misses (full, admission on)
  __shared__ __align__(8) unsigned long long tma_bar[WARPS][TMA_STAGES];
  __shared__ TmaPipe tma_pipe_sh[WARPS];
  extern __shared__ __align__(128) char tma_ring_sh[];  // WARPS x TMA_STAGES x 4 KB (VEC == 16)
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  SegDesc* sd = seg_sh[wib];
  unsigned long long* acc = cnt_sh[wib];
  if (lane < K_N) acc[lane] = 0;
  TmaPipe& pipe = tma_pipe_sh[wib];
  if (VEC == 16 && lane == 0) {
    for (int s = 0; s < TMA_STAGES; s++) mbar_init(&tma_bar[wib][s]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    pipe.phase = 0;
    pipe.pend = 0;
    pipe.live = 1;
  }
  __syncwarp();
  // a shard admits every miss until its clock hand has gone round once (the
  // cache is full); read once per block, a stale "not full" only admits more
  if (threadIdx.x < GIDS_MAX_WORLD)
    gate_sh[threadIdx.x] = threadIdx.x < a.c.world && a.c.sh[threadIdx.x].seen &&
                           ld_relaxed<SYS>(a.c.sh[threadIdx.x].clock) >= a.c.n_slots;
  __syncthreads();
  const uint32_t seg_shift = a.seg_shift;
  const uint32_t seg_mask = (1u << seg_shift) - 1u;
  const uint32_t rpc = 32u >> seg_shift;
  const uint32_t shift = a.c.page_shift;
  const uint64_t psize = a.c.page_size;
  const bool have_cache = a.c.n_slots != 0;
  const uint64_t n_warps = (uint64_t)gridDim.x * WARPS;

  int ti = 0;
  for (uint64_t chunk = (uint64_t)blockIdx.x * WARPS + wib; chunk < a.total_chunks; chunk += n_warps) {
    while (ti + 1 < a.k && a.t[ti + 1].chunk_begin <= chunk) ti++;
    const GatherTuple& T = a.t[ti];
    constexpr bool pf = PF;
    const uint64_t row = (chunk - T.chunk_begin) * rpc + ((uint32_t)lane >> seg_shift);
    const uint32_t sidx = (uint32_t)lane & seg_mask;
    const bool row_ok = row < T.n;

    GIDS_PHASE_MARK(tph0);
    // ---- 1. node id, range check, constant CPU buffer lookup
    int64_t id = row_ok ? __ldg(T.idx + row) : 0;
    const uint64_t r = (uint64_t)id + T.key_off;
    const bool bad = row_ok && (id < 0 || r >= a.n_rows);
    const bool live = row_ok && !bad;
    bool pinned = false;
    uint64_t cpu_slot = 0;
    if (live && a.cpu.mode == 1) {
      pinned = r < a.cpu.seq_len;
      cpu_slot = r;
    } else if (live && a.cpu.mode == 2) {
      const uint64_t w = r >> 6;
      if (w < a.cpu.nwords) {
        const unsigned long long bits = __ldg(a.cpu.bits + w);
        const unsigned long long below = bits & ((1ull << (r & 63)) - 1ull);
        if ((bits >> (r & 63)) & 1ull) {
          pinned = true;
          cpu_slot = (uint64_t)__ldg(a.cpu.rank + w) + (uint64_t)__popcll(below);
        }
      }
    }

    // ---- page segment of this lane, and the shard that owns the page
    const uint64_t b0 = r * a.src_stride;
    const uint64_t p_first = b0 >> shift;
    const uint64_t p_last = (b0 + a.row_bytes - 1) >> shift;
    const uint64_t p = p_first + sidx;
    const bool seg_ok = live && !pinned && p <= p_last;
    uint32_t s0 = 0, s1 = 0;
    if (seg_ok) {
      const uint64_t pb = p << shift;
      s0 = (uint32_t)((pb > b0 ? pb : b0) - b0);
      const uint64_t pe = pb + psize, re = b0 + a.row_bytes;
      s1 = (uint32_t)((pe < re ? pe : re) - b0);
    }
    // the shard that holds the line and its page-table entry there: line
    // p % world at p / world, or a replicated line in this rank's own shard
    uint32_t owner = 0u;
    uint64_t lp = p;  // index in the owner's page table
    if (SYS) {
      const LineHome h = line_home(a.c, seg_ok ? p : 0ull);
      owner = seg_ok ? h.owner : 0u;
      lp = h.entry;
    }
    const DevShard& S = a.c.sh[owner];

    // ---- 2. warp dedup + acquire (one leader per distinct page)
    const unsigned long long key = seg_ok ? (unsigned long long)p : (~0ull - (unsigned long long)lane);
    const unsigned eq = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(eq) - 1;
    const bool is_leader = seg_ok && leader == lane;
    const unsigned cnt = __popc(eq);
    int cls = CLS_NONE;
    uint64_t slot = 0;
    unsigned long long* stw = S.state + (seg_ok ? lp : 0);
    const bool took_ref = is_leader && have_cache;
    if (is_leader) {
      if (!have_cache) {
        cls = CLS_BYPASS;
      } else {
        const unsigned long long old = atom_add_acquire<SYS>(stw, cnt);
        if (old & ST_VALID) {
          cls = CLS_HIT;
          slot = old >> ST_SLOT_SHIFT;
        } else if (old & ST_BUSY) {
          cls = CLS_WAIT;
        } else {
          // a miss: without an admission bit from an earlier miss in this
          // window, read the line straight from the backing store
          // (a line that window buffering has pinned for later batches is
          // admitted at once)
          // (a line with a permanent pin counts as pinned for good). With the
          // pinned-only policy the cache holds the permanently pinned lines
          // alone and every other line is read through.
          bool admit = true;
          // A prefetch applies the same rule without setting the admission
          // bit: it inserts the lines the gather would insert (pinned for a
          // later batch, or missed before in this window) ahead of time, and
          // leaves lines the gather would read through to that gather, so the
          // cache holds what it would hold without the prefetch.
          if (a.c.pinned_only) {
            admit = S.wb && (ld_relaxed_u32<SYS>(S.wb + lp) & WB_PERMANENT) != 0u;
          } else if (gate_sh[owner] && !(S.wb && ld_relaxed_u32<SYS>(S.wb + lp) > cnt)) {
            const unsigned long long bit = 1ull << (lp & 63);
            admit = ((pf ? ld_relaxed<SYS>(S.seen + (lp >> 6)) : atom_or_relaxed<SYS>(S.seen + (lp >> 6), bit)) &
                     bit) != 0;
          }
          if (!admit) {
            cls = CLS_BYPASS;
          } else {
            const unsigned long long prev = atom_or_acquire<SYS>(stw, ST_BUSY);
            if (prev & ST_VALID) {
              cls = CLS_HIT;
              slot = prev >> ST_SLOT_SHIFT;
            } else if (prev & ST_BUSY) {
              cls = CLS_WAIT;
            } else {
              cls = CLS_OWN;
            }
          }
        }
      }
    }

    // output row and, for cache-path lanes, the segment's place in its page
    char* const orow = row_ok && !pf ? T.out + row * (uint64_t)a.row_bytes : nullptr;
    const uint32_t in_pg = seg_ok ? (uint32_t)((b0 + s0) - (p << shift)) : 0u;
    bool forwarded = false;

    GIDS_PHASE_MARK(tph1);
    // ---- 3. fills: per owning shard, a warp-cooperative clock sweep for
    //         victim slots (32 candidates per atomic on that shard's hand)
    unsigned pending = __ballot_sync(0xffffffffu, cls == CLS_OWN);
    if (pending) {
      unsigned todo = pending;
      while (todo) {
        const uint32_t tgt = __shfl_sync(0xffffffffu, owner, __ffs(todo) - 1);
        unsigned grp = todo & __ballot_sync(0xffffffffu, owner == tgt);
        todo &= ~grp;
        const DevShard& V = a.c.sh[tgt];
        for (uint32_t round = 0; grp && round < a.sweep_limit; round++) {
          // the hand passes only as many slots as there are owners to place,
          // doubling per round when candidates are still in use: passing more
          // would spend chances of slots no fill needed and age the cache
          // faster than lines are replaced
          const uint32_t m = min(32u, (uint32_t)__popc(grp) << min(round, 5u));
          unsigned long long base = 0;
          if (lane == 0) base = atom_add_relaxed<SYS>(V.clock, (unsigned long long)m);
          base = __shfl_sync(0xffffffffu, base, 0);
          const bool looks = (uint32_t)lane < m;
          const uint64_t s = (base + (uint64_t)lane) % a.c.n_slots;
          const unsigned long long q = looks ? ld_relaxed<SYS>(V.slot_page + s) : 0ull;
          bool cand = false;
          unsigned long long expect = 0;
          if (!looks) {
          } else if (q == SLOT_EMPTY) {
            cand = true;
          } else if (const unsigned char rr = V.slot_ref[s]) {
            V.slot_ref[s] = rr - 1;  // the clock hand spends one chance
          } else {
            const unsigned long long st = ld_relaxed<SYS>(V.state + q);
            if (st == (((unsigned long long)s << ST_SLOT_SHIFT) | ST_VALID) &&
                (!V.wb || ld_relaxed_u32<SYS>(V.wb + q) == 0)) {
              cand = true;
              expect = st;
            }
          }
          unsigned cmask = __ballot_sync(0xffffffffu, cand);
          while (cmask && grp) {
            const int c = __ffs(cmask) - 1;
            cmask &= cmask - 1;
            const int o = __ffs(grp) - 1;
            const unsigned long long newp = __shfl_sync(0xffffffffu, (unsigned long long)lp, o);
            int ok = 0;
            if (lane == c) {
              if (q == SLOT_EMPTY) {
                ok = atom_cas_acq_rel<SYS>(V.slot_page + s, SLOT_EMPTY, newp) == SLOT_EMPTY;
              } else if (atom_cas_acq_rel<SYS>(V.state + q, expect, 0ull) == expect) {
                atom_exch_relaxed<SYS>(V.slot_page + s, newp);
                atomicAdd(acc + K_EVICT, 1ull);
                ok = 1;
              }
            }
            ok = __shfl_sync(0xffffffffu, ok, c);
            if (ok) {
              const unsigned long long sl = __shfl_sync(0xffffffffu, (unsigned long long)s, c);
              if (lane == o) slot = sl;
              grp &= ~(1u << o);
              pending &= ~(1u << o);
            }
          }
        }
      }
      // owners without a slot give the fill up and read the backing store
      if ((pending >> lane) & 1u) {
        atom_and_relaxed<SYS>(stw, ~ST_BUSY);
        cls = CLS_BYPASS;
      }
      unsigned fills = __ballot_sync(0xffffffffu, cls == CLS_OWN);
      if (shift <= 12) {
        // Lines of at most 4 KB: one 4 KB block of 8 vectors per lane covers
        // 8 >> (shift - 9) lines, so that many fills share one round trip over
        // the host link. Vector q of every lane belongs to line q >> (shift - 9)
        // of the batch: warp-uniform, so owners are broadcast reads.
        const uint32_t qsh = shift - 9;
        const int per_batch = 8 >> qsh;
        unsigned char* const bl = fill_lane[wib];
        while (fills) {
          int nb = 0;
          if (lane == 0) {
            unsigned f = fills;
            for (; nb < per_batch && f; nb++) {
              bl[nb] = (unsigned char)(__ffs(f) - 1);
              f &= f - 1;
            }
          }
          nb = __shfl_sync(0xffffffffu, nb, 0);
          __syncwarp();
          unsigned batch = 0;
          for (int j = 0; j < nb; j++) batch |= 1u << bl[j];
          fills &= ~batch;
          const uint32_t qmask = (1u << qsh) - 1u;
          int4 v[INFLIGHT];
          const char* sq = nullptr;
#pragma unroll
          for (int q = 0; q < INFLIGHT; q++) {
            const int j = q >> qsh;
            if (j < nb) {
              if (((uint32_t)q & qmask) == 0) {  // first vector of line j: its source address
                const unsigned long long po = __shfl_sync(0xffffffffu, (unsigned long long)p, bl[j]);
                sq = backing_addr(a.b, po, shift);
              }
              const uint32_t off = (((uint32_t)q << 9) + ((uint32_t)lane << 4)) & (a.c.page_size - 1u);
              v[q] = __ldcg(reinterpret_cast<const int4*>(sq + off));
            }
          }
          char* dq = nullptr;
          unsigned mm = 0;
#pragma unroll
          for (int q = 0; q < INFLIGHT; q++) {
            const int j = q >> qsh;
            if (j < nb) {
              if (((uint32_t)q & qmask) == 0) {  // first vector of line j: its slot and readers
                const int o = bl[j];
                const unsigned long long so = __shfl_sync(0xffffffffu, (unsigned long long)slot, o);
                const uint32_t ow = __shfl_sync(0xffffffffu, owner, o);
                dq = a.c.sh[ow].slots + (so << shift);
                mm = __shfl_sync(0xffffffffu, eq, o);  // lanes whose rows read line j
                if (VEC == 16 && !pf && ((mm >> lane) & 1u)) forwarded = true;
              }
              const uint32_t off = (((uint32_t)q << 9) + ((uint32_t)lane << 4)) & (a.c.page_size - 1u);
              __stcg(reinterpret_cast<int4*>(dq + off), v[q]);
              if (VEC == 16 && !pf) {  // fill-forward: the rows of line j straight from registers
                unsigned rest = mm;
                while (rest) {
                  const int m = __ffs(rest) - 1;
                  rest &= rest - 1;
                  const uint32_t jip = __shfl_sync(0xffffffffu, in_pg, m);
                  const uint32_t jln = __shfl_sync(0xffffffffu, s1 - s0, m);
                  const unsigned long long jdp =
                      __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(orow + s0), m);
                  if (off >= jip && off < jip + jln)
                    __stcs(reinterpret_cast<int4*>(reinterpret_cast<char*>(jdp) + (off - jip)), v[q]);
                }
              }
            }
          }
          __syncwarp();
          if ((batch >> lane) & 1u) {
            // the release reduction orders the warp's slot stores (made visible
            // to this lane by __syncwarp) before the VALID bit
            red_add_release<SYS>(stw, ((unsigned long long)slot << ST_SLOT_SHIFT) + (ST_VALID - ST_BUSY));
            atomicAdd(acc + K_READIO, 1ull);
            if (pf) atomicAdd(acc + K_PREFETCH, 1ull);
          }
          __syncwarp();
        }
      }
      while (fills) {  // lines larger than 4 KB: one fill at a time, 4 KB blocks
        const int o = __ffs(fills) - 1;
        fills &= fills - 1;
        const unsigned long long po = __shfl_sync(0xffffffffu, (unsigned long long)p, o);
        const unsigned long long so = __shfl_sync(0xffffffffu, (unsigned long long)slot, o);
        const uint32_t ow = __shfl_sync(0xffffffffu, owner, o);
        const unsigned mem = __shfl_sync(0xffffffffu, eq, o);  // lanes whose rows read line po
        if (VEC == 16 && !pf) {
          fill_page<true>(backing_addr(a.b, po, shift), a.c.sh[ow].slots + (so << shift), a.c.page_size, lane, mem,
                          in_pg, s1 - s0, orow + s0);
          if ((mem >> lane) & 1u) forwarded = true;
        } else {
          fill_page<false>(backing_addr(a.b, po, shift), a.c.sh[ow].slots + (so << shift), a.c.page_size, lane,
                           0u, 0u, 0u, nullptr);
        }
        __syncwarp();
        if (lane == o) {
          red_add_release<SYS>(stw, (so << ST_SLOT_SHIFT) + (ST_VALID - ST_BUSY));
          acc[K_READIO]++;  // only lane o touches it here
          if (pf) acc[K_PREFETCH]++;
        }
      }
    }

    // ---- 4. bounded wait for pages filled by other warps (or other GPUs);
    //         a prefetch does not wait: the line is on its way into the cache
    if (pf && cls == CLS_WAIT) cls = CLS_BYPASS;
    if (__any_sync(0xffffffffu, cls == CLS_WAIT)) {
      unsigned ns = 32;
      for (uint32_t it = 0;; it++) {
        if (cls == CLS_WAIT) {
          const unsigned long long v = ld_acquire<SYS>(stw);
          if (v & ST_VALID) {
            cls = CLS_WAITED;
            slot = v >> ST_SLOT_SHIFT;
          } else if (!(v & ST_BUSY)) {
            cls = CLS_BYPASS;  // the filler gave up
          }
        }
        if (!__any_sync(0xffffffffu, cls == CLS_WAIT) || it + 1 >= a.spin_limit) break;
        __nanosleep(ns);
        if (ns < 2048) ns <<= 1;
      }
      if (cls == CLS_WAIT) {
        cls = CLS_BYPASS;
        atomicAdd(acc + K_TIMEOUT, 1ull);
      }
    }

    GIDS_PHASE_MARK(tph2);
    // ---- 5. segment table and copy
    const int gcls = __shfl_sync(0xffffffffu, cls, leader);
    const unsigned long long gslot = __shfl_sync(0xffffffffu, (unsigned long long)slot, leader);
    const char* src = nullptr;
    char* dst = nullptr;
    uint32_t len = 0;
    if (pf) {
      // a prefetch copies nothing out
    } else if (bad && sidx == 0) {
      len = a.row_bytes;  // zero row
      dst = orow;
    } else if (pinned && sidx == 0) {
      src = a.cpu.buf + cpu_slot * a.cpu.stride;
      dst = orow;
      len = a.row_bytes;
    } else if (seg_ok && !forwarded) {
      if (gcls == CLS_BYPASS)
        src = backing_addr(a.b, p, shift) + in_pg;
      else
        src = S.slots + (gslot << shift) + in_pg;
      dst = orow + s0;
      len = s1 - s0;
    }
    // slot-sourced segments go to the TMA pipeline (from the end of the table),
    // the rest (host, constant CPU buffer, zero rows) to the vector copy
    const bool via_tma = VEC == 16 && len && seg_ok && !forwarded && gcls != CLS_BYPASS && pipe.live;
    const unsigned tm = __ballot_sync(0xffffffffu, via_tma);
    const unsigned has = __ballot_sync(0xffffffffu, len != 0 && !via_tma);
    const unsigned below = (1u << lane) - 1u;
    if (via_tma)
      sd[31 - __popc(tm & below)] = SegDesc{src, dst, len, 0u};
    else if (len)
      sd[__popc(has & below)] = SegDesc{src, dst, len, 0u};
    __syncwarp();
    const int nt = __popc(tm);
    if (VEC == 16 && nt && lane == 0)
      pipe.issue(sd + (32 - nt), nt, tma_ring_sh + (size_t)wib * TMA_STAGES * TMA_STAGE_BYTES, tma_bar[wib]);
    copy_segments<VEC>(sd, __popc(has), lane);  // overlaps the bulk loads in flight
    bool keep_refs = false;
    if (VEC == 16 && nt) {
      bool ok = true;
      if (lane == 0) ok = pipe.drain();
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        // A bulk load did not complete within the wait limit. The warp records
        // it (GIDS_E_CUDA at the host), stops using the ring for good, and copies
        // this chunk's slot segments through registers (rewriting any bytes the
        // pipeline already stored with the same values). Loads still in flight
        // write only into the ring, which nothing reads any more, and read only
        // slots this chunk holds references on. Invariant: those references
        // are dropped only once every load of the ring has completed
        // (quiesce); if the loads are still outstanding after a second bounded
        // wait, the chunk keeps its references (the lines stay resident until
        // flush_cache) so no slot a load still reads can be evicted and
        // refilled. Kernel exit waits for them once more (below); a load that
        // never completes at all is the one case left undefined (the CTA exits
        // with it in flight), and it is reported.
        int q = 1;
        if (lane == 0) {
          pipe.live = 0;
          *reinterpret_cast<volatile int*>(a.host_err) = 2;
          q = pipe.quiesce();
        }
        keep_refs = __shfl_sync(0xffffffffu, q, 0) == 0;
        copy_segments<VEC>(sd + (32 - nt), nt, lane);
      }
    }
    __syncwarp();

    GIDS_PHASE_MARK(tph3);
    // ---- release, clock reference bit, window-buffer consumption
    if (took_ref && !keep_refs) {
      red_add_release<SYS>(stw, (unsigned long long)(-(long long)cnt));
      // one more chance, up to the ceiling (the static policy holds only
      // permanently pinned lines, which the clock never evicts: no counter)
      if (gcls != CLS_BYPASS && !a.c.pinned_only) {
        const unsigned char rr = S.slot_ref[gslot];
        if (rr < a.c.ref_max) S.slot_ref[gslot] = rr + 1;
      }
      // the gather of the row consumes its window pins (none to read unless
      // window buffering has marked lines since the pins were last cleared)
      if (S.wb && !pf && a.c.wb_marks) wb_consume<SYS>(S.wb + lp, cnt);
    }

#ifdef GIDS_PHASE_TIMERS
    {
      const unsigned long long tph4 = phase_clock();
      if (lane == 0) {
        acc[K_TLOOK] += tph1 - tph0;
        acc[K_TFILL] += tph2 - tph1;
        acc[K_TCOPY] += tph3 - tph2;
        acc[K_TREL] += tph4 - tph3;
      }
      __syncwarp();
    }
#endif
    // ---- counters
    if (bad && sidx == 0 && !pf) *reinterpret_cast<volatile int*>(a.host_err) = 1;
    const unsigned r0 = sidx == 0;
    const bool cached = seg_ok && (gcls == CLS_HIT || gcls == CLS_OWN || gcls == CLS_WAITED);
    const unsigned n_rows_c = __popc(__ballot_sync(0xffffffffu, row_ok && r0));
    const unsigned n_cpu = __popc(__ballot_sync(0xffffffffu, pinned && r0));
    const unsigned n_bad = __popc(__ballot_sync(0xffffffffu, bad && r0));
    const unsigned n_acc = __popc(__ballot_sync(0xffffffffu, seg_ok));
    const unsigned n_hit = __popc(__ballot_sync(0xffffffffu, seg_ok && gcls == CLS_HIT));
    const unsigned n_miss = __popc(__ballot_sync(0xffffffffu, seg_ok && (gcls == CLS_OWN || gcls == CLS_WAITED)));
    const unsigned n_byp = __popc(__ballot_sync(0xffffffffu, seg_ok && gcls == CLS_BYPASS));
    const unsigned sl = seg_ok ? s1 - s0 : 0u;  // segment bytes, copied or forwarded
    const unsigned lh = __reduce_add_sync(0xffffffffu, seg_ok && gcls == CLS_HIT ? sl : 0u);
    const unsigned lm = __reduce_add_sync(0xffffffffu, seg_ok && (gcls == CLS_OWN || gcls == CLS_WAITED) ? sl : 0u);
    const unsigned lb = __reduce_add_sync(0xffffffffu, seg_ok && gcls == CLS_BYPASS ? sl : 0u);
    const unsigned lc = __reduce_add_sync(0xffffffffu, pinned && r0 ? len : 0u);
    const unsigned lpeer = SYS ? __reduce_add_sync(0xffffffffu, cached && owner != a.c.rank && !forwarded ? sl : 0u)
                               : 0u;
    if (lane == 0 && !pf) {  // a prefetch counts only the lines it inserted
      acc[K_ROWS] += n_rows_c;
      acc[K_CPU] += n_cpu;
      acc[K_BAD] += n_bad;
      acc[K_ACCESS] += n_acc;
      acc[K_HIT] += n_hit;
      acc[K_MISS] += n_miss;
      acc[K_BYPASS] += n_byp;
      acc[K_BHIT] += lh;
      acc[K_BMISS] += lm;
      acc[K_BBYP] += lb;
      acc[K_BCPU] += lc;
      acc[K_BPEER] += lpeer;
    }
    __syncwarp();
  }

  __syncwarp();
  if (lane == 0) {
    if (VEC == 16) {
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // the output's bulk stores
      // loads given up on earlier: one more bounded wait before the CTA exits
      if (pipe.pend && !pipe.quiesce()) *reinterpret_cast<volatile int*>(a.host_err) = 2;
    }
#pragma unroll
    for (int i = 0; i < K_N; i++)
      if (acc[i]) atomicAdd(a.stats + kStatMap[i], acc[i]);
  }
}

// Window buffering: one thread per node id, +1 on the pin counter of every
// page its row touches, in the shard that owns the page (gids_kernel.cu:246-256
// marks one page per id). WB_UNMARK: -1 instead (saturating at 0), the marks
// of a window that will not be gathered are taken back. WB_PIN / WB_UNPIN:
// set / clear the permanent-pin bit of those pages.
__global__ void wb_mark_kernel(const __grid_constant__ WbArgs a) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  const int64_t id = a.idx[i];
  const int64_t rs = id + a.off;
  if (id < 0 || rs < 0 || (uint64_t)rs >= a.n_rows) return;  // the gather reports bad ids
  const uint64_t b0 = (uint64_t)rs * a.stride;
  const uint64_t p0 = b0 >> a.page_shift, p1 = (b0 + a.row_bytes - 1) >> a.page_shift;
  for (uint64_t p = p0; p <= p1; p++) {
    unsigned int* w = a.wb[0] + p;
    if (a.world > 1) {
      const LineHome h = line_home(a.home, p);
      w = a.wb[h.owner] + h.entry;
    }
    switch (a.mode) {
      case WB_MARK:
        if (a.world == 1)
          atomicAdd(w, 1u);
        else
          atomicAdd_system(w, 1u);
        break;
      case WB_UNMARK:
        if (a.world == 1)
          wb_consume<false>(w, 1u);
        else
          wb_consume<true>(w, 1u);
        break;
      case WB_PIN:
        if (a.world == 1)
          atomicOr(w, WB_PERMANENT);
        else
          atomicOr_system(w, WB_PERMANENT);
        break;
      default:
        if (a.world == 1)
          atomicAnd(w, ~WB_PERMANENT);
        else
          atomicAnd_system(w, ~WB_PERMANENT);
        break;
    }
  }
}

// Host-link probe: every warp reads `read_bytes` (512, 1024, 2048 or 4096)
// from the start of pseudo-random lines of the backing store, eight 16-byte
// vectors in flight per lane as in the gather's host copies, and stores them
// to a device buffer. Measures what the link delivers for the gather's own
// access size and footprint.
__global__ void __launch_bounds__(GATHER_THREADS, 2)
    host_probe_kernel(const DevBacking b, uint64_t n_lines, uint32_t line_shift, uint32_t read_bytes,
                      uint64_t reads, int4* __restrict__ dst, uint64_t dst_vecs, uint64_t seed) {
  const int lane = threadIdx.x & 31;
  const uint32_t per_round = 32u * 16u * INFLIGHT / read_bytes;  // reads per 4 KB round of a warp (>= 1)
  const uint32_t vecs = read_bytes / 16u;
  const uint64_t w = (uint64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  const uint64_t nw = (uint64_t)gridDim.x * WARPS;
  for (uint64_t r = w; r * per_round < reads; r += nw) {
    int4 v[INFLIGHT];
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++) {
      const uint32_t e = (uint32_t)q * 32u + (uint32_t)lane;  // vector index within the round
      const uint64_t k = r * per_round + e / vecs;             // read index
      unsigned long long z = seed + k * 0x9E3779B97F4A7C15ull;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      z ^= z >> 31;
      v[q] = __ldcg(reinterpret_cast<const int4*>(backing_addr(b, z % n_lines, line_shift)) + (e % vecs));
    }
#pragma unroll
    for (int q = 0; q < INFLIGHT; q++)
      __stcs(dst + ((r * (32u * INFLIGHT) + (uint64_t)q * 32u + (uint64_t)lane) % dst_vecs), v[q]);
  }
}

}  // namespace

void launch_host_probe(const DevBacking& b, uint64_t n_lines, uint32_t line_shift, uint32_t read_bytes,
                       uint64_t reads, void* dst, uint64_t dst_bytes, uint64_t seed, cudaStream_t st) {
  int sms = 0, dev = 0;
  GIDS_CUDA(cudaGetDevice(&dev));
  GIDS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  host_probe_kernel<<<2 * sms, GATHER_THREADS, 0, st>>>(b, n_lines, line_shift, read_bytes, reads,
                                                        reinterpret_cast<int4*>(dst), dst_bytes / 16, seed);
  GIDS_CUDA(cudaGetLastError());
}

constexpr size_t kTmaRingBytes = (size_t)WARPS * TMA_STAGES * TMA_STAGE_BYTES;

// the 16-byte-vector kernels take the TMA ring as dynamic shared memory; the
// attribute belongs to the current device, so it is set once per device
template <bool SYS>
static void allow_tma_ring() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  GIDS_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && done[dev]) return;
  GIDS_CUDA(cudaFuncSetAttribute(gather_kernel<16, SYS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kTmaRingBytes));
  if (dev >= 0 && dev < 64) done[dev] = true;
}

template <bool SYS>
static void launch_scoped(const GatherArgs& a, int vec, int grid, cudaStream_t st, bool prefetch) {
  if (prefetch) {  // copies nothing out: no TMA ring, any vector width
    gather_kernel<8, SYS, true><<<grid, GATHER_THREADS, 0, st>>>(a);
    return;
  }
  switch (vec) {
    case 16:
      allow_tma_ring<SYS>();
      gather_kernel<16, SYS><<<grid, GATHER_THREADS, kTmaRingBytes, st>>>(a);
      break;
    case 8: gather_kernel<8, SYS><<<grid, GATHER_THREADS, 0, st>>>(a); break;
    case 4: gather_kernel<4, SYS><<<grid, GATHER_THREADS, 0, st>>>(a); break;
    case 2: gather_kernel<2, SYS><<<grid, GATHER_THREADS, 0, st>>>(a); break;
    default: throw Error(GIDS_E_INVAL, "unsupported vector width");
  }
}

void launch_gather(const GatherArgs& a, int vec, bool sys, int grid, cudaStream_t st, bool prefetch) {
  if (sys)
    launch_scoped<true>(a, vec, grid, st, prefetch);
  else
    launch_scoped<false>(a, vec, grid, st, prefetch);
  GIDS_CUDA(cudaGetLastError());
}

template <bool SYS>
static int occupancy(int vec) {
  int n = 0;
  switch (vec) {
    case 16:
      allow_tma_ring<SYS>();
      GIDS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gather_kernel<16, SYS>, GATHER_THREADS, kTmaRingBytes));
      break;
    case 8: GIDS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gather_kernel<8, SYS>, GATHER_THREADS, 0)); break;
    case 4: GIDS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gather_kernel<4, SYS>, GATHER_THREADS, 0)); break;
    case 2: GIDS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gather_kernel<2, SYS>, GATHER_THREADS, 0)); break;
    default: throw Error(GIDS_E_INVAL, "unsupported vector width");
  }
  return n;
}

int gather_blocks_per_sm(int vec, bool sys) { return sys ? occupancy<true>(vec) : occupancy<false>(vec); }

void launch_wb_mark(const WbArgs& a, cudaStream_t st) {
  if (!a.n) return;
  const unsigned blocks = (unsigned)((a.n + 255) / 256);
  wb_mark_kernel<<<blocks, 256, 0, st>>>(a);
  GIDS_CUDA(cudaGetLastError());
}

}  // namespace gids
