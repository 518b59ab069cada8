// Multi-layer neighbour sampler over a CSC graph, and the in-degree-normalised
// PageRank of the constant CPU buffer's pin list, for sm_100a.
//
// Sampler: the node ids fetch_feature gathers come from DGL's
// MultiLayerNeighborSampler in the reference (GIDS_Setup/GIDS/GIDS.py:178-201,
// evaluation/homogenous_train.py:201-203). For fanouts [f_0 .. f_L-1], hop h
// (from the seeds outward) keeps, for every node of the current node set,
// min(f, in_degree) of its in-edges, and appends the new sources in order of
// first appearance; the final node set (seeds first) is the minibatch's
// input_nodes. The edges a node keeps are the ones with the smallest key
//   key(v, j) = (mix(mix(v * G + seed_h) + (j + 1) * M2) >> 25) << 24 | j
// (mix = the SplitMix64 finalizer; seed_h per sampler seed, call and hop), in
// increasing key order: a pure function of integers, so the torch
// restatement in GIDS/synthetic.py draws the same minibatch on any device.
//
// One call runs entirely on the device, with no host synchronisation between
// hops: the sizes of the node set and of each hop's candidates live in a small
// control block in device memory, and every kernel reads them there.
//   seeds  -> candidates [0, n_seeds)
//   hop h  -> one warp per node of the set picks its edges; candidate slot
//             i * f + r holds the r-th kept source of node i (or -1)
// After each step the candidates go through the same dedup: every candidate
// is inserted into an open-addressing hash table in HBM whose 64-bit word
// packs (node + 1) above its smallest position so far, so one atomicMin keeps
// the first occurrence; candidates whose own position is that minimum are new
// (nodes already in the set have smaller positions), and an order-preserving
// compaction (tile counts, one scan block, scatter) appends them.
//
// PageRank: page_rank_node_list_gen.py:126-134 (compute_pagerank): K times,
// pv = pv / in_degree; pv[v] = sum over in-edges u -> v of pv[u];
// pv = (1 - d) / N + d * pv, in float32. One warp per node sums its in-edges
// in CSC order, one add at a time, so the result is the sequential float32
// sum (the oracle's); nodes without in-edges contribute 0 (the reference
// divides by zero there).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "gids_internal.hpp"

namespace gids {
namespace {

constexpr int SMP_THREADS = 256;
constexpr int TILE = 4096;  // candidates per compaction tile (256 threads x 16)
constexpr int PER_THREAD = TILE / SMP_THREADS;
constexpr int POS_BITS = 30;  // candidate position bits of a table word
constexpr unsigned long long POS_MASK = (1ull << POS_BITS) - 1ull;
constexpr unsigned long long G_MUL = 0x9E3779B97F4A7C15ull;
constexpr unsigned long long M2_MUL = 0x94D049BB133111EBull;

__host__ __device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned long long edge_key(unsigned long long seed_h, unsigned long long v,
                                                       unsigned long long j) {
  unsigned long long z = mix64(v * G_MUL + seed_h);
  z = mix64(z + (j + 1ull) * M2_MUL);
  return ((z >> 25) << 24) | j;
}

struct SamplerCtl {
  unsigned long long n_nodes;     // nodes in the set so far
  unsigned long long pos_base;    // first position of the next round of candidates
  unsigned long long n_cand;      // candidates of the current round
  unsigned long long out_base;    // n_nodes before the current round's appends
  unsigned long long round_base;  // pos_base of the current round
  unsigned int err;  // 1: capacity exceeded, 2: table full, 4: seed outside the graph, 8: edge source outside
  unsigned int pad;
};

struct Graph {
  const long long* indptr;  // [n + 1]
  const void* indices;      // [edges], int32 or int64
  int index_bytes;
  unsigned long long n;
};

__device__ __forceinline__ long long edge_src(const Graph& g, unsigned long long e) {
  return g.index_bytes == 4 ? (long long)__ldg(reinterpret_cast<const int*>(g.indices) + e)
                            : __ldg(reinterpret_cast<const long long*>(g.indices) + e);
}

// The table word of node v: probe from its hash; insert it with position
// `pos` if absent, else keep the smaller position. Returns false if the
// table is full (cannot happen while it holds at most half its size).
__device__ __forceinline__ bool table_insert(unsigned long long* tab, unsigned long long mask, long long v,
                                             unsigned long long pos) {
  const unsigned long long tag = (unsigned long long)(v + 1) << POS_BITS;
  const unsigned long long word = tag | pos;
  unsigned long long h = mix64((unsigned long long)v) & mask;
  for (unsigned long long probe = 0; probe <= mask; probe++) {
    unsigned long long cur = tab[h];
    if (cur == 0ull) {
      cur = atomicCAS(tab + h, 0ull, word);
      if (cur == 0ull) return true;
    }
    if ((cur & ~POS_MASK) == tag) {
      atomicMin(tab + h, word);
      return true;
    }
    h = (h + 1ull) & mask;
  }
  return false;
}

__device__ __forceinline__ unsigned long long table_pos(const unsigned long long* tab, unsigned long long mask,
                                                        long long v) {
  const unsigned long long tag = (unsigned long long)(v + 1) << POS_BITS;
  unsigned long long h = mix64((unsigned long long)v) & mask;
  for (unsigned long long probe = 0; probe <= mask; probe++) {
    const unsigned long long cur = tab[h];
    if ((cur & ~POS_MASK) == tag) return cur & POS_MASK;
    if (cur == 0ull) break;
    h = (h + 1ull) & mask;
  }
  return ~0ull;
}

// ---- round 0: the seeds are the candidates
__global__ void seeds_kernel(const long long* __restrict__ seeds, unsigned long long n, long long* __restrict__ cand,
                             unsigned long long* __restrict__ tab, unsigned long long mask, unsigned long long n_graph,
                             SamplerCtl* ctl) {
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const long long v = seeds[i];
    cand[i] = v;
    if (v < 0 || (unsigned long long)v >= n_graph) {
      atomicOr(&ctl->err, 4u);
      cand[i] = -1;
      continue;
    }
    if (!table_insert(tab, mask, v, i)) atomicOr(&ctl->err, 2u);
  }
}

// ---- one hop: a warp per node of the set keeps min(f, deg) in-edges of
// smallest key; candidate slot i * f + r <- r-th kept source (or -1)
__global__ void __launch_bounds__(SMP_THREADS) hop_kernel(const Graph g, const long long* __restrict__ nodes,
                                                          long long* __restrict__ cand, unsigned long long cand_cap,
                                                          unsigned long long* __restrict__ tab,
                                                          unsigned long long mask, int f,
                                                          unsigned long long seed_h, SamplerCtl* ctl) {
  __shared__ unsigned long long sk[SMP_THREADS / 32][32];
  __shared__ unsigned int sj[SMP_THREADS / 32][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned long long n = ctl->n_nodes;
  const unsigned long long base = ctl->pos_base;
  if (n * (unsigned long long)f > cand_cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&ctl->err, 1u);
    return;
  }
  const unsigned long long nw = (unsigned long long)gridDim.x * (SMP_THREADS / 32);
  for (unsigned long long i = (unsigned long long)blockIdx.x * (SMP_THREADS / 32) + w; i < n; i += nw) {
    const long long v = nodes[i];
    const unsigned long long e0 = (unsigned long long)__ldg(g.indptr + v);
    const unsigned long long deg = (unsigned long long)__ldg(g.indptr + v + 1) - e0;
    const unsigned long long take = deg < (unsigned long long)f ? deg : (unsigned long long)f;
    unsigned long long kept_j = ~0ull;  // lane r < take: edge index of the r-th kept edge
    if (deg <= 32) {
      const unsigned long long k = (unsigned long long)lane < deg ? edge_key(seed_h, (unsigned long long)v, lane)
                                                                  : ~0ull;
      unsigned int rank = 0;
#pragma unroll 8
      for (int m = 0; m < 32; m++) rank += __shfl_sync(0xffffffffu, k, m) < k;
      if ((unsigned long long)lane < deg && rank < (unsigned int)f) {
        sk[w][rank] = k;
        sj[w][rank] = (unsigned int)lane;
      }
      __syncwarp();
      if ((unsigned long long)lane < take) kept_j = sj[w][lane];
      __syncwarp();
    } else {
      // running selection over tiles of 32 edges: lanes r < f hold the r-th
      // smallest key so far; each tile is merged by ranking all 64 entries
      unsigned long long bk = ~0ull;
      unsigned int bj = 0;
      for (unsigned long long t = 0; t < deg; t += 32) {
        const unsigned long long j = t + (unsigned long long)lane;
        const unsigned long long nk = j < deg ? edge_key(seed_h, (unsigned long long)v, j) : ~0ull;
        unsigned int rb = (unsigned int)lane, rn = 0;
#pragma unroll 8
        for (int m = 0; m < 32; m++) {
          const unsigned long long ob = __shfl_sync(0xffffffffu, bk, m);
          const unsigned long long on = __shfl_sync(0xffffffffu, nk, m);
          rb += on < bk;
          rn += (ob < nk) + (on < nk);
        }
        // ~0 entries are padding: they never rank below f among real keys
        // only when fewer than f real keys exist, and those slots are unused
        if (lane < f && bk != ~0ull && rb < (unsigned int)f) {
          sk[w][rb] = bk;
          sj[w][rb] = bj;
        }
        if (nk != ~0ull && rn < (unsigned int)f) {
          sk[w][rn] = nk;
          sj[w][rn] = (unsigned int)j;
        }
        __syncwarp();
        const unsigned long long have = t + 32 < deg ? t + 32 : deg;
        if ((unsigned long long)lane < (have < (unsigned long long)f ? have : (unsigned long long)f)) {
          bk = sk[w][lane];
          bj = sj[w][lane];
        } else {
          bk = ~0ull;
        }
        __syncwarp();
      }
      if ((unsigned long long)lane < take) kept_j = bj;
    }
    if (lane < f) {
      const unsigned long long slot = i * (unsigned long long)f + (unsigned long long)lane;
      long long src = -1;
      if ((unsigned long long)lane < take) {
        src = edge_src(g, e0 + kept_j);
        if (src < 0 || (unsigned long long)src >= g.n) {  // a malformed graph: drop the edge, report it
          atomicOr(&ctl->err, 8u);
          src = -1;
        } else if (!table_insert(tab, mask, src, base + slot)) {
          atomicOr(&ctl->err, 2u);
        }
      }
      cand[slot] = src;
    }
  }
}

// candidates of the current round, never beyond the buffer (a round that
// would overflow it has set the capacity error and written nothing past it)
__device__ __forceinline__ unsigned long long round_cands(const SamplerCtl* ctl, int f, unsigned long long n_seeds,
                                                          unsigned long long cand_cap) {
  const unsigned long long nc = f ? ctl->n_nodes * (unsigned long long)f : n_seeds;
  return nc < cand_cap ? nc : cand_cap;
}

// ---- compaction: flag the first occurrences, count them per tile
__global__ void __launch_bounds__(SMP_THREADS) flag_kernel(const long long* __restrict__ cand,
                                                           unsigned char* __restrict__ flag,
                                                           unsigned int* __restrict__ tile_cnt,
                                                           const unsigned long long* __restrict__ tab,
                                                           unsigned long long mask, int f,
                                                           unsigned long long n_seeds, unsigned long long cand_cap,
                                                           const SamplerCtl* ctl) {
  __shared__ unsigned int red[SMP_THREADS / 32];
  const unsigned long long nc = round_cands(ctl, f, n_seeds, cand_cap);
  const unsigned long long base = ctl->pos_base;
  const unsigned long long tiles = (nc + TILE - 1) / TILE;
  for (unsigned long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    unsigned int c = 0;
    for (int q = 0; q < PER_THREAD; q++) {
      const unsigned long long i = t * TILE + (unsigned long long)q * SMP_THREADS + threadIdx.x;
      if (i >= nc) break;
      const long long v = cand[i];
      const unsigned char fl = v >= 0 && table_pos(tab, mask, v) == base + i;
      flag[i] = fl;
      c += fl;
    }
    c = __reduce_add_sync(0xffffffffu, c);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned int s = 0;
      for (int k = 0; k < SMP_THREADS / 32; k++) s += red[k];
      tile_cnt[t] = s;
    }
    __syncthreads();
  }
}

// one block: exclusive scan of the tile counts, then the round's bookkeeping
__global__ void __launch_bounds__(1024) scan_kernel(unsigned int* __restrict__ tile_cnt, int f,
                                                    unsigned long long n_seeds, unsigned long long cand_cap,
                                                    unsigned long long node_cap, SamplerCtl* ctl) {
  __shared__ unsigned long long warp_tot[32];
  __shared__ unsigned long long carry;
  const unsigned long long nc = round_cands(ctl, f, n_seeds, cand_cap);
  const unsigned long long tiles = (nc + TILE - 1) / TILE;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (unsigned long long b = 0; b < tiles; b += 1024) {
    const unsigned long long t = b + threadIdx.x;
    const unsigned long long v = t < tiles ? tile_cnt[t] : 0u;
    unsigned long long incl = v;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
      unsigned long long x = warp_tot[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      warp_tot[lane] = x;  // inclusive over warps
    }
    __syncthreads();
    const unsigned long long before = carry + (w ? warp_tot[w - 1] : 0ull) + incl - v;
    if (t < tiles) tile_cnt[t] = (unsigned int)before;  // tile offsets within the round (fit: < 2^30)
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_tot[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ctl->n_cand = nc;
    ctl->round_base = ctl->pos_base;
    ctl->pos_base += nc;
    ctl->out_base = ctl->n_nodes;
    unsigned long long add = carry;
    if (ctl->n_nodes + add > node_cap) {
      ctl->err |= 1u;
      add = node_cap - ctl->n_nodes;
    }
    ctl->n_nodes += add;
  }
}

// scatter the flagged candidates to nodes[out_base + rank], in candidate order
__global__ void __launch_bounds__(SMP_THREADS) scatter_kernel(const long long* __restrict__ cand,
                                                              const unsigned char* __restrict__ flag,
                                                              const unsigned int* __restrict__ tile_off,
                                                              long long* __restrict__ nodes,
                                                              unsigned long long node_cap, const SamplerCtl* ctl) {
  __shared__ unsigned int warp_tot[SMP_THREADS / 32];
  const unsigned long long nc = ctl->n_cand;
  const unsigned long long out_base = ctl->out_base;
  const unsigned long long tiles = (nc + TILE - 1) / TILE;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (unsigned long long t = blockIdx.x; t < tiles; t += gridDim.x) {
    // thread k of the tile owns candidates t*TILE + k*PER_THREAD + [0, PER_THREAD)
    const unsigned long long i0 = t * TILE + (unsigned long long)threadIdx.x * PER_THREAD;
    unsigned int mine = 0;
    for (int q = 0; q < PER_THREAD; q++) mine += (i0 + q < nc) ? flag[i0 + q] : 0u;
    unsigned int incl = mine;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    unsigned int wbefore = 0;
    for (int k = 0; k < w; k++) wbefore += warp_tot[k];
    unsigned long long pos = out_base + tile_off[t] + wbefore + incl - mine;
    for (int q = 0; q < PER_THREAD; q++) {
      const unsigned long long i = i0 + q;
      if (i < nc && flag[i]) {
        if (pos < node_cap) nodes[pos] = cand[i];
        pos++;
      }
    }
    __syncthreads();
  }
}

// ---- PageRank (float32, sequential sum per node in CSC order)
__global__ void pr_init_kernel(float* __restrict__ pv, unsigned long long n, float v0) {
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x)
    pv[i] = v0;
}

__global__ void pr_norm_kernel(const Graph g, const float* __restrict__ pv, float* __restrict__ norm) {
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < g.n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const long long d = __ldg(g.indptr + i + 1) - __ldg(g.indptr + i);
    norm[i] = d > 0 ? __fdiv_rn(pv[i], (float)d) : 0.0f;
  }
}

__global__ void __launch_bounds__(SMP_THREADS) pr_gather_kernel(const Graph g, const float* __restrict__ norm,
                                                                float* __restrict__ pv, float teleport,
                                                                float damping) {
  const int lane = threadIdx.x & 31;
  const unsigned long long nw = (unsigned long long)gridDim.x * (SMP_THREADS / 32);
  for (unsigned long long v = (unsigned long long)blockIdx.x * (SMP_THREADS / 32) + (threadIdx.x >> 5); v < g.n;
       v += nw) {
    const unsigned long long e0 = (unsigned long long)__ldg(g.indptr + v);
    const unsigned long long deg = (unsigned long long)__ldg(g.indptr + v + 1) - e0;
    float s = 0.0f;
    for (unsigned long long t = 0; t < deg; t += 32) {
      const unsigned long long j = t + (unsigned long long)lane;
      const float x = j < deg ? __ldg(norm + edge_src(g, e0 + j)) : 0.0f;
      const int m = (int)(deg - t < 32 ? deg - t : 32);
      for (int k = 0; k < m; k++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, x, k));  // in edge order
    }
    if (lane == 0) pv[v] = __fadd_rn(teleport, __fmul_rn(damping, s));
  }
}

// top-k order: value descending, node id ascending, as one ascending 64-bit key
__global__ void pr_key_kernel(const float* __restrict__ pv, unsigned long long n, unsigned long long* __restrict__ key) {
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    unsigned int b = __float_as_uint(pv[i]);
    // order-preserving map of a float's bits onto unsigned integers
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    key[i] = ((unsigned long long)(0xFFFFFFFFu - b) << 32) | (unsigned long long)i;
  }
}

// out-degree of every node: the number of in-edges it is the source of, i.e.
// how often neighbour sampling can reach it (the rank of a static hot set)
__global__ void outdeg_kernel(const void* __restrict__ indices, int index_bytes, unsigned long long n_edges,
                              unsigned long long n, unsigned int* __restrict__ counts,
                              unsigned int* __restrict__ bad) {
  for (unsigned long long e = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; e < n_edges;
       e += (unsigned long long)gridDim.x * blockDim.x) {
    const long long v = index_bytes == 4 ? (long long)__ldg(reinterpret_cast<const int*>(indices) + e)
                                         : __ldg(reinterpret_cast<const long long*>(indices) + e);
    if (v >= 0 && (unsigned long long)v < n)
      atomicAdd(counts + v, 1u);
    else
      atomicOr(bad, 1u);
  }
}

int grid_for(int dev, unsigned long long work, int per_block) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned long long want = (work + per_block - 1) / per_block;
  return (int)std::max<unsigned long long>(1, std::min<unsigned long long>(want, (unsigned long long)sms * 8));
}

}  // namespace

// ------------------------------------------------------------------ host side
struct Sampler {
  int device = 0;
  Graph g{};
  std::vector<int> fanouts;
  unsigned long long seed = 0, calls = 0;
  unsigned long long max_seeds = 0, node_cap = 0, cand_cap = 0, tab_mask = 0, tile_cap = 0;
  long long* d_cand = nullptr;
  unsigned char* d_flag = nullptr;
  unsigned int* d_tile = nullptr;
  unsigned long long* d_tab = nullptr;
  SamplerCtl* d_ctl = nullptr;
  SamplerCtl* h_ctl = nullptr;  // pinned copy of the control block

  ~Sampler() {
    cudaFree(d_cand);
    cudaFree(d_flag);
    cudaFree(d_tile);
    cudaFree(d_tab);
    cudaFree(d_ctl);
    if (h_ctl) cudaFreeHost(h_ctl);
  }
};

// 64-bit key seed of one hop of one call (GIDS/synthetic.py hop_seed)
static unsigned long long hop_seed(unsigned long long seed, unsigned long long call, unsigned long long hop) {
  return mix64(seed * 0x9E3779B97F4A7C15ull + call * 0xD1B54A32D192ED03ull + hop * 0x8CB92BA72F3D8DD7ull +
               0x632BE59BD9B4E019ull);
}

Sampler* sampler_create(int device, const int64_t* indptr, const void* indices, int index_bytes, uint64_t n_nodes,
                        const int* fanouts, int n_layers, uint64_t max_seeds, uint64_t seed) {
  GIDS_CHECK(indptr && indices, GIDS_E_INVAL, "null graph array");
  GIDS_CHECK(index_bytes == 4 || index_bytes == 8, GIDS_E_INVAL, "index_bytes must be 4 or 8");
  GIDS_CHECK(n_nodes > 0 && n_nodes < (1ull << (64 - POS_BITS)) - 2, GIDS_E_INVAL, "node count out of range");
  GIDS_CHECK(fanouts && n_layers >= 1 && n_layers <= 16, GIDS_E_INVAL, "1..16 layers");
  GIDS_CHECK(max_seeds > 0, GIDS_E_INVAL, "max_seeds must be > 0");
  std::unique_ptr<Sampler> s(new Sampler());
  s->device = device;
  s->g = Graph{reinterpret_cast<const long long*>(indptr), indices, index_bytes, n_nodes};
  s->seed = seed;
  // capacities: the node set grows by at most f per node per hop (and never
  // beyond the graph); a hop's candidates are (set size) x f
  unsigned long long nodes = max_seeds, cand = max_seeds, total_pos = max_seeds;
  for (int h = n_layers - 1; h >= 0; h--) {  // hops run from the last fanout to the first
    const int f = fanouts[h];
    GIDS_CHECK(f >= 1 && f <= 32, GIDS_E_UNSUPPORTED, "fanouts must be in [1, 32]");
    s->fanouts.push_back(f);
    const unsigned long long c = std::min<unsigned long long>(nodes, n_nodes) * (unsigned long long)f;
    cand = std::max(cand, c);
    total_pos += c;
    nodes = std::min<unsigned long long>(nodes + c, n_nodes);
  }
  GIDS_CHECK(total_pos < (1ull << POS_BITS), GIDS_E_UNSUPPORTED, "minibatch too large for the sampler's table");
  s->max_seeds = max_seeds;
  s->node_cap = nodes;
  s->cand_cap = cand;
  unsigned long long t = 1;
  while (t < 2 * nodes + 1024) t <<= 1;
  s->tab_mask = t - 1;
  s->tile_cap = (cand + TILE - 1) / TILE;
  DeviceGuard dg(device);
  GIDS_CUDA(cudaMalloc(&s->d_cand, cand * sizeof(long long)));
  GIDS_CUDA(cudaMalloc(&s->d_flag, cand));
  GIDS_CUDA(cudaMalloc(&s->d_tile, s->tile_cap * sizeof(unsigned int)));
  GIDS_CUDA(cudaMalloc(&s->d_tab, t * sizeof(unsigned long long)));
  GIDS_CUDA(cudaMalloc(&s->d_ctl, sizeof(SamplerCtl)));
  GIDS_CUDA(cudaHostAlloc(&s->h_ctl, sizeof(SamplerCtl), cudaHostAllocDefault));
  return s.release();
}

void sampler_destroy(Sampler* s) {
  if (!s) return;
  DeviceGuard dg(s->device);
  cudaDeviceSynchronize();
  delete s;
}

uint64_t sampler_capacity(const Sampler* s) { return s->node_cap; }

// One minibatch: out_nodes[0, *count) = input nodes (seeds first). count_dev
// (device) receives the count without a host synchronisation; with host_count
// the call waits for the stream and returns it (and checks the error flags).
void sampler_sample(Sampler* s, const int64_t* seeds, uint64_t n_seeds, int64_t* out_nodes, uint64_t out_cap,
                    uint64_t* count_dev, uint64_t* host_count, int64_t call, cudaStream_t st) {
  GIDS_CHECK(n_seeds <= s->max_seeds, GIDS_E_INVAL, "more seeds than the sampler was created for");
  GIDS_CHECK(out_nodes && out_cap >= s->node_cap, GIDS_E_INVAL,
             "output capacity below gids_sampler_capacity(): " + std::to_string(s->node_cap));
  GIDS_CHECK(n_seeds == 0 || seeds, GIDS_E_INVAL, "null seeds");
  DeviceGuard dg(s->device);
  const unsigned long long c = call >= 0 ? (unsigned long long)call : s->calls;
  s->calls = c + 1;
  long long* nodes = reinterpret_cast<long long*>(out_nodes);
  GIDS_CUDA(cudaMemsetAsync(s->d_tab, 0, (s->tab_mask + 1) * sizeof(unsigned long long), st));
  GIDS_CUDA(cudaMemsetAsync(s->d_ctl, 0, sizeof(SamplerCtl), st));
  const int dev = s->device;
  const int gt = grid_for(dev, s->tile_cap * (unsigned long long)TILE, TILE);
  if (n_seeds) {
    seeds_kernel<<<grid_for(dev, n_seeds, SMP_THREADS), SMP_THREADS, 0, st>>>(
        reinterpret_cast<const long long*>(seeds), n_seeds, s->d_cand, s->d_tab, s->tab_mask, s->g.n, s->d_ctl);
    flag_kernel<<<gt, SMP_THREADS, 0, st>>>(s->d_cand, s->d_flag, s->d_tile, s->d_tab, s->tab_mask, 0, n_seeds,
                                           s->cand_cap, s->d_ctl);
    scan_kernel<<<1, 1024, 0, st>>>(s->d_tile, 0, n_seeds, s->cand_cap, s->node_cap, s->d_ctl);
    scatter_kernel<<<gt, SMP_THREADS, 0, st>>>(s->d_cand, s->d_flag, s->d_tile, nodes, s->node_cap, s->d_ctl);
    for (size_t h = 0; h < s->fanouts.size(); h++) {
      const int f = s->fanouts[h];
      hop_kernel<<<grid_for(dev, s->node_cap * 32ull, SMP_THREADS), SMP_THREADS, 0, st>>>(
          s->g, nodes, s->d_cand, s->cand_cap, s->d_tab, s->tab_mask, f, hop_seed(s->seed, c, h), s->d_ctl);
      flag_kernel<<<gt, SMP_THREADS, 0, st>>>(s->d_cand, s->d_flag, s->d_tile, s->d_tab, s->tab_mask, f, 0,
                                             s->cand_cap, s->d_ctl);
      scan_kernel<<<1, 1024, 0, st>>>(s->d_tile, f, 0, s->cand_cap, s->node_cap, s->d_ctl);
      scatter_kernel<<<gt, SMP_THREADS, 0, st>>>(s->d_cand, s->d_flag, s->d_tile, nodes, s->node_cap, s->d_ctl);
    }
  }
  GIDS_CUDA(cudaGetLastError());
  if (count_dev)
    GIDS_CUDA(cudaMemcpyAsync(count_dev, &s->d_ctl->n_nodes, sizeof(uint64_t), cudaMemcpyDeviceToDevice, st));
  if (host_count) {
    GIDS_CUDA(cudaMemcpyAsync(s->h_ctl, s->d_ctl, sizeof(SamplerCtl), cudaMemcpyDeviceToHost, st));
    GIDS_CUDA(cudaStreamSynchronize(st));
    const unsigned int err = s->h_ctl->err;
    GIDS_CHECK(!(err & 4u), GIDS_E_RANGE, "a seed id lies outside the graph");
    GIDS_CHECK(!(err & 8u), GIDS_E_RANGE, "an edge of the CSC graph has a source outside the graph");
    GIDS_CHECK(!(err & 3u), GIDS_E_INVAL, "sampler capacity exceeded (internal error)");
    *host_count = s->h_ctl->n_nodes;
  }
}

// PageRank of page_rank_node_list_gen.py:126-134 in float32 into pv[n], and
// the top-k order keys (value descending, node id ascending) into keys[n] if
// keys is not null.
void pagerank(int device, const int64_t* indptr, const void* indices, int index_bytes, uint64_t n, int iters,
              double damping, float* pv, uint64_t* keys, cudaStream_t st) {
  GIDS_CHECK(indptr && indices && pv, GIDS_E_INVAL, "null array");
  GIDS_CHECK(index_bytes == 4 || index_bytes == 8, GIDS_E_INVAL, "index_bytes must be 4 or 8");
  GIDS_CHECK(n > 0 && n < (1ull << 32), GIDS_E_INVAL, "node count must be in [1, 2^32)");
  GIDS_CHECK(iters >= 0, GIDS_E_INVAL, "iters must be >= 0");
  DeviceGuard dg(device);
  const Graph g{reinterpret_cast<const long long*>(indptr), indices, index_bytes, n};
  float* norm = nullptr;
  GIDS_CUDA(cudaMallocAsync(&norm, n * sizeof(float), st));
  // the reference's scalars (Python floats applied to float32 tensors):
  // torch.ones(N) / N divides in float32; (1 - DAMP) / N is a double
  // rounded to float32 when added; DAMP * pv multiplies by float32(DAMP)
  const float v0 = 1.0f / (float)n;
  const float teleport = (float)((1.0 - damping) / (double)n);
  const float damp32 = (float)damping;
  const int ge = grid_for(device, n, SMP_THREADS);
  pr_init_kernel<<<ge, SMP_THREADS, 0, st>>>(pv, n, v0);
  for (int k = 0; k < iters; k++) {
    pr_norm_kernel<<<ge, SMP_THREADS, 0, st>>>(g, pv, norm);
    pr_gather_kernel<<<grid_for(device, n * 32ull, SMP_THREADS), SMP_THREADS, 0, st>>>(g, norm, pv, teleport,
                                                                                      damp32);
  }
  if (keys) pr_key_kernel<<<ge, SMP_THREADS, 0, st>>>(pv, n, reinterpret_cast<unsigned long long*>(keys));
  GIDS_CUDA(cudaGetLastError());
  GIDS_CUDA(cudaFreeAsync(norm, st));
}

// Out-degree histogram of a CSC graph's sources into counts[n] (device).
void out_degree(int device, const void* indices, int index_bytes, uint64_t n_edges, uint64_t n, uint32_t* counts,
                cudaStream_t st) {
  GIDS_CHECK(counts && (indices || n_edges == 0), GIDS_E_INVAL, "null array");
  GIDS_CHECK(index_bytes == 4 || index_bytes == 8, GIDS_E_INVAL, "index_bytes must be 4 or 8");
  GIDS_CHECK(n > 0, GIDS_E_INVAL, "node count must be > 0");
  DeviceGuard dg(device);
  unsigned int* bad = nullptr;
  GIDS_CUDA(cudaMallocAsync(&bad, sizeof(unsigned int), st));
  GIDS_CUDA(cudaMemsetAsync(bad, 0, sizeof(unsigned int), st));
  GIDS_CUDA(cudaMemsetAsync(counts, 0, n * sizeof(uint32_t), st));
  if (n_edges)
    outdeg_kernel<<<grid_for(device, n_edges, SMP_THREADS), SMP_THREADS, 0, st>>>(indices, index_bytes, n_edges, n,
                                                                                  counts, bad);
  GIDS_CUDA(cudaGetLastError());
  unsigned int h = 0;
  GIDS_CUDA(cudaMemcpyAsync(&h, bad, sizeof(h), cudaMemcpyDeviceToHost, st));
  GIDS_CUDA(cudaFreeAsync(bad, st));
  GIDS_CUDA(cudaStreamSynchronize(st));
  GIDS_CHECK(h == 0, GIDS_E_RANGE, "an edge of the CSC graph has a source outside the graph");
}

}  // namespace gids
