/*
 * gids_oracle.c -- CPU restatement of the GIDS feature-gather path.
 *
 * TEST INFRASTRUCTURE ONLY. It checks results, nothing more: only tests/, the smoke
 * entry point and the bench's CPU-baseline leg load it. The product library
 * never links or calls it.
 *
 * What it restates (paths relative to the reference project):
 *   - read_feature_kernel             gids_module/gids_kernel.cu:60-86
 *       out[w*dim + t] = feat[(idx[w] + key_off) * cache_dim + t], t < dim
 *   - the mmap baseline gather        evaluation/dataloader.py:166-169 (np.memmap
 *       row-major [N, dim] table) + evaluation/homogenous_train_baseline.py:244
 *       (DGL srcdata gather == torch.index_select(feat, 0, input_nodes))
 *   - page / stripe mapping           gids_module/include/page_cache_backup.h:626-652
 *       (get_backing_page_, get_backing_ctrl_ with STRIPE) and :1146-1152
 *       (range_d_t::get_page): page p = byte >> log2(page_size),
 *       controller = p % n_ctrls, device page = page_start + p / n_ctrls.
 *   - the synthetic feature generator used by the benchmarks: element e of
 *       stream `seed` is the e-th output of SplitMix64 (Steele, Lea, Flood,
 *       "Fast splittable pseudorandom number generators", OOPSLA 2014)
 *       seeded with `seed`, mapped to the element type with integer-only
 *       arithmetic so that every value is exact.
 *
 * Parity status: the gather semantics are pinned against golden vectors made
 * by running the reference's own memmap loader (IGB260M.paper_feat) and
 * torch.index_select; see tests/golden/make_golden.py.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define GO_KIND_F32_UNIFORM 1
#define GO_KIND_F16_BYTESUM 2
#define GO_KIND_I64_RAW 3
#define GO_KIND_F16_NORMAL 4

#define GO_GOLDEN 0x9E3779B97F4A7C15ULL

static inline uint64_t go_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

/* e-th output (e = 0, 1, ...) of SplitMix64 seeded with `seed`. */
uint64_t go_synth_u64(uint64_t seed, uint64_t e) { return go_mix(seed + (e + 1) * GO_GOLDEN); }

int go_kind_elem_bytes(int kind) {
  switch (kind) {
    case GO_KIND_F32_UNIFORM: return 4;
    case GO_KIND_F16_BYTESUM: return 2;
    case GO_KIND_I64_RAW: return 8;
    case GO_KIND_F16_NORMAL: return 2;
    default: return 0;
  }
}

/* uniform[-1, 1): top 24 bits k of the hash, value k * 2^-23 - 1 (exact in fp32) */
static inline uint32_t go_f32_bits(uint64_t h) {
  uint32_t k = (uint32_t)(h >> 40);
  float v = (float)k * (1.0f / 8388608.0f) - 1.0f;
  uint32_t b;
  memcpy(&b, &v, 4);
  return b;
}

/* approximately normal: m = (sum of the 8 bytes of the hash) - 1020, value m * 2^-8.
 * |m| <= 1020 < 2^11, so the value is exact in fp16; the half bits are built
 * directly from m. */
static inline uint16_t go_f16_bits(uint64_t h) {
  int32_t s = 0;
  for (int i = 0; i < 8; i++) s += (int32_t)((h >> (8 * i)) & 0xFF);
  int32_t m = s - 1020;
  if (m == 0) return 0;
  uint16_t sign = m < 0 ? 0x8000 : 0;
  uint32_t a = (uint32_t)(m < 0 ? -m : m);
  int e = 31 - __builtin_clz(a); /* a = 1.f * 2^e, value = 1.f * 2^(e-8) */
  uint16_t expf = (uint16_t)(e - 8 + 15);
  uint16_t mant = (uint16_t)((a << (10 - e)) & 0x3FF);
  return (uint16_t)(sign | (expf << 10) | mant);
}

/* normal(0, 1) by the Box-Muller transform (Box and Muller, 1958) of the
 * hash's two 32-bit halves: u1 = (hi + 1) 2^-32 in (0, 1], u2 = lo 2^-32 in
 * [0, 1), sqrt(-2 ln u1) cos(2 pi u2) in double, rounded to fp16 by the
 * compiler's _Float16 conversion (round to nearest even) */
static inline uint16_t go_f16_normal_bits(uint64_t h) {
  double u1 = ((double)(h >> 32) + 1.0) * 0x1p-32;
  double u2 = (double)(h & 0xFFFFFFFFull) * 0x1p-32;
  _Float16 v = (_Float16)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
  uint16_t b;
  memcpy(&b, &v, 2);
  return b;
}

/* writes the element e of `kind`/`seed` to dst (elem_bytes bytes) */
static inline void go_synth_elem(int kind, uint64_t seed, uint64_t e, void *dst) {
  uint64_t h = go_synth_u64(seed, e);
  if (kind == GO_KIND_F32_UNIFORM) {
    uint32_t b = go_f32_bits(h);
    memcpy(dst, &b, 4);
  } else if (kind == GO_KIND_F16_BYTESUM) {
    uint16_t b = go_f16_bits(h);
    memcpy(dst, &b, 2);
  } else if (kind == GO_KIND_F16_NORMAL) {
    uint16_t b = go_f16_normal_bits(h);
    memcpy(dst, &b, 2);
  } else {
    memcpy(dst, &h, 8);
  }
}

/* ---------------------------------------------------------------- threads */
typedef struct {
  void (*fn)(void *, uint64_t, uint64_t);
  void *arg;
  uint64_t lo, hi;
} go_job_t;

static void *go_run(void *p) {
  go_job_t *j = (go_job_t *)p;
  j->fn(j->arg, j->lo, j->hi);
  return 0;
}

static void go_parallel(void (*fn)(void *, uint64_t, uint64_t), void *arg, uint64_t n, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((uint64_t)threads > n) threads = n ? (int)n : 1;
  pthread_t th[256];
  go_job_t jobs[256];
  for (int t = 0; t < threads; t++) {
    jobs[t].fn = fn;
    jobs[t].arg = arg;
    jobs[t].lo = n / threads * t;
    jobs[t].hi = t == threads - 1 ? n : n / threads * (t + 1);
    if (t) pthread_create(&th[t], 0, go_run, &jobs[t]);
  }
  go_run(&jobs[0]);
  for (int t = 1; t < threads; t++) pthread_join(th[t], 0);
}

/* ------------------------------------------------------- table generation */
typedef struct {
  int kind;
  uint64_t seed, first;
  char *dst;
  int eb;
} go_fill_t;

static void go_fill_part(void *p, uint64_t lo, uint64_t hi) {
  go_fill_t *f = (go_fill_t *)p;
  for (uint64_t i = lo; i < hi; i++) go_synth_elem(f->kind, f->seed, f->first + i, f->dst + i * f->eb);
}

/* dst[i] = element (first + i) of the synthetic stream, i < n. Row-major
 * tables are filled with first = row0 * cache_dim. */
int go_synth_fill(int kind, uint64_t seed, uint64_t first, uint64_t n, void *dst, int threads) {
  int eb = go_kind_elem_bytes(kind);
  if (!eb) return -1;
  go_fill_t f = {kind, seed, first, (char *)dst, eb};
  go_parallel(go_fill_part, &f, n, threads);
  return 0;
}

/* --------------------------------------------------------------- gathers */
typedef struct {
  const char *table;
  uint64_t rows;
  uint64_t src_stride, row_bytes;
  const int64_t *ids;
  uint64_t key_off;
  char *out;
  volatile int bad;
} go_gather_t;

static void go_gather_part(void *p, uint64_t lo, uint64_t hi) {
  go_gather_t *g = (go_gather_t *)p;
  for (uint64_t i = lo; i < hi; i++) {
    int64_t id = g->ids[i];
    uint64_t r = (uint64_t)id + g->key_off;
    if (id < 0 || r >= g->rows) {
      g->bad = 1;
      memset(g->out + i * g->row_bytes, 0, g->row_bytes);
      continue;
    }
    memcpy(g->out + i * g->row_bytes, g->table + r * g->src_stride, g->row_bytes);
  }
}

/* index_select restatement: out[i, 0:dim] = table[ids[i] + key_off, 0:dim],
 * table rows have cache_dim elements. Returns -2 if any id is out of range
 * (that row is zero-filled). */
int go_gather(const void *table, uint64_t table_rows, uint32_t elem_bytes, uint32_t cache_dim, uint32_t dim,
              const int64_t *ids, int64_t n, uint64_t key_off, void *out, int threads) {
  if (dim > cache_dim || n < 0) return -1;
  go_gather_t g = {(const char *)table, table_rows, (uint64_t)cache_dim * elem_bytes, (uint64_t)dim * elem_bytes,
                   ids, key_off, (char *)out, 0};
  go_parallel(go_gather_part, &g, (uint64_t)n, threads);
  return g.bad ? -2 : 0;
}

/* Expected gather output computed from the generator, with no table:
 * element index e = (ids[i] + key_off) * cache_dim + c, value = synth(e mod wrap)
 * (wrap == 0: no wrap). Used at sizes where no table can be materialised. */
typedef struct {
  int kind;
  uint64_t seed, wrap, rows;
  uint32_t cache_dim, dim;
  int eb;
  const int64_t *ids;
  uint64_t key_off;
  char *out;
  volatile int bad;
} go_gsyn_t;

static void go_gsyn_part(void *p, uint64_t lo, uint64_t hi) {
  go_gsyn_t *g = (go_gsyn_t *)p;
  for (uint64_t i = lo; i < hi; i++) {
    int64_t id = g->ids[i];
    uint64_t r = (uint64_t)id + g->key_off;
    char *o = g->out + i * (uint64_t)g->dim * g->eb;
    if (id < 0 || r >= g->rows) {
      g->bad = 1;
      memset(o, 0, (uint64_t)g->dim * g->eb);
      continue;
    }
    for (uint32_t c = 0; c < g->dim; c++) {
      uint64_t e = r * g->cache_dim + c;
      if (g->wrap) e %= g->wrap;
      go_synth_elem(g->kind, g->seed, e, o + (uint64_t)c * g->eb);
    }
  }
}

int go_gather_synth(int kind, uint64_t seed, uint64_t wrap_elems, uint64_t table_rows, uint32_t cache_dim,
                    uint32_t dim, const int64_t *ids, int64_t n, uint64_t key_off, void *out, int threads) {
  int eb = go_kind_elem_bytes(kind);
  if (!eb || dim > cache_dim || n < 0) return -1;
  go_gsyn_t g = {kind, seed, wrap_elems, table_rows, cache_dim, dim, eb, ids, key_off, (char *)out, 0};
  go_parallel(go_gsyn_part, &g, (uint64_t)n, threads);
  return g.bad ? -2 : 0;
}

/* ------------------------------------------------------- stripe mapping */
/* Logical page p of a range striped over n_ctrls devices starting at device
 * page `page_start` (page_cache_backup.h:626-652, STRIPE). wrap_pages > 0
 * models a device whose physical capacity holds wrap_pages logical pages:
 * page p is stored where page (p mod wrap_pages) would be. */
void go_stripe_locate(uint64_t p, uint64_t n_ctrls, uint64_t page_start, uint64_t wrap_pages, uint64_t *ctrl,
                      uint64_t *dev_page) {
  uint64_t q = wrap_pages ? p % wrap_pages : p;
  *ctrl = q % n_ctrls;
  *dev_page = page_start + q / n_ctrls;
}

/* Build the per-device images of a striped backing store from a row-major
 * logical byte image: dev[c][(page_start + q / n) * page_size + o] =
 * logical[q * page_size + o] for q % n == c. Pages at device index below
 * page_start are left untouched. Used to check the product's writer. */
int go_stripe_image(const void *logical, uint64_t logical_bytes, uint32_t page_size, uint64_t n_ctrls,
                    uint64_t page_start, void **dev, uint64_t dev_bytes) {
  if (!page_size || !n_ctrls) return -1;
  const char *src = (const char *)logical;
  uint64_t pages = (logical_bytes + page_size - 1) / page_size;
  for (uint64_t q = 0; q < pages; q++) {
    uint64_t c = q % n_ctrls, dp = page_start + q / n_ctrls;
    uint64_t off = dp * page_size;
    uint64_t len = logical_bytes - q * page_size < page_size ? logical_bytes - q * page_size : page_size;
    if (off + len > dev_bytes) return -2;
    memcpy((char *)dev[c] + off, src + q * page_size, len);
  }
  return 0;
}
