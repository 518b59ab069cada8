/*
 * sampler_oracle.c -- CPU restatement of the minibatch sampler and of the
 * pin-list PageRank that feed the GIDS feature gather.
 *
 * TEST INFRASTRUCTURE ONLY: it checks results. Only tests/ load it (through
 * oracle/oracle.py); the product library never links or calls it.
 *
 * Sampler: DGL's MultiLayerNeighborSampler as the reference's loaders use it
 * (GIDS_Setup/GIDS/GIDS.py:178-201, evaluation/homogenous_train.py:201-203),
 * over a CSC graph (in-edges of v: indices[indptr[v] .. indptr[v+1])), with
 * the random choice made explicit: at hop h (hops run from the last fanout to
 * the first) every node v of the current set keeps the min(fanout, in_degree)
 * in-edges j of smallest
 *     key(v, j) = (mix(mix(v * G + seed_h) + (j + 1) * M2) >> 25) << 24 | j
 * in increasing key order, where mix is the SplitMix64 finalizer (Steele, Lea,
 * Flood, OOPSLA 2014) and seed_h = mix(seed * G + call * C1 + hop * C2 + C3);
 * the kept sources not yet in the set are appended in order of first
 * appearance. The seeds, duplicates removed in order, come first.
 *
 * PageRank: compute_pagerank of evaluation/page_rank_node_list_gen.py:126-134
 * in float32, as the reference runs it on torch tensors:
 *     pv = ones(N) / N
 *     K times: pv = pv / in_degree          (float32 division)
 *              pv[v] = sum over in-edges u -> v of pv[u]   (in CSC order)
 *              pv = (1 - d) / N + d * pv    (the double (1-d)/N and d rounded to
 *                                            float32; multiply, then add)
 * A node without in-edges divides by zero in the reference; here its share
 * is 0. The pin_file is the top-k of pv (page_rank_node_list_gen.py:282-285),
 * ordered by value descending, node id ascending.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline uint64_t so_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

uint64_t go_hop_seed(uint64_t seed, uint64_t call, uint64_t hop) {
  return so_mix(seed * 0x9E3779B97F4A7C15ULL + call * 0xD1B54A32D192ED03ULL + hop * 0x8CB92BA72F3D8DD7ULL +
                0x632BE59BD9B4E019ULL);
}

uint64_t go_edge_key(uint64_t seed_h, uint64_t v, uint64_t j) {
  uint64_t z = so_mix(v * 0x9E3779B97F4A7C15ULL + seed_h);
  z = so_mix(z + (j + 1) * 0x94D049BB133111EBULL);
  return ((z >> 25) << 24) | j;
}

static inline int64_t so_src(const void *indices, int index_bytes, uint64_t e) {
  return index_bytes == 4 ? (int64_t)((const int32_t *)indices)[e] : ((const int64_t *)indices)[e];
}

/* Returns the number of input nodes written to out (at most out_cap), or
 * -1 (bad arguments), -2 (a seed outside the graph), -3 (out_cap too small),
 * -4 (out of memory). */
int64_t go_sample(const int64_t *indptr, const void *indices, int index_bytes, uint64_t n_nodes, const int *fanouts,
                  int n_layers, const int64_t *seeds, uint64_t n_seeds, uint64_t seed, uint64_t call, int64_t *out,
                  uint64_t out_cap) {
  if (!indptr || !indices || !fanouts || n_layers < 1 || (index_bytes != 4 && index_bytes != 8)) return -1;
  unsigned char *in_set = (unsigned char *)calloc(n_nodes ? n_nodes : 1, 1);
  if (!in_set) return -4;
  uint64_t n = 0;
  int64_t rc = 0;
  for (uint64_t i = 0; i < n_seeds; i++) {
    const int64_t v = seeds[i];
    if (v < 0 || (uint64_t)v >= n_nodes) {
      rc = -2;
      goto done;
    }
    if (in_set[v]) continue;
    if (n >= out_cap) {
      rc = -3;
      goto done;
    }
    in_set[v] = 1;
    out[n++] = v;
  }
  for (int h = 0; h < n_layers; h++) {
    const int f = fanouts[n_layers - 1 - h];
    if (f < 1 || f > 64) {
      rc = -1;
      goto done;
    }
    const uint64_t sh = go_hop_seed(seed, call, (uint64_t)h);
    const uint64_t frontier = n;  /* every node of the set before this hop */
    for (uint64_t i = 0; i < frontier; i++) {
      const int64_t v = out[i];
      const uint64_t e0 = (uint64_t)indptr[v], deg = (uint64_t)(indptr[v + 1] - indptr[v]);
      /* the f smallest keys, kept sorted by insertion */
      uint64_t best_k[64], best_j[64];
      int m = 0;
      for (uint64_t j = 0; j < deg; j++) {
        const uint64_t k = go_edge_key(sh, (uint64_t)v, j);
        if (m == f && k >= best_k[m - 1]) continue;
        int p = m < f ? m++ : f - 1;
        while (p > 0 && best_k[p - 1] > k) {
          best_k[p] = best_k[p - 1];
          best_j[p] = best_j[p - 1];
          p--;
        }
        best_k[p] = k;
        best_j[p] = j;
      }
      for (int r = 0; r < m; r++) {
        const int64_t s = so_src(indices, index_bytes, e0 + best_j[r]);
        if (s < 0 || (uint64_t)s >= n_nodes || in_set[s]) continue;
        if (n >= out_cap) {
          rc = -3;
          goto done;
        }
        in_set[s] = 1;
        out[n++] = s;
      }
    }
  }
  rc = (int64_t)n;
done:
  free(in_set);
  return rc;
}

/* float32 PageRank into pv[n]; returns 0, or -1 on bad arguments / -4 out of memory */
int go_pagerank_f32(const int64_t *indptr, const void *indices, int index_bytes, uint64_t n, int iters, double damping,
                    float *pv) {
  if (!indptr || !indices || !pv || !n || iters < 0 || (index_bytes != 4 && index_bytes != 8)) return -1;
  float *norm = (float *)malloc(n * sizeof(float));
  if (!norm) return -4;
  const float v0 = 1.0f / (float)n;
  const float teleport = (float)((1.0 - damping) / (double)n);
  const float d32 = (float)damping;
  for (uint64_t i = 0; i < n; i++) pv[i] = v0;
  for (int k = 0; k < iters; k++) {
    for (uint64_t i = 0; i < n; i++) {
      const int64_t deg = indptr[i + 1] - indptr[i];
      norm[i] = deg > 0 ? pv[i] / (float)deg : 0.0f;
    }
    for (uint64_t v = 0; v < n; v++) {
      float s = 0.0f;
      for (int64_t e = indptr[v]; e < indptr[v + 1]; e++) s = s + norm[so_src(indices, index_bytes, (uint64_t)e)];
      const float t = d32 * s;
      pv[v] = teleport + t;
    }
  }
  free(norm);
  return 0;
}

/* Top-k of pv: ids by value descending, node id ascending. */
static const float *so_pv;
static int so_cmp(const void *a, const void *b) {
  const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
  if (so_pv[x] > so_pv[y]) return -1;
  if (so_pv[x] < so_pv[y]) return 1;
  return x < y ? -1 : (x > y);
}

int go_topk_desc(const float *pv, uint64_t n, uint64_t k, int64_t *out) {
  if (!pv || !out || k > n) return -1;
  int64_t *ids = (int64_t *)malloc((n ? n : 1) * sizeof(int64_t));
  if (!ids) return -4;
  for (uint64_t i = 0; i < n; i++) ids[i] = (int64_t)i;
  so_pv = pv;
  qsort(ids, n, sizeof(int64_t), so_cmp);
  memcpy(out, ids, k * sizeof(int64_t));
  free(ids);
  return 0;
}
