/* Page-cache policy simulator over minibatch line traces.
 *
 * Replays the line references of a sequence of minibatches (one int32 line id
 * per reference, minibatch lengths alongside, both .npy files as written by
 * trace.py) through the replacement policies of the gather kernel and prints
 * the hit ratio per minibatch. Used to choose the kernel's policy; it is not
 * part of the library.
 *
 *   policy "seq":  one reference at a time, a clock whose hand passes exactly
 *                  the slots it needs (the sequential ideal);
 *   policy "warp": references in chunks of 32 (one warp's rows), each shard's
 *                  new lines placed by sweep rounds of m candidates, m = 32
 *                  ("warp32", the first kernel) or m = lines still to place,
 *                  doubling per round ("warpN", the current kernel).
 * Admission (window W, in multiples of the total slots; 0 = off): once a
 * shard's hand has gone round, a line is inserted only on its A-th miss since
 * the last clear of the admission counts (A = 2 by default: the first miss
 * reads through). ref_max: clock chances added per hit.
 *
 * Build: gcc -O2 -o cachesim cachesim.c
 * Run:   cachesim trace.npy trace_len.npy n_lines slots_per_shard \
 *                 policy,shards,ref_max,window[,admit] ...
 *        e.g. cachesim t.npy t_len.npy 100000000 10485760 warpN,1,3,2 seq,1,1,0
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int32_t* trace;
static int64_t* lens;
static int nb;
static int64_t nlines, nslots;

static void* load_npy(const char* path, long* n) {
  FILE* f = fopen(path, "rb");
  if (!f) { perror(path); exit(1); }
  fseek(f, 0, SEEK_END);
  long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  char* b = malloc(sz);
  if (!b || fread(b, 1, sz, f) != (size_t)sz) { fprintf(stderr, "cannot read %s\n", path); exit(1); }
  fclose(f);
  long o = 0;
  while (o < sz && b[o++] != '\n') {}  /* the .npy header ends with a newline */
  *n = sz - o;
  return b + o;
}

static void run(const char* policy, int S, int K, double W, int A) {
  const int warp = strncmp(policy, "warp", 4) == 0;
  const int m32 = strcmp(policy, "warp32") == 0;
  int32_t* state = malloc(nlines * 4);  /* slot within the owner's shard, or -1 */
  int32_t* tag = malloc(S * nslots * 4);
  uint8_t* ref = calloc(S * nslots, 1);
  uint8_t* seen = calloc(nlines + 1, 1);  /* misses of each line in the window */
  memset(state, 0xff, nlines * 4);
  memset(tag, 0xff, S * nslots * 4);
  int64_t hand[64] = {0}, since = 0, pos = 0;
  printf("%s shards=%d ref_max=%d window=%.1f admit=%d:", policy, S, K, W, A);
  for (int b = 0; b < nb; b++) {
    const int64_t n = lens[b];
    int64_t hits = 0;
    since += n;
    if (W > 0 && since > W * nslots * S) { memset(seen, 0, nlines + 1); since = n; }
    int gate[64];
    for (int r = 0; r < S; r++) gate[r] = W > 0 && hand[r] >= nslots;  /* read once per launch */
    const int64_t chunk = warp ? 32 : 1;
    for (int64_t c = 0; c < n; c += chunk) {
      int32_t own[32];
      int no = 0;
      for (int64_t i = c; i < c + chunk && i < n; i++) {
        const int32_t l = trace[pos + i];
        const int r = l % S;
        const int32_t s = state[l];
        if (s >= 0) {
          hits++;
          uint8_t* rf = &ref[r * nslots + s];
          if (*rf < K) (*rf)++;
          continue;
        }
        if (gate[r]) {
          if (seen[l] < 255) seen[l]++;
          if (seen[l] < A) continue;  /* an early miss: read through, not inserted */
        }
        own[no++] = l;
      }
      for (int r = 0; r < S; r++) {
        int32_t need[32];
        int nn = 0, got = 0;
        for (int i = 0; i < no; i++)
          if (own[i] % S == r) need[nn++] = own[i];
        /* the warp sweeps give up after 64 rounds, as the kernel does; the sequential clock
           always places (at most ref_max + 1 passes over the slots) */
        const int64_t max_rounds = warp ? 64 : (int64_t)(K + 1) * nslots + 1;
        for (int64_t round = 0; got < nn && round < max_rounds; round++) {
          int m = warp ? (m32 ? 32 : (nn - got) << (round < 5 ? (int)round : 5)) : 1;
          if (m > 32) m = 32;
          const int64_t base = hand[r];
          hand[r] += m;
          for (int k = 0; k < m; k++) {
            const int64_t s = (base + k) % nslots;
            uint8_t* rf = &ref[r * nslots + s];
            int32_t* tg = &tag[r * nslots + s];
            if (*tg >= 0 && *rf) { (*rf)--; continue; }
            if (got < nn) {
              if (*tg >= 0) state[*tg] = -1;
              *tg = need[got];
              state[need[got]] = (int32_t)s;
              *rf = 1;
              got++;
            }
          }
        }
      }
    }
    pos += n;
    printf(" %.3f", (double)hits / n);
  }
  printf("\n");
  fflush(stdout);
  free(state); free(tag); free(ref); free(seen);
}

int main(int argc, char** argv) {
  if (argc < 6) { fprintf(stderr, "usage: cachesim trace.npy len.npy n_lines slots_per_shard policy,S,K,W ...\n"); return 2; }
  long n;
  trace = load_npy(argv[1], &n);
  lens = load_npy(argv[2], &n);
  nb = (int)(n / 8);
  nlines = atol(argv[3]);
  nslots = atol(argv[4]);
  for (int a = 5; a < argc; a++) {
    char pol[16];
    int S, K, A = 2;
    double W;
    const int got = sscanf(argv[a], "%15[^,],%d,%d,%lf,%d", pol, &S, &K, &W, &A);
    if (got < 4 || S < 1 || S > 64 || A < 1) { fprintf(stderr, "bad spec %s\n", argv[a]); return 2; }
    run(pol, S, K, W, A);
  }
  return 0;
}
