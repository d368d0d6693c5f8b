/* split_c_host.c - the library's multi-GPU sequence split driven from a plain
 * C host: no Python, no framework, no CUDA headers (host buffers only).
 *
 *   split_c_host <rank> <world> <id-file>
 *
 * Every rank builds the same seeded K/V for two sequences, keeps its
 * page-aligned slice of the positions in its own caches on GPU <rank>, and
 * runs eakv_decode_attention_split_host over a communicator whose NCCL id
 * rank 0 writes to <id-file> (the others wait for it, bounded). Each rank
 * also decodes the whole sequences on its own GPU with
 * eakv_decode_attention_host and checks the merged result against that,
 * element by element, within 1e-4 abs + 1e-4 rel. Prints "ok <max error>"
 * and exits 0 on success.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "eakv_nccl.h"

enum { L = 2, NKV = 4, NQ = 16, HD = 128, S = 1000, B = 2 };

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;

static double uniform01(void) {   /* splitmix64 */
  uint64_t z = (rng_state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return ((z >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static float normal(void) {       /* Box-Muller */
  double u = uniform01(), v = uniform01();
  return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

static int fail(const char *what) {
  fprintf(stderr, "%s: %s\n", what, eakv_last_error_string());
  return 1;
}

int main(int argc, char **argv) {
  if (argc != 4) {
    fprintf(stderr, "usage: %s <rank> <world> <id-file>\n", argv[0]);
    return 2;
  }
  const int rank = atoi(argv[1]), world = atoi(argv[2]);
  const char *id_path = argv[3];
  if (eakv_set_device(rank) != EAKV_OK) return fail("set_device");

  /* the same data on every rank: kv[b][l][kv][h][t][d], q[b][l][h][d] */
  const size_t per_seq = (size_t)L * 2 * NKV * S * HD;
  float *kv = malloc(B * per_seq * sizeof(float));
  float *q = malloc((size_t)B * L * NQ * HD * sizeof(float));
  float *out = malloc((size_t)B * L * NQ * HD * sizeof(float));
  float *ref = malloc((size_t)B * L * NQ * HD * sizeof(float));
  for (size_t i = 0; i < B * per_seq; i++) kv[i] = normal();
  for (size_t i = 0; i < (size_t)B * L * NQ * HD; i++) q[i] = normal();

  /* reference: the whole sequences on this rank's GPU */
  eakv_cache_t *full[B];
  for (int b = 0; b < B; b++) {
    full[b] = eakv_cache_create(L, NKV, HD, S);
    if (!full[b] || eakv_cache_load_raw(full[b], kv + b * per_seq, S) != EAKV_OK)
      return fail("full cache");
  }
  if (eakv_decode_attention_host((const eakv_cache_t *const *)full, B, q, NQ, ref, NULL) !=
      EAKV_OK)
    return fail("decode_attention_host");

  /* this rank's page-aligned slice [lo, hi) of every sequence */
  int per = (S + world - 1) / world;
  per = (per + 63) / 64 * 64;
  const int lo = rank * per < S ? rank * per : S;
  const int hi = rank == world - 1 ? S : (lo + per < S ? lo + per : S);
  const int n = hi - lo;
  float *slice = malloc((size_t)L * 2 * NKV * (n > 0 ? n : 1) * HD * sizeof(float));
  eakv_cache_t *mine[B];
  for (int b = 0; b < B; b++) {
    mine[b] = eakv_cache_create(L, NKV, HD, n > 0 ? n : 1);
    if (!mine[b]) return fail("slice cache");
    if (n > 0) {
      for (int lk = 0; lk < L * 2 * NKV; lk++)
        memcpy(slice + (size_t)lk * n * HD, kv + b * per_seq + ((size_t)lk * S + lo) * HD,
               (size_t)n * HD * sizeof(float));
      if (eakv_cache_load_raw(mine[b], slice, n) != EAKV_OK) return fail("slice load");
    }
  }

  /* the NCCL id travels through a file: rank 0 writes it, the others wait */
  char id[EAKV_NCCL_ID_BYTES];
  if (rank == 0) {
    char tmp[4096];
    snprintf(tmp, sizeof tmp, "%s.tmp", id_path);
    if (eakv_nccl_unique_id(id) != EAKV_OK) return fail("nccl_unique_id");
    FILE *f = fopen(tmp, "wb");
    if (!f || fwrite(id, 1, sizeof id, f) != sizeof id || fclose(f) != 0) return 1;
    if (rename(tmp, id_path) != 0) return 1;
  } else {
    FILE *f = NULL;
    for (int i = 0; i < 600 && !f; i++) {   /* at most 60 s */
      f = fopen(id_path, "rb");
      if (!f) usleep(100000);
    }
    if (!f || fread(id, 1, sizeof id, f) != sizeof id) return 1;
    fclose(f);
  }
  void *comm = NULL;
  if (eakv_nccl_comm_init(&comm, world, id, rank, rank) != EAKV_OK) return fail("comm_init");
  if (eakv_decode_attention_split_host((const eakv_cache_t *const *)mine, B, q, NQ, out, comm,
                                       NULL) != EAKV_OK)
    return fail("decode_attention_split_host");

  double worst = 0.0;
  int bad = 0;
  for (size_t i = 0; i < (size_t)B * L * NQ * HD; i++) {
    const double e = fabs((double)out[i] - (double)ref[i]);
    if (!(e <= 1e-4 + 1e-4 * fabs((double)ref[i]))) bad++;
    if (e > worst) worst = e;
  }
  eakv_nccl_comm_destroy(comm);
  for (int b = 0; b < B; b++) {
    eakv_cache_free(mine[b]);
    eakv_cache_free(full[b]);
  }
  free(kv);
  free(q);
  free(out);
  free(ref);
  free(slice);
  if (bad) {
    fprintf(stderr, "rank %d: %d elements outside the bar, worst %.3e\n", rank, bad, worst);
    return 1;
  }
  printf("ok %.3e\n", worst);
  return 0;
}
