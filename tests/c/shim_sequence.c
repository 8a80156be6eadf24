/* The call sequence of the Rust shim (CudaEngine::load and
 * Engine::forward) through the C ABI, in C: laya_open_empty, one
 * laya_upload_weight_f32_graph per tensor with exactly what the reference's
 * unchanged loader hands out (Tensors::f32 values, Tensors::dims dims,
 * src/weights.rs:270-295), laya_finalize, laya_forward.  The tensors come
 * from a dump file written by a stand-in for that loader (tests/
 * test_shim_c.py); the result must equal, bit for bit, a second engine
 * opened with laya_open on the same GGUF.
 *
 * Usage: shim_sequence DUMP GGUF DEVICE
 * Dump: u32 count, then per tensor u32 name length, the name, u32 ndims,
 * i64 dims[ndims], f32 values (graph layout).
 * Exit status: 0 equal outputs; 1 a mismatch; 2 bad input; 3 the first
 * engine call failed (e.g. no usable GPU), its status printed. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "laya_b200.h"

static int fail(const char* what, int rc) {
  fprintf(stderr, "%s failed: status %d: %s\n", what, rc, laya_last_error());
  return rc;
}

static int read_u32(FILE* f, uint32_t* v) { return fread(v, 4, 1, f) == 1; }

int main(int argc, char** argv) {
  if (argc != 4) {
    fprintf(stderr, "usage: %s DUMP GGUF DEVICE\n", argv[0]);
    return 2;
  }
  const int device = atoi(argv[3]);
  laya_engine* shim = NULL;
  int rc = laya_open_empty(device, &shim);
  if (rc != LAYA_OK) {
    fail("laya_open_empty", rc);
    return 3;
  }
  FILE* f = fopen(argv[1], "rb");
  if (!f) {
    fprintf(stderr, "cannot open %s\n", argv[1]);
    laya_close(shim);
    return 2;
  }
  uint32_t count = 0;
  if (!read_u32(f, &count)) return 2;
  for (uint32_t t = 0; t < count; ++t) {
    uint32_t nlen = 0, nd = 0;
    char name[256];
    int64_t dims[4];
    if (!read_u32(f, &nlen) || nlen == 0 || nlen >= sizeof name || fread(name, 1, nlen, f) != nlen) return 2;
    name[nlen] = 0;
    if (!read_u32(f, &nd) || nd == 0 || nd > 4 || fread(dims, 8, nd, f) != nd) return 2;
    size_t el = 1;
    for (uint32_t d = 0; d < nd; ++d) el *= (size_t)dims[d];
    float* v = (float*)malloc(el * sizeof(float));
    if (!v || fread(v, sizeof(float), el, f) != el) return 2;
    rc = laya_upload_weight_f32_graph(shim, name, v, dims, (int)nd);
    free(v);
    if (rc != LAYA_OK) return fail(name, rc);
  }
  fclose(f);
  if ((rc = laya_finalize(shim)) != LAYA_OK) return fail("laya_finalize", rc);

  /* two sequences: 16 and 11 real tokens, 3 markers slots (one masked) */
  enum { N = 2, L = 16, K = 3 };
  int64_t ids[N * L], att[N * L], mpos[N * K] = {2, 5, 9, 3, 7, 0}, mmask[N * K] = {1, 1, 1, 1, 1, 0}, qtype[N] = {0, 2};
  for (int i = 0; i < N * L; ++i) {
    ids[i] = (i * 7919 + 13) % 50280;
    att[i] = (i / L == 1 && i % L >= 11) ? 0 : 1;
    if (!att[i]) ids[i] = 0;
  }
  ids[0] = 50281;
  ids[L] = 50281;
  for (int b = 0; b < N; ++b)
    for (int j = 0; j < K; ++j)
      if (mmask[b * K + j]) ids[b * L + mpos[b * K + j]] = 50284;
  laya_req req = {N, L, K, ids, att, mpos, mmask, qtype};
  float lg_shim[N * K], act_shim[N * 2], lg_ref[N * K], act_ref[N * 2];
  if ((rc = laya_forward(shim, &req, lg_shim, act_shim)) != LAYA_OK) return fail("laya_forward (shim)", rc);

  laya_engine* ref = NULL;
  if ((rc = laya_open(device, argv[2], &ref)) != LAYA_OK) return fail("laya_open", rc);
  if ((rc = laya_forward(ref, &req, lg_ref, act_ref)) != LAYA_OK) return fail("laya_forward (laya_open)", rc);
  int same = memcmp(lg_shim, lg_ref, sizeof lg_ref) == 0 && memcmp(act_shim, act_ref, sizeof act_ref) == 0;
  for (int i = 0; i < N * K; ++i) printf("logit %d: %.9g %.9g\n", i, lg_shim[i], lg_ref[i]);
  for (int i = 0; i < N * 2; ++i) printf("act %d: %.9g %.9g\n", i, act_shim[i], act_ref[i]);
  int finite = 1;
  for (int i = 0; i < N * K; ++i) finite &= isfinite(lg_shim[i]) != 0;
  laya_close(ref);
  laya_close(shim);
  printf(same && finite ? "shim sequence: identical outputs\n" : "shim sequence: MISMATCH\n");
  return same && finite ? 0 : 1;
}
