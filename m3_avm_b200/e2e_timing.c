/*
 * e2e_timing.c -- times the host-buffer GEMV call of libm3gemv from C.
 *
 * A Rust caller binds the C ABI directly (no interpreter between it and the
 * library), so this is the cost such a caller pays per call of
 * m3g_offload_matvec: copy x in, run the GEMV on resident weights, copy y
 * out, check the kernel status, return.  The weights (GGUF bytes read from a
 * file) are uploaded as `copies` resident tensors and the calls rotate over
 * them, so every call streams its weights from HBM rather than L2.
 *
 *   m3g_e2e_timing <weights file> <dtype> <in_dim> <out_dim> <copies> <calls> <warmup>
 *
 * Prints one JSON object: the mean and the best of 8 windows, in
 * microseconds per call, measured with CLOCK_MONOTONIC around the calls.
 */
#define _POSIX_C_SOURCE 199309L
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <time.h>

#include "m3gemv.h"

static double now_s(void) {
  struct timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

int main(int argc, char** argv) {
  if (argc != 8) {
    fprintf(stderr, "usage: %s weights dtype in_dim out_dim copies calls warmup\n", argv[0]);
    return 2;
  }
  const char* path = argv[1];
  const uint32_t dtype = (uint32_t)strtoul(argv[2], NULL, 10);
  const uint64_t in_dim = strtoull(argv[3], NULL, 10), out_dim = strtoull(argv[4], NULL, 10);
  const int copies = atoi(argv[5]), calls = atoi(argv[6]), warmup = atoi(argv[7]);
  if (copies < 1 || calls < 8 || warmup < 0) {
    fprintf(stderr, "need copies >= 1, calls >= 8, warmup >= 0\n");
    return 2;
  }
  FILE* f = fopen(path, "rb");
  if (!f) {
    perror(path);
    return 1;
  }
  fseek(f, 0, SEEK_END);
  const long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  uint8_t* raw = (uint8_t*)malloc((size_t)n);
  if (!raw || fread(raw, 1, (size_t)n, f) != (size_t)n) {
    fprintf(stderr, "cannot read %s\n", path);
    return 1;
  }
  fclose(f);

  m3g_offload* ctx = NULL;
  if (m3g_offload_create(0, in_dim, out_dim, &ctx) != M3G_OK) {
    fprintf(stderr, "m3g_offload_create: %s\n", m3g_last_error());
    return 1;
  }
  for (int c = 0; c < copies; ++c) {
    if (m3g_offload_upload(ctx, (uint64_t)c, dtype, raw, (uint64_t)n, in_dim, out_dim) != M3G_OK) {
      fprintf(stderr, "m3g_offload_upload: %s\n", m3g_last_error());
      return 1;
    }
  }
  float* x = (float*)malloc(sizeof(float) * in_dim);
  float* y = (float*)malloc(sizeof(float) * out_dim);
  uint32_t s = 12345u;
  for (uint64_t i = 0; i < in_dim; ++i) {  /* any finite x: the timing does not depend on its values */
    s = s * 1664525u + 1013904223u;
    x[i] = (float)((int32_t)(s >> 8) - (1 << 23)) / (float)(1 << 23);
  }
  for (int i = 0; i < warmup; ++i) {
    if (m3g_offload_matvec(ctx, (uint64_t)(i % copies), x, in_dim, out_dim, y) != M3G_OK) {
      fprintf(stderr, "m3g_offload_matvec: %s\n", m3g_last_error());
      return 1;
    }
  }
  const int windows = 8, per = calls / windows;
  double best = 1e30, total = 0.0;
  int done = 0;
  for (int w = 0; w < windows; ++w) {
    const double t0 = now_s();
    for (int i = 0; i < per; ++i, ++done) {
      if (m3g_offload_matvec(ctx, (uint64_t)(done % copies), x, in_dim, out_dim, y) != M3G_OK) {
        fprintf(stderr, "m3g_offload_matvec: %s\n", m3g_last_error());
        return 1;
      }
    }
    const double dt = now_s() - t0;
    total += dt;
    if (dt / per < best) best = dt / per;
  }
  printf("{\"us_per_call\": %.3f, \"best_window_us_per_call\": %.3f, \"calls\": %d, \"copies\": %d, "
         "\"y0\": %.6g}\n",
         1e6 * total / done, 1e6 * best, done, copies, (double)y[0]);
  m3g_offload_destroy(ctx);
  free(raw);
  free(x);
  free(y);
  return 0;
}
