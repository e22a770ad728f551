/* Tabulate every finite binary32 input x where the host libm expf(x) differs
 * from exp(x) rounded once to binary32 (the device computes the latter).
 *
 * rai-infer's attention softmax tail and MoE router call f32::exp, which is
 * the host libm's expf; it is not correctly rounded for a small fraction of
 * inputs, and the decode path quantizes its activations to int8, so a 1-ulp
 * softmax difference can move a quantization step. The device applies this
 * table on top of its correctly rounded exp to return exactly what the host
 * libm returns.
 *
 * Output (little-endian): u32 magic "EXP2", u32 count, the 32-byte
 * NUL-padded glibc version string the table was made with, count sorted u32
 * input bit patterns, count u32 result bit patterns. The library refuses a
 * table made with another glibc than the one it runs with.
 *
 *   gcc -O2 -fopenmp gen_expf_table.c -o gen -lm && ./gen out.bin
 */
#include <gnu/libc-version.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static int differs(uint32_t u, uint32_t* got) {
  float x, g, d;
  memcpy(&x, &u, 4);
  if (isnan(x)) return 0;
  g = expf(x);
  d = (float)exp((double)x);
  uint32_t gb, db;
  memcpy(&gb, &g, 4);
  memcpy(&db, &d, 4);
  *got = gb;
  return gb != db;
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const int nthreads = omp_get_max_threads();
  const uint64_t total = 1ull << 32;
  uint32_t** keys = calloc(nthreads, sizeof(uint32_t*));
  uint32_t** vals = calloc(nthreads, sizeof(uint32_t*));
  size_t* counts = calloc(nthreads, sizeof(size_t));
  size_t* caps = calloc(nthreads, sizeof(size_t));
#pragma omp parallel
  {
    int t = omp_get_thread_num();
    uint64_t lo = total * t / nthreads, hi = total * (t + 1) / nthreads;
    caps[t] = 1 << 16;
    keys[t] = malloc(caps[t] * 4);
    vals[t] = malloc(caps[t] * 4);
    for (uint64_t v = lo; v < hi; ++v) {
      uint32_t got;
      if (differs((uint32_t)v, &got)) {
        if (counts[t] == caps[t]) {
          caps[t] *= 2;
          keys[t] = realloc(keys[t], caps[t] * 4);
          vals[t] = realloc(vals[t], caps[t] * 4);
        }
        keys[t][counts[t]] = (uint32_t)v;
        vals[t][counts[t]] = got;
        counts[t]++;
      }
    }
  }
  size_t n = 0;
  for (int t = 0; t < nthreads; ++t) n += counts[t];
  FILE* f = fopen(argv[1], "wb");
  if (!f) return 1;
  uint32_t hdr[2] = {0x32505845u, (uint32_t)n};
  char ver[32] = {0};
  strncpy(ver, gnu_get_libc_version(), sizeof(ver) - 1);
  fwrite(hdr, 4, 2, f);
  fwrite(ver, 1, sizeof(ver), f);
  /* thread ranges are ascending, so concatenation is sorted */
  for (int t = 0; t < nthreads; ++t) fwrite(keys[t], 4, counts[t], f);
  for (int t = 0; t < nthreads; ++t) fwrite(vals[t], 4, counts[t], f);
  fclose(f);
  printf("%zu exceptions\n", n);
  return 0;
}
