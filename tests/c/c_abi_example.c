/* A plain C caller of the library (no torch, no C++), runnable.
 * Reads a problem from stdin (m n k group, then x as fp16 bits, qweight as int32, scales and
 * zeros as fp16 bits, all as decimal integers), runs the CPU path int4gemv_sequential on host
 * buffers, prints y's fp16 bits; then checks that a bad argument is rejected with a message. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "int4gemv_b200.h"

static int read_all(void* dst, size_t count, int bytes) {
  for (size_t i = 0; i < count; ++i) {
    long long v;
    if (scanf("%lld", &v) != 1) return 0;
    if (bytes == 2) ((uint16_t*)dst)[i] = (uint16_t)v;
    else ((int32_t*)dst)[i] = (int32_t)v;
  }
  return 1;
}

int main(void) {
  long long m, n, k, g;
  if (scanf("%lld %lld %lld %lld", &m, &n, &k, &g) != 4) return 2;
  uint16_t* x = malloc(sizeof(uint16_t) * m * k);
  int32_t* q = malloc(sizeof(int32_t) * n * (k / 8));
  uint16_t* s = malloc(sizeof(uint16_t) * n * (k / g));
  uint16_t* z = malloc(sizeof(uint16_t) * n * (k / g));
  uint16_t* y = malloc(sizeof(uint16_t) * m * n);
  if (!read_all(x, m * k, 2) || !read_all(q, n * (k / 8), 4) || !read_all(s, n * (k / g), 2) ||
      !read_all(z, n * (k / g), 2)) {
    return 3;
  }
  if (int4gemv_sequential(y, x, q, s, z, m, n, k, g, 1) != INT4GEMV_OK) {
    fprintf(stderr, "%s\n", int4gemv_last_error());
    return 4;
  }
  for (long long i = 0; i < m * n; ++i) printf("%u\n", (unsigned)y[i]);
  /* group 100 does not divide K: rejected before any work, with the reference's message */
  if (int4gemv_sequential(y, x, q, s, z, m, n, k, 100, 1) != INT4GEMV_ERR_INVALID) return 5;
  if (strstr(int4gemv_last_error(), "group_size 100") == NULL) return 6;
  printf("version %d\n", int4gemv_version());
  free(x); free(q); free(s); free(z); free(y);
  return 0;
}
