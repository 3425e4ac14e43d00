/*
 * CPU oracle for the W4A16 GEMV path. TEST INFRASTRUCTURE ONLY: the tests, the smoke check and
 * the CPU-baseline leg of bench.py call this as the checker. Nothing in the shipped library links
 * or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference project (Yu-TingLee/int4-GEMV-cuda):
 *   - quantize / pack / unpack / dequantize    int4gemv/quant.py:14-53
 *   - the single-threaded CPU GEMV             csrc/sequential.cpp:11-54
 *   - the fp32 dequantise-then-matmul oracle   int4gemv/reference.py:8-10 (here accumulated in
 *     double, so it is a tighter reference than torch's fp32 matmul, whose summation order is
 *     BLAS-specific and not reproducible)
 *
 * Layout (csrc/w4a16.h:10-16): x [M, K] fp16, qweight [N, K/8] int32 with weight k of a row in
 * bits 4*(k%8) .. 4*(k%8)+3 of word k/8, scales and zeros [N, K/group] fp16, y [M, N] fp16.
 *
 * Build with -O2 -ffp-contract=off and without -ffast-math: every float operation below then
 * rounds exactly as the reference's C++ and torch code does (IEEE binary32, round to nearest even),
 * which makes `oracle_sequential` bit-exact with csrc/sequential.cpp and `oracle_quantize` /
 * `oracle_dequantize` bit-exact with int4gemv/quant.py.
 *
 * Pinned by tests/test_oracle.py against golden vectors made by the reference itself
 * (tests/golden/make_golden.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* IEEE binary16 <-> binary32. _Float16 conversions in GCC are exact (half -> float) and round to
 * nearest even (float -> half), the same as c10::Half and torch's .half(). */
static inline float h2f(uint16_t bits) {
  _Float16 h;
  memcpy(&h, &bits, sizeof h);
  return (float)h;
}

static inline uint16_t f2h(float f) {
  _Float16 h = (_Float16)f;
  uint16_t bits;
  memcpy(&bits, &h, sizeof bits);
  return bits;
}

void oracle_half_to_float(const uint16_t* in, float* out, int64_t count) {
  for (int64_t i = 0; i < count; ++i) out[i] = h2f(in[i]);
}

void oracle_float_to_half(const float* in, uint16_t* out, int64_t count) {
  for (int64_t i = 0; i < count; ++i) out[i] = f2h(in[i]);
}

/* quant.py:40-44: q[n, 8w + j] = (qweight[n, w] >> 4j) & 0xF. */
void oracle_unpack(const int32_t* qweight, int32_t* q, int64_t n, int64_t k) {
  const int64_t words = k / 8;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t w = 0; w < words; ++w) {
      const uint32_t word = (uint32_t)qweight[r * words + w];
      for (int j = 0; j < 8; ++j) q[r * k + 8 * w + j] = (int32_t)((word >> (4 * j)) & 0xFu);
    }
  }
}

/* quant.py:32-37: word = sum over j of q[8w + j] << 4j, computed there in int64 and cast to int32,
 * i.e. modulo 2^32. Values outside 0..15 are not masked: they carry into the neighbouring
 * nibbles exactly as in the reference. For 0..15 this is the inverse of unpack. */
void oracle_pack(const int32_t* q, int32_t* qweight, int64_t n, int64_t k) {
  const int64_t words = k / 8;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t w = 0; w < words; ++w) {
      uint32_t word = 0; /* unsigned arithmetic wraps modulo 2^32 */
      for (int j = 0; j < 8; ++j) word += (uint32_t)q[r * k + 8 * w + j] << (4 * j);
      qweight[r * words + w] = (int32_t)word;
    }
  }
}

/* quant.py:47-53: w = (float(q) - float(z)) * float(s), one fp32 subtraction and one fp32
 * multiplication per weight. */
void oracle_dequantize(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                       float* w, int64_t n, int64_t k, int64_t group_size) {
  const int64_t words = k / 8;
  const int64_t groups = k / group_size;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t i = 0; i < k; ++i) {
      const uint32_t word = (uint32_t)qweight[r * words + i / 8];
      const float q = (float)((word >> (4 * (i % 8))) & 0xFu);
      const float s = h2f(scales[r * groups + i / group_size]);
      const float z = h2f(zeros[r * groups + i / group_size]);
      w[r * k + i] = (q - z) * s;
    }
  }
}

/* quant.py:14-29, bit for bit:
 *   lo = min(min over group, 0); hi = max(max over group, 0)
 *   s  = fp16(max((hi - lo) / 15, 1e-6f)) read back as fp32
 *   z  = clamp(rint(-lo / s), 0, 15)
 *   q  = clamp(rint(w / s + z), 0, 15)        rint = round half to even, as torch.round
 * then pack. */
void oracle_quantize(const float* w, int32_t* qweight, uint16_t* scales, uint16_t* zeros,
                     int32_t* q_scratch, int64_t n, int64_t k, int64_t group_size) {
  const int64_t groups = k / group_size;
  for (int64_t r = 0; r < n; ++r) {
    for (int64_t g = 0; g < groups; ++g) {
      const float* wg = w + r * k + g * group_size;
      float lo = wg[0], hi = wg[0];
      for (int64_t i = 1; i < group_size; ++i) {
        if (wg[i] < lo) lo = wg[i];
        if (wg[i] > hi) hi = wg[i];
      }
      if (lo > 0.0f) lo = 0.0f;
      if (hi < 0.0f) hi = 0.0f;
      float s = (hi - lo) / 15.0f;
      if (s < 1e-6f) s = 1e-6f;
      const uint16_t s_bits = f2h(s);
      s = h2f(s_bits);
      float z = nearbyintf(-lo / s);
      if (z < 0.0f) z = 0.0f;
      if (z > 15.0f) z = 15.0f;
      scales[r * groups + g] = s_bits;
      zeros[r * groups + g] = f2h(z);
      for (int64_t i = 0; i < group_size; ++i) {
        const float t = wg[i] / s;
        float v = nearbyintf(t + z);
        if (v < 0.0f) v = 0.0f;
        if (v > 15.0f) v = 15.0f;
        q_scratch[r * k + g * group_size + i] = (int32_t)v;
      }
    }
  }
  oracle_pack(q_scratch, qweight, n, k);
}

/* csrc/sequential.cpp:11-54, in the same order of operations: for each output row and group, the
 * 128 (group_size) weights are dequantised into w[] as (q - z) * s; for each row m of x a fp32 dot
 * product over the group is accumulated left to right and then added to acc[m]; at the end acc is
 * rounded to fp16. w_scratch holds group_size floats, acc_scratch holds m floats and
 * x_scratch m * k floats. */
void oracle_sequential(const uint16_t* x, const int32_t* qweight, const uint16_t* scales,
                       const uint16_t* zeros, uint16_t* y, int64_t m, int64_t n, int64_t k,
                       int64_t group_size, float* x_scratch, float* w_scratch,
                       float* acc_scratch) {
  const int64_t groups = k / group_size;
  const int64_t words = k / 8;
  for (int64_t i = 0; i < m * k; ++i) x_scratch[i] = h2f(x[i]);
  for (int64_t row = 0; row < n; ++row) {
    for (int64_t r = 0; r < m; ++r) acc_scratch[r] = 0.0f;
    for (int64_t g = 0; g < groups; ++g) {
      const float s = h2f(scales[row * groups + g]);
      const float z = h2f(zeros[row * groups + g]);
      const int32_t* wordp = qweight + row * words + g * (group_size / 8);
      for (int64_t i = 0; i < group_size; ++i) {
        const uint32_t q = ((uint32_t)wordp[i / 8] >> (4 * (i % 8))) & 0xFu;
        w_scratch[i] = ((float)q - z) * s;
      }
      for (int64_t r = 0; r < m; ++r) {
        const float* xg = x_scratch + r * k + g * group_size;
        float sum = 0.0f;
        for (int64_t i = 0; i < group_size; ++i) sum += xg[i] * w_scratch[i];
        acc_scratch[r] += sum;
      }
    }
    for (int64_t r = 0; r < m; ++r) y[r * n + row] = f2h(acc_scratch[r]);
  }
}

/* reference.py:8-10, x.float() @ dequantize(W).T, with the dot products accumulated in double.
 * Output fp32 [M, N]. w_scratch holds k floats. */
void oracle_reference(const uint16_t* x, const int32_t* qweight, const uint16_t* scales,
                      const uint16_t* zeros, float* y, int64_t m, int64_t n, int64_t k,
                      int64_t group_size, float* w_scratch) {
  for (int64_t row = 0; row < n; ++row) {
    oracle_dequantize(qweight + row * (k / 8), scales + row * (k / group_size),
                      zeros + row * (k / group_size), w_scratch, 1, k, group_size);
    for (int64_t r = 0; r < m; ++r) {
      double acc = 0.0;
      for (int64_t i = 0; i < k; ++i) acc += (double)h2f(x[r * k + i]) * (double)w_scratch[i];
      y[r * n + row] = (float)acc;
    }
  }
}
