/*
 * C restatement of the reference's CPU GEMM check: TEST INFRASTRUCTURE ONLY (only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs load it; the product never does).
 *
 *   oracle_bf16_to_f32 / oracle_f32_to_bf16: the codec of
 *     scripts/generate_fixed_bf16_dataset.py:32-48 (RNE by adding 0x7FFF + lsb, no NaN case).
 *   oracle_gemm_f64: C = A_q . B_q accumulated in double over BF16 inputs, row-major, the
 *     exact-as-possible value that the float32 numpy product of generator :122 approximates.
 *   oracle_gemm_f32_rows: float32 accumulation in plain k order over a row band, the scalar
 *     CPU baseline used by the benchmark's "port" leg when numpy/BLAS is not used.
 *   oracle_check: the runner's pass rule |out-ref| <= atol + rtol*|ref| and its statistics
 *     (src/runner/main.cpp:324-365), except that a NaN output fails here.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

void oracle_bf16_to_f32(const uint16_t* in, float* out, int64_t count) {
  for (int64_t i = 0; i < count; ++i) out[i] = bits_to_f32(in[i]);
}

void oracle_f32_to_bf16(const float* in, uint16_t* out, int64_t count) {
  for (int64_t i = 0; i < count; ++i) {
    uint32_t u;
    memcpy(&u, &in[i], sizeof u);
    const uint32_t lsb = (u >> 16) & 1u;
    out[i] = (uint16_t)((u + 0x7FFFu + lsb) >> 16);
  }
}

void oracle_gemm_f64(const uint16_t* a, const uint16_t* b, double* c, int m, int n, int k) {
  for (int i = 0; i < m; ++i) {
    double* crow = c + (int64_t)i * n;
    for (int j = 0; j < n; ++j) crow[j] = 0.0;
    for (int p = 0; p < k; ++p) {
      const double av = (double)bits_to_f32(a[(int64_t)i * k + p]);
      if (av == 0.0) continue;
      const uint16_t* brow = b + (int64_t)p * n;
      for (int j = 0; j < n; ++j) crow[j] += av * (double)bits_to_f32(brow[j]);
    }
  }
}

void oracle_gemm_f32_rows(const uint16_t* a, const uint16_t* b, float* c, int row_begin,
                          int row_end, int n, int k) {
  for (int i = row_begin; i < row_end; ++i) {
    float* crow = c + (int64_t)(i - row_begin) * n;
    for (int j = 0; j < n; ++j) crow[j] = 0.0f;
    for (int p = 0; p < k; ++p) {
      const float av = bits_to_f32(a[(int64_t)i * k + p]);
      const uint16_t* brow = b + (int64_t)p * n;
      for (int j = 0; j < n; ++j) crow[j] += av * bits_to_f32(brow[j]);
    }
  }
}

/* stats[0]=max_abs stats[1]=max_rel stats[2]=mean_abs; returns 1 when every element passes. */
int oracle_check(const uint16_t* out, const float* ref, int64_t count, double atol, double rtol,
                 double* stats) {
  int passed = 1;
  double max_abs = 0.0, max_rel = 0.0, sum = 0.0;
  for (int64_t i = 0; i < count; ++i) {
    const double o = (double)bits_to_f32(out[i]);
    const double r = (double)ref[i];
    const double e = fabs(o - r);
    const double rel = e / (fabs(r) > 1.0e-12 ? fabs(r) : 1.0e-12);
    if (e > max_abs) max_abs = e;
    if (rel > max_rel) max_rel = rel;
    sum += e;
    /* Written as !(e <= tol) so that a NaN output fails; the reference's `e > tol` lets a
       NaN through (main.cpp:354), which this checker deliberately does not copy. */
    if (!(e <= atol + rtol * fabs(r))) passed = 0;
  }
  stats[0] = max_abs;
  stats[1] = max_rel;
  stats[2] = count ? sum / (double)count : 0.0;
  return passed;
}
