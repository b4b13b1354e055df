/*
 * CPU restatement (test oracle / "port" CPU baseline) of the reference's
 * source-exact FP4 linear: mosaicvm/kernels/fp4_source.py:132-156 and
 * mosaicvm/bench/vnni_source_kernel.c:8-47.
 *
 * y[m][n] = sum over 32-wide K groups g (ascending) of
 *           fp32(exact_int_dot(512*A, 2*W)) * (1/1024) * sa[m][g/4] * sw[n][g]
 * accumulated in fp32.  A = E4M3 codes (every finite code times 512 is an
 * integer), W = E2M1 codes (times 2 is an integer in [-12, 12]).
 * Plain C + OpenMP over output rows; no ISA-specific intrinsics.
 */
#include <stdint.h>
#include <stddef.h>

static int32_t e4m3_q512(uint8_t b) {
  /* value * 512 of an E4M3 (fn) code, as an exact integer; NaN codes map to 0 */
  int s = (b >> 7) & 1, e = (b >> 3) & 0xF, m = b & 7;
  int32_t v;
  if (e == 0xF && m == 7) return 0;
  if (e == 0) v = m;                       /* m * 2^-9 * 512 */
  else v = (8 + m) << (e - 1);             /* (1 + m/8) * 2^(e-7) * 512 */
  return s ? -v : v;
}

static const int8_t E2M1_Q2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

void fp4_linear_port(const uint8_t *q, const float *sa, const uint8_t *packed, const float *sw, float *y,
                     int M, int N, int K) {
  const int G = K / 32;
  #pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    int8_t w[32];
    for (int m = 0; m < M; m++) {
      float acc = 0.0f;
      for (int g = 0; g < G; g++) {
        const uint8_t *pw = packed + (size_t)n * (K / 2) + (size_t)g * 16;
        for (int i = 0; i < 16; i++) {
          w[2 * i] = E2M1_Q2[pw[i] & 0xF];
          w[2 * i + 1] = E2M1_Q2[pw[i] >> 4];
        }
        const uint8_t *pa = q + (size_t)m * K + (size_t)g * 32;
        int64_t dot = 0;
        for (int i = 0; i < 32; i++) dot += (int64_t)e4m3_q512(pa[i]) * w[i];
        float part = (float)dot * (1.0f / 1024.0f);
        part = part * sa[(size_t)m * (K / 128) + g / 4];
        part = part * sw[(size_t)n * G + g];
        acc = acc + part;
      }
      y[(size_t)m * N + n] = acc;
    }
  }
}
