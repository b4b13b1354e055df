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

/*
 * fp32-activation linear on the dequantised weights (the bf16 path of the
 * oracle, mosaicvm/model/layers.py:348-366 on runtime/fp8.py:19-34 weights):
 * y[m][n] = sum_k x[m][k] * E2M1(code[n][k]) * sw[n][k/32], accumulated in
 * double and rounded once to fp32 (every product is exact in double).
 */
static const float E2M1_F[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                 -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

void fp4_linear_f32(const float *x, const uint8_t *packed, const float *sw, float *y, int M, int N, int K) {
  const int G = K / 32;
  #pragma omp parallel
  {
    double *wrow = (double *)__builtin_alloca(sizeof(double) * (size_t)K);
    #pragma omp for schedule(static)
    for (int n = 0; n < N; n++) {
      const uint8_t *pw = packed + (size_t)n * (K / 2);
      for (int g = 0; g < G; g++) {
        const double s = (double)sw[(size_t)n * G + g];
        for (int i = 0; i < 16; i++) {
          const uint8_t b = pw[g * 16 + i];
          wrow[g * 32 + 2 * i] = (double)E2M1_F[b & 0xF] * s;
          wrow[g * 32 + 2 * i + 1] = (double)E2M1_F[b >> 4] * s;
        }
      }
      for (int m = 0; m < M; m++) {
        const float *xr = x + (size_t)m * K;
        double acc = 0.0;
        for (int k = 0; k < K; k++) acc += (double)xr[k] * wrow[k];
        y[(size_t)m * N + n] = (float)acc;
      }
    }
  }
}

/*
 * Operand preparation of the reference's AVX-VNNI CPU kernel, in C (its own
 * numpy preparation, mosaicvm/bench/vnni_source.py:38-54, takes ~0.3 s per
 * V3 gate/up matrix): weights as 2*E2M1 int8 tiled [N/8][K/4][8][4] and the
 * per-32 int32 weight sums [N][K/32].
 */
void vnni_prepare(const uint8_t *packed, int N, int K, int8_t *tiled, int32_t *sums) {
  const int G = K / 32;
  #pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    const uint8_t *pw = packed + (size_t)n * (K / 2);
    for (int g = 0; g < G; g++) {
      int32_t s = 0;
      for (int i = 0; i < 32; i++) {
        const int c = g * 32 + i;
        const uint8_t b = pw[c >> 1];
        const int8_t q = E2M1_Q2[(c & 1) ? (b >> 4) : (b & 0xF)];
        s += q;
        tiled[(((size_t)(n >> 3) * (K >> 2) + (c >> 2)) << 5) + ((n & 7) << 2) + (c & 3)] = q;
      }
      sums[(size_t)n * G + g] = s;
    }
  }
}
