/*
 * C restatement of the coalesced GEMV model (reference src/pck/gemv.py:71-101,
 * `emulate_gemv_coalesced`) — TEST INFRASTRUCTURE ONLY: the parity checker and the timed
 * CPU baseline. The product never links or calls this file.
 *
 * Y[b, i] = sum_j W[i, j] * X[b, j] with binary32 products and additions in the kernel
 * order: chain t (0 <= t < threads) owns the vectors t, t + threads, t + 2*threads, ...
 * of `vec` consecutive columns and adds its terms one after another (the first term is
 * taken as is; columns >= n contribute +0); then the chains of each group of 32 are
 * reduced by halving (a[i] += a[i + 16], ..., a[i] += a[i + 1]) and the threads/32 group
 * sums are halved the same way.
 *
 * Built with -O2 -ffp-contract=off and without fast math, so every product and every sum
 * is one correctly rounded binary32 operation (x86-64 SSE arithmetic, subnormals kept).
 * Rows are split across OpenMP threads; the arithmetic per row is sequential.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { WEIGHT_BF16 = 0, WEIGHT_E4M3 = 1 };

static float g_e4m3[256];
static int g_e4m3_ready = 0;

static float bf16_bits_to_float(uint16_t bits) {
  uint32_t u = (uint32_t)bits << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* E4M3 (no infinities; S.1111.111 is NaN): 3 mantissa bits, exponent bias 7. */
static void init_e4m3(void) {
  if (g_e4m3_ready) return;
  for (int b = 0; b < 256; ++b) {
    const int sign = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) {
      v = NAN;
    } else if (e == 0) {
      v = ldexpf((float)m, -9); /* m/8 * 2^-6 */
    } else {
      v = ldexpf((float)(8 + m), e - 10); /* (1 + m/8) * 2^(e-7) */
    }
    g_e4m3[b] = sign ? -v : v;
  }
  g_e4m3_ready = 1;
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static void halve(float* a, int len) {
  for (int h = len / 2; h >= 1; h /= 2) {
    for (int i = 0; i < h; ++i) a[i] = a[i] + a[i + h];
  }
}

/* Returns 0 on success, a positive code for a rejected argument. */
int oracle_gemv_coalesced(const void* W, int weight_format, const uint16_t* X, float* Y,
                          int64_t m, int64_t n, int64_t batch, int threads, int vec,
                          int cpu_threads) {
  if (m < 0 || n < 1 || batch < 1) return 1;
  if (threads < 32 || threads > 4096 || (threads & (threads - 1))) return 2;
  if (vec < 1) return 3;
  if (weight_format != WEIGHT_BF16 && weight_format != WEIGHT_E4M3) return 4;
  init_e4m3();
  const int64_t vectors = (n + vec - 1) / vec;
  const int64_t per_thread = (vectors + threads - 1) / threads;
  const int groups = threads / 32;

  float* xf = (float*)malloc(sizeof(float) * (size_t)(n * batch));
  if (!xf) return 5;
  for (int64_t j = 0; j < n * batch; ++j) xf[j] = bf16_bits_to_float(X[j]);

  int bad = 0;
#pragma omp parallel num_threads(cpu_threads > 0 ? cpu_threads : 1)
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)threads);
    float* wrow = (float*)malloc(sizeof(float) * (size_t)n);
    if (!acc || !wrow) {
#pragma omp atomic write
      bad = 1;
    } else {
#pragma omp for schedule(static)
      for (int64_t i = 0; i < m; ++i) {
        if (weight_format == WEIGHT_BF16) {
          const uint16_t* w = (const uint16_t*)W + i * n;
          for (int64_t j = 0; j < n; ++j) wrow[j] = bf16_bits_to_float(w[j]);
        } else {
          const uint8_t* w = (const uint8_t*)W + i * n;
          for (int64_t j = 0; j < n; ++j) wrow[j] = g_e4m3[w[j]];
        }
        for (int64_t b = 0; b < batch; ++b) {
          const float* x = xf + b * n;
          for (int64_t v = 0; v < per_thread; ++v) {
            for (int t = 0; t < threads; ++t) {
              const int64_t base = (v * threads + t) * vec;
              for (int k = 0; k < vec; ++k) {
                const int64_t col = base + k;
                const float p = col < n ? wrow[col] * x[col] : 0.0f;
                if (v == 0 && k == 0) {
                  acc[t] = p;
                } else {
                  acc[t] = acc[t] + p;
                }
              }
            }
          }
          for (int g = 0; g < groups; ++g) halve(acc + 32 * g, 32);
          /* group sums sit at acc[32 g]; gather and halve them */
          for (int g = 0; g < groups; ++g) acc[g] = acc[32 * g];
          halve(acc, groups);
          Y[b * m + i] = acc[0];
        }
      }
    }
    free(acc);
    free(wrow);
  }
  free(xf);
  return bad ? 5 : 0;
}
