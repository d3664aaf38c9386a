/*
 * CPU restatement of QwenEdit's fused NVFP4 Triton kernels — TEST ORACLE (see oracle/__init__.py).
 *
 * Follows multi_turn/fibo/fp4.py:
 *   _e2m1           :37-43   thresholds {>0.25, >=0.75, >1.25, >=1.75, >2.5, >=3.5, >5.0}, sign bit 3
 *   _quantize_store :46-61   16-value groups: sf = e4m3(gs * (amax * (1/6))); scale = 1 / (sf * (1 / gs));
 *                            codes = e2m1(v * scale); byte = even | odd << 4; 128x4-swizzled scale offsets
 *   _norm_scale_fp4_kernel :64-80  rstd = rsqrt(sum(x*x) / K + eps); y = bf16(bf16(bf16(x*rstd) * w) * bf16(1 + mod));
 *                            mod = noisy or clean per token mask; rows past M store zero scales
 *   _silu_mul_fp4_kernel   :83-91  y = bf16(bf16(g / (1 + exp(-g))) * v)
 * with the roundings the GPU executes (bf16 round-to-nearest-even, e4m3 round-to-nearest-even with
 * saturation, IEEE fp32 arithmetic). Choices where the reference leaves the bits to the backend:
 *   - tl.sum order: numpy's pairwise summation over the zero-padded next_pow2(K) block (what the reference
 *     kernel executes under Triton's interpreter, where tl.sum is np.sum);
 *   - rsqrt: 1 / sqrt with both steps correctly rounded (the interpreter's definition);
 *   - exp: Cody-Waite reduction + degree-7 Taylor polynomial with fmaf + exact 2^n rebuild (< 1 ulp).
 * Build: oracle/Makefile (gcc, -ffp-contract=off so no multiply-add is fused behind our back).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float f_from_u(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t u_from_f(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

float ref_bf16_to_f(uint16_t h) { return f_from_u((uint32_t)h << 16); }

uint16_t ref_f_to_bf16(float f) {
  uint32_t u = u_from_f(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float ref_bf16_round(float f) { return ref_bf16_to_f(ref_f_to_bf16(f)); }

/* e4m3 (bias 7, no infinities, 0x7f NaN): round to nearest even, saturate to +-448. */
uint8_t ref_e4m3(float v) {
  if (isnan(v)) return 0x7f;
  uint8_t sign = signbit(v) ? 0x80 : 0;
  float a = fabsf(v);
  if (a >= 448.0f) return sign | 0x7e;
  if (a == 0.0f) return sign;
  int e;
  frexpf(a, &e);
  int E = e - 1;          /* 2^E <= a < 2^(E+1) */
  if (E < -6) E = -6;     /* subnormal spacing below 2^-6 */
  float spacing = ldexpf(1.0f, E - 3);
  float qv = rintf(a / spacing);
  if (E == -6 && qv < 8.0f) return sign | (uint8_t)qv;
  if (qv >= 16.0f) {
    qv = 8.0f;
    E += 1;
  }
  return sign | (uint8_t)(((E + 7) << 3) | ((int)qv - 8));
}

float ref_e4m3_value(uint8_t b) {
  uint32_t e = (b >> 3) & 15u, m = b & 7u;
  if (e == 15u && m == 7u) return NAN;
  float mag = e == 0 ? (float)m * 0.001953125f : ldexpf((float)(8u + m), (int)e - 10);
  return (b & 0x80u) ? -mag : mag;
}

uint8_t ref_e2m1(float v) {
  float a = fabsf(v);
  int c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
  return (uint8_t)(c | ((v < 0.0f) << 3));
}

static float pow2i(int e) { return f_from_u((uint32_t)(e + 127) << 23); }

float ref_exp(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208404541015625f) return 0.0f;
  float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.428606765330187045e-06f, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333377e-3f);
  p = fmaf(p, r, 4.16666679e-2f);
  p = fmaf(p, r, 1.66666672e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  int e1 = ni / 2, e2 = ni - e1;
  return (p * pow2i(e1)) * pow2i(e2);
}

/* numpy's pairwise summation (float32 accumulators): blocks of <= 128 with 8 interleaved partial sums,
 * halved at multiples of 8 above that. */
static float pairwise(const float *a, int64_t n) {
  if (n < 8) {
    float res = 0.0f;
    for (int64_t i = 0; i < n; ++i) res += a[i];
    return res;
  }
  if (n <= 128) {
    float r[8];
    int64_t i;
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    for (i = 8; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
    return res;
  }
  int64_t n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise(a, n2) + pairwise(a + n2, n - n2);
}

float ref_pairwise_sum(const float *a, int64_t n) { return pairwise(a, n); }

static int64_t sf_offset(int64_t m, int64_t g, int64_t K) {
  return (m / 128) * (K / 64 * 512) + (g / 4) * 512 + (m % 32) * 16 + (m % 128 / 32) * 4 + g % 4;
}

/* quantise one row's K values y (already bf16-rounded) */
static void quantize_row(const float *y, int64_t m, int64_t K, float gs, uint8_t *q, uint8_t *sf) {
  float inv_gs = 1.0f / gs;
  for (int64_t g = 0; g < K / 16; ++g) {
    const float *v = y + g * 16;
    float amax = 0.0f;
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    uint8_t sb = ref_e4m3(gs * (amax * 0.16666667163372039795f));
    float sff = ref_e4m3_value(sb);
    float scale = sff != 0.0f ? 1.0f / (sff * inv_gs) : 0.0f;
    for (int i = 0; i < 16; i += 2) {
      uint8_t lo = ref_e2m1(v[i] * scale), hi = ref_e2m1(v[i + 1] * scale);
      q[m * (K / 2) + g * 8 + i / 2] = (uint8_t)(lo | (hi << 4));
    }
    sf[sf_offset(m, g, K)] = sb;
  }
}

static int64_t next_pow2(int64_t k) {
  int64_t p = 1;
  while (p < k) p <<= 1;
  return p;
}

/* Returns 0 on success, -1 on bad sizes. Scratch: 2 * next_pow2(K) floats from the caller. */
int ref_norm_scale_fp4(const uint16_t *x, const uint16_t *w, const uint16_t *noisy, const uint16_t *clean,
                       const uint8_t *mask, const uint16_t *shift, const uint16_t *shift_clean, float gs, int64_t M,
                       int64_t S, int64_t K, int64_t mod_stride, float eps, uint8_t *q, uint8_t *sf, float *scratch) {
  if (K % 64 || S <= 0 || M % S) return -1;
  int64_t P = next_pow2(K);
  int64_t padded = (M + 127) / 128 * 128;
  float *sq = scratch, *y = scratch + P;
  for (int64_t m = 0; m < padded; ++m) {
    if (m >= M) {
      for (int64_t g = 0; g < K / 16; ++g) sf[sf_offset(m, g, K)] = 0;
      continue;
    }
    const uint16_t *xr = x + m * K;
    for (int64_t j = 0; j < P; ++j) {
      float v = j < K ? ref_bf16_to_f(xr[j]) : 0.0f;
      sq[j] = v * v;
    }
    float rstd = 1.0f / sqrtf(pairwise(sq, P) / (float)K + eps);
    int64_t b = m / S;
    int use_noisy = mask == NULL || mask[m % S] != 0;
    const uint16_t *mod = (use_noisy ? noisy : clean) + b * mod_stride;
    const uint16_t *shb = use_noisy ? shift : shift_clean;
    const uint16_t *sh = shb ? shb + b * mod_stride : NULL;
    for (int64_t j = 0; j < K; ++j) {
      float v = ref_bf16_round(ref_bf16_to_f(xr[j]) * rstd);
      v = ref_bf16_round(v * ref_bf16_to_f(w[j]));
      v = ref_bf16_round(v * ref_bf16_round(1.0f + ref_bf16_to_f(mod[j])));
      if (sh) v = ref_bf16_round(v + ref_bf16_to_f(sh[j]));
      y[j] = v;
    }
    quantize_row(y, m, K, gs, q, sf);
  }
  return 0;
}

/* bf16 bits of bf16(g / (1 + exp(-g))) for bf16 bits g (the SiLU value the silu_mul kernel multiplies). */
uint16_t ref_silu_bf16(uint16_t g) {
  float x = ref_bf16_to_f(g);
  return ref_f_to_bf16(x / (1.0f + ref_exp(-x)));
}

/* Scratch: K floats. */
int ref_silu_mul_fp4(const uint16_t *gate, const uint16_t *value, float gs, int64_t M, int64_t K, uint8_t *q,
                     uint8_t *sf, float *scratch) {
  if (K % 64) return -1;
  int64_t padded = (M + 127) / 128 * 128;
  for (int64_t m = 0; m < padded; ++m) {
    if (m >= M) {
      for (int64_t g = 0; g < K / 16; ++g) sf[sf_offset(m, g, K)] = 0;
      continue;
    }
    for (int64_t j = 0; j < K; ++j) {
      float g = ref_bf16_to_f(gate[m * K + j]);
      float v = ref_bf16_to_f(value[m * K + j]);
      float s = ref_bf16_round(g / (1.0f + ref_exp(-g)));
      scratch[j] = ref_bf16_round(s * v);
    }
    quantize_row(scratch, m, K, gs, q, sf);
  }
  return 0;
}
