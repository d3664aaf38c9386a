// Per-step latent ops next to the prefix cache, each one launch instead of a chain of eager torch ops:
//
//   mask blend  multi_turn/pipeline/masking.py:82-89   (MaskState.blend, called once per denoising step from
//               pipeline/hooks.py:223): keep = (1 - s) x0 + s eps; out = m lat + (1 - m) keep
//   compose     multi_turn/pipeline/hooks.py:234-247   (_compose): a stored version's latents with one box of
//               latent cells replaced by a crop's latents
//   crop        multi_turn/state.py:52-62              (stored_latents with a crop box)
//
// The blend reproduces torch's eager arithmetic exactly: every tensor op computes in fp32 and rounds its result
// to the latent dtype (bf16 / fp16 round to nearest even; fp32 is one fp32 rounding), in the reference's order,
// with the `.to(dtype)` conversions of the mask and of sigma done first. No contraction into FMAs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "qe_cuda.cuh"
#include "qeb200.h"

namespace qe {
namespace {

enum { kF32 = 0, kBF16 = 1, kF16 = 2, kScalarPair = 3 };

template <int kT>
struct Elem;
template <>
struct Elem<kF32> {
  using T = float;
  static __device__ __forceinline__ float load(const T *p, int64_t i) { return p[i]; }
  static __device__ __forceinline__ void store(T *p, int64_t i, float v) { p[i] = v; }
  static __device__ __forceinline__ float rnd(float v) { return v; }
};
template <>
struct Elem<kBF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(const T *p, int64_t i) { return __bfloat162float(p[i]); }
  static __device__ __forceinline__ void store(T *p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float rnd(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <>
struct Elem<kF16> {
  using T = __half;
  static __device__ __forceinline__ float load(const T *p, int64_t i) { return __half2float(p[i]); }
  static __device__ __forceinline__ void store(T *p, int64_t i, float v) { p[i] = __float2half_rn(v); }
  static __device__ __forceinline__ float rnd(float v) { return __half2float(__float2half_rn(v)); }
};

// a value of dtype `t` at p[i], as fp32 (the mask and sigma may come in fp32 or in the latent dtype)
__device__ __forceinline__ float load_any(const void *p, int t, int64_t i) {
  switch (t) {
    case kBF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    case kF16: return __half2float(static_cast<const __half *>(p)[i]);
    default: return static_cast<const float *>(p)[i];
  }
}

struct BlendParams {
  const void *lat, *x0, *eps, *mask, *sigma;
  void *out;
  int64_t B, N, C;
  int64_t x0_bstride, eps_bstride, mask_bstride;  // elements between batch entries (0: broadcast)
  int32_t mask_channels;                          // 1 (broadcast over C) or C
  int32_t mask_dtype, sigma_dtype;
};

template <int kT>
__global__ void __launch_bounds__(256) mask_blend_kernel(BlendParams p) {
  using E = Elem<kT>;
  using T = typename E::T;
  // sigma.to(dtype); 1 - sigma (masking.py:87-88). kScalarPair: a Python-float sigma, for which torch keeps
  // both s and (1 - s) in fp32 (computed on the host) and rounds only the products
  float s, oms;
  if (p.sigma_dtype == kScalarPair) {
    s = static_cast<const float *>(p.sigma)[0];
    oms = static_cast<const float *>(p.sigma)[1];
  } else {
    s = E::rnd(load_any(p.sigma, p.sigma_dtype, 0));
    oms = E::rnd(__fsub_rn(1.0f, s));
  }
  const int64_t total = p.B * p.N * p.C;
  const T *lat = static_cast<const T *>(p.lat);
  const T *x0 = static_cast<const T *>(p.x0);
  const T *eps = static_cast<const T *>(p.eps);
  T *out = static_cast<T *>(p.out);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t c = i % p.C;
    const int64_t bn = i / p.C;
    const int64_t n = bn % p.N, b = bn / p.N;
    const int64_t nc = n * p.C + c;
    const float a = E::rnd(__fmul_rn(oms, E::load(x0, b * p.x0_bstride + nc)));
    const float e = E::rnd(__fmul_rn(s, E::load(eps, b * p.eps_bstride + nc)));
    const float keep = E::rnd(__fadd_rn(a, e));
    const int64_t mi = b * p.mask_bstride + n * p.mask_channels + (p.mask_channels == 1 ? 0 : c);
    const float m = E::rnd(load_any(p.mask, p.mask_dtype, mi));  // editable.to(dtype)
    const float ml = E::rnd(__fmul_rn(m, E::load(lat, i)));
    const float omm = E::rnd(__fsub_rn(1.0f, m));
    const float mk = E::rnd(__fmul_rn(omm, keep));
    E::store(out, i, __fadd_rn(ml, mk));
  }
}

// The same blend, 8 channels of one latent cell per thread: the cell's (b, n) index is found once per 8 values
// with 32-bit arithmetic (B * N * C / 8 < 2^31, C a multiple of 8), the three latent tensors move as 16-byte
// (32-byte for fp32) vectors and a per-cell mask (mask_channels == 1) is loaded once. Same op order and roundings
// per value as mask_blend_kernel.
template <int kT>
struct Vec8;
template <>
struct Vec8<kBF16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = u;
  }
};
template <>
struct Vec8<kF16> {
  static __device__ __forceinline__ void load(const __half *p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ void store(__half *p, const float (&v)[8]) {
    uint4 u;
    __half2 *h = reinterpret_cast<__half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = u;
  }
};
template <>
struct Vec8<kF32> {
  static __device__ __forceinline__ void load(const float *p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float *p, const float (&v)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

template <int kT>
__global__ void __launch_bounds__(256) mask_blend_vec_kernel(BlendParams p) {
  using E = Elem<kT>;
  using T = typename E::T;
  float s, oms;
  if (p.sigma_dtype == kScalarPair) {
    s = static_cast<const float *>(p.sigma)[0];
    oms = static_cast<const float *>(p.sigma)[1];
  } else {
    s = E::rnd(load_any(p.sigma, p.sigma_dtype, 0));
    oms = E::rnd(__fsub_rn(1.0f, s));
  }
  const uint32_t vpc = uint32_t(p.C >> 3), N = uint32_t(p.N);
  const uint32_t total = uint32_t(p.B) * N * vpc;
  const T *lat = static_cast<const T *>(p.lat);
  const T *x0 = static_cast<const T *>(p.x0);
  const T *eps = static_cast<const T *>(p.eps);
  T *out = static_cast<T *>(p.out);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t cell = i / vpc, ch = (i - cell * vpc) * 8;
    const uint32_t b = cell / N, n = cell - b * N;
    const int64_t nc = int64_t(n) * p.C + ch;
    float xl[8], xx[8], xe[8], m8[8];
    Vec8<kT>::load(lat + int64_t(i) * 8, xl);
    Vec8<kT>::load(x0 + int64_t(b) * p.x0_bstride + nc, xx);
    Vec8<kT>::load(eps + int64_t(b) * p.eps_bstride + nc, xe);
    const int64_t mrow = int64_t(b) * p.mask_bstride + int64_t(n) * p.mask_channels;
    if (p.mask_channels == 1) {
      const float m = E::rnd(load_any(p.mask, p.mask_dtype, mrow));  // editable.to(dtype)
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = m;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = E::rnd(load_any(p.mask, p.mask_dtype, mrow + ch + k));
    }
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float a = E::rnd(__fmul_rn(oms, xx[k]));
      const float e = E::rnd(__fmul_rn(s, xe[k]));
      const float keep = E::rnd(__fadd_rn(a, e));
      const float ml = E::rnd(__fmul_rn(m8[k], xl[k]));
      const float omm = E::rnd(__fsub_rn(1.0f, m8[k]));
      const float mk = E::rnd(__fmul_rn(omm, keep));
      o[k] = __fadd_rn(ml, mk);
    }
    Vec8<kT>::store(out + int64_t(i) * 8, o);
  }
}

// out[h, w, C] = base everywhere, crop[(y - y0), (x - x0), C] inside the box; 16-byte vectors when C allows
template <typename V>
__global__ void __launch_bounds__(256) compose_kernel(const V *base, const V *crop, V *out, int64_t h, int64_t w,
                                                     int64_t cv, int64_t x0, int64_t y0, int64_t x1, int64_t y1) {
  const int64_t total = h * w * cv;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t v = i % cv, cell = i / cv;
    const int64_t y = cell / w, x = cell % w;
    if (y >= y0 && y < y1 && x >= x0 && x < x1) {
      out[i] = crop[((y - y0) * (x1 - x0) + (x - x0)) * cv + v];
    } else {
      out[i] = base[i];
    }
  }
}

// out[(y - y0), (x - x0), C] = src[y, x, C] for the box (stored_latents with a crop)
template <typename V>
__global__ void __launch_bounds__(256) crop_kernel(const V *src, V *out, int64_t w, int64_t cv, int64_t x0, int64_t y0,
                                                   int64_t x1, int64_t y1) {
  const int64_t bw = x1 - x0;
  const int64_t total = (y1 - y0) * bw * cv;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t v = i % cv, cell = i / cv;
    const int64_t y = y0 + cell / bw, x = x0 + cell % bw;
    out[i] = src[(y * w + x) * cv + v];
  }
}

int grid_for(int64_t total) {
  const int64_t blocks = (total + 255) / 256;
  return int(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count()) * 8)));
}

}  // namespace
}  // namespace qe

using qe::fail;

extern "C" {

int qe_mask_blend(const void *latents, const void *x0, const void *eps, const void *mask, const void *sigma,
                  void *out, int64_t B, int64_t N, int64_t C, int64_t x0_bstride, int64_t eps_bstride,
                  int64_t mask_bstride, int32_t mask_channels, int32_t dtype, int32_t mask_dtype, int32_t sigma_dtype,
                  void *stream) {
  QE_CHECK_ARG(B >= 0 && N >= 0 && C > 0, "qe_mask_blend: bad sizes");
  QE_CHECK_ARG(dtype >= 0 && dtype <= 2 && mask_dtype >= 0 && mask_dtype <= 2 && sigma_dtype >= 0 && sigma_dtype <= 3,
               "qe_mask_blend: dtype codes are 0 (f32), 1 (bf16), 2 (f16); sigma also 3 (host pair)");
  QE_CHECK_ARG(mask_channels == 1 || mask_channels == C, "qe_mask_blend: mask_channels must be 1 or C");
  QE_CHECK_ARG(x0_bstride >= 0 && eps_bstride >= 0 && mask_bstride >= 0, "qe_mask_blend: negative batch stride");
  const int64_t total = B * N * C;
  if (total == 0) return qe::ok();
  QE_CHECK_ARG(latents && x0 && eps && mask && sigma && out, "qe_mask_blend: null argument");
  qe::BlendParams p{latents, x0, eps, mask, sigma, out, B, N, C, x0_bstride, eps_bstride, mask_bstride,
                    mask_channels, mask_dtype, sigma_dtype};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t esz = dtype == qe::kF32 ? 4 : 2;
  const bool vec = C % 8 == 0 && total / 8 < (int64_t(1) << 31) && N < (int64_t(1) << 31) &&
                   x0_bstride % 8 == 0 && eps_bstride % 8 == 0 && qe::aligned16(latents) && qe::aligned16(x0) &&
                   qe::aligned16(eps) && qe::aligned16(out) && (esz * 8) % 16 == 0;
  if (vec) {
    const int grid = qe::grid_for(total / 8);
    switch (dtype) {
      case qe::kBF16: qe::mask_blend_vec_kernel<qe::kBF16><<<grid, 256, 0, st>>>(p); break;
      case qe::kF16: qe::mask_blend_vec_kernel<qe::kF16><<<grid, 256, 0, st>>>(p); break;
      default: qe::mask_blend_vec_kernel<qe::kF32><<<grid, 256, 0, st>>>(p); break;
    }
    int s = qe::cuda_status(cudaGetLastError(), "qe_mask_blend launch");
    return s ? s : qe::ok();
  }
  const int grid = qe::grid_for(total);
  switch (dtype) {
    case qe::kBF16: qe::mask_blend_kernel<qe::kBF16><<<grid, 256, 0, st>>>(p); break;
    case qe::kF16: qe::mask_blend_kernel<qe::kF16><<<grid, 256, 0, st>>>(p); break;
    default: qe::mask_blend_kernel<qe::kF32><<<grid, 256, 0, st>>>(p); break;
  }
  int s = qe::cuda_status(cudaGetLastError(), "qe_mask_blend launch");
  return s ? s : qe::ok();
}

int qe_latent_compose(const void *base, const void *crop, void *out, int64_t h, int64_t w, int64_t row_bytes,
                      int64_t x0, int64_t y0, int64_t x1, int64_t y1, void *stream) {
  QE_CHECK_ARG(h > 0 && w > 0 && row_bytes > 0 && 0 <= x0 && x0 < x1 && x1 <= w && 0 <= y0 && y0 < y1 && y1 <= h,
               "qe_latent_compose: box outside the grid or bad sizes");
  QE_CHECK_ARG(base && crop && out, "qe_latent_compose: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (row_bytes % 16 == 0 && qe::aligned16(base) && qe::aligned16(crop) && qe::aligned16(out)) {
    const int64_t cv = row_bytes / 16;
    qe::compose_kernel<int4><<<qe::grid_for(h * w * cv), 256, 0, st>>>(
        static_cast<const int4 *>(base), static_cast<const int4 *>(crop), static_cast<int4 *>(out), h, w, cv, x0, y0,
        x1, y1);
  } else {
    QE_CHECK_ARG(row_bytes % 2 == 0, "qe_latent_compose: row_bytes must be even");
    const int64_t cv = row_bytes / 2;
    qe::compose_kernel<uint16_t><<<qe::grid_for(h * w * cv), 256, 0, st>>>(
        static_cast<const uint16_t *>(base), static_cast<const uint16_t *>(crop), static_cast<uint16_t *>(out), h, w,
        cv, x0, y0, x1, y1);
  }
  int s = qe::cuda_status(cudaGetLastError(), "qe_latent_compose launch");
  return s ? s : qe::ok();
}

int qe_latent_crop(const void *src, void *out, int64_t h, int64_t w, int64_t row_bytes, int64_t x0, int64_t y0,
                   int64_t x1, int64_t y1, void *stream) {
  QE_CHECK_ARG(h > 0 && w > 0 && row_bytes > 0 && 0 <= x0 && x0 < x1 && x1 <= w && 0 <= y0 && y0 < y1 && y1 <= h,
               "qe_latent_crop: box outside the grid or bad sizes");
  QE_CHECK_ARG(src && out, "qe_latent_crop: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t cells = (y1 - y0) * (x1 - x0);
  if (row_bytes % 16 == 0 && qe::aligned16(src) && qe::aligned16(out)) {
    const int64_t cv = row_bytes / 16;
    qe::crop_kernel<int4><<<qe::grid_for(cells * cv), 256, 0, st>>>(static_cast<const int4 *>(src),
                                                                      static_cast<int4 *>(out), w, cv, x0, y0, x1, y1);
  } else {
    QE_CHECK_ARG(row_bytes % 2 == 0, "qe_latent_crop: row_bytes must be even");
    const int64_t cv = row_bytes / 2;
    qe::crop_kernel<uint16_t><<<qe::grid_for(cells * cv), 256, 0, st>>>(
        static_cast<const uint16_t *>(src), static_cast<uint16_t *>(out), w, cv, x0, y0, x1, y1);
  }
  int s = qe::cuda_status(cudaGetLastError(), "qe_latent_crop launch");
  return s ? s : qe::ok();
}

}  // extern "C"
