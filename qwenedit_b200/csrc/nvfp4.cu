// Fused NVFP4 activation quantisers for the Fibo DiT producers.
//
// Replaces the Triton kernels of multi_turn/fibo/fp4.py:
//   _norm_scale_fp4_kernel (:64-80)  RMSNorm -> *w -> *(1 + adaLN scale) [-> + shift] -> NVFP4
//   _silu_mul_fp4_kernel   (:83-91)  SiLU(gate) * value -> NVFP4
//   _quantize_store / _e2m1 (:37-61) 16-element groups: e4m3 block scale, e2m1 codes, 128x4-swizzled scales
//
// Arithmetic follows the reference dataflow op for op in fp32, with the roundings a GPU executes:
// bf16 round-to-nearest-even at every `.to(tl.bfloat16)`, e4m3 round-to-nearest-even with saturation,
// IEEE division and square root. The row sum of squares uses numpy's pairwise order over the
// power-of-two block the reference kernel reduces (zero-padded to next_pow2(K)): 128-element leaves,
// each with eight interleaved accumulators, combined by a balanced binary tree. SiLU's exponential is
// computed by Cody-Waite reduction (two-constant ln 2 split), a degree-7 Taylor polynomial in Horner
// form with fused multiply-adds, and exact exponent reconstruction; it is within one ulp of exp.
//
// Layout on the device: one warp per row for norm_scale (the row is staged once through shared memory
// in a leaf-major, XOR-swizzled layout so both the coalesced fill and the per-leaf reduction are
// bank-conflict free; the element-wise pass reads it back coalesced); one 16-byte vector (8 values)
// per lane for silu_mul, four vectors in flight per lane. A 16-value group is a lane pair: its amax is
// one shuffle, each lane packs its 8 codes into a 32-bit store, and each quad of groups (one row, four
// consecutive scales) is written as one 32-bit store.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>

#include "qe_cuda.cuh"

namespace qe {
namespace {

// ---- scalar primitives (identical in the CPU oracle) ------------------------------------------
__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }

// e4m3 round-to-nearest-even with saturation to +-448; returns the byte and its exact value.
__device__ __forceinline__ uint32_t e4m3_byte(float v) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(0.0f), "f"(v));
  return uint32_t(out) & 0xffu;
}

// exact value of an e4m3 byte (bias 7, subnormals at exponent field 0, 0x7f/0xff = NaN)
__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  const uint32_t e = (byte >> 3) & 15u, m = byte & 7u;
  if (e == 15u && m == 7u) return __int_as_float(0x7fc00000);
  const float mag = e == 0u ? float(m) * 0.001953125f : float(8u + m) * __int_as_float(int(e + 117u) << 23);
  return (byte & 0x80u) ? -mag : mag;
}

// round to the nearest e2m1 value {0, .5, 1, 1.5, 2, 3, 4, 6} (ties to even code, saturating);
// sign in bit 3 (fibo/fp4.py:37-43)
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float a = fabsf(v);
  uint32_t c = uint32_t(a > 0.25f) + uint32_t(a >= 0.75f) + uint32_t(a > 1.25f) + uint32_t(a >= 1.75f) +
               uint32_t(a > 2.5f) + uint32_t(a >= 3.5f) + uint32_t(a > 5.0f);
  return c | (uint32_t(v < 0.0f) << 3);
}

__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// exp(x) within one ulp: Cody-Waite reduction + degree-7 Taylor (Horner, fma) + exponent rebuild.
__device__ __forceinline__ float exp_cw(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541015625f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.428606765330187045e-06f, r);
  float p = 1.98412698e-4f;
  p = __fmaf_rn(p, r, 1.38888889e-3f);
  p = __fmaf_rn(p, r, 8.33333377e-3f);
  p = __fmaf_rn(p, r, 4.16666679e-2f);
  p = __fmaf_rn(p, r, 1.66666672e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = int(n);
  const int e1 = ni / 2, e2 = ni - e1;
  return __fmul_rn(__fmul_rn(p, pow2i(e1)), pow2i(e2));
}

// Byte offset of the e4m3 scale of (row m, group g) in the 128x4-swizzled layout (fibo/fp4.py:59-60).
__device__ __forceinline__ int64_t sf_offset(int64_t m, int64_t g, int64_t K) {
  return (m >> 7) * (K / 64 * 512) + (g >> 2) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (g & 3);
}

// Quantise the 8 values this lane holds (one half of a 16-value group; the partner is lane ^ 1):
// returns the 4 packed code bytes and writes the group's scale byte to *sf_byte.
__device__ __forceinline__ uint32_t quantize8(const float (&y)[8], float gs, float inv_gs, uint32_t *sf_byte) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const uint32_t sb = e4m3_byte(__fmul_rn(gs, __fmul_rn(amax, 0.16666667163372039795f)));
  const float sff = e4m3_value(sb);
  const float scale = sff != 0.0f ? __fdiv_rn(1.0f, __fmul_rn(sff, inv_gs)) : 0.0f;
  uint32_t packed = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) packed |= e2m1_code(__fmul_rn(y[e], scale)) << (4 * e);
  *sf_byte = sb;
  return packed;
}

// Lanes t, t+2, t+4, t+6 (t % 8 == 0) own four consecutive groups of one row: collect their scale
// bytes into lane t as one little-endian word.
__device__ __forceinline__ uint32_t gather_sf_quad(uint32_t sb) {
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, sb, 2);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, sb, 4);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, sb, 6);
  return sb | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

// ---- RMSNorm + adaLN -> NVFP4 ------------------------------------------------------------------
struct NormParams {
  const uint4 *x;
  const uint4 *w;
  const __nv_bfloat16 *noisy, *clean, *shift, *shift_clean;
  const uint8_t *mask;
  const float *gs;
  uint32_t *q;
  uint8_t *sf;
  int64_t M, S, K, mod_stride, padded;
  int32_t leaves;      // P / 128 leaves (P = next_pow2(K) >= 128), or 1 when P == 64
  int32_t leaf_len;    // 128, or 64 when P == 64
  int32_t mods_vec;    // mod / shift rows are 16-byte aligned
  int32_t row_chunks;  // 16-byte chunks of shared memory per warp (whole 256-byte leaves)
  float eps;
};

// smem chunk index of 16-byte chunk g of a row: leaf-major, XOR swizzle on the chunk within its leaf
__device__ __forceinline__ int swz(int g) {
  const int leaf = g >> 4, c = g & 15;
  return (leaf << 4) | (c ^ (leaf & 15));
}

__device__ __forceinline__ void load_mod8(const __nv_bfloat16 *row, int64_t col, bool vec, float (&out)[8]) {
  if (vec) {
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row + col));
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[2 * i] = bf16_lo(u[i]);
      out[2 * i + 1] = bf16_hi(u[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = __bfloat162float(row[col + i]);
  }
}

template <int kWarps>
__global__ void __launch_bounds__(kWarps * 32) norm_scale_fp4_kernel(NormParams p) {
  extern __shared__ uint4 smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int chunks = int(p.K >> 3);          // 16-byte chunks per row
  uint4 *row_s = smem + int64_t(wid) * p.row_chunks;
  const int64_t warp0 = int64_t(blockIdx.x) * kWarps + wid;
  const int64_t nwarps = int64_t(gridDim.x) * kWarps;
  const float gs = __ldg(p.gs);
  const float inv_gs = __fdiv_rn(1.0f, gs);
  const float kf = float(p.K);

  for (int64_t m = warp0; m < p.padded; m += nwarps) {
    if (m >= p.M) {  // padding rows of the last 128-row tile: zero scales, no codes
      for (int g = lane * 4; g < chunks / 2; g += 128)
        *reinterpret_cast<uint32_t *>(p.sf + sf_offset(m, g, p.K)) = 0u;
      continue;
    }
    // stage the row: coalesced 16-byte loads -> swizzled leaf-major shared memory
    const uint4 *xr = p.x + m * chunks;
    for (int g = lane; g < chunks; g += 32) {
      const int4 v = ld_stream(reinterpret_cast<const int4 *>(xr + g));
      row_s[swz(g)] = make_uint4(uint32_t(v.x), uint32_t(v.y), uint32_t(v.z), uint32_t(v.w));
    }
    __syncwarp();

    // sum of squares, numpy pairwise order: leaf j = elements [leaf_len*j, leaf_len*j + leaf_len); lane l
    // owns leaves l, l+32, l+64, l+96; each round's 32 leaves reduce by a butterfly (a balanced tree), and
    // the rounds (halves / quarters of the padded block) combine as a balanced tree
    const int rounds = p.leaves > 32 ? p.leaves / 32 : 1;  // 1, 2 or 4
    float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (r < rounds) {
        const int leaf = lane + 32 * r;
        float s = 0.0f;
        if (leaf < p.leaves && leaf * p.leaf_len < p.K) {
          float acc[8];
          const int nchunk = min(p.leaf_len / 8, int((p.K - int64_t(leaf) * p.leaf_len) / 8));
          for (int c = 0; c < nchunk; ++c) {
            const uint4 v = row_s[(leaf << 4) | (c ^ (leaf & 15))];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float a = bf16_lo(u[i]), b = bf16_hi(u[i]);
              const float a2 = __fmul_rn(a, a), b2 = __fmul_rn(b, b);
              acc[2 * i] = c == 0 ? a2 : __fadd_rn(acc[2 * i], a2);
              acc[2 * i + 1] = c == 0 ? b2 : __fadd_rn(acc[2 * i + 1], b2);
            }
          }
          s = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                        __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
        part[r] = s;
      }
    }
    const float total = rounds == 1   ? part[0]
                        : rounds == 2 ? __fadd_rn(part[0], part[1])
                                      : __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, kf), p.eps)));

    const int64_t b = m / p.S;
    const bool use_noisy = p.mask == nullptr || __ldg(p.mask + (m % p.S)) != 0;
    const __nv_bfloat16 *mod_row = (use_noisy ? p.noisy : p.clean) + b * p.mod_stride;
    const __nv_bfloat16 *sh_base = use_noisy ? p.shift : p.shift_clean;
    const __nv_bfloat16 *sh_row = sh_base ? sh_base + b * p.mod_stride : nullptr;
    uint32_t *q_row = p.q + m * (p.K / 8);

    for (int g0 = 0; g0 < chunks; g0 += 32) {
      const int g = g0 + lane;
      const bool live = g < chunks;  // chunks is a multiple of 8: quads of groups stay whole
      float y[8];
      if (live) {
        const uint4 xv = row_s[swz(g)];
        const uint4 wv = __ldg(p.w + g);
        float mv[8], sv[8];
        load_mod8(mod_row, int64_t(g) * 8, p.mods_vec, mv);
        if (sh_row) load_mod8(sh_row, int64_t(g) * 8, p.mods_vec, sv);
        const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
        const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xf = (i & 1) ? bf16_hi(xu[i >> 1]) : bf16_lo(xu[i >> 1]);
          const float wf = (i & 1) ? bf16_hi(wu[i >> 1]) : bf16_lo(wu[i >> 1]);
          float v = bf16_round(__fmul_rn(xf, rstd));
          v = bf16_round(__fmul_rn(v, wf));
          v = bf16_round(__fmul_rn(v, bf16_round(__fadd_rn(1.0f, mv[i]))));
          if (sh_row) v = bf16_round(__fadd_rn(v, sv[i]));
          y[i] = v;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = 0.0f;
      }
      uint32_t sb;
      const uint32_t packed = quantize8(y, gs, inv_gs, &sb);
      const uint32_t quad = gather_sf_quad(sb);
      if (live) {
        q_row[g] = packed;
        if ((lane & 7) == 0) *reinterpret_cast<uint32_t *>(p.sf + sf_offset(m, g >> 1, p.K)) = quad;
      }
    }
    __syncwarp();
  }
}

// ---- SiLU(gate) * value -> NVFP4 ---------------------------------------------------------------
struct SiluParams {
  const uint4 *gate;
  const uint4 *value;
  const float *gs;
  uint32_t *q;
  uint8_t *sf;
  int64_t M, K, padded;
};

constexpr int kSiluThreads = 256;
constexpr int kSiluVec = 4;  // 16-byte vectors per lane in flight

__global__ void __launch_bounds__(kSiluThreads) silu_mul_fp4_kernel(SiluParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t cpr = p.K >> 3;  // chunks per row
  const int64_t total = p.M * cpr;
  const int64_t warp = (int64_t(blockIdx.x) * kSiluThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kSiluThreads) >> 5;
  const float gs = __ldg(p.gs);
  const float inv_gs = __fdiv_rn(1.0f, gs);

  for (int64_t base = warp * 32 * kSiluVec; base < total; base += nwarps * 32 * kSiluVec) {
    uint4 gv[kSiluVec], vv[kSiluVec];
#pragma unroll
    for (int u = 0; u < kSiluVec; ++u) {
      const int64_t c = base + u * 32 + lane;
      if (c < total) {
        const int4 a = ld_stream(reinterpret_cast<const int4 *>(p.gate + c));
        const int4 b = ld_stream(reinterpret_cast<const int4 *>(p.value + c));
        gv[u] = make_uint4(a.x, a.y, a.z, a.w);
        vv[u] = make_uint4(b.x, b.y, b.z, b.w);
      }
    }
#pragma unroll
    for (int u = 0; u < kSiluVec; ++u) {
      const int64_t c = base + u * 32 + lane;
      const bool live = c < total;  // total is a multiple of 8 chunks: quads stay whole
      float y[8];
      if (live) {
        const uint32_t gu[4] = {gv[u].x, gv[u].y, gv[u].z, gv[u].w};
        const uint32_t vu[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float g = (i & 1) ? bf16_hi(gu[i >> 1]) : bf16_lo(gu[i >> 1]);
          const float v = (i & 1) ? bf16_hi(vu[i >> 1]) : bf16_lo(vu[i >> 1]);
          const float s = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, exp_cw(-g))));
          y[i] = bf16_round(__fmul_rn(s, v));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = 0.0f;
      }
      uint32_t sb;
      const uint32_t packed = quantize8(y, gs, inv_gs, &sb);
      const uint32_t quad = gather_sf_quad(sb);
      if (live) {
        p.q[c] = packed;
        if ((lane & 7) == 0) {
          const int64_t m = c / cpr, g = c - m * cpr;
          *reinterpret_cast<uint32_t *>(p.sf + sf_offset(m, g >> 1, p.K)) = quad;
        }
      }
    }
  }
  // zero scales of the padding rows M .. padded-1 (4 scale bytes per store)
  const int64_t pad_words = (p.padded - p.M) * (p.K / 64);
  for (int64_t i = warp * 32 + lane; i < pad_words; i += nwarps * 32) {
    const int64_t m = p.M + i / (p.K / 64), g = (i % (p.K / 64)) * 4;
    *reinterpret_cast<uint32_t *>(p.sf + sf_offset(m, g, p.K)) = 0u;
  }
}

int64_t pad128(int64_t m) { return (m + 127) / 128 * 128; }

int64_t next_pow2(int64_t k) {
  int64_t p = 1;
  while (p < k) p <<= 1;
  return p;
}

}  // namespace
}  // namespace qe

using qe::fail;

extern "C" {

int qe_norm_scale_fp4(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                      const void *shift, const void *shift_clean, const float *gs, int64_t M, int64_t S,
                      int64_t K, int64_t mod_stride, float eps, uint8_t *q, uint8_t *sf, void *stream) {
  if (!x || !w || !noisy || !gs || !q || !sf) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: null argument");
  if (mask && !clean) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: a token mask needs `clean` rows");
  if (mask && shift && !shift_clean)
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: a token mask with a shift needs `shift_clean` rows");
  if (M < 0 || S <= 0 || K <= 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: bad sizes M=%lld S=%lld K=%lld",
                                             (long long)M, (long long)S, (long long)K);
  if (K % 64 != 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K=%lld must be a multiple of 64", (long long)K);
  if (K > 16384) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K=%lld above the supported 16384", (long long)K);
  if (M % S != 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: M=%lld is not a multiple of S=%lld",
                               (long long)M, (long long)S);
  if (mod_stride < 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: negative mod_stride");
  if (!qe::aligned16(x) || !qe::aligned16(w))
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: x and w must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(sf) & 3))
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: q and sf must be 4-byte aligned");
  const int64_t padded = qe::pad128(M);
  if (padded == 0) return qe::ok();
  qe::NormParams p{};
  p.x = static_cast<const uint4 *>(x);
  p.w = static_cast<const uint4 *>(w);
  p.noisy = static_cast<const __nv_bfloat16 *>(noisy);
  p.clean = static_cast<const __nv_bfloat16 *>(clean);
  p.shift = static_cast<const __nv_bfloat16 *>(shift);
  p.shift_clean = static_cast<const __nv_bfloat16 *>(shift_clean);
  p.mask = mask;
  p.gs = gs;
  p.q = reinterpret_cast<uint32_t *>(q);
  p.sf = sf;
  p.M = M;
  p.S = S;
  p.K = K;
  p.mod_stride = mod_stride;
  p.padded = padded;
  p.eps = eps;
  const int64_t P = qe::next_pow2(K);
  p.leaf_len = P >= 128 ? 128 : int32_t(P);
  p.leaves = int32_t(P / p.leaf_len);
  bool vec = (mod_stride % 8) == 0;
  for (const void *ptr : {noisy, clean, shift, shift_clean})
    if (ptr && !qe::aligned16(ptr)) vec = false;
  p.mods_vec = vec ? 1 : 0;
  // shared memory: one staged row per warp in whole 256-byte leaves (the swizzle stays inside a leaf)
  p.row_chunks = int32_t((K + 127) / 128 * 16);
  const size_t per_warp = size_t(p.row_chunks) * 16;
  constexpr size_t kSmemMax = 227 * 1024;
  const int warps = per_warp * 8 <= kSmemMax ? 8 : 4;
  const size_t smem = per_warp * size_t(warps);
  if (smem > kSmemMax) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K too large for one row per warp");
  // the shared-memory opt-in is per device context: remember it per device
  static bool attr_set[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  auto kernel = warps == 8 ? qe::norm_scale_fp4_kernel<8> : qe::norm_scale_fp4_kernel<4>;
  if (!attr_set[dev][warps == 8]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemMax));
    if (e != cudaSuccess) return qe::cuda_status(e, "qe_norm_scale_fp4: smem attribute");
    attr_set[dev][warps == 8] = true;
  }
  const int64_t blocks_needed = (padded + warps - 1) / warps;
  const int per_sm = std::max<int>(1, int(kSmemMax / std::max<size_t>(smem, 1)));
  const int64_t blocks =
      std::max<int64_t>(1, std::min<int64_t>(blocks_needed, int64_t(qe::sm_count()) * std::min(per_sm, 64 / warps)));
  kernel<<<dim3(unsigned(blocks)), dim3(warps * 32), smem, static_cast<cudaStream_t>(stream)>>>(p);
  int s = qe::cuda_status(cudaGetLastError(), "qe_norm_scale_fp4 launch");
  return s ? s : qe::ok();
}

int qe_silu_mul_fp4(const void *gate, const void *value, const float *gs, int64_t M, int64_t K, uint8_t *q,
                    uint8_t *sf, void *stream) {
  if (!gate || !value || !gs || !q || !sf) return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: null argument");
  if (M < 0 || K <= 0) return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: bad sizes");
  if (K % 64 != 0) return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: K=%lld must be a multiple of 64", (long long)K);
  if (!qe::aligned16(gate) || !qe::aligned16(value))
    return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: gate and value must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(sf) & 3))
    return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: q and sf must be 4-byte aligned");
  const int64_t padded = qe::pad128(M);
  if (padded == 0) return qe::ok();
  qe::SiluParams p{};
  p.gate = static_cast<const uint4 *>(gate);
  p.value = static_cast<const uint4 *>(value);
  p.gs = gs;
  p.q = reinterpret_cast<uint32_t *>(q);
  p.sf = sf;
  p.M = M;
  p.K = K;
  p.padded = padded;
  const int64_t work = std::max<int64_t>(M * (K / 8), (padded - M) * (K / 64));
  const int64_t per_block = int64_t(qe::kSiluThreads) * qe::kSiluVec;
  int64_t blocks = (work + per_block - 1) / per_block;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(qe::sm_count()) * 8));
  qe::silu_mul_fp4_kernel<<<dim3(unsigned(blocks)), dim3(qe::kSiluThreads), 0, static_cast<cudaStream_t>(stream)>>>(p);
  int s = qe::cuda_status(cudaGetLastError(), "qe_silu_mul_fp4 launch");
  return s ? s : qe::ok();
}

}  // extern "C"
