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

// ---- packed arithmetic (Blackwell f32x2 / bf16x2) ----------------------------------------------
// A bf16x2 word holds elements 2i (low half) and 2i+1 (high half); an f32x2 pair keeps the same order.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 up2(f32x2 r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bf16x2 word -> exact f32x2
__device__ __forceinline__ f32x2 bf2_f2(uint32_t u) {
  return pk2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// f32x2 -> bf16x2 word, each half rounded to nearest even
__device__ __forceinline__ uint32_t f2_bf2(f32x2 v) {
  const float2 f = up2(v);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f.y), "f"(f.x));
  return r;
}
// bf16 x bf16 and bf16 + bf16 are exact (or far from a bf16 midpoint) in fp32, so these single-rounding
// bf16x2 ops equal "fp32 op, then round to bf16", the reference's sequence
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// two fp32 -> two e2m1 codes (round to nearest even on {0,.5,1,1.5,2,3,4,6}, saturating, sign in bit 3);
// the low nibble holds the low element. These are exactly the reference's thresholds
// {>0.25, >=0.75, >1.25, >=1.75, >2.5, >=3.5, >5}; the caller passes +0.0 for a -0.0 product.
__device__ __forceinline__ uint32_t e2m1x2(f32x2 v) {
  const float2 f = up2(v);
  uint16_t r;
  asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n cvt.u16.u8 %0, t;\n}\n"
      : "=h"(r)
      : "f"(f.y), "f"(f.x));
  return r;
}

// exp(x) within one ulp, for two lanes at once: Cody-Waite reduction with a two-constant ln 2 split,
// degree-7 Taylor polynomial in Horner form with fused multiply-adds, exact 2^n rebuild in two factors.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

__device__ __forceinline__ f32x2 exp_cw2(f32x2 x2) {
  const float2 x = up2(x2);
  // n = rint(x * log2 e) by adding and removing 1.5 * 2^23 (round-to-nearest-even for |n| < 2^22, the range
  // that matters); the integer n sits in the low mantissa bits of the biased sum
  // (multiply, then add: the product is rounded to fp32 first, exactly as rintf(x * log2e) sees it)
  const f32x2 biased = add2(mul2(x2, pk2(1.44269504088896341f, 1.44269504088896341f)),
                            pk2(12582912.0f, 12582912.0f));
  const float2 bs = up2(biased);
  const float2 nf = up2(add2(biased, pk2(-12582912.0f, -12582912.0f)));
  const f32x2 nn = pk2(-nf.x, -nf.y);
  f32x2 r = fma2(nn, pk2(0.693145751953125f, 0.693145751953125f), x2);
  r = fma2(nn, pk2(1.428606765330187045e-06f, 1.428606765330187045e-06f), r);
  f32x2 p = pk2(1.98412698e-4f, 1.98412698e-4f);
  p = fma2(p, r, pk2(1.38888889e-3f, 1.38888889e-3f));
  p = fma2(p, r, pk2(8.33333377e-3f, 8.33333377e-3f));
  p = fma2(p, r, pk2(4.16666679e-2f, 4.16666679e-2f));
  p = fma2(p, r, pk2(1.66666672e-1f, 1.66666672e-1f));
  p = fma2(p, r, pk2(0.5f, 0.5f));
  p = fma2(p, r, pk2(1.0f, 1.0f));
  p = fma2(p, r, pk2(1.0f, 1.0f));
  const int ix = __float_as_int(bs.x) - 0x4b400000, iy = __float_as_int(bs.y) - 0x4b400000;
  const int ax = ix >> 1, ay = iy >> 1;
  const float2 e = up2(mul2(mul2(p, pk2(pow2i(ax), pow2i(ay))), pk2(pow2i(ix - ax), pow2i(iy - ay))));
  float ox = e.x, oy = e.y;
  if (!(x.x <= 88.72283935546875f)) ox = x.x != x.x ? x.x : __int_as_float(0x7f800000);
  if (x.x < -103.97208404541015625f) ox = 0.0f;
  if (!(x.y <= 88.72283935546875f)) oy = x.y != x.y ? x.y : __int_as_float(0x7f800000);
  if (x.y < -103.97208404541015625f) oy = 0.0f;
  return pk2(ox, oy);
}

// Byte offset of the e4m3 scale of (row m, group g) in the 128x4-swizzled layout (fibo/fp4.py:59-60).
__device__ __forceinline__ int64_t sf_offset(int64_t m, int64_t g, int64_t K) {
  return (m >> 7) * (K / 64 * 512) + (g >> 2) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (g & 3);
}

constexpr uint32_t kAbs2 = 0x7fff7fffu;
constexpr uint32_t kOne2 = 0x3f803f80u;  // bf16x2 (1.0, 1.0)

// Quantise one 16-value group held as 8 bf16x2 words: returns the 16 codes as 8 bytes (two words, the even
// column of each pair in the low nibble) and the group's e4m3 scale byte (fibo/fp4.py:46-61).
__device__ __forceinline__ uint2 quantize16(const uint32_t (&y)[8], float gs, float inv_gs, uint32_t &sb) {
  const uint32_t m01 = bmax2(y[0] & kAbs2, y[1] & kAbs2), m23 = bmax2(y[2] & kAbs2, y[3] & kAbs2);
  const uint32_t m45 = bmax2(y[4] & kAbs2, y[5] & kAbs2), m67 = bmax2(y[6] & kAbs2, y[7] & kAbs2);
  const uint32_t m = bmax2(bmax2(m01, m23), bmax2(m45, m67));
  const float amax = fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
  sb = e4m3_byte(__fmul_rn(gs, __fmul_rn(amax, 0.16666667163372039795f)));
  const float sff = e4m3_value(sb);
  const float scale = sff != 0.0f ? __frcp_rn(__fmul_rn(sff, inv_gs)) : 0.0f;
  const f32x2 scale2 = pk2(scale, scale), zero2 = pk2(0.0f, 0.0f);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = e2m1x2(fma2(bf2_f2(y[i]), scale2, zero2));
  return make_uint2(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24), c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24));
}

__device__ __forceinline__ void unpack16(const uint4 &a, const uint4 &b, uint32_t (&w)[8]) {
  w[0] = a.x;
  w[1] = a.y;
  w[2] = a.z;
  w[3] = a.w;
  w[4] = b.x;
  w[5] = b.y;
  w[6] = b.z;
  w[7] = b.w;
}

__device__ __forceinline__ uint4 ld16(const uint4 *p) {
  const int4 v = ld_stream(reinterpret_cast<const int4 *>(p));
  return make_uint4(uint32_t(v.x), uint32_t(v.y), uint32_t(v.z), uint32_t(v.w));
}

// zero the scales of padding row m (rows M .. pad128(M)-1 of the last 128-row tile), 4 bytes per store
__device__ __forceinline__ void zero_sf_row(uint8_t *sf, int64_t m, int64_t K, int lane) {
  for (int g = lane * 4; g < int(K / 16); g += 128) *reinterpret_cast<uint32_t *>(sf + sf_offset(m, g, K)) = 0u;
}

// ---- RMSNorm + adaLN -> NVFP4 ------------------------------------------------------------------
struct NormParams {
  const uint4 *x;
  const uint4 *w;
  const __nv_bfloat16 *noisy, *clean, *shift, *shift_clean;
  const uint8_t *mask;
  const float *gs;
  uint8_t *q;
  uint8_t *sf;
  int64_t M, S, K, mod_stride, padded;
  int32_t leaves;      // P / 128 leaves (P = next_pow2(K) >= 128), or 1 when P == 64
  int32_t leaf_len;    // 128, or 64 when P == 64
  int32_t mods_vec;    // mod / shift rows are 16-byte aligned
  int32_t row_chunks;  // 16-byte chunks of shared memory per warp (whole 256-byte leaves)
  float eps;
};

// smem chunk index of 16-byte chunk c of a row: leaf-major, XOR swizzle on the chunk within its leaf
__device__ __forceinline__ int swz(int c) {
  const int leaf = c >> 4;
  return (leaf << 4) | ((c & 15) ^ (leaf & 15));
}

// 8 bf16 modulation values starting at `col` as 4 bf16x2 words
__device__ __forceinline__ void load_mod8(const __nv_bfloat16 *row, int64_t col, bool vec, uint32_t *out) {
  if (vec) {
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row + col));
    out[0] = v.x;
    out[1] = v.y;
    out[2] = v.z;
    out[3] = v.w;
  } else {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(row + col);
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = uint32_t(__ldg(h + 2 * i)) | (uint32_t(__ldg(h + 2 * i + 1)) << 16);
  }
}

constexpr int kMaxRegGroups = 8;  // rows up to K = 4096 stay in registers between the two passes

// One warp per row. Lane l owns the 16-value groups g = l + 32 i of the row (two 16-byte chunks each):
// pass 1 loads them (1 KiB of the row per warp instruction pair) and stages them in leaf-major shared memory
// for the ordered sum of squares; pass 2 quantises each group from registers (K <= 4096) or shared memory.
template <int kWarps, bool kRegs>
__global__ void __launch_bounds__(kWarps * 32) norm_scale_fp4_kernel(NormParams p) {
  extern __shared__ uint4 smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int gpr = int(p.K >> 4);           // 16-value groups per row
  const int gpl = (gpr + 31) >> 5;         // groups per lane
  uint4 *row_s = smem + int64_t(wid) * p.row_chunks;
  const int64_t warp0 = int64_t(blockIdx.x) * kWarps + wid;
  const int64_t nwarps = int64_t(gridDim.x) * kWarps;
  const float gs = __ldg(p.gs);
  const float inv_gs = __fdiv_rn(1.0f, gs);
  const float kf = float(p.K);

  for (int64_t m = warp0; m < p.padded; m += nwarps) {
    if (m >= p.M) {
      zero_sf_row(p.sf, m, p.K, lane);
      continue;
    }
    const uint4 *xr = p.x + m * (p.K >> 3);
    uint4 xa[kRegs ? kMaxRegGroups : 1], xb[kRegs ? kMaxRegGroups : 1];
#pragma unroll
    for (int i = 0; i < (kRegs ? kMaxRegGroups : 1); ++i) {
      if (kRegs && i < gpl) {
        const int g = lane + 32 * i;
        if (g < gpr) {
          xa[i] = ld16(xr + 2 * g);
          xb[i] = ld16(xr + 2 * g + 1);
          row_s[swz(2 * g)] = xa[i];
          row_s[swz(2 * g + 1)] = xb[i];
        }
      }
    }
    if (!kRegs) {
      for (int g = lane; g < gpr; g += 32) {
        row_s[swz(2 * g)] = ld16(xr + 2 * g);
        row_s[swz(2 * g + 1)] = ld16(xr + 2 * g + 1);
      }
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
          // eight running sums (element 8c + e goes to sum e) as four f32x2 pairs; each square is rounded
          // before it is added, as x * x followed by a sum does
          f32x2 acc[4];
          const int nchunk = min(p.leaf_len / 8, int((p.K - int64_t(leaf) * p.leaf_len) / 8));
          {
            const uint4 v = row_s[(leaf << 4) | (leaf & 15)];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const f32x2 f = bf2_f2(u[i]);
              acc[i] = mul2(f, f);
            }
          }
          for (int c = 1; c < nchunk; ++c) {
            const uint4 v = row_s[(leaf << 4) | (c ^ (leaf & 15))];
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const f32x2 f = bf2_f2(u[i]);
              acc[i] = add2(acc[i], mul2(f, f));
            }
          }
          // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))
          const float2 a0 = up2(acc[0]), a1 = up2(acc[1]), a2 = up2(acc[2]), a3 = up2(acc[3]);
          const float2 t = up2(add2(pk2(a0.x, a2.x), pk2(a0.y, a2.y)));
          const float2 u2 = up2(add2(pk2(a1.x, a3.x), pk2(a1.y, a3.y)));
          const float2 v2 = up2(add2(pk2(t.x, t.y), pk2(u2.x, u2.y)));
          s = __fadd_rn(v2.x, v2.y);
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
    const f32x2 rstd2 = pk2(rstd, rstd);

    const int64_t b = m / p.S;
    const bool use_noisy = p.mask == nullptr || __ldg(p.mask + (m % p.S)) != 0;
    const __nv_bfloat16 *mod_row = (use_noisy ? p.noisy : p.clean) + b * p.mod_stride;
    const __nv_bfloat16 *sh_base = use_noisy ? p.shift : p.shift_clean;
    const __nv_bfloat16 *sh_row = sh_base ? sh_base + b * p.mod_stride : nullptr;
    uint8_t *q_row = p.q + m * (p.K >> 1);

    auto group = [&](int g, const uint4 &x0, const uint4 &x1) {
      uint32_t xu[8], wu[8], mv[8], sv[8];
      unpack16(x0, x1, xu);
      unpack16(__ldg(p.w + 2 * g), __ldg(p.w + 2 * g + 1), wu);
      load_mod8(mod_row, int64_t(g) * 16, p.mods_vec, mv);
      load_mod8(mod_row, int64_t(g) * 16 + 8, p.mods_vec, mv + 4);
      if (sh_row) {
        load_mod8(sh_row, int64_t(g) * 16, p.mods_vec, sv);
        load_mod8(sh_row, int64_t(g) * 16 + 8, p.mods_vec, sv + 4);
      }
      uint32_t y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // bf16(bf16(bf16(x * rstd) * w) * bf16(1 + mod)) [+ shift, rounded]
        uint32_t v = f2_bf2(mul2(bf2_f2(xu[i]), rstd2));
        v = bmul2(v, wu[i]);
        v = bmul2(v, badd2(kOne2, mv[i]));
        if (sh_row) v = badd2(v, sv[i]);
        y[i] = v;
      }
      uint32_t sb;
      const uint2 codes = quantize16(y, gs, inv_gs, sb);
      *reinterpret_cast<uint2 *>(q_row + int64_t(g) * 8) = codes;
      p.sf[sf_offset(m, g, p.K)] = uint8_t(sb);
    };
    if (kRegs) {
#pragma unroll
      for (int i = 0; i < kMaxRegGroups; ++i) {
        const int g = lane + 32 * i;
        if (i < gpl && g < gpr) group(g, xa[i], xb[i]);
      }
    } else {
      for (int g = lane; g < gpr; g += 32) group(g, row_s[swz(2 * g)], row_s[swz(2 * g + 1)]);
    }
    __syncwarp();
  }
}

// ---- SiLU(gate) * value -> NVFP4 ---------------------------------------------------------------
struct SiluParams {
  const uint4 *gate;
  const uint4 *value;
  const float *gs;
  uint8_t *q;
  uint8_t *sf;
  int64_t M, K, padded;
};

constexpr int kSiluThreads = 256;
constexpr int kSiluItems = 2;  // warp items (32 groups each) in flight per iteration

// A warp item is 32 consecutive 16-value groups of one row, one group per lane; kSiluItems items per
// iteration so every lane has 8 16-byte loads in flight before it computes.
__global__ void __launch_bounds__(kSiluThreads, 2) silu_mul_fp4_kernel(SiluParams p) {
  const int lane = threadIdx.x & 31;
  const int gpr = int(p.K >> 4);
  const int segs = (gpr + 31) >> 5;
  const int64_t items = p.M * segs;
  const int64_t warp = (int64_t(blockIdx.x) * kSiluThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kSiluThreads) >> 5;
  const float gs = __ldg(p.gs);
  const float inv_gs = __fdiv_rn(1.0f, gs);

  for (int64_t it0 = warp; it0 < items; it0 += nwarps * kSiluItems) {
    uint4 ga[kSiluItems], gb[kSiluItems], va[kSiluItems], vb[kSiluItems];
    int64_t row[kSiluItems];
    int grp[kSiluItems];
#pragma unroll
    for (int u = 0; u < kSiluItems; ++u) {
      const int64_t it = it0 + int64_t(u) * nwarps;
      row[u] = it / segs;
      grp[u] = int(it - row[u] * segs) * 32 + lane;
      if (it < items && grp[u] < gpr) {
        const int64_t c = row[u] * (p.K >> 3) + 2 * grp[u];
        ga[u] = ld16(p.gate + c);
        gb[u] = ld16(p.gate + c + 1);
        va[u] = ld16(p.value + c);
        vb[u] = ld16(p.value + c + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < kSiluItems; ++u) {
      const int64_t it = it0 + int64_t(u) * nwarps;
      if (!(it < items && grp[u] < gpr)) continue;
      uint32_t gw[8], vw[8], y[8];
      unpack16(ga[u], gb[u], gw);
      unpack16(va[u], vb[u], vw);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // bf16(bf16(g / (1 + exp(-g))) * v)
        const f32x2 g2 = bf2_f2(gw[i]);
        const float2 g = up2(g2);
        const float2 d = up2(add2(pk2(1.0f, 1.0f), exp_cw2(pk2(-g.x, -g.y))));
        y[i] = bmul2(f2_bf2(pk2(__fdiv_rn(g.x, d.x), __fdiv_rn(g.y, d.y))), vw[i]);
      }
      uint32_t sb;
      const uint2 codes = quantize16(y, gs, inv_gs, sb);
      *reinterpret_cast<uint2 *>(p.q + row[u] * (p.K >> 1) + int64_t(grp[u]) * 8) = codes;
      p.sf[sf_offset(row[u], grp[u], p.K)] = uint8_t(sb);
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
  p.q = q;
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
  static bool attr_set[64][4] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  const bool regs = K <= 16 * 32 * qe::kMaxRegGroups;
  auto kernel = warps == 8 ? (regs ? qe::norm_scale_fp4_kernel<8, true> : qe::norm_scale_fp4_kernel<8, false>)
                           : (regs ? qe::norm_scale_fp4_kernel<4, true> : qe::norm_scale_fp4_kernel<4, false>);
  const int variant = (warps == 8 ? 2 : 0) + (regs ? 1 : 0);
  if (!attr_set[dev][variant]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemMax));
    if (e != cudaSuccess) return qe::cuda_status(e, "qe_norm_scale_fp4: smem attribute");
    attr_set[dev][variant] = true;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, warps * 32, smem) != cudaSuccess || occ < 1) occ = 1;
  const int64_t blocks_needed = (padded + warps - 1) / warps;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(blocks_needed, int64_t(qe::sm_count()) * occ));
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
  p.q = q;
  p.sf = sf;
  p.M = M;
  p.K = K;
  p.padded = padded;
  const int64_t items = M * ((K / 16 + 31) / 32);  // warp items: 32 groups of one row
  const int64_t warps_per_block = qe::kSiluThreads / 32;
  int64_t blocks = (std::max<int64_t>(items, (padded - M) * (K / 64) / 32) + warps_per_block - 1) / warps_per_block;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qe::silu_mul_fp4_kernel, qe::kSiluThreads, 0) != cudaSuccess ||
      occ < 1)
    occ = 2;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(qe::sm_count()) * occ));
  qe::silu_mul_fp4_kernel<<<dim3(unsigned(blocks)), dim3(qe::kSiluThreads), 0, static_cast<cudaStream_t>(stream)>>>(p);
  int s = qe::cuda_status(cudaGetLastError(), "qe_silu_mul_fp4 launch");
  return s ? s : qe::ok();
}

}  // extern "C"
