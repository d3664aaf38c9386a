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
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
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

// exact value of an e4m3 byte (every e4m3 value, NaN included, is an f16 value): the byte is placed in both
// halves so the result does not depend on which half the conversion reads
__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  const uint16_t pair = uint16_t(byte | (byte << 8));
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(pair));
  return __half2float(__ushort_as_half(uint16_t(h2 & 0xffffu)));
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
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
// bf16x2 word -> exact f32x2, on the FMA pipe: x * 1 + (-0) with bf16 multiplicands is x exactly (the -0
// addend keeps the sign of a zero)
__device__ __forceinline__ f32x2 bf2_f2(uint32_t u) {
  float lo, hi;
  asm("{\n .reg .b16 l, h, one;\n mov.b32 {l, h}, %2;\n mov.b16 one, 0x3f80;\n"
      " fma.rn.f32.bf16 %0, l, one, %3;\n fma.rn.f32.bf16 %1, h, one, %3;\n}\n"
      : "=f"(lo), "=f"(hi)
      : "r"(u), "f"(-0.0f));
  return pk2(lo, hi);
}

// a0 += lo(u)^2, a1 += hi(u)^2 with one rounding each: the square of a bf16 value is exact in fp32, so this
// equals rounding x * x and then adding it
__device__ __forceinline__ void sq_acc2(uint32_t u, float &a0, float &a1) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n"
      " fma.rn.f32.bf16 %0, l, l, %0;\n fma.rn.f32.bf16 %1, h, h, %1;\n}\n"
      : "+f"(a0), "+f"(a1)
      : "r"(u));
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
// Four f32x2 pairs -> eight e2m1 codes in one word (pair i in byte i, its low element in the low nibble):
// round to nearest even on {0, .5, 1, 1.5, 2, 3, 4, 6}, saturating, sign in bit 3. These are exactly the
// reference's thresholds {>0.25, >=0.75, >1.25, >=1.75, >2.5, >=3.5, >5}; callers pass +0.0 for a -0.0
// product (the reference's sign bit is `v < 0`).
__device__ __forceinline__ uint32_t e2m1x8(f32x2 a, f32x2 b, f32x2 c, f32x2 d) {
  const float2 fa = up2(a), fb = up2(b), fc = up2(c), fd = up2(d);
  uint32_t r;
  asm("{\n .reg .b8 t0, t1, t2, t3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 t0, %2, %1;\n"
      " cvt.rn.satfinite.e2m1x2.f32 t1, %4, %3;\n"
      " cvt.rn.satfinite.e2m1x2.f32 t2, %6, %5;\n"
      " cvt.rn.satfinite.e2m1x2.f32 t3, %8, %7;\n"
      " mov.b32 %0, {t0, t1, t2, t3};\n}\n"
      : "=r"(r)
      : "f"(fa.x), "f"(fa.y), "f"(fb.x), "f"(fb.y), "f"(fc.x), "f"(fc.y), "f"(fd.x), "f"(fd.y));
  return r;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// exp(-g) for SiLU's denominator, two lanes at once, within one ulp of exp: Cody-Waite reduction of x = -g
// with a two-constant ln 2 split, degree-7 Taylor polynomial in Horner form with fused multiply-adds, then
// p * 2^n as an exact p * 2^(n-1) times 2 (which overflows to +inf as exp does). Evaluated without
// negating anything: with n from x and r' = -(x - n ln2) computed from g, Horner on r' with alternating-sign
// coefficients yields (-1)^k times each Horner partial of the polynomial in r, so the result is bit for bit
// p(r). g is first clamped to [-89, 80]: for x = -g above 88.7228 both give +inf, and below -17.4 exp(x) < 2^-25
// so 1 + exp(x) rounds to 1 either way; the SiLU value is bit-identical to the unclamped exp with its special
// cases (a NaN gate stays NaN through the division).
__device__ __forceinline__ f32x2 exp_neg_silu2(f32x2 g2) {
  float2 g = up2(g2);
  g.x = fminf(fmaxf(g.x, -89.0f), 80.0f);
  g.y = fminf(fmaxf(g.y, -89.0f), 80.0f);
  g2 = pk2(g.x, g.y);
  // biased = RN(RN(x log2 e) + 1.5 * 2^23) = 1.5 * 2^23 + rint(x log2 e), ties to even; x log2 e = -(g log2 e)
  const f32x2 c2 = pk2(12582912.0f, 12582912.0f);
  const f32x2 biased = sub2(c2, mul2(g2, pk2(1.44269504088896341f, 1.44269504088896341f)));
  const f32x2 n2 = sub2(biased, c2);  // n, exactly
  f32x2 rn = fma2(n2, pk2(0.693145751953125f, 0.693145751953125f), g2);  // -(x - n ln2_hi)
  rn = fma2(n2, pk2(1.428606765330187045e-06f, 1.428606765330187045e-06f), rn);
  f32x2 p = pk2(-1.98412698e-4f, -1.98412698e-4f);
  p = fma2(p, rn, pk2(1.38888889e-3f, 1.38888889e-3f));
  p = fma2(p, rn, pk2(-8.33333377e-3f, -8.33333377e-3f));
  p = fma2(p, rn, pk2(4.16666679e-2f, 4.16666679e-2f));
  p = fma2(p, rn, pk2(-1.66666672e-1f, -1.66666672e-1f));
  p = fma2(p, rn, pk2(0.5f, 0.5f));
  p = fma2(p, rn, pk2(-1.0f, -1.0f));
  p = fma2(p, rn, pk2(1.0f, 1.0f));
  // 2^(n-1) from the bits of biased (0x4b400000 + n): ((n - 1) + 127) << 23 == (bits << 23) + (126 << 23) mod 2^32
  const float2 bs = up2(biased);
  const f32x2 half_scale = pk2(__uint_as_float((__float_as_uint(bs.x) << 23) + (126u << 23)),
                               __uint_as_float((__float_as_uint(bs.y) << 23) + (126u << 23)));
  return mul2(mul2(p, half_scale), pk2(2.0f, 2.0f));
}

// RN(a / b) rounded on to bf16, for b >= 1: a reciprocal-estimate quotient is within a few ulps of the
// correctly rounded one, so it rounds to the same bf16 unless it sits within 8 ulps of a bf16 midpoint (or
// b is huge); those rare cases take the IEEE division.
__device__ __forceinline__ float div_for_bf16(float a, float b) {
  const float q = __fmul_rn(a, rcp_approx(b));
  const uint32_t low = __float_as_uint(q) & 0xffffu;
  if (low - 0x7ff8u <= 16u || !(b < 1.2676506e30f)) return __fdiv_rn(a, b);  // 2^100
  return q;
}

// Byte offset of the e4m3 scale of (row m, group g) in the 128x4-swizzled layout (fibo/fp4.py:59-60).
__device__ __forceinline__ int64_t sf_offset(int64_t m, int64_t g, int64_t K) {
  return (m >> 7) * (K / 64 * 512) + (g >> 2) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (g & 3);
}

constexpr uint32_t kAbs2 = 0x7fff7fffu;
constexpr uint32_t kOne2 = 0x3f803f80u;  // bf16x2 (1.0, 1.0)

// max(|a|, |b|) per half; the sign bit it leaves (the XOR of the inputs' signs) is masked off by the caller
__device__ __forceinline__ uint32_t bamax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// bf16x2 word whose halves are both max |y| over the 16 values of a group
__device__ __forceinline__ uint32_t absmax16(const uint32_t (&y)[8]) {
  const uint32_t a = bamax2(y[0], y[1]), b = bamax2(y[2], y[3]), c = bamax2(y[4], y[5]), d = bamax2(y[6], y[7]);
  const uint32_t m = bamax2(bamax2(a, b), bamax2(c, d));
  return bamax2(m, __byte_perm(m, 0, 0x1032)) & kAbs2;
}

// ---- how the reference's fp32 divisions and reciprocal square root are evaluated --------------------------
// The reference leaves them to the compiler: `1.0 / gs` and `1.0 / (sff * (1.0 / gs))` of the quantiser
// (fibo/fp4.py:53-55), `sum / K` and `tl.rsqrt` of the norm (fibo/fp4.py:70). `numerics` packs one choice per
// site: bits 0-1 the quantiser's reciprocals, bits 2-3 the norm's mean division (0 = IEEE round-to-nearest,
// 1 = div.full.f32, 2 = div.approx.f32, 3 = rcp.approx.f32 then multiply), bits 4-5 the reciprocal square root
// (0 = 1 / sqrt, both correctly rounded; 1 = rsqrt.approx.f32). 0 everywhere is IEEE arithmetic, the rounding
// the CPU restatement uses.
__device__ __forceinline__ float div_sel(float a, float b, int how) {
  float r;
  switch (how) {
    case 1: asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
    case 2: asm("div.approx.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b)); return r;
    case 3: asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(b)); return __fmul_rn(a, r);
    default: return __fdiv_rn(a, b);
  }
}
__device__ __forceinline__ float rstd_sel(float mean_eps, int how) {
  if (how == 1) {
    float r;
    asm("rsqrt.approx.f32 %0, %1;" : "=f"(r) : "f"(mean_eps));
    return r;
  }
  return __fdiv_rn(1.0f, __fsqrt_rn(mean_eps));
}

// The reciprocal scale the quantiser multiplies by, for every e4m3 scale byte sb:
// 1 / (e4m3(sb) * (1 / gs)), or 0 for a zero scale (fibo/fp4.py:53-55). 256 floats, built per CTA.
constexpr int kScaleTab = 256;
__device__ __forceinline__ void build_scale_table(float *tab, float gs, int numerics) {
  const int how = numerics & 3;
  const float inv_gs = div_sel(1.0f, gs, how);
  for (int b = threadIdx.x; b < kScaleTab; b += blockDim.x) {
    const float sff = e4m3_value(uint32_t(b));
    tab[b] = sff != 0.0f ? div_sel(1.0f, __fmul_rn(sff, inv_gs), how) : 0.0f;
  }
}

// Quantise one 16-value group held as 8 bf16x2 words: returns the 16 codes as 8 bytes (two words, the even
// column of each pair in the low nibble) and the group's e4m3 scale byte (fibo/fp4.py:46-61).
__device__ __forceinline__ uint2 quantize16(const uint32_t (&y)[8], float gs, const float *scale_tab,
                                            uint32_t &sb) {
  const float amax = __uint_as_float(absmax16(y) << 16);
  sb = e4m3_byte(__fmul_rn(gs, __fmul_rn(amax, 0.16666667163372039795f)));
  const float scale = scale_tab[sb];
  const f32x2 scale2 = pk2(scale, scale), zero2 = pk2(0.0f, 0.0f);
  f32x2 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = fma2(bf2_f2(y[i]), scale2, zero2);
  return make_uint2(e2m1x8(v[0], v[1], v[2], v[3]), e2m1x8(v[4], v[5], v[6], v[7]));
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

// 32 bytes (one 16-value bf16 group) in one 256-bit streaming load; p must be 32-byte aligned. A warp request
// then covers 32 whole sectors instead of touching 32 sectors twice, half of each per 16-byte load.
__device__ __forceinline__ void ld32(const uint4 *p, uint4 &a, uint4 &b) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "l"(p));
}

// zero the scales of padding row m (rows M .. pad128(M)-1 of the last 128-row tile), 4 bytes per store
__device__ __forceinline__ void zero_sf_row(uint8_t *sf, int64_t m, int64_t K, int lane) {
  for (int g = lane * 4; g < int(K / 16); g += 128) *reinterpret_cast<uint32_t *>(sf + sf_offset(m, g, K)) = 0u;
}

// ---- programmatic dependent launch ------------------------------------------------------------------
// The quantisers are launched so that the next kernel on the stream may start its CTAs while this one's last
// CTAs finish (cudaLaunchAttributeProgrammaticStreamSerialization). Before its first global read a kernel waits
// for the grids it depends on to complete and their writes to be visible (griddepcontrol.wait; a no-op when it
// was launched without the attribute), and it allows its own dependents to launch right away
// (griddepcontrol.launch_dependents): they take SMs only as this kernel's CTAs leave them.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
  int32_t row_chunks;  // 16-byte chunks of one row buffer (whole 256-byte leaves)
  int32_t batches;     // modulation rows staged per variant
  int32_t variants;    // 1, or 2 with a token mask (noisy, clean)
  float eps;
  float *amax;         // amax mode: max |y| over the whole tensor (the calibration pre-pass)
  int32_t numerics;    // evaluation of the reference's divisions / rsqrt (div_sel, rstd_sel)
};

// Shared-memory chunk of 16-byte chunk c of a row: leaf-major with an XOR swizzle inside the leaf, chosen so
// the three access patterns are free of bank conflicts: the coalesced fill (8 consecutive chunks), the
// ordered reduction (lane j walks leaf j) and the per-group reads (lane l takes chunks 2l and 2l+1).
__device__ __forceinline__ int swz(int c) {
  const int leaf = c >> 4;
  return (leaf << 4) | ((c & 15) ^ (leaf & 15) ^ ((c >> 3) & 1));
}

// Per-column constant rows (w, bf16(1 + scale), shift) are stored group-interleaved: the two chunks of group
// g at g and half + g, so the per-group reads of a quarter warp hit 8 different bank groups.
__device__ __forceinline__ int gix(int c, int half) { return (c & 1) ? half + (c >> 1) : (c >> 1); }

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

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(
                   smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Bytes of the per-CTA constant tables: w, then (batches x variants) rows of bf16(1 + scale), then as many
// shift rows when there is a shift.
inline size_t norm_table_bytes(int64_t K, int64_t rows, bool shift) {
  return size_t(K) * 2 * size_t(1 + rows * (shift ? 2 : 1));
}

constexpr int pow2_at_least(int k) { return k <= 1 ? 1 : 2 * pow2_at_least((k + 1) / 2); }

// ---- tensor memory (TMEM) as per-lane constant storage -----------------------------------------
// With the row width fixed at compile time, lane l of every warp reads the same per-column constants (those of
// its groups g = l + 32 i) for every row. They are written once per CTA into TMEM lane l of each 32-lane
// quarter and read back with tcgen05.ld, which keeps them off the shared-memory data path that the row
// buffers use. A warp w can only address TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31.
constexpr uint32_t kTmemCols = 256;  // allocation per CTA (at most two such CTAs share an SM's 512 columns)
// scale table, then a 128-byte slot holding the TMEM address (keeps the row buffers 128-byte aligned, which
// their bank-conflict-free swizzle relies on)
constexpr int kHeadUint4 = kScaleTab / 4 + 8;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// whole warp: allocate kTmemCols columns, write the TMEM address to *slot, give up further allocations
__device__ __forceinline__ void tmem_alloc(uint32_t *slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(kTmemCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTmemCols) : "memory");
}
__device__ __forceinline__ void tmem_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 8 consecutive columns at a and at b (this thread's lane), waited for inside the same statement so that no
// instruction can read the registers before they are written
__device__ __forceinline__ void tmem_ld8x2(uint32_t a, uint32_t b, uint32_t (&x)[8], uint32_t (&y)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%16];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%17];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
        "=r"(y[0]), "=r"(y[1]), "=r"(y[2]), "=r"(y[3]), "=r"(y[4]), "=r"(y[5]), "=r"(y[6]), "=r"(y[7])
      : "r"(a), "r"(b)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8x3(uint32_t a, uint32_t b, uint32_t c, uint32_t (&x)[8], uint32_t (&y)[8],
                                           uint32_t (&z)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%24];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%25];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%26];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]),
        "=r"(y[0]), "=r"(y[1]), "=r"(y[2]), "=r"(y[3]), "=r"(y[4]), "=r"(y[5]), "=r"(y[6]), "=r"(y[7]),
        "=r"(z[0]), "=r"(z[1]), "=r"(z[2]), "=r"(z[3]), "=r"(z[4]), "=r"(z[5]), "=r"(z[6]), "=r"(z[7])
      : "r"(a), "r"(b), "r"(c)
      : "memory");
}

// One warp per row, rows strided over the grid. Each warp owns two row buffers in shared memory: while it
// quantises row m from one, cp.async streams its next row into the other. The per-column constants (w, the
// pre-rounded bf16(1 + scale) rows of every batch and mask variant, the shift rows) come from global memory
// (kTab 0), from tables the CTA stages in shared memory (kTab 1), or from TMEM (kTab 2, compile-time K only).
// In the element-wise pass lane l owns the 16-value groups g = l + 32 i.
// kK != 0 specialises the row width at compile time (every per-row loop unrolled, swizzled addresses
// hoisted out of the row loop); kK == 0 reads K from the parameters.
// kAmax: the calibration pre-pass — the same y, reduced to max |y| instead of quantised and stored.
template <int kK, int kWarps, int kTab, bool kShift, bool kAmax>
__global__ void __launch_bounds__(kWarps * 32) norm_scale_fp4_kernel(NormParams p) {
  static_assert(kTab != 2 || (kK != 0 && (kK / 16) % 32 == 0 && kWarps >= 4),
                "TMEM tables need a compile-time K of whole 512-column blocks and four warps");
  constexpr bool kTables = kTab == 1;
  constexpr bool kTmem = kTab == 2;

  extern __shared__ uint4 smem[];
  constexpr int kP = kK ? pow2_at_least(kK) : 0;
  constexpr int kLeafLen = kP >= 128 ? 128 : kP;
  const int K = kK ? kK : int(p.K);
  const int leaf_len = kK ? kLeafLen : p.leaf_len;
  const int leaves = kK ? kP / kLeafLen : p.leaves;
  const int row_chunks = kK ? (kK + 127) / 128 * 16 : p.row_chunks;
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int gpr = K >> 4;  // 16-value groups per row
  const int kc = K >> 3;   // 16-byte chunks per row
  const int half = gpr;    // group-interleaved table: second chunks start here
  const int mod_rows = p.batches * p.variants;
  float *scale_tab = reinterpret_cast<float *>(smem);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kScaleTab / 4);
  uint4 *w_s = smem + kHeadUint4;
  uint4 *m1_s = w_s + (kTables ? kc : 0);
  uint4 *sh_s = m1_s + (kTables ? kc * mod_rows : 0);
  uint4 *bufs = sh_s + (kTables && kShift ? kc * mod_rows : 0) + wid * 2 * row_chunks;
  // warps are numbered CTA-minor, so consecutive rows go to different SMs and every SM gets the same number of
  // rows (to within one per warp slot) whatever M is
  const int64_t warp0 = int64_t(wid) * gridDim.x + blockIdx.x;
  const int64_t nwarps = int64_t(gridDim.x) * kWarps;
  pdl_enter();
  const float gs = kAmax ? 1.0f : __ldg(p.gs);
  const float kf = float(K);
  if (!kAmax) build_scale_table(scale_tab, gs, p.numerics);

  auto fetch = [&](int64_t row, uint4 *dst) {  // issue the async copy of one row (no-op past M)
    if (row < p.M) {
      const uint4 *src = p.x + row * kc;
      if (kK) {
#pragma unroll
        for (int j = 0; j < (kK / 8 + 31) / 32; ++j) {
          const int c = lane + 32 * j;
          if ((kK / 8) % 32 == 0 || c < kc) cp_async16(dst + swz(c), src + c);
        }
      } else {
        for (int c = lane; c < kc; c += 32) cp_async16(dst + swz(c), src + c);
      }
    }
    cp_async_commit();
  };
  fetch(warp0, bufs);
  uint32_t amax_w = 0u;  // kAmax: running bf16x2 max of |y|

  if (kTables) {
    for (int c = threadIdx.x; c < kc; c += kWarps * 32) w_s[gix(c, half)] = __ldg(p.w + c);
    for (int t = 0; t < mod_rows; ++t) {
      const int b = t / p.variants;
      const bool noisy = (t % p.variants) == 0;
      const __nv_bfloat16 *mrow = (noisy ? p.noisy : p.clean) + b * p.mod_stride;
      const __nv_bfloat16 *srow = kShift ? (noisy ? p.shift : p.shift_clean) + b * p.mod_stride : nullptr;
      for (int c = threadIdx.x; c < kc; c += kWarps * 32) {
        uint32_t mv[4];
        load_mod8(mrow, int64_t(c) * 8, p.mods_vec, mv);
        m1_s[t * kc + gix(c, half)] =
            make_uint4(badd2(kOne2, mv[0]), badd2(kOne2, mv[1]), badd2(kOne2, mv[2]), badd2(kOne2, mv[3]));
        if (kShift) {
          uint32_t sv[4];
          load_mod8(srow, int64_t(c) * 8, p.mods_vec, sv);
          sh_s[t * kc + gix(c, half)] = make_uint4(sv[0], sv[1], sv[2], sv[3]);
        }
      }
    }
  }
  // TMEM columns of lane l: w of its groups i = 0 .. gpl-1 at 8 i, then bf16(1 + scale) of table row t at
  // 8 gpl (1 + t) + 8 i, then shift row t at 8 gpl (1 + mod_rows + t) + 8 i
  constexpr int kGpl = kK ? (kK / 16 + 31) / 32 : 1;  // groups per lane
  uint32_t tlane = 0;
  if constexpr (kTmem) {
    __syncwarp();
    if (wid == 0) tmem_alloc(tmem_slot);
    tmem_fence_before_sync();
    __syncthreads();
    tmem_fence_after_sync();
    tlane = *tmem_slot + (uint32_t(32 * (wid & 3)) << 16);
    {  // the kWarps / 4 warps of each lane quarter share the writes of that quarter's copy. Table row r of
       // group i sits at column 8 kGpl r + 8 i: r = 0 is w, r = 1 + t the bf16(1 + scale) row t, r = 1 + mod_rows
       // + t the shift row t. A writer loads every row of its group before storing any, so the global loads are
       // in flight together instead of one by one behind the stores.
      constexpr int kWriters = kWarps / 4;
      constexpr int kMaxRows = int(kTmemCols) / (8 * kGpl);  // rows that fit the allocation (checked by the host)
      const int rows = 1 + mod_rows * (kShift ? 2 : 1);
#pragma unroll
      for (int i = 0; i < kGpl; ++i) {
        if (i % kWriters != (wid >> 2) % kWriters) continue;
        const int g = lane + 32 * i;
        uint32_t v[kMaxRows][8];
        unpack16(__ldg(p.w + 2 * g), __ldg(p.w + 2 * g + 1), v[0]);
#pragma unroll
        for (int r = 1; r < kMaxRows; ++r) {
          if (r >= rows) break;
          const bool is_shift = r > mod_rows;
          const int t = is_shift ? r - 1 - mod_rows : r - 1;
          const int bt = t / p.variants;
          const bool noisy = (t % p.variants) == 0;
          const __nv_bfloat16 *row =
              (is_shift ? (noisy ? p.shift : p.shift_clean) : (noisy ? p.noisy : p.clean)) + bt * p.mod_stride;
          load_mod8(row, int64_t(g) * 16, p.mods_vec, v[r]);
          load_mod8(row, int64_t(g) * 16 + 8, p.mods_vec, v[r] + 4);
        }
#pragma unroll
        for (int r = 0; r < kMaxRows; ++r) {
          if (r >= rows) break;
          if (r >= 1 && r <= mod_rows) {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[r][k] = badd2(kOne2, v[r][k]);
          }
          tmem_st8(tlane + 8 * kGpl * r + 8 * i, v[r]);
        }
      }
      tmem_wait_st();
    }
    tmem_fence_before_sync();
  }
  __syncthreads();  // scale table (and constant tables) visible to every warp
  if constexpr (kTmem) tmem_fence_after_sync();

  // row m = b * S + s; b, s and b % batches advance by fixed steps instead of dividing per row
  const int S = int(p.S);
  int b = int(warp0 / S), s = int(warp0 % S), bb = b % p.batches;
  const int db = int(nwarps / S), ds = int(nwarps % S), dbb = db % p.batches;
  auto advance = [&]() {
    s += ds;
    b += db;
    bb += dbb;
    if (s >= S) {
      s -= S;
      ++b;
      ++bb;
    }
    if (bb >= p.batches) bb -= p.batches;
  };
  // chunk index of x chunk 2g (g = lane + 32 i) inside a row buffer: swz(2 (lane + 32 i)) written out
  const int x_lane = ((lane >> 3) << 4) + ((2 * lane & 15) ^ (lane >> 3) ^ ((lane >> 2) & 1));

  // one row: quantise (or reduce, kAmax) row m held in shared memory at row_s
  auto row_body = [&](int64_t m, const uint4 *row_s) {
    if (m >= p.M) {  // padding rows of the last 128-row tile: zero scales, no codes
      if (!kAmax) zero_sf_row(p.sf, m, K, lane);
      return;
    }

    // sum of squares, numpy pairwise order: leaf j = elements [leaf_len*j, leaf_len*j + leaf_len); lane l
    // owns leaves l, l+32, l+64, l+96; each round's 32 leaves reduce by a butterfly (a balanced tree), and
    // the rounds (halves / quarters of the padded block) combine as a balanced tree
    const int rounds = leaves > 32 ? leaves / 32 : 1;  // 1, 2 or 4
    float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (r < rounds) {
        const int leaf = lane + 32 * r;
        float sum = 0.0f;
        if (leaf < leaves && leaf * leaf_len < K) {
          // eight running sums (element 8c + e goes to sum e); the first chunk seeds them (0 + x*x = x*x)
          float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
          const int nchunk = min(leaf_len / 8, (K - leaf * leaf_len) / 8);
          const uint4 *leaf_s = row_s + (leaf << 4);
          const int key = leaf & 15;  // swz inside a leaf: chunk c sits at c ^ key ^ (c >> 3 & 1)
          auto chunk = [&](int c) {
            const uint4 v = leaf_s[c ^ key ^ ((c >> 3) & 1)];
            sq_acc2(v.x, acc[0], acc[1]);
            sq_acc2(v.y, acc[2], acc[3]);
            sq_acc2(v.z, acc[4], acc[5]);
            sq_acc2(v.w, acc[6], acc[7]);
          };
          if (nchunk == 16) {
#pragma unroll
            for (int c = 0; c < 16; ++c) chunk(c);
          } else {
            for (int c = 0; c < nchunk; ++c) chunk(c);
          }
          // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))
          const f32x2 t = add2(pk2(acc[0], acc[2]), pk2(acc[1], acc[3]));
          const f32x2 u2 = add2(pk2(acc[4], acc[6]), pk2(acc[5], acc[7]));
          const float2 tt = up2(t), uu = up2(u2);
          const float2 v2 = up2(add2(pk2(tt.x, uu.x), pk2(tt.y, uu.y)));
          sum = __fadd_rn(v2.x, v2.y);
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
        part[r] = sum;
      }
    }
    const float total = rounds == 1   ? part[0]
                        : rounds == 2 ? __fadd_rn(part[0], part[1])
                                      : __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
    const float rstd = rstd_sel(__fadd_rn(div_sel(total, kf, (p.numerics >> 2) & 3), p.eps), (p.numerics >> 4) & 3);
    const f32x2 rstd2 = pk2(rstd, rstd);

    const bool use_noisy = p.mask == nullptr || __ldg(p.mask + s) != 0;
    const int t = bb * p.variants + (use_noisy ? 0 : 1);  // batches == 1: one shared row
    const uint4 *m1_row = m1_s + t * kc;
    const uint4 *sh_row_s = sh_s + t * kc;
    const __nv_bfloat16 *mod_row = (use_noisy ? p.noisy : p.clean) + int64_t(b) * p.mod_stride;
    const __nv_bfloat16 *sh_base = use_noisy ? p.shift : p.shift_clean;
    const __nv_bfloat16 *sh_row = kShift ? sh_base + int64_t(b) * p.mod_stride : nullptr;
    uint8_t *q_row = p.q + m * (K >> 1);
    // scale-byte offset = row part + group part (fibo/fp4.py:60)
    const int64_t sf_row = (m >> 7) * (K / 64 * 512) + (m & 31) * 16 + ((m & 127) >> 5) * 4;

    auto group = [&](int g, int xi, int i) {  // xi: chunk index of x chunk 2g in the row buffer; g = lane + 32 i
      uint32_t xu[8], wu[8], mv[8], sv[8];
      unpack16(row_s[xi], row_s[xi ^ 1], xu);
      if constexpr (kTmem) {
        const uint32_t aw = tlane + 8 * i, am = tlane + 8 * kGpl * (1 + t) + 8 * i;
        if (kShift) {
          tmem_ld8x3(aw, am, tlane + 8 * kGpl * (1 + mod_rows + t) + 8 * i, wu, mv, sv);
        } else {
          tmem_ld8x2(aw, am, wu, mv);
        }
      } else if (kTables) {
        unpack16(w_s[g], w_s[half + g], wu);
        unpack16(m1_row[g], m1_row[half + g], mv);
        if (kShift) unpack16(sh_row_s[g], sh_row_s[half + g], sv);
      } else {
        uint32_t md[8];
        unpack16(__ldg(p.w + 2 * g), __ldg(p.w + 2 * g + 1), wu);
        load_mod8(mod_row, int64_t(g) * 16, p.mods_vec, md);
        load_mod8(mod_row, int64_t(g) * 16 + 8, p.mods_vec, md + 4);
#pragma unroll
        for (int i = 0; i < 8; ++i) mv[i] = badd2(kOne2, md[i]);
        if (kShift) {
          load_mod8(sh_row, int64_t(g) * 16, p.mods_vec, sv);
          load_mod8(sh_row, int64_t(g) * 16 + 8, p.mods_vec, sv + 4);
        }
      }
      uint32_t y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // bf16(bf16(bf16(x * rstd) * w) * bf16(1 + mod)) [+ shift, rounded]
        uint32_t v = f2_bf2(mul2(bf2_f2(xu[i]), rstd2));
        v = bmul2(v, wu[i]);
        v = bmul2(v, mv[i]);
        if (kShift) v = badd2(v, sv[i]);
        y[i] = v;
      }
      if constexpr (kAmax) {
#pragma unroll
        for (int i = 0; i < 8; ++i) amax_w = bamax2(amax_w, y[i]);
      } else {
        uint32_t sb;
        const uint2 codes = quantize16(y, gs, scale_tab, sb);
        *reinterpret_cast<uint2 *>(q_row + g * 8) = codes;
        p.sf[sf_row + (g >> 2) * 512 + (g & 3)] = uint8_t(sb);
      }
    };
    if (kK) {
      if (kTmem) __syncwarp();  // tcgen05.ld is warp-collective
      // g = lane + 32 i: chunk 2g is at x_lane + 64 i with the swizzle key's bits 2-3 advanced by i
#pragma unroll
      for (int i = 0; i < (kK / 16 + 31) / 32; ++i) {
        const int g = lane + 32 * i;
        if ((kK / 16) % 32 == 0 || g < gpr) group(g, (x_lane + 64 * i) ^ (4 * (i & 3)), i);
      }
    } else {
      int g = lane;
      for (; g + 32 < gpr; g += 64) {  // two independent groups per iteration
        group(g, swz(2 * g), 0);
        group(g + 32, swz(2 * g + 64), 0);
      }
      if (g < gpr) group(g, swz(2 * g), 0);
    }
  };

  int cur = 0;
  for (int64_t m = warp0; m < p.padded; m += nwarps, cur ^= 1, advance()) {
    fetch(m + nwarps, bufs + (cur ^ 1) * row_chunks);
    cp_async_wait_1();  // this row's copies (all but the newest group) have landed
    __syncwarp();
    row_body(m, bufs + cur * row_chunks);
    __syncwarp();  // every lane is done with this buffer before it is refilled
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if constexpr (kAmax) {
    amax_w &= kAbs2;
    float v = fmaxf(__uint_as_float(amax_w << 16), __uint_as_float(amax_w & 0xffff0000u));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int *>(p.amax), __float_as_uint(v));  // v >= 0
  }
  if constexpr (kTmem) {  // every warp's TMEM reads are complete before the columns are released
    tmem_fence_before_sync();
    __syncthreads();
    if (wid == 0) {
      tmem_fence_after_sync();
      tmem_dealloc(*tmem_slot);
    }
  }
}

// 1: launch the quantisers with programmatic stream serialization (default); 0: plain stream order
std::atomic<int> g_nvfp4_pdl{1};

template <typename Params>
cudaError_t launch_pdl(void (*kernel)(Params), unsigned blocks, unsigned threads, size_t smem, cudaStream_t stream,
                       const Params &p) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_nvfp4_pdl.load(std::memory_order_relaxed) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int kK, int kWarps, int kTab, bool kShift, bool kAmax>
int launch_norm_typed(const NormParams &p, size_t smem, cudaStream_t stream) {
  auto kernel = norm_scale_fp4_kernel<kK, kWarps, kTab, kShift, kAmax>;
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!attr_set[dev].load(std::memory_order_relaxed)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return cuda_status(e, "qe_norm_scale_fp4: smem attribute");
    attr_set[dev].store(true, std::memory_order_relaxed);
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kWarps * 32, smem) != cudaSuccess || occ < 1)
    occ = 1;
  // TMEM tables: at most two CTAs per SM, so their allocations always fit the SM's 512 columns
  if (kTab == 2 && occ > int(512 / kTmemCols)) occ = int(512 / kTmemCols);
  const int64_t blocks_needed = (p.padded + kWarps - 1) / kWarps;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(blocks_needed, int64_t(sm_count()) * occ));
  return cuda_status(launch_pdl(kernel, unsigned(blocks), unsigned(kWarps * 32), smem, stream, p),
                     "qe_norm_scale_fp4 launch");
}

template <int kK, int kTab, bool kShift, bool kAmax>
int launch_norm_warps(int warps, const NormParams &p, size_t smem, cudaStream_t stream) {
  if constexpr (kTab == 2) {  // 16 or 8 warps: one CTA per SM
    if (warps == 16) return launch_norm_typed<kK, 16, kTab, kShift, kAmax>(p, smem, stream);
    return launch_norm_typed<kK, 8, kTab, kShift, kAmax>(p, smem, stream);
  } else {
    switch (warps) {
      case 16: return launch_norm_typed<kK, 16, kTab, kShift, kAmax>(p, smem, stream);
      case 8: return launch_norm_typed<kK, 8, kTab, kShift, kAmax>(p, smem, stream);
      case 6: return launch_norm_typed<kK, 6, kTab, kShift, kAmax>(p, smem, stream);
      case 4: return launch_norm_typed<kK, 4, kTab, kShift, kAmax>(p, smem, stream);
      default: return launch_norm_typed<kK, 2, kTab, kShift, kAmax>(p, smem, stream);
    }
  }
}

template <int kK, bool kAmax>
int launch_norm_k(int tab, bool shift, int warps, const NormParams &p, size_t smem, cudaStream_t st) {
  if constexpr (kK != 0) {
    if (tab == 2)
      return shift ? launch_norm_warps<kK, 2, true, kAmax>(warps, p, smem, st)
                   : launch_norm_warps<kK, 2, false, kAmax>(warps, p, smem, st);
  }
  return tab == 1 ? (shift ? launch_norm_warps<kK, 1, true, kAmax>(warps, p, smem, st)
                           : launch_norm_warps<kK, 1, false, kAmax>(warps, p, smem, st))
                  : (shift ? launch_norm_warps<kK, 0, true, kAmax>(warps, p, smem, st)
                           : launch_norm_warps<kK, 0, false, kAmax>(warps, p, smem, st));
}

// 0: per-column constants in TMEM where eligible (default); 1: never TMEM (shared-memory / global tables);
// 2: always global memory
std::atomic<int> g_norm_table_mode{0};
bool tmem_tables_enabled() { return g_norm_table_mode.load(std::memory_order_relaxed) == 0; }
// Below this many rows the per-CTA TMEM setup (allocation, table writes, fences) can cost more than the shared-
// memory traffic it saves. K = 3072, device time TMEM vs shared memory, back to back: with 3 constant rows per
// group (w, bf16(1 + scale), shift) equal at 4,096-6,144 rows, 18.1 vs 18.7 us at 8,192, 21.5 vs 22.2 us at
// 10,240; with 5 (a token mask doubles the modulation rows) 21.0 vs 20.4 us at 8,192. From 12,288 rows TMEM wins
// for every layout (52.1 vs 57.0 us at 32,768).
constexpr int64_t kTmemMinRows = 12288;

// SiLU table home: 0 = by size (default), 1 = shared memory, 2 = global memory through L1
std::atomic<int> g_silu_table_mode{0};
// by size: the L1 form below this many rows (no 128 KiB staging per CTA; device time 5.4 vs 8.1 us at one
// row, equal at 1,024, slower from 4,096 rows: 54.6 vs 50.4 us, K = 12288)
constexpr int64_t kSiluL1Rows = 1024;
// load schedule of the SiLU kernel: 0 = load then compute, 1 = pipelined with one item per iteration
// (1024 threads), 2 = pipelined with two items per iteration (512 threads)
std::atomic<int> g_silu_pipeline{1};
// how the reference's fp32 divisions and rsqrt are evaluated (div_sel / rstd_sel bit fields). The default,
// 1 | 1 << 2 | 1 << 4 (div.full.f32 for the quantiser's reciprocals and the norm's mean, rsqrt.approx.f32), is
// what reproduces the reference's Triton kernels as this image's Triton compiles them for sm_100: measured on a
// B200, codes and scales bit-identical on the reference test's shapes and on the benchmark's SiLU shapes (T up to
// 32768) and norm shapes up to T = 16384; 2 codes of 100.7 M differ at T = 32768 (the row sum's reduction order).
// 0 (IEEE everywhere) is the rounding of the CPU restatement.
constexpr int kNumericsTritonGpu = 1 | (1 << 2) | (1 << 4);
std::atomic<int> g_nvfp4_numerics{kNumericsTritonGpu};

// Row widths with a compile-time specialisation: 3072 (the Fibo / Qwen-Image DiT hidden size); any other
// multiple of 64 takes the runtime-K kernel.
constexpr int64_t kFixedK = 3072;
template <bool kAmax>
int launch_norm(int tab, bool shift, int warps, const NormParams &p, size_t smem, cudaStream_t st) {
  if (p.K == kFixedK) return launch_norm_k<kFixedK, kAmax>(tab, shift, warps, p, smem, st);
  return launch_norm_k<0, kAmax>(tab, shift, warps, p, smem, st);
}

// ---- SiLU(gate) * value -> NVFP4 ---------------------------------------------------------------
// bf16(silu(g)) depends on the 16 bits of g alone, so it is a 65,536-entry table, computed once per device
// by silu_table_kernel with the exact arithmetic below (Cody-Waite exp, IEEE-rounded quotient) and staged
// in shared memory by each CTA of silu_mul_fp4_kernel: per element the SiLU costs one shared-memory load.
constexpr int kSiluTable = 65536;

// bf16 bits of bf16(g / (1 + exp(-g))) for the two bf16 values of word w
__device__ __forceinline__ uint32_t silu_bf16x2(uint32_t w) {
  const f32x2 g2 = bf2_f2(w);
  const float2 g = up2(g2);
  const float2 d = up2(add2(pk2(1.0f, 1.0f), exp_neg_silu2(g2)));
  return f2_bf2(pk2(div_for_bf16(g.x, d.x), div_for_bf16(g.y, d.y)));
}

__global__ void __launch_bounds__(256) silu_table_kernel(uint32_t *table) {
  const uint32_t i = blockIdx.x * 256 + threadIdx.x;  // one word = entries 2i, 2i+1
  if (i < kSiluTable / 2) table[i] = silu_bf16x2((2 * i) | ((2 * i + 1) << 16));
}

struct SiluParams {
  const uint4 *gate;
  const uint4 *value;
  const float *gs;
  const uint4 *table;  // kSiluTable bf16 entries
  uint8_t *q;
  uint8_t *sf;
  float *amax;  // amax mode: max |y| over the whole tensor (the calibration pre-pass)
  int64_t M, K, padded;
  int32_t wide;  // gate and value are 32-byte aligned: one 256-bit load per lane and tensor
  int32_t numerics;  // evaluation of the quantiser's reciprocals (div_sel)
};

constexpr int kSiluThreads = 1024;  // one CTA per SM (the table takes 128 KiB of shared memory)

__device__ __forceinline__ uint32_t silu_lookup(const uint16_t *tab, uint32_t w) {
  return uint32_t(tab[w & 0xffffu]) | (uint32_t(tab[w >> 16]) << 16);
}
__device__ __forceinline__ uint32_t silu_lookup_l1(const uint16_t *tab, uint32_t w) {
  return uint32_t(__ldg(tab + (w & 0xffffu))) | (uint32_t(__ldg(tab + (w >> 16))) << 16);
}

// A warp item is 32 consecutive 16-value groups of one row, one group per lane (4 16-byte loads per lane).
// With kPipe the loads of the next iteration's items are issued before the current ones are computed, so the
// global-load latency is hidden behind the table lookups and the quantisation; without, the items are loaded,
// then computed. Items are tracked as (row, 32-group segment) and advanced without division.
// kL1: the SiLU table is read from global memory through the L1 cache instead of being staged in shared
// memory (no 128 KiB copy per CTA before the first row; lookups of the values a row actually uses stay in L1).
// kAmax: the calibration pre-pass — the same y, reduced to max |y| instead of quantised and stored.
// kSched: 0 = load then compute (2 items, 1024 threads); 1 = pipelined, 1 item per iteration, 1024 threads
// (the default: 32 warps per SM with 4 loads each in flight, 64 registers; 0.90 of HBM at T=16384 against
// 0.87 for 2 = pipelined with 2 items per iteration and 512 threads, and 0.81 for 0).
constexpr int silu_threads(int sched) { return sched == 2 ? kSiluThreads / 2 : kSiluThreads; }
constexpr int silu_items(int sched) { return sched == 1 ? 1 : 2; }

template <bool kAmax, bool kL1, int kSched>
__global__ void __launch_bounds__(silu_threads(kSched), 1) silu_mul_fp4_kernel(SiluParams p) {
  constexpr bool kPipe = kSched != 0;
  constexpr int kThreads = silu_threads(kSched);
  constexpr int kItems = silu_items(kSched);
  extern __shared__ uint4 tab4[];
  float *scale_tab = reinterpret_cast<float *>(tab4 + (kL1 ? 0 : kSiluTable / 8));
  pdl_enter();
  if (!kL1)
    for (int i = threadIdx.x; i < kSiluTable / 8; i += kThreads) tab4[i] = __ldg(p.table + i);
  const float gs = kAmax ? 1.0f : __ldg(p.gs);
  if (!kAmax) build_scale_table(scale_tab, gs, p.numerics);
  __syncthreads();
  const uint16_t *tab = kL1 ? reinterpret_cast<const uint16_t *>(p.table) : reinterpret_cast<const uint16_t *>(tab4);
  const int lane = threadIdx.x & 31;
  const int gpr = int(p.K >> 4);
  const int segs = (gpr + 31) >> 5;
  const int64_t warp = int64_t(threadIdx.x >> 5) * gridDim.x + blockIdx.x;  // CTA-minor: items spread over SMs
  const int64_t nwarps = int64_t(gridDim.x) * (kThreads >> 5);
  const int64_t drow = nwarps / segs;
  const int dseg = int(nwarps - drow * segs);
  uint32_t amax_w = 0u;  // kAmax: running bf16x2 max of |y|

  struct Item {
    int64_t row;
    int seg;
  };
  auto next = [&](Item it) {  // the item nwarps further on
    it.row += drow;
    it.seg += dseg;
    if (it.seg >= segs) {
      it.seg -= segs;
      ++it.row;
    }
    return it;
  };
  struct Data {
    uint4 ga, gb, va, vb;
  };
  auto valid = [&](const Item &it) { return it.row < p.M && it.seg * 32 + lane < gpr; };
  auto load = [&](const Item &it, Data &d) {
    if (valid(it)) {
      const int64_t c = it.row * (p.K >> 3) + 2 * (it.seg * 32 + lane);
      if (p.wide) {  // rows are whole 128-byte lines (K % 64 == 0), so every group is 32-byte aligned
        ld32(p.gate + c, d.ga, d.gb);
        ld32(p.value + c, d.va, d.vb);
      } else {
        d.ga = ld16(p.gate + c);
        d.gb = ld16(p.gate + c + 1);
        d.va = ld16(p.value + c);
        d.vb = ld16(p.value + c + 1);
      }
    }
  };
  auto compute = [&](const Item &it, const Data &d) {
    if (!valid(it)) return;
    const int grp = it.seg * 32 + lane;
    uint32_t gw[8], vw[8], y[8];
    unpack16(d.ga, d.gb, gw);
    unpack16(d.va, d.vb, vw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // bf16(silu(g) * v)
      y[i] = bmul2(kL1 ? silu_lookup_l1(tab, gw[i]) : silu_lookup(tab, gw[i]), vw[i]);
    }
    if constexpr (kAmax) {
#pragma unroll
      for (int i = 0; i < 8; ++i) amax_w = bamax2(amax_w, y[i]);
    } else {
      uint32_t sb;
      const uint2 codes = quantize16(y, gs, scale_tab, sb);
      *reinterpret_cast<uint2 *>(p.q + it.row * (p.K >> 1) + int64_t(grp) * 8) = codes;
      p.sf[sf_offset(it.row, grp, p.K)] = uint8_t(sb);
    }
  };

  Item cur[kItems];
  cur[0] = Item{warp / segs, int(warp % segs)};
#pragma unroll
  for (int u = 1; u < kItems; ++u) cur[u] = next(cur[u - 1]);
  Data dc[kItems];
  if constexpr (kPipe) {
#pragma unroll
    for (int u = 0; u < kItems; ++u) load(cur[u], dc[u]);
  }
  while (cur[0].row < p.M) {
    Item nx[kItems];
    nx[0] = next(cur[kItems - 1]);
#pragma unroll
    for (int u = 1; u < kItems; ++u) nx[u] = next(nx[u - 1]);
    Data dn[kItems];
    if constexpr (kPipe) {
#pragma unroll
      for (int u = 0; u < kItems; ++u) load(nx[u], dn[u]);  // next iteration's loads go out first
    } else {
#pragma unroll
      for (int u = 0; u < kItems; ++u) load(cur[u], dc[u]);
    }
#pragma unroll
    for (int u = 0; u < kItems; ++u) compute(cur[u], dc[u]);
#pragma unroll
    for (int u = 0; u < kItems; ++u) {
      cur[u] = nx[u];
      if constexpr (kPipe) dc[u] = dn[u];
    }
  }
  if constexpr (kAmax) {
    amax_w &= kAbs2;
    float v = fmaxf(__uint_as_float(amax_w << 16), __uint_as_float(amax_w & 0xffff0000u));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int *>(p.amax), __float_as_uint(v));  // v >= 0
    return;
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

namespace qe {
namespace {
int norm_scale_impl(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                    const void *shift, const void *shift_clean, const float *gs, int64_t M, int64_t S, int64_t K,
                    int64_t mod_stride, float eps, uint8_t *q, uint8_t *sf, float *amax, void *stream) {
  // with M = 0 the row buffers may be null (empty tensors)
  if (!w || !noisy || (M > 0 && (!x || (!amax && (!gs || !q || !sf)))))
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: null argument");
  if (mask && !clean) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: a token mask needs `clean` rows");
  if (mask && shift && !shift_clean)
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: a token mask with a shift needs `shift_clean` rows");
  if (M < 0 || S <= 0 || K <= 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: bad sizes M=%lld S=%lld K=%lld",
                                             (long long)M, (long long)S, (long long)K);
  if (K % 64 != 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K=%lld must be a multiple of 64", (long long)K);
  if (K > 16384) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K=%lld above the supported 16384", (long long)K);
  if (!qe::aligned16(x)) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: x must be 16-byte aligned");
  if (M % S != 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: M=%lld is not a multiple of S=%lld",
                               (long long)M, (long long)S);
  if (M > (int64_t(1) << 30)) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: M=%lld above 2^30 rows", (long long)M);
  if (mod_stride < 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: negative mod_stride");
  if (!qe::aligned16(x) || !qe::aligned16(w))
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: x and w must be 16-byte aligned");
  if (!amax && ((reinterpret_cast<uintptr_t>(q) & 7) || (reinterpret_cast<uintptr_t>(sf) & 3)))
    return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: q must be 8-byte and sf 4-byte aligned");
  const int64_t padded = amax ? M : qe::pad128(M);  // the pre-pass writes no padding scales
  if (amax) {
    cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return qe::cuda_status(e, "qe_norm_scale_amax: clear");
  }
  if (padded == 0) return 0;
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
  p.numerics = qe::g_nvfp4_numerics.load(std::memory_order_relaxed);
  p.amax = amax;
  const int64_t P = qe::next_pow2(K);
  p.leaf_len = P >= 128 ? 128 : int32_t(P);
  p.leaves = int32_t(P / p.leaf_len);
  bool vec = (mod_stride % 8) == 0;
  for (const void *ptr : {noisy, clean, shift, shift_clean})
    if (ptr && !qe::aligned16(ptr)) vec = false;
  p.mods_vec = vec ? 1 : 0;
  // shared memory: two row buffers per warp (whole 256-byte leaves) plus, when they fit, the per-column
  // constant tables; pick the warps per CTA that keep the most warps resident per SM
  p.row_chunks = int32_t((K + 127) / 128 * 16);
  p.batches = int32_t(mod_stride == 0 ? 1 : (M / S));
  p.variants = mask ? 2 : 1;
  const bool has_shift = shift != nullptr;
  const size_t row_pair = 2 * size_t(p.row_chunks) * 16;
  constexpr size_t kSmemMax = 227 * 1024;
  constexpr size_t kHead = qe::kHeadUint4 * 16;
  const size_t tables = qe::norm_table_bytes(K, int64_t(p.batches) * p.variants, has_shift);
  // per-column constants: TMEM when K is the specialised width and they fit the allocation, else shared-memory
  // tables up to 64 KiB, else global memory
  const int64_t tmem_cols = 8 * ((K / 16 + 31) / 32) * (1 + int64_t(p.batches) * p.variants * (has_shift ? 2 : 1));
  int tab = tables <= 64 * 1024 ? 1 : 0;
  if (K == qe::kFixedK && tmem_cols <= int64_t(qe::kTmemCols) && qe::tmem_tables_enabled() && M >= qe::kTmemMinRows)
    tab = 2;
  if (qe::g_norm_table_mode.load(std::memory_order_relaxed) == 2) tab = 0;  // constants read from global memory
  int best_warps = 0, best_resident = 0;
  size_t best_smem = 0;
  for (int w : {16, 8, 6, 4, 2}) {
    if (tab == 2 && w < 8) continue;
    const size_t smem = kHead + size_t(w) * row_pair + (tab == 1 ? tables : 0);
    if (smem > kSmemMax) continue;
    const int per_sm = std::min<int>(int(kSmemMax / smem), 32 / w);
    if (per_sm * w > best_resident) {
      best_resident = per_sm * w;
      best_warps = w;
      best_smem = smem;
    }
  }
  if (best_warps == 0) return fail(QE_ERR_INVALID, "qe_norm_scale_fp4: K too large for two rows per warp");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return amax ? qe::launch_norm<true>(tab, has_shift, best_warps, p, best_smem, st)
              : qe::launch_norm<false>(tab, has_shift, best_warps, p, best_smem, st);
}
}  // namespace
}  // namespace qe

extern "C" {

int qe_norm_scale_fp4(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                      const void *shift, const void *shift_clean, const float *gs, int64_t M, int64_t S,
                      int64_t K, int64_t mod_stride, float eps, uint8_t *q, uint8_t *sf, void *stream) {
  int s = qe::norm_scale_impl(x, w, noisy, clean, mask, shift, shift_clean, gs, M, S, K, mod_stride, eps, q, sf,
                              nullptr, stream);
  return s ? s : qe::ok();
}

int qe_norm_scale_amax(const void *x, const void *w, const void *noisy, const void *clean, const uint8_t *mask,
                       const void *shift, const void *shift_clean, int64_t M, int64_t S, int64_t K,
                       int64_t mod_stride, float eps, float *amax, void *stream) {
  if (!amax) return fail(QE_ERR_INVALID, "qe_norm_scale_amax: null amax");
  int s = qe::norm_scale_impl(x, w, noisy, clean, mask, shift, shift_clean, nullptr, M, S, K, mod_stride, eps,
                              nullptr, nullptr, amax, stream);
  return s ? s : qe::ok();
}

int qe_set_silu_table_mode(int32_t mode) {
  if (mode < 0 || mode > 2) return fail(QE_ERR_INVALID, "qe_set_silu_table_mode: mode must be 0, 1 or 2");
  qe::g_silu_table_mode.store(mode, std::memory_order_relaxed);
  return qe::ok();
}

int qe_set_silu_pipeline(int32_t on) {
  if (on < 0 || on > 2) return fail(QE_ERR_INVALID, "qe_set_silu_pipeline: 0, 1 or 2");
  qe::g_silu_pipeline.store(on, std::memory_order_relaxed);
  return qe::ok();
}

int qe_set_nvfp4_numerics(int32_t numerics) {
  if (numerics < 0 || numerics > 0x1f)
    return fail(QE_ERR_INVALID, "qe_set_nvfp4_numerics: bits 0-1 and 2-3 in 0..3, bit 4 in 0..1");
  qe::g_nvfp4_numerics.store(numerics, std::memory_order_relaxed);
  return qe::ok();
}

int qe_set_nvfp4_pdl(int32_t on) {
  if (on != 0 && on != 1) return fail(QE_ERR_INVALID, "qe_set_nvfp4_pdl: 0 or 1");
  qe::g_nvfp4_pdl.store(on, std::memory_order_relaxed);
  return qe::ok();
}

int qe_set_norm_table_mode(int32_t mode) {
  if (mode < 0 || mode > 2) return fail(QE_ERR_INVALID, "qe_set_norm_table_mode: mode must be 0, 1 or 2");
  qe::g_norm_table_mode.store(mode, std::memory_order_relaxed);
  return qe::ok();
}

int qe_silu_table_init(uint16_t *table, void *stream) {
  if (!table) return fail(QE_ERR_INVALID, "qe_silu_table_init: null table");
  if (!qe::aligned16(table)) return fail(QE_ERR_INVALID, "qe_silu_table_init: table must be 16-byte aligned");
  qe::silu_table_kernel<<<dim3(qe::kSiluTable / 2 / 256), dim3(256), 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint32_t *>(table));
  int s = qe::cuda_status(cudaGetLastError(), "qe_silu_table_init launch");
  return s ? s : qe::ok();
}

}  // extern "C"

namespace qe {
namespace {
int silu_mul_impl(const void *gate, const void *value, const float *gs, int64_t M, int64_t K, uint8_t *q,
                  uint8_t *sf, const uint16_t *silu_table, float *amax, void *stream) {
  // with M = 0 the row buffers may be null (empty tensors)
  if (!silu_table || (M > 0 && (!gate || !value || (!amax && (!gs || !q || !sf)))))
    return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: null argument");
  if (M < 0 || K <= 0) return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: bad sizes");
  if (K % 64 != 0) return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: K=%lld must be a multiple of 64", (long long)K);
  if (!aligned16(gate) || !aligned16(value) || !aligned16(silu_table))
    return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: gate, value and the table must be 16-byte aligned");
  if (!amax && ((reinterpret_cast<uintptr_t>(q) & 7) || (reinterpret_cast<uintptr_t>(sf) & 3)))
    return fail(QE_ERR_INVALID, "qe_silu_mul_fp4: q must be 8-byte and sf 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (amax) {
    cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float), st);
    if (e != cudaSuccess) return cuda_status(e, "qe_silu_mul_amax: clear");
  }
  const int64_t padded = pad128(M);
  if (padded == 0) return 0;
  SiluParams p{};
  p.gate = static_cast<const uint4 *>(gate);
  p.value = static_cast<const uint4 *>(value);
  p.gs = gs;
  p.table = reinterpret_cast<const uint4 *>(silu_table);
  p.q = q;
  p.sf = sf;
  p.amax = amax;
  p.M = M;
  p.K = K;
  p.padded = padded;
  p.wide = ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(value)) & 31) == 0 ? 1 : 0;
  p.numerics = qe::g_nvfp4_numerics.load(std::memory_order_relaxed);
  const int mode = g_silu_table_mode.load(std::memory_order_relaxed);
  const bool l1 = mode == 2 || (mode == 0 && M < kSiluL1Rows);
  const int sched = g_silu_pipeline.load(std::memory_order_relaxed);
  const size_t smem = (l1 ? 0 : size_t(kSiluTable) * 2) + kScaleTab * sizeof(float);
  static std::atomic<bool> attr_set[12][64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  using Kernel = void (*)(SiluParams);
  static const Kernel kernels[12] = {
      silu_mul_fp4_kernel<false, false, 0>, silu_mul_fp4_kernel<false, true, 0>,
      silu_mul_fp4_kernel<true, false, 0>,  silu_mul_fp4_kernel<true, true, 0>,
      silu_mul_fp4_kernel<false, false, 1>, silu_mul_fp4_kernel<false, true, 1>,
      silu_mul_fp4_kernel<true, false, 1>,  silu_mul_fp4_kernel<true, true, 1>,
      silu_mul_fp4_kernel<false, false, 2>, silu_mul_fp4_kernel<false, true, 2>,
      silu_mul_fp4_kernel<true, false, 2>,  silu_mul_fp4_kernel<true, true, 2>};
  const int variant = sched * 4 + (amax ? 2 : 0) + (l1 ? 1 : 0);
  const Kernel kernel = kernels[variant];
  const int threads = silu_threads(sched);
  if (!attr_set[variant][dev].load(std::memory_order_relaxed)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return cuda_status(e, "qe_silu_mul_fp4: smem attribute");
    attr_set[variant][dev].store(true, std::memory_order_relaxed);
  }
  const int64_t items = M * ((K / 16 + 31) / 32);  // warp items: 32 groups of one row
  const int64_t warps_per_block = threads / 32;
  const int64_t pad_items = amax ? 0 : (padded - M) * (K / 64) / 32;
  int64_t blocks = (std::max<int64_t>(items, pad_items) + warps_per_block - 1) / warps_per_block;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count())));
  return cuda_status(launch_pdl(kernel, unsigned(blocks), unsigned(threads), smem, st, p), "qe_silu_mul_fp4 launch");
}
}  // namespace
}  // namespace qe

extern "C" {

int qe_silu_mul_fp4(const void *gate, const void *value, const float *gs, int64_t M, int64_t K, uint8_t *q,
                    uint8_t *sf, const uint16_t *silu_table, void *stream) {
  int s = qe::silu_mul_impl(gate, value, gs, M, K, q, sf, silu_table, nullptr, stream);
  return s ? s : qe::ok();
}

int qe_silu_mul_amax(const void *gate, const void *value, int64_t M, int64_t K, const uint16_t *silu_table,
                     float *amax, void *stream) {
  if (!amax) return fail(QE_ERR_INVALID, "qe_silu_mul_amax: null amax");
  int s = qe::silu_mul_impl(gate, value, nullptr, M, K, nullptr, nullptr, silu_table, amax, stream);
  return s ? s : qe::ok();
}

}  // extern "C"
