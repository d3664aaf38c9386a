// Paged joint attention: attention of a block of queries over the cached prefix K/V, read straight from the
// prefix pool through the block table, together with the step's own K/V, in one kernel.
//
// Replaces, for the DiT prefix cache, the per-step materialisation the reference does before its attention:
// multi_turn/pipeline/hooks.py:101-105 gathers the matched prefix (PagedKVPool.gather, cache/paged.py:106-113,
// kv.index_select of 2 * L * H * D values per token) and hooks.py:81-83 hands the per-layer K/V views to the
// model's joint attention, which concatenates them with the step's own K/V. Here the attention reads the K/V tiles
// from the pool pages themselves (TMA tile loads addressed by the block table) and no gathered copy exists.
// The same kernel covers the text encoder's partial hit (cache/encoder.py:173-190): grouped-query heads and a
// bottom-right causal mask on the step's own (tail) keys.
//
// Per CTA: two 128-query tiles of one query head (M = 256), head_dim 128, bf16 in, fp32 accumulation, bf16 out;
// or one tile (q_tiles = 1, warps 4-7 idle) when one-tile CTAs fit on the SMs in one wave, so that a small grid
// (the encoder tail's 28 heads x 256 queries) runs twice the CTAs, each with half the work.
//   warp 8       TMA producer: the Q tiles once, then per 128-key tile the K tile and the V tile into a
//                two-stage ring each (pool pages: 4-D tensor maps [D, H, row-in-page, page] of the K or V plane of
//                the layer; the step's own keys: 3-D maps [D, H, token])
//   warp 9       tcgen05.mma issuer (one thread) and owner of the 512 tensor-memory columns:
//                S_t = Q_t K^T (SS form, both operands K-major in 128-byte swizzled shared memory) and
//                O_t += P_t V (TS form: P_t from tensor memory, V MN-major in shared memory)
//   warps 0-7    softmax, one warpgroup per Q tile, one thread per query row (tensor-memory lane = row):
//                S row from tensor memory, masking, online max with a lazy rescale of O (only when the max
//                grows by more than 2^8), exp2, row sum, P written back over S as bf16, and the epilogue
//                O / l -> bf16 (+ log-sum-exp)
// Tensor memory: S0 | O0 | S1 | O1, 128 fp32 columns each; P_t (bf16 pairs) overwrites the first 64 columns of S_t.
// The MMAs of one thread execute in issue order, so PV_t(j) reads P_t(j) before QK_t(j+1) rewrites S_t.
// Every mbarrier wait is bounded (kWaitNs); on expiry the CTA records QE_ERR_TIMEOUT in the error flag (bit 2),
// drains what it issued and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "qe_cuda.cuh"

namespace qe {
namespace {

constexpr int kHeadDim = 128;
constexpr int kTile = 128;                       // queries per Q tile, keys per K/V tile
constexpr int kQTiles = 2;                       // Q tiles per CTA at most (AttnParams::q_tiles: 1 or 2)
constexpr int kTileBytes = kTile * kHeadDim * 2;  // 32 KiB: one Q, K or V tile
constexpr int kHalfBytes = kTileBytes / 2;        // 16 KiB: 128 rows x 64 dims, one 128-byte swizzle span per row
constexpr int kThreads = 320;                     // 8 softmax warps, the producer, the MMA warp
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the running max grows by more than this (log2 units)
constexpr float kHalfSumBound = 16384.0f;  // 64 keys x 2^kRescaleLog2: a larger half-tile sum has a p above 2^8

// shared memory, from a 1024-byte aligned base
constexpr int kQOff = 0;
constexpr int kKOff = kQOff + kQTiles * kTileBytes;  // 2 stages
constexpr int kVOff = kKOff + 2 * kTileBytes;        // 2 stages
constexpr int kBarOff = kVOff + 2 * kTileBytes;
enum Bar { kQFull = 0, kKFull = 1, kKEmpty = 3, kVFull = 5, kVEmpty = 7, kSFull = 9, kPReady = 11, kOFinal = 13,
           kDrain = 14, kNumBars = 15 };
constexpr int kSlotOff = kBarOff + kNumBars * 8;  // tensor-memory base address
constexpr int kAbortOff = kSlotOff + 4;
constexpr int kSmemBytes = kAbortOff + 4 + 1024;  // + slack to align the base

struct AttnParams {
  const int32_t *block_table;
  int32_t page_size, n_prefix, prefix_tiles, pool_pages, last_page, tail_rows;
  // fused append of the own K/V tiles into the pool (qe_paged_attention_append): the own tokens' page ids, the
  // index of their last page and its valid rows; null when not appending
  const int32_t *append_table;
  int32_t append_last_page, append_tail_rows;
  int32_t n_q, n_local, heads_q, group, causal;
  int32_t q_tiles;  // Q tiles per CTA: 2, or 1 for grids that fit one wave of one-tile CTAs
  float scale_log2;
  __nv_bfloat16 *out;
  int64_t out_token_stride, out_head_stride;  // elements
  float *lse;
  int32_t *err;
};

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase of `parity` to complete. Gives up (false) after kWaitNs or once another role of the
// CTA has given up; the first to give up records the timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort, int32_t *err) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > kWaitNs) {
        *abort = 1;
        if (err) atomicOr(err, 2);
        return false;
      }
    }
  }
}

// ---- TMA ----------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1, int32_t c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
// shared -> global tensor store (bulk group); rows outside the map's extents are not written
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, uint32_t src, int32_t c0, int32_t c1, int32_t c2,
                                             int32_t c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// ---- tcgen05 ------------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle: start address, leading / stride byte offsets (16-byte
// units), descriptor version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3fffu) | (uint64_t((lbo >> 4) & 0x3fffu) << 16) |
         (uint64_t((sbo >> 4) & 0x3fffu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator (bit 4), bf16 A (bits 7-9 = 1) and B (bits 10-12 = 1),
// A K-major, B K-major (QK) or MN-major (PV, bit 16), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kTile >> 3) << 17) |
                              (uint32_t(kTile >> 4) << 24);
constexpr uint32_t kIdescPV = kIdescQK | (1u << 16);

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's lane, waited for inside the statement (no register is read early)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 columns issued without waiting; tmem_ld_wait then waits for every load this thread has in flight and, by
// taking the registers as read-write operands, keeps the compiler from reading them any earlier
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// packed pairs of fp32 (Blackwell f32x2 arithmetic: one instruction for two lanes' worth of work)
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
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {  // two bf16 products, round to nearest
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Own-key tiles query-tile CTA x reads: all of them, or under the causal mask those up to the last own key its
// last query sees.
__device__ __forceinline__ int own_key_tiles(const AttnParams &p, int x) {
  if (p.n_local <= 0) return 0;
  int last_key = p.n_local - 1;
  if (p.causal) last_key = min(last_key, min((x + 1) * p.q_tiles * kTile, p.n_q) - 1 + p.n_local - p.n_q);
  return last_key >= 0 ? last_key / kTile + 1 : 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    paged_attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kpool,
                           const __grid_constant__ CUtensorMap tm_vpool, const __grid_constant__ CUtensorMap tm_ktail,
                           const __grid_constant__ CUtensorMap tm_vtail, const __grid_constant__ CUtensorMap tm_klocal,
                           const __grid_constant__ CUtensorMap tm_vlocal, const __grid_constant__ CUtensorMap tm_kapp,
                           const __grid_constant__ CUtensorMap tm_vapp, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bars = sbase + kBarOff;
  auto bar = [&](int i) { return bars + 8u * uint32_t(i); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kSlotOff);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + kAbortOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int q_tiles = p.q_tiles;
  const int q0 = blockIdx.x * (q_tiles * kTile);
  const int hq = blockIdx.y;
  const int hkv = hq / p.group;
  // key tiles: the prefix's, then the visible ones of the step's own keys
  const int local_tiles = own_key_tiles(p, blockIdx.x);
  const int n_tiles = p.prefix_tiles + local_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(kQFull), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kKFull + s), 1);
      mbar_init(bar(kKEmpty + s), 1);
      mbar_init(bar(kVFull + s), 1);
      mbar_init(bar(kVEmpty + s), 1);
      mbar_init(bar(kSFull + s), 1);
      mbar_init(bar(kPReady + s), 4);  // one arrival per softmax warp of the tile
    }
    mbar_init(bar(kOFinal), 1);
    mbar_init(bar(kDrain), 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // ---- producer: Q once, then K_j and V_j through two-stage rings ----
      mbar_expect_tx(bar(kQFull), q_tiles * kTileBytes);
      for (int t = 0; t < q_tiles; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sbase + kQOff + t * kTileBytes + h * kHalfBytes, &tm_q, h * 64, hq, q0 + t * kTile, bar(kQFull));
      const int P = p.page_size;
      auto load_tile = [&](int it, uint32_t dst, bool is_v, uint32_t full) {
        if (it < p.prefix_tiles) {
          const CUtensorMap *full_map = is_v ? &tm_vpool : &tm_kpool;
          const CUtensorMap *tail_map = is_v ? &tm_vtail : &tm_ktail;
          const int k0 = it * kTile;
          if (P >= kTile) {  // the tile lies inside one page
            const int pi = k0 / P;
            int page = __ldg(p.block_table + pi);
            if (page < 0 || page >= p.pool_pages) {
              if (p.err) atomicOr(p.err, 1);
              page = p.pool_pages;  // out of the map: the copy reads zeros
            }
            const CUtensorMap *map = pi == p.last_page ? tail_map : full_map;
            for (int h = 0; h < 2; ++h) tma_load_4d(dst + h * kHalfBytes, map, h * 64, hkv, k0 % P, page, full);
          } else {  // kTile / P pages per tile
            for (int sub = 0; sub < kTile / P; ++sub) {
              const int key = k0 + sub * P;
              const int pi = key / P;
              int page = p.pool_pages;  // past the prefix: zeros
              const CUtensorMap *map = full_map;
              if (key < p.n_prefix) {
                page = __ldg(p.block_table + pi);
                if (page < 0 || page >= p.pool_pages) {
                  if (p.err) atomicOr(p.err, 1);
                  page = p.pool_pages;
                }
                if (pi == p.last_page) map = tail_map;
              }
              for (int h = 0; h < 2; ++h)
                tma_load_4d(dst + h * kHalfBytes + sub * P * 128, map, h * 64, hkv, 0, page, full);
            }
          }
        } else {
          const int l0 = (it - p.prefix_tiles) * kTile;
          for (int h = 0; h < 2; ++h)
            tma_load_3d(dst + h * kHalfBytes, is_v ? &tm_vlocal : &tm_klocal, h * 64, hkv, l0, full);
        }
      };
      // Fused append: each own K/V tile j is stored into the pool pages of the own tokens (the last page through
      // a map whose row extent ends at the last token, so nothing past it is written) by exactly one of the CTAs
      // that load it: r = j mod (query-tile CTAs x group) names a query head of the group (r / G) and a query-tile
      // CTA (r mod G); under the causal mask, when that CTA does not load tile j, the first CTA that does stores
      // it (the loaded own tiles grow with the query tile). A stage is reloaded only after its stores read it.
      auto stores_tile = [&](int it) -> bool {
        if (p.append_table == nullptr || it < p.prefix_tiles) return false;
        const int G = int(gridDim.x);
        const int j = it - p.prefix_tiles;
        const int r = j % (G * p.group);
        if (hq % p.group != r / G) return false;
        const int xc = r % G, x = int(blockIdx.x);
        if (xc == x) return true;
        return xc < x && j >= own_key_tiles(p, x - 1);
      };
      auto store_tile = [&](int it, uint32_t src, bool is_v) {
        const CUtensorMap *full_map = is_v ? &tm_vpool : &tm_kpool;
        const CUtensorMap *tail_map = is_v ? &tm_vapp : &tm_kapp;
        const int l0 = (it - p.prefix_tiles) * kTile;
        const int rows = P >= kTile ? kTile : P;
        for (int sub = 0; sub < kTile / rows; ++sub) {
          const int key = l0 + sub * rows;
          if (key >= p.n_local) break;
          const int pi = key / P;
          const int page = __ldg(p.append_table + pi);
          if (page < 0 || page >= p.pool_pages) {
            if (p.err) atomicOr(p.err, 1);
            continue;
          }
          const CUtensorMap *map = pi == p.append_last_page ? tail_map : full_map;
          for (int h = 0; h < 2; ++h)
            tma_store_4d(map, src + h * kHalfBytes + sub * rows * 128, h * 64, hkv, key % P, page);
        }
      };
      bool ok = true, stored = false;
      for (int it = 0; it < n_tiles && ok; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        ok = mbar_wait(bar(kKEmpty + s), ph ^ 1, abort, p.err);
        if (!ok) break;
        if (stored) {  // the stores of an earlier tile may still read this stage
          bulk_wait_read_all();
          stored = false;
        }
        mbar_expect_tx(bar(kKFull + s), kTileBytes);
        load_tile(it, sbase + kKOff + s * kTileBytes, false, bar(kKFull + s));
        ok = mbar_wait(bar(kVEmpty + s), ph ^ 1, abort, p.err);
        if (!ok) break;
        mbar_expect_tx(bar(kVFull + s), kTileBytes);
        load_tile(it, sbase + kVOff + s * kTileBytes, true, bar(kVFull + s));
        if (stores_tile(it)) {
          ok = mbar_wait(bar(kKFull + s), ph, abort, p.err) && mbar_wait(bar(kVFull + s), ph, abort, p.err);
          if (!ok) break;
          store_tile(it, sbase + kKOff + s * kTileBytes, false);
          store_tile(it, sbase + kVOff + s * kTileBytes, true);
          bulk_commit();
          stored = true;
        }
      }
      if (p.append_table) bulk_wait_all();  // the appended rows are in global memory before the CTA retires
      if (!ok) {  // give the copies already issued time to land before the CTA's shared memory is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---- MMA issuer ----
      const uint32_t q_addr = sbase + kQOff, k_addr = sbase + kKOff, v_addr = sbase + kVOff;
      auto qk = [&](int t, int ks) {  // S_t = Q_t K^T over the 128 head dims, 8 steps of 16
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = uint32_t((k >> 2) * kHalfBytes + (k & 3) * 32);
          mma_ss(tmem + t * 256, sw128_desc(q_addr + t * kTileBytes + off, 16, 1024),
                 sw128_desc(k_addr + ks * kTileBytes + off, 16, 1024), kIdescQK, k > 0);
        }
      };
      auto pv = [&](int t, int vs, bool acc) {  // O_t += P_t V over 128 keys, 8 steps of 16
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ts(tmem + t * 256 + 128, tmem + t * 256 + 8 * k,
                 sw128_desc(v_addr + vs * kTileBytes + k * 2048, kHalfBytes, 1024), kIdescPV, acc || k > 0);
      };
      bool ok = mbar_wait(bar(kQFull), 0, abort, p.err);
      if (ok && n_tiles > 0) {
        ok = mbar_wait(bar(kKFull), 0, abort, p.err);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < q_tiles; ++t) {
            qk(t, 0);
            mma_commit(bar(kSFull + t));
          }
          mma_commit(bar(kKEmpty));
        }
        for (int it = 0; it < n_tiles && ok; ++it) {
          const int s = it & 1;
          ok = mbar_wait(bar(kVFull + s), (it >> 1) & 1, abort, p.err);
          if (!ok) break;
          const int s1 = (it + 1) & 1;
          for (int t = 0; t < q_tiles && ok; ++t) {
            ok = mbar_wait(bar(kPReady + t), it & 1, abort, p.err);
            if (!ok) break;
            tc_fence_after();
            pv(t, s, it > 0);
            if (it + 1 < n_tiles) {
              if (t == 0) {
                ok = mbar_wait(bar(kKFull + s1), ((it + 1) >> 1) & 1, abort, p.err);
                if (!ok) break;
                tc_fence_after();
              }
              qk(t, s1);
              mma_commit(bar(kSFull + t));
            }
          }
          if (!ok) break;
          mma_commit(bar(kVEmpty + s));
          if (it + 1 < n_tiles) mma_commit(bar(kKEmpty + s1));
        }
      }
      mma_commit(bar(kOFinal));
      if (!ok) {  // wait (bounded) for the MMAs already issued before the tensor memory is released
        mma_commit(bar(kDrain));
        const uint64_t t0 = globaltimer();
        while (!mbar_try(bar(kDrain), 0) && globaltimer() - t0 < kWaitNs) {
        }
      }
    }
  } else if ((warp >> 2) < q_tiles) {
    // ---- softmax warpgroups: warp w handles tile w / 4, tensor-memory lanes 32 (w % 4) .. + 31 (the warps of
    // a tile the CTA does not have go straight to the final barrier) ----
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const int qi = q0 + t * kTile + row;
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    const uint32_t s_col = lane_base + t * 256, o_col = s_col + 128;
    const int causal_shift = p.n_local - p.n_q;  // query i sees own keys j <= i + causal_shift
    float m_use = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int it = 0; it < n_tiles; ++it) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kSFull + t), it & 1, abort, p.err));
      if (!ok) break;
      tc_fence_after();
      // visible keys of this tile: [0, limit)
      int limit;
      if (it < p.prefix_tiles) {
        limit = p.n_prefix - it * kTile;
      } else {
        const int l0 = (it - p.prefix_tiles) * kTile;
        limit = p.n_local - l0;
        if (p.causal) limit = min(limit, qi + causal_shift - l0 + 1);
      }
      // Tiles whose 128 keys are all visible to every row of the warp skip the per-key masks (warp-uniform).
      const bool masked = __any_sync(0xffffffffu, limit < kTile);
      // One pass over S once every row of the warp has a finite reference max m_use: p = 2^(s scale_log2 - m_use)
      // with no max. A half tile (64 keys) whose p all stay <= 2^8 sums to <= 2^14, so a row whose max grew by more
      // than 2^8 shows (at the latest once its growth makes a half sum pass 2^14; until then its p stay <= 2^14).
      // Half A (keys 0-63) is written as P once no row's half sum passed the bound (else the two-pass path runs
      // from the intact S); then half B. A row that passes in half B: its max over half B is read from S (those
      // columns are not written yet); if it grew by more than 2^8, m_use moves up by a whole number k of octaves,
      // the row's O, half-A P and row sum scale by 2^-k exactly, and half B is redone.
      bool two_pass = true;
      if (__all_sync(0xffffffffu, m_use != -INFINITY)) {
        const f32x2 scale2 = pk2(p.scale_log2, p.scale_log2);
        f32x2 nbase2 = pk2(-m_use, -m_use);
        f32x2 la[2] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)}, lb[2] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
        uint32_t buf[2][32], pw[32];
        // 32 keys of chunk c: p = 2^(s scale_log2 - m_use) (hidden keys 0), row sums, P words 16 (c % 2) ..
        auto chunk32 = [&](int c, const uint32_t(&b)[32], f32x2(&ls)[2]) {
          float pv[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x = up2(fma2(pk2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1])), scale2, nbase2));
            pv[2 * i] = ex2(x.x);
            pv[2 * i + 1] = ex2(x.y);
          }
          if (masked) {
#pragma unroll
            for (int i = 0; i < 32; ++i) pv[i] = 32 * c + i < limit ? pv[i] : 0.0f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            ls[i & 1] = add2(ls[i & 1], pk2(pv[2 * i], pv[2 * i + 1]));
            pw[16 * (c & 1) + i] = pack_bf16(pv[2 * i], pv[2 * i + 1]);
          }
        };
        auto store_half = [&](uint32_t col) {  // P words 0-31 to columns col .. col + 31
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pw[i];
          tmem_st16(col, w);
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pw[16 + i];
          tmem_st16(col + 16, w);
        };
        auto half_sum = [&](const f32x2(&ls)[2]) {
          const float2 a = up2(add2(ls[0], ls[1]));
          return a.x + a.y;
        };
        tmem_ld32_async(s_col, buf[0]);
        tmem_ld_wait(buf[0]);
        tmem_ld32_async(s_col + 32, buf[1]);
        chunk32(0, buf[0], la);
        tmem_ld_wait(buf[1]);
        tmem_ld32_async(s_col + 64, buf[0]);  // half B's first chunk arrives during chunk 1
        chunk32(1, buf[1], la);
        tmem_ld_wait(buf[0]);
        const float suma = half_sum(la);
        if (!__any_sync(0xffffffffu, suma > kHalfSumBound)) {
          two_pass = false;
          store_half(s_col);
          auto half_b = [&]() {  // buf[0] holds chunk 2
            tmem_ld32_async(s_col + 96, buf[1]);
            chunk32(2, buf[0], lb);
            tmem_ld_wait(buf[1]);
            chunk32(3, buf[1], lb);
          };
          half_b();
          float lsum = l + suma, sumb = half_sum(lb);
          if (__any_sync(0xffffffffu, sumb > kHalfSumBound)) {
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            tmem_ld32_async(s_col + 96, buf[1]);
            tmem_ld32_async(s_col + 64, buf[0]);
            tmem_ld_wait(buf[1]);
            tmem_ld_wait(buf[0]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  v[j] = 64 + 32 * h + i + j < limit ? __uint_as_float(buf[h][i + j]) : -INFINITY;
                m4[0] = max3(m4[0], v[0], v[1]);
                m4[1] = max3(m4[1], v[2], v[3]);
                m4[2] = max3(m4[2], v[4], v[5]);
                m4[3] = max3(m4[3], v[6], v[7]);
              }
            }
            const float mb = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * p.scale_log2;
            const bool grow = mb > m_use + kRescaleLog2;
            if (__any_sync(0xffffffffu, grow)) {
              const int k = grow ? int(ceilf(fminf(mb - m_use, 1000.0f))) : 0;
              const uint32_t fb = k <= 126 ? uint32_t(127 - k) << 23 : 0u;  // 2^-k (0 below the normal range)
              const float f = __uint_as_float(fb);
              const uint32_t f2 = (fb >> 16) | (fb & 0xffff0000u);  // the same as a bf16 pair
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float o[32];
                uint32_t w[32];
                tmem_ld32(o_col + 32 * c, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(o[i] * f);
                tmem_st32(o_col + 32 * c, w);
              }
              tmem_wait_st();  // half A's P is in tensor memory before it is read back
              {
                float pa[32];
                uint32_t w[32];
                tmem_ld32(s_col, pa);
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = bmul2(__float_as_uint(pa[i]), f2);
                tmem_st32(s_col, w);
              }
              lsum *= f;
              m_use += float(k);
              nbase2 = pk2(-m_use, -m_use);
              lb[0] = lb[1] = pk2(0.0f, 0.0f);
              half_b();  // buf[0] still holds chunk 2
              sumb = half_sum(lb);
            }
          }
          store_half(s_col + 32);
          l = lsum + sumb;
        }
      }
      if (two_pass) {
        // pass 1: the row's max of the raw scores over the visible keys (S stays in tensor memory, read 32
        // columns at a time; four independent three-input max chains), scaled once afterwards (scale > 0)
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        {
          uint32_t buf[2][32];
          tmem_ld32_async(s_col, buf[0]);
          tmem_ld_wait(buf[0]);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c + 1 < 4) tmem_ld32_async(s_col + 32 * (c + 1), buf[(c + 1) & 1]);  // next chunk in flight
            float chunk[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) chunk[i] = __uint_as_float(buf[c & 1][i]);
            if (masked) {
#pragma unroll
              for (int i = 0; i < 32; ++i) chunk[i] = 32 * c + i < limit ? chunk[i] : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              m4[0] = max3(m4[0], chunk[i], chunk[i + 1]);
              m4[1] = max3(m4[1], chunk[i + 2], chunk[i + 3]);
              m4[2] = max3(m4[2], chunk[i + 4], chunk[i + 5]);
              m4[3] = max3(m4[3], chunk[i + 6], chunk[i + 7]);
            }
            if (c + 1 < 4) tmem_ld_wait(buf[(c + 1) & 1]);
          }
        }
        const float mx = max3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * p.scale_log2;
        // A row moves its reference max only when its max grew by more than 2^8 (also when m_use is still -inf and
        // a key is visible); its O (earlier tiles' sums at the old max) is scaled down to match. The tensor-memory
        // accesses are warp-collective, so a warp rescales together: rows that keep their max scale by 1.
        const bool grow = mx > m_use + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          const float f = grow && m_use != -INFINITY ? ex2(m_use - mx) : 1.0f;
          if (it > 0) {  // before the first P V, O holds nothing yet
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float o[32];
              uint32_t w[32];
              tmem_ld32(o_col + 32 * c, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(o[i] * f);
              tmem_st32(o_col + 32 * c, w);
            }
          }
          l *= f;
          if (grow) m_use = mx;
        }
        // pass 2: p = 2^(s scale_log2 - base) (one FFMA and one ex2 per key) as bf16 pairs written over the S
        // columns already read: chunk c's 32 scores (columns 32c ..) become P columns 16c .. 16c + 15. The row sum
        // runs in eight independent partial sums.
        const float nbase = m_use == -INFINITY ? 0.0f : -m_use;
        const f32x2 scale2 = pk2(p.scale_log2, p.scale_log2), nbase2 = pk2(nbase, nbase);
        f32x2 l4[4] = {pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f), pk2(0.0f, 0.0f)};
        {
          uint32_t buf[2][32];
          tmem_ld32_async(s_col, buf[0]);
          tmem_ld_wait(buf[0]);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c + 1 < 4) tmem_ld32_async(s_col + 32 * (c + 1), buf[(c + 1) & 1]);  // next chunk in flight
            float chunk[32];
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 x = up2(fma2(pk2(__uint_as_float(buf[c & 1][2 * i]), __uint_as_float(buf[c & 1][2 * i + 1])),
                                        scale2, nbase2));
              chunk[2 * i] = ex2(x.x);
              chunk[2 * i + 1] = ex2(x.y);
            }
            if (masked) {
#pragma unroll
              for (int i = 0; i < 32; ++i) chunk[i] = 32 * c + i < limit ? chunk[i] : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              l4[i & 3] = add2(l4[i & 3], pk2(chunk[2 * i], chunk[2 * i + 1]));
              w[i] = pack_bf16(chunk[2 * i], chunk[2 * i + 1]);
            }
            tmem_st16(s_col + 16 * c, w);  // columns 16c .. 16c + 15: already read, not those in flight
            if (c + 1 < 4) tmem_ld_wait(buf[(c + 1) & 1]);
          }
        }
        {
          const float2 a = up2(add2(add2(l4[0], l4[1]), add2(l4[2], l4[3])));
          l += a.x + a.y;
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();  // every lane's P is written before the warp's one arrival
      if (lane == 0) mbar_arrive(bar(kPReady + t));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(kOFinal), 0, abort, p.err));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool store = qi < p.n_q;
      __nv_bfloat16 *dst = p.out + int64_t(qi) * p.out_token_stride + int64_t(hq) * p.out_head_stride;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(o_col + 32 * c, o);  // warp-collective: every lane loads, only valid rows store
        if (l == 0.0f) {  // a row that saw no key: zeros (its O columns were never written)
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.0f;
        }
        if (store) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 pk;
            pk.x = pack_bf16(o[8 * v + 0] * inv, o[8 * v + 1] * inv);
            pk.y = pack_bf16(o[8 * v + 2] * inv, o[8 * v + 3] * inv);
            pk.z = pack_bf16(o[8 * v + 4] * inv, o[8 * v + 5] * inv);
            pk.w = pack_bf16(o[8 * v + 6] * inv, o[8 * v + 7] * inv);
            *reinterpret_cast<uint4 *>(dst + 32 * c + 8 * v) = pk;
          }
        }
      }
      if (store && p.lse) {
        const float ln2 = 0.69314718055994530942f;
        p.lse[int64_t(hq) * p.n_q + qi] = l > 0.0f ? (m_use + __log2f(l)) * ln2 : -INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---- host ---------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// bf16 tensor map with a 128-byte swizzle; dims / strides innermost first (strides of dims 1.. in bytes)
int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
             const uint32_t *box, const char *what) {
  auto fn = encode_fn();
  if (!fn) return fail(QE_ERR_CUDA, "qe_paged_attention: cuTensorMapEncodeTiled unavailable");
  const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void *>(base),
                  reinterpret_cast<const cuuint64_t *>(dims), reinterpret_cast<const cuuint64_t *>(strides),
                  reinterpret_cast<const cuuint32_t *>(box), elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QE_ERR_INVALID, "qe_paged_attention: tensor map for %s rejected (%d)", what, int(r));
  return QE_OK;
}

bool al16(int64_t v) { return v % 16 == 0; }

}  // namespace
}  // namespace qe

using qe::fail;

namespace qe {
namespace {
// Q tiles per CTA (process-wide): 0 = by grid size (default), 1 or 2 forced
std::atomic<int> g_attention_q_tiles{0};

int paged_attention_impl(const void *q, int64_t q_token_stride, int64_t q_head_stride, int32_t n_q, int32_t heads_q,
                         const void *k_pool, const void *v_pool, int64_t pool_rows, int32_t heads_kv,
                         const int32_t *block_table, int32_t page_size, int32_t n_prefix, const void *k_local,
                         const void *v_local, int64_t local_token_stride, int64_t local_head_stride, int32_t n_local,
                         int32_t causal, float scale, void *out, int64_t out_token_stride, int64_t out_head_stride,
                         float *lse, const int32_t *append_table, int32_t *err_flag, void *stream) {
  QE_CHECK_ARG(n_q >= 0 && n_prefix >= 0 && n_local >= 0, "qe_paged_attention: negative size");
  QE_CHECK_ARG(heads_q >= 1 && heads_kv >= 1 && heads_q % heads_kv == 0 && heads_q <= 65535,
               "qe_paged_attention: heads_q must be a positive multiple of heads_kv (at most 65535)");
  QE_CHECK_ARG(append_table == nullptr || n_q > 0, "qe_paged_attention_append: no queries (the appending CTAs "
               "are query-tile CTAs)");
  if (n_q == 0) return ok();
  QE_CHECK_ARG(q && out, "qe_paged_attention: null q or out");
  QE_CHECK_ARG(n_prefix + n_local >= 1, "qe_paged_attention: no keys (n_prefix + n_local == 0)");
  QE_CHECK_ARG(aligned16(q) && aligned16(out) && al16(q_token_stride) && al16(q_head_stride) &&
                   al16(out_token_stride) && al16(out_head_stride) && q_head_stride >= 256 &&
                   out_head_stride >= 256 && q_token_stride > 0 && out_token_stride > 0,
               "qe_paged_attention: q / out must be 16-byte aligned with 16-byte multiple strides, rows of 128 bf16");
  QE_CHECK_ARG(std::isfinite(scale) && scale > 0.0f, "qe_paged_attention: scale must be positive and finite");
  int32_t prefix_tiles = 0, pool_pages = 0, last_page = -1, tail_rows = 0;
  const bool append = append_table != nullptr;
  QE_CHECK_ARG(!append || n_local > 0, "qe_paged_attention_append: nothing to append (n_local == 0)");
  if (n_prefix > 0 || append) {
    QE_CHECK_ARG(k_pool && v_pool && (block_table || n_prefix == 0),
                 "qe_paged_attention: null pool plane or block table");
    QE_CHECK_ARG(aligned16(k_pool) && aligned16(v_pool), "qe_paged_attention: pool planes must be 16-byte aligned");
    QE_CHECK_ARG(page_size >= 8 && ((kTile % page_size) == 0 || (page_size % kTile) == 0) && page_size <= 1 << 20,
                 "qe_paged_attention: page_size must be a divisor of 128 (>= 8) or a multiple of 128");
    QE_CHECK_ARG(pool_rows >= page_size && pool_rows % page_size == 0 && pool_rows / page_size < (int64_t(1) << 31),
                 "qe_paged_attention: pool_rows must be a positive multiple of page_size");
    prefix_tiles = (n_prefix + kTile - 1) / kTile;
    pool_pages = int32_t(pool_rows / page_size);
    if (n_prefix > 0) {
      last_page = (n_prefix - 1) / page_size;
      tail_rows = n_prefix - last_page * page_size;
    }
  }
  if (n_local > 0) {
    QE_CHECK_ARG(k_local && v_local && aligned16(k_local) && aligned16(v_local) && al16(local_token_stride) &&
                     al16(local_head_stride) && local_token_stride > 0 && local_head_stride >= 256,
                 "qe_paged_attention: local K / V must be 16-byte aligned with 16-byte multiple strides");
  }
  CUtensorMap maps[9];
  std::memset(maps, 0, sizeof(maps));
  const uint32_t box3[3] = {64, 1, uint32_t(kTile)};
  int s;
  {
    const uint64_t dims[3] = {uint64_t(kHeadDim), uint64_t(heads_q), uint64_t(n_q)};
    const uint64_t strides[2] = {uint64_t(q_head_stride), uint64_t(q_token_stride)};
    if ((s = make_map(&maps[0], q, 3, dims, strides, box3, "q"))) return s;
  }
  const int64_t row_bytes = int64_t(heads_kv) * kHeadDim * 2;
  if (n_prefix > 0 || append) {
    const uint32_t box_rows = uint32_t(std::min(page_size, kTile));
    const uint32_t box4[4] = {64, 1, box_rows, 1};
    const uint64_t strides[3] = {uint64_t(kHeadDim * 2), uint64_t(row_bytes), uint64_t(row_bytes * page_size)};
    const uint64_t full[4] = {uint64_t(kHeadDim), uint64_t(heads_kv), uint64_t(page_size), uint64_t(pool_pages)};
    const uint64_t tail[4] = {uint64_t(kHeadDim), uint64_t(heads_kv), uint64_t(tail_rows), uint64_t(pool_pages)};
    if ((s = make_map(&maps[1], k_pool, 4, full, strides, box4, "the K pool"))) return s;
    if ((s = make_map(&maps[2], v_pool, 4, full, strides, box4, "the V pool"))) return s;
    if (n_prefix > 0) {
      if ((s = make_map(&maps[3], k_pool, 4, tail, strides, box4, "the K pool tail"))) return s;
      if ((s = make_map(&maps[4], v_pool, 4, tail, strides, box4, "the V pool tail"))) return s;
    }
    if (append) {  // the own tokens' last page: rows past the last own token are outside the map, never written
      const int64_t app_last = (int64_t(n_local) - 1) / page_size;
      const uint64_t app_tail[4] = {uint64_t(kHeadDim), uint64_t(heads_kv),
                                    uint64_t(int64_t(n_local) - app_last * page_size), uint64_t(pool_pages)};
      if ((s = make_map(&maps[7], k_pool, 4, app_tail, strides, box4, "the K append tail"))) return s;
      if ((s = make_map(&maps[8], v_pool, 4, app_tail, strides, box4, "the V append tail"))) return s;
    }
  }
  if (n_local > 0) {
    const uint64_t dims[3] = {uint64_t(kHeadDim), uint64_t(heads_kv), uint64_t(n_local)};
    const uint64_t strides[2] = {uint64_t(local_head_stride), uint64_t(local_token_stride)};
    if ((s = make_map(&maps[5], k_local, 3, dims, strides, box3, "local K"))) return s;
    if ((s = make_map(&maps[6], v_local, 3, dims, strides, box3, "local V"))) return s;
  }
  AttnParams p{};
  p.block_table = block_table;
  p.page_size = page_size;
  p.n_prefix = n_prefix;
  p.prefix_tiles = prefix_tiles;
  p.pool_pages = pool_pages;
  p.last_page = last_page;
  p.tail_rows = tail_rows;
  p.append_table = append_table;
  p.append_last_page = append ? (n_local - 1) / page_size : -1;
  p.append_tail_rows = append ? n_local - p.append_last_page * page_size : 0;
  p.n_q = n_q;
  p.n_local = n_local;
  p.heads_q = heads_q;
  p.group = heads_q / heads_kv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.44269504088896341f;
  p.out = static_cast<__nv_bfloat16 *>(out);
  p.out_token_stride = out_token_stride / 2;
  p.out_head_stride = out_head_stride / 2;
  p.lse = lse;
  p.err = err_flag;

  static std::atomic<bool> attr_done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!attr_done[dev].load(std::memory_order_relaxed)) {
    cudaError_t e = cudaFuncSetAttribute(paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "qe_paged_attention: smem attribute");
    attr_done[dev].store(true, std::memory_order_relaxed);
  }
  // one-tile CTAs when all of them fit on the SMs at once (twice the CTAs of a grid that would leave most SMs
  // idle, each CTA with half the work); else two tiles per CTA, whose softmax phases hide each other's
  int q_tiles = g_attention_q_tiles.load(std::memory_order_relaxed);
  if (q_tiles == 0) q_tiles = int64_t((n_q + kTile - 1) / kTile) * heads_q <= int64_t(sm_count()) ? 1 : 2;
  p.q_tiles = q_tiles;
  const dim3 grid(unsigned((n_q + q_tiles * kTile - 1) / (q_tiles * kTile)), unsigned(heads_q));
  paged_attention_kernel<<<grid, dim3(kThreads), kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
      maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], maps[6], maps[7], maps[8], p);
  s = cuda_status(cudaGetLastError(), "qe_paged_attention launch");
  return s ? s : ok();
}
}  // namespace
}  // namespace qe

extern "C" int qe_paged_attention(const void *q, int64_t q_token_stride, int64_t q_head_stride, int32_t n_q,
                                  int32_t heads_q, const void *k_pool, const void *v_pool, int64_t pool_rows,
                                  int32_t heads_kv, const int32_t *block_table, int32_t page_size, int32_t n_prefix,
                                  const void *k_local, const void *v_local, int64_t local_token_stride,
                                  int64_t local_head_stride, int32_t n_local, int32_t causal, float scale, void *out,
                                  int64_t out_token_stride, int64_t out_head_stride, float *lse, int32_t *err_flag,
                                  void *stream) {
  return qe::paged_attention_impl(q, q_token_stride, q_head_stride, n_q, heads_q, k_pool, v_pool, pool_rows, heads_kv,
                                  block_table, page_size, n_prefix, k_local, v_local, local_token_stride,
                                  local_head_stride, n_local, causal, scale, out, out_token_stride, out_head_stride, lse,
                                  nullptr, err_flag, stream);
}

extern "C" int qe_set_attention_q_tiles(int32_t q_tiles) {
  if (q_tiles < 0 || q_tiles > 2) return qe::fail(QE_ERR_INVALID, "qe_set_attention_q_tiles: 0, 1 or 2");
  qe::g_attention_q_tiles.store(q_tiles, std::memory_order_relaxed);
  return qe::ok();
}

extern "C" int qe_paged_attention_append(const void *q, int64_t q_token_stride, int64_t q_head_stride, int32_t n_q,
                                         int32_t heads_q, const void *k_pool, const void *v_pool, int64_t pool_rows,
                                         int32_t heads_kv, const int32_t *block_table, int32_t page_size,
                                         int32_t n_prefix, const void *k_local, const void *v_local,
                                         int64_t local_token_stride, int64_t local_head_stride, int32_t n_local,
                                         int32_t causal, float scale, void *out, int64_t out_token_stride,
                                         int64_t out_head_stride, float *lse, const int32_t *append_table,
                                         int32_t *err_flag, void *stream) {
  if (!append_table || !err_flag)
    return qe::fail(QE_ERR_INVALID, "qe_paged_attention_append: null append table or error flag");
  return qe::paged_attention_impl(q, q_token_stride, q_head_stride, n_q, heads_q, k_pool, v_pool, pool_rows, heads_kv,
                                  block_table, page_size, n_prefix, k_local, v_local, local_token_stride,
                                  local_head_stride, n_local, causal, scale, out, out_token_stride, out_head_stride, lse,
                                  append_table, err_flag, stream);
}
