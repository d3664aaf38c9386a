// Paged K/V gather and append for the prefix pools.
//
// Replaces, on the device, the data movement of QwenEdit's PagedKVPool:
//   gather  multi_turn/cache/paged.py:106-113   kv.index_select(2, indices)  (and encoder.py:114 extra rows)
//   write   multi_turn/cache/paged.py:115-116   kv.index_copy_(2, indices, kv_new)
//   store   multi_turn/pipeline/hooks.py:136-138  2*L per-layer index_copy_ -> one launch (pointer form)
//
// A pool is a stack of planes (layer x {K,V}), each [rows, row_bytes]; a token's K or V for one layer is
// one row of H*D elements (6 KB for the Qwen-Image DiT, 1 KB for the text encoder). Every row copy is
// a vectorised, fully coalesced warp copy, all loads of a pass issued before the matching stores: on 32-byte
// aligned planes rows move in 256-bit vectors (lane i: bytes [32 i, 32 i + 32) of each 1 KiB stripe, 8 in
// flight per lane), else in 16-byte vectors (lane i: bytes [16 i, 16 i + 16) of each 512-byte stripe, 8 or 16
// in flight per lane); rows of at most 1 KiB go several per warp pass. Each warp walks its
// rows through the slot list (token-granular, page_size 1) or the block table (page_size P). The grid is
// persistent: a multiple of the SM count, warps striding over the (plane, token) rows.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "qe_cuda.cuh"

namespace qe {

int sm_count() {
  static std::atomic<int> cached[64];  // per device, filled on first use (relaxed: any thread may fill it)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  int c = cached[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
    cached[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

namespace {

constexpr int kThreads = 256;

struct Planes {
  char *base;
  int64_t outer, inner;
  int32_t per_outer;
  __device__ __forceinline__ char *plane(int32_t p) const {
    return base + int64_t(p / per_outer) * outer + int64_t(p % per_outer) * inner;
  }
};

struct CopyParams {
  Planes pool;
  Planes other;                    // the gather destination / append source
  const void *const *other_ptrs;   // per-plane source pointers (pointer form), else null
  int64_t pool_rows;
  int64_t n_tokens;
  int64_t row_bytes;
  const int64_t *slots;            // token form
  const int32_t *pages;            // block-table form
  int32_t page_size;
  int32_t n_planes;
  int32_t *err;
};

enum { kSlots = 0, kPages = 1 };

// Error-flag bits a copy kernel may set: an out-of-range slot or page (that row is skipped), a bounded wait that
// gave up (bulk kernel), and a per-plane source pointer (pointer form) that is null or not aligned to the
// vector width the launch chose (that plane is skipped: a misaligned vector load would fault the kernel).
constexpr int32_t kErrSlot = 1, kErrTimeout = 2, kErrSrcPtr = 4;

// Pointer form: the source plane's base, or null when it is null or not `align`-byte aligned (flagged).
__device__ __forceinline__ const char *checked_src(const CopyParams &p, int32_t plane, uint32_t align, bool report) {
  const char *ptr = static_cast<const char *>(p.other_ptrs[plane]);
  if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & (align - 1u)) != 0) {
    if (report && p.err) atomicOr(p.err, kErrSrcPtr);
    return nullptr;
  }
  return ptr;
}

// 32 bytes: one 256-bit load / store per lane (sm_100), so a warp request covers 1 KiB
struct alignas(32) Vec32 {
  uint32_t w[8];
};

template <typename V>
__device__ __forceinline__ V load_v(const V *p) {
  return *p;
}
template <>
__device__ __forceinline__ int4 load_v<int4>(const int4 *p) {
  return ld_stream(p);
}
template <>
__device__ __forceinline__ Vec32 load_v<Vec32>(const Vec32 *p) {
  Vec32 v;
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]), "=r"(v.w[6]),
                 "=r"(v.w[7])
               : "l"(p));
  return v;
}
template <typename V>
__device__ __forceinline__ void store_v(V *p, V v) {
  *p = v;
}
template <>
__device__ __forceinline__ void store_v<int4>(int4 *p, int4 v) {
  st_stream(p, v);
}
template <>
__device__ __forceinline__ void store_v<Vec32>(Vec32 *p, Vec32 v) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
               "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
               : "memory");
}

// kUnroll vectors per lane are loaded before any is stored: 16 for rows of 6 KiB and more (a whole DiT row in
// flight per warp), 8 for smaller rows.
template <typename V, int kMode, bool kGather, bool kPtrs, int kUnroll>
__global__ void __launch_bounds__(kThreads) paged_copy_kernel(CopyParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kThreads) >> 5;
  const int64_t rows = int64_t(p.n_planes) * p.n_tokens;
  const int64_t vpr = p.row_bytes / int64_t(sizeof(V));

  for (int64_t r = warp; r < rows; r += nwarps) {
    const int32_t plane = int32_t(r / p.n_tokens);
    const int64_t t = r - int64_t(plane) * p.n_tokens;
    int64_t slot;
    if (kMode == kSlots) {
      slot = __ldg(p.slots + t);
    } else {
      const int64_t page = __ldg(p.pages + t / p.page_size);
      slot = page * p.page_size + t % p.page_size;
    }
    if (slot < 0 || slot >= p.pool_rows) {  // out-of-range slot: skip the row, report it
      if (lane == 0 && p.err) atomicOr(p.err, kErrSlot);
      continue;
    }
    char *pool_row = p.pool.plane(plane) + slot * p.row_bytes;
    const char *other_row;
    if (kPtrs) {
      const char *src_plane = checked_src(p, plane, sizeof(V), lane == 0);
      if (src_plane == nullptr) continue;  // null or misaligned source plane: skipped, reported
      other_row = src_plane + t * p.row_bytes;
    } else {
      other_row = p.other.plane(plane) + t * p.row_bytes;
    }
    const V *src = reinterpret_cast<const V *>(kGather ? pool_row : other_row);
    V *dst = reinterpret_cast<V *>(kGather ? const_cast<char *>(other_row) : pool_row);
    for (int64_t v0 = 0; v0 < vpr; v0 += 32 * kUnroll) {
      V buf[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t v = v0 + k * 32 + lane;
        if (v < vpr) buf[k] = load_v<V>(src + v);
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t v = v0 + k * 32 + lane;
        if (v < vpr) store_v<V>(dst + v, buf[k]);
      }
    }
  }
}

// Short rows (eight or more fit in 32 x kUnroll vectors: the 1 KiB encoder rows, 768 B head-sharded DiT rows
// at 8 GPUs): one warp moves R = (32 kUnroll) / vpr consecutive tokens of one plane per pass, so each
// lane still has kUnroll loads in flight (16 of 16 bytes, or 8 of 32 bytes on 32-byte aligned planes: the same
// bytes with half the memory instructions). Lane i < R holds token i's slot; the other lanes read it with a
// shuffle. On the contiguous side (the gather output, the append source) the R rows are one run, so those
// accesses stay fully coalesced across row boundaries.
constexpr int kRowsUnroll = 16;

template <typename V, int kMode, bool kGather, bool kPtrs, int kUnroll = kRowsUnroll>
__global__ void __launch_bounds__(kThreads) paged_copy_rows_kernel(CopyParams p, int32_t rows_per_pass) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kThreads) >> 5;
  const int64_t vpr = p.row_bytes / int64_t(sizeof(V));
  const int R = rows_per_pass;
  const int64_t blocks_per_plane = (p.n_tokens + R - 1) / R;
  const int64_t items = int64_t(p.n_planes) * blocks_per_plane;

  for (int64_t it = warp; it < items; it += nwarps) {
    const int32_t plane = int32_t(it / blocks_per_plane);
    const int64_t t0 = (it - int64_t(plane) * blocks_per_plane) * R;
    // lane i < R: the slot of token t0 + i (-1 past the end), and the out-of-range report
    int64_t my_slot = -1;
    if (lane < R && t0 + lane < p.n_tokens) {
      const int64_t t = t0 + lane;
      if (kMode == kSlots) {
        my_slot = __ldg(p.slots + t);
      } else {
        my_slot = int64_t(__ldg(p.pages + t / p.page_size)) * p.page_size + t % p.page_size;
      }
      if (my_slot < 0 || my_slot >= p.pool_rows) {
        if (p.err) atomicOr(p.err, kErrSlot);
        my_slot = -2;  // skipped
      }
    }
    char *pool_plane = p.pool.plane(plane);
    const char *other_plane =
        kPtrs ? checked_src(p, plane, sizeof(V), lane == 0) : static_cast<const char *>(p.other.plane(plane));
    if (other_plane == nullptr) continue;  // pointer form: null or misaligned source plane, skipped and reported
    // the R rows of the pass are one run on the contiguous side: vector v of the pass is run[v]
    V *run = reinterpret_cast<V *>(const_cast<char *>(other_plane) + t0 * p.row_bytes);
    V buf[kUnroll];
    uint32_t valid = 0u;
    // (row, vector) of vector lane + 32 k of the pass, advanced by 32 per k
    int ri = int(lane / vpr);
    int64_t vec = lane - int64_t(ri) * vpr;
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int64_t slot = __shfl_sync(0xffffffffu, my_slot, ri < 32 ? ri : 0);
      if (ri < R && slot >= 0) {
        valid |= 1u << k;
        buf[k] = kGather ? load_v<V>(reinterpret_cast<const V *>(pool_plane + slot * p.row_bytes) + vec)
                         : load_v<V>(run + lane + 32 * k);
      }
      vec += 32;
      while (vec >= vpr) {
        vec -= vpr;
        ++ri;
      }
    }
    if (kGather) {
#pragma unroll
      for (int k = 0; k < kUnroll; ++k)
        if (valid & (1u << k)) store_v<V>(run + lane + 32 * k, buf[k]);
    } else {  // walk the pass again for the pool rows
      ri = int(lane / vpr);
      vec = lane - int64_t(ri) * vpr;
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t slot = __shfl_sync(0xffffffffu, my_slot, ri < 32 ? ri : 0);
        if (valid & (1u << k)) store_v<V>(reinterpret_cast<V *>(pool_plane + slot * p.row_bytes) + vec, buf[k]);
        vec += 32;
        while (vec >= vpr) {
          vec -= vpr;
          ++ri;
        }
      }
    }
  }
}

// Gather into a head-major layout with room for a tail: out[plane][h][t] (head stride and token stride free)
// = pool row slots[t] of plane, head h. For the text encoder's partial hit (cache/encoder.py:173-182), which
// gathers the prefix [L, 2, m, H, D] and then, per layer, transposes it and concatenates the tail K/V into a
// fresh [1, H, m + n, D] tensor: written here once, straight into a [L, 2, H, m + n, D] buffer whose last n
// positions the caller fills per layer. One warp moves R consecutive tokens of one plane per pass (256-bit
// vectors, 8 per lane in flight, when every address is 32-byte aligned; else 16-byte vectors, 16 in flight);
// lane i < R holds token i's slot.
struct HeadsParams {
  Planes pool;
  Planes out;
  int64_t pool_rows, n_tokens, row_bytes, head_bytes, out_head_stride, out_token_stride;
  const int64_t *slots;
  int32_t n_planes, rows_per_pass;
  int32_t head_shift;  // log2(head_bytes / vector bytes) when that is a power of two, else -1
  int32_t *err;
};

// Loads of a pass first (kUnroll vectors per lane, a validity bitmask), then a second walk over the same vectors
// for their head-major destinations, so no destination pointer is kept live across the loads; the head of a
// vector is a shift when the head size is a power of two (head_shift >= 0). V = int4 with 16 vectors per lane,
// or Vec32 (256-bit loads and stores, every address 32-byte aligned) with 8: the same bytes in flight with half
// the memory instructions.
template <typename V, int kUnroll>
__global__ void __launch_bounds__(kThreads, 2) gather_heads_kernel(HeadsParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kThreads) >> 5;
  const int vpr = int(p.row_bytes / int64_t(sizeof(V))), vph = int(p.head_bytes / int64_t(sizeof(V)));
  const int R = p.rows_per_pass;
  const int64_t blocks_per_plane = (p.n_tokens + R - 1) / R;
  const int64_t items = int64_t(p.n_planes) * blocks_per_plane;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int32_t plane = int32_t(it / blocks_per_plane);
    const int64_t t0 = (it - int64_t(plane) * blocks_per_plane) * R;
    int64_t my_slot = -1;
    if (lane < R && t0 + lane < p.n_tokens) {
      my_slot = __ldg(p.slots + t0 + lane);
      if (my_slot < 0 || my_slot >= p.pool_rows) {
        if (p.err) atomicOr(p.err, kErrSlot);
        my_slot = -2;
      }
    }
    const char *pool_plane = p.pool.plane(plane);
    char *out_plane = p.out.plane(plane) + t0 * p.out_token_stride;
    for (int base = 0; base < R * vpr; base += 32 * kUnroll) {
      V buf[kUnroll];
      uint32_t valid = 0u;
      int ri = (base + lane) / vpr, vin = (base + lane) - ri * vpr;
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t slot = __shfl_sync(0xffffffffu, my_slot, ri < 32 ? ri : 0);
        if (ri < R && slot >= 0) {
          valid |= 1u << k;
          buf[k] = load_v<V>(reinterpret_cast<const V *>(pool_plane + slot * p.row_bytes) + vin);
        }
        vin += 32;
        while (vin >= vpr) {
          vin -= vpr;
          ++ri;
        }
      }
      ri = (base + lane) / vpr;
      vin = (base + lane) - ri * vpr;
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        if (valid & (1u << k)) {
          const int h = p.head_shift >= 0 ? vin >> p.head_shift : vin / vph;
          const int w = vin - h * vph;
          V *dst = reinterpret_cast<V *>(out_plane + h * p.out_head_stride + int64_t(ri) * p.out_token_stride) + w;
          if constexpr (sizeof(V) == 32) {  // a plain (not streaming) 256-bit store: the buffer is read next
            const Vec32 &v = reinterpret_cast<const Vec32 &>(buf[k]);
            asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(v.w[0]), "r"(v.w[1]),
                         "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
                         : "memory");
          } else {
            *dst = buf[k];
          }
        }
        vin += 32;
        while (vin >= vpr) {
          vin -= vpr;
          ++ri;
        }
      }
    }
  }
}

// ---- TMA bulk-copy variant --------------------------------------------------------------------
// One elected thread per CTA drives the copy engine: cp.async.bulk global->shared (completion counted in
// bytes on a per-stage mbarrier) then cp.async.bulk shared->global, kStages chunks of up to kChunk bytes in
// flight. A chunk is either a byte range of one page run (block-table form: one load, one store) or up to
// kChunk / row_bytes consecutive tokens (slot form: one op per scattered row, one op for the contiguous
// side). Every mbarrier wait is bounded (kWaitNs); on expiry the kernel records QE_ERR_TIMEOUT in the error
// flag, drains what it issued (bounded again) and returns.
constexpr int kStages = 6;
constexpr int kChunk = 32 * 1024;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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

// bounded wait on an mbarrier phase; false when it gave up
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitNs) return false;
  }
  return true;
}

__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_smem),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void bulk_store(void *dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct BulkGeom {
  int64_t chunks_per_plane;  // chunks of one plane
  int64_t chunks_per_run;    // block-table form: chunks of one full page run
  int64_t rows_per_chunk;    // slot form: tokens per chunk
};

// Issue the loads (kLoad) or the stores (!kLoad) of chunk c; returns the bytes moved into shared memory.
template <int kMode, bool kGather, bool kPtrs, bool kLoad>
__device__ __forceinline__ uint32_t bulk_chunk(const CopyParams &p, const BulkGeom &g, int64_t c, uint32_t stage,
                                               uint32_t bar) {
  const int32_t plane = int32_t(c / g.chunks_per_plane);
  const int64_t rem = c - int64_t(plane) * g.chunks_per_plane;
  char *pool_plane = p.pool.plane(plane);
  char *oth_plane = kPtrs ? const_cast<char *>(checked_src(p, plane, 16, false)) : p.other.plane(plane);
  if (kPtrs && oth_plane == nullptr) return 0;  // skipped plane (reported by bulk_chunk_bytes)
  if (kMode == kPages) {
    const int64_t run = rem / g.chunks_per_run;
    const int64_t k = rem - run * g.chunks_per_run;
    const int64_t t0 = run * p.page_size;
    const int64_t rows = min(int64_t(p.page_size), p.n_tokens - t0);
    const int64_t off = k * kChunk;
    const int64_t run_bytes = rows * p.row_bytes;
    if (off >= run_bytes) return 0;
    const uint32_t bytes = uint32_t(min(int64_t(kChunk), run_bytes - off));
    const int64_t page = __ldg(p.pages + run);
    if (page < 0 || (page + 1) * p.page_size > p.pool_rows) {
      if (kLoad && p.err) atomicOr(p.err, kErrSlot);
      return 0;
    }
    char *pool_ptr = pool_plane + page * p.page_size * p.row_bytes + off;
    char *oth_ptr = oth_plane + t0 * p.row_bytes + off;
    if (kLoad) {
      bulk_load(stage, kGather ? pool_ptr : oth_ptr, bytes, bar);
    } else {
      bulk_store(kGather ? oth_ptr : pool_ptr, stage, bytes);
    }
    return bytes;
  } else {
    const int64_t t0 = rem * g.rows_per_chunk;
    const int64_t rows = min(g.rows_per_chunk, p.n_tokens - t0);
    if (rows <= 0) return 0;
    const uint32_t rb = uint32_t(p.row_bytes);
    uint32_t moved = 0;
    // the contiguous side (gather: output rows t0..; append: source rows t0..) is one op
    if constexpr (kLoad == !kGather) {  // the contiguous side
      char *oth_ptr = oth_plane + t0 * p.row_bytes;
      if (kLoad) {
        bulk_load(stage, oth_ptr, uint32_t(rows) * rb, bar);
      } else {
        bulk_store(oth_ptr, stage, uint32_t(rows) * rb);
      }
      return uint32_t(rows) * rb;
    } else {
    for (int64_t i = 0; i < rows; ++i) {
      const int64_t slot = __ldg(p.slots + t0 + i);
      if (slot < 0 || slot >= p.pool_rows) {
        if (kLoad && p.err) atomicOr(p.err, kErrSlot);
        continue;  // skipped row: its bytes are not expected
      }
      char *pool_ptr = pool_plane + slot * p.row_bytes;
      if (kLoad) {
        bulk_load(stage + uint32_t(i) * rb, pool_ptr, rb, bar);
      } else {
        bulk_store(pool_ptr, stage + uint32_t(i) * rb, rb);
      }
      moved += rb;
    }
    return moved;
    }
  }
}

// bytes the loads of chunk c will deliver (the mbarrier's transaction count), computed before issuing
template <int kMode, bool kGather, bool kPtrs>
__device__ __forceinline__ uint32_t bulk_chunk_bytes(const CopyParams &p, const BulkGeom &g, int64_t c) {
  const int32_t plane = int32_t(c / g.chunks_per_plane);
  const int64_t rem = c - int64_t(plane) * g.chunks_per_plane;
  if (kPtrs && checked_src(p, plane, 16, true) == nullptr) return 0;  // null or misaligned source plane
  if (kMode == kPages) {
    const int64_t run = rem / g.chunks_per_run;
    const int64_t k = rem - run * g.chunks_per_run;
    const int64_t rows = min(int64_t(p.page_size), p.n_tokens - run * p.page_size);
    const int64_t off = k * kChunk, run_bytes = rows * p.row_bytes;
    if (off >= run_bytes) return 0;
    const int64_t page = __ldg(p.pages + run);
    if (page < 0 || (page + 1) * p.page_size > p.pool_rows) return 0;
    return uint32_t(min(int64_t(kChunk), run_bytes - off));
  }
  const int64_t t0 = rem * g.rows_per_chunk;
  const int64_t rows = min(g.rows_per_chunk, p.n_tokens - t0);
  if (rows <= 0) return 0;
  if (!kGather) return uint32_t(rows * p.row_bytes);
  uint32_t bytes = 0;
  for (int64_t i = 0; i < rows; ++i) {
    const int64_t slot = __ldg(p.slots + t0 + i);
    if (slot >= 0 && slot < p.pool_rows) bytes += uint32_t(p.row_bytes);
  }
  return bytes;
}

template <int kMode, bool kGather, bool kPtrs>
__global__ void __launch_bounds__(32) paged_bulk_kernel(CopyParams p, BulkGeom g) {
  extern __shared__ __align__(128) uint8_t stage_mem[];
  __shared__ __align__(8) uint64_t bars[kStages];
  if (threadIdx.x != 0) return;  // one thread issues every copy; the copy engine does the rest
  const int64_t total = g.chunks_per_plane * p.n_planes;
  const int64_t first = blockIdx.x, stride = gridDim.x;
  const int64_t mine = first < total ? (total - first + stride - 1) / stride : 0;
  if (mine == 0) return;
  const uint32_t base = smem_u32(stage_mem);
  for (int s = 0; s < kStages; ++s) mbar_init(smem_u32(&bars[s]));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  auto issue_load = [&](int64_t i) {
    const int64_t c = first + i * stride;
    const uint32_t s = uint32_t(i % kStages);
    const uint32_t bar = smem_u32(&bars[s]);
    const uint32_t bytes = bulk_chunk_bytes<kMode, kGather, kPtrs>(p, g, c);
    mbar_expect(bar, bytes);
    if (bytes) bulk_chunk<kMode, kGather, kPtrs, true>(p, g, c, base + s * kChunk, bar);
  };

  const int64_t prologue = min(mine, int64_t(kStages));
  for (int64_t i = 0; i < prologue; ++i) issue_load(i);
  bool ok = true;
  int64_t i = 0;
  for (; i < mine; ++i) {
    const uint32_t s = uint32_t(i % kStages);
    if (!mbar_wait(smem_u32(&bars[s]), uint32_t((i / kStages) & 1))) {
      ok = false;
      break;
    }
    bulk_chunk<kMode, kGather, kPtrs, false>(p, g, first + i * stride, base + s * kChunk, 0);
    bulk_commit();
    // refill the stage of chunk i-1 once its store has finished reading shared memory
    if (i >= 1 && i - 1 + kStages < mine) {
      bulk_wait_read_1();
      issue_load(i - 1 + kStages);
    }
  }
  if (!ok) {
    if (p.err) atomicOr(p.err, kErrTimeout);
    // drain the loads still in flight (each wait bounded again) so no copy lands in a retired CTA
    const int64_t issued = min(mine, (i >= 1 ? i - 1 + kStages : int64_t(kStages)));
    for (int64_t j = i; j < issued; ++j) mbar_wait(smem_u32(&bars[j % kStages]), uint32_t((j / kStages) & 1));
  }
  bulk_wait_all();
}

int bulk_launch_check(const CopyParams &p, int align) {
  if (align < 16 || p.row_bytes > kChunk || p.row_bytes % 16) return 0;
  return 1;
}

// 0 auto, 1 warp LDG/STG, 2 TMA bulk, 3 warp LDG/STG with one row per warp pass, 4 warp LDG/STG with 16-byte
// vectors only
std::atomic<int> g_copy_mode{0};

template <int kMode, bool kGather, bool kPtrs>
int launch_bulk(const CopyParams &p, cudaStream_t stream) {
  static std::atomic<bool> attr_done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!attr_done[dev].load(std::memory_order_relaxed)) {
    cudaError_t e = cudaFuncSetAttribute(paged_bulk_kernel<kMode, kGather, kPtrs>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kStages * kChunk);
    if (e != cudaSuccess) return cuda_status(e, "paged bulk copy: smem attribute");
    attr_done[dev].store(true, std::memory_order_relaxed);
  }
  BulkGeom g{};
  if (kMode == kPages) {
    g.chunks_per_run = (int64_t(p.page_size) * p.row_bytes + kChunk - 1) / kChunk;
    const int64_t runs = (p.n_tokens + p.page_size - 1) / p.page_size;
    g.chunks_per_plane = runs * g.chunks_per_run;
  } else {
    g.rows_per_chunk = kChunk / p.row_bytes;
    g.chunks_per_plane = (p.n_tokens + g.rows_per_chunk - 1) / g.rows_per_chunk;
  }
  const int64_t total = g.chunks_per_plane * p.n_planes;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(total, int64_t(sm_count())));
  paged_bulk_kernel<kMode, kGather, kPtrs><<<dim3(unsigned(blocks)), dim3(32), kStages * kChunk, stream>>>(p, g);
  return cuda_status(cudaGetLastError(), "paged bulk copy launch");
}

template <typename V, int kMode, bool kGather, bool kPtrs, int kUnroll>
int launch_unrolled(const CopyParams &p, cudaStream_t stream) {
  static std::atomic<int> cached_blocks{0};
  int blocks_per_sm = cached_blocks.load(std::memory_order_relaxed);
  if (blocks_per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &blocks_per_sm, paged_copy_kernel<V, kMode, kGather, kPtrs, kUnroll>, kThreads, 0) != cudaSuccess ||
        blocks_per_sm <= 0)
      blocks_per_sm = 2;
    cached_blocks.store(blocks_per_sm, std::memory_order_relaxed);
  }
  const int64_t rows = int64_t(p.n_planes) * p.n_tokens;
  const int64_t warps_per_block = kThreads / 32;
  int64_t blocks = std::min<int64_t>((rows + warps_per_block - 1) / warps_per_block, int64_t(sm_count()) * blocks_per_sm);
  blocks = std::max<int64_t>(blocks, 1);
  paged_copy_kernel<V, kMode, kGather, kPtrs, kUnroll><<<dim3(unsigned(blocks)), dim3(kThreads), 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "paged copy launch");
}

template <typename V, int kMode, bool kGather, bool kPtrs, int kUnroll = kRowsUnroll>
int launch_rows(const CopyParams &p, int rows_per_pass, cudaStream_t stream) {
  static std::atomic<int> cached_blocks{0};
  int blocks_per_sm = cached_blocks.load(std::memory_order_relaxed);
  if (blocks_per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks_per_sm,
                                                      paged_copy_rows_kernel<V, kMode, kGather, kPtrs, kUnroll>,
                                                      kThreads, 0) != cudaSuccess ||
        blocks_per_sm <= 0)
      blocks_per_sm = 2;
    cached_blocks.store(blocks_per_sm, std::memory_order_relaxed);
  }
  const int64_t items = int64_t(p.n_planes) * ((p.n_tokens + rows_per_pass - 1) / rows_per_pass);
  const int64_t warps_per_block = kThreads / 32;
  int64_t blocks = std::min<int64_t>((items + warps_per_block - 1) / warps_per_block, int64_t(sm_count()) * blocks_per_sm);
  blocks = std::max<int64_t>(blocks, 1);
  paged_copy_rows_kernel<V, kMode, kGather, kPtrs, kUnroll>
      <<<dim3(unsigned(blocks)), dim3(kThreads), 0, stream>>>(p, int32_t(rows_per_pass));
  return cuda_status(cudaGetLastError(), "paged copy launch");
}

template <typename V, int kMode, bool kGather, bool kPtrs>
int launch_typed(const CopyParams &p, cudaStream_t stream) {
  const int64_t vpr = p.row_bytes / int64_t(sizeof(V));
  // rows of at most 1 KiB (eight or more per warp pass): the short-row kernel. Measured on 60-layer 2K gathers:
  // 768 B rows 0.86 of HBM vs 0.63 one row per pass; 1.5 KiB rows 0.87 vs 0.94 (the per-vector shuffle and row
  // arithmetic cost more than the extra loads in flight gain). g_copy_mode 3 forces the one-row kernel.
  const int64_t per_pass = std::min<int64_t>(32 * kRowsUnroll / std::max<int64_t>(vpr, 1), 32);
  if (g_copy_mode.load(std::memory_order_relaxed) != 3 && per_pass >= 8)
    return launch_rows<V, kMode, kGather, kPtrs>(p, int(per_pass), stream);
  if (vpr >= 32 * 12) return launch_unrolled<V, kMode, kGather, kPtrs, 16>(p, stream);
  return launch_unrolled<V, kMode, kGather, kPtrs, 8>(p, stream);
}

bool planes_aligned(const qe_planes &pl, int a) {
  return (reinterpret_cast<uintptr_t>(pl.base) % a) == 0 && pl.outer_stride % a == 0 && pl.inner_stride % a == 0;
}

template <int kMode, bool kGather, bool kPtrs>
int launch(const CopyParams &p, int align, cudaStream_t stream) {
  const int mode = g_copy_mode.load(std::memory_order_relaxed);
  if (mode == 2 && bulk_launch_check(p, align)) return launch_bulk<kMode, kGather, kPtrs>(p, stream);
  // rows above 1 KiB (one row per warp pass) on 32-byte aligned planes: 256-bit vectors, 8 per lane in flight
  // (the same bytes as 16 of 16 bytes, half the instructions and L1 requests)
  if (align >= 32 && mode != 4 && (p.row_bytes > 1024 || mode == 3))
    return launch_unrolled<Vec32, kMode, kGather, kPtrs, 8>(p, stream);
  // rows of at most 1 KiB on 32-byte aligned planes (eight or more per warp pass): the short-row kernel with
  // 256-bit vectors, 8 per lane in flight
  if (align >= 32 && mode != 4 && 32 * 8 / (p.row_bytes / 32) >= 8)
    return launch_rows<Vec32, kMode, kGather, kPtrs, 8>(
        p, int(std::min<int64_t>(32 * 8 / (p.row_bytes / 32), 32)), stream);
  if (align >= 16) return launch_typed<int4, kMode, kGather, kPtrs>(p, stream);
  if (align >= 4) return launch_typed<uint32_t, kMode, kGather, kPtrs>(p, stream);
  return launch_typed<uint8_t, kMode, kGather, kPtrs>(p, stream);
}

Planes to_planes(const qe_planes &q) {
  Planes p;
  p.base = static_cast<char *>(q.base);
  p.outer = q.outer_stride;
  p.inner = q.inner_stride;
  p.per_outer = q.planes_inner > 0 ? q.planes_inner : 1;
  return p;
}

int common_checks(const char *fn, const qe_planes &pool, int64_t pool_rows, int32_t n_planes, int64_t row_bytes,
                  int64_t n_tokens) {
  if (!pool.base) return fail(QE_ERR_INVALID, "%s: null pool", fn);
  if (pool.planes_inner < 1) return fail(QE_ERR_INVALID, "%s: planes_inner must be >= 1", fn);
  if (n_planes < 0 || n_tokens < 0) return fail(QE_ERR_INVALID, "%s: negative size", fn);
  if (row_bytes <= 0) return fail(QE_ERR_INVALID, "%s: row_bytes must be positive", fn);
  if (pool_rows <= 0) return fail(QE_ERR_INVALID, "%s: pool_rows must be positive", fn);
  return QE_OK;
}

// Largest vector width (32, 16, 4 or 1 bytes) every address of the copy is aligned to.
int align_of(const qe_planes &a, const qe_planes *b, int64_t row_bytes) {
  for (int w : {32, 16, 4}) {
    if (row_bytes % w == 0 && planes_aligned(a, w) && (!b || planes_aligned(*b, w))) return w;
  }
  return 1;
}

}  // namespace
}  // namespace qe

using qe::fail;

extern "C" {

int qe_gather_slots(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                    const int64_t *slots, int64_t n_tokens, int32_t *err_flag, void *stream) {
  int s = qe::common_checks("qe_gather_slots", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!out.base || !slots) return fail(QE_ERR_INVALID, "qe_gather_slots: null output or slots");
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other = qe::to_planes(out);
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.slots = slots;
  p.n_planes = n_planes;
  p.err = err_flag;
  s = qe::launch<qe::kSlots, true, false>(p, qe::align_of(pool, &out, row_bytes), static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

int qe_gather_pages(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                    const int32_t *block_table, int32_t page_size, int64_t n_tokens, int32_t *err_flag,
                    void *stream) {
  int s = qe::common_checks("qe_gather_pages", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (page_size < 1) return fail(QE_ERR_INVALID, "qe_gather_pages: page_size must be >= 1");
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!out.base || !block_table) return fail(QE_ERR_INVALID, "qe_gather_pages: null output or block table");
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other = qe::to_planes(out);
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.pages = block_table;
  p.page_size = page_size;
  p.n_planes = n_planes;
  p.err = err_flag;
  s = qe::launch<qe::kPages, true, false>(p, qe::align_of(pool, &out, row_bytes), static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

int qe_append_slots(qe_planes pool, int64_t pool_rows, qe_planes src, int32_t n_planes, int64_t row_bytes,
                    const int64_t *slots, int64_t n_tokens, int32_t *err_flag, void *stream) {
  int s = qe::common_checks("qe_append_slots", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!src.base || !slots) return fail(QE_ERR_INVALID, "qe_append_slots: null source or slots");
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other = qe::to_planes(src);
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.slots = slots;
  p.n_planes = n_planes;
  p.err = err_flag;
  s = qe::launch<qe::kSlots, false, false>(p, qe::align_of(pool, &src, row_bytes), static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

int qe_append_pages(qe_planes pool, int64_t pool_rows, qe_planes src, int32_t n_planes, int64_t row_bytes,
                    const int32_t *block_table, int32_t page_size, int64_t n_tokens, int32_t *err_flag,
                    void *stream) {
  int s = qe::common_checks("qe_append_pages", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (page_size < 1) return fail(QE_ERR_INVALID, "qe_append_pages: page_size must be >= 1");
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!src.base || !block_table) return fail(QE_ERR_INVALID, "qe_append_pages: null source or block table");
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other = qe::to_planes(src);
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.pages = block_table;
  p.page_size = page_size;
  p.n_planes = n_planes;
  p.err = err_flag;
  s = qe::launch<qe::kPages, false, false>(p, qe::align_of(pool, &src, row_bytes), static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

int qe_append_slots_ptrs(qe_planes pool, int64_t pool_rows, const void *const *src_ptrs, int32_t n_planes,
                         int64_t row_bytes, const int64_t *slots, int64_t n_tokens, int32_t *err_flag,
                         void *stream) {
  int s = qe::common_checks("qe_append_slots_ptrs", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!src_ptrs || !slots) return fail(QE_ERR_INVALID, "qe_append_slots_ptrs: null source pointers or slots");
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other_ptrs = src_ptrs;
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.slots = slots;
  p.n_planes = n_planes;
  p.err = err_flag;
  // Source pointers are only known on the device; the Python side checks each one for 16-byte
  // alignment before uploading the array, so the width follows the pool and the row size, up to 16 bytes.
  s = qe::launch<qe::kSlots, false, true>(p, std::min(16, qe::align_of(pool, nullptr, row_bytes)),
                                          static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

int qe_gather_slots_heads(qe_planes pool, int64_t pool_rows, qe_planes out, int32_t n_planes, int64_t row_bytes,
                          int64_t head_bytes, int64_t out_head_stride, int64_t out_token_stride, const int64_t *slots,
                          int64_t n_tokens, int32_t *err_flag, void *stream) {
  QE_CHECK_ARG(n_planes >= 1 && pool_rows >= 1 && n_tokens >= 0, "qe_gather_slots_heads: bad sizes");
  QE_CHECK_ARG(head_bytes > 0 && head_bytes % 16 == 0 && row_bytes % head_bytes == 0,
               "qe_gather_slots_heads: head_bytes must be a multiple of 16 dividing row_bytes");
  QE_CHECK_ARG(out_head_stride % 16 == 0 && out_token_stride % 16 == 0 && out_head_stride >= 0 && out_token_stride >= 0,
               "qe_gather_slots_heads: output strides must be non-negative multiples of 16 bytes");
  QE_CHECK_ARG(pool.planes_inner >= 1 && out.planes_inner >= 1, "qe_gather_slots_heads: planes_inner must be >= 1");
  QE_CHECK_ARG(pool.base && out.base && qe::planes_aligned(pool, 16) && qe::planes_aligned(out, 16),
               "qe_gather_slots_heads: planes must be 16-byte aligned");
  QE_CHECK_ARG(n_tokens == 0 || slots, "qe_gather_slots_heads: null slots");
  if (n_tokens == 0) return qe::ok();
  qe::HeadsParams p{};
  p.pool = qe::to_planes(pool);
  p.out = qe::to_planes(out);
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.head_bytes = head_bytes;
  p.out_head_stride = out_head_stride;
  p.out_token_stride = out_token_stride;
  p.slots = slots;
  p.n_planes = n_planes;
  // 256-bit vectors when every address of the copy is 32-byte aligned (the encoder's 1 KiB rows of 256-byte heads
  // into a buffer from the caching allocator), unless the copy mode asks for 16-byte vectors
  const bool wide = qe::g_copy_mode.load(std::memory_order_relaxed) != 4 && row_bytes % 32 == 0 &&
                    head_bytes % 32 == 0 && out_head_stride % 32 == 0 && out_token_stride % 32 == 0 &&
                    qe::planes_aligned(pool, 32) && qe::planes_aligned(out, 32);
  const int64_t vec = wide ? 32 : 16, unroll = wide ? 8 : qe::kRowsUnroll;
  p.rows_per_pass = int32_t(std::max<int64_t>(1, std::min<int64_t>(32 * unroll / (row_bytes / vec), 32)));
  p.head_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((int64_t(1) << sh) == head_bytes / vec) p.head_shift = sh;
  p.err = err_flag;
  const int64_t items = int64_t(n_planes) * ((n_tokens + p.rows_per_pass - 1) / p.rows_per_pass);
  const int64_t warps_per_block = qe::kThreads / 32;
  int64_t blocks = std::min<int64_t>((items + warps_per_block - 1) / warps_per_block, int64_t(qe::sm_count()) * 2);
  blocks = std::max<int64_t>(blocks, 1);
  if (wide)
    qe::gather_heads_kernel<qe::Vec32, 8>
        <<<dim3(unsigned(blocks)), dim3(qe::kThreads), 0, static_cast<cudaStream_t>(stream)>>>(p);
  else
    qe::gather_heads_kernel<int4, qe::kRowsUnroll>
        <<<dim3(unsigned(blocks)), dim3(qe::kThreads), 0, static_cast<cudaStream_t>(stream)>>>(p);
  int s = qe::cuda_status(cudaGetLastError(), "qe_gather_slots_heads launch");
  return s ? s : qe::ok();
}

int qe_set_paged_copy_mode(int32_t mode) {
  if (mode < 0 || mode > 4) return fail(QE_ERR_INVALID, "qe_set_paged_copy_mode: mode must be 0, 1, 2, 3 or 4");
  qe::g_copy_mode.store(mode, std::memory_order_relaxed);
  return qe::ok();
}

const char *qe_version(void) { return "qeb200 0.1.0 (sm_100a)"; }

}  // extern "C"

// ---- variant of qe_append_slots_ptrs that allocates nothing ----------------------------------------
// The per-plane source-pointer table lives in this module's own device memory: a file-scope array that
// every GPU loading the library holds until exit. Host code must not pass the array's name to a kernel (in
// host code it is only a stand-in symbol); its device address comes from cudaGetSymbolAddress, taken once
// per device with that device current.
namespace qe {
constexpr int32_t kStaticMaxPlanes = 1024;  // 8 KiB of pointers: 512 layers of K and V
}  // namespace qe

static __device__ __align__(256) const void *g_static_src_ptrs[qe::kStaticMaxPlanes];

namespace qe {
namespace {
// One lock per device, held from the table write through the kernel launch, so that two host threads issuing on
// the same stream cannot interleave as write A, write B, kernel A, kernel B (kernel A would read B's pointers).
std::mutex g_static_table_lock[64];

int static_ptr_table(int *dev_out, const void *const **out) {
  static std::atomic<const void *const *> addr[64];  // per device: the table's device address
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "qe_append_slots_ptrs_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(QE_ERR_INVALID, "qe_append_slots_ptrs_noalloc: device %d above 63", dev);
  *dev_out = dev;
  const void *const *table = addr[dev].load(std::memory_order_relaxed);
  if (!table) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_src_ptrs);
    if (e != cudaSuccess) return cuda_status(e, "qe_append_slots_ptrs_noalloc: cudaGetSymbolAddress");
    table = static_cast<const void *const *>(ptr);
    addr[dev].store(table, std::memory_order_relaxed);
  }
  *out = table;
  return QE_OK;
}
}  // namespace
}  // namespace qe

extern "C" int qe_append_slots_ptrs_noalloc(qe_planes pool, int64_t pool_rows, const void *const *src_ptrs_host,
                                            int32_t n_planes, int64_t row_bytes, const int64_t *slots,
                                            int64_t n_tokens, int32_t *err_flag, void *stream) {
  int s = qe::common_checks("qe_append_slots_ptrs_noalloc", pool, pool_rows, n_planes, row_bytes, n_tokens);
  if (s) return s;
  if (n_planes > qe::kStaticMaxPlanes)
    return fail(QE_ERR_INVALID, "qe_append_slots_ptrs_noalloc: %d planes exceed the static table's %d", n_planes,
                qe::kStaticMaxPlanes);
  if (n_planes == 0 || n_tokens == 0) return qe::ok();
  if (!src_ptrs_host || !slots) return fail(QE_ERR_INVALID, "qe_append_slots_ptrs_noalloc: null source pointers or slots");
  // the vector width also follows the source pointers, which are known here on the host
  int align = qe::align_of(pool, nullptr, row_bytes);
  for (int32_t i = 0; i < n_planes; ++i) {
    if (!src_ptrs_host[i]) return fail(QE_ERR_INVALID, "qe_append_slots_ptrs_noalloc: null source pointer %d", i);
    while (align > 1 && (reinterpret_cast<uintptr_t>(src_ptrs_host[i]) % align) != 0)
      align = align == 32 ? 16 : align == 16 ? 4 : 1;
  }
  const void *const *table = nullptr;
  int dev = 0;
  s = qe::static_ptr_table(&dev, &table);
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> hold(qe::g_static_table_lock[dev]);
  // The table is written on the caller's stream ahead of the kernel that reads it. A pageable host array is
  // staged by the copy before this call returns; a pinned one is read by the GPU when the stream reaches the
  // copy, so it must stay unchanged until then.
  s = qe::cuda_status(cudaMemcpyAsync(const_cast<const void **>(table), src_ptrs_host, size_t(n_planes) * sizeof(void *),
                                      cudaMemcpyHostToDevice, st),
                      "qe_append_slots_ptrs_noalloc: pointer table copy");
  if (s) return s;
  qe::CopyParams p{};
  p.pool = qe::to_planes(pool);
  p.other_ptrs = table;
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.row_bytes = row_bytes;
  p.slots = slots;
  p.n_planes = n_planes;
  p.err = err_flag;
  s = qe::launch<qe::kSlots, false, true>(p, align, st);
  return s ? s : qe::ok();
}
