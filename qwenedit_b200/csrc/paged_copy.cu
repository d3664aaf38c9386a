// Paged K/V gather and append for the prefix pools.
//
// Replaces, on the device, the data movement of QwenEdit's PagedKVPool:
//   gather  multi_turn/cache/paged.py:106-113   kv.index_select(2, indices)  (and encoder.py:114 extra rows)
//   write   multi_turn/cache/paged.py:115-116   kv.index_copy_(2, indices, kv_new)
//   store   multi_turn/pipeline/hooks.py:136-138  2*L per-layer index_copy_ -> one launch (pointer form)
//
// A pool is a stack of planes (layer x {K,V}), each [rows, row_bytes]; a token's K or V for one layer is
// one row of H*D elements (6 KB for the Qwen-Image DiT, 1 KB for the text encoder). Every row copy is
// a 16-byte-vectorised, fully coalesced warp copy: lane i moves bytes [16 i, 16 i + 16) of each 512-byte
// stripe, with up to kUnroll loads in flight per lane before the matching stores. Each warp walks its
// rows through the slot list (token-granular, page_size 1) or the block table (page_size P). The grid is
// persistent: a multiple of the SM count, warps striding over the (plane, token) rows.
#include <algorithm>
#include <cstdint>

#include "qe_cuda.cuh"

namespace qe {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;

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

template <typename V>
__device__ __forceinline__ V load_v(const V *p) {
  return *p;
}
template <>
__device__ __forceinline__ int4 load_v<int4>(const int4 *p) {
  return ld_stream(p);
}
template <typename V>
__device__ __forceinline__ void store_v(V *p, V v) {
  *p = v;
}
template <>
__device__ __forceinline__ void store_v<int4>(int4 *p, int4 v) {
  st_stream(p, v);
}

template <typename V, int kMode, bool kGather, bool kPtrs>
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
      if (lane == 0 && p.err) atomicOr(p.err, 1);
      continue;
    }
    char *pool_row = p.pool.plane(plane) + slot * p.row_bytes;
    const char *other_row;
    if (kPtrs) {
      other_row = static_cast<const char *>(p.other_ptrs[plane]) + t * p.row_bytes;
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

template <typename V, int kMode, bool kGather, bool kPtrs>
int launch_typed(const CopyParams &p, cudaStream_t stream) {
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, paged_copy_kernel<V, kMode, kGather, kPtrs>, kThreads, 0) !=
            cudaSuccess ||
        b <= 0)
      b = 4;
    blocks_per_sm = b;
  }
  const int64_t rows = int64_t(p.n_planes) * p.n_tokens;
  const int64_t warps_per_block = kThreads / 32;
  int64_t blocks = std::min<int64_t>((rows + warps_per_block - 1) / warps_per_block, int64_t(sm_count()) * blocks_per_sm);
  blocks = std::max<int64_t>(blocks, 1);
  paged_copy_kernel<V, kMode, kGather, kPtrs><<<dim3(unsigned(blocks)), dim3(kThreads), 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "paged copy launch");
}

bool planes_aligned(const qe_planes &pl, int a) {
  return (reinterpret_cast<uintptr_t>(pl.base) % a) == 0 && pl.outer_stride % a == 0 && pl.inner_stride % a == 0;
}

template <int kMode, bool kGather, bool kPtrs>
int launch(const CopyParams &p, int align, cudaStream_t stream) {
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

// Largest vector width (16, 4 or 1 bytes) every address of the copy is aligned to.
int align_of(const qe_planes &a, const qe_planes *b, int64_t row_bytes) {
  for (int w : {16, 4}) {
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
  // alignment before uploading the array, so the width follows the pool and the row size.
  s = qe::launch<qe::kSlots, false, true>(p, qe::align_of(pool, nullptr, row_bytes), static_cast<cudaStream_t>(stream));
  return s ? s : qe::ok();
}

const char *qe_version(void) { return "qeb200 0.1.0 (sm_100a)"; }

}  // extern "C"
