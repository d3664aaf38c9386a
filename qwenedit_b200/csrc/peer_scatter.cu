// Head-sharded prefix pools across the GPUs of one node: the append that scatters new K/V heads to their
// owners over NVLink, and the CUDA IPC plumbing that maps the owners' pools into each rank.
//
// QwenEdit keeps a session's whole-prefix K/V on one GPU and turns the pool off under tensor or sequence
// parallelism (multi_turn/pipeline/encoding.py:214-220: "TP/SP shard or exchange it"). Here each rank r of an
// n-GPU group owns heads [r H/n, (r+1) H/n) of every pooled token; all ranks run the same prefix-index
// decisions, so a token has the same slot on every rank. Gathers stay local (each rank reads its own heads).
// When a rank holds new K/V for a slice of the tokens with all heads (sequence parallel, before the
// all-to-all), qe_append_scatter writes head slice r of each of its rows straight into rank r's pool through
// the peer mapping: the all-to-all and the pool append are one kernel, and the bytes cross NVLink once.
//
// No kernel here waits on another rank: visibility of the peer writes is the caller's stream-ordered barrier
// after the launch (an NCCL all-reduce on the same stream), never a spin on a flag.
#include <algorithm>
#include <cstdint>
#include <cstring>

#include "qe_cuda.cuh"
#include "qeb200.h"

namespace qe {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kScatterThreads = 256;
constexpr int kScatterUnroll = 16;  // vectors per lane in flight: a 8 KiB row per warp pass

struct ScatterParams {
  char *peer[kMaxPeers];  // every rank's pool base, rank order (this rank's own pool included)
  int64_t outer, inner;   // pool plane geometry, identical on every rank
  int32_t per_outer;
  int32_t n_peers;
  const char *src;
  int64_t src_outer, src_inner;
  int32_t src_per_outer;
  int32_t n_planes;
  int64_t pool_rows, n_tokens;
  int64_t slice_vecs;  // 16-byte vectors of one rank's head slice of a row
  const int64_t *slots;
  int32_t *err;
};

// One warp per (plane, token) source row: the whole row (all heads) is loaded, then vector v goes to rank
// v / slice_vecs at offset v % slice_vecs of that rank's row `slot`.
__global__ void __launch_bounds__(kScatterThreads) append_scatter_kernel(ScatterParams p) {
  __shared__ char *peer[kMaxPeers];  // indexed by a runtime rank: kept out of the parameter space
  if (threadIdx.x < kMaxPeers) peer[threadIdx.x] = p.peer[threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = int64_t(threadIdx.x >> 5) * gridDim.x + blockIdx.x;
  const int64_t nwarps = int64_t(gridDim.x) * (kScatterThreads / 32);
  const int64_t items = int64_t(p.n_planes) * p.n_tokens;
  const int64_t row_vecs = p.slice_vecs * p.n_peers;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int32_t plane = int32_t(it / p.n_tokens);
    const int64_t t = it - int64_t(plane) * p.n_tokens;
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0 || slot >= p.pool_rows) {
      if (lane == 0) atomicOr(p.err, 1);
      continue;
    }
    const int4 *src = reinterpret_cast<const int4 *>(p.src + int64_t(plane / p.src_per_outer) * p.src_outer +
                                                     int64_t(plane % p.src_per_outer) * p.src_inner) +
                      t * row_vecs;
    const int64_t dst_off = int64_t(plane / p.per_outer) * p.outer + int64_t(plane % p.per_outer) * p.inner +
                            slot * (p.slice_vecs << 4);
    for (int64_t base = 0; base < row_vecs; base += 32 * kScatterUnroll) {
      int4 buf[kScatterUnroll];
#pragma unroll
      for (int u = 0; u < kScatterUnroll; ++u) {
        const int64_t v = base + lane + 32 * u;
        if (v < row_vecs) buf[u] = ld_stream(src + v);
      }
      // (rank, offset) of vector base + lane, then advanced by 32 per step (slice_vecs may be below 32)
      int64_t r = (base + lane) / p.slice_vecs;
      int64_t w = (base + lane) - r * p.slice_vecs;
#pragma unroll
      for (int u = 0; u < kScatterUnroll; ++u) {
        if (base + lane + 32 * u < row_vecs) {
          int4 *dst = reinterpret_cast<int4 *>(peer[r] + dst_off) + w;
          *dst = buf[u];
        }
        w += 32;
        while (w >= p.slice_vecs) {
          w -= p.slice_vecs;
          ++r;
        }
        if (r >= p.n_peers) break;  // past the row (later u are out of range too)
      }
    }
  }
}

}  // namespace
}  // namespace qe

using qe::fail;

extern "C" {

int qe_ipc_alloc(int64_t bytes, void **ptr, uint8_t *handle) {
  QE_CHECK_ARG(bytes > 0 && ptr && handle, "qe_ipc_alloc: bad arguments");
  *ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, size_t(bytes));
  if (e != cudaSuccess) return qe::cuda_status(e, "qe_ipc_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return qe::cuda_status(e, "qe_ipc_alloc: cudaIpcGetMemHandle");
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return qe::ok();
}

int qe_ipc_free(void *ptr) {
  QE_CHECK_ARG(ptr, "qe_ipc_free: null pointer");
  int s = qe::cuda_status(cudaFree(ptr), "qe_ipc_free");
  return s ? s : qe::ok();
}

int qe_ipc_open(const uint8_t *handle, void **ptr) {
  QE_CHECK_ARG(handle && ptr, "qe_ipc_open: bad arguments");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return qe::cuda_status(e, "qe_ipc_open: cudaIpcOpenMemHandle");
  *ptr = p;
  return qe::ok();
}

int qe_ipc_close(void *ptr) {
  QE_CHECK_ARG(ptr, "qe_ipc_close: null pointer");
  int s = qe::cuda_status(cudaIpcCloseMemHandle(ptr), "qe_ipc_close");
  return s ? s : qe::ok();
}

int qe_append_scatter(const void *const *peer_pools, int32_t n_peers, qe_planes pool, int64_t pool_rows,
                      qe_planes src, int32_t n_planes, int64_t slice_bytes, const int64_t *slots, int64_t n_tokens,
                      int32_t *err_flag, void *stream) {
  QE_CHECK_ARG(peer_pools && n_peers >= 1 && n_peers <= qe::kMaxPeers, "qe_append_scatter: 1..8 peer pools");
  QE_CHECK_ARG(n_planes >= 1 && pool_rows >= 1 && n_tokens >= 0 && err_flag, "qe_append_scatter: bad sizes");
  QE_CHECK_ARG(slice_bytes > 0 && slice_bytes % 16 == 0, "qe_append_scatter: slice_bytes must be a multiple of 16");
  QE_CHECK_ARG(pool.planes_inner >= 1 && src.planes_inner >= 1, "qe_append_scatter: planes_inner must be >= 1");
  QE_CHECK_ARG(pool.outer_stride % 16 == 0 && pool.inner_stride % 16 == 0 && src.outer_stride % 16 == 0 &&
                   src.inner_stride % 16 == 0,
               "qe_append_scatter: plane strides must be multiples of 16 bytes");
  if (n_tokens == 0) return qe::ok();
  QE_CHECK_ARG(src.base && qe::aligned16(src.base), "qe_append_scatter: source must be 16-byte aligned");
  QE_CHECK_ARG(slots, "qe_append_scatter: null slots");
  qe::ScatterParams p{};
  for (int r = 0; r < n_peers; ++r) {
    QE_CHECK_ARG(peer_pools[r] && qe::aligned16(peer_pools[r]), "qe_append_scatter: peer pool %d null or unaligned",
                 r);
    p.peer[r] = static_cast<char *>(const_cast<void *>(peer_pools[r]));
  }
  p.outer = pool.outer_stride;
  p.inner = pool.inner_stride;
  p.per_outer = pool.planes_inner;
  p.n_peers = n_peers;
  p.src = static_cast<const char *>(src.base);
  p.src_outer = src.outer_stride;
  p.src_inner = src.inner_stride;
  p.src_per_outer = src.planes_inner;
  p.n_planes = n_planes;
  p.pool_rows = pool_rows;
  p.n_tokens = n_tokens;
  p.slice_vecs = slice_bytes / 16;
  p.slots = slots;
  p.err = err_flag;
  const int64_t items = int64_t(n_planes) * n_tokens;
  const int64_t warps_per_block = qe::kScatterThreads / 32;
  int64_t blocks = (items + warps_per_block - 1) / warps_per_block;
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(qe::sm_count()) * 8));
  qe::append_scatter_kernel<<<dim3(unsigned(blocks)), dim3(qe::kScatterThreads), 0,
                              static_cast<cudaStream_t>(stream)>>>(p);
  int s = qe::cuda_status(cudaGetLastError(), "qe_append_scatter launch");
  return s ? s : qe::ok();
}

}  // extern "C"
