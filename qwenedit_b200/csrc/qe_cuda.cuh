// Device-side helpers shared by the libqeb200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "qe_common.h"

namespace qe {

// Number of SMs of the current device (cached per device).
int sm_count();

// Turn a launch / runtime error into a status + message.
inline int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return QE_OK;
  return fail(QE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 128-bit streaming load that bypasses L1 allocation (each byte of a page copy is read exactly once).
__device__ __forceinline__ int4 ld_stream(const int4 *p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 128-bit store with evict-first L2 policy (the destination is not re-read by this kernel).
__device__ __forceinline__ void st_stream(int4 *p, int4 v) {
  asm volatile("st.global.cs.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace qe
