// Shared helpers for the path-ordered geometric attention kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/hoa.h"

#define HOA_DEVICE __device__ __forceinline__

namespace hoa {

// element loads / stores for the two activation types the ABI accepts
HOA_DEVICE float load_elem(const void* p, long long i, int dtype) {
  if (dtype == HOA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

HOA_DEVICE void store_elem(void* p, long long i, int dtype, float v) {
  if (dtype == HOA_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// Record the first device-side failure so that the host can read it later.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HOA_OK : HOA_ERR_LAUNCH;
}

// Smallest supported padded head dimension >= d, or 0.
inline int padded_dim(int d) {
  static const int dims[] = {8, 16, 32, 48, 64, 96, 120};
  for (int p : dims)
    if (d <= p) return p;
  return 0;
}

}  // namespace hoa
