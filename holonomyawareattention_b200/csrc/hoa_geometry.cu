// The path products themselves, for forward(..., return_geometry=True):
//   P_t = R_t C_{t/chunk}
// (core/attention_fast_chunked.py:89-94 and the {"C": P, "H": Hol} return at
// :175-177; Hol is the carry scan's total_out).  R_t are the chunk-local
// products written by the link kernel, C_k the carries of the carry scan.
//
// Not on the hot path (the forward never materialises P): a register-tiled
// FFMA product per position.  One CTA takes up to kGeoPos positions of one
// chunk; C_k stays in shared memory, R_t is staged there per position, and a
// 16 x 16 thread grid computes the d x d result with TT x TT strided tiles
// (thread (ty, tx) owns rows ty + 16 i and columns tx + 16 j, so the writes of
// a warp are contiguous and its shared-memory reads conflict-free).
#include "hoa_common.cuh"

namespace hoa {

constexpr int kGeoPos = 16;

template <int TT>
__global__ void __launch_bounds__(256) compose_paths_kernel(const float* __restrict__ R,
                                                            const float* __restrict__ C, void* P,
                                                            int p_dtype, int T, int d, int chunk,
                                                            int K, int nsub) {
  extern __shared__ float sm[];
  const int ld = d + 1;
  float* sC = sm;               // C_k   [d][d + 1]
  float* sR = sm + d * ld;      // R_t   [d][d + 1]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int sub = blockIdx.x % nsub;
  const int k = (blockIdx.x / nsub) % K;
  const long long bh = blockIdx.x / ((long long)nsub * K);
  const int t0 = k * chunk + sub * kGeoPos;
  const int t1 = min(min(t0 + kGeoPos, (k + 1) * chunk), T);
  const int dd = d * d;
  const float* Ck = C + (bh * K + k) * (long long)dd;
  for (int i = tid; i < dd; i += 256) sC[(i / d) * ld + i % d] = Ck[i];
  for (int t = t0; t < t1; ++t) {
    const long long pos = bh * T + t;
    __syncthreads();                                   // sR free (and sC loaded)
    const float* Rt = R + pos * dd;
    for (int i = tid; i < dd; i += 256) sR[(i / d) * ld + i % d] = Rt[i];
    __syncthreads();
    float acc[TT][TT];
#pragma unroll
    for (int i = 0; i < TT; ++i)
#pragma unroll
      for (int j = 0; j < TT; ++j) acc[i][j] = 0.f;
    for (int kk = 0; kk < d; ++kk) {
      float a[TT], b[TT];
#pragma unroll
      for (int i = 0; i < TT; ++i) {
        const int row = ty + 16 * i;
        a[i] = row < d ? sR[row * ld + kk] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < TT; ++j) {
        const int col = tx + 16 * j;
        b[j] = col < d ? sC[kk * ld + col] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < TT; ++i)
#pragma unroll
        for (int j = 0; j < TT; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < TT; ++i) {
      const int row = ty + 16 * i;
      if (row >= d) continue;
#pragma unroll
      for (int j = 0; j < TT; ++j) {
        const int col = tx + 16 * j;
        if (col < d) store_elem(P, pos * dd + (long long)row * d + col, p_dtype, acc[i][j]);
      }
    }
  }
}

template <int TT>
int launch_compose_paths(const float* R, const float* C, void* P, int p_dtype, int BH, int T, int d,
                         int chunk, cudaStream_t s) {
  const int K = ceil_div(T, chunk);
  const int nsub = ceil_div(min(chunk, T), kGeoPos);
  const long long blocks = (long long)BH * K * nsub;
  if (blocks > 0x7fffffffLL) return HOA_ERR_UNSUPPORTED;
  const size_t smem = (size_t)2 * d * (d + 1) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(compose_paths_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  compose_paths_kernel<TT><<<(unsigned)blocks, 256, smem, s>>>(R, C, P, p_dtype, T, d, chunk, K, nsub);
  return launch_status();
}

}  // namespace hoa

using namespace hoa;

extern "C" int hoa_compose_paths(const float* R, const float* C, void* P, int p_dtype, int BH, int T,
                                 int d, int chunk, void* stream) {
  if (!R || !C || !P || BH < 1 || T < 1 || d < 1 || chunk < 1) return HOA_ERR_INVALID_ARG;
  if (p_dtype != HOA_F32 && p_dtype != HOA_BF16) return HOA_ERR_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tt = (d + 15) / 16;          // tile edge: rows and columns per thread
  switch (tt) {
    case 1: return launch_compose_paths<1>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 2: return launch_compose_paths<2>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 3: return launch_compose_paths<3>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 4: return launch_compose_paths<4>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 5: return launch_compose_paths<5>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 6: return launch_compose_paths<6>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 7: return launch_compose_paths<7>(R, C, P, p_dtype, BH, T, d, chunk, s);
    case 8: return launch_compose_paths<8>(R, C, P, p_dtype, BH, T, d, chunk, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}
