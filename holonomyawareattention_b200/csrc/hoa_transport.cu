// Kernel (4): inverse transport of the attention output,
//   out_t = P_t o_t = R_t (C_{t/chunk} o_t)
// (core/attention_fast_chunked.py:171, `einsum("bhide,bhie->bhid", P, o)`),
// written as (B, T, H, d) — the (B, T, D) input of the `out` projection
// (core/attention_fast_chunked.py:172).
//
// HBM-bound: every position streams its own d x d product R_t (fp32) once.
// One warp per position; each d-row is read as float4s by 8 lanes (128 B
// contiguous per row segment) and reduced with three shuffles.
#include "hoa_common.cuh"

namespace hoa {

constexpr int kXWarps = 8;

// y[e] = sum_f Mat[e][f] x[f] for e < d.  x, y in shared memory; Mat row-major in global.
HOA_DEVICE void warp_matvec(const float* __restrict__ Mat, const float* __restrict__ x,
                            float* __restrict__ y, int d, int lane) {
  const int sub = lane & 7, rsel = lane >> 3;
  if ((d & 3) == 0) {
    const int nc = d >> 2;                       // float4 chunks per row
    for (int e0 = 0; e0 < d; e0 += 4) {
      const int e = e0 + rsel;
      float part = 0.f;
      if (e < d) {
        const float4* row = reinterpret_cast<const float4*>(Mat + (long long)e * d);
        for (int c = sub; c < nc; c += 8) {
          const float4 m = __ldg(row + c);
          const float* xv = x + 4 * c;
          part = fmaf(m.x, xv[0], part);
          part = fmaf(m.y, xv[1], part);
          part = fmaf(m.z, xv[2], part);
          part = fmaf(m.w, xv[3], part);
        }
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      if (sub == 0 && e < d) y[e] = part;
    }
  } else {
    for (int e0 = 0; e0 < d; e0 += 4) {
      const int e = e0 + rsel;
      float part = 0.f;
      if (e < d)
        for (int f = sub; f < d; f += 8) part = fmaf(__ldg(Mat + (long long)e * d + f), x[f], part);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      part += __shfl_xor_sync(0xffffffffu, part, 4);
      if (sub == 0 && e < d) y[e] = part;
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kXWarps * 32)
out_transport_kernel(const float* __restrict__ o, const float* __restrict__ R,
                     const float* __restrict__ C, int chunk, int K, void* out, int out_dtype,
                     int H, int T, int d, long long npos) {
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* xo = smem + warp * 2 * d;        // o_t, then R_t w
  float* w = xo + d;                      // C_k o_t
  const long long pos = (long long)blockIdx.x * kXWarps + warp;
  if (pos >= npos) return;
  const long long chain = pos / T;
  const int t = (int)(pos % T);
  const int b = (int)(chain / H), h = (int)(chain % H);
  for (int e = lane; e < d; e += 32) xo[e] = o[pos * d + e];
  __syncwarp();
  warp_matvec(C + ((long long)chain * K + t / chunk) * d * d, xo, w, d, lane);
  warp_matvec(R + pos * d * d, w, xo, d, lane);
  const long long obase = (((long long)b * T + t) * H + h) * d;
  for (int e = lane; e < d; e += 32) store_elem(out, obase + e, out_dtype, xo[e]);
}

}  // namespace hoa

using namespace hoa;

extern "C" int hoa_out_transport(const float* o, const float* R, const float* C, int chunk,
                                 void* out, int out_dtype, int B, int H, int T, int d,
                                 void* stream) {
  if (!o || !R || !C || !out || B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  if (out_dtype != HOA_F32 && out_dtype != HOA_BF16) return HOA_ERR_UNSUPPORTED;
  const long long npos = (long long)B * H * T;
  const size_t smem = (size_t)kXWarps * 2 * d * sizeof(float);
  const long long blocks = (npos + kXWarps - 1) / kXWarps;
  if (blocks > 0x7fffffffLL) return HOA_ERR_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  out_transport_kernel<<<(unsigned)blocks, kXWarps * 32, smem, s>>>(
      o, R, C, chunk, ceil_div(T, chunk), out, out_dtype, H, T, d, npos);
  return launch_status();
}
