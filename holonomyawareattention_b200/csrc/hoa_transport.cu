// Kernel (4): inverse transport of the attention output,
//   out_t = P_t o_t = R_t (C_{t/chunk} o_t)
// (core/attention_fast_chunked.py:171, `einsum("bhide,bhie->bhid", P, o)`),
// written as (B, T, H, d) — the (B, T, D) input of the `out` projection
// (core/attention_fast_chunked.py:172).
//
// HBM-bound: every position streams its own d x d product R_t (fp32) once.
// One warp per position; each d-row of R_t is read as float4s by 8 lanes
// (128 B contiguous per row segment) and reduced with three shuffles.
#include "hoa_common.cuh"

namespace hoa {

constexpr int kXWarps = 16;     // 16 warps x 128 positions per CTA: measured best of 4-32 warps, 32-128 positions

// y = Mat x for a compile-time d (multiple of 4): 4 rows per pass, 8 lanes per
// row with float4 loads; the passes are unrolled in groups of 4 so that 12
// loads per lane are in flight together (Mat streams from HBM once).
template <int D>
HOA_DEVICE void warp_matvec_fixed(const float* __restrict__ Mat, const float* __restrict__ x,
                                  float* __restrict__ y, int lane) {
  constexpr int NC = D / 4;                      // float4 chunks per row
  constexpr int PER = (NC + 7) / 8;              // chunks per lane and row
  const int sub = lane & 7, rsel = lane >> 3;
#pragma unroll 4
  for (int e0 = 0; e0 < D; e0 += 4) {
    const int e = e0 + rsel;
    const float4* row = reinterpret_cast<const float4*>(Mat + (long long)e * D);
    float4 m[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = sub + 8 * k;
      m[k] = c < NC ? __ldg(row + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float part = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = sub + 8 * k;
      if (c < NC) {
        const float* xv = x + 4 * c;
        part = fmaf(m[k].x, xv[0], part);
        part = fmaf(m[k].y, xv[1], part);
        part = fmaf(m[k].z, xv[2], part);
        part = fmaf(m[k].w, xv[3], part);
      }
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    if (sub == 0) y[e] = part;
  }
  __syncwarp();
}

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

// Positions per CTA: a run of consecutive positions of one chain inside one
// chunk, so that the chunk's carry C_k is read from global memory once per
// CTA (into shared memory, rows padded to d+1 words) instead of once per
// position; only R_t streams from HBM.
constexpr int kXPos = 128;

// DF: the head dim the R_t matvec is unrolled for (64, 96 or 120), or 0 for any d;
// one instantiation per width keeps each at its own register count (occupancy).
template <int DF>
__global__ void __launch_bounds__(kXWarps * 32)
out_transport_kernel(const float* __restrict__ o, const float* __restrict__ R,
                     const float* __restrict__ C, int chunk, int K, int nsub, void* out, int out_dtype,
                     int BH, int H, int T, int d) {
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = d + 1;
  float* Cs = smem;                               // [d][d+1]
  float* xo = smem + d * ld + warp * 2 * d;       // o_t, then R_t w
  float* w = xo + d;                              // C_k o_t
  const long long chain = blockIdx.x / ((long long)K * nsub);
  const int rem = (int)(blockIdx.x % ((long long)K * nsub));
  const int kc = rem / nsub, sb = rem % nsub;
  const int t_begin = kc * chunk + sb * kXPos;
  const int t_end = min(min(t_begin + kXPos, (kc + 1) * chunk), T);
  if (t_begin >= t_end) return;                   // block-uniform
  const float* Cg = C + ((long long)chain * K + kc) * d * d;
#ifdef HOA_DEBUG_BOUNDS
  const bool c_ok = HOA_IN(((long long)chain * K + kc) * d * d, d * d, (long long)BH * K * d * d);
  for (int i = threadIdx.x; i < d * d; i += blockDim.x) Cs[(i / d) * ld + i % d] = c_ok ? Cg[i] : 0.f;
#else
  for (int i = threadIdx.x; i < d * d; i += blockDim.x) Cs[(i / d) * ld + i % d] = Cg[i];
#endif
  __syncthreads();
  const int b = (int)(chain / H), h = (int)(chain % H);
  for (int t = t_begin + warp; t < t_end; t += kXWarps) {
    const long long pos = chain * T + t;
#ifdef HOA_DEBUG_BOUNDS
    // o_t, R_t and out_t inside their buffers; the position is skipped if not (warp-uniform)
    if (!(HOA_IN(pos * d, d, (long long)BH * T * d) && HOA_IN(pos * d * d, d * d, (long long)BH * T * d * d) &&
          HOA_IN((((long long)b * T + t) * H + h) * d, d, (long long)BH * T * d)))
      continue;
#endif
    for (int e = lane; e < d; e += 32) xo[e] = o[pos * d + e];
    __syncwarp();
    for (int e = lane; e < d; e += 32) {          // w = C_k o_t (rows of C_k from shared memory)
      const float* crow = Cs + e * ld;
      float acc = 0.f;
      for (int f = 0; f < d; ++f) acc = fmaf(crow[f], xo[f], acc);
      w[e] = acc;
    }
    __syncwarp();
    if constexpr (DF > 0) warp_matvec_fixed<DF>(R + pos * d * d, w, xo, lane);
    else warp_matvec(R + pos * d * d, w, xo, d, lane);
    const long long obase = (((long long)b * T + t) * H + h) * d;
    for (int e = lane; e < d; e += 32) store_elem(out, obase + e, out_dtype, xo[e]);
    __syncwarp();
  }
}

}  // namespace hoa

using namespace hoa;

extern "C" int hoa_out_transport(const float* o, const float* R, const float* C, int chunk,
                                 void* out, int out_dtype, int B, int H, int T, int d,
                                 void* stream) {
  if (!o || !R || !C || !out || B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  if (out_dtype != HOA_F32 && out_dtype != HOA_BF16) return HOA_ERR_UNSUPPORTED;
  const int K = ceil_div(T, chunk);
  const int nsub = ceil_div(min(chunk, T), kXPos);
  const long long blocks = (long long)B * H * K * nsub;
  if (blocks > 0x7fffffffLL || d > 128) return HOA_ERR_UNSUPPORTED;
  const size_t smem = (size_t)(d * (d + 1) + kXWarps * 2 * d) * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* kern = d == 96 ? out_transport_kernel<96> : d == 64 ? out_transport_kernel<64>
              : d == 120 ? out_transport_kernel<120> : out_transport_kernel<0>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  kern<<<(unsigned)blocks, kXWarps * 32, smem, s>>>(o, R, C, chunk, K, nsub, out, out_dtype, B * H, H, T, d);
  return launch_status();
}
