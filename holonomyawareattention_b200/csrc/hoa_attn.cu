// Kernel (3), fp32 path: causal online-softmax attention over the transported
// q^, k^, v^, written as the normalised o (fp32, (B*H, T, d)); the inverse
// transport (kernel 4) follows in hoa_transport.cu.
//
// Reference semantics (SiddhiMali/HolonomyAwareAttention):
//   scores q^_i . k^_j * scale, tril mask with finfo.min, online softmax,
//   o / l.clamp_min(1e-20)                    core/attention_fast_chunked.py:119-168
//
// SIMT variant: q^/k^/v^ in fp32 (or bf16), every product and the softmax in
// fp32, so fp32 inputs keep fp32 accuracy.  One CTA per (64-query tile, chain).
#include "hoa_common.cuh"

namespace hoa {

constexpr int kBQ = 64, kBK = 64, kAttnThreads = 256;
constexpr int kLDT = kBQ + 4;   // row stride of the transposed tiles (keeps float4 alignment)

template <int DA> struct AttnCfg {
  static constexpr int CPT = DA / 16;    // output columns per thread
  static constexpr size_t kQt = (size_t)DA * kLDT, kKt = (size_t)DA * kLDT, kVs = (size_t)kBK * DA,
                          kPt = (size_t)kBK * kLDT;
  static constexpr size_t kSmem = (kQt + kKt + kVs + kPt) * sizeof(float);
};

struct AttnArgs {
  const void* qh; const void* kh; const void* vh; int hat_dtype;
  float* o; float scale;
  int Tq, Tk, q_offset, d;   // query rows are global positions q_offset .. q_offset + Tq - 1
};

template <int N>
HOA_DEVICE void lds4(const float* __restrict__ p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      float4 t = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  } else if constexpr (N % 2 == 0) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      float2 t = reinterpret_cast<const float2*>(p)[i];
      v[2 * i] = t.x; v[2 * i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = p[i];
  }
}

template <int DA>
__global__ void __launch_bounds__(kAttnThreads) attn_fwd_simt_kernel(AttnArgs p) {
  using Cf = AttnCfg<DA>;
  constexpr int CPT = Cf::CPT;
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;                 // [DA][kLDT]   q^ transposed
  float* Kt = Qt + Cf::kQt;         // [DA][kLDT]   k^ transposed
  float* Vs = Kt + Cf::kKt;         // [kBK][DA]    v^ row-major
  float* Pt = Vs + Cf::kVs;         // [kBK][kLDT]  probabilities transposed

  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int r0 = ty * 4, c0 = tx * 4;
  const int chain = blockIdx.y;
  const int qtile = gridDim.x - 1 - blockIdx.x;     // heaviest causal tiles first
  const int q0 = qtile * kBQ;                        // local row of this tile
  const int d = p.d, Tq = p.Tq, Tk = p.Tk;
  const int gq0 = p.q_offset + q0;                   // its global position
  const int nkt = min((gq0 + kBQ - 1) / kBK, (Tk - 1) / kBK) + 1;
  const long long qbase = (long long)chain * Tq * d;
  const long long kbase = (long long)chain * Tk * d;
  const long long BH = gridDim.y;
  // (debug build) the query tile inside q^; a tile outside is read as zeros
  const bool q_ok = HOA_IN(qbase + (long long)q0 * d, (long long)min(kBQ, Tq - q0) * d, BH * Tq * d);

  for (int i = tid; i < kBQ * DA; i += kAttnThreads) {
    const int r = i / DA, e = i % DA;
    const int t = q0 + r;
    Qt[e * kLDT + r] = (t < Tq && e < d && q_ok) ? load_elem(p.qh, qbase + (long long)t * d + e, p.hat_dtype)
                                                 : 0.f;
  }

  float mrow[4], lrow[4], o[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) o[i][j] = 0.f;
  }

  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * kBK;
    __syncthreads();
    const bool kv_ok = HOA_IN(kbase + (long long)k0 * d, (long long)min(kBK, Tk - k0) * d, BH * Tk * d);
    for (int i = tid; i < kBK * DA; i += kAttnThreads) {
      const int r = i / DA, e = i % DA;
      const int t = k0 + r;
      const bool ok = t < Tk && e < d && kv_ok;
      const long long off = kbase + (long long)t * d + e;
      Kt[e * kLDT + r] = ok ? load_elem(p.kh, off, p.hat_dtype) : 0.f;
      Vs[r * DA + e] = ok ? load_elem(p.vh, off, p.hat_dtype) : 0.f;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int e = 0; e < DA; ++e) {
      float qa[4], kb[4];
      lds4<4>(Qt + e * kLDT + r0, qa);
      lds4<4>(Kt + e * kLDT + c0, kb);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], kb[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = gq0 + r0 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + c0 + j;
        s[i][j] = (kj <= qi && kj < Tk) ? s[i][j] * p.scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(mrow[i], mx);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      const float corr = expf(mrow[i] - mref);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = expf(s[i][j] - mref);
        s[i][j] = pv;
        rs += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      lrow[i] = lrow[i] * corr + rs;
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < CPT; ++j) o[i][j] *= corr;
#pragma unroll
      for (int j = 0; j < 4; ++j) Pt[(c0 + j) * kLDT + r0 + i] = s[i][j];
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < kBK; ++j) {
      float pa[4], vb[CPT];
      lds4<4>(Pt + j * kLDT + r0, pa);
      lds4<CPT>(Vs + j * DA + tx * CPT, vb);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < CPT; ++jj) o[i][jj] = fmaf(pa[i], vb[jj], o[i][jj]);
    }
  }

  // ---- epilogue: o / l ------------------------------------------------------
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = q0 + r0 + i;
    if (t >= Tq || !HOA_IN(((long long)chain * Tq + t) * d, d, BH * Tq * d)) continue;
    const float inv = 1.f / fmaxf(lrow[i], 1e-20f);
    float* orow = p.o + ((long long)chain * Tq + t) * d;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int e = tx * CPT + j;
      if (e < d) orow[e] = o[i][j] * inv;
    }
  }
}

template <int DA>
int launch_attn(const AttnArgs& a, int BH, cudaStream_t s) {
  using Cf = AttnCfg<DA>;
  if (cudaFuncSetAttribute(attn_fwd_simt_kernel<DA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)Cf::kSmem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  dim3 grid((unsigned)ceil_div(a.Tq, kBQ), (unsigned)BH);
  attn_fwd_simt_kernel<DA><<<grid, kAttnThreads, Cf::kSmem, s>>>(a);
  return launch_status();
}

}  // namespace hoa

using namespace hoa;

extern "C" int hoa_attn_fwd(const void* qh, const void* kh, const void* vh, int hat_dtype,
                            float* o, float softmax_scale, int BH, int Tq, int Tk, int q_offset,
                            int d, void* stream) {
  if (!qh || !kh || !vh || !o || BH < 1 || Tq < 1 || Tk < 1 || d < 1) return HOA_ERR_INVALID_ARG;
  if (q_offset < 0 || q_offset + Tq > Tk) return HOA_ERR_INVALID_ARG;
  if (hat_dtype != HOA_F32 && hat_dtype != HOA_BF16) return HOA_ERR_UNSUPPORTED;
  if (BH > 65535) return HOA_ERR_UNSUPPORTED;
  AttnArgs a{qh, kh, vh, hat_dtype, o, softmax_scale, Tq, Tk, q_offset, d};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int da = ((d + 15) / 16) * 16;
  switch (da) {
    case 16: return launch_attn<16>(a, BH, s);
    case 32: return launch_attn<32>(a, BH, s);
    case 48: return launch_attn<48>(a, BH, s);
    case 64: return launch_attn<64>(a, BH, s);
    case 80: return launch_attn<80>(a, BH, s);
    case 96: return launch_attn<96>(a, BH, s);
    case 112: return launch_attn<112>(a, BH, s);
    case 128: return launch_attn<128>(a, BH, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}
