// The module's general forms (core/attention.py:69-195), beside the causal
// tril hot path: any attention mask, the wrap pairs of the arc transport, the
// inert ablation.  All fp32.
//
// * hoa_attn_general_fwd: softmax over ALL keys of the chain, masked entries
//   at -FLT_MAX (finfo.min, core/attention_fast_chunked.py:142-148), the
//   pairs j <= i scored and weighted with (k^_j, v^_j) and the wrap pairs
//   j > i, when given, with (kw_j, vw_j) = (Hol k^_j, Hol v^_j): the arc
//   transport j -> i through the closing edge is P_i Hol P_j^T
//   (core/attention.py:156-165).
// * hoa_chain_matvec: y_t = M x_t (or M^T x_t) with one d x d matrix per chain
//   (Hol k^, Hol v^).
// * hoa_apply_paths: y_t = P_t x_t or P_t^T x_t with P_t = R_t C_{t/chunk}
//   (the inert ablation's transports q~ = P q and out = P^T o,
//   core/attention.py:166-169).
#include <cfloat>

#include "hoa_common.cuh"

namespace hoa {

// ---------------------------------------------------------------------------
// attention over all keys
// ---------------------------------------------------------------------------
constexpr int kGQ = 64, kGK = 64, kGThreads = 256;
constexpr int kGLD = kGQ + 4;

template <int DA> struct GenCfg {
  static constexpr int CPT = DA / 16;
  static constexpr size_t kT = (size_t)DA * kGLD, kV = (size_t)kGK * DA, kP = (size_t)kGK * kGLD;
  static constexpr size_t kSmem = (3 * kT + 2 * kV + 2 * kP) * sizeof(float);
};

struct GenArgs {
  const float* qh; const float* kh; const float* vh; const float* kw; const float* vw;
  const uint8_t* mask;   // (T, T) row-major, nonzero = allowed; nullptr = all allowed
  float* o; float scale; int T, d;
};

template <int DA>
__global__ void __launch_bounds__(kGThreads) attn_general_kernel(GenArgs p) {
  using Cf = GenCfg<DA>;
  constexpr int CPT = Cf::CPT;
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;                  // [DA][kGLD]
  float* Kb = Qt + Cf::kT;           // [DA][kGLD]  k^ transposed
  float* Kw = Kb + Cf::kT;           // [DA][kGLD]  wrap keys transposed
  float* Vb = Kw + Cf::kT;           // [kGK][DA]
  float* Vw = Vb + Cf::kV;           // [kGK][DA]
  float* Pb = Vw + Cf::kV;           // [kGK][kGLD] weights of the pairs j <= i
  float* Pw = Pb + Cf::kP;           // [kGK][kGLD] weights of the wrap pairs

  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int r0 = ty * 4, c0 = tx * 4;
  const int chain = blockIdx.y;
  const int q0 = blockIdx.x * kGQ;
  const int d = p.d, T = p.T;
  const bool wrap = p.kw != nullptr;
  const long long base = (long long)chain * T * d;

  for (int i = tid; i < kGQ * DA; i += kGThreads) {
    const int r = i / DA, e = i % DA;
    const int t = q0 + r;
    Qt[e * kGLD + r] = (t < T && e < d) ? p.qh[base + (long long)t * d + e] : 0.f;
  }
  float mrow[4], lrow[4], o[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) o[i][j] = 0.f;
  }

  const int nkt = (T + kGK - 1) / kGK;
  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * kGK;
    // which key sets this tile needs: j <= i for every pair (below the
    // diagonal), j > i for every pair (above it), or both
    const bool below = k0 + kGK - 1 <= q0;
    const bool above = k0 >= q0 + kGQ;
    const bool use_b = !wrap || !above;
    const bool use_w = wrap && !below;
    __syncthreads();
    for (int i = tid; i < kGK * DA; i += kGThreads) {
      const int r = i / DA, e = i % DA;
      const int t = k0 + r;
      const bool ok = t < T && e < d;
      const long long off = base + (long long)t * d + e;
      if (use_b) {
        Kb[e * kGLD + r] = ok ? p.kh[off] : 0.f;
        Vb[r * DA + e] = ok ? p.vh[off] : 0.f;
      }
      if (use_w) {
        Kw[e * kGLD + r] = ok ? p.kw[off] : 0.f;
        Vw[r * DA + e] = ok ? p.vw[off] : 0.f;
      }
    }
    __syncthreads();

    float sb[4][4], sw[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) { sb[i][j] = 0.f; sw[i][j] = 0.f; }
    if (use_b) {
#pragma unroll 4
      for (int e = 0; e < DA; ++e) {
        const float4 qa = *reinterpret_cast<const float4*>(Qt + e * kGLD + r0);
        const float4 kb = *reinterpret_cast<const float4*>(Kb + e * kGLD + c0);
        const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) sb[i][j] = fmaf(qv[i], kv[j], sb[i][j]);
      }
    }
    if (use_w) {
#pragma unroll 4
      for (int e = 0; e < DA; ++e) {
        const float4 qa = *reinterpret_cast<const float4*>(Qt + e * kGLD + r0);
        const float4 kb = *reinterpret_cast<const float4*>(Kw + e * kGLD + c0);
        const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) sw[i][j] = fmaf(qv[i], kv[j], sw[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qi = q0 + r0 + i;
      float s[4];
      bool isb[4];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kj = k0 + c0 + j;
        isb[j] = !wrap || kj <= qi;
        float v = (isb[j] ? sb[i][j] : sw[i][j]) * p.scale;
        if (kj >= T) {
          v = -INFINITY;                                          // no such key
        } else if (p.mask != nullptr && qi < T && p.mask[(long long)qi * T + kj] == 0) {
          v = -FLT_MAX;                                           // masked: finfo.min
        }
        s[j] = v;
        mx = fmaxf(mx, v);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(mrow[i], mx);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      const float corr = expf(mrow[i] - mref);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = expf(s[j] - mref);
        s[j] = pv;
        rs += pv;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      lrow[i] = lrow[i] * corr + rs;
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < CPT; ++j) o[i][j] *= corr;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        Pb[(c0 + j) * kGLD + r0 + i] = isb[j] ? s[j] : 0.f;
        Pw[(c0 + j) * kGLD + r0 + i] = isb[j] ? 0.f : s[j];
      }
    }
    __syncthreads();
    if (use_b) {
#pragma unroll 4
      for (int j = 0; j < kGK; ++j) {
        const float4 pa = *reinterpret_cast<const float4*>(Pb + j * kGLD + r0);
        const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
        for (int jj = 0; jj < CPT; ++jj) {
          const float vb = Vb[j * DA + tx * CPT + jj];
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i][jj] = fmaf(pv[i], vb, o[i][jj]);
        }
      }
    }
    if (use_w) {
#pragma unroll 4
      for (int j = 0; j < kGK; ++j) {
        const float4 pa = *reinterpret_cast<const float4*>(Pw + j * kGLD + r0);
        const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
        for (int jj = 0; jj < CPT; ++jj) {
          const float vw = Vw[j * DA + tx * CPT + jj];
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i][jj] = fmaf(pv[i], vw, o[i][jj]);
        }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = q0 + r0 + i;
    if (t >= T) continue;
    const float inv = 1.f / fmaxf(lrow[i], 1e-20f);
    float* orow = p.o + base + (long long)t * d;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int e = tx * CPT + j;
      if (e < d) orow[e] = o[i][j] * inv;
    }
  }
}

template <int DA>
int launch_attn_general(const GenArgs& a, int BH, cudaStream_t s) {
  using Cf = GenCfg<DA>;
  if (cudaFuncSetAttribute(attn_general_kernel<DA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)Cf::kSmem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  dim3 grid((unsigned)ceil_div(a.T, kGQ), (unsigned)BH);
  attn_general_kernel<DA><<<grid, kGThreads, Cf::kSmem, s>>>(a);
  return launch_status();
}

// ---------------------------------------------------------------------------
// per-chain and per-position matrix-vector products
// ---------------------------------------------------------------------------
constexpr int kMvWarps = 8, kMvPos = 64;

// z[e] = sum_f A[e][f] x[f] (tr = false) or sum_f A[f][e] x[f] (tr = true), A in
// shared memory with row stride d + 1 (odd for even d: lanes e hit distinct banks
// either way); lane e computes outputs e, e + 32, ...
HOA_DEVICE void smem_matvec(const float* A, const float* x, float* z, int d, bool tr, int lane) {
  const int ld = d + 1;
  for (int e = lane; e < d; e += 32) {
    float acc = 0.f;
    if (tr) {
      for (int f = 0; f < d; ++f) acc = fmaf(A[f * ld + e], x[f], acc);
    } else {
      for (int f = 0; f < d; ++f) acc = fmaf(A[e * ld + f], x[f], acc);
    }
    z[e] = acc;
  }
  __syncwarp();
}

// y_t = M x_t (tr = 0) or M^T x_t, M (d x d) per chain.  One CTA per
// (chain, run of kMvPos positions), a warp per position.
__global__ void __launch_bounds__(kMvWarps * 32) chain_matvec_kernel(const float* __restrict__ x,
                                                                     const float* __restrict__ M,
                                                                     float* __restrict__ y, int tr,
                                                                     int T, int d, int nrun) {
  extern __shared__ float sm[];
  const int ld = d + 1;
  float* sM = sm;
  float* sx = sm + d * ld + (threadIdx.x >> 5) * 2 * d;
  float* sz = sx + d;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long bh = blockIdx.x / nrun;
  const int t0 = (blockIdx.x % nrun) * kMvPos, t1 = min(t0 + kMvPos, T);
  const float* Mb = M + bh * (long long)d * d;
  for (int i = threadIdx.x; i < d * d; i += blockDim.x) sM[(i / d) * ld + i % d] = Mb[i];
  __syncthreads();
  for (int t = t0 + warp; t < t1; t += kMvWarps) {
    const long long off = (bh * T + t) * (long long)d;
    for (int e = lane; e < d; e += 32) sx[e] = x[off + e];
    __syncwarp();
    smem_matvec(sM, sx, sz, d, tr != 0, lane);
    for (int e = lane; e < d; e += 32) y[off + e] = sz[e];
    __syncwarp();
  }
}

// y_t = P_t x_t = R_t (C_k x_t) (tr = 0) or P_t^T x_t = C_k^T (R_t^T x_t) (tr = 1),
// k = t / chunk.  One CTA per (chain, chunk, run of kMvPos positions), C_k in
// shared memory, R_t streamed row by row (coalesced across lanes).
__global__ void __launch_bounds__(kMvWarps * 32) apply_paths_kernel(
    const float* __restrict__ x, const float* __restrict__ R, const float* __restrict__ C, int chunk,
    int K, int nsub, float* __restrict__ y, int tr, int T, int d) {
  extern __shared__ float sm[];
  const int ld = d + 1;
  float* sC = sm;
  float* sx = sm + d * ld + (threadIdx.x >> 5) * 2 * d;
  float* sz = sx + d;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = blockIdx.x % nsub;
  const int k = (blockIdx.x / nsub) % K;
  const long long bh = blockIdx.x / ((long long)nsub * K);
  const int t0 = k * chunk + sub * kMvPos;
  const int t1 = min(min(t0 + kMvPos, (k + 1) * chunk), T);
  const float* Ck = C + (bh * K + k) * (long long)d * d;
  for (int i = threadIdx.x; i < d * d; i += blockDim.x) sC[(i / d) * ld + i % d] = Ck[i];
  __syncthreads();
  for (int t = t0 + warp; t < t1; t += kMvWarps) {
    const long long pos = bh * T + t;
    const float* Rt = R + pos * (long long)d * d;
    for (int e = lane; e < d; e += 32) sx[e] = x[pos * d + e];
    __syncwarp();
    if (!tr) {
      smem_matvec(sC, sx, sz, d, false, lane);              // z = C_k x
      for (int e = 0; e < d; ++e) {                         // y_e = sum_f R[e][f] z_f
        float part = 0.f;
        for (int f = lane; f < d; f += 32) part = fmaf(Rt[(long long)e * d + f], sz[f], part);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) sx[e] = part;                        // x no longer needed
      }
      __syncwarp();
      for (int e = lane; e < d; e += 32) y[pos * d + e] = sx[e];
    } else {
      float zl[4] = {0.f, 0.f, 0.f, 0.f};                   // z_e = sum_f R[f][e] x_f, e = lane + 32 i
      for (int f = 0; f < d; ++f) {
        const float xf = sx[f];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = lane + 32 * i;
          if (e < d) zl[i] = fmaf(Rt[(long long)f * d + e], xf, zl[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (lane + 32 * i < d) sz[lane + 32 * i] = zl[i];
      __syncwarp();
      smem_matvec(sC, sz, sx, d, true, lane);               // y = C_k^T z
      for (int e = lane; e < d; e += 32) y[pos * d + e] = sx[e];
    }
    __syncwarp();
  }
}

}  // namespace hoa

using namespace hoa;

extern "C" int hoa_attn_general_fwd(const float* qh, const float* kh, const float* vh,
                                    const float* kw, const float* vw, const uint8_t* mask,
                                    float* o, float softmax_scale, int BH, int T, int d,
                                    void* stream) {
  if (!qh || !kh || !vh || !o || BH < 1 || T < 1 || d < 1) return HOA_ERR_INVALID_ARG;
  if ((kw == nullptr) != (vw == nullptr)) return HOA_ERR_INVALID_ARG;
  if (BH > 65535 || d > 128) return HOA_ERR_UNSUPPORTED;
  GenArgs a{qh, kh, vh, kw, vw, mask, o, softmax_scale, T, d};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int da = ((d + 15) / 16) * 16;
  switch (da) {
    case 16: return launch_attn_general<16>(a, BH, s);
    case 32: return launch_attn_general<32>(a, BH, s);
    case 48: return launch_attn_general<48>(a, BH, s);
    case 64: return launch_attn_general<64>(a, BH, s);
    case 80: return launch_attn_general<80>(a, BH, s);
    case 96: return launch_attn_general<96>(a, BH, s);
    case 112: return launch_attn_general<112>(a, BH, s);
    case 128: return launch_attn_general<128>(a, BH, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

extern "C" int hoa_chain_matvec(const float* x, const float* M, float* y, int transpose, int BH, int T,
                                int d, void* stream) {
  if (!x || !M || !y || BH < 1 || T < 1 || d < 1) return HOA_ERR_INVALID_ARG;
  if (d > 128) return HOA_ERR_UNSUPPORTED;
  const int nrun = ceil_div(T, kMvPos);
  const long long blocks = (long long)BH * nrun;
  if (blocks > 0x7fffffffLL) return HOA_ERR_UNSUPPORTED;
  const size_t smem = (size_t)(d * (d + 1) + kMvWarps * 2 * d) * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(chain_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return HOA_ERR_LAUNCH;
  chain_matvec_kernel<<<(unsigned)blocks, kMvWarps * 32, smem, s>>>(x, M, y, transpose, T, d, nrun);
  return launch_status();
}

extern "C" int hoa_apply_paths(const float* x, const float* R, const float* C, int chunk, float* y,
                               int transpose, int BH, int T, int d, void* stream) {
  if (!x || !R || !C || !y || BH < 1 || T < 1 || d < 1 || chunk < 1) return HOA_ERR_INVALID_ARG;
  if (d > 128) return HOA_ERR_UNSUPPORTED;
  const int K = ceil_div(T, chunk);
  const int nsub = ceil_div(min(chunk, T), kMvPos);
  const long long blocks = (long long)BH * K * nsub;
  if (blocks > 0x7fffffffLL) return HOA_ERR_UNSUPPORTED;
  const size_t smem = (size_t)(d * (d + 1) + kMvWarps * 2 * d) * sizeof(float);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(apply_paths_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return HOA_ERR_LAUNCH;
  apply_paths_kernel<<<(unsigned)blocks, kMvWarps * 32, smem, s>>>(x, R, C, chunk, K, nsub, y, transpose,
                                                                    T, d);
  return launch_status();
}
