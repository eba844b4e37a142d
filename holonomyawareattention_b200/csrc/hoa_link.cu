// Kernels (1) and (2): link rotations G_t = expm(skew(edge_scale * a_t)) and the
// ordered prefix composition P_{t+1} = G_t P_t, chunked so that every
// (chain, chunk) unit runs independently, then joined by a carry scan.
//
// Reference semantics (SiddhiMali/HolonomyAwareAttention):
//   skew_from_vec            core/utils.py:4-27   (row-major strict upper triangle, A[j,i] = -A[i,j])
//   so_exp = matrix_exp      core/utils.py:30-52
//   a_all * edge_scale       core/attention_fast_chunked.py:77
//   prefix loop              core/attention_fast_chunked.py:89-94
//   transport q^ = P^T q     core/attention_fast_chunked.py:108-110
//
// Arithmetic is fp32 throughout (FFMA).  Each unit keeps four d x d matrices
// in shared memory: the running local product R, the generator A (later G^T),
// and two operand buffers.  Each thread owns a TM x TN tile of every product.
#include <atomic>

#include "hoa_sm100.cuh"

namespace hoa {

// ---------------------------------------------------------------------------
// Degree-8 Taylor polynomial of exp(A) in three matrix products
// (Bader, Blanes & Casas, Mathematics 7 (2019) 1174, the 3-product T8 scheme):
//   A2 = A^2
//   A4 = A2 (x1 A + x2 A2)
//   A8 = (x3 A2 + A4)(x4 I + x5 A + x6 A2 + x7 A4)
//   T8 = I + A + y2 A2 + A8            == sum_{k=0..8} A^k / k!   (exact identity)
// Matching the coefficients of A^2..A^8 gives x1 = 4 x2 and, with z = x3/x2,
// z^2 + 4 z - 704 = 0; we take z = -2 + sqrt(708) (the root with small
// coefficients) and fix the free scale by x4 = 1:
//   x2 = (1/6 - 11 z/2520)/4, x1 = 4 x2, x3 = z x2, x5 = 11/(2520 x2),
//   x6 = (1/1008 - z/40320)/x2, x7 = 1/(40320 x2^2), y2 = 1/2 - x3 x4.
// (Values below evaluated in double precision from those formulas.)
// ---------------------------------------------------------------------------
__constant__ float kT8[8] = {
    0.059249617736388274f,  // x1
    0.014812404434097069f,  // x2
    0.36450763864714936f,   // x3
    1.0f,                   // x4
    0.29469080354241967f,   // x5
    0.025771599210148963f,  // x6
    0.11303901220301756f,   // x7
    0.13549236135285064f,   // y2
};

// Largest theta = sqrt(||A^2||_1) >= ||A||_2 for which the Taylor remainder
// sum_{k>=9} theta^k/k! stays below 3e-8 (< half an fp32 ulp of 1).  For a
// skew-symmetric (normal) A the remainder bound holds in the 2-norm, and e^A
// is orthogonal, so this is a relative bound.  Larger norms are scaled by
// 2^-s and squared s times.
constexpr float kTheta8 = 0.6f;

template <int DP> struct LinkTile;
template <> struct LinkTile<8>   { static constexpr int TM = 2, TN = 2; };
template <> struct LinkTile<16>  { static constexpr int TM = 2, TN = 2; };
template <> struct LinkTile<32>  { static constexpr int TM = 4, TN = 4; };
template <> struct LinkTile<48>  { static constexpr int TM = 6, TN = 6; };
template <> struct LinkTile<64>  { static constexpr int TM = 8, TN = 8; };
template <> struct LinkTile<96>  { static constexpr int TM = 6, TN = 6; };
template <> struct LinkTile<120> { static constexpr int TM = 8, TN = 8; };

template <int DP> struct LinkCfg {
  static constexpr int TM = LinkTile<DP>::TM, TN = LinkTile<DP>::TN;
  static constexpr int GX = DP / TN, GY = DP / TM;     // thread grid over the output
  static constexpr int ACTIVE = GX * GY;
  static constexpr int NT = ACTIVE <= 32 ? 32 : ((ACTIVE + 31) / 32) * 32;
  static constexpr int MAT = DP * DP;                   // floats per matrix (row stride DP)
  static constexpr size_t kLinkSmem = (4 * MAT + 4 * DP) * sizeof(float);
  static constexpr size_t kScanSmem = (2 * MAT) * sizeof(float);
};

template <int N>
HOA_DEVICE void lds_vec(const float* __restrict__ p, float (&v)[N]) {
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

// acc[i][j] += sum_k X[r0+i][k] * Y[k][c0+j], with X supplied column-major
// (Xt[k][r] = X[r][k]) and Y row-major, both DP x DP with row stride DP.
template <int DP, int TM, int TN>
HOA_DEVICE void mm_acc(const float* __restrict__ Xt, const float* __restrict__ Y, int r0, int c0,
                       float (&acc)[TM][TN]) {
#pragma unroll 4
  for (int k = 0; k < DP; ++k) {
    float xa[TM], yb[TN];
    lds_vec<TM>(Xt + k * DP + r0, xa);
    lds_vec<TN>(Y + k * DP + c0, yb);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(xa[i], yb[j], acc[i][j]);
  }
}

template <int TM, int TN>
HOA_DEVICE void zero_acc(float (&acc)[TM][TN]) {
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
}

// Row of the strict-upper-triangle entry idx: largest i with S_i <= idx,
// S_i = i (2d - i - 1) / 2 (row-major order of core/utils.py:20-26).
HOA_DEVICE int triu_row(int idx, int d) {
  const float b = 2.f * d - 1.f;
  int i = (int)floorf((b - sqrtf(fmaxf(b * b - 8.f * idx, 0.f))) * 0.5f);
  i = max(0, min(i, d - 2));
  while (i + 1 <= d - 2 && (i + 1) * (2 * d - i - 2) / 2 <= idx) ++i;
  while (i > 0 && i * (2 * d - i - 1) / 2 > idx) --i;
  return i;
}

struct LinkArgs {
  const void* a; int a_dtype; bool a_banked; int a_stride;  // element type, layout, floats per head
  const float* a_bias; float edge_scale;
  const void* qkv; int qkv_dtype;
  float* R; float* U; float* M;
  int B, H, T, d, chunk, K;
};

// One CTA per (chain, chunk).  For every position t of the chunk it writes
// R_t and U_t = R_t^T [q_t, k_t, v_t], then folds edge t into R.
template <int DP>
__global__ void __launch_bounds__(LinkCfg<DP>::NT, 1) link_local_kernel(LinkArgs p) {
  using C = LinkCfg<DP>;
  constexpr int TM = C::TM, TN = C::TN, NT = C::NT;
  extern __shared__ __align__(16) float smem[];
  float* bufR = smem;              // running local product R (row-major)
  float* bufA = bufR + C::MAT;     // A, later G^T
  float* buf1 = bufA + C::MAT;     // A2, later L^T
  float* buf2 = buf1 + C::MAT;     // T1 = x1 A + x2 A2, later the right factor of A8
  float* svec = buf2 + C::MAT;     // q, k, v of the current position (3*DP)
  float* colsum = svec + 3 * DP;   // column abs-sums of A2 (DP)
  __shared__ int s_squarings;

  const int tid = threadIdx.x;
  const int chain = blockIdx.x / p.K;
  const int kc = blockIdx.x % p.K;
  const int b = chain / p.H, h = chain % p.H;
  const int d = p.d;
  const int m = d * (d - 1) / 2;
  const int t0 = kc * p.chunk;
  const int t1 = min(t0 + p.chunk, p.T);
  const bool active = tid < C::ACTIVE;
  const int r0 = (tid / C::GX) * TM, c0 = (tid % C::GX) * TN;

  for (int i = tid; i < C::MAT; i += NT) bufR[i] = (i / DP == i % DP) ? 1.f : 0.f;
  __syncthreads();

  float acc[TM][TN];
  float E[TM][TN];
  const long long BH = (long long)p.B * p.H;
  for (int t = t0; t < t1; ++t) {
    // ---- position t: R_t and the locally transported q, k, v -------------
    const long long pos = (long long)chain * p.T + t;
    const long long qbase = (((long long)b * p.T + t) * p.H + h) * 3LL * d;
    const long long abase = (((long long)b * p.T + t) * p.H + h) * (long long)p.a_stride;
    // (debug build) every buffer range of this position; a failed one is skipped
    const bool r_ok = HOA_IN(pos * d * d, d * d, BH * p.T * d * d);
    const bool q_ok = HOA_IN(qbase, 3 * d, BH * p.T * 3 * d);
    const bool a_ok = HOA_IN(abase, p.a_stride, BH * p.T * p.a_stride);
    const bool u_ok = HOA_IN(pos * 3 * d, 3 * d, BH * p.T * 3 * d);
    float* Rg = p.R + pos * d * d;
    if (r_ok)
      for (int i = tid; i < d * d; i += NT) Rg[i] = bufR[(i / d) * DP + (i % d)];
    for (int i = tid; i < 3 * DP; i += NT) {
      const int v = i / DP, e = i % DP;
      svec[i] = (e < d && q_ok) ? load_elem(p.qkv, qbase + (long long)v * d + e, p.qkv_dtype) : 0.f;
    }
    // ---- edge t: A = skew(edge_scale * a_t) ------------------------------
    for (int idx = tid; idx < m; idx += NT) {
      const int i = triu_row(idx, d);
      const int j = idx - i * (2 * d - i - 1) / 2 + i + 1;
      const int slot = p.a_banked ? gen_banked_slot(i, j, d) : idx;
      float av = a_ok ? load_elem(p.a, abase + slot, p.a_dtype) : 0.f;
      if (p.a_bias != nullptr) av += p.a_bias[(long long)h * p.a_stride + slot];
      const float v = __fmul_rn(av, p.edge_scale);
      bufA[i * DP + j] = v;
      bufA[j * DP + i] = -v;
    }
    for (int i = tid; i < DP; i += NT) { bufA[i * DP + i] = 0.f; colsum[i] = 0.f; }
    if (d < DP) {
      for (int i = tid; i < DP * (DP - d); i += NT) {
        const int r = i / (DP - d), c = d + i % (DP - d);
        bufA[r * DP + c] = 0.f;
        bufA[c * DP + r] = 0.f;
      }
    }
    __syncthreads();
    float* Ug = p.U + pos * 3 * d;
    for (int i = tid; i < 3 * d; i += NT) {
      const int v = i / d, e = i % d;
      float s = 0.f;
      for (int r = 0; r < d; ++r) s = fmaf(bufR[r * DP + e], svec[v * DP + r], s);
      if (u_ok) Ug[i] = s;
    }

    // ---- A2 = A A = -(A^T A); theta^2 = ||A2||_1 -------------------------
    zero_acc(acc);
    if (active) {
      mm_acc<DP, TM, TN>(bufA, bufA, r0, c0, acc);
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        float cs = 0.f;
#pragma unroll
        for (int i = 0; i < TM; ++i) cs += fabsf(acc[i][j]);
        atomicAdd(&colsum[c0 + j], cs);
      }
    }
    __syncthreads();
    if (tid < 32) {
      float mx = 0.f;
      for (int c = tid; c < DP; c += 32) mx = fmaxf(mx, colsum[c]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (tid == 0) {
        float theta = sqrtf(mx);
        int s = 0;
        while (theta > kTheta8 && s < 64) { theta *= 0.5f; ++s; }
        s_squarings = s;
      }
    }
    __syncthreads();
    const int nsq = s_squarings;
    const float sa = ldexpf(1.f, -nsq), sa2 = ldexpf(1.f, -2 * nsq);
    const float x1 = kT8[0], x2 = kT8[1], x3 = kT8[2], x4 = kT8[3], x5 = kT8[4], x6 = kT8[5],
                x7 = kT8[6], y2 = kT8[7];

    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int o = (r0 + i) * DP + c0 + j;
          const float a2 = -acc[i][j] * sa2;
          buf1[o] = a2;
          buf2[o] = x1 * (bufA[o] * sa) + x2 * a2;
        }
    }
    __syncthreads();

    // ---- A4 = A2 T1 (A2 symmetric, so buf1 serves as its transpose) -------
    zero_acc(acc);
    if (active) mm_acc<DP, TM, TN>(buf1, buf2, r0, c0, acc);
    __syncthreads();
    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int r = r0 + i, c = c0 + j, o = r * DP + c;
          const float a = bufA[o] * sa, a2 = buf1[o], a4 = acc[i][j];
          const float id = (r == c) ? 1.f : 0.f;
          buf2[o] = x4 * id + x5 * a + x6 * a2 + x7 * a4;   // right factor
          E[i][j] = id + a + y2 * a2;                          // I + A + y2 A2
          acc[i][j] = x3 * a2 + a4;                            // left factor L
        }
    }
    __syncthreads();
    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) buf1[(c0 + j) * DP + r0 + i] = acc[i][j];   // L^T
    }
    __syncthreads();

    // ---- G = E + L Rf; then s squarings ------------------------------------
    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = E[i][j];
      mm_acc<DP, TM, TN>(buf1, buf2, r0, c0, acc);
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) bufA[(c0 + j) * DP + r0 + i] = acc[i][j];   // G^T
    }
    for (int sq = 0; sq < nsq; ++sq) {
      __syncthreads();
      if (active) {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) buf2[(r0 + i) * DP + c0 + j] = acc[i][j];   // G
      }
      __syncthreads();
      zero_acc(acc);
      if (active) mm_acc<DP, TM, TN>(bufA, buf2, r0, c0, acc);
      __syncthreads();
      if (active) {
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) bufA[(c0 + j) * DP + r0 + i] = acc[i][j];
      }
    }
    __syncthreads();

    // ---- R <- G R ----------------------------------------------------------
    zero_acc(acc);
    if (active) mm_acc<DP, TM, TN>(bufA, bufR, r0, c0, acc);
    __syncthreads();
    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) bufR[(r0 + i) * DP + c0 + j] = acc[i][j];
    }
    __syncthreads();
  }
  // chunk total: R after the chunk's last edge
  float* Mg = p.M + ((long long)chain * p.K + kc) * d * d;
  if (HOA_IN(((long long)chain * p.K + kc) * d * d, d * d, BH * p.K * d * d))
    for (int i = tid; i < d * d; i += NT) Mg[i] = bufR[(i / d) * DP + (i % d)];
}

// ---------------------------------------------------------------------------
// The same unit for DP = 120 with every operand row-major.  Thread (ty, tx) of
// the GR x 15 grid owns rows ty + GR i (i < RI, GR = DP / RI) and columns
// 4 tx + j, 60 + 4 tx + j (j < 4) of every product.  A product reads its left
// operand as float4 runs along k of the thread's RI rows (the row offsets of a
// warp fall on different banks) and its right operand as two float4 of row k
// (15 contiguous float4 per warp), and every result is stored row-major, so no
// product needs a transposed operand and no store is bank-conflicted.  Each output element accumulates the same
// terms in the same k order as link_local_kernel, so R, U and M agree with it
// (up to the rounding of the column sums behind the squaring count).
// ---------------------------------------------------------------------------
template <int DP> struct LinkRm {
  static constexpr int RI = 8;                          // rows per thread (8 x 8 tiles, 225 threads)
  static constexpr int GR = DP / RI;                    // row groups (thread rows ty + GR i)
  static constexpr int GC = DP / 8;                     // column groups: two runs of 4 columns
  static constexpr int HALF = DP / 2;                   // column offset of the second float4 run
  static constexpr int ACTIVE = GR * GC;
  static constexpr int NT = ((ACTIVE + 31) / 32) * 32;
  static_assert(DP % 8 == 0 && DP % RI == 0 && HALF == 4 * GC, "two runs of 4 GC columns");
};

// (a0, a1) = fma((x, x), (y0, y1), (a0, a1)): one packed fp32 FMA instruction, each lane
// rounded as fmaf rounds it (sm_100 fma.rn.f32x2), half the instructions of two fmaf.
HOA_DEVICE void fma2(float& a0, float& a1, unsigned long long xx, float y0, float y1) {
  unsigned long long a, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(y0), "f"(y1));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(xx), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(a));
}

template <int DP>
HOA_DEVICE void mm_rm(const float* __restrict__ X, const float* __restrict__ Y, int ty, int tx,
                      float (&acc)[LinkRm<DP>::RI][8]) {
  constexpr int RI = LinkRm<DP>::RI, GR = LinkRm<DP>::GR, HALF = LinkRm<DP>::HALF;
  const float* xr = X + ty * DP;
  const float* yc = Y + 4 * tx;
#pragma unroll 2
  for (int k0 = 0; k0 < DP; k0 += 4) {
    float4 xv[RI];
#pragma unroll
    for (int i = 0; i < RI; ++i) xv[i] = *reinterpret_cast<const float4*>(xr + i * GR * DP + k0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float4 y0 = *reinterpret_cast<const float4*>(yc + (k0 + kk) * DP);
      const float4 y1 = *reinterpret_cast<const float4*>(yc + (k0 + kk) * DP + HALF);
#pragma unroll
      for (int i = 0; i < RI; ++i) {
        const float x = kk == 0 ? xv[i].x : (kk == 1 ? xv[i].y : (kk == 2 ? xv[i].z : xv[i].w));
        unsigned long long xx;
        asm("mov.b64 %0, {%1, %1};" : "=l"(xx) : "f"(x));
        fma2(acc[i][0], acc[i][1], xx, y0.x, y0.y);
        fma2(acc[i][2], acc[i][3], xx, y0.z, y0.w);
        fma2(acc[i][4], acc[i][5], xx, y1.x, y1.y);
        fma2(acc[i][6], acc[i][7], xx, y1.z, y1.w);
      }
    }
  }
}

// Offset of the thread's element (i, h) (h: column run 0 / 1) in a row-major DP x DP matrix.
template <int DP>
HOA_DEVICE int rm_off(int ty, int tx, int i, int h) {
  return (ty + i * LinkRm<DP>::GR) * DP + 4 * tx + h * LinkRm<DP>::HALF;
}

template <int DP>
HOA_DEVICE void st_rm(float* __restrict__ Z, int ty, int tx, const float (&acc)[LinkRm<DP>::RI][8]) {
#pragma unroll
  for (int i = 0; i < LinkRm<DP>::RI; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h)
      *reinterpret_cast<float4*>(Z + rm_off<DP>(ty, tx, i, h)) =
          make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]);
}

template <int DP>
HOA_DEVICE float4 ld_rm(const float* __restrict__ Z, int ty, int tx, int i, int h) {
  return *reinterpret_cast<const float4*>(Z + rm_off<DP>(ty, tx, i, h));
}

HOA_DEVICE float f4_at(const float4& v, int c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

// Element e of row pair q of the strict upper triangle of a d x d matrix: the
// pair is row q followed by row d - 2 - q (d - 1 - q and q + 1 elements, d in all;
// for even d the middle row q = d/2 - 1 stands alone).  Returns false past the
// pair's end or past the last pair (q >= d/2); m = d (d - 1) / 2 elements in all.
HOA_DEVICE bool pair_elem(int q, int e, int d, int& row, int& col) {
  const int len1 = d - 1 - q;
  const int q2 = d - 2 - q;
  const int len = q2 == q ? len1 : d;
  const bool first = e < len1;
  row = first ? q : q2;
  col = row + 1 + (first ? e : e - len1);
  return q < d / 2 && e < len;
}

template <int DP>
__global__ void __launch_bounds__(LinkRm<DP>::NT, 1) link_local_rm_kernel(LinkArgs p) {
  using C = LinkCfg<DP>;
  using Rm = LinkRm<DP>;
  constexpr int NT = Rm::NT, RI = Rm::RI, GR = Rm::GR, HALF = Rm::HALF;
  extern __shared__ __align__(16) float smem[];
  float* bufR = smem;              // running local product R
  float* bufA = bufR + C::MAT;     // A, later G
  float* buf1 = bufA + C::MAT;     // A2s, later L
  float* buf2 = buf1 + C::MAT;     // T1, later the right factor Rf of A8
  float* svec = buf2 + C::MAT;     // q, k, v of the current position (3*DP)
  float* colsum = svec + 3 * DP;   // column abs-sums of A2 (DP)
  __shared__ int s_squarings;

  const int tid = threadIdx.x;
  const int chain = blockIdx.x / p.K;
  const int kc = blockIdx.x % p.K;
  const int b = chain / p.H, h = chain % p.H;
  const int d = p.d;
  const int m = d * (d - 1) / 2;
  const int t0 = kc * p.chunk;
  const int t1 = min(t0 + p.chunk, p.T);
  const bool active = tid < Rm::ACTIVE;
  const int ty = tid / Rm::GC, tx = tid % Rm::GC;
  // R_t leaves as float4 rows when it has no padding and R is 16-byte aligned
  const bool r_vec = d == DP && (reinterpret_cast<uintptr_t>(p.R) & 15) == 0;
  constexpr int NW = NT / 32;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kPairsPerWarp = (DP / 2 + NW - 1) / NW;         // row pairs per warp (d/2 pairs)
  constexpr int kPairChunks = (DP + 31) / 32;                   // a pair holds d <= DP elements
  constexpr int kVecPer = (3 * DP + NT - 1) / NT;               // q, k, v elements per thread

  for (int i = tid; i < C::MAT; i += NT) bufR[i] = (i / DP == i % DP) ? 1.f : 0.f;
  __syncthreads();

  float acc[RI][8];
  const long long BH = (long long)p.B * p.H;
  for (int t = t0; t < t1; ++t) {
    // ---- position t: R_t and the locally transported q, k, v -------------
    const long long pos = (long long)chain * p.T + t;
    const long long qbase = (((long long)b * p.T + t) * p.H + h) * 3LL * d;
    const long long abase = (((long long)b * p.T + t) * p.H + h) * (long long)p.a_stride;
    // (debug build) every buffer range of this position; a failed one is skipped
    const bool r_ok = HOA_IN(pos * d * d, d * d, BH * p.T * d * d);
    const bool q_ok = HOA_IN(qbase, 3 * d, BH * p.T * 3 * d);
    const bool a_ok = HOA_IN(abase, p.a_stride, BH * p.T * p.a_stride);
    const bool u_ok = HOA_IN(pos * 3 * d, 3 * d, BH * p.T * 3 * d);
    // ---- this position's inputs: every load is issued before any is used -----
    // The generator row a_t in row pairs: warp w takes pairs q = w, w + NW, ... of
    // rows q and d - 2 - q of the strict upper triangle (d elements together; the
    // middle row of an even d alone), lane l their elements l, l + 32, ...
    // (the element indices do not change with t; an opaque copy of d keeps the
    // compiler from holding all of them in registers across the position loop)
    int dl;
    asm volatile("mov.b32 %0, %1;" : "=r"(dl) : "r"(d));
    // (packed layout only: the banked one needs d % 32 == 0, which no d of this kernel has;
    // the element type is chosen outside the unrolled loops, so that no branch separates
    // the loads and they are all in flight together)
    float gv[kPairsPerWarp][kPairChunks];
    auto load_gen = [&](auto tag) {
      using TA = decltype(tag);
      const TA* ag = static_cast<const TA*>(p.a) + abase;
#pragma unroll
      for (int u = 0; u < kPairsPerWarp; ++u)
#pragma unroll
        for (int c = 0; c < kPairChunks; ++c) {
          int row, col;
          const bool ok = pair_elem(warp + u * NW, lane + 32 * c, dl, row, col) && a_ok;
          const int idx = row * (2 * dl - row - 1) / 2 + col - row - 1;
          gv[u][c] = ok ? static_cast<float>(ag[ok ? idx : 0]) : 0.f;
        }
    };
    if (p.a_dtype == HOA_BF16) load_gen(__nv_bfloat16{});
    else load_gen(float{});
    float qv[kVecPer];
#pragma unroll
    for (int u = 0; u < kVecPer; ++u) {
      const int i = tid + u * NT, v = i / DP, e = i % DP;
      qv[u] = (i < 3 * DP && e < d && q_ok) ? load_elem(p.qkv, qbase + (long long)v * d + e, p.qkv_dtype) : 0.f;
    }
    float* Rg = p.R + pos * d * d;
    if (r_ok) {
      if (r_vec) {
        for (int i = tid; i < DP * DP / 4; i += NT)
          reinterpret_cast<float4*>(Rg)[i] = reinterpret_cast<const float4*>(bufR)[i];
      } else {
        for (int i = tid; i < d * d; i += NT) Rg[i] = bufR[(i / d) * DP + (i % d)];
      }
    }
#pragma unroll
    for (int u = 0; u < kVecPer; ++u)
      if (tid + u * NT < 3 * DP) svec[tid + u * NT] = qv[u];
    if (p.a_bias != nullptr) {
      const float* bh = p.a_bias + (long long)h * p.a_stride;
#pragma unroll
      for (int u = 0; u < kPairsPerWarp; ++u)
#pragma unroll
        for (int c = 0; c < kPairChunks; ++c) {
          int row, col;
          if (pair_elem(warp + u * NW, lane + 32 * c, dl, row, col))
            gv[u][c] += bh[row * (2 * dl - row - 1) / 2 + col - row - 1];
        }
    }
    // ---- edge t: A = skew(edge_scale * a_t) ------------------------------
#pragma unroll
    for (int u = 0; u < kPairsPerWarp; ++u)
#pragma unroll
      for (int c = 0; c < kPairChunks; ++c) {
        int row, col;
        if (pair_elem(warp + u * NW, lane + 32 * c, dl, row, col)) {
          const float v = __fmul_rn(gv[u][c], p.edge_scale);
          bufA[row * DP + col] = v;
          bufA[col * DP + row] = -v;
        }
      }
    for (int i = tid; i < DP; i += NT) { bufA[i * DP + i] = 0.f; colsum[i] = 0.f; }
    if (d < DP) {
      for (int i = tid; i < DP * (DP - d); i += NT) {
        const int r = i / (DP - d), c = d + i % (DP - d);
        bufA[r * DP + c] = 0.f;
        bufA[c * DP + r] = 0.f;
      }
    }
    __syncthreads();
    // U_t = R_t^T [q, k, v]: thread e < DP sums column e of R against all three
    // (over the padded width: R's padding rows and the vectors' padding are 0)
    float* Ug = p.U + pos * 3 * d;
    if (tid < DP) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 8
      for (int r = 0; r < DP; ++r) {
        const float x = bufR[r * DP + tid];
        s0 = fmaf(x, svec[r], s0);
        s1 = fmaf(x, svec[DP + r], s1);
        s2 = fmaf(x, svec[2 * DP + r], s2);
      }
      if (tid < d && u_ok) {
        Ug[tid] = s0;
        Ug[d + tid] = s1;
        Ug[2 * d + tid] = s2;
      }
    }

    // ---- the products ----------------------------------------------------------
    // step kind 0: A2 = A A          1: A4 = A2s T1        2: G = E + L Rf
    //           3: G <- G G (s times) 4: R <- G R
    // One call site of mm_rm serves every product (a single copy of its unrolled
    // loop in the instruction cache); E waits in bufA in place of A for step 2.
    const float x1 = kT8[0], x2 = kT8[1], x3 = kT8[2], x4 = kT8[3], x5 = kT8[4], x6 = kT8[5],
                x7 = kT8[6], y2 = kT8[7];
    int nsq = 0;
    float sa = 1.f, sa2 = 1.f;
    for (int step = 0;; ++step) {
      const int kind = step < 3 ? step : (step < 3 + nsq ? 3 : 4);
      const float* X = (kind == 1 || kind == 2) ? buf1 : bufA;
      const float* Y = (kind == 0 || kind == 3) ? bufA : (kind == 4 ? bufR : buf2);
      if (active) {
        if (kind == 2) {
#pragma unroll
          for (int i = 0; i < RI; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float4 e = ld_rm<DP>(bufA, ty, tx, i, hh);
              acc[i][4 * hh] = e.x; acc[i][4 * hh + 1] = e.y; acc[i][4 * hh + 2] = e.z; acc[i][4 * hh + 3] = e.w;
            }
        } else {
          zero_acc(acc);
        }
        mm_rm<DP>(X, Y, ty, tx, acc);
      }
      if (kind == 0) {
        // theta^2 = ||A2||_1 -> the squaring count; then A2s -> buf1, T1 = x1 As + x2 A2s -> buf2
        if (active) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float cs = 0.f;
#pragma unroll
            for (int i = 0; i < RI; ++i) cs += fabsf(acc[i][j]);
            atomicAdd(&colsum[4 * tx + (j & 3) + (j >> 2) * HALF], cs);
          }
        }
        __syncthreads();
        if (tid < 32) {
          float mx = 0.f;
          for (int c = tid; c < DP; c += 32) mx = fmaxf(mx, colsum[c]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          if (tid == 0) {
            float theta = sqrtf(mx);
            int sc = 0;
            while (theta > kTheta8 && sc < 64) { theta *= 0.5f; ++sc; }
            s_squarings = sc;
          }
        }
        __syncthreads();
        nsq = s_squarings;
        sa = ldexpf(1.f, -nsq);
        sa2 = ldexpf(1.f, -2 * nsq);
        if (active) {
#pragma unroll
          for (int i = 0; i < RI; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float4 av = ld_rm<DP>(bufA, ty, tx, i, hh);
              float a2[4], t1v[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                a2[c] = acc[i][4 * hh + c] * sa2;
                t1v[c] = x1 * (f4_at(av, c) * sa) + x2 * a2[c];
              }
              const int o = rm_off<DP>(ty, tx, i, hh);
              *reinterpret_cast<float4*>(buf1 + o) = make_float4(a2[0], a2[1], a2[2], a2[3]);
              *reinterpret_cast<float4*>(buf2 + o) = make_float4(t1v[0], t1v[1], t1v[2], t1v[3]);
            }
        }
        __syncthreads();
      } else if (kind == 1) {
        // Rf -> buf2, E = I + As + y2 A2s -> bufA, L = x3 A2s + A4 -> buf1
        __syncthreads();
        if (active) {
#pragma unroll
          for (int i = 0; i < RI; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float4 av = ld_rm<DP>(bufA, ty, tx, i, hh);
              const float4 a2v = ld_rm<DP>(buf1, ty, tx, i, hh);
              const int r = ty + i * GR;
              float rf[4], ev[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const int col = 4 * tx + hh * HALF + c;
                const float a = f4_at(av, c) * sa, a2 = f4_at(a2v, c), a4 = acc[i][4 * hh + c];
                const float id = (r == col) ? 1.f : 0.f;
                rf[c] = x4 * id + x5 * a + x6 * a2 + x7 * a4;   // right factor
                ev[c] = id + a + y2 * a2;                       // I + A + y2 A2
                acc[i][4 * hh + c] = x3 * a2 + a4;              // left factor L
              }
              const int o = rm_off<DP>(ty, tx, i, hh);
              *reinterpret_cast<float4*>(buf2 + o) = make_float4(rf[0], rf[1], rf[2], rf[3]);
              *reinterpret_cast<float4*>(bufA + o) = make_float4(ev[0], ev[1], ev[2], ev[3]);
            }
        }
        __syncthreads();
        if (active) st_rm<DP>(buf1, ty, tx, acc);
        __syncthreads();
      } else if (kind == 2) {
        if (active) st_rm<DP>(bufA, ty, tx, acc);              // G (each thread its own E slots)
        __syncthreads();
      } else {
        __syncthreads();
        if (active) st_rm<DP>(kind == 3 ? bufA : bufR, ty, tx, acc);
        __syncthreads();
        if (kind == 4) break;
      }
    }
  }
  // chunk total: R after the chunk's last edge
  float* Mg = p.M + ((long long)chain * p.K + kc) * d * d;
  if (HOA_IN(((long long)chain * p.K + kc) * d * d, d * d, BH * p.K * d * d))
    for (int i = tid; i < d * d; i += NT) Mg[i] = bufR[(i / d) * DP + (i % d)];
}

// C_0 = carry_in (or I), C_{k+1} = M_k C_k.  One CTA per chain.
template <int DP>
__global__ void __launch_bounds__(LinkCfg<DP>::NT, 1)
carry_scan_kernel(const float* __restrict__ M, const float* __restrict__ carry_in,
                  float* __restrict__ Cout, float* __restrict__ total_out, int K, int d) {
  using Cf = LinkCfg<DP>;
  constexpr int TM = Cf::TM, TN = Cf::TN, NT = Cf::NT;
  extern __shared__ __align__(16) float smem[];
  float* bufC = smem;             // current carry (row-major)
  float* bufX = bufC + Cf::MAT;   // M_k^T
  const int tid = threadIdx.x;
  const int chain = blockIdx.x;
  const bool active = tid < Cf::ACTIVE;
  const int r0 = (tid / Cf::GX) * TM, c0 = (tid % Cf::GX) * TN;
  const long long BH = gridDim.x;
  const bool cin_ok = HOA_IN((long long)chain * d * d, d * d, BH * d * d);

  for (int i = tid; i < Cf::MAT; i += NT) {
    const int r = i / DP, c = i % DP;
    float v = (r == c) ? 1.f : 0.f;
    if (carry_in != nullptr && r < d && c < d && cin_ok) v = carry_in[(long long)chain * d * d + r * d + c];
    bufC[i] = v;
    bufX[i] = (r == c) ? 1.f : 0.f;
  }
  __syncthreads();
  float acc[TM][TN];
  for (int k = 0; k < K; ++k) {
    const bool k_ok = HOA_IN(((long long)chain * K + k) * d * d, d * d, BH * K * d * d);
    float* Cg = Cout + ((long long)chain * K + k) * d * d;
    if (k_ok)
      for (int i = tid; i < d * d; i += NT) Cg[i] = bufC[(i / d) * DP + (i % d)];
    const float* Mg = M + ((long long)chain * K + k) * d * d;
    for (int i = tid; i < d * d; i += NT) bufX[(i % d) * DP + (i / d)] = k_ok ? Mg[i] : 0.f;
    __syncthreads();
    zero_acc(acc);
    if (active) mm_acc<DP, TM, TN>(bufX, bufC, r0, c0, acc);
    __syncthreads();
    if (active) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) bufC[(r0 + i) * DP + c0 + j] = acc[i][j];
    }
    __syncthreads();
  }
  if (total_out != nullptr && HOA_IN((long long)chain * d * d, d * d, BH * d * d)) {
    float* Tg = total_out + (long long)chain * d * d;
    for (int i = tid; i < d * d; i += NT) Tg[i] = bufC[(i / d) * DP + (i % d)];
  }
}

// hat_v[t] = C_k^T U_v[t] for v in {q, k, v}.  One CTA per (chain, chunk).
// q^ and k^ are written (B*H, T, d); v^ likewise, or transposed as
// (B*H, d, vt_stride) when vt_stride > 0 (the K-major layout the tensor-core
// attention reads for its P V product).  Each step is a [96 x DP] x [DP x DP]
// product: rows = 32 positions x (q, k, v), register-tiled 6 x TN per thread.
constexpr int kApplyPos = 32;
constexpr int kApplyRows = 3 * kApplyPos;                 // 96
constexpr int kApplyLd = kApplyRows + 1;                  // row stride of the transposed U tile (odd: no bank conflicts)

template <int DP> struct ApplyCfg {
  static constexpr int TN = DP >= 120 ? 8 : (DP >= 96 ? 6 : (DP >= 64 ? 4 : (DP >= 48 ? 3 : (DP >= 32 ? 2 : 1))));
  static constexpr int CG = DP / TN;                      // column groups
  static constexpr int TR = 6;                            // rows per thread
  static constexpr int RG = kApplyRows / TR;              // 16 row groups
  static constexpr int ACTIVE = RG * CG;
  static constexpr int NT = ((ACTIVE + 31) / 32) * 32;
  static constexpr size_t kSmem = (size_t)(DP * DP + DP * kApplyLd + DP * kApplyPos) * sizeof(float);
  static constexpr int kLoadPer = (kApplyRows * DP + NT - 1) / NT;   // U elements per thread and tile
};

template <int DP>
__global__ void __launch_bounds__(ApplyCfg<DP>::NT)
carry_apply_kernel(const float* __restrict__ U, const float* __restrict__ Cin, void* qh, void* kh,
                   void* vh, int hat_dtype, int vt_stride, int T, int d, int chunk, int K) {
  using Cf = ApplyCfg<DP>;
  constexpr int TN = Cf::TN, TR = Cf::TR, NT = Cf::NT;
  extern __shared__ __align__(16) float smem[];
  float* Cs = smem;                      // [DP][DP]: C_k, zero-padded
  float* Ut = Cs + DP * DP;              // [DP][kApplyLd]: U tile transposed (r, row = pos*3 + v)
  float* Vt = Ut + DP * kApplyLd;        // [DP][kApplyPos]: v^ staged for the transposed write
  const int tid = threadIdx.x;
  const int chain = blockIdx.x / K;
  const int kc = blockIdx.x % K;
  const int t0 = kc * chunk, t1 = min(t0 + chunk, T);
  const bool active = tid < Cf::ACTIVE;
  const int rg = tid / Cf::CG, cg = tid % Cf::CG;
  const int row0 = rg * TR, col0 = cg * TN;
  const long long BH = gridDim.x / K;
  const float* Cg = Cin + ((long long)chain * K + kc) * d * d;
  const bool c_ok = HOA_IN(((long long)chain * K + kc) * d * d, d * d, BH * K * d * d);
  for (int i = tid; i < DP * DP; i += NT) {
    const int r = i / DP, e = i % DP;
    Cs[i] = (r < d && e < d && c_ok) ? Cg[r * d + e] : 0.f;
  }
  // the U tile of the next step is loaded into registers while this one is computed
  float pre[Cf::kLoadPer];
  auto load_tile = [&](int tb) {
    const int np = HOA_IN(((long long)chain * T + tb) * 3 * d, (long long)min(kApplyPos, t1 - tb) * 3 * d,
                          BH * T * 3 * d) ? min(kApplyPos, t1 - tb) : 0;   // (debug build) 0: skipped
    const float* Ug = U + ((long long)chain * T + tb) * 3 * d;
#pragma unroll
    for (int k = 0; k < Cf::kLoadPer; ++k) {
      const int i = tid + k * NT;
      const int row = i / DP, r = i % DP;           // row = pos*3 + v
      pre[k] = (i < kApplyRows * DP && row / 3 < np && r < d) ? Ug[(long long)row * d + r] : 0.f;
    }
  };
  if (t0 < t1) load_tile(t0);
  for (int tb = t0; tb < t1; tb += kApplyPos) {
    // (debug build) the hats of this tile inside their buffers, else the tile is not written
    const int np = (HOA_IN(((long long)chain * T + tb) * d, (long long)min(kApplyPos, t1 - tb) * d, BH * T * d) &&
                    (vt_stride == 0 || HOA_IN((long long)chain * d * vt_stride, (long long)d * vt_stride,
                                              BH * d * vt_stride)))
                       ? min(kApplyPos, t1 - tb) : 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < Cf::kLoadPer; ++k) {
      const int i = tid + k * NT;
      if (i < kApplyRows * DP) Ut[(i % DP) * kApplyLd + i / DP] = pre[k];
    }
    __syncthreads();
    if (tb + kApplyPos < t1) load_tile(tb + kApplyPos);
    float acc[TR][TN];
#pragma unroll
    for (int i = 0; i < TR; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
    if (active) {
#pragma unroll 4
      for (int r = 0; r < DP; ++r) {
        float xa[TR], yb[TN];
#pragma unroll
        for (int i = 0; i < TR; ++i) xa[i] = Ut[r * kApplyLd + row0 + i];
#pragma unroll
        for (int j = 0; j < TN; ++j) yb[j] = Cs[r * DP + col0 + j];
        if constexpr (TN % 2 == 0) {                    // packed pairs of columns (fma.rn.f32x2)
#pragma unroll
          for (int i = 0; i < TR; ++i) {
            unsigned long long xx;
            asm("mov.b64 %0, {%1, %1};" : "=l"(xx) : "f"(xa[i]));
#pragma unroll
            for (int j = 0; j < TN; j += 2) fma2(acc[i][j], acc[i][j + 1], xx, yb[j], yb[j + 1]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < TR; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(xa[i], yb[j], acc[i][j]);
        }
      }
#pragma unroll
      for (int i = 0; i < TR; ++i) {
        const int row = row0 + i, pp = row / 3, v = row % 3;
        if (pp >= np) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int e = col0 + j;
          if (e >= d) continue;
          if (v < 2) store_elem(v == 0 ? qh : kh, ((long long)chain * T + tb + pp) * d + e, hat_dtype, acc[i][j]);
          else if (vt_stride > 0) Vt[e * kApplyPos + pp] = acc[i][j];
          else store_elem(vh, ((long long)chain * T + tb + pp) * d + e, hat_dtype, acc[i][j]);
        }
      }
    }
    if (vt_stride > 0) {
      __syncthreads();
      for (int i = tid; i < d * kApplyPos; i += NT) {
        const int e = i / kApplyPos, pp = i % kApplyPos;
        if (pp < np)
          store_elem(vh, ((long long)chain * d + e) * vt_stride + tb + pp, hat_dtype, Vt[e * kApplyPos + pp]);
      }
    }
  }
}

template <int DP>
int launch_carry_apply(const float* U, const float* C, void* qh, void* kh, void* vh,
                       int hat_dtype, int vt_stride, int BH, int T, int d, int chunk,
                       cudaStream_t s) {
  using Cf = ApplyCfg<DP>;
  if (cudaFuncSetAttribute(carry_apply_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)Cf::kSmem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  const int K = ceil_div(T, chunk);
  carry_apply_kernel<DP><<<(unsigned)((long long)BH * K), Cf::NT, Cf::kSmem, s>>>(
      U, C, qh, kh, vh, hat_dtype, vt_stride, T, d, chunk, K);
  return launch_status();
}

template <int DP>
int launch_link_local(const LinkArgs& a, cudaStream_t s) {
  using C = LinkCfg<DP>;
  // DP = 120 runs the row-major variant (same results, fewer shared-memory wavefronts)
  void (*kern)(LinkArgs);
  int nt;
  if constexpr (DP == 120) {
    if (a.a_banked) return HOA_ERR_UNSUPPORTED;   // the banked layout needs d % 32 == 0
    kern = link_local_rm_kernel<DP>;
    nt = LinkRm<DP>::NT;
  } else {
    kern = link_local_kernel<DP>;
    nt = C::NT;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kLinkSmem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  const long long units = (long long)a.B * a.H * a.K;
  kern<<<(unsigned)units, nt, C::kLinkSmem, s>>>(a);
  return launch_status();
}

template <int DP>
int launch_carry_scan(const float* M, const float* cin, float* C, float* tot, int BH, int K, int d,
                      cudaStream_t s) {
  using Cf = LinkCfg<DP>;
  if (cudaFuncSetAttribute(carry_scan_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)Cf::kScanSmem) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  carry_scan_kernel<DP><<<BH, Cf::NT, Cf::kScanSmem, s>>>(M, cin, C, tot, K, d);
  return launch_status();
}

}  // namespace hoa

using namespace hoa;

static bool valid_dtype(int t) { return t == HOA_F32 || t == HOA_BF16; }

extern "C" int hoa_abi_version(void) { return 2; }

// Process-wide bound of the abortable device-side waits (hoa_set_wait_bound).
// Read at each launch of a kernel with such waits and passed as an argument.
static std::atomic<long long> g_wait_bound{sm100::kMaxWaitCycles};

long long hoa::wait_bound_cycles() { return g_wait_bound.load(std::memory_order_relaxed); }

#ifdef HOA_DEBUG_BOUNDS
namespace {
constexpr int kMaxDbgUnits = 32;
hoa::DbgSyncFn g_dbg_fns[kMaxDbgUnits];
int g_dbg_count = 0;                 // zero-initialised before any registration runs
}  // namespace
void hoa::dbg_register(DbgSyncFn fn) {
  if (g_dbg_count < kMaxDbgUnits) g_dbg_fns[g_dbg_count++] = fn;
}
extern "C" int hoa_debug_bounds(int extent_shift, int* status) {
  if (status == nullptr || extent_shift < 0 || extent_shift > 30) return HOA_ERR_INVALID_ARG;
  *status = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return HOA_ERR_LAUNCH;
  for (int i = 0; i < g_dbg_count; ++i) {
    const int st = g_dbg_fns[i](extent_shift, status);
    if (st != HOA_OK) return st;
  }
  return HOA_OK;
}
#else
extern "C" int hoa_debug_bounds(int extent_shift, int* status) {
  if (status != nullptr) *status = 0;
  (void)extent_shift;
  return HOA_ERR_UNSUPPORTED;
}
#endif

extern "C" int hoa_set_wait_bound(long long max_cycles) {
  if (max_cycles < 0 || max_cycles > sm100::kMaxWaitCycles) return HOA_ERR_INVALID_ARG;
  g_wait_bound.store(max_cycles == 0 ? sm100::kMaxWaitCycles : max_cycles, std::memory_order_relaxed);
  return HOA_OK;
}

extern "C" int hoa_gen_stride(int d, int banked) {
  if (d < 2) return 0;
  return banked ? gen_banked_stride(d) : d * (d - 1) / 2;
}

extern "C" int hoa_gen_banked_map(int d, int* slot_of_index) {
  if (slot_of_index == nullptr || d < 2) return HOA_ERR_INVALID_ARG;
  if (gen_banked_stride(d) == 0) return HOA_ERR_UNSUPPORTED;
  int idx = 0;
  for (int i = 0; i < d; ++i)
    for (int j = i + 1; j < d; ++j) slot_of_index[idx++] = gen_banked_slot(i, j, d);
  return HOA_OK;
}
extern "C" int hoa_max_head_dim(void) { return 120; }

extern "C" const char* hoa_status_string(int st) {
  switch (st) {
    case HOA_OK: return "ok";
    case HOA_ERR_INVALID_ARG: return "invalid argument";
    case HOA_ERR_UNSUPPORTED: return "unsupported head dimension or dtype";
    case HOA_ERR_LAUNCH: return "CUDA launch failed";
    case HOA_ERR_WORKSPACE: return "workspace too small";
    case HOA_ERR_TIMEOUT: return "device-side wait timed out";
    case HOA_ERR_BOUNDS: return "device-side index check failed (debug build)";
    default: return "unknown status";
  }
}

// Link-kernel CTAs resident per SM: the tensor-core kernel (d in {32, 48, 64,
// 96}) is bound by its TMEM columns (5 d, rounded up to a power of two, of
// 512) and, at d = 32, by its registers (LtLayout::kMinBlocks); the SIMT
// kernel by its shared-memory footprint.
static int link_ctas_per_sm(int d) {
  if (d == 32) return 1;     // TMEM would allow two; 2 x 544 threads do not fit the registers
  if (d == 48 || d == 64 || d == 96) {
    const int cols = 5 * d <= 128 ? 128 : (5 * d <= 256 ? 256 : 512);
    return 512 / cols;
  }
  const int dp = padded_dim(d);
  const size_t smem = (size_t)(4 * dp * dp + 4 * dp) * sizeof(float);
  int per_sm = (int)(228 * 1024 / (smem + 1024));
  return per_sm < 1 ? 1 : (per_sm > 8 ? 8 : per_sm);
}

// Chunk length: every (chain, chunk) unit is one CTA and all units are about
// equally long, so the link kernel takes about ceil(units / slots) unit-times.
// The planner picks the number of chunks per chain K that minimises
// ceil(chains K / slots) (chunk + c0), c0 ~ 2 positions of per-CTA start-up,
// over chunks of at least 16 positions: K chosen so that the last wave is
// nearly full (at B16 T4096 H16 on 148 SMs, 1024 units in 7 waves rather than
// 1216 in 8.2).
extern "C" int hoa_plan_chunk(int B, int H, int T, int d, int num_sms) {
  if (T < 16) return T > 0 ? T : 1;
  const long long chains = (long long)B * H;
  const long long slots = (long long)(num_sms > 0 ? num_sms : 148) * link_ctas_per_sm(d);
  constexpr long long kStartup = 2;          // per-CTA start-up, in positions
  long long best_cost = -1, best_chunk = T;
  for (long long K = 1; K <= T / 16; ++K) {
    const long long chunk = (T + K - 1) / K;
    const long long units = chains * ((T + chunk - 1) / chunk);
    const long long waves = (units + slots - 1) / slots;
    const long long cost = waves * (chunk + kStartup);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_chunk = chunk;
    }
  }
  return (int)best_chunk;
}

namespace hoa {
int link_local_tc(const void* a_all, int a_dtype, const float* a_bias, float edge_scale, const void* qkv,
                  int qkv_dtype, float* R, float* U, float* M, int* status, int B, int H, int T,
                  int d, int chunk, cudaStream_t s);
}

// The tensor-core kernel serves d in {32, 48, 64, 96} with fp32 generators; every
// other shape runs the SIMT kernel.  Both compute the same fp32-accurate result.
static int link_local_dispatch(const void* a_all, int a_dtype, const float* a_bias, float edge_scale, const void* qkv,
                               int qkv_dtype, float* R, float* U, float* M, int* status, int B,
                               int H, int T, int d, int chunk, void* stream) {
  if (!a_all || !qkv || !R || !U || !M || B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  if (!valid_dtype(gen_elem_dtype(a_dtype)) || !valid_dtype(qkv_dtype)) return HOA_ERR_UNSUPPORTED;
  const int a_stride = gen_row_stride(a_dtype, d);
  if (a_stride == 0) return HOA_ERR_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tc = link_local_tc(a_all, a_dtype, a_bias, edge_scale, qkv, qkv_dtype, R, U, M, status,
                               B, H, T, d, chunk, s);
  if (tc != HOA_ERR_UNSUPPORTED) return tc;
  LinkArgs a{a_all, gen_elem_dtype(a_dtype), gen_is_banked(a_dtype), a_stride, a_bias, edge_scale,
             qkv, qkv_dtype, R, U, M, B, H, T, d, chunk, ceil_div(T, chunk)};
  switch (padded_dim(d)) {
    case 8: return launch_link_local<8>(a, s);
    case 16: return launch_link_local<16>(a, s);
    case 32: return launch_link_local<32>(a, s);
    case 48: return launch_link_local<48>(a, s);
    case 64: return launch_link_local<64>(a, s);
    case 96: return launch_link_local<96>(a, s);
    case 120: return launch_link_local<120>(a, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

extern "C" int hoa_link_local(const void* a_all, int a_dtype, const float* a_bias,
                              float edge_scale, const void* qkv, int qkv_dtype, float* R, float* U,
                              float* M, int* status, int B, int H, int T, int d, int chunk,
                              void* stream) {
  return link_local_dispatch(a_all, a_dtype, a_bias, edge_scale, qkv, qkv_dtype, R, U, M, status,
                             B, H, T, d, chunk, stream);
}

extern "C" int hoa_carry_scan(const float* M, const float* carry_in, float* C, float* total_out,
                              int BH, int K, int d, void* stream) {
  if (!M || !C || BH < 1 || K < 1 || d < 1) return HOA_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (padded_dim(d)) {
    case 8: return launch_carry_scan<8>(M, carry_in, C, total_out, BH, K, d, s);
    case 16: return launch_carry_scan<16>(M, carry_in, C, total_out, BH, K, d, s);
    case 32: return launch_carry_scan<32>(M, carry_in, C, total_out, BH, K, d, s);
    case 48: return launch_carry_scan<48>(M, carry_in, C, total_out, BH, K, d, s);
    case 64: return launch_carry_scan<64>(M, carry_in, C, total_out, BH, K, d, s);
    case 96: return launch_carry_scan<96>(M, carry_in, C, total_out, BH, K, d, s);
    case 120: return launch_carry_scan<120>(M, carry_in, C, total_out, BH, K, d, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

extern "C" int hoa_carry_apply(const float* U, const float* C, void* qh, void* kh, void* vh,
                               int hat_dtype, int vt_stride, int BH, int T, int d, int chunk,
                               void* stream) {
  if (!U || !C || !qh || !kh || !vh || BH < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  if (!valid_dtype(hat_dtype)) return HOA_ERR_UNSUPPORTED;
  if (vt_stride != 0 && vt_stride < T) return HOA_ERR_INVALID_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (padded_dim(d)) {
    case 8: return launch_carry_apply<8>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 16: return launch_carry_apply<16>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 32: return launch_carry_apply<32>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 48: return launch_carry_apply<48>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 64: return launch_carry_apply<64>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 96: return launch_carry_apply<96>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    case 120: return launch_carry_apply<120>(U, C, qh, kh, vh, hat_dtype, vt_stride, BH, T, d, chunk, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

// ---------------------------------------------------------------------------
// whole core region
// ---------------------------------------------------------------------------
namespace {
struct CoreLayout {
  size_t status, R, U, M, C, qh, kh, vh, o, total;
  bool tc;
  int vt_stride;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The tensor-core attention serves bf16 hats with d % 8 == 0, d <= 128 (TMA
// row alignment, one TMEM accumulator); fp32 hats keep the fp32 SIMT attention.
bool use_tc(int hat_dtype, int d) { return hat_dtype == HOA_BF16 && d % 8 == 0 && d <= 128; }

CoreLayout core_layout(int B, int H, int T, int d, int chunk, int hat_dtype) {
  const size_t BH = (size_t)B * H;
  const size_t K = (size_t)((T + chunk - 1) / chunk);
  const size_t hs = hat_dtype == HOA_BF16 ? 2 : 4;
  CoreLayout L{};
  L.tc = use_tc(hat_dtype, d);
  L.vt_stride = L.tc ? hoa_vt_stride(T) : 0;
  size_t off = 0;
  L.status = off; off = align256(off + 256);
  L.R = off; off = align256(off + BH * T * d * d * sizeof(float));
  L.U = off; off = align256(off + BH * T * 3 * d * sizeof(float));
  L.M = off; off = align256(off + BH * K * d * d * sizeof(float));
  L.C = off; off = align256(off + BH * K * d * d * sizeof(float));
  L.qh = off; off = align256(off + BH * T * d * hs);
  L.kh = off; off = align256(off + BH * T * d * hs);
  L.vh = off; off = align256(off + BH * (L.tc ? (size_t)L.vt_stride * d : (size_t)T * d) * hs);
  L.o = off; off = align256(off + BH * T * d * sizeof(float));
  L.total = off;
  return L;
}
}  // namespace

extern "C" size_t hoa_core_workspace_bytes(int B, int H, int T, int d, int chunk, int hat_dtype) {
  if (B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1) return 0;
  return core_layout(B, H, T, d, chunk, hat_dtype).total;
}

extern "C" int hoa_core_forward(const void* a_all, int a_dtype, const float* a_bias,
                                float edge_scale, const void* qkv,
                                int qkv_dtype, void* out, int out_dtype, int hat_dtype,
                                float softmax_scale, const float* carry_in, float* total_out,
                                int B, int H, int T, int d, int chunk, void* workspace,
                                size_t workspace_bytes, void* stream) {
  if (!a_all || !qkv || !out || !workspace || B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  if (!valid_dtype(gen_elem_dtype(a_dtype)) || gen_row_stride(a_dtype, d) == 0 ||
      !valid_dtype(qkv_dtype) || !valid_dtype(out_dtype) || !valid_dtype(hat_dtype))
    return HOA_ERR_UNSUPPORTED;
  if (padded_dim(d) == 0) return HOA_ERR_UNSUPPORTED;
  const CoreLayout L = core_layout(B, H, T, d, chunk, hat_dtype);
  if (workspace_bytes < L.total) return HOA_ERR_WORKSPACE;
  char* w = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(w + L.status);
  float* R = reinterpret_cast<float*>(w + L.R);
  float* U = reinterpret_cast<float*>(w + L.U);
  float* M = reinterpret_cast<float*>(w + L.M);
  float* C = reinterpret_cast<float*>(w + L.C);
  void* qh = w + L.qh;
  void* kh = w + L.kh;
  void* vh = w + L.vh;
  float* o = reinterpret_cast<float*>(w + L.o);
  const int K = ceil_div(T, chunk);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return HOA_ERR_LAUNCH;
  int st = link_local_dispatch(a_all, a_dtype, a_bias, edge_scale, qkv, qkv_dtype, R, U, M,
                               status, B, H, T, d, chunk, stream);
  if (st != HOA_OK) return st;
  st = hoa_carry_scan(M, carry_in, C, total_out, B * H, K, d, stream);
  if (st != HOA_OK) return st;
  st = hoa_carry_apply(U, C, qh, kh, vh, hat_dtype, L.vt_stride, B * H, T, d, chunk, stream);
  if (st != HOA_OK) return st;
  st = L.tc ? hoa_attn_tc_fwd(qh, kh, vh, o, status, softmax_scale, B * H, T, T, 0, d, stream)
            : hoa_attn_fwd(qh, kh, vh, hat_dtype, o, softmax_scale, B * H, T, T, 0, d, stream);
  if (st != HOA_OK) return st;
  return hoa_out_transport(o, R, C, chunk, out, out_dtype, B, H, T, d, stream);
}
