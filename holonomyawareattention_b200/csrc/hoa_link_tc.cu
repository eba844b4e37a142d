// Kernels (1)+(2) on tcgen05: link rotations G_t = expm(skew(edge_scale a_t))
// and the local prefix products R_{t+1} = G_t R_t, fp32-accurate through
// 3xTF32 (x = hi + lo, both tf32; X Y ~ Xhi Yhi + Xhi Ylo + Xlo Yhi).
//
// Same contract and reference semantics as link_local_kernel in hoa_link.cu
// (core/utils.py:4-52, core/attention_fast_chunked.py:77, 86-94, 108-110);
// this variant serves d in {32, 48, 64, 96} with fp32 generators.
//
// One CTA per (chain, chunk): 4 TMEM lane groups x 4 (or 2) column groups of
// warps; the thread at (lane group g, lane l, column group q) owns row 32g + l
// (TMEM lane = row of every accumulator) and a quarter (or half) of its columns.  Every product D = X Y
// takes X as rows (K-major) and Y as the rows of Y^T (K-major B operand), in
// the 128B-swizzled layout; the matrices are polynomials in the skew A, so
// p(A)^T = p(-A) gives most transposes for free:
//   P1  D1 = A A^T = -A^2            X = Y^T = A rows (one buffer)
//   P2  D2 = A2s T1 = A4             Y^T = T1^T = -x1 As + x2 A2s  (As = A 2^-s, A2s = A^2 4^-s)
//   P3  D2 = L F                     L = x3 A2s + A4, F = x5 As + x6 A2s + x7 A4 (= Rf - x4 I);
//                                    F^T needs A4^T, read back through a padded shared-memory transpose
//       N  = G - I = As + (y2 + x3 x4) A2s + x4 A4 + D2      (fp32, CUDA cores)
//       s squarings: N <- 2N + N N   (N^T by the same transpose)
//   P4  D1 = R^T N^T                 A operand R^T (hi, lo) from TMEM, B = N rows
//       R_{t+1}^T = R^T + D1         (fp32, CUDA cores; R^T kept exactly in TMEM)
// Keeping the identity out of every tensor-core product makes the MMA's own
// accumulation rounding scale with the small delta (|N| ~ |A|), not with |G R|.
// The running product lives in TMEM as R^T split exactly into tf32 hi and the
// fp32 remainder lo (R^T = hi + lo), the A operand the next composition needs.
// The generator and q, k, v of the next position arrive by 1-D bulk TMA copies
// into a double-buffered stage; the next position's A-build and its P1 run
// while the current composition P4 and its readout complete (two commit
// barriers, alternating TMEM roles).
#include "hoa_sm100.cuh"

namespace hoa {
using namespace sm100;

// T8 coefficients (derivation in hoa_link.cu).
__constant__ float kT8tc[8] = {
    0.059249617736388274f, 0.014812404434097069f, 0.36450763864714936f, 1.0f,
    0.29469080354241967f,  0.025771599210148963f, 0.11303901220301756f, 0.13549236135285064f,
};
constexpr float kTheta8tc = 0.6f;

template <int DP>
struct LtLayout {
  // Thread layout: 4 TMEM lane groups (warps w % 4) x CQ column groups (warps w / 4).
  static constexpr int CQ = (DP % 32 == 0) ? 4 : 2;
  static constexpr int CW = DP / CQ;                   // columns per thread
  static constexpr int NCH = CW / 8;                   // 8-column chunks per thread
  static constexpr int NT = 128 * CQ;
  static_assert(CW % 8 == 0, "column groups must be multiples of 8");
  static constexpr int NSLAB = (DP + 31) / 32;
  static constexpr int kSlab = DP * 128;               // DP rows of 128 bytes
  static constexpr int kMat = NSLAB * kSlab;           // one split (hi or lo) of one matrix
  // An A operand is read as 128 rows (M = 128), i.e. 128 - DP rows past the
  // end of its last slab; the scratch that follows covers that.
  static constexpr int offYhi = 0;
  static constexpr int offYlo = kMat;
  static constexpr int offXhi = 2 * kMat;
  static constexpr int offXlo = 3 * kMat;
  static constexpr int offXT = 4 * kMat;               // fp32 scratch: [DP][DP+1] transpose, or reductions
  static constexpr int kXTmat = DP * (DP + 1) * 4;
  static constexpr int kXTred = CQ * 3 * 128 * 4;
  static constexpr int kXTbytes = kXTmat > kXTred ? kXTmat : kXTred;
  static constexpr int kXend = offXlo + (NSLAB - 1) * kSlab + 128 * 128;
  static constexpr int kEnd0 = offXT + kXTbytes > kXend ? offXT + kXTbytes : kXend;
  static constexpr int offStage = (kEnd0 + 1023) / 1024 * 1024;
  // one stage: the generator a_t (fp32) followed by q, k, v of position t (up to fp32)
  static constexpr int kGenBytes = (DP * (DP - 1) / 2) * 4;
  static constexpr int kStage = (kGenBytes + 3 * DP * 4 + 127) / 128 * 128;
  static constexpr int offRed = offStage + 2 * kStage;
  static constexpr int offBar = offRed + 64;
  static constexpr int kBytes = offBar + 64;
  // TMEM: R^T hi, R^T lo, A, D1, D2 (DP columns each), rounded up to a power of two.
  static constexpr uint32_t kTmemCols = 5 * DP <= 128 ? 128 : (5 * DP <= 256 ? 256 : 512);
  // Request enough shared memory that no more CTAs share an SM than its 512
  // TMEM columns can serve (an allocation would otherwise wait for a peer).
  static constexpr int kMaxCtas = 512 / kTmemCols;
  static constexpr int kMinAlloc = 233472 / (kMaxCtas + 1);
  static constexpr int kAlloc = (kBytes + 1024 > kMinAlloc) ? kBytes + 1024 : kMinAlloc;
  static_assert(kSlab % 1024 == 0, "slabs must stay 1024-aligned");
  static_assert(kAlloc <= 232448, "shared memory budget");
};

struct LinkTcArgs {
  const float* a; const float* a_bias; float edge_scale;
  const void* qkv; int qkv_dtype;
  float* R; float* U; float* M;
  int* status;
  int B, H, T, chunk, K;
};

// Row r, columns [c0, c0+8) of A = skew(edge_scale * a) from the staged vector.
// S_i = i (2d - i - 1) / 2 is the offset of row i's strict upper triangle.
template <int DP>
HOA_DEVICE void skew_row8(const float* __restrict__ av, float es, int r, int c0, float (&v)[8]) {
  const int Sr = r * (2 * DP - r - 1) / 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = c0 + i;
    float x = 0.f;
    if (c > r) x = __fmul_rn(av[Sr + c - r - 1], es);
    else if (c < r) x = -__fmul_rn(av[c * (2 * DP - c - 1) / 2 + r - c - 1], es);
    v[i] = x;
  }
}

// Write 8 values of row `row`, columns [c0, c0+8), as tf32 hi (rounded) and
// lo = x - hi (exact; the tensor core reads its leading tf32 bits) into two
// swizzled operand buffers.
template <int DP>
HOA_DEVICE void put_row8(uint8_t* hi_buf, uint8_t* lo_buf, int row, int c0, const float (&v)[8]) {
  using L = LtLayout<DP>;
  const int slab = c0 >> 5;
  const int ch0 = (c0 & 31) >> 2;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    float h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = to_tf32(v[4 * q + i]);
      l[i] = v[4 * q + i] - h[i];
    }
    const uint32_t off = slab * L::kSlab + sw128_offset(row, ch0 + q);
    *reinterpret_cast<float4*>(hi_buf + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo_buf + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// 3-pass SS product D = X Y with X given as rows and Y as the rows of Y^T
// (both K-major, 128B-swizzled).
template <int DP>
HOA_DEVICE void issue_ss(uint32_t d_tmem, uint32_t xhi, uint32_t xlo, uint32_t yhi, uint32_t ylo) {
  using L = LtLayout<DP>;
  constexpr uint32_t id = make_idesc(kFmtTF32, 128, DP);
  const uint32_t xs[3] = {xhi, xhi, xlo};
  const uint32_t ys[3] = {yhi, ylo, yhi};
#pragma unroll
  for (int ps = 0; ps < 3; ++ps)
#pragma unroll
    for (int kk = 0; kk < DP / 8; ++kk) {
      const uint32_t off = (kk >> 2) * L::kSlab + (kk & 3) * 32;
      mma_tf32(d_tmem, desc_sw128(xs[ps] + off), desc_sw128(ys[ps] + off), id, (ps | kk) ? 1u : 0u);
    }
}

// 3-pass TS product D = A B^T: A from TMEM (hi, lo columns), B rows K-major in shared memory.
template <int DP>
HOA_DEVICE void issue_ts(uint32_t d_tmem, uint32_t ahi, uint32_t alo, uint32_t bhi, uint32_t blo) {
  using L = LtLayout<DP>;
  constexpr uint32_t id = make_idesc(kFmtTF32, 128, DP);
  const uint32_t as[3] = {ahi, ahi, alo};
  const uint32_t bs[3] = {bhi, blo, bhi};
#pragma unroll
  for (int ps = 0; ps < 3; ++ps)
#pragma unroll
    for (int kk = 0; kk < DP / 8; ++kk) {
      const uint32_t ba = bs[ps] + (kk >> 2) * L::kSlab + (kk & 3) * 32;
      mma_tf32_ts(d_tmem, as[ps] + kk * 8, desc_sw128(ba), id, (ps | kk) ? 1u : 0u);
    }
}

// Barrier for operand hand-over: generic shared-memory writes become visible
// to the tensor core, TMEM accesses are ordered around the barrier.
HOA_DEVICE void operand_barrier() {
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

template <int DP>
__global__ void __launch_bounds__(LtLayout<DP>::NT, 1) link_tc_kernel(LinkTcArgs p) {
  using L = LtLayout<DP>;
  constexpr int NCH = L::NCH, CW = L::CW, CQ = L::CQ, NT = L::NT;
  constexpr int m = DP * (DP - 1) / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint8_t* Yhi = sm + L::offYhi;
  uint8_t* Ylo = sm + L::offYlo;
  uint8_t* Xhi = sm + L::offXhi;
  uint8_t* Xlo = sm + L::offXlo;
  float* XT = reinterpret_cast<float*>(sm + L::offXT);
  uint8_t* stage_base = sm + L::offStage;
  float* sred = reinterpret_cast<float*>(sm + L::offRed);
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(sm + L::offBar);  // P2, P3, squarings, P4
  uint64_t* bar_p1 = bar_mma + 1;                                    // P1
  uint64_t* bar_a = bar_mma + 2;                                     // two: one per stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_a + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lid = tid & 31;
  const int g = warp & 3, q = warp >> 2;
  const int r = g * 32 + lid;                            // this thread's row
  const int c0 = q * CW;                                 // ... and its first column
  const bool row_ok = r < DP;
  const int chain = blockIdx.x / p.K;
  const int kc = blockIdx.x % p.K;
  const int b = chain / p.H, h = chain % p.H;
  const int t0 = kc * p.chunk;
  const int t1 = min(t0 + p.chunk, p.T);
  const float es = p.edge_scale;
  const int qkv_bytes = 3 * DP * (p.qkv_dtype == HOA_BF16 ? 2 : 4);
  const uint32_t stage_tx = (uint32_t)(L::kGenBytes + qkv_bytes);

  if (tid == 0) {
    mbar_init(bar_mma, 1);
    mbar_init(bar_p1, 1);
    mbar_init(&bar_a[0], 1);
    mbar_init(&bar_a[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t lane = static_cast<uint32_t>(g * 32) << 16;
  const uint32_t cRhi = tbase, cRlo = tbase + DP, cA = tbase + 2 * DP, cD1 = tbase + 3 * DP,
                 cD2 = tbase + 4 * DP;
  const uint32_t sXhi = smem_u32(Xhi), sXlo = smem_u32(Xlo), sYhi = smem_u32(Yhi),
                 sYlo = smem_u32(Ylo);

  auto stage_gen = [&](int s) { return reinterpret_cast<float*>(stage_base + s * L::kStage); };
  auto stage_qkv = [&](int s) { return stage_base + s * L::kStage + L::kGenBytes; };
  auto fetch = [&](int s, int t) {        // thread 0: a_t and (q, k, v)_t into stage s
    const long long row = ((long long)b * p.T + t) * p.H + h;
    mbar_arrive_expect_tx(&bar_a[s], stage_tx);
    bulk_load(stage_gen(s), p.a + row * m, L::kGenBytes, &bar_a[s]);
    bulk_load(stage_qkv(s),
              static_cast<const uint8_t*>(p.qkv) + row * (long long)qkv_bytes, qkv_bytes, &bar_a[s]);
  };
  // the generator bias of this chain's head, held in registers (a few per thread)
  constexpr int kBiasPer = (m + NT - 1) / NT;
  float breg[kBiasPer];
#pragma unroll
  for (int k = 0; k < kBiasPer; ++k) {
    const int i = tid + k * NT;
    breg[k] = (p.a_bias != nullptr && i < m) ? p.a_bias[(long long)h * m + i] : 0.f;
  }
  auto add_bias = [&](int s) {            // all threads; a barrier must follow
    if (p.a_bias == nullptr) return;
    float* av = stage_gen(s);
#pragma unroll
    for (int k = 0; k < kBiasPer; ++k) {
      const int i = tid + k * NT;
      if (i < m) av[i] += breg[k];
    }
  };
  // A rows (this thread's columns) from stage s -> TMEM (fp32) and X (tf32 hi, lo)
  auto build_a = [&](int s) {
    const float* av = stage_gen(s);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float v[8];
      if (row_ok) skew_row8<DP>(av, es, r, c0 + 8 * j, v);
      else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
      }
      tmem_st8(cA + lane + c0 + 8 * j, v);
      if (row_ok) put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, v);
    }
    tmem_wait_st();
  };

  bool bad = false;
  uint32_t ph_mma = 0, ph_p1 = 0, ph_a0 = 0, ph_a1 = 0;
  auto wait_stage = [&](int s) {
    if (s == 0) { bad |= !mbar_wait(&bar_a[0], ph_a0); ph_a0 ^= 1; }
    else { bad |= !mbar_wait(&bar_a[1], ph_a1); ph_a1 ^= 1; }
  };

  // ---- prologue: position t0 (R = I, U = (q, k, v)), A(t0), and P1(t0) -> D2
  if (tid == 0) fetch(0, t0);
  wait_stage(0);
  add_bias(0);
  __syncthreads();
  {
    const long long pos = (long long)chain * p.T + t0;
    float* Rg = p.R + pos * DP * DP;
    for (int i = tid; i < DP * DP; i += NT) Rg[i] = (i / DP == i % DP) ? 1.f : 0.f;
    float* Ug = p.U + pos * 3 * DP;
    const uint8_t* qv = stage_qkv(0);
    for (int i = tid; i < 3 * DP; i += NT) Ug[i] = load_elem(qv, i, p.qkv_dtype);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float v[8], z[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { v[i] = (c0 + 8 * j + i == r) ? 1.f : 0.f; z[i] = 0.f; }
      tmem_st8(cRhi + lane + c0 + 8 * j, v);
      tmem_st8(cRlo + lane + c0 + 8 * j, z);
    }
  }
  build_a(0);
  operand_barrier();
  if (tid == 0 && !bad) {
    issue_ss<DP>(cD2, sXhi, sXlo, sXhi, sXlo);      // D = A A^T = -A^2
    tc_commit(bar_p1);
  }

  const float x1 = kT8tc[0], x2 = kT8tc[1], x3 = kT8tc[2], x4 = kT8tc[3], x5 = kT8tc[4],
              x6 = kT8tc[5], x7 = kT8tc[6], y2 = kT8tc[7];

  for (int t = t0; t < t1; ++t) {
    const int it = t - t0;
    const int sidx = it & 1;
    // TMEM roles alternate: P holds P1(t) = -A^2, Q the other accumulator
    const uint32_t cP = sidx ? cD1 : cD2, cQ = sidx ? cD2 : cD1;
    const bool last = (t + 1 == t1);
    if (__syncthreads_or(bad)) { bad = true; break; }
    if (tid == 0 && !last) {                 // stage sidx^1 was last read two positions ago
      fence_proxy_async_smem();
      fetch(sidx ^ 1, t + 1);
    }

    // ---- theta^2 = ||A^2||_1 (A^2 symmetric: max row abs-sum) ---------------
    bad |= !mbar_wait(bar_p1, ph_p1);
    ph_p1 ^= 1;
    tc_fence_after();
    {
      float v[NCH][8];
#pragma unroll
      for (int j = 0; j < NCH; ++j) tmem_ld8(cP + lane + c0 + 8 * j, v[j]);
      tmem_wait_ld();
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < NCH; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) rs += fabsf(v[j][i]);
      XT[q * 128 + r] = row_ok ? rs : 0.f;
      __syncthreads();
      if (q == 0) {
        float full = 0.f;
#pragma unroll
        for (int qq = 0; qq < CQ; ++qq) full += XT[qq * 128 + r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) full = fmaxf(full, __shfl_xor_sync(0xffffffffu, full, o));
        if (lid == 0) sred[g] = full;
      }
      __syncthreads();
    }
    int nsq = 0;
    {
      float theta = sqrtf(fmaxf(fmaxf(sred[0], sred[1]), fmaxf(sred[2], sred[3])));
      while (theta > kTheta8tc && nsq < 64) { theta *= 0.5f; ++nsq; }
    }
    const float sa = ldexpf(1.f, -nsq);
    const float sa2 = -ldexpf(1.f, -2 * nsq);    // A2s = -P * 4^-s

    // ---- P2: X = A2s rows, Y^T = T1^T = -x1 As + x2 A2s rows; Q = A4 -------------
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float a2[8], a[8];
      tmem_ld8(cP + lane + c0 + 8 * j, a2);
      tmem_ld8(cA + lane + c0 + 8 * j, a);
      tmem_wait_ld();
      if (row_ok) {
        float t1v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a2[i] *= sa2;
          t1v[i] = x2 * a2[i] - x1 * (a[i] * sa);
        }
        put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, a2);
        put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, t1v);
      }
    }
    operand_barrier();
    if (tid == 0 && !bad) {
      issue_ss<DP>(cQ, sXhi, sXlo, sYhi, sYlo);
      tc_commit(bar_mma);
    }
    bad |= !mbar_wait(bar_mma, ph_mma);
    ph_mma ^= 1;
    tc_fence_after();

    // ---- A4 -> transpose scratch, so that each thread can read its part of A4^T
    {
      float a4[NCH][8];
#pragma unroll
      for (int j = 0; j < NCH; ++j) tmem_ld8(cQ + lane + c0 + 8 * j, a4[j]);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) XT[r * (DP + 1) + c0 + 8 * j + i] = a4[j][i];
      }
    }
    __syncthreads();

    // ---- P3: X = L rows, Y^T = F^T rows; N0 = As + (y2 + x3 x4) A2s + x4 A4 -> P
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float a2[8], a4[8], a[8], n0[8];
      tmem_ld8(cP + lane + c0 + 8 * j, a2);
      tmem_ld8(cQ + lane + c0 + 8 * j, a4);
      tmem_ld8(cA + lane + c0 + 8 * j, a);
      tmem_wait_ld();
      if (row_ok) {
        float lv[8], fv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int col = c0 + 8 * j + i;
          const float a2s = a2[i] * sa2;
          const float as = a[i] * sa;
          const float a4t = XT[col * (DP + 1) + r];               // A4^T[r][col] = A4[col][r]
          lv[i] = x3 * a2s + a4[i];
          fv[i] = x6 * a2s + x7 * a4t - x5 * as;
          n0[i] = as + (y2 + x3 * x4) * a2s + x4 * a4[i];
        }
        put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, lv);
        put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, fv);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) n0[i] = 0.f;
      }
      tmem_st8(cP + lane + c0 + 8 * j, n0);
    }
    tmem_wait_st();
    operand_barrier();
    if (tid == 0 && !bad) {
      issue_ss<DP>(cQ, sXhi, sXlo, sYhi, sYlo);        // Q = L F
      tc_commit(bar_mma);
    }
    bad |= !mbar_wait(bar_mma, ph_mma);
    ph_mma ^= 1;
    tc_fence_after();

    // ---- N = G - I = N0 + L F, then s squarings N <- 2N + N N; N rows -> Y ------
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float n0[8], nv[8];
      tmem_ld8(cP + lane + c0 + 8 * j, n0);
      tmem_ld8(cQ + lane + c0 + 8 * j, nv);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 8; ++i) nv[i] += n0[i];
        if (nsq > 0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) XT[r * (DP + 1) + c0 + 8 * j + i] = nv[i];
        } else {
          put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nv);
        }
      }
    }
    for (int sq = 0; sq < nsq; ++sq) {      // N <- 2N + N N: X = N rows, Y^T = N^T rows
      __syncthreads();                       // N complete in the scratch
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          float nv[8], nt[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            nv[i] = XT[r * (DP + 1) + c0 + 8 * j + i];
            nt[i] = XT[(c0 + 8 * j + i) * (DP + 1) + r];
          }
          put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, nv);
          put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nt);
        }
      }
      operand_barrier();
      if (tid == 0 && !bad) {
        issue_ss<DP>(cQ, sXhi, sXlo, sYhi, sYlo);
        tc_commit(bar_mma);
      }
      bad |= !mbar_wait(bar_mma, ph_mma);
      ph_mma ^= 1;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float nv[8];
        tmem_ld8(cQ + lane + c0 + 8 * j, nv);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 8; ++i) nv[i] = fmaf(2.f, XT[r * (DP + 1) + c0 + 8 * j + i], nv[i]);
          if (sq + 1 < nsq) {
#pragma unroll
            for (int i = 0; i < 8; ++i) XT[r * (DP + 1) + c0 + 8 * j + i] = nv[i];
          } else {
            put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nv);
          }
        }
      }
    }
    operand_barrier();

    // ---- P4: P = R^T N^T (issued; its readout overlaps the next position's P1)
    if (tid == 0 && !bad) {
      issue_ts<DP>(cP, cRhi, cRlo, sYhi, sYlo);
      tc_commit(bar_mma);
    }

    // ---- next position: A(t+1) -> X and TMEM, P1(t+1) -> Q (queued behind P4)
    if (!last) {
      wait_stage(sidx ^ 1);
      add_bias(sidx ^ 1);
      __syncthreads();
      build_a(sidx ^ 1);
      operand_barrier();
      if (tid == 0 && !bad) {
        issue_ss<DP>(cQ, sXhi, sXlo, sXhi, sXlo);
        tc_commit(bar_p1);
      }
    }

    // ---- R_{t+1}^T = R^T + P (R^T = hi + lo exactly); write R_{t+1} and U_{t+1},
    //      or the chunk total after the chunk's last edge.
    bad |= !mbar_wait(bar_mma, ph_mma);
    ph_mma ^= 1;
    tc_fence_after();
    const long long pos1 = (long long)chain * p.T + t + 1;
    float* Rg = last ? p.M + ((long long)chain * p.K + kc) * DP * DP : p.R + pos1 * DP * DP;
    const uint8_t* qv = stage_qkv(sidx ^ 1);
    float u0 = 0.f, u1 = 0.f, u2 = 0.f;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      float rh[8], rl[8], dv[8];
      tmem_ld8(cRhi + lane + c0 + 8 * j, rh);
      tmem_ld8(cRlo + lane + c0 + 8 * j, rl);
      tmem_ld8(cP + lane + c0 + 8 * j, dv);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = (rh[i] + rl[i]) + dv[i];
        rh[i] = to_tf32(v);
        rl[i] = v - rh[i];
        dv[i] = v;
      }
      tmem_st8(cRhi + lane + c0 + 8 * j, rh);
      tmem_st8(cRlo + lane + c0 + 8 * j, rl);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = c0 + 8 * j + i;                 // dv[i] = R_{t+1}[k][r]
          Rg[(long long)k * DP + r] = dv[i];
          if (!last) {
            u0 = fmaf(dv[i], load_elem(qv, k, p.qkv_dtype), u0);
            u1 = fmaf(dv[i], load_elem(qv, DP + k, p.qkv_dtype), u1);
            u2 = fmaf(dv[i], load_elem(qv, 2 * DP + k, p.qkv_dtype), u2);
          }
        }
      }
    }
    tmem_wait_st();
    if (!last) {                                         // U_{t+1}: sum the column groups
      XT[(q * 3 + 0) * 128 + r] = u0;
      XT[(q * 3 + 1) * 128 + r] = u1;
      XT[(q * 3 + 2) * 128 + r] = u2;
      __syncthreads();
      if (q == 0 && row_ok) {
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int qq = 0; qq < CQ; ++qq) {
          s0 += XT[(qq * 3 + 0) * 128 + r];
          s1 += XT[(qq * 3 + 1) * 128 + r];
          s2 += XT[(qq * 3 + 2) * 128 + r];
        }
        float* Ug = p.U + pos1 * 3 * DP;
        Ug[r] = s0;
        Ug[DP + r] = s1;
        Ug[2 * DP + r] = s2;
      }
    }
    tc_fence_before();
  }

  bad = __syncthreads_or(bad);
  if (bad && tid == 0 && p.status != nullptr) atomicExch(p.status, HOA_ERR_TIMEOUT);
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, L::kTmemCols);
}

template <int DP>
int launch_link_tc(const LinkTcArgs& a, cudaStream_t s) {
  using L = LtLayout<DP>;
  if (cudaFuncSetAttribute(link_tc_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kAlloc) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  const long long units = (long long)a.B * a.H * a.K;
  link_tc_kernel<DP><<<(unsigned)units, L::NT, L::kAlloc, s>>>(a);
  return launch_status();
}

// Entry used by hoa_link_local: returns HOA_ERR_UNSUPPORTED when this variant
// does not serve the shape (the caller then runs the SIMT kernel).
int link_local_tc(const void* a_all, int a_dtype, const float* a_bias, float edge_scale, const void* qkv,
                  int qkv_dtype, float* R, float* U, float* M, int* status, int B, int H, int T,
                  int d, int chunk, cudaStream_t s) {
  if (a_dtype != HOA_F32 || (reinterpret_cast<uintptr_t>(a_all) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(qkv) & 15) != 0)
    return HOA_ERR_UNSUPPORTED;
  LinkTcArgs a{static_cast<const float*>(a_all), a_bias, edge_scale, qkv, qkv_dtype, R, U, M, status,
               B, H, T, chunk, ceil_div(T, chunk)};
  switch (d) {
    case 32: return launch_link_tc<32>(a, s);
    case 48: return launch_link_tc<48>(a, s);
    case 64: return launch_link_tc<64>(a, s);
    case 96: return launch_link_tc<96>(a, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

}  // namespace hoa
