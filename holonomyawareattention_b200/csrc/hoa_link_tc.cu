// Kernels (1)+(2) on tcgen05: link rotations G_t = expm(skew(edge_scale a_t))
// and the local prefix products R_{t+1} = G_t R_t, fp32-accurate through
// 3xTF32 (x = hi + lo, both tf32; X Y ~ Xhi Yhi + Xhi Ylo + Xlo Yhi).
//
// Same contract and reference semantics as link_local_kernel in hoa_link.cu
// (core/utils.py:4-52, core/attention_fast_chunked.py:77, 86-94, 108-110);
// this variant serves d in {32, 48, 64, 96} with fp32 generators.
//
// One CTA per (chain, chunk).  Compute warps form 4 TMEM lane groups x CQ
// column groups; the thread at (lane group g, lane l, column group q) owns row
// 32g + l (TMEM lane = row of every accumulator) and 1/CQ of its columns.  One
// more warp only issues the tensor-core products.  Every product D = X Y takes
// X as rows (K-major) and Y as the rows of Y^T (K-major B operand), in the
// 128B-swizzled layout; the matrices are polynomials in the skew A, so
// p(A)^T = p(-A) gives most transposes for free:
//   P1  Q = A A^T = -A^2             X = Y^T = A rows (one shared-memory buffer)
//   P2  Q = A2s T1 = A4              Y^T = T1^T = -x1 As + x2 A2s  (As = A 2^-s, A2s = A^2 4^-s)
//   P3  Q = L F                      L = x3 A2s + A4, F = x5 As + x6 A2s + x7 A4 (= Rf - x4 I);
//                                    F^T needs A4^T, read back through a padded shared-memory transpose
//       N  = G - I = As + (y2 + x3 x4) A2s + x4 A4 + Q       (fp32, CUDA cores)
//       s squarings: N <- 2N + N N   (N^T by the same transpose)
//   P4  P = R^T N^T                  A operand R^T (hi, lo) from TMEM, B = N rows
//       R_{t+1}^T = R^T + P          (fp32, CUDA cores; R^T kept exactly in TMEM)
// In P2 and P3 the tf32 high parts of X sit in TMEM (the columns of P, free
// between the readout of one composition and the issue of the next), so two of
// the three passes read only the B tile from shared memory.
// Keeping the identity out of every tensor-core product makes the MMA's own
// accumulation rounding scale with the small delta (|N| ~ |A|), not with |G R|.
// The running product lives in TMEM as R^T split exactly into tf32 hi and the
// fp32 remainder lo (R^T = hi + lo), the A operand the next composition needs.
// The generator and q, k, v of the next position arrive by 1-D bulk TMA copies
// into a double-buffered stage.  Operands are handed to the MMA warp one
// 8-column chunk at a time (an mbarrier per chunk), so a product starts on its
// first K-steps while later ones are still being written.
#include <utility>

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
  // Compute threads: 4 TMEM lane groups (warps w % 4) x CQ column groups
  // (warps w / 4); one more warp issues the tensor-core products.
  // (d = 96 uses 3 column groups: with 13 warps every SM sub-partition holds
  // at most 4, which leaves 128 registers per thread.)
  static constexpr int CQ = (DP == 96) ? 3 : ((DP % 32 == 0) ? 4 : 2);
  static constexpr int CW = DP / CQ;                   // columns per thread
  static constexpr int NCH = CW / 8;                   // 8-column chunks per thread
  static constexpr int NT = 128 * CQ;                  // compute threads
  static constexpr int NW = NT / 32;                   // compute warps
  // + the MMA warp.  At d = 96 lane group 3 holds only padding rows, so the fourth SM
  // sub-partition (warps 3, 7, 11, 15) has spare issue slots: the block gets 16 warps and
  // warp 15 issues the products (warps 12-14 only take part in the block-wide barriers),
  // instead of sharing sub-partition 0 with three compute warps (link -2.6..-4.9%).
  static constexpr int kMmaWarp = DP == 96 ? 15 : NW;
  static constexpr int NTHREADS = DP == 96 ? 512 : NT + 32;
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
  static constexpr int offXT = 4 * kMat;               // fp32 [DP][DP+1] transpose scratch
  static constexpr int kXTbytes = DP * (DP + 1) * 4;
  static constexpr int kXend = offXlo + (NSLAB - 1) * kSlab + 128 * 128;
  static constexpr int kEnd0 = offXT + kXTbytes > kXend ? offXT + kXTbytes : kXend;
  static constexpr int offStage = (kEnd0 + 1023) / 1024 * 1024;
  // one stage: the generator a_t (fp32) followed by q, k, v of position t (up to fp32);
  // room for the larger (banked) generator layout where it exists
  static constexpr int kGenPacked = DP * (DP - 1) / 2;
  static constexpr int kGenBanked =
      DP % 32 == 0 ? 1024 * ((DP / 32) * (DP / 32 - 1) / 2) + 512 * (DP / 32) : kGenPacked;
  static constexpr int kGenBytes = kGenBanked * 4;
  static constexpr int kStage = (kGenBytes + 3 * DP * 4 + 127) / 128 * 128;
  static constexpr int offU = offStage + 2 * kStage;   // U partial sums [CQ][3][128]
  static constexpr int offMisc = offU + CQ * 3 * 128 * 4;
  static constexpr int offBar = offMisc + 64;
  // banked layout: the slot of every (column v, lane u) of a diagonal block, uint16 [32][32]
  static constexpr int offDiag = offBar + 128;
  static constexpr int kBytes = offDiag + 32 * 32 * 2;
  static_assert(NCH <= 4, "one operand barrier per column chunk, at most 4");
  // TMEM: R^T hi, R^T lo, A, P, Q (DP columns each), rounded up to a power of two.
  static constexpr uint32_t kTmemCols = 5 * DP <= 128 ? 128 : (5 * DP <= 256 ? 256 : 512);
  // Request enough shared memory that no more CTAs share an SM than its 512
  // TMEM columns can serve (an allocation would otherwise wait for a peer).
  static constexpr int kMaxCtas = 512 / kTmemCols;
  // CTAs per SM the registers must leave room for: at d = 48 two CTAs share the SM's TMEM
  // (256 columns each), which 2 x 288 threads fit only at <= 112 registers a thread
  // (unbounded the compiler takes 168, and one CTA per SM); at d = 32 two would need
  // <= 60 registers for 2 x 544 threads, so one CTA runs (hoa_plan_chunk models both).
  static constexpr int kMinBlocks = DP == 48 ? 2 : 1;
  static constexpr int kMinAlloc = 233472 / (kMaxCtas + 1);
  static constexpr int kAlloc = (kBytes + 1024 > kMinAlloc) ? kBytes + 1024 : kMinAlloc;
  static_assert(kSlab % 1024 == 0, "slabs must stay 1024-aligned");
  static_assert(kAlloc <= 232448, "shared memory budget");
};

struct LinkTcArgs {
  const float* a; const float* a_bias; float edge_scale;   // a: generator rows, packed or banked
  const void* qkv;
  float* R; float* U; float* M;
  int* status;
  int B, H, T, chunk, K;
  long long max_wait;   // bound of the abortable waits, SM cycles (wait_bound_cycles())
};

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

// Split 8 values of row `row`, columns [c0, c0+8): the tf32 high parts are
// returned in hi (for TMEM), the fp32 remainders lo = x - hi go to the
// swizzled operand buffer lo_buf.
template <int DP>
HOA_DEVICE void split_row8(uint8_t* lo_buf, int row, int c0, const float (&v)[8], float (&hi)[8]) {
  using L = LtLayout<DP>;
  const int slab = c0 >> 5;
  const int ch0 = (c0 & 31) >> 2;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    float l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      hi[4 * q + i] = to_tf32(v[4 * q + i]);
      l[i] = v[4 * q + i] - hi[4 * q + i];
    }
    const uint32_t off = slab * L::kSlab + sw128_offset(row, ch0 + q);
    *reinterpret_cast<float4*>(lo_buf + off) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// One 8-column chunk j of every column group (K-steps q * NCH + j) of a 3-pass
// SS product D = X Y, X given as rows and Y as the rows of Y^T (both K-major,
// 128B-swizzled).  Chunk 0 (q = 0, first pass) starts the accumulation.  The
// operands come as base descriptors: a K-step's descriptor is the base plus
// its byte offset / 16 (the start-address field cannot carry: shared
// addresses stay below 2^18).
template <int DP, int J>
HOA_DEVICE void issue_ss_chunk(uint32_t d_tmem, uint64_t xhi, uint64_t xlo, uint64_t yhi, uint64_t ylo) {
  using L = LtLayout<DP>;
  constexpr uint32_t id = make_idesc(kFmtTF32, 128, DP);
#pragma unroll
  for (int q = 0; q < L::CQ; ++q) {
    constexpr int kNch = L::NCH;
    const int kk = q * kNch + J;
    const uint64_t off = (uint64_t)(((kk >> 2) * L::kSlab + (kk & 3) * 32) >> 4);
    mma_tf32(d_tmem, xhi + off, yhi + off, id, (J | q) ? 1u : 0u);
    mma_tf32(d_tmem, xhi + off, ylo + off, id, 1u);
    mma_tf32(d_tmem, xlo + off, yhi + off, id, 1u);
  }
}

// The same for a 3-pass TS product D = A B^T: A from TMEM (hi, lo columns),
// B rows K-major in shared memory (base descriptors).
template <int DP, int J>
HOA_DEVICE void issue_ts_chunk(uint32_t d_tmem, uint32_t ahi, uint32_t alo, uint64_t bhi, uint64_t blo) {
  using L = LtLayout<DP>;
  constexpr uint32_t id = make_idesc(kFmtTF32, 128, DP);
#pragma unroll
  for (int q = 0; q < L::CQ; ++q) {
    constexpr int kNch = L::NCH;
    const int kk = q * kNch + J;
    const uint64_t off = (uint64_t)(((kk >> 2) * L::kSlab + (kk & 3) * 32) >> 4);
    mma_tf32_ts(d_tmem, ahi + kk * 8, bhi + off, id, (J | q) ? 1u : 0u);
    mma_tf32_ts(d_tmem, ahi + kk * 8, blo + off, id, 1u);
    mma_tf32_ts(d_tmem, alo + kk * 8, bhi + off, id, 1u);
  }
}

// The same for a 3-pass product whose A operand is split between TMEM (tf32
// high parts, two TS passes) and shared memory (remainders, one SS pass).
template <int DP, int J>
HOA_DEVICE void issue_mixed_chunk(uint32_t d_tmem, uint32_t ahi, uint64_t xlo, uint64_t yhi, uint64_t ylo) {
  using L = LtLayout<DP>;
  constexpr uint32_t id = make_idesc(kFmtTF32, 128, DP);
#pragma unroll
  for (int q = 0; q < L::CQ; ++q) {
    constexpr int kNch = L::NCH;
    const int kk = q * kNch + J;
    const uint64_t off = (uint64_t)(((kk >> 2) * L::kSlab + (kk & 3) * 32) >> 4);
    mma_tf32_ts(d_tmem, ahi + kk * 8, yhi + off, id, (J | q) ? 1u : 0u);
    mma_tf32_ts(d_tmem, ahi + kk * 8, ylo + off, id, 1u);
    mma_tf32(d_tmem, xlo + off, yhi + off, id, 1u);
  }
}

// f(std::integral_constant<int, 0>{}), ..., f(std::integral_constant<int, N - 1>{})
template <int... Is, class F>
HOA_DEVICE void unroll_impl(std::integer_sequence<int, Is...>, F&& f) {
  (f(std::integral_constant<int, Is>{}), ...);
}
template <int N, class F>
HOA_DEVICE void unroll(F&& f) {
  unroll_impl(std::make_integer_sequence<int, N>{}, f);
}

// Hand-over of operands from the compute warps to the MMA warp: each thread
// makes its generic shared-memory writes visible to the tensor core's proxy
// and orders its TMEM accesses; the warp converges and one lane arrives (the
// barrier counts one arrival per compute warp).
HOA_DEVICE void hand_over(uint64_t* bar, int lid) {
  fence_proxy_async_smem();
  tc_fence_before();
  __syncwarp();
  if (lid == 0) mbar_arrive(bar);
}

// Loads of the per-position vectors q, k, v (8 consecutive elements from
// shared memory: one 16-byte load for bf16, two for fp32).
template <bool QB16>
HOA_DEVICE void load8(const uint8_t* base, int i0, float (&v)[8]) {
  if constexpr (QB16) {
    const uint4 w = *reinterpret_cast<const uint4*>(base + 2 * i0);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(ws[i] << 16);
      v[2 * i + 1] = __uint_as_float(ws[i] & 0xffff0000u);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(base + 4 * i0);
    const float4 b = *reinterpret_cast<const float4*>(base + 4 * i0 + 16);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Warp roles.  Compute warps 0 .. NW-1 own the rows (TMEM lanes) and do all
// elementwise work; warp kMmaWarp (one elected lane) only issues the products.
// Each product's operands are handed over through an mbarrier (one arrival per
// compute warp) and its completion is signalled by tcgen05.commit, so the
// issuing thread never stalls the elementwise work.  Per position t, with
// fixed TMEM roles (cA: A, then N0; cQ: every expm product; cP: the
// composition), the tensor-core order is P2(t), P3(t) [, squarings], P4(t),
// P1(t+1), and the compute warps overlap
//   build A(t+1)                    with P4(t),
//   R_{t+1} = R_t + P4 into TMEM    with P1(t+1),
//   R_{t+1}, U_{t+1} to global      with P2(t+1).
template <int DP, bool QB16, bool BANKED>
__global__ void __launch_bounds__(LtLayout<DP>::NTHREADS, LtLayout<DP>::kMinBlocks) link_tc_kernel(LinkTcArgs p) {
  using L = LtLayout<DP>;
  constexpr int NCH = L::NCH, CW = L::CW, CQ = L::CQ, NT = L::NT, NW = L::NW;
  static_assert(!BANKED || DP % 32 == 0, "the banked generator layout needs d % 32 == 0");
  constexpr int m = BANKED ? L::kGenBanked : L::kGenPacked;   // floats per generator row
  constexpr int kQkvBytes = 3 * DP * (QB16 ? 2 : 4);
  constexpr uint32_t kNamed = 1;                          // named barrier of the compute warps
  extern __shared__ uint8_t smem_raw[];
  // 1024-aligned base by pointer arithmetic on the shared array, so that the
  // compiler keeps every derived pointer in the shared address space
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* Yhi = sm + L::offYhi;
  uint8_t* Ylo = sm + L::offYlo;
  uint8_t* Xhi = sm + L::offXhi;
  uint8_t* Xlo = sm + L::offXlo;
  float* XT = reinterpret_cast<float*>(sm + L::offXT);
  uint8_t* stage_base = sm + L::offStage;
  float* sU = reinterpret_cast<float*>(sm + L::offU);
  int* smax = reinterpret_cast<int*>(sm + L::offMisc);           // [2][4] theta^2 partial maxima
  int* s_nsq = smax + 8;                                           // squarings of this position
  volatile int* s_abort = smax + 9;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::offBar);
  uint16_t* dtab = reinterpret_cast<uint16_t*>(sm + L::offDiag);
  // operands ready (compute -> MMA), one barrier per column chunk j: P1 has its
  // own set (its hand-over follows P4's without a wait in between); P2, P3,
  // squarings and P4 share the other
  uint64_t* ops_main = bars + 0;   // [NCH]
  uint64_t* ops_p1 = bars + 4;     // [NCH]
  uint64_t* done_p1 = bars + 8;    // product complete (MMA -> compute)
  uint64_t* done_mma = bars + 9;   // P2, P3, squarings
  uint64_t* done_p4 = bars + 10;
  uint64_t* done_fin = bars + 11;
  uint64_t* bar_a = bars + 12;     // two: one per stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int tid = threadIdx.x, warp = tid >> 5, lid = tid & 31;
  const int chain = blockIdx.x / p.K;
  const int kc = blockIdx.x % p.K;
  const int b = chain / p.H, h = chain % p.H;
  const int t0 = kc * p.chunk;
  const int t1 = min(t0 + p.chunk, p.T);

  if (tid == 0) {
    for (int i = 0; i < 14; ++i) mbar_init(&bars[i], (i < 8) ? NW : 1);
    for (int i = 0; i < 8; ++i) smax[i] = 0;
    *s_nsq = 0;
    *s_abort = 0;
    fence_mbar_init();
  }
  if constexpr (BANKED) {
    for (int i = threadIdx.x; i < 32 * 32; i += blockDim.x) {
      const int v = i >> 5, u = i & 31;
      dtab[i] = (uint16_t)(u == v ? 0 : gen_banked_diag(u, v));
    }
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t cRhi = tbase, cRlo = tbase + DP, cA = tbase + 2 * DP, cP = tbase + 3 * DP,
                 cQ = tbase + 4 * DP;
  const uint32_t sXhi = smem_u32(Xhi), sXlo = smem_u32(Xlo), sYhi = smem_u32(Yhi),
                 sYlo = smem_u32(Ylo);
  bool bad = false;

  if (warp == L::kMmaWarp) {
    // ------------------------------------------------------------ MMA warp
    if (lid == 0) {
      uint32_t ph_main = 0, ph_p1 = 0;   // bit j: phase parity of barrier j of the set
      const uint64_t dXhi = desc_sw128(sXhi), dXlo = desc_sw128(sXlo), dYhi = desc_sw128(sYhi),
                     dYlo = desc_sw128(sYlo);
      // waits for chunk j of the set, then issues that chunk of the product
      auto wait_chunk = [&](uint64_t* set, uint32_t& ph, int j) {
        const bool ok = mbar_wait_abortable(&set[j], (ph >> j) & 1u, s_abort, p.max_wait);
        ph ^= 1u << j;
        if (ok) tc_fence_after();
        return ok;
      };
      // waits for each chunk of the set in turn and issues it (issue(jc), jc a compile-time index)
      auto product = [&](uint64_t* set, uint32_t& ph, auto&& issue) {
        bool ok = true;
        unroll<NCH>([&](auto jc) {
          if (ok) {
            ok = wait_chunk(set, ph, decltype(jc)::value);
            if (ok) issue(jc);
          }
        });
        return ok;
      };
      auto ss_xx = [&](auto jc) { issue_ss_chunk<DP, decltype(jc)::value>(cQ, dXhi, dXlo, dXhi, dXlo); };
      auto ss_xy = [&](auto jc) { issue_ss_chunk<DP, decltype(jc)::value>(cQ, dXhi, dXlo, dYhi, dYlo); };
      auto ts_ry = [&](auto jc) { issue_ts_chunk<DP, decltype(jc)::value>(cP, cRhi, cRlo, dYhi, dYlo); };
      auto mx_py = [&](auto jc) { issue_mixed_chunk<DP, decltype(jc)::value>(cQ, cP, dXlo, dYhi, dYlo); };
      bool ok = product(ops_p1, ph_p1, ss_xx);                               // Q = A A^T = -A^2
      if (ok) tc_commit(done_p1);
      for (int t = t0; t < t1 && ok; ++t) {
        // P2 (Q = A2s T1); the squaring count is published before chunk 0's hand-over
        int nsq = 0;
        ok = product(ops_main, ph_main, [&](auto jc) {
          if constexpr (decltype(jc)::value == 0) nsq = *s_nsq;
          mx_py(jc);
        });
        if (!ok) break;
        tc_commit(done_mma);
        ok = product(ops_main, ph_main, mx_py);                           // Q = L F
        if (ok) tc_commit(done_mma);
        for (int sq = 0; sq < nsq && ok; ++sq) {                         // Q = N N
          ok = product(ops_main, ph_main, ss_xy);
          if (ok) tc_commit(done_mma);
        }
        if (!ok || !product(ops_main, ph_main, ts_ry)) break;            // P = R^T N^T
        tc_commit(done_p4);
        if (t + 1 < t1) {
          ok = product(ops_p1, ph_p1, ss_xx);
          if (ok) tc_commit(done_p1);
        }
      }
      // every product issued above has completed before TMEM is released
      tc_commit(done_fin);
      bad |= !mbar_wait(done_fin, 0);
    }
    __syncwarp();
  } else if (warp < NW) {
    // -------------------------------------------------------- compute warps
    const int g = warp & 3, q = warp >> 2;
    const int r = g * 32 + lid;                          // this thread's row
    const int c0 = q * CW;                               // ... and its first column
    const bool row_ok = r < DP;
    const uint32_t lane = static_cast<uint32_t>(g * 32) << 16;
    const float es = p.edge_scale;
    const float x1 = kT8tc[0], x2 = kT8tc[1], x3 = kT8tc[2], x4 = kT8tc[3], x5 = kT8tc[4],
                x6 = kT8tc[5], x7 = kT8tc[6], y2 = kT8tc[7];
    const float c2 = y2 + x3 * x4;

    const long long nrows = (long long)p.B * p.T * p.H;    // rows of a_all and of qkv
    const long long BHT = nrows;                            // positions of R and U
    auto stage_gen = [&](int s) { return reinterpret_cast<float*>(stage_base + s * L::kStage); };
    auto stage_qkv = [&](int s) { return stage_base + s * L::kStage + L::kGenBytes; };
    auto fetch = [&](int s, int t) {        // thread 0: a_t and (q, k, v)_t into stage s
      const long long row = ((long long)b * p.T + t) * p.H + h;
      // (debug build) a source row outside its buffer: no copy, the barrier completes empty
      if (!(HOA_IN(row * m, m, nrows * m) && HOA_IN(row * kQkvBytes, kQkvBytes, nrows * kQkvBytes))) {
        mbar_arrive_expect_tx(&bar_a[s], 0u);
        return;
      }
      mbar_arrive_expect_tx(&bar_a[s], (uint32_t)(m * 4 + kQkvBytes));
      bulk_load(stage_gen(s), p.a + row * m, m * 4, &bar_a[s]);
      bulk_load(stage_qkv(s), static_cast<const uint8_t*>(p.qkv) + row * (long long)kQkvBytes,
                kQkvBytes, &bar_a[s]);
    };
    uint32_t ph_a[2] = {0, 0};
    uint32_t pend = 0;                      // thread 0: stages with a copy in flight
    // A stage stays marked in flight until its wait has seen the copy land: after
    // an abort the drain below waits for it with the full bound.
    auto wait_stage = [&](int s) {
      const bool ok = mbar_wait_abortable(&bar_a[s], ph_a[s], s_abort, p.max_wait);
      bad |= !ok;
      if (ok) {
        ph_a[s] ^= 1;
        pend &= ~(1u << s);
      }
    };
    // the generator bias of this chain's head (read through the cache: every
    // CTA of the head reads the same m floats)
    const float* bias_h = p.a_bias != nullptr ? p.a_bias + (long long)h * m : nullptr;
    // A(t) from stage s -> TMEM cA and X (tf32 hi, lo).  First the packed upper
    // triangle (plus bias, times edge_scale) is expanded into the transpose
    // scratch, U[row][col] = a[S_row + col - row - 1] with S_row = row (2d - row - 1) / 2;
    // then every thread reads its row segment, A[r][c] = U[r][c] (c > r),
    // -U[c][r] (c < r), 0 (c = r).
    // Banked layout: every thread reads its row segment straight from the stage,
    // with no transpose scratch and no barrier (gen_banked_slot gives the
    // layout).  A warp's columns lie in one block of 32, so the case (upper
    // rows of an off-diagonal block pair, lower rows, or a diagonal block) is
    // warp-uniform.  Same values as build_a below: A[r][c] = +-(a + bias) * es.
    auto build_a_banked = [&](int s) {
      const float* av = stage_gen(s);
      constexpr int NB = DP / 32;
      static_assert(!BANKED || (CW <= 32 && 32 % CW == 0), "a warp's columns must lie in one block of 32");
      const int bc = c0 >> 5, cv = c0 & 31;        // column block and first column offset
      float ev[NCH][8];
      if (!row_ok) {
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) ev[j][i] = 0.f;
      } else if (g < bc) {                         // upper rows: this lane's line, 16-byte loads
        const int bp = g * NB - g * (g + 1) / 2 + (bc - g - 1);
        const int line = (bp * 32 + lid) * 32, sw = lid & 7;
        auto slot = [&](int j, int k) { return line + 4 * ((((cv + 8 * j) >> 2) + (k >> 2)) ^ sw) + (k & 3); };
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const float4 x = *reinterpret_cast<const float4*>(av + slot(j, 4 * h2));
            ev[j][4 * h2] = x.x; ev[j][4 * h2 + 1] = x.y; ev[j][4 * h2 + 2] = x.z; ev[j][4 * h2 + 3] = x.w;
          }
        if (bias_h != nullptr) {
#pragma unroll
          for (int j = 0; j < NCH; ++j)
#pragma unroll
            for (int k = 0; k < 8; ++k) ev[j][k] += __ldg(bias_h + slot(j, k));
        }
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int k = 0; k < 8; ++k) ev[j][k] = __fmul_rn(ev[j][k], es);
      } else if (g > bc) {                         // lower rows: one line per column
        const int bp = bc * NB - bc * (bc + 1) / 2 + (g - bc - 1);
        const int line0 = (bp * 32 + cv) * 32;
        // (cv + 8j + i) mod 8 = i
        auto slot = [&](int j, int i) { return line0 + (8 * j + i) * 32 + (lid ^ (4 * i)); };
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) ev[j][i] = av[slot(j, i)];
        if (bias_h != nullptr) {
#pragma unroll
          for (int j = 0; j < NCH; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) ev[j][i] += __ldg(bias_h + slot(j, i));
        }
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) ev[j][i] = -__fmul_rn(ev[j][i], es);
      } else {                                     // diagonal block
        const int base = ((NB * (NB - 1) / 2) * 32 + g * 16) * 32;
        // branch-free: every lane loads, the lane with u = v from the block's first
        // slot (in range; its value is discarded), so the warp's 32 loads stay one access;
        // the slots come from the per-CTA table (gen_banked_diag, 0 for u = v)
        auto slot = [&](int v) { return base + dtab[v * 32 + lid]; };
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) ev[j][i] = av[slot(cv + 8 * j + i)];
        if (bias_h != nullptr) {
#pragma unroll
          for (int j = 0; j < NCH; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) ev[j][i] += __ldg(bias_h + slot(cv + 8 * j + i));
        }
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int v = cv + 8 * j + i;
            const float x = __fmul_rn(ev[j][i], es);
            ev[j][i] = (v == lid) ? 0.f : ((v < lid) ? -x : x);
          }
      }
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        tmem_st8(cA + lane + c0 + 8 * j, ev[j]);
        if (row_ok) put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, ev[j]);
        hand_over(&ops_p1[j], lid);                       // P1 may start on this chunk
      }
      tmem_wait_st();
    };
    auto build_a = [&](int s) {
      if constexpr (BANKED) {
        build_a_banked(s);
        return;
      }
      const float* av = stage_gen(s);
      // a warp per row, lanes along it; every load of the warp is issued before
      // its stores (fixed trip counts, predicated), so their latencies overlap
      constexpr int kRows = (DP - 1 + NW - 1) / NW, kSlots = (DP - 1 + 31) / 32;
      float ev[kRows][kSlots];
#pragma unroll
      for (int k = 0; k < kRows; ++k) {
        const int row = warp + k * NW;
        const int base = row * (2 * DP - row - 1) / 2 - row - 1;
#pragma unroll
        for (int u = 0; u < kSlots; ++u) {
          const int col = row + 1 + lid + 32 * u;
          ev[k][u] = (row < DP - 1 && col < DP) ? av[base + col] : 0.f;
        }
      }
      if (bias_h != nullptr) {
#pragma unroll
        for (int k = 0; k < kRows; ++k) {
          const int row = warp + k * NW;
          const int base = row * (2 * DP - row - 1) / 2 - row - 1;
#pragma unroll
          for (int u = 0; u < kSlots; ++u) {
            const int col = row + 1 + lid + 32 * u;
            if (row < DP - 1 && col < DP) ev[k][u] += __ldg(bias_h + base + col);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kRows; ++k) {
        const int row = warp + k * NW;
#pragma unroll
        for (int u = 0; u < kSlots; ++u) {
          const int col = row + 1 + lid + 32 * u;
          if (row < DP - 1 && col < DP) XT[row * (DP + 1) + col] = __fmul_rn(ev[k][u], es);
        }
      }
      named_sync(kNamed, NT);
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float v[8];
        const int rr = row_ok ? r : 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = c0 + 8 * j + i;
          const float up = XT[rr * (DP + 1) + c];
          const float lo = XT[c * (DP + 1) + rr];
          v[i] = (row_ok && c > r) ? up : ((row_ok && c < r) ? -lo : 0.f);
        }
        tmem_st8(cA + lane + c0 + 8 * j, v);
        if (row_ok) put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, v);
        hand_over(&ops_p1[j], lid);                       // P1 may start on this chunk
      }
      tmem_wait_st();
    };
    auto touch_rows = [&](float (&v)[NCH][8]) {
#pragma unroll
      for (int j = 0; j < NCH; ++j) tmem_touch(v[j]);
    };
    auto ld_rows = [&](uint32_t col, float (&v)[NCH][8]) {
#pragma unroll
      for (int j = 0; j < NCH; ++j) tmem_ld8(col + lane + c0 + 8 * j, v[j]);
    };
    uint32_t ph_p1 = 0, ph_mma = 0, ph_p4 = 0;
    auto wait_done = [&](uint64_t* bar, uint32_t& ph) {
      bad |= !mbar_wait_abortable(bar, ph, s_abort, p.max_wait);
      ph ^= 1;
      tc_fence_after();
    };

    // ---- prologue: stages for t0 (and t0 + 1), R = I, U = (q, k, v), A(t0)
    if (tid == 0) {
      fetch(0, t0);
      pend |= 1u;
      if (t0 + 1 < t1) { fetch(1, t0 + 1); pend |= 2u; }
    }
    wait_stage(0);
    {
      const long long pos = (long long)chain * p.T + t0;
      float* Rg = p.R + pos * DP * DP;
      if (HOA_IN(pos * DP * DP, DP * DP, BHT * DP * DP))
        for (int i = tid; i < DP * DP; i += NT) Rg[i] = (i / DP == i % DP) ? 1.f : 0.f;
      float* Ug = HOA_IN(pos * 3 * DP, 3 * DP, BHT * 3 * DP) ? p.U + pos * 3 * DP : nullptr;
      const uint8_t* qv = stage_qkv(0);
      for (int i = tid; i < 3 * DP; i += NT)
        if (Ug != nullptr) Ug[i] = QB16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(qv)[i])
                     : reinterpret_cast<const float*>(qv)[i];
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

    for (int t = t0; t < t1; ++t) {
      const int it = t - t0;
      const int sidx = it & 1, par = it & 1;
      const bool last = (t + 1 == t1);

      // ---- theta^2 <= sum over column groups of the max row abs-sum of -A^2
      wait_done(done_p1, ph_p1);
      float a2s[NCH][8];
      int nsq;                  // same value in every thread (from the same maxima)
      {
        float av[NCH][8];
        ld_rows(cQ, a2s);
        ld_rows(cA, av);
        tmem_wait_ld();
        touch_rows(a2s);
        touch_rows(av);
        float rs = 0.f;
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) rs += fabsf(a2s[j][i]);
        if (!row_ok) rs = 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rs = fmaxf(rs, __shfl_xor_sync(0xffffffffu, rs, o));
        if (lid == 0) atomicMax(&smax[par * 4 + q], __float_as_int(rs));   // rs >= 0
        if (named_sync_or(kNamed, NT, bad || *s_abort != 0)) { bad = true; break; }
        float th2 = 0.f;
#pragma unroll
        for (int qq = 0; qq < CQ; ++qq) th2 += __int_as_float(smax[par * 4 + qq]);
        if (tid < 4) smax[(par ^ 1) * 4 + tid] = 0;
        nsq = 0;
        float theta = sqrtf(th2);
        while (theta > kTheta8tc && nsq < 64) { theta *= 0.5f; ++nsq; }
        if (tid == 0) *s_nsq = nsq;
        const float sa = ldexpf(1.f, -nsq);
        const float sa2 = -ldexpf(1.f, -2 * nsq);        // A2s = -Q * 4^-s
        // ---- P2 operands: X = A2s rows, Y^T = T1^T = -x1 As + x2 A2s rows
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          float t1v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            a2s[j][i] *= sa2;
            t1v[i] = x2 * a2s[j][i] - x1 * (av[j][i] * sa);
          }
          float hv[8];
          if (row_ok) {
            split_row8<DP>(Xlo, r, c0 + 8 * j, a2s[j], hv);
            put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, t1v);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) hv[i] = 0.f;
          }
          tmem_st8(cP + lane + c0 + 8 * j, hv);             // A2s high parts: the TS operand
          tmem_wait_st();
          hand_over(&ops_main[j], lid);
        }
      }
      const float sa = ldexpf(1.f, -nsq);
      named_sync(kNamed, NT);                             // (as after N below)

      // ---- while P2 runs: R_t and U_t to global (t > t0; R_t^T row r is in TMEM)
      if (t > t0) {
        const long long pos = (long long)chain * p.T + t;
        // (debug build) R_t outside its buffer: not written
        float* Rg = HOA_IN(pos * DP * DP, DP * DP, BHT * DP * DP) ? p.R + pos * DP * DP : nullptr;
        const uint8_t* qv = stage_qkv(sidx);
        float u0 = 0.f, u1 = 0.f, u2 = 0.f;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          float rh[1][8], rl[1][8];
          tmem_ld8(cRhi + lane + c0 + 8 * j, rh[0]);
          tmem_ld8(cRlo + lane + c0 + 8 * j, rl[0]);
          tmem_wait_ld();
          tmem_touch(rh[0]);
          tmem_touch(rl[0]);
          float qa[8], ka[8], va[8];
          load8<QB16>(qv, c0 + 8 * j, qa);
          load8<QB16>(qv, DP + c0 + 8 * j, ka);
          load8<QB16>(qv, 2 * DP + c0 + 8 * j, va);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float v = rh[0][i] + rl[0][i];        // R_t[k][r], k = c0 + 8j + i
            if (row_ok && Rg != nullptr) Rg[(long long)(c0 + 8 * j + i) * DP + r] = v;
            u0 = fmaf(v, qa[i], u0);
            u1 = fmaf(v, ka[i], u1);
            u2 = fmaf(v, va[i], u2);
          }
        }
        sU[(q * 3 + 0) * 128 + r] = u0;
        sU[(q * 3 + 1) * 128 + r] = u1;
        sU[(q * 3 + 2) * 128 + r] = u2;
      }

      // ---- A4 = A2s T1 -> transpose scratch (this thread's row stays in registers)
      wait_done(done_mma, ph_mma);
      float a4[NCH][8];
      {
        ld_rows(cQ, a4);
        tmem_wait_ld();
        touch_rows(a4);
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < NCH; ++j)
#pragma unroll
            for (int i = 0; i < 8; ++i) XT[r * (DP + 1) + c0 + 8 * j + i] = a4[j][i];
        }
      }
      named_sync(kNamed, NT);
      float n0r[NCH][8];                                  // N0, kept until N is formed
      // ---- P3 operands: X = L rows, Y^T = F^T rows; N0 = As + c2 A2s + x4 A4 (registers).
      //      A4 comes from registers and A4^T from the scratch, not from Q: P3
      //      starts overwriting Q as soon as the first chunk is handed over.
      {
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          float av[8], hv[8];
          float (&n0)[8] = n0r[j];
          tmem_ld8(cA + lane + c0 + 8 * j, av);
          tmem_wait_ld();
          tmem_touch(av);
          if (row_ok) {
            float lv[8], fv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int col = c0 + 8 * j + i;
              const float as = av[i] * sa;
              const float a4t = XT[col * (DP + 1) + r];             // A4^T[r][col] = A4[col][r]
              lv[i] = x3 * a2s[j][i] + a4[j][i];
              fv[i] = x6 * a2s[j][i] + x7 * a4t - x5 * as;
              n0[i] = as + c2 * a2s[j][i] + x4 * a4[j][i];
            }
            split_row8<DP>(Xlo, r, c0 + 8 * j, lv, hv);
            put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, fv);
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) { n0[i] = 0.f; hv[i] = 0.f; }
          }
          tmem_st8(cP + lane + c0 + 8 * j, hv);             // L high parts: the TS operand
          tmem_wait_st();
          hand_over(&ops_main[j], lid);
        }
        tmem_wait_st();
      }

      // ---- after the P3 hand-overs (off the path to P3, which waits for every warp's
      //      chunks): U_t from the column groups' partial sums, and the stage refill
      if (t > t0 && q == 0 && row_ok) {                   // U_t: sum the column groups
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int qq = 0; qq < CQ; ++qq) {
          s0 += sU[(qq * 3 + 0) * 128 + r];
          s1 += sU[(qq * 3 + 1) * 128 + r];
          s2 += sU[(qq * 3 + 2) * 128 + r];
        }
        const long long upos = ((long long)chain * p.T + t) * 3 * DP;
        if (HOA_IN(upos, 3 * DP, BHT * 3 * DP)) {
          float* Ug = p.U + upos;
          Ug[r] = s0;
          Ug[DP + r] = s1;
          Ug[2 * DP + r] = s2;
        }
      }
      // stage sidx is free: position t + 2 (no new copy once a wait has given up:
      // the stage may still hold a copy in flight, which the drain waits for)
      if (tid == 0 && t + 2 < t1 && !bad && *s_abort == 0) {
        fence_proxy_async_smem();
        fetch(sidx, t + 2);
        pend |= 1u << sidx;
      }

      // ---- N = G - I = N0 + L F, then nsq squarings N <- 2N + N N; N rows -> Y
      wait_done(done_mma, ph_mma);
      {
        float nv[NCH][8];
        ld_rows(cQ, nv);
        tmem_wait_ld();
        touch_rows(nv);
        const float (&n0)[NCH][8] = n0r;
#pragma unroll
        for (int j = 0; j < NCH; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) nv[j][i] += n0[j][i];
        if (nsq == 0) {
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            if (row_ok) put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nv[j]);
            hand_over(&ops_main[j], lid);                 // P4 may start on this chunk
          }
        } else {
          for (int sq = 0; sq < nsq; ++sq) {
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < NCH; ++j)
#pragma unroll
                for (int i = 0; i < 8; ++i) XT[r * (DP + 1) + c0 + 8 * j + i] = nv[j][i];
            }
            named_sync(kNamed, NT);                       // N complete in the scratch
            if (row_ok) {                                 // X = N rows, Y^T = N^T rows
#pragma unroll
              for (int j = 0; j < NCH; ++j) {
                float nt[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) nt[i] = XT[(c0 + 8 * j + i) * (DP + 1) + r];
                put_row8<DP>(Xhi, Xlo, r, c0 + 8 * j, nv[j]);
                put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nt);
              }
            }
#pragma unroll
            for (int j = 0; j < NCH; ++j) hand_over(&ops_main[j], lid);
            wait_done(done_mma, ph_mma);
            float dq[NCH][8];
            ld_rows(cQ, dq);
            tmem_wait_ld();
            touch_rows(dq);
#pragma unroll
            for (int j = 0; j < NCH; ++j)
#pragma unroll
              for (int i = 0; i < 8; ++i) nv[j][i] = fmaf(2.f, nv[j][i], dq[j][i]);
          }
          if (row_ok) {
#pragma unroll
            for (int j = 0; j < NCH; ++j) put_row8<DP>(Yhi, Ylo, r, c0 + 8 * j, nv[j]);
          }
#pragma unroll
          for (int j = 0; j < NCH; ++j) hand_over(&ops_main[j], lid);
        }
      }
      // Every compute warp has handed N over before any starts on A(t+1): a product
      // starts on a chunk only once all warps have handed it over, and three warps
      // share each SM sub-partition, so a warp that runs ahead only takes issue slots
      // from the ones P4 waits for (measured: -1.2% link time with the barrier after
      // the P2 operands below).
      named_sync(kNamed, NT);

      // ---- while P4 runs: A(t+1) -> cA and X, then P1(t+1) is queued
      if (!last) {
        wait_stage(sidx ^ 1);
        build_a(sidx ^ 1);
      }

      // ---- while P1(t+1) runs: R_{t+1}^T = R^T + P (R^T = hi + lo exactly) in TMEM,
      //      or the chunk total after the chunk's last edge
      wait_done(done_p4, ph_p4);
      {
        const bool m_ok = HOA_IN(((long long)chain * p.K + kc) * DP * DP, DP * DP,
                                 (long long)p.B * p.H * p.K * DP * DP);
        float* Mg = p.M + ((long long)chain * p.K + kc) * DP * DP;
#pragma unroll
        for (int j = 0; j < NCH; ++j) {
          float rh[8], rl[8], dv[8];
          tmem_ld8(cRhi + lane + c0 + 8 * j, rh);
          tmem_ld8(cRlo + lane + c0 + 8 * j, rl);
          tmem_ld8(cP + lane + c0 + 8 * j, dv);
          tmem_wait_ld();
          tmem_touch(rh);
          tmem_touch(rl);
          tmem_touch(dv);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float v = (rh[i] + rl[i]) + dv[i];
            rh[i] = to_tf32(v);
            rl[i] = v - rh[i];
            if (last && row_ok && m_ok) Mg[(long long)(c0 + 8 * j + i) * DP + r] = v;
          }
          tmem_st8(cRhi + lane + c0 + 8 * j, rh);
          tmem_st8(cRlo + lane + c0 + 8 * j, rl);
        }
        tmem_wait_st();
        tc_fence_before();
      }
    }
    // copies still in flight (only after an abort) land before the CTA exits
    if (tid == 0) {
      if (pend & 1u) bad |= !mbar_wait(&bar_a[0], ph_a[0]);
      if (pend & 2u) bad |= !mbar_wait(&bar_a[1], ph_a[1]);
    }
  }

  bad = __syncthreads_or(bad || *s_abort != 0);
  if (bad && tid == 0 && p.status != nullptr) atomicExch(p.status, HOA_ERR_TIMEOUT);
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tbase, L::kTmemCols);
}

template <int DP, bool QB16, bool BANKED>
int launch_link_tc(const LinkTcArgs& a, cudaStream_t s) {
  using L = LtLayout<DP>;
  if (cudaFuncSetAttribute(link_tc_kernel<DP, QB16, BANKED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kAlloc) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  const long long units = (long long)a.B * a.H * a.K;
  link_tc_kernel<DP, QB16, BANKED><<<(unsigned)units, L::NTHREADS, L::kAlloc, s>>>(a);
  return launch_status();
}

template <int DP, bool BANKED>
int launch_link_tc_dt(const LinkTcArgs& a, int qkv_dtype, cudaStream_t s) {
  return qkv_dtype == HOA_BF16 ? launch_link_tc<DP, true, BANKED>(a, s)
                               : launch_link_tc<DP, false, BANKED>(a, s);
}

template <int DP>
int launch_link_tc_layout(const LinkTcArgs& a, int qkv_dtype, bool banked, cudaStream_t s) {
  if constexpr (DP % 32 == 0) {
    if (banked) return launch_link_tc_dt<DP, true>(a, qkv_dtype, s);
  } else {
    if (banked) return HOA_ERR_UNSUPPORTED;
  }
  return launch_link_tc_dt<DP, false>(a, qkv_dtype, s);
}

// Entry used by hoa_link_local: returns HOA_ERR_UNSUPPORTED when this variant
// does not serve the shape (the caller then runs the SIMT kernel).
int link_local_tc(const void* a_all, int a_dtype, const float* a_bias, float edge_scale, const void* qkv,
                  int qkv_dtype, float* R, float* U, float* M, int* status, int B, int H, int T,
                  int d, int chunk, cudaStream_t s) {
  if (gen_elem_dtype(a_dtype) != HOA_F32 || (qkv_dtype != HOA_F32 && qkv_dtype != HOA_BF16) ||
      (reinterpret_cast<uintptr_t>(a_all) & 15) != 0 || (reinterpret_cast<uintptr_t>(qkv) & 15) != 0)
    return HOA_ERR_UNSUPPORTED;
  const bool banked = gen_is_banked(a_dtype);
  LinkTcArgs a{static_cast<const float*>(a_all), a_bias, edge_scale, qkv, R, U, M, status,
               B, H, T, chunk, ceil_div(T, chunk), wait_bound_cycles()};
  switch (d) {
    case 32: return launch_link_tc_layout<32>(a, qkv_dtype, banked, s);
    case 48: return launch_link_tc_layout<48>(a, qkv_dtype, banked, s);
    case 64: return launch_link_tc_layout<64>(a, qkv_dtype, banked, s);
    case 96: return launch_link_tc_layout<96>(a, qkv_dtype, banked, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}

}  // namespace hoa
