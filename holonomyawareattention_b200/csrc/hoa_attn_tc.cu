// Kernel (3), bf16 path: causal online-softmax attention on tcgen05 / TMEM.
//
// Reference semantics (SiddhiMali/HolonomyAwareAttention):
//   s_ij = q^_i . k^_j * scale, tril mask, online softmax, o / l.clamp_min(1e-20)
//   core/attention_fast_chunked.py:119-168
//
// One CTA per (pair of 128-query tiles, chain); the warp roles and the TMEM
// plan are described at the kernel.  Output: o / l in fp32, (B*H, Tq, d),
// consumed by the inverse transport (kernel 4).
// Queries may be a shard of the sequence: local row i is global position
// q_offset + i and attends to keys 0 .. q_offset + i of the (gathered) key set.
#include <cudaTypedefs.h>

#include "hoa_sm100.cuh"

namespace hoa {
using namespace sm100;

// Warp roles (320 threads):
//   warps 0-3  softmax of Q tile 0 (row r of the tile = TMEM lane r = thread r)
//   warps 4-7  softmax of Q tile 1
//   warp 8     issues the tcgen05 products (one elected lane)
//   warp 9     issues the TMA loads: both Q tiles once, then K and V^T tiles
//              through a 2-stage ring
// Per key tile j, for each Q tile i (two tiles keep the tensor core busy while
// the other tile's softmax runs):
//   S_i = Q_i K_j^T     SS, M=128, N=128 keys, K=d      -> TMEM columns S_i
//   P_i = exp2(S_i * scale * log2e - m_i) as bf16, written back over S_i
//   O_i += P_i V_j      TS (P from TMEM), N=d (padded to 16), K=128 keys -> TMEM O_i
// The reference point m_i of the exponent moves only when a row's running
// maximum grows by more than 8 (a factor 256): then that warp rescales its
// rows of O_i in TMEM (after the previous P V of the tile has completed) and
// l_i.  Between moves P <= 256, exact in the sums; the result o = O / l is
// the same softmax, with the final division by l as in the reference.
constexpr int kFaThreads = 320;
constexpr int kFaRescaleLog2 = 8;

template <int DP16>
struct FaLayout {
  static constexpr int NKB = (DP16 + 63) / 64;        // 64-column boxes of a Q or K tile
  static constexpr int kBlk = 128 * 128;              // bytes: 128 rows x 128 B
  static constexpr int kQ = NKB * kBlk;               // one Q (or K) tile
  static constexpr int kVblk = DP16 * 128;            // one 64-key box of V^T
  static constexpr int kStage = kQ + 2 * kVblk;       // K tile + V^T tile (128 keys)
  static constexpr int NS = 2;
  static constexpr int offQ = 0;                      // Q tiles 0 and 1
  static constexpr int offStage = 2 * kQ;
  static constexpr int offBar = offStage + NS * kStage;
  static constexpr int kBytes = offBar + 256;
  static constexpr int kAlloc = kBytes + 1024;        // slack to align the base to 1024
  static_assert(kVblk % 1024 == 0, "V^T blocks must stay 1024-aligned");
  static_assert(kAlloc <= 232448, "shared memory budget");
  // TMEM columns: S_0, S_1 (128 each), O_0, O_1 (128 each, DP16 used)
  static constexpr uint32_t colS0 = 0, colS1 = 128, colO0 = 256, colO1 = 384;
};

struct AttnTcArgs {
  float* o;
  int* status;
  int Tq, Tk, q_offset, d;   // query rows are global positions q_offset .. q_offset + Tq - 1
  float scale_log2;
  long long max_wait;        // bound of the abortable waits, SM cycles (wait_bound_cycles())
};

HOA_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// key tiles (of 128) that the query rows starting at global position gq0 see
HOA_DEVICE int fa_key_tiles(int gq0, int Tk) { return min((gq0 + 127) / 128, (Tk - 1) / 128) + 1; }

template <int DP16>
__global__ void __launch_bounds__(kFaThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, AttnTcArgs p) {
  using L = FaLayout<DP16>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-aligned base by pointer arithmetic on the shared array, so that the
  // compiler keeps every derived pointer in the shared address space
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::offBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;      // [2]
  uint64_t* kv_empty = bars + 3;     // [2]
  uint64_t* s_full = bars + 5;       // [2] per Q tile
  uint64_t* p_full = bars + 7;       // [2] per Q tile
  uint64_t* pv_done = bars + 9;      // [2] per Q tile
  uint64_t* fin = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 13);

  const int tid = threadIdx.x, warp = tid >> 5, lid = tid & 31;
  const int chain = blockIdx.y;
  const int nqt = (p.Tq + 127) / 128;
  const int pair = gridDim.x - 1 - blockIdx.x;     // heaviest causal pairs first
  const int Tk = p.Tk;
  int n_t[2];                                       // key tiles of each Q tile (0: absent)
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int qt = 2 * pair + i;
    n_t[i] = qt < nqt ? fa_key_tiles(p.q_offset + qt * 128, Tk) : 0;
  }
  const int nkt = max(n_t[0], n_t[1]);

  if (tid == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], (i == 7 || i == 8) ? 4 : 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool bad = false;

  if (warp == 9) {
    // ------------------------------------------------------------------ TMA
    if (lid == 0) {
      const uint32_t kq = L::kQ;
      mbar_arrive_expect_tx(q_full, (n_t[1] > 0 ? 2u : 1u) * kq);
      for (int i = 0; i < 2; ++i)
        if (n_t[i] > 0)
          for (int kb = 0; kb < L::NKB; ++kb)
            tma_load_3d(sm + L::offQ + i * L::kQ + kb * L::kBlk, &tq, q_full, kb * 64,
                        (2 * pair + i) * 128, chain);
      const uint32_t v_bytes = 2u * 64u * (uint32_t)p.d * 2u;
      int issued[2] = {0, 0};
      for (int j = 0; j < nkt; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait_abortable(&kv_empty[s], ((j >> 1) - 1) & 1, s_abort, p.max_wait)) { bad = true; break; }
        uint8_t* st = sm + L::offStage + s * L::kStage;
        mbar_arrive_expect_tx(&kv_full[s], kq + v_bytes);
        for (int kb = 0; kb < L::NKB; ++kb) tma_load_3d(st + kb * L::kBlk, &tk, &kv_full[s], kb * 64, j * 128, chain);
        tma_load_3d(st + L::kQ, &tv, &kv_full[s], j * 128, 0, chain);
        tma_load_3d(st + L::kQ + L::kVblk, &tv, &kv_full[s], j * 128 + 64, 0, chain);
        issued[s] = j + 1;
      }
      // copies in flight land before the CTA exits (the last fill of each stage)
      for (int s = 0; s < 2; ++s)
        if (issued[s] > 0) bad |= !mbar_wait(&kv_full[s], ((issued[s] - 1) >> 1) & 1);
      bad |= !mbar_wait(q_full, 0);
    }
    __syncwarp();
  } else if (warp == 8) {
    // ------------------------------------------------------------------ MMA
    if (lid == 0) {
      constexpr uint32_t idS = make_idesc(kFmtBF16, 128, 128);
      constexpr uint32_t idO = make_idesc(kFmtBF16, 128, DP16);
      constexpr int KSTEPS = DP16 / 16;
      const uint64_t dQ[2] = {desc_sw128(smem_u32(sm + L::offQ)), desc_sw128(smem_u32(sm + L::offQ + L::kQ))};
      const uint32_t colS[2] = {tmem + L::colS0, tmem + L::colS1};
      const uint32_t colO[2] = {tmem + L::colO0, tmem + L::colO1};
      bool ok = mbar_wait_abortable(q_full, 0, s_abort, p.max_wait);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait_abortable(&kv_full[s], (j >> 1) & 1, s_abort, p.max_wait);
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + L::offStage + s * L::kStage);
        const uint64_t dK = desc_sw128(st), dV = desc_sw128(st + L::kQ);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (j >= n_t[i]) continue;
#pragma unroll
          for (int kk = 0; kk < KSTEPS; ++kk) {
            const uint64_t off = (uint64_t)(((kk >> 2) * L::kBlk + (kk & 3) * 32) >> 4);
            mma_bf16(colS[i], dQ[i] + off, dK + off, idS, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[i]);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (j >= n_t[i] || !ok) continue;
          ok = mbar_wait_abortable(&p_full[i], j & 1, s_abort, p.max_wait);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t boff = (uint64_t)(((kk >> 2) * L::kVblk + (kk & 3) * 32) >> 4);
            mma_bf16_ts(colO[i], colS[i] + kk * 8, dV + boff, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&pv_done[i]);
        }
        tc_commit(&kv_empty[s]);
      }
      if (!ok) bad = true;
      tc_commit(fin);
      bad |= !mbar_wait(fin, 0);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    const int i = warp >> 2;                         // Q tile of this warpgroup
    const int r = tid & 127;                         // row in the tile = TMEM lane
    const uint32_t lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t cS = tmem + (i ? L::colS1 : L::colS0) + lane;
    const uint32_t cO = tmem + (i ? L::colO1 : L::colO0) + lane;
    const int ni = n_t[i];
    const int qi = p.q_offset + (2 * pair + i) * 128 + r;   // global query position
    const float c = p.scale_log2;
    float m_ref = -INFINITY, l_run = 0.f;
    for (int j = 0; j < ni; ++j) {
      bad |= !mbar_wait_abortable(&s_full[i], j & 1, s_abort, p.max_wait);
      tc_fence_after();
      const int k0 = j * 128;
      const bool diag = k0 + 127 > qi || k0 + 127 >= Tk;          // some key of the tile masked
      float sv[4][32];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(cS + 32 * q4, sv[q4]);
      tmem_wait_ld();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_touch(sv[q4]);
      if (diag) {
#pragma unroll
        for (int k = 0; k < 128; ++k)
          if (k0 + k > qi || k0 + k >= Tk) sv[k >> 5][k & 31] = -INFINITY;
      }
      float mx[4];                                   // 4 independent partial maxima
#pragma unroll
      for (int u = 0; u < 4; ++u) mx[u] = sv[0][u];
#pragma unroll
      for (int k = 4; k < 128; ++k) mx[k & 3] = fmaxf(mx[k & 3], sv[k >> 5][k & 31]);
      const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float m_cand = mt * c;
      const bool move = m_cand > m_ref + (float)kFaRescaleLog2;    // also the first tile (m_ref = -inf)
      const float m_new = move ? m_cand : m_ref;
      const float corr = move ? exp2f(m_ref - m_new) : 1.f;        // 0 on the first tile
      if (__any_sync(0xffffffffu, move) && j > 0) {
        // rescale this warp's rows of O once the previous P V has completed
        bad |= !mbar_wait_abortable(&pv_done[i], (j - 1) & 1, s_abort, p.max_wait);
        tc_fence_after();
#pragma unroll
        for (int c16 = 0; c16 < DP16 / 16; ++c16) {
          float ov[16];
          tmem_ld16(cO + 16 * c16, ov);
          tmem_wait_ld();
          tmem_touch(ov);
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] *= corr;
          tmem_st16(cO + 16 * c16, ov);
        }
      }
      l_run *= corr;
      m_ref = m_new;
      // P = exp2(s c - m) as bf16 pairs over the first 64 columns of S (all of S is
      // in registers already)
      float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};   // 8 independent partial sums
#pragma unroll
      for (int h = 0; h < 4; ++h) {                  // 32 keys -> 16 packed columns
        float pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = exp2f(fmaf(sv[h][2 * e], c, -m_ref));
          const float p1 = exp2f(fmaf(sv[h][2 * e + 1], c, -m_ref));
          ps[(2 * e) & 7] += p0;
          ps[(2 * e + 1) & 7] += p1;
          pk[e] = __uint_as_float(pack_bf16x2(p0, p1));
        }
        tmem_st16(cS + 16 * h, pk);
      }
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lid == 0) mbar_arrive(&p_full[i]);
    }
    // ---- epilogue: o = O / l for the rows of this tile that exist
    if (ni > 0) {
      bad |= !mbar_wait_abortable(&pv_done[i], (ni - 1) & 1, s_abort, p.max_wait);
      tc_fence_after();
      const int lrow = (2 * pair + i) * 128 + r;     // local query row
      const float inv = 1.f / fmaxf(l_run, 1e-20f);
      float* orow = p.o + ((long long)chain * p.Tq + lrow) * p.d;
      // (debug build) the output row inside o, else not written
      const bool o_ok = lrow < p.Tq &&
                        HOA_IN(((long long)chain * p.Tq + lrow) * p.d, p.d, (long long)gridDim.y * p.Tq * p.d);
#pragma unroll
      for (int c16 = 0; c16 < DP16 / 16; ++c16) {
        float ov[16];
        tmem_ld16(cO + 16 * c16, ov);
        tmem_wait_ld();
        tmem_touch(ov);
        if (o_ok && !bad) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (16 * c16 + e < p.d) orow[16 * c16 + e] = ov[e] * inv;
        }
      }
    }
  }

  bad = __syncthreads_or(bad || *s_abort != 0);
  if (bad && tid == 0 && p.status != nullptr) atomicExch(p.status, HOA_ERR_TIMEOUT);
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// 3-D bf16 map over (x fastest, y, z) with a {64, box_y, 1} box, 128B swizzle, zero OOB fill.
static bool make_map(CUtensorMap* m, const void* base, uint64_t x, uint64_t y, uint64_t z,
                     uint64_t stride_y_bytes, uint64_t stride_z_bytes, uint32_t box_y) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[3] = {x, y, z};
  cuuint64_t strides[2] = {stride_y_bytes, stride_z_bytes};
  cuuint32_t box[3] = {64, box_y, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DP16>
static int launch_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                     const AttnTcArgs& a, int BH, cudaStream_t s) {
  using L = FaLayout<DP16>;
  if (cudaFuncSetAttribute(attn_tc_kernel<DP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kAlloc) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  dim3 grid((unsigned)ceil_div(ceil_div(a.Tq, 128), 2), (unsigned)BH);
  attn_tc_kernel<DP16><<<grid, kFaThreads, L::kAlloc, s>>>(mq, mk, mv, a);
  return launch_status();
}

}  // namespace hoa

using namespace hoa;

// Row stride (elements) of the v^T buffer: T rounded up to a multiple of 8, so
// that every row starts 16-byte aligned (TMA requirement).
extern "C" int hoa_vt_stride(int T) { return ((T + 7) / 8) * 8; }

extern "C" int hoa_attn_tc_fwd(const void* qh, const void* kh, const void* vhT, float* o,
                               int* status, float softmax_scale, int BH, int Tq, int Tk,
                               int q_offset, int d, void* stream) {
  if (!qh || !kh || !vhT || !o || BH < 1 || Tq < 1 || Tk < 1 || d < 1) return HOA_ERR_INVALID_ARG;
  if (q_offset < 0 || q_offset + Tq > Tk) return HOA_ERR_INVALID_ARG;
  if (BH > 65535 || d > 128 || d % 8 != 0) return HOA_ERR_UNSUPPORTED;
  const int dp16 = ((d + 15) / 16) * 16;
  const uint64_t tp = (uint64_t)hoa_vt_stride(Tk);
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, qh, d, Tq, BH, (uint64_t)d * 2, (uint64_t)Tq * d * 2, 128) ||
      !make_map(&mk, kh, d, Tk, BH, (uint64_t)d * 2, (uint64_t)Tk * d * 2, 128) ||
      !make_map(&mv, vhT, Tk, d, BH, tp * 2, tp * d * 2, (uint32_t)d))
    return HOA_ERR_INVALID_ARG;
  AttnTcArgs a{o, status, Tq, Tk, q_offset, d, softmax_scale * 1.4426950408889634f,
               wait_bound_cycles()};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dp16) {
    case 16: return launch_tc<16>(mq, mk, mv, a, BH, s);
    case 32: return launch_tc<32>(mq, mk, mv, a, BH, s);
    case 48: return launch_tc<48>(mq, mk, mv, a, BH, s);
    case 64: return launch_tc<64>(mq, mk, mv, a, BH, s);
    case 80: return launch_tc<80>(mq, mk, mv, a, BH, s);
    case 96: return launch_tc<96>(mq, mk, mv, a, BH, s);
    case 112: return launch_tc<112>(mq, mk, mv, a, BH, s);
    case 128: return launch_tc<128>(mq, mk, mv, a, BH, s);
    default: return HOA_ERR_UNSUPPORTED;
  }
}
