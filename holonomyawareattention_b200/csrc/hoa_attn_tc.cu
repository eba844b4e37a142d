// Kernel (3), bf16 path: causal online-softmax attention on tcgen05 / TMEM.
//
// Reference semantics (SiddhiMali/HolonomyAwareAttention):
//   s_ij = q^_i . k^_j * scale, tril mask, online softmax, o / l.clamp_min(1e-20)
//   core/attention_fast_chunked.py:119-168
//
// One CTA (4 warps) per (128-query tile, chain).  Thread 0 issues the TMA loads
// (128B-swizzled bf16 tiles of q^, k^ and v^T) and the tcgen05 MMAs; all 128
// threads run the softmax, one query row each (TMEM lane = row):
//   S   = Q K^T      M=128, N=128 keys, K=d     -> TMEM columns [0, 128)
//   P   = exp2(S*scale*log2e - m) as bf16, written to shared memory (swizzled)
//   O_j = P V        M=128, N=d (padded to 16),  K=128 keys -> TMEM columns [128, 128+d)
//   o  <- o * exp2(m_old - m_new) + O_j  (fp32, per-row accumulator in shared memory)
// Output: o / l in fp32, (B*H, Tq, d), consumed by the inverse transport (kernel 4).
// Queries may be a shard of the sequence: local row i is global position
// q_offset + i and attends to keys 0 .. q_offset + i of the (gathered) key set.
#include <cudaTypedefs.h>

#include "hoa_sm100.cuh"

namespace hoa {
using namespace sm100;

constexpr int kTcThreads = 128;

template <int DP16>
struct TcLayout {
  static constexpr int NKB = (DP16 + 63) / 64;        // 64-column blocks of the Q / K tiles
  static constexpr int kBlk = 128 * 128;              // bytes: 128 rows x 128 B
  static constexpr int kVblk = DP16 * 128;            // bytes per 64-key block of V^T
  static constexpr int offQ = 0;
  static constexpr int offK = offQ + NKB * kBlk;
  static constexpr int offV = offK + NKB * kBlk;
  static constexpr int offP = offV + 2 * kVblk;
  static constexpr int offO = offP + 2 * kBlk;         // fp32 accumulator, [DP16][128 rows]
  static constexpr int offBar = offO + DP16 * 128 * 4;
  static constexpr int kBytes = offBar + 64;
  static constexpr int kAlloc = kBytes + 1024;        // slack to align the base to 1024
  static_assert(kVblk % 1024 == 0, "V^T blocks must stay 1024-aligned");
};

struct AttnTcArgs {
  float* o;
  int* status;
  int Tq, Tk, q_offset, d;   // query rows are global positions q_offset .. q_offset + Tq - 1
  float scale_log2;
};

HOA_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int DP16>
__global__ void __launch_bounds__(kTcThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, AttnTcArgs p) {
  using L = TcLayout<DP16>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-aligned base by pointer arithmetic on the shared array, so that the
  // compiler keeps every derived pointer in the shared address space
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = sm + L::offQ;
  uint8_t* sK = sm + L::offK;
  uint8_t* sV = sm + L::offV;
  uint8_t* sP = sm + L::offP;
  float* sO = reinterpret_cast<float*>(sm + L::offO);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + L::offBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_mma + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int chain = blockIdx.y;
  const int qt = gridDim.x - 1 - blockIdx.x;     // heaviest causal tiles first
  const int q0 = qt * 128;                        // local query row of this tile
  const int Tq = p.Tq, Tk = p.Tk, d = p.d;
  const int gq0 = p.q_offset + q0;                // global position of its first row
  const int nkt = min((gq0 + 127) / 128, (Tk - 1) / 128) + 1;   // key tiles this tile sees

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 128;
  const uint32_t lane = static_cast<uint32_t>(warp * 32) << 16;

  constexpr uint32_t idS = make_idesc(kFmtBF16, 128, 128);
  constexpr uint32_t idO = make_idesc(kFmtBF16, 128, DP16);
  constexpr int KSTEPS = DP16 / 16;
  const uint32_t qk_bytes = L::NKB * L::kBlk;
  const uint32_t v_bytes = 2u * 64u * (uint32_t)d * 2u;
  uint32_t ph_tma = 0, ph_mma = 0;

  if (tid == 0) {
    mbar_arrive_expect_tx(bar_tma, qk_bytes);
    for (int kb = 0; kb < L::NKB; ++kb) tma_load_3d(sQ + kb * L::kBlk, &tq, bar_tma, kb * 64, q0, chain);
  }
  // `bad` records a bounded wait that gave up; the loop is left only at its
  // top, by a block-uniform vote, so every thread reaches the same barriers.
  bool bad = !mbar_wait(bar_tma, ph_tma);
  ph_tma ^= 1;

  const int qi = gq0 + tid;                        // this thread's global query position
  float m_run = -INFINITY, l_run = 0.f;
#pragma unroll 8
  for (int e = 0; e < DP16; ++e) sO[e * 128 + tid] = 0.f;    // this row's accumulator

  for (int j = 0; j < nkt; ++j) {
    if (__syncthreads_or(bad)) { bad = true; break; }
    const int k0 = j * 128;
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_tma, qk_bytes + v_bytes);
      for (int kb = 0; kb < L::NKB; ++kb) tma_load_3d(sK + kb * L::kBlk, &tk, bar_tma, kb * 64, k0, chain);
      tma_load_3d(sV, &tv, bar_tma, k0, 0, chain);
      tma_load_3d(sV + L::kVblk, &tv, bar_tma, k0 + 64, 0, chain);
    }
    bad |= !mbar_wait(bar_tma, ph_tma);
    ph_tma ^= 1;
    tc_fence_after();
    if (tid == 0 && !bad) {
      const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        const uint32_t off = (kk >> 2) * L::kBlk + (kk & 3) * 32;
        mma_bf16(tS, desc_sw128(qa + off), desc_sw128(ka + off), idS, kk > 0 ? 1u : 0u);
      }
      tc_commit(bar_mma);
    }
    bad |= !mbar_wait(bar_mma, ph_mma);
    ph_mma ^= 1;
    tc_fence_after();

    // ---- softmax over this tile's 128 keys (row qi) ------------------------
    float mt = -INFINITY;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float v[16];
      tmem_ld16(tS + lane + c * 16, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int key = k0 + c * 16 + i;
        if (key <= qi && key < Tk) mt = fmaxf(mt, v[i]);
      }
    }
    const float m_new = fmaxf(m_run, mt * p.scale_log2);
    const float corr = exp2f(m_run - m_new);
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float v[16];
      tmem_ld16(tS + lane + c * 16, v);
      tmem_wait_ld();
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int key = k0 + c * 16 + i;
        const float p0 = (key <= qi && key < Tk) ? exp2f(fmaf(v[i], p.scale_log2, -m_new)) : 0.f;
        const float p1 =
            (key + 1 <= qi && key + 1 < Tk) ? exp2f(fmaf(v[i + 1], p.scale_log2, -m_new)) : 0.f;
        rs += p0 + p1;
        pk[i >> 1] = pack_bf16x2(p0, p1);
      }
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int gg = c * 2 + g;                 // 16-byte chunk index along the 128 keys
        uint4 val = make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
        *reinterpret_cast<uint4*>(sP + (gg >> 3) * L::kBlk + sw128_offset(tid, gg & 7)) = val;
      }
    }
    l_run = l_run * corr + rs;
    m_run = m_new;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && !bad) {
      const uint32_t pa = smem_u32(sP), va = smem_u32(sV);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * L::kBlk + (kk & 3) * 32;
        const uint32_t boff = (kk >> 2) * L::kVblk + (kk & 3) * 32;
        mma_bf16(tO, desc_sw128(pa + aoff), desc_sw128(va + boff), idO, kk > 0 ? 1u : 0u);
      }
      tc_commit(bar_mma);
    }
    bad |= !mbar_wait(bar_mma, ph_mma);
    ph_mma ^= 1;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < DP16 / 16; ++c) {
      float v[16];
      tmem_ld16(tO + lane + c * 16, v);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float* a = sO + (c * 16 + i) * 128 + tid;
        *a = fmaf(*a, corr, v[i]);
      }
    }
    tc_fence_before();
  }

  bad = __syncthreads_or(bad);
  if (q0 + tid < Tq && !bad) {
    const float inv = 1.f / fmaxf(l_run, 1e-20f);
    float* orow = p.o + ((long long)chain * Tq + q0 + tid) * d;
    for (int e = 0; e < d; ++e) orow[e] = sO[e * 128 + tid] * inv;
  }
  if (bad && tid == 0 && p.status != nullptr) atomicExch(p.status, HOA_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
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
  using L = TcLayout<DP16>;
  if (cudaFuncSetAttribute(attn_tc_kernel<DP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kAlloc) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  dim3 grid((unsigned)ceil_div(a.Tq, 128), (unsigned)BH);
  attn_tc_kernel<DP16><<<grid, kTcThreads, L::kAlloc, s>>>(mq, mk, mv, a);
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
  AttnTcArgs a{o, status, Tq, Tk, q_offset, d, softmax_scale * 1.4426950408889634f};
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
