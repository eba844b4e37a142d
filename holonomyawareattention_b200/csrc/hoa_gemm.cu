// hoa_edge_gemm: the second layer of the edge MLP, a = hidden W^T + bias, as one
// cuBLASLt GEMM (bf16 operands, fp32 accumulation and output) whose epilogue
// adds the fp32 bias — a plain library GEMM (core/attention_fast_chunked.py:76).
// Row-major operands are handed to cuBLASLt (column-major) as their transposes:
// the row-major M x N result is the column-major N x M product D_cm = A_cm B_cm
// with A_cm = wt (row-major K x N) viewed as N x K (leading dimension N) and
// B_cm = hidden (row-major M x K) viewed as K x M (leading dimension K); the
// bias runs along D_cm's rows (length N).
#include <cublasLt.h>
#include <cuda_fp8.h>

#include <map>
#include <mutex>
#include <tuple>

#include "hoa_common.cuh"

namespace {

struct GemmPlan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, d = nullptr;
  cublasLtMatmulAlgo_t algo{};
  size_t ws = 0;
};

std::mutex g_mu;
cublasLtHandle_t g_handle = nullptr;
using PlanKey = std::tuple<int, int, int, int, size_t>;  // M, N, K, kind (0 / 1: bf16 without / with
                                                         // bias, 2: fp8 accumulate), workspace bytes
std::map<PlanKey, GemmPlan> g_plans;

void destroy_plan(GemmPlan& p) {
  if (p.a) cublasLtMatrixLayoutDestroy(p.a);
  if (p.b) cublasLtMatrixLayoutDestroy(p.b);
  if (p.d) cublasLtMatrixLayoutDestroy(p.d);
  if (p.op) cublasLtMatmulDescDestroy(p.op);
  p = GemmPlan{};
}

// Plan for (M, N, K): descriptors and the first algorithm of cuBLASLt's heuristic
// that fits the workspace.  (Timing the heuristic's other candidates on first use
// picked slower ones: under the power cap each candidate runs at another clock.)
// Called under g_mu.
int make_plan(GemmPlan& p, int M, int N, int K, bool bias, size_t ws_bytes) {
  if (cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS)
    return HOA_ERR_LAUNCH;
  const cublasOperation_t tn = CUBLAS_OP_N;
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSA, &tn, sizeof(tn));
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSB, &tn, sizeof(tn));
  if (bias) {
    const cublasLtEpilogue_t ep = CUBLASLT_EPILOGUE_BIAS;
    const cudaDataType_t bt = CUDA_R_32F;
    cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_EPILOGUE, &ep, sizeof(ep));
    cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bt, sizeof(bt));
  }
  if (cublasLtMatrixLayoutCreate(&p.a, CUDA_R_16BF, N, K, N) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&p.b, CUDA_R_16BF, K, M, K) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&p.d, CUDA_R_32F, N, M, N) != CUBLAS_STATUS_SUCCESS)
    return HOA_ERR_LAUNCH;
  cublasLtMatmulPreference_t pref = nullptr;
  if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) return HOA_ERR_LAUNCH;
  cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes,
                                       sizeof(ws_bytes));
  cublasLtMatmulHeuristicResult_t res[1];
  int found = 0;
  const cublasStatus_t st =
      cublasLtMatmulAlgoGetHeuristic(g_handle, p.op, p.a, p.b, p.d, p.d, pref, 1, res, &found);
  cublasLtMatmulPreferenceDestroy(pref);
  if (st != CUBLAS_STATUS_SUCCESS || found < 1) return HOA_ERR_UNSUPPORTED;
  p.algo = res[0].algo;
  p.ws = res[0].workspaceSize;
  return HOA_OK;
}

}  // namespace

extern "C" int hoa_edge_gemm(const void* hidden, const void* wt, const float* bias, float* out, int M,
                             int N, int K, void* workspace, size_t workspace_bytes, void* stream) {
  if (!hidden || !wt || !out || M < 1 || N < 1 || K < 1 || (workspace_bytes > 0 && !workspace))
    return HOA_ERR_INVALID_ARG;
  // one lock covers plan lookup, the per-call bias pointer on the shared
  // descriptor and the enqueue of the matmul that reads it
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_handle == nullptr && cublasLtCreate(&g_handle) != CUBLAS_STATUS_SUCCESS) return HOA_ERR_LAUNCH;
  const PlanKey key{M, N, K, bias != nullptr ? 1 : 0, workspace_bytes};
  auto it = g_plans.find(key);
  if (it == g_plans.end()) {
    GemmPlan p;
    const int st = make_plan(p, M, N, K, bias != nullptr, workspace_bytes);
    if (st != HOA_OK) {
      destroy_plan(p);
      return st;
    }
    it = g_plans.emplace(key, p).first;
  }
  const GemmPlan& plan = it->second;
  if (bias != nullptr)
    cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias));
  const float one = 1.f, zero = 0.f;
  const cublasStatus_t st =
      cublasLtMatmul(g_handle, plan.op, &one, wt, plan.a, hidden, plan.b, &zero, out, plan.d, out, plan.d,
                     &plan.algo, workspace, plan.ws, reinterpret_cast<cudaStream_t>(stream));
  return st == CUBLAS_STATUS_SUCCESS ? HOA_OK : HOA_ERR_LAUNCH;
}

// hoa_edge_gemm_fp8_acc: out (M x N, fp32, row-major) += alpha * lo (M x K, e4m3) W^T, with
// W (N x K, e4m3) the output projection's weight as stored (rows = outputs).  Both operands
// are K-major, cuBLASLt's FP8 form: D_cm (N x M) = op(A) B with A = W viewed as K x N
// (transposed) and B = lo viewed as K x M; C = D = out (beta = 1).
namespace {
int make_plan_fp8(GemmPlan& p, int M, int N, int K, size_t ws_bytes) {
  if (cublasLtMatmulDescCreate(&p.op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS)
    return HOA_ERR_LAUNCH;
  const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta));
  cublasLtMatmulDescSetAttribute(p.op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb));
  if (cublasLtMatrixLayoutCreate(&p.a, CUDA_R_8F_E4M3, K, N, K) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&p.b, CUDA_R_8F_E4M3, K, M, K) != CUBLAS_STATUS_SUCCESS ||
      cublasLtMatrixLayoutCreate(&p.d, CUDA_R_32F, N, M, N) != CUBLAS_STATUS_SUCCESS)
    return HOA_ERR_LAUNCH;
  cublasLtMatmulPreference_t pref = nullptr;
  if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) return HOA_ERR_LAUNCH;
  cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes,
                                       sizeof(ws_bytes));
  cublasLtMatmulHeuristicResult_t res[1];
  int found = 0;
  const cublasStatus_t st =
      cublasLtMatmulAlgoGetHeuristic(g_handle, p.op, p.a, p.b, p.d, p.d, pref, 1, res, &found);
  cublasLtMatmulPreferenceDestroy(pref);
  if (st != CUBLAS_STATUS_SUCCESS || found < 1) return HOA_ERR_UNSUPPORTED;
  p.algo = res[0].algo;
  p.ws = res[0].workspaceSize;
  return HOA_OK;
}
}  // namespace

extern "C" int hoa_edge_gemm_fp8_acc(const void* lo, const void* w, float* out, float alpha, int M, int N,
                                     int K, void* workspace, size_t workspace_bytes, void* stream) {
  if (!lo || !w || !out || M < 1 || N < 1 || K < 1 || (workspace_bytes > 0 && !workspace))
    return HOA_ERR_INVALID_ARG;
  if ((K & 15) != 0 || (N & 15) != 0 || (M & 15) != 0) return HOA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_handle == nullptr && cublasLtCreate(&g_handle) != CUBLAS_STATUS_SUCCESS) return HOA_ERR_LAUNCH;
  const PlanKey key{M, N, K, 2, workspace_bytes};
  auto it = g_plans.find(key);
  if (it == g_plans.end()) {
    GemmPlan p;
    const int st = make_plan_fp8(p, M, N, K, workspace_bytes);
    if (st != HOA_OK) {
      destroy_plan(p);
      return st;
    }
    it = g_plans.emplace(key, p).first;
  }
  const GemmPlan& plan = it->second;
  const float one = 1.f;
  const cublasStatus_t st =
      cublasLtMatmul(g_handle, plan.op, &alpha, w, plan.a, lo, plan.b, &one, out, plan.d, out, plan.d,
                     &plan.algo, workspace, plan.ws, reinterpret_cast<cudaStream_t>(stream));
  return st == CUBLAS_STATUS_SUCCESS ? HOA_OK : HOA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// The edge MLP's hidden layer between its two GEMMs: g = GELU(h) (exact erf,
// nn.GELU(), core/attention_fast_chunked.py:56-58; evaluated as
// x * 0.5 * (1 + erf(x / sqrt 2)) in fp32, the expression PyTorch's GELU uses),
// written as the bf16 operand of the second GEMM: [g_hi] or, split, [g_hi | g_lo]
// with g_hi = bf16(g) and g_lo = bf16(g - g_hi).  One pass over h instead of a
// GELU pass, a rounding copy and (split) a subtraction and a second copy.
namespace {

__global__ void edge_gelu_split_kernel(const float* __restrict__ h, __nv_bfloat16* __restrict__ out,
                                       long long rows, int cols, int split) {
  const int c4 = cols >> 2;
  const long long n4 = rows * c4;
  const float kAlpha = 0.70710678118654752440f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / c4;
    const int c = (int)(i % c4) * 4;
    const float4 x = *reinterpret_cast<const float4*>(h + r * cols + c);
    const float xv[4] = {x.x, x.y, x.z, x.w};
    uint32_t hw[4], lw[4];                           // bf16 bit patterns
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = xv[k] * 0.5f * (1.0f + erff(xv[k] * kAlpha));
      const __nv_bfloat16 hb = __float2bfloat16_rn(g);
      hw[k] = __bfloat16_as_ushort(hb);
      lw[k] = __bfloat16_as_ushort(__float2bfloat16_rn(g - __bfloat162float(hb)));
    }
    const long long ld = split ? 2LL * cols : cols;
    __nv_bfloat16* o = out + r * ld + c;
    *reinterpret_cast<uint2*>(o) = make_uint2(hw[0] | (hw[1] << 16), hw[2] | (hw[3] << 16));
    if (split)
      *reinterpret_cast<uint2*>(o + cols) = make_uint2(lw[0] | (lw[1] << 16), lw[2] | (lw[3] << 16));
  }
}

}  // namespace

extern "C" int hoa_edge_gelu_split(const float* h, void* out, long long rows, int cols, int split,
                                   void* stream) {
  if (!h || !out || rows < 1 || cols < 4 || (cols & 3) != 0) return HOA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) & 15) != 0 || (reinterpret_cast<uintptr_t>(out) & 7) != 0)
    return HOA_ERR_INVALID_ARG;
  const long long n4 = rows * (cols >> 2);
  long long blocks = (n4 + 255) / 256;
  if (blocks > 148LL * 64) blocks = 148LL * 64;
  edge_gelu_split_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      h, static_cast<__nv_bfloat16*>(out), rows, cols, split ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? HOA_OK : HOA_ERR_LAUNCH;
}

// The same hidden layer for the fp8 form: g_hi = bf16(g) (rows x cols, bf16) and the remainder
// g - g_hi, which is at most 2^-9 |g|, times lo_scale (a power of two) in e4m3 with saturation
// (rows x cols, one byte each), the operand of hoa_edge_gemm_fp8_acc.
namespace {

__global__ void edge_gelu_split8_kernel(const float* __restrict__ h, __nv_bfloat16* __restrict__ hi,
                                        uint8_t* __restrict__ lo, long long rows, int cols, float lo_scale) {
  const int c4 = cols >> 2;
  const long long n4 = rows * c4;
  const float kAlpha = 0.70710678118654752440f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / c4;
    const int c = (int)(i % c4) * 4;
    const float4 x = *reinterpret_cast<const float4*>(h + r * cols + c);
    const float xv[4] = {x.x, x.y, x.z, x.w};
    uint32_t hw[4], lw = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = xv[k] * 0.5f * (1.0f + erff(xv[k] * kAlpha));
      const __nv_bfloat16 hb = __float2bfloat16_rn(g);
      hw[k] = __bfloat16_as_ushort(hb);
      const __nv_fp8_storage_t l8 =
          __nv_cvt_float_to_fp8((g - __bfloat162float(hb)) * lo_scale, __NV_SATFINITE, __NV_E4M3);
      lw |= (uint32_t)l8 << (8 * k);
    }
    *reinterpret_cast<uint2*>(hi + r * cols + c) = make_uint2(hw[0] | (hw[1] << 16), hw[2] | (hw[3] << 16));
    *reinterpret_cast<uint32_t*>(lo + r * cols + c) = lw;
  }
}

}  // namespace

extern "C" int hoa_edge_gelu_split8(const float* h, void* hi, void* lo, long long rows, int cols,
                                    float lo_scale, void* stream) {
  if (!h || !hi || !lo || rows < 1 || cols < 4 || (cols & 3) != 0 || !(lo_scale > 0.f))
    return HOA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(h) & 15) != 0 || (reinterpret_cast<uintptr_t>(hi) & 7) != 0 ||
      (reinterpret_cast<uintptr_t>(lo) & 3) != 0)
    return HOA_ERR_INVALID_ARG;
  const long long n4 = rows * (cols >> 2);
  long long blocks = (n4 + 255) / 256;
  if (blocks > 148LL * 64) blocks = 148LL * 64;
  edge_gelu_split8_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      h, static_cast<__nv_bfloat16*>(hi), static_cast<uint8_t*>(lo), rows, cols, lo_scale);
  return cudaGetLastError() == cudaSuccess ? HOA_OK : HOA_ERR_LAUNCH;
}
