// hoa_edge_gemm: the second layer of the edge MLP, a = hidden W^T + bias, as one
// cuBLASLt GEMM (bf16 operands, fp32 accumulation and output) whose epilogue
// adds the fp32 bias — a plain library GEMM (core/attention_fast_chunked.py:76).
// Row-major operands are handed to cuBLASLt (column-major) as their transposes:
// the row-major M x N result is the column-major N x M product D_cm = A_cm B_cm
// with A_cm = wt (row-major K x N) viewed as N x K (leading dimension N) and
// B_cm = hidden (row-major M x K) viewed as K x M (leading dimension K); the
// bias runs along D_cm's rows (length N).
#include <cublasLt.h>

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
using PlanKey = std::tuple<int, int, int, bool, size_t>;  // M, N, K, bias, workspace bytes
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
  const PlanKey key{M, N, K, bias != nullptr, workspace_bytes};
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
