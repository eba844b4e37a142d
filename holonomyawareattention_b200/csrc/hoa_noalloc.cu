// hoa_core_forward_noalloc: the core region for callers that cannot allocate
// device memory at call time (for example an inference-engine plugin whose
// enqueue callback must not call cudaMalloc, or a process whose device memory
// is reserved in full by another allocator).  It runs exactly the kernels of
// hoa_core_forward; only the scratch differs: it lives in a static device
// array compiled into this file, so nothing is allocated per call.
//
// Limits and sharing, stated for users:
//   * the array holds HOA_NOALLOC_SCRATCH_BYTES (16 MiB); every GPU on which
//     this part of the library is loaded keeps it until the process exits;
//   * problems that need more scratch (hoa_core_workspace_bytes) are rejected
//     with HOA_ERR_WORKSPACE before any GPU work is enqueued;
//   * all calls on a device share the one array and it keeps the last call's
//     contents; the status word at its start is cleared by every call, and
//     every other byte a call reads was written earlier in the same call.
//     Calls that overlap on the GPU (different streams, or several host
//     threads) race on the array: serialise them;
//   * the status word (0, or HOA_ERR_TIMEOUT when a bounded device-side wait
//     gave up) is at hoa_noalloc_status_word(): read it once the call's stream
//     has completed, before the next call on that device clears it.
#include <cuda.h>

#include <mutex>

#include "hoa_common.cuh"

static __device__ __align__(256) unsigned char g_noalloc_scratch[HOA_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};   // context the cached address belongs to

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the current CUDA context (0 when it cannot be read).  A device
// reset destroys the context and the module with the array; the next context
// gets a new id, so the cached address is looked up again.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur == nullptr || get_id == nullptr || get_cur(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of g_noalloc_scratch on the current device.  Host code may
// not use the array's name as a device pointer (it names a host-side stand-in),
// so the address is looked up with that device current (cudaGetSymbolAddress)
// the first time a device (or a new context on it, after a reset) is seen, and
// cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HOA_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return HOA_ERR_UNSUPPORTED;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    // (also makes the device's primary context current if no call has yet)
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return HOA_ERR_LAUNCH;
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = current_context_id();
  }
  *out = g_noalloc_ptr[dev];
  return HOA_OK;
}
}  // namespace

extern "C" int hoa_noalloc_status_word(int** dev_status) {
  if (dev_status == nullptr) return HOA_ERR_INVALID_ARG;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != HOA_OK) return st;
  // hoa_core_forward keeps its status word in the first bytes of its workspace
  *dev_status = static_cast<int*>(scratch);
  return HOA_OK;
}

extern "C" int hoa_core_forward_noalloc(const void* a_all, int a_dtype, const float* a_bias,
                                        float edge_scale,
                                        const void* qkv, int qkv_dtype, void* out, int out_dtype,
                                        int hat_dtype, float softmax_scale, const float* carry_in,
                                        float* total_out, int B, int H, int T, int d, int chunk,
                                        void* stream) {
  if (!a_all || !qkv || !out || B < 1 || H < 1 || T < 1 || d < 1 || chunk < 1)
    return HOA_ERR_INVALID_ARG;
  const size_t need = hoa_core_workspace_bytes(B, H, T, d, chunk, hat_dtype);
  if (need == 0) return HOA_ERR_INVALID_ARG;
  if (need > (size_t)HOA_NOALLOC_SCRATCH_BYTES) return HOA_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != HOA_OK) return st;
  return hoa_core_forward(a_all, a_dtype, a_bias, edge_scale, qkv, qkv_dtype, out, out_dtype, hat_dtype,
                          softmax_scale, carry_in, total_out, B, H, T, d, chunk, scratch,
                          (size_t)HOA_NOALLOC_SCRATCH_BYTES, stream);
}
