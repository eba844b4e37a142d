// hoa_selftest_wait: exercises the bounded mbarrier waits (sm100::mbar_wait_abortable)
// that every kernel of the library relies on, on barriers that nothing arrives at.
// Warp 0 gives up after max_cycles and raises the CTA's abort flag; warp 1, bounded by
// the library's full limit, must then give up on the flag.
#include "hoa_sm100.cuh"

namespace hoa {
using namespace sm100;

__global__ void __launch_bounds__(64) selftest_wait_kernel(int* out, long long max_cycles) {
  __shared__ uint64_t bars[2];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lid = tid & 31;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* ab = &abort_flag;
  __shared__ int res[2];
  __shared__ long long w1_cycles;
  // every lane of a warp waits (no divergence before the barrier below)
  if (warp == 0) {
    const bool ok = mbar_wait_abortable(&bars[0], 0, ab, max_cycles);
    if (lid == 0) res[0] = ok ? 1 : 0;
  } else {
    const long long c0 = clock64();
    const bool ok = mbar_wait_abortable(&bars[1], 0, ab);
    const long long dt = clock64() - c0;
    if (lid == 0) {
      res[1] = ok ? 1 : 0;
      w1_cycles = dt;
    }
  }
  __syncwarp();
  __syncthreads();
  if (tid == 0) {
    out[0] = (res[0] == 0 && *ab != 0) ? HOA_ERR_TIMEOUT : HOA_OK;
    out[1] = (res[1] == 0 && *ab != 0) ? 1 : 0;
    out[2] = (int)min(w1_cycles >> 10, (long long)0x7fffffff);
    out[3] = (res[0] == 0 && res[1] == 0) ? 1 : 0;
  }
}

}  // namespace hoa

extern "C" int hoa_selftest_wait(int* out, long long max_cycles, void* stream) {
  if (out == nullptr || max_cycles < 1 || max_cycles > 1000000000ll) return HOA_ERR_INVALID_ARG;
  hoa::selftest_wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(out, max_cycles);
  return hoa::launch_status();
}
