// Shared helpers for the path-ordered geometric attention kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/hoa.h"

#define HOA_DEVICE __device__ __forceinline__
#define HOA_HD __host__ __device__ __forceinline__

namespace hoa {

// element loads / stores for the two activation types the ABI accepts
HOA_DEVICE float load_elem(const void* p, long long i, int dtype) {
  if (dtype == HOA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

HOA_DEVICE void store_elem(void* p, long long i, int dtype, float v) {
  if (dtype == HOA_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

inline int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// ---- debug bounds checks (libhoa_debug.so, -DHOA_DEBUG_BOUNDS) ----------------
// HOA_IN(first, count, extent): the element range [first, first + count) lies in
// [0, extent) (extent shifted right by the test hook of hoa_debug_bounds).  In
// the debug build a failed check records HOA_ERR_BOUNDS in this translation
// unit's debug word and the caller skips the access; the product build compiles
// every check to `true`.
#ifdef HOA_DEBUG_BOUNDS
static __device__ int g_hoa_dbg_status;
static __device__ int g_hoa_dbg_shift;
HOA_DEVICE bool dbg_in(long long first, long long count, long long extent) {
  if (first >= 0 && count >= 0 && first + count <= (extent >> g_hoa_dbg_shift)) return true;
  atomicCAS(&g_hoa_dbg_status, 0, HOA_ERR_BOUNDS);
  return false;
}
#define HOA_IN(first, count, extent) \
  ::hoa::dbg_in((long long)(first), (long long)(count), (long long)(extent))
// Each translation unit registers a host function that reads and clears its
// debug word and sets its extent shift (hoa_debug_bounds calls them all).
using DbgSyncFn = int (*)(int shift, int* status);
void dbg_register(DbgSyncFn fn);
namespace {
int dbg_sync_tu(int shift, int* status) {
  int st = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&st, g_hoa_dbg_status, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_hoa_dbg_status, &zero, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_hoa_dbg_shift, &shift, sizeof(int)) != cudaSuccess)
    return HOA_ERR_LAUNCH;
  if (st != 0 && *status == 0) *status = st;
  return HOA_OK;
}
struct DbgRegistration {
  DbgRegistration() { dbg_register(dbg_sync_tu); }
};
DbgRegistration g_dbg_registration;
}  // namespace
#else
#define HOA_IN(first, count, extent) true
#endif

// Bound, in SM cycles, of the abortable device-side waits of the kernels
// launched from now on (hoa_set_wait_bound; the library default unless a test
// shortened it).  Defined in hoa_link.cu.
long long wait_bound_cycles();

// Record the first device-side failure so that the host can read it later.
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HOA_OK : HOA_ERR_LAUNCH;
}

// Smallest supported padded head dimension >= d, or 0.
inline int padded_dim(int d) {
  static const int dims[] = {8, 16, 32, 48, 64, 96, 120};
  for (int p : dims)
    if (d <= p) return p;
  return 0;
}

// ---- generator layouts (HOA_GEN_BANKED) ----------------------------------
// d = 32 nb.  The d x d skew matrix splits into nb x nb blocks of 32; entry
// {i, j} has i in block a, j in block b, a <= b, offsets u = i mod 32 and
// v = j mod 32.  The slots are laid out for the link kernel's reads, where a
// warp holds 32 consecutive rows r and walks the columns c of one block:
// * off-diagonal pair (a < b), bp its row-major index among the pairs a < b:
//   line 32 bp + u (32 slots) holds row u's entries, entry v at position
//   v ^ 4 (u mod 8).  The warp of the upper rows (r in block a) reads each
//   lane's own line with 16-byte loads, 8 lanes hitting 8 distinct 16-byte bank
//   groups; the warp of the lower rows (r in block b) reads one whole line per
//   column (positions lane ^ const), one access per column.
// * diagonal block: slot 32 k + s with bank s = (u + v) mod 32, 16 slots per
//   bank (15 for even s; one unused).  Within a bank the entries are the pairs
//   {u, s - u}; with w = (u - ceil(s/2)) mod 32 the partner has 31 - w (odd s)
//   or 32 - w (even s), so min(w, partner) numbers the pairs (the w of u = v,
//   excluded, is 0 or 16).
HOA_HD int gen_banked_stride(int d) {
  if (d <= 0 || d % 32 != 0) return 0;
  const int nb = d / 32;
  return 1024 * (nb * (nb - 1) / 2) + 512 * nb;
}

// slot of the two offsets u != v of one diagonal block, within that block's range
HOA_HD int gen_banked_diag(int u, int v) {
  const int s = (u + v) & 31, e = s & 1;
  const int w = (u - ((s + 1) >> 1)) & 31;
  const int kd = (w < 32 - e - w ? w : 32 - e - w) - 1 + e;
  return kd * 32 + s;
}

HOA_HD int gen_banked_slot(int i, int j, int d) {   // i != j
  if (i > j) { const int t = i; i = j; j = t; }
  const int nb = d >> 5;
  const int a = i >> 5, b = j >> 5, u = i & 31, v = j & 31;
  if (a < b) {
    const int bp = a * nb - a * (a + 1) / 2 + (b - a - 1);
    return (bp * 32 + u) * 32 + (v ^ (4 * (u & 7)));
  }
  return ((nb * (nb - 1) / 2) * 32 + a * 16) * 32 + gen_banked_diag(u, v);
}

// a_dtype with the layout flag: the element type, and whether it is banked.
inline int gen_elem_dtype(int a_dtype) { return a_dtype & ~HOA_GEN_BANKED; }
inline bool gen_is_banked(int a_dtype) { return (a_dtype & HOA_GEN_BANKED) != 0; }
// Floats per head of the generator row, or 0 for an unsupported combination.
inline int gen_row_stride(int a_dtype, int d) {
  if (!gen_is_banked(a_dtype)) return d * (d - 1) / 2;
  return gen_elem_dtype(a_dtype) == HOA_F32 ? gen_banked_stride(d) : 0;
}

}  // namespace hoa
