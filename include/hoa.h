/*
 * hoa.h — C ABI of the B200 (sm_100a) path-ordered geometric attention forward.
 *
 * The library (libhoa.so) implements the causal forward of
 * PathOrderedGeometricMHA from SiddhiMali/HolonomyAwareAttention between the
 * PyTorch projections: it takes the edge-MLP output a_all and the qkv
 * projection, and returns the per-head outputs that feed the `out` Linear.
 *
 *   G_t  = expm(skew(edge_scale * a_t))          t = 0 .. T-2   (edge t joins t, t+1)
 *   P_0  = I,  P_{t+1} = G_t P_t
 *   q^_t = P_t^T q_t,  k^_t = P_t^T k_t,  v^_t = P_t^T v_t
 *   o_i  = P_i * sum_{j<=i} softmax_j(q^_i . k^_j * softmax_scale) v^_j
 *
 * Layout conventions (row-major, contiguous):
 *   a_all  (B, T, H, m)    m = d(d-1)/2, row-major strict upper triangle per head
 *   qkv    (B, T, H, 3d)   per head [q | k | v]  (the reference's qkv(x).view(B,T,H,3d))
 *   out    (B, T, H, d)    i.e. the (B, T, D) input of the `out` projection
 *   chain c = b*H + h.  Rotations are always fp32.
 *
 * Rules of the ABI: no entry point allocates or synchronises; all work is
 * enqueued on the caller's stream (`stream` is a cudaStream_t, NULL = legacy
 * default stream).  Scratch comes from the caller through `workspace`
 * (hoa_core_workspace_bytes).  Every entry point returns a hoa_status.
 *
 * Process-wide state (everything else keeps none, and may be called from
 * several host threads on different data):
 *   - hoa_edge_gemm and hoa_edge_gemm_fp8_acc keep one cuBLASLt handle and a
 *     plan per GEMM shape, and serialise their calls with a lock;
 *   - hoa_core_forward_noalloc computes in one static device array per GPU,
 *     shared by all its calls (see there), and caches that array's address
 *     per device;
 *   - hoa_set_wait_bound sets the bound of the device-side waits of every
 *     kernel launched after it (a diagnostic; the default is seconds).
 * Kernels whose bounded waits can give up report HOA_ERR_TIMEOUT through a
 * device status word (hoa_core_forward: the first 4 bytes of the workspace;
 * the stage entry points: their `status` argument).  The status of a launch is
 * known only once its stream has completed: read the word then.
 */
#ifndef HOA_H_
#define HOA_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HOA_OK = 0,
  HOA_ERR_INVALID_ARG = 1,   /* null pointer, bad shape, misaligned pointer */
  HOA_ERR_UNSUPPORTED = 2,   /* head dim or dtype outside the compiled set  */
  HOA_ERR_LAUNCH = 3,        /* CUDA launch failed (cudaGetLastError)       */
  HOA_ERR_WORKSPACE = 4,     /* workspace too small                          */
  HOA_ERR_TIMEOUT = 5,       /* a bounded device-side wait gave up           */
  HOA_ERR_BOUNDS = 6         /* debug build: a device-side index check failed */
} hoa_status;

typedef enum { HOA_F32 = 0, HOA_BF16 = 1 } hoa_dtype;

/*
 * Generator layout flag, OR'ed into `a_dtype` (with HOA_F32 only, for head
 * dims d % 32 == 0).  Without it the d(d-1)/2 generators of a head are packed
 * as the reference packs them: the strict upper triangle row by row
 * (core/utils.py skew_from_vec; entry (i, j), i < j, at i(2d-i-1)/2 + j-i-1).
 * With it each head holds hoa_gen_stride(d, 1) floats and entry {i, j} sits at
 * slot 32k + ((i + j) mod 32): a permutation of the same values (plus a few
 * unused slots) chosen so that the link kernel reads each row of the skew
 * matrix from shared memory without bank conflicts.  A caller gets this layout
 * for free by permuting the output rows of the generator projection once
 * (hoa_gen_banked_map).  Both layouts give bit-identical results.
 */
#define HOA_GEN_BANKED 0x100

/* Library facts. */
int hoa_abi_version(void);
int hoa_max_head_dim(void);
const char* hoa_status_string(int status);

/* Chunk length used to split each (b,h) rotation chain into independent
 * chunks (composed locally, then joined by hoa_carry_scan).  `num_sms` is the
 * device's SM count.  Returns a length in [16, T] (T when T < 16) chosen so
 * that the link kernel's (chain, chunk) units fill whole waves of the GPU. */
int hoa_plan_chunk(int B, int H, int T, int d, int num_sms);

/*
 * The edge MLP's hidden layer as the bf16 operand of hoa_edge_gemm:
 * g = GELU(h) (exact erf, nn.GELU(); core/attention_fast_chunked.py:56-58) for
 * h (rows, cols) fp32, written as out (rows, cols) = bf16(g), or with split
 * (rows, 2 cols) = [bf16(g) | bf16(g - bf16(g))].  cols % 4 == 0, h 16-byte
 * aligned.  No reference counterpart beyond the GELU itself.
 */
int hoa_edge_gelu_split(const float* h, void* out, long long rows, int cols, int split, void* stream);

/* Floats per head of the generator row: d(d-1)/2 (banked = 0) or the banked
 * layout's size (banked = 1; 0 when d % 32 != 0). */
int hoa_gen_stride(int d, int banked);

/* slot_of_index[i] (i < d(d-1)/2, reference order) = the banked slot of
 * reference entry i.  Returns HOA_ERR_UNSUPPORTED when d % 32 != 0. */
int hoa_gen_banked_map(int d, int* slot_of_index);

/* Bytes of scratch hoa_core_forward needs.  The first 4 bytes of the
 * workspace receive a device status word (0, or HOA_ERR_TIMEOUT when a
 * bounded device-side wait gave up); read it after the stream completes. */
size_t hoa_core_workspace_bytes(int B, int H, int T, int d, int chunk, int hat_dtype);

/*
 * Whole core region in one call: kernels (1)-(4).
 * Replaces the reference's core region between the projections:
 *   core/attention_fast_chunked.py:86-95   so_exp(skew_from_vec(a)) + prefix loop
 *   core/attention_fast_chunked.py:108-110 transport q^, k^, v^
 *   core/attention_fast_chunked.py:119-171 causal fold and out_i = P_i o_i
 * (kernel/attention_kernel.py:215-216 `_geometry` + `HoloAttnFn.apply`).
 * a_dtype / qkv_dtype / out_dtype: HOA_F32 or HOA_BF16.  `a_bias` (nullable,
 * (H*m) fp32) is added to every generator before the edge_scale multiply — the
 * edge MLP's output bias, so that the projection GEMM may leave it out
 * (core/attention_fast_chunked.py:76-77).  hat_dtype is the
 * dtype of the transported q^/k^/v^ fed to attention: HOA_BF16 runs the
 * tcgen05 tensor-core attention (d % 8 == 0, d <= 128), HOA_F32 the fp32 SIMT
 * attention.  `carry_in` (nullable, (B*H, d, d) fp32) is P at the first
 * position (a previous shard's product; NULL = identity); `total_out`
 * (nullable, (B*H, d, d)) receives the product through the last edge
 * t = T-1 (for a full sequence that edge is the closing edge, and total_out
 * is the holonomy G_close P_{T-1}, core/attention_fast_chunked.py:95).
 */
int hoa_core_forward(const void* a_all, int a_dtype, const float* a_bias, float edge_scale,
                     const void* qkv, int qkv_dtype,
                     void* out, int out_dtype, int hat_dtype, float softmax_scale,
                     const float* carry_in, float* total_out,
                     int B, int H, int T, int d, int chunk,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Kernels (1)+(2), local part: per (chain, chunk) unit, builds
 * G_t = expm(skew(edge_scale*a_t)) in fp32 and the local products
 * R_{t0} = I, R_{t+1} = G_t R_t over the chunk's edges.
 * Writes R (B*H, T, d, d) fp32 — R_t for every position —, the locally
 * transported vectors U (B*H, T, 3, d) fp32 = R_t^T [q_t, k_t, v_t], and the
 * chunk totals M (B*H, K, d, d) = R after the chunk's last edge.
 * `status` (nullable device int) receives HOA_ERR_TIMEOUT if a bounded
 * device-side wait gave up (the word is only ever set, never cleared).
 * Replaces core/attention_fast_chunked.py:86-94 (with core/utils.py:4-52)
 * and the transport at :108-110, split into independent chunks.
 */
int hoa_link_local(const void* a_all, int a_dtype, const float* a_bias, float edge_scale,
                   const void* qkv, int qkv_dtype,
                   float* R, float* U, float* M, int* status,
                   int B, int H, int T, int d, int chunk, void* stream);

/*
 * Kernel (2), carry: C_0 = carry_in (or I), C_{k+1} = M_k C_k for the K
 * chunks of each chain; writes C (B*H, K, d, d) and, if total_out != NULL,
 * C_K.  Joins the chunks so that P_t = R_t C_{t/chunk}
 * (core/attention_fast_chunked.py:91-94 re-associated).
 */
int hoa_carry_scan(const float* M, const float* carry_in, float* C, float* total_out,
                   int BH, int K, int d, void* stream);

/*
 * Kernel (2), transport: q^_t = C_k^T U_q[t] (likewise k, v) in hat_dtype.
 * q^, k^: (B*H, T, d).  v^: (B*H, T, d) when vt_stride == 0, else transposed
 * as (B*H, d, vt_stride) with vt_stride = hoa_vt_stride(T) (the layout
 * hoa_attn_tc_fwd reads).  Completes core/attention_fast_chunked.py:108-110.
 */
int hoa_carry_apply(const float* U, const float* C, void* qh, void* kh, void* vh,
                    int hat_dtype, int vt_stride, int BH, int T, int d, int chunk,
                    void* stream);

/* Row stride (elements) of the transposed v^ buffer: T rounded up to 8. */
int hoa_vt_stride(int T);

/*
 * Kernel (3), fp32 path: causal online-softmax attention with every product
 * in fp32.  q^ is (B*H, Tq, d), k^ and v^ (B*H, Tk, d), in fp32 (or bf16).
 * Query row i is global position q_offset + i and attends to keys
 * 0 .. q_offset + i (q_offset + Tq <= Tk; a whole sequence is Tq = Tk,
 * q_offset = 0; a sequence shard passes its offset and the gathered keys).
 * Writes the normalised o = softmax(q^ k^T * scale) v^ as (B*H, Tq, d) fp32.
 * Replaces core/attention_fast_chunked.py:119-168 (kernel/attention_kernel.py:122-134
 * run_fwd_kernel) for the causal tril mask.
 */
int hoa_attn_fwd(const void* qh, const void* kh, const void* vh, int hat_dtype,
                 float* o, float softmax_scale, int BH, int Tq, int Tk, int q_offset,
                 int d, void* stream);

/*
 * Kernel (3), bf16 path on tcgen05/TMEM: same contract as hoa_attn_fwd with
 * bf16 q^ (B*H, Tq, d), k^ (B*H, Tk, d) and v^ transposed
 * (B*H, d, hoa_vt_stride(Tk)); fp32 accumulation.  d % 8 == 0, d <= 128.
 * `status` (nullable device int) receives HOA_ERR_TIMEOUT if a bounded wait
 * gave up.
 */
int hoa_attn_tc_fwd(const void* qh, const void* kh, const void* vhT, float* o, int* status,
                    float softmax_scale, int BH, int Tq, int Tk, int q_offset, int d,
                    void* stream);

/*
 * The path products P_t = R_t C_{t/chunk} (B*H, T, d, d) in p_dtype, from the
 * link kernel's R and the carry scan's C: the "C" entry of the reference's
 * forward(..., return_geometry=True) (core/attention_fast_chunked.py:89-94,
 * 175-177; its "H" entry, the holonomy, is hoa_carry_scan's total_out).  Not on
 * the forward's path, which never materialises P.
 */
int hoa_compose_paths(const float* R, const float* C, void* P, int p_dtype, int BH, int T, int d,
                      int chunk, void* stream);

/*
 * General forms of the module (core/attention.py:69-195) beside the causal
 * tril path, all fp32, (B*H, T, d) row-major vectors:
 *
 * hoa_attn_general_fwd — softmax over all keys of a chain: o_i =
 *   sum_j softmax_j(q^_i . key_ij * scale) value_ij / l.clamp_min(1e-20), with
 *   key/value_ij = k^_j / v^_j for j <= i and, when kw/vw are given (both or
 *   neither), kw_j / vw_j for the wrap pairs j > i (the arc transport through
 *   the closing edge, core/attention.py:156-165: kw = Hol k^, vw = Hol v^).
 *   mask: (T, T) bytes, nonzero = allowed, NULL = all allowed; masked scores
 *   sit at -FLT_MAX as the reference's finfo.min (a fully masked row averages
 *   uniformly, core/attention_fast_chunked.py:142-148).  d <= 128.
 * hoa_chain_matvec — y_t = M x_t (transpose = 0) or M^T x_t, M (B*H, d, d).
 * hoa_apply_paths — y_t = P_t x_t (transpose = 0) or P_t^T x_t with
 *   P_t = R_t C_{t/chunk} (the inert ablation's transports,
 *   core/attention.py:166-169).
 */
int hoa_attn_general_fwd(const float* qh, const float* kh, const float* vh, const float* kw,
                         const float* vw, const unsigned char* mask, float* o, float softmax_scale,
                         int BH, int T, int d, void* stream);
int hoa_chain_matvec(const float* x, const float* M, float* y, int transpose, int BH, int T, int d,
                     void* stream);
int hoa_apply_paths(const float* x, const float* R, const float* C, int chunk, float* y, int transpose,
                    int BH, int T, int d, void* stream);

/*
 * Kernel (4): inverse transport out_t = R_t (C_{t/chunk} o_t), written to
 * out (B, T, H, d) in out_dtype — the input of the `out` projection.
 * Replaces core/attention_fast_chunked.py:171.
 */
int hoa_out_transport(const float* o, const float* R, const float* C, int chunk,
                      void* out, int out_dtype, int B, int H, int T, int d, void* stream);

/* Size of the static scratch behind hoa_core_forward_noalloc: 16 MiB. */
#define HOA_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/*
 * hoa_core_forward_noalloc — no counterpart in the reference.  Same
 * computation and arguments as hoa_core_forward minus the workspace, for
 * callers that cannot allocate device memory when they call in (for example
 * an inference-engine plugin whose enqueue callback must not call cudaMalloc,
 * or a process whose device memory is reserved in full by another allocator).
 * Its scratch is a static device array of HOA_NOALLOC_SCRATCH_BYTES inside
 * the library, which every GPU that loads it keeps until the process exits;
 * nothing is allocated per call.  Problems whose hoa_core_workspace_bytes
 * exceeds that size return HOA_ERR_WORKSPACE without enqueuing work.
 * It runs on the current device, and `stream` must belong to that device.
 * The first call on each device (and the first after a device reset, which
 * gives the device a new context) looks up the array's device address
 * (cudaGetSymbolAddress) and caches it, so make that first call before any
 * stream capture.  All calls share the array and it keeps the last call's
 * contents: calls that overlap on the GPU (other streams, other host
 * threads) race on it, so serialise them.  The call's device status word
 * (0, or HOA_ERR_TIMEOUT when a bounded device-side wait gave up) is cleared
 * at the start of every call and lies in the array: hoa_noalloc_status_word.
 */
int hoa_core_forward_noalloc(const void* a_all, int a_dtype, const float* a_bias,
                             float edge_scale,
                             const void* qkv, int qkv_dtype,
                             void* out, int out_dtype, int hat_dtype, float softmax_scale,
                             const float* carry_in, float* total_out,
                             int B, int H, int T, int d, int chunk, void* stream);

/*
 * hoa_noalloc_status_word — no counterpart in the reference.  The device
 * address, on the current device, of the status word that the last
 * hoa_core_forward_noalloc call on that device wrote: read it (4 bytes, e.g.
 * with cudaMemcpy) once that call's stream has completed.  Allocates nothing;
 * like hoa_core_forward_noalloc, its first call on a device does the address
 * look-up, so make it before any stream capture.
 */
int hoa_noalloc_status_word(int** dev_status);

/*
 * hoa_set_wait_bound — no counterpart in the reference.  A diagnostic: the
 * bound, in SM cycles, of the device-side waits (on TMA and tensor-core
 * completion) of every kernel launched after the call, process-wide.
 * 0 restores the default (4e9 cycles, i.e. seconds); the maximum is the
 * default.  A short bound makes a real forward's waits give up: the kernels
 * then leave early without faulting (each waits, with the default bound, for
 * its copies and products in flight, frees its tensor memory and returns) and
 * report HOA_ERR_TIMEOUT in their status word; the output is not valid.
 */
int hoa_set_wait_bound(long long max_cycles);

/*
 * hoa_debug_bounds — no counterpart in the reference.  Device-side index
 * checks of the debug build (libhoa_debug.so, built with -DHOA_DEBUG_BOUNDS;
 * compute-sanitizer is not available where this library is tested).  In that
 * build every kernel of the core path checks, before each global access, that
 * the element range a unit (a position, a chunk, a row) touches lies inside
 * the extent its buffer has for the launch's shape; a check that fails
 * records HOA_ERR_BOUNDS and the access is skipped (never performed; a
 * skipped TMA copy completes its barrier with zero bytes), so nothing faults
 * or traps.  The call returns in *status (host int) the first code recorded
 * since the previous call on this device (0 if none) and clears it, after
 * waiting for the device to finish; it then sets every check to compare
 * against extents shifted right by `extent_shift` (0 = the true extents; a
 * test hook: 1 makes the checks treat every buffer as half as long, so they
 * fire on accesses that are really in bounds).  The product build returns
 * HOA_ERR_UNSUPPORTED.
 */
int hoa_debug_bounds(int extent_shift, int* status);

/*
 * hoa_edge_gemm — the second layer of the edge MLP (core/attention_fast_chunked.py:76,
 * `edge_mlp[2]`, whose output is the a_all of hoa_core_forward) as one cuBLASLt GEMM, a plain
 * library GEMM: out (M x N, fp32, row-major) = hidden (M x K, bf16, row-major) * wt (K x N,
 * bf16, row-major, i.e. W^T) + bias (N floats, nullable), fp32 accumulation, the bias added in
 * the GEMM's epilogue.  workspace: caller-owned cuBLASLt scratch (32 MiB is plenty).  The plan
 * of each shape is made once and cached; calls are serialised inside the library.
 */
int hoa_edge_gemm(const void* hidden, const void* wt, const float* bias, float* out, int M, int N,
                  int K, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The low half of the edge MLP's second layer in fp8 (the same layer as hoa_edge_gemm,
 * core/attention_fast_chunked.py:76; the reference computes it in one fp32 GEMM): with
 * g = g_hi + g_lo, g_hi = bf16(g), the layer is W g_hi + W g_lo; the first term is a bf16
 * hoa_edge_gemm and the second, whose terms are at most 2^-9 of the first's, this call:
 *   hoa_edge_gelu_split8: g = GELU(h) (exact erf) for h (rows, cols) fp32 -> hi (rows, cols)
 *     = bf16(g) and lo (rows, cols) = e4m3(lo_scale * (g - bf16(g))), saturating (one byte
 *     each); cols % 4 == 0, h 16-byte aligned, lo_scale > 0 (a power of two keeps it exact);
 *   hoa_edge_gemm_fp8_acc: out (M x N, fp32, row-major) += alpha * lo (M x K, e4m3,
 *     row-major) * w^T, w (N x K, e4m3, row-major: the weight as nn.Linear stores it), fp32
 *     accumulation; alpha undoes the two operands' scales.  M, N, K multiples of 16.
 * The plan of each shape is made once and cached; calls are serialised inside the library.
 */
int hoa_edge_gelu_split8(const float* h, void* hi, void* lo, long long rows, int cols, float lo_scale,
                         void* stream);
int hoa_edge_gemm_fp8_acc(const void* lo, const void* w, float* out, float alpha, int M, int N, int K,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * hoa_selftest_wait — no counterpart in the reference.  Diagnostic for the
 * bounded device-side waits every kernel of this library uses (mbarrier waits
 * on TMA and tensor-core completion): one CTA of two warps waits on two
 * mbarriers that nothing arrives at.  Warp 0 waits with a bound of max_cycles
 * SM cycles, gives up and raises the CTA's abort flag; warp 1 waits with the
 * library's full bound (seconds) but on the abort flag as well, so it must
 * give up as soon as warp 0 does.  Results, written to out[0..3] (device,
 * 4 ints): out[0] = HOA_ERR_TIMEOUT when warp 0 gave up, out[1] = 1 when
 * warp 1 left on the abort flag, out[2] = warp 1's wait in units of 1024
 * cycles, out[3] = 1 when both waits returned false.  Nothing faults or hangs:
 * the GPU context stays usable.  max_cycles must be in [1, 1e9].
 */
int hoa_selftest_wait(int* out, long long max_cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HOA_H_ */
