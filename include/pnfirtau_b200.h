/*
 * pnfirtau_b200.h - C ABI of the B200-native pn_fir_tau attention operator.
 *
 * One shared library (libpnfirtau_b200.so) exports these entry points. Every
 * pointer is a DEVICE pointer unless stated otherwise, strides are in ELEMENTS,
 * the CUDA stream is passed as an opaque `void*` (a cudaStream_t) and comes
 * last. No entry point allocates device memory: outputs and workspaces are
 * owned by the caller (the reference's Python wrappers allocate with
 * torch.empty / torch.zeros and hand raw pointers to the kernels, which is the
 * convention kept here). All launches are asynchronous on `stream` and are
 * legal inside CUDA-graph capture.
 *
 * Return value of every entry point: PNFT_OK (0) on success, a negative
 * PNFT_E* code for invalid arguments or a CUDA launch error. The message of
 * the last failure on the calling thread is available from pnft_last_error().
 * Kernels that wait on hardware barriers write a positive PNFT_DEV_* code to
 * the caller's `status` word instead of hanging (device memory, read after a
 * synchronisation, or mapped pinned host memory, see pnft_mapped_status_ptr).
 *
 * Reference interface replaced (paths inside the reference project):
 *   src/triton_pnfirtau.py  - Triton kernels + autograd wrappers
 *   src/pnfirtau_attention.py - eager primitives (power_norm_peak_gate, causal_fir)
 */
#ifndef PNFIRTAU_B200_H
#define PNFIRTAU_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PNFT_API __attribute__((visibility("default")))
#else
#define PNFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types of the tensors handed to the kernels */
#define PNFT_DTYPE_F32 0
#define PNFT_DTYPE_BF16 1
#define PNFT_DTYPE_F16 2

/* host-side status codes */
#define PNFT_OK 0
#define PNFT_EINVAL (-1)       /* bad shape / stride / pointer / parameter */
#define PNFT_EUNSUPPORTED (-2) /* valid request this build cannot serve   */
#define PNFT_ECUDA (-3)        /* CUDA runtime / launch error              */

/* device-reported status codes (written to the caller's status word) */
#define PNFT_DEV_OK 0
#define PNFT_DEV_WAIT_TIMEOUT 1 /* a pipeline mbarrier wait hit its bound */
#define PNFT_DEV_BAD_INDEX 2    /* pnft_lm_xent: a target outside [0, V) (not ignore_index) */

/* silence modes of power_norm_peak_gate (src/pnfirtau_attention.py:108-116) */
#define PNFT_SILENCE_PEAK 0
#define PNFT_SILENCE_MASS_RELU 1
#define PNFT_SILENCE_MASS_POW 2

/* flags of the flash entry points */
#define PNFT_FLASH_FORCE_GENERIC 0x1 /* use the SIMT kernel even where tcgen05 applies */
/* Ordered dQ accumulation: the backward adds the dQ contributions of the key
 * tiles of each 64-row query tile in key order (per-tile turn counters in the
 * workspace, work taken in ticket order), so dq is bitwise reproducible run to
 * run; dk, dv, dtau and the FIR's dk / dtaps always are. Slower backward. */
#define PNFT_FLASH_DETERMINISTIC 0x2
#define PNFT_FLASH_PREFER_SM100 0x4  /* tcgen05 kernels wherever their shape rules allow */
/* Test-only: the tcgen05 kernels' elementwise warps make their first pipeline
 * wait on a barrier that nothing arrives on, so every CTA takes the timeout path
 * after the 1 s limit (status word set to PNFT_DEV_WAIT_TIMEOUT, the other roles
 * unwind, copies drain, TMEM is freed). The outputs of such a call are invalid.
 * No effect on the generic kernels. */
#define PNFT_FLASH_TEST_STALL 0x100

/* Tap count of the FIR fused into the flash kernels (pnft_flash_fwd_fir): the
 * module's causal filter on the keys, PnFirConfig.fir_k = 7
 * (src/pnfirtau_attention.py:35-47). */
#define PNFT_FIR_FUSED_TAPS 7

/* Library version (major*10000 + minor*100 + patch). */
PNFT_API int pnft_version(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads); lets callers attribute launches in a timed region. */
PNFT_API uint64_t pnft_launch_count(void);

/* Message of the last failed call on this thread ("" if none). Host pointer. */
PNFT_API const char* pnft_last_error(void);

/* Device capabilities relevant to kernel selection. Host pointers out.
 * has_sm100a: 1 if the device is compute capability 10.0 (the sm_100a cubins
 * of this library run on it). */
PNFT_API int pnft_query_caps(int device, int* cc_major, int* cc_minor, int* sm_count,
                    int* smem_optin_bytes, int* has_sm100a);

/* Device address of a status word in pinned host memory (cudaHostAlloc /
 * cudaMallocHost, which unified addressing maps into every device): the
 * kernels' `status` argument may be that address, so a failure they report is
 * visible to the host by reading the word, with no copy and no synchronisation.
 * Returns PNFT_EINVAL if host_word is not such memory. Host pointers in and out. */
PNFT_API int pnft_mapped_status_ptr(void* host_word, void** device_ptr);

/* ------------------------------------------------------------------------- */
/* Depthwise causal FIR along N of x[B,N,C]                                   */
/* ------------------------------------------------------------------------- */

/* y[b,n,c] = sum_{u<ntaps} taps[ntaps-1-u] * x[b,n-u,c]   (x[b,<0,c] = 0),
 * fp32 accumulation, y in the dtype of x. taps: fp32[ntaps], index ntaps-1 is
 * lag 0 (oldest lag first, as the reference's fir_taps buffer).
 * Replaces: src/triton_pnfirtau.py:40-87 (_causal_fir7_fwd_kernel) and its
 * launch in _TritonCausalFir7Fn.forward (:631-658); also the eager
 * causal_fir (src/pnfirtau_attention.py:65-74) for any ntaps <= 64. */
PNFT_API int pnft_fir_fwd(const void* x, int64_t sxb, int64_t sxn, int64_t sxc, const float* taps,
                 int ntaps, void* y, int64_t syb, int64_t syn, int64_t syc, int64_t B,
                 int64_t N, int64_t C, int dtype, void* stream);

/* Transpose (anti-causal) FIR: gx[b,n,c] = sum_u taps[ntaps-1-u] * gy[b,n+u,c].
 * If x != NULL, also the tap gradient dtaps[ntaps-1-u] = sum gy[b,n,c]*x[b,n-u,c],
 * reduced deterministically (fixed order, fp64) into dtaps (fp32[ntaps]).
 * `workspace` must hold pnft_fir_bwd_workspace_size(B,N,C,ntaps) bytes when
 * x != NULL (may be NULL otherwise). gx may be NULL to compute dtaps only.
 * Replaces: src/triton_pnfirtau.py:89-135 (_causal_fir7_bwd_kernel) and
 * _TritonCausalFir7Fn.backward (:660-682), which returns no tap gradient. */
PNFT_API int pnft_fir_bwd(const void* gy, int64_t sgb, int64_t sgn, int64_t sgc, const float* taps,
                 int ntaps, void* gx, int64_t sxb, int64_t sxn, int64_t sxc, const void* x,
                 int64_t s0b, int64_t s0n, int64_t s0c, float* dtaps, void* workspace,
                 size_t workspace_bytes, int64_t B, int64_t N, int64_t C, int dtype,
                 void* stream);

PNFT_API size_t pnft_fir_bwd_workspace_size(int64_t B, int64_t N, int64_t C, int ntaps);

/* pnft_fir_bwd with the tap gradient, for callers that cannot allocate device
 * memory on the library's behalf: code that runs while a stream is being
 * captured (cudaMalloc is not permitted then), serving loops that must never
 * enter the allocator after start-up, and foreign-language bindings that only
 * receive the input and output buffers from a host runtime owning all device
 * memory. The per-block partial sums that pnft_fir_bwd keeps in the caller's
 * workspace live instead in a static 128 KiB device array of the library,
 * which every GPU that loads the library holds until the process exits.
 * x and dtaps are required; gx may be NULL. ntaps above 64 is rejected with
 * PNFT_EINVAL. The first call on each device looks the array's address up
 * (make that first call before any stream capture). All calls share the
 * array, so calls that overlap on the GPU (other streams or threads) race;
 * each call overwrites every element it reads, so none needs clearing.
 * Results equal pnft_fir_bwd's. No counterpart in the reference (an addition
 * of this library). */
PNFT_API int pnft_fir_bwd_noalloc(const void* gy, int64_t sgb, int64_t sgn, int64_t sgc,
                                  const float* taps, int ntaps, void* gx, int64_t sxb, int64_t sxn,
                                  int64_t sxc, const void* x, int64_t s0b, int64_t s0n, int64_t s0c,
                                  float* dtaps, int64_t B, int64_t N, int64_t C, int dtype,
                                  void* stream);

/* ------------------------------------------------------------------------- */
/* Row-fused score -> weight op over R rows of length N                      */
/* ------------------------------------------------------------------------- */

/* For every row r (causal column limit t = r % N when causal != 0):
 *   s = raw*scale - tau[0]; u = relu(s) on valid columns; pw = u^p;
 *   strength = peak | sum u | sum pw (silence_mode); gate = strength/(strength+gamma)
 *   (1 when has_gamma == 0); w = pw * gate / (sum pw + 1e-12).
 * Stats (fp32/int32 [R]): stat_m = peak, stat_z = sum pw + 1e-12,
 * stat_nmax = #columns with u == peak, stat_strength = strength.
 * Silent rows (peak <= 0) write w = 0, M = 0, Z = 1e-12, Nmax = 0.
 * p: exponent; p == 10 and p == 2 use repeated multiplication, other p powf.
 * Replaces: src/triton_pnfirtau.py:141-212 (_pn_fir_tau_row_fwd_kernel) and
 * _TritonPnFirTauScoresFn.forward (:694-752); the silence modes other than
 * "peak" and general p follow power_norm_peak_gate (src/pnfirtau_attention.py:87-119). */
PNFT_API int pnft_rows_fwd(const void* raw, int64_t raw_row_stride, const float* tau, void* w,
                  int64_t w_row_stride, float* stat_m, float* stat_z, int32_t* stat_nmax,
                  float* stat_strength, int64_t R, int64_t N, float scale, float p,
                  float gamma, int has_gamma, int silence_mode, int causal, int dtype,
                  void* stream);

/* Analytic backward of pnft_rows_fwd: graw (dtype of raw) and the per-row
 * tau gradient dtau_rows (fp32 [R], = -sum_j du). If dtau != NULL the rows are
 * also reduced deterministically in fp64 into dtau[0] (fp32).
 * Replaces: src/triton_pnfirtau.py:214-303 (_pn_fir_tau_row_bwd_kernel) and
 * _TritonPnFirTauScoresFn.backward (:754-785). */
PNFT_API int pnft_rows_bwd(const void* gw, int64_t gw_row_stride, const void* raw,
                  int64_t raw_row_stride, const float* tau, const float* stat_m,
                  const float* stat_z, const int32_t* stat_nmax, const float* stat_strength,
                  void* graw, int64_t graw_row_stride, float* dtau_rows, float* dtau,
                  int64_t R, int64_t N, float scale, float p, float gamma, int has_gamma,
                  int silence_mode, int causal, int dtype, void* stream);

/* Deterministic fp64 sum of n fp32 values into out[0] (fp32). */
PNFT_API int pnft_sum_f32(const float* x, int64_t n, float* out, void* stream);

/* ------------------------------------------------------------------------- */
/* Flash pn_fir_tau attention (p = 10)                                       */
/* ------------------------------------------------------------------------- */

/* q,k,v: [B,H,N,D] with arbitrary 4-D element strides sq/sk/sv/so (host
 * arrays of 4 int64: b,h,n,d); out in the same dtype with strides so.
 * Stats stat_m/stat_z (fp32) and stat_nmax (int32) are contiguous [B,H,N];
 * stat_arg (int32 [B,H,N]) receives the first key index attaining each row's
 * peak (-1 for silent rows): the backward routes the gate gradient of a row
 * with a single maximum to that key, independently of how S is recomputed.
 * gamma is used when has_gamma != 0 (reference: gamma is not None and > 0).
 * out_f32 (optional, may be NULL): fp32 [B,H,N,D] contiguous copy of the
 * output before rounding to the input dtype; handing it to pnft_flash_bwd keeps
 * the per-row term <dO,O>/gate exact (u^10 rows are so peaked that dP - <dO,O>
 * cancels at the peak and would amplify bf16 rounding of O into the gradients).
 * tile_flags (optional, may be NULL): uint8 [B*H, ceil(N/64), ceil(N/64)],
 * zeroed by the caller; the kernel sets entry (bh, qi, kj) to 1 for every
 * 64x64 tile it processed as live (some u > 0) and leaves skipped silent
 * tiles and tiles above the causal diagonal at 0 - the silent-tile decisions
 * of experiments/exp4b_mha6_instrumentation.py:91-111.
 * status: int32 word the device can write (device memory, or mapped pinned host
 * memory, see pnft_mapped_status_ptr; may be NULL), set to PNFT_DEV_* if a
 * pipeline wait times out (never cleared by the library).
 * Replaces: src/triton_pnfirtau.py:313-443 (_flash_pn_fir_tau_fwd_kernel) and
 * _FlashPnFirTauFn.forward (:814-898). */
PNFT_API int pnft_flash_fwd(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                   const void* v, const int64_t* sv, const float* tau, void* out,
                   const int64_t* so, float* out_f32, float* stat_m, float* stat_z, int32_t* stat_nmax,
                   int32_t* stat_arg, int64_t B, int64_t H, int64_t N, int64_t D, float scale,
                   float gamma, int has_gamma, int causal, int dtype, int flags, uint8_t* tile_flags,
                   int32_t* status, void* stream);

/* Backward of pnft_flash_fwd. out_f32: the forward's fp32 output copy, or NULL
 * to use `out`. dout has strides sdo; dq/dk/dv (dtype of q)
 * strides sdq/sdk/sdv. dtau: fp32[1], the tau gradient reduced in fp64 in a
 * fixed order. workspace: pnft_flash_bwd_workspace_size(...) bytes (the fp32 dQ
 * accumulator, per-row coefficients and per-tile tau partials).
 * Replaces: src/triton_pnfirtau.py:445-621 (_flash_pn_fir_tau_bwd_kernel) and
 * _FlashPnFirTauFn.backward (:900-968). */
PNFT_API int pnft_flash_bwd(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                   const void* v, const int64_t* sv, const float* tau, const void* out,
                   const int64_t* so, const float* out_f32, const void* dout, const int64_t* sdo,
                   const float* stat_m, const float* stat_z, const int32_t* stat_nmax,
                   const int32_t* stat_arg, void* dq, const int64_t* sdq, void* dk, const int64_t* sdk, void* dv,
                   const int64_t* sdv, float* dtau, void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t H, int64_t N, int64_t D, float scale, float gamma,
                   int has_gamma, int causal, int dtype, int flags, int32_t* status,
                   void* stream);

PNFT_API size_t pnft_flash_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D, int flags);

/* pnft_flash_fwd with the causal FIR on the keys fused into the kernels' K-tile
 * load: k is the RAW K (the projection output); each K tile is staged by TMA with
 * its 8 preceding rows (zeros before the sequence start) and filtered in shared
 * memory into k~ = causal_fir(k, taps), bit-identical to pnft_fir_fwd, before the
 * QK^T MMA. taps: device fp32[PNFT_FIR_FUSED_TAPS], index 6 = lag 0. The other
 * arguments as pnft_flash_fwd. Served by the sm_100a kernels only (bf16, head dims
 * that are multiples of 16 up to 128, 16-byte aligned rows with unit head-dim
 * stride); other inputs return PNFT_EUNSUPPORTED.
 * Replaces: triton_causal_fir(k) followed by flash_pn_fir_tau_attention in
 * PnFirTauFlashMHA.forward (src/pnfirtau_attention.py:285-316,
 * src/triton_pnfirtau.py:685-691, 971-983). */
PNFT_API int pnft_flash_fwd_fir(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                       const float* taps, int ntaps, const void* v, const int64_t* sv, const float* tau,
                       void* out, const int64_t* so, float* out_f32, float* stat_m, float* stat_z,
                       int32_t* stat_nmax, int32_t* stat_arg, int64_t B, int64_t H, int64_t N, int64_t D,
                       float scale, float gamma, int has_gamma, int causal, int dtype, int flags,
                       uint8_t* tile_flags, int32_t* status, void* stream);

/* Backward of pnft_flash_fwd_fir. The kernel re-filters its K tile from the raw k
 * in shared memory and writes d(k~) to the workspace; the transposed FIR
 * (pnft_fir_bwd) then gives dk, the gradient of the RAW k (strides sdk), and
 * dtaps (fp32[PNFT_FIR_FUSED_TAPS], may be NULL). k and dk need unit head-dim
 * stride and either adjacent (h, d) axes (the module's [B,N,H*D] view) or
 * adjacent (b, h) axes (a contiguous [B,H,N,D] tensor). workspace:
 * pnft_flash_bwd_fir_workspace_size(...) bytes, 256-byte aligned. The other
 * arguments as pnft_flash_bwd.
 * Replaces: the backward of the same composition (src/triton_pnfirtau.py:445-621,
 * 629-682). */
PNFT_API int pnft_flash_bwd_fir(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                       const float* taps, int ntaps, const void* v, const int64_t* sv, const float* tau,
                       const void* out, const int64_t* so, const float* out_f32, const void* dout,
                       const int64_t* sdo, const float* stat_m, const float* stat_z,
                       const int32_t* stat_nmax, const int32_t* stat_arg, void* dq, const int64_t* sdq,
                       void* dk, const int64_t* sdk, void* dv, const int64_t* sdv, float* dtau,
                       float* dtaps, void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                       int64_t N, int64_t D, float scale, float gamma, int has_gamma, int causal, int dtype,
                       int flags, int32_t* status, void* stream);

PNFT_API size_t pnft_flash_bwd_fir_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D, int flags);

/* Which kernel family pnft_flash_fwd / pnft_flash_bwd would launch for these
 * arguments: 1 = sm_100a tcgen05/TMA kernels, 0 = generic SIMT kernels. */
PNFT_API int pnft_flash_path(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                    const void* v, const int64_t* sv, int64_t D, int dtype, int flags);

/* ---------------------------------------------------------------------------
 * LM training step around the operator (the caller in the reference's
 * language-model experiments, experiments/exp4_wikitext2_lm.py).
 * ------------------------------------------------------------------------- */

/* Next-token cross-entropy of the LM head, loss and logit gradient in one pass.
 * logits: bf16 [M, ld] row-major; columns [V, ld) are padding and excluded.
 * On return `logits` holds the gradient s * (softmax(row) - onehot(target)) for
 * columns < V and 0 for the padding, with s = grad_scale * (*grad_scale_dev if
 * grad_scale_dev is not NULL; a device float, e.g. 1/number of counted rows);
 * row_loss[m] (fp32) = logsumexp(row m) - row m[target m]. Rows whose target
 * equals ignore_index get loss 0 and gradient 0. A target outside [0, V) that is
 * not ignore_index gives that row a NaN loss, no one-hot term, and sets the
 * status word to PNFT_DEV_BAD_INDEX. targets: int64 [M].
 * Replaces: nn.functional.cross_entropy(logits, targets) (mean reduction,
 * ignore_index) and its autograd backward (experiments/exp4_wikitext2_lm.py:714-719). */
PNFT_API int pnft_lm_xent(void* logits, int64_t ld, const int64_t* targets, int64_t ignore_index, float* row_loss,
                 int64_t M, int64_t V, float grad_scale, const float* grad_scale_dev, int32_t* status,
                 void* stream);

/* LayerNorm over the last C elements of M rows (row strides sx / sy in
 * elements, unit column stride): y = (x - mean) * rstd * gamma + beta with
 * rstd = 1/sqrt(var + eps) (biased variance); gamma / beta may be NULL (1 / 0).
 * Writes mean[M] and rstd[M] (fp32) for the backward. x and y are float32 or
 * bfloat16 (x_dtype / y_dtype: PNFT_DTYPE_*), arithmetic in fp32.
 * Replaces: nn.LayerNorm.forward in the Pre-LN blocks
 * (experiments/exp4_wikitext2_lm.py:183-200, 203-247). */
PNFT_API int pnft_layernorm_fwd(const void* x, int64_t sx, const float* gamma, const float* beta, float eps, void* y,
                       int64_t sy, float* mean, float* rstd, int64_t M, int64_t C, int x_dtype, int y_dtype,
                       void* stream);

/* Backward of pnft_layernorm_fwd: dx (the type of x, row stride sdx) and, when
 * dgamma / dbeta are not NULL, the parameter gradients (fp32 [C]) summed over
 * the rows in a fixed order (bitwise reproducible). dy is float32 or bfloat16.
 * workspace: pnft_layernorm_bwd_workspace_size(M, C) bytes when dgamma or
 * dbeta is requested (else may be NULL).
 * Replaces: the autograd backward of nn.LayerNorm (same call sites). */
PNFT_API int pnft_layernorm_bwd(const void* dy, int64_t sdy, const void* x, int64_t sx, const float* gamma,
                       const float* mean, const float* rstd, void* dx, int64_t sdx, float* dgamma, float* dbeta,
                       void* workspace, size_t workspace_bytes, int64_t M, int64_t C, int dy_dtype, int x_dtype,
                       void* stream);

PNFT_API size_t pnft_layernorm_bwd_workspace_size(int64_t M, int64_t C);

/* Residual add fused with the LayerNorm that follows it (the Pre-LN block's
 * `x + branch(...)` then `ln(x)`): s = x + r in x's type (r: r_dtype, float32 or
 * bfloat16; strides sr / ss), then y = LN(s) as pnft_layernorm_fwd. With r NULL
 * this is pnft_layernorm_fwd (s unused).
 * Replaces: the residual adds and nn.LayerNorm calls of the Pre-LN blocks
 * (experiments/exp4_wikitext2_lm.py:183-200) and the final ln_f (:203-247). */
PNFT_API int pnft_add_layernorm_fwd(const void* x, int64_t sx, const void* r, int64_t sr, int r_dtype, void* s,
                           int64_t ss, const float* gamma, const float* beta, float eps, void* y, int64_t sy,
                           float* mean, float* rstd, int64_t M, int64_t C, int x_dtype, int y_dtype, void* stream);

/* Backward of pnft_add_layernorm_fwd. x is the LayerNorm input (s of the
 * forward). dx (x's type, may be NULL) = gs + LN'(dy), with gs (x's type, may
 * be NULL) the gradient already flowing into s from the residual path; dr (may
 * be NULL, dr_dtype) receives the same values (the gradient of the residual
 * branch r); at least one of dx / dr. dgamma / dbeta / workspace as
 * pnft_layernorm_bwd.
 * Replaces: the autograd backward of the same composition, including the
 * residual gradient accumulation and the cast of the branch's gradient. */
PNFT_API int pnft_add_layernorm_bwd(const void* dy, int64_t sdy, const void* gs, int64_t sgs, const void* x,
                           int64_t sx, const float* gamma, const float* mean, const float* rstd, void* dx,
                           int64_t sdx, void* dr, int64_t sdr, int dr_dtype, float* dgamma, float* dbeta,
                           void* workspace, size_t workspace_bytes, int64_t M, int64_t C, int dy_dtype,
                           int x_dtype, void* stream);

/* Bias gradient of a Linear layer: out[c] = sum over the M rows of g[r, c]
 * (fp32, summed in a fixed order for a given GPU). g: float32 or bfloat16,
 * row stride sg. workspace: pnft_colsum_workspace_size(M, C) bytes.
 * Replaces: grad_output.sum(0) in the backward of the MLP's nn.Linear layers
 * (experiments/exp4_wikitext2_lm.py:183-200). */
PNFT_API int pnft_colsum(const void* g, int64_t sg, float* out, void* workspace, size_t workspace_bytes, int64_t M,
                int64_t C, int dtype, void* stream);

PNFT_API size_t pnft_colsum_workspace_size(int64_t M, int64_t C);

/* Backward of the MLP's exact (erf) GELU fused with the first Linear's bias
 * gradient: da[r, c] = dh[r, c] * GELU'(a[r, c]) (written in `dtype`), and
 * db[c] = sum over rows of da[r, c] as stored (fp32, fixed order). a is the
 * GELU input. workspace: pnft_colsum_workspace_size(M, C) bytes. table: as
 * pnft_gelu_fwd (GELU' of bfloat16 a; NULL: computed per CTA).
 * Replaces: nn.GELU's backward and grad_output.sum(0) of the first nn.Linear
 * (same call sites). */
/* Weight gradient of a Linear layer: C[M x N] (fp32, row stride ldc) = A^T B,
 * A [K x M] and B [K x N] bfloat16 rows (row strides lda / ldb, multiples of 8;
 * M and N multiples of 8; 16-byte aligned bases), i.e. dW = dY^T X with K the
 * token count. tcgen05 MMAs with the K reduction split over the SMs; the splits'
 * fp32 partials (workspace: pnft_gemm_at_b_workspace_size(K, M, N) bytes,
 * 16-byte aligned; 0 bytes when one split suffices) are added in a fixed order.
 * sm_100 devices only (PNFT_EUNSUPPORTED elsewhere). status: as the flash entry
 * points (bounded pipeline waits).
 * Replaces: the weight-gradient GEMM of nn.Linear's backward in the Pre-LN
 * blocks (experiments/exp4_wikitext2_lm.py:183-200). */
PNFT_API int pnft_gemm_at_b(const void* a, int64_t lda, const void* b, int64_t ldb, float* c, int64_t ldc,
                   void* workspace, size_t workspace_bytes, int64_t K, int64_t M, int64_t N, int dtype,
                   int32_t* status, void* stream);

PNFT_API size_t pnft_gemm_at_b_workspace_size(int64_t K, int64_t M, int64_t N);

/* Floats of the GELU lookup table (GELU and GELU' of every bfloat16 a with
 * |a| in [2^-16, 16)), built by pnft_gelu_table. */
#define PNFT_GELU_TABLE_FLOATS 10240

/* Builds the GELU lookup table (PNFT_GELU_TABLE_FLOATS fp32, 16-byte aligned)
 * that pnft_gelu_fwd / pnft_gelu_bwd_colsum copy into shared memory. */
PNFT_API int pnft_gelu_table(float* table, void* stream);

/* y = GELU(a) = a * Phi(a) (the exact, erf form of nn.GELU()), rows of C
 * elements with row strides sa / sy; float32 or bfloat16, arithmetic in fp32.
 * bfloat16 rows look GELU up in `table` (pnft_gelu_table's output; NULL: every
 * CTA computes its own copy, same values). Values outside the table's range
 * use the formula.
 * Replaces: nn.GELU's forward in the MLP (experiments/exp4_wikitext2_lm.py:183-200). */
PNFT_API int pnft_gelu_fwd(const void* a, int64_t sa, void* y, int64_t sy, int64_t M, int64_t C, int dtype,
                  const float* table, void* stream);

PNFT_API int pnft_gelu_bwd_colsum(const void* dh, int64_t sdh, const void* a, int64_t sa, void* da, int64_t sda,
                         float* db, void* workspace, size_t workspace_bytes, int64_t M, int64_t C, int dtype,
                         const float* table, void* stream);

/* bfloat16 copies of `count` fp32 tensors in one launch. `table` (device
 * memory, int64 rows of {src address, dst address, element count}) names each
 * tensor; dst[e] = src[e] rounded to nearest even for e < count of that row.
 * max_n: the largest element count (sizes the grid).
 * Replaces: the per-GEMM weight / bias casts of bf16 autocast in the LM step
 * (torch.autocast around experiments/exp4_wikitext2_lm.py:712-729). */
PNFT_API int pnft_cast_bf16(const int64_t* table, int count, int64_t max_n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PNFIRTAU_B200_H */
