// C-ABI entry points of the flash op plus library-wide plumbing (version,
// last-error message, device capabilities). Argument checking happens here so
// the kernels can assume well-formed shapes.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "flash.cuh"

namespace pnft {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<uint64_t> g_launches{0};

int check_launch(const char* what, int nlaunch) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    g_launches.fetch_add((uint64_t)nlaunch, std::memory_order_relaxed);
    return PNFT_OK;
  }
  return fail(PNFT_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace pnft

using namespace pnft;

extern "C" uint64_t pnft_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int pnft_version(void) { return 100; }

extern "C" const char* pnft_last_error(void) { return g_err; }

extern "C" int pnft_query_caps(int device, int* cc_major, int* cc_minor, int* sm_count, int* smem_optin_bytes,
                               int* has_sm100a) {
  cudaDeviceProp p;
  const cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return fail(PNFT_ECUDA, "query_caps: %s", cudaGetErrorString(e));
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (smem_optin_bytes) *smem_optin_bytes = (int)p.sharedMemPerBlockOptin;
  if (has_sm100a) *has_sm100a = (p.major == 10 && p.minor == 0) ? 1 : 0;
  return PNFT_OK;
}

extern "C" int pnft_mapped_status_ptr(void* host_word, void** device_ptr) {
  if (!host_word || !device_ptr) return fail(PNFT_EINVAL, "mapped_status_ptr: null pointer");
  *device_ptr = nullptr;
  void* d = nullptr;
  const cudaError_t e = cudaHostGetDevicePointer(&d, host_word, 0);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // not sticky: clear it for the caller's next launch check
    return fail(PNFT_EINVAL, "mapped_status_ptr: %s (the word must be pinned host memory mapped into the device)",
                cudaGetErrorString(e));
  }
  *device_ptr = d;
  return PNFT_OK;
}

static int fill_common(FlashArgs& a, const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                       const void* v, const int64_t* sv, const float* tau, int64_t B, int64_t H, int64_t N,
                       int64_t D, float scale, float gamma, int has_gamma, int causal, int dtype, int flags,
                       int32_t* status) {
  memset(&a, 0, sizeof(a));
  if (B < 0 || H < 0 || N < 0 || D < 0)
    return fail(PNFT_EINVAL, "flash: negative size B=%lld H=%lld N=%lld D=%lld", (long long)B, (long long)H,
                (long long)N, (long long)D);
  if (dtype < PNFT_DTYPE_F32 || dtype > PNFT_DTYPE_F16) return fail(PNFT_EINVAL, "flash: unknown dtype %d", dtype);
  if (D > 128) return fail(PNFT_EUNSUPPORTED, "flash: head dim %lld > 128 is not supported", (long long)D);
  if (B * H > 65535LL * 1024) return fail(PNFT_EUNSUPPORTED, "flash: B*H = %lld too large", (long long)(B * H));
  if (has_gamma && !(gamma > 0.f)) return fail(PNFT_EINVAL, "flash: has_gamma set with gamma <= 0");
  if (!sq || !sk || !sv) return fail(PNFT_EINVAL, "flash: null stride array");
  a.q = q; a.k = k; a.v = v; a.tau = tau;
  for (int i = 0; i < 4; ++i) { a.sq[i] = sq[i]; a.sk[i] = sk[i]; a.sv[i] = sv[i]; }
  a.B = B; a.H = H; a.N = N; a.D = D; a.acc_d = acc_width(D); a.scale = scale; a.gamma = gamma; a.has_gamma = has_gamma;
  a.causal = causal; a.dtype = dtype; a.flags = flags; a.status = status;
  return PNFT_OK;
}

static bool use_sm100(const FlashArgs& a) {
  if (a.flags & PNFT_FLASH_FORCE_GENERIC) return false;
  return flash_sm100_supported(a);
}

extern "C" int pnft_flash_path(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                               const int64_t* sv, int64_t D, int dtype, int flags) {
  FlashArgs a;
  float tau_dummy = 0.f;
  if (fill_common(a, q, sq, k, sk, v, sv, &tau_dummy, 1, 1, 1, D, 1.f, 0.5f, 1, 1, dtype, flags, nullptr)) return 0;
  return use_sm100(a) ? 1 : 0;
}

static int flash_fwd_entry(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                           const int64_t* sv, const float* tau, void* out, const int64_t* so, float* out_f32,
                           float* stat_m, float* stat_z, int32_t* stat_nmax, int32_t* stat_arg, int64_t B, int64_t H,
                           int64_t N, int64_t D, float scale, float gamma, int has_gamma, int causal, int dtype,
                           int flags, uint8_t* tile_flags, int32_t* status, void* stream, const float* fir_taps,
                           int fir_ntaps) {
  FlashArgs a;
  int rc = fill_common(a, q, sq, k, sk, v, sv, tau, B, H, N, D, scale, gamma, has_gamma, causal, dtype, flags, status);
  if (rc) return rc;
  a.tile_flags = tile_flags;
  a.fir_taps = fir_taps;
  a.fir_ntaps = fir_ntaps;
  if (B * H * N == 0) return PNFT_OK;
  if (D == 0) return fail(PNFT_EINVAL, "flash fwd: head dim 0");
  if (!q || !k || !v || !tau || !out || !so || !stat_m || !stat_z || !stat_nmax || !stat_arg)
    return fail(PNFT_EINVAL, "flash fwd: null pointer");
  a.out = out;
  a.out32 = out_f32;
  for (int i = 0; i < 4; ++i) a.so[i] = so[i];
  a.stat_m = stat_m; a.stat_z = stat_z; a.stat_nmax = stat_nmax; a.stat_arg = stat_arg;
  cudaStream_t st = as_stream(stream);
  if (use_sm100(a)) return flash_fwd_sm100(a, st);
  if (fir_taps)
    return fail(PNFT_EUNSUPPORTED, "flash fwd: the fused FIR runs on the sm_100a kernels only (bf16, head dims multiples of 16 up to 128, "
                                   "16-byte aligned rows with unit head-dim stride)");
  return flash_fwd_generic(a, st);
}

extern "C" int pnft_flash_fwd(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                              const int64_t* sv, const float* tau, void* out, const int64_t* so, float* out_f32,
                              float* stat_m, float* stat_z, int32_t* stat_nmax, int32_t* stat_arg, int64_t B,
                              int64_t H, int64_t N, int64_t D, float scale, float gamma, int has_gamma, int causal,
                              int dtype, int flags, uint8_t* tile_flags, int32_t* status, void* stream) {
  return flash_fwd_entry(q, sq, k, sk, v, sv, tau, out, so, out_f32, stat_m, stat_z, stat_nmax, stat_arg, B, H, N, D,
                         scale, gamma, has_gamma, causal, dtype, flags, tile_flags, status, stream, nullptr, 0);
}

extern "C" int pnft_flash_fwd_fir(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                                  const float* taps, int ntaps, const void* v, const int64_t* sv, const float* tau,
                                  void* out, const int64_t* so, float* out_f32, float* stat_m, float* stat_z,
                                  int32_t* stat_nmax, int32_t* stat_arg, int64_t B, int64_t H, int64_t N, int64_t D,
                                  float scale, float gamma, int has_gamma, int causal, int dtype, int flags,
                                  uint8_t* tile_flags, int32_t* status, void* stream) {
  if (!taps) return fail(PNFT_EINVAL, "flash fwd fir: null taps");
  return flash_fwd_entry(q, sq, k, sk, v, sv, tau, out, so, out_f32, stat_m, stat_z, stat_nmax, stat_arg, B, H, N, D,
                         scale, gamma, has_gamma, causal, dtype, flags, tile_flags, status, stream, taps, ntaps);
}

extern "C" size_t pnft_flash_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D, int flags) {
  (void)flags;
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0) return 0;
  return bwd_workspace_layout(B, H, N, D).total;
}

static int flash_bwd_entry(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                           const int64_t* sv, const float* tau, const void* out, const int64_t* so,
                           const float* out_f32, const void* dout, const int64_t* sdo, const float* stat_m,
                           const float* stat_z, const int32_t* stat_nmax, const int32_t* stat_arg, void* dq,
                           const int64_t* sdq, void* dk, const int64_t* sdk, void* dv, const int64_t* sdv, float* dtau,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D,
                           float scale, float gamma, int has_gamma, int causal, int dtype, int flags, int32_t* status,
                           void* stream, const float* fir_taps, int fir_ntaps) {
  FlashArgs a;
  int rc = fill_common(a, q, sq, k, sk, v, sv, tau, B, H, N, D, scale, gamma, has_gamma, causal, dtype, flags, status);
  if (rc) return rc;
  a.fir_taps = fir_taps;
  a.fir_ntaps = fir_ntaps;
  cudaStream_t st = as_stream(stream);
  if (!dtau) return fail(PNFT_EINVAL, "flash bwd: null dtau");
  if (B * H * N == 0) {
    if (cudaMemsetAsync(dtau, 0, sizeof(float), st) != cudaSuccess) return check_launch("flash bwd: dtau memset");
    return PNFT_OK;
  }
  if (D == 0) return fail(PNFT_EINVAL, "flash bwd: head dim 0");
  if (!q || !k || !v || !tau || !out || !so || !dout || !sdo || !stat_m || !stat_z || !stat_nmax || !stat_arg || !dq ||
      !sdq || !dk || !sdk || !dv || !sdv)
    return fail(PNFT_EINVAL, "flash bwd: null pointer");
  const BwdWorkspace w = bwd_workspace_layout(B, H, N, D);
  if (!workspace || workspace_bytes < w.total)
    return fail(PNFT_EINVAL, "flash bwd: workspace of %zu bytes < required %zu", workspace_bytes, w.total);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return fail(PNFT_EINVAL, "flash bwd: workspace not 256-byte aligned");
  a.out_c = out; a.out32 = const_cast<float*>(out_f32); a.dout = dout; a.dq = dq; a.dk = dk; a.dv = dv; a.dtau = dtau;
  for (int i = 0; i < 4; ++i) { a.so[i] = so[i]; a.sdo[i] = sdo[i]; a.sdq[i] = sdq[i]; a.sdk[i] = sdk[i]; a.sdv[i] = sdv[i]; }
  a.stat_m = const_cast<float*>(stat_m); a.stat_z = const_cast<float*>(stat_z);
  a.stat_nmax = const_cast<int32_t*>(stat_nmax);
  a.stat_arg = const_cast<int32_t*>(stat_arg);
  char* ws = static_cast<char*>(workspace);
  a.dq_acc = reinterpret_cast<float*>(ws + w.off_dq);
  {
    const size_t recs = (size_t)(B * H * rec_rows(N));
    a.coefP = reinterpret_cast<float4*>(ws + w.off_coef);
    a.tiev = reinterpret_cast<float*>(a.coefP + recs / 2);
    a.argv = reinterpret_cast<int32_t*>(a.tiev + recs);
    a.pcmpv = reinterpret_cast<float*>(a.argv + recs);
  }
  a.live64 = reinterpret_cast<int32_t*>(ws + w.off_live);
  a.dtau_part = reinterpret_cast<float*>(ws + w.off_part);
  a.dq_sem = reinterpret_cast<int32_t*>(ws + w.off_sem);
  a.dq_ticket = a.dq_sem + (B * H) * ((N + 63) / 64);
  a.dq_scale = 1.f;
  if (use_sm100(a)) return flash_bwd_sm100(a, st);
  if (fir_taps) return fail(PNFT_EUNSUPPORTED, "flash bwd: the fused FIR runs on the sm_100a kernels only");
  return flash_bwd_generic(a, st);
}

extern "C" int pnft_flash_bwd(const void* q, const int64_t* sq, const void* k, const int64_t* sk, const void* v,
                              const int64_t* sv, const float* tau, const void* out, const int64_t* so,
                              const float* out_f32, const void* dout, const int64_t* sdo, const float* stat_m, const float* stat_z,
                              const int32_t* stat_nmax, const int32_t* stat_arg, void* dq, const int64_t* sdq, void* dk,
                              const int64_t* sdk, void* dv, const int64_t* sdv, float* dtau, void* workspace,
                              size_t workspace_bytes, int64_t B, int64_t H, int64_t N, int64_t D, float scale,
                              float gamma, int has_gamma, int causal, int dtype, int flags, int32_t* status,
                              void* stream) {
  return flash_bwd_entry(q, sq, k, sk, v, sv, tau, out, so, out_f32, dout, sdo, stat_m, stat_z, stat_nmax, stat_arg,
                         dq, sdq, dk, sdk, dv, sdv, dtau, workspace, workspace_bytes, B, H, N, D, scale, gamma,
                         has_gamma, causal, dtype, flags, status, stream, nullptr, 0);
}

// ---- fused-FIR backward: flash backward on the filtered keys (its d(k~) into the
// workspace), then the transposed FIR for dk and the tap gradient
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct FirBwdPlan {
  int64_t Bf, Cf;          // the FIR's [Bf, N, Cf] view of k / dk / d(k~)
  int64_t sk_b, sk_n;      // k in that view (channel stride 1)
  int64_t sdk_b, sdk_n;    // dk in that view
  int64_t sg_b, sg_n;      // d(k~) in that view (contiguous)
  int64_t st[4];           // d(k~) as [B,H,N,D]
};

// k and dk as [B, N, H*D] (head dims adjacent: the module's view of the qkv
// projection) or as [B*H, N, D] (b and h adjacent: a contiguous tensor).
static bool fir_bwd_plan(const int64_t* sk, const int64_t* sdk, int64_t B, int64_t H, int64_t N, int64_t D,
                         FirBwdPlan* pl) {
  if (sk[3] != 1 || sdk[3] != 1) return false;
  if ((H == 1 || (sk[1] == D && sdk[1] == D))) {
    *pl = FirBwdPlan{B, H * D, sk[0], sk[2], sdk[0], sdk[2], N * H * D, H * D, {N * H * D, D, H * D, 1}};
    return true;
  }
  if (sk[0] == H * sk[1] && sdk[0] == H * sdk[1]) {
    *pl = FirBwdPlan{B * H, D, sk[1], sk[2], sdk[1], sdk[2], N * D, D, {H * N * D, N * D, D, 1}};
    return true;
  }
  return false;
}

extern "C" size_t pnft_flash_bwd_fir_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D, int flags) {
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0) return 0;
  const size_t fir_ws = std::max(pnft_fir_bwd_workspace_size(B, N, H * D, PNFT_FIR_FUSED_TAPS),
                                 pnft_fir_bwd_workspace_size(B * H, N, D, PNFT_FIR_FUSED_TAPS));
  return align256(pnft_flash_bwd_workspace_size(B, H, N, D, flags)) + align256((size_t)(B * H * N * D) * 2) +
         align256(fir_ws);
}

extern "C" int pnft_flash_bwd_fir(const void* q, const int64_t* sq, const void* k, const int64_t* sk,
                                  const float* taps, int ntaps, const void* v, const int64_t* sv, const float* tau,
                                  const void* out, const int64_t* so, const float* out_f32, const void* dout,
                                  const int64_t* sdo, const float* stat_m, const float* stat_z,
                                  const int32_t* stat_nmax, const int32_t* stat_arg, void* dq, const int64_t* sdq,
                                  void* dk, const int64_t* sdk, void* dv, const int64_t* sdv, float* dtau,
                                  float* dtaps, void* workspace, size_t workspace_bytes, int64_t B, int64_t H,
                                  int64_t N, int64_t D, float scale, float gamma, int has_gamma, int causal, int dtype,
                                  int flags, int32_t* status, void* stream) {
  if (!taps || !sk || !sdk || !dk) return fail(PNFT_EINVAL, "flash bwd fir: null taps, dk or strides");
  if (ntaps != PNFT_FIR_FUSED_TAPS) return fail(PNFT_EUNSUPPORTED, "flash bwd fir: fused FIR needs %d taps", PNFT_FIR_FUSED_TAPS);
  if (B < 0 || H < 0 || N < 0 || D < 0) return fail(PNFT_EINVAL, "flash bwd fir: negative size");
  cudaStream_t st = as_stream(stream);
  if (B * H * N * D == 0) {
    if (dtaps && cudaMemsetAsync(dtaps, 0, sizeof(float) * ntaps, st) != cudaSuccess)
      return check_launch("flash bwd fir: dtaps memset");
    return pnft_flash_bwd(q, sq, k, sk, v, sv, tau, out, so, out_f32, dout, sdo, stat_m, stat_z, stat_nmax, stat_arg,
                          dq, sdq, dk, sdk, dv, sdv, dtau, workspace, workspace_bytes, B, H, N, D, scale, gamma,
                          has_gamma, causal, dtype, flags, status, stream);
  }
  FirBwdPlan pl;
  if (!fir_bwd_plan(sk, sdk, B, H, N, D, &pl))
    return fail(PNFT_EUNSUPPORTED, "flash bwd fir: k and dk need unit head-dim stride and adjacent (h, d) or (b, h) axes");
  const size_t need = pnft_flash_bwd_fir_workspace_size(B, H, N, D, flags);
  if (!workspace || workspace_bytes < need)
    return fail(PNFT_EINVAL, "flash bwd fir: workspace of %zu bytes < required %zu", workspace_bytes, need);
  char* ws = static_cast<char*>(workspace);
  const size_t flash_ws = align256(pnft_flash_bwd_workspace_size(B, H, N, D, flags));
  void* dkt = ws + flash_ws;                               // d(k~), bf16
  char* fir_ws = ws + flash_ws + align256((size_t)(B * H * N * D) * 2);
  int rc = flash_bwd_entry(q, sq, k, sk, v, sv, tau, out, so, out_f32, dout, sdo, stat_m, stat_z, stat_nmax, stat_arg,
                           dq, sdq, dkt, pl.st, dv, sdv, dtau, workspace, flash_ws, B, H, N, D, scale, gamma,
                           has_gamma, causal, dtype, flags, status, stream, taps, ntaps);
  if (rc) return rc;
  return pnft_fir_bwd(dkt, pl.sg_b, pl.sg_n, 1, taps, ntaps, dk, pl.sdk_b,
                      pl.sdk_n, 1, dtaps ? k : nullptr, pl.sk_b, pl.sk_n, 1, dtaps, fir_ws,
                      need - (size_t)(fir_ws - ws), pl.Bf, N, pl.Cf, dtype, stream);
}
