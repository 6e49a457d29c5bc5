// Row-fused score -> weight op of pn_fir_tau over R rows of length N
// (the materialised-scores path behind triton_pn_fir_tau_scores and the
// return_weights=True module path).
//
// Forward, per row (src/triton_pnfirtau.py:141-212; silence modes and general
// p from power_norm_peak_gate, src/pnfirtau_attention.py:87-119):
//   s = raw*scale - tau ; u = relu(s) on valid columns (causal: col <= r % N)
//   pw = u^p ; mass = sum pw ; z = mass + 1e-12
//   strength = max u | sum u | mass  ; gate = strength/(strength+gamma) (or 1)
//   w = pw * (gate / z); stats M = peak, Z = z, Nmax = #(u == peak), S = strength
//   rows with peak <= 0 are silent: w = 0, M = 0, Z = 1e-12, Nmax = 0.
// Backward (src/triton_pnfirtau.py:214-303, generalised to the three modes):
//   D = sum dy * pw/z
//   du = p*u^(p-1) * [ gate/z * (dy - D) + (mass_pow) D*gamma/(mass+gamma)^2 ]
//        + (peak) [u == peak] * D*gamma/(peak+gamma)^2 / Nmax
//        + (mass_relu) D*gamma/(sum u + gamma)^2          on u > 0, else 0
//   graw = du*scale ; dtau_row = -sum du
// A block of 256 threads serves 256/TPR rows; each thread keeps up to
// ROW_CACHE of its row's values in registers so the row is read once.
#include "common.cuh"

namespace pnft {

constexpr int ROW_THREADS = 256;
constexpr int ROW_CACHE = 16;

struct RowParams {
  const void* raw;
  int64_t raw_stride;
  const void* gw;
  int64_t gw_stride;
  void* out;
  int64_t out_stride;
  const float* tau;
  float* m;
  float* z;
  int32_t* nmax;
  float* strength;
  const float* cm;
  const float* cz;
  const int32_t* cnmax;
  const float* cstrength;
  float* dtau_rows;
  int64_t R, N;
  float scale, p, gamma;
  int has_gamma, mode, causal, pmode;  // pmode: 10, 2 or 0 (general)
};

template <int TPR>
struct RowReduce {
  static constexpr int W = TPR / 32;  // warps per row (TPR >= 32)
  // sm: ROW_THREADS/32 floats of scratch, shared by the block
  __device__ static float sum(float v, float* sm) {
    v = group_sum<32>(v);
    if constexpr (W == 1) return v;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sm[warp] = v;
    __syncthreads();
    const int first = (warp / W) * W;
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < W; ++i) t += sm[first + i];
    return t;
  }
  __device__ static float max(float v, float* sm) {
    v = group_max<32>(v);
    if constexpr (W == 1) return v;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sm[warp] = v;
    __syncthreads();
    const int first = (warp / W) * W;
    float t = sm[first];
#pragma unroll
    for (int i = 1; i < W; ++i) t = fmaxf(t, sm[first + i]);
    return t;
  }
};

__device__ __forceinline__ float pow_p(float u, int pmode, float p) {
  if (pmode == 10) {
    const float u2 = u * u, u4 = u2 * u2;
    return u4 * u4 * u2;
  }
  if (pmode == 2) return u * u;
  return u > 0.f ? powf(u, p) : 0.f;
}
__device__ __forceinline__ float pow_pm1(float u, int pmode, float p) {
  if (pmode == 10) {
    const float u2 = u * u, u4 = u2 * u2, u8 = u4 * u4;
    return u8 * u;
  }
  if (pmode == 2) return u;
  return u > 0.f ? powf(u, p - 1.f) : 0.f;
}

template <typename T, int TPR>
__global__ void __launch_bounds__(ROW_THREADS) rows_fwd_kernel(RowParams P) {
  __shared__ float sm[ROW_THREADS / 32];
  constexpr int RPB = ROW_THREADS / TPR;
  const int64_t r = (int64_t)blockIdx.x * RPB + threadIdx.x / TPR;
  const int l = threadIdx.x % TPR;
  const bool row_ok = r < P.R;
  const int64_t limit = !row_ok ? 0 : (P.causal ? min(r % P.N + 1, P.N) : P.N);
  const T* raw = static_cast<const T*>(P.raw) + (row_ok ? r * P.raw_stride : 0);
  const float tau = __ldg(P.tau);
  float uc[ROW_CACHE];
  float peak = 0.f, mass = 0.f, sumu = 0.f;
#pragma unroll
  for (int k = 0; k < ROW_CACHE; ++k) {
    const int64_t j = l + (int64_t)k * TPR;
    float u = 0.f;
    if (j < limit) {
      const float s = to_f32<T>(raw[j]) * P.scale - tau;
      u = s > 0.f ? s : 0.f;
    }
    uc[k] = u;
    peak = fmaxf(peak, u);
    mass += pow_p(u, P.pmode, P.p);
    sumu += u;
  }
  for (int64_t j = l + (int64_t)ROW_CACHE * TPR; j < limit; j += TPR) {
    const float s = to_f32<T>(raw[j]) * P.scale - tau;
    const float u = s > 0.f ? s : 0.f;
    peak = fmaxf(peak, u);
    mass += pow_p(u, P.pmode, P.p);
    sumu += u;
  }
  peak = RowReduce<TPR>::max(peak, sm);
  mass = RowReduce<TPR>::sum(mass, sm);
  sumu = RowReduce<TPR>::sum(sumu, sm);
  float cnt = 0.f;
#pragma unroll
  for (int k = 0; k < ROW_CACHE; ++k) cnt += (peak > 0.f && uc[k] == peak) ? 1.f : 0.f;
  for (int64_t j = l + (int64_t)ROW_CACHE * TPR; j < limit; j += TPR) {
    const float s = to_f32<T>(raw[j]) * P.scale - tau;
    const float u = s > 0.f ? s : 0.f;
    cnt += (peak > 0.f && u == peak) ? 1.f : 0.f;
  }
  cnt = RowReduce<TPR>::sum(cnt, sm);
  if (!row_ok) return;
  T* w = static_cast<T*>(P.out) + r * P.out_stride;
  const bool silent = !(peak > 0.f);
  float coef = 0.f, z = 1e-12f, strength = 0.f;
  if (!silent) {
    z = mass + 1e-12f;
    strength = P.mode == PNFT_SILENCE_PEAK ? peak : (P.mode == PNFT_SILENCE_MASS_RELU ? sumu : mass);
    const float gate = P.has_gamma ? strength / (strength + P.gamma) : 1.f;
    coef = gate / z;
  }
#pragma unroll
  for (int k = 0; k < ROW_CACHE; ++k) {
    const int64_t j = l + (int64_t)k * TPR;
    if (j < P.N) w[j] = from_f32<T>(silent ? 0.f : pow_p(uc[k], P.pmode, P.p) * coef);
  }
  for (int64_t j = l + (int64_t)ROW_CACHE * TPR; j < P.N; j += TPR) {
    float v = 0.f;
    if (!silent && j < limit) {
      const float s = to_f32<T>(raw[j]) * P.scale - tau;
      const float u = s > 0.f ? s : 0.f;
      v = pow_p(u, P.pmode, P.p) * coef;
    }
    w[j] = from_f32<T>(v);
  }
  if (l == 0) {
    P.m[r] = silent ? 0.f : peak;
    P.z[r] = z;
    P.nmax[r] = silent ? 0 : (int32_t)cnt;
    if (P.strength) P.strength[r] = strength;
  }
}

template <typename T, int TPR>
__global__ void __launch_bounds__(ROW_THREADS) rows_bwd_kernel(RowParams P) {
  __shared__ float sm[ROW_THREADS / 32];
  constexpr int RPB = ROW_THREADS / TPR;
  const int64_t r = (int64_t)blockIdx.x * RPB + threadIdx.x / TPR;
  const int l = threadIdx.x % TPR;
  const bool row_ok = r < P.R;
  const float peak = row_ok ? P.cm[r] : 0.f;
  const bool silent = !(peak > 0.f);
  // silent rows: zero gradient without reading scores or dy (the reference's short circuit)
  const int64_t limit = (!row_ok || silent) ? 0 : (P.causal ? min(r % P.N + 1, P.N) : P.N);
  const T* raw = static_cast<const T*>(P.raw) + (row_ok ? r * P.raw_stride : 0);
  const T* gw = static_cast<const T*>(P.gw) + (row_ok ? r * P.gw_stride : 0);
  const float tau = __ldg(P.tau);
  const float z = row_ok ? P.cz[r] : 1.f;
  float uc[ROW_CACHE], dyc[ROW_CACHE];
  float D = 0.f;
#pragma unroll
  for (int k = 0; k < ROW_CACHE; ++k) {
    const int64_t j = l + (int64_t)k * TPR;
    float u = 0.f, dy = 0.f;
    if (j < limit) {
      const float s = to_f32<T>(raw[j]) * P.scale - tau;
      u = s > 0.f ? s : 0.f;
      dy = to_f32<T>(gw[j]);
    }
    uc[k] = u;
    dyc[k] = dy;
    D += dy * (pow_p(u, P.pmode, P.p) / z);
  }
  for (int64_t j = l + (int64_t)ROW_CACHE * TPR; j < limit; j += TPR) {
    const float s = to_f32<T>(raw[j]) * P.scale - tau;
    const float u = s > 0.f ? s : 0.f;
    D += to_f32<T>(gw[j]) * (pow_p(u, P.pmode, P.p) / z);
  }
  D = RowReduce<TPR>::sum(D, sm);
  float gate = 1.f, tie = 0.f, add_all = 0.f, add_pw = 0.f;
  if (row_ok && !silent) {
    const float strength = P.cstrength ? P.cstrength[r] : peak;
    if (P.has_gamma) {
      const float sg = strength + P.gamma;
      gate = strength / sg;
      const float dg = D * (P.gamma / (sg * sg));
      if (P.mode == PNFT_SILENCE_PEAK) tie = dg / (float)P.cnmax[r];
      else if (P.mode == PNFT_SILENCE_MASS_RELU) add_all = dg;
      else add_pw = dg;
    }
  }
  const float cnorm = P.p * gate / z;
  float dtau = 0.f;
  T* g = static_cast<T*>(P.out) + (row_ok ? r * P.out_stride : 0);
#pragma unroll
  for (int k = 0; k < ROW_CACHE; ++k) {
    const int64_t j = l + (int64_t)k * TPR;
    const float u = uc[k];
    float du = 0.f;
    if (u > 0.f) {
      const float upm1 = pow_pm1(u, P.pmode, P.p);
      du = cnorm * upm1 * (dyc[k] - D) + P.p * upm1 * add_pw + add_all + (u == peak ? tie : 0.f);
    }
    dtau -= du;
    if (row_ok && j < P.N) g[j] = from_f32<T>(du * P.scale);
  }
  for (int64_t j = l + (int64_t)ROW_CACHE * TPR; j < P.N; j += TPR) {
    float du = 0.f;
    if (j < limit) {
      const float s = to_f32<T>(raw[j]) * P.scale - tau;
      const float u = s > 0.f ? s : 0.f;
      if (u > 0.f) {
        const float upm1 = pow_pm1(u, P.pmode, P.p);
        du = cnorm * upm1 * (to_f32<T>(gw[j]) - D) + P.p * upm1 * add_pw + add_all + (u == peak ? tie : 0.f);
      }
    }
    dtau -= du;
    if (row_ok) g[j] = from_f32<T>(du * P.scale);
  }
  dtau = RowReduce<TPR>::sum(dtau, sm);
  if (row_ok && l == 0) P.dtau_rows[r] = dtau;
}

// Deterministic fp64 reduction of n floats into out[0].
__global__ void __launch_bounds__(1024) sum_f32_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ out) {
  __shared__ double sm[1024];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 1024) s += (double)x[i];
  sm[threadIdx.x] = s;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) sm[threadIdx.x] += sm[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[0] = (float)sm[0];
}

template <typename T, bool FWD>
static void rows_launch(const RowParams& P, cudaStream_t st) {
  auto go = [&](auto tpr_c) {
    constexpr int TPR = decltype(tpr_c)::value;
    constexpr int RPB = ROW_THREADS / TPR;
    const int64_t grid = (P.R + RPB - 1) / RPB;
    if (FWD) rows_fwd_kernel<T, TPR><<<(unsigned)grid, ROW_THREADS, 0, st>>>(P);
    else rows_bwd_kernel<T, TPR><<<(unsigned)grid, ROW_THREADS, 0, st>>>(P);
  };
  if (P.N <= 32 * ROW_CACHE) go(std::integral_constant<int, 32>{});
  else if (P.N <= 64 * ROW_CACHE) go(std::integral_constant<int, 64>{});
  else if (P.N <= 128 * ROW_CACHE) go(std::integral_constant<int, 128>{});
  else go(std::integral_constant<int, 256>{});
}

static int rows_check(const RowParams& P) {
  if (P.R < 0 || P.N < 0) return fail(PNFT_EINVAL, "rows: negative size");
  if (P.R > ((int64_t)1 << 31) * (ROW_THREADS / 32)) return fail(PNFT_EINVAL, "rows: too many rows");
  if (P.mode < 0 || P.mode > 2) return fail(PNFT_EINVAL, "rows: unknown silence mode %d", P.mode);
  if (P.has_gamma && !(P.gamma > 0.f)) return fail(PNFT_EINVAL, "rows: has_gamma with gamma <= 0");
  if (!P.tau) return fail(PNFT_EINVAL, "rows: null tau");
  return PNFT_OK;
}

static int pmode_of(float p) { return p == 10.f ? 10 : (p == 2.f ? 2 : 0); }

}  // namespace pnft

using namespace pnft;

extern "C" int pnft_sum_f32(const float* x, int64_t n, float* out, void* stream) {
  if (!out || (n > 0 && !x) || n < 0) return fail(PNFT_EINVAL, "sum_f32: bad arguments");
  sum_f32_kernel<<<1, 1024, 0, as_stream(stream)>>>(x, n, out);
  return check_launch("sum_f32");
}

extern "C" int pnft_rows_fwd(const void* raw, int64_t raw_row_stride, const float* tau, void* w,
                             int64_t w_row_stride, float* stat_m, float* stat_z, int32_t* stat_nmax,
                             float* stat_strength, int64_t R, int64_t N, float scale, float p, float gamma,
                             int has_gamma, int silence_mode, int causal, int dtype, void* stream) {
  RowParams P{};
  P.raw = raw; P.raw_stride = raw_row_stride; P.out = w; P.out_stride = w_row_stride; P.tau = tau;
  P.m = stat_m; P.z = stat_z; P.nmax = stat_nmax; P.strength = stat_strength;
  P.R = R; P.N = N; P.scale = scale; P.p = p; P.gamma = gamma; P.has_gamma = has_gamma;
  P.mode = silence_mode; P.causal = causal; P.pmode = pmode_of(p);
  int rc = rows_check(P);
  if (rc) return rc;
  if (R == 0) return PNFT_OK;
  if (N == 0) return fail(PNFT_EINVAL, "rows fwd: N == 0 with R > 0");
  if (!raw || !w || !stat_m || !stat_z || !stat_nmax) return fail(PNFT_EINVAL, "rows fwd: null pointer");
  PNFT_DISPATCH_DTYPE(dtype, T, rows_launch<T, true>(P, as_stream(stream)));
  return check_launch("rows fwd");
}

extern "C" int pnft_rows_bwd(const void* gw, int64_t gw_row_stride, const void* raw, int64_t raw_row_stride,
                             const float* tau, const float* stat_m, const float* stat_z,
                             const int32_t* stat_nmax, const float* stat_strength, void* graw,
                             int64_t graw_row_stride, float* dtau_rows, float* dtau, int64_t R, int64_t N,
                             float scale, float p, float gamma, int has_gamma, int silence_mode, int causal,
                             int dtype, void* stream) {
  RowParams P{};
  P.raw = raw; P.raw_stride = raw_row_stride; P.gw = gw; P.gw_stride = gw_row_stride; P.out = graw;
  P.out_stride = graw_row_stride; P.tau = tau; P.cm = stat_m; P.cz = stat_z; P.cnmax = stat_nmax;
  P.cstrength = stat_strength; P.dtau_rows = dtau_rows; P.R = R; P.N = N; P.scale = scale; P.p = p;
  P.gamma = gamma; P.has_gamma = has_gamma; P.mode = silence_mode; P.causal = causal; P.pmode = pmode_of(p);
  int rc = rows_check(P);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  if (R > 0) {
    if (N == 0) return fail(PNFT_EINVAL, "rows bwd: N == 0 with R > 0");
    if (!raw || !gw || !graw || !stat_m || !stat_z || !stat_nmax || !dtau_rows)
      return fail(PNFT_EINVAL, "rows bwd: null pointer");
    if (silence_mode != PNFT_SILENCE_PEAK && has_gamma && !stat_strength)
      return fail(PNFT_EINVAL, "rows bwd: silence mode %d needs stat_strength", silence_mode);
    PNFT_DISPATCH_DTYPE(dtype, T, rows_launch<T, false>(P, st));
    rc = check_launch("rows bwd");
    if (rc) return rc;
  }
  if (dtau) return pnft_sum_f32(dtau_rows, R, dtau, stream);
  return PNFT_OK;
}
