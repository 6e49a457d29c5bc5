// Depthwise causal FIR along the sequence axis of x[B,N,C] (and its transpose
// and tap gradient). HBM-bound: every element is read once and written once;
// threads own 16-byte channel vectors so a warp moves 512 contiguous bytes per
// row, and each thread walks a run of consecutive rows (32, 16 or 8: the longest
// that still fills every SM) keeping the K-1 previous rows in registers
// (the halo rows are re-read from L1/L2, never from DRAM twice in practice). A run
// that lies inside the sequence loads eight rows at a time before using them, so
// each thread keeps eight 16-byte loads in flight.
//
// Semantics follow the reference kernels src/triton_pnfirtau.py:40-135:
//   fwd  y[b,n,c]  = sum_{u=0}^{K-1} taps[K-1-u] * x[b,n-u,c]   (x[<0] = 0)
//   bwd  gx[b,n,c] = sum_{u=0}^{K-1} taps[K-1-u] * gy[b,n+u,c]  (gy[>=N] = 0)
// with fp32 accumulation and the output in the input dtype. The tap gradient
// (absent in the reference, whose taps are a non-trainable buffer,
// src/triton_pnfirtau.py:682) is dtaps[K-1-u] = sum gy[b,n,c] * x[b,n-u,c].
#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace pnft {

constexpr int FIR_TN = 8;         // consecutive rows per thread
constexpr int FIR_MAX_TAPS = 64;  // runtime-K kernels
constexpr int FIR_THREADS = 256;
constexpr int FIR_DTAPS_MAX_BLOCKS = 512;

template <typename T, int VEC>
__device__ __forceinline__ void ld_vec(const T* p, float (&f)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f32<T>(p[i]);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void st_vec(T* p, const float (&f)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 r;
    T* e = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < VEC; ++i) e[i] = from_f32<T>(f[i]);
    *reinterpret_cast<uint4*>(p) = r;
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) p[i] = from_f32<T>(f[i]);
  }
}

struct FirGeom {
  const void* in;
  void* out;
  int64_t sib, sin, sic, sob, son, soc;
  int64_t B, N, C;
};

// Sliding-window kernel with compile-time tap count. DIR = +1: causal fwd
// (window over past rows), DIR = -1: transpose (window over future rows).
template <typename T, int VEC, int K, int DIR, int TN = FIR_TN>
__global__ void __launch_bounds__(FIR_THREADS) fir_sliding_kernel(FirGeom g, const float* __restrict__ taps) {
  constexpr int BATCH = TN < 8 ? TN : 8;  // row loads in flight per thread on the fast path
  const T* __restrict__ x = static_cast<const T*>(g.in);
  T* __restrict__ y = static_cast<T*>(g.out);
  float h[K];  // h[u] multiplies the input at lag u
#pragma unroll
  for (int u = 0; u < K; ++u) h[u] = __ldg(taps + (K - 1 - u));
  const int64_t CV = (g.C + VEC - 1) / VEC;
  const int64_t chunks = (g.N + TN - 1) / TN;
  const int64_t items = g.B * chunks * CV;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t cv = it % CV;
    const int64_t rest = it / CV;
    const int64_t chunk = rest % chunks;
    const int64_t b = rest / chunks;
    const int64_t c0 = cv * VEC;
    const T* xb = x + b * g.sib + c0 * g.sic;
    T* yb = y + b * g.sob + c0 * g.soc;
    float win[K][VEC];
    const int64_t n_first = chunk * TN;
    const int64_t n_last = min(n_first + TN, g.N) - 1;
    if (DIR > 0) {
      if (VEC * sizeof(T) == 16 && TN % BATCH == 0 && n_first >= K - 1 && n_first + TN <= g.N) {
        // interior run: the K-1 halo rows and the first BATCH rows requested together
        uint4 hr[K - 1], raw[BATCH];
#pragma unroll
        for (int u = 1; u < K; ++u) hr[u - 1] = __ldg(reinterpret_cast<const uint4*>(xb + (n_first - u) * g.sin));
#pragma unroll
        for (int t0 = 0; t0 < TN; t0 += BATCH) {
#pragma unroll
          for (int t = 0; t < BATCH; ++t) raw[t] = __ldg(reinterpret_cast<const uint4*>(xb + (n_first + t0 + t) * g.sin));
          if (t0 == 0) {
#pragma unroll
            for (int u = 1; u < K; ++u) {
              const T* e = reinterpret_cast<const T*>(&hr[u - 1]);
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = to_f32<T>(e[v]);
            }
          }
#pragma unroll
          for (int t = 0; t < BATCH; ++t) {
            const T* e = reinterpret_cast<const T*>(&raw[t]);
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[0][v] = to_f32<T>(e[v]);
            float acc[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float a = win[0][v] * h[0];
#pragma unroll
              for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
              acc[v] = a;
            }
            st_vec<T, VEC>(yb + (n_first + t0 + t) * g.son, acc);
#pragma unroll
            for (int u = K - 1; u > 0; --u)
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
          }
        }
        continue;
      }
      // win[u] = x[n-u]; prime lags 1..K-1 for n = n_first
#pragma unroll
      for (int u = 1; u < K; ++u) {
        const int64_t n = n_first - u;
        if (n >= 0) {
          if constexpr (VEC > 1) ld_vec<T, VEC>(xb + n * g.sin, win[u]);
          else win[u][0] = to_f32<T>(xb[n * g.sin]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) win[u][v] = 0.f;
        }
      }
      if (VEC * sizeof(T) == 16 && TN % BATCH == 0 && n_first + TN <= g.N) {
        // whole chunk inside the sequence: BATCH rows' loads issued before their use
#pragma unroll
        for (int t0 = 0; t0 < TN; t0 += BATCH) {
          uint4 raw[BATCH];
#pragma unroll
          for (int t = 0; t < BATCH; ++t) raw[t] = __ldg(reinterpret_cast<const uint4*>(xb + (n_first + t0 + t) * g.sin));
#pragma unroll
          for (int t = 0; t < BATCH; ++t) {
            const T* e = reinterpret_cast<const T*>(&raw[t]);
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[0][v] = to_f32<T>(e[v]);
            float acc[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float a = win[0][v] * h[0];
#pragma unroll
              for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
              acc[v] = a;
            }
            st_vec<T, VEC>(yb + (n_first + t0 + t) * g.son, acc);
#pragma unroll
            for (int u = K - 1; u > 0; --u)
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
          }
        }
        continue;
      }
#pragma unroll
      for (int t = 0; t < TN; ++t) {
        const int64_t n = n_first + t;
        if (n <= n_last) {
          if constexpr (VEC > 1) ld_vec<T, VEC>(xb + n * g.sin, win[0]);
          else win[0][0] = to_f32<T>(xb[n * g.sin]);
          float acc[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            float a = win[0][v] * h[0];
#pragma unroll
            for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
            acc[v] = a;
          }
          if constexpr (VEC > 1) st_vec<T, VEC>(yb + n * g.son, acc);
          else yb[n * g.son] = from_f32<T>(acc[0]);
#pragma unroll
          for (int u = K - 1; u > 0; --u)
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
        }
      }
    } else {
      if (VEC * sizeof(T) == 16 && TN % BATCH == 0 && n_last + K - 1 < g.N && n_first + TN <= g.N) {
        // interior run: the K-1 halo rows and the last BATCH rows requested together
        uint4 hr[K - 1], raw[BATCH];
#pragma unroll
        for (int u = 1; u < K; ++u) hr[u - 1] = __ldg(reinterpret_cast<const uint4*>(xb + (n_last + u) * g.sin));
#pragma unroll
        for (int t0 = TN - BATCH; t0 >= 0; t0 -= BATCH) {
#pragma unroll
          for (int t = 0; t < BATCH; ++t) raw[t] = __ldg(reinterpret_cast<const uint4*>(xb + (n_first + t0 + t) * g.sin));
          if (t0 == TN - BATCH) {
#pragma unroll
            for (int u = 1; u < K; ++u) {
              const T* e = reinterpret_cast<const T*>(&hr[u - 1]);
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = to_f32<T>(e[v]);
            }
          }
#pragma unroll
          for (int t = BATCH - 1; t >= 0; --t) {
            const T* e = reinterpret_cast<const T*>(&raw[t]);
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[0][v] = to_f32<T>(e[v]);
            float acc[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float a = win[0][v] * h[0];
#pragma unroll
              for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
              acc[v] = a;
            }
            st_vec<T, VEC>(yb + (n_first + t0 + t) * g.son, acc);
#pragma unroll
            for (int u = K - 1; u > 0; --u)
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
          }
        }
        continue;
      }
      // win[u] = gy[n+u]; prime lags 1..K-1 for n = n_last
#pragma unroll
      for (int u = 1; u < K; ++u) {
        const int64_t n = n_last + u;
        if (n < g.N) {
          if constexpr (VEC > 1) ld_vec<T, VEC>(xb + n * g.sin, win[u]);
          else win[u][0] = to_f32<T>(xb[n * g.sin]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) win[u][v] = 0.f;
        }
      }
      if (VEC * sizeof(T) == 16 && TN % BATCH == 0 && n_first + TN <= g.N) {
        // whole chunk inside the sequence: BATCH rows' loads issued before their use
#pragma unroll
        for (int t0 = TN - BATCH; t0 >= 0; t0 -= BATCH) {
          uint4 raw[BATCH];
#pragma unroll
          for (int t = 0; t < BATCH; ++t) raw[t] = __ldg(reinterpret_cast<const uint4*>(xb + (n_first + t0 + t) * g.sin));
#pragma unroll
          for (int t = BATCH - 1; t >= 0; --t) {
            const T* e = reinterpret_cast<const T*>(&raw[t]);
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[0][v] = to_f32<T>(e[v]);
            float acc[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
              float a = win[0][v] * h[0];
#pragma unroll
              for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
              acc[v] = a;
            }
            st_vec<T, VEC>(yb + (n_first + t0 + t) * g.son, acc);
#pragma unroll
            for (int u = K - 1; u > 0; --u)
#pragma unroll
              for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
          }
        }
        continue;
      }
#pragma unroll
      for (int t = TN - 1; t >= 0; --t) {
        const int64_t n = n_first + t;
        if (n <= n_last) {
          if constexpr (VEC > 1) ld_vec<T, VEC>(xb + n * g.sin, win[0]);
          else win[0][0] = to_f32<T>(xb[n * g.sin]);
          float acc[VEC];
#pragma unroll
          for (int v = 0; v < VEC; ++v) {
            float a = win[0][v] * h[0];
#pragma unroll
            for (int u = 1; u < K; ++u) a = fmaf(win[u][v], h[u], a);
            acc[v] = a;
          }
          if constexpr (VEC > 1) st_vec<T, VEC>(yb + n * g.son, acc);
          else yb[n * g.son] = from_f32<T>(acc[0]);
#pragma unroll
          for (int u = K - 1; u > 0; --u)
#pragma unroll
            for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
        }
      }
    }
  }
}

// Any tap count (1..FIR_MAX_TAPS), any strides: one output element per thread.
template <typename T, int DIR>
__global__ void __launch_bounds__(FIR_THREADS) fir_generic_kernel(FirGeom g, const float* __restrict__ taps, int K) {
  const T* __restrict__ x = static_cast<const T*>(g.in);
  T* __restrict__ y = static_cast<T*>(g.out);
  const int64_t total = g.B * g.N * g.C;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < total;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = it % g.C;
    const int64_t n = (it / g.C) % g.N;
    const int64_t b = it / (g.C * g.N);
    const T* xb = x + b * g.sib + c * g.sic;
    float a = 0.f;
    for (int u = 0; u < K; ++u) {
      const int64_t src = DIR > 0 ? n - u : n + u;  // causal: past rows; transpose: future rows
      if (src < 0 || src >= g.N) continue;
      a = fmaf(to_f32<T>(xb[src * g.sin]), __ldg(taps + (K - 1 - u)), a);
    }
    y[b * g.sob + n * g.son + c * g.soc] = from_f32<T>(a);
  }
}

// Tap gradient, one lag per grid row: partial[u][blockIdx.x] =
// sum over this block's elements of gy[b,n,c] * x[b,n-u,c].
template <typename T>
__global__ void __launch_bounds__(FIR_THREADS) fir_dtaps_partial_kernel(
    const T* __restrict__ gy, int64_t sgb, int64_t sgn, int64_t sgc, const T* __restrict__ x,
    int64_t sxb, int64_t sxn, int64_t sxc, int64_t B, int64_t N, int64_t C, float* __restrict__ partial) {
  __shared__ float red[FIR_THREADS / 32];
  const int u = blockIdx.y;
  const int64_t total = B * N * C;
  float acc = 0.f;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < total;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = it % C;
    const int64_t n = (it / C) % N;
    const int64_t b = it / (C * N);
    if (n - u < 0) continue;
    acc = fmaf(to_f32<T>(gy[b * sgb + n * sgn + c * sgc]), to_f32<T>(x[b * sxb + (n - u) * sxn + c * sxc]), acc);
  }
  const float s = block_sum(acc, red);
  if (threadIdx.x == 0) partial[(int64_t)u * gridDim.x + blockIdx.x] = s;
}

// Tap gradient in one pass over gy and x (16-byte channel vectors, unit channel
// stride): a thread owns VEC channels of a run of TN rows, keeps x[n-K+1..n] in a
// register window and adds gy[n,c] * x[n-u,c] to acc[u] for every lag u at once,
// so gy and x are read once (plus the K-1 halo rows of each run, from L1/L2)
// instead of once per lag. Grid-stride over (b, run, channel vector) with a fixed
// grid; partial[u][block] = the block's sum for lag u (reduced in fp64 in block
// order by fir_dtaps_final_kernel, so the result is deterministic).
template <typename T, int VEC, int K, int TN>
__global__ void __launch_bounds__(FIR_THREADS) fir_dtaps_sliding_kernel(
    const T* __restrict__ gy, int64_t sgb, int64_t sgn, const T* __restrict__ x, int64_t sxb, int64_t sxn,
    int64_t B, int64_t N, int64_t C, float* __restrict__ partial) {
  __shared__ float red[K][FIR_THREADS / 32];
  float acc[K];
#pragma unroll
  for (int u = 0; u < K; ++u) acc[u] = 0.f;
  const int64_t CV = C / VEC, chunks = (N + TN - 1) / TN, items = B * chunks * CV;
  for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t cv = it % CV, rest = it / CV, chunk = rest % chunks, b = rest / chunks;
    const T* xb = x + b * sxb + cv * VEC;
    const T* gb = gy + b * sgb + cv * VEC;
    const int64_t n0 = chunk * TN;
    float win[K][VEC];  // win[u] = x[n-u]
    const int rows = (int)min((int64_t)TN, N - n0);
    auto step = [&](const uint4& xr, const uint4& gr) {
      float gv[VEC];
      const T* xe = reinterpret_cast<const T*>(&xr);
      const T* ge = reinterpret_cast<const T*>(&gr);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        win[0][v] = to_f32<T>(xe[v]);
        gv[v] = to_f32<T>(ge[v]);
      }
#pragma unroll
      for (int u = 0; u < K; ++u)
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[u] = fmaf(gv[v], win[u][v], acc[u]);
#pragma unroll
      for (int u = K - 1; u > 0; --u)
#pragma unroll
        for (int v = 0; v < VEC; ++v) win[u][v] = win[u - 1][v];
    };
    if (rows == TN && n0 >= K - 1) {
      // interior run: the halo rows of x and every row of x and gy requested before use
      uint4 hr[K - 1], xr[TN], gr[TN];
#pragma unroll
      for (int u = 1; u < K; ++u) hr[u - 1] = __ldg(reinterpret_cast<const uint4*>(xb + (n0 - u) * sxn));
#pragma unroll
      for (int t = 0; t < TN; ++t) {
        xr[t] = __ldg(reinterpret_cast<const uint4*>(xb + (n0 + t) * sxn));
        gr[t] = __ldg(reinterpret_cast<const uint4*>(gb + (n0 + t) * sgn));
      }
#pragma unroll
      for (int u = 1; u < K; ++u) {
        const T* e = reinterpret_cast<const T*>(&hr[u - 1]);
#pragma unroll
        for (int v = 0; v < VEC; ++v) win[u][v] = to_f32<T>(e[v]);
      }
#pragma unroll
      for (int t = 0; t < TN; ++t) step(xr[t], gr[t]);
    } else {
#pragma unroll
      for (int u = 1; u < K; ++u) {
        if (n0 - u >= 0) {
          ld_vec<T, VEC>(xb + (n0 - u) * sxn, win[u]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) win[u][v] = 0.f;
        }
      }
      for (int t = 0; t < rows; ++t)
        step(__ldg(reinterpret_cast<const uint4*>(xb + (n0 + t) * sxn)),
             __ldg(reinterpret_cast<const uint4*>(gb + (n0 + t) * sgn)));
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int u = 0; u < K; ++u) {
    const float s = group_sum<32>(acc[u]);
    if (lane == 0) red[u][warp] = s;
  }
  __syncthreads();
  if (threadIdx.x < K) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < FIR_THREADS / 32; ++w) s += red[threadIdx.x][w];
    partial[(int64_t)threadIdx.x * gridDim.x + blockIdx.x] = s;
  }
}

// dtaps[K-1-u] = fp64 sum over the partials of lag u: one warp per lag, lane l adds
// blocks l, l+32, ... in order, then a fixed butterfly across the lanes, so the
// rounding is the same on every run.
__global__ void fir_dtaps_final_kernel(const float* __restrict__ partial, int nblk, int K, float* __restrict__ dtaps) {
  const int u = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (u >= K) return;
  double s = 0.0;
  for (int i = lane; i < nblk; i += 32) s += (double)partial[(int64_t)u * nblk + i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) dtaps[K - 1 - u] = (float)s;
}
static void dtaps_final(const float* part, int nblk, int K, float* dtaps, cudaStream_t st) {
  constexpr int WARPS = 8;
  fir_dtaps_final_kernel<<<(K + WARPS - 1) / WARPS, 32 * WARPS, 0, st>>>(part, nblk, K, dtaps);
}

static int grid_for(int64_t items) {
  int64_t g = (items + FIR_THREADS - 1) / FIR_THREADS;
  if (g < 1) g = 1;
  if (g > (int64_t)1 << 20) g = (int64_t)1 << 20;
  return (int)g;
}

template <typename T>
static bool vec_ok(const FirGeom& g) {
  constexpr int VEC = 16 / sizeof(T);
  const uintptr_t a = reinterpret_cast<uintptr_t>(g.in), b = reinterpret_cast<uintptr_t>(g.out);
  return g.sic == 1 && g.soc == 1 && g.C % VEC == 0 && a % 16 == 0 && b % 16 == 0 && g.sin % VEC == 0 &&
         g.sib % VEC == 0 && g.son % VEC == 0 && g.sob % VEC == 0;
}

template <typename T, int DIR>
static int fir_launch(const FirGeom& g, const float* taps, int K, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  if (K == 7) {
    const int64_t chunks = (g.N + FIR_TN - 1) / FIR_TN;
    if (vec_ok<T>(g)) {
      // the longest run of rows per thread (the 6-row halo, the index math and the
      // load round trips amortised over 32, 16 or 8 rows) that still gives at least
      // 1.5 blocks of 256 threads per SM of a B200 (measured: 32-row runs 14.7 us
      // against 24.0 us for 8-row runs on [8, 4096, 512]; on [32, 512, 256], where
      // longer runs leave SMs idle, 8-row runs 7.5 us against 9.6 us for 4-row runs)
      const int64_t CV = g.C / VEC, enough = 148 * FIR_THREADS * 3 / 2;
      const int64_t items32 = g.B * ((g.N + 31) / 32) * CV, items16 = g.B * ((g.N + 15) / 16) * CV;
      if (items32 >= enough) {
        fir_sliding_kernel<T, VEC, 7, DIR, 32><<<grid_for(items32), FIR_THREADS, 0, st>>>(g, taps);
      } else if (items16 >= enough) {
        fir_sliding_kernel<T, VEC, 7, DIR, 16><<<grid_for(items16), FIR_THREADS, 0, st>>>(g, taps);
      } else {
        fir_sliding_kernel<T, VEC, 7, DIR><<<grid_for(g.B * chunks * CV), FIR_THREADS, 0, st>>>(g, taps);
      }
    } else {
      const int64_t items = g.B * chunks * g.C;
      fir_sliding_kernel<T, 1, 7, DIR><<<grid_for(items), FIR_THREADS, 0, st>>>(g, taps);
    }
  } else {
    fir_generic_kernel<T, DIR><<<grid_for(g.B * g.N * g.C), FIR_THREADS, 0, st>>>(g, taps, K);
  }
  return check_launch(DIR > 0 ? "fir fwd" : "fir bwd");
}

static int64_t dtaps_blocks(int64_t B, int64_t N, int64_t C) {
  int64_t g = (B * N * C + FIR_THREADS - 1) / FIR_THREADS;
  if (g < 1) g = 1;
  if (g > FIR_DTAPS_MAX_BLOCKS) g = FIR_DTAPS_MAX_BLOCKS;
  return g;
}

// Tap-gradient partials: the one-pass sliding kernel for 7 taps on 16-byte
// aligned rows with unit channel stride, else the per-lag kernel. Returns the
// number of blocks (<= dtaps_blocks(B, N, C)) whose partials partial[u][block]
// the final reduction sums.
template <typename T>
static int dtaps_partials(const T* gy, int64_t sgb, int64_t sgn, int64_t sgc, const T* x, int64_t sxb, int64_t sxn,
                          int64_t sxc, int64_t B, int64_t N, int64_t C, int K, float* part, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int TN = 8;
  const int nmax = (int)dtaps_blocks(B, N, C);
  const bool vec = K == 7 && sgc == 1 && sxc == 1 && C % VEC == 0 && sgn % VEC == 0 && sgb % VEC == 0 &&
                   sxn % VEC == 0 && sxb % VEC == 0 && reinterpret_cast<uintptr_t>(gy) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0;
  if (vec) {
    const int64_t items = B * ((N + TN - 1) / TN) * (C / VEC);
    int nblk = (int)std::min<int64_t>(nmax, (items + FIR_THREADS - 1) / FIR_THREADS);
    if (nblk < 1) nblk = 1;
    fir_dtaps_sliding_kernel<T, VEC, 7, TN><<<nblk, FIR_THREADS, 0, st>>>(gy, sgb, sgn, x, sxb, sxn, B, N, C, part);
    return nblk;
  }
  fir_dtaps_partial_kernel<T><<<dim3(nmax, K), FIR_THREADS, 0, st>>>(gy, sgb, sgn, sgc, x, sxb, sxn, sxc, B, N, C,
                                                                    part);
  return nmax;
}

// Scratch of pnft_fir_bwd_noalloc: the per-block, per-lag partial sums of the tap
// gradient (at most FIR_MAX_TAPS lags x FIR_DTAPS_MAX_BLOCKS blocks = 128 KiB).
// It lives in the module image, so every GPU that loads the library holds it
// until the process exits. Each call writes every slot it later reads before
// reading it, so nothing has to start at zero; two calls that overlap on the
// GPU (different streams, or host threads) share it and race.
static __device__ __align__(256) float g_dtaps_scratch[FIR_MAX_TAPS * FIR_DTAPS_MAX_BLOCKS];

constexpr int kMaxDevices = 64;

// Device address of g_dtaps_scratch on the current device, looked up once per
// device (the host-side symbol is only a stand-in, never a device address).
static int dtaps_scratch_ptr(float** out) {
  static std::mutex mu;
  static float* ptrs[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(PNFT_ECUDA, "fir bwd noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(PNFT_EUNSUPPORTED, "fir bwd noalloc: device %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dtaps_scratch);
    if (e != cudaSuccess)
      return fail(PNFT_ECUDA, "fir bwd noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    ptrs[dev] = static_cast<float*>(p);
  }
  *out = ptrs[dev];
  return PNFT_OK;
}

}  // namespace pnft

using namespace pnft;

extern "C" size_t pnft_fir_bwd_workspace_size(int64_t B, int64_t N, int64_t C, int ntaps) {
  if (B <= 0 || N <= 0 || C <= 0 || ntaps <= 0) return 0;
  return (size_t)dtaps_blocks(B, N, C) * (size_t)ntaps * sizeof(float);
}

static int fir_check_common(const void* in, const void* out, const float* taps, int ntaps, int64_t B,
                            int64_t N, int64_t C, bool need_out) {
  if (B < 0 || N < 0 || C < 0) return fail(PNFT_EINVAL, "fir: negative size B=%lld N=%lld C=%lld", (long long)B, (long long)N, (long long)C);
  if (ntaps < 1 || ntaps > FIR_MAX_TAPS) return fail(PNFT_EINVAL, "fir: ntaps=%d outside [1,%d]", ntaps, FIR_MAX_TAPS);
  if (!in || (need_out && !out) || !taps) return fail(PNFT_EINVAL, "fir: null pointer");
  return PNFT_OK;
}

extern "C" int pnft_fir_fwd(const void* x, int64_t sxb, int64_t sxn, int64_t sxc, const float* taps, int ntaps,
                            void* y, int64_t syb, int64_t syn, int64_t syc, int64_t B, int64_t N, int64_t C,
                            int dtype, void* stream) {
  if (B == 0 || N == 0 || C == 0) return PNFT_OK;
  int rc = fir_check_common(x, y, taps, ntaps, B, N, C, true);
  if (rc) return rc;
  FirGeom g{x, y, sxb, sxn, sxc, syb, syn, syc, B, N, C};
  PNFT_DISPATCH_DTYPE(dtype, T, return fir_launch<T, +1>(g, taps, ntaps, as_stream(stream)));
  return PNFT_OK;
}

extern "C" int pnft_fir_bwd(const void* gy, int64_t sgb, int64_t sgn, int64_t sgc, const float* taps, int ntaps,
                            void* gx, int64_t sxb, int64_t sxn, int64_t sxc, const void* x, int64_t s0b,
                            int64_t s0n, int64_t s0c, float* dtaps, void* workspace, size_t workspace_bytes,
                            int64_t B, int64_t N, int64_t C, int dtype, void* stream) {
  int rc = fir_check_common(gy, gx, taps, ntaps, B, N, C, false);
  if (rc) return rc;
  if (!gx && !x) return fail(PNFT_EINVAL, "fir bwd: nothing to compute (gx and x are both NULL)");
  cudaStream_t st = as_stream(stream);
  if (x) {
    if (!dtaps) return fail(PNFT_EINVAL, "fir bwd: x given but dtaps is NULL");
    if (B == 0 || N == 0 || C == 0) {
      if (cudaMemsetAsync(dtaps, 0, sizeof(float) * ntaps, st) != cudaSuccess) return check_launch("fir dtaps memset");
    } else {
      const size_t need = pnft_fir_bwd_workspace_size(B, N, C, ntaps);
      if (!workspace || workspace_bytes < need)
        return fail(PNFT_EINVAL, "fir bwd: workspace of %zu bytes < required %zu", workspace_bytes, need);
      int nblk = 0;
      float* part = static_cast<float*>(workspace);
      PNFT_DISPATCH_DTYPE(dtype, T, {
        nblk = dtaps_partials<T>(static_cast<const T*>(gy), sgb, sgn, sgc, static_cast<const T*>(x), s0b, s0n, s0c,
                                 B, N, C, ntaps, part, st);
      });
      dtaps_final(part, nblk, ntaps, dtaps, st);
      rc = check_launch("fir dtaps", 2);
      if (rc) return rc;
    }
  }
  if (gx && B > 0 && N > 0 && C > 0) {
    FirGeom g{gy, gx, sgb, sgn, sgc, sxb, sxn, sxc, B, N, C};
    PNFT_DISPATCH_DTYPE(dtype, T, return fir_launch<T, -1>(g, taps, ntaps, st));
  }
  return PNFT_OK;
}

// Allocation-free variant of pnft_fir_bwd for callers that cannot hand the
// library device memory of its choosing (see the header): identical results,
// with the tap-gradient partial sums kept in the static g_dtaps_scratch. The
// first call on a device looks the scratch address up (keep that first call
// out of any stream capture); calls that overlap on the GPU share the scratch.
extern "C" int pnft_fir_bwd_noalloc(const void* gy, int64_t sgb, int64_t sgn, int64_t sgc, const float* taps,
                                    int ntaps, void* gx, int64_t sxb, int64_t sxn, int64_t sxc, const void* x,
                                    int64_t s0b, int64_t s0n, int64_t s0c, float* dtaps, int64_t B, int64_t N,
                                    int64_t C, int dtype, void* stream) {
  if (ntaps > FIR_MAX_TAPS)
    return fail(PNFT_EINVAL, "fir bwd noalloc: ntaps=%d exceeds the %d lags its static scratch holds", ntaps,
                FIR_MAX_TAPS);
  int rc = fir_check_common(gy, gx, taps, ntaps, B, N, C, false);
  if (rc) return rc;
  if (!x || !dtaps) return fail(PNFT_EINVAL, "fir bwd noalloc: x and dtaps are required (tap gradient entry point)");
  cudaStream_t st = as_stream(stream);
  if (B == 0 || N == 0 || C == 0) {
    if (cudaMemsetAsync(dtaps, 0, sizeof(float) * ntaps, st) != cudaSuccess) return check_launch("fir dtaps memset", 0);
    return PNFT_OK;
  }
  float* part = nullptr;
  rc = dtaps_scratch_ptr(&part);
  if (rc) return rc;
  int nblk = 0;  // <= dtaps_blocks(B, N, C) <= FIR_DTAPS_MAX_BLOCKS by construction
  PNFT_DISPATCH_DTYPE(dtype, T, {
    nblk = dtaps_partials<T>(static_cast<const T*>(gy), sgb, sgn, sgc, static_cast<const T*>(x), s0b, s0n, s0c, B, N,
                             C, ntaps, part, st);
  });
  dtaps_final(part, nblk, ntaps, dtaps, st);
  rc = check_launch("fir dtaps noalloc", 2);
  if (rc) return rc;
  if (gx) {
    FirGeom g{gy, gx, sgb, sgn, sgc, sxb, sxn, sxc, B, N, C};
    PNFT_DISPATCH_DTYPE(dtype, T, return fir_launch<T, -1>(g, taps, ntaps, st));
  }
  return PNFT_OK;
}
