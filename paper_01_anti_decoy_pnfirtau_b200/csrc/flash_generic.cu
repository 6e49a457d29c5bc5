// Generic (SIMT, fp32-FMA) flash pn_fir_tau kernels: any dtype, any strides,
// head dim D <= 128, any N. They serve every shape the tcgen05 kernels do not
// (fp32 inputs for the reference's fp32 parity harness, D of 16/32, odd
// strides) and define the arithmetic the fast kernels are checked against.
//
// Forward (src/triton_pnfirtau.py:313-443), per 64-query block:
//   for each 64-key tile j <= the diagonal (causal):
//     S = Q K^T ; s = S*scale - tau ; u = relu(s) on col <= row
//     if max(u) over the tile <= 0: skip (no u^10, no V load, no PV)
//     peak' = max(peak, rowmax u); ties counted against peak'; mass += sum u^10
//     acc += u^10 V
//   O = acc * gate/(mass+1e-12), gate = peak/(peak+gamma) (1 without gamma, 0 if silent)
// Backward (src/triton_pnfirtau.py:445-621), per 64-key block, over query
// blocks at or below the diagonal: recompute S and u, W = u^10*gate/z,
// dV += W^T dO, dP = dO V^T, du = 10*gate/z*u^9*(dP - D) + [u==peak]*tie,
// dS = du*scale, dK += dS^T Q, dQ += dS K (fp32 atomics), dtau -= sum du.
// D = <dO,O>/gate and the tie coefficient are per-row values computed once by
// flash_bwd_prep.
//
// S is recomputed in the backward by the same `tile_dot` routine (same FMA
// order), so u == peak identifies exactly the forward's maxima.
#include <type_traits>

#include "flash.cuh"

namespace pnft {

constexpr int GB = 64;        // query and key tile
constexpr int GTHREADS = 256; // 16 row groups x 16 column groups

template <int DP>
struct GenSmem {
  static constexpr int LD = DP + 1;  // padded row: conflict-free row and column walks
  static constexpr int TILE = GB * LD;
  static constexpr int LDP = GB + 1;
  static constexpr size_t fwd_bytes = (size_t)(3 * TILE + GB * LDP) * sizeof(float);
  static constexpr size_t bwd_bytes = (size_t)(4 * TILE + 2 * GB * LDP + 4 * GB + 3 * GB) * sizeof(float);
};

// dst[r][e] (row stride ld) = src[n0 + r, e] for r < 64, e < DP; zero outside N/D.
template <typename T, int DP>
__device__ __forceinline__ void load_tile(float* __restrict__ dst, const T* __restrict__ src, int64_t s_n,
                                          int64_t s_d, int64_t n0, int64_t N, int D) {
  constexpr int LD = DP + 1;
  for (int idx = threadIdx.x; idx < GB * DP; idx += GTHREADS) {
    const int r = idx / DP, e = idx % DP;
    const int64_t n = n0 + r;
    float v = 0.f;
    if (n < N && e < D) v = to_f32<T>(src[n * s_n + e * s_d]);
    dst[r * LD + e] = v;
  }
}

// acc[ii][jj] = sum_e A[rg+16ii][e] * Bm[cg+16jj][e]  (both row-major, ld = DP+1)
template <int DP>
__device__ __forceinline__ void tile_dot(float (&acc)[4][4], const float* __restrict__ A,
                                         const float* __restrict__ Bm, int rg, int cg) {
  constexpr int LD = DP + 1;
#pragma unroll
  for (int ii = 0; ii < 4; ++ii)
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[ii][jj] = 0.f;
#pragma unroll 8
  for (int e = 0; e < DP; ++e) {
    float a[4], bv[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) a[ii] = A[(rg + 16 * ii) * LD + e];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) bv[jj] = Bm[(cg + 16 * jj) * LD + e];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) acc[ii][jj] = fmaf(a[ii], bv[jj], acc[ii][jj]);
  }
}

__device__ __forceinline__ float pow10f_(float u) {
  const float u2 = u * u, u4 = u2 * u2;
  return u4 * u4 * u2;
}

template <typename T, int DP>
__global__ void __launch_bounds__(GTHREADS) flash_fwd_generic_kernel(FlashArgs a) {
  extern __shared__ float smem[];
  using SM = GenSmem<DP>;
  constexpr int LD = SM::LD, LDP = SM::LDP, NJ = DP / 16;
  float* sQ = smem;
  float* sK = sQ + SM::TILE;
  float* sV = sK + SM::TILE;
  float* sP = sV + SM::TILE;
  const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  const int64_t q0 = (int64_t)blockIdx.x * GB;
  const int64_t bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int D = (int)a.D;
  const int64_t N = a.N;
  const T* Q = static_cast<const T*>(a.q) + b * a.sq[0] + h * a.sq[1];
  const T* K = static_cast<const T*>(a.k) + b * a.sk[0] + h * a.sk[1];
  const T* V = static_cast<const T*>(a.v) + b * a.sv[0] + h * a.sv[1];
  load_tile<T, DP>(sQ, Q, a.sq[2], a.sq[3], q0, N, D);
  const float tau = __ldg(a.tau);
  float peak[4], mass[4], acc[4][NJ];
  int nmax[4], arg[4];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    peak[ii] = 0.f; mass[ii] = 0.f; nmax[ii] = 0; arg[ii] = -1;
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) acc[ii][jj] = 0.f;
  }
  const int64_t hi = a.causal ? min(q0 + GB, N) : N;
  for (int64_t k0 = 0; k0 < hi; k0 += GB) {
    __syncthreads();
    load_tile<T, DP>(sK, K, a.sk[2], a.sk[3], k0, N, D);
    __syncthreads();
    float u[4][4];
    tile_dot<DP>(u, sQ, sK, rg, cg);
    int live = 0;
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int64_t row = q0 + rg + 16 * ii;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int64_t col = k0 + cg + 16 * jj;
        const bool valid = row < N && col < N && (!a.causal || col <= row);
        const float s = u[ii][jj] * a.scale - tau;
        u[ii][jj] = (valid && s > 0.f) ? s : 0.f;
        live |= u[ii][jj] > 0.f;
      }
    }
    if (!__syncthreads_or(live)) continue;  // silent tile: no u^10, no V load, no PV
    if (a.tile_flags && tid == 0) {
      const int64_t nt = (N + GB - 1) / GB;
      a.tile_flags[(bh * nt + blockIdx.x) * nt + k0 / GB] = 1;
    }
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      float tmax = fmaxf(fmaxf(u[ii][0], u[ii][1]), fmaxf(u[ii][2], u[ii][3]));
      tmax = group_max<16>(tmax);
      const float np = fmaxf(peak[ii], tmax);
      int cnt = 0, first = 0x7fffffff;
      float rm = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const bool hit = np > 0.f && u[ii][jj] == np;
        cnt += hit ? 1 : 0;
        if (hit) first = min(first, (int)(k0 + cg + 16 * jj));
        const float pw = pow10f_(u[ii][jj]);
        rm += pw;
        sP[(rg + 16 * ii) * LDP + cg + 16 * jj] = pw;
      }
      cnt = group_sum_i<16>(cnt);
      first = group_min_i<16>(first);
      rm = group_sum<16>(rm);
      if (np > peak[ii]) arg[ii] = first;  // a tie with an earlier tile keeps the earlier key
      nmax[ii] = np > peak[ii] ? cnt : nmax[ii] + cnt;
      peak[ii] = np;
      mass[ii] += rm;
    }
    load_tile<T, DP>(sV, V, a.sv[2], a.sv[3], k0, N, D);
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < GB; ++j) {
      float p[4], vv[NJ];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) p[ii] = sP[(rg + 16 * ii) * LDP + j];
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) vv[jj] = sV[j * LD + cg + 16 * jj];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) acc[ii][jj] = fmaf(p[ii], vv[jj], acc[ii][jj]);
    }
  }
  T* O = static_cast<T*>(a.out) + b * a.so[0] + h * a.so[1];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int64_t row = q0 + rg + 16 * ii;
    if (row >= N) continue;
    const float z = mass[ii] + 1e-12f;
    float gate = 0.f;
    if (peak[ii] > 0.f) gate = a.has_gamma ? peak[ii] / (peak[ii] + a.gamma) : 1.f;
    const float so = gate / z;
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) {
      const int e = cg + 16 * jj;
      if (e < D) {
        O[row * a.so[2] + e * a.so[3]] = from_f32<T>(acc[ii][jj] * so);
        if (a.out32) a.out32[(bh * N + row) * D + e] = acc[ii][jj] * so;
      }
    }
    if (cg == 0) {
      const int64_t si = bh * N + row;
      a.stat_m[si] = peak[ii];
      a.stat_z[si] = z;
      a.stat_nmax[si] = nmax[ii];
      a.stat_arg[si] = arg[ii];
    }
  }
}

// Per query row (RowCoef in flash.cuh): D = <dO,O>/gate (0 if gate == 0) and
// tie = D*gamma/(peak+gamma)^2/Nmax (0 without gamma or for silent rows). One
// block per (64-row tile, b*h) also records whether any row of the tile is live.
template <typename T>
__global__ void __launch_bounds__(256) flash_bwd_prep_kernel(FlashArgs a) {
  // 8 lanes per row, 4 rows per warp and pass, 2 passes: 64 rows per block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane >> 3, sl = lane & 7;
  const int64_t bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int64_t nt = (a.N + 63) / 64, npad = nt * 64;
  // bf16 dO: 16-byte loads, lane sl reads head dims [8sl + 64k, +8) of dO and the fp32 O
  const bool vec = std::is_same<T, __nv_bfloat16>::value && a.out32 && (a.D % 64) == 0 && a.sdo[3] == 1 && (a.sdo[2] % 8) == 0 &&
                   (a.sdo[1] % 8) == 0 && (a.sdo[0] % 8) == 0 && (reinterpret_cast<uintptr_t>(a.dout) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.out32) & 15) == 0;
  {  // this block's rows of the fp32 dQ accumulator start at zero (the backward adds into them)
    const int64_t n0 = (int64_t)blockIdx.x * 64, cnt = (min((int64_t)64, a.N - n0)) * a.acc_d;
    float* z = a.dq_acc + (bh * a.N + n0) * a.acc_d;
    if ((reinterpret_cast<uintptr_t>(z) & 15) == 0 && (cnt & 3) == 0) {
      for (int64_t i = threadIdx.x; i < cnt / 4; i += blockDim.x) reinterpret_cast<float4*>(z)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int64_t i = threadIdx.x; i < cnt; i += blockDim.x) z[i] = 0.f;
    }
  }
  int live = 0, multi = 0;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int64_t n = (int64_t)blockIdx.x * 64 + warp * 8 + pass * 4 + sub;
    const bool ok = n < a.N;
    const int64_t r = bh * a.N + (ok ? n : 0);
    const T* O = static_cast<const T*>(a.out_c) + b * a.so[0] + h * a.so[1] + (ok ? n : 0) * a.so[2];
    const T* dO = static_cast<const T*>(a.dout) + b * a.sdo[0] + h * a.sdo[1] + (ok ? n : 0) * a.sdo[2];
    float dot = 0.f;
    if (ok && vec) {
      for (int e0 = 8 * sl; e0 < a.D; e0 += 64) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(dO + e0));
        const float4* o4 = reinterpret_cast<const float4*>(a.out32 + r * a.D + e0);
        const float4 o0 = __ldg(o4), o1 = __ldg(o4 + 1);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float os[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dot = fmaf(__uint_as_float(ws[i] << 16), os[2 * i], dot);
          dot = fmaf(__uint_as_float(ws[i] & 0xffff0000u), os[2 * i + 1], dot);
        }
      }
    } else if (ok) {
      if (a.out32) {
        const float* O32 = a.out32 + r * a.D;
        for (int e = sl; e < a.D; e += 8) dot = fmaf(to_f32<T>(dO[e * a.sdo[3]]), O32[e], dot);
      } else {
        for (int e = sl; e < a.D; e += 8) dot = fmaf(to_f32<T>(dO[e * a.sdo[3]]), to_f32<T>(O[e * a.so[3]]), dot);
      }
    }
    dot = group_sum<8>(dot);
    const float peak = ok ? a.stat_m[r] : 0.f;
    live |= peak > 0.f;
    if (sl == 0) {
      // rows past N get the record of a silent row (the tile loads read all 64)
      float c1 = 0.f, Dg = 0.f, tie = 0.f;
      int arg = -1, nm = 0;
      float pcmp = __int_as_float(0x7fc00000);  // NaN never compares equal
      if (ok) {
        const float z = a.stat_z[r];
        nm = a.stat_nmax[r];
        arg = a.stat_arg[r];
        float gate = 0.f;
        if (peak > 0.f) gate = a.has_gamma ? peak / (peak + a.gamma) : 1.f;
        Dg = gate > 0.f ? dot / gate : 0.f;
        if (a.has_gamma && peak > 0.f) {
          const float pg = peak + a.gamma;
          tie = Dg * (a.gamma / (pg * pg)) / (float)nm;  // d out / d peak per maximum (du units)
        }
        c1 = gate / z;
        // single maximum: matched by key index; genuine ties (Nmax > 1): by value
        if (nm > 1) pcmp = peak;
      }
      const int64_t rr = bh * npad + n;
      float* cp = reinterpret_cast<float*>(a.coefP) + (rr >> 1) * 4 + (rr & 1);
      cp[0] = c1;
      cp[2] = -Dg;
      a.tiev[rr] = 0.1f * tie;  // dS = scale * du; dS' = dS / (10 scale)
      a.argv[rr] = arg;
      a.pcmpv[rr] = pcmp;
      if (nm > 1) multi = 1;
    }
  }
  live = __syncthreads_or(live);
  multi = __syncthreads_or(multi);
  if (threadIdx.x == 0) {
    a.live64[bh * nt + blockIdx.x] = (live ? kLiveRow : 0) | (multi ? kMultiTie : 0);
    a.dq_sem[bh * nt + blockIdx.x] = 0;  // no dQ contribution added yet (deterministic mode)
    if (bh == 0 && blockIdx.x == 0) *a.dq_ticket = 0;
  }
}

template <typename T, int DP>
__global__ void __launch_bounds__(GTHREADS) flash_bwd_generic_kernel(FlashArgs a) {
  extern __shared__ float smem[];
  using SM = GenSmem<DP>;
  constexpr int LD = SM::LD, LDP = SM::LDP, NJ = DP / 16;
  float* sK = smem;
  float* sV = sK + SM::TILE;
  float* sQ = sV + SM::TILE;
  float* sdO = sQ + SM::TILE;
  float* sW = sdO + SM::TILE;
  float* sdS = sW + GB * LDP;
  float4* sC = reinterpret_cast<float4*>(sdS + GB * LDP);  // {-, gate/z, 10*scale*gate/z, D}
  float* sTie = reinterpret_cast<float*>(sC + GB);          // scale * tie coefficient
  int* sArg = reinterpret_cast<int*>(sTie + GB);            // argmax key of the row
  float* sPc = reinterpret_cast<float*>(sArg + GB);         // peak for the value test (NaN: unused)
  const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  // deterministic mode: key blocks add their dQ contributions to each query tile in
  // key order (turn counters); blocks take their (key block, b*h) from a ticket in
  // grid order, so a block only ever waits for blocks that started before it
  const bool det = (a.flags & PNFT_FLASH_DETERMINISTIC) != 0;
  int64_t kt_ = blockIdx.x, bh_ = blockIdx.y;
  if (det) {
    __shared__ int s_ticket;
    if (tid == 0) s_ticket = atomicAdd(a.dq_ticket, 1);
    __syncthreads();
    kt_ = s_ticket % (int)gridDim.x;
    bh_ = s_ticket / (int)gridDim.x;
  }
  const int64_t kt = kt_, k0 = kt * GB;
  const int64_t bh = bh_, b = bh / a.H, h = bh % a.H;
  const int D = (int)a.D;
  const int64_t N = a.N;
  int32_t* sem_bh = a.dq_sem + bh * ((N + GB - 1) / GB);
  // this block's turn on query tile q0 (det mode): wait for the lower key blocks,
  // optionally add (plain read-modify-write through L2), pass the turn on
  auto det_turn_wait = [&](int64_t q0) {
    if (tid == 0) turn_wait(sem_bh + q0 / GB, (int)kt, a.status, nullptr);
    __syncthreads();
  };
  auto det_turn_pass = [&](int64_t q0) {
    __syncthreads();
    if (tid == 0) turn_pass(sem_bh + q0 / GB);
  };
  const T* Q = static_cast<const T*>(a.q) + b * a.sq[0] + h * a.sq[1];
  const T* K = static_cast<const T*>(a.k) + b * a.sk[0] + h * a.sk[1];
  const T* V = static_cast<const T*>(a.v) + b * a.sv[0] + h * a.sv[1];
  const T* dO = static_cast<const T*>(a.dout) + b * a.sdo[0] + h * a.sdo[1];
  float* dQa = a.dq_acc + bh * N * a.acc_d;
  load_tile<T, DP>(sK, K, a.sk[2], a.sk[3], k0, N, D);
  load_tile<T, DP>(sV, V, a.sv[2], a.sv[3], k0, N, D);
  const float tau = __ldg(a.tau);
  float dk[4][NJ], dv[4][NJ];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii)
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) dk[ii][jj] = dv[ii][jj] = 0.f;
  float dtau = 0.f;
  const int64_t lo = a.causal ? k0 : 0;
  // query tiles in ascending order; deterministic mode walks them downwards, so the
  // blocks of a head reach a query tile at about the same time and the key-ordered
  // dQ additions seldom wait
  const int64_t nqt = (N - lo + GB - 1) / GB;
  for (int64_t it = 0; it < nqt; ++it) {
    const int64_t q0 = lo + (det ? nqt - 1 - it : it) * GB;
    __syncthreads();
    int live_row = 0;
    if (tid < GB) {
      const int64_t row = q0 + tid;
      RowCoef c{0.f, 0.f, 0.f, 0.f};
      int arg = -1;
      float pcmp = __int_as_float(0x7fc00000);
      if (row < N) {
        const int64_t rr = bh * rec_rows(N) + row;
        c = load_row_coef(a.coefP, a.tiev, rr, a.scale);
        arg = a.argv[rr];
        pcmp = a.pcmpv[rr];
      }
      sC[tid] = make_float4(0.f, c.c1, c.c10, c.D);  // -, gate/z, 10*scale*gate/z, D
      sTie[tid] = c.tie;
      sArg[tid] = arg;
      sPc[tid] = pcmp;
      live_row = arg >= 0;
    }
    if (!__syncthreads_or(live_row)) {  // every query row of the block is silent
      if (det) {
        det_turn_wait(q0);
        det_turn_pass(q0);
      }
      continue;
    }
    load_tile<T, DP>(sQ, Q, a.sq[2], a.sq[3], q0, N, D);
    __syncthreads();
    float u[4][4];
    tile_dot<DP>(u, sQ, sK, rg, cg);
    int live = 0;
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int64_t row = q0 + rg + 16 * ii;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int64_t col = k0 + cg + 16 * jj;
        const bool valid = row < N && col < N && (!a.causal || col <= row);
        const float s = u[ii][jj] * a.scale - tau;
        u[ii][jj] = (valid && s > 0.f) ? s : 0.f;
        live |= u[ii][jj] > 0.f;
      }
    }
    if (!__syncthreads_or(live)) {  // silent tile
      if (det) {
        det_turn_wait(q0);
        det_turn_pass(q0);
      }
      continue;
    }
    load_tile<T, DP>(sdO, dO, a.sdo[2], a.sdo[3], q0, N, D);
    __syncthreads();
    float dp[4][4];
    tile_dot<DP>(dp, sdO, sV, rg, cg);
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int r = rg + 16 * ii;
      const float4 c = sC[r];  // -, gate/z, 10*scale*gate/z, D
      const float tie = sTie[r], pcmp = sPc[r];
      const int arg = sArg[r];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float x = u[ii][jj];
        const float x2 = x * x, x4 = x2 * x2, x8 = x4 * x4, x9 = x8 * x;
        const float w = x8 * x2 * c.y;
        float ds = 0.f;  // du * scale
        if (x > 0.f) {
          ds = c.z * x9 * (dp[ii][jj] - c.w);
          if ((int)(k0 + cg + 16 * jj) == arg || x == pcmp) ds += tie;
        }
        dtau += ds;
        sW[r * LDP + cg + 16 * jj] = w;
        sdS[r * LDP + cg + 16 * jj] = ds;
      }
    }
    __syncthreads();
    // dV[key][e] += sum_q W[q][key] dO[q][e];  dK[key][e] += sum_q dS[q][key] Q[q][e]
#pragma unroll 4
    for (int qq = 0; qq < GB; ++qq) {
      float w[4], s[4], d[NJ], qv[NJ];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        w[ii] = sW[qq * LDP + rg + 16 * ii];
        s[ii] = sdS[qq * LDP + rg + 16 * ii];
      }
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) {
        d[jj] = sdO[qq * LD + cg + 16 * jj];
        qv[jj] = sQ[qq * LD + cg + 16 * jj];
      }
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          dv[ii][jj] = fmaf(w[ii], d[jj], dv[ii][jj]);
          dk[ii][jj] = fmaf(s[ii], qv[jj], dk[ii][jj]);
        }
    }
    // dQ[q][e] += sum_key dS[q][key] K[key][e]
    float dq[4][NJ];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) dq[ii][jj] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < GB; ++kk) {
      float s[4], kv[NJ];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) s[ii] = sdS[(rg + 16 * ii) * LDP + kk];
#pragma unroll
      for (int jj = 0; jj < NJ; ++jj) kv[jj] = sK[kk * LD + cg + 16 * jj];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) dq[ii][jj] = fmaf(s[ii], kv[jj], dq[ii][jj]);
    }
    if (det) {
      // this block's turn: every load of its dQ elements issued before the first add
      det_turn_wait(q0);
      float old[4][NJ];
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          const int64_t row = q0 + rg + 16 * ii;
          const int e = cg + 16 * jj;
          old[ii][jj] = (row < N && e < D) ? __ldcg(dQa + row * a.acc_d + e) : 0.f;
        }
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          const int64_t row = q0 + rg + 16 * ii;
          const int e = cg + 16 * jj;
          if (row < N && e < D) __stcg(dQa + row * a.acc_d + e, old[ii][jj] + dq[ii][jj]);
        }
      det_turn_pass(q0);
    } else {
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int64_t row = q0 + rg + 16 * ii;
        if (row >= N) continue;
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          const int e = cg + 16 * jj;
          if (e < D) atomicAdd(dQa + row * a.acc_d + e, dq[ii][jj]);
        }
      }
    }
  }
  T* dK = static_cast<T*>(a.dk) + b * a.sdk[0] + h * a.sdk[1];
  T* dV = static_cast<T*>(a.dv) + b * a.sdv[0] + h * a.sdv[1];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int64_t key = k0 + rg + 16 * ii;
    if (key >= N) continue;
#pragma unroll
    for (int jj = 0; jj < NJ; ++jj) {
      const int e = cg + 16 * jj;
      if (e < D) {
        dK[key * a.sdk[2] + e * a.sdk[3]] = from_f32<T>(dk[ii][jj]);
        dV[key * a.sdv[2] + e * a.sdv[3]] = from_f32<T>(dv[ii][jj]);
      }
    }
  }
  __shared__ float red[GTHREADS / 32];
  const float t = block_sum(dtau, red);  // sum of du*scale over this key block
  if (tid == 0) a.dtau_part[bh * gridDim.x + kt] = -t / a.scale;
}

// dtau = fixed-order fp64 sum of the backward's tau partials, by one block of 256
// threads (block (0,0) of the dQ cast, which runs after the backward kernel)
__device__ __forceinline__ void tau_partials_sum(const FlashArgs& a) {
  __shared__ double sm[256];
  double v = 0.0;
  for (int64_t i = threadIdx.x; i < a.n_dtau_part; i += 256) v += (double)a.dtau_part[i];
  sm[threadIdx.x] = v;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) sm[threadIdx.x] += sm[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) a.dtau[0] = (float)sm[0];
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  static_assert(sizeof(T) == 2, "16-bit element type");
  const T l = from_f32<T>(lo), u = from_f32<T>(hi);
  uint16_t bl, bu;
  memcpy(&bl, &l, 2);
  memcpy(&bu, &u, 2);
  return (uint32_t)bl | ((uint32_t)bu << 16);
}

// dQ = dq_scale * dq_acc for head dims 64 / 128 (SH = log2(D / 8)), unit inner
// stride, 16-byte aligned rows: grid (rows * D / 8 / 256, B * H), one 16-byte store
// per thread, no 64-bit divisions.
template <typename T, int SH>
__global__ void __launch_bounds__(256) dq_cast_rows_kernel(FlashArgs a) {
  if (blockIdx.x == 0 && blockIdx.y == 0) tau_partials_sum(a);
  const int bh = blockIdx.y, b = bh / (int)a.H, h = bh - b * (int)a.H;
  const uint32_t li = blockIdx.x * 256u + threadIdx.x;
  const int64_t n = li >> SH;
  if (n >= a.N) return;
  constexpr int D = 8 << SH;
  const int c = (int)(li & ((1u << SH) - 1)) * 8;
  const float4* row4 = reinterpret_cast<const float4*>(a.dq_acc + ((int64_t)bh * a.N + n) * D);
  const int c4 = c >> 2;  // 16-byte chunks c4, c4 + 1 of the row (swizzled: D == 64 only)
  float4 f0 = __ldcs(row4 + (a.acc_swz ? acc_chunk(c4, n) : c4));
  float4 f1 = __ldcs(row4 + (a.acc_swz ? acc_chunk(c4 + 1, n) : c4 + 1));
  const float fs = a.dq_scale;
  uint4 w;
  w.x = pack2<T>(fs * f0.x, fs * f0.y);
  w.y = pack2<T>(fs * f0.z, fs * f0.w);
  w.z = pack2<T>(fs * f1.x, fs * f1.y);
  w.w = pack2<T>(fs * f1.z, fs * f1.w);
  T* dst = static_cast<T*>(a.dq) + b * a.sdq[0] + h * a.sdq[1] + n * a.sdq[2] + c;
  *reinterpret_cast<uint4*>(dst) = w;
}

template <typename T>
__global__ void __launch_bounds__(256) dq_cast_kernel(FlashArgs a) {
  if (blockIdx.x == 0) tau_partials_sum(a);
  T* dq = static_cast<T*>(a.dq);
  const float fs = a.dq_scale;
  const bool vec = (a.D % 8) == 0 && a.sdq[3] == 1 && (a.sdq[2] % 8) == 0 && (a.sdq[1] % 8) == 0 &&
                   (a.sdq[0] % 8) == 0 && (reinterpret_cast<uintptr_t>(a.dq) % 16) == 0;
  if (vec) {  // 8 consecutive head dims per thread: two float4 loads, one or two 16-byte stores
    const int64_t per_row = a.D / 8, total = a.B * a.H * a.N * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t row = i / per_row, c = (i - row * per_row) * 8;
      const int64_t n = row % a.N, bh = row / a.N, b = bh / a.H, h = bh % a.H;
      const float4* row4 = reinterpret_cast<const float4*>(a.dq_acc + row * a.acc_d);
      const int c4 = (int)(c >> 2);
      float4 f0 = row4[a.acc_swz ? acc_chunk(c4, n) : c4], f1 = row4[a.acc_swz ? acc_chunk(c4 + 1, n) : c4 + 1];
      f0.x *= fs; f0.y *= fs; f0.z *= fs; f0.w *= fs;
      f1.x *= fs; f1.y *= fs; f1.z *= fs; f1.w *= fs;
      T* dst = dq + b * a.sdq[0] + h * a.sdq[1] + n * a.sdq[2] + c;
      if constexpr (sizeof(T) == 2) {
        uint4 w;
        T* e = reinterpret_cast<T*>(&w);
        e[0] = from_f32<T>(f0.x); e[1] = from_f32<T>(f0.y); e[2] = from_f32<T>(f0.z); e[3] = from_f32<T>(f0.w);
        e[4] = from_f32<T>(f1.x); e[5] = from_f32<T>(f1.y); e[6] = from_f32<T>(f1.z); e[7] = from_f32<T>(f1.w);
        *reinterpret_cast<uint4*>(dst) = w;
      } else {
        reinterpret_cast<float4*>(dst)[0] = f0;
        reinterpret_cast<float4*>(dst)[1] = f1;
      }
    }
    return;
  }
  const int64_t total = a.B * a.H * a.N * a.D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i % a.D, n = (i / a.D) % a.N, bh = i / (a.D * a.N), b = bh / a.H, h = bh % a.H;
    const int64_t ep = a.acc_swz ? (int64_t)((acc_chunk((int)(e >> 2), n) << 2) | (int)(e & 3)) : e;
    dq[b * a.sdq[0] + h * a.sdq[1] + n * a.sdq[2] + e * a.sdq[3]] = from_f32<T>(fs * a.dq_acc[(bh * a.N + n) * a.acc_d + ep]);
  }
}

static unsigned grid_cap(int64_t items, int per_block) {
  int64_t g = (items + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > 65535LL * 32) g = 65535LL * 32;
  return (unsigned)g;
}

BwdWorkspace bwd_workspace_layout(int64_t B, int64_t H, int64_t N, int64_t D) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  BwdWorkspace w{};
  const size_t rows = (size_t)(B * H * N), recs = (size_t)(B * H * rec_rows(N));
  const size_t ntiles64 = (size_t)(B * H) * (size_t)((N + GB - 1) / GB);
  w.off_dq = 0;
  w.off_coef = up(rows * (size_t)acc_width(D) * sizeof(float));
  // coefP (two floats per row), tiev, argv, pcmpv: recs records each
  w.off_live = w.off_coef + up(recs * (sizeof(float2) + sizeof(float) + sizeof(int32_t) + sizeof(float)));
  w.off_part = w.off_live + up(ntiles64 * sizeof(int32_t));
  w.off_sem = w.off_part + up(ntiles64 * sizeof(float));
  w.total = w.off_sem + up((ntiles64 + 1) * sizeof(int32_t));  // turn counters + work ticket
  return w;
}

template <typename T, int DP>
static int fwd_launch(const FlashArgs& a, cudaStream_t st) {
  constexpr size_t smem = GenSmem<DP>::fwd_bytes;
  auto kern = flash_fwd_generic_kernel<T, DP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return check_launch("flash fwd generic: smem attribute");
  dim3 grid((unsigned)((a.N + GB - 1) / GB), (unsigned)(a.B * a.H));
  kern<<<grid, GTHREADS, smem, st>>>(a);
  return check_launch("flash fwd generic");
}

template <typename T, int DP>
static int bwd_launch(const FlashArgs& a, cudaStream_t st) {
  constexpr size_t smem = GenSmem<DP>::bwd_bytes;
  auto kern = flash_bwd_generic_kernel<T, DP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return check_launch("flash bwd generic: smem attribute");
  dim3 grid((unsigned)((a.N + GB - 1) / GB), (unsigned)(a.B * a.H));
  kern<<<grid, GTHREADS, smem, st>>>(a);
  return check_launch("flash bwd generic");
}

#define PNFT_DISPATCH_DP(D, DPV, ...)                                                    \
  if ((D) <= 16) {                                                                       \
    constexpr int DPV = 16;                                                              \
    __VA_ARGS__;                                                                         \
  } else if ((D) <= 32) {                                                                \
    constexpr int DPV = 32;                                                              \
    __VA_ARGS__;                                                                         \
  } else if ((D) <= 64) {                                                                \
    constexpr int DPV = 64;                                                              \
    __VA_ARGS__;                                                                         \
  } else if ((D) <= 128) {                                                               \
    constexpr int DPV = 128;                                                             \
    __VA_ARGS__;                                                                         \
  } else {                                                                               \
    return fail(PNFT_EUNSUPPORTED, "flash: head dim %lld > 128 is not supported", (long long)(D)); \
  }

int flash_fwd_generic(const FlashArgs& a, cudaStream_t st) {
  PNFT_DISPATCH_DTYPE(a.dtype, T, { PNFT_DISPATCH_DP(a.D, DP, return fwd_launch<T, DP>(a, st)); });
  return PNFT_OK;
}

int flash_bwd_prep(const FlashArgs& a, cudaStream_t st) {
  PNFT_DISPATCH_DTYPE(a.dtype, T, {
    flash_bwd_prep_kernel<T><<<dim3((unsigned)((a.N + 63) / 64), (unsigned)(a.B * a.H)), 256, 0, st>>>(a);
  });
  return check_launch("flash bwd prep");
}

// the dQ cast (and tau sum) in element type T: the row kernel for 16-bit types with
// head dim 64 / 128 and 16-byte aligned rows, else the grid-stride kernel
template <typename T>
static void dq_cast_launch(const FlashArgs& a, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    const bool rows = (a.D == 64 || a.D == 128) && a.sdq[3] == 1 && (a.sdq[2] % 8) == 0 && (a.sdq[1] % 8) == 0 &&
                      (a.sdq[0] % 8) == 0 && (reinterpret_cast<uintptr_t>(a.dq) % 16) == 0 && a.B * a.H <= 65535 &&
                      a.N * (a.D / 8) < ((int64_t)1 << 31);
    if (rows) {
      const dim3 grid((unsigned)((a.N * (a.D / 8) + 255) / 256), (unsigned)(a.B * a.H));
      if (a.D == 64) dq_cast_rows_kernel<T, 3><<<grid, 256, 0, st>>>(a);
      else dq_cast_rows_kernel<T, 4><<<grid, 256, 0, st>>>(a);
      return;
    }
  }
  const int64_t items = a.B * a.H * a.N * (a.D % 8 == 0 ? a.D / 8 : a.D);
  dq_cast_kernel<T><<<grid_cap(items, 256), 256, 0, st>>>(a);
}

int flash_bwd_finish(const FlashArgs& a, cudaStream_t st) {
  PNFT_DISPATCH_DTYPE(a.dtype, T, { dq_cast_launch<T>(a, st); });
  return check_launch("flash bwd dq cast + tau sum");
}

int flash_bwd_generic(const FlashArgs& a0, cudaStream_t st) {
  FlashArgs a = a0;
  a.n_dtau_part = a.B * a.H * ((a.N + GB - 1) / GB);
  int rc = flash_bwd_prep(a, st);
  if (rc) return rc;
  PNFT_DISPATCH_DTYPE(a.dtype, T, {
    PNFT_DISPATCH_DP(a.D, DP, { rc = bwd_launch<T, DP>(a, st); });
  });
  if (rc) return rc;
  return flash_bwd_finish(a, st);
}

}  // namespace pnft
