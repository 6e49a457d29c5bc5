// Kernels of the LM training step around the attention operator (the caller in
// the reference's language-model experiments, experiments/exp4_wikitext2_lm.py):
//
//  * lm_xent: next-token cross-entropy of the LM head, loss AND logit gradient
//    in one pass over the logits (replaces nn.functional.cross_entropy and its
//    autograd backward, exp4_wikitext2_lm.py:714-719). Each row of logits is
//    staged into shared memory by a 1-D bulk copy (cp.async.bulk, a ring of up
//    to three rows per CTA, one persistent CTA per SM), reduced there (max,
//    then one exponential per element, kept in fp16 beside its sum), and
//    overwritten in place in HBM by scale * (softmax - onehot). HBM traffic is
//    one read and one write of the logits, against the eager path's logit
//    copies, log-softmax output and its backward re-reads.
//
//  * (add_)layernorm_fwd / _bwd: nn.LayerNorm of the Pre-LN blocks
//    (exp4_wikitext2_lm.py:183-200), optionally fused with the residual add
//    before it. One warp per row with the row held in registers; the forward
//    writes the normalised row directly in the type of the GEMM that consumes
//    it (bf16 under autocast) and keeps mean and 1/std; the backward gives dx
//    (plus the residual path's gradient, and the branch's gradient in its own
//    type) and per-CTA partial sums of dgamma / dbeta, which a second kernel
//    adds in a fixed order (bitwise reproducible).
//
//  * colsum / gelu_bwd_colsum / gelu_fwd: the MLP's bias gradients as
//    fixed-order column sums, the GELU backward fused with the first of them,
//    and the GELU forward; bf16 GELU and GELU' come from a per-device table over
//    the bf16 bit patterns (pnft_gelu_table) copied into shared memory.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace pnft {
namespace {

using sm100::Abort;
using sm100::smem_u32;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kEBias = 15.f;  // log2 of the scale of the fp16 copy of exp(x - max)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& u, float f[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// =====================================================================================
// cross-entropy of the LM head
// =====================================================================================

constexpr int XT = 512;  // threads of a cross-entropy CTA
constexpr int XW = XT / 32;
constexpr int kXentMaxStages = 3;

struct XentArgs {
  __nv_bfloat16* logits;  // [M, ld] in: logits, out: gradient
  int64_t ld;
  const int64_t* tgt;     // [M]
  int64_t ignore;         // target value that excludes a row
  float* row_loss;        // [M]
  int64_t M, V;
  float scale;            // gradient scale (times *scale_dev when given)
  const float* scale_dev;
  int32_t* status;
  uint32_t row_bytes;     // staged bytes per row (ld * 2)
  int stages;
};

// Block-wide reduction over the XT threads; every thread gets the result. The
// warps' partials are combined in warp order, so the result is reproducible.
template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  v = MAX ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < XW; ++w) r = MAX ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

// 2^x on the MUFU pipe (subnormal results flush to 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One row: src holds the logits (shared memory, or the global row itself), dst
// receives the gradient (the global row). VEC: 16-byte vectors (ld % 8 == 0 and
// 16-byte aligned rows). An ignored row gets loss 0 and gradient 0; a target
// outside [0, V) gets loss NaN, the softmax without the one-hot term, and the
// status word PNFT_DEV_BAD_INDEX.
//
// VEC path, three passes over the row: (A) the maximum M; (B) e = 2^((x-M)log2e
// + 15) once per element, summed in fp32 and written back over the row as fp16
// (the staged copy in shared memory, or the global row that receives the
// gradient); (C) gradient = e * scale/sum, packed to bf16. One exponential per
// element. The 2^15 bias keeps e in [2^-14, 2^15], fp16's normal range, for
// every element within 2^-29 of the row's largest probability (smaller ones
// contribute below 2^-29 / sum to the gradient), so the fp16 copy adds at most
// 2^-12 relative to the single bf16 rounding of the gradient; the factor
// cancels in e/sum and is taken out of the loss exactly. Columns in
// [V, 8*ceil(V/8)) are read as -inf: they drop out of M and give e = 0.
template <bool VEC>
__device__ __forceinline__ void xent_row(const __nv_bfloat16* src, __nv_bfloat16* dst, const XentArgs& a,
                                         int64_t t, float scale, float* loss_out, float* red_m, float* red_s) {
  const int tid = threadIdx.x;
  if (t == a.ignore) {
    if (VEC) {
      for (int64_t v = tid; v < a.ld / 8; v += XT) reinterpret_cast<uint4*>(dst)[v] = make_uint4(0, 0, 0, 0);
    } else {
      for (int64_t c = tid; c < a.ld; c += XT) dst[c] = __float2bfloat16_rn(0.f);
    }
    if (tid == 0) *loss_out = 0.f;
    return;
  }
  const bool bad = t < 0 || t >= a.V;
  // the target's logit is read before the first barrier below: after it, the row
  // is overwritten (by e, and on the global path by the gradient)
  float xt = 0.f;
  if (tid == 0 && !bad) xt = __bfloat162float(src[t]);

  if constexpr (VEC) {
    const uint32_t V = (uint32_t)a.V, nfull = V / 8, nv = (V + 7) / 8, nld = (uint32_t)(a.ld / 8);
    const uint4* sv = reinterpret_cast<const uint4*>(src);
    uint4* ev = const_cast<uint4*>(sv);  // e (fp16) overwrites the row it came from
    // (A) maximum
    float m = -INFINITY;
#pragma unroll 2
    for (uint32_t v = tid; v < nv; v += XT) {
      float f[8];
      unpack8(sv[v], f);
      if (v >= nfull) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (v * 8 + k >= V) f[k] = -INFINITY;
      }
      m = fmaxf(m, fmaxf(fmaxf(fmaxf(f[0], f[1]), fmaxf(f[2], f[3])), fmaxf(fmaxf(f[4], f[5]), fmaxf(f[6], f[7]))));
    }
    const float M = block_reduce<true>(m, red_m);
    // (B) e and its sum
    const float2 l2e = make_float2(kLog2e, kLog2e), nm = make_float2(kEBias - M * kLog2e, kEBias - M * kLog2e);
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll 2
    for (uint32_t v = tid; v < nv; v += XT) {
      float f[8];
      unpack8(sv[v], f);
      if (v >= nfull) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (v * 8 + k >= V) f[k] = -INFINITY;
      }
      uint32_t h[4];
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        const float2 x = __ffma2_rn(make_float2(f[k], f[k + 1]), l2e, nm);
        const float2 e = make_float2(ex2(x.x), ex2(x.y));
        s2 = __fadd2_rn(s2, e);
        const __half2 hh = __floats2half2_rn(e.x, e.y);
        h[k / 2] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      ev[v] = make_uint4(h[0], h[1], h[2], h[3]);
    }
    const float S = block_reduce<false>(s2.x + s2.y, red_s);
    if (tid == 0) {
      if (bad) {
        *loss_out = NAN;
        sm100::report_status(a.status, PNFT_DEV_BAD_INDEX);
      } else {
        *loss_out = M + (logf(S) - kEBias * kLn2) - xt;  // logsumexp(row) - row[t]
      }
    }
    // (C) gradient = scale * softmax - scale * onehot; padding columns get 0
    const float inv = scale / S;
    const float2 inv2 = make_float2(inv, inv);
    const uint32_t tcol = bad ? 0xffffffffu : (uint32_t)t;
    uint4* dv = reinterpret_cast<uint4*>(dst);
#pragma unroll 2
    for (uint32_t v = tid; v < nld; v += XT) {
      uint4 out = make_uint4(0, 0, 0, 0);
      if (v < nv) {
        const uint4 u = ev[v];
        const uint32_t hw[4] = {u.x, u.y, u.z, u.w};
        float g[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&hw[k]));
          const float2 q = __fmul2_rn(e, inv2);
          g[2 * k] = q.x;
          g[2 * k + 1] = q.y;
        }
        const uint32_t d = tcol - v * 8;
        if (d < 8u) {  // this vector holds the target column
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (d == (uint32_t)k) g[k] -= scale;
        }
        out = make_uint4(sm100::pack_bf16x2(g[0], g[1]), sm100::pack_bf16x2(g[2], g[3]),
                         sm100::pack_bf16x2(g[4], g[5]), sm100::pack_bf16x2(g[6], g[7]));
      }
      dv[v] = out;
    }
  } else {
    const int64_t V = a.V, ld = a.ld;
    float m = -INFINITY;
    for (int64_t c = tid; c < V; c += XT) m = fmaxf(m, __bfloat162float(src[c]));
    m = block_reduce<true>(m, red_m);
    const float m2 = m * kLog2e;
    float s = 0.f;
    for (int64_t c = tid; c < V; c += XT) s += exp2f(fmaf(__bfloat162float(src[c]), kLog2e, -m2));
    s = block_reduce<false>(s, red_s);
    if (tid == 0) {
      if (bad) {
        *loss_out = NAN;
        sm100::report_status(a.status, PNFT_DEV_BAD_INDEX);
      } else {
        *loss_out = m + logf(s) - xt;
      }
    }
    const float inv = scale / s;
    for (int64_t c = tid; c < ld; c += XT) {
      float g = 0.f;
      if (c < V) {
        g = exp2f(fmaf(__bfloat162float(src[c]), kLog2e, -m2)) * inv;
        if (c == t) g -= scale;
      }
      dst[c] = __float2bfloat16_rn(g);
    }
  }
}

// Persistent: CTA b takes rows b, b + grid, b + 2*grid, ... and keeps up to
// `stages` of them in flight as bulk copies while it works on the oldest.
__global__ void __launch_bounds__(XT, 1) xent_staged_kernel(XentArgs a) {
  extern __shared__ __align__(128) uint8_t xsm[];
  __shared__ __align__(8) uint64_t full[kXentMaxStages];
  __shared__ float red_m[XW], red_s[XW];
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  const int64_t first = blockIdx.x, step = gridDim.x;
  if (first >= a.M) return;
  const int64_t nrow = (a.M - first + step - 1) / step;
  const int S = a.stages;
  const float scale = a.scale * (a.scale_dev ? *a.scale_dev : 1.f);
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) sm100::mbar_init(smem_u32(&full[s]), 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  const uint32_t base = smem_u32(xsm);
  int64_t issued = 0;  // rows whose copy has been issued (thread 0's count)
  auto issue = [&](int64_t i) {
    const int s = (int)(i % S);
    const uint32_t bar = smem_u32(&full[s]);
    sm100::mbar_arrive_expect_tx(bar, a.row_bytes);
    sm100::bulk_load(base + (uint32_t)s * a.row_bytes, a.logits + (first + i * step) * a.ld, a.row_bytes, bar);
  };
  if (tid == 0)
    for (; issued < std::min<int64_t>(S, nrow); ++issued) issue(issued);
  const Abort ab{&abort_flag, a.status};
  int64_t i = 0;
  for (; i < nrow; ++i) {
    const int s = (int)(i % S);
    const int64_t row = first + i * step;
    const int64_t t = a.tgt[row];
    const bool ok = sm100::warp_wait(smem_u32(&full[s]), (uint32_t)((i / S) & 1), ab);
    if (__syncthreads_or(!ok)) break;
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(xsm + (size_t)s * a.row_bytes);  // e is written here too
    xent_row<true>(src, a.logits + row * a.ld, a, t, scale, a.row_loss + row, red_m, red_s);
    // the row's generic-proxy writes (e) are ordered before the bulk copy that
    // refills the stage, and the stage is fully read before it is refilled
    sm100::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0 && issued < nrow) issue(issued++);
  }
  if (i < nrow && tid == 0) {
    // a wait gave up: let this CTA's outstanding copies land before it exits
    for (int64_t j = i; j < issued; ++j) sm100::drain_wait(smem_u32(&full[j % S]), (uint32_t)((j / S) & 1));
  }
}

// Rows too long to stage (or not 16-byte aligned): one CTA per row straight
// from global memory (the row's re-reads come from L2).
template <bool VEC>
__global__ void __launch_bounds__(XT) xent_global_kernel(XentArgs a) {
  __shared__ float red_m[XW], red_s[XW];
  const float scale = a.scale * (a.scale_dev ? *a.scale_dev : 1.f);
  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    __nv_bfloat16* r = a.logits + row * a.ld;
    xent_row<VEC>(r, r, a, a.tgt[row], scale, a.row_loss + row, red_m, red_s);
    __syncthreads();
  }
}

int device_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// =====================================================================================
// LayerNorm, optionally fused with the residual add before it
// =====================================================================================

constexpr int LT = 256;  // threads of a LayerNorm / column-sum CTA
constexpr int LWARPS = LT / 32;
constexpr int kLnMaxBlocks = 1024;  // bound on the partial-sum blocks (workspace size)

// s = x + r (when r is given; s is written in x's type), y = LN(s) (LN(x) without r).
struct LnFwdArgs {
  const void* x;
  int64_t sx;
  const void* r;  // residual branch (may be null), type r_dt
  int64_t sr;
  int r_dt;
  void* s;        // x + r (x's type); null without r
  int64_t ss;
  const float* gamma;
  const float* beta;
  float eps;
  void* y;
  int64_t sy;
  float* mean;
  float* rstd;
  int64_t M;
  int C;
};

// dx = gs + LN'(dy) in x's type (gs: gradient already flowing into s, may be
// null); dr (may be null) = the same values in dr_dt (the residual branch's
// gradient); x here is the LN input (s of the forward).
struct LnBwdArgs {
  const void* dy;
  int64_t sdy;
  const void* gs;
  int64_t sgs;
  const void* x;
  int64_t sx;
  const float* gamma;
  const float* mean;
  const float* rstd;
  void* dx;
  int64_t sdx;
  void* dr;
  int64_t sdr;
  int dr_dt;
  float* part;  // [2][C][nblk] partial dgamma / dbeta (column-major in the blocks), or null
  int64_t M;
  int C;
};

__device__ __forceinline__ void load4(const float* p, float f[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float f[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  f[0] = __uint_as_float(v.x << 16), f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16), f[3] = __uint_as_float(v.y & 0xffff0000u);
}
__device__ __forceinline__ void store4(float* p, const float f[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float f[4]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(sm100::pack_bf16x2(f[0], f[1]), sm100::pack_bf16x2(f[2], f[3]));
}
// runtime-typed variants (f32 / bf16), the type uniform over the launch
__device__ __forceinline__ void load4(const void* p, int64_t off, int dt, float f[4]) {
  if (dt == PNFT_DTYPE_BF16) load4(static_cast<const __nv_bfloat16*>(p) + off, f);
  else load4(static_cast<const float*>(p) + off, f);
}
__device__ __forceinline__ void store4(void* p, int64_t off, int dt, const float f[4]) {
  if (dt == PNFT_DTYPE_BF16) store4(static_cast<__nv_bfloat16*>(p) + off, f);
  else store4(static_cast<float*>(p) + off, f);
}
__device__ __forceinline__ float load1(const void* p, int64_t off, int dt) {
  return dt == PNFT_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[off])
                               : static_cast<const float*>(p)[off];
}
__device__ __forceinline__ void store1(void* p, int64_t off, int dt, float v) {
  if (dt == PNFT_DTYPE_BF16) static_cast<__nv_bfloat16*>(p)[off] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[off] = v;
}

// VPL > 0: lane l owns columns 4*(32k + l) .. +3 for k < VPL (C <= 128*VPL,
// C % 4 == 0, vector-aligned rows); the row lives in registers. VPL == 0: any
// C and strides, scalar passes over the row.
template <int VPL, typename TX, typename TY>
__global__ void __launch_bounds__(LT) ln_fwd_kernel(LnFwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarp = (int64_t)gridDim.x * LWARPS;
  const int C = a.C;
  const float invC = 1.f / (float)C;
  const TX* __restrict__ x = static_cast<const TX*>(a.x);
  TY* __restrict__ y = static_cast<TY*>(a.y);
  TX* __restrict__ sum = static_cast<TX*>(a.s);
  if constexpr (VPL > 0) {
    float g[VPL][4], b[VPL][4];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c = 4 * (32 * k + lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[k][j] = (a.gamma && c < C) ? a.gamma[c + j] : 1.f;
        b[k][j] = (a.beta && c < C) ? a.beta[c + j] : 0.f;
      }
    }
    for (int64_t row = (int64_t)blockIdx.x * LWARPS + (threadIdx.x >> 5); row < a.M; row += nwarp) {
      float v[VPL][4];
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
          load4(x + row * a.sx + c, v[k]);
          if (a.r) {
            float rr[4];
            load4(a.r, row * a.sr + c, a.r_dt, rr);
#pragma unroll
            for (int j = 0; j < 4; ++j) v[k][j] = (float)from_f32<TX>(v[k][j] + rr[j]);  // s in x's type
            store4(sum + row * a.ss + c, v[k]);
          }
          s += (v[k][0] + v[k][1]) + (v[k][2] + v[k][3]);
        } else {
          v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.f;
        }
      }
      const float mu = warp_sum(s) * invC;
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float d = v[k][j] - mu;
            q = fmaf(d, d, q);
          }
        }
      }
      const float r = rsqrtf(warp_sum(q) * invC + a.eps);
      TY* yr = y + row * a.sy;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
          float o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = fmaf((v[k][j] - mu) * r, g[k][j], b[k][j]);
          store4(yr + c, o);
        }
      }
      if (lane == 0) {
        a.mean[row] = mu;
        a.rstd[row] = r;
      }
    }
  } else {
    for (int64_t row = (int64_t)blockIdx.x * LWARPS + (threadIdx.x >> 5); row < a.M; row += nwarp) {
      // the LN input: x, or s = x + r written first (and re-read from there)
      const TX* in = x + row * a.sx;
      if (a.r) {
        TX* sr = sum + row * a.ss;
        for (int c = lane; c < C; c += 32) sr[c] = from_f32<TX>(to_f32(in[c]) + load1(a.r, row * a.sr + c, a.r_dt));
        __syncwarp();
        in = sr;
      }
      float s = 0.f;
      for (int c = lane; c < C; c += 32) s += to_f32(in[c]);
      const float mu = warp_sum(s) * invC;
      float q = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float d = to_f32(in[c]) - mu;
        q = fmaf(d, d, q);
      }
      const float r = rsqrtf(warp_sum(q) * invC + a.eps);
      TY* yr = y + row * a.sy;
      for (int c = lane; c < C; c += 32) {
        const float gg = a.gamma ? a.gamma[c] : 1.f, bb = a.beta ? a.beta[c] : 0.f;
        yr[c] = from_f32<TY>(fmaf((to_f32(in[c]) - mu) * r, gg, bb));
      }
      if (lane == 0) {
        a.mean[row] = mu;
        a.rstd[row] = r;
      }
    }
  }
}

// dx = gs + rstd * (dy*g - mean(dy*g) - xhat * mean(dy*g*xhat)); per-CTA
// partial sums of dgamma = sum dy*xhat and dbeta = sum dy over this CTA's rows
// (vector path only; the scalar path leaves them to ln_bwd_params_kernel).
template <int VPL, typename TDY, typename TX>
__global__ void __launch_bounds__(LT, 2) ln_bwd_kernel(LnBwdArgs a) {
  extern __shared__ float lsm[];  // [LWARPS][C] (vector path with partials)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nwarp = (int64_t)gridDim.x * LWARPS;
  const int C = a.C;
  const float invC = 1.f / (float)C;
  const TDY* __restrict__ dy = static_cast<const TDY*>(a.dy);
  const TX* __restrict__ x = static_cast<const TX*>(a.x);
  const TX* __restrict__ gs = static_cast<const TX*>(a.gs);
  TX* __restrict__ dx = static_cast<TX*>(a.dx);
  if constexpr (VPL > 0) {
    float g[VPL][4], dg[VPL][4], db[VPL][4];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int c = 4 * (32 * k + lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g[k][j] = (a.gamma && c < C) ? a.gamma[c + j] : 1.f;
        dg[k][j] = db[k][j] = 0.f;
      }
    }
    // rows up to 256 columns are software-pipelined: the next row's loads are
    // issued before this row's reductions, so each warp keeps two rows of loads
    // in flight (wider rows would need more registers than two CTAs per SM allow)
    constexpr bool kPipe = VPL <= 2;
    float cgy[VPL][4], cx[VPL][4], cgs[VPL][4], cmu = 0.f, cr = 0.f;
    auto load_row = [&](int64_t row, float (&gy_)[VPL][4], float (&x_)[VPL][4], float (&gs_)[VPL][4], float& mu_,
                        float& r_) {
      mu_ = a.mean[row];
      r_ = a.rstd[row];
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
          load4(dy + row * a.sdy + c, gy_[k]);
          load4(x + row * a.sx + c, x_[k]);
          if (gs) load4(gs + row * a.sgs + c, gs_[k]);
        }
      }
    };
    int64_t row = (int64_t)blockIdx.x * LWARPS + warp;
    if (kPipe && row < a.M) load_row(row, cgy, cx, cgs, cmu, cr);
    for (; row < a.M; row += nwarp) {
      float ngy[VPL][4], nx[VPL][4], ngs[VPL][4], nmu = 0.f, nr = 0.f;
      if constexpr (kPipe) {
        if (row + nwarp < a.M) load_row(row + nwarp, ngy, nx, ngs, nmu, nr);
      } else {
        load_row(row, cgy, cx, cgs, cmu, cr);
      }
      const float mu = cmu, r = cr;
      float xh[VPL][4];
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            xh[k][j] = (cx[k][j] - mu) * r;
            const float ag = cgy[k][j] * g[k][j];
            s1 += ag;
            s2 = fmaf(ag, xh[k][j], s2);
            dg[k][j] = fmaf(cgy[k][j], xh[k][j], dg[k][j]);
            db[k][j] += cgy[k][j];
          }
        }
      }
      s1 = warp_sum(s1) * invC;
      s2 = warp_sum(s2) * invC;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C) {
          float o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[j] = r * (cgy[k][j] * g[k][j] - s1 - xh[k][j] * s2);
            if (gs) o[j] += cgs[k][j];
          }
          if (dx) store4(dx + row * a.sdx + c, o);
          if (a.dr) store4(a.dr, row * a.sdr + c, a.dr_dt, o);
        }
      }
      if constexpr (kPipe) {
#pragma unroll
        for (int k = 0; k < VPL; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) cgy[k][j] = ngy[k][j], cx[k][j] = nx[k][j], cgs[k][j] = ngs[k][j];
        cmu = nmu, cr = nr;
      }
    }
    if (!a.part) return;
    // this CTA's partial dgamma, then dbeta: warps' sums added in warp order
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int c = 4 * (32 * k + lane);
        if (c < C)
#pragma unroll
          for (int j = 0; j < 4; ++j) lsm[warp * C + c + j] = pass == 0 ? dg[k][j] : db[k][j];
      }
      __syncthreads();
      for (int c = threadIdx.x; c < C; c += LT) {
        float acc = lsm[c];
#pragma unroll
        for (int w = 1; w < LWARPS; ++w) acc += lsm[w * C + c];
        a.part[((int64_t)pass * C + c) * gridDim.x + blockIdx.x] = acc;
      }
      __syncthreads();
    }
  } else {
    for (int64_t row = (int64_t)blockIdx.x * LWARPS + warp; row < a.M; row += nwarp) {
      const float mu = a.mean[row], r = a.rstd[row];
      const TDY* dyr = dy + row * a.sdy;
      const TX* xr = x + row * a.sx;
      float s1 = 0.f, s2 = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float ag = to_f32(dyr[c]) * (a.gamma ? a.gamma[c] : 1.f);
        s1 += ag;
        s2 = fmaf(ag, (to_f32(xr[c]) - mu) * r, s2);
      }
      s1 = warp_sum(s1) * invC;
      s2 = warp_sum(s2) * invC;
      for (int c = lane; c < C; c += 32) {
        const float ag = to_f32(dyr[c]) * (a.gamma ? a.gamma[c] : 1.f);
        float o = r * (ag - s1 - (to_f32(xr[c]) - mu) * r * s2);
        if (gs) o += to_f32(gs[row * a.sgs + c]);
        if (dx) dx[row * a.sdx + c] = from_f32<TX>(o);
        if (a.dr) store1(a.dr, row * a.sdr + c, a.dr_dt, o);
      }
    }
  }
}

// Scalar-path partial sums: CTA b sums dgamma / dbeta over its contiguous
// block of rows, one thread per column (coalesced across the CTA).
template <typename TDY, typename TX>
__global__ void __launch_bounds__(LT) ln_bwd_params_kernel(LnBwdArgs a, int64_t rows_per_blk) {
  const TDY* dy = static_cast<const TDY*>(a.dy);
  const TX* x = static_cast<const TX*>(a.x);
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_blk, r1 = std::min<int64_t>(a.M, r0 + rows_per_blk);
  for (int c = threadIdx.x; c < a.C; c += LT) {
    float sg = 0.f, sb = 0.f;
    for (int64_t row = r0; row < r1; ++row) {
      const float d = to_f32(dy[row * a.sdy + c]);
      sg = fmaf(d, (to_f32(x[row * a.sx + c]) - a.mean[row]) * a.rstd[row], sg);
      sb += d;
    }
    a.part[(int64_t)c * gridDim.x + blockIdx.x] = sg;
    a.part[((int64_t)a.C + c) * gridDim.x + blockIdx.x] = sb;
  }
}

// out[r] = sum over blocks b of part[r][b] for the R = K*C rows of partials
// (row r < C goes to out0[r], row C + r to out1[r]); one warp per row: lane l
// adds blocks l, l+32, ... in order (coalesced), then a fixed butterfly adds the
// lanes. The order is fixed for a given nblk.
__global__ void __launch_bounds__(LT) sum_partials_kernel(const float* part, int nblk, int R, int C, float* out0,
                                                          float* out1) {
  const int r = blockIdx.x * LWARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= R) return;
  float* out = r < C ? out0 : out1;
  if (!out) return;
  const float* row = part + (int64_t)r * nblk;
  float acc = 0.f;
#pragma unroll 4
  for (int b = lane; b < nblk; b += 32) acc += row[b];
  acc = warp_sum(acc);
  if (lane == 0) out[r < C ? r : r - C] = acc;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Vector path: C % 4 == 0, C <= 512, and every row of every operand starting on
// a 16-byte boundary (strides % 4, 16-byte bases; null pointers are ignored).
int ln_vpl(int C, std::initializer_list<std::pair<const void*, int64_t>> rows) {
  if (C % 4 != 0 || C > 512) return 0;
  for (const auto& pr : rows)
    if (pr.first && (pr.second % 4 || !aligned16(pr.first))) return 0;
  return (C + 127) / 128;
}

// CTAs of `kern` resident per SM (computed once per kernel; the same on every
// sm_100a device).
template <typename K>
int resident_per_sm(K kern, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, LT, smem) != cudaSuccess || n < 1) n = 1;
  return n;
}

// One wave of resident CTAs (no partial second wave), at most one CTA per `rows_per_cta` rows.
int wave_grid(int64_t M, int64_t rows_per_cta, int per_sm, int cap) {
  return (int)std::max<int64_t>(
      1, std::min<int64_t>({(M + rows_per_cta - 1) / rows_per_cta, (int64_t)per_sm * device_sms(), (int64_t)cap}));
}

template <int VPL, typename TX, typename TY>
void ln_fwd_go(const LnFwdArgs& a, cudaStream_t st) {
  static const int per_sm = resident_per_sm(ln_fwd_kernel<VPL, TX, TY>, 0);
  ln_fwd_kernel<VPL, TX, TY><<<wave_grid(a.M, LWARPS, per_sm, 1 << 20), LT, 0, st>>>(a);
}

template <typename TX, typename TY>
int ln_fwd_launch(const LnFwdArgs& a, int vpl, cudaStream_t st) {
  switch (vpl) {
    case 1: ln_fwd_go<1, TX, TY>(a, st); break;
    case 2: ln_fwd_go<2, TX, TY>(a, st); break;
    case 3: ln_fwd_go<3, TX, TY>(a, st); break;
    case 4: ln_fwd_go<4, TX, TY>(a, st); break;
    default: ln_fwd_go<0, TX, TY>(a, st); break;
  }
  return check_launch("layernorm fwd");
}

// The backward's grid (also its number of partial sums): one wave on this GPU,
// so the parameter gradients' summation order is fixed for a given GPU model.
template <int VPL, typename TDY, typename TX>
int ln_bwd_go(const LnBwdArgs& a, cudaStream_t st) {
  static const int per_sm = resident_per_sm(ln_bwd_kernel<VPL, TDY, TX>, VPL > 0 ? sizeof(float) * LWARPS * 512 : 0);
  const int nblk = wave_grid(a.M, LWARPS, per_sm, kLnMaxBlocks);
  const size_t smem = (VPL > 0 && a.part) ? sizeof(float) * LWARPS * a.C : 0;
  ln_bwd_kernel<VPL, TDY, TX><<<nblk, LT, smem, st>>>(a);
  return nblk;
}

template <typename TDY, typename TX>
int ln_bwd_launch(const LnBwdArgs& a, int vpl, float* dgamma, float* dbeta, cudaStream_t st) {
  int nblk = 1, n = 1;
  switch (vpl) {
    case 1: nblk = ln_bwd_go<1, TDY, TX>(a, st); break;
    case 2: nblk = ln_bwd_go<2, TDY, TX>(a, st); break;
    case 3: nblk = ln_bwd_go<3, TDY, TX>(a, st); break;
    case 4: nblk = ln_bwd_go<4, TDY, TX>(a, st); break;
    default: nblk = ln_bwd_go<0, TDY, TX>(a, st); break;
  }
  if (a.part) {
    if (vpl == 0) {
      ln_bwd_params_kernel<TDY, TX><<<nblk, LT, 0, st>>>(a, (a.M + nblk - 1) / nblk);
      ++n;
    }
    sum_partials_kernel<<<(2 * a.C + LWARPS - 1) / LWARPS, LT, 0, st>>>(a.part, nblk, 2 * a.C, a.C, dgamma, dbeta);
    ++n;
  }
  return check_launch("layernorm bwd", n);
}

bool ln_dtype_ok(int dt) { return dt == PNFT_DTYPE_F32 || dt == PNFT_DTYPE_BF16; }

int ln_fwd_entry(const LnFwdArgs& a, int x_dtype, int y_dtype, cudaStream_t st) {
  const int vpl = ln_vpl(a.C, {{a.x, a.sx}, {a.y, a.sy}, {a.r, a.sr}, {a.s, a.ss}});
  if (x_dtype == PNFT_DTYPE_F32)
    return y_dtype == PNFT_DTYPE_F32 ? ln_fwd_launch<float, float>(a, vpl, st)
                                     : ln_fwd_launch<float, __nv_bfloat16>(a, vpl, st);
  return y_dtype == PNFT_DTYPE_F32 ? ln_fwd_launch<__nv_bfloat16, float>(a, vpl, st)
                                   : ln_fwd_launch<__nv_bfloat16, __nv_bfloat16>(a, vpl, st);
}

int ln_bwd_entry(const LnBwdArgs& a, int dy_dtype, int x_dtype, float* dgamma, float* dbeta, cudaStream_t st) {
  const int vpl = ln_vpl(a.C, {{a.dy, a.sdy}, {a.x, a.sx}, {a.gs, a.sgs}, {a.dx, a.sdx}, {a.dr, a.sdr}});
  if (x_dtype == PNFT_DTYPE_F32)
    return dy_dtype == PNFT_DTYPE_F32 ? ln_bwd_launch<float, float>(a, vpl, dgamma, dbeta, st)
                                      : ln_bwd_launch<__nv_bfloat16, float>(a, vpl, dgamma, dbeta, st);
  return dy_dtype == PNFT_DTYPE_F32 ? ln_bwd_launch<float, __nv_bfloat16>(a, vpl, dgamma, dbeta, st)
                                    : ln_bwd_launch<__nv_bfloat16, __nv_bfloat16>(a, vpl, dgamma, dbeta, st);
}

// =====================================================================================
// Linear-layer bias gradients: column sums, optionally fused with the GELU backward
// =====================================================================================

// exact (erf) GELU and its derivative Phi(a) + a * phi(a)
__device__ __forceinline__ float gelu_exact(float a) {
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  return 0.5f * a * (1.f + erff(a * kInvSqrt2));
}
__device__ __forceinline__ float gelu_grad(float a) {
  constexpr float kInvSqrt2 = 0.70710678118654752f, kInvSqrt2Pi = 0.39894228040143268f;
  return 0.5f * (1.f + erff(a * kInvSqrt2)) + a * kInvSqrt2Pi * expf(-0.5f * a * a);
}

// For bf16 inputs GELU and GELU' depend only on the 16-bit pattern of a. A CTA
// tabulates them (the same fp32 formulas) in shared memory for |a| in
// [2^-16, 16), 2 signs x 20 binades x 128 mantissas, and looks elements up
// there; the rare |a| outside the range take the formula.
constexpr int kGeluE0 = 111;  // biased exponent of 2^-16
constexpr int kGeluNE = 20;   // binades up to 2^4
constexpr int kGeluN = 2 * kGeluNE * 128;

__device__ __forceinline__ float gelu_table_arg(int i) {
  const uint32_t sign = (uint32_t)i / (kGeluNE * 128), rem = (uint32_t)i % (kGeluNE * 128);
  return __uint_as_float(((sign << 15) | ((kGeluE0 + rem / 128) << 7) | (rem % 128)) << 16);
}

// The CTA's shared-memory table: copied from `src` (built once per device by
// pnft_gelu_table) when given, else computed here.
template <bool GRAD>
__device__ __forceinline__ void gelu_table_init(float* tbl, const float* src) {
  if (src) {
    const float4* s4 = reinterpret_cast<const float4*>(src + (GRAD ? kGeluN : 0));
    for (int i = threadIdx.x; i < kGeluN / 4; i += blockDim.x) reinterpret_cast<float4*>(tbl)[i] = __ldg(s4 + i);
  } else {
    for (int i = threadIdx.x; i < kGeluN; i += blockDim.x) {
      const float a = gelu_table_arg(i);
      tbl[i] = GRAD ? gelu_grad(a) : gelu_exact(a);
    }
  }
}

__global__ void gelu_table_kernel(float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < kGeluN) {
    const float a = gelu_table_arg(i);
    out[i] = gelu_exact(a);
    out[kGeluN + i] = gelu_grad(a);
  }
}

// Table index of a bf16 bit pattern: sign-major, then binade, then mantissa, i.e.
// (bits & 0x7FFF) - (kGeluE0 << 7) + sign * kGeluNE * 128 over a contiguous range.
// Outside the table GELU has closed forms to fp32 precision: for |a| >= 16,
// Phi(a) is 1 or 0 and a*phi(a) underflows (GELU = a or -0, GELU' = 1 or 0;
// NaN and -inf give NaN like the erf formula); for |a| < 2^-16, Phi(a) =
// 0.5 + a*phi(0) and phi(a) = phi(0) to within a relative a^2 (GELU =
// 0.5a + phi(0)a^2, GELU' = 0.5 + 2 phi(0) a).
template <bool GRAD>
__device__ __forceinline__ float gelu_lookup(const float* tbl, uint32_t bits16) {
  constexpr float kPhi0 = 0.39894228040143268f;  // 1/sqrt(2 pi)
  const uint32_t mag = bits16 & 0x7FFFu, off = mag - ((uint32_t)kGeluE0 << 7);
  if (off < (uint32_t)(kGeluNE * 128)) return tbl[off + (bits16 >> 15) * (kGeluNE * 128)];
  const float a = __uint_as_float(bits16 << 16);
  if (mag >= (uint32_t)(kGeluE0 + kGeluNE) << 7) return GRAD ? (a >= 0.f ? 1.f : a * 0.f) : (a >= 0.f ? a : a * 0.f);
  return GRAD ? fmaf(a, 2.f * kPhi0, 0.5f) : fmaf(kPhi0 * a, a, 0.5f * a);
}

struct ColArgs {
  const void* g;  // [M, C] rows of the incoming gradient
  int64_t sg;
  const void* a;  // GELU input (null: plain column sum)
  int64_t sa;
  void* da;       // g * gelu'(a) (written when a is given)
  int64_t sda;
  float* part;    // [C][nblk]
  const float* table;  // pnft_gelu_table output, or null
  int64_t M;
  int C;
  int64_t rows_per_blk;
};

// CTA b covers rows [b*rows_per_blk, ...) (contiguous). VW columns per thread
// (VW = 8: 16-byte bf16 vectors; VW = 1: scalar). Threads are laid out as
// `par` row lanes x `jn` column vectors; each accumulates its column vector
// over its row lane's rows, the row lanes are then added in order in shared
// memory: part[c][b] is a fixed-order sum for a given grid.
template <typename T, int VW>
__global__ void __launch_bounds__(LT) colsum_kernel(ColArgs p) {
  __shared__ float red[LT * VW];
  constexpr bool kTable = VW == 8;  // bf16 vectors: GELU' from the table
  __shared__ float gtab[kTable ? kGeluN : 1];
  if (kTable && p.a) {
    gelu_table_init<true>(gtab, p.table);
    __syncthreads();
  }
  // distinct buffers: the next rows' loads may move above this row's stores
  const T* __restrict__ g = static_cast<const T*>(p.g);
  const T* __restrict__ av = static_cast<const T*>(p.a);
  T* __restrict__ da = static_cast<T*>(p.da);
  const int vpr = p.C / VW;                 // column vectors per row
  const int jn = vpr < LT ? vpr : LT;       // vectors processed side by side
  const int par = LT / jn;                  // row lanes
  const int tj = threadIdx.x % jn, trp = threadIdx.x / jn;
  const int64_t r0 = (int64_t)blockIdx.x * p.rows_per_blk, r1 = std::min<int64_t>(p.M, r0 + p.rows_per_blk);
  for (int j0 = 0; j0 < vpr; j0 += jn) {
    const int j = j0 + tj;
    float acc[VW];
#pragma unroll
    for (int k = 0; k < VW; ++k) acc[k] = 0.f;
    if (trp < par && j < vpr) {
#pragma unroll 4
      for (int64_t row = r0 + trp; row < r1; row += par) {
        float f[VW];
        if constexpr (VW == 8) {
          unpack8(*reinterpret_cast<const uint4*>(g + row * p.sg + (int64_t)j * 8), f);
        } else {
          f[0] = to_f32(g[row * p.sg + j]);
        }
        if (av) {
          if constexpr (VW == 8) {
            const uint4 u = *reinterpret_cast<const uint4*>(av + row * p.sa + (int64_t)j * 8);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              o[k] = sm100::pack_bf16x2(f[2 * k] * gelu_lookup<true>(gtab, w[k] & 0xFFFFu),
                                        f[2 * k + 1] * gelu_lookup<true>(gtab, w[k] >> 16));
              // the stored (rounded) values are what gets summed
              f[2 * k] = __uint_as_float(o[k] << 16);
              f[2 * k + 1] = __uint_as_float(o[k] & 0xffff0000u);
            }
            *reinterpret_cast<uint4*>(da + row * p.sda + (int64_t)j * 8) = make_uint4(o[0], o[1], o[2], o[3]);
          } else {
            f[0] = (float)from_f32<T>(f[0] * gelu_grad(to_f32(av[row * p.sa + j])));
            da[row * p.sda + j] = from_f32<T>(f[0]);
          }
        }
#pragma unroll
        for (int k = 0; k < VW; ++k) acc[k] += f[k];
      }
    }
#pragma unroll
    for (int k = 0; k < VW; ++k) red[threadIdx.x * VW + k] = acc[k];
    __syncthreads();
    if (trp == 0 && j < vpr) {
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        float s = red[tj * VW + k];
        for (int q = 1; q < par; ++q) s += red[(q * jn + tj) * VW + k];
        p.part[((int64_t)j * VW + k) * gridDim.x + blockIdx.x] = s;
      }
    }
    __syncthreads();
  }
}

// rows per CTA: at least 16, and about 32K elements per CTA
int64_t col_rows(int64_t C) { return std::max<int64_t>(16, (32768 + C - 1) / C); }
int col_blocks(int64_t M, int64_t C) {
  return (int)std::min<int64_t>((M + col_rows(C) - 1) / col_rows(C), kLnMaxBlocks);
}

template <typename T, int VW>
int colsum_launch(ColArgs p, float* out, cudaStream_t st) {
  static const int per_sm = resident_per_sm(colsum_kernel<T, VW>, 0);
  const int nblk = wave_grid(p.M, col_rows(p.C), per_sm, col_blocks(p.M, p.C));
  p.rows_per_blk = (p.M + nblk - 1) / nblk;
  colsum_kernel<T, VW><<<nblk, LT, 0, st>>>(p);
  sum_partials_kernel<<<(p.C + LWARPS - 1) / LWARPS, LT, 0, st>>>(p.part, nblk, p.C, p.C, out, nullptr);
  return check_launch("column sum", 2);
}

int col_entry(ColArgs p, float* out, int dtype, cudaStream_t st) {
  if (dtype == PNFT_DTYPE_BF16 && p.C % 8 == 0 && p.sg % 8 == 0 && aligned16(p.g) &&
      (!p.a || (p.sa % 8 == 0 && p.sda % 8 == 0 && aligned16(p.a) && aligned16(p.da))))
    return colsum_launch<__nv_bfloat16, 8>(p, out, st);
  if (dtype == PNFT_DTYPE_BF16) return colsum_launch<__nv_bfloat16, 1>(p, out, st);
  return colsum_launch<float, 1>(p, out, st);
}

// y = GELU(a) (exact erf form), rows of C elements with row strides sa / sy.
// bf16 with 16-byte vectors: table lookups; otherwise the formula per element.
template <typename T, bool VEC>
__global__ void __launch_bounds__(LT) gelu_fwd_kernel(const T* __restrict__ a, int64_t sa, T* __restrict__ y, int64_t sy,
                                                     int64_t M, int C, const float* __restrict__ table) {
  __shared__ float gtab[VEC ? kGeluN : 1];
  if constexpr (VEC) {
    gelu_table_init<false>(gtab, table);
    __syncthreads();
    // thread -> fixed column vector j of its rows (no index division in the loop)
    const int vpr = C / 8;
    const int jn = vpr < LT ? vpr : LT, par = LT / jn;
    const int tj = threadIdx.x % jn, trp = threadIdx.x / jn;
    if (trp < par) {
      for (int j = tj; j < vpr; j += jn) {
#pragma unroll 4
        for (int64_t row = (int64_t)blockIdx.x * par + trp; row < M; row += (int64_t)gridDim.x * par) {
          const uint4 u = *reinterpret_cast<const uint4*>(a + row * sa + (int64_t)j * 8);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            o[k] = sm100::pack_bf16x2(gelu_lookup<false>(gtab, w[k] & 0xFFFFu), gelu_lookup<false>(gtab, w[k] >> 16));
          *reinterpret_cast<uint4*>(y + row * sy + (int64_t)j * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  } else {
    const int64_t n = M * C;
    for (int64_t i = (int64_t)blockIdx.x * LT + threadIdx.x; i < n; i += (int64_t)gridDim.x * LT) {
      const int64_t row = i / C;
      const int c = (int)(i - row * C);
      y[row * sy + c] = from_f32<T>(gelu_exact(to_f32(a[row * sa + c])));
    }
  }
}

template <typename T, bool VEC>
int gelu_fwd_launch(const void* a, int64_t sa, void* y, int64_t sy, int64_t M, int64_t C, const float* table,
                    cudaStream_t st) {
  static const int per_sm = resident_per_sm(gelu_fwd_kernel<T, VEC>, 0);
  // vector path: a CTA covers LT / (C/8) rows per pass (at least one); scalar path: LT elements
  const int64_t rows_per_pass = VEC ? std::max<int64_t>(1, LT / std::max<int64_t>(1, C / 8)) : 1;
  const int64_t items = VEC ? (M + rows_per_pass - 1) / rows_per_pass : (M * C + LT - 1) / LT;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items, (int64_t)per_sm * device_sms()));
  gelu_fwd_kernel<T, VEC><<<grid, LT, 0, st>>>(static_cast<const T*>(a), sa, static_cast<T*>(y), sy, M, (int)C, table);
  return check_launch("gelu fwd");
}

// ---------------------------------------------------------------- bf16 copies of parameters
// Tensor i of the table (rows of {src, dst, n}): dst[e] = bf16(src[e]) for e < n,
// round to nearest even (the cast autocast does per GEMM). blockIdx.y = tensor,
// grid-stride over its elements 8 at a time (two 16-byte loads, one 16-byte
// store) when both pointers are 16-byte aligned.
__global__ void __launch_bounds__(256) cast_bf16_multi_kernel(const int64_t* __restrict__ table) {
  const int64_t* row = table + 3 * blockIdx.y;
  const float* src = reinterpret_cast<const float*>(row[0]);
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(row[1]);
  const int64_t n = row[2];
  const int64_t step = (int64_t)gridDim.x * 256;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    const int64_t n8 = n / 8;
    for (int64_t v = (int64_t)blockIdx.x * 256 + threadIdx.x; v < n8; v += step) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(src) + 2 * v);
      const float4 b = __ldcs(reinterpret_cast<const float4*>(src) + 2 * v + 1);
      uint4 w;
      w.x = sm100::pack_bf16x2(a.x, a.y);
      w.y = sm100::pack_bf16x2(a.z, a.w);
      w.z = sm100::pack_bf16x2(b.x, b.y);
      w.w = sm100::pack_bf16x2(b.z, b.w);
      reinterpret_cast<uint4*>(dst)[v] = w;
    }
    for (int64_t e = 8 * n8 + (int64_t)blockIdx.x * 256 + threadIdx.x; e < n; e += step)
      dst[e] = __float2bfloat16_rn(src[e]);
  } else {
    for (int64_t e = (int64_t)blockIdx.x * 256 + threadIdx.x; e < n; e += step) dst[e] = __float2bfloat16_rn(src[e]);
  }
}

}  // namespace
}  // namespace pnft

using namespace pnft;

extern "C" int pnft_cast_bf16(const int64_t* table, int count, int64_t max_n, void* stream) {
  if (count < 0 || count > 65535 || max_n < 0) return fail(PNFT_EINVAL, "cast bf16: bad count %d / max_n %lld", count, (long long)max_n);
  if (count == 0 || max_n == 0) return PNFT_OK;
  if (!table) return fail(PNFT_EINVAL, "cast bf16: null table");
  // enough blocks for the largest tensor to keep every SM busy; smaller ones exit early
  const int64_t want = (max_n + 8 * 256 - 1) / (8 * 256);
  const int gx = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sms() * 8));
  cast_bf16_multi_kernel<<<dim3((unsigned)gx, (unsigned)count), 256, 0, as_stream(stream)>>>(table);
  return check_launch("cast bf16");
}

extern "C" int pnft_lm_xent(void* logits, int64_t ld, const int64_t* targets, int64_t ignore_index,
                            float* row_loss, int64_t M, int64_t V, float grad_scale, const float* grad_scale_dev,
                            int32_t* status, void* stream) {
  if (M < 0 || V < 0 || ld < V || ld >= (int64_t)1 << 30)
    return fail(PNFT_EINVAL, "lm_xent: need M >= 0 and 2^30 > ld >= V >= 0 (M=%lld V=%lld ld=%lld)", (long long)M,
                (long long)V, (long long)ld);
  if (M == 0) return PNFT_OK;
  if (V == 0) return fail(PNFT_EINVAL, "lm_xent: V must be positive");
  if (!logits || !targets || !row_loss) return fail(PNFT_EINVAL, "lm_xent: null pointer");
  cudaStream_t st = as_stream(stream);
  XentArgs a{static_cast<__nv_bfloat16*>(logits), ld, targets, ignore_index, row_loss, M, V, grad_scale,
             grad_scale_dev, status, 0, 0};
  const bool vec = ld % 8 == 0 && reinterpret_cast<uintptr_t>(logits) % 16 == 0;
  const int64_t row_bytes = ld * 2;
  int dev_smem = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&dev_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int64_t budget = (int64_t)dev_smem - 1024;  // the kernel's static shared memory
  const int stages = vec && row_bytes > 0 ? (int)std::min<int64_t>(kXentMaxStages, budget / row_bytes) : 0;
  if (stages >= 2) {
    a.row_bytes = (uint32_t)row_bytes;
    a.stages = stages;
    const int smem = stages * (int)row_bytes;
    if (cudaFuncSetAttribute(xent_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return check_launch("lm_xent smem attribute", 0);
    const int grid = (int)std::min<int64_t>(M, device_sms());
    xent_staged_kernel<<<grid, XT, smem, st>>>(a);
  } else {
    const int grid = (int)std::min<int64_t>(M, (int64_t)device_sms() * 4);
    if (vec)
      xent_global_kernel<true><<<grid, XT, 0, st>>>(a);
    else
      xent_global_kernel<false><<<grid, XT, 0, st>>>(a);
  }
  return check_launch("lm_xent");
}

static int ln_shape_check(const char* what, int64_t M, int64_t C, int dt_a, int dt_b) {
  if (M < 0 || C <= 0 || C > (1 << 24))
    return fail(PNFT_EINVAL, "%s: bad shape M=%lld C=%lld", what, (long long)M, (long long)C);
  if (!ln_dtype_ok(dt_a) || !ln_dtype_ok(dt_b)) return fail(PNFT_EUNSUPPORTED, "%s: float32 or bfloat16 expected", what);
  return PNFT_OK;
}

extern "C" int pnft_add_layernorm_fwd(const void* x, int64_t sx, const void* r, int64_t sr, int r_dtype, void* s,
                                      int64_t ss, const float* gamma, const float* beta, float eps, void* y,
                                      int64_t sy, float* mean, float* rstd, int64_t M, int64_t C, int x_dtype,
                                      int y_dtype, void* stream) {
  if (int rc = ln_shape_check("layernorm fwd", M, C, x_dtype, y_dtype)) return rc;
  if (r && !ln_dtype_ok(r_dtype)) return fail(PNFT_EUNSUPPORTED, "layernorm fwd: residual must be float32 or bfloat16");
  if (M == 0) return PNFT_OK;
  if (!x || !y || !mean || !rstd || (r && !s)) return fail(PNFT_EINVAL, "layernorm fwd: null pointer");
  if (sx < C || sy < C || (r && (sr < C || ss < C))) return fail(PNFT_EINVAL, "layernorm fwd: row strides must be >= C");
  LnFwdArgs a{x, sx, r, sr, r_dtype, r ? s : nullptr, ss, gamma, beta, eps, y, sy, mean, rstd, M, (int)C};
  return ln_fwd_entry(a, x_dtype, y_dtype, as_stream(stream));
}

extern "C" int pnft_layernorm_fwd(const void* x, int64_t sx, const float* gamma, const float* beta, float eps, void* y,
                                  int64_t sy, float* mean, float* rstd, int64_t M, int64_t C, int x_dtype,
                                  int y_dtype, void* stream) {
  return pnft_add_layernorm_fwd(x, sx, nullptr, 0, 0, nullptr, 0, gamma, beta, eps, y, sy, mean, rstd, M, C, x_dtype,
                                y_dtype, stream);
}

extern "C" size_t pnft_layernorm_bwd_workspace_size(int64_t M, int64_t C) {
  if (M <= 0 || C <= 0) return 0;
  return sizeof(float) * 2 * (size_t)C * (size_t)std::min<int64_t>((M + LWARPS - 1) / LWARPS, kLnMaxBlocks);
}

extern "C" int pnft_add_layernorm_bwd(const void* dy, int64_t sdy, const void* gs, int64_t sgs, const void* x,
                                      int64_t sx, const float* gamma, const float* mean, const float* rstd, void* dx,
                                      int64_t sdx, void* dr, int64_t sdr, int dr_dtype, float* dgamma, float* dbeta,
                                      void* workspace, size_t workspace_bytes, int64_t M, int64_t C, int dy_dtype,
                                      int x_dtype, void* stream) {
  if (int rc = ln_shape_check("layernorm bwd", M, C, dy_dtype, x_dtype)) return rc;
  if (dr && !ln_dtype_ok(dr_dtype)) return fail(PNFT_EUNSUPPORTED, "layernorm bwd: dr must be float32 or bfloat16");
  cudaStream_t st = as_stream(stream);
  const bool params = dgamma || dbeta;
  if (M == 0) {
    if (dgamma && cudaMemsetAsync(dgamma, 0, sizeof(float) * C, st) != cudaSuccess) return check_launch("layernorm bwd memset", 0);
    if (dbeta && cudaMemsetAsync(dbeta, 0, sizeof(float) * C, st) != cudaSuccess) return check_launch("layernorm bwd memset", 0);
    return PNFT_OK;
  }
  if (!dy || !x || !mean || !rstd || (!dx && !dr)) return fail(PNFT_EINVAL, "layernorm bwd: null pointer");
  if (sdy < C || sx < C || (dx && sdx < C) || (gs && sgs < C) || (dr && sdr < C))
    return fail(PNFT_EINVAL, "layernorm bwd: row strides must be >= C");
  if (params) {
    const size_t need = pnft_layernorm_bwd_workspace_size(M, C);
    if (!workspace || workspace_bytes < need)
      return fail(PNFT_EINVAL, "layernorm bwd: workspace of %zu bytes < required %zu", workspace_bytes, need);
  }
  LnBwdArgs a{dy, sdy, gs, sgs, x, sx, gamma, mean, rstd, dx, sdx, dr, sdr, dr_dtype,
              params ? static_cast<float*>(workspace) : nullptr, M, (int)C};
  return ln_bwd_entry(a, dy_dtype, x_dtype, dgamma, dbeta, st);
}

extern "C" int pnft_layernorm_bwd(const void* dy, int64_t sdy, const void* x, int64_t sx, const float* gamma,
                                  const float* mean, const float* rstd, void* dx, int64_t sdx, float* dgamma,
                                  float* dbeta, void* workspace, size_t workspace_bytes, int64_t M, int64_t C,
                                  int dy_dtype, int x_dtype, void* stream) {
  if (!dx && M > 0) return fail(PNFT_EINVAL, "layernorm bwd: null pointer");
  return pnft_add_layernorm_bwd(dy, sdy, nullptr, 0, x, sx, gamma, mean, rstd, dx, sdx, nullptr, 0, 0, dgamma, dbeta,
                                workspace, workspace_bytes, M, C, dy_dtype, x_dtype, stream);
}

extern "C" size_t pnft_colsum_workspace_size(int64_t M, int64_t C) {
  if (M <= 0 || C <= 0) return 0;
  return sizeof(float) * (size_t)C * (size_t)col_blocks(M, C);
}

static int col_check(const char* what, const void* g, int64_t sg, float* out, void* ws, size_t wsb, int64_t M,
                     int64_t C, int dtype) {
  if (M < 0 || C <= 0 || C > (1 << 24)) return fail(PNFT_EINVAL, "%s: bad shape M=%lld C=%lld", what, (long long)M, (long long)C);
  if (!ln_dtype_ok(dtype)) return fail(PNFT_EUNSUPPORTED, "%s: float32 or bfloat16 expected", what);
  if (!out || (M > 0 && !g)) return fail(PNFT_EINVAL, "%s: null pointer", what);
  if (M > 0 && sg < C) return fail(PNFT_EINVAL, "%s: row stride must be >= C", what);
  const size_t need = pnft_colsum_workspace_size(M, C);
  if (M > 0 && (!ws || wsb < need)) return fail(PNFT_EINVAL, "%s: workspace of %zu bytes < required %zu", what, wsb, need);
  return PNFT_OK;
}

extern "C" int pnft_colsum(const void* g, int64_t sg, float* out, void* workspace, size_t workspace_bytes, int64_t M,
                           int64_t C, int dtype, void* stream) {
  if (int rc = col_check("colsum", g, sg, out, workspace, workspace_bytes, M, C, dtype)) return rc;
  cudaStream_t st = as_stream(stream);
  if (M == 0) return cudaMemsetAsync(out, 0, sizeof(float) * C, st) == cudaSuccess ? PNFT_OK : check_launch("colsum", 0);
  ColArgs p{g, sg, nullptr, 0, nullptr, 0, static_cast<float*>(workspace), nullptr, M, (int)C, 0};
  return col_entry(p, out, dtype, st);
}

extern "C" int pnft_gelu_bwd_colsum(const void* dh, int64_t sdh, const void* a, int64_t sa, void* da, int64_t sda,
                                    float* db, void* workspace, size_t workspace_bytes, int64_t M, int64_t C,
                                    int dtype, const float* table, void* stream) {
  if (int rc = col_check("gelu_bwd_colsum", dh, sdh, db, workspace, workspace_bytes, M, C, dtype)) return rc;
  if (M > 0 && (!a || !da || sa < C || sda < C)) return fail(PNFT_EINVAL, "gelu_bwd_colsum: bad a / da");
  cudaStream_t st = as_stream(stream);
  if (M == 0) return cudaMemsetAsync(db, 0, sizeof(float) * C, st) == cudaSuccess ? PNFT_OK : check_launch("gelu_bwd_colsum", 0);
  if (table && reinterpret_cast<uintptr_t>(table) % 16) return fail(PNFT_EINVAL, "gelu_bwd_colsum: table not 16-byte aligned");
  ColArgs p{dh, sdh, a, sa, da, sda, static_cast<float*>(workspace), table, M, (int)C, 0};
  return col_entry(p, db, dtype, st);
}

extern "C" int pnft_gelu_table(float* table, void* stream) {
  if (!table) return fail(PNFT_EINVAL, "gelu table: null pointer");
  if (reinterpret_cast<uintptr_t>(table) % 16) return fail(PNFT_EINVAL, "gelu table: not 16-byte aligned");
  gelu_table_kernel<<<(kGeluN + 255) / 256, 256, 0, as_stream(stream)>>>(table);
  return check_launch("gelu table");
}

extern "C" int pnft_gelu_fwd(const void* a, int64_t sa, void* y, int64_t sy, int64_t M, int64_t C, int dtype,
                             const float* table, void* stream) {
  if (M < 0 || C <= 0 || C > (1 << 24)) return fail(PNFT_EINVAL, "gelu fwd: bad shape M=%lld C=%lld", (long long)M, (long long)C);
  if (!ln_dtype_ok(dtype)) return fail(PNFT_EUNSUPPORTED, "gelu fwd: float32 or bfloat16 expected");
  if (M == 0) return PNFT_OK;
  if (!a || !y) return fail(PNFT_EINVAL, "gelu fwd: null pointer");
  if (sa < C || sy < C) return fail(PNFT_EINVAL, "gelu fwd: row strides must be >= C");
  cudaStream_t st = as_stream(stream);
  if (dtype == PNFT_DTYPE_BF16) {
    if (C % 8 == 0 && sa % 8 == 0 && sy % 8 == 0 && aligned16(a) && aligned16(y))
      return gelu_fwd_launch<__nv_bfloat16, true>(a, sa, y, sy, M, C, table, st);
    return gelu_fwd_launch<__nv_bfloat16, false>(a, sa, y, sy, M, C, table, st);
  }
  return gelu_fwd_launch<float, false>(a, sa, y, sy, M, C, table, st);
}
