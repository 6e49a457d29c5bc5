// Weight gradient of a Linear layer, dW = dY^T X, for the LM training step
// around the attention operator (the Pre-LN blocks' projections and MLP,
// experiments/exp4_wikitext2_lm.py:183-200): C[M x N] (fp32) = A^T B with A
// [K x M] and B [K x N] bf16 row-major, K the token count (16384 at config 4)
// and M, N the layer's widths (256..1024).
//
// The output has few 128x128 tiles (4..16) and a long reduction, which leaves a
// GEMM library with few CTAs, each looping over all of K. Here the reduction is
// split: CTA (tile, s) accumulates rows [s*kchunk, (s+1)*kchunk) of K in TMEM
// with tcgen05 MMAs (M = 128, N = 256 or 128, both operands MN-major from
// 128-byte-swizzled TMA tiles, a ring of 64-row stages), writes its fp32 partial, and a
// second kernel adds the splits' partials in split order (deterministic).
#include <string.h>

#include <algorithm>

#include "flash.cuh"
#include "sm100_ptx.cuh"

namespace pnft {
namespace {

using namespace sm100;

constexpr int GM = 128;  // output rows (A columns) per CTA: TMEM lanes
constexpr int GK = 64;   // K rows per stage
constexpr int GGROUP = GK * 128;              // one 64-column group of a stage's A or B tile (bytes)
constexpr int A_BYTES = (GM / 64) * GGROUP;   // 16 KB
constexpr int GTHREADS = 192;                 // producer warp, MMA warp, 4 epilogue warps

// GN output columns (B columns) per CTA = TMEM columns of the accumulator. 128
// (6 stages): a 256-wide tile brings fewer bytes per FLOP into the SM but fits
// only 4 stages, and measured slower at config 4's shapes (16.6 against 14.0 µs
// per weight gradient inside the LM step).
template <int GN>
struct GemmCfg {
  static constexpr int B_BYTES = (GN / 64) * GGROUP;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = GN == 256 ? 4 : 6;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static_assert(STAGE_BYTES % 1024 == 0, "128-byte swizzle atoms stay 1024-byte aligned");
};

struct GemmParams {
  CUtensorMap ta;  // A [K rows x M cols]
  CUtensorMap tb;  // B [K rows x N cols]
  float* part;     // [splits][M][N] fp32 (the output itself when there is one split)
  int64_t ldp;     // row stride of part (elements)
  int64_t split_stride;  // elements between splits' partials
  int M, N;
  int64_t K;
  int kchunk;      // K rows per split, a multiple of GK
  int tiles_n;
  int32_t* status;
};

template <int GN>
__global__ void __launch_bounds__(GTHREADS, 1) gemm_at_b_kernel(const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<GN>;
  constexpr int GSTAGES = Cfg::STAGES, STAGE_BYTES = Cfg::STAGE_BYTES;
  extern __shared__ __align__(1024) uint8_t gsm_raw[];
  uint8_t* gsm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(gsm);
  __shared__ __align__(8) uint64_t bars[2 * GSTAGES + 1];  // full[s], empty[s], done
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = blockIdx.x / p.tiles_n, nt = blockIdx.x % p.tiles_n;
  const int m0 = mt * GM, n0 = nt * GN;
  const int64_t k0 = (int64_t)blockIdx.y * p.kchunk;
  const int nk = (int)((std::min<int64_t>(p.K, k0 + p.kchunk) - k0 + GK - 1) / GK);
  auto bar = [&](int i) -> uint32_t { return smem_u32(&bars[i]); };
  auto sA = [&](int s) -> uint32_t { return sb + (uint32_t)(s * STAGE_BYTES); };
  auto sB = [&](int s) -> uint32_t { return sb + (uint32_t)(s * STAGE_BYTES + A_BYTES); };
  const Abort ab{&abort_flag, p.status};

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < GSTAGES; ++s) {
      mbar_init(bar(s), 1);
      mbar_init(bar(GSTAGES + s), 1);
    }
    mbar_init(bar(2 * GSTAGES), 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.ta);
    prefetch_tmap(&p.tb);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), GN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(&tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % GSTAGES;
        // stage s is free once the MMAs of its previous use completed (the first
        // use waits on the phase before the barrier's first, which counts as done)
        if (!mbar_wait(bar(GSTAGES + s), ((i / GSTAGES) & 1) ^ 1, ab)) break;
        mbar_arrive_expect_tx(bar(s), STAGE_BYTES);
        const int kr = (int)(k0 + (int64_t)i * GK);
#pragma unroll
        for (int g = 0; g < GM / 64; ++g) tma_load_2d(sA(s) + g * GGROUP, &p.ta, bar(s), m0 + 64 * g, kr);
#pragma unroll
        for (int g = 0; g < GN / 64; ++g) tma_load_2d(sB(s) + g * GGROUP, &p.tb, bar(s), n0 + 64 * g, kr);
        issued = i + 1;
      }
      // never leave a copy in flight into this CTA's shared memory
      for (int i = issued - 1; i >= 0 && i > issued - 1 - GSTAGES; --i)
        drain_wait(bar(i % GSTAGES), (i / GSTAGES) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16(GM, GN, 1, 1, 1);  // bf16, A and B MN-major
      for (int i = 0; i < nk; ++i) {
        const int s = i % GSTAGES;
        if (!mbar_wait(bar(s), (i / GSTAGES) & 1, ab)) break;
        tc_fence_after();
        const uint32_t da = sw128_desc(sA(s), GGROUP), db = sw128_desc(sB(s), GGROUP);
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)  // 16 K rows = 2048 bytes per MMA
          mma_ss(tmem, da + kk * 128, db + kk * 128, ID, (i | kk) != 0);
        mma_commit(bar(GSTAGES + s));
      }
      mma_commit(bar(2 * GSTAGES));
      drain_wait(bar(2 * GSTAGES), 0);  // no MMA may still be writing TMEM at teardown
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int wq = warp & 3;  // TMEM lane quadrant this warp may read
    const int row = m0 + 32 * wq + lane;
    if (warp_wait(bar(2 * GSTAGES), 0, ab)) {
      tc_fence_after();
      float* dst = p.part + (int64_t)blockIdx.y * p.split_stride + (int64_t)row * p.ldp + n0;
#pragma unroll 1
      for (int c = 0; c < GN; c += 32) {
        uint32_t r[32];
        tmem_load32(tmem + ((uint32_t)(32 * wq) << 16) + (uint32_t)c, r);
        if (row < p.M) {
          if (n0 + c + 32 <= p.N) {
#pragma unroll
            for (int v = 0; v < 32; v += 4)
              *reinterpret_cast<float4*>(dst + c + v) =
                  make_float4(__uint_as_float(r[v]), __uint_as_float(r[v + 1]), __uint_as_float(r[v + 2]),
                              __uint_as_float(r[v + 3]));
          } else {
#pragma unroll
            for (int v = 0; v < 32; ++v)
              if (n0 + c + v < p.N) dst[c + v] = __uint_as_float(r[v]);
          }
        }
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, GN);
  }
}

// C[m][n] = sum over splits s (in order) of part[s][m][n], four columns per
// thread (M*N/4 < 2^31 items); the splits' loads are issued eight at a time.
__global__ void __launch_bounds__(256) gemm_sum_splits_kernel(const float* part, int64_t split_stride, int splits,
                                                              int M, int N, float* c, int64_t ldc) {
  const int n4 = N / 4;
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= M * n4) return;
  const int m = i / n4, q = i - m * n4;
  const float* src = part + (int64_t)m * N + 4 * q;
  float4 acc = *reinterpret_cast<const float4*>(src);
#pragma unroll 8
  for (int s = 1; s < splits; ++s) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(src + s * split_stride));
    acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
  }
  *reinterpret_cast<float4*>(c + (int64_t)m * ldc + 4 * q) = acc;
}

int gemm_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  return n;
}

// Tile width and split of K: enough CTAs for one per SM, at least 512 rows (8
// stages) per split (shorter splits cost more in partial sums than they gain).
struct SplitPlan {
  int gn, tiles, tiles_n, splits, kchunk;
};
SplitPlan plan_splits(int64_t K, int64_t M, int64_t N) {
  SplitPlan sp;
  sp.gn = 128;
  sp.tiles_n = (int)((N + sp.gn - 1) / sp.gn);
  sp.tiles = (int)((M + GM - 1) / GM) * sp.tiles_n;
  const int64_t max_splits = std::max<int64_t>(1, K / 512);
  const int64_t want = std::max<int64_t>(1, (gemm_sms() + sp.tiles / 2) / sp.tiles);
  int64_t s = std::min(max_splits, want);
  int64_t chunk = (K + s - 1) / s;
  chunk = (chunk + GK - 1) / GK * GK;
  sp.kchunk = (int)chunk;
  sp.splits = (int)((K + chunk - 1) / chunk);
  return sp;
}

}  // namespace
}  // namespace pnft

using namespace pnft;

extern "C" size_t pnft_gemm_at_b_workspace_size(int64_t K, int64_t M, int64_t N) {
  if (K <= 0 || M <= 0 || N <= 0) return 0;
  const SplitPlan sp = plan_splits(K, M, N);
  return sp.splits > 1 ? sizeof(float) * (size_t)sp.splits * (size_t)M * (size_t)N : 0;
}

extern "C" int pnft_gemm_at_b(const void* a, int64_t lda, const void* b, int64_t ldb, float* c, int64_t ldc,
                              void* workspace, size_t workspace_bytes, int64_t K, int64_t M, int64_t N, int dtype,
                              int32_t* status, void* stream) {
  if (K < 0 || M <= 0 || N <= 0 || M > (1 << 24) || N > (1 << 24) || K >= ((int64_t)1 << 31))
    return fail(PNFT_EINVAL, "gemm_at_b: bad shape K=%lld M=%lld N=%lld", (long long)K, (long long)M, (long long)N);
  if (dtype != PNFT_DTYPE_BF16) return fail(PNFT_EUNSUPPORTED, "gemm_at_b: bfloat16 operands only");
  if (!a || !b || !c) return fail(PNFT_EINVAL, "gemm_at_b: null pointer");
  cudaStream_t st = as_stream(stream);
  if (K == 0) {
    for (int64_t m = 0; m < M; ++m)
      if (cudaMemsetAsync(c + m * ldc, 0, sizeof(float) * N, st) != cudaSuccess) return check_launch("gemm_at_b memset", 0);
    return PNFT_OK;
  }
  if (lda < M || ldb < N || ldc < N) return fail(PNFT_EINVAL, "gemm_at_b: leading dimensions below the widths");
  if (lda % 8 || ldb % 8 || M % 8 || N % 8 || reinterpret_cast<uintptr_t>(a) % 16 ||
      reinterpret_cast<uintptr_t>(b) % 16)
    return fail(PNFT_EUNSUPPORTED, "gemm_at_b: rows must be 16-byte aligned (widths and strides multiples of 8)");
  if (ldc % 4 || reinterpret_cast<uintptr_t>(c) % 16)
    return fail(PNFT_EUNSUPPORTED, "gemm_at_b: the output's rows must be 16-byte aligned");
  if (!device_is_sm100()) return fail(PNFT_EUNSUPPORTED, "gemm_at_b: needs an sm_100 device");
  const SplitPlan sp = plan_splits(K, M, N);
  GemmParams p;
  memset(&p, 0, sizeof(p));
  int rc = tma_map_rows(&p.ta, a, M, K, lda, GK);
  if (!rc) rc = tma_map_rows(&p.tb, b, N, K, ldb, GK);
  if (rc) return rc;
  if (sp.splits > 1) {
    const size_t need = pnft_gemm_at_b_workspace_size(K, M, N);
    if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 16)
      return fail(PNFT_EINVAL, "gemm_at_b: workspace of %zu bytes < required %zu (16-byte aligned)", workspace_bytes,
                  need);
    p.part = static_cast<float*>(workspace);
    p.ldp = N;
    p.split_stride = M * N;
  } else {
    p.part = c;
    p.ldp = ldc;
    p.split_stride = 0;
  }
  p.M = (int)M;
  p.N = (int)N;
  p.K = K;
  p.kchunk = sp.kchunk;
  p.tiles_n = sp.tiles_n;
  p.status = status;
  if (sp.gn == 256) {
    if (cudaFuncSetAttribute(gemm_at_b_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<256>::SMEM) !=
        cudaSuccess)
      return check_launch("gemm_at_b smem attribute", 0);
    gemm_at_b_kernel<256><<<dim3(sp.tiles, sp.splits), GTHREADS, GemmCfg<256>::SMEM, st>>>(p);
  } else {
    if (cudaFuncSetAttribute(gemm_at_b_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<128>::SMEM) !=
        cudaSuccess)
      return check_launch("gemm_at_b smem attribute", 0);
    gemm_at_b_kernel<128><<<dim3(sp.tiles, sp.splits), GTHREADS, GemmCfg<128>::SMEM, st>>>(p);
  }
  int n = 1;
  if (sp.splits > 1) {
    const int64_t items = M * (N / 4);
    gemm_sum_splits_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(p.part, p.split_stride, sp.splits,
                                                                           (int)M, (int)N, c, ldc);
    ++n;
  }
  return check_launch("gemm_at_b", n);
}
