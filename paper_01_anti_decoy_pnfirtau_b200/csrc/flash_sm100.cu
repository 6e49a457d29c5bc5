// sm_100a flash pn_fir_tau kernels: TMA -> shared memory, tcgen05 MMAs with
// TMEM accumulators, warp-specialised pipelines. bf16 inputs, head dim 64/128 (smaller
// head dims that are multiples of 16 run zero-padded: the TMA loads fill the missing
// head dims with zeros and the epilogue stores only the real ones).
//
// Forward, one CTA per (128 query rows, b*h), 192 threads, two CTAs per SM (each
// holds 256 of the 512 TMEM columns; the two CTAs' tile phases are independent,
// so one CTA's loads, hand-offs and MMAs overlap the other's elementwise work):
//   warp 0      TMA producer: Q once; K and V tile j+1 while tile j is computed.
//   warp 1      MMA issuer and TMEM owner: S_j = Q K_j^T (SS, M=128, N=64) into
//               one of two S buffers; O += P_j V_j (TS: P read from TMEM) for the
//               live 64-key tiles only.
//   warps 2-5   one elementwise group of four warps (covering the four TMEM lane
//               quadrants, warp % 4) owning all 64 key columns of every tile (per
//               warp and tile the bookkeeping is amortised over 64 columns, half
//               the per-element cost of two groups of 32), thread = TMEM lane = query row:
//               s = S*scale - tau (packed f32x2 FMA, rounded once), u = max(s, 0),
//               row max via 3-input max, per-warp silent vote, u^10 by repeated
//               squaring (no exp), running peak / tie count / argmax / mass, and
//               P = u^10 split into two bf16 terms P_hi + P_lo written back over
//               the tile's own S columns in TMEM for the two PV MMAs.
// TMEM (256 columns per CTA): S/P buffers [0,64) and [64,128), O [128, 128+D).
// With the fused FIR, warps 2-3 filter the K tiles (fir_tile.cuh), the
// elementwise warps are 4-7 and the CTA runs alone on its SM.
// Epilogue: O * gate/(mass + 1e-12) with gate = peak/(peak+gamma), stats M, Z,
// Nmax, argmax.
// Semantics follow src/triton_pnfirtau.py:313-443 (the reference skips 64x64
// tiles; here the skip unit is 128 query rows x 64 keys, and the optional
// tile_flags record reports the 64x64 decisions of the same u values).
//
// Every mbarrier wait is bounded (sm100_ptx.cuh): on timeout the CTA sets the
// caller's status word, drains its own TMA/MMA work and frees TMEM.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "fir_tile.cuh"
#include "flash.cuh"
#include "sm100_ptx.cuh"

namespace pnft {

using namespace sm100;

namespace {

constexpr int FM = 128;  // query rows per CTA (TMEM lanes)
constexpr int FN = 64;   // keys per tile
constexpr int FQ = 64;                  // key columns per elementwise group
constexpr int NQW = FN / FQ;            // elementwise groups of four warps
// warp 0 producer, warp 1 MMA issuer, elementwise warps from EW0 on (with the
// fused FIR, warps 2-3 filter K and the elementwise warps start at 4)
template <bool FIR> constexpr int ew0() { return FIR ? 4 : 2; }
template <bool FIR> constexpr int f_threads() { return 32 * ew0<FIR>() + 128 * NQW; }

// barrier slots
enum : int {
  B_QFULL = 0,
  B_KFULL = 1,   // [2]
  B_KEMPTY = 3,  // [2]
  B_VFULL = 5,   // [2]
  B_VEMPTY = 7,  // [2]
  B_SFULL = 9,   // [2]
  B_PFULL = 11,  // [2]
  B_OFULL = 13,
  B_FLAG = 14,  // plain arrive after the o_written flag is stored (release for the flag)
  B_RAWFULL = 15,   // [2] fused FIR: raw K rows (with halo) landed
  B_RAWEMPTY = 17,  // [2] fused FIR: raw stage read by the filter warps
  B_STALL = 19,     // test-only: a barrier nothing arrives on (PNFT_FLASH_TEST_STALL)
  B_COUNT = 20
};

// Fused FIR: raw K rows [128 j - FIR_HALO, 128 j + 128) of tile j are staged by TMA
// and warps 2-3 write K~ = causal_fir(K) rows of the tile into the K stage for the
// MMA (fir_tile.cuh).
constexpr int RAW_ROWS = FN + FIR_HALO;

template <int D>
struct FwdLayout {
  static constexpr int GROUP = FM * 128;            // bytes of one 64-column (128 B) group of a Q tile
  static constexpr int KGROUP = FN * 128;           // same for a K / V tile
  static constexpr int QBYTES = FM * D * 2;
  static constexpr int KBYTES = FN * D * 2;
  static constexpr int VBYTES = FN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QBYTES;       // 2 stages
  static constexpr int OFF_V = OFF_K + 2 * KBYTES;   // 2 stages
  static constexpr int OFF_BAR = OFF_V + 2 * VBYTES;
  static constexpr int OFF_TMEM = OFF_BAR + B_COUNT * 8;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_OWR = OFF_ABORT + 4;
  // u8 [2 buf][NQW column groups][4 warps]: one word per group, nonzero when any warp saw a live row
  static constexpr int OFF_VPART = OFF_OWR + 8;
  static constexpr int OFF_STATS = OFF_VPART + 2 * NQW * 4;  // float [NQW][4][128]: peak, mass, count, argmax
  // float4 per row (16-byte aligned for the vector loads): running peaks of the column groups
  // (slots past NQW stay zero)
  static constexpr int OFF_RPK = (OFF_STATS + NQW * 4 * FM * 4 + 15) & ~15;
  static_assert(OFF_RPK % 16 == 0, "float4 rows need 16-byte alignment");
  // d=64 only (d=128 has no room): per elementwise lane the FQ s-values of the tile
  // that set its column block's peak, rows FQ*4 + 16 B apart (an odd number of 16-byte
  // units: conflict-free 16-byte stores)
  static constexpr bool DEFER = D == 64;
  static constexpr int REC_STRIDE = FQ * 4 + 16;
  static constexpr int OFF_REC = OFF_RPK + FM * 16;
  static_assert(OFF_REC % 16 == 0, "16-byte rows");
  static constexpr int END = OFF_REC + (DEFER ? NQW * FM * REC_STRIDE : 0);
  static constexpr int ALLOC = END + 1024;           // slack to align the base to 1024
  static constexpr int SMEM = ALLOC;  // two CTAs per SM, 256 TMEM columns each
  // fused FIR: raw K stages after the rest (1024-aligned for the 128-byte swizzle)
  static constexpr int RAWGROUP = RAW_ROWS * 128;    // one 64-column group of a raw stage
  static constexpr int RAWBYTES = (D / 64) * RAWGROUP;
  static constexpr int NRAW = D == 64 ? 2 : 1;
  static constexpr int OFF_RAW = (END + 1023) & ~1023;
  static constexpr int SMEM_FIR = OFF_RAW + NRAW * RAWBYTES + 1024;
  static_assert(SMEM <= 227 * 1024 && SMEM_FIR <= 227 * 1024, "shared memory budget");
};

// S buffer s at [FN s, FN s + FN); group g's P_hi / P_lo of that tile overwrite its
// own S columns [FN s + 32 g, +16) / [+16, +16) once they are in registers.
constexpr uint32_t TM_S = 0, TM_O = 2 * FN, TM_COLS = 256;
static_assert(TM_O + 128 <= TM_COLS, "TMEM budget (d <= 128)");

struct FwdParams {
  CUtensorMap tq, tk, tv;
  CUtensorMap tkr;    // fused FIR: raw K, RAW_ROWS-row boxes
  const float* taps;  // fused FIR: fp32[FIR_TAPS], index FIR_TAPS-1 = lag 0
  void* out;
  int64_t so[4];
  float* out32;
  float* stat_m;
  float* stat_z;
  int32_t* stat_nmax;
  int32_t* stat_arg;
  uint8_t* tile_flags;
  const float* tau;
  int32_t* status;
  int H, N, nq, nk;
  int dreal;  // the operands' head dim: D when D is 64 / 128, else zero-padded to D by the TMA loads
  float scale, gamma;
  int has_gamma, causal;
  int stall;  // PNFT_FLASH_TEST_STALL: the elementwise warps first wait on B_STALL
  int hgroup;  // heads per group of the CTA order (work_item)
};

template <int D, bool FIR>
__global__ void __launch_bounds__(f_threads<FIR>(), FIR ? 1 : 2) flash_fwd_sm100_kernel(const __grid_constant__ FwdParams p) {
  using L = FwdLayout<D>;
  constexpr int DG = D / 64;  // 64-column groups of a row
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // offset from the __shared__ array itself, so the compiler keeps shared-space accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb0 = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // b*h runs fastest and the query tiles go from the last (longest causal rows)
  // down: the grid starts with its longest CTAs, so none starts late
  int bh, qt;
  work_item((int)(blockIdx.y * gridDim.x + blockIdx.x), (int)gridDim.x, p.nq, p.hgroup, &bh, &qt);
  qt = p.nq - 1 - qt;
  const int b = bh / p.H, hd = bh % p.H;
  const int q0 = qt * FM;
  const int ntiles = p.causal ? min(p.nk, (q0 + FM + FN - 1) / FN) : p.nk;
  auto bar = [&](int i) -> uint32_t { return sb0 + L::OFF_BAR + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_ABORT);
  volatile uint8_t* vpart = smem + L::OFF_VPART;
  const Abort ab{abort_flag, p.status};

  if (threadIdx.x == 0) {
    mbar_init(bar(B_QFULL), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_KFULL + i), FIR ? 2 : 1);  // fused FIR: one arrive per filter warp
      mbar_init(bar(B_RAWFULL + i), 1);
      mbar_init(bar(B_RAWEMPTY + i), 2);
      mbar_init(bar(B_KEMPTY + i), 1);
      mbar_init(bar(B_VFULL + i), 1);
      mbar_init(bar(B_VEMPTY + i), 1);
      mbar_init(bar(B_SFULL + i), 1);
      mbar_init(bar(B_PFULL + i), 4 * NQW);
    }
    mbar_init(bar(B_OFULL), 1);
    mbar_init(bar(B_FLAG), 1);
    mbar_init(bar(B_STALL), 1);
    *abort_flag = 0;
    *reinterpret_cast<volatile int*>(smem + L::OFF_OWR) = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tq);
    prefetch_tmap(FIR ? &p.tkr : &p.tk);
    prefetch_tmap(&p.tv);
  }
  if (warp == 1) {
    tmem_alloc(sb0 + L::OFF_TMEM, TM_COLS);
    tmem_relinquish();
  }
  for (int i = threadIdx.x; i < FM * 4; i += blockDim.x) reinterpret_cast<float*>(smem + L::OFF_RPK)[i] = 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::OFF_TMEM);
  const uint32_t sQ = sb0 + L::OFF_Q;
  auto sK = [&](int s) -> uint32_t { return sb0 + L::OFF_K + (uint32_t)s * L::KBYTES; };
  auto sV = [&](int s) -> uint32_t { return sb0 + L::OFF_V + (uint32_t)s * L::VBYTES; };
  auto sRaw = [&](int s) -> uint32_t { return sb0 + L::OFF_RAW + (uint32_t)s * L::RAWBYTES; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int k_last = -1, v_last = -1;
      mbar_arrive_expect_tx(bar(B_QFULL), L::QBYTES);
      for (int g = 0; g < DG; ++g) tma_load_4d(sQ + g * L::GROUP, &p.tq, bar(B_QFULL), 64 * g, q0, hd, b);
      auto issue_k = [&](int j) -> bool {
        if constexpr (FIR) {
          // raw rows [j*FN - RAW_HALO, (j+1)*FN) into a raw stage; the filter warps fill K
          const int r = j % L::NRAW;
          if (!mbar_wait(bar(B_RAWEMPTY + r), ((j / L::NRAW) & 1) ^ 1, ab)) return false;
          mbar_arrive_expect_tx(bar(B_RAWFULL + r), L::RAWBYTES);
          for (int g = 0; g < DG; ++g)
            tma_load_4d(sRaw(r) + g * L::RAWGROUP, &p.tkr, bar(B_RAWFULL + r), 64 * g, j * FN - FIR_HALO, hd, b);
        } else {
          const int s = j & 1;
          if (!mbar_wait(bar(B_KEMPTY + s), ((j >> 1) & 1) ^ 1, ab)) return false;
          mbar_arrive_expect_tx(bar(B_KFULL + s), L::KBYTES);
          for (int g = 0; g < DG; ++g) tma_load_4d(sK(s) + g * L::KGROUP, &p.tk, bar(B_KFULL + s), 64 * g, j * FN, hd, b);
        }
        k_last = j;
        return true;
      };
      // V is fetched with its K tile, not after the silence vote: the vote still
      // skips the PV MMAs of silent halves, but a V fetch on the critical path
      // of every tile costs more than the L2 traffic it saves
      auto issue_v = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(bar(B_VEMPTY + s), ((j >> 1) & 1) ^ 1, ab)) return false;
        mbar_arrive_expect_tx(bar(B_VFULL + s), L::VBYTES);
        for (int hh = 0; hh < FN / 64; ++hh)
          for (int g = 0; g < DG; ++g)
            tma_load_4d(sV(s) + g * L::KGROUP + hh * 64 * 128, &p.tv, bar(B_VFULL + s), 64 * g,
                        j * FN + 64 * hh, hd, b);
        v_last = j;
        return true;
      };
      bool ok = issue_k(0) && issue_v(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles) ok = issue_k(j + 1) && issue_v(j + 1);
      }
      // drain: never leave a copy in flight into this CTA's shared memory
      drain_wait(bar(B_QFULL), 0);
      if constexpr (FIR) {
        for (int j = k_last; j >= 0 && j > k_last - L::NRAW; --j)
          drain_wait(bar(B_RAWFULL + j % L::NRAW), (j / L::NRAW) & 1);
      } else {
        for (int j = k_last; j >= 0 && j > k_last - 2; --j) drain_wait(bar(B_KFULL + (j & 1)), (j >> 1) & 1);
      }
      for (int j = v_last; j >= 0 && j > v_last - 2; --j) drain_wait(bar(B_VFULL + (j & 1)), (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(FM, FN, 1, 0, 0);
      constexpr uint32_t ID_O = idesc_f16(FM, D, 1, 0, 1);
      uint32_t o_acc = 0;
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        // buffer s last held P_{j-2}: its PV MMAs were issued before this one and
        // tcgen05 MMAs of one thread execute in order
        if (!mbar_wait(bar(B_KFULL + s), (j >> 1) & 1, ab)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::GROUP + (kk & 3) * 32, koff = (kk >> 2) * L::KGROUP + (kk & 3) * 32;
          mma_ss(tmem + TM_S + (uint32_t)FN * s, sw128_desc(sQ + off, 16), sw128_desc(sK(s) + koff, 16), ID_S,
                 kk > 0);
        }
        mma_commit(bar(B_SFULL + s));
        mma_commit(bar(B_KEMPTY + s));
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(bar(B_PFULL + s), (j >> 1) & 1, ab)) return false;
        if (!mbar_wait(bar(B_VFULL + s), (j >> 1) & 1, ab)) return false;
        tc_fence_after();
        for (int g = 0; g < NQW; ++g) {
          // the four warps' votes of this column block, published before their PFULL arrives
          if (!reinterpret_cast<volatile const uint32_t*>(vpart)[s * NQW + g]) continue;  // silent: P is zero
#pragma unroll
          for (int kq = 0; kq < FQ / 16; ++kq) {
            const int kk = g * (FQ / 16) + kq;  // 16 keys per MMA
            const uint32_t a_hi = tmem + TM_S + (uint32_t)FN * s + (uint32_t)FQ * g + 8u * kq;
            const uint32_t bdesc = sw128_desc(sV(s) + kk * 2048, L::KGROUP);
            mma_ts(tmem + TM_O, a_hi, bdesc, ID_O, o_acc);             // O += P_hi V
            mma_ts(tmem + TM_O, a_hi + FQ / 2, bdesc, ID_O, 1u);       // O += P_lo V
            o_acc = 1;
          }
        }
        mma_commit(bar(B_VEMPTY + s));
        return true;
      };
      if (mbar_wait(bar(B_QFULL), 0, ab)) {
        bool ok = true;
        for (int j = 0; ok && j < ntiles; ++j) {
          ok = issue_s(j);
          if (ok && j >= 1) ok = issue_pv(j - 1);
        }
        if (ok) issue_pv(ntiles - 1);
      }
      *reinterpret_cast<volatile int*>(smem + L::OFF_OWR) = (int)o_acc;
      mbar_arrive(bar(B_FLAG));
      mma_commit(bar(B_OFULL));
      drain_wait(bar(B_OFULL), 0);  // no MMA may still be writing TMEM at teardown
    }
  } else if (warp < ew0<FIR>()) {
    // ------------------------------------------------------------ fused FIR filter (warps 2-3)
    if constexpr (FIR) {
      // 64 threads: column pair ct % 32 of every group, output rows [64 (ct / 32), +64)
      const int ct = threadIdx.x - 64;
      float2 h[FIR_TAPS];
      fir_load_taps(p.taps, h);
      for (int j = 0; j < ntiles; ++j) {
        const int r = j % L::NRAW, s = j & 1;
        if (!warp_wait(bar(B_RAWFULL + r), (j / L::NRAW) & 1, ab)) break;
        if (!warp_wait(bar(B_KEMPTY + s), ((j >> 1) & 1) ^ 1, ab)) break;  // S of tile j-2 has read stage s
#pragma unroll
        for (int g = 0; g < DG; ++g)
          fir_filter_rows<FN / 2>(smem + L::OFF_RAW + r * L::RAWBYTES + g * L::RAWGROUP,
                                  smem + L::OFF_K + s * L::KBYTES + g * L::KGROUP, ct & 31, (ct >> 5) * (FN / 2), h);
        fence_proxy_async_smem();  // the tensor core reads K through the async proxy
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(B_KFULL + s));
          mbar_arrive(bar(B_RAWEMPTY + r));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ elementwise
    const int ew = warp - ew0<FIR>(), g = ew >> 2, wq = warp & 3;  // group g owns key columns [FQ g, FQ g + FQ)
    const int rl = 32 * wq + lane;  // TMEM lane = local query row
    const int row = q0 + rl;
    const uint32_t lane_off = (uint32_t)(32 * wq) << 16;
    const float tau = __ldg(p.tau);
    // h = (S*scale - tau)/2, rounded once, two columns per packed f32x2 FMA. The
    // halving is exact, so maxima and ties of h are those of s, and the relu
    // u = max(s, 0) = h + |h| is one FMA-pipe add instead of an ALU max. Peaks are
    // kept as h until the epilogue doubles them.
    const float2 sc2 = make_float2(0.5f * p.scale, 0.5f * p.scale), nt2 = make_float2(-0.5f * tau, -0.5f * tau);
    const int nT64 = (p.N + 63) >> 6;
    float peak = 0.f, cnt = 0.f;
    int arg = -1;  // first key attaining the running peak in this column block
    // deferred search (d=64): the tile that set the peak is saved; `arg` holds its
    // first key and `cnt` counts only the maxima of later tiles equal to the peak
    float* rec = reinterpret_cast<float*>(smem + L::OFF_REC + (g * FM + rl) * L::REC_STRIDE);
    // running peaks of this row's column groups; a group whose tile maximum is
    // below the row's best so far can never hold the row maximum, so it skips the
    // per-column search (the estimate may lag: that only costs extra searches)
    float4* rpk = reinterpret_cast<float4*>(smem + L::OFF_RPK) + rl;  // zeroed before the first __syncthreads
    float2 ms[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // mass partial sums
    // `dead` (warp-uniform) turns the rest of the loop into no-ops after an
    // abort, while every warp still passes the named barriers.
    bool dead = false;
    // test-only (p.stall): the first wait is on B_STALL, which nothing completes,
    // so the warps run it out and unwind like any timed-out wait
    const uint32_t bar_s0 = p.stall ? bar(B_STALL) : bar(B_SFULL);
    for (int j = 0; j < ntiles; ++j) {
      const int s = j & 1;
      if (!dead) dead = !warp_wait(j == 0 ? bar_s0 : bar(B_SFULL + s), (j >> 1) & 1, ab);
      const uint32_t scol = tmem + lane_off + TM_S + (uint32_t)FN * s + (uint32_t)FQ * g;
      static_assert(FQ == 32 || FQ == 64, "32 or 64 key columns per warp");
      uint32_t r[FQ / 32][32];
      if (!dead) {
        tc_fence_after();
        if constexpr (FQ == 64) tmem_load32x2(scol, r[0], scol + 32, r[FQ / 32 - 1]);
        else tmem_load32(scol, r[0]);
      }
      float x[FQ];
#pragma unroll
      for (int c = 0; c < FQ; c += 2) {
        const float2 a = __ffma2_rn(make_float2(__uint_as_float(r[c >> 5][c & 31]), __uint_as_float(r[c >> 5][(c & 31) + 1])), sc2, nt2);
        x[c] = a.x;
        x[c + 1] = a.y;
      }
      const int kb = j * FN + FQ * g;
      int lim = row < p.N ? (p.causal ? row : p.N - 1) - kb : -1;  // last valid column offset
      if (dead) lim = -1;                                                // after an abort: silent
      if (lim < FQ - 1) {
#pragma unroll
        for (int c = 0; c < FQ; ++c) x[c] = c > lim ? -1.f : x[c];
      }
      // row maximum as four independent 3-input max chains of FQ/4 columns (dependency
      // depth ~FQ/8 + 2 instead of FQ/2)
      constexpr int MQ = FQ / 4;
      float mc[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        mc[k] = max3(x[k * MQ], x[k * MQ + 1], x[k * MQ + 2]);
#pragma unroll
        for (int c = 3; c + 1 < MQ; c += 2) mc[k] = max3(mc[k], x[k * MQ + c], x[k * MQ + c + 1]);
        if constexpr (MQ % 2 == 0) mc[k] = fmaxf(mc[k], x[k * MQ + MQ - 1]);
      }
      const float m = max3(mc[0], mc[1], fmaxf(mc[2], mc[3]));
      // silent vote of this warp's 32 rows; the MMA issuer ORs the four warps of
      // the column block after PFULL completes (no barrier between the warps). A silent
      // warp writes zeros: another warp's rows may keep the column block live.
      const unsigned live_w = __any_sync(0xffffffffu, m > 0.f);
      if (lane == 0) {
        vpart[(s * NQW + g) * 4 + wq] = live_w ? 1 : 0;
        if (p.tile_flags && live_w) {
          const int qi = (q0 >> 6) + (wq >> 1), kj = kb >> 6;
          if (qi < nT64 && kj < nT64) p.tile_flags[((int64_t)bh * nT64 + qi) * nT64 + kj] = 1;
        }
      }
      if (live_w && !dead) {
        const float mu = m > 0.f ? m : 0.f;  // row max of u/2 over this column block of the tile
        const float4 rp4 = *rpk;
        const float row_best = fmaxf(fmaxf(rp4.x, rp4.y), fmaxf(rp4.z, rp4.w));
        if (mu > 0.f && mu >= fmaxf(peak, row_best)) {
          if (L::DEFER && mu > peak) {
            // new peak: save the tile's values, search them once after the loop
#pragma unroll
            for (int k = 0; k < FQ / 4; ++k)
              reinterpret_cast<float4*>(rec)[k] = make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]);
            arg = kb;
            cnt = 0.f;
          } else {
            // columns attaining the maximum as a bit mask: count and first key
            unsigned long long mk = 0ull;
#pragma unroll
            for (int i = 0; i < FQ; ++i) mk |= x[i] == m ? 1ull << i : 0ull;
            const float c = (float)__popcll(mk);
            if (mu > peak) arg = kb + __ffsll((long long)mk) - 1;  // equal to an earlier tile's peak: keep the earlier key
            cnt = mu > peak ? c : cnt + c;
          }
          peak = mu;
          reinterpret_cast<float*>(rpk)[g] = peak;
        }
        // P = u^10 as P_hi + P_lo (two bf16 terms: P_hi truncated, P_lo = P - P_hi exact
        // then rounded, ~2^-17 relative): O, and with it the
        // backward's <dO,O>/gate, stays fp32-accurate; the tau gradient is a small
        // residual of cancelling per-row sums and needs that accuracy
        // Quarters of 16 columns, each stored as soon as it is packed (fewer live
        // registers): P_hi / P_lo over this group's own S columns
        // [FQ g + 8hh, +8) / [FQ g + FQ/2 + 8hh, +8).
        const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
        for (int hh = 0; hh < FQ / 16; ++hh) {
          uint32_t hi[8], lo[8];
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const int c = 8 * hh + cc;
            const float2 u =
                make_float2(__fadd_rn(x[2 * c], fabsf(x[2 * c])), __fadd_rn(x[2 * c + 1], fabsf(x[2 * c + 1])));
            const float2 u2 = __fmul2_rn(u, u), u4 = __fmul2_rn(u2, u2);
            const float2 pw = __fmul2_rn(__fmul2_rn(u4, u4), u2);
            ms[c & 1] = __fadd2_rn(ms[c & 1], pw);
            // P_hi = P truncated to bf16 (its low 16 bits cleared), packed by one byte permute
            const uint32_t bx = __float_as_uint(pw.x), by = __float_as_uint(pw.y);
            hi[cc] = __byte_perm(bx, by, 0x7632);
            const float2 hf = make_float2(__uint_as_float(bx & 0xffff0000u), __uint_as_float(by & 0xffff0000u));
            const float2 lf = __ffma2_rn(hf, neg1, pw);  // exact: pw - hi
            lo[cc] = pack_bf16x2(lf.x, lf.y);
          }
          tmem_st8(scol + 8 * hh, hi);
          tmem_st8(scol + FQ / 2 + 8 * hh, lo);
        }
        tmem_wait_st();
      } else if (!dead) {
        uint32_t zr[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) zr[c] = 0u;
#pragma unroll
        for (int c = 0; c < FQ; c += 16) tmem_st16(scol + c, zr);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PFULL + s));
    }
    if (L::DEFER && peak > 0.f) {
      // search of the saved tile: its maximum equals the column block's peak
      unsigned long long mk = 0ull;
#pragma unroll
      for (int k = 0; k < FQ / 4; ++k) {
        const float4 v4 = reinterpret_cast<const float4*>(rec)[k];
        mk |= (unsigned long long)((v4.x == peak ? 1u : 0u) | (v4.y == peak ? 2u : 0u) | (v4.z == peak ? 4u : 0u) |
                                   (v4.w == peak ? 8u : 0u))
              << (4 * k);
      }
      cnt += (float)__popcll(mk);
      arg += __ffsll((long long)mk) - 1;
    }
    // ---- epilogue: merge the column groups of every row, scale O, store
    float* st = reinterpret_cast<float*>(smem + L::OFF_STATS);
    const float mass_q = (ms[0].x + ms[0].y) + (ms[1].x + ms[1].y);
    st[(g * 4 + 0) * FM + rl] = peak;
    st[(g * 4 + 1) * FM + rl] = mass_q;
    st[(g * 4 + 2) * FM + rl] = cnt;
    st[(g * 4 + 3) * FM + rl] = __int_as_float(arg);
    named_bar_sync(1 + NQW, 128 * NQW);
    float pk = 0.f, mass = 0.f;
#pragma unroll
    for (int q = 0; q < NQW; ++q) {
      pk = fmaxf(pk, st[(q * 4 + 0) * FM + rl]);
      mass += st[(q * 4 + 1) * FM + rl];
    }
    // first key of the row maximum: each column block kept its earliest key (an earlier
    // tile wins a tie), so the smallest key over the column blocks holding the maximum
    float nm = 0.f;
    int amax = -1;
    if (pk > 0.f) {
#pragma unroll
      for (int q = 0; q < NQW; ++q) {
        if (st[(q * 4 + 0) * FM + rl] == pk) {
          nm += st[(q * 4 + 2) * FM + rl];
          const int aq = __float_as_int(st[(q * 4 + 3) * FM + rl]);
          amax = amax < 0 ? aq : min(amax, aq);
        }
      }
    }
    pk *= 2.f;  // h -> s
    const float z = mass + 1e-12f;
    float gate = 0.f;
    if (pk > 0.f) gate = p.has_gamma ? pk / (pk + p.gamma) : 1.f;
    const float so = gate / z;
    const bool o_ok = warp_wait(bar(B_OFULL), 0, ab) && warp_wait(bar(B_FLAG), 0, ab);
    tc_fence_after();
    const bool o_written = o_ok && *reinterpret_cast<volatile int*>(smem + L::OFF_OWR) != 0;
    __nv_bfloat16* O = static_cast<__nv_bfloat16*>(p.out) + (int64_t)b * p.so[0] + (int64_t)hd * p.so[1] +
                       (int64_t)row * p.so[2];
#pragma unroll
    for (int cb = 0; cb < D / NQW; cb += 16) {  // group g writes head dims [g*D/NQW, (g+1)*D/NQW)
      const int d0 = g * (D / NQW) + cb;
      if (d0 >= p.dreal) break;  // zero-padded head dims: computed, never stored (warp-uniform)
      uint32_t r[16];
      if (o_written) {
        tmem_load16(tmem + lane_off + TM_O + (uint32_t)d0, r);
      }
      if (row < p.N && o_ok && p.out32) {
        float4* o32 = reinterpret_cast<float4*>(p.out32 + ((int64_t)bh * p.N + row) * p.dreal + d0);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float4 f;
          f.x = o_written ? __uint_as_float(r[4 * v + 0]) * so : 0.f;
          f.y = o_written ? __uint_as_float(r[4 * v + 1]) * so : 0.f;
          f.z = o_written ? __uint_as_float(r[4 * v + 2]) * so : 0.f;
          f.w = o_written ? __uint_as_float(r[4 * v + 3]) * so : 0.f;
          o32[v] = f;
        }
      }
      if (row < p.N && o_ok) {
        if (p.so[3] == 1 && (reinterpret_cast<uintptr_t>(O + d0) & 15) == 0) {
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = o_written ? __uint_as_float(r[8 * v + 2 * e]) * so : 0.f;
              const float hi = o_written ? __uint_as_float(r[8 * v + 2 * e + 1]) * so : 0.f;
              wp[e] = pack_bf16x2(lo, hi);
            }
            *reinterpret_cast<uint4*>(O + d0 + 8 * v) = w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            O[(int64_t)(d0 + e) * p.so[3]] = __float2bfloat16_rn(o_written ? __uint_as_float(r[e]) * so : 0.f);
        }
      }
    }
    if (g == 0 && row < p.N && o_ok) {
      const int64_t si = (int64_t)bh * p.N + row;
      p.stat_m[si] = pk;
      p.stat_z[si] = z;
      p.stat_nmax[si] = (int32_t)nm;
      p.stat_arg[si] = amax;
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_COLS);
  }
}

}  // namespace

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

int tma_map_bhnd(CUtensorMap* m, const void* base, const int64_t* s, int64_t B, int64_t H, int64_t N, int64_t D,
                 int rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(PNFT_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)s[2] * 2, (cuuint64_t)s[1] * 2, (cuuint64_t)s[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PNFT_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PNFT_OK;
}

int tma_map_rows(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t row_stride, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(PNFT_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PNFT_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return PNFT_OK;
}

bool tma_ok_bhnd(const void* ptr, const int64_t* s) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  if (s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (s[i] <= 0 || (s[i] % 8) != 0 || s[i] >= ((int64_t)1 << 38)) return false;
  return true;
}

int head_group(int64_t BH, int64_t head_bytes) {
  if (const char* e = getenv("PNFT_HEAD_GROUP")) {
    const long g = strtol(e, nullptr, 10);
    if (g > 0) return (int)std::min<int64_t>(g, BH);
  }
  const int64_t budget = (int64_t)80 << 20;
  const int64_t g = std::max<int64_t>(1, budget / std::max<int64_t>(head_bytes, 1));
  return (int)std::min<int64_t>(g, BH);
}

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return false;
  return major == 10 && minor == 0;
}

// Both passes of a bf16 call run on the same kernel family: the backward's tie
// test u == peak needs the forward's S recomputed by the same arithmetic.
bool flash_sm100_supported(const FlashArgs& a) {
  if (a.dtype != PNFT_DTYPE_BF16) return false;
  // head dims that are multiples of 16 up to 128; below 64 (or between 64 and 128) the
  // TMA loads zero-fill the operands to 64 (128) head dims, which changes no product
  if (a.D < 16 || a.D > 128 || a.D % 16 != 0) return false;
  if (a.N < 1 || a.N > (int64_t)1 << 30) return false;
  if (!tma_ok_bhnd(a.q, a.sq) || !tma_ok_bhnd(a.k, a.sk) || !tma_ok_bhnd(a.v, a.sv)) return false;
  return device_is_sm100();
}

int flash_fwd_sm100(const FlashArgs& a, cudaStream_t st) {
  FwdParams p;
  memset(&p, 0, sizeof(p));
  int rc = tma_map_bhnd(&p.tq, a.q, a.sq, a.B, a.H, a.N, a.D, FM);
  if (!rc) rc = tma_map_bhnd(&p.tk, a.k, a.sk, a.B, a.H, a.N, a.D, FN);
  if (!rc) rc = tma_map_bhnd(&p.tv, a.v, a.sv, a.B, a.H, a.N, a.D, 64);
  if (rc) return rc;
  p.out = a.out;
  for (int i = 0; i < 4; ++i) p.so[i] = a.so[i];
  p.out32 = a.out32;
  p.stat_m = a.stat_m;
  p.stat_z = a.stat_z;
  p.stat_nmax = a.stat_nmax;
  p.stat_arg = a.stat_arg;
  p.tile_flags = a.tile_flags;
  p.tau = a.tau;
  p.status = a.status;
  p.H = (int)a.H;
  p.N = (int)a.N;
  p.dreal = (int)a.D;
  p.nq = (int)((a.N + FM - 1) / FM);
  p.nk = (int)((a.N + FN - 1) / FN);
  p.scale = a.scale;
  p.gamma = a.gamma;
  p.has_gamma = a.has_gamma;
  p.causal = a.causal;
  p.stall = (a.flags & PNFT_FLASH_TEST_STALL) ? 1 : 0;
  p.hgroup = head_group(a.B * a.H, a.N * a.D * 4);  // K and V of a head, re-read by its query tiles
  if (p.nq > 65535) return fail(PNFT_EUNSUPPORTED, "flash fwd sm100: N = %lld needs more than 65535 query tiles", (long long)a.N);
  const dim3 grid((unsigned)(a.B * a.H), (unsigned)p.nq);
  auto launch = [&](auto kern, int smem) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return check_launch("flash fwd sm100: smem attribute", 0);
    kern<<<grid, a.fir_taps ? f_threads<true>() : f_threads<false>(), smem, st>>>(p);
    return check_launch("flash fwd sm100");
  };
  if (a.fir_taps) {
    if (a.fir_ntaps != FIR_TAPS) return fail(PNFT_EUNSUPPORTED, "flash fwd sm100: fused FIR needs %d taps", FIR_TAPS);
    rc = tma_map_bhnd(&p.tkr, a.k, a.sk, a.B, a.H, a.N, a.D, RAW_ROWS);
    if (rc) return rc;
    p.taps = a.fir_taps;
    if (a.D <= 64) return launch(flash_fwd_sm100_kernel<64, true>, FwdLayout<64>::SMEM_FIR);
    return launch(flash_fwd_sm100_kernel<128, true>, FwdLayout<128>::SMEM_FIR);
  }
  if (a.D <= 64) return launch(flash_fwd_sm100_kernel<64, false>, FwdLayout<64>::SMEM);
  return launch(flash_fwd_sm100_kernel<128, false>, FwdLayout<128>::SMEM);
}

}  // namespace pnft
