// sm_100a backward of flash pn_fir_tau (bf16, head dim 64/128; smaller head dims that
// are multiples of 16 zero-padded to them, as in the forward).
//
// One CTA per (128 keys, b*h), KV-parallel over the 64-query tiles at or below
// the causal diagonal whose rows are not all silent (per-tile flags from the
// prep kernel). 512 threads:
//   warp 0       TMA producer: K, V once; per query tile Q, dO (4 stages for
//                D=64, 2 for D=128) and the tile's per-row coefficient records.
//   warp 1       MMA issuer + TMEM owner (a converged warp; one elected lane
//                issues, descriptors are precomputed bases plus constant
//                offsets). Per tile t:
//                  S^T = K Q^T, dP^T = V dO^T            (SS, M=128 keys, N=64)
//                then for tile t-1 (overlapping tile t's elementwise work):
//                  dV += P^T dO   (TS: P^T bf16 from TMEM)
//                  dK += dS^T Q   (SS: dS^T bf16 from shared memory)
//                  dQ of a pair of query tiles = dS K (SS, M = 128 queries,
//                  N = head dims; D=64), or dQ^T = K^T dS^T per tile (SS,
//                  M = head dims; D=128), into TMEM
//   warps 4-11   elementwise, thread = TMEM lane = key; warpgroup g owns query
//                columns [32g, 32g+32). Each thread pulls its whole S/dP slice
//                into registers and releases TMEM at once, then computes
//                u = relu(S*scale - tau), W = c1 u^10 (-> P^T in TMEM) and
//                dS' = c1 u^9 (dP - D) + [key == argmax] tie/10 (-> smem,
//                128-byte swizzled), dS' = dS / (10 scale); the factor is applied
//                to dK here and to dQ by the cast kernel, and dtau = -10 sum dS'.
//                Two columns at a time in packed f32x2 arithmetic; masking only
//                on tiles that cross the diagonal or a sequence end; the gate
//                term is one patched entry per row (value tests only on tiles
//                holding a row with several maxima).
//   warps 12-15  dQ drain: TMEM -> fp32 staging tile in smem (D=64: each
//                thread one query row, 16-byte stores in acc_chunk order) -> one
//                cp.reduce.async.bulk add into the fp32 dQ accumulator (in
//                deterministic mode: a read-modify-write of the tile once the
//                lower key tiles of the head have added theirs, so the fp32
//                additions happen in key order on every run).
// Finally the elementwise warps write dK, dV (bf16) from TMEM.
// TMEM columns: see BwdLayout (D=64: S/dP x2 [0,256), dV, dK, dQ of a tile pair
//               [384,448); D=128: S/dP [0,128), P^T x2, dV, dK, dQ^T [448,512)).
// Semantics: src/triton_pnfirtau.py:445-621 with the per-row terms of
// flash_bwd_prep (RowCoef). S is recomputed by the tensor core exactly as in
// the tcgen05 forward, so u == peak finds the forward's maxima.
#include <string.h>

#include <type_traits>

#include "fir_tile.cuh"
#include "flash.cuh"
#include "sm100_ptx.cuh"

namespace pnft {

using namespace sm100;

namespace {

constexpr int BN = 128;  // keys per CTA (TMEM lanes)
constexpr int BM = 64;   // queries per tile
// two elementwise warpgroups of 32 query columns per warp: half the per-tile
// bookkeeping of four groups of 16 per score element, and 128 registers per thread
constexpr int NEW = 2;                       // elementwise warpgroups
constexpr int CW = BM / NEW;                 // query columns per elementwise warp
constexpr int W_DRAIN = 4 + 4 * NEW;         // first dQ drain warp
constexpr int B_THREADS = 32 * (W_DRAIN + 4);

enum : int {
  C_KV = 0,
  C_QDFULL = 1,    // [4]
  C_QDEMPTY = 5,   // [4]
  C_SDPFULL = 9,   // [2] (one per S/dP buffer)
  C_SDPEMPTY = 11, // single-buffer layout only
  C_PDSFULL = 12,  // [2]
  C_PDSEMPTY = 14, // [4] (one per dS buffer)
  C_DQFULL = 18,   // [2]
  C_DQEMPTY = 20,  // [2]
  C_DKV = 22,
  C_FLAG = 23,  // plain arrive after dkv_written is stored (release for the flag)
  C_KRAW = 24,  // fused FIR: raw K rows (with halo) landed
  C_STALL = 25, // test-only: a barrier nothing arrives on (PNFT_FLASH_TEST_STALL)
  C_COUNT = 26
};

template <int D>
struct BwdLayout {
  static constexpr int NQS = D == 64 ? 4 : 2;    // Q / dO / coefficient stages
  static constexpr int KGROUP = BN * 128;  // one 64-column group of the K / V tile
  static constexpr int QGROUP = BM * 128;  // one 64-column group of a Q / dO tile
  static constexpr int KBYTES = BN * D * 2;
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int NDQ = D == 64 ? 2 : 1;   // dQ buffers in TMEM
  // D=64: dQ of two consecutive tiles in one MMA sequence (M = 128 queries from two
  // adjacent dS tiles, N = 64 head dims)
  static constexpr bool DQ_PAIR = D == 64;
  static constexpr int NSTG = D == 64 ? 2 : 1;  // dQ staging tiles in smem
  static constexpr int STG_BYTES = BM * D * 4;
  static constexpr int DS_BYTES = BN * BM * 2;
  // dS^T tiles in smem. d=64: four, so the elementwise warps' tile j+2 waits only
  // for its S/dP (whose MMAs follow dV/dK of tile j) and not for dQ of tile j, the
  // last reader of dS_j. d=128 has room for two.
  static constexpr int NDS = D == 64 ? 4 : 2;
  // per query tile: 32 coefficient pairs {c1, c1, -D, -D}, tie/10, argmax, tie peak
  static constexpr int CF_P = 0, CF_TIE = BM * 8, CF_ARG = BM * 12, CF_PC = BM * 16, COEF_BYTES = BM * 20;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KBYTES;
  static constexpr int OFF_Q = OFF_V + KBYTES;
  static constexpr int OFF_DO = OFF_Q + NQS * QBYTES;
  static constexpr int OFF_DS = OFF_DO + NQS * QBYTES;
  static constexpr int OFF_STG = OFF_DS + NDS * DS_BYTES;
  static constexpr int OFF_COEF = OFF_STG + NSTG * STG_BYTES;
  static constexpr int OFF_BAR = OFF_COEF + NQS * COEF_BYTES;
  static constexpr int OFF_TMEM = OFF_BAR + C_COUNT * 8;
  static constexpr int OFF_ABORT = OFF_TMEM + 4;
  static constexpr int OFF_DKVW = OFF_ABORT + 4;
  static constexpr int OFF_RED = OFF_DKVW + 8;  // one float per elementwise warp
  static constexpr int OFF_TKT = OFF_RED + 4 * 4 * NEW;  // deterministic mode: this CTA's work ticket
  static constexpr int END = OFF_TKT + 16;
  static constexpr int SMEM = END + 1024;
  // TMEM. D=64: two S/dP buffers [128b, 128b+128) (S at +0, dP at +64); a warp
  // writes the packed P^T of each 16-query group over the first 8 of that group's S
  // columns (its own columns) once they are in registers, so buffer b is free again once dV of its tile has been issued
  // (MMAs of one thread run in order). dV [256,320) dK [320,384) dQ of a tile pair
  // [384,448).
  // D=128: one S/dP buffer [0,128), P^T x2 [128,192), dV [192,320), dK [320,448),
  // dQ^T [448,512).
  static constexpr int NSB = D == 64 ? 2 : 1;
  static constexpr uint32_t TM_DV = NSB == 2 ? 256 : 192, TM_DK = TM_DV + D, TM_DQ = TM_DK + D;
  static_assert(TM_DQ + 64 * NDQ <= 512, "TMEM budget");
  __device__ static constexpr uint32_t tm_s(int b) { return 128u * (uint32_t)b; }
  __device__ static constexpr uint32_t tm_dp(int b) { return 128u * (uint32_t)b + 64u; }
  // packed P^T columns of queries [16k, 16k+16) of the tile in PDS buffer s
  __device__ static constexpr uint32_t tm_p(int s, int k) {
    return NSB == 2 ? 128u * (uint32_t)s + 16u * (uint32_t)k : 128u + 32u * (uint32_t)s + 8u * (uint32_t)k;
  }
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  // fused FIR: the raw K rows [k0 - FIR_HALO, k0 + BN) are staged in the dS / dQ
  // staging area, unused until the first tile's elementwise work (which follows
  // the filtered K through the S MMA)
  static constexpr int RAWGROUP = (BN + FIR_HALO) * 128;
  static constexpr int OFF_RAW = OFF_DS;
  static_assert((D / 64) * RAWGROUP <= OFF_COEF - OFF_DS, "raw K fits the dS / staging area");
  static_assert(OFF_RAW % 1024 == 0, "swizzle atoms");
};

struct BwdParams {
  CUtensorMap tk, tv, tq, tdo;
  CUtensorMap tkr;    // fused FIR: raw K, BN + FIR_HALO rows per box
  const float* taps;  // fused FIR: fp32[FIR_TAPS], index FIR_TAPS-1 = lag 0
  const float4* coefP;
  const float* tiev;
  const int32_t* argv;
  const float* pcmpv;
  int64_t npad;  // records per head
  const int32_t* live64;
  float* dq_acc;
  void* dk;
  int64_t sdk[4];
  void* dv;
  int64_t sdv[4];
  float* dtau_part;
  const float* tau;
  int32_t* status;
  int H, N, nq64, nkt;
  int dreal;  // the operands' head dim (zero-padded to D by the TMA loads when smaller)
  float scale;
  int causal;
  int stall;  // PNFT_FLASH_TEST_STALL: the elementwise warps first wait on C_STALL
  // PNFT_FLASH_DETERMINISTIC: work items in ticket order; the dQ drain adds each tile
  // into the accumulator after the lower key tiles of its head (turn counters)
  int det;
  int32_t* sem;     // [B*H, nq64]
  int32_t* ticket;  // [1]
  int hgroup;       // heads per group of the CTA order (work_item)
};

// Warp-cooperative walk over the query tiles [i0, n) whose live bit is set: 32
// flags per ballot, the next 32 already loaded (one flag per lane), so moving
// from tile to tile never waits on global memory. All 32 lanes call next().
// Ascending by default; descending (from n-1 down to i0) in deterministic mode,
// where every CTA of a head then reaches a given query tile at about the same
// step, so the key-ordered dQ additions seldom wait.
struct LiveTiles {
  const int32_t* f;
  int n, i0, base;  // ascending: chunk [base, base+32); descending: chunk [base-31, base]
  bool desc;
  uint32_t live, multi;
  int32_t ahead;  // this lane's flag of the next chunk
  __device__ __forceinline__ int32_t flag(int j) const { return j >= i0 && j < n ? f[j] : 0; }
  __device__ __forceinline__ LiveTiles(const int32_t* flags, int i0_, int n_, bool desc_ = false)
      : f(flags), n(n_), i0(i0_), base(desc_ ? n_ - 1 : i0_), desc(desc_) {
    const int lane = threadIdx.x & 31;
    const int32_t cur = flag(desc ? base - lane : base + lane);
    ahead = flag(desc ? base - 32 - lane : base + 32 + lane);
    live = __ballot_sync(0xffffffffu, cur & kLiveRow);
    multi = __ballot_sync(0xffffffffu, cur & kMultiTie);
  }
  // Next live tile, -1 past the end; *is_multi: the tile holds a row with several maxima.
  __device__ __forceinline__ int next(bool* is_multi) {
    while (!live) {
      if (desc ? base - 32 < i0 : base + 32 >= n) return -1;
      base += desc ? -32 : 32;
      live = __ballot_sync(0xffffffffu, ahead & kLiveRow);
      multi = __ballot_sync(0xffffffffu, ahead & kMultiTie);
      const int lane = (int)(threadIdx.x & 31);
      ahead = flag(desc ? base - 32 - lane : base + 32 + lane);
    }
    const int bit = __ffs(live) - 1;
    live &= live - 1;
    *is_multi = (multi >> bit) & 1u;
    return desc ? base - bit : base + bit;
  }
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int D, bool FIR>
__global__ void __launch_bounds__(B_THREADS, 1) flash_bwd_sm100_kernel(const __grid_constant__ BwdParams p) {
  using L = BwdLayout<D>;
  constexpr int DG = D / 64;
  constexpr int NQS = L::NQS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // offset from the __shared__ array itself, so the compiler keeps shared-space accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb0 = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // b*h runs fastest and key tile 0 (the most causal query tiles) comes first:
  // the grid starts with its longest CTAs, so none starts late. Deterministic mode
  // takes the same order from a work ticket, so every CTA whose dQ additions a CTA
  // waits for (the lower key tiles of its head) started before it.
  int kt_, bh_, w = (int)(blockIdx.y * gridDim.x + blockIdx.x);
  if (p.det) {
    volatile int* tk = reinterpret_cast<volatile int*>(smem + L::OFF_TKT);
    if (threadIdx.x == 0) *tk = atomicAdd(p.ticket, 1);
    __syncthreads();
    w = *tk;
  }
  // heads in groups sized to L2 (work_item): in deterministic mode the lower key
  // tiles of a head still come earlier in the order, within its group
  work_item(w, (int)gridDim.x, p.nkt, p.hgroup, &bh_, &kt_);
  const int kt = kt_, bh = bh_, b = bh / p.H, hd = bh % p.H;
  const int k0 = kt * BN;
  const int i_first = p.causal ? k0 / BM : 0;
  const int32_t* live = p.live64 + (int64_t)bh * p.nq64;
  auto bar = [&](int i) -> uint32_t { return sb0 + L::OFF_BAR + 8u * (uint32_t)i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_ABORT);
  volatile int* dkv_written = reinterpret_cast<volatile int*>(smem + L::OFF_DKVW);
  const Abort ab{abort_flag, p.status};
  const uint32_t sK = sb0 + L::OFF_K, sV = sb0 + L::OFF_V;
  auto sQ = [&](int s) -> uint32_t { return sb0 + L::OFF_Q + (uint32_t)s * L::QBYTES; };
  auto sdO = [&](int s) -> uint32_t { return sb0 + L::OFF_DO + (uint32_t)s * L::QBYTES; };
  auto sdS = [&](int s) -> uint32_t { return sb0 + L::OFF_DS + (uint32_t)s * L::DS_BYTES; };

  if (threadIdx.x == 0) {
    mbar_init(bar(C_KV), FIR ? 2 : 1);  // fused FIR: + one arrive once K~ is written
    mbar_init(bar(C_KRAW), 1);
    mbar_init(bar(C_SDPFULL), 1);
    mbar_init(bar(C_SDPFULL + 1), 1);
    mbar_init(bar(C_SDPEMPTY), 4 * NEW);
    for (int i = 0; i < NQS; ++i) {
      mbar_init(bar(C_QDFULL + i), 1);
      mbar_init(bar(C_QDEMPTY + i), 1);
    }
    for (int i = 0; i < L::NDS; ++i) mbar_init(bar(C_PDSEMPTY + i), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(C_PDSFULL + i), 4 * NEW);
      mbar_init(bar(C_DQFULL + i), 1);
      mbar_init(bar(C_DQEMPTY + i), 4);
    }
    mbar_init(bar(C_DKV), 1);
    mbar_init(bar(C_FLAG), 1);
    mbar_init(bar(C_STALL), 1);
    *abort_flag = 0;
    *dkv_written = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(FIR ? &p.tkr : &p.tk);
    prefetch_tmap(&p.tv);
    prefetch_tmap(&p.tq);
    prefetch_tmap(&p.tdo);
  }
  if (warp == 1) {
    tmem_alloc(sb0 + L::OFF_TMEM, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L::OFF_TMEM);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (converged warp, lane 0 issues)
    if (lane == 0) {
      if constexpr (FIR) {
        // raw K with its causal halo for the elementwise warps to filter into sK
        mbar_arrive_expect_tx(bar(C_KRAW), DG * L::RAWGROUP);
        for (int g = 0; g < DG; ++g)
          tma_load_4d(sb0 + L::OFF_RAW + g * L::RAWGROUP, &p.tkr, bar(C_KRAW), 64 * g, k0 - FIR_HALO, hd, b);
        mbar_arrive_expect_tx(bar(C_KV), L::KBYTES);
        for (int g = 0; g < DG; ++g) tma_load_4d(sV + g * L::KGROUP, &p.tv, bar(C_KV), 64 * g, k0, hd, b);
      } else {
        mbar_arrive_expect_tx(bar(C_KV), 2 * L::KBYTES);
        for (int g = 0; g < DG; ++g) {
          tma_load_4d(sK + g * L::KGROUP, &p.tk, bar(C_KV), 64 * g, k0, hd, b);
          tma_load_4d(sV + g * L::KGROUP, &p.tv, bar(C_KV), 64 * g, k0, hd, b);
        }
      }
    }
    __syncwarp();
    LiveTiles lt(live, i_first, p.nq64, p.det != 0);
    int t = 0;
    bool ok = true, mt;
    for (int i; ok && (i = lt.next(&mt)) >= 0;) {
      const int s = t % NQS;
      if (!(ok = warp_wait(bar(C_QDEMPTY + s), ((t / NQS) & 1) ^ 1, ab))) break;
      if (lane == 0) {
        const int q0 = i * BM;
        const uint32_t full = bar(C_QDFULL + s);
        mbar_arrive_expect_tx(full, 2 * L::QBYTES + L::COEF_BYTES);
        for (int g = 0; g < DG; ++g) {
          tma_load_4d(sQ(s) + g * L::QGROUP, &p.tq, full, 64 * g, q0, hd, b);
          tma_load_4d(sdO(s) + g * L::QGROUP, &p.tdo, full, 64 * g, q0, hd, b);
        }
        // 64 records always: each head's records are padded to whole 64-row tiles
        const int64_t rec = (int64_t)bh * p.npad + q0;
        const uint32_t cb = sb0 + L::OFF_COEF + s * L::COEF_BYTES;
        bulk_load(cb + L::CF_P, p.coefP + rec / 2, BM * 8, full);
        bulk_load(cb + L::CF_TIE, p.tiev + rec, BM * 4, full);
        bulk_load(cb + L::CF_ARG, p.argv + rec, BM * 4, full);
        bulk_load(cb + L::CF_PC, p.pcmpv + rec, BM * 4, full);
      }
      __syncwarp();
      ++t;
    }
    if (lane == 0) {
      drain_wait(bar(C_KV), 0);
      if (FIR) drain_wait(bar(C_KRAW), 0);
      for (int u = t - 1; u >= 0 && u > t - 1 - NQS; --u) drain_wait(bar(C_QDFULL + u % NQS), (u / NQS) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (converged warp)
    constexpr uint32_t ID_S = idesc_f16(BN, BM, 1, 0, 0);   // S^T, dP^T: K-major A and B
    constexpr uint32_t ID_G = idesc_f16(BN, D, 1, 0, 1);    // dV (A in TMEM), dK (A K-major); B MN-major
    constexpr uint32_t ID_DQ = idesc_f16(D, BM, 1, 1, 1);   // dQ^T: M = head dims
    // dQ of a tile pair, not transposed: M = the pair's 128 queries (A = dS, queries
    // contiguous in the dS^T tiles), N = head dims (B = K, head dims contiguous)
    constexpr uint32_t ID_DQ2 = idesc_f16(2 * BM, D, 1, 1, 1);
    // Descriptors of k-step 0; a k-step moves +32 B inside a 128-byte K-major row
    // (+2 in descriptor units, +GROUP bytes across 64-column groups) or +16 rows
    // (2048 B, +128) of an MN-major tile.
    const uint32_t dKk = sw128_desc(sK, 16), dVk = sw128_desc(sV, 16);
    const uint32_t dKmn = sw128_desc(sK, L::KGROUP);
    const uint32_t dQk = sw128_desc(sQ(0), 16), dOk = sw128_desc(sdO(0), 16);
    const uint32_t dQmn = sw128_desc(sQ(0), L::QGROUP), dOmn = sw128_desc(sdO(0), L::QGROUP);
    const uint32_t dSk = sw128_desc(sdS(0), 16), dSmn = sw128_desc(sdS(0), L::KGROUP);
    constexpr uint32_t QSTEP = L::QBYTES >> 4, DSSTEP = L::DS_BYTES >> 4;
    auto kmaj = [](int kk, int group) -> uint32_t { return (uint32_t)(((kk >> 2) * group + (kk & 3) * 32) >> 4); };
    constexpr int NSB = L::NSB;
    auto issue_sdp = [&](int t) -> bool {
      const int qs = t % NQS, sb = t % NSB;
      if (!warp_wait(bar(C_QDFULL + qs), (t / NQS) & 1, ab)) return false;
      if (NSB == 1 && !warp_wait(bar(C_SDPEMPTY), (t & 1) ^ 1, ab)) return false;
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tmem + L::tm_s(sb), dKk + kmaj(kk, L::KGROUP), dQk + qs * QSTEP + kmaj(kk, L::QGROUP), ID_S, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(tmem + L::tm_dp(sb), dVk + kmaj(kk, L::KGROUP), dOk + qs * QSTEP + kmaj(kk, L::QGROUP), ID_S, kk > 0);
        mma_commit(bar(C_SDPFULL + sb));
      }
      __syncwarp();
      return true;
    };
    auto dvdk = [&](int u) -> bool {
      const int s = u & 1, qs = u % NQS, ds = u % L::NDS;
      if (!warp_wait(bar(C_PDSFULL + s), (u >> 1) & 1, ab)) return false;
      tc_fence_after();
      const uint32_t acc0 = u > 0 ? 1u : 0u;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          mma_ts(tmem + L::TM_DV, tmem + L::tm_p(s, kk), dOmn + qs * QSTEP + kk * 128, ID_G, acc0 | (uint32_t)kk);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          mma_ss(tmem + L::TM_DK, dSk + ds * DSSTEP + kk * 2, dQmn + qs * QSTEP + kk * 128, ID_G, acc0 | (uint32_t)kk);
        mma_commit(bar(C_QDEMPTY + qs));  // Q / dO of tile u are no longer needed
      }
      __syncwarp();
      return true;
    };
    // dQ of tiles u and u+1 (u even; `two` false for a last tile alone, whose partner
    // rows the drain ignores): the dS tiles u % NDS and u % NDS + 1 are adjacent, one
    // 64-query atom apart, so the MN-major descriptor of tile u spans both (its atom
    // stride is the dS tile size). TMEM lane = query of the pair, column = head dim.
    auto dq_pair = [&](int u, bool two) -> bool {
      const int ds = u % L::NDS;
      if (!warp_wait(bar(C_DQEMPTY), ((u >> 1) & 1) ^ 1, ab)) return false;
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ss(tmem + L::TM_DQ, dSmn + ds * DSSTEP + kk * 128, dKmn + kk * 128, ID_DQ2, kk > 0);
        mma_commit(bar(C_DQFULL));
        mma_commit(bar(C_PDSEMPTY + ds));
        if (two) mma_commit(bar(C_PDSEMPTY + ds + 1));
      }
      __syncwarp();
      return true;
    };
    static_assert(!L::DQ_PAIR || (L::NDS % 2 == 0 && L::DS_BYTES == L::KGROUP), "tile pairs in adjacent dS tiles");
    auto dq = [&](int u) -> bool {
      const int ds = u % L::NDS, bq = u % L::NDQ;
      if (!warp_wait(bar(C_DQEMPTY + bq), ((u / L::NDQ) & 1) ^ 1, ab)) return false;
      tc_fence_after();
      if (elect_one()) {
        // dQ^T[D x 64 q] = K^T[D x keys] dS^T[keys x q]: both operands MN-major in smem
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_ss(tmem + L::TM_DQ + 64u * bq, dKmn + kk * 128, dSmn + ds * DSSTEP + kk * 128, ID_DQ, kk > 0);
        mma_commit(bar(C_DQFULL + bq));
        mma_commit(bar(C_PDSEMPTY + ds));  // dS_u (and, for d=128, P^T_u) are free
      }
      __syncwarp();
      return true;
    };
    int t = 0;  // tiles whose S / dP are issued
    bool ok = warp_wait(bar(C_KV), 0, ab), mt;
    LiveTiles lt(live, i_first, p.nq64, p.det != 0);
    if constexpr (NSB == 2) {
      // S/dP run two tiles ahead: per step j, dV/dK of tile j, then S/dP of tile
      // j+2 (into tile j's buffer, behind dV(j) in the MMA pipe), then dQ of tile j.
      int T = 0;  // live tiles known so far
      bool more = true;
      auto discover = [&]() { if (more && lt.next(&mt) >= 0) ++T; else more = false; };
      discover();
      discover();
      for (int u = 0; ok && u < T && u < 2; ++u) {
        ok = issue_sdp(u);
        t = u + 1;
      }
      for (int j = 0; ok && j < T; ++j) {
        if (!(ok = dvdk(j))) break;
        discover();
        if (j + 2 < T) {
          if (!(ok = issue_sdp(j + 2))) break;
          t = j + 3;
        }
        if constexpr (L::DQ_PAIR) {
          if ((j & 1) && !(ok = dq_pair(j - 1, true))) break;
        } else {
          if (!(ok = dq(j))) break;
        }
      }
      if constexpr (L::DQ_PAIR) {
        if (ok && (T & 1)) ok = dq_pair(T - 1, false);
      }
    } else {
      // one S/dP buffer: S/dP of tile j once every warp has read tile j-1's, then
      // dV, dK, dQ of tile j-1
      for (int i; ok && (i = lt.next(&mt)) >= 0;) {
        if (!(ok = issue_sdp(t))) break;
        if (t >= 1 && !(ok = dvdk(t - 1))) break;
        if (t >= 1 && !(ok = dq(t - 1))) break;
        ++t;
      }
      if (ok && t >= 1) ok = dvdk(t - 1) && dq(t - 1);
    }
    if (elect_one()) {  // the same lane as every issue above: a commit tracks its own thread's MMAs
      *dkv_written = (ok && t >= 1) ? 1 : 0;
      mbar_arrive(bar(C_FLAG));
      mma_commit(bar(C_DKV));
      drain_wait(bar(C_DKV), 0);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < W_DRAIN) {
    // ------------------------------------------------------------ elementwise
    const int ew = warp - 4, hh = ew >> 2, wq = warp & 3;
    const int rl = 32 * wq + lane;
    const int key = k0 + rl, kb = k0 + 32 * wq;  // this thread's key, the warp's first key
    const uint32_t lane_off = (uint32_t)(32 * wq) << 16;
    const float tau = __ldg(p.tau);
    // s = S*scale - tau rounded once; relu(s) is bit-identical to the forward's u
    const float2 sc2 = make_float2(p.scale, p.scale), nt2 = make_float2(-tau, -tau);
    const int lim = key < p.N ? (p.causal ? key : 0) : 0x7fffffff;  // first valid query of this key
    float2 ds_sum = make_float2(0.f, 0.f);
    bool dead = false;
    if constexpr (FIR) {
      // K~ = causal_fir(K) into sK: thread -> (column pair, group, block of rows)
      constexpr int NB = 128 * NEW / (32 * DG), NR = BN / NB;
      const int et = threadIdx.x - 128, cp = et & 31, g = (et >> 5) % DG, rb = (et >> 5) / DG;
      float2 h[FIR_TAPS];
      fir_load_taps(p.taps, h);
      if (!dead) dead = !warp_wait(bar(C_KRAW), 0, ab);
      if (!dead) fir_filter_rows<NR>(smem + L::OFF_RAW + g * L::RAWGROUP, smem + L::OFF_K + g * L::KGROUP, cp, rb * NR, h);
      fence_proxy_async_smem();  // the tensor core reads K through the async proxy
      named_bar_sync(3, 128 * NEW);
      if (et == 0) mbar_arrive(bar(C_KV));
    }
    int t = 0;
    LiveTiles lt(live, i_first, p.nq64, p.det != 0);
    bool multi_tile;
    for (int i; (i = lt.next(&multi_tile)) >= 0;) {
      const int s = t & 1, qs = t % NQS, ds = t % L::NDS;
      const int q0 = i * BM;
      // S/dP of this tile, its coefficient records, and a free dS buffer (d=128:
      // also a free P^T buffer; d=64 writes P^T over its own S columns)
      const int sb = t % L::NSB;
      // test-only (p.stall): the first tile waits on C_STALL, which nothing
      // completes, so the warps run the wait out and unwind like any timeout
      if (!dead)
        dead = !warp_wait3(t == 0 && p.stall ? bar(C_STALL) : bar(C_SDPFULL + sb), (t / L::NSB) & 1,
                           bar(C_QDFULL + qs), (t / NQS) & 1, bar(C_PDSEMPTY + ds), ((t / L::NDS) & 1) ^ 1, ab);
      uint32_t rs[CW], rp[CW];
      if (!dead) {
        tc_fence_after();
        if constexpr (CW == 32)
          tmem_load32x2(tmem + lane_off + L::tm_s(sb) + (uint32_t)(CW * hh), rs,
                        tmem + lane_off + L::tm_dp(sb) + (uint32_t)(CW * hh), rp);
        else
          tmem_load16x2(tmem + lane_off + L::tm_s(sb) + (uint32_t)(CW * hh), rs,
                        tmem + lane_off + L::tm_dp(sb) + (uint32_t)(CW * hh), rp);
        if constexpr (L::NSB == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C_SDPEMPTY));
        }
        const uint8_t* cfb = smem + L::OFF_COEF + qs * L::COEF_BYTES;
        const float4* cp4 = reinterpret_cast<const float4*>(cfb + L::CF_P) + (CW / 2) * hh;  // this warp's pairs
        const float* tiew = reinterpret_cast<const float*>(cfb + L::CF_TIE) + CW * hh;
        const int* argw = reinterpret_cast<const int*>(cfb + L::CF_ARG) + CW * hh;
        const float* pcw = reinterpret_cast<const float*>(cfb + L::CF_PC) + CW * hh;
        const int qb = q0 + CW * hh;  // first query of this warp's columns
        // This warp's CW columns. MASK: zero u past the diagonal / the sequence
        // ends. MULTI: per-element gate-gradient test (value ties); otherwise the
        // single argmax entry of each row is patched in afterwards.
        auto slice = [&](auto mask_c, auto multi_c) {
          constexpr bool MASK = decltype(mask_c)::value, MULTI = decltype(multi_c)::value;
          uint32_t pw_pk[CW / 2], ds_pk[CW / 2];
#pragma unroll
          for (int c2 = 0; c2 < CW / 2; ++c2) {
            const int c = 2 * c2;
            const float4 cf = cp4[c2];  // c1 pair, -D pair
            float2 x = __ffma2_rn(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sc2, nt2);
            if constexpr (MASK) {
              const int q = qb + c;
              if (!(q >= lim && q < p.N)) x.x = -1.f;
              if (!(q + 1 >= lim && q + 1 < p.N)) x.y = -1.f;
            }
            const float2 u = make_float2(fmaxf(x.x, 0.f), fmaxf(x.y, 0.f));
            const float2 u2 = __fmul2_rn(u, u), u4 = __fmul2_rn(u2, u2), u8 = __fmul2_rn(u4, u4);
            const float2 g = __fmul2_rn(__fmul2_rn(u8, u), make_float2(cf.x, cf.y));  // c1 u^9
            const float2 w = __fmul2_rn(g, u);                                        // c1 u^10
            const float2 dp = make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1]));
            float2 ds = __fmul2_rn(g, __fadd2_rn(dp, make_float2(cf.z, cf.w)));
            if constexpr (MULTI) {
              if (u.x > 0.f && (key == argw[c] || u.x == pcw[c])) ds.x += tiew[c];
              if (u.y > 0.f && (key == argw[c + 1] || u.y == pcw[c + 1])) ds.y += tiew[c + 1];
            }
            ds_sum = __fadd2_rn(ds_sum, ds);
            pw_pk[c2] = pack_bf16x2(w.x, w.y);
            ds_pk[c2] = pack_bf16x2(ds.x, ds.y);
          }
#pragma unroll
          for (int k = 0; k < CW / 16; ++k)
            tmem_st8(tmem + lane_off + L::tm_p(s, (CW / 16) * hh + k), *reinterpret_cast<const uint32_t(*)[8]>(pw_pk + 8 * k));
#pragma unroll
          for (int cc = 0; cc < CW / 8; ++cc) {
            const uint32_t chunk = (CW / 8) * hh + cc;  // 16-byte chunk of the 128-byte key row
            st_shared_v4(sdS(ds) + rl * 128 + ((chunk ^ (rl & 7)) << 4), ds_pk[4 * cc], ds_pk[4 * cc + 1],
                         ds_pk[4 * cc + 2], ds_pk[4 * cc + 3]);
          }
        };
        static_assert(CW == 16 || CW == 32, "16 or 32 query columns per warp");
        using T_ = std::true_type;
        using F_ = std::false_type;
        const bool edge = (p.causal && qb < kb + 31) || qb + CW > p.N || kb + 32 > p.N;
        if (multi_tile) {
          slice(T_{}, T_{});
        } else {
          if (edge) slice(T_{}, F_{});
          else slice(F_{}, F_{});
          // Gate gradient of the rows whose argmax key is one of this warp's keys:
          // lane c < CW patches column c's entry (key row arg - k0) of the bf16 dS tile.
          __syncwarp();
          const int col = CW * hh + lane;
          const int l = lane < CW ? argw[lane] - kb : -1;
          if ((unsigned)l < 32u) {
            const float tie = tiew[lane];
            const int r = 32 * wq + l;
            const uint32_t addr = sdS(ds) + r * 128 + ((((uint32_t)col >> 3) ^ (r & 7)) << 4) + (col & 7) * 2;
            unsigned short hv;
            asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hv) : "r"(addr) : "memory");
            const float nv = __bfloat162float(__ushort_as_bfloat16(hv)) + tie;
            hv = __bfloat16_as_ushort(__float2bfloat16_rn(nv));
            asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(hv) : "memory");
            ds_sum.x += tie;
          }
        }
        tmem_wait_st();
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C_PDSFULL + s));
      ++t;
    }
    // ---- dK, dV: rows of this CTA's keys, warpgroup g writes head dims [g*D/NEW, (g+1)*D/NEW)
    const bool ok = warp_wait(bar(C_DKV), 0, ab) && warp_wait(bar(C_FLAG), 0, ab);
    tc_fence_after();
    const bool have = ok && *dkv_written != 0;
    const float dk_scale = 10.f * p.scale;  // dS' -> dS
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      __nv_bfloat16* G = static_cast<__nv_bfloat16*>(m == 0 ? p.dv : p.dk);
      const int64_t* sg = m == 0 ? p.sdv : p.sdk;
      const uint32_t tcol = m == 0 ? L::TM_DV : L::TM_DK;
      const float f = m == 0 ? 1.f : dk_scale;
      __nv_bfloat16* row = G + (int64_t)b * sg[0] + (int64_t)hd * sg[1] + (int64_t)key * sg[2];
#pragma unroll
      for (int cb = 0; cb < D / NEW; cb += 16) {
        const int d0 = hh * (D / NEW) + cb;
        if (d0 >= p.dreal) break;  // zero-padded head dims: never stored (warp-uniform)
        uint32_t r[16];
        if (have) {
          tmem_load16(tmem + lane_off + tcol + (uint32_t)d0, r);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) r[e] = 0u;
        }
        if (key < p.N && ok) {
          if (sg[3] == 1 && (reinterpret_cast<uintptr_t>(row + d0) & 15) == 0) {
#pragma unroll
            for (int v = 0; v < 2; ++v) {
              uint4 w;
              w.x = pack_bf16x2(f * __uint_as_float(r[8 * v + 0]), f * __uint_as_float(r[8 * v + 1]));
              w.y = pack_bf16x2(f * __uint_as_float(r[8 * v + 2]), f * __uint_as_float(r[8 * v + 3]));
              w.z = pack_bf16x2(f * __uint_as_float(r[8 * v + 4]), f * __uint_as_float(r[8 * v + 5]));
              w.w = pack_bf16x2(f * __uint_as_float(r[8 * v + 6]), f * __uint_as_float(r[8 * v + 7]));
              *reinterpret_cast<uint4*>(row + d0 + 8 * v) = w;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              row[(int64_t)(d0 + e) * sg[3]] = __float2bfloat16_rn(f * __uint_as_float(r[e]));
          }
        }
      }
    }
    // ---- tau gradient partial of this CTA (fixed reduction order): -sum dS / scale = -10 sum dS'
    float v = ds_sum.x + ds_sum.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
    if (lane == 0) red[ew] = v;
    named_bar_sync(3, 128 * NEW);
    if (ew == 0 && lane == 0) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < 4 * NEW; ++w) tot += red[w];
      p.dtau_part[(int64_t)bh * p.nkt + kt] = -10.f * tot;
    }
  } else if (warp >= W_DRAIN) {
    // ------------------------------------------------------------ dQ drain
    const int wq = warp & 3;
    const uint32_t lane_off = (uint32_t)(32 * wq) << 16;
    const bool leader = warp == W_DRAIN && lane == 0;
    bool dead = false;
    // deterministic mode: add the staged fp32 tiles of query tiles ia and (if ib >= 0)
    // ib (rows of 64 x D, the accumulator's own layout) once the lower key tiles of
    // this head have added theirs, then pass both turns on; all 128 drain threads.
    // Both tiles' turns are awaited together and all their loads issued before the
    // first add, so a pair costs one turn wait and one L2 round trip.
    const int dt = threadIdx.x - 32 * W_DRAIN;
    auto ordered_add = [&](int ia, const float* stga, int ib, const float* stgb) {
      int32_t* sema = p.sem + (int64_t)bh * p.nq64 + ia;
      int32_t* semb = ib >= 0 ? p.sem + (int64_t)bh * p.nq64 + ib : nullptr;
      if (leader) {
        turn_wait(sema, kt, p.status, abort_flag);
        if (semb) turn_wait(semb, kt, p.status, abort_flag);
      }
      named_bar_sync(4, 128);
      if (!dead) {
        // loads of up to 8 float4 per thread (both tiles of a pair at d = 64, half a
        // tile at d = 128) issued before their adds
        constexpr int PER = BM * D / 4 / 128;   // float4 per drain thread and tile
        constexpr int NT = L::DQ_PAIR ? 2 : 1;  // tiles per drain step
        constexpr int CH = PER * NT > 8 ? 8 : PER * NT;
        auto addr = [&](int c, int* e, int* t) {  // c-th float4 of this thread -> tile, element
          *t = c / PER;
          *e = dt + 128 * (c % PER);
        };
#pragma unroll
        for (int c0 = 0; c0 < PER * NT; c0 += CH) {
          float4 a[CH];
#pragma unroll
          for (int k = 0; k < CH; ++k) {
            int e, t;
            addr(c0 + k, &e, &t);
            const int i = t == 0 ? ia : ib;
            if (i >= 0 && e < min(BM, p.N - i * BM) * (D / 4))
              a[k] = __ldcg(reinterpret_cast<const float4*>(p.dq_acc + ((int64_t)bh * p.N + (int64_t)i * BM) * D) + e);
          }
#pragma unroll
          for (int k = 0; k < CH; ++k) {
            int e, t;
            addr(c0 + k, &e, &t);
            const int i = t == 0 ? ia : ib;
            if (i >= 0 && e < min(BM, p.N - i * BM) * (D / 4)) {
              const float4 b4 = reinterpret_cast<const float4*>(t == 0 ? stga : stgb)[e];
              a[k].x += b4.x;
              a[k].y += b4.y;
              a[k].z += b4.z;
              a[k].w += b4.w;
              __stcg(reinterpret_cast<float4*>(p.dq_acc + ((int64_t)bh * p.N + (int64_t)i * BM) * D) + e, a[k]);
            }
          }
        }
      }
      named_bar_sync(4, 128);
      if (leader) {
        turn_pass(sema);
        if (semb) turn_pass(semb);
      }
    };
    LiveTiles lt(live, i_first, p.nq64, p.det != 0);
    bool mt;
    if constexpr (L::DQ_PAIR) {
      // tile pairs: TMEM lane = query of the pair (quadrants 0-1: tile A, 2-3: tile
      // B), columns = head dims; each thread stores its query's row of 64 head dims
      // as 16 chunks of 16 bytes into the row-major staging tile (chunks swizzled by
      // acc_chunk, the accumulator's own order)
      static_assert(L::NSTG == 2 && D == 64, "one staging tile per tile of a pair, rows of 64 head dims");
      const int tsel = wq >> 1, ql = 32 * (wq & 1) + lane;  // tile of the pair, row in that tile
      for (int pr = 0;; ++pr) {
        const int ia = lt.next(&mt);
        if (ia < 0) break;
        const int ib = lt.next(&mt);  // -1: tile A is the last one
        const bool two = ib >= 0;
        if (!dead) dead = !warp_wait(bar(C_DQFULL), pr & 1, ab);
        if (leader) bulk_wait_read<0>();  // the previous pair's reduces have read both staging tiles
        named_bar_sync(4, 128);
        if (!dead) tc_fence_after();
        float* stg = reinterpret_cast<float*>(smem + L::OFF_STG + tsel * L::STG_BYTES);  // [64 q][D]
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // head dims [32h, 32h + 32)
          uint32_t r[32];
          if (!dead) tmem_load32(tmem + lane_off + L::TM_DQ + 32u * h, r);
          if (!dead && (tsel == 0 || two)) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              reinterpret_cast<float4*>(stg + ql * D)[acc_chunk(8 * h + v, ql)] =
                  make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]), __uint_as_float(r[4 * v + 2]),
                              __uint_as_float(r[4 * v + 3]));
          }
        }
        if (!dead) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C_DQEMPTY));
        }
        fence_proxy_async_smem();
        named_bar_sync(4, 128);
        if (p.det) {
          ordered_add(ia, reinterpret_cast<const float*>(smem + L::OFF_STG), two ? ib : -1,
                      reinterpret_cast<const float*>(smem + L::OFF_STG + L::STG_BYTES));
        } else if (leader && !dead) {
          const int qa = ia * BM;
          bulk_reduce_add_f32(p.dq_acc + ((int64_t)bh * p.N + qa) * D, smem_u32(smem + L::OFF_STG),
                              (uint32_t)(min(BM, p.N - qa) * D * 4));
          if (two) {
            const int qb2 = ib * BM;
            bulk_reduce_add_f32(p.dq_acc + ((int64_t)bh * p.N + qb2) * D, smem_u32(smem + L::OFF_STG + L::STG_BYTES),
                                (uint32_t)(min(BM, p.N - qb2) * D * 4));
          }
          bulk_commit();
        }
      }
    } else {
    int t = 0;
    for (int i; (i = lt.next(&mt)) >= 0;) {
      const int bq = t % L::NDQ, sg = t % L::NSTG;
      const int q0 = i * BM;
      if (!dead) dead = !warp_wait(bar(C_DQFULL + bq), (t / L::NDQ) & 1, ab);
      if (leader) bulk_wait_read<L::NSTG - 1>();  // the staging tile's previous reduce has read it
      named_bar_sync(4, 128);
      float* stg = reinterpret_cast<float*>(smem + L::OFF_STG + sg * L::STG_BYTES);  // [64 q][D] fp32
      // dQ^T accumulator, columns = the 64 queries. D=128 (M=128): head dim d in
      // lane d. D=64 (M=64 layout): head dim 16*wq + l in lane l < 16 of quadrant wq.
      const bool holds = D == 128 || lane < 16;
      const int d = D == 128 ? 32 * wq + lane : 16 * wq + lane;
      if (!dead) tc_fence_after();
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {  // 32 query columns at a time
        uint32_t r[32];
        if (!dead) {
          tmem_load32(tmem + lane_off + L::TM_DQ + 64u * bq + 32u * h2, r);
        }
        if (h2 == 1 && !dead) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C_DQEMPTY + bq));
        }
        if (holds && !dead) {
#pragma unroll
          for (int q = 0; q < 32; ++q) stg[(32 * h2 + q) * D + d] = __uint_as_float(r[q]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(4, 128);
      if (p.det) {
        ordered_add(i, stg, -1, nullptr);
      } else if (leader && !dead) {
        const int rows = min(BM, p.N - q0);
        bulk_reduce_add_f32(p.dq_acc + ((int64_t)bh * p.N + q0) * D, smem_u32(stg), (uint32_t)(rows * D * 4));
        bulk_commit();
      }
      ++t;
    }
    }
    if (leader) bulk_wait_all();
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int flash_bwd_sm100(const FlashArgs& a0, cudaStream_t st) {
  if (!tma_ok_bhnd(a0.dout, a0.sdo))
    return fail(PNFT_EINVAL,
                "flash bwd: dout needs unit head-dim stride and 16-byte aligned rows when q/k/v take the sm100 path");
  FlashArgs a = a0;
  const int nkt = (int)((a.N + BN - 1) / BN);
  a.n_dtau_part = a.B * a.H * nkt;
  a.dq_scale = 10.f * a.scale;  // the kernel accumulates dS' = dS / (10 scale) into dQ
  a.acc_swz = a.D <= 64 ? 1 : 0;  // d = 64 kernel: tile-pair dQ rows stored in acc_chunk order
  int rc = flash_bwd_prep(a, st);
  if (rc) return rc;
  BwdParams p;
  memset(&p, 0, sizeof(p));
  if (a.fir_taps) {
    if (a.fir_ntaps != FIR_TAPS) return fail(PNFT_EUNSUPPORTED, "flash bwd sm100: fused FIR needs %d taps", FIR_TAPS);
    rc = tma_map_bhnd(&p.tkr, a.k, a.sk, a.B, a.H, a.N, a.D, BN + FIR_HALO);
    p.taps = a.fir_taps;
  } else {
    rc = tma_map_bhnd(&p.tk, a.k, a.sk, a.B, a.H, a.N, a.D, BN);
  }
  if (!rc) rc = tma_map_bhnd(&p.tv, a.v, a.sv, a.B, a.H, a.N, a.D, BN);
  if (!rc) rc = tma_map_bhnd(&p.tq, a.q, a.sq, a.B, a.H, a.N, a.D, BM);
  if (!rc) rc = tma_map_bhnd(&p.tdo, a.dout, a.sdo, a.B, a.H, a.N, a.D, BM);
  if (rc) return rc;
  p.coefP = a.coefP;
  p.tiev = a.tiev;
  p.argv = a.argv;
  p.pcmpv = a.pcmpv;
  p.npad = rec_rows(a.N);
  p.live64 = a.live64;
  p.dq_acc = a.dq_acc;
  p.dk = a.dk;
  p.dv = a.dv;
  for (int i = 0; i < 4; ++i) {
    p.sdk[i] = a.sdk[i];
    p.sdv[i] = a.sdv[i];
  }
  p.dtau_part = a.dtau_part;
  p.tau = a.tau;
  p.status = a.status;
  p.H = (int)a.H;
  p.N = (int)a.N;
  p.dreal = (int)a.D;
  p.nq64 = (int)((a.N + BM - 1) / BM);
  p.nkt = nkt;
  p.scale = a.scale;
  p.causal = a.causal;
  p.stall = (a.flags & PNFT_FLASH_TEST_STALL) ? 1 : 0;
  p.det = (a.flags & PNFT_FLASH_DETERMINISTIC) ? 1 : 0;
  // Q, dO (bf16) and the fp32 dQ accumulator of a head, re-read by its key tiles
  p.hgroup = head_group(a.B * a.H, a.N * a.D * 8);
  p.sem = a.dq_sem;
  p.ticket = a.dq_ticket;
  if (nkt > 65535) return fail(PNFT_EUNSUPPORTED, "flash bwd sm100: N = %lld needs more than 65535 key tiles", (long long)a.N);
  const dim3 grid((unsigned)(a.B * a.H), (unsigned)nkt);
  auto launch = [&](auto kern, int smem) -> int {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return check_launch("flash bwd sm100: smem attribute", 0);
    kern<<<grid, B_THREADS, smem, st>>>(p);
    return check_launch("flash bwd sm100");
  };
  if (a.fir_taps)
    rc = a.D <= 64 ? launch(flash_bwd_sm100_kernel<64, true>, BwdLayout<64>::SMEM)
                   : launch(flash_bwd_sm100_kernel<128, true>, BwdLayout<128>::SMEM);
  else
    rc = a.D <= 64 ? launch(flash_bwd_sm100_kernel<64, false>, BwdLayout<64>::SMEM)
                   : launch(flash_bwd_sm100_kernel<128, false>, BwdLayout<128>::SMEM);
  if (rc) return rc;
  return flash_bwd_finish(a, st);
}

}  // namespace pnft
