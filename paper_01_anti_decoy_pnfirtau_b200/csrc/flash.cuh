// Argument bundle and internal entry points of the flash pn_fir_tau kernels.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace pnft {

struct FlashArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* out_c;  // bwd: forward output
  const void* dout;
  void* out;          // fwd: output
  float* out32;       // optional fp32 [B,H,N,D] contiguous copy of the output
  void* dq;
  void* dk;
  void* dv;
  int64_t sq[4], sk[4], sv[4], so[4], sdo[4], sdq[4], sdk[4], sdv[4];
  const float* tau;
  float* stat_m;
  float* stat_z;
  int32_t* stat_nmax;
  int32_t* stat_arg;   // first key index attaining the row peak (-1: silent row)
  float* dtau;
  int32_t* status;
  uint8_t* tile_flags;  // optional [B*H, nT64, nT64] live-tile record
  // fused FIR (sm100 kernels only): k is the raw K and the kernels filter each K
  // tile with these causal taps (fp32[fir_ntaps], index fir_ntaps-1 = lag 0)
  const float* fir_taps;
  int fir_ntaps;
  int64_t B, H, N, D;
  float scale, gamma;
  int has_gamma, causal, dtype, flags;
  // bwd workspace carve-up
  float* dq_acc;       // fp32 [B,H,N,acc_d] contiguous
  int64_t acc_d;       // row stride of dq_acc: acc_width(D)
  int acc_swz;         // rows of dq_acc hold their 16-byte chunks in acc_chunk order (the d=64 tcgen05 backward)
  // per-row backward coefficients (see below): record of row n of head bh at
  // r = bh * rec_rows(N) + n; the padding rows past N hold silent-row records
  float4* coefP;       // rows 2j, 2j+1 interleaved: {c1_0, c1_1, -D_0, -D_1}
  float* tiev;         // tie / 10 (the gate term in units of 10*scale)
  int32_t* argv;       // argmax key (-1: silent row)
  float* pcmpv;        // peak for the value test (NaN when Nmax == 1)
  int32_t* live64;     // [B*H, ceil(N/64)]: bit 0 any row live (peak > 0), bit 1 any row with Nmax > 1
  float* dtau_part;    // per (bh, key tile) partial of -sum du
  int64_t n_dtau_part;
  // deterministic mode (PNFT_FLASH_DETERMINISTIC): per (bh, 64-row query tile) turn
  // counters of the dQ accumulator and the work-ticket counter, zeroed by the prep kernel
  int32_t* dq_sem;     // [B*H, ceil(N/64)]
  int32_t* dq_ticket;  // [1]
  float dq_scale;      // factor the dQ cast applies to the fp32 accumulator
};

// Per query row backward coefficients (c1 = gate/z, D = <dO,O>/gate,
// tie = scale * D * gamma/(peak+gamma)^2 / Nmax, pcmp = peak when Nmax > 1
// else NaN):
//   W  = c1 * u^10                  (the normalised, gated weight: P)
//   dS = 10*scale*c1 * u^9 * (dP - D) + [key == argmax || u == pcmp] * tie
// The records hold c1, -D and tie/10 (the tcgen05 kernel works with
// dS' = dS / (10*scale)). A row with one maximum takes the gate gradient at its
// recorded argmax (exact whatever arithmetic recomputes S); genuine ties
// (Nmax > 1) are found by value and split evenly, like the eager amax
// backward. A silent row has argmax -1 and all-zero coefficients.
constexpr int kLiveRow = 1, kMultiTie = 2;  // live64 bits

struct RowCoef {
  float c1, c10, D, tie;  // tie and c10 in dS units (scale included)
};
__device__ __forceinline__ RowCoef load_row_coef(const float4* coefP, const float* tiev, int64_t r, float scale) {
  const float* p = reinterpret_cast<const float*>(coefP) + (r >> 1) * 4 + (r & 1);
  const float c1 = p[0], ts = 10.f * scale;
  return RowCoef{c1, ts * c1, -p[2], ts * tiev[r]};
}

// Rows per head in the coefficient arrays: N rounded up to whole 64-row tiles,
// so every tile's records start 256-byte aligned and a tile load never reads
// past its head.
__host__ __device__ __forceinline__ int64_t rec_rows(int64_t N) { return (N + 63) / 64 * 64; }

// Swizzled dQ accumulator rows (acc_swz, 64 floats per row): the 16-byte chunk c of
// row n sits at chunk c ^ (n & 15). A drain thread then stores a whole row of one
// query as 16-byte stores while the 32 rows of a warp fall in distinct bank groups.
__host__ __device__ __forceinline__ int acc_chunk(int c, int64_t n) { return c ^ (int)(n & 15); }

// Workspace layout shared by both kernel families (256-byte aligned sections).
struct BwdWorkspace {
  size_t off_dq, off_coef, off_live, off_part, off_sem, total;
};
BwdWorkspace bwd_workspace_layout(int64_t B, int64_t H, int64_t N, int64_t D);
// Row width of the fp32 dQ accumulator: the sm_100a kernels compute head dims that
// are multiples of 16 below 64 (or between 64 and 128) zero-padded to 64 (128), and
// add whole padded rows into it; every kernel family uses the same layout.
inline int64_t acc_width(int64_t D) {
  if (D > 0 && D % 16 == 0 && D < 64) return 64;
  if (D > 64 && D % 16 == 0 && D < 128) return 128;
  return D;
}

int flash_fwd_generic(const FlashArgs& a, cudaStream_t st);
int flash_bwd_generic(const FlashArgs& a, cudaStream_t st);
// Shared pieces of the backward: per-row coefficients and the dQ cast.
int flash_bwd_prep(const FlashArgs& a, cudaStream_t st);
int flash_bwd_finish(const FlashArgs& a, cudaStream_t st);

// sm_100a tcgen05/TMA kernels (bf16, D a multiple of 16 up to 128; computed as 64 or 128).
bool flash_sm100_supported(const FlashArgs& a);
int flash_fwd_sm100(const FlashArgs& a, cudaStream_t st);
int flash_bwd_sm100(const FlashArgs& a, cudaStream_t st);

// CTA order of the tcgen05 kernels: work item w (a CTA's linear block index, or
// its ticket) -> head bh and tile index t. Heads are taken in groups of G: inside a
// group the tile index runs slowest and the head fastest (the longest tiles of the
// group first), and the groups follow one another, so the per-head data that the
// CTAs in flight re-read (K/V in the forward; Q, dO and the dQ accumulator in the
// backward) stays within L2 on long sequences. G >= number of heads is the plain
// order: tile slowest, head fastest.
__device__ __forceinline__ void work_item(int w, int BH, int nT, int G, int* bh, int* t) {
  const int full = BH / G * G;  // heads in complete groups
  if (w < full * nT) {
    const int gsz = G * nT, g = w / gsz, r = w - g * gsz;
    *t = r / G;
    *bh = g * G + r % G;
  } else {
    const int r = w - full * nT, last = BH - full;
    *t = r / last;
    *bh = full + r % last;
  }
}
// Heads per group for a per-head working set of `head_bytes`: the groups in flight
// re-read about 80 MB (the 126 MB L2 keeps streamed tiles too). PNFT_HEAD_GROUP in
// the environment (a positive head count) overrides the choice.
int head_group(int64_t BH, int64_t head_bytes);

// Host helpers shared by the sm_100a kernels: a 4-D TMA map {D, N, H, B} over a
// bf16 [B,H,N,D] view with element strides s (box {64, rows}, 128-byte swizzle),
// the stride/alignment rule such a map needs, and the device check.
int tma_map_bhnd(CUtensorMap* m, const void* base, const int64_t* s, int64_t B, int64_t H, int64_t N, int64_t D,
                 int rows);
bool tma_ok_bhnd(const void* ptr, const int64_t* s);
// 2-D bf16 map over `rows` rows of `cols` elements (row stride in elements, a
// multiple of 8; base 16-byte aligned): boxes of 64 columns x box_rows rows,
// 128-byte swizzled, out-of-range elements read as zero.
int tma_map_rows(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t row_stride, int box_rows);
bool device_is_sm100();

}  // namespace pnft
