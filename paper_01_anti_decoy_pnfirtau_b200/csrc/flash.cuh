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
  int64_t B, H, N, D;
  float scale, gamma;
  int has_gamma, causal, dtype, flags;
  // bwd workspace carve-up
  float* dq_acc;       // fp32 [B,H,N,D] contiguous
  float4* coef;        // [B*H*N + 64] records of 2 float4 (RowCoef), zero tail
  int32_t* live64;     // [B*H, ceil(N/64)]: 1 if any row of the 64-row tile has peak > 0
  float* dtau_part;    // per (bh, key tile) partial of -sum du
  int64_t n_dtau_part;
};

// Per query row backward coefficients, two float4 per row:
//   c0 = {peak, gate/z, 10*scale*gate/z, D = <dO,O>/gate}
//   c1 = {tie = scale * D*gamma/(peak+gamma)^2/Nmax, argmax key (int bits),
//         peak for the value test (NaN when Nmax == 1), 0}
// so that dS = 10*scale*gate/z * u^9 * (dP - D) + [key == argmax || u == c1.z] * tie:
// a row with one maximum takes the gate gradient at its recorded argmax (exact
// whatever arithmetic recomputes S); genuine ties (Nmax > 1) are found by value.
constexpr int kCoefStride = 2;  // float4 per row

// Workspace layout shared by both kernel families (256-byte aligned sections).
struct BwdWorkspace {
  size_t off_dq, off_coef, off_live, off_part, total;
};
BwdWorkspace bwd_workspace_layout(int64_t B, int64_t H, int64_t N, int64_t D);

int flash_fwd_generic(const FlashArgs& a, cudaStream_t st);
int flash_bwd_generic(const FlashArgs& a, cudaStream_t st);
// Shared pieces of the backward: per-row coefficients and the dQ cast.
int flash_bwd_prep(const FlashArgs& a, cudaStream_t st);
int flash_bwd_finish(const FlashArgs& a, cudaStream_t st);

// sm_100a tcgen05/TMA kernels (bf16, D in {64,128}).
bool flash_sm100_supported(const FlashArgs& a);
int flash_fwd_sm100(const FlashArgs& a, cudaStream_t st);
int flash_bwd_sm100(const FlashArgs& a, cudaStream_t st);

// Host helpers shared by the sm_100a kernels: a 4-D TMA map {D, N, H, B} over a
// bf16 [B,H,N,D] view with element strides s (box {64, rows}, 128-byte swizzle),
// the stride/alignment rule such a map needs, and the device check.
int tma_map_bhnd(CUtensorMap* m, const void* base, const int64_t* s, int64_t B, int64_t H, int64_t N, int64_t D,
                 int rows);
bool tma_ok_bhnd(const void* ptr, const int64_t* s);
bool device_is_sm100();

}  // namespace pnft
