// Argument bundle and internal entry points of the flash pn_fir_tau kernels.
#pragma once

#include "common.cuh"

namespace pnft {

struct FlashArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* out_c;  // bwd: forward output
  const void* dout;
  void* out;          // fwd: output
  void* dq;
  void* dk;
  void* dv;
  int64_t sq[4], sk[4], sv[4], so[4], sdo[4], sdq[4], sdk[4], sdv[4];
  const float* tau;
  float* stat_m;
  float* stat_z;
  int32_t* stat_nmax;
  float* dtau;
  int32_t* status;
  uint8_t* tile_flags;  // optional [B*H, nT64, nT64] live-tile record
  int64_t B, H, N, D;
  float scale, gamma;
  int has_gamma, causal, dtype, flags;
  // bwd workspace carve-up
  float* dq_acc;       // fp32 [B,H,N,D] contiguous
  float4* coef;        // [B,H,N]: {peak, gate/z, <dO,O>/gate, tie coefficient}
  float* dtau_part;    // per (bh, key tile) partial of -sum du
  int64_t n_dtau_part;
};

// Workspace layout shared by both kernel families (256-byte aligned sections).
struct BwdWorkspace {
  size_t off_dq, off_coef, off_part, total;
};
BwdWorkspace bwd_workspace_layout(int64_t B, int64_t H, int64_t N, int64_t D);

int flash_fwd_generic(const FlashArgs& a, cudaStream_t st);
int flash_bwd_generic(const FlashArgs& a, cudaStream_t st);
// Shared pieces of the backward: per-row coefficients and the dQ cast.
int flash_bwd_prep(const FlashArgs& a, cudaStream_t st);
int flash_bwd_finish(const FlashArgs& a, cudaStream_t st);

// sm_100a tcgen05/TMA kernels (bf16/fp16, D in {64,128}); return
// PNFT_EUNSUPPORTED when the arguments do not fit them.
bool flash_sm100_supported(const FlashArgs& a);
int flash_fwd_sm100(const FlashArgs& a, cudaStream_t st);
int flash_bwd_sm100(const FlashArgs& a, cudaStream_t st);

}  // namespace pnft
