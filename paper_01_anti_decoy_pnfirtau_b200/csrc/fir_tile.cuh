// Causal FIR of a K tile in shared memory, for the tcgen05 flash kernels' fused
// K-tile load (K~ = causal_fir(K), the module's 7-tap filter on the keys).
//
// The raw rows [k0 - FIR_HALO, k0 + rows) of one 64-column group are staged by
// TMA (rows before the sequence start read as zero, the filter's causal padding)
// as 128-byte rows in the 128-byte swizzle; the filtered rows go to the MMA's K
// tile in the same layout. The arithmetic is that of pnft_fir_fwd (csrc/fir.cu):
// fp32, the product of lag 0 first, then FMAs of lags 1..6, rounded to bf16, so a
// fused tile is bit-identical to the standalone filter's output.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace pnft {

using sm100::pack_bf16x2;

constexpr int FIR_TAPS = PNFT_FIR_FUSED_TAPS;  // the module's filter length (PnFirConfig.fir_k)
constexpr int FIR_HALO = 8;  // staged rows before the tile: >= FIR_TAPS - 1, one swizzle atom

// h[u] = (taps[FIR_TAPS-1-u], same): the weight of the input at lag u
__device__ __forceinline__ void fir_load_taps(const float* taps, float2 (&h)[FIR_TAPS]) {
#pragma unroll
  for (int u = 0; u < FIR_TAPS; ++u) {
    const float t = __ldg(taps + (FIR_TAPS - 1 - u));
    h[u] = make_float2(t, t);
  }
}

// Output rows [r0, r0 + NR) of column pair cp (columns 2cp, 2cp+1) of one group;
// r0 a multiple of 8. raw: the staged group (row i = input row k0 - FIR_HALO + i);
// dst: the tile group (row n = output row k0 + n); both shared-memory pointers.
// 32 threads with consecutive cp and the same rows touch one 128-byte row: no
// bank conflicts. Fully unrolled: the window rotates by renaming, every row
// address is a constant offset (r0 is a multiple of the 8-row swizzle period),
// and plain loads / stores leave the compiler free to run the rows' loads ahead.
template <int NR>
__device__ __forceinline__ void fir_filter_rows(const uint8_t* raw, uint8_t* dst, int cp, int r0,
                                                const float2 (&h)[FIR_TAPS]) {
  static_assert(FIR_HALO % 8 == 0, "row offsets keep the swizzle phase");
  const uint32_t cb = (uint32_t)(cp & 3) * 4u;  // byte inside the 16-byte chunk
  const uint32_t ch = (uint32_t)(cp >> 2);      // 16-byte chunk of the row
  uint32_t col[8];                              // swizzled column offset per row phase
#pragma unroll
  for (int i = 0; i < 8; ++i) col[i] = ((ch ^ (uint32_t)i) << 4) + cb;
  const uint8_t* rb = raw + r0 * 128;
  uint8_t* db = dst + r0 * 128;
  auto ld = [&](int rr) -> float2 {  // staged row r0 + rr
    const uint32_t w = *reinterpret_cast<const uint32_t*>(rb + rr * 128 + col[rr & 7]);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  };
  float2 x[NR + FIR_TAPS - 1];  // x[i] = input row r0 + i - (FIR_TAPS - 1)
#pragma unroll
  for (int i = 0; i < FIR_TAPS - 1; ++i) x[i] = ld(FIR_HALO - (FIR_TAPS - 1) + i);
#pragma unroll
  for (int n = 0; n < NR; ++n) {
    x[n + FIR_TAPS - 1] = ld(n + FIR_HALO);
    float2 a = __fmul2_rn(x[n + FIR_TAPS - 1], h[0]);
#pragma unroll
    for (int u = 1; u < FIR_TAPS; ++u) a = __ffma2_rn(x[n + FIR_TAPS - 1 - u], h[u], a);
    *reinterpret_cast<uint32_t*>(db + n * 128 + col[n & 7]) = pack_bf16x2(a.x, a.y);
  }
}

}  // namespace pnft
