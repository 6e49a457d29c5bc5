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

// Output rows [r0, r0 + NR) of column pair cp (columns 2cp, 2cp+1) of one group.
// raw: shared address of the staged group (row i = input row k0 - FIR_HALO + i);
// dst: shared address of the tile group (row n = output row k0 + n). 32 threads
// with consecutive cp and the same rows touch one 128-byte row: no bank conflicts.
template <int NR>
__device__ __forceinline__ void fir_filter_rows(uint32_t raw, uint32_t dst, int cp, int r0,
                                                const float2 (&h)[FIR_TAPS]) {
  const uint32_t cb = (uint32_t)(cp & 3) * 4u;  // byte inside the 16-byte chunk
  const uint32_t ch = (uint32_t)(cp >> 2);      // 16-byte chunk of the row
  auto ld = [&](int rr) -> float2 {
    uint32_t w;
    asm volatile("ld.shared.b32 %0, [%1];"
                 : "=r"(w)
                 : "r"(raw + (uint32_t)rr * 128u + ((ch ^ (uint32_t)(rr & 7)) << 4) + cb));
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  };
  float2 x[FIR_TAPS];  // x[u]: input at lag u of the current output row
#pragma unroll
  for (int u = 1; u < FIR_TAPS; ++u) x[u] = ld(r0 + FIR_HALO - u);
#pragma unroll 4
  for (int n = r0; n < r0 + NR; ++n) {
    x[0] = ld(n + FIR_HALO);
    float2 a = __fmul2_rn(x[0], h[0]);
#pragma unroll
    for (int u = 1; u < FIR_TAPS; ++u) a = __ffma2_rn(x[u], h[u], a);
    const uint32_t w = pack_bf16x2(a.x, a.y);
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst + (uint32_t)n * 128u + ((ch ^ (uint32_t)(n & 7)) << 4) + cb),
                 "r"(w)
                 : "memory");
#pragma unroll
    for (int u = FIR_TAPS - 1; u > 0; --u) x[u] = x[u - 1];
  }
}

}  // namespace pnft
