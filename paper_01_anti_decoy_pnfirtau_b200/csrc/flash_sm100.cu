// sm_100a tcgen05 / TMA / TMEM flash pn_fir_tau kernels (bf16, fp16).
#include "flash.cuh"

namespace pnft {

bool flash_sm100_supported(const FlashArgs& a) {
  (void)a;
  return false;
}

int flash_fwd_sm100(const FlashArgs& a, cudaStream_t st) {
  (void)a; (void)st;
  return fail(PNFT_EUNSUPPORTED, "flash fwd sm100: not built");
}

int flash_bwd_sm100(const FlashArgs& a, cudaStream_t st) {
  (void)a; (void)st;
  return fail(PNFT_EUNSUPPORTED, "flash bwd sm100: not built");
}

}  // namespace pnft
