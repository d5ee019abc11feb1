// Super-tile instances (several M blocks per tile, BN <= 64) of the halo conv kernel.
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool F16, bool SILU, bool RES>
HaloKernel pick(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<F16, 16, SILU, RES, false, true>, halo_threads<16>()};
    case 32: return {conv_halo_kernel<F16, 32, SILU, RES, false, true>, halo_threads<32>()};
    case 64: return {conv_halo_kernel<F16, 64, SILU, RES, false, true>, halo_threads<64>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_mb(bool f16, int bn, bool silu, bool res) {
  if (f16) {
    if (res) return silu ? pick<true, true, true>(bn) : HaloKernel{nullptr, 0};
    return silu ? pick<true, true, false>(bn) : pick<true, false, false>(bn);
  }
  if (silu) return res ? pick<false, true, true>(bn) : pick<false, true, false>(bn);
  return res ? pick<false, false, true>(bn) : pick<false, false, false>(bn);
}
}  // namespace aexrt
