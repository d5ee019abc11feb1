// pg16 (INT8_PERGROUP) instances of the halo conv kernel.
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool SILU, bool RES>
HaloKernel pick(int bn) {
  switch (bn) {
    case 64: return {conv_halo_kernel<false, 64, SILU, RES, true>, halo_threads<64>()};
    case 128: return {conv_halo_kernel<false, 128, SILU, RES, true>, halo_threads<128>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_pg(int bn, bool silu, bool res) {
  if (silu) return res ? pick<true, true>(bn) : pick<true, false>(bn);
  return res ? pick<false, true>(bn) : pick<false, false>(bn);
}
}  // namespace aexrt
