// Per-tensor int8 instances of the halo conv kernel (conv_halo.cuh), SiLU epilogue.
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool RES>
HaloKernel pick(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<false, 16, true, RES>, halo_threads<16>()};
    case 32: return {conv_halo_kernel<false, 32, true, RES>, halo_threads<32>()};
    case 64: return {conv_halo_kernel<false, 64, true, RES>, halo_threads<64>()};
    case 128: return {conv_halo_kernel<false, 128, true, RES>, halo_threads<128>()};
    case 256: return {conv_halo_kernel<false, 256, true, RES>, halo_threads<256>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_i8_silu(int bn, bool res) { return res ? pick<true>(bn) : pick<false>(bn); }
}  // namespace aexrt
