// fp16 (detect head) instances of the halo conv kernel (conv_halo.cuh).
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool SILU>
HaloKernel pick(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<true, 16, SILU, false>, halo_threads<16>()};
    case 32: return {conv_halo_kernel<true, 32, SILU, false>, halo_threads<32>()};
    case 64: return {conv_halo_kernel<true, 64, SILU, false>, halo_threads<64>()};
    case 128: return {conv_halo_kernel<true, 128, SILU, false>, halo_threads<128>()};
    case 256: return {conv_halo_kernel<true, 256, SILU, false>, halo_threads<256>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_f16(int bn, bool silu) { return silu ? pick<true>(bn) : pick<false>(bn); }
}  // namespace aexrt
