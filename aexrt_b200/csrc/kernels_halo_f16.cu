// fp16 instances of the halo conv kernel (conv_halo.cuh): the detect head, the stem-side convs, and
// convs an engine keeps in fp16 (SiLU convs may carry a C2f residual).
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool SILU, bool RES>
HaloKernel pick(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<true, 16, SILU, RES>, halo_threads<16>()};
    case 32: return {conv_halo_kernel<true, 32, SILU, RES>, halo_threads<32>()};
    case 64: return {conv_halo_kernel<true, 64, SILU, RES>, halo_threads<64>()};
    case 128: return {conv_halo_kernel<true, 128, SILU, RES>, halo_threads<128>()};
    case 256: return {conv_halo_kernel<true, 256, SILU, RES>, halo_threads<256>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_f16(int bn, bool silu, bool res) {
  if (res) return silu ? pick<true, true>(bn) : HaloKernel{nullptr, 0};
  return silu ? pick<true, false>(bn) : pick<false, false>(bn);
}
}  // namespace aexrt
