// Quantize-on-load instances of the halo conv kernel (conv_halo.cuh): int8 plans that read fp16
// NHWC sources and convert them to int8 codes in shared memory.  Per tensor (SiLU with and without
// the C2f residual, linear); the super-tile and pg16 forms are in kernels_halo_ql_mb.cu.
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool SILU, bool RES>
HaloKernel pick(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<false, 16, SILU, RES, false, false, true>, halo_threads<16, true>()};
    case 32: return {conv_halo_kernel<false, 32, SILU, RES, false, false, true>, halo_threads<32, true>()};
    case 64: return {conv_halo_kernel<false, 64, SILU, RES, false, false, true>, halo_threads<64, true>()};
    case 128: return {conv_halo_kernel<false, 128, SILU, RES, false, false, true>, halo_threads<128, true>()};
    case 256: return {conv_halo_kernel<false, 256, SILU, RES, false, false, true>, halo_threads<256, true>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_ql(int bn, bool silu, bool res) {
  if (silu) return res ? pick<true, true>(bn) : pick<true, false>(bn);
  return res ? HaloKernel{nullptr, 0} : pick<false, false>(bn);
}
}  // namespace aexrt
