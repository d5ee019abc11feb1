// Quantize-on-load instances of the halo conv kernel (conv_halo.cuh): super-tiles (BN <= 64,
// SiLU) and pg16 (BN 64 / 128).
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool RES>
HaloKernel pick_mb(int bn) {
  switch (bn) {
    case 16: return {conv_halo_kernel<false, 16, true, RES, false, true, true>, halo_threads<16, true>()};
    case 32: return {conv_halo_kernel<false, 32, true, RES, false, true, true>, halo_threads<32, true>()};
    case 64: return {conv_halo_kernel<false, 64, true, RES, false, true, true>, halo_threads<64, true>()};
    default: return {nullptr, 0};
  }
}
template <bool SILU, bool RES>
HaloKernel pick_pg(int bn) {
  switch (bn) {
    case 64: return {conv_halo_kernel<false, 64, SILU, RES, true, false, true>, halo_threads<64, true>()};
    case 128: return {conv_halo_kernel<false, 128, SILU, RES, true, false, true>, halo_threads<128, true>()};
    default: return {nullptr, 0};
  }
}
}  // namespace

HaloKernel halo_kernel_ql_mb(int bn, bool silu, bool res) {
  if (!silu) return HaloKernel{nullptr, 0};
  return res ? pick_mb<true>(bn) : pick_mb<false>(bn);
}

HaloKernel halo_kernel_ql_pg(int bn, bool silu, bool res) {
  if (silu) return res ? pick_pg<true, true>(bn) : pick_pg<true, false>(bn);
  return res ? HaloKernel{nullptr, 0} : pick_pg<false, false>(bn);
}
}  // namespace aexrt
