// Instances of the slot-streaming conv kernel (conv_tc.cuh).
#include "kernels.cuh"

namespace aexrt {
namespace {
template <bool F16, bool PG>
KernelFn kernel_for_bn(int bn) {
  switch (bn) {
    case 16: return conv_tc_kernel<F16, PG, 16>;
    case 32: return conv_tc_kernel<F16, PG, 32>;
    case 64: return conv_tc_kernel<F16, PG, 64>;
    case 128: return conv_tc_kernel<F16, PG, 128>;
    case 256:
      if constexpr (!PG) return conv_tc_kernel<F16, PG, 256>;
      return nullptr;
    default: return nullptr;
  }
}
}  // namespace

KernelFn kernel_for(bool f16, bool pg, int bn) {
  if (f16) return kernel_for_bn<true, false>(bn);
  return pg ? kernel_for_bn<false, true>(bn) : kernel_for_bn<false, false>(bn);
}
}  // namespace aexrt
