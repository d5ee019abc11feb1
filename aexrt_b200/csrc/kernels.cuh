// Kernel selection across the translation units that instantiate the conv
// kernels (kernels_slot.cu, kernels_halo_*.cu): each unit compiles one family
// of template instances, so the library builds in parallel.
#pragma once
#include <cuda.h>

#include "conv_halo.cuh"
#include "conv_tc.cuh"
#include "stem.cuh"

namespace aexrt {

using KernelFn = void (*)(const CUtensorMap, const ConvTcParams);
using HaloFn = void (*)(const CUtensorMap, const ConvHaloParams);

struct HaloKernel {
  HaloFn fn;
  int threads;
};

// Slot-streaming kernel for (fp16, pg16, BN); nullptr when not instantiated.
KernelFn kernel_for(bool f16, bool pg, int bn);

// Halo kernel families: per tensor (int8 SiLU / linear, fp16), super-tiles (BN <= 64) and
// pg16 (BN 64/128).
HaloKernel halo_kernel_i8_silu(int bn, bool res);
HaloKernel halo_kernel_i8_linear(int bn, bool res);
HaloKernel halo_kernel_f16(int bn, bool silu, bool res);
HaloKernel halo_kernel_mb(bool f16, int bn, bool silu, bool res);
HaloKernel halo_kernel_pg(int bn, bool silu, bool res);
// quantize on load (int8 plans reading fp16 NHWC sources): per tensor, super-tiles, pg16
HaloKernel halo_kernel_ql(int bn, bool silu, bool res);
HaloKernel halo_kernel_ql_mb(int bn, bool silu, bool res);
HaloKernel halo_kernel_ql_pg(int bn, bool silu, bool res);

// Residuals (the C2f tail) are instantiated for every int8 conv and for fp16 SiLU convs; a
// combination without an instance returns {nullptr, 0}.
inline HaloKernel halo_kernel_for(bool f16, int bn, bool silu, bool res, bool pg = false, bool mb = false,
                                  bool ql = false) {
  if (ql) {
    if (f16) return HaloKernel{nullptr, 0};
    return mb ? halo_kernel_ql_mb(bn, silu, res) : (pg ? halo_kernel_ql_pg(bn, silu, res) : halo_kernel_ql(bn, silu, res));
  }
  if (mb) return halo_kernel_mb(f16, bn, silu, res);
  if (pg) return f16 ? HaloKernel{nullptr, 0} : halo_kernel_pg(bn, silu, res);
  if (f16) return halo_kernel_f16(bn, silu, res);
  return silu ? halo_kernel_i8_silu(bn, res) : halo_kernel_i8_linear(bn, res);
}

// The image stem (stem.cuh): one unit per output width (16, 32, 48, 64), fp16 or fp32 images.
// Widths 16 and 32 run stem_pair_kernel, 48 and 64 stem_conv_kernel; each launcher sizes its own grid.
#define AEXRT_STEM_DECL(OC)                                                                                        \
  void launch_stem_##OC(bool silu, bool f16_images, const void* images, int n, int h, int w, int oh, int ow,      \
                        int stride, __half* out, int out_ldc, int out_coff, uint32_t* amax, int amax_stride,      \
                        int amax_goff, const StemWeights& wt, cudaStream_t st);
AEXRT_STEM_DECL(16)
AEXRT_STEM_DECL(32)
AEXRT_STEM_DECL(48)
AEXRT_STEM_DECL(64)
#undef AEXRT_STEM_DECL

inline void launch_stem(int oc, bool silu, bool f16_images, const void* images, int n, int h, int w, int oh, int ow,
                        int stride, __half* out, int out_ldc, int out_coff, uint32_t* amax, int amax_stride,
                        int amax_goff, const StemWeights& wt, cudaStream_t st) {
  auto* fn = oc == 16 ? launch_stem_16 : oc == 32 ? launch_stem_32 : oc == 48 ? launch_stem_48 : launch_stem_64;
  fn(silu, f16_images, images, n, h, w, oh, ow, stride, out, out_ldc, out_coff, amax, amax_stride, amax_goff, wt, st);
}

}  // namespace aexrt
