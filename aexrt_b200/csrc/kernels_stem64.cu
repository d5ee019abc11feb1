// Instances of the image-stem conv (stem.cuh) for 64 output channels: the one-pixel form.
#include "kernels.cuh"
#include "launch.cuh"

namespace aexrt {
namespace {
template <bool SILU, typename T>
void go(const void* images, int n, int h, int w, int oh, int ow, int stride, __half* out, int out_ldc, int out_coff,
        uint32_t* amax, int amax_stride, int amax_goff, const StemWeights& wt, cudaStream_t st) {
  const dim3 grid((oh * ow + 255) / 256, n);
  launch_kernel(stem_conv_kernel<64, SILU, T>, dim3(grid), dim3(256), 0, st,
      static_cast<const T*>(images), h, w, oh, ow, stride, out, out_ldc, out_coff, amax, amax_stride, amax_goff, wt);
}
}  // namespace

void launch_stem_64(bool silu, bool f16_images, const void* images, int n, int h, int w, int oh, int ow, int stride,
                    __half* out, int out_ldc, int out_coff, uint32_t* amax, int amax_stride, int amax_goff,
                    const StemWeights& wt, cudaStream_t st) {
  if (f16_images)
    (silu ? go<true, __half> : go<false, __half>)(images, n, h, w, oh, ow, stride, out, out_ldc, out_coff, amax,
                                                 amax_stride, amax_goff, wt, st);
  else
    (silu ? go<true, float> : go<false, float>)(images, n, h, w, oh, ow, stride, out, out_ldc, out_coff, amax,
                                               amax_stride, amax_goff, wt, st);
}
}  // namespace aexrt
