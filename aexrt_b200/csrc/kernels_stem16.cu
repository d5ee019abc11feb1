// Instances of the image-stem conv (stem.cuh) for 16 output channels: the two-pixel form.
#include "kernels.cuh"
#include "launch.cuh"

namespace aexrt {
namespace {
template <bool SILU, typename T, int S>
void go(const void* images, int n, int h, int w, int oh, int ow, __half* out, int out_ldc, int out_coff,
        uint32_t* amax, int amax_stride, int amax_goff, const StemWeights& wt, cudaStream_t st) {
  const dim3 grid((oh * ((ow + 1) / 2) + 255) / 256, n);
  launch_kernel(stem_pair_kernel<16, SILU, T, S>, dim3(grid), dim3(256), 0, st,
      static_cast<const T*>(images), h, w, oh, ow, out, out_ldc, out_coff, amax, amax_stride, amax_goff, wt);
}

template <bool SILU, typename T>
void go_s(int stride, const void* images, int n, int h, int w, int oh, int ow, __half* out, int out_ldc, int out_coff,
          uint32_t* amax, int amax_stride, int amax_goff, const StemWeights& wt, cudaStream_t st) {
  (stride == 2 ? go<SILU, T, 2> : go<SILU, T, 1>)(images, n, h, w, oh, ow, out, out_ldc, out_coff, amax, amax_stride,
                                                  amax_goff, wt, st);
}
}  // namespace

void launch_stem_16(bool silu, bool f16_images, const void* images, int n, int h, int w, int oh, int ow, int stride,
                    __half* out, int out_ldc, int out_coff, uint32_t* amax, int amax_stride, int amax_goff,
                    const StemWeights& wt, cudaStream_t st) {
  if (f16_images)
    (silu ? go_s<true, __half> : go_s<false, __half>)(stride, images, n, h, w, oh, ow, out, out_ldc, out_coff, amax,
                                                     amax_stride, amax_goff, wt, st);
  else
    (silu ? go_s<true, float> : go_s<false, float>)(stride, images, n, h, w, oh, ow, out, out_ldc, out_coff, amax,
                                                   amax_stride, amax_goff, wt, st);
}
}  // namespace aexrt
