// Direct fp16 conv for the image stem: 3 input channels, 3x3 window, read
// straight from the NCHW image batch (fp16 or fp32).
//
// The stem of the YOLO graphs (Conv(3, c, 3, 2) + SiLU, the reference's first
// fp16 command) has K = 27: a tensor-core tile would need the image repacked
// into 8-channel fp16 slabs (5 of 8 channels padding) and still be bound by
// that repack's traffic.  Here each thread computes one output pixel x OC
// channels with fp32 FMAs whose weight operands come from the kernel's
// parameter space (constant bank, broadcast), so the image is read once and
// the fp16 NHWC output written once.  Numerics match the fp16 conv plans:
// inputs and weights rounded to fp16, fp32 accumulation, fp32 bias + SiLU,
// fp16 output.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "conv_tc.cuh"

namespace aexrt {

constexpr int kStemIC = 3;
constexpr int kStemMaxOC = 64;

struct StemWeights {
  float w[kStemMaxOC * kStemIC * 9];  // [oc][ic][kh][kw], fp16-rounded
  float b[kStemMaxOC];
};

__device__ __forceinline__ float stem_load(const float* p) { return __ldg(p); }
__device__ __forceinline__ float stem_load(const __half* p) { return __half2float(__ldg(p)); }

// grid (ceil(oh*ow / 256), n); block 256, one output pixel per thread.  TIn: float or
// __half images (fp16 images are already what the conv rounds its inputs to).
template <int OC, bool kSilu, typename TIn>
__global__ void __launch_bounds__(256) stem_conv_kernel(const TIn* __restrict__ x, int h, int w, int oh, int ow,
                                                        int stride, __half* __restrict__ out, int out_ldc,
                                                        int out_coff, uint32_t* __restrict__ amax, int amax_stride,
                                                        int amax_goff, const __grid_constant__ StemWeights wt) {
  static_assert(OC % 16 == 0 && OC <= kStemMaxOC, "OC must be a multiple of 16, at most 64");
  constexpr int kGroups = OC / 16;
  __shared__ uint32_t s_amax[kGroups];
  const int n = blockIdx.y;
  if (threadIdx.x < kGroups) s_amax[threadIdx.x] = 0u;
  __syncthreads();
  float run[kGroups];
#pragma unroll
  for (int g = 0; g < kGroups; ++g) run[g] = 0.0f;
  const int npix = oh * ow;
  const size_t plane = static_cast<size_t>(h) * w;
  const TIn* img = x + static_cast<size_t>(n) * kStemIC * plane;
  // one pixel per thread: no loop for the compiler to hoist the weight operands out of
  const int pix = blockIdx.x * blockDim.x + threadIdx.x;
  if (pix < npix) {
    const int oy = pix / ow, ox = pix - (pix / ow) * ow;
    const int iy0 = oy * stride - 1, ix0 = ox * stride - 1;
    float xv[kStemIC * 9];
#pragma unroll
    for (int ic = 0; ic < kStemIC; ++ic)
#pragma unroll
      for (int kh = 0; kh < 3; ++kh)
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          const int iy = iy0 + kh, ix = ix0 + kw;
          const bool in = iy >= 0 && iy < h && ix >= 0 && ix < w;
          const float v = in ? stem_load(img + ic * plane + static_cast<size_t>(iy) * w + ix) : 0.0f;
          xv[(ic * 3 + kh) * 3 + kw] = __half2float(__float2half_rn(v));
        }
    __half* orow = out + (static_cast<size_t>(n) * npix + pix) * out_ldc + out_coff;
#pragma unroll
    for (int o8 = 0; o8 < OC / 8; ++o8) {
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int oc = o8 * 8 + i;
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kStemIC * 9; ++k) acc = fmaf(xv[k], wt.w[oc * kStemIC * 9 + k], acc);
        y[i] = acc + wt.b[oc];
        if constexpr (kSilu) y[i] = silu_fast(y[i]);
      }
      __align__(16) __half2 hv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) hv[i] = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
      *reinterpret_cast<uint4*>(orow + o8 * 8) = *reinterpret_cast<const uint4*>(hv);
      const __half2 m = __hmax2(__hmax2(__habs2(hv[0]), __habs2(hv[1])), __hmax2(__habs2(hv[2]), __habs2(hv[3])));
      run[o8 / 2] = fmaxf(run[o8 / 2], fmaxf(__low2float(m), __high2float(m)));
    }
  }
  if (amax != nullptr) {
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const uint32_t r = __reduce_max_sync(0xffffffffu, __float_as_uint(run[g]));
      if ((threadIdx.x & 31) == 0 && r != 0u) atomicMax(&s_amax[g], r);
    }
    __syncthreads();
    if (threadIdx.x < kGroups && s_amax[threadIdx.x] != 0u)
      atomicMax(&amax[static_cast<size_t>(n) * amax_stride + amax_goff + threadIdx.x], s_amax[threadIdx.x]);
  }
}

}  // namespace aexrt
