// Direct fp16 conv for the image stem: 3 input channels, 3x3 window, read
// straight from the NCHW image batch (fp16 or fp32).
//
// The stem of the YOLO graphs (Conv(3, c, 3, 2) + SiLU, the reference's first
// fp16 command) has K = 27: a tensor-core tile would need the image repacked
// into 8-channel fp16 slabs (5 of 8 channels padding) and still be bound by
// that repack's traffic.  Here each thread computes output pixels x OC
// channels with fp32 FMAs whose weight operands come from the kernel's
// parameter space (constant bank, broadcast), so the image is read once and
// the fp16 NHWC output written once.  Numerics match the fp16 conv plans:
// inputs and weights rounded to fp16, fp32 accumulation, fp32 bias + SiLU,
// fp16 output.
//
// Two forms with the same per-output arithmetic (the same fma chain over
// k = 0..26 from 0, then + bias), so their outputs are bit-identical:
//   * stem_pair_kernel (OC <= 32): two horizontally adjacent output pixels per
//     thread, the two fma chains run as one packed f32x2 fma per tap and
//     channel; the weight operand is the tap's fp32 weight in both halves
//     (packed in the kernel: faster than a pre-duplicated 64-bit parameter).  The
//     kernel is issue-bound (about 1170 instructions per pixel in the
//     one-pixel form), and the pair form halves the fma instructions and
//     shares the overlapping window columns;
//   * stem_conv_kernel (OC 48, 64): one output pixel per thread, where the
//     pair form's registers would spill.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "conv_tc.cuh"
#include "ptx.cuh"

namespace aexrt {

constexpr int kStemIC = 3;
constexpr int kStemMaxOC = 64;
constexpr int kStemPairMaxOC = 32;  // widths that run stem_pair_kernel

struct StemWeights {
  float w[kStemMaxOC * kStemIC * 9];  // [oc][ic][kh][kw], fp16-rounded
  float b[kStemMaxOC];
};

// One tap as the conv consumes it: the image value rounded to fp16 (fp16 images already are).
__device__ __forceinline__ float stem_load(const float* p) { return __half2float(__float2half_rn(__ldg(p))); }
__device__ __forceinline__ float stem_load(const __half* p) { return __half2float(__ldg(p)); }

// grid (ceil(oh*ow / 256), n); block 256, one output pixel per thread.  TIn: float or
// __half images (fp16 images are already what the conv rounds its inputs to).
template <int OC, bool kSilu, typename TIn>
__global__ void __launch_bounds__(256) stem_conv_kernel(const TIn* __restrict__ x, int h, int w, int oh, int ow,
                                                        int stride, __half* __restrict__ out, int out_ldc,
                                                        int out_coff, uint32_t* __restrict__ amax, int amax_stride,
                                                        int amax_goff, const __grid_constant__ StemWeights wt) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
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
          xv[(ic * 3 + kh) * 3 + kw] = in ? stem_load(img + ic * plane + static_cast<size_t>(iy) * w + ix) : 0.0f;
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

// grid (ceil(oh * ceil(ow / 2) / 256), n); block 256.  Thread q owns output pixels (oy, ox) and
// (oy, ox + 1), ox = 2 * (q mod ceil(ow / 2)); the second is skipped where ox + 1 == ow.  The two
// windows span columns ix0 .. ix0 + S + 2 of each input row.
template <int OC, bool kSilu, typename TIn, int S>
__global__ void __launch_bounds__(256, 3) stem_pair_kernel(const TIn* __restrict__ x, int h, int w, int oh, int ow,
                                                           __half* __restrict__ out, int out_ldc, int out_coff,
                                                           uint32_t* __restrict__ amax, int amax_stride, int amax_goff,
                                                           const __grid_constant__ StemWeights wt) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  static_assert(OC % 16 == 0 && OC <= kStemPairMaxOC, "OC must be 16 or 32");
  constexpr int kGroups = OC / 16;
  constexpr int kCols = S + 3;
  __shared__ uint32_t s_amax[kGroups];
  const int n = blockIdx.y;
  if (threadIdx.x < kGroups) s_amax[threadIdx.x] = 0u;
  __syncthreads();
  float run[kGroups];
#pragma unroll
  for (int g = 0; g < kGroups; ++g) run[g] = 0.0f;
  const int ppr = (ow + 1) >> 1;
  const size_t plane = static_cast<size_t>(h) * w;
  const TIn* img = x + static_cast<size_t>(n) * kStemIC * plane;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q < oh * ppr) {
    const int oy = q / ppr, ox = 2 * (q - oy * ppr);
    const bool second = ox + 1 < ow;
    const int iy0 = oy * S - 1, ix0 = ox * S - 1;
    uint64_t xp[kStemIC * 9];  // (pixel ox tap, pixel ox + 1 tap)
#pragma unroll
    for (int ic = 0; ic < kStemIC; ++ic)
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        const int iy = iy0 + kh;
        const bool row_in = iy >= 0 && iy < h;
        float col[kCols];
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          const int ix = ix0 + j;
          const bool in = row_in && ix >= 0 && ix < w;
          col[j] = in ? stem_load(img + ic * plane + static_cast<size_t>(iy) * w + ix) : 0.0f;
        }
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) xp[(ic * 3 + kh) * 3 + kw] = f2_pack(col[kw], col[kw + S]);
      }
    __half* oa = out + (static_cast<size_t>(n) * oh * ow + static_cast<size_t>(oy) * ow + ox) * out_ldc + out_coff;
#pragma unroll
    for (int o8 = 0; o8 < OC / 8; ++o8) {
      float ya[8], yb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int oc = o8 * 8 + i;
        uint64_t acc = 0ull;
#pragma unroll
        for (int k = 0; k < kStemIC * 9; ++k) {
          const float wv = wt.w[oc * kStemIC * 9 + k];
          acc = f2_fma(xp[k], f2_pack(wv, wv), acc);
        }
        f2_unpack(acc, ya[i], yb[i]);
        ya[i] = ya[i] + wt.b[oc];
        yb[i] = yb[i] + wt.b[oc];
        if constexpr (kSilu) {
          ya[i] = silu_fast(ya[i]);
          yb[i] = silu_fast(yb[i]);
        }
      }
      __align__(16) __half2 ha[4], hb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ha[i] = __floats2half2_rn(ya[2 * i], ya[2 * i + 1]);
        hb[i] = __floats2half2_rn(yb[2 * i], yb[2 * i + 1]);
      }
      *reinterpret_cast<uint4*>(oa + o8 * 8) = *reinterpret_cast<const uint4*>(ha);
      __half2 m = __hmax2(__hmax2(__habs2(ha[0]), __habs2(ha[1])), __hmax2(__habs2(ha[2]), __habs2(ha[3])));
      if (second) {
        *reinterpret_cast<uint4*>(oa + out_ldc + o8 * 8) = *reinterpret_cast<const uint4*>(hb);
        m = __hmax2(m, __hmax2(__hmax2(__habs2(hb[0]), __habs2(hb[1])), __hmax2(__habs2(hb[2]), __habs2(hb[3]))));
      }
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
