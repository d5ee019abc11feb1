// Element-wise graph ops of reference engines that the W8A8 runtime meets
// outside its fused forms: a MAXPOOL that is not part of an SPPF cascade and a
// BINARY Add that cannot become a conv epilogue residual (the reference's
// generic fp32 MAXPOOL / BINARY shaders, recorded by record_direct_logical_command,
// native/aexrt_d3d12_runtime.cpp:28307-28330).  Activations here are fp16 NHWC
// channel slices; the input of an op may be a concatenation of up to
// kMaxGraphParts slices, each optionally read through a nearest 2x upsample.
// Both ops max |y| per (image, 16-channel group) into the output buffer's amax
// slots when the output feeds an int8 conv.
#pragma once
#include "ptx.cuh"
#include <cuda_fp16.h>

#include <cstdint>

namespace aexrt {

constexpr int kMaxGraphParts = 8;

struct GraphParts {
  int nparts;
  const __half* ptr[kMaxGraphParts];
  int ldc[kMaxGraphParts], coff[kMaxGraphParts], ch[kMaxGraphParts], up[kMaxGraphParts];
  int h[kMaxGraphParts], w[kMaxGraphParts];  // stored dims of each part's buffer
};

// x[img][y][x][c] of the concatenation (y, x at the consumer's resolution)
__device__ __forceinline__ float parts_at(const GraphParts& p, int img, int y, int x, int c) {
  int i = 0;
  while (i + 1 < p.nparts && c >= p.ch[i]) {
    c -= p.ch[i];
    ++i;
  }
  const int yy = y / p.up[i], xx = x / p.up[i];
  return __half2float(p.ptr[i][((static_cast<long>(img) * p.h[i] + yy) * p.w[i] + xx) * p.ldc[i] + p.coff[i] + c]);
}

__device__ __forceinline__ void store_amax(uint32_t* amax, int amax_stride, int img, int c, float y) {
  if (amax) atomicMax(amax + static_cast<long>(img) * amax_stride + c / 16, __float_as_uint(fabsf(y)));
}

// MaxPool (kernel k, stride s, padding p, padded positions ignored as -inf) of an n x h x w x c input.
// Thread = one output element.
__global__ void maxpool_nhwc_kernel(const GraphParts in, int n, int h, int w, int c, int k, int s, int pad, int oh,
                                    int ow, __half* __restrict__ out, int out_ldc, uint32_t* __restrict__ amax,
                                    int amax_stride) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  const long total = static_cast<long>(n) * oh * ow * c;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int ch = static_cast<int>(idx % c);
  const long pix = idx / c;
  const int ox = static_cast<int>(pix % ow), oy = static_cast<int>((pix / ow) % oh);
  const int img = static_cast<int>(pix / (static_cast<long>(ow) * oh));
  float m = -INFINITY;
  for (int dy = 0; dy < k; ++dy) {
    const int y = oy * s - pad + dy;
    if (y < 0 || y >= h) continue;
    for (int dx = 0; dx < k; ++dx) {
      const int x = ox * s - pad + dx;
      if (x < 0 || x >= w) continue;
      m = fmaxf(m, parts_at(in, img, y, x, ch));
    }
  }
  const __half hv = __float2half_rn(m);
  out[pix * out_ldc + ch] = hv;
  store_amax(amax, amax_stride, img, ch, __half2float(hv));
}

// out = a + b (fp32 sum of the fp16 operands, rounded to fp16), same n x h x w x c shape.
__global__ void add_nhwc_kernel(const GraphParts a, const GraphParts b, int n, int h, int w, int c,
                                __half* __restrict__ out, int out_ldc, uint32_t* __restrict__ amax, int amax_stride) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  const long total = static_cast<long>(n) * h * w * c;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int ch = static_cast<int>(idx % c);
  const long pix = idx / c;
  const int x = static_cast<int>(pix % w), y = static_cast<int>((pix / w) % h);
  const int img = static_cast<int>(pix / (static_cast<long>(w) * h));
  const __half hv = __float2half_rn(parts_at(a, img, y, x, ch) + parts_at(b, img, y, x, ch));
  out[pix * out_ldc + ch] = hv;
  store_amax(amax, amax_stride, img, ch, __half2float(hv));
}

}  // namespace aexrt
