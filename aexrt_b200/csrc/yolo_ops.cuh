// The non-convolution ops of the YOLO graphs around the W8A8 path: the SPPF
// max-pool cascade and the detect-head decode (DFL softmax + anchor decode +
// class sigmoid).  Both are small HBM-bound element passes.
#pragma once
#include "ptx.cuh"
#include <cuda_fp16.h>

#include <cstdint>

namespace aexrt {

// SPPF (YOLOv8: cv1 -> m -> m -> m with m = MaxPool2d(5, 1, 2), concatenated):
// the three cascaded 5x5 pools equal single 5x5 / 9x9 / 13x13 max windows of
// the input (clipped at the border), so one pass writes all three slices.
// Thread = one pixel x 8 channels.  Also max-es |y| per 16-channel group into
// the amax slots of the destination buffer.
__global__ void sppf_pool_kernel(const __half* __restrict__ x, int n, int h, int w, int c, int ldc, int coff,
                                 __half* __restrict__ out, int out_ldc, int out_coff, uint32_t* __restrict__ amax,
                                 int amax_stride, int amax_goff) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  const int vec = c / 8;
  const long total = static_cast<long>(n) * h * w * vec;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int cv = static_cast<int>(idx % vec) * 8;
  const long pix = idx / vec;
  const int xw = static_cast<int>(pix % w);
  const int yh = static_cast<int>((pix / w) % h);
  const int img = static_cast<int>(pix / (static_cast<long>(w) * h));
  __half2 m5[4], m9[4], m13[4];
  const __half2 ninf = __halves2half2(__ushort_as_half(0xFC00), __ushort_as_half(0xFC00));
#pragma unroll
  for (int i = 0; i < 4; ++i) m5[i] = m9[i] = m13[i] = ninf;
  for (int dy = -6; dy <= 6; ++dy) {
    const int yy = yh + dy;
    if (yy < 0 || yy >= h) continue;
    for (int dx = -6; dx <= 6; ++dx) {
      const int xx = xw + dx;
      if (xx < 0 || xx >= w) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(x + ((static_cast<long>(img) * h + yy) * w + xx) * ldc + coff + cv);
      const __half2* hv = reinterpret_cast<const __half2*>(&v);
      const int ad = max(abs(dy), abs(dx));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        m13[i] = __hmax2(m13[i], hv[i]);
        if (ad <= 4) m9[i] = __hmax2(m9[i], hv[i]);
        if (ad <= 2) m5[i] = __hmax2(m5[i], hv[i]);
      }
    }
  }
  __half* o = out + pix * out_ldc + out_coff + cv;
  *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(m5);
  *reinterpret_cast<uint4*>(o + c) = *reinterpret_cast<const uint4*>(m9);
  *reinterpret_cast<uint4*>(o + 2 * c) = *reinterpret_cast<const uint4*>(m13);
  if (amax != nullptr) {
    float a[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[0] = fmaxf(a[0], fmaxf(fabsf(__low2float(m5[i])), fabsf(__high2float(m5[i]))));
      a[1] = fmaxf(a[1], fmaxf(fabsf(__low2float(m9[i])), fabsf(__high2float(m9[i]))));
      a[2] = fmaxf(a[2], fmaxf(fabsf(__low2float(m13[i])), fabsf(__high2float(m13[i]))));
    }
    uint32_t* slot = amax + static_cast<long>(img) * amax_stride + amax_goff;
#pragma unroll
    for (int k = 0; k < 3; ++k) atomicMax(slot + (k * c + cv) / 16, __float_as_uint(a[k]));
  }
}

// SPPF from shared memory: one block holds an image's whole map for a block of
// `cb` channels, computes the row maxima of the 5/9/13 windows (separable), then
// the column maxima, and writes the three pooled slices.  amax per 16-channel
// group is reduced in shared memory (one global atomic per group and block).
__global__ void __launch_bounds__(256) sppf_smem_kernel(const __half* __restrict__ x, int h, int w, int c, int ldc,
                                                       int coff, int cb, __half* __restrict__ out, int out_ldc,
                                                       int out_coff, uint32_t* __restrict__ amax, int amax_stride,
                                                       int amax_goff) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  extern __shared__ __align__(16) __half sm[];  // [4][h*w][cb]: input, then row maxima for 5, 9, 13
  __shared__ uint32_t s_amax[3 * 16];           // cb <= 256 -> <= 16 groups per slice
  const int n = blockIdx.y;
  const int c0 = blockIdx.x * cb;
  const int hw = h * w;
  const int vec = cb / 8;
  const int plane = hw * cb;
  for (int i = threadIdx.x; i < 3 * 16; i += blockDim.x) s_amax[i] = 0u;
  for (int idx = threadIdx.x; idx < hw * vec; idx += blockDim.x) {
    const int pix = idx / vec, v = idx - (idx / vec) * vec;
    *reinterpret_cast<uint4*>(sm + pix * cb + 8 * v) =
        *reinterpret_cast<const uint4*>(x + (static_cast<size_t>(n) * hw + pix) * ldc + coff + c0 + 8 * v);
  }
  __syncthreads();
  const __half2 ninf = __halves2half2(__ushort_as_half(0xFC00), __ushort_as_half(0xFC00));
  for (int idx = threadIdx.x; idx < hw * vec; idx += blockDim.x) {
    const int pix = idx / vec, v = idx - (idx / vec) * vec;
    const int yy = pix / w, xx = pix - (pix / w) * w;
    __half2 m5[4], m9[4], m13[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) m5[i] = m9[i] = m13[i] = ninf;
    for (int dx = -6; dx <= 6; ++dx) {
      const int xs = xx + dx;
      if (xs < 0 || xs >= w) continue;
      const uint4 t = *reinterpret_cast<const uint4*>(sm + (yy * w + xs) * cb + 8 * v);
      const __half2* t2 = reinterpret_cast<const __half2*>(&t);
      const int ad = abs(dx);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        m13[i] = __hmax2(m13[i], t2[i]);
        if (ad <= 4) m9[i] = __hmax2(m9[i], t2[i]);
        if (ad <= 2) m5[i] = __hmax2(m5[i], t2[i]);
      }
    }
    *reinterpret_cast<uint4*>(sm + plane + pix * cb + 8 * v) = *reinterpret_cast<const uint4*>(m5);
    *reinterpret_cast<uint4*>(sm + 2 * plane + pix * cb + 8 * v) = *reinterpret_cast<const uint4*>(m9);
    *reinterpret_cast<uint4*>(sm + 3 * plane + pix * cb + 8 * v) = *reinterpret_cast<const uint4*>(m13);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < hw * vec; idx += blockDim.x) {
    const int pix = idx / vec, v = idx - (idx / vec) * vec;
    const int yy = pix / w, xx = pix - (pix / w) * w;
    __half* o = out + (static_cast<size_t>(n) * hw + pix) * out_ldc + out_coff + c0 + 8 * v;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int r = k == 0 ? 2 : (k == 1 ? 4 : 6);
      __half2 m[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) m[i] = ninf;
      for (int dy = -r; dy <= r; ++dy) {
        const int ys = yy + dy;
        if (ys < 0 || ys >= h) continue;
        const uint4 t = *reinterpret_cast<const uint4*>(sm + (k + 1) * plane + (ys * w + xx) * cb + 8 * v);
        const __half2* t2 = reinterpret_cast<const __half2*>(&t);
#pragma unroll
        for (int i = 0; i < 4; ++i) m[i] = __hmax2(m[i], t2[i]);
      }
      *reinterpret_cast<uint4*>(o + k * c) = *reinterpret_cast<const uint4*>(m);
      if (amax != nullptr) {
        const __half2 a = __hmax2(__hmax2(__habs2(m[0]), __habs2(m[1])), __hmax2(__habs2(m[2]), __habs2(m[3])));
        atomicMax(&s_amax[k * 16 + (8 * v) / 16], __float_as_uint(fmaxf(__low2float(a), __high2float(a))));
      }
    }
  }
  __syncthreads();
  if (amax != nullptr) {
    const int g = cb / 16;
    for (int i = threadIdx.x; i < 3 * g; i += blockDim.x) {
      const int k = i / g, gi = i - (i / g) * g;
      const uint32_t val = s_amax[k * 16 + gi];
      if (val) atomicMax(&amax[static_cast<size_t>(n) * amax_stride + amax_goff + (k * c + c0) / 16 + gi], val);
    }
  }
}

constexpr int kMaxLevels = 3;

struct DecodeParams {
  const __half* box[kMaxLevels];  // NHWC [n][h][w][4*reg_max] box-distribution logits (slice)
  const __half* cls[kMaxLevels];  // NHWC [n][h][w][nc] class logits (slice)
  int box_ldc[kMaxLevels], box_coff[kMaxLevels], cls_ldc[kMaxLevels], cls_coff[kMaxLevels];
  int h[kMaxLevels], w[kMaxLevels];
  float stride[kMaxLevels];
  int levels, n, nc, reg_max, anchors;
  float* out;  // [n][4 + nc][anchors]: cx, cy, w, h (input pixels) then class probabilities
};

// One thread per (image, anchor): DFL expectation of each side's distribution
// (softmax over reg_max bins), distance -> box around the anchor centre, and a
// sigmoid per class.  Matches the anchor-free YOLOv8 head (ultralytics Detect).
__global__ void yolo_decode_kernel(const DecodeParams p) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long>(p.n) * p.anchors) return;
  const int img = static_cast<int>(idx / p.anchors);
  int a = static_cast<int>(idx % p.anchors);
  int lv = 0;
  while (lv < p.levels - 1 && a >= p.h[lv] * p.w[lv]) {
    a -= p.h[lv] * p.w[lv];
    ++lv;
  }
  const int gy = a / p.w[lv], gx = a % p.w[lv];
  const long pix = (static_cast<long>(img) * p.h[lv] + gy) * p.w[lv] + gx;
  const __half* bl = p.box[lv] + pix * p.box_ldc[lv] + p.box_coff[lv];
  float dist[4];
  if (p.reg_max == 16 && (reinterpret_cast<uintptr_t>(bl) & 15) == 0) {
    // 64 logits as eight 16-byte loads, all issued before use
    uint4 raw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = reinterpret_cast<const uint4*>(bl)[i];
#pragma unroll
    for (int side = 0; side < 4; ++side) {
      const __half* hv = reinterpret_cast<const __half*>(&raw[2 * side]);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) mx = fmaxf(mx, __half2float(hv[i]));
      float den = 0.f, num = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float e = __expf(__half2float(hv[i]) - mx);
        den += e;
        num += e * static_cast<float>(i);
      }
      dist[side] = num / den;
    }
  } else {
    for (int side = 0; side < 4; ++side) {
      float mx = -INFINITY;
      for (int i = 0; i < p.reg_max; ++i) mx = fmaxf(mx, __half2float(bl[side * p.reg_max + i]));
      float den = 0.f, num = 0.f;
      for (int i = 0; i < p.reg_max; ++i) {
        const float e = __expf(__half2float(bl[side * p.reg_max + i]) - mx);
        den += e;
        num += e * static_cast<float>(i);
      }
      dist[side] = num / den;
    }
  }
  const float cx = gx + 0.5f, cy = gy + 0.5f, st = p.stride[lv];
  const float x1 = cx - dist[0], y1 = cy - dist[1], x2 = cx + dist[2], y2 = cy + dist[3];
  const long plane = p.anchors;
  float* o = p.out + static_cast<long>(img) * (4 + p.nc) * plane + (idx % p.anchors);
  o[0] = (x1 + x2) * 0.5f * st;
  o[plane] = (y1 + y2) * 0.5f * st;
  o[2 * plane] = (x2 - x1) * st;
  o[3 * plane] = (y2 - y1) * st;
  const __half* cl = p.cls[lv] + pix * p.cls_ldc[lv] + p.cls_coff[lv];
  for (int k = 0; k < p.nc; ++k) o[(4 + k) * plane] = 1.0f / (1.0f + __expf(-__half2float(cl[k])));
}

}  // namespace aexrt
