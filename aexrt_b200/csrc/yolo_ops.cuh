// The non-convolution ops of the YOLO graphs around the W8A8 path: the SPPF
// max-pool cascade and the detect-head decode (DFL softmax + anchor decode +
// class sigmoid).  Both are small HBM-bound element passes.
#pragma once
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
