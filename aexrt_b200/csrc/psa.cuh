// The two fp16 ops of the YOLOv11 graphs that stay off the W8A8 path: the depthwise 3x3 conv
// (DWConv in the detect head's class branch, and the positional-encoding conv of the C2PSA
// attention block) and the C2PSA multi-head self-attention over the smallest feature map.  The
// reference keeps both in its generic fp16 kernels: its int8 guard refuses grouped convs
// (native/aexrt_d3d12_runtime.cpp:9404) and attention lowers to MATMUL / SOFTMAX commands
// (runtime.cpp:17305-17307).  Both kernels read and write NHWC fp16 channel slices.
#pragma once
#include "ptx.cuh"
#include <cuda_fp16.h>

#include <cstdint>

namespace aexrt {

// Depthwise 3x3 conv, pad 1, stride 1 or 2: one thread = one output pixel x 8 channels, fp32
// accumulation in (kh, kw) order from the bias, optional SiLU y / (1 + e^-y), fp16 store.
// Output channel c reads input channel coff + (c / grp) * grp_stride + grp_off + c % grp (grp = C
// is a plain slice; the C2PSA positional encoding reads the per-head v channels of the qkv
// tensor).  w9: [9][C] fp32 (fp16-rounded weights), bias: [C] fp32.
__global__ void dwconv3x3_kernel(const __half* __restrict__ x, int n, int h, int w, int c, int ldc, int coff, int grp,
                                 int grp_stride, int grp_off, const float* __restrict__ w9,
                                 const float* __restrict__ bias, int stride, int silu, int oh, int ow,
                                 __half* __restrict__ out, int out_ldc, int out_coff) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  const int vec = c / 8;
  const long total = static_cast<long>(n) * oh * ow * vec;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c0 = static_cast<int>(idx % vec) * 8;
  const long pix = idx / vec;
  const int ox = static_cast<int>(pix % ow);
  const int oy = static_cast<int>((pix / ow) % oh);
  const int img = static_cast<int>(pix / (static_cast<long>(ow) * oh));
  const int ic0 = coff + (c0 / grp) * grp_stride + grp_off + c0 % grp;  // 8 channels never straddle a group
  float acc[8];
  {
    const float4 b0 = *reinterpret_cast<const float4*>(bias + c0);
    const float4 b1 = *reinterpret_cast<const float4*>(bias + c0 + 4);
    acc[0] = b0.x; acc[1] = b0.y; acc[2] = b0.z; acc[3] = b0.w;
    acc[4] = b1.x; acc[5] = b1.y; acc[6] = b1.z; acc[7] = b1.w;
  }
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int iy = oy * stride + kh - 1;
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const int ix = ox * stride + kw - 1;
      if (iy < 0 || iy >= h || ix < 0 || ix >= w) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(x + ((static_cast<long>(img) * h + iy) * w + ix) * ldc + ic0);
      const __half2* hv = reinterpret_cast<const __half2*>(&v);
      const float* wt = w9 + (kh * 3 + kw) * c + c0;
      const float4 w0 = *reinterpret_cast<const float4*>(wt);
      const float4 w1 = *reinterpret_cast<const float4*>(wt + 4);
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hv[i]);
        acc[2 * i] = fmaf(f.x, ww[2 * i], acc[2 * i]);
        acc[2 * i + 1] = fmaf(f.y, ww[2 * i + 1], acc[2 * i + 1]);
      }
    }
  }
  __align__(16) __half2 o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a = acc[2 * i], b = acc[2 * i + 1];
    if (silu) {
      a = a / (1.0f + expf(-a));
      b = b / (1.0f + expf(-b));
    }
    o[i] = __floats2half2_rn(a, b);
  }
  *reinterpret_cast<uint4*>(out + ((static_cast<long>(img) * oh + oy) * ow + ox) * out_ldc + out_coff + c0) =
      *reinterpret_cast<const uint4*>(o);
}

// C2PSA attention (ultralytics Attention: qkv conv -> per head q, k (key_dim) and v (64 channels)
// -> softmax(q^T k * scale) -> v @ attn^T, plus the positional encoding pe(v)), one CTA per
// (head, image).  The head's q, k and v (its 2 * key_dim + 64 consecutive qkv channels of every
// pixel) are staged in shared memory as fp16 (k transposed, so that lanes read consecutive keys);
// each warp takes query pixels in turn: lane-parallel scores over the keys, a warp softmax in
// fp32, then lane l accumulates output channels 2l and 2l + 1 over every key, adds pe and stores
// fp16.  The |y| maxima of each 16-channel group are max-ed into the amax slots of the output
// (the next conv is int8).
constexpr int kPsaThreads = 256;
constexpr int kPsaHeadDim = 64;

__host__ __device__ inline size_t psa_smem_bytes(int l, int kd) {
  // q [L][kd], kT [kd][L], v [L][64] fp16; per-warp probability rows [8][L] fp32; group maxima
  return static_cast<size_t>(l) * kd * 2 * 2 + static_cast<size_t>(l) * kPsaHeadDim * 2 +
         static_cast<size_t>(kPsaThreads / 32) * l * 4 + 16 * 4;
}

__global__ void __launch_bounds__(kPsaThreads) psa_attention_kernel(
    const __half* __restrict__ qkv, int l, int ldc, int coff, int kd, float scale, const __half* __restrict__ pe,
    int pe_ldc, int pe_coff, __half* __restrict__ out, int out_ldc, int out_coff, uint32_t* __restrict__ amax,
    int amax_stride, int amax_goff) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  extern __shared__ __align__(16) uint8_t smem[];
  const int head = blockIdx.x, img = blockIdx.y;
  const int per_head = 2 * kd + kPsaHeadDim;
  __half* sq = reinterpret_cast<__half*>(smem);  // [L][kd]
  __half* skt = sq + static_cast<size_t>(l) * kd;  // [kd][L]
  __half* sv = skt + static_cast<size_t>(l) * kd;  // [L][64]
  float* sp = reinterpret_cast<float*>(sv + static_cast<size_t>(l) * kPsaHeadDim);  // [8][L]
  uint32_t* sgmax = reinterpret_cast<uint32_t*>(sp + static_cast<size_t>(kPsaThreads / 32) * l);  // [4]
  if (threadIdx.x < 4) sgmax[threadIdx.x] = 0u;
  const __half* src = qkv + static_cast<size_t>(img) * l * ldc + coff + head * per_head;
  // stage the head's channels: 8 channels (16 bytes) per load
  const int vecs = per_head / 8;
  for (int e = threadIdx.x; e < l * vecs; e += blockDim.x) {
    const int j = e / vecs, cv = (e - j * vecs) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(j) * ldc + cv);
    const __half* hv = reinterpret_cast<const __half*>(&v);
    if (cv < kd) {
      *reinterpret_cast<uint4*>(sq + static_cast<size_t>(j) * kd + cv) = v;
    } else if (cv < 2 * kd) {
#pragma unroll
      for (int i = 0; i < 8; ++i) skt[static_cast<size_t>(cv - kd + i) * l + j] = hv[i];
    } else {
      *reinterpret_cast<uint4*>(sv + static_cast<size_t>(j) * kPsaHeadDim + cv - 2 * kd) = v;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* prow = sp + static_cast<size_t>(warp) * l;
  float gmax = 0.0f;  // max |y| of this lane's two channels (one 16-channel group per 8 lanes)
  for (int i = warp; i < l; i += kPsaThreads / 32) {
    // scores of query i against keys j = lane + 32 t
    float mx = -INFINITY;
    for (int j0 = 0; j0 < l; j0 += 32) {
      const int j = j0 + lane;
      float s = -INFINITY;
      if (j < l) {
        float acc = 0.0f;
        for (int d = 0; d < kd; ++d)
          acc = fmaf(__half2float(sq[static_cast<size_t>(i) * kd + d]), __half2float(skt[static_cast<size_t>(d) * l + j]), acc);
        s = acc * scale;
        prow[j] = s;
      }
      mx = fmaxf(mx, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int j = lane; j < l; j += 32) {
      const float e = expf(prow[j] - mx);
      prow[j] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    __syncwarp();
    // output channels 2*lane, 2*lane + 1: sum_j p_j * v[j][c]
    float a0 = 0.0f, a1 = 0.0f;
    for (int j = 0; j < l; ++j) {
      const float pj = prow[j] * inv;
      const float2 vv = __half22float2(reinterpret_cast<const __half2*>(sv + static_cast<size_t>(j) * kPsaHeadDim)[lane]);
      a0 = fmaf(pj, vv.x, a0);
      a1 = fmaf(pj, vv.y, a1);
    }
    const int ch = head * kPsaHeadDim + 2 * lane;
    const float2 pv = __half22float2(
        *reinterpret_cast<const __half2*>(pe + (static_cast<size_t>(img) * l + i) * pe_ldc + pe_coff + ch));
    const __half2 y = __floats2half2_rn(a0 + pv.x, a1 + pv.y);
    *reinterpret_cast<__half2*>(out + (static_cast<size_t>(img) * l + i) * out_ldc + out_coff + ch) = y;
    const __half2 ay = __habs2(y);
    gmax = fmaxf(gmax, fmaxf(__low2float(ay), __high2float(ay)));
    __syncwarp();  // prow is rewritten by the next query
  }
  if (amax != nullptr) {
    // lanes 8g .. 8g + 7 hold group g of this head's 64 channels
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
    if ((lane & 7) == 0 && gmax > 0.0f) atomicMax(&sgmax[lane >> 3], __float_as_uint(gmax));
    __syncthreads();
    if (threadIdx.x < 4 && sgmax[threadIdx.x] != 0u)
      atomicMax(&amax[static_cast<size_t>(img) * amax_stride + amax_goff + head * 4 + threadIdx.x], sgmax[threadIdx.x]);
  }
}

}  // namespace aexrt
