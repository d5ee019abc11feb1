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

// Depthwise 3x3 conv, pad 1, stride 1 or 2: one thread = kDwRun consecutive output pixels of a row
// x 8 channels.  Per kernel row the thread loads the input row segment its pixels cover once (16-byte
// loads, coalesced across the channel groups of a pixel) and that row's three taps of its weights,
// so inputs and weights are reused across the run instead of reloaded per pixel.  fp32 accumulation
// from the bias in (kh, kw) order, optional SiLU y / (1 + e^-y), fp16 stores.  Output channel c reads
// input channel coff + (c / grp) * grp_stride + grp_off + c % grp (grp = C is a plain slice; the C2PSA
// positional encoding reads the per-head v channels of the qkv tensor).  w9: [9][C] fp32
// (fp16-rounded weights), bias: [C] fp32.
constexpr int kDwRun = 4;

template <int S>
__global__ void __launch_bounds__(256) dwconv3x3_kernel(const __half* __restrict__ x, int n, int h, int w, int c,
                                                        int ldc, int coff, int grp, int grp_stride, int grp_off,
                                                        const float* __restrict__ w9, const float* __restrict__ bias,
                                                        int silu, int oh, int ow, __half* __restrict__ out, int out_ldc,
                                                        int out_coff) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  constexpr int kSeg = (kDwRun - 1) * S + 3;  // input columns of one kernel row
  const int vec = c / 8;
  const int runs = (ow + kDwRun - 1) / kDwRun;
  const long total = static_cast<long>(n) * oh * runs * vec;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c0 = static_cast<int>(idx % vec) * 8;
  const long rr = idx / vec;
  const int ox0 = static_cast<int>(rr % runs) * kDwRun;
  const int oy = static_cast<int>((rr / runs) % oh);
  const int img = static_cast<int>(rr / (static_cast<long>(runs) * oh));
  const int ic0 = coff + (c0 / grp) * grp_stride + grp_off + c0 % grp;  // 8 channels never straddle a group
  float acc[kDwRun][8];
  {
    const float4 b0 = *reinterpret_cast<const float4*>(bias + c0);
    const float4 b1 = *reinterpret_cast<const float4*>(bias + c0 + 4);
#pragma unroll
    for (int r = 0; r < kDwRun; ++r) {
      acc[r][0] = b0.x; acc[r][1] = b0.y; acc[r][2] = b0.z; acc[r][3] = b0.w;
      acc[r][4] = b1.x; acc[r][5] = b1.y; acc[r][6] = b1.z; acc[r][7] = b1.w;
    }
  }
  const int ix0 = ox0 * S - 1;
#pragma unroll
  for (int kh = 0; kh < 3; ++kh) {
    const int iy = oy * S + kh - 1;
    if (iy < 0 || iy >= h) continue;
    const __half* row = x + (static_cast<long>(img) * h + iy) * w * static_cast<long>(ldc) + ic0;
    uint4 seg[kSeg];
#pragma unroll
    for (int j = 0; j < kSeg; ++j) {
      const int ix = ix0 + j;
      seg[j] = (ix >= 0 && ix < w) ? *reinterpret_cast<const uint4*>(row + static_cast<long>(ix) * ldc)
                                   : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int kw = 0; kw < 3; ++kw) {
      const float* wt = w9 + (kh * 3 + kw) * c + c0;
      const float4 w0 = *reinterpret_cast<const float4*>(wt);
      const float4 w1 = *reinterpret_cast<const float4*>(wt + 4);
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int r = 0; r < kDwRun; ++r) {
        // padding taps read zeros, which add exact zeros (fma(0, w, acc) == acc for finite w)
        const __half2* hv = reinterpret_cast<const __half2*>(&seg[r * S + kw]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(hv[i]);
          acc[r][2 * i] = fmaf(f.x, ww[2 * i], acc[r][2 * i]);
          acc[r][2 * i + 1] = fmaf(f.y, ww[2 * i + 1], acc[r][2 * i + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kDwRun; ++r) {
    if (ox0 + r >= ow) break;
    __align__(16) __half2 o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = acc[r][2 * i], b = acc[r][2 * i + 1];
      if (silu) {
        a = a / (1.0f + expf(-a));
        b = b / (1.0f + expf(-b));
      }
      o[i] = __floats2half2_rn(a, b);
    }
    *reinterpret_cast<uint4*>(out + ((static_cast<long>(img) * oh + oy) * ow + ox0 + r) * out_ldc + out_coff + c0) =
        *reinterpret_cast<const uint4*>(o);
  }
}

// C2PSA attention (ultralytics Attention: qkv conv -> per head q, k (key_dim) and v (64 channels)
// -> softmax(q^T k * scale) -> v @ attn^T, plus the positional encoding pe(v)), one CTA per
// (head, image, query split: gridDim.z CTAs share a head's queries, so that small batches still
// fill the SMs).  The head's q, k and v (its 2 * key_dim + 64 consecutive qkv channels of every
// pixel) are staged in shared memory as fp16; k rows are padded by 16 bytes so that eight lanes
// reading eight keys' 16-byte chunks hit eight bank groups.  Each warp takes kPsaQ query pixels at
// a time, so every key and value load serves kPsaQ queries: lane-parallel scores over the keys
// (in chunks of 128 keys, 8 key dims per load), a warp softmax per query in fp32, then lane l
// accumulates output channels 2l and 2l + 1 of all kPsaQ queries over every key, adds pe and stores
// fp16.  The |y| maxima of each 16-channel group are max-ed into the amax slots of the output (the
// next conv is int8).
constexpr int kPsaThreads = 256;
constexpr int kPsaHeadDim = 64;
constexpr int kPsaQ = 4;  // queries per warp pass

__host__ __device__ inline size_t psa_smem_bytes(int l, int kd) {
  // q [L][kd], k [L][kd + 8], v [L][64] fp16; per-warp probabilities [8][L][kPsaQ] fp32; group maxima
  return static_cast<size_t>(l) * kd * 2 + static_cast<size_t>(l) * (kd + 8) * 2 +
         static_cast<size_t>(l) * kPsaHeadDim * 2 + static_cast<size_t>(kPsaThreads / 32) * l * kPsaQ * 4 + 16 * 4;
}

__device__ __forceinline__ void psa_h8_to_f8(const uint4& v, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
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
  const int kstride = kd + 8;  // halfs per padded k row
  __half* sq = reinterpret_cast<__half*>(smem);                    // [L][kd]
  __half* sk = sq + static_cast<size_t>(l) * kd;                   // [L][kd + 8]
  __half* sv = sk + static_cast<size_t>(l) * kstride;              // [L][64]
  float* sp = reinterpret_cast<float*>(sv + static_cast<size_t>(l) * kPsaHeadDim);  // [8][L][kPsaQ]
  uint32_t* sgmax = reinterpret_cast<uint32_t*>(sp + static_cast<size_t>(kPsaThreads / 32) * l * kPsaQ);  // [4]
  if (threadIdx.x < 4) sgmax[threadIdx.x] = 0u;
  const __half* src = qkv + static_cast<size_t>(img) * l * ldc + coff + head * per_head;
  // stage the head's channels: 8 channels (16 bytes) per load
  const int vecs = per_head / 8;
  for (int e = threadIdx.x; e < l * vecs; e += blockDim.x) {
    const int j = e / vecs, cv = (e - j * vecs) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(j) * ldc + cv);
    if (cv < kd) {
      *reinterpret_cast<uint4*>(sq + static_cast<size_t>(j) * kd + cv) = v;
    } else if (cv < 2 * kd) {
      *reinterpret_cast<uint4*>(sk + static_cast<size_t>(j) * kstride + cv - kd) = v;
    } else {
      *reinterpret_cast<uint4*>(sv + static_cast<size_t>(j) * kPsaHeadDim + cv - 2 * kd) = v;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* prow = sp + static_cast<size_t>(warp) * l * kPsaQ;  // [L][kPsaQ]
  float gmax = 0.0f;  // max |y| of this lane's two channels (one 16-channel group per 8 lanes)
  const int qstep = (kPsaThreads / 32) * kPsaQ * static_cast<int>(gridDim.z);
  for (int i0 = (static_cast<int>(blockIdx.z) * (kPsaThreads / 32) + warp) * kPsaQ; i0 < l; i0 += qstep) {
    int qi[kPsaQ];  // the pass's queries (a short last pass repeats its last query; only real ones are stored)
#pragma unroll
    for (int q = 0; q < kPsaQ; ++q) qi[q] = min(i0 + q, l - 1);
    // scores, 128 keys (4 per lane) at a time
    for (int j0 = 0; j0 < l; j0 += 128) {
      float acc[kPsaQ][4];
#pragma unroll
      for (int q = 0; q < kPsaQ; ++q)
#pragma unroll
        for (int t = 0; t < 4; ++t) acc[q][t] = 0.0f;
      for (int d = 0; d < kd; d += 8) {
        float kf[4][8];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int j = min(j0 + 32 * t + lane, l - 1);
          psa_h8_to_f8(*reinterpret_cast<const uint4*>(sk + static_cast<size_t>(j) * kstride + d), kf[t]);
        }
#pragma unroll
        for (int q = 0; q < kPsaQ; ++q) {
          float qf[8];
          psa_h8_to_f8(*reinterpret_cast<const uint4*>(sq + static_cast<size_t>(qi[q]) * kd + d), qf);
#pragma unroll
          for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[q][t] = fmaf(qf[e], kf[t][e], acc[q][t]);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int j = j0 + 32 * t + lane;
        if (j < l)
          *reinterpret_cast<float4*>(prow + static_cast<size_t>(j) * kPsaQ) =
              make_float4(acc[0][t] * scale, acc[1][t] * scale, acc[2][t] * scale, acc[3][t] * scale);
      }
    }
    __syncwarp();
    // softmax over the keys, per query (unnormalised exponentials stored; 1/sum kept)
    float inv[kPsaQ];
#pragma unroll
    for (int q = 0; q < kPsaQ; ++q) {
      float mx = -INFINITY;
      for (int j = lane; j < l; j += 32) mx = fmaxf(mx, prow[static_cast<size_t>(j) * kPsaQ + q]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sum = 0.0f;
      for (int j = lane; j < l; j += 32) {
        const float e = expf(prow[static_cast<size_t>(j) * kPsaQ + q] - mx);
        prow[static_cast<size_t>(j) * kPsaQ + q] = e;
        sum += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      inv[q] = 1.0f / sum;
    }
    __syncwarp();
    // output channels 2*lane, 2*lane + 1 of every query: sum_j p_qj * v[j][c]
    float a0[kPsaQ], a1[kPsaQ];
#pragma unroll
    for (int q = 0; q < kPsaQ; ++q) a0[q] = a1[q] = 0.0f;
    for (int j = 0; j < l; ++j) {
      const float4 pj = *reinterpret_cast<const float4*>(prow + static_cast<size_t>(j) * kPsaQ);
      const float pq[kPsaQ] = {pj.x, pj.y, pj.z, pj.w};
      const float2 vv = __half22float2(reinterpret_cast<const __half2*>(sv + static_cast<size_t>(j) * kPsaHeadDim)[lane]);
#pragma unroll
      for (int q = 0; q < kPsaQ; ++q) {
        a0[q] = fmaf(pq[q], vv.x, a0[q]);
        a1[q] = fmaf(pq[q], vv.y, a1[q]);
      }
    }
    const int ch = head * kPsaHeadDim + 2 * lane;
#pragma unroll
    for (int q = 0; q < kPsaQ; ++q) {
      if (i0 + q >= l) break;
      const int i = i0 + q;
      const float2 pv = __half22float2(
          *reinterpret_cast<const __half2*>(pe + (static_cast<size_t>(img) * l + i) * pe_ldc + pe_coff + ch));
      const __half2 y = __floats2half2_rn(a0[q] * inv[q] + pv.x, a1[q] * inv[q] + pv.y);
      *reinterpret_cast<__half2*>(out + (static_cast<size_t>(img) * l + i) * out_ldc + out_coff + ch) = y;
      const __half2 ay = __habs2(y);
      gmax = fmaxf(gmax, fmaxf(__low2float(ay), __high2float(ay)));
    }
    __syncwarp();  // prow is rewritten by the next pass
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
