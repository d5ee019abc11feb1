// tcgen05 implicit-GEMM convolution for sm_100a: the W8A8 conv (kernels 51/52/53
// of the reference, native/aexrt_d3d12_runtime.cpp:4614-4923 and the LTS
// variants :3371-3812) and, with kF16, the fp16 convs around it.
//
// GEMM view: M = output pixels of one spatial tile of one image (TH x TW <= 128),
// N = output channels (BN per tile), K = "slots" of 16 bytes: one slot is one
// kernel tap of one 16-channel slab (int8) or 8-channel slab (fp16).
//
// Activation operand: the int8 (or fp16) activation lives in HBM as
//   stride-1 consumers: [image][slab][H][W][16 bytes]
//   stride-2 consumers: [image][slab][H][2 (column parity)][W/2][16 bytes]
// so one TMA tiled box of (16*TW bytes, TH rows) -- TW output columns of one
// tap -- lands in shared memory as TH*TW contiguous 16-byte rows: exactly one K
// chunk of the canonical K-major no-swizzle UMMA layout.  A stride-2 tap reads
// one column parity, which the parity-split layout makes contiguous.  Halo and
// padding come from the TMA's out-of-range zero fill.
//
// Weight operand: pre-packed on the host as [n_tile][slot][BN][16 bytes], so a
// stage's worth of B is one contiguous cp.async.bulk copy.
//
// The kernel is persistent (one CTA per SM walks a static list of tiles) and
// keeps two TMEM accumulators, so the epilogue of one accumulation unit overlaps
// the MMAs of the next.  An accumulation unit is a whole tile for per-tensor
// scaling, or one 16-channel input slab for pg16 scaling (INT8_PERGROUP): K is
// then ordered (slab, tap) and each slab's int32 sub-sum is drained into fp32
// registers scaled by that slab's activation scale, in ascending group order as
// the reference's LTS kernels do (runtime.cpp:3450-3468, 3594-3618).
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = TMEM allocator +
// MMA issuer, warps 2..9 = epilogue (each owns one TMEM lane quadrant and one
// half of the BN columns).
#pragma once
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace aexrt {

constexpr int kConvThreads = 320;
constexpr int kSlotBytes = 16;

struct ConvTcParams {
  // geometry
  int n_img, slabs;
  int oc, oh, ow;
  int ksize, stride, pad;
  int tw, th, tiles_w, tiles_h;
  int n_tiles;      // output-channel tiles
  int total_tiles;  // n_img * tiles_h * tiles_w * n_tiles
  int q_total;      // K slots including pads (even)
  int sps;          // slots per pipeline stage (even)
  int stages;       // pipeline depth
  int kk_p;         // pg16: slots per group (taps rounded up to even)
  int silu;
  const uint8_t* w_packed;  // [n_tile][q_total][BN][16]
  // scales (int8 only): per image record [1 + slabs] of fp32 amax values
  const float* scale_rec;
  const float* w_scale;
  const float* bias;
  // optional residual (fp16 NHWC slice), added after SiLU
  const __half* res;
  int res_ldc, res_coff;
  // output (fp16 NHWC slice)
  __half* out;
  int out_ldc, out_coff;
  int out_vec, res_vec;  // 1 when 8-channel (16-byte) vector access is aligned for out / res
  // optional next-layer amax (float bits, per image, per 16-channel group)
  uint32_t* amax_out;
  int amax_stride, amax_goff;
  // optional int32 accumulator dump: per-tensor [pixel][oc]; pg16 [group][pixel][oc]
  int32_t* acc_dump;
  uint32_t* status;
};

// Shared-memory plan of one CTA (identical on host and device).
struct ConvSmemPlan {
  int a_slot_stride;  // bytes between K slots of the A operand (LBO), multiple of 128
  int a_box_bytes;    // bytes one activation TMA box delivers
  int a_stage_bytes;
  int b_stage_bytes;
  int stage_bytes;
  int bar_offset;
  int total_bytes;
};

__host__ __device__ inline ConvSmemPlan conv_smem_plan(int tw, int th, int sps, int stages, int bn) {
  ConvSmemPlan s;
  const int rows = tw * th;
  s.a_slot_stride = ((rows + 7) / 8) * 8 * kSlotBytes;
  s.a_box_bytes = rows * kSlotBytes;
  s.a_stage_bytes = sps * s.a_slot_stride;
  s.b_stage_bytes = sps * bn * kSlotBytes;
  s.stage_bytes = s.a_stage_bytes + s.b_stage_bytes;
  // 2 KB of slack after the stages: an M=128 MMA reads 128 rows from every slot.
  s.bar_offset = stages * s.stage_bytes + 2048;
  s.total_bytes = s.bar_offset + (2 * stages + 4) * 8 + 16;
  return s;
}

struct TileCoord {
  int img, oh0, ow0, n_tile;
};

__device__ __forceinline__ TileCoord tile_coord(const ConvTcParams& p, int t) {
  TileCoord c;
  const int m_tile = t / p.n_tiles;
  c.n_tile = t - m_tile * p.n_tiles;
  const int per_img = p.tiles_w * p.tiles_h;
  c.img = m_tile / per_img;
  const int r = m_tile - c.img * per_img;
  c.oh0 = (r / p.tiles_w) * p.th;
  c.ow0 = (r % p.tiles_w) * p.tw;
  return c;
}

template <bool kPG>
__device__ __forceinline__ int decode_slot(const ConvTcParams& p, int q, int& slab) {
  const int kk = p.ksize * p.ksize;
  int tap;
  if (kPG) {
    slab = q / p.kk_p;
    tap = q - slab * p.kk_p;
    if (tap >= kk || slab >= p.slabs) tap = -1;
  } else {
    tap = q / p.slabs;
    slab = q - tap * p.slabs;
    if (tap >= kk) tap = -1;
  }
  return tap;
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}

__device__ __forceinline__ float tanh_approx(float x) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// SiLU through the identity sigmoid(y) = (1 + tanh(y/2)) / 2: one MUFU op per element.
__device__ __forceinline__ float silu_fast(float y) {
  const float h = 0.5f * y;
  return fmaf(h, tanh_approx(h), h);
}

// Epilogue of 8 consecutive output channels of one pixel: `acc` already holds
// the dequantized sum (int8) or the fp32 accumulator (fp16); applies the
// per-channel scale, bias, SiLU, residual, stores fp16 and returns the max
// |fp16 output| bits for the next layer's amax.
template <bool kF16>
__device__ __forceinline__ uint32_t epilogue8(const ConvTcParams& p, const float (&acc)[8], int oc_base, bool valid,
                                              size_t pix) {
  const bool full8 = oc_base + 8 <= p.oc;  // all 8 channels exist (else only oc < p.oc is touched)
  float wsc[8], bia[8];
  if (full8) {
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + oc_base);
    const float4 b0 = __ldg(b4), b1 = __ldg(b4 + 1);
    bia[0] = b0.x; bia[1] = b0.y; bia[2] = b0.z; bia[3] = b0.w;
    bia[4] = b1.x; bia[5] = b1.y; bia[6] = b1.z; bia[7] = b1.w;
    if (!kF16) {
      const float4* s4 = reinterpret_cast<const float4*>(p.w_scale + oc_base);
      const float4 s0 = __ldg(s4), s1 = __ldg(s4 + 1);
      wsc[0] = s0.x; wsc[1] = s0.y; wsc[2] = s0.z; wsc[3] = s0.w;
      wsc[4] = s1.x; wsc[5] = s1.y; wsc[6] = s1.z; wsc[7] = s1.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      bia[i] = oc_base + i < p.oc ? __ldg(p.bias + oc_base + i) : 0.0f;
      wsc[i] = (!kF16 && oc_base + i < p.oc) ? __ldg(p.w_scale + oc_base + i) : 0.0f;
    }
  }
  float res[8];
  const bool has_res = p.res != nullptr && valid && oc_base < p.oc;
  if (has_res) {
    const __half* rp = p.res + pix * p.res_ldc + p.res_coff + oc_base;
    if (full8 && p.res_vec) {
      const uint4 r = *reinterpret_cast<const uint4*>(rp);
      const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(rh[i]);
        res[2 * i] = f.x;
        res[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) res[i] = oc_base + i < p.oc ? __half2float(rp[i]) : 0.0f;
    }
  }
  __align__(16) __half2 hv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float y[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int k = 2 * i + j;
      float v = kF16 ? acc[k] + bia[k] : fmaf(acc[k], wsc[k], bia[k]);
      if (p.silu) v = silu_fast(v);
      if (has_res) v += res[k];
      y[j] = oc_base + k < p.oc ? v : 0.0f;
    }
    hv[i] = __floats2half2_rn(y[0], y[1]);
  }
  const __half2 m01 = __hmax2(__habs2(hv[0]), __habs2(hv[1]));
  const __half2 m23 = __hmax2(__habs2(hv[2]), __habs2(hv[3]));
  const __half2 m = __hmax2(m01, m23);
  const float amax = fmaxf(__low2float(m), __high2float(m));
  if (valid && oc_base < p.oc) {
    __half* op = p.out + pix * p.out_ldc + p.out_coff + oc_base;
    if (full8 && p.out_vec) {
      *reinterpret_cast<uint4*>(op) = *reinterpret_cast<const uint4*>(hv);
    } else {
      const __half* h = reinterpret_cast<const __half*>(hv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (oc_base + i < p.oc) op[i] = h[i];
    }
  }
  return valid ? __float_as_uint(amax) : 0u;
}

template <bool kF16, bool kPG, int BN>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap act_map, const ConvTcParams p) {
  constexpr int kHalf = BN / 2;       // columns per epilogue warp
  constexpr int kChunks = kHalf / 8;  // 8-column chunks per epilogue warp
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN must be a multiple of 16 in [16, 256]");
  static_assert(!kPG || (!kF16 && BN <= 128), "pg16 is int8-only and keeps BN/2 fp32 partials per thread");
  constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;

  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const ConvSmemPlan sp = conv_smem_plan(p.tw, p.th, p.sps, p.stages, BN);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bar_offset);  // [stages]
  uint64_t* empty = full + p.stages;                                     // [stages]
  uint64_t* acc_full = full + 2 * p.stages;                              // [2]
  uint64_t* acc_empty = acc_full + 2;                                    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int rows = p.th * p.tw;
  const int ksteps_per_unit = kPG ? p.kk_p / 2 : p.q_total / 2;
  const size_t w_tile_bytes = static_cast<size_t>(p.q_total) * BN * kSlotBytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&act_map);
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = tile_coord(p, t);
        const uint8_t* w_tile = p.w_packed + static_cast<size_t>(tc.n_tile) * w_tile_bytes;
        for (int q0 = 0; q0 < p.q_total; q0 += p.sps, ++it) {
          const int s = it % p.stages;
          if (it >= p.stages && !mbar_wait_bounded(&empty[s], ((it / p.stages) - 1) & 1, p.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int rem = min(p.sps, p.q_total - q0);
          uint8_t* a_dst = smem + s * sp.stage_bytes;
          uint8_t* b_dst = a_dst + sp.a_stage_bytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rem * (sp.a_box_bytes + BN * kSlotBytes)));
          for (int j = 0; j < rem; ++j) {
            int slab;
            const int tap = decode_slot<kPG>(p, q0 + j, slab);
            int sn = tc.img * p.slabs + slab;
            int kh = 0, kw = 0;
            if (tap < 0) {
              sn = p.n_img * p.slabs;  // fully out of range: the TMA zero-fills the slot
            } else {
              kh = tap / p.ksize;
              kw = tap - kh * p.ksize;
            }
            void* dst = a_dst + j * sp.a_slot_stride;
            if (p.stride == 1) {
              tma_load_3d(dst, &act_map, &full[s], kSlotBytes / (kF16 ? 2 : 1) * (tc.ow0 + kw - p.pad),
                          tc.oh0 + kh - p.pad, sn);
            } else {
              // input column 2*ow + kw - 1 == 2*(ow + dw) + pw  (same for rows)
              const int pw = (kw + 1) & 1, dw = (kw - 1 - pw) / 2;
              const int ph = (kh + 1) & 1, dh = (kh - 1 - ph) / 2;
              tma_load_5d(dst, &act_map, &full[s], kSlotBytes / (kF16 ? 2 : 1) * (tc.ow0 + dw), pw, ph, tc.oh0 + dh, sn);
            }
          }
          bulk_load(b_dst, w_tile + static_cast<size_t>(q0) * BN * kSlotBytes, static_cast<uint32_t>(rem * BN * kSlotBytes),
                    &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc<kF16>(BN);
      int it = 0, u = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        for (int q0 = 0; q0 < p.q_total && ok; q0 += p.sps, ++it) {
          const int s = it % p.stages;
          if (!mbar_wait_bounded(&full[s], (it / p.stages) & 1, p.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int rem = min(p.sps, p.q_total - q0);
          const uint32_t a_base = smem_u32(smem + s * sp.stage_bytes);
          const uint32_t b_base = a_base + sp.a_stage_bytes;
          for (int j = 0; j < rem / 2; ++j) {
            const int ks = q0 / 2 + j;
            const int kin = ks % ksteps_per_unit;
            const int buf = u & 1;
            if (kin == 0 && u >= 2) {
              if (!mbar_wait_bounded(&acc_empty[buf], ((u - 2) >> 1) & 1, p.status, kStatusTimeoutAccEmpty)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            const uint64_t a_desc = smem_desc_kmajor_noswizzle(a_base + 2 * j * sp.a_slot_stride, sp.a_slot_stride, 128);
            const uint64_t b_desc = smem_desc_kmajor_noswizzle(b_base + 2 * j * BN * kSlotBytes, BN * kSlotBytes, 128);
            tc_mma<kF16>(tmem_base + buf * BN, a_desc, b_desc, idesc, kin == 0 ? 0u : 1u);
            if (kin == ksteps_per_unit - 1) {
              tc_commit(&acc_full[buf]);
              ++u;
            }
          }
          tc_commit(&empty[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int colh = (warp - 2) >> 2;  // which half of the BN columns
    const int row = quad * 32 + lane;  // tile row == TMEM lane
    const int r_h = row / p.tw;
    const int r_w = row - r_h * p.tw;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int col0 = colh * kHalf;
    const size_t npix = static_cast<size_t>(p.n_img) * p.oh * p.ow;
    int u = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      const TileCoord tc = tile_coord(p, t);
      const int oy = tc.oh0 + r_h, ox = tc.ow0 + r_w;
      const bool valid = row < rows && oy < p.oh && ox < p.ow;
      const size_t pix = (static_cast<size_t>(tc.img) * p.oh + (valid ? oy : 0)) * p.ow + (valid ? ox : 0);
      const int n0 = tc.n_tile * BN;
      const float* rec = kF16 ? nullptr : p.scale_rec + static_cast<size_t>(tc.img) * (1 + p.slabs);

      if constexpr (!kPG) {
        const int buf = u & 1;
        if (!mbar_wait_bounded(&acc_full[buf], (u >> 1) & 1, p.status, kStatusTimeoutAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float in_scale = kF16 ? 1.0f : __fdiv_rn(rec[0], 127.0f);
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          uint32_t v[8];
          tmem_ld_x8(lane_addr + buf * BN + col0 + c * 8, v);
          tmem_ld_wait();
          if (c == kChunks - 1) {
            // every column of this accumulator has been read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          const int oc_base = n0 + col0 + c * 8;
          float acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            acc[i] = kF16 ? __uint_as_float(v[i]) : __fmul_rn(static_cast<float>(static_cast<int32_t>(v[i])), in_scale);
          if (!kF16 && p.acc_dump != nullptr && valid) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (oc_base + i < p.oc) p.acc_dump[pix * p.oc + oc_base + i] = static_cast<int32_t>(v[i]);
          }
          const uint32_t m = __reduce_max_sync(0xffffffffu, epilogue8<kF16>(p, acc, oc_base, valid, pix));
          if (p.amax_out != nullptr && lane == 0 && oc_base < p.oc && m != 0u) {
            atomicMax(&p.amax_out[static_cast<size_t>(tc.img) * p.amax_stride + p.amax_goff + oc_base / 16], m);
          }
        }
        ++u;
      } else {
        float fp[kHalf];
        for (int g = 0; g < p.slabs; ++g) {
          const int buf = u & 1;
          if (!mbar_wait_bounded(&acc_full[buf], (u >> 1) & 1, p.status, kStatusTimeoutAccFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float gs = __fdiv_rn(rec[1 + g], 127.0f);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            uint32_t v[8];
            tmem_ld_x8(lane_addr + buf * BN + col0 + c * 8, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float term = __fmul_rn(static_cast<float>(static_cast<int32_t>(v[i])), gs);
              fp[c * 8 + i] = g == 0 ? term : __fadd_rn(fp[c * 8 + i], term);
            }
            if (p.acc_dump != nullptr && valid) {
              const int oc_base = n0 + col0 + c * 8;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (oc_base + i < p.oc)
                  p.acc_dump[(static_cast<size_t>(g) * npix + pix) * p.oc + oc_base + i] = static_cast<int32_t>(v[i]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
          ++u;
        }
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          const int oc_base = n0 + col0 + c * 8;
          float acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = fp[c * 8 + i];
          const uint32_t m = __reduce_max_sync(0xffffffffu, epilogue8<false>(p, acc, oc_base, valid, pix));
          if (p.amax_out != nullptr && lane == 0 && oc_base < p.oc && m != 0u) {
            atomicMax(&p.amax_out[static_cast<size_t>(tc.img) * p.amax_stride + p.amax_goff + oc_base / 16], m);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace aexrt
