// tcgen05 implicit-GEMM convolution for sm_100a: the W8A8 conv (kernels 51/52/53
// of the reference, native/aexrt_d3d12_runtime.cpp:4614-4923 and the LTS
// variants :3371-3812) and, with kF16, the fp16 convs around it.
//
// GEMM view: M = output pixels of one spatial tile of one image (TH x TW <= 128),
// N = output channels (BN per CTA), K = "slots" of 16 bytes: one slot is one
// kernel tap of one 16-channel slab (int8) or 8-channel slab (fp16).
//
// Activation operand: the int8 (or fp16) activation lives in HBM as
//   [image][slab][H][W][16 bytes]
// so a TMA tiled box (16 B, TW, TH, 1 slab) lands in shared memory as TH*TW
// contiguous 16-byte rows: exactly one K chunk of the canonical K-major
// no-swizzle UMMA layout.  Halo / padding rows come from the TMA's out-of-range
// zero fill.  Stride 2 reads the same bytes through a 5-D view that splits W and
// H into (pair, phase), so every tap of a 3x3/s2 conv is again a plain box.
//
// Weight operand: pre-packed on the host as [slot][OC][16 bytes]; one TMA box
// (16 B, BN, SPS) fills a whole pipeline stage.
//
// Accumulators live in TMEM.  Per-tensor scaling accumulates all of K into one
// buffer; pg16 scaling (INT8_PERGROUP) orders K by (slab, tap) and drains each
// slab's int32 sub-sum from one of two ping-pong TMEM buffers into fp32
// registers, multiplying by that slab's activation scale in ascending group
// order as the reference's LTS kernels do (runtime.cpp:3450-3468, 3594-3618).
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
  int n_img, slabs, in_h, in_w;  // activation view (in_h/in_w: dims of the packed buffer)
  int oc, oh, ow;
  int ksize, stride, pad;
  int tw, th, tiles_w, tiles_h;
  int q_total;  // K slots including pads (even)
  int sps;      // slots per pipeline stage (even)
  int stages;   // pipeline depth
  int kk_p;     // pg16: slots per group (taps rounded up to even)
  int silu;
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

// Epilogue of 8 consecutive output channels of one pixel: scale, bias, SiLU,
// residual, fp16 store; returns the max |fp16 output| bits for the amax.
template <bool kF16>
__device__ __forceinline__ uint32_t epilogue8(const ConvTcParams& p, const float (&acc)[8], int oc_base, bool valid,
                                              size_t pix) {
  float res[8];
  const bool has_res = p.res != nullptr && valid && oc_base < p.oc;
  const bool full8 = oc_base + 8 <= p.oc;  // all 8 channels exist (else only oc < p.oc is touched)
  if (has_res) {
    const __half* rp = p.res + pix * p.res_ldc + p.res_coff + oc_base;
    if (full8 && p.res_vec) {
      const uint4 r = *reinterpret_cast<const uint4*>(rp);
      const __half* rh = reinterpret_cast<const __half*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) res[i] = __half2float(rh[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) res[i] = oc_base + i < p.oc ? __half2float(rp[i]) : 0.0f;
    }
  }
  __align__(16) __half hv[8];
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int oc = oc_base + i;
    float y = 0.0f;
    if (oc < p.oc) {
      y = kF16 ? __fadd_rn(acc[i], p.bias[oc]) : __fadd_rn(__fmul_rn(acc[i], p.w_scale[oc]), p.bias[oc]);
      if (p.silu) {
        const float e = __expf(fminf(-y, 80.0f));
        y = __fdividef(y, 1.0f + e);
      }
      if (has_res) y = __fadd_rn(y, res[i]);
    }
    hv[i] = __float2half_rn(y);
    amax_bits = max(amax_bits, __float_as_uint(fabsf(__half2float(hv[i]))));
  }
  if (valid && oc_base < p.oc) {
    __half* op = p.out + pix * p.out_ldc + p.out_coff + oc_base;
    if (full8 && p.out_vec) {
      *reinterpret_cast<uint4*>(op) = *reinterpret_cast<const uint4*>(hv);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (oc_base + i < p.oc) op[i] = hv[i];
    }
  }
  return valid ? amax_bits : 0u;
}

template <bool kF16, bool kPG, int BN>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap act_map, const __grid_constant__ CUtensorMap w_map,
                   const ConvTcParams p) {
  constexpr int kChanPerSlot = kF16 ? 8 : 16;
  constexpr int kHalf = BN / 2;       // columns per epilogue warp
  constexpr int kChunks = kHalf / 8;  // 8-column chunks per epilogue warp
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN must be a multiple of 16 in [16, 256]");
  static_assert(!kPG || (!kF16 && BN <= 128), "pg16 is int8-only and keeps BN/2 fp32 partials per thread");
  constexpr int kBufs = kPG ? 2 : 1;
  constexpr uint32_t kTmemCols = (kBufs * BN <= 32) ? 32 : (kBufs * BN <= 64) ? 64 : (kBufs * BN <= 128) ? 128 : 256;

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
  const int m_tile = blockIdx.x;
  const int tiles_per_img = p.tiles_w * p.tiles_h;
  const int img = m_tile / tiles_per_img;
  const int t_in = m_tile - img * tiles_per_img;
  const int oh0 = (t_in / p.tiles_w) * p.th;
  const int ow0 = (t_in % p.tiles_w) * p.tw;
  const int n0 = blockIdx.y * BN;

  const int groups = kPG ? p.slabs : 1;
  const int ksteps = p.q_total / 2;
  const int ksteps_per_group = kPG ? p.kk_p / 2 : ksteps;
  const int ksteps_per_stage = p.sps / 2;
  const int stage_iters = (p.q_total + p.sps - 1) / p.sps;

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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&act_map);
    tma_prefetch_desc(&w_map);
  }
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
      const uint32_t tx = static_cast<uint32_t>(p.sps * sp.a_box_bytes + sp.b_stage_bytes);
      for (int it = 0; it < stage_iters; ++it) {
        const int s = it % p.stages;
        if (it >= p.stages) {
          if (!mbar_wait_bounded(&empty[s], ((it / p.stages) - 1) & 1, p.status, kStatusTimeoutEmpty)) break;
        }
        uint8_t* a_dst = smem + s * sp.stage_bytes;
        uint8_t* b_dst = a_dst + sp.a_stage_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        for (int j = 0; j < p.sps; ++j) {
          int slab;
          const int tap = decode_slot<kPG>(p, it * p.sps + j, slab);
          int sn = img * p.slabs + slab;
          int kh = 0, kw = 0;
          if (tap < 0) {
            sn = p.n_img * p.slabs;  // fully out of range: the TMA zero-fills the slot
          } else {
            kh = tap / p.ksize;
            kw = tap - kh * p.ksize;
          }
          void* dst = a_dst + j * sp.a_slot_stride;
          if (p.stride == 1) {
            tma_load_4d(dst, &act_map, &full[s], 0, ow0 + kw - p.pad, oh0 + kh - p.pad, sn);
          } else {
            // input column 2*ow + kw - 1 == 2*(ow + dw) + pw  (same for rows)
            const int pw = (kw + 1) & 1, dw = (kw - 1 - pw) / 2;
            const int ph = (kh + 1) & 1, dh = (kh - 1 - ph) / 2;
            tma_load_5d(dst, &act_map, &full[s], pw * kChanPerSlot, ow0 + dw, ph, oh0 + dh, sn);
          }
        }
        tma_load_3d(b_dst, &w_map, &full[s], 0, n0, it * p.sps);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc<kF16>(BN);
      for (int ks = 0; ks < ksteps; ++ks) {
        const int it = ks / ksteps_per_stage;
        const int j = ks - it * ksteps_per_stage;
        const int s = it % p.stages;
        if (j == 0) {
          if (!mbar_wait_bounded(&full[s], (it / p.stages) & 1, p.status, kStatusTimeoutFull)) break;
          tc_fence_after();
        }
        const int g = ks / ksteps_per_group;
        const int kin = ks - g * ksteps_per_group;
        const int buf = kPG ? (g & 1) : 0;
        if (kPG && kin == 0 && g >= 2) {
          if (!mbar_wait_bounded(&acc_empty[buf], ((g - 2) >> 1) & 1, p.status, kStatusTimeoutAccEmpty)) break;
          tc_fence_after();
        }
        const uint32_t a_addr = smem_u32(smem + s * sp.stage_bytes + (2 * j) * sp.a_slot_stride);
        const uint32_t b_addr = smem_u32(smem + s * sp.stage_bytes + sp.a_stage_bytes + (2 * j) * BN * kSlotBytes);
        const uint64_t a_desc = smem_desc_kmajor_noswizzle(a_addr, sp.a_slot_stride, 128);
        const uint64_t b_desc = smem_desc_kmajor_noswizzle(b_addr, BN * kSlotBytes, 128);
        tc_mma<kF16>(tmem_base + buf * BN, a_desc, b_desc, idesc, kin == 0 ? 0u : 1u);
        if (j == ksteps_per_stage - 1 || ks == ksteps - 1) tc_commit(&empty[s]);
        if (kin == ksteps_per_group - 1) tc_commit(&acc_full[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int colh = (warp - 2) >> 2;  // which half of the BN columns
    const int row = quad * 32 + lane;  // tile row == TMEM lane
    const int r_h = row / p.tw;
    const int r_w = row - r_h * p.tw;
    const int oy = oh0 + r_h, ox = ow0 + r_w;
    const bool valid = row < rows && oy < p.oh && ox < p.ow;
    const size_t npix = static_cast<size_t>(p.n_img) * p.oh * p.ow;
    const size_t pix = (static_cast<size_t>(img) * p.oh + (valid ? oy : 0)) * p.ow + (valid ? ox : 0);
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int col0 = colh * kHalf;
    const float* rec = kF16 ? nullptr : p.scale_rec + static_cast<size_t>(img) * (1 + p.slabs);

    if constexpr (!kPG) {
      if (mbar_wait_bounded(&acc_full[0], 0, p.status, kStatusTimeoutAccFull)) {
        tc_fence_after();
        const float in_scale = kF16 ? 1.0f : __fdiv_rn(rec[0], 127.0f);
#pragma unroll 1
        for (int c = 0; c < kChunks; ++c) {
          uint32_t v[8];
          tmem_ld_x8(lane_addr + col0 + c * 8, v);
          tmem_ld_wait();
          float acc[8];
          const int oc_base = n0 + col0 + c * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            acc[i] = kF16 ? __uint_as_float(v[i]) : __fmul_rn(static_cast<float>(static_cast<int32_t>(v[i])), in_scale);
          }
          if (!kF16 && p.acc_dump != nullptr && valid) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (oc_base + i < p.oc) p.acc_dump[pix * p.oc + oc_base + i] = static_cast<int32_t>(v[i]);
          }
          const uint32_t m = __reduce_max_sync(0xffffffffu, epilogue8<kF16>(p, acc, oc_base, valid, pix));
          if (p.amax_out != nullptr && lane == 0 && oc_base < p.oc) {
            atomicMax(&p.amax_out[static_cast<size_t>(img) * p.amax_stride + p.amax_goff + oc_base / 16], m);
          }
        }
      }
    } else {
      float fp[kHalf];
      bool ok = true;
      for (int g = 0; g < groups; ++g) {
        const int buf = g & 1;
        ok = mbar_wait_bounded(&acc_full[buf], (g >> 1) & 1, p.status, kStatusTimeoutAccFull);
        if (!ok) break;
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
      }
      if (ok) {
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          const int oc_base = n0 + col0 + c * 8;
          float acc[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = fp[c * 8 + i];
          const uint32_t m = __reduce_max_sync(0xffffffffu, epilogue8<false>(p, acc, oc_base, valid, pix));
          if (p.amax_out != nullptr && lane == 0 && oc_base < p.oc) {
            atomicMax(&p.amax_out[static_cast<size_t>(img) * p.amax_stride + p.amax_goff + oc_base / 16], m);
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
