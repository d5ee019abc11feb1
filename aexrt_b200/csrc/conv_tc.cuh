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

template <int CW>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[CW]) {
  static_assert(CW == 8 || CW == 16, "8 or 16 columns");
  if constexpr (CW == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
  } else {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
  }
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

__device__ __forceinline__ void load8f(const float* src, bool full, int n_valid, float (&dst)[8]) {
  if (full) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
    dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = i < n_valid ? __ldg(src + i) : 0.0f;
  }
}

// Epilogue of 8 consecutive output channels of one pixel: `acc` holds the
// dequantized sum (int8: already multiplied by the activation scale) or the
// fp32 accumulator (fp16); applies the per-channel weight scale, bias, SiLU,
// residual, stores fp16 and returns the max |fp16 output| for the next
// layer's amax.
template <bool kF16>
__device__ __forceinline__ float epilogue8(const ConvTcParams& p, const float (&acc)[8], int oc_base, bool valid,
                                           size_t pix) {
  const int n_valid = p.oc - oc_base;
  const bool full8 = n_valid >= 8;
  float wsc[8], bia[8];
  load8f(p.bias + oc_base, full8, n_valid, bia);
  if (!kF16) load8f(p.w_scale + oc_base, full8, n_valid, wsc);
  float res[8];
  const bool has_res = p.res != nullptr && valid && n_valid > 0;
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
      for (int i = 0; i < 8; ++i) res[i] = i < n_valid ? __half2float(rp[i]) : 0.0f;
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
      y[j] = k < n_valid ? v : 0.0f;
    }
    hv[i] = __floats2half2_rn(y[0], y[1]);
  }
  const __half2 m = __hmax2(__hmax2(__habs2(hv[0]), __habs2(hv[1])), __hmax2(__habs2(hv[2]), __habs2(hv[3])));
  if (valid && n_valid > 0) {
    __half* op = p.out + pix * p.out_ldc + p.out_coff + oc_base;
    if (full8 && p.out_vec) {
      *reinterpret_cast<uint4*>(op) = *reinterpret_cast<const uint4*>(hv);
    } else {
      const __half* h = reinterpret_cast<const __half*>(hv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < n_valid) op[i] = h[i];
    }
  }
  return valid ? fmaxf(__low2float(m), __high2float(m)) : 0.0f;
}

// Warp-wide max of the per-lane amax of one 16-channel group (or 8-channel
// half of one) and a single atomic per warp.
__device__ __forceinline__ void amax_commit(const ConvTcParams& p, float m, int img, int oc_base, int lane) {
  const uint32_t r = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
  if (p.amax_out != nullptr && lane == 0 && oc_base < p.oc && r != 0u)
    atomicMax(&p.amax_out[static_cast<size_t>(img) * p.amax_stride + p.amax_goff + oc_base / 16], r);
}

template <bool kF16, bool kPG, int BN>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap act_map, const ConvTcParams p) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  constexpr int kHalf = BN / 2;                  // columns per epilogue warp
  constexpr int CW = kHalf >= 16 ? 16 : 8;       // columns per TMEM load
  constexpr int kChunks = kHalf / CW;
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
  const int stages_per_tile = (p.q_total + p.sps - 1) / p.sps;

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
  // each persistent CTA takes one contiguous run of tiles, so consecutive tiles of one image
  // fold their |y| maxima in registers before one atomic per image and group
  const int t_begin = static_cast<int>(static_cast<long long>(blockIdx.x) * p.total_tiles / gridDim.x);
  const int t_end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.total_tiles / gridDim.x);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane j issues the TMA box of slot j of the stage (slots decode in
    // parallel); lane 0 also arms the barrier and issues the weight copy.
    const size_t w_tile_bytes = static_cast<size_t>(p.q_total) * BN * kSlotBytes;
    const int x_per_px = kSlotBytes / (kF16 ? 2 : 1);  // tensor-map elements per pixel of one slab
    int s = 0, it = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int t = t_begin; t < t_end && ok; ++t) {
      const TileCoord tc = tile_coord(p, t);
      const uint8_t* w_tile = p.w_packed + static_cast<size_t>(tc.n_tile) * w_tile_bytes;
      for (int st = 0, q0 = 0; st < stages_per_tile; ++st, q0 += p.sps) {
        if (it >= p.stages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.status, kStatusTimeoutEmpty)) {
          ok = false;
          break;
        }
        const int rem = min(p.sps, p.q_total - q0);
        uint8_t* a_dst = smem + s * sp.stage_bytes;
        if (lane == 0)
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rem * (sp.a_box_bytes + BN * kSlotBytes)));
        __syncwarp();
        if (lane < rem) {
          int slab;
          const int tap = decode_slot<kPG>(p, q0 + lane, slab);
          int sn = tc.img * p.slabs + slab;
          int kh = 0, kw = 0;
          if (tap < 0) {
            sn = p.n_img * p.slabs;  // fully out of range: the TMA zero-fills the slot
          } else {
            kh = tap / p.ksize;
            kw = tap - kh * p.ksize;
          }
          void* dst = a_dst + lane * sp.a_slot_stride;
          if (p.stride == 1) {
            tma_load_3d(dst, &act_map, &full[s], x_per_px * (tc.ow0 + kw - p.pad), tc.oh0 + kh - p.pad, sn);
          } else {
            // input column 2*ow + kw - 1 == 2*(ow + dw) + pw  (same for rows)
            const int pw = (kw + 1) & 1, dw = (kw - 1 - pw) / 2;
            const int ph2 = (kh + 1) & 1, dh = (kh - 1 - ph2) / 2;
            tma_load_5d(dst, &act_map, &full[s], x_per_px * (tc.ow0 + dw), pw, ph2, tc.oh0 + dh, sn);
          }
        }
        if (lane == 0)
          bulk_load(a_dst + sp.a_stage_bytes, w_tile + static_cast<size_t>(q0) * BN * kSlotBytes,
                    static_cast<uint32_t>(rem * BN * kSlotBytes), &full[s]);
        ++it;
        if (++s == p.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc<kF16>(BN);
      const int ksteps_per_unit = kPG ? p.kk_p / 2 : p.q_total / 2;
      const uint32_t smem_base = smem_u32(smem);
      const uint64_t a_desc0 = smem_desc_kmajor_noswizzle(smem_base, sp.a_slot_stride, 128);
      const uint64_t b_desc0 = smem_desc_kmajor_noswizzle(smem_base + sp.a_stage_bytes, BN * kSlotBytes, 128);
      const uint64_t a_inc = static_cast<uint64_t>((2 * sp.a_slot_stride) >> 4);
      const uint64_t b_inc = static_cast<uint64_t>((2 * BN * kSlotBytes) >> 4);
      const uint64_t stage_inc = static_cast<uint64_t>(sp.stage_bytes >> 4);
      int s = 0, u = 0, kin = 0, buf = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t) {
        for (int st = 0, q0 = 0; st < stages_per_tile; ++st, q0 += p.sps) {
          if (!mbar_wait_bounded(&full[s], ph, p.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int ksteps = min(p.sps, p.q_total - q0) >> 1;
          uint64_t ad = a_desc0 + s * stage_inc;
          uint64_t bd = b_desc0 + s * stage_inc;
          for (int j = 0; j < ksteps; ++j) {
            if (kin == 0) {
              buf = u & 1;
              if (u >= 2) {
                if (!mbar_wait_bounded(&acc_empty[buf], ((u - 2) >> 1) & 1, p.status, kStatusTimeoutAccEmpty)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
              }
            }
            tc_mma<kF16>(tmem_base + buf * BN, ad, bd, idesc, kin == 0 ? 0u : 1u);
            ad += a_inc;
            bd += b_inc;
            if (++kin == ksteps_per_unit) {
              tc_commit(&acc_full[buf]);
              ++u;
              kin = 0;
            }
          }
          tc_commit(&empty[s]);
          if (++s == p.stages) {
            s = 0;
            ph ^= 1u;
          }
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
    float run_max[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) run_max[c] = 0.0f;
    int run_key = -1, run_img = 0, run_oc = 0;  // (image, n-tile) the maxima belong to
    auto flush_amax = [&]() {
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        amax_commit(p, run_max[c], run_img, run_oc + c * CW, lane);
        run_max[c] = 0.0f;
      }
    };
    for (int t = t_begin; t < t_end && ok; ++t) {
      const TileCoord tc = tile_coord(p, t);
      if (!kPG && p.amax_out != nullptr && tc.img * p.n_tiles + tc.n_tile != run_key) {
        if (run_key >= 0) flush_amax();
        run_key = tc.img * p.n_tiles + tc.n_tile;
        run_img = tc.img;
        run_oc = tc.n_tile * BN + col0;
      }
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
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          uint32_t v[CW];
          tmem_ld<CW>(lane_addr + buf * BN + col0 + c * CW, v);
          tmem_ld_wait();
          if (c == kChunks - 1) {
            // every column of this accumulator has been read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          const int oc_c = n0 + col0 + c * CW;
          if (!kF16 && p.acc_dump != nullptr && valid) {
#pragma unroll
            for (int i = 0; i < CW; ++i)
              if (oc_c + i < p.oc) p.acc_dump[pix * p.oc + oc_c + i] = static_cast<int32_t>(v[i]);
          }
          float m = 0.0f;
#pragma unroll
          for (int h8 = 0; h8 < CW / 8; ++h8) {
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t bits = v[h8 * 8 + i];
              acc[i] = kF16 ? __uint_as_float(bits) : static_cast<float>(static_cast<int32_t>(bits)) * in_scale;
            }
            m = fmaxf(m, epilogue8<kF16>(p, acc, oc_c + h8 * 8, valid, pix));
          }
          run_max[c] = fmaxf(run_max[c], m);
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
            uint32_t v[CW];
            tmem_ld<CW>(lane_addr + buf * BN + col0 + c * CW, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < CW; ++i) {
              // fp += fl32(S) * gs, one fused multiply-add per group in ascending order
              const float sv = static_cast<float>(static_cast<int32_t>(v[i]));
              fp[c * CW + i] = g == 0 ? __fmul_rn(sv, gs) : fmaf(sv, gs, fp[c * CW + i]);
            }
            if (p.acc_dump != nullptr && valid) {
              const int oc_c = n0 + col0 + c * CW;
#pragma unroll
              for (int i = 0; i < CW; ++i)
                if (oc_c + i < p.oc)
                  p.acc_dump[(static_cast<size_t>(g) * npix + pix) * p.oc + oc_c + i] = static_cast<int32_t>(v[i]);
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
          const int oc_c = n0 + col0 + c * CW;
          float m = 0.0f;
#pragma unroll
          for (int h8 = 0; h8 < CW / 8; ++h8) {
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fp[c * CW + h8 * 8 + i];
            m = fmaxf(m, epilogue8<false>(p, acc, oc_c + h8 * 8, valid, pix));
          }
          amax_commit(p, m, tc.img, oc_c, lane);  // pg16 keeps its registers for the partial sums
        }
      }
    }
    if (!kPG && p.amax_out != nullptr && run_key >= 0) flush_amax();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace aexrt
