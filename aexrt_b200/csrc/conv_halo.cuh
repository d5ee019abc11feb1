// Halo-tile tcgen05 convolution: the per-tensor W8A8 conv (kernels 51/52/53,
// native/aexrt_d3d12_runtime.cpp:4614-4762) and the fp16 convs, with the whole
// weight tile resident in shared memory and each activation slab loaded ONCE
// per output tile.
//
// Each output tile is TH rows x TW columns of one image, computed on an M grid
// of TH rows with a row pitch P >= TW (the extra columns are junk rows of the
// MMA that the epilogue drops).  For a stride-1 3x3 conv the tile's input halo
// ((TH+2) x P pixels of one 16-byte slab chunk) is one TMA box; the MMA of tap
// (kh, kw) reads that halo through a descriptor whose start address is shifted
// by kh*P + kw rows -- the canonical K-major no-swizzle UMMA layout only needs
// 16-byte aligned starts, so a shifted window is itself a valid operand.  A
// stride-2 conv loads the halo of each of the four (row, column) parities of
// the parity-split input layout ((TH+1) x P pixels each, P = TW+1) and a tap
// reads its parity's halo with a shift of 0 or 1 row/column.  A 1x1 conv loads
// the TH x TW tile itself.
//
// One MMA K step covers two 16-byte chunks: the same pixel window of two
// consecutive slabs (LBO = bytes of one slab's halo).  Pipeline stages carry
// the halo of one slab pair; all K of the CTA's output-channel tile
// ([slab pair][tap][2][BN][16 B]) stays resident.  Activation traffic from L2
// drops from 9x the input (one box per tap) to ~1.3x (one halo per tile), and
// weight traffic to one copy per CTA.
#pragma once
#include "codes.cuh"
#include "conv_tc.cuh"

namespace aexrt {

// Quantize on load: an int8 plan can read fp16 NHWC sources (the producers' outputs, a
// concatenation of up to kQlMaxParts slices, each optionally read through a nearest 2x upsample)
// instead of pre-quantized slab16 codes.  The producer warp loads each slab's fp16 box into a raw
// ring; kQlWarps converter warps turn it into int8 codes in the A stage (the quantizer's arithmetic:
// code = low byte of round_half_even(fl32(x * fl32(127 / amax))), 0 when amax <= 0) and hand the
// stage to the MMA.  The activation scales come from the producers' amax slots, so the separate
// quantize launch and its int8 write + read disappear.
constexpr int kQlMaxParts = 4;
constexpr int kQlMaxRaw = 4;
constexpr int kQlWarps = 4;

struct ConvHaloParams {
  int n_img, slabs, slab_pairs;
  int oc, oh, ow;
  int ksize, stride;
  int tw, th, pitch;        // output tile and M-grid row pitch
  int halo_rows;            // rows (pixels) of one halo box
  int boxes_per_slab;       // 1 (s1, 1x1) or 4 (s2 parities)
  int tiles_w, tiles_h, n_tiles, m_tiles, total_tiles;
  int taps;                 // 9 or 1
  int stages;
  const uint8_t* w_packed;  // [n_tile][slab_pair][tap][2][BN][16]
  int w_tile_bytes;
  int oc_alloc;             // n_tiles * BN: length of the (zero-padded) w_scale and bias vectors
  const float* scale_rec;
  const float* w_scale;
  const float* bias;
  const __half* res;
  int res_ldc, res_coff;
  __half* out;
  int out_ldc, out_coff;
  int out_vec, res_vec;
  uint32_t* amax_out;
  int amax_stride, amax_goff;
  int32_t* acc_dump;
  uint32_t* status;
  int silu;
  int contiguous;           // tile order: 0 strided over CTAs, 1 one contiguous run per CTA
  int nhwc;                 // fp16 stride 1: act_map is the NHWC activation (channel, x, y, image) itself
  int issuers;              // MMA issuing threads (1 or 2; 2 needs a half ring to hold a whole tile)
  // pg16 (INT8_PERGROUP): every slab is its own accumulation unit; a K step pairs two taps of
  // one slab (tap_a[m], tap_b[m] < 0: the second half of K has zero weights)
  int tap_pairs;
  int tap_a[5], tap_b[5];
  // super-tiles (per tensor): a tile is mblocks M blocks of th rows stacked vertically, sharing one
  // halo box per slab and one pipeline step; nacc TMEM buffers of mblocks*BN columns each
  int mblocks, nacc, tmem_cols;
  // quantize on load (kQL instances): sources, raw ring, per-source staging boxes and amax slots
  int ql_parts;
  int ql_raw_slots, ql_raw_bytes;     // raw ring: slots, bytes of one slot (two slabs)
  int ql_mode;                        // 0 per tensor, 1 pg16 (every slab its own group's scale)
  int ql_slab0[kQlMaxParts];          // first slab of each source
  int ql_up[kQlMaxParts];             // 1 or 2 (nearest 2x upsample)
  int ql_box_w[kQlMaxParts], ql_box_h[kQlMaxParts];  // staging box of one slab, pixels
  int ql_groups[kQlMaxParts];         // amax groups of each source (one per slab it fills)
  const uint32_t* ql_amax[kQlMaxParts];
  int ql_amax_stride[kQlMaxParts], ql_amax_goff[kQlMaxParts];
  // int32 accumulators convert through the exact small-integer path (the host bounds every
  // |accumulator| <= 2^22 from the weight codes)
  int acc_small;
  // staged output (out_nbuf > 0): each epilogue group of four warps (one per TMEM lane quadrant)
  // writes its column block of a tile into a swizzled shared-memory box and one thread stores
  // the box with a TMA tensor store; out_nbuf buffers of out_gbytes per group
  int out_nbuf, out_gbytes;
  CUtensorMap ql_map[kQlMaxParts];    // (channel, x, y, image) maps of the fp16 NHWC slices
  CUtensorMap out_map;                // (channel, x, y, image) over the output slice; box = one group's block
};

// Shared-memory bytes of the staged output of one plan: 4 epilogue groups x nbuf buffers, each
// one group's column block (kCols channels) of every pixel of a (super-)tile, 1024-aligned.
__host__ __device__ constexpr int halo_out_cols(int bn, bool pg) {
  return (bn == 64 && !pg) ? 32 : (bn >= 64 ? bn / 4 : 16);
}
__host__ __device__ inline int halo_out_gbytes(int bn, bool pg, int tile_px) {
  return ((tile_px * halo_out_cols(bn, pg) * 2 + 1023) / 1024) * 1024;
}

struct HaloSmemPlan {
  int slab_bytes;   // one slab's halo (all parity boxes), multiple of 128
  int stage_bytes;  // two slabs
  int a_bytes;      // all stages
  int raw_offset;   // quantize on load: the fp16 raw ring
  int out_offset;   // staged output buffers (1024-aligned)
  int b_offset;
  int sb_offset;
  int am_offset;    // per-tile amax reduction ring (strided order): [8][16] maxima + [8][4] counters
  int gs_offset;    // pg16: per epilogue warp, the current image's group scales [16][kMaxSlabsPg]
  int bar_offset;
  int total_bytes;
};

constexpr int kMaxAcc = 16;                 // TMEM accumulator buffers (narrow tiles keep more in flight)
constexpr int kMaxSlabsPg = 64;             // pg16 group-scale table per epilogue warp (up to 1024 input channels)
constexpr int kAmaxRing = 2 * kMaxAcc;      // >= 2 x accumulator buffers: a slot is reset before any warp reuses it

__host__ __device__ inline HaloSmemPlan halo_smem_plan(int halo_rows, int boxes_per_slab, int stages,
                                                       int w_tile_bytes, int oc_alloc, int raw_total = 0,
                                                       int out_total = 0, bool pg = false) {
  HaloSmemPlan s;
  const int box_bytes = ((halo_rows * kSlotBytes + 127) / 128) * 128;
  s.slab_bytes = box_bytes * boxes_per_slab;
  s.stage_bytes = 2 * s.slab_bytes;
  // 4 KB of slack: a shifted 128-row window may run past the last halo row
  s.a_bytes = stages * s.stage_bytes + 4096;
  s.raw_offset = ((s.a_bytes + 127) / 128) * 128;
  s.out_offset = ((s.raw_offset + raw_total + 1023) / 1024) * 1024;
  s.b_offset = ((s.out_offset + out_total + 1023) / 1024) * 1024;
  s.sb_offset = s.b_offset + ((w_tile_bytes + 127) / 128) * 128;  // w_scale[oc_alloc], bias[oc_alloc]
  s.am_offset = s.sb_offset + ((8 * oc_alloc + 127) / 128) * 128;
  s.gs_offset = s.am_offset + kAmaxRing * (16 + 4) * 4;
  s.bar_offset = s.gs_offset + (pg ? 16 * kMaxSlabsPg * 4 : 0);
  // barriers: full[stages], empty[stages], acc_full[16], acc_empty[16], w_full[2], sb_full, raw_full[4],
  // raw_empty[4]; then the TMEM address
  s.total_bytes = s.bar_offset + (2 * stages + 2 * kMaxAcc + 3 + 2 * kQlMaxRaw) * 8 + 16;
  return s;
}

// Epilogue: 16 warps, 4 per TMEM lane quadrant.  The four warps of a quadrant
// split the tile's columns into halo_col_blocks blocks; the spare warps (BN < 64,
// and BN = 64 per tensor) form tile groups that take alternate tiles
// (accumulator buffers), so narrow layers get the same epilogue throughput per
// SM as wide ones.
template <int BN>
constexpr int halo_epi_warps() {
  return 16;
}
template <int BN, bool kPG = false>
constexpr int halo_col_blocks() {
  // BN 64 (per tensor): two 32-column blocks and two tile groups, so that the four warps of an SM
  // sub-partition work on two tiles at once (3x3 64->64 @80 batch 64: 37.9 against 39.9 us with four
  // 16-column blocks); 128 and 256 keep four blocks (two tile groups measured slower there)
  return (BN == 64 && !kPG) ? 2 : (BN >= 64 ? 4 : BN / 16);
}
// MMA issuers: tcgen05.mma issue blocks while the tensor core is busy, so one
// issuing thread leaves the tensor core idle during its per-tile barrier waits
// and commits; two issuers (tiles alternate between them) hide each other's.
// With two, the stage ring is split in halves, one per issuer, so that every
// ring slot still has a single consumer taking its phases in order (mbarrier
// parity waits are only unambiguous one phase ahead).
constexpr int kMmaIssuers = 2;
template <int BN, bool kQL = false>
constexpr int halo_threads() {
  // producer, epilogue, issuers (warp 1 and warp 2 + epilogue warps), then the converters
  return 32 * (1 + halo_epi_warps<BN>() + kMmaIssuers + (kQL ? kQlWarps : 0));
}

// Sixteen fp16 values (two 16-byte chunks) -> sixteen int8 codes, the quantizer's arithmetic
// (codes8 in quant.cuh): the 1.5*2^23 rounding when every |x * mult| < 2^22, else float-to-int.
__device__ __forceinline__ uint4 ql_codes16(const uint4& a, const uint4& b, float mult) {
  const __half2* ha = reinterpret_cast<const __half2*>(&a);
  const __half2* hb = reinterpret_cast<const __half2*>(&b);
  __half2 m = __habs2(ha[0]);
#pragma unroll
  for (int e = 1; e < 4; ++e) m = __hmax2(m, __habs2(ha[e]));
#pragma unroll
  for (int e = 0; e < 4; ++e) m = __hmax2(m, __habs2(hb[e]));
  const bool magic = fmaxf(__low2float(m), __high2float(m)) * mult < 4194304.0f;
  uint4 r;
  if (magic) {
    codes8<true>(a, mult, r.x, r.y);
    codes8<true>(b, mult, r.z, r.w);
  } else {
    codes8<false>(a, mult, r.x, r.y);
    codes8<false>(b, mult, r.z, r.w);
  }
  return r;
}

// Source (part) of slab `slab` of the concatenated input.
__device__ __forceinline__ int ql_part_of(const ConvHaloParams& p, int slab) {
  int k = 0;
#pragma unroll
  for (int j = 1; j < kQlMaxParts; ++j)
    if (j < p.ql_parts && slab >= p.ql_slab0[j]) k = j;
  return k;
}

// amax of 16-channel group g of source k for image img (float bits in the producers' slots).
__device__ __forceinline__ float ql_group_amax(const ConvHaloParams& p, int k, int img, int g) {
  return __uint_as_float(
      __ldg(p.ql_amax[k] + static_cast<size_t>(img) * p.ql_amax_stride[k] + p.ql_amax_goff[k] + g));
}

// Per-tensor amax of image img: the max over every group of every source (the quantizer's `at`).
__device__ __forceinline__ float ql_tensor_amax(const ConvHaloParams& p, int img) {
  float at = 0.0f;
  for (int k = 0; k < p.ql_parts; ++k)
    for (int g = 0; g < p.ql_groups[k]; ++g) at = fmaxf(at, ql_group_amax(p, k, img, g));
  return at;
}

__device__ __forceinline__ float ql_mult(float a) { return a > 0.0f ? __fdiv_rn(127.0f, a) : 0.0f; }

// Epilogue of 8 consecutive output channels of one pixel (full-width fast path
// when all 8 channels exist and the row is 16-byte aligned): scale, bias,
// SiLU, residual, fp16 store.  Returns the max |fp16 output| of the 8 values.
// `sscale` / `sbias` point at this 8-column group's weight scale and bias in the
// CTA's resident weight tile (shared memory; zero past the last channel).  For
// SiLU layers both vectors hold half the plan's values, so the affine step
// yields h = y/2 directly (exact: halving commutes with rounding) and
// SiLU(y) = y * sigmoid(y) = h + h * tanh(h).  This scalar form serves
// partial chunks; halo_epilogue16_packed below is the full-chunk path.
template <bool kF16, bool kSilu, bool kRes>
__device__ __forceinline__ float halo_epilogue8(const ConvHaloParams& p, const uint32_t* v, float in_scale, int oc,
                                                const float* sscale, const float* sbias, bool valid, __half* out_row,
                                                const __half* res_row) {
  const int n_valid = p.oc - oc;
  float y[8];
  {
    const float4 b0 = *reinterpret_cast<const float4*>(sbias);
    const float4 b1 = *reinterpret_cast<const float4*>(sbias + 4);
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    if constexpr (kF16) {
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = kSilu ? fmaf(__uint_as_float(v[i]), 0.5f, bb[i]) : __uint_as_float(v[i]) + bb[i];
    } else {
      const float4 s0 = *reinterpret_cast<const float4*>(sscale);
      const float4 s1 = *reinterpret_cast<const float4*>(sscale + 4);
      const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = fmaf(static_cast<float>(static_cast<int32_t>(v[i])) * in_scale, ss[i], bb[i]);
    }
  }
  if constexpr (kSilu) {
    // y holds h = y/2 (halved scale and bias): SiLU(y) = h + h * tanh(h)
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = fmaf(y[i], tanh_approx(y[i]), y[i]);
  }
  const bool vec = n_valid >= 8 && p.out_vec;
  if constexpr (kRes) {
    if (valid) {
      if (n_valid >= 8 && p.res_vec) {
        const uint4 r = *reinterpret_cast<const uint4*>(res_row + oc);
        const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(rh[i]);
          y[2 * i] += f.x;
          y[2 * i + 1] += f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < n_valid) y[i] += __half2float(res_row[oc + i]);
      }
    }
  }
  if (n_valid < 8) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i >= n_valid) y[i] = 0.0f;
  }
  __align__(16) __half2 hv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) hv[i] = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
  if (valid) {
    if (vec) {
      *reinterpret_cast<uint4*>(out_row + oc) = *reinterpret_cast<const uint4*>(hv);
    } else if (n_valid > 0) {
      const __half* h = reinterpret_cast<const __half*>(hv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < n_valid) out_row[oc + i] = h[i];
    }
  }
  const __half2 m = __hmax2(__hmax2(__habs2(hv[0]), __habs2(hv[1])), __hmax2(__habs2(hv[2]), __habs2(hv[3])));
  return valid ? fmaxf(__low2float(m), __high2float(m)) : 0.0f;
}

// The epilogue of 16 consecutive output channels of one pixel when all 16
// exist and the output (and residual) rows allow 16-byte accesses: the same
// arithmetic as halo_epilogue8, element for element, with the affine, SiLU
// and residual steps on packed fp32 pairs (fma/mul/add .f32x2).  Returns the
// max |fp16 output| as a half2 pair (the caller folds it).
template <bool kF16, bool kSilu, bool kRes>
__device__ __forceinline__ __half2 halo_epilogue16_packed(const uint32_t* v, float in_scale, const float* sscale,
                                                          const float* sbias, bool valid, __half* out,
                                                          const __half* res) {
  const uint64_t s2 = f2_pack(in_scale, in_scale);
  const uint64_t half2c = f2_pack(0.5f, 0.5f);
  __half2 m = __float2half2_rn(0.0f);
#pragma unroll
  for (int h8 = 0; h8 < 2; ++h8) {
    const float4 b0 = *reinterpret_cast<const float4*>(sbias + 8 * h8);
    const float4 b1 = *reinterpret_cast<const float4*>(sbias + 8 * h8 + 4);
    const uint64_t bb[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y), f2_pack(b1.z, b1.w)};
    uint64_t y[4];
    if constexpr (kF16) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t a = f2_pack(__uint_as_float(v[8 * h8 + 2 * i]), __uint_as_float(v[8 * h8 + 2 * i + 1]));
        y[i] = kSilu ? f2_fma(a, half2c, bb[i]) : f2_add(a, bb[i]);
      }
    } else {
      const float4 c0 = *reinterpret_cast<const float4*>(sscale + 8 * h8);
      const float4 c1 = *reinterpret_cast<const float4*>(sscale + 8 * h8 + 4);
      const uint64_t ss[4] = {f2_pack(c0.x, c0.y), f2_pack(c0.z, c0.w), f2_pack(c1.x, c1.y), f2_pack(c1.z, c1.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t a = f2_pack(static_cast<float>(static_cast<int32_t>(v[8 * h8 + 2 * i])),
                                   static_cast<float>(static_cast<int32_t>(v[8 * h8 + 2 * i + 1])));
        y[i] = f2_fma(f2_mul(a, s2), ss[i], bb[i]);
      }
    }
    if constexpr (kSilu) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float h0, h1;
        f2_unpack(y[i], h0, h1);
        y[i] = f2_fma(y[i], f2_pack(tanh_approx(h0), tanh_approx(h1)), y[i]);
      }
    }
    if constexpr (kRes) {
      if (valid) {
        const uint4 r = *reinterpret_cast<const uint4*>(res + 8 * h8);
        const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(rh[i]);
          y[i] = f2_add(y[i], f2_pack(f.x, f.y));
        }
      }
    }
    __align__(16) __half2 hv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a, b;
      f2_unpack(y[i], a, b);
      hv[i] = __floats2half2_rn(a, b);
      m = __hmax2(m, __habs2(hv[i]));
    }
    if (valid) *reinterpret_cast<uint4*>(out + 8 * h8) = *reinterpret_cast<const uint4*>(hv);
  }
  return valid ? m : __float2half2_rn(0.0f);
}

// The staged epilogue of 16 consecutive output channels of one pixel: the arithmetic of
// halo_epilogue16_packed (scale, bias, SiLU, residual, fp16), with the results returned as two
// 16-byte chunks `o` instead of stored.  `r` holds the 16 residual values (zero where absent);
// the scale and bias vectors are zero-padded, so channels past the last one compute zeros.
// kSmall: the accumulators convert through acc2_to_f2's exact small-integer path.
template <bool kF16, bool kSilu, bool kRes, bool kSmall>
__device__ __forceinline__ __half2 halo_epi16(const uint32_t* v, uint64_t s2, const float* sscale, const float* sbias,
                                              const uint4* r, uint4* o) {
  const uint64_t half2c = f2_pack(0.5f, 0.5f);
  __half2 m = __float2half2_rn(0.0f);
#pragma unroll
  for (int h8 = 0; h8 < 2; ++h8) {
    const float4 b0 = *reinterpret_cast<const float4*>(sbias + 8 * h8);
    const float4 b1 = *reinterpret_cast<const float4*>(sbias + 8 * h8 + 4);
    const uint64_t bb[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y), f2_pack(b1.z, b1.w)};
    uint64_t y[4];
    if constexpr (kF16) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t a = f2_pack(__uint_as_float(v[8 * h8 + 2 * i]), __uint_as_float(v[8 * h8 + 2 * i + 1]));
        y[i] = kSilu ? f2_fma(a, half2c, bb[i]) : f2_add(a, bb[i]);
      }
    } else {
      const float4 c0 = *reinterpret_cast<const float4*>(sscale + 8 * h8);
      const float4 c1 = *reinterpret_cast<const float4*>(sscale + 8 * h8 + 4);
      const uint64_t ss[4] = {f2_pack(c0.x, c0.y), f2_pack(c0.z, c0.w), f2_pack(c1.x, c1.y), f2_pack(c1.z, c1.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t a = acc2_to_f2<kSmall>(v[8 * h8 + 2 * i], v[8 * h8 + 2 * i + 1]);
        y[i] = f2_fma(f2_mul(a, s2), ss[i], bb[i]);
      }
    }
    if constexpr (kSilu) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float h0, h1;
        f2_unpack(y[i], h0, h1);
        y[i] = f2_fma(y[i], f2_pack(tanh_approx(h0), tanh_approx(h1)), y[i]);
      }
    }
    if constexpr (kRes) {
      const __half2* rh = reinterpret_cast<const __half2*>(&r[h8]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(rh[i]);
        y[i] = f2_add(y[i], f2_pack(f.x, f.y));
      }
    }
    __half2* hv = reinterpret_cast<__half2*>(&o[h8]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a, b;
      f2_unpack(y[i], a, b);
      hv[i] = __floats2half2_rn(a, b);
      m = __hmax2(m, __habs2(hv[i]));
    }
  }
  return m;
}

// The 16 residual values of channels [oc, oc + 16) of one pixel row (zero past the last channel
// or for an invalid pixel): two 16-byte loads when the whole group exists and the row allows it.
__device__ __forceinline__ void halo_load_res16(const ConvHaloParams& p, const __half* res_row, int oc, bool valid,
                                                uint4* r) {
  r[0] = r[1] = make_uint4(0u, 0u, 0u, 0u);
  if (!valid) return;
  const int n_valid = p.oc - oc;
  if (n_valid >= 16 && p.res_vec) {
    r[0] = *reinterpret_cast<const uint4*>(res_row + oc);
    r[1] = *reinterpret_cast<const uint4*>(res_row + oc + 8);
  } else {
    __half* h = reinterpret_cast<__half*>(r);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < n_valid) h[i] = res_row[oc + i];
  }
}

// Byte offset of 16-byte chunk `c` of staging row `row` inside one group's output box: rows of
// kCols fp16 channels, chunks permuted by the TMA swizzle of that row width (32, 64 or 128 bytes:
// chunk bits XOR address bits 7.. of the row), so that eight consecutive rows written by eight
// lanes land in eight distinct bank groups.
template <int kCols>
__device__ __forceinline__ uint32_t halo_stage_off(int row, int c) {
  static_assert(kCols == 16 || kCols == 32 || kCols == 64, "staged output rows are 32, 64 or 128 bytes");
  const int sw = kCols == 64 ? (row & 7) : (kCols == 32 ? ((row >> 1) & 3) : ((row >> 2) & 1));
  return static_cast<uint32_t>(row * (2 * kCols) + ((c ^ sw) << 4));
}

// pg16 final epilogue of 8 consecutive channels from the fp32 group sums `fp2` (packed pairs):
// y = fma(fp, w_scale, bias) (the reference's `fp * scale + bias`, which its shader compiler may contract), then
// SiLU (halved vectors, as above), residual, fp16 store.  Packed when all 8
// channels exist and the rows allow 16-byte accesses.  Returns max |fp16 y|.
template <bool kSilu, bool kRes>
__device__ __forceinline__ float halo_pg_finish8(const ConvHaloParams& p, const uint64_t* fp2, int oc,
                                                 const float* sscale, const float* sbias, bool valid, __half* out_row,
                                                 const __half* res_row) {
  const int n_valid = p.oc - oc;
  const bool full = n_valid >= 8 && p.out_vec && (!kRes || p.res_vec);
  const float4 c0 = *reinterpret_cast<const float4*>(sscale), c1 = *reinterpret_cast<const float4*>(sscale + 4);
  const float4 b0 = *reinterpret_cast<const float4*>(sbias), b1 = *reinterpret_cast<const float4*>(sbias + 4);
  const uint64_t ss[4] = {f2_pack(c0.x, c0.y), f2_pack(c0.z, c0.w), f2_pack(c1.x, c1.y), f2_pack(c1.z, c1.w)};
  const uint64_t bb[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y), f2_pack(b1.z, b1.w)};
  float y[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t v = f2_fma(fp2[i], ss[i], bb[i]);
    if constexpr (kSilu) {
      float h0, h1;
      f2_unpack(v, h0, h1);
      v = f2_fma(v, f2_pack(tanh_approx(h0), tanh_approx(h1)), v);
    }
    f2_unpack(v, y[2 * i], y[2 * i + 1]);
  }
  if constexpr (kRes) {
    if (valid) {
      if (full) {
        const uint4 r = *reinterpret_cast<const uint4*>(res_row + oc);
        const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(rh[i]);
          y[2 * i] += f.x;
          y[2 * i + 1] += f.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i < n_valid) y[i] += __half2float(res_row[oc + i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i >= n_valid) y[i] = 0.0f;
  __align__(16) __half2 hv[4];
  __half2 m = __float2half2_rn(0.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    hv[i] = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
    m = __hmax2(m, __habs2(hv[i]));
  }
  if (valid) {
    if (full) {
      *reinterpret_cast<uint4*>(out_row + oc) = *reinterpret_cast<const uint4*>(hv);
    } else {
      const __half* h = reinterpret_cast<const __half*>(hv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < n_valid) out_row[oc + i] = h[i];
    }
  }
  return valid ? fmaxf(__low2float(m), __high2float(m)) : 0.0f;
}

// pg16, staged: the arithmetic of halo_pg_finish8 for 8 channels with the residual values `r`
// (zero where absent), returned as one 16-byte chunk.
template <bool kSilu, bool kRes>
__device__ __forceinline__ __half2 halo_pg_vals8(const uint64_t* fp2, const float* sscale, const float* sbias,
                                                 const uint4& r, uint4& o) {
  const float4 c0 = *reinterpret_cast<const float4*>(sscale), c1 = *reinterpret_cast<const float4*>(sscale + 4);
  const float4 b0 = *reinterpret_cast<const float4*>(sbias), b1 = *reinterpret_cast<const float4*>(sbias + 4);
  const uint64_t ss[4] = {f2_pack(c0.x, c0.y), f2_pack(c0.z, c0.w), f2_pack(c1.x, c1.y), f2_pack(c1.z, c1.w)};
  const uint64_t bb[4] = {f2_pack(b0.x, b0.y), f2_pack(b0.z, b0.w), f2_pack(b1.x, b1.y), f2_pack(b1.z, b1.w)};
  const __half2* rh = reinterpret_cast<const __half2*>(&r);
  __half2* hv = reinterpret_cast<__half2*>(&o);
  __half2 m = __float2half2_rn(0.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t v = f2_fma(fp2[i], ss[i], bb[i]);
    if constexpr (kSilu) {
      float h0, h1;
      f2_unpack(v, h0, h1);
      v = f2_fma(v, f2_pack(tanh_approx(h0), tanh_approx(h1)), v);
    }
    float y0, y1;
    f2_unpack(v, y0, y1);
    if constexpr (kRes) {
      const float2 f = __half22float2(rh[i]);
      y0 += f.x;
      y1 += f.y;
    }
    hv[i] = __floats2half2_rn(y0, y1);
    m = __hmax2(m, __habs2(hv[i]));
  }
  return m;
}

// A conv tile index t = ((nt * n_img + img) * tiles_h + row) * tiles_w + col as its digits.
struct TileCursor {
  int col, row, img, nt;
  __device__ __forceinline__ void set(int t, const ConvHaloParams& p) {
    col = t % p.tiles_w;
    t /= p.tiles_w;
    row = t % p.tiles_h;
    t /= p.tiles_h;
    img = t % p.n_img;
    nt = t / p.n_img;
  }
  // this += d (every digit of d below its radix, so one carry per digit suffices)
  __device__ __forceinline__ void advance(const TileCursor& d, const ConvHaloParams& p) {
    col += d.col;
    int c = col >= p.tiles_w;
    col -= c ? p.tiles_w : 0;
    row += d.row + c;
    c = row >= p.tiles_h;
    row -= c ? p.tiles_h : 0;
    img += d.img + c;
    c = img >= p.n_img;
    img -= c ? p.n_img : 0;
    nt += d.nt + c;
  }
};

template <bool kF16, int BN, bool kSilu, bool kRes, bool kPG = false, bool kMB = false, bool kQL = false>
__global__ void __launch_bounds__(halo_threads<BN, kQL>(), 1)
    conv_halo_kernel(const __grid_constant__ CUtensorMap act_map, const __grid_constant__ ConvHaloParams p) {
  static_assert(!kMB || (!kPG && BN <= 64), "super-tiles: per tensor, BN <= 64");
  static_assert(!kQL || !kF16, "quantize on load: int8 plans");
  static_assert(!kPG || (!kF16 && (BN == 64 || BN == 128)), "pg16 halo: int8, BN 64 or 128 (no epilogue tile groups)");
  constexpr int kEpiWarps = halo_epi_warps<BN>();
  constexpr int kColBlocks = halo_col_blocks<BN, kPG>();
  constexpr int kTileGroups = 4 / kColBlocks;   // epilogue tile groups (tiles i with i % groups == g)
  constexpr int kCols = BN / kColBlocks;        // columns per epilogue warp
  constexpr int CW = (kCols >= 32 && !kPG) ? 32 : 16;  // columns per TMEM load (pg16 keeps fp32 sums live)
  constexpr int kChunks = kCols / CW;
  // accumulator buffers in TMEM, p.nacc of p.mblocks*BN columns each (the host keeps nacc a
  // multiple of the issuers and of the epilogue tile groups): the MMA runs up to nacc tiles ahead
  // of the epilogue.  pg16: accumulation units are (tile, slab), 512 / BN buffers of BN columns.
  // super-tile instances (kMB) stack up to kMaxMB M blocks; the others keep compile-time counts
  constexpr int kMaxMB = kMB ? (BN <= 32 ? 4 : 2) : 1;
  constexpr int kAccFixed = kPG ? 512 / BN : (BN <= 16 ? 16 : (BN <= 32 ? 8 : (BN <= 128 ? 4 : 2)));
  constexpr int kAcc = kPG ? kAccFixed : kMaxAcc;  // pg16 count; bound of nacc otherwise
  const int nacc = kMaxMB == 1 ? kAccFixed : p.nacc;
  const int acc_cols = kMaxMB == 1 ? BN : p.mblocks * BN;
  const uint32_t tmem_cols = static_cast<uint32_t>(p.tmem_cols);
  constexpr int kCS = kF16 ? 8 : 16;  // tensor-map elements per 16-byte chunk

  extern __shared__ __align__(1024) uint8_t smem[];
  // programmatic dependent launch (ptx.cuh): the next kernel may be scheduled right away.  The set-up
  // below and the loads of the plan's own weights, scales and biases touch no memory another kernel
  // writes; every role that reads activations, scale records or amax slots, or writes outputs, first
  // waits for the previous grid (the producer before its first activation box, the epilogue and the
  // converters on entry; the MMA issuers only touch shared memory and TMEM).
  grid_dep_launch();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const HaloSmemPlan sp = halo_smem_plan(p.halo_rows, p.boxes_per_slab, p.stages, p.w_tile_bytes, p.oc_alloc,
                                         kQL ? p.ql_raw_slots * p.ql_raw_bytes : 0, 4 * p.out_nbuf * p.out_gbytes,
                                         kPG);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + sp.bar_offset);
  uint64_t* empty = full + p.stages;
  uint64_t* acc_full = full + 2 * p.stages;  // [kAcc]
  uint64_t* acc_empty = acc_full + kMaxAcc;  // [kAcc]
  uint64_t* w_full = acc_empty + kMaxAcc;
  uint64_t* sb_full = w_full + 2;
  uint64_t* raw_full = sb_full + 1;         // [kQlMaxRaw]: fp16 boxes of a stage landed
  uint64_t* raw_empty = raw_full + kQlMaxRaw;  // [kQlMaxRaw]: the converters have read them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_empty + kQlMaxRaw);
  const int box_bytes = sp.slab_bytes / p.boxes_per_slab;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < nacc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * kColBlocks);  // the warps of the tile group that drains buffer b
    }
    mbar_init(&w_full[0], 1);
    mbar_init(&w_full[1], p.issuers);  // every active issuer releases the old weights
    mbar_init(sb_full, 1);
    if constexpr (kQL) {
      for (int r = 0; r < p.ql_raw_slots; ++r) {
        mbar_init(&raw_full[r], 1);
        mbar_init(&raw_empty[r], 1);
      }
    }
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < kAmaxRing * (16 + 4); i += blockDim.x) reinterpret_cast<uint32_t*>(smem + sp.am_offset)[i] = 0u;
  if (warp == 0 && lane == 0) {
    if constexpr (kQL) {
      for (int k = 0; k < p.ql_parts; ++k) tma_prefetch_desc(&p.ql_map[k]);
    } else {
      tma_prefetch_desc(&act_map);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Tiles are ordered n-tile major, so a persistent CTA keeps one weight tile for long runs.
  // Strided order (CTA b takes b, b+G, ...): concurrent CTAs work on neighbouring tiles; the
  // |y| maxima of a tile are reduced across its four lane quadrants in shared memory (one
  // atomic per tile and 16-channel group).  Contiguous order (one run per CTA): consecutive
  // tiles of one image fold their maxima in registers (one atomic per run, image and group).
  // Every role walks k = b, b+G, ... (G CTAs); the i-th tile of CTA b is t = k (strided) or
  // t = run_start + i (contiguous: CTA b owns as many tiles as the strided walk gives it).
  const int run_start = static_cast<int>(blockIdx.x) * (p.total_tiles / static_cast<int>(gridDim.x)) +
                        min(static_cast<int>(blockIdx.x), p.total_tiles % static_cast<int>(gridDim.x));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(sb_full, static_cast<uint32_t>(8 * p.oc_alloc));
      bulk_load(smem + sp.sb_offset, p.w_scale, static_cast<uint32_t>(4 * p.oc_alloc), sb_full);
      bulk_load(smem + sp.sb_offset + 4 * p.oc_alloc, p.bias, static_cast<uint32_t>(4 * p.oc_alloc), sb_full);
    }
    // Lane-parallel issue: the CTA's stages (tile i, slab pair pr) are numbered q = i * pairs + pr
    // and handed out in groups of up to min(32, stages) consecutive stages with one weight tile;
    // lane j of the warp computes stage q0 + j's coordinates, waits for its ring slot and issues
    // its boxes, so the per-stage integer arithmetic and barrier latencies overlap across lanes.
    const int my_tiles = static_cast<int>(blockIdx.x) < p.total_tiles
                             ? (p.total_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    const int total_q = my_tiles * p.slab_pairs;
    const int R = p.issuers, H = p.stages / p.issuers;  // rings and slots per ring
    // quantize on load: stages go to the raw ring (one slot per stage, in order); the converters
    // fill the A stages
    const int group = kQL ? min(32, p.ql_raw_slots) : min(32, H);
    const int per_img = p.tiles_w * p.tiles_h;
    const int nbox = 2 * p.boxes_per_slab;
    const uint32_t stage_tx = static_cast<uint32_t>(nbox * p.halo_rows * kSlotBytes);
    int cur_n = -1, wloads = 0;
    bool ok = true, deps = false;
    for (int q0 = 0; q0 < total_q && ok;) {
      const int q = q0 + lane;
      const int i = q / p.slab_pairs;
      const int pr = q - i * p.slab_pairs;
      const int t = p.contiguous ? run_start + i : static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
      const int n_tile = t / p.m_tiles;
      const int m_tile = t - n_tile * p.m_tiles;
      const int img = m_tile / per_img;
      const int r = m_tile - img * per_img;
      const int oh0 = (r / p.tiles_w) * p.th * p.mblocks, ow0 = (r % p.tiles_w) * p.tw;
      const int n_first = __shfl_sync(0xffffffffu, n_tile, 0);
      // n-tiles never decrease along q: the stages of this group form a prefix of the lanes
      const bool mine = lane < group && q < total_q && n_tile == n_first;
      const int count = __popc(__ballot_sync(0xffffffffu, mine));
      if (n_first != cur_n) {
        // a new weight tile: wait until every MMA reading the old one has completed
        if (wloads > 0 && !mbar_wait_bounded(&w_full[1], (wloads - 1) & 1, p.status, kStatusTimeoutEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&w_full[0], static_cast<uint32_t>(p.w_tile_bytes));
          const uint8_t* src = p.w_packed + static_cast<size_t>(n_first) * p.w_tile_bytes;
          for (int off = 0; off < p.w_tile_bytes; off += 32768)
            bulk_load(smem + sp.b_offset + off, src + off, static_cast<uint32_t>(min(32768, p.w_tile_bytes - off)),
                      &w_full[0]);
        }
        __syncwarp();
        cur_n = n_first;
        ++wloads;
      }
      if (!deps) {
        grid_dep_wait();  // the first weight tile is on its way; activations come from the previous kernel
        deps = true;
      }
      bool lane_ok = true;
      if (kQL && mine) {
        const int rr = q % p.ql_raw_slots;
        const uint32_t rph = static_cast<uint32_t>(q / p.ql_raw_slots) & 1u;
        lane_ok = q < p.ql_raw_slots || mbar_wait_bounded(&raw_empty[rr], rph ^ 1u, p.status, kStatusTimeoutEmpty);
        if (lane_ok) {
          const int o = p.ksize == 3 ? 1 : 0;
          int kp[2] = {-1, -1};
          uint32_t tx = 0;
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const int slab = 2 * pr + which;
            if (slab < p.slabs) {
              kp[which] = ql_part_of(p, slab);
              tx += static_cast<uint32_t>(32 * p.ql_box_w[kp[which]] * p.ql_box_h[kp[which]]);
            }
          }
          mbar_arrive_expect_tx(&raw_full[rr], tx);
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const int k = kp[which];
            if (k < 0) continue;  // odd slab count: the converters write zero codes
            int x, y;
            if (p.stride == 2) {
              x = 2 * (ow0 - 1);
              y = 2 * (oh0 - 1);
            } else if (p.ql_up[k] == 2) {
              x = (ow0 - o) >> 1;  // floor for negative coordinates too
              y = (oh0 - o) >> 1;
            } else {
              x = ow0 - o;
              y = oh0 - o;
            }
            uint8_t* dst = smem + sp.raw_offset + rr * p.ql_raw_bytes + which * (p.ql_raw_bytes / 2);
            tma_load_4d(dst, &p.ql_map[k], &raw_full[rr], 16 * (2 * pr + which - p.ql_slab0[k]), x, y, img);
          }
        }
      } else if (!kQL && mine) {
        // tile i's stages go to ring i % R, in that ring's own order
        const int qr = (i / R) * p.slab_pairs + pr;
        const int s = (i % R) * H + qr % H;
        const uint32_t ph = static_cast<uint32_t>(qr / H) & 1u;
        lane_ok = qr < H || mbar_wait_bounded(&empty[s], ph ^ 1u, p.status, kStatusTimeoutEmpty);
        if (lane_ok) {
          mbar_arrive_expect_tx(&full[s], stage_tx);
          for (int b = 0; b < nbox; ++b) {
            const int which = b >= p.boxes_per_slab ? 1 : 0;  // slab of the pair
            const int box = b - which * p.boxes_per_slab;
            const int slab = 2 * pr + which;
            const int sn = slab < p.slabs ? img * p.slabs + slab : p.n_img * p.slabs;  // odd count: zero slab
            uint8_t* dst = smem + s * sp.stage_bytes + which * sp.slab_bytes + box * box_bytes;
            if (p.nhwc) {
              // 8 channels x pitch pixels x halo rows of the NHWC tensor land exactly as the slab8
              // box would; a zero slab (odd slab count) reads channels past the extent: zero fill
              const int o = p.ksize == 3 ? 1 : 0;
              tma_load_4d(dst, &act_map, &full[s], 8 * slab, ow0 - o, oh0 - o, img);
            } else if (p.stride == 2) {
              tma_load_5d(dst, &act_map, &full[s], kCS * (ow0 - 1), box & 1, box >> 1, oh0 - 1, sn);
            } else if (p.ksize == 3) {
              tma_load_3d(dst, &act_map, &full[s], kCS * (ow0 - 1), oh0 - 1, sn);
            } else {
              tma_load_3d(dst, &act_map, &full[s], kCS * ow0, oh0, sn);
            }
          }
        }
      }
      ok = __all_sync(0xffffffffu, lane_ok);
      q0 += count;
    }
  } else if (warp == 1 || warp == 2 + kEpiWarps) {
    // ------------------------------------------------------------ MMA issuers
    const int me = warp == 1 ? 0 : 1;  // issues the tiles i with i % p.issuers == me, from ring me
    if (lane == 0 && me < p.issuers) {
      const uint32_t idesc = make_idesc<kF16>(BN);
      // descriptor of (stage 0, tap 0) and per-tap start offsets, in 16-byte descriptor units
      const uint64_t a_desc0 = smem_desc_kmajor_noswizzle(smem_u32(smem), sp.slab_bytes, 128);
      const uint64_t b_desc0 = smem_desc_kmajor_noswizzle(smem_u32(smem + sp.b_offset), BN * kSlotBytes, 128);
      const uint32_t b_step = (2 * BN * kSlotBytes) >> 4;  // one (pair, tap) of resident B
      const uint32_t stage_step = sp.stage_bytes >> 4;
      const uint32_t mb_step = (p.th * p.pitch * kSlotBytes) >> 4;  // one M block of halo rows
      uint32_t tap_off[9];
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) {
        const int kh = tap / 3, kw = tap % 3;
        uint32_t off = 0;
        if (p.stride == 2) {
          // parity box of the tap, shifted by 0 (kh/kw == 0) or 1 pixel
          off = ((((kh + 1) & 1) * 2 + ((kw + 1) & 1)) * box_bytes + ((kh ? 1 : 0) * p.pitch + (kw ? 1 : 0)) * kSlotBytes);
        } else if (p.ksize == 3) {
          off = (kh * p.pitch + kw) * kSlotBytes;
        }
        tap_off[tap] = off >> 4;
      }
      const int H = p.stages / p.issuers;
      // pg16: per tap pair m, the A descriptor of (stage 0, slab 0): start at tap a, LBO = tap b - tap a
      uint64_t pair_desc[5];
      if constexpr (kPG) {
#pragma unroll
        for (int m = 0; m < 5; ++m) {
          const int ta = m < p.tap_pairs ? p.tap_a[m] : 0, tb = m < p.tap_pairs ? p.tap_b[m] : -1;
          const uint32_t oa = tap_off[ta] << 4;
          const uint32_t lbo = tb >= 0 ? (tap_off[tb] << 4) - oa : 16u;
          pair_desc[m] = smem_desc_kmajor_noswizzle(smem_u32(smem) + oa, lbo, 128);
        }
      }
      const uint32_t slab_step = sp.slab_bytes >> 4;
      int uu = 0;  // pg16: this issuer's accumulation units so far
      int s = me * H, cur_n = -1, wloads = 0;  // s, ph: position in this issuer's ring
      uint32_t ph = 0;
      bool ok = true, need_w = false;
      int n_tile = -1, n_end = 0;  // current n-tile and the first tile index past it (no division per tile)
      for (int k = blockIdx.x, i = 0; k < p.total_tiles && ok; k += gridDim.x, ++i) {
        const int t = p.contiguous ? run_start + i : k;
        if (t >= n_end) {
          n_tile = t / p.m_tiles;
          n_end = (n_tile + 1) * p.m_tiles;
        }
        if (n_tile != cur_n) {
          // every issuer releases the old weights at the change (after its own MMAs that read
          // them), once it has seen them arrive: its releases then stay one per weight load
          if (wloads > 0) {
            if (need_w && !mbar_wait_bounded(&w_full[0], (wloads - 1) & 1, p.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            need_w = false;
            tc_commit(&w_full[1]);
          }
          cur_n = n_tile;
          ++wloads;
          need_w = true;
        }
        if (i % p.issuers == me) {
          if (need_w) {
            if (!mbar_wait_bounded(&w_full[0], (wloads - 1) & 1, p.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            need_w = false;
          }
          if constexpr (kPG) {
            // pg16: every slab is an accumulation unit in this issuer's half of the buffers;
            // a K step pairs two taps of the slab (the reference's per-group sub-sums)
            const int Hh = kAcc / p.issuers;
            for (int pr = 0; pr < p.slab_pairs && ok; ++pr) {
              if (!mbar_wait_bounded(&full[s], ph, p.status, kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              for (int which = 0; which < 2; ++which) {
                const int slab = 2 * pr + which;
                if (slab >= p.slabs) break;
                const int buf = me * Hh + uu % Hh;
                if (uu >= Hh) {
                  if (!mbar_wait_bounded(&acc_empty[buf], ((uu / Hh) - 1) & 1, p.status, kStatusTimeoutAccEmpty)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                }
                const uint32_t d = tmem_base + buf * BN;
                const uint32_t a_off = s * stage_step + which * slab_step;
                const uint64_t bslab = b_desc0 + ((static_cast<uint32_t>(slab * p.tap_pairs) * b_step));
#pragma unroll
                for (int m = 0; m < 5; ++m)
                  if (m < p.tap_pairs) tc_mma<false>(d, pair_desc[m] + a_off, bslab + m * b_step, idesc, m ? 1u : 0u);
                tc_commit(&acc_full[buf]);
                ++uu;
              }
              if (!ok) break;
              tc_commit(&empty[s]);
              if (++s == (me + 1) * H) {
                s = me * H;
                ph ^= 1u;
              }
            }
            continue;
          }
          const int u = i;
          const int buf = u % nacc;
          if (u >= nacc) {
            if (!mbar_wait_bounded(&acc_empty[buf], ((u / nacc) - 1) & 1, p.status, kStatusTimeoutAccEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint32_t d = tmem_base + buf * acc_cols;
          for (int pr = 0; pr < p.slab_pairs; ++pr) {
            if (!mbar_wait_bounded(&full[s], ph, p.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ad = a_desc0 + s * stage_step;
            const uint64_t bpr = b_desc0 + static_cast<uint32_t>(pr * p.taps) * b_step;
#pragma unroll
            for (int mb = 0; mb < kMaxMB; ++mb) {
              if (mb >= p.mblocks) break;
              // M block mb starts mb*th rows down the (shared) halo of every box
              const uint64_t amb = ad + mb * mb_step;
              const uint32_t dmb = d + mb * BN;
              uint64_t bd = bpr;
              if (p.taps == 9) {
#pragma unroll
                for (int tap = 0; tap < 9; ++tap) {
                  tc_mma<kF16>(dmb, amb + tap_off[tap], bd, idesc, (pr | tap) ? 1u : 0u);
                  bd += b_step;
                }
              } else {
                tc_mma<kF16>(dmb, amb, bd, idesc, pr ? 1u : 0u);
              }
            }
            tc_commit(&empty[s]);
            if (++s == (me + 1) * H) {
              s = me * H;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit(&acc_full[buf]);
        }
      }
    }
  } else if (kQL && warp >= 3 + kEpiWarps) {
    // ------------------------------------------------------------ converters (quantize on load)
    // Every stage, in the producer's order: wait for its fp16 boxes in the raw ring and for its A
    // slot (the stage ring of the tile's issuer), write the int8 codes of both slabs in the TMA
    // layout the MMA descriptors expect, then release the raw slot and fill the A slot.
    constexpr int kCT = 32 * kQlWarps;
    grid_dep_wait();  // the sources and their amax slots come from earlier kernels
    const int ct = static_cast<int>(threadIdx.x) - 32 * (3 + kEpiWarps);
    const int my_tiles = static_cast<int>(blockIdx.x) < p.total_tiles
                             ? (p.total_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    const int total_q = my_tiles * p.slab_pairs;
    const int R = p.issuers, H = p.stages / p.issuers;
    const int per_img = p.tiles_w * p.tiles_h;
    const int o = p.ksize == 3 ? 1 : 0;
    int cur_img = -1;
    float mult_t = 0.0f;
    for (int q = 0; q < total_q; ++q) {
      const int i = q / p.slab_pairs;
      const int pr = q - i * p.slab_pairs;
      const int t = p.contiguous ? run_start + i : static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
      const int m_tile = t % p.m_tiles;
      const int img = m_tile / per_img;
      const int r = m_tile - img * per_img;
      const int oh0 = (r / p.tiles_w) * p.th * p.mblocks, ow0 = (r % p.tiles_w) * p.tw;
      const int rr = q % p.ql_raw_slots;
      const int qr = (i / R) * p.slab_pairs + pr;
      const int s = (i % R) * H + qr % H;
      bool ok = mbar_wait_bounded(&raw_full[rr], static_cast<uint32_t>(q / p.ql_raw_slots) & 1u, p.status,
                                  kStatusTimeoutFull);
      ok = ok && (qr < H || mbar_wait_bounded(&empty[s], (static_cast<uint32_t>(qr / H) & 1u) ^ 1u, p.status,
                                              kStatusTimeoutEmpty));
      // the converter threads leave together if any of them gave up (they share a named barrier)
      uint32_t all_ok;
      asm volatile(
          "{\n\t.reg .pred pa, pb;\n\tsetp.ne.u32 pa, %1, 0;\n\tbar.red.and.pred pb, 1, %2, pa;\n\t"
          "selp.u32 %0, 1, 0, pb;\n\t}"
          : "=r"(all_ok)
          : "r"(ok ? 1u : 0u), "r"(kCT)
          : "memory");
      if (!all_ok) break;
      if (p.ql_mode == 0 && img != cur_img) {
        mult_t = ql_mult(ql_tensor_amax(p, img));
        cur_img = img;
      }
      const uint8_t* raw = smem + sp.raw_offset + rr * p.ql_raw_bytes;
      uint8_t* stage = smem + s * sp.stage_bytes;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const int slab = 2 * pr + which;
        const int k = slab < p.slabs ? ql_part_of(p, slab) : 0;
        const float mult = slab >= p.slabs ? 0.0f
                           : (p.ql_mode == 0 ? mult_t
                                             : ql_mult(ql_group_amax(p, k, img, slab - p.ql_slab0[k])));
        const uint8_t* src = raw + which * (p.ql_raw_bytes / 2);
        uint8_t* dst = stage + which * sp.slab_bytes;
        const int bw = p.ql_box_w[k], up = p.ql_up[k];
        const int units = p.halo_rows * p.boxes_per_slab;
        for (int u = ct; u < units; u += kCT) {
          const int box = u / p.halo_rows;
          const int rem = u - box * p.halo_rows;
          const int row = rem / p.pitch, col = rem - row * p.pitch;
          uint4 code = make_uint4(0u, 0u, 0u, 0u);
          if (mult != 0.0f) {
            int sy, sx;
            if (p.stride == 2) {  // parity box (row parity box >> 1, column parity box & 1)
              sy = 2 * row + (box >> 1);
              sx = 2 * col + (box & 1);
            } else if (up == 2) {
              sy = ((oh0 - o + row) >> 1) - ((oh0 - o) >> 1);
              sx = ((ow0 - o + col) >> 1) - ((ow0 - o) >> 1);
            } else {
              sy = row;
              sx = col;
            }
            const uint4* v = reinterpret_cast<const uint4*>(src + (sy * bw + sx) * 32);
            code = ql_codes16(v[0], v[1], mult);
          }
          *reinterpret_cast<uint4*>(dst + box * (sp.slab_bytes / p.boxes_per_slab) + rem * kSlotBytes) = code;
        }
      }
      // the codes are generic-proxy writes read by the tensor core (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory");
      if (ct == 0) {
        mbar_arrive(&full[s]);
        mbar_arrive(&raw_empty[rr]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // scale records and residuals come from earlier kernels; outputs may still be read
    const int quad = warp & 3;                   // TMEM lane quadrant this warp may access
    const int colq = ((warp - 2) >> 2) % kColBlocks;  // which kCols-wide column block
    const int tgroup = ((warp - 2) >> 2) / kColBlocks;  // which tiles: i % kTileGroups == tgroup
    const int row = quad * 32 + lane;
    const int r_h = row / p.pitch;
    const int r_w = row - r_h * p.pitch;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int col0 = colq * kCols;
    const int per_img = p.tiles_w * p.tiles_h;
    const float* s_scale = reinterpret_cast<const float*>(smem + sp.sb_offset);  // [oc_alloc]
    const float* s_bias = s_scale + p.oc_alloc;
    mbar_wait_bounded(sb_full, 0, p.status, kStatusTimeoutFull);
    constexpr int kGroups = kChunks * (CW / 16);  // 16-channel amax groups of this warp
    float run_max[kGroups];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) run_max[g] = 0.0f;
    int run_key = -1, run_img = 0, run_oc = 0;  // (n-tile, image) the maxima belong to
    auto flush_amax = [&]() {
#pragma unroll
      for (int g = 0; g < kGroups; ++g) {
        const uint32_t mr = __reduce_max_sync(0xffffffffu, __float_as_uint(run_max[g]));
        const int oc_g = run_oc + 16 * g;
        if (lane == 0 && oc_g < p.oc && mr != 0u)
          atomicMax(&p.amax_out[static_cast<size_t>(run_img) * p.amax_stride + p.amax_goff + oc_g / 16], mr);
        run_max[g] = 0.0f;
      }
    };
    uint32_t* am_ring = reinterpret_cast<uint32_t*>(smem + sp.am_offset);  // [kAmaxRing][16] maxima
    uint32_t* am_count = am_ring + kAmaxRing * 16;                          // [kAmaxRing][4] arrivals
    int ep_img = -1;       // the image whose activation scale ep_scale holds (per tensor)
    float ep_scale = 0.0f;
    int gs_img = -1;       // pg16: the image whose group scales this warp's table holds
    // Staged output: the four warps of this warp's group (one per TMEM lane quadrant, the same
    // column block and tile group) write their column block of a tile into a swizzled box in
    // shared memory; after a named barrier the group's first thread stores the box with one TMA
    // store.  A thread whose wait gives up keeps walking its tiles (without waiting) so that the
    // group's barriers always see all four warps.
    const bool staged = p.out_nbuf > 0;
    const int sgroup = (warp - 2) >> 2;
    const bool st_issuer = staged && warp == 2 + 4 * sgroup && lane == 0;
    uint8_t* const sbuf0 = smem + sp.out_offset + sgroup * p.out_nbuf * p.out_gbytes;
    const int srow0 = (r_h < p.th && r_w < p.tw) ? r_h * p.tw + r_w : -1;  // staging row (M block 0)
    int jj = 0;         // this group's tiles so far: staging buffer jj % out_nbuf
    bool alive = true;  // every wait of this warp so far succeeded
    // This warp's tiles are t0, t0 + step, t0 + 2 step, ... (t0: its tile group's first tile; step:
    // kTileGroups tiles in contiguous order, kTileGroups * gridDim.x in strided order).  A tile index is
    // the mixed-radix number (n-tile, image, tile row, tile column); the cursor holds those digits and
    // adds the step's digits with carries, so no tile needs an integer division.
    TileCursor cur, stp;
    {
      const int t0 = p.contiguous ? run_start + tgroup : static_cast<int>(blockIdx.x) + tgroup * static_cast<int>(gridDim.x);
      cur.set(t0, p);
      stp.set(kTileGroups * (p.contiguous ? 1 : static_cast<int>(gridDim.x)), p);
    }
    for (int k = blockIdx.x, i = 0; k < p.total_tiles; k += gridDim.x, ++i) {
      if (kTileGroups > 1 && i % kTileGroups != tgroup) continue;
      if (i != tgroup) cur.advance(stp, p);
      const int u = i;  // the tile's place in this CTA's sequence: accumulator buffer and phase
      const int n_tile = cur.nt;
      const int img = cur.img;
      const int oy = cur.row * p.th * p.mblocks + r_h, ox = cur.col * p.tw + r_w;
      const bool valid = r_h < p.th && r_w < p.tw && oy < p.oh && ox < p.ow;
      const size_t pix = (static_cast<size_t>(img) * p.oh + (valid ? oy : 0)) * p.ow + (valid ? ox : 0);
      __half* out_row = p.out + pix * p.out_ldc + p.out_coff;
      const __half* res_row = kRes ? p.res + pix * p.res_ldc + p.res_coff : nullptr;
      const int n0 = n_tile * BN;
      uint8_t* const sbuf = sbuf0 + (staged ? (jj % p.out_nbuf) * p.out_gbytes : 0);
      if (staged && p.out_nbuf == 1 && jj > 0) {
        // one buffer: the previous tile's store must have read it before anyone writes it again
        if (st_issuer) bulk_wait_read_all();
        named_bar_sync(2 + sgroup, 128);
      }
      if (p.amax_out != nullptr && p.contiguous && n_tile * p.n_img + img != run_key) {
        if (run_key >= 0) flush_amax();
        run_key = n_tile * p.n_img + img;
        run_img = img;
        run_oc = n0 + col0;
      }
      if constexpr (kPG) {
        // pg16: drain the tile's slab units in ascending group order into fp32 sums,
        // fp = sum_g fl32(fl32(S_g) * fl32(amax_g / 127)), then the final epilogue
        // the image's group scales fl32(amax_g / 127), computed once per image into this warp's table
        float* gs_tab = reinterpret_cast<float*>(smem + sp.gs_offset) + (warp - 2) * kMaxSlabsPg;
        if (img != gs_img) {
          __syncwarp();
          const float* rec = kQL ? nullptr : p.scale_rec + static_cast<size_t>(img) * (1 + p.slabs);
          for (int g = lane; g < p.slabs; g += 32) {
            float ag;
            if constexpr (kQL) {
              const int kq = ql_part_of(p, g);
              ag = ql_group_amax(p, kq, img, g - p.ql_slab0[kq]);
            } else {
              ag = __ldg(rec + 1 + g);
            }
            gs_tab[g] = __fdiv_rn(ag, 127.0f);
          }
          __syncwarp();
          gs_img = img;
        }
        const int Hh = kAcc / p.issuers;
        const int r_iss = i % p.issuers;
        const int ubase = (i / p.issuers) * p.slabs;
        uint64_t fp2[kCols / 2];  // packed fp32 pairs of the group sums
        for (int g = 0; g < p.slabs; ++g) {
          const int uu = ubase + g;
          const int gbuf = r_iss * Hh + uu % Hh;
          const float gs = gs_tab[g];
          const uint64_t gs2 = f2_pack(gs, gs);
          if (alive && !mbar_wait_bounded(&acc_full[gbuf], (uu / Hh) & 1, p.status, kStatusTimeoutAccFull))
            alive = false;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            uint32_t v[CW];
            const uint32_t taddr = lane_addr + gbuf * BN + col0 + c * CW;
            if constexpr (CW == 32) {
              tmem_ld_32x32(taddr, v);
            } else {
              tmem_ld<16>(taddr, v);
            }
            tmem_ld_wait();
            if (c == kChunks - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[gbuf]);
            }
            const int oc_c = n0 + col0 + c * CW;
            if (p.acc_dump != nullptr && valid) {
              const size_t npix = static_cast<size_t>(p.n_img) * p.oh * p.ow;
#pragma unroll
              for (int j = 0; j < CW; ++j)
                if (oc_c + j < p.oc) p.acc_dump[(static_cast<size_t>(g) * npix + pix) * p.oc + oc_c + j] = static_cast<int32_t>(v[j]);
            }
#pragma unroll
            for (int j = 0; j < CW / 2; ++j) {
              // fp += fl32(S) * gs in ascending group order, one fused multiply-add per group (the
              // slot kernel's `fp + S * gs` contracts the same way; ptxas also fuses a packed
              // mul.rn + add.rn pair, so the fma is written out).  Plain conversions: the exact
              // small-integer path (two integer adds and a packed add per pair) measured 9 % slower
              // here, where the drain is issue-bound (C1 batch 64: 140.8 against 129.0 us)
              const uint64_t s2 = acc2_to_f2<false>(v[2 * j], v[2 * j + 1]);
              fp2[c * (CW / 2) + j] = g == 0 ? f2_mul(s2, gs2) : f2_fma(s2, gs2, fp2[c * (CW / 2) + j]);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
#pragma unroll
          for (int g16 = 0; g16 < CW / 16; ++g16) {
            const int lc = n0 + col0 + c * CW + 16 * g16;
            float mg;
            if (staged) {
              uint4 rr[2], o[2];
              if constexpr (kRes) halo_load_res16(p, res_row, lc, valid, rr);
              const __half2 m2 = __hmax2(
                  halo_pg_vals8<kSilu, kRes>(fp2 + (c * CW + 16 * g16) / 2, s_scale + lc, s_bias + lc, rr[0], o[0]),
                  halo_pg_vals8<kSilu, kRes>(fp2 + (c * CW + 16 * g16 + 8) / 2, s_scale + lc + 8, s_bias + lc + 8,
                                             rr[1], o[1]));
              if (srow0 >= 0) {
                const int cc = (c * CW + 16 * g16) >> 3;
                *reinterpret_cast<uint4*>(sbuf + halo_stage_off<kCols>(srow0, cc)) = o[0];
                *reinterpret_cast<uint4*>(sbuf + halo_stage_off<kCols>(srow0, cc + 1)) = o[1];
              }
              mg = valid ? fmaxf(__low2float(m2), __high2float(m2)) : 0.0f;
            } else {
              const float m0 = halo_pg_finish8<kSilu, kRes>(p, fp2 + (c * CW + 16 * g16) / 2, lc, s_scale + lc,
                                                            s_bias + lc, valid, out_row, res_row);
              const float m1 = halo_pg_finish8<kSilu, kRes>(p, fp2 + (c * CW + 16 * g16 + 8) / 2, lc + 8,
                                                            s_scale + lc + 8, s_bias + lc + 8, valid, out_row, res_row);
              mg = fmaxf(m0, m1);
            }
            run_max[c * (CW / 16) + g16] = fmaxf(run_max[c * (CW / 16) + g16], mg);
          }
        }
      } else {
      const int buf = u % nacc;
      // the image's activation scale fl32(amax / 127), computed once per image (the scale record is
      // ready before the launch: read it while the accumulator fills)
      if (!kF16 && img != ep_img) {
        float amax_in;
        if constexpr (kQL) {
          amax_in = ql_tensor_amax(p, img);
        } else {
          amax_in = __ldg(p.scale_rec + static_cast<size_t>(img) * (1 + p.slabs));
        }
        ep_scale = __fdiv_rn(amax_in, 127.0f);
        ep_img = img;
      }
      if (alive && !mbar_wait_bounded(&acc_full[buf], (u / nacc) & 1, p.status, kStatusTimeoutAccFull)) alive = false;
      tc_fence_after();
      const float in_scale = kF16 ? 1.0f : ep_scale;
      const uint64_t s2 = f2_pack(in_scale, in_scale);
      const int oy0 = cur.row * p.th * p.mblocks + r_h;
      for (int mb = 0; mb < kMaxMB; ++mb) {
        if (mb >= p.mblocks) break;
        // M block mb of the super-tile: rows mb*th.. of the tile, columns mb*BN.. of the buffer
        const int oyb = oy0 + mb * p.th;
        const bool vb = r_h < p.th && r_w < p.tw && oyb < p.oh && ox < p.ow;
        const size_t pixb = (static_cast<size_t>(img) * p.oh + (vb ? oyb : 0)) * p.ow + (vb ? ox : 0);
        __half* outb = p.out + pixb * p.out_ldc + p.out_coff;
        const __half* resb = kRes ? p.res + pixb * p.res_ldc + p.res_coff : nullptr;
        const int srow = srow0 >= 0 ? srow0 + mb * p.th * p.tw : -1;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          uint32_t v[CW];
          const uint32_t taddr = lane_addr + buf * acc_cols + mb * BN + col0 + c * CW;
          if constexpr (CW == 32) {
            tmem_ld_32x32(taddr, v);
          } else {
            tmem_ld<16>(taddr, v);
          }
          tmem_ld_wait();
          if (c == kChunks - 1 && (kMaxMB == 1 || mb == p.mblocks - 1)) {
            // every column of this accumulator has been read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
          const int oc_c = n0 + col0 + c * CW;
          if (!kF16 && p.acc_dump != nullptr && vb) {
#pragma unroll
            for (int i = 0; i < CW; ++i)
              if (oc_c + i < p.oc) p.acc_dump[pixb * p.oc + oc_c + i] = static_cast<int32_t>(v[i]);
          }
          if (staged) {
#pragma unroll
            for (int g = 0; g < CW / 16; ++g) {
              const int lc = oc_c + 16 * g;  // output channel (the vectors are zero-padded to oc_alloc)
              uint4 rr[2], o[2];
              if constexpr (kRes) halo_load_res16(p, resb, lc, vb, rr);
              __half2 m2;
              if (kF16 || !p.acc_small)
                m2 = halo_epi16<kF16, kSilu, kRes, false>(v + 16 * g, s2, s_scale + lc, s_bias + lc, rr, o);
              else
                m2 = halo_epi16<kF16, kSilu, kRes, !kF16>(v + 16 * g, s2, s_scale + lc, s_bias + lc, rr, o);
              if (srow >= 0) {
                const int cc = (c * CW + 16 * g) >> 3;
                *reinterpret_cast<uint4*>(sbuf + halo_stage_off<kCols>(srow, cc)) = o[0];
                *reinterpret_cast<uint4*>(sbuf + halo_stage_off<kCols>(srow, cc + 1)) = o[1];
              }
              const float mg = vb ? fmaxf(__low2float(m2), __high2float(m2)) : 0.0f;
              run_max[c * (CW / 16) + g] = fmaxf(run_max[c * (CW / 16) + g], mg);
            }
            continue;
          }
          // the whole chunk exists and its rows allow 16-byte accesses: packed path (warp-uniform)
          const bool packed = oc_c + CW <= p.oc && p.out_vec && (!kRes || p.res_vec);
#pragma unroll
          for (int g = 0; g < CW / 16; ++g) {
            const int lc = oc_c + 16 * g;  // output channel (the vectors are zero-padded to oc_alloc)
            float mg;
            if (packed) {
              const __half2 m2 = halo_epilogue16_packed<kF16, kSilu, kRes>(
                  v + 16 * g, in_scale, s_scale + lc, s_bias + lc, vb, outb + lc, kRes ? resb + lc : nullptr);
              mg = fmaxf(__low2float(m2), __high2float(m2));
            } else {
              const float m0 = halo_epilogue8<kF16, kSilu, kRes>(p, v + 16 * g, in_scale, lc, s_scale + lc,
                                                                 s_bias + lc, vb, outb, resb);
              const float m1 = halo_epilogue8<kF16, kSilu, kRes>(p, v + 16 * g + 8, in_scale, lc + 8,
                                                                 s_scale + lc + 8, s_bias + lc + 8, vb, outb, resb);
              mg = fmaxf(m0, m1);
            }
            run_max[c * (CW / 16) + g] = fmaxf(run_max[c * (CW / 16) + g], mg);
          }
        }
      }
      }  // per-tensor
      if (staged) {
        // the group's box is complete once all four warps pass the barrier; the issuer's wait
        // before it guarantees that the previous tile's store has read the other buffer
        fence_proxy_async_smem();
        if (st_issuer) bulk_wait_read_all();
        named_bar_sync(2 + sgroup, 128);
        if (st_issuer && n0 + col0 < p.oc) {  // a column block past the last channel has nothing to store
          tma_store_4d(&p.out_map, sbuf, n0 + col0, cur.col * p.tw, cur.row * p.th * p.mblocks, img);
          bulk_commit_group();
        }
        ++jj;
      }
      if (p.amax_out != nullptr && !p.contiguous) {
        // this tile's maxima: warp max, then shared max over the four lane quadrants; the last
        // quadrant to arrive at this (ring slot, column block) issues the global atomics
        const int slot = u % kAmaxRing;
        uint32_t wmax[kGroups];
#pragma unroll
        for (int g = 0; g < kGroups; ++g) {
          wmax[g] = __reduce_max_sync(0xffffffffu, __float_as_uint(run_max[g]));
          run_max[g] = 0.0f;
        }
        if (lane == 0) {
#pragma unroll
          for (int g = 0; g < kGroups; ++g)
            if (wmax[g] != 0u) atomicMax(&am_ring[slot * 16 + col0 / 16 + g], wmax[g]);
          __threadfence_block();
          if (atomicAdd(&am_count[slot * 4 + colq], 1u) == 3u) {
            __threadfence_block();
            am_count[slot * 4 + colq] = 0u;
#pragma unroll
            for (int g = 0; g < kGroups; ++g) {
              const uint32_t v = atomicExch(&am_ring[slot * 16 + col0 / 16 + g], 0u);
              const int oc_g = n0 + col0 + 16 * g;
              if (v != 0u && oc_g < p.oc)
                atomicMax(&p.amax_out[static_cast<size_t>(img) * p.amax_stride + p.amax_goff + oc_g / 16], v);
            }
          }
        }
      }
    }
    if (p.amax_out != nullptr && p.contiguous && run_key >= 0) flush_amax();
    if (st_issuer) bulk_wait_all();  // the last boxes are written before the CTA's shared memory goes away
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace aexrt
