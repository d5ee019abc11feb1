// Single-pass amax + quantize of an NCHW fp16 activation whose 16-channel strips
// fit in shared memory (the standalone tensor of the reference's
// record_int8_prequant_activation, native/aexrt_d3d12_runtime.cpp:21466-21665;
// amax shader :3212-3275, pack shader :3277-3361).
//
// The two-kernel form reads the tensor twice (amax, then quantize) and pays a
// launch in between.  Here one thread-block cluster owns one image and one CTA
// owns a pixel slice of one 16-channel strip (the strip's 16 planes of H * W
// fp16 are contiguous in NCHW; slices keep a CTA's shared memory small enough
// for two CTAs per SM, so one loads while the other computes):
//   1. the CTA bulk-copies its 16 plane segments into shared memory, two planes
//      per mbarrier, and maxes |x| over each pair as it lands;
//   2. the CTAs of the cluster exchange their maxima through distributed shared
//      memory (group amax = max over the strip's slices, per-tensor amax = max
//      over the image);
//   3. each CTA quantizes its slice from shared memory into the slab16 layout
//      (one pixel = one 16-byte row of 16 codes, two pixels per thread with
//      packed fp32 products, coalesced stores) and the first slice of each strip
//      writes the scale-record slot and amax slot.
// HBM sees each input byte once and each code once.  The arithmetic is that of
// the two-kernel path: amax as fp16 |x| maxima, multiplier fl32(127 / amax)
// (0 when amax <= 0), code = low byte of round_half_even(fl32(x * mult)).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace aexrt {

constexpr int kClusterQuantThreads = 512;
constexpr int kClusterQuantChunks = 8;      // mbarriers: two channel planes each
constexpr int kClusterQuantMaxCtas = 8;     // portable cluster size
// dynamic shared memory of one CTA's strip slice: at most two CTAs per SM
constexpr int kClusterQuantMaxSliceBytes = 112 * 1024;
constexpr uint32_t kSliceFailed = 0x80000000u;

// Codes of one channel for two pixels: low byte of round_half_even(fl32(x * mult)) by the
// 1.5 * 2^23 addend, exact because |x * mult| <= 127 here (x is bounded by the amax that mult
// comes from).  The product is rounded on its own (packed multiply, then separate adds).
__device__ __forceinline__ void codes_pair(__half2 h, uint64_t m2, uint32_t& a, uint32_t& b) {
  const float2 f = __half22float2(h);
  float x, y;
  f2_unpack(f2_mul(f2_pack(f.x, f.y), m2), x, y);
  a = __float_as_uint(__fadd_rn(x, 12582912.0f));
  b = __float_as_uint(__fadd_rn(y, 12582912.0f));
}

// grid (groups * slices, n), cluster (groups * slices, 1, 1), block kClusterQuantThreads; CTA rank r
// owns pixels [s * hw_s, (s + 1) * hw_s) of 16-channel strip g = r / slices, s = r % slices;
// dynamic smem = 32 * hw_s bytes ([16 channels][hw_s] fp16).
// amax_g: [n][groups_total] uint32 float bits (stored: no clearing pass), or null.
// status: bit kStatusTimeoutFull when a copy did not land within wait_limit cycles; then no CTA of
// that image's cluster writes q, rec or amax_g (the maxima would be incomplete).
__global__ void __launch_bounds__(kClusterQuantThreads, 2)
    amax_quant_cluster_kernel(const __half* __restrict__ x, int c, int hw, int slices, int mode,
                              uint8_t* __restrict__ q, float* __restrict__ rec, uint32_t* __restrict__ amax_g,
                              int groups_total, int group_offset, uint32_t* status, long long wait_limit) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  extern __shared__ __align__(128) unsigned char strip_smem[];
  __shared__ __align__(8) uint64_t bar[kClusterQuantChunks];
  __shared__ uint32_t s_warp[32];
  // this slice's amax bits, read by the peer CTAs; bit 31 (never set in the bits of an |x| maximum)
  // marks a slice whose copies did not all land in time
  __shared__ uint32_t s_slice_amax;
  __shared__ float s_amax_t, s_amax_grp;
  __shared__ int s_ok, s_cluster_ok;
  const int ctas = gridDim.x, n = blockIdx.y;
  const int g = blockIdx.x / slices, sl = blockIdx.x - g * slices;
  const int groups = ctas / slices;
  const int hw_s = hw / slices;
  const uint32_t plane_bytes = 2u * static_cast<uint32_t>(hw_s);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // channel plane ch of this slice starts at element ((n * c + 16 g + ch) * hw + sl * hw_s)
  const __half* src = x + (static_cast<size_t>(n) * c + static_cast<size_t>(g) * 16) * hw + static_cast<size_t>(sl) * hw_s;
  if (tid == 0) {
    for (int k = 0; k < kClusterQuantChunks; ++k) mbar_init(&bar[k], 1);
    fence_mbar_init();
    s_ok = 1;
  }
  __syncthreads();
  if (tid == 0) {
    for (int k = 0; k < kClusterQuantChunks; ++k) {
      mbar_arrive_expect_tx(&bar[k], 2 * plane_bytes);
      for (int ch = 2 * k; ch < 2 * k + 2; ++ch)
        bulk_load(strip_smem + ch * plane_bytes, src + static_cast<size_t>(ch) * hw, plane_bytes, &bar[k]);
    }
  }
  // ---- 1. slice amax, two planes at a time as they land (16-byte vectors, |x| max in fp16)
  __half2 hm = __float2half2_rn(0.0f);
  bool ok = true;
  for (int k = 0; k < kClusterQuantChunks; ++k) {
    if (!mbar_wait_bounded_limit(&bar[k], 0, status, kStatusTimeoutFull, wait_limit)) {
      ok = false;
      break;
    }
    const uint32_t end = (2 * k + 2) * plane_bytes;
    for (uint32_t b = 2 * k * plane_bytes + 16u * tid; b < end; b += 16u * kClusterQuantThreads) {
      const uint4 v = *reinterpret_cast<const uint4*>(strip_smem + b);
      const __half2* h2 = reinterpret_cast<const __half2*>(&v);
      hm = __hmax2(hm, __hmax2(__hmax2(__habs2(h2[0]), __habs2(h2[1])), __hmax2(__habs2(h2[2]), __habs2(h2[3]))));
    }
  }
  if (!ok) s_ok = 0;
  uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(__low2float(hm), __high2float(hm))));
  if (lane == 0) s_warp[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = __reduce_max_sync(0xffffffffu, lane < kClusterQuantThreads / 32 ? s_warp[lane] : 0u);
    if (lane == 0) s_slice_amax = m | (s_ok ? 0u : kSliceFailed);
  }
  // ---- 2. group and per-tensor amax over the cluster's slices (distributed shared memory)
  cluster_sync_all();
  if (tid == 0) {
    uint32_t t = 0, gm = 0, failed = 0;
    for (int r = 0; r < ctas; ++r) {
      const uint32_t v = ld_peer_u32(&s_slice_amax, static_cast<uint32_t>(r));
      failed |= v & kSliceFailed;
      t = max(t, v & ~kSliceFailed);
      if (r / slices == g) gm = max(gm, v & ~kSliceFailed);
    }
    s_amax_t = __uint_as_float(t);
    s_amax_grp = __uint_as_float(gm);
    // one slice short of data makes the image's maxima wrong: then no CTA of the cluster writes
    s_cluster_ok = failed ? 0 : 1;
  }
  __syncthreads();
  const float amax_grp = s_amax_grp, amax_t = s_amax_t;
  const float a = mode == 1 ? amax_grp : amax_t;
  const float mult = a > 0.0f ? __fdiv_rn(127.0f, a) : 0.0f;
  // ---- 3. quantize from shared memory: two pixels per thread, one 16-byte slab row each
  if (s_cluster_ok) {
    const uint64_t m2 = f2_pack(mult, mult);
    uint8_t* dst = q + ((static_cast<size_t>(n) * groups + g) * hw + static_cast<size_t>(sl) * hw_s) * 16;
    for (int p = 2 * tid; p < hw_s; p += 2 * kClusterQuantThreads) {
      uint32_t ca[16], cb[16];
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        const __half2 h = *reinterpret_cast<const __half2*>(strip_smem + ch * plane_bytes + 2 * p);
        codes_pair(h, m2, ca[ch], cb[ch]);
      }
      uint32_t wa[4], wb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wa[j] = __byte_perm(__byte_perm(ca[4 * j], ca[4 * j + 1], 0x0040), __byte_perm(ca[4 * j + 2], ca[4 * j + 3], 0x0040),
                            0x5410);
        wb[j] = __byte_perm(__byte_perm(cb[4 * j], cb[4 * j + 1], 0x0040), __byte_perm(cb[4 * j + 2], cb[4 * j + 3], 0x0040),
                            0x5410);
      }
      uint4* o = reinterpret_cast<uint4*>(dst + static_cast<size_t>(p) * 16);
      o[0] = make_uint4(wa[0], wa[1], wa[2], wa[3]);
      o[1] = make_uint4(wb[0], wb[1], wb[2], wb[3]);
    }
    if (tid == 0 && sl == 0) {
      float* r = rec + static_cast<size_t>(n) * (1 + groups);
      r[1 + g] = amax_grp;
      if (g == 0) r[0] = amax_t;
      if (amax_g) amax_g[static_cast<size_t>(n) * groups_total + group_offset + g] = __float_as_uint(amax_grp);
    }
  } else if (tid == 0 && !s_ok) {
    // a copy that has not landed may still write this CTA's shared memory: wait for it with the
    // full limit (whatever limit the first wait had), so the CTA does not exit under its copies
    for (int k = 0; k < kClusterQuantChunks; ++k) mbar_wait_bounded(&bar[k], 0, status, kStatusTimeoutFull);
  }
  // peers may still be reading s_slice_amax: leave the cluster together (the CTA's threads converge
  // first: thread 0 may come from the wait above, and the cluster barrier is warp-aligned)
  __syncthreads();
  cluster_sync_all();
}

}  // namespace aexrt
