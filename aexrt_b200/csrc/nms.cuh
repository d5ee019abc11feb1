// YOLO post-process on the GPU: confidence filter, class-wise NMS, top-k.
//
// The reference records three D3D12 dispatches per frame for this
// (native/aexrt_d3d12_runtime.cpp:27104-27219): a decode-filter shader that
// appends candidates with an atomic counter (:15300-15355), an O(count^2)
// "mark" shader (:15637-15691) and a rank-by-counting top-k shader
// (:15693-15733).  Here one thread-block cluster of 1-8 CTAs owns one image and
// does all three in shared memory, so a batch is one launch and nothing but
// the detections and their count reaches HBM.  Every CTA of the cluster runs
// steps 1-2 on the same data (they come out identical); the rows of step 3
// are spread over the cluster's warps, and CTA 0 gathers the suppressed bits
// (mode 0) or the matrix rows (mode 1) through distributed shared memory and
// runs step 4.  Small batches take 8 CTAs per image, so that the O(count^2)
// pair tests of one image spread over eight SMs:
//
//   1. filter: the CTA walks the anchors in blocks of blockDim; a ballot +
//      warp-total scan compacts the passing anchors in ASCENDING ANCHOR ORDER
//      (one of the orders the reference's atomic append can produce; fixed
//      here so that results are deterministic) up to max_candidates;
//   2. rank: a bitonic sort of 64-bit keys (score descending, candidate index
//      ascending: exactly the shaders' "higher" relation), then the candidates
//      are permuted into rank order;
//   3. suppress: for rank r < rank j, same class, IoU > threshold, r suppresses
//      j.  A warp owns a row r and lane l tests column 32w + l, so one ballot is
//      one 32-bit word of row r and the lanes read consecutive boxes (no bank
//      conflicts).  Mode 0 (the reference's GPU "mark" rule) drops j if ANY
//      higher-ranked box suppresses it: the words are OR-ed per column word in
//      shared memory, no matrix is stored.  Mode 1 (the greedy rule of
//      yolo_postprocess, src/aexrt/yolo.py:996-1007) keeps the suppression
//      matrix (rank x 32-bit words in shared memory) and one warp scans it in
//      rank order, each kept row OR-ing its word into the removed set held one
//      word per lane;
//   4. top-k: the kept set is the complement of the suppressed bits; a box's
//      output slot is the popcount of kept bits before it; rows past the count
//      are zeroed (the reference leaves them as they were).
//
// Box and IoU arithmetic uses explicit round-to-nearest intrinsics (no FMA
// contraction) in the reference's operation order, so the kept set and the
// output rows are bit-identical to a float32 restatement on the CPU.  The
// division of IoU = inter / den is only carried out when the quotient lies
// within a relative 2^-20 of the threshold: outside that band the products
// den * thr * (1 +- 2^-20) (each off by at most 2^-23 relative) already decide
// fl(inter / den) > thr the same way.
#pragma once
#include "ptx.cuh"
#include <cstdint>

namespace aexrt {

constexpr int kNmsThreads = 512;
constexpr int kNmsMaxCandidates = 1024;  // 2 per thread; greedy matrix 1024 x 32 words = 128 KB

struct NmsParams {
  const float* y;        // [n][channels][anchors] (or [n][anchors][channels] when channels_last)
  int anchors, channels, nc, has_obj, channels_last;
  float conf, iou;
  int max_cand, max_det, mode, pow2;  // pow2 = sort width >= max_cand
  int csize;             // CTAs per image: one thread-block cluster of csize CTAs (1, 2, 4 or 8)
  float* dets;           // [n][max_det][6]: x1, y1, x2, y2, score, class
  uint32_t* counts;      // [n]
};

// Shared-memory bytes of one CTA (mode 1 adds the suppression matrix).
// The per-candidate arrays are sized for an even count so that the 8-byte keys after them stay aligned.
__host__ __device__ inline size_t nms_smem_bytes(int max_cand, int pow2, int mode) {
  const int words = (max_cand + 31) / 32;
  const size_t even = static_cast<size_t>((max_cand + 1) & ~1);
  size_t b = even * (16 + 4 + 4 + 4) + static_cast<size_t>(pow2) * 8 + 64 * 4 + 32 * 4;
  if (mode == 1) b += static_cast<size_t>(max_cand) * words * 4;
  return b;
}

__device__ __forceinline__ float nms_area(float4 a) {
  return __fmul_rn(fmaxf(0.f, __fsub_rn(a.z, a.x)), fmaxf(0.f, __fsub_rn(a.w, a.y)));
}

// fl(IoU(a, b)) > thr, IoU = inter / max(area_a + area_b - inter, 1e-7) in the shader's order.
// thr_lo / thr_hi = fl(thr * (1 -+ 2^-20)); fast = thr is in [1e-20, 1e20] (products stay normal).
__device__ __forceinline__ bool nms_suppresses(float4 a, float area_a, float4 b, float area_b, float thr,
                                               float thr_lo, float thr_hi, bool fast) {
  const float x1 = fmaxf(a.x, b.x), y1 = fmaxf(a.y, b.y);
  const float x2 = fminf(a.z, b.z), y2 = fminf(a.w, b.w);
  const float inter = __fmul_rn(fmaxf(0.f, __fsub_rn(x2, x1)), fmaxf(0.f, __fsub_rn(y2, y1)));
  const float den = fmaxf(__fsub_rn(__fadd_rn(area_a, area_b), inter), 1e-7f);
  if (fast) {
    if (inter > __fmul_rn(den, thr_hi)) return true;
    if (inter < __fmul_rn(den, thr_lo)) return false;
  }
  return __fdiv_rn(inter, den) > thr;
}

// Float -> uint32 whose unsigned order is the float order (+0 and -0 made equal first).
__device__ __forceinline__ uint32_t nms_orderable(float f) {
  const uint32_t u = __float_as_uint(__fadd_rn(f, 0.f));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kNmsThreads) yolo_nms_kernel(const NmsParams p) {
  grid_dep_launch();
  grid_dep_wait();  // programmatic dependent launch: see ptx.cuh
  extern __shared__ __align__(16) unsigned char nms_smem[];
  const int MC = p.max_cand;
  const int MCe = (MC + 1) & ~1;  // array stride: keeps `key` 8-byte aligned
  const int W = (MC + 31) / 32;
  float4* box = reinterpret_cast<float4*>(nms_smem);
  float* score = reinterpret_cast<float*>(box + MCe);
  float* cls = score + MCe;
  float* area = cls + MCe;
  uint64_t* key = reinterpret_cast<uint64_t*>(area + MCe);  // 28 * MCe bytes before it: a multiple of 8
  uint32_t* supp = reinterpret_cast<uint32_t*>(key + p.pow2);  // 32 words: suppressed / removed bits
  int* scan = reinterpret_cast<int*>(supp + 32);               // warp totals + running count
  uint32_t* mask = reinterpret_cast<uint32_t*>(scan + 64);     // mode 1: [MC][W]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int img = blockIdx.x / p.csize;
  // the cluster's CTAs run steps 1-2 alike on the same data and share step 3's rows; CTA 0 of the
  // cluster collects the suppressed bits and writes the detections
  const uint32_t crank = p.csize > 1 ? cluster_rank() : 0u;
  const float* y = p.y + static_cast<long>(img) * p.channels * p.anchors;
  const int off = p.has_obj ? 5 : 4;
  // element (ch, a) of this image's output0
  auto at = [&](int ch, int a) -> float {
    return p.channels_last ? y[static_cast<long>(a) * p.channels + ch] : y[static_cast<long>(ch) * p.anchors + a];
  };

  // ---- 1. filter + compaction in anchor order
  if (tid == 0) scan[32] = 0;
  if (tid < 32) supp[tid] = 0;
  __syncthreads();
  for (int base = 0; base < p.anchors; base += kNmsThreads) {
    const int running = scan[32];
    if (running >= MC) break;  // block-uniform
    const int a = base + tid;
    bool pass = false;
    float best = 0.f;
    int best_c = 0;
    if (a < p.anchors) {
      const float obj = p.has_obj ? at(4, a) : 1.f;
      best = p.has_obj ? __fmul_rn(obj, at(off, a)) : at(off, a);
      for (int c = 1; c < p.nc; ++c) {
        const float s = p.has_obj ? __fmul_rn(obj, at(off + c, a)) : at(off + c, a);
        if (s > best) {
          best = s;
          best_c = c;
        }
      }
      pass = !(best < p.conf);
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, pass);
    if (lane == 0) scan[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      const int v = lane < kNmsThreads / 32 ? scan[lane] : 0;
      int incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += t;
      }
      if (lane < kNmsThreads / 32) scan[lane] = incl - v;  // exclusive warp offsets
      if (lane == 31) scan[33] = incl;                     // block total
    }
    __syncthreads();
    const int pos = running + scan[warp] + __popc(bal & ((1u << lane) - 1u));
    if (pass && pos < MC) {
      const float cx = at(0, a), cy = at(1, a), w = at(2, a), h = at(3, a);
      const float hw = __fmul_rn(w, 0.5f), hh = __fmul_rn(h, 0.5f);
      box[pos] = make_float4(__fsub_rn(cx, hw), __fsub_rn(cy, hh), __fadd_rn(cx, hw), __fadd_rn(cy, hh));
      score[pos] = best;
      cls[pos] = static_cast<float>(best_c);
    }
    __syncthreads();
    if (tid == 0) scan[32] = running + scan[33];
    __syncthreads();
  }
  const int count = min(scan[32], MC);

  // ---- 2. rank: bitonic sort of (score desc, index asc), then permute into rank order
  for (int i = tid; i < p.pow2; i += kNmsThreads)
    key[i] = i < count ? (static_cast<uint64_t>(~nms_orderable(score[i])) << 32) | static_cast<uint32_t>(i)
                       : ~0ull;
  __syncthreads();
  for (int k = 2; k <= p.pow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < p.pow2; i += kNmsThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t ka = key[i], kb = key[ixj];
          const bool up = (i & k) == 0;
          if ((ka > kb) == up) {
            key[i] = kb;
            key[ixj] = ka;
          }
        }
      }
      __syncthreads();
    }
  }
  float4 rb[2];
  float rs[2], rc[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r = tid + t * kNmsThreads;
    if (r < count) {
      const int ci = static_cast<int>(static_cast<uint32_t>(key[r]));
      rb[t] = box[ci];
      rs[t] = score[ci];
      rc[t] = cls[ci];
    }
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r = tid + t * kNmsThreads;
    if (r < count) {
      box[r] = rb[t];
      score[r] = rs[t];
      cls[r] = rc[t];
      area[r] = nms_area(rb[t]);
    }
  }
  __syncthreads();

  // ---- 3. suppression words: bit j of word (r, w) = rank r suppresses rank j = 32w + bit
  const int wc = (count + 31) / 32;
  const bool fast = p.iou >= 1e-20f && p.iou <= 1e20f;
  const float thr_hi = __fmul_rn(p.iou, 1.0f + 0x1p-20f), thr_lo = __fmul_rn(p.iou, 1.0f - 0x1p-20f);
  // rows round-robin over the warps of the cluster; the greedy rule's matrix rows go to CTA 0
  constexpr int kWarps = kNmsThreads / 32;
  for (int r = warp + kWarps * static_cast<int>(crank); r < count; r += kWarps * p.csize) {
    const float4 br = box[r];
    const float cr = cls[r], ar = area[r];
    const int w0 = (r + 1) >> 5;  // first word holding a column > r
    if (p.mode == 1)
      for (int w = lane; w < w0; w += 32) {
        if (crank == 0)
          mask[r * W + w] = 0u;
        else
          st_peer_u32(&mask[r * W + w], 0, 0u);
      }
    for (int w = w0; w < wc; ++w) {
      const int j = w * 32 + lane;
      const bool s = j > r && j < count && cls[j] == cr &&
                     nms_suppresses(br, ar, box[j], area[j], p.iou, thr_lo, thr_hi, fast);
      const uint32_t bits = __ballot_sync(0xffffffffu, s);
      if (lane == 0) {
        if (p.mode == 1) {
          if (crank == 0)
            mask[r * W + w] = bits;
          else
            st_peer_u32(&mask[r * W + w], 0, bits);
        } else if (bits) {
          atomicOr(&supp[w], bits);
        }
      }
    }
  }
  __syncthreads();
  if (p.csize > 1) {
    // every CTA's rows are in (mode 1: CTA 0's matrix; mode 0: each CTA's own words); CTA 0 ORs the
    // words of the others, which stay resident until it has read them (second barrier)
    cluster_sync_all();
    if (p.mode == 0 && crank == 0 && tid < wc) {
      uint32_t v = supp[tid];
      for (int r = 1; r < p.csize; ++r) v |= ld_peer_u32(&supp[tid], static_cast<uint32_t>(r));
      supp[tid] = v;
    }
    cluster_sync_all();
    if (crank != 0) return;
  }
  if (p.mode == 1 && warp == 0) {
    // greedy: rows in rank order; a row that is still standing removes what it suppresses
    uint32_t removed = 0;  // word `lane`
    for (int r = 0; r < count; ++r) {
      const uint32_t word = __shfl_sync(0xffffffffu, removed, r >> 5);
      if (!((word >> (r & 31)) & 1u) && lane < wc) removed |= mask[r * W + lane];
    }
    supp[lane] = removed;
  }
  __syncthreads();

  // ---- 4. top-k: kept = not suppressed; slot = kept ranks before this one
  int total = 0;
  for (int w = 0; w < wc; ++w) {
    const uint32_t valid = (w == wc - 1 && (count & 31)) ? ((1u << (count & 31)) - 1u) : 0xffffffffu;
    total += __popc(~supp[w] & valid);
  }
  for (int r = tid; r < count; r += kNmsThreads) {
    const int w = r >> 5;
    if ((supp[w] >> (r & 31)) & 1u) continue;
    int slot = __popc(~supp[w] & ((1u << (r & 31)) - 1u));
    for (int v = 0; v < w; ++v) slot += __popc(~supp[v]);
    if (slot < p.max_det) {
      float* d = p.dets + (static_cast<long>(img) * p.max_det + slot) * 6;
      const float4 b = box[r];
      d[0] = b.x;
      d[1] = b.y;
      d[2] = b.z;
      d[3] = b.w;
      d[4] = score[r];
      d[5] = cls[r];
    }
  }
  // rows past the count are zeroed, so a detection buffer's contents depend only on this image
  const int kept = min(total, p.max_det);
  float* tail = p.dets + (static_cast<long>(img) * p.max_det + kept) * 6;
  for (int e = tid; e < (p.max_det - kept) * 6; e += kNmsThreads) tail[e] = 0.f;
  if (tid == 0) p.counts[img] = static_cast<uint32_t>(kept);
}

}  // namespace aexrt
