// C ABI of the B200 W8A8 backend (declared in include/aexrt_b200.h).
//
// Host side of the hot path: layout-8 weight quantization and repack into the
// K-slot layout the tcgen05 kernel streams, the reference's int8 shape guard,
// TMA descriptor encoding, tile / pipeline selection and the launches.  All
// launches are asynchronous and allocate nothing; only plan creation allocates
// (the packed weights, scales, bias and a status word).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/aexrt_b200.h"
#include "conv_halo.cuh"
#include "kernels.cuh"
#include "nms.cuh"
#include "psa.cuh"
#include "quant.cuh"
#include "quant_cluster.cuh"
#include "stem.cuh"
#include "yolo_ops.cuh"
#include "launch.cuh"

using namespace aexrt;

namespace {

thread_local std::string g_last_error;

int fail(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return 0;
}

bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  fail("%s: %s", what, cudaGetErrorString(e));
  return false;
}

// cuTensorMapEncodeTiled, fetched through the runtime so the library does not
// link libcuda directly (it must load on machines without a GPU driver).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled unavailable (no CUDA driver)") != 0;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail("TMA base address must be 16-byte aligned") != 0;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) s[i - 1] = strides_bytes[i - 1];
  }
  const CUresult r = fn(map, dt, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r)) != 0;
  return true;
}

// Output tile (tw x th <= 128 pixels) maximising the useful fraction of the
// 128-row MMA tile; ties prefer fewer, wider tiles.  max_tw keeps one TMA box
// row (tw pixels of 16 bytes) within the 256-element box limit.
void pick_tile(int oh, int ow, int max_tw, int& tw, int& th) {
  double best = -1.0;
  tw = th = 1;
  for (int w = 1; w <= std::min(ow, max_tw); ++w) {
    const int h = std::min(oh, 128 / w);
    const long tiles = static_cast<long>((oh + h - 1) / h) * ((ow + w - 1) / w);
    const double util = static_cast<double>(oh) * ow / (static_cast<double>(tiles) * 128.0);
    if (util > best + 1e-9) {
      best = util;
      tw = w;
      th = h;
    }
  }
}

}  // namespace

namespace aexrt {
// The library's one thread-local error message, shared by the runtime translation units.
void set_last_error(const char* msg) { g_last_error = msg; }
// Launch flags of this thread (aexrt_b200_set_launch_flags), read by launch_kernel (launch.cuh).
thread_local uint32_t g_launch_flags = 0;
uint32_t launch_flags() { return g_launch_flags; }
}  // namespace aexrt

struct AexrtB200ConvPlan {
  AexrtConv2DDesc desc{};
  uint32_t kind = 0, kernel_id = 0, flags = 0;
  bool f16 = false, pg = false;
  int k = 1, stride = 1, pad = 0;
  int slabs = 0;         // input slabs (16 ch int8, 8 ch fp16)
  int in_hp = 0, in_wp = 0;
  int tw = 0, th = 0, tiles_w = 0, tiles_h = 0;
  int bn = 0, n_tiles = 0, oc_alloc = 0;
  int q_total = 0, kk_p = 0, sps = 0, stages = 0, smem = 0;
  int grid = 0;          // persistent CTAs (one per SM, at most one per tile)
  int total_tiles = 0;
  // halo variant (conv_halo.cuh): whole weight tile resident, one halo per slab and tile
  bool halo = false;
  // quantize on load (AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD, int8 halo plans): fp16 NHWC sources are
  // loaded into a raw ring of ql_raw slots of ql_raw_bytes and converted in shared memory
  bool ql = false;
  int ql_raw = 0, ql_raw_bytes = 0;
  int order = 0;  // halo tile order (see conv_halo.cuh): 0 auto, 1 strided, 2 contiguous
  // pg16 halo: K steps pair two taps of one slab, ordered by their shared-memory offset
  int tap_pairs = 0, tap_a[5] = {0, 0, 0, 0, 0}, tap_b[5] = {-1, -1, -1, -1, -1};
  int mblocks = 1, nacc = 4, tmem_cols = 512;  // super-tile M blocks, TMEM buffers and columns
  // plan bit 30: two MMA issuers even when half the stage ring holds less than a tile (the default
  // for per-tensor plans since it was measured faster; the bit is kept for tuned maps)
  bool two_issuers = false;
  // staged output (conv_halo.cuh): buffers per epilogue group (0: direct stores) and their bytes
  int out_nbuf = 0, out_gbytes = 0;
  // every |int32 accumulator| <= 2^22 (bounded from the weight codes): exact fast conversion
  bool acc_small = false;
  int pitch = 0, halo_rows = 0, boxes_per_slab = 1, slab_pairs = 0, taps = 1, w_tile_bytes = 0, m_tiles = 0;
  void* d_w = nullptr;   // [n_tile][q_total][bn][16 bytes]
  float* d_scale = nullptr;
  float* d_bias = nullptr;
  // SiLU plans: [scale/2 | bias/2] for the halo epilogue, which forms h = y/2 directly
  float* d_half_sb = nullptr;
  uint32_t* d_status = nullptr;
  int device = 0;
  // image stem (fp16, 3 input channels, 3x3): direct kernel reading fp16 or fp32 NCHW images
  bool image_input = false;
  StemWeights stem{};
};

namespace {

// Kernel instances live in their own translation units (kernels_*.cu), compiled in parallel.
// Dynamic shared memory of a conv CTA: the B200's 227 KB.  Halo pipelines and weights take at
// most kConvStageBudget of it; the rest goes first to the staged output buffers.
constexpr int kMaxConvSmem = 227 * 1024;
constexpr int kConvStageBudget = 200 * 1024;
// The activation kernels put the image index in a grid's y or z dimension.
constexpr uint32_t kMaxImagesPerLaunch = 65535;
// Halo tile: output tw x th on an M grid of pitch = tw + (2 for 3x3 s1, 1 for 3x3 s2, 0 for 1x1)
// <= max_pitch (one TMA box row of pitch pixels within the 256-element limit), th*pitch <= 128.
bool pick_halo_tile(int oh, int ow, int k, int s, int max_pitch, int& tw, int& th, int& pitch) {
  const int extra = k == 1 ? 0 : (s == 1 ? 2 : 1);
  double best = -1.0;
  for (int w = 1; w + extra <= max_pitch && w <= ow; ++w) {
    const int pt = w + extra;
    const int h = std::min(oh, 128 / pt);
    if (h < 1) continue;
    const long tiles = static_cast<long>((oh + h - 1) / h) * ((ow + w - 1) / w);
    const double util = static_cast<double>(oh) * ow / (static_cast<double>(tiles) * 128.0);
    if (util > best + 1e-9) {
      best = util;
      tw = w;
      th = h;
      pitch = pt;
    }
  }
  return best > 0.0;
}

int choose_bn(int oc, bool pg, uint32_t requested) {
  if (requested) return static_cast<int>(requested);
  const int cands[] = {256, 128, 64, 32, 16};
  int best = 16;
  long best_waste = 1L << 40;
  for (int c : cands) {
    if (pg && c > 128) continue;
    const int tiles = (oc + c - 1) / c;
    const long waste = static_cast<long>(tiles) * c - oc;
    if (waste < best_waste) {  // first (largest) tile with the least padding
      best_waste = waste;
      best = c;
    }
  }
  return best;
}

bool check_desc_int8(const AexrtConv2DDesc& d, uint32_t kernel_id, bool pg) {
  // can_use_conv_int8 (native/aexrt_d3d12_runtime.cpp:9398-9422)
  if (d.groups != 1 || d.in_channels % 4 || d.out_channels % 4)
    return fail("int8 conv needs groups == 1, in_channels %% 4 == 0, out_channels %% 4 == 0") != 0;
  if (d.dilation_h != 1 || d.dilation_w != 1) return fail("int8 conv needs dilation 1") != 0;
  if (kernel_id == 51) {
    if (d.kernel_h != 1 || d.kernel_w != 1 || d.stride_h != 1 || d.stride_w != 1 || d.pad_top || d.pad_left)
      return fail("kernel 51 needs a 1x1 stride-1 conv without padding") != 0;
    if (d.out_channels % 8 || d.in_h != d.out_h || d.in_w != d.out_w)
      return fail("kernel 51 needs out_channels %% 8 == 0 and same spatial size") != 0;
  } else if (kernel_id == 52 || kernel_id == 53) {
    if (d.kernel_h != 3 || d.kernel_w != 3 || d.pad_top != 1 || d.pad_left != 1)
      return fail("kernels 52/53 need a 3x3 conv with padding 1") != 0;
    if (kernel_id == 52) {
      if (d.stride_h != 1 || d.stride_w != 1 || d.in_h != d.out_h || d.in_w != d.out_w)
        return fail("kernel 52 needs stride 1 and same spatial size") != 0;
    } else {
      if (d.stride_h != 2 || d.stride_w != 2 || d.in_h < d.out_h * 2 - 1 || d.in_w < d.out_w * 2 - 1)
        return fail("kernel 53 needs stride 2 and in >= 2*out-1") != 0;
      if (d.out_h != (d.in_h + 1) / 2 || d.out_w != (d.in_w + 1) / 2)
        return fail("kernel 53 output size must be ceil(in/2)") != 0;
    }
  } else {
    return fail("unknown int8 kernel id %u (expected 51, 52 or 53)", kernel_id) != 0;
  }
  if (pg && d.in_channels % 16) return fail("pg16 scaling needs in_channels %% 16 == 0") != 0;
  if (d.batch == 0 || d.out_h == 0 || d.out_w == 0) return fail("empty conv") != 0;
  return true;
}

cudaError_t set_halo_smem(bool f16, int bn, bool silu, bool pg, bool mb, bool ql) {
  for (int res = 0; res < 2; ++res) {
    const HaloFn fn = halo_kernel_for(f16, bn, silu, res, pg, mb, ql).fn;
    if (!fn) continue;  // no residual instance for this combination
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxConvSmem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

AexrtB200ConvPlan* build_plan(const AexrtConv2DDesc& d, uint32_t kind, uint32_t kernel_id, uint32_t flags, bool f16,
                              const void* host_w, const float* scale, const float* bias, uint32_t block_n) {
  if (kind != AEXRT_B200_KIND_CONV && kind != AEXRT_B200_KIND_CONV_SILU) {
    fail("kind must be CONV (1) or CONV_SILU (2)");
    return nullptr;
  }
  if (!host_w || !bias || (!f16 && !scale)) {
    fail("null weight/scale/bias pointer");
    return nullptr;
  }
  auto* p = new AexrtB200ConvPlan();
  p->desc = d;
  p->kind = kind;
  p->kernel_id = kernel_id;
  p->flags = flags;
  p->f16 = f16;
  p->pg = !f16 && (flags & AEXRT_B200_PLAN_FLAG_INT8_PERGROUP);
  p->k = static_cast<int>(d.kernel_h);
  p->stride = static_cast<int>(d.stride_h);
  p->pad = static_cast<int>(d.pad_top);
  const int cps = f16 ? 8 : 16;  // channels per slot
  const int ic = static_cast<int>(d.in_channels), oc = static_cast<int>(d.out_channels);
  const int kk = p->k * p->k;
  p->slabs = (ic + cps - 1) / cps;
  p->in_hp = static_cast<int>(d.in_h) + (p->stride == 2 ? (d.in_h & 1) : 0);
  p->in_wp = static_cast<int>(d.in_w) + (p->stride == 2 ? (d.in_w & 1) : 0);
  pick_tile(static_cast<int>(d.out_h), static_cast<int>(d.out_w), f16 ? 32 : 16, p->tw, p->th);
  p->tiles_w = (static_cast<int>(d.out_w) + p->tw - 1) / p->tw;
  p->tiles_h = (static_cast<int>(d.out_h) + p->th - 1) / p->th;
  const uint32_t variant = (block_n >> 16) & 0xF;  // 0 auto, 1 slot streaming, 2 halo
  const uint32_t order = (block_n >> 20) & 0xF;    // halo tile order: 0 auto, 1 strided, 2 contiguous
  const int mblocks_cap = static_cast<int>((block_n >> 24) & 0xF);  // super-tile M blocks: 0 auto, else at most
  // staged TMA-store epilogue: bit 29 asks for it, bit 28 forces direct stores (the default).  Measured
  // at batch 64: 1x1 128->128 @40 24.6 us staged against 26.7 us direct, but the 3x3 layers ran 4-9 %
  // slower staged (the per-tile barrier holds the four warps of a column block in step), and the
  // YOLOv8n-320 step at batch 256 was 1.3 % slower even with only its 1x1 convs staged
  const bool direct_store = ((block_n >> 28) & 1u) != 0 || ((block_n >> 29) & 1u) == 0;
  p->two_issuers = !p->pg && ((block_n >> 30) & 1u) != 0;
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  block_n &= 0xFFFF;
  p->bn = choose_bn(oc, p->pg, block_n);
  if (!block_n) {
    // small grids (one or a few images): narrower output-channel tiles until the conv spreads over at
    // least a third of the SMs, so that each CTA loads and multiplies a smaller weight tile (the
    // latency of a batch-1 layer is one CTA's weight load, MMAs and epilogue)
    const long m_tiles = static_cast<long>(d.batch) * p->tiles_h * p->tiles_w;
    while (p->bn > (p->pg ? 64 : 32) && m_tiles * ((oc + p->bn - 1) / p->bn) * 3 < sms) p->bn /= 2;
  }
  if (!kernel_for(f16, p->pg, p->bn)) {
    fail("unsupported block_n %d", p->bn);
    delete p;
    return nullptr;
  }
  p->n_tiles = (oc + p->bn - 1) / p->bn;
  p->oc_alloc = p->n_tiles * p->bn;
  if (p->pg) {
    p->kk_p = (kk + 1) & ~1;
    p->q_total = p->slabs * p->kk_p;
  } else {
    p->kk_p = 0;
    p->q_total = (kk * p->slabs + 1) & ~1;
  }
  p->sps = std::min(16, p->q_total);
  {
    // one persistent CTA per SM: spend up to ~200 KB of shared memory on pipeline stages
    const ConvSmemPlan one = conv_smem_plan(p->tw, p->th, p->sps, 1, p->bn);
    const int budget = 200 * 1024;
    const int st = std::max(2, std::min((budget - 2048 - 256) / one.stage_bytes, 8));
    p->stages = st;
    p->smem = conv_smem_plan(p->tw, p->th, p->sps, st, p->bn).total_bytes;
  }
  p->total_tiles = static_cast<int>(d.batch) * p->tiles_h * p->tiles_w * p->n_tiles;

  // ---- halo variant: per-tensor int8, fp16, or pg16 with 64/128-wide output tiles, when the whole
  // weight tile fits next to >= 2 stages (with an automatic tile width, narrower output-channel
  // tiles are tried before giving up)
  if (variant != 1) {
    int tw = 0, th = 0, pitch = 0;
    const int taps = kk;
    const int pairs = (p->slabs + 1) / 2;
    const int tap_pairs = (kk + 1) / 2;
    // (pg16: the epilogue's per-warp group-scale table holds kMaxSlabsPg slabs)
    const bool tile_ok = pick_halo_tile(static_cast<int>(d.out_h), static_cast<int>(d.out_w), p->k, p->stride,
                                        f16 ? 32 : 16, tw, th, pitch) &&
                         !(p->pg && p->slabs > kMaxSlabsPg);
    const int bn_min = p->pg ? 64 : 16;
    for (int bn = p->bn; tile_ok && !p->halo && bn >= bn_min; bn = block_n ? 0 : bn / 2) {
      if (p->pg && bn != 64 && bn != 128) continue;
      const int n_tiles = (oc + bn - 1) / bn;
      const int oc_alloc = n_tiles * bn;
      // resident weights: [pair][tap][2][bn][16] (per tensor) or [slab][tap pair][2][bn][16] (pg16)
      const int w_tile = p->pg ? p->slabs * tap_pairs * 2 * bn * 16 : pairs * taps * 2 * bn * 16;
      // super-tiles for narrow per-tensor tiles: stack M blocks (halving the per-tile pipeline costs
      // each time) while the map has the rows and the batch still gives every SM >= 2 tiles
      // (3x3 stride 1 only: there they also share halo rows; measured no gain for 1x1 and stride 2)
      int mblocks = 1;
      const int kernel_mb = p->pg || bn > 64 ? 1 : (bn <= 32 ? 4 : 2);  // the kernel's kMaxMB
      if (p->k == 3 && p->stride == 1 && mblocks_cap != 1) {
        const int max_r = std::min(kernel_mb, mblocks_cap ? mblocks_cap : kernel_mb);
        const long tw_tiles = (static_cast<long>(d.out_w) + tw - 1) / tw;
        while (mblocks * 2 <= max_r && mblocks * 2 * th <= static_cast<int>(d.out_h) &&
               static_cast<long>(d.batch) * ((d.out_h + mblocks * 2 * th - 1) / (mblocks * 2 * th)) * tw_tiles *
                       n_tiles >= 2L * sms)
          mblocks *= 2;
      }
      const int boxes = p->stride == 2 ? 4 : 1;
      const int budget = kConvStageBudget - 1024;
      const bool want_ql = !f16 && (flags & AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD);
      int halo_h = 0, st = 0, raw_slots = 0, raw_bytes = 0, out_nbuf = 0, out_gbytes = 0;
      for (;; mblocks /= 2) {
        // keep >= 4 stages (and a whole tile per issuer half ring) for a super-tile, else fewer blocks
        halo_h = mblocks * th + (p->k == 1 ? 0 : (p->stride == 1 ? 2 : 1));
        const HaloSmemPlan one = halo_smem_plan(halo_h * pitch, boxes, 1, w_tile, oc_alloc, 0, 0, p->pg);
        // quantize on load: a raw ring of 3 (else 2) slots, each the fp16 boxes of one stage (twice
        // its int8 bytes), while >= 4 stages remain
        raw_slots = 0;
        raw_bytes = want_ql ? 2 * one.stage_bytes : 0;
        for (int rs = want_ql ? 3 : 0; rs >= 2; --rs) {
          if ((budget - one.total_bytes - rs * raw_bytes) / one.stage_bytes + 1 >= 4) {
            raw_slots = rs;
            break;
          }
        }
        st = std::min(16, (budget - one.total_bytes - raw_slots * raw_bytes) / one.stage_bytes + 1);
        if (mblocks == 1 || st >= std::max(4, 2 * pairs)) break;
      }
      // staged output: two buffers per epilogue group (else one) from the whole 227 KB, while the
      // pipeline keeps min(st, max(4, 2 * pairs)) stages; the TMA box holds <= 256 rows
      if (st >= 2 && mblocks * th <= 256 && !direct_store) {
        const HaloSmemPlan one = halo_smem_plan(halo_h * pitch, boxes, 1, w_tile, oc_alloc, 0, 0, p->pg);
        const int gbytes = halo_out_gbytes(bn, p->pg, mblocks * th * tw);
        const int keep = std::min(st, std::max(4, 2 * pairs));
        for (int nb = 2; nb >= 1; --nb) {
          const int total = one.total_bytes + raw_slots * raw_bytes + 4 * nb * gbytes + 2048;  // + alignment
          const int st_o = std::min(16, (kMaxConvSmem - 1024 - total) / one.stage_bytes + 1);
          if (st_o >= keep) {
            out_nbuf = nb;
            out_gbytes = gbytes;
            st = std::min(st, st_o);
            break;
          }
        }
      }
      if (st >= 2) {
        // TMEM accumulators: nacc buffers of mblocks*bn columns (a multiple of the two issuers and of
        // the epilogue tile groups); pg16 uses 512 / bn units of bn columns
        const int acc_cols = mblocks * bn;
        int nacc = p->pg ? 512 / bn
                         : (mblocks > 1 ? std::min(16, 512 / acc_cols)
                                        : (bn <= 16 ? 16 : (bn <= 32 ? 8 : (bn <= 128 ? 4 : 2))));
        int cols = 32;
        while (cols < nacc * (p->pg ? bn : acc_cols)) cols *= 2;
        p->mblocks = mblocks;
        p->nacc = nacc;
        p->tmem_cols = cols;
        p->bn = bn;
        p->n_tiles = n_tiles;
        p->oc_alloc = oc_alloc;
        p->halo = true;
        p->ql = raw_slots > 0;
        p->ql_raw = raw_slots;
        p->ql_raw_bytes = raw_slots > 0 ? raw_bytes : 0;
        p->order = static_cast<int>(order);
        p->tw = tw;
        p->th = th;
        p->pitch = pitch;
        p->halo_rows = halo_h * pitch;
        p->boxes_per_slab = boxes;
        p->slab_pairs = pairs;
        p->taps = taps;
        p->w_tile_bytes = w_tile;
        p->stages = st;
        p->out_nbuf = out_nbuf;
        p->out_gbytes = out_gbytes;
        p->smem = halo_smem_plan(p->halo_rows, boxes, st, w_tile, p->oc_alloc, p->ql_raw * p->ql_raw_bytes,
                                 4 * out_nbuf * out_gbytes, p->pg)
                      .total_bytes;
        p->tiles_w = (static_cast<int>(d.out_w) + tw - 1) / tw;
        p->tiles_h = (static_cast<int>(d.out_h) + mblocks * th - 1) / (mblocks * th);
        p->m_tiles = static_cast<int>(d.batch) * p->tiles_h * p->tiles_w;
        p->total_tiles = p->m_tiles * p->n_tiles;
        if (p->pg) {
          // tap offsets inside a stage slab (the kernel's tap_off), then pairs in ascending order
          const int box_bytes = ((p->halo_rows * 16 + 127) / 128) * 128;
          int order_t[9], off[9];
          for (int tap = 0; tap < kk; ++tap) {
            const int kh = tap / 3, kw = tap % 3;
            off[tap] = 0;
            if (p->stride == 2)
              off[tap] = (((kh + 1) & 1) * 2 + ((kw + 1) & 1)) * box_bytes + ((kh ? 1 : 0) * pitch + (kw ? 1 : 0)) * 16;
            else if (p->k == 3)
              off[tap] = (kh * pitch + kw) * 16;
            order_t[tap] = tap;
          }
          std::sort(order_t, order_t + kk, [&](int a, int b) { return off[a] < off[b]; });
          p->tap_pairs = tap_pairs;
          for (int m = 0; m < tap_pairs; ++m) {
            p->tap_a[m] = order_t[2 * m];
            p->tap_b[m] = 2 * m + 1 < kk ? order_t[2 * m + 1] : -1;
          }
        }
      }
    }
    if (variant == 2 && !p->halo) {
      fail("halo variant does not fit this conv");
      delete p;
      return nullptr;
    }
  }

  // int8 accumulators are bounded by 128 * sum_k |w[o][k]| (|activation code| <= 127 when its scale
  // comes from the tensor's amax): within 2^22 the epilogue converts them on full-rate pipes
  if (!f16) {
    long worst = 0;
    const int8_t* wc = static_cast<const int8_t*>(host_w);
    for (int o = 0; o < oc; ++o) {
      long s = 0;
      for (size_t j = 0; j < static_cast<size_t>(ic) * kk; ++j) s += std::abs(static_cast<int>(wc[static_cast<size_t>(o) * ic * kk + j]));
      worst = std::max(worst, s);
    }
    p->acc_small = 128L * worst <= (1L << 22);
  }

  // ---- weight repack.  Slot streaming: [n_tile][slot][bn][16 bytes] (one stage of B is one
  // contiguous run).  Halo: [n_tile][slab pair][tap][2][bn][16 bytes] (the resident tile).
  const size_t slot_row = 16;
  std::vector<uint8_t> packed(static_cast<size_t>(p->halo ? p->n_tiles * p->w_tile_bytes
                                                          : static_cast<size_t>(p->q_total) * p->oc_alloc * slot_row),
                              0);
  if (p->halo && p->pg) {
    // pg16 halo: [n_tile][slab][tap pair][2 (tap a, tap b)][bn][16 bytes]; a missing tap b is zero
    for (int nt = 0; nt < p->n_tiles; ++nt)
      for (int slab = 0; slab < p->slabs; ++slab)
        for (int m = 0; m < p->tap_pairs; ++m)
          for (int ch = 0; ch < 2; ++ch) {
            const int tap = ch ? p->tap_b[m] : p->tap_a[m];
            if (tap < 0) continue;
            for (int on = 0; on < p->bn; ++on) {
              const int o = nt * p->bn + on;
              if (o >= oc) continue;
              uint8_t* dst = packed.data() + static_cast<size_t>(nt) * p->w_tile_bytes +
                             ((((static_cast<size_t>(slab) * p->tap_pairs + m) * 2 + ch) * p->bn) + on) * slot_row;
              for (int c = 0; c < cps; ++c) {
                const int ci = slab * cps + c;
                if (ci >= ic) continue;
                dst[c] = static_cast<uint8_t>(
                    static_cast<const int8_t*>(host_w)[(static_cast<size_t>(o) * ic + ci) * kk + tap]);
              }
            }
          }
  } else if (p->halo) {
    for (int nt = 0; nt < p->n_tiles; ++nt)
      for (int pr = 0; pr < p->slab_pairs; ++pr)
        for (int tap = 0; tap < kk; ++tap)
          for (int ch = 0; ch < 2; ++ch) {
            const int slab = 2 * pr + ch;
            if (slab >= p->slabs) continue;
            for (int on = 0; on < p->bn; ++on) {
              const int o = nt * p->bn + on;
              if (o >= oc) continue;
              uint8_t* dst = packed.data() + static_cast<size_t>(nt) * p->w_tile_bytes +
                             ((((static_cast<size_t>(pr) * kk + tap) * 2 + ch) * p->bn) + on) * slot_row;
              for (int c = 0; c < cps; ++c) {
                const int ci = slab * cps + c;
                if (ci >= ic) continue;
                const size_t src = (static_cast<size_t>(o) * ic + ci) * kk + tap;
                if (f16) {
                  const __half h = __float2half_rn(static_cast<const float*>(host_w)[src]);
                  std::memcpy(dst + 2 * c, &h, 2);
                } else {
                  dst[c] = static_cast<uint8_t>(static_cast<const int8_t*>(host_w)[src]);
                }
              }
            }
          }
  }
  for (int q = 0; q < (p->halo ? 0 : p->q_total); ++q) {
    int tap, slab;
    if (p->pg) {
      slab = q / p->kk_p;
      tap = q - slab * p->kk_p;
      if (tap >= kk || slab >= p->slabs) tap = -1;
    } else {
      tap = q / p->slabs;
      slab = q - tap * p->slabs;
      if (tap >= kk) tap = -1;
    }
    if (tap < 0) continue;
    for (int o = 0; o < oc; ++o) {
      const int nt = o / p->bn, on = o - nt * p->bn;
      uint8_t* dst = packed.data() + ((static_cast<size_t>(nt) * p->q_total + q) * p->bn + on) * slot_row;
      for (int c = 0; c < cps; ++c) {
        const int ci = slab * cps + c;
        if (ci >= ic) continue;
        const size_t src = (static_cast<size_t>(o) * ic + ci) * kk + tap;
        if (f16) {
          const __half h = __float2half_rn(static_cast<const float*>(host_w)[src]);
          std::memcpy(dst + 2 * c, &h, 2);
        } else {
          dst[c] = static_cast<uint8_t>(static_cast<const int8_t*>(host_w)[src]);
        }
      }
    }
  }
  bool ok = cuda_ok(cudaGetDevice(&p->device), "cudaGetDevice") &&
            cuda_ok(cudaMalloc(&p->d_w, packed.size()), "cudaMalloc(weights)") &&
            cuda_ok(cudaMemcpy(p->d_w, packed.data(), packed.size(), cudaMemcpyHostToDevice), "copy weights") &&
            cuda_ok(cudaMalloc(reinterpret_cast<void**>(&p->d_bias), sizeof(float) * p->oc_alloc), "cudaMalloc(bias)") &&
            cuda_ok(cudaMemset(p->d_bias, 0, sizeof(float) * p->oc_alloc), "memset(bias)") &&
            cuda_ok(cudaMemcpy(p->d_bias, bias, sizeof(float) * oc, cudaMemcpyHostToDevice), "copy bias") &&
            cuda_ok(cudaMalloc(reinterpret_cast<void**>(&p->d_status), sizeof(uint32_t)), "cudaMalloc(status)") &&
            cuda_ok(cudaMemset(p->d_status, 0, sizeof(uint32_t)), "memset(status)");
  if (ok) {
    // per-output-channel weight scale, zero-padded to the n-tile multiple (1.0 for fp16 plans)
    std::vector<float> sc(p->oc_alloc, 0.0f);
    for (int o = 0; o < oc; ++o) sc[o] = f16 ? 1.0f : scale[o];
    ok = cuda_ok(cudaMalloc(reinterpret_cast<void**>(&p->d_scale), sizeof(float) * p->oc_alloc), "cudaMalloc(scale)") &&
         cuda_ok(cudaMemcpy(p->d_scale, sc.data(), sizeof(float) * p->oc_alloc, cudaMemcpyHostToDevice), "copy scale");
    if (ok && kind == AEXRT_B200_KIND_CONV_SILU) {
      std::vector<float> hsb(2 * static_cast<size_t>(p->oc_alloc), 0.0f);
      for (int o = 0; o < oc; ++o) {
        hsb[o] = 0.5f * sc[o];
        hsb[p->oc_alloc + o] = 0.5f * bias[o];
      }
      ok = cuda_ok(cudaMalloc(reinterpret_cast<void**>(&p->d_half_sb), sizeof(float) * hsb.size()), "cudaMalloc(sb)") &&
           cuda_ok(cudaMemcpy(p->d_half_sb, hsb.data(), sizeof(float) * hsb.size(), cudaMemcpyHostToDevice), "copy sb");
    }
  }
  if (ok) {
    int sms = 0;
    ok = cuda_ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device), "SM count");
    p->grid = std::max(1, std::min(p->total_tiles, sms));
  }
  if (ok) {
    // the attribute is a per-kernel cap shared by every plan of this instance: set it to the
    // largest dynamic shared memory any plan may request, never to this plan's size
    ok = p->smem <= kMaxConvSmem &&
         cuda_ok(p->halo ? set_halo_smem(f16, p->bn, kind == AEXRT_B200_KIND_CONV_SILU, p->pg, p->mblocks > 1, false)
                         : cudaFuncSetAttribute(kernel_for(f16, p->pg, p->bn),
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxConvSmem),
                 "cudaFuncSetAttribute");
    if (ok && p->ql)
      ok = cuda_ok(set_halo_smem(false, p->bn, kind == AEXRT_B200_KIND_CONV_SILU, p->pg, p->mblocks > 1, true),
                   "cudaFuncSetAttribute");
    if (p->smem > kMaxConvSmem) fail("conv plan needs %d bytes of shared memory", p->smem);
  }
  if (!ok) {
    aexrt_b200_conv_plan_destroy(p);
    return nullptr;
  }
  return p;
}

bool encode_act_map(const AexrtB200ConvPlan* p, const void* x, CUtensorMap* map) {
  const uint64_t hp = p->in_hp, wp = p->in_wp;
  const uint64_t sn = static_cast<uint64_t>(p->slabs) * p->desc.batch;
  const uint32_t ce = p->f16 ? 8 : 16;  // elements per 16-byte slot (one pixel of one slab)
  const CUtensorMapDataType dt = p->f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  if (p->halo) {
    const uint32_t box_x = ce * static_cast<uint32_t>(p->pitch);  // one box row = pitch pixels
    const uint32_t box_h = static_cast<uint32_t>(p->halo_rows / p->pitch);
    if (p->stride == 1) {
      const uint64_t dims[3] = {ce * wp, hp, sn};
      const uint64_t strides[2] = {16 * wp, 16 * wp * hp};
      const uint32_t box[3] = {box_x, box_h, 1};
      return encode_map(map, dt, 3, x, dims, strides, box);
    }
    const uint64_t dims[5] = {ce * wp / 2, 2, 2, hp / 2, sn};
    const uint64_t strides[4] = {8 * wp, 16 * wp, 32 * wp, 16 * wp * hp};
    const uint32_t box[5] = {box_x, 1, 1, box_h, 1};
    return encode_map(map, dt, 5, x, dims, strides, box);
  }
  const uint32_t box_x = ce * static_cast<uint32_t>(p->tw);  // one box row = tw pixels
  if (p->stride == 1) {
    // [image*slab][H][W*16 bytes]
    const uint64_t dims[3] = {ce * wp, hp, sn};
    const uint64_t strides[2] = {16 * wp, 16 * wp * hp};
    const uint32_t box[3] = {box_x, static_cast<uint32_t>(p->th), 1};
    return encode_map(map, dt, 3, x, dims, strides, box);
  }
  // [image*slab][H/2][2 (row parity)][2 (column parity)][W/2 * 16 bytes]
  const uint64_t dims[5] = {ce * wp / 2, 2, 2, hp / 2, sn};
  const uint64_t strides[4] = {8 * wp, 16 * wp, 32 * wp, 16 * wp * hp};
  const uint32_t box[5] = {box_x, 1, 1, static_cast<uint32_t>(p->th), 1};
  return encode_map(map, dt, 5, x, dims, strides, box);
}

// The quantize-on-load fields of a launch (aexrt_b200_conv_w8a8_sources): sources and their maps.
struct QlLaunch {
  int parts = 0, mode = 0;
  int slab0[kQlMaxParts] = {}, up[kQlMaxParts] = {}, box_w[kQlMaxParts] = {}, box_h[kQlMaxParts] = {};
  int groups[kQlMaxParts] = {}, amax_stride[kQlMaxParts] = {}, amax_goff[kQlMaxParts] = {};
  const uint32_t* amax[kQlMaxParts] = {};
  CUtensorMap map[kQlMaxParts];
};

// nhwc_map: an fp16 stride-1 halo plan reading the NHWC activation directly (see aexrt_b200_conv_f16_nhwc)
// ql: an int8 plan converting fp16 NHWC sources on load (x and scale_rec unused)
int launch_conv(const AexrtB200ConvPlan* p, const void* x, const float* scale_rec, const void* res, uint32_t res_ldc,
                uint32_t res_coff, void* out, uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out,
                uint32_t amax_stride, uint32_t amax_goff, int32_t* acc_dump, void* stream,
                const CUtensorMap* nhwc_map = nullptr, const QlLaunch* ql = nullptr) {
  if (!p) return fail("null plan");
  if ((!x && !ql) || !out) return fail("null input/output pointer");
  if (!p->f16 && !scale_rec && !ql) return fail("null scale record");
  const uint32_t oc = p->desc.out_channels;
  if (out_ldc < out_coff + oc || reinterpret_cast<uintptr_t>(out) % 2)
    return fail("output slice out of range (need coff + oc <= ldc)");
  if (res && (res_ldc < res_coff + oc || reinterpret_cast<uintptr_t>(res) % 2))
    return fail("residual slice out of range (need coff + oc <= ldc)");
  if (amax_out && (amax_goff * 16 + oc > amax_stride * 16 || out_coff % 16))
    return fail("amax_out slots out of range (need amax_goff + ceil(oc/16) <= amax_stride, coff %% 16 == 0)");
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail("packed input must be 16-byte aligned");
  CUtensorMap act_map;
  if (nhwc_map)
    act_map = *nhwc_map;
  else if (ql)
    std::memset(&act_map, 0, sizeof(act_map));  // unused: the sources' maps travel in the params
  else if (!encode_act_map(p, x, &act_map))
    return 0;
  const int out_vec = (out_ldc % 8 == 0 && out_coff % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) ? 1 : 0;
  const int res_vec = (res && res_ldc % 8 == 0 && res_coff % 8 == 0 && reinterpret_cast<uintptr_t>(res) % 16 == 0) ? 1 : 0;
  if (p->halo) {
    ConvHaloParams h{};
    h.n_img = static_cast<int>(p->desc.batch);
    h.slabs = p->slabs;
    h.slab_pairs = p->slab_pairs;
    h.oc = static_cast<int>(oc);
    h.oh = static_cast<int>(p->desc.out_h);
    h.ow = static_cast<int>(p->desc.out_w);
    h.ksize = p->k;
    h.stride = p->stride;
    h.tw = p->tw;
    h.th = p->th;
    h.pitch = p->pitch;
    h.halo_rows = p->halo_rows;
    h.boxes_per_slab = p->boxes_per_slab;
    h.tiles_w = p->tiles_w;
    h.tiles_h = p->tiles_h;
    h.n_tiles = p->n_tiles;
    h.m_tiles = p->m_tiles;
    h.total_tiles = p->total_tiles;
    h.taps = p->taps;
    h.stages = p->stages;
    h.w_packed = static_cast<const uint8_t*>(p->d_w);
    // auto: contiguous runs when the epilogue maxes |y| for the next layer (their register
    // folding saves the amax atomics) or when there are several weight tiles (a run stays on
    // one, where the strided walk reloads weights at every n-tile), strided otherwise
    // (neighbouring tiles run together)
    h.contiguous = (p->order == 2 || (p->order == 0 && (amax_out != nullptr || p->n_tiles > 1))) ? 1 : 0;
    // two MMA issuers when each half of the stage ring holds a whole tile's stages, and for every
    // per-tensor plan with >= 4 stages (each issuer then walks its half ring through its own tiles'
    // stages).  Measured with the default tiles: YOLOv8n-320 2.564 against 2.600 ms per step at
    // batch 256, 1.074 against 1.083 at 64, 0.500 against 0.501 at 1; YOLOv11s-320 batch 64 2.167
    // against 2.194 (one issuer where a half ring held less than a tile).  pg16 keeps the first rule
    h.issuers = (2 * p->slab_pairs <= p->stages || ((!p->pg || p->two_issuers) && p->stages >= 4)) ? 2 : 1;
    h.w_tile_bytes = p->w_tile_bytes;
    h.oc_alloc = p->oc_alloc;
    h.scale_rec = scale_rec;
    // SiLU epilogues take half the scale and bias (they form h = y/2, see conv_halo.cuh)
    h.w_scale = p->d_half_sb ? p->d_half_sb : p->d_scale;
    h.bias = p->d_half_sb ? p->d_half_sb + p->oc_alloc : p->d_bias;
    h.res = static_cast<const __half*>(res);
    h.res_ldc = static_cast<int>(res_ldc);
    h.res_coff = static_cast<int>(res_coff);
    h.out = static_cast<__half*>(out);
    h.out_ldc = static_cast<int>(out_ldc);
    h.out_coff = static_cast<int>(out_coff);
    h.out_vec = out_vec;
    h.res_vec = res_vec;
    h.acc_small = p->acc_small ? 1 : 0;
    if (p->out_nbuf > 0 && out_vec) {
      // staged output: the output slice as (channel, x, y, image), one box per epilogue group's
      // column block of a (super-)tile, swizzled by its row width (conv_halo.cuh halo_stage_off)
      const int cols = halo_out_cols(p->bn, p->pg);
      const uint64_t ldc = out_ldc, ow = p->desc.out_w, oh = p->desc.out_h;
      const uint64_t dims[4] = {oc, ow, oh, p->desc.batch};
      const uint64_t strides[3] = {2 * ldc, 2 * ldc * ow, 2 * ldc * ow * oh};
      const uint32_t box[4] = {static_cast<uint32_t>(cols), static_cast<uint32_t>(p->tw),
                               static_cast<uint32_t>(p->th * p->mblocks), 1};
      const CUtensorMapSwizzle sw = cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                               : (cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
      if (!encode_map(&h.out_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, static_cast<const __half*>(out) + out_coff, dims,
                      strides, box, sw))
        return 0;
      h.out_nbuf = p->out_nbuf;
      h.out_gbytes = p->out_gbytes;
    }
    h.amax_out = amax_out;
    h.amax_stride = static_cast<int>(amax_stride);
    h.amax_goff = static_cast<int>(amax_goff);
    h.acc_dump = acc_dump;
    h.status = p->d_status;
    h.silu = p->kind == AEXRT_B200_KIND_CONV_SILU;
    h.nhwc = nhwc_map ? 1 : 0;
    h.mblocks = p->mblocks;
    h.nacc = p->nacc;
    h.tmem_cols = p->tmem_cols;
    h.tap_pairs = p->tap_pairs;
    for (int m = 0; m < 5; ++m) {
      h.tap_a[m] = p->tap_a[m];
      h.tap_b[m] = p->tap_b[m];
    }
    if (ql) {
      h.ql_parts = ql->parts;
      h.ql_raw_slots = p->ql_raw;
      h.ql_raw_bytes = p->ql_raw_bytes;
      h.ql_mode = ql->mode;
      for (int k = 0; k < kQlMaxParts; ++k) {
        h.ql_slab0[k] = ql->slab0[k];
        h.ql_up[k] = ql->up[k];
        h.ql_box_w[k] = ql->box_w[k];
        h.ql_box_h[k] = ql->box_h[k];
        h.ql_groups[k] = ql->groups[k];
        h.ql_amax[k] = ql->amax[k];
        h.ql_amax_stride[k] = ql->amax_stride[k];
        h.ql_amax_goff[k] = ql->amax_goff[k];
        if (k < ql->parts) h.ql_map[k] = ql->map[k];
      }
    }
    const HaloKernel k = halo_kernel_for(p->f16, p->bn, h.silu != 0, res != nullptr, p->pg, p->mblocks > 1, ql != nullptr);
    if (!k.fn) return fail("no conv kernel instance for this combination (linear fp16 residual, or quantize on load)");
    // with programmatic dependent launch, CTAs of this conv may be placed while the previous conv still
    // runs: more than half of an SM's shared memory keeps two conv CTAs (each owning the SM's TMEM)
    // off one SM, so that the persistent grid still spreads one CTA per SM
    const int smem = (aexrt::launch_flags() & aexrt::kLaunchProgrammatic) ? std::max(p->smem, kMaxConvSmem / 2 + 1024)
                                                                          : p->smem;
    launch_kernel(k.fn, dim3(p->grid), dim3(k.threads), smem, static_cast<cudaStream_t>(stream), act_map, h);
    return cuda_ok(cudaGetLastError(), "conv launch") ? 1 : 0;
  }
  ConvTcParams prm{};
  prm.n_img = static_cast<int>(p->desc.batch);
  prm.slabs = p->slabs;
  prm.oc = static_cast<int>(oc);
  prm.oh = static_cast<int>(p->desc.out_h);
  prm.ow = static_cast<int>(p->desc.out_w);
  prm.ksize = p->k;
  prm.stride = p->stride;
  prm.pad = p->pad;
  prm.tw = p->tw;
  prm.th = p->th;
  prm.tiles_w = p->tiles_w;
  prm.tiles_h = p->tiles_h;
  prm.n_tiles = p->n_tiles;
  prm.total_tiles = p->total_tiles;
  prm.w_packed = static_cast<const uint8_t*>(p->d_w);
  prm.q_total = p->q_total;
  prm.sps = p->sps;
  prm.stages = p->stages;
  prm.kk_p = p->kk_p;
  prm.silu = p->kind == AEXRT_B200_KIND_CONV_SILU;
  prm.scale_rec = scale_rec;
  prm.w_scale = p->d_scale;
  prm.bias = p->d_bias;
  prm.res = static_cast<const __half*>(res);
  prm.res_ldc = static_cast<int>(res_ldc);
  prm.res_coff = static_cast<int>(res_coff);
  prm.out = static_cast<__half*>(out);
  prm.out_ldc = static_cast<int>(out_ldc);
  prm.out_coff = static_cast<int>(out_coff);
  prm.out_vec = (out_ldc % 8 == 0 && out_coff % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) ? 1 : 0;
  prm.res_vec = (res && res_ldc % 8 == 0 && res_coff % 8 == 0 && reinterpret_cast<uintptr_t>(res) % 16 == 0) ? 1 : 0;
  prm.amax_out = amax_out;
  prm.amax_stride = static_cast<int>(amax_stride);
  prm.amax_goff = static_cast<int>(amax_goff);
  prm.acc_dump = acc_dump;
  prm.status = p->d_status;
  KernelFn fn = kernel_for(p->f16, p->pg, p->bn);
  launch_kernel(fn, dim3(p->grid), dim3(kConvThreads), p->smem, static_cast<cudaStream_t>(stream), act_map, prm);
  return cuda_ok(cudaGetLastError(), "conv launch") ? 1 : 0;
}

// NHWC sources whose slices all allow 16-byte loads (and, for int8, whose
// slabs do not straddle two sources): the coalesced row kernel applies.
bool rows_ok(const QuantParams& q, bool i8) {
  for (int i = 0; i < q.nsrc; ++i) {
    const QuantSrc& s = q.src[i];
    if (s.layout != 0 || s.ch % 8 || s.ldc % 8 || s.coff % 8 || reinterpret_cast<uintptr_t>(s.ptr) % 16) return false;
    if (i8 && i + 1 < q.nsrc && s.ch % 16) return false;
  }
  return q.slabs <= kMaxSlabs;
}

// One source at full resolution with no padding rows or columns: the source pixel is the linear
// pixel index (the destination too, unless a stride-2 consumer splits the columns by parity).
bool rows_linear(const QuantParams& q) {
  return q.nsrc == 1 && q.src[0].up == 1 && q.hp == q.h && q.wp == q.w && q.src[0].src_h == q.h &&
         q.src[0].src_w == q.w;
}

// Picks the quantize kernel: NHWC sources (16-byte aligned slices, enforced by
// the entry points) go through the coalesced row kernel, stride-1 NCHW fp16
// with H*W % 4 == 0 through the register-transpose kernel, anything else
// (more than 1024 channels, NCHW with ragged planes) through the per-slab
// generic kernel.
void launch_quantize(const QuantParams& q, cudaStream_t st) {
  if (rows_ok(q, true)) {
    const int pw = rows_pixels_per_warp(q, true);
    const int groups = rows_channel_groups(q, true);
    const long items = static_cast<long>((q.hp * q.wp + pw - 1) / pw) * groups;  // one warp each
    const dim3 grid(static_cast<unsigned>((items + 7) / 8), q.n);
    if (rows_linear(q))
      launch_kernel(quant_rows_kernel<true, true>, dim3(grid), dim3(256), 0, st, q, pw, groups);
    else
      launch_kernel(quant_rows_kernel<true, false>, dim3(grid), dim3(256), 0, st, q, pw, groups);
  } else if (q.nsrc == 1 && q.src[0].layout == 1 && !q.split && (q.h * q.w) % 4 == 0 && q.slabs <= kMaxSlabs) {
    const dim3 grid((q.h * q.w / 4 + 255) / 256, q.slabs, q.n);
    launch_kernel(quantize_nchw_kernel, dim3(grid), dim3(256), 0, st, q);
  } else {
    const dim3 grid((q.hp * q.wp + 255) / 256, q.slabs, q.n);
    launch_kernel(quantize_i8_kernel, dim3(grid), dim3(256), 0, st, q);
  }
}

void launch_pack(const QuantParams& q, cudaStream_t st) {
  if (q.nsrc == 1 && q.src[0].layout == 2 && q.src[0].ch <= 8 && q.src[0].up == 1) {
    // images (fp32 NCHW, <= 8 channels): one slab, four pixels per thread
    const int quads = q.hp * ((q.wp + 3) / 4);
    const dim3 grid((quads + 255) / 256, q.n);
    launch_kernel(pack_nchw_f32_kernel, dim3(grid), dim3(256), 0, st,
        static_cast<const float*>(q.src[0].ptr), q.src[0].ch, q.h, q.w, q.hp, q.wp, q.split,
        static_cast<__half*>(q.out));
    return;
  }
  if (rows_ok(q, false)) {
    const int pw = rows_pixels_per_warp(q, false);
    const int groups = rows_channel_groups(q, false);
    const long items = static_cast<long>((q.hp * q.wp + pw - 1) / pw) * groups;
    const dim3 grid(static_cast<unsigned>((items + 7) / 8), q.n);
    if (rows_linear(q))
      launch_kernel(quant_rows_kernel<false, true>, dim3(grid), dim3(256), 0, st, q, pw, groups);
    else
      launch_kernel(quant_rows_kernel<false, false>, dim3(grid), dim3(256), 0, st, q, pw, groups);
  } else {
    const dim3 grid((q.hp * q.wp + 255) / 256, q.slabs, q.n);
    launch_kernel(pack_f16_kernel, dim3(grid), dim3(256), 0, st, q);
  }
}

void quant_params_common(QuantParams& q, const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w,
                         uint32_t layout, uint32_t ldc, uint32_t coff, const uint32_t* amax_groups,
                         uint32_t groups_total, uint32_t group_offset) {
  std::memset(&q, 0, sizeof(q));
  q.nsrc = 1;
  QuantSrc& s = q.src[0];
  s.ptr = x;
  s.layout = static_cast<int>(layout);
  s.ldc = static_cast<int>(layout == AEXRT_B200_LAYOUT_NHWC_F16 ? ldc : c);
  s.coff = static_cast<int>(layout == AEXRT_B200_LAYOUT_NHWC_F16 ? coff : 0);
  s.ch = static_cast<int>(c);
  s.up = 1;
  s.src_h = static_cast<int>(h);
  s.src_w = static_cast<int>(w);
  s.amax_g = amax_groups;
  s.amax_stride = static_cast<int>(groups_total);
  s.amax_goff = static_cast<int>(group_offset);
  q.n = static_cast<int>(n);
  q.h = static_cast<int>(h);
  q.w = static_cast<int>(w);
  q.c_total = static_cast<int>(c);
}

}  // namespace

extern "C" {

uint32_t aexrt_b200_abi_version(void) { return AEXRT_B200_ABI_VERSION; }

int aexrt_b200_set_launch_flags(uint32_t flags) {
  if (flags & ~static_cast<uint32_t>(AEXRT_B200_LAUNCH_PROGRAMMATIC)) return fail("unknown launch flags 0x%x", flags);
  aexrt::g_launch_flags = flags;
  return 1;
}

uint32_t aexrt_b200_get_launch_flags(void) { return aexrt::g_launch_flags; }

const char* aexrt_b200_get_last_error(void) { return g_last_error.c_str(); }

int aexrt_b200_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int aexrt_b200_quantize_conv_weight_int8(const float* weight, uint32_t out_channels, uint32_t in_channels,
                                         uint32_t kernel_elems, uint32_t fp16_engine, int8_t* codes_out,
                                         float* scale_out) {
  if (!weight || !codes_out || !scale_out) return fail("null pointer");
  const size_t row = static_cast<size_t>(in_channels) * kernel_elems;
  std::vector<float> src(row);
  for (uint32_t o = 0; o < out_channels; ++o) {
    float amax = 0.0f;
    for (size_t i = 0; i < row; ++i) {
      float v = weight[o * row + i];
      if (fp16_engine) v = __half2float(__float2half_rn(v));
      src[i] = v;
      amax = std::max(amax, std::fabs(v));
    }
    // engine.py:2450-2457 — every operation rounds to fp32
    volatile float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    volatile float inv = 1.0f / scale;
    for (size_t i = 0; i < row; ++i) {
      volatile float prod = src[i] * inv;
      volatile float mag = std::fabs(prod) + 0.5f;
      float q = std::floor(mag);
      if (prod < 0.0f) q = -q;
      if (prod == 0.0f) q = 0.0f;
      q = std::min(127.0f, std::max(-127.0f, q));
      codes_out[o * row + i] = static_cast<int8_t>(q);
    }
    scale_out[o] = scale;
  }
  return 1;
}

int aexrt_b200_act_amax_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout,
                            uint32_t ldc, uint32_t coff, uint32_t* amax_groups, uint32_t groups_total,
                            uint32_t group_offset, uint32_t zero_first, void* stream) {
  if (!x || !amax_groups) return fail("null pointer");
  const uint32_t groups = (c + 15) / 16;
  if (group_offset + groups > groups_total) return fail("amax group range exceeds groups_total");
  if (n > kMaxImagesPerLaunch) return fail("at most %u images per call (grid dimension limit)", kMaxImagesPerLaunch);
  if (n == 0 || c == 0 || h == 0 || w == 0) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int hw = static_cast<int>(h * w);
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail("x must be 16-byte aligned");
  // NCHW with enough (image, group) strips to fill the GPU: one block per strip stores its
  // maximum, so zero_first needs no clearing pass
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool one_block = layout == AEXRT_B200_LAYOUT_NCHW_F16 && zero_first &&
                         static_cast<long>(n) * groups >= static_cast<long>(sms);
  if (zero_first && !one_block) {
    if (!cuda_ok(cudaMemset2DAsync(amax_groups + group_offset, groups_total * 4, 0, groups * 4, n, st), "memset amax"))
      return 0;
  }
  if (layout == AEXRT_B200_LAYOUT_NCHW_F16) {
    const int chunk = one_block ? 16 * hw : 32768;  // halves per block (chunked: 64 KB)
    const int blocks = static_cast<int>((16ull * hw + chunk - 1) / chunk);
    launch_kernel(amax_nchw_f16_kernel, dim3(blocks, groups, n), dim3(one_block ? 512 : 256), 0, st,
        static_cast<const __half*>(x), static_cast<int>(c), hw, static_cast<int>(groups_total), chunk,
        amax_groups + group_offset, one_block ? 1 : 0);
  } else if (layout == AEXRT_B200_LAYOUT_NHWC_F16) {
    if (ldc < coff + c || ldc % 8 || coff % 8 || reinterpret_cast<uintptr_t>(x) % 16)
      return fail("NHWC slice must be 16-byte aligned (ldc, coff multiples of 8)");
    const int vec = static_cast<int>((c + 7) / 8);
    const int ppb = std::max(1, 2048 / vec);
    const int blocks = (hw + ppb - 1) / ppb;
    launch_kernel(amax_nhwc_f16_kernel, dim3(blocks, n), dim3(256), groups * 4, st,
        static_cast<const __half*>(x), hw, static_cast<int>(c), static_cast<int>(ldc), static_cast<int>(coff),
        static_cast<int>(groups), ppb, amax_groups + group_offset, static_cast<int>(groups_total));
  } else {
    return fail("amax supports fp16 NCHW or NHWC input");
  }
  return cuda_ok(cudaGetLastError(), "amax launch") ? 1 : 0;
}

uint64_t aexrt_b200_packed_act_bytes(uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t stride) {
  const uint64_t hp = h + (stride == 2 ? (h & 1) : 0), wp = w + (stride == 2 ? (w & 1) : 0);
  return static_cast<uint64_t>(n) * ((c + 15) / 16) * hp * wp * 16;
}

uint64_t aexrt_b200_packed_f16_bytes(uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t stride) {
  const uint64_t hp = h + (stride == 2 ? (h & 1) : 0), wp = w + (stride == 2 ? (w & 1) : 0);
  return static_cast<uint64_t>(n) * ((c + 7) / 8) * hp * wp * 16;
}

int aexrt_b200_act_quantize_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout,
                                uint32_t ldc, uint32_t coff, const uint32_t* amax_groups, uint32_t groups_total,
                                uint32_t group_offset, uint32_t mode, uint32_t consumer_stride, void* q_out,
                                float* scale_rec, void* stream) {
  if (!x || !amax_groups || !q_out) return fail("null pointer");
  if (layout > AEXRT_B200_LAYOUT_NCHW_F16) return fail("quantize supports fp16 NHWC or NCHW input");
  if (mode > 1) return fail("mode must be 0 (per tensor) or 1 (pg16)");
  if (mode == 1 && c % 16) return fail("pg16 needs c %% 16 == 0");
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail("x must be 16-byte aligned");
  if (layout == AEXRT_B200_LAYOUT_NHWC_F16 && (ldc < coff + c || ldc % 8 || coff % 8))
    return fail("NHWC slice must be 16-byte aligned (ldc, coff multiples of 8)");
  if (group_offset + (c + 15) / 16 > groups_total) return fail("amax group range exceeds groups_total");
  if (reinterpret_cast<uintptr_t>(q_out) % 16) return fail("q_out must be 16-byte aligned");
  if (n > kMaxImagesPerLaunch) return fail("at most %u images per call (grid dimension limit)", kMaxImagesPerLaunch);
  if (n == 0 || c == 0 || h == 0 || w == 0) return 1;
  QuantParams q;
  quant_params_common(q, x, n, c, h, w, layout, ldc, coff, amax_groups, groups_total, group_offset);
  q.slabs = static_cast<int>((c + 15) / 16);
  q.hp = static_cast<int>(h + (consumer_stride == 2 ? (h & 1) : 0));
  q.wp = static_cast<int>(w + (consumer_stride == 2 ? (w & 1) : 0));
  q.mode = static_cast<int>(mode);
  q.split = consumer_stride == 2 ? 1 : 0;
  q.out = q_out;
  q.rec = scale_rec;
  launch_quantize(q, static_cast<cudaStream_t>(stream));
  return cuda_ok(cudaGetLastError(), "quantize launch") ? 1 : 0;
}

}  // extern "C"

namespace {

// Status word of the activation kernels that wait on their own copies (one per device, resolved
// once per device like the allocation-free scratch below).
static __device__ uint32_t g_act_status;
std::mutex g_act_mutex;
uint32_t* g_act_status_ptr[128] = {};
size_t g_cluster_smem_raised[128] = {};
int g_cluster_fits[128][kClusterQuantMaxCtas + 1] = {};  // per cluster size: 0 unknown, 1 schedulable, -1 not

uint32_t* act_status_word(int dev) {
  std::lock_guard<std::mutex> lock(g_act_mutex);
  if (!g_act_status_ptr[dev]) {
    void* ptr = nullptr;
    if (!cuda_ok(cudaGetSymbolAddress(&ptr, g_act_status), "cudaGetSymbolAddress")) return nullptr;
    g_act_status_ptr[dev] = static_cast<uint32_t*>(ptr);
  }
  return g_act_status_ptr[dev];
}

// Pixel slices per 16-channel strip for the single-pass cluster kernel, or 0 when it does not apply:
// stride-1 consumers of NCHW fp16 tensors with whole 16-channel groups, strips x slices within one
// cluster, slices of whole 16-byte plane segments that fit one CTA's shared memory.
int cluster_quant_slices(uint32_t c, uint32_t hw, const void* x, const void* q) {
  if (c % 16 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(q) % 16) return 0;
  const uint32_t groups = c / 16;
  for (uint32_t s = 1; s <= 4 && groups * s <= static_cast<uint32_t>(kClusterQuantMaxCtas); s *= 2) {
    if (hw % (8 * s)) break;
    if (32ull * (hw / s) <= static_cast<uint64_t>(kClusterQuantMaxSliceBytes)) return static_cast<int>(s);
  }
  return 0;
}

cudaLaunchConfig_t cluster_quant_config(unsigned ctas, unsigned n, size_t smem, cudaStream_t st,
                                        cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(ctas, n, 1);
  cfg.blockDim = dim3(kClusterQuantThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = ctas;
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Prepares the kernel on the current device (smem attribute, cluster occupancy at the largest
// slice), once per device and cluster size: returns 1 ready, 0 not schedulable (use the two-kernel
// path), -1 error.
int cluster_quant_prepare(int dev, int ctas) {
  std::lock_guard<std::mutex> lock(g_act_mutex);
  if (!g_cluster_smem_raised[dev]) {
    if (!cuda_ok(cudaFuncSetAttribute(amax_quant_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kClusterQuantMaxSliceBytes),
                 "cluster quantize smem attribute"))
      return -1;
    g_cluster_smem_raised[dev] = kClusterQuantMaxSliceBytes;
  }
  int& fits = g_cluster_fits[dev][ctas];
  if (fits == 0) {
    cudaLaunchAttribute attr{};
    const cudaLaunchConfig_t cfg = cluster_quant_config(static_cast<unsigned>(ctas), 1, kClusterQuantMaxSliceBytes,
                                                        nullptr, &attr);
    int clusters = 0;
    if (!cuda_ok(cudaOccupancyMaxActiveClusters(&clusters, amax_quant_cluster_kernel, &cfg), "cluster occupancy"))
      return -1;
    fits = clusters > 0 ? 1 : -1;
  }
  return fits > 0 ? 1 : 0;
}

// aexrt_b200_act_amax_quantize_f16 with the cluster kernel's first copy wait limited to
// wait_limit cycles (the second, which keeps a CTA from exiting under its own copies, always
// has the full limit).
int amax_quantize_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t mode,
                      uint32_t* amax_groups, uint32_t groups_total, uint32_t group_offset, void* q_out,
                      float* scale_rec, void* stream, long long wait_limit) {
  if (!x || !amax_groups || !q_out || !scale_rec) return fail("null pointer");
  if (n > kMaxImagesPerLaunch) return fail("at most %u images per call (grid dimension limit)", kMaxImagesPerLaunch);
  if (mode > 1) return fail("mode must be 0 (per tensor) or 1 (pg16)");
  if (mode == 1 && c % 16) return fail("pg16 needs c %% 16 == 0");
  const uint32_t groups = (c + 15) / 16;
  if (group_offset + groups > groups_total) return fail("amax group range exceeds groups_total");
  if (n == 0 || c == 0 || h == 0 || w == 0) return 1;
  const uint32_t hw = h * w;
  int dev = 0;
  if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return 0;
  if (dev < 0 || dev >= 128) return fail("device index %d out of range", dev);
  const int slices = cluster_quant_slices(c, hw, x, q_out);
  if (slices) {
    const int ctas = static_cast<int>(groups) * slices;
    const int ready = cluster_quant_prepare(dev, ctas);
    if (ready < 0) return 0;
    uint32_t* status = act_status_word(dev);
    if (!status) return 0;
    if (ready > 0) {
      cudaLaunchAttribute attr{};
      const cudaLaunchConfig_t cfg = cluster_quant_config(static_cast<unsigned>(ctas), n, 32ull * (hw / slices),
                                                          static_cast<cudaStream_t>(stream), &attr);
      return cuda_ok(cudaLaunchKernelEx(&cfg, amax_quant_cluster_kernel, static_cast<const __half*>(x),
                                        static_cast<int>(c), static_cast<int>(hw), slices, static_cast<int>(mode),
                                        static_cast<uint8_t*>(q_out), scale_rec, amax_groups,
                                        static_cast<int>(groups_total), static_cast<int>(group_offset), status,
                                        wait_limit),
                     "cluster quantize launch")
                 ? 1
                 : 0;
    }
  }
  // two passes: amax into the caller's slots, then quantize
  if (!aexrt_b200_act_amax_f16(x, n, c, h, w, AEXRT_B200_LAYOUT_NCHW_F16, c, 0, amax_groups, groups_total,
                               group_offset, 1, stream))
    return 0;
  return aexrt_b200_act_quantize_f16(x, n, c, h, w, AEXRT_B200_LAYOUT_NCHW_F16, c, 0, amax_groups, groups_total,
                                     group_offset, mode, 1, q_out, scale_rec, stream);
}

// Whether a cluster of csize post-process CTAs with smem bytes each can be scheduled on the current
// device (asked once per device, cluster size and the largest size seen; the kernel's shared-memory
// attribute is raised before).
bool nms_cluster_fits(int csize, size_t smem) {
  static std::mutex mu;
  static size_t ok_upto[128][9] = {};  // per device and cluster size: largest smem known schedulable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128 || csize > 8) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (smem <= ok_upto[dev][csize]) return true;
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = launch_config(dim3(csize), dim3(aexrt::kNmsThreads), smem, nullptr,
                                               static_cast<unsigned>(csize), attr);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, aexrt::yolo_nms_kernel, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();  // a refused query leaves no sticky error: the launch takes one CTA per image
    return false;
  }
  ok_upto[dev][csize] = smem;
  return true;
}

}  // namespace

extern "C" {

int aexrt_b200_act_amax_quantize_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t mode,
                                     uint32_t* amax_groups, uint32_t groups_total, uint32_t group_offset,
                                     void* q_out, float* scale_rec, void* stream) {
  return amax_quantize_f16(x, n, c, h, w, mode, amax_groups, groups_total, group_offset, q_out, scale_rec, stream,
                           kWaitLimitCycles);
}

int aexrt_b200_act_amax_quantize_f16_wait_limit(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w,
                                                uint32_t mode, uint32_t* amax_groups, uint32_t groups_total,
                                                uint32_t group_offset, void* q_out, float* scale_rec,
                                                uint64_t wait_limit_cycles, void* stream) {
  const long long lim = wait_limit_cycles > static_cast<uint64_t>(kWaitLimitCycles)
                            ? kWaitLimitCycles
                            : static_cast<long long>(wait_limit_cycles);
  return amax_quantize_f16(x, n, c, h, w, mode, amax_groups, groups_total, group_offset, q_out, scale_rec, stream, lim);
}

int aexrt_b200_act_status(uint32_t* status) {
  if (!status) return fail("null pointer");
  int dev = 0;
  if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return 0;
  if (dev < 0 || dev >= 128) return fail("device index %d out of range", dev);
  uint32_t* word = act_status_word(dev);
  if (!word) return 0;
  if (!cuda_ok(cudaMemcpy(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost), "read status")) return 0;
  return cuda_ok(cudaMemset(word, 0, sizeof(uint32_t)), "clear status") ? 1 : 0;
}

int aexrt_b200_pack_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout, uint32_t ldc,
                        uint32_t coff, uint32_t consumer_stride, void* out, void* stream) {
  if (!x || !out) return fail("null pointer");
  if (layout > AEXRT_B200_LAYOUT_NCHW_F32) return fail("unknown layout");
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail("x must be 16-byte aligned");
  if (layout == AEXRT_B200_LAYOUT_NHWC_F16 && (ldc < coff + c || ldc % 8 || coff % 8))
    return fail("NHWC slice must be 16-byte aligned (ldc, coff multiples of 8)");
  if (reinterpret_cast<uintptr_t>(out) % 16) return fail("out must be 16-byte aligned");
  if (n > kMaxImagesPerLaunch) return fail("at most %u images per call (grid dimension limit)", kMaxImagesPerLaunch);
  if (n == 0 || c == 0 || h == 0 || w == 0) return 1;
  QuantParams q;
  quant_params_common(q, x, n, c, h, w, layout, ldc, coff, nullptr, 0, 0);
  q.slabs = static_cast<int>((c + 7) / 8);
  q.split = consumer_stride == 2 ? 1 : 0;
  q.hp = static_cast<int>(h + (consumer_stride == 2 ? (h & 1) : 0));
  q.wp = static_cast<int>(w + (consumer_stride == 2 ? (w & 1) : 0));
  q.out = out;
  launch_pack(q, static_cast<cudaStream_t>(stream));
  return cuda_ok(cudaGetLastError(), "pack launch") ? 1 : 0;
}

AexrtB200ConvPlan* aexrt_b200_conv_plan_create(const AexrtConv2DDesc* desc, uint32_t kind, uint32_t kernel_id,
                                               uint32_t flags, const int8_t* codes, const float* w_scale,
                                               const float* bias, uint32_t block_n) {
  if (!desc) {
    fail("null desc");
    return nullptr;
  }
  const bool pg = flags & AEXRT_B200_PLAN_FLAG_INT8_PERGROUP;
  if (!check_desc_int8(*desc, kernel_id, pg)) return nullptr;
  return build_plan(*desc, kind, kernel_id, flags, false, codes, w_scale, bias, block_n);
}

AexrtB200ConvPlan* aexrt_b200_conv_plan_create_f16(const AexrtConv2DDesc* desc, uint32_t kind, const float* weight,
                                                   const float* bias, uint32_t block_n) {
  if (!desc) {
    fail("null desc");
    return nullptr;
  }
  const AexrtConv2DDesc& d = *desc;
  const bool k_ok = (d.kernel_h == 1 && d.kernel_w == 1 && d.pad_top == 0 && d.pad_left == 0) ||
                    (d.kernel_h == 3 && d.kernel_w == 3 && d.pad_top == 1 && d.pad_left == 1);
  const bool s_ok = (d.stride_h == 1 && d.stride_w == 1) || (d.stride_h == 2 && d.stride_w == 2 && d.kernel_h == 3);
  if (!k_ok || !s_ok || d.groups != 1 || d.dilation_h != 1 || d.dilation_w != 1) {
    fail("fp16 conv supports 1x1 s1 p0 and 3x3 s1/s2 p1, groups 1");
    return nullptr;
  }
  const uint32_t oh = (d.in_h + 2 * d.pad_top - d.kernel_h) / d.stride_h + 1;
  const uint32_t ow = (d.in_w + 2 * d.pad_left - d.kernel_w) / d.stride_w + 1;
  if (d.out_h != oh || d.out_w != ow || d.batch == 0) {
    fail("fp16 conv output size mismatch");
    return nullptr;
  }
  AexrtB200ConvPlan* p = build_plan(d, kind, 0, 0, true, weight, nullptr, bias, block_n);
  const uint32_t oc = d.out_channels;
  if (p && d.in_channels == static_cast<uint32_t>(kStemIC) && d.kernel_h == 3 && oc % 16 == 0 &&
      oc <= static_cast<uint32_t>(kStemMaxOC)) {
    p->image_input = true;
    for (uint32_t i = 0; i < oc * kStemIC * 9; ++i) p->stem.w[i] = __half2float(__float2half_rn(weight[i]));
    for (uint32_t i = 0; i < oc; ++i) p->stem.b[i] = bias[i];
  }
  return p;
}

int aexrt_b200_conv_f16_image(const AexrtB200ConvPlan* p, const void* images, uint32_t layout, void* out,
                              uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride,
                              uint32_t amax_goff, void* stream) {
  if (!p) return fail("null plan");
  if (layout != AEXRT_B200_LAYOUT_NCHW_F16 && layout != AEXRT_B200_LAYOUT_NCHW_F32)
    return fail("images must be NCHW fp16 or fp32");
  if (!p->image_input) return fail("plan does not take images directly (need fp16, 3 input channels, 3x3, oc %% 16 == 0 <= 64)");
  if (!images || !out) return fail("null input/output pointer");
  if (p->desc.batch > kMaxImagesPerLaunch) return fail("stem: at most %u images per launch", kMaxImagesPerLaunch);
  const uint32_t oc = p->desc.out_channels;
  if (out_ldc < out_coff + oc || out_ldc % 8 || out_coff % 8 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail("output slice must fit (coff + oc <= ldc) with ldc, coff multiples of 8 and a 16-byte aligned base");
  if (amax_out && (amax_goff * 16 + oc > amax_stride * 16 || out_coff % 16))
    return fail("amax_out slots out of range (need amax_goff + ceil(oc/16) <= amax_stride, coff %% 16 == 0)");
  const int oh = static_cast<int>(p->desc.out_h), ow = static_cast<int>(p->desc.out_w);
  auto* st = static_cast<cudaStream_t>(stream);
  const bool silu = p->kind == AEXRT_B200_KIND_CONV_SILU;
  auto* o = static_cast<__half*>(out);
  const int h = static_cast<int>(p->desc.in_h), w = static_cast<int>(p->desc.in_w), s = p->stride;
  launch_stem(static_cast<int>(oc), silu, layout == AEXRT_B200_LAYOUT_NCHW_F16, images, static_cast<int>(p->desc.batch),
              h, w, oh, ow, s, o, static_cast<int>(out_ldc), static_cast<int>(out_coff), amax_out,
              static_cast<int>(amax_stride), static_cast<int>(amax_goff), p->stem, st);
  return cuda_ok(cudaGetLastError(), "stem conv launch") ? 1 : 0;
}

int aexrt_b200_conv_plan_info(const AexrtB200ConvPlan* p, AexrtB200ConvPlanInfo* info) {
  if (!p || !info) return fail("null pointer");
  AexrtB200ConvPlanInfo i{};
  i.struct_size = sizeof(i);
  i.kernel_id = p->kernel_id;
  i.flags = p->flags;
  i.kind = p->kind;
  i.is_f16 = p->f16;
  i.tile_w = p->tw;
  i.tile_h = p->th;
  i.block_n = p->bn;
  i.k_slots = p->q_total;
  i.stages = p->stages;
  i.smem_bytes = p->smem;
  i.grid_m = p->desc.batch * p->tiles_h * p->tiles_w;
  i.grid_n = p->n_tiles;
  i.grid = p->grid;
  i.variant = p->halo ? 2u : 1u;
  i.pitch = p->pitch;
  i.image_input = p->image_input ? 1u : 0u;
  i.quant_on_load = p->ql ? 1u : 0u;
  i.staged_out = static_cast<uint32_t>(p->out_nbuf);
  i.in_hp = p->in_hp;
  i.in_wp = p->in_wp;
  *info = i;
  return 1;
}

void aexrt_b200_conv_plan_destroy(AexrtB200ConvPlan* p) {
  if (!p) return;
  if (p->d_w) cudaFree(p->d_w);
  if (p->d_scale) cudaFree(p->d_scale);
  if (p->d_bias) cudaFree(p->d_bias);
  if (p->d_half_sb) cudaFree(p->d_half_sb);
  if (p->d_status) cudaFree(p->d_status);
  delete p;
}

int aexrt_b200_conv_w8a8(const AexrtB200ConvPlan* plan, const void* q_act, const float* scale_rec,
                         const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out, uint32_t out_ldc,
                         uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride, uint32_t amax_goff,
                         int32_t* acc_dump, void* stream) {
  if (plan && plan->f16) return fail("plan is fp16; use aexrt_b200_conv_f16");
  return launch_conv(plan, q_act, scale_rec, residual, res_ldc, res_coff, out, out_ldc, out_coff, amax_out,
                     amax_stride, amax_goff, acc_dump, stream);
}

int aexrt_b200_conv_w8a8_sources(const AexrtB200ConvPlan* plan, const AexrtB200ActSource* srcs, uint32_t nsrc,
                                 const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out,
                                 uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride,
                                 uint32_t amax_goff, int32_t* acc_dump, void* stream) {
  if (!plan) return fail("null plan");
  if (plan->f16 || !plan->ql)
    return fail("conv_w8a8_sources: needs an int8 plan created with AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD "
                "(info.quant_on_load = 1)");
  if (!srcs || nsrc == 0 || nsrc > static_cast<uint32_t>(kQlMaxParts))
    return fail("conv_w8a8_sources: between 1 and %d sources", kQlMaxParts);
  const AexrtConv2DDesc& d = plan->desc;
  QlLaunch ql;
  ql.parts = static_cast<int>(nsrc);
  ql.mode = plan->pg ? 1 : 0;
  const int halo_h = plan->halo_rows / plan->pitch;
  uint32_t ch = 0;
  for (uint32_t i = 0; i < nsrc; ++i) {
    const AexrtB200ActSource& a = srcs[i];
    if (!a.ptr || !a.amax_groups) return fail("source %u: null pointer", i);
    if (a.layout != AEXRT_B200_LAYOUT_NHWC_F16) return fail("source %u: fp16 NHWC slices only", i);
    if (a.channels < 16 || (i + 1 < nsrc && a.channels % 16) || a.coff % 16 || a.ldc % 8 ||
        a.ldc < a.coff + a.channels || reinterpret_cast<uintptr_t>(a.ptr) % 16)
      return fail("source %u: >= 16 channels (a multiple of 16 but for the last), coff %% 16 == 0, ldc %% 8 == 0, "
                  "16-byte aligned", i);
    if ((a.upsample != 1 && a.upsample != 2) || (a.upsample == 2 && plan->stride != 1))
      return fail("source %u: upsample 1, or 2 for a stride-1 conv", i);
    if (a.src_h * a.upsample != d.in_h || a.src_w * a.upsample != d.in_w)
      return fail("source %u: spatial size does not match the conv input", i);
    if (a.amax_goff * 16 + a.channels > a.amax_stride * 16) return fail("source %u: amax slots out of range", i);
    ql.slab0[i] = static_cast<int>(ch / 16);
    ql.up[i] = static_cast<int>(a.upsample);
    if (plan->stride == 2) {
      ql.box_w[i] = 2 * plan->pitch;
      ql.box_h[i] = 2 * halo_h;
    } else if (a.upsample == 2) {
      ql.box_w[i] = plan->pitch / 2 + 2;
      ql.box_h[i] = halo_h / 2 + 2;
    } else {
      ql.box_w[i] = plan->pitch;
      ql.box_h[i] = halo_h;
    }
    if (32 * ql.box_w[i] * ql.box_h[i] > plan->ql_raw_bytes / 2)
      return fail("source %u: staging box larger than the plan's raw slot", i);
    ql.groups[i] = static_cast<int>((a.channels + 15) / 16);
    ql.amax[i] = a.amax_groups;
    ql.amax_stride[i] = static_cast<int>(a.amax_stride);
    ql.amax_goff[i] = static_cast<int>(a.amax_goff);
    // the slice viewed from its channel offset: (channel, x, y, image)
    const uint64_t dims[4] = {a.channels, a.src_w, a.src_h, d.batch};
    const uint64_t strides[3] = {2ull * a.ldc, 2ull * a.ldc * a.src_w, 2ull * a.ldc * a.src_w * a.src_h};
    const uint32_t box[4] = {16, static_cast<uint32_t>(ql.box_w[i]), static_cast<uint32_t>(ql.box_h[i]), 1};
    if (!encode_map(&ql.map[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, static_cast<const __half*>(a.ptr) + a.coff, dims,
                    strides, box))
      return 0;
    ch += a.channels;
  }
  if (ch != d.in_channels) return fail("sources hold %u channels, the conv %u", ch, d.in_channels);
  return launch_conv(plan, nullptr, nullptr, residual, res_ldc, res_coff, out, out_ldc, out_coff, amax_out, amax_stride,
                     amax_goff, acc_dump, stream, nullptr, &ql);
}

int aexrt_b200_conv_f16(const AexrtB200ConvPlan* plan, const void* x_slab8, const void* residual, uint32_t res_ldc,
                        uint32_t res_coff, void* out, uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out,
                        uint32_t amax_stride, uint32_t amax_goff, void* stream) {
  if (plan && !plan->f16) return fail("plan is int8; use aexrt_b200_conv_w8a8");
  return launch_conv(plan, x_slab8, nullptr, residual, res_ldc, res_coff, out, out_ldc, out_coff, amax_out,
                     amax_stride, amax_goff, nullptr, stream);
}

int aexrt_b200_conv_f16_nhwc(const AexrtB200ConvPlan* plan, const void* x, uint32_t ldc, uint32_t coff,
                             const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out, uint32_t out_ldc,
                             uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride, uint32_t amax_goff,
                             void* stream) {
  if (!plan) return fail("null plan");
  if (!plan->f16) return fail("conv_f16_nhwc: plan is int8; use aexrt_b200_conv_w8a8");
  if (!plan->halo || plan->stride != 1 || plan->image_input)
    return fail("conv_f16_nhwc: needs a stride-1 halo plan (info.variant 2); pack with aexrt_b200_pack_f16 instead");
  const uint32_t ic = plan->desc.in_channels;
  if (!x) return fail("null input pointer");
  if (ic % 8 || ldc % 8 || coff % 8 || coff + ic > ldc || reinterpret_cast<uintptr_t>(x) % 16)
    return fail("conv_f16_nhwc: input slice needs in_channels, ldc and coff multiples of 8, coff + in_channels <= "
                "ldc and a 16-byte aligned base");
  // [image][H][W][ldc] fp16 viewed from channel coff: (channel, x, y, image); a halo box is 8 channels x
  // pitch pixels x (halo rows / pitch) rows, which fills shared memory exactly as the slab8 box does
  const uint64_t w = plan->desc.in_w, h = plan->desc.in_h;
  const uint64_t dims[4] = {ic, w, h, plan->desc.batch};
  const uint64_t strides[3] = {2ull * ldc, 2ull * ldc * w, 2ull * ldc * w * h};
  const uint32_t box[4] = {8, static_cast<uint32_t>(plan->pitch), static_cast<uint32_t>(plan->halo_rows / plan->pitch),
                           1};
  CUtensorMap map;
  if (!encode_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, static_cast<const __half*>(x) + coff, dims, strides, box))
    return 0;
  return launch_conv(plan, x, nullptr, residual, res_ldc, res_coff, out, out_ldc, out_coff, amax_out, amax_stride,
                     amax_goff, nullptr, stream, &map);
}

int aexrt_b200_conv_status(const AexrtB200ConvPlan* plan, uint32_t* status) {
  if (!plan || !status) return fail("null pointer");
  if (!cuda_ok(cudaMemcpy(status, plan->d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "read status")) return 0;
  return cuda_ok(cudaMemset(plan->d_status, 0, sizeof(uint32_t)), "clear status") ? 1 : 0;
}

static bool fill_sources(QuantParams& q, const AexrtB200ActSource* srcs, uint32_t nsrc, uint32_t n, uint32_t h,
                         uint32_t w, int cps, bool need_amax) {
  if (!srcs || nsrc == 0 || nsrc > static_cast<uint32_t>(kMaxQuantSrc))
    return fail("between 1 and %d sources", kMaxQuantSrc) != 0;
  if (n > kMaxImagesPerLaunch) return fail("at most %u images per call (grid dimension limit)", kMaxImagesPerLaunch) != 0;
  std::memset(&q, 0, sizeof(q));
  q.nsrc = static_cast<int>(nsrc);
  q.n = static_cast<int>(n);
  q.h = static_cast<int>(h);
  q.w = static_cast<int>(w);
  int total = 0;
  for (uint32_t i = 0; i < nsrc; ++i) {
    const AexrtB200ActSource& a = srcs[i];
    QuantSrc& d = q.src[i];
    if (!a.ptr || (need_amax && !a.amax_groups)) return fail("source %u: null pointer", i) != 0;
    if (a.layout > AEXRT_B200_LAYOUT_NCHW_F32 || (need_amax && a.layout == AEXRT_B200_LAYOUT_NCHW_F32))
      return fail("source %u: unsupported layout", i) != 0;
    if (a.upsample != 1 && a.upsample != 2) return fail("source %u: upsample must be 1 or 2", i) != 0;
    if (a.src_h * a.upsample != h || a.src_w * a.upsample != w) return fail("source %u: spatial size mismatch", i) != 0;
    if (i + 1 < nsrc && a.channels % cps) return fail("source %u: channels must be a multiple of %d", i, cps) != 0;
    if (a.layout == AEXRT_B200_LAYOUT_NHWC_F16 &&
        (a.ldc < a.coff + a.channels || a.ldc % 8 || a.coff % 8 || reinterpret_cast<uintptr_t>(a.ptr) % 16))
      return fail("source %u: NHWC slice must be 16-byte aligned (ldc, coff multiples of 8)", i) != 0;
    if (need_amax && (a.coff % 16 || a.amax_goff * 16 + a.channels > a.amax_stride * 16))
      return fail("source %u: amax slots out of range", i) != 0;
    d.ptr = a.ptr;
    d.layout = static_cast<int>(a.layout);
    d.ldc = static_cast<int>(a.layout == AEXRT_B200_LAYOUT_NHWC_F16 ? a.ldc : a.channels);
    d.coff = static_cast<int>(a.layout == AEXRT_B200_LAYOUT_NHWC_F16 ? a.coff : 0);
    d.ch = static_cast<int>(a.channels);
    d.up = static_cast<int>(a.upsample);
    d.src_h = static_cast<int>(a.src_h);
    d.src_w = static_cast<int>(a.src_w);
    d.amax_g = a.amax_groups;
    d.amax_stride = static_cast<int>(a.amax_stride);
    d.amax_goff = static_cast<int>(a.amax_goff);
    total += static_cast<int>(a.channels);
  }
  q.c_total = total;
  return true;
}

int aexrt_b200_act_quantize_concat(const AexrtB200ActSource* srcs, uint32_t nsrc, uint32_t n, uint32_t h, uint32_t w,
                                   uint32_t mode, uint32_t consumer_stride, void* q_out, float* scale_rec,
                                   void* stream) {
  QuantParams q;
  if (!fill_sources(q, srcs, nsrc, n, h, w, 16, true)) return 0;
  if (!q_out || reinterpret_cast<uintptr_t>(q_out) % 16) return fail("q_out must be a 16-byte aligned pointer");
  if (mode > 1 || (mode == 1 && q.c_total % 16)) return fail("bad mode (pg16 needs channels %% 16 == 0)");
  if (n == 0 || h == 0 || w == 0) return 1;
  q.slabs = (q.c_total + 15) / 16;
  q.hp = static_cast<int>(h + (consumer_stride == 2 ? (h & 1) : 0));
  q.wp = static_cast<int>(w + (consumer_stride == 2 ? (w & 1) : 0));
  q.mode = static_cast<int>(mode);
  q.split = consumer_stride == 2 ? 1 : 0;
  q.out = q_out;
  q.rec = scale_rec;
  launch_quantize(q, static_cast<cudaStream_t>(stream));
  return cuda_ok(cudaGetLastError(), "quantize launch") ? 1 : 0;
}

int aexrt_b200_pack_f16_concat(const AexrtB200ActSource* srcs, uint32_t nsrc, uint32_t n, uint32_t h, uint32_t w,
                               uint32_t consumer_stride, void* out, void* stream) {
  QuantParams q;
  if (!fill_sources(q, srcs, nsrc, n, h, w, 8, false)) return 0;
  if (!out || reinterpret_cast<uintptr_t>(out) % 16) return fail("out must be a 16-byte aligned pointer");
  if (n == 0 || h == 0 || w == 0) return 1;
  q.slabs = (q.c_total + 7) / 8;
  q.hp = static_cast<int>(h + (consumer_stride == 2 ? (h & 1) : 0));
  q.wp = static_cast<int>(w + (consumer_stride == 2 ? (w & 1) : 0));
  q.split = consumer_stride == 2 ? 1 : 0;
  q.out = out;
  launch_pack(q, static_cast<cudaStream_t>(stream));
  return cuda_ok(cudaGetLastError(), "pack launch") ? 1 : 0;
}

int aexrt_b200_sppf_pool(const void* x, uint32_t n, uint32_t h, uint32_t w, uint32_t c, uint32_t ldc, uint32_t coff,
                         void* out, uint32_t out_ldc, uint32_t out_coff, uint32_t* amax, uint32_t amax_stride,
                         uint32_t amax_goff, void* stream) {
  if (!x || !out) return fail("null pointer");
  if (c % 16 || ldc % 8 || coff % 8 || out_ldc % 8 || out_coff % 16 || ldc < coff + c || out_ldc < out_coff + 3 * c ||
      reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail("sppf: c %% 16 == 0 and 16-byte aligned slices required");
  if (amax && amax_goff * 16 + 3 * c > amax_stride * 16) return fail("sppf: amax slots out of range");
  if (n > kMaxImagesPerLaunch) return fail("sppf: at most %u images per call", kMaxImagesPerLaunch);
  const long total = static_cast<long>(n) * h * w * (c / 8);
  if (total == 0) return 1;
  {
    // whole map per (image, channel block) in shared memory when it fits; blocks of at most 32
    // channels, so that small maps still give every SM several blocks (the passes are latency-bound)
    int cb = 32;
    while (cb > 16 && (c % cb || 4L * h * w * cb * 2 > 160 * 1024)) cb /= 2;
    const long smem = 4L * h * w * cb * 2;
    if (c % cb == 0 && smem <= 160 * 1024) {
      // per call: the attribute belongs to the current device's context
      if (!cuda_ok(cudaFuncSetAttribute(sppf_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024),
                   "cudaFuncSetAttribute"))
        return 0;
      launch_kernel(sppf_smem_kernel, dim3(c / cb, n), dim3(256), smem, static_cast<cudaStream_t>(stream),
          static_cast<const __half*>(x), h, w, c, ldc, coff, cb, static_cast<__half*>(out), out_ldc, out_coff, amax,
          amax_stride, amax_goff);
      return cuda_ok(cudaGetLastError(), "sppf launch") ? 1 : 0;
    }
  }
  launch_kernel(sppf_pool_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0,
      static_cast<cudaStream_t>(stream),
      static_cast<const __half*>(x), n, h, w, c, ldc, coff, static_cast<__half*>(out), out_ldc, out_coff, amax,
      amax_stride, amax_goff);
  return cuda_ok(cudaGetLastError(), "sppf launch") ? 1 : 0;
}

int aexrt_b200_dwconv3x3_f16(const void* x, uint32_t n, uint32_t h, uint32_t w, uint32_t c, uint32_t ldc,
                             uint32_t coff, uint32_t grp, uint32_t grp_stride, uint32_t grp_off, const float* w9,
                             const float* bias, uint32_t stride, uint32_t silu, void* out, uint32_t out_ldc,
                             uint32_t out_coff, void* stream) {
  if (!x || !out || !w9 || !bias) return fail("dwconv: null pointer");
  if (stride != 1 && stride != 2) return fail("dwconv: stride must be 1 or 2");
  if (grp == 0) grp = c;
  if (grp_stride == 0) grp_stride = grp;
  if (c % 8 || grp % 8 || grp_stride % 8 || grp_off % 8 || ldc % 8 || coff % 8 || out_ldc % 8 || out_coff % 8 ||
      c % grp || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
      reinterpret_cast<uintptr_t>(w9) % 16 || reinterpret_cast<uintptr_t>(bias) % 16)
    return fail("dwconv: channel counts, groups and slices must be multiples of 8 with 16-byte aligned buffers");
  if (ldc < coff + (c / grp - 1) * grp_stride + grp_off + grp || out_ldc < out_coff + c)
    return fail("dwconv: input or output slice out of range");
  const uint32_t oh = (h + 2 - 3) / stride + 1, ow = (w + 2 - 3) / stride + 1;
  const long total = static_cast<long>(n) * oh * ((ow + kDwRun - 1) / kDwRun) * (c / 8);
  if (total == 0) return 1;
  launch_kernel(stride == 1 ? dwconv3x3_kernel<1> : dwconv3x3_kernel<2>,
      dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, static_cast<cudaStream_t>(stream),
      static_cast<const __half*>(x), n, h, w, c, ldc, coff, grp, grp_stride, grp_off, w9, bias, silu ? 1 : 0,
      oh, ow, static_cast<__half*>(out), out_ldc, out_coff);
  return cuda_ok(cudaGetLastError(), "dwconv launch") ? 1 : 0;
}

int aexrt_b200_psa_attention_f16(const void* qkv, uint32_t n, uint32_t h, uint32_t w, uint32_t ldc, uint32_t coff,
                                 uint32_t heads, uint32_t key_dim, uint32_t head_dim, float scale, const void* pe,
                                 uint32_t pe_ldc, uint32_t pe_coff, void* out, uint32_t out_ldc, uint32_t out_coff,
                                 uint32_t* amax, uint32_t amax_stride, uint32_t amax_goff, void* stream) {
  if (!qkv || !pe || !out) return fail("psa attention: null pointer");
  if (head_dim != static_cast<uint32_t>(kPsaHeadDim)) return fail("psa attention: head_dim must be 64");
  if (heads == 0 || key_dim == 0 || key_dim % 8 || ldc % 8 || coff % 8 || pe_ldc % 2 || pe_coff % 2 ||
      out_ldc % 2 || out_coff % 16 || reinterpret_cast<uintptr_t>(qkv) % 16)
    return fail("psa attention: key_dim, ldc and coff multiples of 8, output slice at a 16-channel boundary");
  const uint32_t per_head = 2 * key_dim + head_dim;
  if (ldc < coff + heads * per_head || pe_ldc < pe_coff + heads * head_dim || out_ldc < out_coff + heads * head_dim)
    return fail("psa attention: qkv, pe or output slice out of range");
  if (amax && amax_goff * 16 + heads * head_dim > amax_stride * 16) return fail("psa attention: amax slots out of range");
  if (n > kMaxImagesPerLaunch) return fail("psa attention: at most %u images per call", kMaxImagesPerLaunch);
  const uint32_t l = h * w;
  const size_t smem = psa_smem_bytes(static_cast<int>(l), static_cast<int>(key_dim));
  if (smem > 200 * 1024) return fail("psa attention: a %ux%u map does not fit one CTA's shared memory", h, w);
  if (n == 0 || l == 0) return 1;
  if (!cuda_ok(cudaFuncSetAttribute(psa_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
               "cudaFuncSetAttribute"))
    return 0;
  // split each head's queries over up to 4 CTAs while the grid is below two CTAs per SM
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t pairs = heads * n;
  const uint32_t splits = std::min(4u, std::max(1u, (2u * static_cast<uint32_t>(sms) + pairs - 1) / pairs));
  launch_kernel(psa_attention_kernel, dim3(heads, n, splits), dim3(kPsaThreads), smem, static_cast<cudaStream_t>(stream),
      static_cast<const __half*>(qkv), static_cast<int>(l), ldc, coff, key_dim, scale,
      static_cast<const __half*>(pe), pe_ldc, pe_coff, static_cast<__half*>(out), out_ldc, out_coff, amax,
      amax_stride, amax_goff);
  return cuda_ok(cudaGetLastError(), "psa attention launch") ? 1 : 0;
}

int aexrt_b200_yolo_decode(const AexrtB200DecodeLevel* levels, uint32_t nlevels, uint32_t n, uint32_t nc,
                           uint32_t reg_max, float* out, void* stream) {
  if (!levels || !out || nlevels == 0 || nlevels > static_cast<uint32_t>(kMaxLevels)) return fail("bad decode levels");
  if (reg_max == 0 || reg_max > 64 || nc == 0) return fail("bad nc / reg_max");
  DecodeParams d;
  std::memset(&d, 0, sizeof(d));
  int anchors = 0;
  for (uint32_t i = 0; i < nlevels; ++i) {
    const AexrtB200DecodeLevel& l = levels[i];
    if (!l.box || !l.cls || l.box_ldc < l.box_coff + 4 * reg_max || l.cls_ldc < l.cls_coff + nc)
      return fail("decode level %u: bad slices", i);
    d.box[i] = static_cast<const __half*>(l.box);
    d.cls[i] = static_cast<const __half*>(l.cls);
    d.box_ldc[i] = l.box_ldc;
    d.box_coff[i] = l.box_coff;
    d.cls_ldc[i] = l.cls_ldc;
    d.cls_coff[i] = l.cls_coff;
    d.h[i] = l.h;
    d.w[i] = l.w;
    d.stride[i] = l.stride;
    anchors += static_cast<int>(l.h * l.w);
  }
  d.levels = static_cast<int>(nlevels);
  d.n = static_cast<int>(n);
  d.nc = static_cast<int>(nc);
  d.reg_max = static_cast<int>(reg_max);
  d.anchors = anchors;
  d.out = out;
  const long total = static_cast<long>(n) * anchors;
  if (total == 0) return 1;
  launch_kernel(yolo_decode_kernel, dim3(static_cast<unsigned>((total + 127) / 128)), dim3(128), 0,
      static_cast<cudaStream_t>(stream), d);
  return cuda_ok(cudaGetLastError(), "decode launch") ? 1 : 0;
}

int aexrt_b200_yolo_nms_topk(const float* output0, uint32_t n, uint32_t channels, uint32_t anchors, uint32_t nc,
                             uint32_t has_objectness, uint32_t layout, float conf_threshold, float iou_threshold,
                             uint32_t max_candidates, uint32_t max_detections, uint32_t mode,
                             AexrtYoloDetection* detections, uint32_t* counts, void* stream) {
  if (!output0 || !detections || !counts) return fail("yolo_nms_topk: null pointer");
  if (nc == 0 || channels != (has_objectness ? 5u : 4u) + nc)
    return fail("yolo_nms_topk: channels %u do not match nc %u (objectness %u)", channels, nc, has_objectness);
  if (layout > 2) return fail("yolo_nms_topk: bad layout %u", layout);
  const uint32_t rule = mode & 0xFFu, ctas = (mode >> AEXRT_B200_NMS_CTAS_SHIFT) & 0xFu;
  if (rule > 1 || (mode >> 12) != 0 || (ctas != 0 && ctas != 1 && ctas != 2 && ctas != 4 && ctas != 8))
    return fail("yolo_nms_topk: bad mode 0x%x (rule 0 or 1, CTAs per image 0, 1, 2, 4 or 8)", mode);
  if (max_candidates == 0 || max_candidates > aexrt::kNmsMaxCandidates)
    return fail("yolo_nms_topk: max_candidates %u outside 1..%d", max_candidates, aexrt::kNmsMaxCandidates);
  if (max_detections == 0) return fail("yolo_nms_topk: max_detections must be >= 1");
  if (static_cast<uint64_t>(channels) * anchors > (1ull << 31)) return fail("yolo_nms_topk: output0 too large");
  if (n == 0) return 1;
  aexrt::NmsParams p;
  p.y = output0;
  p.anchors = static_cast<int>(anchors);
  p.channels = static_cast<int>(channels);
  p.nc = static_cast<int>(nc);
  p.has_obj = has_objectness ? 1 : 0;
  p.channels_last = layout == 2 ? 1 : 0;
  p.conf = conf_threshold;
  p.iou = iou_threshold;
  p.max_cand = static_cast<int>(max_candidates);
  p.max_det = static_cast<int>(max_detections);
  p.mode = static_cast<int>(rule);
  p.pow2 = 1;
  while (p.pow2 < p.max_cand) p.pow2 <<= 1;
  p.dets = reinterpret_cast<float*>(detections);
  p.counts = counts;
  const size_t smem = aexrt::nms_smem_bytes(p.max_cand, p.pow2, p.mode);
  if (smem > 48 * 1024) {
    // raised once per device to the largest size seen, so a launch inside a stream capture
    // that an earlier launch prepared makes no attribute call
    static std::mutex mu;
    static size_t raised[128] = {};
    int dev = 0;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return 0;
    if (dev < 0 || dev >= 128) return fail("device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (smem > raised[dev]) {
      if (!cuda_ok(cudaFuncSetAttribute(aexrt::yolo_nms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "nms smem attribute"))
        return 0;
      raised[dev] = smem;
    }
  }
  // CTAs per image: automatic = the widest cluster (at most 8) whose grid still fits two CTAs per SM
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int csize = static_cast<int>(ctas);
  if (csize == 0) {
    csize = 8;
    while (csize > 1 && static_cast<long>(n) * csize > 2L * sms) csize /= 2;
  }
  if (static_cast<uint64_t>(n) * csize > 0x7FFFFFFFull) return fail("yolo_nms_topk: too many images");
  if (csize > 1 && !nms_cluster_fits(csize, smem)) csize = 1;
  p.csize = csize;
  launch_kernel_cluster(aexrt::yolo_nms_kernel, dim3(n * csize), dim3(aexrt::kNmsThreads), smem,
                        static_cast<cudaStream_t>(stream), static_cast<unsigned>(csize), p);
  return cuda_ok(cudaGetLastError(), "nms launch") ? 1 : 0;
}

int aexrt_b200_zero(void* ptr, uint64_t bytes, void* stream) {
  if (!ptr) return fail("null pointer");
  return cuda_ok(cudaMemsetAsync(ptr, 0, bytes, static_cast<cudaStream_t>(stream)), "memset") ? 1 : 0;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Allocation-free amax + quantize
//
// Some callers cannot call cudaMalloc: a real-time loop that forbids allocation
// after start-up (an allocation can stall on the driver), a plugin whose device
// memory is owned by its host's allocator or budget, or an embedded caller with
// no allocator of its own.  For them the per-(image, group) amax slots, which are
// scratch between the amax and the quantize kernels, live in a fixed device
// array owned by the library instead of in caller memory.
// ----------------------------------------------------------------------------

namespace {

constexpr uint32_t kNoAllocAmaxSlots = 65536;  // 256 KB: images x ceil(channels / 16) slots
static __device__ __align__(256) uint32_t g_noalloc_amax[kNoAllocAmaxSlots];

std::mutex g_noalloc_mutex;
uint32_t* g_noalloc_ptr[128] = {};  // device address of g_noalloc_amax, per device

// The host-side name g_noalloc_amax is not a device address: resolve it once per
// device, with that device current.
uint32_t* noalloc_slots() {
  int dev = 0;
  if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
  if (dev < 0 || dev >= 128) {
    fail("device index %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    if (!cuda_ok(cudaGetSymbolAddress(&ptr, g_noalloc_amax), "cudaGetSymbolAddress")) return nullptr;
    g_noalloc_ptr[dev] = static_cast<uint32_t*>(ptr);
  }
  return g_noalloc_ptr[dev];
}

}  // namespace

extern "C" int aexrt_b200_act_quantize_f16_noalloc(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w,
                                                   uint32_t layout, uint32_t ldc, uint32_t coff, uint32_t mode,
                                                   uint32_t consumer_stride, void* q_out, float* scale_rec,
                                                   void* stream) {
  // the image index is a grid dimension of the amax and quantize launches
  if (n > kMaxImagesPerLaunch)
    return fail("act_quantize_noalloc: %u images exceed the %u a call takes", n, kMaxImagesPerLaunch);
  const uint64_t slots = static_cast<uint64_t>(n) * ((c + 15) / 16);
  if (slots > kNoAllocAmaxSlots)
    return fail("act_quantize_noalloc: %llu amax slots (images x ceil(channels/16)) exceed the fixed %u",
                static_cast<unsigned long long>(slots), kNoAllocAmaxSlots);
  uint32_t* amax = noalloc_slots();
  if (!amax) return 0;
  const uint32_t groups = (c + 15) / 16;
  // zero_first clears this call's slots: the array keeps the previous call's maxima
  if (!aexrt_b200_act_amax_f16(x, n, c, h, w, layout, ldc, coff, amax, groups, 0, 1, stream)) return 0;
  return aexrt_b200_act_quantize_f16(x, n, c, h, w, layout, ldc, coff, amax, groups, 0, mode, consumer_stride, q_out,
                                     scale_rec, stream);
}
