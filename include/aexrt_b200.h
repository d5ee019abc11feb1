/*
 * aexrt_b200 — C ABI of the B200 (sm_100a) W8A8 convolution backend.
 *
 * Conventions follow the reference runtime's C ABI (native/aexrt.h):
 *   - every entry point returns int 1 on success and 0 on failure, never aborts,
 *     and records a message retrievable with aexrt_b200_get_last_error()
 *     (reference: aexrt_yolo_get_last_error, aexrt.h:406);
 *   - opaque handles are owned by the library until their destroy call;
 *   - device pointers are plain `void*`/typed pointers into the current CUDA
 *     device's memory and `stream` is a cudaStream_t (NULL = legacy default);
 *   - launches are asynchronous on `stream`; none of them allocates memory.
 *
 * Data layouts used on the device:
 *   fp16 activations: NHWC slices (channel stride `ldc`, channel offset `coff`);
 *   int8 codes:       [image][ceil(C/16)][Hp][Wp][16]   ("slab16");
 *   fp16 conv input:  [image][ceil(C/8)][Hp][Wp][8]     ("slab8");
 *                     for a stride-2 consumer Hp, Wp are rounded up to even and
 *                     each row is stored as [even columns][odd columns];
 *   amax groups:      uint32 float bits, [image][groups_total] (one per 16 channels);
 *   scale record:     float [image][1 + ceil(C/16)]: slot 0 = per-tensor amax,
 *                     slot 1+g = amax of 16-channel group g (the reference's
 *                     amax buffer layout, runtime.cpp:3241-3258, one per image).
 */
#ifndef AEXRT_B200_H
#define AEXRT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with -fvisibility=hidden; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define AEXRT_B200_ABI_VERSION 1u

/* Layout-identical to the reference's AexrtConv2DDesc (native/aexrt.h:98-115). */
typedef struct AexrtConv2DDesc {
    uint32_t batch;
    uint32_t in_channels;
    uint32_t in_h;
    uint32_t in_w;
    uint32_t out_channels;
    uint32_t out_h;
    uint32_t out_w;
    uint32_t kernel_h;
    uint32_t kernel_w;
    uint32_t stride_h;
    uint32_t stride_w;
    uint32_t pad_top;
    uint32_t pad_left;
    uint32_t dilation_h;
    uint32_t dilation_w;
    uint32_t groups;
} AexrtConv2DDesc;

/* Command kinds and plan flags, same values as the reference compiler
 * (src/aexrt/engine.py:85-96, 103-118). */
#define AEXRT_B200_KIND_CONV 1u
#define AEXRT_B200_KIND_CONV_SILU 2u
#define AEXRT_B200_PLAN_FLAG_INT8_PERGROUP (1u << 4)
/* This backend's own plan flag (above the reference's bits 0-4): an int8 plan that
 * reads fp16 NHWC sources and quantizes them on load (aexrt_b200_conv_w8a8_sources). */
#define AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD (1u << 8)

/* Activation layouts accepted by the amax / quantize entry points. */
#define AEXRT_B200_LAYOUT_NHWC_F16 0u
#define AEXRT_B200_LAYOUT_NCHW_F16 1u
#define AEXRT_B200_LAYOUT_NCHW_F32 2u

/* Activation scale modes (the INT8_PERGROUP plan flag selects pg16). */
#define AEXRT_B200_SCALE_PER_TENSOR 0u
#define AEXRT_B200_SCALE_PG16 1u

typedef struct AexrtB200ConvPlan AexrtB200ConvPlan;

/* Read-only description of a conv plan (the analogue of AexrtConvPlanInfo,
 * native/aexrt.h:435-445, for one command). */
typedef struct AexrtB200ConvPlanInfo {
    uint32_t struct_size;
    uint32_t kernel_id;        /* 51 = 1x1, 52 = 3x3 s1, 53 = 3x3 s2 (0 for fp16 plans) */
    uint32_t flags;            /* plan flags (bit 4 = INT8_PERGROUP) */
    uint32_t kind;             /* AEXRT_B200_KIND_CONV or _CONV_SILU */
    uint32_t is_f16;
    uint32_t tile_w, tile_h;   /* spatial output tile (M = tile_w*tile_h <= 128) */
    uint32_t block_n;          /* output channels per CTA */
    uint32_t k_slots;          /* 16-byte K slots incl. padding */
    uint32_t stages;           /* TMA/MMA pipeline depth */
    uint32_t smem_bytes;
    uint32_t grid_m, grid_n;
    uint32_t in_hp, in_wp;     /* packed input buffer dims expected by the launch */
    uint32_t grid;             /* persistent CTAs per launch */
    uint32_t variant;          /* 1 slot streaming, 2 halo tile */
    uint32_t pitch;            /* halo variant: M rows per tile row */
    uint32_t image_input;      /* 1: aexrt_b200_conv_f16_image accepts this plan */
    uint32_t quant_on_load;    /* 1: aexrt_b200_conv_w8a8_sources accepts this plan */
    uint32_t staged_out;       /* halo variant: output tiles staged in shared memory for a TMA store
                                  (buffers per epilogue group; 0: direct stores) */
} AexrtB200ConvPlanInfo;

/* ---------------------------------------------------------------- library */
uint32_t aexrt_b200_abi_version(void);
/* Thread-local message of the last failed call on this thread ("" if none). */
const char* aexrt_b200_get_last_error(void);
/* Launch flags of the calling thread, applied to every later launch it makes
 * through this library (the reference has no counterpart: D3D12 command lists
 * have no dependent-launch overlap).  AEXRT_B200_LAUNCH_PROGRAMMATIC: kernels
 * are launched with programmatic stream serialization, so that each one's
 * launch and set-up (barrier init, TMEM allocation, weight loads) overlap the
 * kernel before it; every kernel waits for its predecessor's grid before it
 * touches activations.  Meant for small batches, where grids use few SMs; it
 * also applies inside CUDA graph capture.  Returns 0 for unknown flags. */
#define AEXRT_B200_LAUNCH_PROGRAMMATIC 1u
int aexrt_b200_set_launch_flags(uint32_t flags);
uint32_t aexrt_b200_get_launch_flags(void);
/* Number of visible CUDA devices (0 when no driver or GPU is present). */
int aexrt_b200_device_count(void);

/* ---------------------------------------------------------------- a1: weights
 * Per-output-channel symmetric int8 quantization of a conv weight
 * [out_channels][in_channels][kernel_elems] (fp32): the layout-8 payload.
 * Replaces src/aexrt/engine.py:2418-2465 (_add_packed_conv_int8) and its C++
 * twin ensure_conv_int8_weight (native/aexrt_d3d12_runtime.cpp:21716-21742);
 * host-side, bit-identical.  fp16_engine=1 rounds the weights through fp16 first. */
int aexrt_b200_quantize_conv_weight_int8(const float* weight, uint32_t out_channels, uint32_t in_channels,
                                         uint32_t kernel_elems, uint32_t fp16_engine, int8_t* codes_out,
                                         float* scale_out);

/* ---------------------------------------------------------------- a3: amax
 * Per-image amax of |x| per 16-channel group (float bits), atomically max-ed
 * into amax_groups[image * groups_total + group_offset + g].  zero_first=1
 * clears this call's slots first.  Replaces aexrt_int8_quant_zero +
 * aexrt_int8_quant_amax (native/aexrt_d3d12_runtime.cpp:3159-3275, recorded by
 * record_int8_prequant_activation :21622-21644); per image instead of over
 * the [C][N*H*W] view, which is the reference's batch-1 behaviour. */
int aexrt_b200_act_amax_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout,
                            uint32_t ldc, uint32_t coff, uint32_t* amax_groups, uint32_t groups_total,
                            uint32_t group_offset, uint32_t zero_first, void* stream);

/* ---------------------------------------------------------------- a4: quantize
 * Bytes of the slab16 int8 buffer a conv with the given stride reads
 * (stride 2 pads H and W up to even). */
uint64_t aexrt_b200_packed_act_bytes(uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t stride);

/* int8 codes q = round_half_even(x * 127/amax) (no clamp, 0 when amax <= 0)
 * into the slab16 layout, plus the per-image scale record the conv reads.
 * mode = AEXRT_B200_SCALE_PER_TENSOR uses max over all groups, PG16 each
 * group's own amax.  Replaces aexrt_int8_quant_pack[_pg]
 * (native/aexrt_d3d12_runtime.cpp:3277-3361, recorder :21646-21659). */
int aexrt_b200_act_quantize_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout,
                                uint32_t ldc, uint32_t coff, const uint32_t* amax_groups, uint32_t groups_total,
                                uint32_t group_offset, uint32_t mode, uint32_t consumer_stride, void* q_out,
                                float* scale_rec, void* stream);

/* ---------------------------------------------------------------- a2/a9: plans
 * Builds a device-resident W8A8 conv plan from layout-8 weights (codes in
 * [oc][ic][kh][kw] order + per-oc fp32 scale) and fp32 bias.  kernel_id is the
 * reference's planned kernel (51 1x1, 52 3x3 s1, 53 3x3 s2) and must pass the
 * reference's guard can_use_conv_int8 (native/aexrt_d3d12_runtime.cpp:9398-9422)
 * plus IC % 16 == 0 when flags has INT8_PERGROUP; the weight repack replaces
 * ensure_conv_int8_weight's uint32 repack (runtime.cpp:21744-21775).
 * block_n = 0 picks the output-channel tile automatically.  Tuning bits above
 * the tile (bits 0-15): bits 16-19 kernel variant (0 auto, 1 slot streaming,
 * 2 halo tile), bits 20-23 halo tile order (0 auto, 1 strided over CTAs,
 * 2 one contiguous run per CTA), bits 24-27 the most M blocks stacked in one
 * halo super-tile (0 auto, 1 none), bit 29 halo epilogue stages each tile in
 * shared memory and writes it with one TMA tensor store per column block,
 * bit 28 it stores each output pixel directly (the default), bit 30 asks for
 * two MMA issuers even when half the stage ring holds less than one tile's
 * stages (per-tensor halo plans with at least 4 stages have two anyway; the
 * bit changes nothing there).  Small grids (one
 * or a few images) pick narrower automatic tiles so that the conv spreads over
 * more SMs.  For int8 plans the results are identical
 * for every choice (integer accumulation); an fp16 plan whose choice moves it
 * between the halo and slot kernels sums K in another order, which can change
 * the last bit of an fp16 output.
 * Allocates device memory (set-up time only).  Returns NULL on error. */
AexrtB200ConvPlan* aexrt_b200_conv_plan_create(const AexrtConv2DDesc* desc, uint32_t kind, uint32_t kernel_id,
                                               uint32_t flags, const int8_t* codes, const float* w_scale,
                                               const float* bias, uint32_t block_n);

/* fp16 conv plan (stem / detect head of the model): fp32 weights are rounded
 * to fp16, accumulation is fp32.  Any k in {1,3}, stride in {1,2}, pad k/2. */
AexrtB200ConvPlan* aexrt_b200_conv_plan_create_f16(const AexrtConv2DDesc* desc, uint32_t kind, const float* weight,
                                                   const float* bias, uint32_t block_n);

int aexrt_b200_conv_plan_info(const AexrtB200ConvPlan* plan, AexrtB200ConvPlanInfo* info);
void aexrt_b200_conv_plan_destroy(AexrtB200ConvPlan* plan);

/* ---------------------------------------------------------------- a6/a7/a10: conv
 * One W8A8 conv launch (per-tensor or pg16 per the plan flags):
 *   y = (sum_k q_a*q_w) * amax/127 * w_scale[oc] + bias[oc]      (per tensor)
 *   y = (sum_g fl32(S_g) * amax_g/127) * w_scale[oc] + bias[oc]  (pg16)
 * then SiLU (CONV_SILU), then + residual (C2f tail, optional), stored as fp16
 * into out[pixel*out_ldc + out_coff + oc].  When amax_out is non-NULL the
 * epilogue also max-es |y| per (image, 16-channel group) into
 * amax_out[image*amax_stride + amax_goff + oc/16] for the next layer.
 * acc_dump (optional, debugging) receives the int32 accumulators:
 * [pixel][oc] per tensor, [group][pixel][oc] for pg16.
 * Replaces the prequant conv kernels 51/52/53 (runtime.cpp:4614-4923), the LTS
 * variants (:3371-3812) and the unfused CONCAT / BINARY Add neighbours. */
int aexrt_b200_conv_w8a8(const AexrtB200ConvPlan* plan, const void* q_act, const float* scale_rec,
                         const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out, uint32_t out_ldc,
                         uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride, uint32_t amax_goff,
                         int32_t* acc_dump, void* stream);

/* fp16 conv launch on slab8 input (see aexrt_b200_pack_f16). */
int aexrt_b200_conv_f16(const AexrtB200ConvPlan* plan, const void* x_slab8, const void* residual, uint32_t res_ldc,
                        uint32_t res_coff, void* out, uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out,
                        uint32_t amax_stride, uint32_t amax_goff, void* stream);

/* fp16 conv launch reading the NHWC fp16 activation x ([batch][in_h][in_w][ldc],
 * channels coff .. coff + in_channels) directly, with no slab8 copy: for
 * stride-1 plans of the halo variant (info.variant == 2).  in_channels, ldc
 * and coff multiples of 8, x 16-byte aligned.  Same result as
 * aexrt_b200_pack_f16 + aexrt_b200_conv_f16, bit for bit.  Replaces the
 * reference's fp16 CONV / CONV_SILU commands of the detect head
 * (record_replay_conv fp16 branch, native/aexrt_d3d12_runtime.cpp:23280). */
int aexrt_b200_conv_f16_nhwc(const AexrtB200ConvPlan* plan, const void* x, uint32_t ldc, uint32_t coff,
                             const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out, uint32_t out_ldc,
                             uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride, uint32_t amax_goff,
                             void* stream);

/* Reads and clears the plan's device status word (synchronises the device).
 * Non-zero bits mean a pipeline wait gave up (see the kernel sources). */
/* The image stem: an fp16 plan with 3 input channels, a 3x3 window (pad 1)
 * and 16/32/48/64 output channels (info.image_input == 1) read straight from
 * the NCHW image batch [batch][3][in_h][in_w], fp16 (layout
 * AEXRT_B200_LAYOUT_NCHW_F16) or fp32 (AEXRT_B200_LAYOUT_NCHW_F32), with no
 * packed copy.
 * Same arithmetic as aexrt_b200_conv_f16 (fp16-rounded inputs and weights,
 * fp32 accumulation, fp32 bias + SiLU, fp16 output); out_ldc and out_coff
 * multiples of 8 (16 with amax_out), out 16-byte aligned.  Replaces the
 * reference's first fp16 conv command with its input conversion
 * (the image upload + NCHW fp16 conv of the stem in prepared replay,
 * native/aexrt_d3d12_runtime.cpp:28758-29010). */
int aexrt_b200_conv_f16_image(const AexrtB200ConvPlan* plan, const void* images, uint32_t layout, void* out,
                              uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride,
                              uint32_t amax_goff, void* stream);

int aexrt_b200_conv_status(const AexrtB200ConvPlan* plan, uint32_t* status);

/* fp16 slab8 repack of an NHWC fp16 or NCHW fp16/fp32 tensor for fp16 convs. */
uint64_t aexrt_b200_packed_f16_bytes(uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t stride);
int aexrt_b200_pack_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout, uint32_t ldc,
                        uint32_t coff, uint32_t consumer_stride, void* out, void* stream);

/* ---------------------------------------------------------------- a10: fused neighbours
 * One input part of a conv whose input is a channel concatenation (CONCAT,
 * engine.py:103-118), optionally read through a nearest 2x upsample (RESIZE)
 * and/or as a channel slice of a wider NHWC buffer (SLICE / C2f split).  The
 * quantizer reads the parts in place, so the concatenated fp16 tensor is never
 * materialised: the reference instead runs CONCAT, then quantizes the
 * concatenated value (its compiler un-fuses concat + conv for the int8 path,
 * src/aexrt/yolo.py:473-487; quantizer recorder runtime.cpp:21466-21665). */
typedef struct AexrtB200ActSource {
    const void* ptr;
    uint32_t layout;              /* AEXRT_B200_LAYOUT_* */
    uint32_t ldc, coff;           /* NHWC slice: channel stride and offset */
    uint32_t channels;            /* multiple of 16 except for the last part (int8) / 8 (fp16) */
    uint32_t upsample;            /* 1, or 2 for nearest-neighbour 2x */
    uint32_t src_h, src_w;        /* spatial dims of this part (consumer dims / upsample) */
    const uint32_t* amax_groups;  /* per (image, group) amax bits of this part's buffer (int8 only) */
    uint32_t amax_stride, amax_goff;
} AexrtB200ActSource;

/* Quantize a concatenation of parts into one slab16 int8 input (+ scale record). */
int aexrt_b200_act_quantize_concat(const AexrtB200ActSource* srcs, uint32_t nsrc, uint32_t n, uint32_t h, uint32_t w,
                                   uint32_t mode, uint32_t consumer_stride, void* q_out, float* scale_rec,
                                   void* stream);

/* fp16 slab8 repack of a concatenation of parts (fp16 convs). */
int aexrt_b200_pack_f16_concat(const AexrtB200ActSource* srcs, uint32_t nsrc, uint32_t n, uint32_t h, uint32_t w,
                               uint32_t consumer_stride, void* out, void* stream);

/* The same W8A8 conv reading its input straight from fp16 NHWC sources (the
 * producers' outputs: a concatenation of up to 4 slices, each optionally read
 * through a nearest 2x upsample for stride-1 convs), for plans created with
 * AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD whose info.quant_on_load is 1.  The conv
 * quantizes each 16-channel slab in shared memory with the scales of the
 * sources' amax slots (AexrtB200ActSource.amax_groups; per tensor or pg16 per the
 * plan), with the arithmetic of aexrt_b200_act_quantize_concat, so codes,
 * accumulators and outputs equal aexrt_b200_act_quantize_concat +
 * aexrt_b200_conv_w8a8 bit for bit, without the int8 codes ever reaching
 * memory: the reference's prequant pass (record_int8_prequant_activation,
 * runtime.cpp:21466-21665) and its conv (:4614-4923) in one launch.  Sources:
 * >= 16 channels each (a multiple of 16 but for the last), coff a multiple of
 * 16, ldc of 8, 16-byte aligned. */
int aexrt_b200_conv_w8a8_sources(const AexrtB200ConvPlan* plan, const AexrtB200ActSource* srcs, uint32_t nsrc,
                                 const void* residual, uint32_t res_ldc, uint32_t res_coff, void* out,
                                 uint32_t out_ldc, uint32_t out_coff, uint32_t* amax_out, uint32_t amax_stride,
                                 uint32_t amax_goff, int32_t* acc_dump, void* stream);


/* SPPF pooling (YOLOv8 SPPF: three cascaded MaxPool2d(5, 1, 2) whose outputs
 * are concatenated; reference kind MAXPOOL, engine.py:103-118): writes the 5x5,
 * 9x9 and 13x13 window maxima of the NHWC slice x into three consecutive
 * c-channel slices of out starting at out_coff, and max-es their |y| per
 * 16-channel group into amax (optional). */
int aexrt_b200_sppf_pool(const void* x, uint32_t n, uint32_t h, uint32_t w, uint32_t c, uint32_t ldc, uint32_t coff,
                         void* out, uint32_t out_ldc, uint32_t out_coff, uint32_t* amax, uint32_t amax_stride,
                         uint32_t amax_goff, void* stream);

/* ---------------------------------------------------------------- YOLOv11 fp16 ops
 * Depthwise 3x3 conv (pad 1, stride 1 or 2) on an NHWC fp16 slice: fp32
 * accumulation from the bias, optional SiLU, fp16 out.  The reference runs
 * grouped convs on its generic fp16 conv path (its int8 guard refuses
 * groups != 1, native/aexrt_d3d12_runtime.cpp:9404).  Output channel k reads
 * input channel coff + (k / grp) * grp_stride + grp_off + k % grp (grp = 0:
 * the plain slice).  w9: device [9][c] fp32 (kh-major taps), bias: device [c]
 * fp32; c, grp, strides and offsets multiples of 8. */
int aexrt_b200_dwconv3x3_f16(const void* x, uint32_t n, uint32_t h, uint32_t w, uint32_t c, uint32_t ldc,
                             uint32_t coff, uint32_t grp, uint32_t grp_stride, uint32_t grp_off, const float* w9,
                             const float* bias, uint32_t stride, uint32_t silu, void* out, uint32_t out_ldc,
                             uint32_t out_coff, void* stream);

/* C2PSA multi-head self-attention over an h x w map (the reference lowers it
 * to MATMUL / SOFTMAX commands, runtime.cpp:17305-17307, 20195, 20305): per
 * image and head, q, k (key_dim channels) and v (head_dim = 64) are that
 * head's consecutive channels of the qkv slice; out = v @ softmax(q^T k *
 * scale)^T + pe (the positional-encoding slice), fp16, with per-16-channel
 * |out| maxima max-ed into amax slots (NULL: none) for an int8 consumer.
 * h * w must fit one CTA's shared memory (up to 20 x 20 at key_dim 32). */
int aexrt_b200_psa_attention_f16(const void* qkv, uint32_t n, uint32_t h, uint32_t w, uint32_t ldc, uint32_t coff,
                                 uint32_t heads, uint32_t key_dim, uint32_t head_dim, float scale, const void* pe,
                                 uint32_t pe_ldc, uint32_t pe_coff, void* out, uint32_t out_ldc, uint32_t out_coff,
                                 uint32_t* amax, uint32_t amax_stride, uint32_t amax_goff, void* stream);

/* One detect level: box-distribution logits (4*reg_max channels) and class
 * logits (nc channels), both fp16 NHWC slices, with the level's stride. */
typedef struct AexrtB200DecodeLevel {
    const void* box;
    uint32_t box_ldc, box_coff;
    const void* cls;
    uint32_t cls_ldc, cls_coff;
    uint32_t h, w;
    float stride;
} AexrtB200DecodeLevel;

/* Anchor-free YOLOv8 decode (DFL expectation over reg_max bins, distance to
 * box, class sigmoid) into out[n][4 + nc][anchors] fp32 (cx, cy, w, h in input
 * pixels, then class scores): the layout of the model's output0 that the
 * reference post-processes (src/aexrt/yolo.py:92-138). */
int aexrt_b200_yolo_decode(const AexrtB200DecodeLevel* levels, uint32_t nlevels, uint32_t n, uint32_t nc,
                           uint32_t reg_max, float* out, void* stream);

/* One detection, layout-identical to the reference's AexrtYoloDetection
 * (native/aexrt.h:25-32): box corners in input pixels, score, class index as float. */
typedef struct AexrtYoloDetection {
    float x1;
    float y1;
    float x2;
    float y2;
    float score;
    float class_id;
} AexrtYoloDetection;

#define AEXRT_B200_NMS_MARK 0u   /* the reference GPU path's rule (runtime.cpp:15637-15691) */
#define AEXRT_B200_NMS_GREEDY 1u /* yolo_postprocess's greedy rule (src/aexrt/yolo.py:996-1007) */
#define AEXRT_B200_NMS_MAX_CANDIDATES 1024u

/* Post-process of a batch of YOLO output0 tensors into detections: replaces the
 * reference's decode-filter, NMS-mark and top-k dispatches
 * (record_yolo_decode_nms_topk, runtime.cpp:27104-27219; shaders :15300-15355,
 * :15637-15733) and, in greedy mode, yolo_postprocess (src/aexrt/yolo.py:92-138).
 *   output0: fp32 [n][channels][anchors] (layout 0 or 1) or [n][anchors][channels]
 *            (layout 2, the shader's channels-last case); channels = 4 (+1 with
 *            objectness) + nc: cx, cy, w, h, [objectness], class scores.
 *   Per image: best class = first maximum of (objectness *) class score, kept when
 *   score >= conf_threshold; the first max_candidates such anchors in anchor order
 *   are the candidates; NMS per class with IoU > iou_threshold; the kept boxes by
 *   (score desc, anchor order) fill detections[img * max_detections ...] and
 *   counts[img] = min(kept, max_detections); the rows after the count are zeroed.
 *   max_candidates <= AEXRT_B200_NMS_MAX_CANDIDATES (the reference default is 512).
 *   mode: the rule (AEXRT_B200_NMS_MARK / _GREEDY) in bits 0-7; bits 8-11 the CTAs
 *   per image (0 automatic: 8 for small batches down to 1 for large ones; else 1, 2,
 *   4 or 8), one thread-block cluster per image that shares the pair tests.  The
 *   detections do not depend on it. */
#define AEXRT_B200_NMS_CTAS_SHIFT 8u
int aexrt_b200_yolo_nms_topk(const float* output0, uint32_t n, uint32_t channels, uint32_t anchors, uint32_t nc,
                             uint32_t has_objectness, uint32_t layout, float conf_threshold, float iou_threshold,
                             uint32_t max_candidates, uint32_t max_detections, uint32_t mode,
                             AexrtYoloDetection* detections, uint32_t* counts, void* stream);

/* cudaMemsetAsync(ptr, 0, bytes, stream): clears amax slots inside a captured graph. */
int aexrt_b200_zero(void* ptr, uint64_t bytes, void* stream);

/* Standalone amax + quantize of an fp16 NCHW tensor for a stride-1 consumer (the
 * activation prequant of record_int8_prequant_activation,
 * native/aexrt_d3d12_runtime.cpp:21466-21665, amax + pack shaders :3212-3361):
 * writes q_out (slab16), scale_rec ([n][1 + ceil(c/16)]) and the per-(image, group)
 * amax bits into amax_groups[n][groups_total] at group_offset (caller memory, no
 * clearing needed).  Same results as aexrt_b200_act_amax_f16 (zero_first) +
 * aexrt_b200_act_quantize_f16, bit for bit.  When c % 16 == 0 and each
 * 16-channel strip splits into 1, 2 or 4 pixel slices (h * w a multiple of 8 per
 * slice, at most 112 KB each, at most 8 slices per image), one thread-block
 * cluster per image reads the tensor once (slices in shared memory, amax
 * exchanged between the CTAs); otherwise it runs those two kernels. */
int aexrt_b200_act_amax_quantize_f16(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t mode,
                                     uint32_t* amax_groups, uint32_t groups_total, uint32_t group_offset,
                                     void* q_out, float* scale_rec, void* stream);

/* The same call with the wait for the strip copies limited to wait_limit_cycles
 * SM clock cycles (capped at the default of 2^30).  For failure-detection tests:
 * a limit of 0 makes the first wait give up unless the data has landed, which
 * sets the status word and leaves that image's outputs unwritten; the kernel
 * still waits, with the full limit, for its own copies before it exits. */
int aexrt_b200_act_amax_quantize_f16_wait_limit(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w,
                                                uint32_t mode, uint32_t* amax_groups, uint32_t groups_total,
                                                uint32_t group_offset, void* q_out, float* scale_rec,
                                                uint64_t wait_limit_cycles, void* stream);

/* Reads and clears this device's activation-kernel status word (synchronises):
 * non-zero means a strip copy of aexrt_b200_act_amax_quantize_f16 did not land
 * within the wait limit; then no output of that image (codes, scale record,
 * amax slots) was written. */
int aexrt_b200_act_status(uint32_t* status);

/* ---------------------------------------------------------------- allocation-free variant
 * amax + quantize in one call for callers that cannot call cudaMalloc (a
 * real-time loop that allocates nothing after start-up, a plugin whose memory
 * belongs to its host's allocator, an embedded caller with no allocator): the
 * per-(image, 16-channel group) amax scratch lives in a fixed device array
 * inside the library instead of caller memory.  No counterpart in the
 * reference (there the amax buffer is allocated by the recorder).
 *   - The caller still passes the input, q_out and scale_rec, as for
 *     aexrt_b200_act_amax_f16 + aexrt_b200_act_quantize_f16, whose results it equals.
 *   - Limit: n * ceil(c / 16) <= 65536 slots (256 KB, held on every GPU that
 *     loads the library until exit); larger calls fail with a message.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress) with that device current: make it before any
 *     stream capture.  Each call clears its slots first.
 *   - The address is cached per device for the life of the process: do not
 *     use the library across a cudaDeviceReset (or any teardown of the
 *     device's primary context) on that device.
 *   - At most 65535 images per call (a grid dimension of the launches).
 *   - Every call shares the one array, so calls that overlap on the GPU (other
 *     streams, other host threads) race; serialize them.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
int aexrt_b200_act_quantize_f16_noalloc(const void* x, uint32_t n, uint32_t c, uint32_t h, uint32_t w, uint32_t layout,
                                        uint32_t ldc, uint32_t coff, uint32_t mode, uint32_t consumer_stride,
                                        void* q_out, float* scale_rec, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* AEXRT_B200_H */
