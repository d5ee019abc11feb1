/*
 * aexrt_yolo.h — the reference runtime's YOLO C ABI, served by libaexrt_b200.so.
 *
 * These are the entry points the reference's ctypes binding NativeCppYoloModel
 * (src/aexrt/cpp_runtime.py:229-662) and its C++ tools (examples/cpp/
 * conv_autotune.cpp, native_yolo_package.cpp) call, with the reference's names,
 * argument meaning, struct layouts and 1/0 status convention
 * (native/aexrt.h:25-51, 98-115, 129-137, 271-486).  Underneath, an .aexrt
 * engine compiled by the reference (`aexrtc build` / build_aexrt_engine) is
 * parsed and validated (engine_file.cu), lowered to the B200 kernels (W8A8
 * tcgen05 convs for planned kernels 51/52/53, fp16 convs for the others, the
 * SPPF pool, the fused YOLO head decode + NMS + top-k), given one arena
 * allocation by a lifetime planner, captured into one CUDA graph and replayed
 * per run on the device's stream.
 *
 * The AexrtDevice handle keeps the reference's "d3d12" constructor names so the
 * binding loads unchanged; on this backend it is a CUDA device and a stream.
 * Counters of D3D12 kernel families and pipeline caches that do not exist here
 * return 0; JSON packages and ONNX files are refused with a message (compile
 * them to .aexrt with the reference compiler).
 */
#ifndef AEXRT_YOLO_H
#define AEXRT_YOLO_H

#include <stdint.h>

#include "aexrt_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct AexrtDevice AexrtDevice;
typedef struct AexrtYoloModel AexrtYoloModel;

/* native/aexrt.h:34-41 (fields filled for the CUDA device: native_fp16_supported = 1). */
typedef struct AexrtD3D12Capabilities {
    uint32_t struct_size;
    uint32_t highest_shader_model;
    uint32_t native_fp16_supported;
    uint32_t wave_mma_tier;
    uint32_t dxc_available;
    uint32_t reserved[3];
} AexrtD3D12Capabilities;

/* native/aexrt.h:43-51: host times of the last aexrt_yolo_run in ms.
 * memcpy_ms: caller input into the pinned staging buffer (0 when the caller
 * wrote aexrt_yolo_input_ptr directly); submit_ms: the upload + graph launch +
 * read-back enqueue; fence_ms: the wait for the stream; readback_ms: copying
 * the detections out. */
typedef struct AexrtYoloRunTiming {
    uint32_t struct_size;
    uint32_t valid;
    double memcpy_ms;
    double submit_ms;
    double fence_ms;
    double readback_ms;
    uint64_t reserved[4];
} AexrtYoloRunTiming;

/* native/aexrt.h:435-445: one CONV / CONV_SILU command for the autotuner. */
typedef struct AexrtConvPlanInfo {
    uint32_t struct_size;
    uint32_t command_index;
    uint32_t kind_is_silu;
    AexrtConv2DDesc desc;
    uint32_t current_algorithm;   /* effective algorithm (after the fail-closed fallback) */
    uint32_t candidate_count;
    uint32_t candidates[32];      /* 51/52/53 when the int8 guard passes, and the fp16 path */
    uint32_t in_fusion_group;     /* 1: the conv carries a fused residual Add; do not override */
    uint32_t planned_algorithm;   /* the engine's planned kernel */
} AexrtConvPlanInfo;

/* ---------------------------------------------------------------- device
 * aexrt.h:129-137.  adapter_index = CUDA device ordinal. */
int aexrt_d3d12_probe(void);
AexrtDevice* aexrt_d3d12_create_device(uint32_t adapter_index);
int aexrt_d3d12_get_capabilities(AexrtDevice* device, AexrtD3D12Capabilities* capabilities);
void aexrt_d3d12_destroy_device(AexrtDevice* device);
/* The same device under this backend's own name. */
AexrtDevice* aexrt_cuda_create_device(uint32_t device_index);

/* ---------------------------------------------------------------- model (aexrt.h:271-486)
 * aexrt_yolo_load_engine: NULL on error (message in aexrt_b200_get_last_error()).
 * The engine's graph batch (value shapes' first dimension, 1 for aexrtc's
 * default) is the batch of one run. */
AexrtYoloModel* aexrt_yolo_load_engine(AexrtDevice* device, const char* engine_path);
AexrtYoloModel* aexrt_yolo_compile_from_package(AexrtDevice* device, const char* package_path);
AexrtYoloModel* aexrt_yolo_compile_from_onnx(AexrtDevice* device, const char* onnx_path);
uint64_t aexrt_yolo_input_element_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_class_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_anchor_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_channel_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_output_layout(AexrtYoloModel* model);
uint32_t aexrt_yolo_has_objectness(AexrtYoloModel* model);
uint32_t aexrt_yolo_package_mode(AexrtYoloModel* model);
uint32_t aexrt_yolo_graph_node_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_graph_value_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_constant_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_prepared_command_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_supported_prepared_command_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_unsupported_prepared_command_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_prepared_skipped_command_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_late_concat_conv1x1_fusion_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_concat_residual_conv1x1_fusion_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_paired_conv3x3_fusion_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_c2f_bottleneck_superblock_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_c2f_tail_residual_fusion_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_head_fusion_enabled(AexrtYoloModel* model);
uint32_t aexrt_yolo_head_final_conv_fusion_enabled(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_conv1x1_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_spatial_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_pack4_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_pack8_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_implicit_gemm_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_implicit_gemm_40x40_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_implicit_gemm_20x20_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_implicit_gemm_10x10_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_exact_40x40_64x64_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_exact_20x20_64x64_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_exact_10x10_128x128_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_exact_20x20_128x64_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_3x3_exact_10x10_256x64_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_tileflow_native_fp16_count(AexrtYoloModel* model);
int aexrt_yolo_is_executable(AexrtYoloModel* model);

/* aexrt.h:391-398: one synchronous inference of an engine whose graph batch is 1.
 * input: fp32 NCHW image, input_element_count elements (may be the pointer
 * aexrt_yolo_input_ptr returned).  Writes min(kept, max_detections) detections
 * ranked by score, and their count.  1 ok / 0 fail (aexrt_yolo_get_last_error). */
int aexrt_yolo_run(AexrtDevice* device, AexrtYoloModel* model, const float* input, uint64_t input_element_count,
                   AexrtYoloDetection* detections, uint32_t max_detections, uint32_t* out_detection_count);

/* aexrt.h:400-403: fp32 NCHW copy of an intermediate value after the last run
 * (elements = the value's element count); value 0xFFFFFFFF or the engine's
 * output value read output0.  Values whose arena slot a later command reuses
 * need aexrt_b200_yolo_set_arena_reuse(model, 0) before the run. */
int aexrt_yolo_debug_output(AexrtYoloModel* model, float* out, uint64_t elements);
int aexrt_yolo_debug_value(AexrtYoloModel* model, uint32_t value_id, float* out, uint64_t elements);
int aexrt_yolo_debug_page(AexrtYoloModel* model, uint32_t page_id, float* out, uint64_t elements);
const char* aexrt_yolo_get_last_error(AexrtYoloModel* model);
int aexrt_yolo_get_last_run_timing(AexrtYoloModel* model, AexrtYoloRunTiming* timing);
/* Runs are synchronous here (one frame in flight): returns 0 detections. */
int aexrt_yolo_flush_pipeline(AexrtYoloModel* model, AexrtYoloDetection* detections, uint32_t max_detections,
                              uint32_t* out_detection_count);
/* Per-launch device times of the last run, recorded when profiling is on
 * (environment AEXRT_NATIVE_D3D12_PROFILE_REPLAY=1 at load, as the reference,
 * or aexrt_b200_yolo_set_profiling): label "cmd#<i> <KIND> <in>-><out> alg=<id>". */
uint32_t aexrt_yolo_profile_event_count(AexrtYoloModel* model);
const char* aexrt_yolo_profile_event_label(AexrtYoloModel* model, uint32_t index);
double aexrt_yolo_profile_event_ms(AexrtYoloModel* model, uint32_t index);
/* aexrt.h:447-463: conv enumeration and algorithm override for the autotuner.
 * An override takes effect at the next run (the model is re-lowered). */
uint32_t aexrt_yolo_conv_plan_count(AexrtYoloModel* model);
int aexrt_yolo_conv_plan_info(AexrtYoloModel* model, uint32_t index, AexrtConvPlanInfo* out_info);
int aexrt_yolo_override_conv_algorithm(AexrtYoloModel* model, uint32_t command_index, uint32_t algorithm_id);
/* aexrt.h:465-468: the pinned host staging buffer of the model input: fp32 NCHW
 * (fp16 after aexrt_b200_yolo_set_input_dtype(model, 1)); a run whose input is
 * this pointer skips the input memcpy. */
void* aexrt_yolo_input_ptr(AexrtYoloModel* model, uint64_t* out_elements);
uint64_t aexrt_yolo_pipeline_cache_size(AexrtYoloModel* model);
int aexrt_yolo_export_pipeline_cache(AexrtYoloModel* model, void* output, uint64_t output_nbytes);
uint32_t aexrt_yolo_dxil_cache_hit_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_shader_cache_hit_count(AexrtYoloModel* model);
uint32_t aexrt_yolo_pso_cache_hit_count(AexrtYoloModel* model);
void aexrt_yolo_destroy(AexrtYoloModel* model);

/* ---------------------------------------------------------------- this backend's extensions
 * Parse and validate an engine image without a GPU (the loader's checks):
 * 1 valid / 0 with the reason in aexrt_b200_get_last_error(). */
int aexrt_b200_engine_validate(const void* bytes, uint64_t size);

/* Load an engine for `images` images per run (a multiple of the engine's graph
 * batch; every image is independent, so a batch-1 engine serves any batch). */
AexrtYoloModel* aexrt_b200_yolo_load_engine_batch(AexrtDevice* device, const char* engine_path, uint32_t images);
uint32_t aexrt_b200_yolo_batch(AexrtYoloModel* model);

/* Synchronous run of a whole batch from host memory: `images` fp32
 * (input_dtype 0) or fp16 (1) NCHW [batch][C][H][W]; per image a count and up to
 * max_detections rows (detections[i * max_detections ...], counts[i]). */
int aexrt_b200_yolo_run_batch(AexrtYoloModel* model, const void* images, uint32_t input_dtype,
                              AexrtYoloDetection* detections, uint32_t max_detections, uint32_t* counts);

/* Device-resident pieces for callers that stream themselves: the input buffer
 * (fp32 or fp16 NCHW per aexrt_b200_yolo_set_input_dtype), output0
 * ([batch][channels][anchors] fp32) and the detection buffer (uint32 counts
 * [batch], then AexrtYoloDetection [batch][max_detections of the manifest]). */
int aexrt_b200_yolo_set_input_dtype(AexrtYoloModel* model, uint32_t input_dtype);
void* aexrt_b200_yolo_device_input(AexrtYoloModel* model);
void* aexrt_b200_yolo_device_output0(AexrtYoloModel* model);
void* aexrt_b200_yolo_device_detections(AexrtYoloModel* model, uint64_t* out_bytes);
/* Enqueues one forward (graph replay) on `stream` (NULL: the device's stream). */
int aexrt_b200_yolo_enqueue(AexrtYoloModel* model, void* stream);
/* Kernel launches in one forward, and bytes of the model's arena / amax slots. */
uint32_t aexrt_b200_yolo_launch_count(AexrtYoloModel* model);
uint64_t aexrt_b200_yolo_arena_bytes(AexrtYoloModel* model);
/* B200 tile choice of one conv command (the block_n bits of
 * aexrt_b200_conv_plan_create: output-channel tile, variant, tile order,
 * stacked M blocks): int8 convs give identical results for every choice,
 * fp16 ones can differ in the last bit (see aexrt_b200_conv_plan_create). */
int aexrt_b200_yolo_override_conv_variant(AexrtYoloModel* model, uint32_t command_index, uint32_t block_n_bits);
int aexrt_b200_yolo_set_profiling(AexrtYoloModel* model, uint32_t enabled);
/* 1 (default): int8 convs quantize their fp16 inputs on load (one launch each);
 * 0: a separate quantize launch writes the int8 codes first.  Same results. */
int aexrt_b200_yolo_set_quant_on_load(AexrtYoloModel* model, uint32_t enabled);
/* 0: every value keeps its own arena slot (so aexrt_yolo_debug_value can read
 * any of them); 1 (default): slots are reused between values whose lifetimes
 * do not overlap. */
int aexrt_b200_yolo_set_arena_reuse(AexrtYoloModel* model, uint32_t enabled);
/* OR of every conv plan's device status word (synchronises). */
int aexrt_b200_yolo_status(AexrtYoloModel* model, uint32_t* status);

/* Lifetime-based arena placement: item i of `bytes` lives over the launches
 * [first[i], last[i]]; offsets receive byte offsets (multiples of alignment)
 * such that items whose lifetimes overlap never overlap in memory; *total is
 * the arena size.  Host only. */
int aexrt_b200_arena_plan(uint32_t count, const uint64_t* bytes, const uint32_t* first, const uint32_t* last,
                          uint64_t alignment, uint64_t* offsets, uint64_t* total);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* AEXRT_YOLO_H */
