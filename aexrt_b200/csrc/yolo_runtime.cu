// The reference's YOLO runtime ABI (include/aexrt_yolo.h) on the B200 kernels.
//
// An engine compiled by the reference (.aexrt, parsed and validated by
// engine_file.cu) is lowered command by command into this backend's launches,
// the way the reference's prepared replay lowers it into D3D12 dispatches
// (ensure_prepared_yolo_replay / record_prepared_physical_stream /
// record_direct_logical_command, native/aexrt_d3d12_runtime.cpp:28307-29010):
//   CONV / CONV_SILU   planned kernel 51/52/53 -> quantize + tcgen05 W8A8 conv
//                      (layout-8 weights of the engine); others -> fp16 conv;
//                      a planned int8 kernel that fails the int8 guard falls back
//                      to the fp16 conv (replay_conv_algorithm, :9424-9503)
//   CONCAT_CONV1X1     fp16 1x1 conv over the concatenated parts (read in place)
//   CONCAT / VIEW / SLICE / RESIZE (channel concat, channel views, nearest 2x)
//                      -> no launch: consumers read the parts in place
//   MAXPOOL x3 (5x5 s1) SPPF cascade -> one SPPF pool launch; other MAXPOOL ->
//                      a generic pool
//   BINARY Add         -> the residual of the conv that produced one operand (when
//                      that conv's output has no other reader), else a generic add
//   YOLO head          the reference's head fusion rule (detect_yolo_head_fusion,
//                      :26956-27100): per-level CONCAT(box 64, class nc) and the
//                      final 3-input CONCAT; those and every later command are
//                      replaced by the decode + filter + NMS + top-k launches
// Activations are fp16 NHWC buffers placed in one device allocation by a
// lifetime planner (aexrt_b200_arena_plan); int8 consumers get per-(image,
// group) amax slots that their producers' epilogues fill.  One forward is
// captured into a CUDA graph and replayed per run on the device's stream.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/aexrt_b200.h"
#include "../../include/aexrt_yolo.h"
#include "engine_file.h"
#include "graph_ops.cuh"
#include "launch.cuh"

using aexrt::engine::Command;
using aexrt::engine::Engine;

namespace aexrt {
void set_last_error(const char* msg);  // capi.cu: the message aexrt_b200_get_last_error returns
}

struct AexrtDevice {
  int cuda_device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
};

namespace {


int set_error(std::string* model_err, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  aexrt::set_last_error(buf);
  if (model_err) *model_err = buf;
  return 0;
}

bool cuda_ok(cudaError_t e, const char* what, std::string* model_err = nullptr) {
  if (e == cudaSuccess) return true;
  set_error(model_err, "%s: %s", what, cudaGetErrorString(e));
  return false;
}

constexpr int kInput = -1;  // part source: the graph input (NCHW images)
constexpr uint32_t kFp16Generic = 0, kFp16Conv1x1 = 1;

struct Part {
  int buf = kInput;
  int coff = 0, ch = 0, up = 1;
};
using Parts = std::vector<Part>;

struct Buffer {
  int c = 0, h = 0, w = 0;  // fp16 NHWC [batch][h][w][c]; c = 0 for raw scratch
  uint64_t bytes = 0, off = 0;
  int first = -1, last = -1;
  bool amax = false;
  uint64_t amax_off = 0;  // in uint32 slots
  int groups = 0;
};

enum OpKind { kOpConv, kOpSppf, kOpMaxPool, kOpAdd, kOpDecode, kOpNms };
enum ConvPath { kPathInt8, kPathInt8Ql, kPathF16Pack, kPathF16Nhwc, kPathStem };

struct Op {
  OpKind kind = kOpConv;
  int cmd = -1;
  std::string label;
  // conv
  AexrtB200ConvPlan* plan = nullptr;
  ConvPath path = kPathInt8;
  bool pg16 = false;
  int k = 1, s = 1, in_h = 0, in_w = 0, ic = 0, oc = 0;
  uint32_t algorithm = 0;
  Parts in;
  int out = -1;
  bool has_res = false;
  Part res;
  int q = -1, rec = -1, x8 = -1;
  // pools / add
  Part x;
  Parts a, b;
  int pool_k = 0, pool_s = 1, pool_p = 0, out_h = 0, out_w = 0, c = 0;
  // head
  Part box[3], cls[3];
  int lh[3] = {0, 0, 0}, lw[3] = {0, 0, 0};
};

struct ConvInfo {
  uint32_t cmd = 0;
  AexrtConv2DDesc desc{};
  bool silu = false;
  uint32_t planned = 0, current = 0;
  std::vector<uint32_t> candidates;
  bool fused_residual = false;
};

}  // namespace

struct AexrtYoloModel {
  AexrtDevice* dev = nullptr;
  Engine eng;
  std::string error;
  uint32_t batch = 1;        // images per run
  uint32_t graph_batch = 1;  // the engine's batch
  uint32_t input_dtype = 0;  // 0 fp32, 1 fp16
  bool profiling = false, reuse = true, dirty = true, head_fusion = false;
  bool quant_on_load = false;  // int8 convs quantize their fp16 inputs on load (else a quantize launch each)
  std::map<uint32_t, uint32_t> overrides, variants;
  // lowered state
  std::vector<Buffer> bufs;
  std::vector<Op> ops;
  std::vector<ConvInfo> convs;
  std::vector<int> value_op;   // producing op of each value (-1)
  std::vector<Parts> vparts;
  std::vector<bool> vdefined;
  uint32_t skipped = 0, launches = 0;
  uint64_t arena_bytes = 0, amax_slots = 0;
  void* d_arena = nullptr;
  uint64_t d_arena_cap = 0;
  uint32_t* d_amax = nullptr;
  uint64_t d_amax_cap = 0;
  void* d_input = nullptr;
  void* h_input = nullptr;
  uint64_t input_bytes = 0;
  float* d_output0 = nullptr;
  uint8_t* d_dets = nullptr;
  uint8_t* h_dets = nullptr;
  uint64_t dets_bytes = 0;
  int channels_in = 3, img_h = 0, img_w = 0;
  cudaGraphExec_t graph = nullptr;
  // profiling
  std::vector<std::string> prof_labels;
  std::vector<double> prof_ms;
  AexrtYoloRunTiming timing{};
  std::mutex mu;
};

namespace {

using namespace aexrt::engine;

// ------------------------------------------------------------------ helpers

uint32_t int8_kernel_for(uint32_t k, uint32_t s) { return k == 1 ? 51u : (s == 1 ? 52u : 53u); }

bool is_int8_id(uint32_t a) { return a == 51 || a == 52 || a == 53; }

AexrtConv2DDesc desc_of(const Command& c, uint32_t batch) {
  AexrtConv2DDesc d{};
  uint32_t* f = reinterpret_cast<uint32_t*>(&d);
  for (int i = 0; i < 16; ++i) f[i] = c.params[i];
  d.batch = batch;
  return d;
}

// can_use_conv_int8 (native/aexrt_d3d12_runtime.cpp:9398-9422) for the command's own planned id
bool int8_guard(const AexrtConv2DDesc& d, uint32_t id, bool pg) {
  if (d.groups != 1 || d.in_channels % 4 || d.out_channels % 4 || d.dilation_h != 1 || d.dilation_w != 1) return false;
  if (pg && d.in_channels % 16) return false;
  if (id == 51)
    return d.kernel_h == 1 && d.kernel_w == 1 && d.stride_h == 1 && d.stride_w == 1 && !d.pad_top && !d.pad_left &&
           d.out_channels % 8 == 0 && d.in_h == d.out_h && d.in_w == d.out_w;
  if (d.kernel_h != 3 || d.kernel_w != 3 || d.pad_top != 1 || d.pad_left != 1) return false;
  if (id == 52) return d.stride_h == 1 && d.stride_w == 1 && d.in_h == d.out_h && d.in_w == d.out_w;
  if (id == 53)
    return d.stride_h == 2 && d.stride_w == 2 && d.in_h >= d.out_h * 2 - 1 && d.in_w >= d.out_w * 2 - 1 &&
           d.out_h == (d.in_h + 1) / 2 && d.out_w == (d.in_w + 1) / 2;
  return false;
}

// The shapes this backend's fp16 conv plans accept.
bool f16_ok(const AexrtConv2DDesc& d) {
  const bool k1 = d.kernel_h == 1 && d.kernel_w == 1 && !d.pad_top && !d.pad_left && d.stride_h == 1 && d.stride_w == 1;
  const bool k3 = d.kernel_h == 3 && d.kernel_w == 3 && d.pad_top == 1 && d.pad_left == 1 &&
                  ((d.stride_h == 1 && d.stride_w == 1) || (d.stride_h == 2 && d.stride_w == 2));
  return (k1 || k3) && d.groups == 1 && d.dilation_h == 1 && d.dilation_w == 1;
}

Parts sub_parts(const Parts& src, int coff, int ch) {
  Parts out;
  int base = 0;
  for (const Part& p : src) {
    const int lo = std::max(coff, base), hi = std::min(coff + ch, base + p.ch);
    if (lo < hi) {
      Part q = p;
      q.coff = p.coff + (lo - base);
      q.ch = hi - lo;
      out.push_back(q);
    }
    base += p.ch;
  }
  return out;
}

// adjacent slices of one buffer merge into one part
Parts merge_parts(const Parts& src) {
  Parts out;
  for (const Part& p : src) {
    if (!out.empty() && out.back().buf == p.buf && out.back().up == p.up && p.buf != kInput &&
        out.back().coff + out.back().ch == p.coff) {
      out.back().ch += p.ch;
    } else {
      out.push_back(p);
    }
  }
  return out;
}

int parts_channels(const Parts& p) {
  int c = 0;
  for (const Part& q : p) c += q.ch;
  return c;
}

// ------------------------------------------------------------------ head fusion (reference rule)

struct HeadFusion {
  bool found = false;
  uint32_t box[3], cls[3], concat_cmd[3], final_cmd = 0;
};

bool alias_of(const Engine& e, uint32_t value, uint32_t source) {
  if (value == source) return true;
  for (const Command& c : e.commands)
    if ((c.kind == kAlias || c.kind == kView) && c.output == value && !c.inputs.empty() && c.inputs[0] == source)
      return true;
  return false;
}

HeadFusion find_head(const Engine& e) {
  // detect_yolo_head_fusion, native/aexrt_d3d12_runtime.cpp:26956-27040
  HeadFusion hf;
  const uint32_t classes = e.manifest.classes();
  struct Cand {
    uint32_t cmd, out, box, cls, hw;
  };
  std::vector<Cand> cands;
  for (uint32_t i = 0; i < e.commands.size(); ++i) {
    const Command& c = e.commands[i];
    if (c.kind != kConcat || c.inputs.size() != 2 || c.params.size() < 10) continue;
    if (c.params[1] != 4 || c.params[2] != 1 || c.params[3] != 2 || c.params[8] != 64 || c.params[9] != classes) continue;
    const Value& bv = e.values[c.inputs[0]];
    const Value& cv = e.values[c.inputs[1]];
    if (bv.shape[1] != 64 || cv.shape[1] != classes || bv.shape[2] != cv.shape[2] || bv.shape[3] != cv.shape[3]) continue;
    cands.push_back({i, c.output, c.inputs[0], c.inputs[1], bv.shape[2] * bv.shape[3]});
  }
  if (cands.size() < 3) return hf;
  std::stable_sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.hw > b.hw; });
  cands.resize(3);
  for (uint32_t i = 0; i < e.commands.size(); ++i) {
    const Command& c = e.commands[i];
    if (c.kind != kConcat || c.inputs.size() != 3 || c.params.size() < 8 || c.params[2] != 3) continue;
    int matched = 0;
    for (const Cand& s : cands)
      for (uint32_t in : c.inputs)
        if (alias_of(e, in, s.out)) {
          ++matched;
          break;
        }
    if (matched == 3) {
      hf.found = true;
      hf.final_cmd = i;
      break;
    }
  }
  if (!hf.found) return hf;
  for (int k = 0; k < 3; ++k) {
    hf.box[k] = cands[k].box;
    hf.cls[k] = cands[k].cls;
    hf.concat_cmd[k] = cands[k].cmd;
  }
  return hf;
}

// ------------------------------------------------------------------ lowering

struct Lowering {
  AexrtYoloModel* m;
  const Engine& e;
  std::vector<int> consumers;  // per value, among executed commands
  std::vector<bool> skip;

  explicit Lowering(AexrtYoloModel* model) : m(model), e(model->eng) {}

  int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return set_error(&m->error, "%s", buf);
  }

  int new_buffer(int c, int h, int w) {
    Buffer b;
    b.c = c;
    b.h = h;
    b.w = w;
    b.bytes = uint64_t(m->batch) * h * w * c * 2;
    m->bufs.push_back(b);
    return static_cast<int>(m->bufs.size()) - 1;
  }

  int new_scratch(uint64_t bytes) {
    Buffer b;
    b.bytes = bytes;
    m->bufs.push_back(b);
    return static_cast<int>(m->bufs.size()) - 1;
  }

  bool parts_of(uint32_t value, Parts* out) {
    if (value == e.manifest.input_value()) {
      const Value& v = e.values[value];
      *out = {Part{kInput, 0, static_cast<int>(v.shape[1]), 1}};
      return true;
    }
    if (value >= m->vparts.size() || !m->vdefined[value]) {
      fail("value %u is read before a supported command produced it", value);
      return false;
    }
    *out = m->vparts[value];
    return true;
  }

  void define(uint32_t value, const Parts& p) {
    m->vparts[value] = p;
    m->vdefined[value] = true;
  }

  // spatial dims of a part as the consumer sees it
  void part_hw(const Part& p, int* h, int* w) {
    if (p.buf == kInput) {
      *h = m->img_h;
      *w = m->img_w;
    } else {
      *h = m->bufs[p.buf].h * p.up;
      *w = m->bufs[p.buf].w * p.up;
    }
  }

  std::vector<float> constant(uint32_t value, size_t want) {
    auto it = e.constants.find(value);
    if (it == e.constants.end() || it->second.data.size() != want) return {};
    return it->second.data;
  }

  bool lower_conv(uint32_t ci, const Command& c, const Parts& in, const std::vector<float>& weight,
                  const std::vector<float>& bias, bool silu, bool allow_int8) {
    AexrtConv2DDesc d = desc_of(c, m->batch);
    if (c.params[0] != m->graph_batch || e.values[c.output].shape[0] != m->graph_batch)
      return fail("conv %u: descriptor batch differs from the graph batch %u", ci, m->graph_batch) != 0;
    int ih = 0, iw = 0;
    part_hw(in[0], &ih, &iw);
    if (parts_channels(in) != static_cast<int>(d.in_channels) || ih != static_cast<int>(d.in_h) ||
        iw != static_cast<int>(d.in_w))
      return fail("conv %u: input parts do not match its descriptor", ci) != 0;
    for (const Part& p : in) {
      int h = 0, w = 0;
      part_hw(p, &h, &w);
      if (h != ih || w != iw) return fail("conv %u: concatenated parts differ in size", ci) != 0;
    }
    ConvInfo info;
    info.cmd = ci;
    info.desc = desc_of(c, m->graph_batch);
    info.silu = silu;
    info.planned = c.planned_kernel;
    const uint32_t iid = int8_kernel_for(d.kernel_h, d.stride_h);
    const bool pg = (c.plan_flags & kPlanInt8PerGroup) != 0;
    if (allow_int8 && int8_guard(d, iid, pg) && in[0].buf != kInput) info.candidates.push_back(iid);
    const uint32_t fid = d.kernel_h == 1 ? kFp16Conv1x1 : kFp16Generic;
    info.candidates.push_back(is_int8_id(c.planned_kernel) || !allow_int8 ? fid : c.planned_kernel);
    uint32_t alg = c.planned_kernel;
    auto ov = m->overrides.find(ci);
    if (ov != m->overrides.end()) alg = ov->second;
    // fail-closed fallback: an int8 id that the guard refuses runs the fp16 conv; so does an input
    // whose concatenated slices do not start on 16-channel groups (the quantizer's slab rule)
    bool parts16 = true;
    for (size_t k = 0; k < in.size(); ++k)
      parts16 = parts16 && in[k].buf != kInput && in[k].coff % 16 == 0 && (k + 1 == in.size() || in[k].ch % 16 == 0);
    bool int8 = allow_int8 && is_int8_id(alg) && alg == iid && int8_guard(d, iid, pg) && parts16;
    if (is_int8_id(alg) && !int8) alg = fid;
    info.current = alg;

    Op op;
    op.kind = kOpConv;
    op.cmd = static_cast<int>(ci);
    op.k = static_cast<int>(d.kernel_h);
    op.s = static_cast<int>(d.stride_h);
    op.in_h = ih;
    op.in_w = iw;
    op.ic = static_cast<int>(d.in_channels);
    op.oc = static_cast<int>(d.out_channels);
    op.in = merge_parts(in);
    op.algorithm = alg;
    op.pg16 = int8 && pg;
    const uint32_t kind = silu ? AEXRT_B200_KIND_CONV_SILU : AEXRT_B200_KIND_CONV;
    const uint32_t vbits = m->variants.count(ci) ? m->variants[ci] : 0u;
    if (int8) {
      std::vector<int8_t> codes(size_t(d.out_channels) * d.in_channels * d.kernel_h * d.kernel_w);
      std::vector<float> scale(d.out_channels);
      auto pk = e.packed.find(c.inputs[1]);
      if (pk != e.packed.end() && pk->second.layout == kLayoutConvInt8 && c.packed_value == c.inputs[1]) {
        // the engine's own layout-8 payload: [oc*ic*kk int8][oc fp32] (src/aexrt/engine.py:2458)
        if (pk->second.in_channels != d.in_channels || pk->second.out_channels != d.out_channels ||
            pk->second.data.size() != codes.size() + 4 * scale.size())
          return fail("conv %u: layout-8 payload does not match the conv", ci) != 0;
        std::memcpy(codes.data(), pk->second.data.data(), codes.size());
        std::memcpy(scale.data(), pk->second.data.data() + codes.size(), 4 * scale.size());
      } else {
        // no layout-8 payload (an override to int8): quantize at load, as the reference does when the
        // engine lacks layout 8 (ensure_conv_int8_weight, runtime.cpp:21716-21742)
        if (!aexrt_b200_quantize_conv_weight_int8(weight.data(), d.out_channels, d.in_channels,
                                                  d.kernel_h * d.kernel_w, e.manifest.precision() == 2,
                                                  codes.data(), scale.data()))
          return fail("conv %u: weight quantization failed", ci) != 0;
      }
      // quantize on load when every part fits its rules: the conv reads the producers' fp16 slices
      bool ql = m->quant_on_load && op.in.size() <= 4;
      for (size_t k = 0; k < op.in.size(); ++k)
        ql = ql && op.in[k].ch >= 16 && (op.in[k].up == 1 || op.s == 1);
      uint32_t pflags = (pg ? AEXRT_B200_PLAN_FLAG_INT8_PERGROUP : 0u) | (ql ? AEXRT_B200_PLAN_FLAG_QUANT_ON_LOAD : 0u);
      op.plan = aexrt_b200_conv_plan_create(&d, kind, iid, pflags, codes.data(), scale.data(), bias.data(), vbits);
      if (!op.plan) return fail("conv %u: %s", ci, aexrt_b200_get_last_error()) != 0;
      AexrtB200ConvPlanInfo pi{};
      aexrt_b200_conv_plan_info(op.plan, &pi);
      if (ql && pi.quant_on_load) {
        op.path = kPathInt8Ql;
      } else {
        op.path = kPathInt8;
        op.q = new_scratch(aexrt_b200_packed_act_bytes(d.batch, d.in_channels, d.in_h, d.in_w, d.stride_h));
        op.rec = new_scratch(uint64_t(d.batch) * (1 + (d.in_channels + 15) / 16) * 4);
      }
    } else {
      if (!f16_ok(d)) return fail("conv %u: shape outside the fp16 conv (k 1 or 3, pad k/2, stride 1/2)", ci) != 0;
      op.plan = aexrt_b200_conv_plan_create_f16(&d, kind, weight.data(), bias.data(), vbits);
      if (!op.plan) return fail("conv %u: %s", ci, aexrt_b200_get_last_error()) != 0;
      AexrtB200ConvPlanInfo pi{};
      aexrt_b200_conv_plan_info(op.plan, &pi);
      const Part& p0 = op.in[0];
      if (op.in.size() == 1 && p0.buf == kInput && pi.image_input && m->input_dtype <= 1) {
        op.path = kPathStem;
      } else if (op.in.size() == 1 && p0.buf != kInput && p0.up == 1 && op.s == 1 && pi.variant == 2 &&
                 op.ic % 8 == 0 && p0.coff % 8 == 0 && m->bufs[p0.buf].c % 8 == 0) {
        op.path = kPathF16Nhwc;
      } else {
        op.path = kPathF16Pack;
        op.x8 = new_scratch(aexrt_b200_packed_f16_bytes(d.batch, d.in_channels, d.in_h, d.in_w, d.stride_h));
      }
    }
    op.out = new_buffer(op.oc, static_cast<int>(d.out_h), static_cast<int>(d.out_w));
    char lab[160];
    std::snprintf(lab, sizeof(lab), "cmd#%u %s %ux%ux%u->%u%s alg=%u", ci, kind_name(c.kind), d.in_channels, d.in_h,
                  d.in_w, d.out_channels, op.s == 2 ? " s2" : "", alg);
    op.label = lab;
    if (allow_int8) m->convs.push_back(info);  // the CONV / CONV_SILU commands (not CONCAT_CONV1X1)
    m->value_op[c.output] = static_cast<int>(m->ops.size());
    m->ops.push_back(op);
    define(c.output, {Part{op.out, 0, op.oc, 1}});
    return true;
  }

  bool run() {
    const uint32_t nv = e.manifest.value_count();
    m->vparts.assign(nv, {});
    m->vdefined.assign(nv, false);
    m->value_op.assign(nv, -1);
    const Value& in = e.values[e.manifest.input_value()];
    if (in.shape[0] == 0 || in.shape[1] == 0) return fail("graph input has an empty shape") != 0;
    m->graph_batch = in.shape[0];
    if (m->batch % m->graph_batch) return fail("batch %u is not a multiple of the engine's %u", m->batch, m->graph_batch) != 0;
    m->channels_in = static_cast<int>(in.shape[1]);
    m->img_h = static_cast<int>(in.shape[2]);
    m->img_w = static_cast<int>(in.shape[3]);
    const HeadFusion hf = find_head(e);
    if (!hf.found) return fail("no YOLO head (per-level box 64 + class CONCATs and a final 3-way CONCAT) in the engine") != 0;
    m->head_fusion = true;
    skip.assign(e.commands.size(), false);
    for (uint32_t i = hf.final_cmd; i < e.commands.size(); ++i) skip[i] = true;
    for (int k = 0; k < 3; ++k) {
      skip[hf.concat_cmd[k]] = true;
      for (uint32_t j = 0; j < hf.final_cmd; ++j) {
        const Command& c = e.commands[j];
        if ((c.kind == kAlias || c.kind == kView) && !c.inputs.empty() &&
            e.commands[hf.concat_cmd[k]].output == c.inputs[0])
          skip[j] = true;
      }
    }
    consumers.assign(nv, 0);
    for (uint32_t i = 0; i < e.commands.size(); ++i)
      if (!skip[i])
        for (uint32_t v : e.commands[i].inputs) consumers[v]++;
    for (int k = 0; k < 3; ++k) {
      consumers[hf.box[k]]++;
      consumers[hf.cls[k]]++;
    }
    m->skipped = 0;
    for (bool s : skip) m->skipped += s ? 1 : 0;

    for (uint32_t i = 0; i < e.commands.size(); ++i) {
      if (skip[i]) continue;
      const Command& c = e.commands[i];
      switch (c.kind) {
        case kConv:
        case kConvSilu: {
          if (c.inputs.size() < 3 || c.params.size() < 16) return fail("conv %u: malformed command", i) != 0;
          Parts in;
          if (!parts_of(c.inputs[0], &in)) return false;
          const AexrtConv2DDesc d = desc_of(c, 1);
          auto w = constant(c.inputs[1], size_t(d.out_channels) * (d.in_channels / std::max(1u, d.groups)) *
                                             d.kernel_h * d.kernel_w);
          auto b = constant(c.inputs[2], d.out_channels);
          if (w.empty() || b.empty()) return fail("conv %u: weight or bias constant missing", i) != 0;
          if (!lower_conv(i, c, in, w, b, c.kind == kConvSilu, true)) return false;
          break;
        }
        case kConcatConv1x1: {
          // params: N, H, W, OC, silu, per-input channels (src/aexrt/yolo.py:793-799)
          if (c.params.size() < 5 || c.inputs.size() < 3) return fail("concat_conv1x1 %u: malformed command", i) != 0;
          if (is_int8_id(c.planned_kernel)) return fail("concat_conv1x1 %u: int8 kernel id on a fused command", i) != 0;
          const size_t nin = c.inputs.size() - 2;
          Parts in;
          for (size_t k = 0; k < nin; ++k) {
            Parts p;
            if (!parts_of(c.inputs[k], &p)) return false;
            in.insert(in.end(), p.begin(), p.end());
          }
          const uint32_t oc = c.params[3], ic = static_cast<uint32_t>(parts_channels(in));
          Command cc = c;
          cc.params.assign(16, 0);
          const uint32_t dd[16] = {m->graph_batch, ic, c.params[1], c.params[2], oc, c.params[1], c.params[2], 1, 1,
                                   1, 1, 0, 0, 1, 1, 1};
          for (int k = 0; k < 16; ++k) cc.params[k] = dd[k];
          cc.inputs = {c.inputs[0], c.inputs[nin], c.inputs[nin + 1]};
          auto w = constant(c.inputs[nin], size_t(oc) * ic);
          auto b = constant(c.inputs[nin + 1], oc);
          if (w.empty() || b.empty()) return fail("concat_conv1x1 %u: weight or bias constant missing", i) != 0;
          if (!lower_conv(i, cc, in, w, b, c.params[4] != 0, false)) return false;
          break;
        }
        case kView: {
          // channel split view at batch 1: (element offset, element count) of the NCHW source
          Parts src;
          if (!parts_of(c.inputs[0], &src)) return false;
          const Value& sv = e.values[c.inputs[0]];
          const uint64_t plane = uint64_t(sv.shape[2]) * sv.shape[3];
          if (c.params.size() < 2 || plane == 0 || c.params[0] % plane || c.params[1] % plane || sv.shape[0] != 1)
            return fail("VIEW %u: not a channel view of a batch-1 NCHW value", i) != 0;
          define(c.output, sub_parts(src, static_cast<int>(c.params[0] / plane), static_cast<int>(c.params[1] / plane)));
          break;
        }
        case kAlias: {
          Parts src;
          if (!parts_of(c.inputs[0], &src)) return false;
          const Value& sv = e.values[c.inputs[0]];
          const Value& ov = e.values[c.output];
          if (std::memcmp(sv.shape, ov.shape, sizeof(sv.shape)) != 0)
            return fail("ALIAS %u: a reshape that moves elements (outside the head) is not supported", i) != 0;
          define(c.output, src);
          break;
        }
        case kSlice: {
          // params: numel, rank, 0, 0, src4[4], out4[4], starts4[4], steps4[4] (src/aexrt/yolo.py:880-884)
          Parts src;
          if (!parts_of(c.inputs[0], &src)) return false;
          if (c.params.size() < 20) return fail("SLICE %u: malformed command", i) != 0;
          const uint32_t* s4 = &c.params[4];
          const uint32_t* o4 = &c.params[8];
          const uint32_t* st = &c.params[12];
          const uint32_t* sp = &c.params[16];
          if (c.params[1] != 4 || st[0] || st[2] || st[3] || sp[0] != 1 || sp[1] != 1 || sp[2] != 1 || sp[3] != 1 ||
              o4[0] != s4[0] || o4[2] != s4[2] || o4[3] != s4[3])
            return fail("SLICE %u: only channel slices of NCHW values are supported", i) != 0;
          define(c.output, sub_parts(src, static_cast<int>(st[1]), static_cast<int>(o4[1])));
          break;
        }
        case kConcat: {
          // params: numel, rank, padded axis, inputs, out4[4], sizes[8], 0, 0
          if (c.params.size() < 4 || c.params[1] != 4 || c.params[2] != 1)
            return fail("CONCAT %u: only channel concat of NCHW values is supported", i) != 0;
          Parts all;
          for (uint32_t v : c.inputs) {
            Parts p;
            if (!parts_of(v, &p)) return false;
            all.insert(all.end(), p.begin(), p.end());
          }
          define(c.output, merge_parts(all));
          break;
        }
        case kResize: {
          // params: n, c, ih, iw, oh, ow
          Parts src;
          if (!parts_of(c.inputs[0], &src)) return false;
          if (c.params.size() < 6 || c.params[4] != 2 * c.params[2] || c.params[5] != 2 * c.params[3])
            return fail("RESIZE %u: only nearest 2x is supported", i) != 0;
          for (Part& p : src) {
            if (p.up != 1 || p.buf == kInput) return fail("RESIZE %u: nested upsample", i) != 0;
            p.up = 2;
          }
          define(c.output, src);
          break;
        }
        case kMaxPool: {
          // params: n, c, ih, iw, oh, ow, kh, kw, sh, sw, ph, pw, dilation
          if (c.params.size() < 13) return fail("MAXPOOL %u: malformed command", i) != 0;
          Parts src;
          if (!parts_of(c.inputs[0], &src)) return false;
          const uint32_t* p = c.params.data();
          const bool sppf5 = p[6] == 5 && p[7] == 5 && p[8] == 1 && p[9] == 1 && p[10] == 2 && p[11] == 2 && p[12] == 1;
          // the SPPF cascade: three 5x5 stride-1 pools, each reading the previous one
          uint32_t j1 = i + 1, j2 = i + 2;
          while (j1 < e.commands.size() && skip[j1]) ++j1;
          j2 = j1 + 1;
          while (j2 < e.commands.size() && skip[j2]) ++j2;
          const bool chain = sppf5 && src.size() == 1 && src[0].buf != kInput && src[0].up == 1 && p[1] % 16 == 0 &&
                             src[0].coff % 8 == 0 && m->bufs[src[0].buf].c % 8 == 0 &&
                             j2 < e.commands.size() && e.commands[j1].kind == kMaxPool &&
                             e.commands[j2].kind == kMaxPool && e.commands[j1].inputs[0] == c.output &&
                             e.commands[j2].inputs[0] == e.commands[j1].output &&
                             e.commands[j1].params == c.params && e.commands[j2].params == c.params &&
                             consumers[c.output] <= 2 && consumers[e.commands[j1].output] <= 2;
          const int ch = static_cast<int>(p[1]);
          if (chain) {
            Op op;
            op.kind = kOpSppf;
            op.cmd = static_cast<int>(i);
            op.x = src[0];
            op.c = ch;
            op.out = new_buffer(3 * ch, static_cast<int>(p[4]), static_cast<int>(p[5]));
            op.label = "cmd#" + std::to_string(i) + " MAXPOOL x3 (SPPF)";
            const int oi = static_cast<int>(m->ops.size());
            m->ops.push_back(op);
            const uint32_t outs[3] = {c.output, e.commands[j1].output, e.commands[j2].output};
            for (int k = 0; k < 3; ++k) {
              define(outs[k], {Part{op.out, k * ch, ch, 1}});
              m->value_op[outs[k]] = oi;
            }
            skip[j1] = skip[j2] = true;
            i = j2;
          } else {
            if (p[12] != 1 || p[6] != p[7] || p[8] != p[9] || p[10] != p[11] || src.size() > aexrt::kMaxGraphParts)
              return fail("MAXPOOL %u: square kernel, stride and padding without dilation only", i) != 0;
            Op op;
            op.kind = kOpMaxPool;
            op.cmd = static_cast<int>(i);
            op.a = src;
            op.pool_k = static_cast<int>(p[6]);
            op.pool_s = static_cast<int>(p[8]);
            op.pool_p = static_cast<int>(p[10]);
            op.c = ch;
            op.in_h = static_cast<int>(p[2]);
            op.in_w = static_cast<int>(p[3]);
            op.out_h = static_cast<int>(p[4]);
            op.out_w = static_cast<int>(p[5]);
            op.out = new_buffer(ch, op.out_h, op.out_w);
            op.label = "cmd#" + std::to_string(i) + " MAXPOOL";
            m->value_op[c.output] = static_cast<int>(m->ops.size());
            m->ops.push_back(op);
            define(c.output, {Part{op.out, 0, ch, 1}});
          }
          break;
        }
        case kBinary: {
          // params: numel, op, rank, 0, out4[4], a4[4], b4[4], astr[4], bstr[4]; op 0 = add
          if (c.params.size() < 16 || c.params[1] != 0 || c.inputs.size() != 2)
            return fail("BINARY %u: only Add is supported outside the head", i) != 0;
          if (std::memcmp(&c.params[4], &c.params[8], 16) || std::memcmp(&c.params[4], &c.params[12], 16))
            return fail("BINARY %u: broadcasting Add is not supported", i) != 0;
          Parts pa, pb;
          if (!parts_of(c.inputs[0], &pa) || !parts_of(c.inputs[1], &pb)) return false;
          // the residual of the conv producing one operand: Add(x, conv(..)) -> conv epilogue + x
          bool fused = false;
          for (int side = 1; side >= 0 && !fused; --side) {
            const uint32_t cv = c.inputs[side];
            const Parts& other = side ? pa : pb;
            const int oi = m->value_op[cv];
            if (oi < 0 || consumers[cv] != 1) continue;
            Op& op = m->ops[oi];
            // int8 convs take a residual; fp16 ones with SiLU too (the C2f bottleneck)
            const bool res_ok = op.path == kPathInt8 || op.path == kPathInt8Ql ||
                                ((op.path == kPathF16Pack || op.path == kPathF16Nhwc) &&
                                                         e.commands[op.cmd].kind == kConvSilu);
            if (op.kind != kOpConv || !res_ok || op.has_res || other.size() != 1 || other[0].up != 1 ||
                other[0].buf == kInput || other[0].ch != op.oc)
              continue;
            op.has_res = true;
            op.res = other[0];
            op.label += " +residual";
            for (ConvInfo& ci : m->convs)
              if (static_cast<int>(ci.cmd) == op.cmd) ci.fused_residual = true;
            define(c.output, m->vparts[cv]);
            m->value_op[c.output] = oi;
            fused = true;
          }
          if (!fused) {
            if (pa.size() > aexrt::kMaxGraphParts || pb.size() > aexrt::kMaxGraphParts)
              return fail("BINARY %u: too many concatenated parts", i) != 0;
            Op op;
            op.kind = kOpAdd;
            op.cmd = static_cast<int>(i);
            op.a = pa;
            op.b = pb;
            op.c = static_cast<int>(c.params[5]);
            op.out_h = static_cast<int>(c.params[6]);
            op.out_w = static_cast<int>(c.params[7]);
            op.out = new_buffer(op.c, op.out_h, op.out_w);
            op.label = "cmd#" + std::to_string(i) + " BINARY add";
            m->value_op[c.output] = static_cast<int>(m->ops.size());
            m->ops.push_back(op);
            define(c.output, {Part{op.out, 0, op.c, 1}});
          }
          break;
        }
        default:
          return fail("command %u (%s) is outside what this backend runs before the YOLO head", i,
                      kind_name(c.kind)) != 0;
      }
    }
    // ---- the head: decode + filter + NMS + top-k from the three levels' box and class logits
    Op dec;
    dec.kind = kOpDecode;
    dec.cmd = static_cast<int>(hf.final_cmd);
    dec.label = "post:yolo_head_decode";
    uint64_t anchors = 0;
    for (int k = 0; k < 3; ++k) {
      Parts bp, cp;
      if (!parts_of(hf.box[k], &bp) || !parts_of(hf.cls[k], &cp)) return false;
      if (bp.size() != 1 || cp.size() != 1 || bp[0].up != 1 || cp[0].up != 1 || bp[0].buf == kInput ||
          cp[0].buf == kInput)
        return fail("YOLO head level %d: box / class logits are not plain buffers", k) != 0;
      dec.box[k] = bp[0];
      dec.cls[k] = cp[0];
      dec.lh[k] = m->bufs[bp[0].buf].h;
      dec.lw[k] = m->bufs[bp[0].buf].w;
      anchors += uint64_t(dec.lh[k]) * dec.lw[k];
    }
    if (anchors != e.manifest.anchors() || e.manifest.channels() != 4 + e.manifest.classes() ||
        e.manifest.objectness())
      return fail("YOLO head: anchors / channels disagree with the manifest") != 0;
    m->ops.push_back(dec);
    Op nms;
    nms.kind = kOpNms;
    nms.cmd = static_cast<int>(hf.final_cmd);
    nms.label = "post:yolo_nms_topk";
    m->ops.push_back(nms);

    // ---- amax slots: every buffer an int8 conv reads gets them, and its producer fills them
    for (const Op& op : m->ops)
      if (op.kind == kOpConv && (op.path == kPathInt8 || op.path == kPathInt8Ql))
        for (const Part& p : op.in) {
          if (p.buf == kInput) return fail("an int8 conv reads the graph input directly") != 0;
          m->bufs[p.buf].amax = true;
        }
    m->amax_slots = 0;
    for (Buffer& b : m->bufs)
      if (b.amax) {
        b.groups = (b.c + 15) / 16;
        b.amax_off = m->amax_slots;
        m->amax_slots += uint64_t(m->batch) * b.groups;
      }
    // ---- lifetimes over the launch order, then the arena
    for (size_t j = 0; j < m->ops.size(); ++j) {
      const Op& op = m->ops[j];
      auto use = [&](int b) {
        if (b < 0) return;
        Buffer& x = m->bufs[b];
        if (x.first < 0) x.first = static_cast<int>(j);
        x.last = std::max(x.last, static_cast<int>(j));
      };
      for (const Part& p : op.in) use(p.buf);
      for (const Part& p : op.a) use(p.buf);
      for (const Part& p : op.b) use(p.buf);
      if (op.has_res) use(op.res.buf);
      if (op.kind == kOpSppf) use(op.x.buf);
      if (op.kind == kOpDecode)
        for (int k = 0; k < 3; ++k) {
          use(op.box[k].buf);
          use(op.cls[k].buf);
        }
      use(op.out);
      use(op.q);
      use(op.rec);
      use(op.x8);
    }
    std::vector<uint64_t> bytes, offs(m->bufs.size());
    std::vector<uint32_t> first, last;
    for (size_t b = 0; b < m->bufs.size(); ++b) {
      const Buffer& x = m->bufs[b];
      bytes.push_back(x.bytes);
      first.push_back(m->reuse ? static_cast<uint32_t>(std::max(0, x.first)) : 0u);
      last.push_back(m->reuse ? static_cast<uint32_t>(std::max(0, x.last)) : 0xFFFFFFFFu);
    }
    uint64_t total = 0;
    if (!aexrt_b200_arena_plan(static_cast<uint32_t>(bytes.size()), bytes.data(), first.data(), last.data(), 256,
                               offs.data(), &total))
      return fail("arena planning failed: %s", aexrt_b200_get_last_error()) != 0;
    for (size_t b = 0; b < m->bufs.size(); ++b) m->bufs[b].off = offs[b];
    m->arena_bytes = total;
    return true;
  }
};

// ------------------------------------------------------------------ device state

void free_lowered(AexrtYoloModel* m) {
  if (m->graph) cudaGraphExecDestroy(m->graph);
  m->graph = nullptr;
  for (Op& op : m->ops)
    if (op.plan) aexrt_b200_conv_plan_destroy(op.plan);
  m->ops.clear();
  m->bufs.clear();
  m->convs.clear();
}

__half* buf_ptr(AexrtYoloModel* m, int b) {
  return reinterpret_cast<__half*>(static_cast<uint8_t*>(m->d_arena) + m->bufs[b].off);
}

void fill_source(AexrtYoloModel* m, const Part& p, bool amax, AexrtB200ActSource* s) {
  std::memset(s, 0, sizeof(*s));
  if (p.buf == kInput) {
    s->ptr = m->d_input;
    s->layout = m->input_dtype == 1 ? AEXRT_B200_LAYOUT_NCHW_F16 : AEXRT_B200_LAYOUT_NCHW_F32;
    s->ldc = static_cast<uint32_t>(m->channels_in);
    s->src_h = static_cast<uint32_t>(m->img_h);
    s->src_w = static_cast<uint32_t>(m->img_w);
  } else {
    const Buffer& b = m->bufs[p.buf];
    s->ptr = buf_ptr(m, p.buf);
    s->layout = AEXRT_B200_LAYOUT_NHWC_F16;
    s->ldc = static_cast<uint32_t>(b.c);
    s->src_h = static_cast<uint32_t>(b.h);
    s->src_w = static_cast<uint32_t>(b.w);
    if (amax) {
      s->amax_groups = m->d_amax + b.amax_off;
      s->amax_stride = static_cast<uint32_t>(b.groups);
      s->amax_goff = static_cast<uint32_t>(p.coff / 16);
    }
  }
  s->coff = static_cast<uint32_t>(p.coff);
  s->channels = static_cast<uint32_t>(p.ch);
  s->upsample = static_cast<uint32_t>(p.up);
}

aexrt::GraphParts graph_parts(AexrtYoloModel* m, const Parts& ps) {
  aexrt::GraphParts g{};
  g.nparts = static_cast<int>(ps.size());
  for (size_t i = 0; i < ps.size(); ++i) {
    const Buffer& b = m->bufs[ps[i].buf];
    g.ptr[i] = buf_ptr(m, ps[i].buf);
    g.ldc[i] = b.c;
    g.coff[i] = ps[i].coff;
    g.ch[i] = ps[i].ch;
    g.up[i] = ps[i].up;
    g.h[i] = b.h;
    g.w[i] = b.w;
  }
  return g;
}

uint32_t* amax_of(AexrtYoloModel* m, int b, int* stride) {
  if (b < 0 || !m->bufs[b].amax) {
    *stride = 0;
    return nullptr;
  }
  *stride = m->bufs[b].groups;
  return m->d_amax + m->bufs[b].amax_off;
}

// Issues one forward on `st`; with `events` (profiling) records a pair around every op.
bool launch_forward(AexrtYoloModel* m, cudaStream_t st, std::vector<std::pair<cudaEvent_t, cudaEvent_t>>* events) {
  void* sv = static_cast<void*>(st);
  const uint32_t n = m->batch;
  if (m->amax_slots && !aexrt_b200_zero(m->d_amax, m->amax_slots * 4, sv))
    return set_error(&m->error, "amax clear: %s", aexrt_b200_get_last_error()) != 0;
  for (size_t j = 0; j < m->ops.size(); ++j) {
    Op& op = m->ops[j];
    if (events) cudaEventRecord((*events)[j].first, st);
    int ok = 1;
    switch (op.kind) {
      case kOpConv: {
        int astride = 0;
        uint32_t* am = amax_of(m, op.out, &astride);
        __half* out = buf_ptr(m, op.out);
        const uint32_t ldc = static_cast<uint32_t>(op.oc);
        if (op.path == kPathInt8) {
          AexrtB200ActSource src[aexrt::kMaxGraphParts];
          if (op.in.size() > aexrt::kMaxGraphParts) return set_error(&m->error, "too many conv input parts") != 0;
          for (size_t i = 0; i < op.in.size(); ++i) fill_source(m, op.in[i], true, &src[i]);
          void* q = buf_ptr(m, op.q);
          float* rec = reinterpret_cast<float*>(buf_ptr(m, op.rec));
          ok = aexrt_b200_act_quantize_concat(src, static_cast<uint32_t>(op.in.size()), n, op.in_h, op.in_w,
                                              op.pg16 ? 1u : 0u, op.s, q, rec, sv);
          if (ok) {
            const void* res = op.has_res ? static_cast<const void*>(buf_ptr(m, op.res.buf)) : nullptr;
            const uint32_t res_ldc = op.has_res ? static_cast<uint32_t>(m->bufs[op.res.buf].c) : 0u;
            ok = aexrt_b200_conv_w8a8(op.plan, q, rec, res, res_ldc, op.has_res ? op.res.coff : 0, out, ldc, 0, am,
                                      astride, 0, nullptr, sv);
          }
        } else if (op.path == kPathInt8Ql) {
          AexrtB200ActSource src[aexrt::kMaxGraphParts];
          for (size_t i = 0; i < op.in.size(); ++i) fill_source(m, op.in[i], true, &src[i]);
          const void* res = op.has_res ? static_cast<const void*>(buf_ptr(m, op.res.buf)) : nullptr;
          const uint32_t res_ldc = op.has_res ? static_cast<uint32_t>(m->bufs[op.res.buf].c) : 0u;
          ok = aexrt_b200_conv_w8a8_sources(op.plan, src, static_cast<uint32_t>(op.in.size()), res, res_ldc,
                                            op.has_res ? op.res.coff : 0, out, ldc, 0, am, astride, 0, nullptr, sv);
        } else if (op.path == kPathStem) {
          ok = aexrt_b200_conv_f16_image(op.plan, m->d_input,
                                         m->input_dtype == 1 ? AEXRT_B200_LAYOUT_NCHW_F16 : AEXRT_B200_LAYOUT_NCHW_F32,
                                         out, ldc, 0, am, astride, 0, sv);
        } else if (op.path == kPathF16Nhwc) {
          const Part& p = op.in[0];
          const void* res = op.has_res ? static_cast<const void*>(buf_ptr(m, op.res.buf)) : nullptr;
          const uint32_t res_ldc = op.has_res ? static_cast<uint32_t>(m->bufs[op.res.buf].c) : 0u;
          ok = aexrt_b200_conv_f16_nhwc(op.plan, buf_ptr(m, p.buf), m->bufs[p.buf].c, p.coff, res, res_ldc,
                                        op.has_res ? op.res.coff : 0, out, ldc, 0, am, astride, 0, sv);
        } else {
          AexrtB200ActSource src[aexrt::kMaxGraphParts];
          if (op.in.size() > aexrt::kMaxGraphParts) return set_error(&m->error, "too many conv input parts") != 0;
          for (size_t i = 0; i < op.in.size(); ++i) fill_source(m, op.in[i], false, &src[i]);
          void* x8 = buf_ptr(m, op.x8);
          ok = aexrt_b200_pack_f16_concat(src, static_cast<uint32_t>(op.in.size()), n, op.in_h, op.in_w, op.s, x8, sv);
          const void* res = op.has_res ? static_cast<const void*>(buf_ptr(m, op.res.buf)) : nullptr;
          const uint32_t res_ldc = op.has_res ? static_cast<uint32_t>(m->bufs[op.res.buf].c) : 0u;
          if (ok)
            ok = aexrt_b200_conv_f16(op.plan, x8, res, res_ldc, op.has_res ? op.res.coff : 0, out, ldc, 0, am, astride,
                                     0, sv);
        }
        break;
      }
      case kOpSppf: {
        int astride = 0;
        uint32_t* am = amax_of(m, op.out, &astride);
        const Buffer& xb = m->bufs[op.x.buf];
        ok = aexrt_b200_sppf_pool(buf_ptr(m, op.x.buf), n, xb.h, xb.w, op.c, xb.c, op.x.coff, buf_ptr(m, op.out),
                                  3 * op.c, 0, am, astride, 0, sv);
        break;
      }
      case kOpMaxPool: {
        int astride = 0;
        uint32_t* am = amax_of(m, op.out, &astride);
        const long total = long(n) * op.out_h * op.out_w * op.c;
        aexrt::launch_kernel(aexrt::maxpool_nhwc_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256),
            0, st,
            graph_parts(m, op.a), n, op.in_h, op.in_w, op.c, op.pool_k, op.pool_s, op.pool_p, op.out_h, op.out_w,
            buf_ptr(m, op.out), op.c, am, astride);
        ok = cudaGetLastError() == cudaSuccess;
        break;
      }
      case kOpAdd: {
        int astride = 0;
        uint32_t* am = amax_of(m, op.out, &astride);
        const long total = long(n) * op.out_h * op.out_w * op.c;
        aexrt::launch_kernel(aexrt::add_nhwc_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0,
            st,
            graph_parts(m, op.a), graph_parts(m, op.b), n, op.out_h, op.out_w, op.c, buf_ptr(m, op.out), op.c, am,
            astride);
        ok = cudaGetLastError() == cudaSuccess;
        break;
      }
      case kOpDecode: {
        AexrtB200DecodeLevel lv[3];
        for (int k = 0; k < 3; ++k) {
          lv[k].box = buf_ptr(m, op.box[k].buf);
          lv[k].box_ldc = static_cast<uint32_t>(m->bufs[op.box[k].buf].c);
          lv[k].box_coff = static_cast<uint32_t>(op.box[k].coff);
          lv[k].cls = buf_ptr(m, op.cls[k].buf);
          lv[k].cls_ldc = static_cast<uint32_t>(m->bufs[op.cls[k].buf].c);
          lv[k].cls_coff = static_cast<uint32_t>(op.cls[k].coff);
          lv[k].h = static_cast<uint32_t>(op.lh[k]);
          lv[k].w = static_cast<uint32_t>(op.lw[k]);
          // the reference's head strides: input height / level height (runtime.cpp:27277-27283)
          lv[k].stride = static_cast<float>(m->img_h) / static_cast<float>(std::max(1, op.lh[k]));
        }
        ok = aexrt_b200_yolo_decode(lv, 3, n, m->eng.manifest.classes(), 16, m->d_output0, sv);
        break;
      }
      case kOpNms: {
        const Manifest& mf = m->eng.manifest;
        uint32_t* counts = reinterpret_cast<uint32_t*>(m->d_dets);
        auto* rows = reinterpret_cast<AexrtYoloDetection*>(m->d_dets + 4 * n);
        ok = aexrt_b200_yolo_nms_topk(m->d_output0, n, mf.channels(), mf.anchors(), mf.classes(), 0, 1, mf.conf,
                                      mf.iou, std::min<uint32_t>(mf.max_candidates(), AEXRT_B200_NMS_MAX_CANDIDATES),
                                      mf.max_detections(), AEXRT_B200_NMS_MARK, rows, counts, sv);
        break;
      }
    }
    if (!ok) return set_error(&m->error, "%s: %s", op.label.c_str(), aexrt_b200_get_last_error()) != 0;
    if (events) cudaEventRecord((*events)[j].second, st);
  }
  return true;
}

uint32_t count_launches(const AexrtYoloModel* m) {
  uint32_t k = m->amax_slots ? 1 : 0;
  for (const Op& op : m->ops)
    k += (op.kind == kOpConv && (op.path == kPathInt8 || op.path == kPathF16Pack)) ? 2 : 1;
  return k;
}

template <typename T>
bool ensure_alloc(T** p, uint64_t* cap, uint64_t want, std::string* err) {
  if (*cap >= want && *p) return true;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (!cuda_ok(cudaMalloc(reinterpret_cast<void**>(p), std::max<uint64_t>(want, 256)), "cudaMalloc(arena)", err))
    return false;
  *cap = want;
  return true;
}

// (Re)builds the lowered model: plans, arena, CUDA graph.  Allocates device memory.
bool prepare(AexrtYoloModel* m) {
  if (!m->dirty && m->graph) return true;
  cudaSetDevice(m->dev->cuda_device);
  free_lowered(m);
  Lowering low(m);
  if (!low.run()) {
    free_lowered(m);
    return false;
  }
  if (!ensure_alloc(&m->d_arena, &m->d_arena_cap, m->arena_bytes, &m->error) ||
      !ensure_alloc(&m->d_amax, &m->d_amax_cap, m->amax_slots * 4, &m->error))
    return false;
  const Manifest& mf = m->eng.manifest;
  const uint64_t in_elems = uint64_t(m->batch) * m->channels_in * m->img_h * m->img_w;
  const uint64_t in_bytes = in_elems * (m->input_dtype == 1 ? 2 : 4);
  if (in_bytes != m->input_bytes) {
    if (m->d_input) cudaFree(m->d_input);
    if (m->h_input) cudaFreeHost(m->h_input);
    m->d_input = m->h_input = nullptr;
    if (!cuda_ok(cudaMalloc(&m->d_input, in_bytes), "cudaMalloc(input)", &m->error) ||
        !cuda_ok(cudaMallocHost(&m->h_input, in_bytes), "cudaMallocHost(input)", &m->error))
      return false;
    m->input_bytes = in_bytes;
  }
  if (!m->d_output0) {
    const uint64_t ob = uint64_t(m->batch) * mf.channels() * mf.anchors() * 4;
    m->dets_bytes = uint64_t(m->batch) * 4 + uint64_t(m->batch) * mf.max_detections() * sizeof(AexrtYoloDetection);
    if (!cuda_ok(cudaMalloc(reinterpret_cast<void**>(&m->d_output0), ob), "cudaMalloc(output0)", &m->error) ||
        !cuda_ok(cudaMalloc(reinterpret_cast<void**>(&m->d_dets), m->dets_bytes), "cudaMalloc(detections)", &m->error) ||
        !cuda_ok(cudaMallocHost(reinterpret_cast<void**>(&m->h_dets), m->dets_bytes), "cudaMallocHost(detections)",
                 &m->error))
      return false;
    cudaMemset(m->d_dets, 0, m->dets_bytes);
  }
  m->launches = count_launches(m);
  // one eager forward first (it also prepares per-device attributes outside capture), then capture
  cudaStream_t st = m->dev->stream;
  if (!launch_forward(m, st, nullptr)) return false;
  if (!cuda_ok(cudaStreamSynchronize(st), "warm-up forward", &m->error)) return false;
  cudaGraph_t g = nullptr;
  if (!cuda_ok(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "begin capture", &m->error)) return false;
  // one image per run (the reference's aexrt_yolo_run): every kernel of the graph is launched with
  // programmatic dependent launch, so its launch and set-up overlap the kernel before it (launch.cuh)
  const uint32_t prev_flags = aexrt_b200_get_launch_flags();
  aexrt_b200_set_launch_flags(m->batch == 1 ? AEXRT_B200_LAUNCH_PROGRAMMATIC : 0u);
  const bool ok = launch_forward(m, st, nullptr);
  aexrt_b200_set_launch_flags(prev_flags);
  const cudaError_t ce = cudaStreamEndCapture(st, &g);
  if (!ok || !cuda_ok(ce, "end capture", &m->error)) {
    if (g) cudaGraphDestroy(g);
    return false;
  }
  const cudaError_t ie = cudaGraphInstantiate(&m->graph, g, 0);
  cudaGraphDestroy(g);
  if (!cuda_ok(ie, "graph instantiate", &m->error)) return false;
  m->dirty = false;
  return true;
}

bool forward(AexrtYoloModel* m, cudaStream_t st) {
  if (!prepare(m)) return false;
  if (m->profiling) {
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev(m->ops.size());
    for (auto& e : ev) {
      cudaEventCreate(&e.first);
      cudaEventCreate(&e.second);
    }
    const bool ok = launch_forward(m, st, &ev) && cuda_ok(cudaStreamSynchronize(st), "profiled forward", &m->error);
    m->prof_labels.clear();
    m->prof_ms.clear();
    for (size_t j = 0; ok && j < m->ops.size(); ++j) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[j].first, ev[j].second);
      m->prof_labels.push_back(m->ops[j].label);
      m->prof_ms.push_back(ms);
    }
    for (auto& e : ev) {
      cudaEventDestroy(e.first);
      cudaEventDestroy(e.second);
    }
    return ok;
  }
  return cuda_ok(cudaGraphLaunch(m->graph, st), "graph launch", &m->error);
}

double ms_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

AexrtYoloModel* load(AexrtDevice* dev, const char* path, uint32_t images) {
  if (!dev || !path) {
    set_error(nullptr, "null device or path");
    return nullptr;
  }
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    set_error(nullptr, "cannot open %s", path);
    return nullptr;
  }
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  auto m = std::make_unique<AexrtYoloModel>();
  std::string err;
  if (!aexrt::engine::parse(bytes.data(), bytes.size(), &m->eng, &err)) {
    set_error(nullptr, "%s: %s", path, err.c_str());
    return nullptr;
  }
  m->dev = dev;
  const uint32_t gb = m->eng.values[m->eng.manifest.input_value()].shape[0];
  m->batch = images ? images : gb;
  const char* prof = std::getenv("AEXRT_NATIVE_D3D12_PROFILE_REPLAY");
  m->profiling = prof && prof[0] && prof[0] != '0';
  std::lock_guard<std::mutex> lock(dev->mu);
  if (!prepare(m.get())) {
    set_error(nullptr, "%s: %s", path, m->error.c_str());
    AexrtYoloModel* raw = m.release();
    aexrt_yolo_destroy(raw);
    return nullptr;
  }
  return m.release();
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ arena planner

int aexrt_b200_arena_plan(uint32_t count, const uint64_t* bytes, const uint32_t* first, const uint32_t* last,
                          uint64_t alignment, uint64_t* offsets, uint64_t* total) {
  if ((count && (!bytes || !first || !last || !offsets)) || !total) return set_error(nullptr, "null pointer");
  if (alignment == 0 || (alignment & (alignment - 1))) return set_error(nullptr, "alignment must be a power of two");
  for (uint32_t i = 0; i < count; ++i)
    if (first[i] > last[i]) return set_error(nullptr, "item %u: first launch after last", i);
  // largest first; each item takes the lowest aligned offset that overlaps in memory no placed item
  // whose lifetime overlaps its own
  std::vector<uint32_t> order(count);
  for (uint32_t i = 0; i < count; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
    return bytes[a] != bytes[b] ? bytes[a] > bytes[b] : first[a] < first[b];
  });
  std::vector<uint32_t> placed;
  uint64_t end = 0;
  auto al = [&](uint64_t v) { return (v + alignment - 1) & ~(alignment - 1); };
  for (uint32_t i : order) {
    std::vector<std::pair<uint64_t, uint64_t>> busy;
    for (uint32_t j : placed)
      if (!(last[j] < first[i] || last[i] < first[j]) && bytes[j]) busy.push_back({offsets[j], offsets[j] + bytes[j]});
    std::sort(busy.begin(), busy.end());
    uint64_t off = 0;
    for (const auto& r : busy) {
      if (off + bytes[i] <= r.first) break;
      off = std::max(off, al(r.second));
    }
    offsets[i] = off;
    end = std::max(end, al(off + bytes[i]));
    placed.push_back(i);
  }
  *total = end;
  return 1;
}

int aexrt_b200_engine_validate(const void* data, uint64_t size) {
  aexrt::engine::Engine e;
  std::string err;
  if (!aexrt::engine::parse(static_cast<const uint8_t*>(data), static_cast<size_t>(size), &e, &err))
    return set_error(nullptr, "%s", err.c_str());
  return 1;
}

// ------------------------------------------------------------------ device

int aexrt_d3d12_probe(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n > 0 ? 1 : 0;
}

AexrtDevice* aexrt_cuda_create_device(uint32_t index) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || static_cast<int>(index) >= n) {
    cudaGetLastError();
    set_error(nullptr, "CUDA device %u not present (%d visible)", index, n);
    return nullptr;
  }
  auto* d = new AexrtDevice();
  d->cuda_device = static_cast<int>(index);
  if (!cuda_ok(cudaSetDevice(d->cuda_device), "cudaSetDevice") ||
      !cuda_ok(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate")) {
    delete d;
    return nullptr;
  }
  return d;
}

AexrtDevice* aexrt_d3d12_create_device(uint32_t adapter_index) { return aexrt_cuda_create_device(adapter_index); }

int aexrt_d3d12_get_capabilities(AexrtDevice* device, AexrtD3D12Capabilities* caps) {
  if (!device || !caps) return set_error(nullptr, "null pointer");
  AexrtD3D12Capabilities c{};
  c.struct_size = sizeof(c);
  c.native_fp16_supported = 1;
  *caps = c;
  return 1;
}

void aexrt_d3d12_destroy_device(AexrtDevice* device) {
  if (!device) return;
  cudaSetDevice(device->cuda_device);
  if (device->stream) cudaStreamDestroy(device->stream);
  delete device;
}

// ------------------------------------------------------------------ model

AexrtYoloModel* aexrt_yolo_load_engine(AexrtDevice* device, const char* path) { return load(device, path, 0); }

AexrtYoloModel* aexrt_b200_yolo_load_engine_batch(AexrtDevice* device, const char* path, uint32_t images) {
  if (images == 0) {
    set_error(nullptr, "images must be >= 1");
    return nullptr;
  }
  return load(device, path, images);
}

AexrtYoloModel* aexrt_yolo_compile_from_package(AexrtDevice*, const char* path) {
  set_error(nullptr, "%s: JSON YOLO packages are the D3D12 compiler's intermediate form; compile them to .aexrt "
                     "(aexrtc build) and load that", path ? path : "(null)");
  return nullptr;
}

AexrtYoloModel* aexrt_yolo_compile_from_onnx(AexrtDevice*, const char* path) {
  set_error(nullptr, "%s: ONNX import needs the reference compiler (aexrtc build model.onnx) and the onnx package; "
                     "load the resulting .aexrt", path ? path : "(null)");
  return nullptr;
}

void aexrt_yolo_destroy(AexrtYoloModel* m) {
  if (!m) return;
  if (m->dev) cudaSetDevice(m->dev->cuda_device);
  free_lowered(m);
  if (m->d_arena) cudaFree(m->d_arena);
  if (m->d_amax) cudaFree(m->d_amax);
  if (m->d_input) cudaFree(m->d_input);
  if (m->h_input) cudaFreeHost(m->h_input);
  if (m->d_output0) cudaFree(m->d_output0);
  if (m->d_dets) cudaFree(m->d_dets);
  if (m->h_dets) cudaFreeHost(m->h_dets);
  delete m;
}

#define AEXRT_MODEL_GETTER(name, expr) \
  uint32_t name(AexrtYoloModel* m) { return m ? static_cast<uint32_t>(expr) : 0u; }
AEXRT_MODEL_GETTER(aexrt_yolo_class_count, m->eng.manifest.classes())
AEXRT_MODEL_GETTER(aexrt_yolo_anchor_count, m->eng.manifest.anchors())
AEXRT_MODEL_GETTER(aexrt_yolo_channel_count, m->eng.manifest.channels())
AEXRT_MODEL_GETTER(aexrt_yolo_output_layout, m->eng.manifest.output_layout())
AEXRT_MODEL_GETTER(aexrt_yolo_has_objectness, m->eng.manifest.objectness())
AEXRT_MODEL_GETTER(aexrt_yolo_package_mode, 2u)
AEXRT_MODEL_GETTER(aexrt_yolo_graph_node_count, m->eng.manifest.nodes())
AEXRT_MODEL_GETTER(aexrt_yolo_graph_value_count, m->eng.manifest.value_count())
AEXRT_MODEL_GETTER(aexrt_yolo_constant_count, m->eng.manifest.constant_count())
AEXRT_MODEL_GETTER(aexrt_yolo_prepared_command_count, m->eng.manifest.command_count())
AEXRT_MODEL_GETTER(aexrt_yolo_supported_prepared_command_count, m->eng.manifest.command_count())
AEXRT_MODEL_GETTER(aexrt_yolo_unsupported_prepared_command_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_prepared_skipped_command_count, m->skipped)
AEXRT_MODEL_GETTER(aexrt_yolo_head_fusion_enabled, m->head_fusion ? 1u : 0u)
AEXRT_MODEL_GETTER(aexrt_b200_yolo_batch, m->batch)
AEXRT_MODEL_GETTER(aexrt_b200_yolo_launch_count, m->launches)
// D3D12 kernel families and fusions that do not exist on this backend
AEXRT_MODEL_GETTER(aexrt_yolo_late_concat_conv1x1_fusion_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_concat_residual_conv1x1_fusion_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_paired_conv3x3_fusion_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_c2f_bottleneck_superblock_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_head_final_conv_fusion_enabled, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_spatial_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_conv1x1_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_pack4_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_pack8_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_implicit_gemm_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_implicit_gemm_40x40_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_implicit_gemm_20x20_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_implicit_gemm_10x10_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_exact_40x40_64x64_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_exact_20x20_64x64_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_exact_10x10_128x128_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_exact_20x20_128x64_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_3x3_exact_10x10_256x64_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_tileflow_native_fp16_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_dxil_cache_hit_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_shader_cache_hit_count, 0u)
AEXRT_MODEL_GETTER(aexrt_yolo_pso_cache_hit_count, 0u)
#undef AEXRT_MODEL_GETTER

uint32_t aexrt_yolo_c2f_tail_residual_fusion_count(AexrtYoloModel* m) {
  if (!m) return 0;
  uint32_t k = 0;
  for (const ConvInfo& c : m->convs) k += c.fused_residual ? 1 : 0;
  return k;
}

uint64_t aexrt_yolo_input_element_count(AexrtYoloModel* m) {
  return m ? uint64_t(m->batch) * m->channels_in * m->img_h * m->img_w : 0;
}

uint64_t aexrt_b200_yolo_arena_bytes(AexrtYoloModel* m) { return m ? m->arena_bytes + m->amax_slots * 4 : 0; }

int aexrt_yolo_is_executable(AexrtYoloModel* m) { return m && !m->ops.empty() ? 1 : 0; }

const char* aexrt_yolo_get_last_error(AexrtYoloModel* m) { return m ? m->error.c_str() : aexrt_b200_get_last_error(); }

void* aexrt_yolo_input_ptr(AexrtYoloModel* m, uint64_t* out_elements) {
  if (!m) return nullptr;
  if (out_elements) *out_elements = aexrt_yolo_input_element_count(m);
  return m->h_input;
}

int aexrt_b200_yolo_set_input_dtype(AexrtYoloModel* m, uint32_t dtype) {
  if (!m) return set_error(nullptr, "null model");
  if (dtype > 1) return set_error(&m->error, "input dtype must be 0 (fp32) or 1 (fp16)");
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->input_dtype != dtype) {
    m->input_dtype = dtype;
    m->dirty = true;
    std::lock_guard<std::mutex> dlock(m->dev->mu);
    if (!prepare(m)) return 0;
  }
  return 1;
}

void* aexrt_b200_yolo_device_input(AexrtYoloModel* m) { return m ? m->d_input : nullptr; }
void* aexrt_b200_yolo_device_output0(AexrtYoloModel* m) { return m ? m->d_output0 : nullptr; }

void* aexrt_b200_yolo_device_detections(AexrtYoloModel* m, uint64_t* out_bytes) {
  if (!m) return nullptr;
  if (out_bytes) *out_bytes = m->dets_bytes;
  return m->d_dets;
}

int aexrt_b200_yolo_enqueue(AexrtYoloModel* m, void* stream) {
  if (!m) return set_error(nullptr, "null model");
  std::lock_guard<std::mutex> lock(m->mu);
  std::lock_guard<std::mutex> dlock(m->dev->mu);
  cudaSetDevice(m->dev->cuda_device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->dev->stream;
  if (!forward(m, st)) {
    aexrt::set_last_error(m->error.c_str());
    return 0;
  }
  return 1;
}

int aexrt_b200_yolo_run_batch(AexrtYoloModel* m, const void* images, uint32_t dtype, AexrtYoloDetection* dets,
                              uint32_t max_det, uint32_t* counts) {
  if (!m || !images || (!dets && max_det) || !counts) return set_error(m ? &m->error : nullptr, "null pointer");
  std::lock_guard<std::mutex> lock(m->mu);
  cudaSetDevice(m->dev->cuda_device);
  if (dtype > 1) return set_error(&m->error, "input dtype must be 0 (fp32) or 1 (fp16)");
  if (dtype != m->input_dtype) {
    m->input_dtype = dtype;
    m->dirty = true;
  }
  std::lock_guard<std::mutex> dlock(m->dev->mu);
  if (!prepare(m)) return 0;
  cudaStream_t st = m->dev->stream;
  AexrtYoloRunTiming t{};
  t.struct_size = sizeof(t);
  auto t0 = std::chrono::steady_clock::now();
  const void* src = images;
  if (images != m->h_input) {
    std::memcpy(m->h_input, images, m->input_bytes);
    t.memcpy_ms = ms_since(t0);
  }
  src = m->h_input;
  auto t1 = std::chrono::steady_clock::now();
  if (!cuda_ok(cudaMemcpyAsync(m->d_input, src, m->input_bytes, cudaMemcpyHostToDevice, st), "input upload", &m->error) ||
      !forward(m, st) ||
      !cuda_ok(cudaMemcpyAsync(m->h_dets, m->d_dets, m->dets_bytes, cudaMemcpyDeviceToHost, st), "read-back", &m->error))
    return 0;
  t.submit_ms = ms_since(t1);
  auto t2 = std::chrono::steady_clock::now();
  if (!cuda_ok(cudaStreamSynchronize(st), "run", &m->error)) return 0;
  t.fence_ms = ms_since(t2);
  auto t3 = std::chrono::steady_clock::now();
  const uint32_t md = m->eng.manifest.max_detections();
  const uint32_t* hc = reinterpret_cast<const uint32_t*>(m->h_dets);
  const auto* rows = reinterpret_cast<const AexrtYoloDetection*>(m->h_dets + 4 * m->batch);
  for (uint32_t i = 0; i < m->batch; ++i) {
    const uint32_t c = std::min(hc[i], max_det);
    counts[i] = c;
    if (c) std::memcpy(dets + size_t(i) * max_det, rows + size_t(i) * md, c * sizeof(AexrtYoloDetection));
  }
  t.readback_ms = ms_since(t3);
  t.valid = 1;
  m->timing = t;
  return 1;
}

int aexrt_yolo_run(AexrtDevice* device, AexrtYoloModel* m, const float* input, uint64_t elements,
                   AexrtYoloDetection* dets, uint32_t max_det, uint32_t* out_count) {
  if (!m) return set_error(nullptr, "null model");
  if (device && device != m->dev) return set_error(&m->error, "the model belongs to another device");
  if (!input || !out_count || (!dets && max_det)) return set_error(&m->error, "null pointer");
  if (m->batch != 1) return set_error(&m->error, "aexrt_yolo_run takes one image; this model runs %u (use "
                                                 "aexrt_b200_yolo_run_batch)", m->batch);
  if (elements != aexrt_yolo_input_element_count(m))
    return set_error(&m->error, "expected %llu input elements, got %llu",
                     static_cast<unsigned long long>(aexrt_yolo_input_element_count(m)),
                     static_cast<unsigned long long>(elements));
  std::vector<AexrtYoloDetection> tmp(std::max<uint32_t>(max_det, 1));
  uint32_t count = 0;
  if (!aexrt_b200_yolo_run_batch(m, input, 0, tmp.data(), max_det, &count)) return 0;
  if (count) std::memcpy(dets, tmp.data(), count * sizeof(AexrtYoloDetection));
  *out_count = count;
  return 1;
}

int aexrt_yolo_flush_pipeline(AexrtYoloModel* m, AexrtYoloDetection*, uint32_t, uint32_t* out_count) {
  if (!m || !out_count) return set_error(m ? &m->error : nullptr, "null pointer");
  *out_count = 0;
  return 1;
}

int aexrt_yolo_get_last_run_timing(AexrtYoloModel* m, AexrtYoloRunTiming* timing) {
  if (!m || !timing) return set_error(m ? &m->error : nullptr, "null pointer");
  if (timing->struct_size && timing->struct_size < sizeof(AexrtYoloRunTiming))
    return set_error(&m->error, "timing struct too small");
  *timing = m->timing;
  return 1;
}

uint32_t aexrt_yolo_profile_event_count(AexrtYoloModel* m) { return m ? static_cast<uint32_t>(m->prof_ms.size()) : 0; }

const char* aexrt_yolo_profile_event_label(AexrtYoloModel* m, uint32_t i) {
  return m && i < m->prof_labels.size() ? m->prof_labels[i].c_str() : nullptr;
}

double aexrt_yolo_profile_event_ms(AexrtYoloModel* m, uint32_t i) {
  return m && i < m->prof_ms.size() ? m->prof_ms[i] : 0.0;
}

int aexrt_b200_yolo_set_profiling(AexrtYoloModel* m, uint32_t enabled) {
  if (!m) return set_error(nullptr, "null model");
  m->profiling = enabled != 0;
  return 1;
}

int aexrt_b200_yolo_set_quant_on_load(AexrtYoloModel* m, uint32_t enabled) {
  if (!m) return set_error(nullptr, "null model");
  if (m->quant_on_load != (enabled != 0)) {
    m->quant_on_load = enabled != 0;
    m->dirty = true;
  }
  return 1;
}

int aexrt_b200_yolo_set_arena_reuse(AexrtYoloModel* m, uint32_t enabled) {
  if (!m) return set_error(nullptr, "null model");
  if (m->reuse != (enabled != 0)) {
    m->reuse = enabled != 0;
    m->dirty = true;
  }
  return 1;
}

uint32_t aexrt_yolo_conv_plan_count(AexrtYoloModel* m) { return m ? static_cast<uint32_t>(m->convs.size()) : 0; }

int aexrt_yolo_conv_plan_info(AexrtYoloModel* m, uint32_t index, AexrtConvPlanInfo* out) {
  if (!m || !out) return set_error(m ? &m->error : nullptr, "null pointer");
  if (index >= m->convs.size()) return set_error(&m->error, "conv plan index %u out of range", index);
  const ConvInfo& c = m->convs[index];
  AexrtConvPlanInfo i{};
  i.struct_size = sizeof(i);
  i.command_index = c.cmd;
  i.kind_is_silu = c.silu ? 1 : 0;
  i.desc = c.desc;
  i.current_algorithm = c.current;
  i.candidate_count = static_cast<uint32_t>(std::min<size_t>(32, c.candidates.size()));
  for (uint32_t k = 0; k < i.candidate_count; ++k) i.candidates[k] = c.candidates[k];
  i.in_fusion_group = c.fused_residual ? 1 : 0;
  i.planned_algorithm = c.planned;
  *out = i;
  return 1;
}

int aexrt_yolo_override_conv_algorithm(AexrtYoloModel* m, uint32_t cmd, uint32_t alg) {
  if (!m) return set_error(nullptr, "null model");
  for (const ConvInfo& c : m->convs) {
    if (c.cmd != cmd) continue;
    if (alg != c.planned && std::find(c.candidates.begin(), c.candidates.end(), alg) == c.candidates.end())
      return set_error(&m->error, "algorithm %u is not a candidate of command %u", alg, cmd);
    m->overrides[cmd] = alg;
    m->dirty = true;
    return 1;
  }
  return set_error(&m->error, "command %u is not a conv of this engine", cmd);
}

int aexrt_b200_yolo_override_conv_variant(AexrtYoloModel* m, uint32_t cmd, uint32_t bits) {
  if (!m) return set_error(nullptr, "null model");
  for (const ConvInfo& c : m->convs)
    if (c.cmd == cmd) {
      m->variants[cmd] = bits;
      m->dirty = true;
      return 1;
    }
  return set_error(&m->error, "command %u is not a conv of this engine", cmd);
}

int aexrt_b200_yolo_status(AexrtYoloModel* m, uint32_t* status) {
  if (!m || !status) return set_error(m ? &m->error : nullptr, "null pointer");
  uint32_t st = 0;
  for (const Op& op : m->ops) {
    if (!op.plan) continue;
    uint32_t v = 0;
    if (!aexrt_b200_conv_status(op.plan, &v)) return set_error(&m->error, "%s", aexrt_b200_get_last_error());
    st |= v;
  }
  *status = st;
  return 1;
}

uint64_t aexrt_yolo_pipeline_cache_size(AexrtYoloModel*) { return 0; }

int aexrt_yolo_export_pipeline_cache(AexrtYoloModel* m, void*, uint64_t) {
  return set_error(m ? &m->error : nullptr, "no pipeline cache: the kernels are compiled ahead of time");
}

int aexrt_yolo_debug_output(AexrtYoloModel* m, float* out, uint64_t elements) {
  return aexrt_yolo_debug_value(m, 0xFFFFFFFFu, out, elements);
}

int aexrt_yolo_debug_value(AexrtYoloModel* m, uint32_t value, float* out, uint64_t elements) {
  if (!m || !out) return set_error(m ? &m->error : nullptr, "null pointer");
  std::lock_guard<std::mutex> lock(m->mu);
  cudaSetDevice(m->dev->cuda_device);
  if (!cuda_ok(cudaStreamSynchronize(m->dev->stream), "sync", &m->error)) return 0;
  const Manifest& mf = m->eng.manifest;
  if (value == 0xFFFFFFFFu || value == mf.output_value()) {
    const uint64_t n = uint64_t(m->batch) * mf.channels() * mf.anchors();
    if (elements != n) return set_error(&m->error, "output0 holds %llu elements", static_cast<unsigned long long>(n));
    return cuda_ok(cudaMemcpy(out, m->d_output0, n * 4, cudaMemcpyDeviceToHost), "read output0", &m->error) ? 1 : 0;
  }
  if (value >= m->vparts.size() || !m->vdefined[value])
    return set_error(&m->error, "value %u has no device storage on this backend", value);
  const Value& v = m->eng.values[value];
  const uint64_t n = uint64_t(m->batch) / m->graph_batch * v.elements;
  if (elements != n) return set_error(&m->error, "value %u holds %llu elements", value, static_cast<unsigned long long>(n));
  const Parts& ps = m->vparts[value];
  const int H = static_cast<int>(v.shape[2]), W = static_cast<int>(v.shape[3]), C = parts_channels(ps);
  if (uint64_t(m->batch) * C * H * W != n) return set_error(&m->error, "value %u is not an NCHW activation", value);
  // with slot reuse, a buffer written after this one over the same bytes has replaced its contents
  for (const Part& p : ps) {
    if (p.buf == kInput) continue;
    const Buffer& b = m->bufs[p.buf];
    for (const Buffer& o : m->bufs)
      if (&o != &b && o.bytes && o.first > b.first && o.off < b.off + b.bytes && b.off < o.off + o.bytes)
        return set_error(&m->error, "value %u's arena slot is reused by later launches: call "
                                    "aexrt_b200_yolo_set_arena_reuse(model, 0) and run again", value);
  }
  int c0 = 0;
  for (const Part& p : ps) {
    if (p.buf == kInput) return set_error(&m->error, "value %u is the graph input", value);
    const Buffer& b = m->bufs[p.buf];
    std::vector<__half> host(size_t(m->batch) * b.h * b.w * b.c);
    if (!cuda_ok(cudaMemcpy(host.data(), buf_ptr(m, p.buf), host.size() * 2, cudaMemcpyDeviceToHost), "read value",
                 &m->error))
      return 0;
    for (uint32_t img = 0; img < m->batch; ++img)
      for (int c = 0; c < p.ch; ++c)
        for (int y = 0; y < H; ++y)
          for (int x = 0; x < W; ++x) {
            const size_t src = ((size_t(img) * b.h + y / p.up) * b.w + x / p.up) * b.c + p.coff + c;
            out[((size_t(img) * C + c0 + c) * H + y) * W + x] = __half2float(host[src]);
          }
    c0 += p.ch;
  }
  return 1;
}

int aexrt_yolo_debug_page(AexrtYoloModel* m, uint32_t, float*, uint64_t) {
  return set_error(m ? &m->error : nullptr, "pages are the D3D12 arena's resources; read values with "
                                            "aexrt_yolo_debug_value");
}

}  // extern "C"
