// Reader of the reference's .aexrt engine container (host code, no GPU needed).
//
// Container format: docs/AEXRT_ENGINE.md:54-587 of the reference, written by
// src/aexrt/engine.py:3952 (_build_container) and its section encoders
// (:2556-2700, :3867-3930, memory_v2.py:572-603, barrier_v2.py:262-285), parsed
// there by parse_aexrt_engine (native/aexrt_d3d12_runtime.cpp:17560).  The
// reader checks what that loader checks before it trusts an engine, and the
// structural rules the format document states for the optional plans, and
// fails closed with a message otherwise.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace aexrt {
namespace engine {

// command kinds (src/aexrt/engine.py:103-118)
enum Kind : uint32_t {
  kConv = 1, kConvSilu = 2, kConcatConv1x1 = 3, kView = 4, kAlias = 5, kSlice = 6, kConcat = 7,
  kResize = 8, kMaxPool = 9, kUnary = 10, kBinary = 11, kMatMul = 12, kTranspose = 13, kSoftmax = 14,
};
constexpr uint32_t kValueInput = 1u << 0, kValueConstant = 1u << 1, kValueArena = 1u << 2, kValueAlias = 1u << 3;
constexpr uint32_t kPlanAuthoritative = 1u << 0, kPlanInt8PerGroup = 1u << 4;
constexpr uint32_t kLayoutConvInt8 = 8;

const char* kind_name(uint32_t kind);

struct Manifest {
  uint32_t u[17] = {};
  uint64_t input_elements = 0, arena_nbytes = 0;
  float conf = 0.25f, iou = 0.45f;
  uint32_t precision() const { return u[2]; }
  uint32_t output_layout() const { return u[4]; }
  uint32_t objectness() const { return u[5]; }
  uint32_t channels() const { return u[6]; }
  uint32_t anchors() const { return u[7]; }
  uint32_t classes() const { return u[8]; }
  uint32_t max_candidates() const { return u[9]; }
  uint32_t max_detections() const { return u[10]; }
  uint32_t nodes() const { return u[11]; }
  uint32_t value_count() const { return u[12]; }
  uint32_t constant_count() const { return u[13]; }
  uint32_t command_count() const { return u[14]; }
  uint32_t input_value() const { return u[15]; }
  uint32_t output_value() const { return u[16]; }
};

struct Value {
  uint32_t id = 0, flags = 0;
  uint64_t elements = 0;
  uint32_t shape[4] = {0, 0, 0, 0};
  uint64_t arena_offset = 0, arena_nbytes = 0;
};

struct Command {
  uint32_t kind = 0, output = 0, planned_kernel = 0, precision = 0;
  std::vector<uint32_t> inputs, params;
  uint32_t plan_flags = 0, packed_value = 0xFFFFFFFFu;  // from the kernel plan
};

struct Constant {
  uint32_t dtype = 0;       // 1 fp32, 2 fp16 (widened here)
  std::vector<float> data;
};

struct Packed {
  uint32_t layout = 0, in_channels = 0, out_channels = 0;
  uint64_t elements = 0;
  std::vector<uint8_t> data;
};

struct MemoryPage {
  uint32_t id = 0, dtype = 0, layout = 0, flags = 0;
  uint64_t nbytes = 0;
};

struct MemoryRecord {
  uint32_t value = 0, flags = 0, page = 0, dtype = 0, layout = 0;
  uint64_t offset = 0, nbytes = 0;
};

struct FusionGroup {
  uint32_t kind = 0, start = 0, end = 0, precision = 0, kernel = 0, flags = 0, aux0 = 0, aux1 = 0;
};

struct PhysicalRecord {
  uint64_t stable_id = 0;
  uint32_t logical_start = 0, logical_end = 0, execution_index = 0, kernel = 0, precision = 0, flags = 0,
           fusion_kind = 0;
  std::vector<uint32_t> logical;  // owned logical command indices (sorted)
};

struct Engine {
  Manifest manifest;
  std::vector<Value> values;
  std::vector<Command> commands;
  std::map<uint32_t, Constant> constants;
  std::map<uint32_t, Packed> packed;
  uint32_t memory_plan_version = 0;  // 1 legacy, 2 paged
  uint64_t memory_alignment = 0;
  std::vector<MemoryPage> pages;
  std::vector<MemoryRecord> memory_records;
  std::vector<FusionGroup> fusion;
  bool has_physical = false, has_barrier = false;
  std::vector<PhysicalRecord> physical;
  uint32_t barrier_records = 0;
  std::vector<uint32_t> section_ids;
};

// Parses and validates an engine image.  Returns false and sets *err on any violation.
bool parse(const uint8_t* data, size_t size, Engine* out, std::string* err);

// The 32-bit CRC of the container's section checksums (IEEE 802.3, reflected, as zlib.crc32).
uint32_t crc32(const uint8_t* data, size_t size);

}  // namespace engine
}  // namespace aexrt
