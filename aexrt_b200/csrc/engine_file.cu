// Reader of the reference's .aexrt engine container (see engine_file.h).
#include "engine_file.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <set>

#include <cuda_fp16.h>

namespace aexrt {
namespace engine {

namespace {

constexpr char kMagic[8] = {'A', 'E', 'X', 'R', 'T', 'E', 'N', 'G'};
constexpr size_t kHeader = 64, kToc = 32;

bool failf(std::string* err, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (err) *err = buf;
  return false;
}

// Little-endian reader over one section; every read is bounds-checked.
struct Reader {
  const uint8_t* p;
  size_t n, at = 0;
  bool ok = true;
  Reader(const uint8_t* d, size_t s, size_t start = 0) : p(d), n(s), at(start) {}
  template <typename T>
  T get() {
    T v{};
    if (!ok || at + sizeof(T) > n) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + at, sizeof(T));
    at += sizeof(T);
    return v;
  }
  uint32_t u32() { return get<uint32_t>(); }
  uint64_t u64() { return get<uint64_t>(); }
  float f32() { return get<float>(); }
};

struct Section {
  const uint8_t* data = nullptr;
  size_t size = 0;
};

uint32_t g_crc_table[256];
bool g_crc_init = [] {
  for (uint32_t i = 0; i < 256; ++i) {
    uint32_t c = i;
    for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
    g_crc_table[i] = c;
  }
  return true;
}();

}  // namespace

uint32_t crc32(const uint8_t* data, size_t size) {
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < size; ++i) c = g_crc_table[(c ^ data[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

const char* kind_name(uint32_t kind) {
  static const char* names[] = {"?",          "CONV",  "CONV_SILU", "CONCAT_CONV1X1", "VIEW",
                                "ALIAS",      "SLICE", "CONCAT",    "RESIZE",         "MAXPOOL",
                                "UNARY",      "BINARY", "MATMUL",   "TRANSPOSE",      "SOFTMAX"};
  return kind <= 14 ? names[kind] : "?";
}

bool parse(const uint8_t* data, size_t size, Engine* out, std::string* err) {
  (void)g_crc_init;
  if (!data || !out) return failf(err, "null engine pointer");
  Engine e;
  // ---- header and section table (docs/AEXRT_ENGINE.md:54-104; runtime.cpp:17560-17597)
  if (size < kHeader || std::memcmp(data, kMagic, 8) != 0) return failf(err, "not an .aexrt engine (bad magic)");
  Reader h(data, size, 8);
  const uint32_t version = h.u32(), header_size = h.u32(), count = h.u32(), flags = h.u32();
  const uint64_t file_size = h.u64(), toc = h.u64(), toc_size = h.u64();
  if (version != 1 || header_size != kHeader) return failf(err, "unsupported engine version %u / header size %u", version, header_size);
  if (!(flags & 1u)) return failf(err, "engine header flag bit 0 is not set");
  if (file_size != size) return failf(err, "file size %zu does not match the header's %llu", size, (unsigned long long)file_size);
  if (toc != kHeader || toc_size != uint64_t(count) * kToc || toc + toc_size > size) return failf(err, "bad section table");
  for (size_t i = 48; i < 64; ++i)
    if (data[i]) return failf(err, "reserved header bytes are not zero");
  if (count < 9 || count > 12) return failf(err, "section count %u outside 9..12", count);
  std::map<uint32_t, Section> sec;
  Reader t(data, size, kHeader);
  for (uint32_t i = 0; i < count; ++i) {
    const uint32_t sid = t.u32(), sflags = t.u32();
    const uint64_t off = t.u64(), sz = t.u64();
    const uint32_t crc = t.u32(), rsv = t.u32();
    (void)sflags;
    if (sid < 1 || sid > 12) return failf(err, "unknown section id %u", sid);
    if (rsv != 0) return failf(err, "section %u: reserved table field is not zero", sid);
    if (sec.count(sid)) return failf(err, "duplicate section %u", sid);
    if (off < toc + toc_size || off > size || sz > size - off) return failf(err, "section %u lies outside the file", sid);
    if (crc32(data + off, static_cast<size_t>(sz)) != crc) return failf(err, "section %u fails its CRC32", sid);
    sec[sid] = Section{data + off, static_cast<size_t>(sz)};
    e.section_ids.push_back(sid);
  }
  for (uint32_t sid = 1; sid <= 9; ++sid)
    if (!sec.count(sid)) return failf(err, "missing section %u", sid);
  if (sec.count(11) && !sec.count(10))
    return failf(err, "section 11 (arena barrier plan) requires section 10 (physical dispatch plan)");

  // ---- manifest (124 bytes; runtime.cpp:17606-17618)
  {
    const Section& s = sec[1];
    if (s.size != 124) return failf(err, "manifest must be 124 bytes");
    Reader r(s.data, s.size);
    for (uint32_t& v : e.manifest.u) v = r.u32();
    e.manifest.input_elements = r.u64();
    e.manifest.arena_nbytes = r.u64();
    e.manifest.conf = r.f32();
    e.manifest.iou = r.f32();
    const uint32_t* u = e.manifest.u;
    if (u[0] != 1) return failf(err, "unsupported manifest version %u", u[0]);
    if (u[1] != 1 || (u[2] != 1 && u[2] != 2) || u[3] != 2 || (u[4] != 1 && u[4] != 2) || u[5] > 1 || !u[6] || !u[7] ||
        !u[8] || !u[12] || !u[14] || u[15] >= u[12] || u[16] >= u[12] || !e.manifest.input_elements ||
        !e.manifest.arena_nbytes)
      return failf(err, "manifest fields out of range (target, precision, mode, layout, counts or value ids)");
  }
  const uint32_t nval = e.manifest.value_count(), ncmd = e.manifest.command_count();

  // ---- values: <II> + 48-byte <IIQ4IQQ> records
  {
    Reader r(sec[2].data, sec[2].size);
    const uint32_t n = r.u32(), rsv = r.u32();
    if (!r.ok || rsv != 0 || n != nval) return failf(err, "values section disagrees with the manifest");
    e.values.resize(n);
    for (uint32_t i = 0; i < n; ++i) {
      Value& v = e.values[i];
      v.id = r.u32();
      v.flags = r.u32();
      v.elements = r.u64();
      for (uint32_t& d : v.shape) d = r.u32();
      v.arena_offset = r.u64();
      v.arena_nbytes = r.u64();
      if (!r.ok) return failf(err, "values section truncated");
      if (v.id != i) return failf(err, "value records are not dense and ordered by id");
      const uint64_t prod = uint64_t(v.shape[0]) * v.shape[1] * v.shape[2] * v.shape[3];
      if (prod != v.elements) return failf(err, "value %u: shape does not hold its element count", i);
      if (!(v.flags & kValueArena) && (v.arena_offset != ~0ull || v.arena_nbytes != 0))
        return failf(err, "value %u: a non-arena value carries an arena range", i);
    }
    if (r.at != sec[2].size) return failf(err, "trailing bytes in the values section");
  }

  // ---- commands: <II> + <6I> header, inputs, params
  {
    Reader r(sec[3].data, sec[3].size);
    const uint32_t n = r.u32(), rsv = r.u32();
    if (!r.ok || rsv != 0 || n != ncmd) return failf(err, "commands section disagrees with the manifest");
    e.commands.resize(n);
    for (uint32_t i = 0; i < n; ++i) {
      Command& c = e.commands[i];
      c.kind = r.u32();
      c.output = r.u32();
      const uint32_t nin = r.u32(), npar = r.u32();
      c.planned_kernel = r.u32();
      c.precision = r.u32();
      if (!r.ok || nin > 4096 || npar > 4096) return failf(err, "commands section truncated");
      c.inputs.resize(nin);
      c.params.resize(npar);
      for (uint32_t& v : c.inputs) v = r.u32();
      for (uint32_t& v : c.params) v = r.u32();
      if (!r.ok) return failf(err, "commands section truncated");
      if (c.kind < 1 || c.kind > 14) return failf(err, "command %u: unknown kind %u", i, c.kind);
      if (c.output >= nval) return failf(err, "command %u references a value outside the value table", i);
      for (uint32_t v : c.inputs)
        if (v >= nval) return failf(err, "command %u references a value outside the value table", i);
    }
    if (r.at != sec[3].size) return failf(err, "trailing bytes in the commands section");
  }

  // ---- kernel plan: <II> (count, version 1) + <6I> records repeating each command
  {
    Reader r(sec[5].data, sec[5].size);
    const uint32_t n = r.u32(), ver = r.u32();
    if (!r.ok || n != ncmd || ver != 1) return failf(err, "kernel plan does not cover the command stream");
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t idx = r.u32(), kind = r.u32(), pk = r.u32(), prec = r.u32(), packed = r.u32(), pf = r.u32();
      if (!r.ok) return failf(err, "kernel plan truncated");
      Command& c = e.commands[i];
      if (idx != i || kind != c.kind || pk != c.planned_kernel || prec != c.precision)
        return failf(err, "kernel plan record %u disagrees with its command", i);
      if (!(pf & kPlanAuthoritative)) return failf(err, "kernel plan record %u is not authoritative", i);
      if (pf & ~0x1Fu) return failf(err, "kernel plan record %u has unknown flag bits", i);
      c.plan_flags = pf;
      c.packed_value = packed;
    }
  }

  // ---- raw constants: <II> + <IIQQQ> (value, dtype, elements, offset, nbytes)
  {
    Reader r(sec[4].data, sec[4].size);
    const uint32_t n = r.u32(), rsv = r.u32();
    if (!r.ok || rsv != 0) return failf(err, "raw constants section truncated");
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t vid = r.u32(), dt = r.u32();
      const uint64_t elems = r.u64(), off = r.u64(), nb = r.u64();
      if (!r.ok) return failf(err, "raw constants section truncated");
      const uint64_t width = dt == 1 ? 4 : (dt == 2 ? 2 : 0);
      if (!width || nb != elems * width || off > sec[4].size || nb > sec[4].size - off || vid >= nval)
        return failf(err, "bad constant record for value %u", vid);
      if (!(e.values[vid].flags & kValueConstant) || e.values[vid].elements != elems)
        return failf(err, "constant record for value %u does not match its value", vid);
      Constant& k = e.constants[vid];
      k.dtype = dt;
      k.data.resize(static_cast<size_t>(elems));
      const uint8_t* src = sec[4].data + off;
      for (uint64_t j = 0; j < elems; ++j) {
        if (dt == 1) {
          std::memcpy(&k.data[j], src + 4 * j, 4);
        } else {
          __half hv;
          std::memcpy(&hv, src + 2 * j, 2);
          k.data[j] = __half2float(hv);
        }
      }
    }
  }

  // ---- packed weights: <II> + <4IQQQ>
  {
    Reader r(sec[6].data, sec[6].size);
    const uint32_t n = r.u32(), rsv = r.u32();
    if (!r.ok || rsv != 0) return failf(err, "packed weights section truncated");
    for (uint32_t i = 0; i < n; ++i) {
      Packed p;
      const uint32_t vid = r.u32();
      p.layout = r.u32();
      p.in_channels = r.u32();
      p.out_channels = r.u32();
      p.elements = r.u64();
      const uint64_t off = r.u64(), nb = r.u64();
      if (!r.ok) return failf(err, "packed weights section truncated");
      if (off > sec[6].size || nb > sec[6].size - off || vid >= nval)
        return failf(err, "packed weights of value %u lie outside their section", vid);
      p.data.assign(sec[6].data + off, sec[6].data + off + nb);
      e.packed[vid] = std::move(p);
    }
  }

  // ---- memory plan (section 7): V2 pages + value records, or the legacy V1 table
  {
    const Section& s = sec[7];
    Reader r(s.data, s.size);
    const uint32_t first = r.u32();
    if (!r.ok) return failf(err, "memory plan truncated");
    if (first == 2) {
      e.memory_plan_version = 2;
      const uint32_t alignment = r.u32(), npages = r.u32(), nrec = r.u32();
      const uint64_t total = r.u64();
      const uint32_t mflags = r.u32(), rsv = r.u32();
      if (!r.ok || alignment < 4 || (alignment & (alignment - 1)) || npages == 0 || npages > 64 || mflags != 1 ||
          rsv != 0 || s.size != 32 + size_t(npages) * 24 + size_t(nrec) * 40)
        return failf(err, "invalid memory plan V2 header");
      if (total != e.manifest.arena_nbytes) return failf(err, "memory plan total differs from the manifest arena size");
      e.memory_alignment = alignment;
      uint64_t sum = 0;
      for (uint32_t i = 0; i < npages; ++i) {
        MemoryPage pg;
        pg.id = r.u32();
        pg.dtype = r.u32();
        pg.layout = r.u32();
        pg.flags = r.u32();
        pg.nbytes = r.u64();
        if (pg.id != i || (pg.dtype != 1 && pg.dtype != 2) || (pg.layout != 1 && pg.layout != 2) ||
            (pg.layout == 2 && pg.dtype != 2) || pg.flags != 1 || pg.nbytes == 0 || pg.nbytes % alignment)
          return failf(err, "invalid memory page %u", i);
        sum += pg.nbytes;
        e.pages.push_back(pg);
      }
      if (sum != total) return failf(err, "memory pages do not add up to the plan total");
      std::set<uint32_t> seen;
      for (uint32_t i = 0; i < nrec; ++i) {
        MemoryRecord m;
        m.value = r.u32();
        m.flags = r.u32();
        m.page = r.u32();
        m.dtype = r.u32();
        m.layout = r.u32();
        const uint32_t rr = r.u32();
        m.offset = r.u64();
        m.nbytes = r.u64();
        if (m.value >= nval || seen.count(m.value) || !(m.flags & kValueArena) || m.page >= npages || rr != 0 ||
            m.dtype != e.pages[m.page].dtype || m.layout != e.pages[m.page].layout || m.offset % alignment ||
            m.nbytes == 0 || m.offset > e.pages[m.page].nbytes || m.nbytes > e.pages[m.page].nbytes - m.offset)
          return failf(err, "invalid memory record %u (value %u)", i, m.value);
        const Value& v = e.values[m.value];
        if (m.nbytes != v.elements * (m.dtype == 2 ? 2 : 4))
          return failf(err, "memory record of value %u does not hold its elements", m.value);
        if (v.arena_offset != m.offset || v.arena_nbytes != m.nbytes)
          return failf(err, "values section and memory plan disagree on value %u", m.value);
        seen.insert(m.value);
        e.memory_records.push_back(m);
      }
    } else {
      // legacy V1: <IIQ> (alignment, value count, total) + <IIQQ> records in one fp32 resource
      e.memory_plan_version = 1;
      const uint32_t alignment = first, nrec = r.u32();
      const uint64_t total = r.u64();
      if (!r.ok || alignment < 4 || (alignment & (alignment - 1)) || s.size != 16 + size_t(nrec) * 24 ||
          total != e.manifest.arena_nbytes)
        return failf(err, "invalid legacy memory plan");
      e.memory_alignment = alignment;
      for (uint32_t i = 0; i < nrec; ++i) {
        MemoryRecord m;
        m.value = r.u32();
        m.flags = r.u32();
        m.offset = r.u64();
        m.nbytes = r.u64();
        if (m.value >= nval || m.offset % alignment || m.offset > total || m.nbytes > total - m.offset)
          return failf(err, "invalid legacy memory record %u", i);
        m.dtype = 1;
        m.layout = 1;
        e.memory_records.push_back(m);
      }
    }
  }

  // ---- fusion plan (section 8): <4I> + <8I> groups
  {
    Reader r(sec[8].data, sec[8].size);
    const uint32_t ver = r.u32(), ngroups = r.u32(), nc = r.u32(), fflags = r.u32();
    if (!r.ok || ver != 1 || nc != ncmd || !(fflags & 1u) || sec[8].size != 16 + size_t(ngroups) * 32)
      return failf(err, "invalid fusion plan header");
    for (uint32_t i = 0; i < ngroups; ++i) {
      FusionGroup g;
      g.kind = r.u32();
      g.start = r.u32();
      g.end = r.u32();
      g.precision = r.u32();
      g.kernel = r.u32();
      g.flags = r.u32();
      g.aux0 = r.u32();
      g.aux1 = r.u32();
      const bool kind_ok = g.kind == 1 || g.kind == 2 || g.kind == 3 || g.kind == 4 || g.kind == 6 || g.kind == 9;
      if (!kind_ok || g.start > g.end || g.end >= ncmd || (g.precision != 1 && g.precision != 2))
        return failf(err, "invalid fusion group %u (kind %u, commands %u..%u)", i, g.kind, g.start, g.end);
      e.fusion.push_back(g);
    }
  }

  // ---- physical dispatch plan V2 (section 10)
  if (sec.count(10)) {
    e.has_physical = true;
    const Section& s = sec[10];
    Reader r(s.data, s.size);
    const uint32_t ver = r.u32(), nrec = r.u32(), nlog = r.u32(), pflags = r.u32(), rsize = r.u32(), nidx = r.u32(),
                   table = r.u32(), rsv = r.u32();
    if (!r.ok || ver != 2 || pflags != 1 || rsv != 0 || rsize != 48 || nlog != ncmd || nidx != ncmd ||
        table != 32 + nrec * 48 || s.size != size_t(table) + size_t(nidx) * 4)
      return failf(err, "invalid physical dispatch plan header");
    std::vector<uint32_t> idx(nidx);
    {
      Reader ti(s.data, s.size, table);
      for (uint32_t& v : idx) v = ti.u32();
    }
    std::vector<int> owner(ncmd, -1);
    std::set<uint64_t> ids;
    uint32_t expect_off = 0;
    int64_t last_exec = -1;
    for (uint32_t i = 0; i < nrec; ++i) {
      PhysicalRecord p;
      p.stable_id = r.u64();
      p.logical_start = r.u32();
      p.logical_end = r.u32();
      p.execution_index = r.u32();
      const uint32_t off = r.u32(), cnt = r.u32();
      p.kernel = r.u32();
      p.precision = r.u32();
      p.flags = r.u32();
      p.fusion_kind = r.u32();
      const uint32_t prsv = r.u32();
      if (!r.ok) return failf(err, "physical dispatch plan truncated");
      if (p.stable_id == 0 || ids.count(p.stable_id) || prsv != 0 || off != expect_off || cnt == 0 ||
          off + cnt > nidx || p.fusion_kind > 9 || (p.precision != 1 && p.precision != 2) || !(p.flags & 1u))
        return failf(err, "invalid physical dispatch record %u", i);
      ids.insert(p.stable_id);
      expect_off += cnt;
      p.logical.assign(idx.begin() + off, idx.begin() + off + cnt);
      for (size_t k = 0; k < p.logical.size(); ++k) {
        const uint32_t li = p.logical[k];
        if (li >= ncmd || (k && li <= p.logical[k - 1]) || owner[li] >= 0)
          return failf(err, "physical dispatch record %u: logical commands not sorted, repeated or out of range", i);
        owner[li] = static_cast<int>(i);
      }
      if (p.logical_start != p.logical.front() || p.logical_end != p.logical.back())
        return failf(err, "physical dispatch record %u: logical range does not match its table entries", i);
      if ((p.fusion_kind == 0) != (cnt == 1))
        return failf(err, "physical dispatch record %u: unfused records own one command, fused ones several", i);
      if (!std::binary_search(p.logical.begin(), p.logical.end(), p.execution_index) ||
          int64_t(p.execution_index) <= last_exec)
        return failf(err, "physical dispatch record %u: execution index outside the record or out of order", i);
      last_exec = p.execution_index;
      if (p.fusion_kind == 0) {
        const Command& c = e.commands[p.logical[0]];
        if (p.kernel != c.planned_kernel || p.flags != c.plan_flags)
          return failf(err, "physical dispatch record %u disagrees with the kernel plan of command %u", i, p.logical[0]);
      }
      e.physical.push_back(std::move(p));
    }
    if (expect_off != nidx) return failf(err, "physical dispatch plan leaves table entries unowned");
    for (uint32_t li = 0; li < ncmd; ++li)
      if (owner[li] < 0) return failf(err, "command %u belongs to no physical dispatch record", li);
  }

  // ---- arena barrier plan V1 (section 11): header rules and record bounds.  The barriers order
  // D3D12 resource states; on CUDA the one stream orders every access, so they are validated only.
  if (sec.count(11)) {
    e.has_barrier = true;
    const Section& s = sec[11];
    Reader r(s.data, s.size);
    const uint32_t ver = r.u32(), bflags = r.u32(), ndisp = r.u32(), npages = r.u32(), nrec = r.u32(),
                   rsize = r.u32(), r0 = r.u32(), r1 = r.u32();
    if (!r.ok || ver != 1 || bflags != 1 || rsize != 40 || r0 || r1 || ndisp != e.physical.size() ||
        e.memory_plan_version != 2 || npages != e.pages.size() || s.size != 32 + size_t(nrec) * 40)
      return failf(err, "invalid arena barrier plan header");
    uint64_t prev = 0;
    for (uint32_t i = 0; i < nrec; ++i) {
      const uint32_t disp = r.u32(), page = r.u32(), kind = r.u32(), before = r.u32(), after = r.u32(), rr = r.u32();
      const uint64_t off = r.u64(), nb = r.u64();
      (void)before;
      (void)after;
      const uint64_t key = (uint64_t(disp) << 32) | page;
      if (disp >= ndisp || page >= npages || kind < 1 || kind > 3 || rr || nb == 0 || off > e.pages[page].nbytes ||
          nb > e.pages[page].nbytes - off || (i && key <= prev))
        return failf(err, "invalid arena barrier record %u", i);
      prev = key;
    }
    e.barrier_records = nrec;
  }
  *out = std::move(e);
  return true;
}

}  // namespace engine
}  // namespace aexrt
