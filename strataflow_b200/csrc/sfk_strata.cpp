// sfk_strata.cpp -- the .strata file reader and its HBM loader (host code).
//
// Replaces, for the HBM-resident engine, the reference's
//   * StrataReader::open            (src/tws/strata_file.cpp:30-230): superblock
//     (v1 / v2 / v3 trailing fields, header CRC32), embedded GGUF metadata,
//     expert index, optional trunk index;
//   * StrataReader::read_bundle     (src/tws/strata_file.cpp:368-444): one
//     (layer, expert) bundle gate|up|down;
//   * Engine::load_strata_weights   (src/model/engine/engine.cpp:556-830) and
//     the hparam read of Engine::load (engine.cpp:1062-1137): hparams from the
//     GGUF keys, trunk tensors walked in GGUF order through the contiguous
//     trunk block, experts from the bundle index.
// The on-disk format is the reference's (src/tws/strata_format.h:77-177), read
// field by field from its documented byte offsets.  LZ-compressed expert
// blobs (v3 kStrataFlagExpertsCompressed) are not decoded: such a file is
// rejected with SFK_ERR_UNSUPPORTED.
//
// Nothing here touches a GPU except sfk_strata_load, which hands each tensor's
// verbatim GGUF bytes to sfk_weights_put / sfk_expert_put.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <tuple>
#include <vector>

#include "sfk.h"
#include "sfk_kernels.cuh"

namespace {

using sfk::set_last_error;

sfk_status sfail(sfk_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return s;
}

// strata_format.h: superblock size, magic, flag bits
constexpr uint32_t SB_SIZE = 128;
constexpr char MAGIC[8] = {'S', 'T', 'R', 'A', 'T', 'A', '0', '1'};
constexpr uint32_t FLAG_COMPRESSED = 1u << 3;
constexpr uint64_t INDEX_ENTRY = 48;  // ExpertIndexEntry
constexpr uint64_t TRUNK_ENTRY = 80;  // TrunkIndexEntry (64-byte name + 2 x u64)

// CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320), as the header CRC
// of strata_format.h specifies it; table-driven.
uint32_t crc32_ieee(const uint8_t* p, size_t n) {
  static const std::array<uint32_t, 256> table = [] {  // built once, thread-safe
    std::array<uint32_t, 256> t{};
    for (uint32_t i = 0; i < 256; ++i) {
      uint32_t c = i;
      for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
      t[i] = c;
    }
    return t;
  }();
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

template <typename T>
T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

// ggml block geometry of the types this library reads: (weights per block,
// bytes per block)
bool type_block(int t, int64_t* blk, int64_t* bytes) {
  switch (t) {
    case SFK_TYPE_F32: *blk = 1; *bytes = 4; return true;
    case SFK_TYPE_F16: *blk = 1; *bytes = 2; return true;
    case SFK_TYPE_Q8_0: *blk = 32; *bytes = 34; return true;
    case SFK_TYPE_Q4_K: *blk = 256; *bytes = 144; return true;
    case SFK_TYPE_Q6_K: *blk = 256; *bytes = 210; return true;
    default: return false;
  }
}

struct TensorInfo {
  std::string name;
  int type = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  uint64_t nbytes = 0;      // ggml_nbytes
  bool expert = false;      // blk.N.ffn_{gate,up,down}_exps.weight: lives in the bundles
  uint64_t trunk_rel = 0;   // byte offset inside the trunk block (trunk tensors)
};

struct KV {
  uint32_t type = 0;
  uint64_t u = 0;  // integer / bool value
  double f = 0.0;  // float value
  std::string s;
};

struct ExpertEntry {
  uint32_t layer, expert;
  uint64_t blob_offset, blob_length, gate_rel, up_rel, down_rel;
};

// GGUF metadata parser over the embedded blob (GGUF v2 / v3: magic "GGUF",
// u32 version, u64 tensor count, u64 KV count, KV pairs, tensor infos).
struct Cursor {
  const uint8_t* p;
  size_t n, off = 0;
  bool ok = true;
  bool need(size_t k) {
    if (!ok || off + k > n) ok = false;
    return ok;
  }
  template <typename T>
  T get() {
    if (!need(sizeof(T))) return T{};
    T v = rd<T>(p + off);
    off += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t len = get<uint64_t>();
    if (!ok || len > (1u << 20) || !need((size_t)len)) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p + off), (size_t)len);
    off += (size_t)len;
    return s;
  }
};

// GGUF value types
enum : uint32_t {
  G_U8 = 0, G_I8 = 1, G_U16 = 2, G_I16 = 3, G_U32 = 4, G_I32 = 5, G_F32 = 6, G_BOOL = 7,
  G_STR = 8, G_ARR = 9, G_U64 = 10, G_I64 = 11, G_F64 = 12
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case G_U8: case G_I8: case G_BOOL: return 1;
    case G_U16: case G_I16: return 2;
    case G_U32: case G_I32: case G_F32: return 4;
    case G_U64: case G_I64: case G_F64: return 8;
    default: return 0;
  }
}

bool read_value(Cursor& c, uint32_t t, KV* out, int depth = 0) {
  if (t == G_STR) {
    std::string s = c.str();
    if (out) out->s = s;
    return c.ok;
  }
  if (t == G_ARR) {
    if (depth > 2) return false;
    const uint32_t et = c.get<uint32_t>();
    const uint64_t cnt = c.get<uint64_t>();
    if (!c.ok) return false;
    if (et == G_STR || et == G_ARR) {
      for (uint64_t i = 0; i < cnt && c.ok; ++i) read_value(c, et, nullptr, depth + 1);
    } else {
      const size_t sz = scalar_size(et);
      if (!sz || cnt > (uint64_t)1 << 40 || !c.need((size_t)(cnt * sz))) return false;
      c.off += (size_t)(cnt * sz);
    }
    return c.ok;
  }
  const size_t sz = scalar_size(t);
  if (!sz || !c.need(sz)) return false;
  const uint8_t* q = c.p + c.off;
  if (out) {
    switch (t) {
      case G_U8: out->u = rd<uint8_t>(q); break;
      case G_I8: out->u = (uint64_t)(int64_t)rd<int8_t>(q); break;
      case G_U16: out->u = rd<uint16_t>(q); break;
      case G_I16: out->u = (uint64_t)(int64_t)rd<int16_t>(q); break;
      case G_U32: out->u = rd<uint32_t>(q); break;
      case G_I32: out->u = (uint64_t)(int64_t)rd<int32_t>(q); break;
      case G_BOOL: out->u = rd<uint8_t>(q); break;
      case G_U64: out->u = rd<uint64_t>(q); break;
      case G_I64: out->u = (uint64_t)rd<int64_t>(q); break;
      case G_F32: out->f = rd<float>(q); break;
      case G_F64: out->f = rd<double>(q); break;
      default: break;
    }
  }
  c.off += sz;
  return true;
}

// blk.N.<suffix>: layer N and the suffix, or -1
int parse_layer(const std::string& name, std::string* suffix) {
  if (name.compare(0, 4, "blk.") != 0) return -1;
  size_t i = 4;
  int l = 0;
  if (i >= name.size() || name[i] < '0' || name[i] > '9') return -1;
  while (i < name.size() && name[i] >= '0' && name[i] <= '9') {
    if (i >= 4 + 6) return -1;  // a layer index of at most six digits
    l = l * 10 + (name[i++] - '0');
  }
  if (i >= name.size() || name[i] != '.') return -1;
  *suffix = name.substr(i + 1);
  return l;
}

bool is_expert_name(const std::string& name) {
  std::string suf;
  if (parse_layer(name, &suf) < 0) return false;
  return suf == "ffn_gate_exps.weight" || suf == "ffn_up_exps.weight" || suf == "ffn_down_exps.weight";
}

// trunk tensor name -> (tensor id, layer) of include/sfk.h, or false
bool trunk_id(const std::string& name, int* tid, int* layer) {
  *layer = 0;
  if (name == "token_embd.weight") { *tid = SFK_T_TOK_EMBD; return true; }
  if (name == "output_norm.weight") { *tid = SFK_T_OUTPUT_NORM; return true; }
  if (name == "output.weight") { *tid = SFK_T_OUTPUT; return true; }
  std::string suf;
  const int l = parse_layer(name, &suf);
  if (l < 0) return false;
  *layer = l;
  static const std::map<std::string, int> ids = {
      {"attn_norm.weight", SFK_T_ATTN_NORM}, {"attn_q.weight", SFK_T_ATTN_Q},
      {"attn_k.weight", SFK_T_ATTN_K},       {"attn_v.weight", SFK_T_ATTN_V},
      {"attn_output.weight", SFK_T_ATTN_OUT}, {"ffn_norm.weight", SFK_T_FFN_NORM},
      {"ffn_gate_inp.weight", SFK_T_FFN_GATE_INP}};
  auto it = ids.find(suf);
  if (it == ids.end()) return false;
  *tid = it->second;
  return true;
}

}  // namespace

struct sfk_strata {
  int fd = -1;
  uint64_t file_size = 0;
  std::string path;
  // superblock
  uint32_t version = 0, flags = 0, n_layers = 0, n_experts = 0, align = 0;
  uint64_t meta_off = 0, meta_size = 0, index_off = 0, index_count = 0, trunk_off = 0, trunk_size = 0;
  uint64_t expert_off = 0, expert_size = 0, trunk_index_off = 0, trunk_index_count = 0;
  uint64_t compress_off = 0, compress_count = 0;
  // GGUF metadata
  std::map<std::string, KV> kv;
  std::vector<TensorInfo> tensors;
  std::map<std::string, size_t> by_name;
  std::vector<ExpertEntry> index;
  std::map<uint64_t, size_t> entry_of;  // (layer << 32 | expert) -> index position

  ~sfk_strata() {
    if (fd >= 0) close(fd);
  }
  bool read_at(void* dst, uint64_t n, uint64_t off) const {
    if (off + n > file_size || off + n < off) return false;
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n > 0) {
      const ssize_t r = pread(fd, d, n > (1u << 30) ? (1u << 30) : (size_t)n, (off_t)off);
      if (r <= 0) return false;
      d += r;
      off += (uint64_t)r;
      n -= (uint64_t)r;
    }
    return true;
  }
  const TensorInfo* find(const std::string& name) const {
    auto it = by_name.find(name);
    return it == by_name.end() ? nullptr : &tensors[it->second];
  }
  int64_t key_int(const std::string& k, int64_t fallback) const {
    auto it = kv.find(k);
    if (it == kv.end()) return fallback;
    const uint32_t t = it->second.type;
    if (t == G_F32 || t == G_F64 || t == G_STR || t == G_ARR) return fallback;
    return (int64_t)it->second.u;  // signed types were stored sign-extended
  }
  double key_float(const std::string& k, double fallback) const {
    auto it = kv.find(k);
    if (it == kv.end()) return fallback;
    if (it->second.type == G_F32 || it->second.type == G_F64) return it->second.f;
    return fallback;
  }
};

namespace {

sfk_status parse_superblock(sfk_strata* s) {
  uint8_t sb[SB_SIZE];
  if (s->file_size < SB_SIZE || !s->read_at(sb, SB_SIZE, 0))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: shorter than the 128-byte superblock", s->path.c_str());
  if (std::memcmp(sb, MAGIC, 8) != 0)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: not a .strata file (magic)", s->path.c_str());
  s->version = rd<uint32_t>(sb + 8);
  s->flags = rd<uint32_t>(sb + 12);
  s->meta_off = rd<uint64_t>(sb + 16);
  s->meta_size = rd<uint64_t>(sb + 24);
  s->index_off = rd<uint64_t>(sb + 32);
  s->index_count = rd<uint64_t>(sb + 40);
  s->trunk_off = rd<uint64_t>(sb + 48);
  s->trunk_size = rd<uint64_t>(sb + 56);
  s->expert_off = rd<uint64_t>(sb + 64);
  s->expert_size = rd<uint64_t>(sb + 72);
  // trailing fields by version (strata_format.h:52-66)
  uint32_t tail;
  if (s->version == 1) {
    tail = 80;
  } else if (s->version == 2) {
    s->trunk_index_off = rd<uint64_t>(sb + 80);
    s->trunk_index_count = rd<uint64_t>(sb + 88);
    tail = 96;
  } else if (s->version == 3) {
    s->trunk_index_off = rd<uint64_t>(sb + 80);
    s->trunk_index_count = rd<uint64_t>(sb + 88);
    s->compress_off = rd<uint64_t>(sb + 96);
    s->compress_count = rd<uint64_t>(sb + 104);
    tail = 112;
  } else {
    return sfail(SFK_ERR_UNSUPPORTED, "%s: .strata version %u (1-3 are read)", s->path.c_str(), s->version);
  }
  s->n_layers = rd<uint32_t>(sb + tail);
  s->n_experts = rd<uint32_t>(sb + tail + 4);
  s->align = rd<uint32_t>(sb + tail + 8);
  const uint32_t crc = rd<uint32_t>(sb + tail + 12);
  if (crc32_ieee(sb, tail + 12) != crc)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: superblock CRC mismatch", s->path.c_str());
  if ((s->flags & FLAG_COMPRESSED) || s->compress_count > 0)
    return sfail(SFK_ERR_UNSUPPORTED,
                 "%s: LZ-compressed expert blobs are not decoded by this loader; pack the file uncompressed",
                 s->path.c_str());
  auto inside = [&](uint64_t off, uint64_t n) { return off <= s->file_size && n <= s->file_size - off; };
  if (!inside(s->meta_off, s->meta_size) || !inside(s->trunk_off, s->trunk_size) ||
      !inside(s->expert_off, s->expert_size) || s->index_count > (1ull << 32) ||
      !inside(s->index_off, s->index_count * INDEX_ENTRY) || s->trunk_index_count > (1ull << 32) ||
      !inside(s->trunk_index_off, s->trunk_index_count * TRUNK_ENTRY))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: a region lies outside the file", s->path.c_str());
  return SFK_OK;
}

sfk_status parse_gguf(sfk_strata* s) {
  std::vector<uint8_t> meta((size_t)s->meta_size);
  if (!s->read_at(meta.data(), s->meta_size, s->meta_off))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: GGUF metadata unreadable", s->path.c_str());
  Cursor c{meta.data(), meta.size()};
  const uint32_t magic = c.get<uint32_t>();
  const uint32_t ver = c.get<uint32_t>();
  if (!c.ok || magic != 0x46554747u /* "GGUF" */ || (ver != 2 && ver != 3))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: embedded metadata is not GGUF v2/v3", s->path.c_str());
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: GGUF counts out of range", s->path.c_str());
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    KV v;
    v.type = c.get<uint32_t>();
    if (!c.ok || !read_value(c, v.type, &v))
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: GGUF key/value %llu unreadable", s->path.c_str(),
                   (unsigned long long)i);
    s->kv[key] = v;
  }
  uint64_t trunk_rel = 0;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    TensorInfo t;
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok || nd < 1 || nd > 4) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor %llu dims", s->path.c_str(),
                                                (unsigned long long)i);
    for (uint32_t d = 0; d < nd; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
    t.type = (int)c.get<uint32_t>();
    (void)c.get<uint64_t>();  // offset in the source GGUF's data section (unused: the trunk is repacked)
    if (!c.ok) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor info %llu unreadable", s->path.c_str(),
                            (unsigned long long)i);
    int64_t blk, bb;
    if (!type_block(t.type, &blk, &bb))
      return sfail(SFK_ERR_UNSUPPORTED, "%s: tensor %s has ggml type %d (F32, F16, Q8_0, Q4_K, Q6_K are read)",
                   s->path.c_str(), t.name.c_str(), t.type);
    bool shape_ok = t.ne[0] > 0 && t.ne[0] % blk == 0;
    for (int d = 0; d < 4; ++d) shape_ok = shape_ok && t.ne[d] > 0 && t.ne[d] < ((int64_t)1 << 31);
    if (shape_ok)  // the byte count must stay far from overflow (no real tensor is near 2^50 bytes)
      shape_ok = (double)(t.ne[0] / blk * bb) * (double)t.ne[1] * (double)t.ne[2] * (double)t.ne[3] < 0x1p50;
    if (!shape_ok) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor %s shape", s->path.c_str(), t.name.c_str());
    t.nbytes = (uint64_t)(t.ne[0] / blk * bb) * (uint64_t)t.ne[1] * (uint64_t)t.ne[2] * (uint64_t)t.ne[3];
    t.expert = is_expert_name(t.name);
    if (!t.expert) {  // trunk tensors sit contiguously in GGUF order (engine.cpp:786-830)
      t.trunk_rel = trunk_rel;
      trunk_rel += t.nbytes;
    }
    s->by_name[t.name] = s->tensors.size();
    s->tensors.push_back(t);
  }
  if (trunk_rel > s->trunk_size)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: trunk tensors (%llu B) exceed the trunk block (%llu B)",
                 s->path.c_str(), (unsigned long long)trunk_rel, (unsigned long long)s->trunk_size);
  // a v2+ trunk index, when present, must agree with the GGUF-order walk
  for (uint64_t i = 0; i < s->trunk_index_count; ++i) {
    uint8_t e[TRUNK_ENTRY];
    if (!s->read_at(e, TRUNK_ENTRY, s->trunk_index_off + i * TRUNK_ENTRY))
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: trunk index unreadable", s->path.c_str());
    const std::string name(reinterpret_cast<const char*>(e), strnlen(reinterpret_cast<const char*>(e), 64));
    const TensorInfo* t = s->find(name);
    if (!t || t->expert || rd<uint64_t>(e + 64) != t->trunk_rel || rd<uint64_t>(e + 72) != t->nbytes)
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: trunk index entry %s disagrees with the GGUF tensor order",
                   s->path.c_str(), name.c_str());
  }
  return SFK_OK;
}

sfk_status parse_index(sfk_strata* s) {
  s->index.resize((size_t)s->index_count);
  for (uint64_t i = 0; i < s->index_count; ++i) {
    uint8_t e[INDEX_ENTRY];
    if (!s->read_at(e, INDEX_ENTRY, s->index_off + i * INDEX_ENTRY))
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: expert index unreadable", s->path.c_str());
    ExpertEntry x{rd<uint32_t>(e), rd<uint32_t>(e + 4), rd<uint64_t>(e + 8), rd<uint64_t>(e + 16),
                  rd<uint64_t>(e + 24), rd<uint64_t>(e + 32), rd<uint64_t>(e + 40)};
    if (x.blob_offset > s->file_size || x.blob_length > s->file_size - x.blob_offset)
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: expert blob (%u, %u) outside the file", s->path.c_str(), x.layer,
                   x.expert);
    s->index[(size_t)i] = x;
    s->entry_of[((uint64_t)x.layer << 32) | x.expert] = (size_t)i;
  }
  return SFK_OK;
}

// bytes of one expert's slice of the stacked tensor blk.L.ffn_<kind>_exps
uint64_t expert_slice(const sfk_strata* s, int layer, const char* kind) {
  const TensorInfo* t = s->find("blk." + std::to_string(layer) + ".ffn_" + kind + "_exps.weight");
  if (!t || t->ne[2] <= 0) return 0;
  return t->nbytes / (uint64_t)t->ne[2];
}

}  // namespace

extern "C" {

SFK_API sfk_status sfk_strata_open(const char* path, sfk_strata** out) {
  if (!path || !out) return sfail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  sfk_strata* s = new (std::nothrow) sfk_strata();
  if (!s) return sfail(SFK_ERR_OUT_OF_MEMORY, "host alloc");
  s->path = path;
  s->fd = open(path, O_RDONLY);
  if (s->fd < 0) {
    delete s;
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: cannot open", path);
  }
  const off_t end = lseek(s->fd, 0, SEEK_END);
  s->file_size = end > 0 ? (uint64_t)end : 0;
  sfk_status st = parse_superblock(s);
  if (!st) st = parse_gguf(s);
  if (!st) st = parse_index(s);
  if (st) {
    delete s;
    return st;
  }
  *out = s;
  return SFK_OK;
}

SFK_API void sfk_strata_close(sfk_strata* s) { delete s; }

SFK_API sfk_status sfk_strata_hparams(const sfk_strata* s, sfk_hparams* hp) {
  if (!s || !hp) return sfail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  auto it = s->kv.find("general.architecture");
  const std::string arch = it == s->kv.end() ? std::string("llama") : it->second.s;
  if (arch != "llama")
    return sfail(SFK_ERR_UNSUPPORTED, "%s: architecture '%s' (llama-arch MoE is read)", s->path.c_str(), arch.c_str());
  const TensorInfo* emb = s->find("token_embd.weight");
  const TensorInfo* out = s->find("output.weight");
  const TensorInfo* q = s->find("blk.0.attn_q.weight");
  const TensorInfo* gate = s->find("blk.0.ffn_gate_exps.weight");
  const TensorInfo* down = s->find("blk.0.ffn_down_exps.weight");
  if (!emb || !out || !q || !gate || !down)
    return sfail(SFK_ERR_UNSUPPORTED, "%s: not a llama-arch MoE (token_embd, output, blk.0.attn_q, "
                 "blk.0.ffn_gate_exps / ffn_down_exps required)", s->path.c_str());
  // engine.cpp:1078-1087, 1131-1137
  hp->n_layer = (int32_t)s->key_int("llama.block_count", 0);
  hp->n_embd = (int32_t)s->key_int("llama.embedding_length", emb->ne[0]);
  hp->n_head = (int32_t)s->key_int("llama.attention.head_count", 0);
  hp->n_head_kv = (int32_t)s->key_int("llama.attention.head_count_kv", hp->n_head);
  hp->n_expert = (int32_t)s->key_int("llama.expert_count", 0);
  hp->n_expert_used = (int32_t)s->key_int("llama.expert_used_count", 0);
  hp->rms_eps = (float)s->key_float("llama.attention.layer_norm_rms_epsilon", 1e-5);
  hp->freq_base = (float)s->key_float("llama.rope.freq_base", 10000.0);
  hp->n_vocab = (int32_t)emb->ne[1];
  hp->n_ff = (int32_t)gate->ne[1];
  if (hp->n_ctx <= 0) hp->n_ctx = (int32_t)s->key_int("llama.context_length", 0);
  hp->type_embd = emb->type;
  hp->type_output = out->type;
  hp->type_attn = q->type;
  hp->type_ffn_gu = gate->type;
  hp->type_ffn_down = down->type;
  hp->head_dim = 0;  // n_embd / n_head (engine.cpp:1137)
  if (hp->n_layer <= 0 || hp->n_head <= 0 || hp->n_embd <= 0 || hp->n_expert <= 0 || hp->n_expert_used <= 0)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: incomplete hparams (block_count, head_count, expert_count, "
                 "expert_used_count)", s->path.c_str());
  if (gate->ne[0] != hp->n_embd || gate->ne[2] != hp->n_expert || down->ne[1] != hp->n_embd ||
      down->ne[0] != hp->n_ff || emb->ne[0] != hp->n_embd)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor shapes disagree with the hparams", s->path.c_str());
  if ((s->n_layers && (int64_t)s->n_layers != hp->n_layer) || (s->n_experts && (int64_t)s->n_experts != hp->n_expert))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: superblock layer/expert counts disagree with GGUF", s->path.c_str());
  return SFK_OK;
}

SFK_API int64_t sfk_strata_n_tensors(const sfk_strata* s) { return s ? (int64_t)s->tensors.size() : 0; }

SFK_API sfk_status sfk_strata_tensor_info(const sfk_strata* s, int64_t i, char* name, size_t name_cap, int32_t* type,
                                          int64_t ne[4], uint64_t* n_bytes, int32_t* is_expert) {
  if (!s || i < 0 || i >= (int64_t)s->tensors.size()) return sfail(SFK_ERR_INVALID_ARGUMENT, "tensor index");
  const TensorInfo& t = s->tensors[(size_t)i];
  if (name && name_cap) {
    std::strncpy(name, t.name.c_str(), name_cap - 1);
    name[name_cap - 1] = 0;
  }
  if (type) *type = t.type;
  if (ne)
    for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
  if (n_bytes) *n_bytes = t.nbytes;
  if (is_expert) *is_expert = t.expert ? 1 : 0;
  return SFK_OK;
}

SFK_API sfk_status sfk_strata_read_trunk(const sfk_strata* s, const char* name, void* host_out, size_t n_bytes) {
  if (!s || !name || !host_out) return sfail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const TensorInfo* t = s->find(name);
  if (!t || t->expert) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: no trunk tensor %s", s->path.c_str(), name);
  if (n_bytes != t->nbytes)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s is %llu bytes, buffer %zu", s->path.c_str(), name,
                 (unsigned long long)t->nbytes, n_bytes);
  if (!s->read_at(host_out, t->nbytes, s->trunk_off + t->trunk_rel))
    return sfail(SFK_ERR_RUNTIME, "%s: read of %s failed", s->path.c_str(), name);
  return SFK_OK;
}

SFK_API size_t sfk_strata_bundle_bytes(const sfk_strata* s, int32_t layer) {
  if (!s) return 0;
  return (size_t)(expert_slice(s, layer, "gate") + expert_slice(s, layer, "up") + expert_slice(s, layer, "down"));
}

SFK_API sfk_status sfk_strata_read_bundle(const sfk_strata* s, int32_t layer, int32_t expert, void* host_out,
                                          size_t n_bytes) {
  if (!s || !host_out) return sfail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  auto it = s->entry_of.find(((uint64_t)(uint32_t)layer << 32) | (uint32_t)expert);
  if (it == s->entry_of.end())
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: no bundle for layer %d expert %d", s->path.c_str(), layer, expert);
  const ExpertEntry& x = s->index[it->second];
  const uint64_t g = expert_slice(s, layer, "gate"), u = expert_slice(s, layer, "up"),
                 d = expert_slice(s, layer, "down");
  if (!g || !u || !d || n_bytes != g + u + d)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: bundle of layer %d is %llu bytes, buffer %zu", s->path.c_str(), layer,
                 (unsigned long long)(g + u + d), n_bytes);
  if (x.gate_rel > x.blob_length || g > x.blob_length - x.gate_rel || x.up_rel > x.blob_length ||
      u > x.blob_length - x.up_rel || x.down_rel > x.blob_length || d > x.blob_length - x.down_rel)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: bundle (%d, %d) slices outside its blob", s->path.c_str(), layer,
                 expert);
  uint8_t* o = static_cast<uint8_t*>(host_out);
  if (!s->read_at(o, g, x.blob_offset + x.gate_rel) || !s->read_at(o + g, u, x.blob_offset + x.up_rel) ||
      !s->read_at(o + g + u, d, x.blob_offset + x.down_rel))
    return sfail(SFK_ERR_RUNTIME, "%s: read of bundle (%d, %d) failed", s->path.c_str(), layer, expert);
  return SFK_OK;
}

SFK_API sfk_status sfk_strata_load(const sfk_strata* s, sfk_engine* eng) {
  if (!s || !eng) return sfail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  // every (layer, expert) needs its bundle: the HBM tier holds all of them
  const int64_t n_layer = s->key_int("llama.block_count", 0), n_expert = s->key_int("llama.expert_count", 0);
  for (int64_t l = 0; l < n_layer; ++l)
    for (int64_t e = 0; e < n_expert; ++e)
      if (!s->entry_of.count(((uint64_t)l << 32) | (uint64_t)e))
        return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: no bundle for layer %lld expert %lld", s->path.c_str(),
                     (long long)l, (long long)e);
  // an expert-parallel engine holds its own experts and, when the heads
  // split, its query / kv heads' rows of Q, K, V and its heads' columns of
  // the output projection (whole quant blocks: the split is 256-column aligned)
  sfk::EngineShard sh{};
  sfk::engine_shard(eng, &sh);
  std::vector<uint8_t> buf, part;
  for (const TensorInfo& t : s->tensors) {
    if (t.expert) continue;
    int tid, layer;
    if (!trunk_id(t.name, &tid, &layer))
      return sfail(SFK_ERR_UNSUPPORTED, "%s: trunk tensor %s has no place in this engine", s->path.c_str(),
                   t.name.c_str());
    buf.resize((size_t)t.nbytes);
    sfk_status st = sfk_strata_read_trunk(s, t.name.c_str(), buf.data(), buf.size());
    if (st) return st;
    int64_t ne[3] = {t.ne[0], t.ne[1], t.ne[2]};
    const uint8_t* src = buf.data();
    size_t n = buf.size();
    if (sh.head_split && (tid == SFK_T_ATTN_Q || tid == SFK_T_ATTN_K || tid == SFK_T_ATTN_V)) {
      const int64_t h0 = tid == SFK_T_ATTN_Q ? sh.q0 : sh.kv0, hn = tid == SFK_T_ATTN_Q ? sh.hq_loc : sh.hkv_loc;
      const uint64_t rowb = t.nbytes / (uint64_t)t.ne[1];  // one output row (head_dim rows per head)
      if ((h0 + hn) * sh.hd > t.ne[1])
        return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s has fewer heads than the engine", s->path.c_str(),
                     t.name.c_str());
      src = buf.data() + (uint64_t)(h0 * sh.hd) * rowb;
      n = (size_t)((uint64_t)(hn * sh.hd) * rowb);
      ne[1] = hn * sh.hd;
    } else if (sh.head_split && tid == SFK_T_ATTN_OUT) {
      int64_t blk, bb;
      type_block(t.type, &blk, &bb);
      const int64_t c0 = (int64_t)sh.q0 * sh.hd, cn = (int64_t)sh.hq_loc * sh.hd;
      if (c0 % blk || cn % blk || c0 + cn > t.ne[0])
        return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s columns do not split on quant blocks", s->path.c_str(),
                     t.name.c_str());
      const uint64_t rowb = (uint64_t)(t.ne[0] / blk * bb), off = (uint64_t)(c0 / blk * bb),
                     len = (uint64_t)(cn / blk * bb);
      part.resize((size_t)(len * (uint64_t)t.ne[1]));
      for (int64_t r = 0; r < t.ne[1]; ++r) memcpy(part.data() + r * len, buf.data() + r * rowb + off, len);
      src = part.data();
      n = part.size();
      ne[0] = cn;
    }
    if ((st = sfk_weights_put(eng, tid, layer, t.type, ne, src, n))) return st;
  }
  for (const ExpertEntry& x : s->index) {
    if ((int)x.expert < sh.e0 || (int)x.expert >= sh.e0 + sh.e_loc) continue;  // another rank's expert
    const size_t n = sfk_strata_bundle_bytes(s, (int32_t)x.layer);
    if (!n) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: layer %u has no expert tensors", s->path.c_str(), x.layer);
    buf.resize(n);
    sfk_status st = sfk_strata_read_bundle(s, (int32_t)x.layer, (int32_t)x.expert, buf.data(), n);
    if (st) return st;
    if ((st = sfk_expert_put(eng, (int)x.layer, (int)x.expert, buf.data(), n))) return st;
  }
  return SFK_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The packer: a GGUF checkpoint -> .strata, the reference's
// pack_gguf_to_strata (src/tws/strata_pack.h:16-46, strata_pack.cpp:251-1108)
// without its optional LZ compression.  Weight bytes are copied verbatim.
//   * Expert tensors are recognised by name: stacked blk.N.ffn_{gate,up,down}
//     _exps.weight (3-D, experts outermost) or legacy per-expert
//     blk.N.ffn_{gate,up,down}.E.weight; a file mixing the two, or one whose
//     metadata declares experts none of which are found, is refused.  Fused
//     gate_up expert tensors are refused (this library's bundles are
//     gate | up | down).
//   * Embedded metadata: the source's own header, key/values and tensor
//     infos verbatim (stacked input), or for legacy input a GGUF prefix built
//     here with the same key/values and stacked _exps tensor declarations.
//   * Layout: superblock (v2) | metadata | expert index | trunk block (4 KiB
//     aligned, every other tensor in source order, no padding) | expert
//     region (4 KiB aligned, one 4 KiB-aligned gate|up|down blob per (layer,
//     expert), layer-major) | trunk index (4 KiB aligned).
// ---------------------------------------------------------------------------
namespace {

constexpr uint64_t IO_ALIGN = 4096;

uint64_t align_up64(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct SrcTensor {
  std::string name;
  uint32_t nd = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  int type = 0;
  uint64_t off = 0;     // from the start of the source file
  uint64_t nbytes = 0;
  int kind = -1;        // expert kind 0 gate, 1 up, 2 down (or -1: trunk)
  int layer = -1, expert = -1;  // expert tensors; expert >= 0: a legacy per-expert tensor
  size_t info_begin = 0, info_end = 0;  // its tensor-info bytes in the source prefix
};

// blk.N.ffn_{gate,up,down}.E.weight -> (layer, kind, expert)
bool legacy_expert(const std::string& name, int* layer, int* kind, int* expert) {
  std::string suf;
  const int l = parse_layer(name, &suf);
  if (l < 0) return false;
  static const char* kinds[3] = {"ffn_gate.", "ffn_up.", "ffn_down."};
  for (int k = 0; k < 3; ++k) {
    const size_t n = strlen(kinds[k]);
    if (suf.compare(0, n, kinds[k]) != 0) continue;
    std::string rest = suf.substr(n);
    if (rest.size() < 8 || rest.compare(rest.size() - 7, 7, ".weight") != 0) return false;
    rest = rest.substr(0, rest.size() - 7);
    if (rest.empty() || rest.size() > 6) return false;
    int e = 0;
    for (char c : rest) {
      if (c < '0' || c > '9') return false;
      e = e * 10 + (c - '0');
    }
    *layer = l;
    *kind = k;
    *expert = e;
    return true;
  }
  return false;
}

int stacked_kind(const std::string& name, int* layer) {
  std::string suf;
  const int l = parse_layer(name, &suf);
  if (l < 0) return -1;
  *layer = l;
  if (suf == "ffn_gate_exps.weight") return 0;
  if (suf == "ffn_up_exps.weight") return 1;
  if (suf == "ffn_down_exps.weight") return 2;
  if (suf == "ffn_gate_up_exps.weight") return 3;
  return -1;
}

struct Out {
  int fd = -1;
  uint64_t pos = 0;
  bool ok = true;
  void write(const void* p, uint64_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    while (ok && n > 0) {
      const ssize_t w = ::write(fd, b, n > (1u << 30) ? (1u << 30) : (size_t)n);
      if (w <= 0) {
        ok = false;
        return;
      }
      b += w;
      n -= (uint64_t)w;
      pos += (uint64_t)w;
    }
  }
  void pad_to(uint64_t target) {
    static const uint8_t zeros[4096] = {};
    while (ok && pos < target) write(zeros, std::min<uint64_t>(sizeof(zeros), target - pos));
  }
  void pwrite_at(const void* p, uint64_t n, uint64_t off) {
    if (ok && ::pwrite(fd, p, (size_t)n, (off_t)off) != (ssize_t)n) ok = false;
  }
};

// copy [off, off + n) of `src` to the output
bool copy_range(int src, uint64_t off, uint64_t n, Out& o, std::vector<uint8_t>& buf) {
  while (o.ok && n > 0) {
    const size_t chunk = (size_t)std::min<uint64_t>(n, buf.size());
    size_t got = 0;
    while (got < chunk) {
      const ssize_t r = pread(src, buf.data() + got, chunk - got, (off_t)(off + got));
      if (r <= 0) return false;
      got += (size_t)r;
    }
    o.write(buf.data(), chunk);
    off += chunk;
    n -= chunk;
  }
  return o.ok;
}

void put_str(std::vector<uint8_t>& v, const std::string& s) {
  const uint64_t n = s.size();
  v.insert(v.end(), reinterpret_cast<const uint8_t*>(&n), reinterpret_cast<const uint8_t*>(&n) + 8);
  v.insert(v.end(), s.begin(), s.end());
}
template <typename T>
void put(std::vector<uint8_t>& v, T x) {
  v.insert(v.end(), reinterpret_cast<const uint8_t*>(&x), reinterpret_cast<const uint8_t*>(&x) + sizeof(T));
}

sfk_status pack(const char* in_path, const char* out_path) {
  const int src = open(in_path, O_RDONLY);
  if (src < 0) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: cannot open", in_path);
  struct Closer {
    int fd;
    ~Closer() { close(fd); }
  } src_closer{src};
  const off_t fsz = lseek(src, 0, SEEK_END);
  if (fsz < 24) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: not a GGUF file (too short)", in_path);
  const uint64_t file_size = (uint64_t)fsz;

  // the metadata prefix: read more of the file until it parses
  std::vector<uint8_t> pre;
  Cursor c{nullptr, 0};
  std::vector<SrcTensor> tensors;
  std::map<std::string, KV> kv;
  std::vector<std::pair<size_t, size_t>> kv_bytes;  // each key/value's bytes in the prefix
  uint64_t n_tensors = 0, n_kv = 0;
  uint32_t gguf_ver = 0;
  for (uint64_t want = std::min<uint64_t>(file_size, 1u << 22);; want = std::min<uint64_t>(file_size, want * 4)) {
    pre.resize((size_t)want);
    size_t got = 0;
    while (got < pre.size()) {
      const ssize_t r = pread(src, pre.data() + got, pre.size() - got, (off_t)got);
      if (r <= 0) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: read failed", in_path);
      got += (size_t)r;
    }
    c = Cursor{pre.data(), pre.size()};
    tensors.clear();
    kv.clear();
    kv_bytes.clear();
    const uint32_t magic = c.get<uint32_t>();
    gguf_ver = c.get<uint32_t>();
    n_tensors = c.get<uint64_t>();
    n_kv = c.get<uint64_t>();
    if (!c.ok || magic != 0x46554747u || (gguf_ver != 2 && gguf_ver != 3))
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: not a GGUF v2/v3 file", in_path);
    if (n_tensors > (1u << 24) || n_kv > (1u << 24))
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: GGUF counts out of range", in_path);
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
      const size_t b = c.off;
      std::string key = c.str();
      KV v;
      v.type = c.get<uint32_t>();
      if (!c.ok || !read_value(c, v.type, &v)) {
        c.ok = false;
        break;
      }
      kv[key] = v;
      kv_bytes.emplace_back(b, c.off);
    }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
      SrcTensor t;
      t.info_begin = c.off;
      t.name = c.str();
      t.nd = c.get<uint32_t>();
      if (!c.ok || t.nd < 1 || t.nd > 4) {
        if (c.ok) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor %llu has %u dims", in_path,
                               (unsigned long long)i, t.nd);
        break;
      }
      for (uint32_t d = 0; d < t.nd; ++d) t.ne[d] = (int64_t)c.get<uint64_t>();
      t.type = (int)c.get<uint32_t>();
      t.off = c.get<uint64_t>();
      t.info_end = c.off;
      tensors.push_back(t);
    }
    if (c.ok) break;
    if (want >= file_size) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: GGUF metadata truncated", in_path);
  }
  uint64_t alignment = 32;
  if (kv.count("general.alignment")) alignment = kv["general.alignment"].u;
  if (alignment == 0 || (alignment & (alignment - 1)))
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: general.alignment %llu", in_path, (unsigned long long)alignment);
  const uint64_t data_off = align_up64(c.off, alignment);
  std::string arch = "llama";
  if (kv.count("general.architecture") && kv["general.architecture"].type == G_STR)
    arch = kv["general.architecture"].s;
  auto key_u = [&](const std::string& k) -> uint64_t {
    auto it = kv.find(k);
    return it == kv.end() || it->second.type == G_STR || it->second.type == G_ARR || it->second.type == G_F32 ||
                   it->second.type == G_F64
               ? 0
               : it->second.u;
  };
  const uint64_t meta_experts = key_u(arch + ".expert_count");

  // classify
  int max_layer = -1, n_exp = 0;
  bool stacked = false, legacy = false;
  for (SrcTensor& t : tensors) {
    int64_t blk, bb;
    if (!type_block(t.type, &blk, &bb))
      return sfail(SFK_ERR_UNSUPPORTED, "%s: tensor %s has ggml type %d (F32, F16, Q8_0, Q4_K, Q6_K are packed)",
                   in_path, t.name.c_str(), t.type);
    bool shape_ok = t.ne[0] > 0 && t.ne[0] % blk == 0;
    for (int d = 0; d < 4; ++d) shape_ok = shape_ok && t.ne[d] > 0 && t.ne[d] < ((int64_t)1 << 31);
    if (!shape_ok) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor %s shape", in_path, t.name.c_str());
    t.nbytes = (uint64_t)(t.ne[0] / blk * bb) * (uint64_t)t.ne[1] * (uint64_t)t.ne[2] * (uint64_t)t.ne[3];
    if (t.off % alignment || data_off + t.off + t.nbytes > file_size || data_off + t.off < data_off)
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor %s lies outside the file", in_path, t.name.c_str());
    t.off += data_off;
    int l = -1, k = stacked_kind(t.name, &l), e = -1;
    if (k == 3)
      return sfail(SFK_ERR_UNSUPPORTED, "%s: fused gate_up expert tensor %s (bundles here are gate | up | down)",
                   in_path, t.name.c_str());
    if (k >= 0) {
      if (t.ne[2] < 1 || t.nbytes % (uint64_t)t.ne[2])
        return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: expert tensor %s is not 3-D with the experts outermost",
                     in_path, t.name.c_str());
      if (n_exp && n_exp != (int)t.ne[2])
        return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: expert tensors disagree on the expert count", in_path);
      n_exp = (int)t.ne[2];
      stacked = true;
    } else if (legacy_expert(t.name, &l, &k, &e)) {
      legacy = true;
    } else {
      continue;  // trunk
    }
    t.kind = k;
    t.layer = l;
    t.expert = e;
    max_layer = std::max(max_layer, l);
  }
  if (stacked && legacy)
    return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: stacked and per-expert expert tensors mixed", in_path);
  if (meta_experts > 0 && !stacked && !legacy)
    return sfail(SFK_ERR_INVALID_ARGUMENT,
                 "%s: the metadata declares %llu experts but no expert tensor was recognised by name", in_path,
                 (unsigned long long)meta_experts);
  const int n_layers = max_layer + 1;
  // expert tensors per (layer, kind[, expert])
  std::map<std::tuple<int, int, int>, const SrcTensor*> xt;
  if (legacy) {
    n_exp = (int)meta_experts;
    if (n_exp == 0)
      for (const SrcTensor& t : tensors)
        if (t.kind >= 0) n_exp = std::max(n_exp, t.expert + 1);
  }
  for (const SrcTensor& t : tensors) {
    if (t.kind < 0) continue;
    if (legacy && t.expert >= n_exp)
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s: expert %d of %d", in_path, t.name.c_str(), t.expert, n_exp);
    const auto key = std::make_tuple(t.layer, t.kind, legacy ? t.expert : 0);
    if (xt.count(key)) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s appears twice", in_path, t.name.c_str());
    xt[key] = &t;
  }
  for (int l = 0; l < n_layers; ++l)
    for (int k = 0; k < 3; ++k)
      for (int e = 0; e < (legacy ? n_exp : 1); ++e)
        if (!xt.count(std::make_tuple(l, k, e)))
          return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: layer %d lacks its %s expert tensor%s", in_path, l,
                       k == 0 ? "gate" : k == 1 ? "up" : "down", legacy ? "s" : "");
  if (legacy)  // every expert of a (layer, kind) must share a shape and type
    for (int l = 0; l < n_layers; ++l)
      for (int k = 0; k < 3; ++k) {
        const SrcTensor* a = xt[std::make_tuple(l, k, 0)];
        for (int e = 1; e < n_exp; ++e) {
          const SrcTensor* b = xt[std::make_tuple(l, k, e)];
          if (b->type != a->type || b->nbytes != a->nbytes || b->ne[0] != a->ne[0] || b->ne[1] != a->ne[1])
            return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: %s differs from %s", in_path, b->name.c_str(),
                         a->name.c_str());
        }
      }
  for (const SrcTensor& t : tensors)
    if (t.kind < 0 && t.name.size() >= 64)
      return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: tensor name %s is too long for the trunk index", in_path,
                   t.name.c_str());

  // embedded metadata
  std::vector<uint8_t> meta;
  if (!legacy) {
    meta.assign(pre.begin(), pre.begin() + (size_t)std::min<uint64_t>(data_off, pre.size()));
    meta.resize((size_t)data_off, 0);  // the alignment padding (zeros)
  } else {
    uint64_t nt = 0;
    for (const SrcTensor& t : tensors) nt += t.kind < 0 ? 1 : 0;
    nt += (uint64_t)n_layers * 3;
    put<uint32_t>(meta, 0x46554747u);
    put<uint32_t>(meta, 3);
    put<uint64_t>(meta, nt);
    put<uint64_t>(meta, n_kv);
    for (const auto& b : kv_bytes) meta.insert(meta.end(), pre.begin() + b.first, pre.begin() + b.second);
    uint64_t doff = 0;
    auto info = [&](const std::string& name, uint32_t nd, const int64_t* ne, int type, uint64_t nbytes) {
      put_str(meta, name);
      put<uint32_t>(meta, nd);
      for (uint32_t d = 0; d < nd; ++d) put<uint64_t>(meta, (uint64_t)ne[d]);
      put<uint32_t>(meta, (uint32_t)type);
      put<uint64_t>(meta, doff);
      doff = align_up64(doff + nbytes, alignment);
    };
    for (const SrcTensor& t : tensors)
      if (t.kind < 0) info(t.name, t.nd, t.ne, t.type, t.nbytes);
    static const char* sfx[3] = {"ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"};
    for (int l = 0; l < n_layers; ++l)
      for (int k : {0, 2, 1}) {  // llama.cpp's per-block order: gate, down, up
        const SrcTensor* a = xt[std::make_tuple(l, k, 0)];
        const int64_t ne[3] = {a->ne[0], a->ne[1], n_exp};
        info("blk." + std::to_string(l) + "." + sfx[k], 3, ne, a->type, a->nbytes * (uint64_t)n_exp);
      }
    meta.resize((size_t)align_up64(meta.size(), alignment), 0);
  }

  Out o;
  o.fd = open(out_path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
  if (o.fd < 0) return sfail(SFK_ERR_INVALID_ARGUMENT, "%s: cannot create", out_path);
  struct Cleanup {
    Out& o;
    const char* path;
    bool keep = false;
    ~Cleanup() {
      close(o.fd);
      if (!keep) unlink(path);
    }
  } cleanup{o, out_path};
  std::vector<uint8_t> buf(64u << 20);
  const uint8_t zsb[SB_SIZE] = {};
  o.write(zsb, SB_SIZE);
  const uint64_t meta_off = o.pos;
  o.write(meta.data(), meta.size());
  const uint64_t index_off = o.pos, n_index = (uint64_t)n_layers * (uint64_t)n_exp;
  std::vector<uint8_t> index((size_t)(n_index * INDEX_ENTRY), 0);
  o.write(index.data(), index.size());
  o.pad_to(align_up64(o.pos, IO_ALIGN));
  const uint64_t trunk_off = o.pos;
  std::vector<uint8_t> tix;
  uint64_t n_trunk = 0;
  for (const SrcTensor& t : tensors) {
    if (t.kind >= 0) continue;
    uint8_t e[TRUNK_ENTRY] = {};
    memcpy(e, t.name.data(), t.name.size());
    const uint64_t rel = o.pos - trunk_off;
    memcpy(e + 64, &rel, 8);
    memcpy(e + 72, &t.nbytes, 8);
    tix.insert(tix.end(), e, e + TRUNK_ENTRY);
    ++n_trunk;
    if (!copy_range(src, t.off, t.nbytes, o, buf))
      return sfail(SFK_ERR_RUNTIME, "%s: copying %s failed", out_path, t.name.c_str());
  }
  const uint64_t trunk_size = o.pos - trunk_off;
  o.pad_to(align_up64(o.pos, IO_ALIGN));
  const uint64_t expert_off = o.pos;
  size_t ii = 0;
  for (int l = 0; l < n_layers; ++l)
    for (int e = 0; e < n_exp; ++e, ++ii) {
      o.pad_to(align_up64(o.pos, IO_ALIGN));
      const uint64_t blob = o.pos;
      uint64_t rel[3] = {};
      for (int k = 0; k < 3; ++k) {
        rel[k] = o.pos - blob;
        const SrcTensor* t = xt[std::make_tuple(l, k, legacy ? e : 0)];
        const uint64_t per = legacy ? t->nbytes : t->nbytes / (uint64_t)n_exp;
        const uint64_t off = legacy ? t->off : t->off + (uint64_t)e * per;
        if (!copy_range(src, off, per, o, buf))
          return sfail(SFK_ERR_RUNTIME, "%s: copying expert (%d, %d) failed", out_path, l, e);
      }
      uint8_t* x = index.data() + ii * INDEX_ENTRY;
      const uint32_t lu = (uint32_t)l, eu = (uint32_t)e;
      const uint64_t len = o.pos - blob;
      memcpy(x, &lu, 4);
      memcpy(x + 4, &eu, 4);
      memcpy(x + 8, &blob, 8);
      memcpy(x + 16, &len, 8);
      memcpy(x + 24, &rel[0], 8);
      memcpy(x + 32, &rel[1], 8);
      memcpy(x + 40, &rel[2], 8);
    }
  const uint64_t expert_size = o.pos - expert_off;
  uint64_t tix_off = 0;
  if (n_trunk) {
    o.pad_to(align_up64(o.pos, IO_ALIGN));
    tix_off = o.pos;
    o.write(tix.data(), tix.size());
  }
  o.pwrite_at(index.data(), index.size(), index_off);
  // superblock (v2): magic, version, flags, eight offsets / sizes, the trunk
  // index, n_layers, n_experts, alignment, then the CRC of all of it
  uint8_t sb[SB_SIZE] = {};
  const uint32_t ver = 2, flags = 1u | 2u | (n_trunk ? 4u : 0u), al = (uint32_t)IO_ALIGN;
  const uint32_t nl = (uint32_t)n_layers, ne = (uint32_t)n_exp;
  const uint64_t meta_size = meta.size();
  memcpy(sb, MAGIC, 8);
  memcpy(sb + 8, &ver, 4);
  memcpy(sb + 12, &flags, 4);
  const uint64_t f8[8] = {meta_off, meta_size, index_off, n_index, trunk_off, trunk_size, expert_off, expert_size};
  memcpy(sb + 16, f8, sizeof(f8));
  memcpy(sb + 80, &tix_off, 8);
  memcpy(sb + 88, &n_trunk, 8);
  memcpy(sb + 96, &nl, 4);
  memcpy(sb + 100, &ne, 4);
  memcpy(sb + 104, &al, 4);
  const uint32_t crc = crc32_ieee(sb, 108);
  memcpy(sb + 108, &crc, 4);
  o.pwrite_at(sb, SB_SIZE, 0);
  if (!o.ok) return sfail(SFK_ERR_RUNTIME, "%s: write failed", out_path);
  cleanup.keep = true;
  return SFK_OK;
}

}  // namespace

extern "C" SFK_API sfk_status sfk_strata_pack(const char* gguf_path, const char* strata_path) {
  if (!gguf_path || !strata_path) return sfail(SFK_ERR_INVALID_ARGUMENT, "null path");
  try {
    return pack(gguf_path, strata_path);
  } catch (const std::bad_alloc&) {
    return sfail(SFK_ERR_OUT_OF_MEMORY, "%s: host allocation failed", gguf_path);
  }
}
