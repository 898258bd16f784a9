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

#include <array>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
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
