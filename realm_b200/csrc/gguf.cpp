// GGUF reader and device model loader.
//
// The parser follows GGUFParser (crates/realm-core/src/formats/gguf.rs:100-479)
// over a read-only mapping of the file: header, metadata key/values and
// tensor infos are decoded once into tables that point into the mapping, so
// tensor bytes are never copied on the host. rb_model_load_gguf then uploads
// each tensor straight from the mapping into a model (Model::load_from_gguf,
// crates/realm-models/src/model.rs:291-540).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/realm_b200.h"

namespace rb {
int fail(int code, const char* fmt, ...);
}
using rb::fail;

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF", little-endian
constexpr uint64_t kDefaultAlignment = 32;

// Elements and bytes of one block of a ggml type (the published GGUF / ggml
// block layouts); {0, 0} for types this library does not know.
struct BlockSize {
  uint32_t elems, bytes;
};
BlockSize ggml_block(int32_t t) {
  switch (t) {
    case 0: return {1, 4};      // F32
    case 1: return {1, 2};      // F16
    case 2: return {32, 18};    // Q4_0
    case 3: return {32, 20};    // Q4_1
    case 6: return {32, 22};    // Q5_0
    case 7: return {32, 24};    // Q5_1
    case 8: return {32, 34};    // Q8_0
    case 9: return {32, 36};    // Q8_1
    case 10: return {256, 84};  // Q2_K
    case 11: return {256, 110}; // Q3_K
    case 12: return {256, 144}; // Q4_K
    case 13: return {256, 176}; // Q5_K
    case 14: return {256, 210}; // Q6_K
    case 15: return {256, 292}; // Q8_K
    case 24: return {1, 1};     // I8
    case 25: return {1, 2};     // I16
    case 26: return {1, 4};     // I32
    case 27: return {1, 8};     // I64
    case 28: return {1, 8};     // F64
    case 30: return {1, 2};     // BF16
    default: return {0, 0};
  }
}

// Size of a fixed-size metadata scalar, 0 for strings / arrays / unknown.
uint32_t scalar_bytes(int32_t t) {
  switch (t) {
    case RB_GGUF_U8: case RB_GGUF_I8: case RB_GGUF_BOOL: return 1;
    case RB_GGUF_U16: case RB_GGUF_I16: return 2;
    case RB_GGUF_U32: case RB_GGUF_I32: case RB_GGUF_F32: return 4;
    case RB_GGUF_U64: case RB_GGUF_I64: case RB_GGUF_F64: return 8;
    default: return 0;
  }
}

struct Str {
  const char* p = nullptr;
  uint64_t n = 0;
};

struct Meta {
  std::string key;
  int32_t type = 0;
  const uint8_t* scalar = nullptr;  // fixed-size scalar value
  Str str;                          // string value
  int32_t elem_type = -1;           // arrays
  uint64_t length = 0;
  const uint8_t* elems = nullptr;   // fixed-size array elements
  std::vector<Str> strs;            // string array elements
};

struct Tensor {
  std::string name;
  int32_t dtype = 0;
  uint32_t n_dims = 0;
  uint64_t dims[4] = {1, 1, 1, 1};
  uint64_t offset = 0, nbytes = 0;
};

// Well-formed UTF-8 (RFC 3629: no overlong forms, no surrogates, <= U+10FFFF),
// the check String::from_utf8 makes on every GGUF string (gguf.rs:302-307).
bool valid_utf8(const uint8_t* s, uint64_t n) {
  uint64_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    int len;
    uint32_t cp, min;
    if ((c & 0xE0) == 0xC0) len = 2, cp = c & 0x1F, min = 0x80;
    else if ((c & 0xF0) == 0xE0) len = 3, cp = c & 0x0F, min = 0x800;
    else if ((c & 0xF8) == 0xF0) len = 4, cp = c & 0x07, min = 0x10000;
    else return false;
    if (n - i < (uint64_t)len) return false;
    for (int k = 1; k < len; ++k) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// Bounds-checked little-endian reader over the mapping.
struct Reader {
  const uint8_t* base;
  uint64_t size, pos = 0;
  int err = 0;

  bool need(uint64_t n) {
    if (err) return false;
    if (n > size - pos) {
      err = fail(RB_ERR_IO, "unexpected end of GGUF data at byte %llu (need %llu more)", (unsigned long long)pos,
                 (unsigned long long)n);
      return false;
    }
    return true;
  }
  template <class T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      std::memcpy(&v, base + pos, sizeof(T));
      pos += sizeof(T);
    }
    return v;
  }
  Str str() {
    Str s;
    const uint64_t n = get<uint64_t>();
    if (!need(n)) return s;
    if (!valid_utf8(base + pos, n)) {
      err = fail(RB_ERR_INVALID, "Invalid UTF-8 in the string at byte %llu", (unsigned long long)pos);
      return s;
    }
    s.p = reinterpret_cast<const char*>(base + pos);
    s.n = n;
    pos += n;
    return s;
  }
  const uint8_t* skip(uint64_t n) {
    if (!need(n)) return nullptr;
    const uint8_t* p = base + pos;
    pos += n;
    return p;
  }
};

}  // namespace

struct rb_gguf {
  const uint8_t* data = nullptr;
  uint64_t size = 0;
  bool mapped = false;
  uint32_t version = 0;
  uint64_t data_offset = 0;
  std::vector<Meta> meta;
  std::unordered_map<std::string, uint32_t> meta_index;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, uint32_t> tensor_index;

  ~rb_gguf() {
    if (mapped && data) munmap(const_cast<uint8_t*>(data), size);
  }
};

namespace {

int parse_value(Reader& r, int32_t type, Meta& m) {
  if (const uint32_t b = scalar_bytes(type)) {
    m.scalar = r.skip(b);
    return r.err;
  }
  if (type == RB_GGUF_STRING) {
    m.str = r.str();
    return r.err;
  }
  if (type == RB_GGUF_ARRAY) {
    m.elem_type = (int32_t)r.get<uint32_t>();
    m.length = r.get<uint64_t>();
    if (r.err) return r.err;
    if (const uint32_t b = scalar_bytes(m.elem_type)) {
      if (m.length > (r.size - r.pos) / b)
        return r.err = fail(RB_ERR_IO, "unexpected end of GGUF data in array %s", m.key.c_str());
      m.elems = r.skip(m.length * b);
      return r.err;
    }
    if (m.elem_type == RB_GGUF_STRING) {
      if (m.length > (r.size - r.pos) / 8)
        return r.err = fail(RB_ERR_IO, "unexpected end of GGUF data in array %s", m.key.c_str());
      m.strs.resize(m.length);
      for (uint64_t i = 0; i < m.length && !r.err; ++i) m.strs[i] = r.str();
      return r.err;
    }
    return fail(RB_ERR_INVALID, "Unknown typed value: %d", m.elem_type);
  }
  return fail(RB_ERR_INVALID, "Unknown metadata value type: %d", type);
}

int parse(rb_gguf& g) {
  Reader r{g.data, g.size};
  const uint32_t magic = r.get<uint32_t>();
  if (r.err) return r.err;
  if (magic != kMagic) return fail(RB_ERR_INVALID, "Invalid GGUF magic: 0x%08X", magic);
  g.version = r.get<uint32_t>();
  if (r.err) return r.err;
  if (g.version < 2 || g.version > 3) return fail(RB_ERR_INVALID, "Unsupported GGUF version: %u", g.version);
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_meta = r.get<uint64_t>();
  if (r.err) return r.err;
  // every entry takes at least 12 bytes: a count beyond that is a corrupt header
  if (n_meta > g.size / 12 || n_tensors > g.size / 12)
    return fail(RB_ERR_INVALID, "GGUF counts out of range: %llu tensors, %llu metadata entries",
                (unsigned long long)n_tensors, (unsigned long long)n_meta);
  g.meta.resize(n_meta);
  for (uint64_t i = 0; i < n_meta; ++i) {
    Meta& m = g.meta[i];
    const Str k = r.str();
    if (r.err) return r.err;
    m.key.assign(k.p, k.n);
    m.type = (int32_t)r.get<uint32_t>();
    if (r.err) return r.err;
    if (int rc = parse_value(r, m.type, m)) return rc;
    g.meta_index[m.key] = (uint32_t)i;  // a repeated key keeps its last value (HashMap::insert)
  }
  g.tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    Tensor& t = g.tensors[i];
    const Str nm = r.str();
    t.n_dims = r.get<uint32_t>();
    if (r.err) return r.err;
    t.name.assign(nm.p, nm.n);
    if (t.n_dims == 0 || t.n_dims > 4) return fail(RB_ERR_INVALID, "tensor %s: %u dimensions", t.name.c_str(), t.n_dims);
    for (uint32_t d = 0; d < t.n_dims; ++d) t.dims[d] = r.get<uint64_t>();
    t.dtype = (int32_t)r.get<uint32_t>();
    t.offset = r.get<uint64_t>();
    if (r.err) return r.err;
    uint64_t numel = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      if (t.dims[d] == 0 || numel > (1ull << 62) / t.dims[d]) return fail(RB_ERR_INVALID, "tensor %s: bad shape", t.name.c_str());
      numel *= t.dims[d];
    }
    const BlockSize b = ggml_block(t.dtype);
    if (b.elems) {
      if (t.dims[0] % b.elems)
        return fail(RB_ERR_INVALID, "tensor %s: row of %llu elements is not whole %u-element blocks", t.name.c_str(),
                    (unsigned long long)t.dims[0], b.elems);
      t.nbytes = numel / b.elems * b.bytes;
    }
    g.tensor_index[t.name] = (uint32_t)i;
  }
  uint64_t align = kDefaultAlignment;
  if (auto it = g.meta_index.find("general.alignment"); it != g.meta_index.end()) {
    const Meta& m = g.meta[it->second];
    uint32_t a = 0;
    if (m.type == RB_GGUF_U32) std::memcpy(&a, m.scalar, 4);
    if (a == 0 || (a & (a - 1))) return fail(RB_ERR_INVALID, "general.alignment must be a power of two u32");
    align = a;
  }
  g.data_offset = (r.pos + align - 1) / align * align;
  for (const Tensor& t : g.tensors) {
    if (t.offset % align) return fail(RB_ERR_INVALID, "tensor %s: offset %llu not a multiple of %llu", t.name.c_str(),
                                      (unsigned long long)t.offset, (unsigned long long)align);
    if (g.data_offset > g.size || t.offset > g.size - g.data_offset || t.nbytes > g.size - g.data_offset - t.offset)
      return fail(RB_ERR_IO, "tensor %s: bytes [%llu, +%llu) beyond the end of the file (%llu bytes)", t.name.c_str(),
                  (unsigned long long)(g.data_offset + t.offset), (unsigned long long)t.nbytes,
                  (unsigned long long)g.size);
  }
  return RB_OK;
}

const Meta* meta_at(rb_gguf* g, uint32_t i) { return (g && i < g->meta.size()) ? &g->meta[i] : nullptr; }

template <class T>
T load(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof v);
  return v;
}

bool meta_u32(const Meta& m, uint32_t& out) {
  switch (m.type) {
    case RB_GGUF_U8: out = load<uint8_t>(m.scalar); return true;
    case RB_GGUF_U16: out = load<uint16_t>(m.scalar); return true;
    case RB_GGUF_U32: out = load<uint32_t>(m.scalar); return true;
    case RB_GGUF_U64: out = (uint32_t)load<uint64_t>(m.scalar); return true;
    case RB_GGUF_I8: out = (uint32_t)(int32_t)load<int8_t>(m.scalar); return true;
    case RB_GGUF_I16: out = (uint32_t)(int32_t)load<int16_t>(m.scalar); return true;
    case RB_GGUF_I32: out = (uint32_t)load<int32_t>(m.scalar); return true;
    case RB_GGUF_I64: out = (uint32_t)load<int64_t>(m.scalar); return true;
    default: return false;
  }
}

bool meta_f32(const Meta& m, float& out) {
  if (m.type == RB_GGUF_F32) out = load<float>(m.scalar);
  else if (m.type == RB_GGUF_F64) out = (float)load<double>(m.scalar);
  else return false;
  return true;
}

}  // namespace

extern "C" {

int32_t rb_gguf_open_memory(const void* bytes, size_t nbytes, rb_gguf** out) {
  if (!out || (!bytes && nbytes)) return fail(RB_ERR_INVALID, "null argument");
  auto* g = new rb_gguf;
  g->data = static_cast<const uint8_t*>(bytes);
  g->size = nbytes;
  if (int rc = parse(*g)) {
    delete g;
    return rc;
  }
  *out = g;
  return RB_OK;
}

int32_t rb_gguf_open(const char* path, rb_gguf** out) {
  if (!path || !out) return fail(RB_ERR_INVALID, "null argument");
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(RB_ERR_IO, "cannot open %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return fail(RB_ERR_IO, "cannot stat %s", path);
  }
  void* p = nullptr;
  if (st.st_size > 0) {
    p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
      close(fd);
      return fail(RB_ERR_IO, "cannot map %s: %s", path, strerror(errno));
    }
  }
  close(fd);
  auto* g = new rb_gguf;
  g->data = static_cast<const uint8_t*>(p);
  g->size = (uint64_t)st.st_size;
  g->mapped = p != nullptr;
  if (int rc = parse(*g)) {
    delete g;
    return rc;
  }
  *out = g;
  return RB_OK;
}

int32_t rb_gguf_close(rb_gguf* g) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  delete g;
  return RB_OK;
}

int32_t rb_gguf_version(rb_gguf* g) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  return (int32_t)g->version;
}

int32_t rb_gguf_data_offset(rb_gguf* g, uint64_t* out) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  *out = g->data_offset;
  return RB_OK;
}

int32_t rb_gguf_tensor_count(rb_gguf* g) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  return (int32_t)g->tensors.size();
}

int32_t rb_gguf_tensor_info(rb_gguf* g, uint32_t i, rb_gguf_tensor* out) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  if (i >= g->tensors.size()) return fail(RB_ERR_OUT_OF_BOUNDS, "tensor %u of %zu", i, g->tensors.size());
  const Tensor& t = g->tensors[i];
  out->name = t.name.c_str();
  out->dtype = t.dtype;
  out->n_dims = t.n_dims;
  std::memcpy(out->dims, t.dims, sizeof out->dims);
  out->offset = t.offset;
  out->file_offset = g->data_offset + t.offset;
  out->nbytes = t.nbytes;
  out->data = g->data ? g->data + g->data_offset + t.offset : nullptr;
  return RB_OK;
}

int32_t rb_gguf_find_tensor(rb_gguf* g, const char* name) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  if (!name) return fail(RB_ERR_INVALID, "null name");
  auto it = g->tensor_index.find(name);
  if (it == g->tensor_index.end()) return fail(RB_ERR_NOT_FOUND, "Tensor not found: %s", name);
  return (int32_t)it->second;
}

int32_t rb_gguf_meta_count(rb_gguf* g) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  return (int32_t)g->meta.size();
}

int32_t rb_gguf_meta_entry(rb_gguf* g, uint32_t i, const char** key, int32_t* type, int32_t* elem_type,
                           uint64_t* length) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m) return fail(RB_ERR_OUT_OF_BOUNDS, "metadata entry %u of %zu", i, g->meta.size());
  if (key) *key = m->key.c_str();
  if (type) *type = m->type;
  if (elem_type) *elem_type = m->elem_type;
  if (length) *length = m->length;
  return RB_OK;
}

int32_t rb_gguf_meta_find(rb_gguf* g, const char* key) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  if (!key) return fail(RB_ERR_INVALID, "null key");
  auto it = g->meta_index.find(key);
  if (it == g->meta_index.end()) return fail(RB_ERR_NOT_FOUND, "metadata key not found: %s", key);
  return (int32_t)it->second;
}

int32_t rb_gguf_meta_u32(rb_gguf* g, uint32_t i, uint32_t* out) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m || !out) return fail(RB_ERR_INVALID, "metadata entry %u", i);
  if (!meta_u32(*m, *out)) return fail(RB_ERR_INVALID, "%s is not an integer", m->key.c_str());
  return RB_OK;
}

int32_t rb_gguf_meta_f32(rb_gguf* g, uint32_t i, float* out) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m || !out) return fail(RB_ERR_INVALID, "metadata entry %u", i);
  if (!meta_f32(*m, *out)) return fail(RB_ERR_INVALID, "%s is not a float", m->key.c_str());
  return RB_OK;
}

int32_t rb_gguf_meta_scalar(rb_gguf* g, uint32_t i, void* out, size_t cap) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m || !out) return fail(RB_ERR_INVALID, "metadata entry %u", i);
  const uint32_t n = scalar_bytes(m->type);
  if (!n) return fail(RB_ERR_INVALID, "%s is not a scalar", m->key.c_str());
  if (cap < n) return fail(RB_ERR_INVALID, "%s: %u bytes do not fit in %zu", m->key.c_str(), n, cap);
  std::memcpy(out, m->scalar, n);
  return (int32_t)n;
}

int32_t rb_gguf_meta_string(rb_gguf* g, uint32_t i, int64_t elem, const char** str, uint64_t* len) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m || !str || !len) return fail(RB_ERR_INVALID, "metadata entry %u", i);
  Str s;
  if (elem < 0) {
    if (m->type != RB_GGUF_STRING) return fail(RB_ERR_INVALID, "%s is not a string", m->key.c_str());
    s = m->str;
  } else {
    if (m->type != RB_GGUF_ARRAY || m->elem_type != RB_GGUF_STRING)
      return fail(RB_ERR_INVALID, "%s is not a string array", m->key.c_str());
    if ((uint64_t)elem >= m->length) return fail(RB_ERR_OUT_OF_BOUNDS, "%s[%lld]", m->key.c_str(), (long long)elem);
    s = m->strs[elem];
  }
  *str = s.p;
  *len = s.n;
  return RB_OK;
}

int32_t rb_gguf_meta_array_data(rb_gguf* g, uint32_t i, const void** data) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  const Meta* m = meta_at(g, i);
  if (!m || !data) return fail(RB_ERR_INVALID, "metadata entry %u", i);
  if (m->type != RB_GGUF_ARRAY || !scalar_bytes(m->elem_type))
    return fail(RB_ERR_INVALID, "%s is not a numeric array", m->key.c_str());
  *data = m->elems;
  return RB_OK;
}

int32_t rb_gguf_model_config(rb_gguf* g, rb_model_config* out) {
  if (!g) return fail(RB_ERR_BAD_HANDLE, "null gguf");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  std::string arch = "unknown";
  if (auto it = g->meta_index.find("general.architecture"); it != g->meta_index.end()) {
    const Meta& m = g->meta[it->second];
    if (m.type == RB_GGUF_STRING) arch.assign(m.str.p, m.str.n);
  }
  // first present key that converts, else the default (gguf.rs:219-285)
  auto u32 = [&](const char* a, const char* b, bool b_arch, uint32_t def) {
    for (const std::string& k : {arch + "." + a, b_arch ? arch + "." + b : std::string(b)}) {
      auto it = g->meta_index.find(k);
      uint32_t v;
      if (it != g->meta_index.end()) return meta_u32(g->meta[it->second], v) ? v : def;
    }
    return def;
  };
  auto f32 = [&](const char* a, const char* b, float def) {
    for (const std::string& k : {arch + "." + a, std::string(b)}) {
      auto it = g->meta_index.find(k);
      float v;
      if (it != g->meta_index.end()) return meta_f32(g->meta[it->second], v) ? v : def;
    }
    return def;
  };
  std::memset(out, 0, sizeof *out);
  out->vocab = u32("vocab_size", "vocab_size", false, 32000);
  out->hidden = u32("embedding_length", "hidden_size", true, 2048);
  out->n_layers = u32("block_count", "num_layers", true, 22);
  out->n_heads = u32("attention.head_count", "num_heads", true, 32);
  out->n_kv_heads = u32("attention.head_count_kv", "num_kv_heads", true, 4);
  out->ffn = u32("feed_forward_length", "intermediate_size", true, 5632);
  out->max_seq = u32("context_length", "max_seq_len", true, 2048);
  out->rms_eps = f32("attention.layer_norm_rms_epsilon", "rms_norm_eps", 1e-5f);
  out->layer_eps = out->rms_eps;
  out->rope_theta = f32("rope.freq_base", "rope_theta", 10000.0f);
  out->head_dim = out->n_heads ? out->hidden / out->n_heads : 0;
  return RB_OK;
}

int32_t rb_model_load_gguf(rb_ctx* ctx, rb_gguf* g, const rb_model_config* cfg, int32_t* model) {
  if (!ctx || !g || !cfg || !model) return fail(RB_ERR_BAD_HANDLE, "null argument");
  const rb_model_config& c = *cfg;
  auto find = [&](const std::string& name) -> const Tensor* {
    auto it = g->tensor_index.find(name);
    return it == g->tensor_index.end() ? nullptr : &g->tensors[it->second];
  };
  struct Item {
    int32_t which, layer;
    const Tensor* t;
    uint64_t rows, cols;  // expected
  };
  std::vector<Item> items;
  const Tensor* embd = find("token_embd.weight");
  if (!embd) return fail(RB_ERR_NOT_FOUND, "Missing token embeddings (token_embd.weight)");
  const Tensor* onorm = find("output_norm.weight");
  if (!onorm) return fail(RB_ERR_NOT_FOUND, "Tensor not found: output_norm.weight");
  const Tensor* out = find("output.weight");
  if (!out) out = find("lm_head.weight");
  if (!out) out = embd;  // tied: the LM head reads the embedding table as [vocab][hidden]
  const uint64_t H = c.hidden, Q = (uint64_t)c.n_heads * c.head_dim, KV = (uint64_t)c.n_kv_heads * c.head_dim;
  items.push_back({RB_W_TOKEN_EMBD, -1, embd, c.vocab, H});
  items.push_back({RB_W_OUTPUT_NORM, -1, onorm, 1, H});
  items.push_back({RB_W_OUTPUT, -1, out, c.vocab, H});
  static const struct { int32_t which; const char* name; } kLayer[] = {
      {RB_W_ATTN_NORM, "attn_norm"}, {RB_W_Q, "attn_q"},     {RB_W_K, "attn_k"},
      {RB_W_V, "attn_v"},           {RB_W_O, "attn_output"}, {RB_W_FFN_NORM, "ffn_norm"},
      {RB_W_GATE, "ffn_gate"},      {RB_W_UP, "ffn_up"},     {RB_W_DOWN, "ffn_down"}};
  for (uint32_t l = 0; l < c.n_layers; ++l)
    for (const auto& e : kLayer) {
      const std::string name = "blk." + std::to_string(l) + "." + e.name + ".weight";
      const Tensor* t = find(name);
      if (!t) return fail(RB_ERR_NOT_FOUND, "Tensor not found: %s", name.c_str());
      uint64_t rows = 1, cols = H;
      switch (e.which) {
        case RB_W_Q: rows = Q; break;
        case RB_W_K: case RB_W_V: rows = KV; break;
        case RB_W_O: rows = H; cols = Q; break;
        case RB_W_GATE: case RB_W_UP: rows = c.ffn; break;
        case RB_W_DOWN: rows = H; cols = c.ffn; break;
        default: break;
      }
      items.push_back({e.which, (int32_t)l, t, rows, cols});
    }
  for (const Item& it : items) {
    const Tensor& t = *it.t;
    const uint64_t rows = t.n_dims >= 2 ? t.dims[1] : 1;
    bool ok = t.dims[0] == it.cols && rows == it.rows;
    for (uint32_t d = 2; d < t.n_dims; ++d) ok = ok && t.dims[d] == 1;
    if (!ok)
      return fail(RB_ERR_INVALID, "%s: shape [%llu, %llu] in the file, [%llu, %llu] expected from the config",
                  t.name.c_str(), (unsigned long long)t.dims[0], (unsigned long long)rows,
                  (unsigned long long)it.cols, (unsigned long long)it.rows);
  }
  int32_t h = -1;
  if (int rc = rb_model_create(ctx, cfg, &h)) return rc;
  for (const Item& it : items) {
    const Tensor& t = *it.t;
    const uint8_t* src = g->data + g->data_offset + t.offset;
    const bool norm = it.which == RB_W_OUTPUT_NORM || it.which == RB_W_ATTN_NORM || it.which == RB_W_FFN_NORM;
    int rc;
    if (norm && t.dtype == RB_F16) {
      std::vector<float> w(it.cols);
      for (uint64_t i = 0; i < it.cols; ++i) {
        // binary16 -> binary32, exact (IEEE 754 widening)
        const uint16_t b = load<uint16_t>(src + 2 * i);
        const uint32_t sign = (uint32_t)(b >> 15) << 31, e = (b >> 10) & 31, f = b & 1023;
        float v;
        if (e == 0) v = std::ldexp((float)f, -24);
        else if (e == 31) v = f ? NAN : INFINITY;
        else v = std::ldexp((float)(f | 1024), (int)e - 25);
        uint32_t bits;
        std::memcpy(&bits, &v, 4);
        bits |= sign;
        std::memcpy(&w[i], &bits, 4);
      }
      rc = rb_model_set_weight(ctx, h, it.which, it.layer, RB_F32, w.data(), w.size() * 4, RB_PTR_HOST);
    } else {
      rc = rb_model_set_weight(ctx, h, it.which, it.layer, t.dtype, src, t.nbytes, RB_PTR_HOST);
    }
    if (rc < 0) {
      std::string msg = t.name;  // keep the tensor's name in the message
      char buf[512];
      rb_last_error(buf, sizeof buf);
      msg += ": ";
      msg += buf;
      rb_model_destroy(ctx, h);
      return fail(rc, "%s", msg.c_str());
    }
  }
  if (int rc = rb_model_finalize(ctx, h)) {
    rb_model_destroy(ctx, h);
    return rc;
  }
  *model = h;
  return RB_OK;
}

}  // extern "C"
