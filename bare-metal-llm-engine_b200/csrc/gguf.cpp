// gguf.cpp -- read-only GGUF model files, memory-mapped, feeding the projections.
//
// The engine plans a GGUF-style mmap'd loader whose ~50 weight tensors alias one
// mapped region (README.md:247, Module 7; include/engine/tensor.hpp:19-23) but
// has none.  This is its read side for the weights the projections consume.
//
// Layout of a GGUF file (versions 2 and 3; all integers little-endian):
//   u32 magic "GGUF", u32 version, u64 tensor_count, u64 metadata_kv_count;
//   metadata: { string key, u32 value_type, value } x kv_count, where a string
//     is { u64 length, bytes } and an array is { u32 elem_type, u64 count,
//     elements };
//   tensor table: { string name, u32 n_dims, u64 dims[n_dims], u32 ggml_type,
//     u64 offset } x tensor_count;
//   padding to general.alignment (default 32), then the tensor data, each
//     tensor at its offset (a multiple of the alignment) from that point.
// Every read goes through a cursor that checks the remaining length first, so
// a malformed or truncated file is an ENGINE_ERR_FORMAT, never an out-of-range
// read.  Tensor data is not copied: a tensor is a pointer into the mapping.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "host.h"

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr uint64_t kDefaultAlign = 32;
constexpr size_t kChunk = size_t(16) << 20;  // pinned bounce buffer, bytes

// Block size (elements) and block bytes of the GGML types with fixed-size
// blocks; 0 marks a code the loader does not know (its tensors get nbytes 0).
struct TypeSize {
  int32_t block;
  int32_t bytes;
};
TypeSize ggml_type_size(uint32_t t) {
  switch (t) {
    case 0: return {1, 4};       // F32
    case 1: return {1, 2};       // F16
    case 2: return {32, 18};     // Q4_0: f16 d, 16 nibble bytes
    case 3: return {32, 20};     // Q4_1: f16 d, f16 m, 16 nibble bytes
    case 6: return {32, 22};     // Q5_0
    case 7: return {32, 24};     // Q5_1
    case 8: return {32, 34};     // Q8_0: f16 d, 32 int8
    case 9: return {32, 36};     // Q8_1
    case 10: return {256, 84};   // Q2_K
    case 11: return {256, 110};  // Q3_K
    case 12: return {256, 144};  // Q4_K
    case 13: return {256, 176};  // Q5_K
    case 14: return {256, 210};  // Q6_K
    case 15: return {256, 292};  // Q8_K
    case 24: return {1, 1};      // I8
    case 25: return {1, 2};      // I16
    case 26: return {1, 4};      // I32
    case 27: return {1, 8};      // I64
    case 28: return {1, 8};      // F64
    case 30: return {1, 2};      // BF16
    default: return {0, 0};
  }
}

int scalar_bytes(uint32_t vt) {
  switch (vt) {
    case ENGINE_GGUF_UINT8: case ENGINE_GGUF_INT8: case ENGINE_GGUF_BOOL: return 1;
    case ENGINE_GGUF_UINT16: case ENGINE_GGUF_INT16: return 2;
    case ENGINE_GGUF_UINT32: case ENGINE_GGUF_INT32: case ENGINE_GGUF_FLOAT32: return 4;
    case ENGINE_GGUF_UINT64: case ENGINE_GGUF_INT64: case ENGINE_GGUF_FLOAT64: return 8;
    default: return 0;
  }
}

struct Meta {
  std::string key;
  int32_t type = 0;
  int32_t elem_type = -1;  // arrays only
  uint64_t count = 1;      // arrays: element count
  bool is_int = false, is_float = false;
  int64_t i = 0;
  bool u64_big = false;    // a UINT64 above INT64_MAX
  double f = 0.0;
  std::string s;
};

struct GTensor {
  std::string name;
  int32_t type = 0;
  int32_t n_dims = 0;
  int64_t dims[4] = {1, 1, 1, 1};
  uint64_t rel = 0, offset = 0, nbytes = 0;
};

class Cursor {
 public:
  Cursor(const uint8_t* p, uint64_t size) : p_(p), size_(size) {}
  uint64_t pos() const { return pos_; }
  uint64_t left() const { return size_ - pos_; }
  template <typename T>
  bool get(T* v) {
    if (left() < sizeof(T)) return false;
    std::memcpy(v, p_ + pos_, sizeof(T));
    pos_ += sizeof(T);
    return true;
  }
  bool str(std::string* s) {
    uint64_t n = 0;
    if (!get(&n) || n > left()) return false;
    s->assign(reinterpret_cast<const char*>(p_ + pos_), static_cast<size_t>(n));
    pos_ += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (n > left()) return false;
    pos_ += n;
    return true;
  }

 private:
  const uint8_t* p_;
  uint64_t size_;
  uint64_t pos_ = 0;
};

}  // namespace

struct engine_gguf {
  int fd = -1;
  void* map = nullptr;
  uint64_t size = 0;
  int32_t version = 0;
  uint64_t alignment = kDefaultAlign;
  uint64_t data_start = 0;
  std::vector<Meta> meta;
  std::unordered_map<std::string, size_t> meta_index;
  std::vector<GTensor> tensors;
  std::unordered_map<std::string, size_t> tensor_index;
  // pinned double buffers for engine_gguf_load_tensor (allocated on first use)
  void* pin[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  int dev = -1;
};

namespace {

using b200::set_error;

int fmt_error(const std::string& msg) { return set_error(ENGINE_ERR_FORMAT, "gguf: " + msg); }

// Reads one metadata value of type `vt` into `m` (scalars and strings keep
// their value; arrays keep their element type and count).  `depth` bounds the
// nesting of arrays of arrays.
bool read_value(Cursor& c, uint32_t vt, Meta* m, int depth, std::string* why) {
  const int sb = scalar_bytes(vt);
  if (sb > 0) {
    uint64_t raw = 0;
    if (c.left() < static_cast<uint64_t>(sb)) return (*why = "truncated value", false);
    uint8_t b[8] = {};
    for (int k = 0; k < sb; ++k) c.get(&b[k]);
    std::memcpy(&raw, b, 8);
    if (m == nullptr) return true;
    switch (vt) {
      case ENGINE_GGUF_UINT8: m->i = static_cast<uint8_t>(raw); break;
      case ENGINE_GGUF_INT8: m->i = static_cast<int8_t>(raw); break;
      case ENGINE_GGUF_UINT16: m->i = static_cast<uint16_t>(raw); break;
      case ENGINE_GGUF_INT16: m->i = static_cast<int16_t>(raw); break;
      case ENGINE_GGUF_UINT32: m->i = static_cast<uint32_t>(raw); break;
      case ENGINE_GGUF_INT32: m->i = static_cast<int32_t>(raw); break;
      case ENGINE_GGUF_BOOL: m->i = (raw & 0xff) != 0; break;
      case ENGINE_GGUF_UINT64:
        m->i = static_cast<int64_t>(raw);
        m->u64_big = raw > static_cast<uint64_t>(INT64_MAX);
        break;
      case ENGINE_GGUF_INT64: m->i = static_cast<int64_t>(raw); break;
      case ENGINE_GGUF_FLOAT32: {
        float f;
        std::memcpy(&f, b, 4);
        m->f = f;
        break;
      }
      case ENGINE_GGUF_FLOAT64: std::memcpy(&m->f, b, 8); break;
      default: break;
    }
    m->is_float = vt == ENGINE_GGUF_FLOAT32 || vt == ENGINE_GGUF_FLOAT64;
    m->is_int = !m->is_float;
    return true;
  }
  if (vt == ENGINE_GGUF_STRING) {
    std::string tmp;
    if (!c.str(m ? &m->s : &tmp)) return (*why = "truncated string", false);
    return true;
  }
  if (vt == ENGINE_GGUF_ARRAY) {
    uint32_t et = 0;
    uint64_t n = 0;
    if (!c.get(&et) || !c.get(&n)) return (*why = "truncated array header", false);
    if (m) {
      m->elem_type = static_cast<int32_t>(et);
      m->count = n;
    }
    const int eb = scalar_bytes(et);
    if (eb > 0) {
      if (n > c.left() / static_cast<uint64_t>(eb)) return (*why = "truncated array", false);
      return c.skip(n * static_cast<uint64_t>(eb)) || (*why = "truncated array", false);
    }
    if (et == ENGINE_GGUF_STRING) {
      if (n > c.left() / 8) return (*why = "truncated array", false);  // >= 8 bytes each
      for (uint64_t k = 0; k < n; ++k) {
        uint64_t len = 0;
        if (!c.get(&len) || !c.skip(len)) return (*why = "truncated string in array", false);
      }
      return true;
    }
    if (et == ENGINE_GGUF_ARRAY) {
      if (depth >= 2) return (*why = "arrays nested more than two deep", false);
      if (n > c.left() / 12) return (*why = "truncated array", false);  // >= 12 bytes each
      for (uint64_t k = 0; k < n; ++k)
        if (!read_value(c, et, nullptr, depth + 1, why)) return false;
      return true;
    }
    return (*why = "array of unknown value type " + std::to_string(et), false);
  }
  return (*why = "unknown value type " + std::to_string(vt), false);
}

int parse(engine_gguf* g) {
  Cursor c(static_cast<const uint8_t*>(g->map), g->size);
  uint32_t magic = 0, version = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!c.get(&magic) || magic != kMagic) return fmt_error("not a GGUF file (bad magic)");
  if (!c.get(&version)) return fmt_error("truncated header");
  if (version != 2 && version != 3)
    return fmt_error("unsupported GGUF version " + std::to_string(version) + " (2 and 3 are read)");
  g->version = static_cast<int32_t>(version);
  if (!c.get(&n_tensors) || !c.get(&n_kv)) return fmt_error("truncated header");
  // Each entry takes at least 13 (metadata) or 24 (tensor) bytes: counts beyond
  // what the file can hold are malformed, and are rejected before reserving.
  if (n_kv > c.left() / 13) return fmt_error("metadata count exceeds the file");
  if (n_tensors > c.left() / 24) return fmt_error("tensor count exceeds the file");

  g->meta.reserve(static_cast<size_t>(n_kv));
  for (uint64_t k = 0; k < n_kv; ++k) {
    Meta m;
    uint32_t vt = 0;
    std::string why;
    if (!c.str(&m.key)) return fmt_error("truncated metadata key");
    if (!c.get(&vt)) return fmt_error("truncated metadata entry '" + m.key + "'");
    m.type = static_cast<int32_t>(vt);
    if (!read_value(c, vt, &m, 0, &why)) return fmt_error("metadata '" + m.key + "': " + why);
    if (g->meta_index.count(m.key)) return fmt_error("duplicate metadata key '" + m.key + "'");
    g->meta_index[m.key] = g->meta.size();
    g->meta.push_back(std::move(m));
  }
  auto al = g->meta_index.find("general.alignment");
  if (al != g->meta_index.end()) {
    const Meta& m = g->meta[al->second];
    if (!m.is_int || m.i <= 0 || (m.i & (m.i - 1)) != 0 || m.i > (1 << 20))
      return fmt_error("general.alignment must be a power of two up to 1 MiB");
    g->alignment = static_cast<uint64_t>(m.i);
  }

  g->tensors.reserve(static_cast<size_t>(n_tensors));
  for (uint64_t k = 0; k < n_tensors; ++k) {
    GTensor t;
    uint32_t nd = 0, ty = 0;
    if (!c.str(&t.name)) return fmt_error("truncated tensor name");
    if (!c.get(&nd)) return fmt_error("truncated tensor '" + t.name + "'");
    if (nd < 1 || nd > 4)
      return fmt_error("tensor '" + t.name + "' has " + std::to_string(nd) + " dims (1..4)");
    t.n_dims = static_cast<int32_t>(nd);
    uint64_t elems = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      uint64_t v = 0;
      if (!c.get(&v)) return fmt_error("truncated tensor '" + t.name + "'");
      if (v > (uint64_t(1) << 40) || (v != 0 && elems > (uint64_t(1) << 62) / v))
        return fmt_error("tensor '" + t.name + "' is too large");
      elems *= v;
      t.dims[d] = static_cast<int64_t>(v);
    }
    if (!c.get(&ty) || !c.get(&t.rel)) return fmt_error("truncated tensor '" + t.name + "'");
    t.type = static_cast<int32_t>(ty);
    const TypeSize ts = ggml_type_size(ty);
    if (ts.block > 0) {
      if (t.dims[0] % ts.block != 0)
        return fmt_error("tensor '" + t.name + "': dims[0] = " + std::to_string(t.dims[0]) +
                         " is not a multiple of its type's block of " + std::to_string(ts.block));
      t.nbytes = elems / static_cast<uint64_t>(ts.block) * static_cast<uint64_t>(ts.bytes);
    }
    if (t.rel % g->alignment != 0)
      return fmt_error("tensor '" + t.name + "' data offset is not a multiple of the alignment");
    if (g->tensor_index.count(t.name)) return fmt_error("duplicate tensor name '" + t.name + "'");
    g->tensor_index[t.name] = g->tensors.size();
    g->tensors.push_back(std::move(t));
  }

  const uint64_t here = c.pos();
  g->data_start = (here + g->alignment - 1) / g->alignment * g->alignment;
  for (GTensor& t : g->tensors) {
    if (t.rel > g->size || g->data_start > g->size - t.rel ||
        t.nbytes > g->size - g->data_start - t.rel)
      return fmt_error("tensor '" + t.name + "' extends past the end of the file");
    t.offset = g->data_start + t.rel;
  }
  return ENGINE_OK;
}

void release(engine_gguf* g) {
  for (int b = 0; b < 2; ++b) {
    if (g->ev[b]) {
      cudaEventSynchronize(g->ev[b]);  // this handle's own copies finish before their buffers go
      cudaEventDestroy(g->ev[b]);
    }
    if (g->pin[b]) cudaFreeHost(g->pin[b]);
  }
  if (g->map) munmap(g->map, static_cast<size_t>(g->size));
  if (g->fd >= 0) close(g->fd);
  delete g;
}

const Meta* find_meta(const engine_gguf* g, const char* key) {
  if (key == nullptr) return nullptr;
  auto it = g->meta_index.find(key);
  return it == g->meta_index.end() ? nullptr : &g->meta[it->second];
}

}  // namespace

extern "C" {

int engine_gguf_open(const char* path, engine_gguf_t** out) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(path != nullptr && out != nullptr, "gguf_open: null pointer");
  *out = nullptr;
  auto* g = new engine_gguf;
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    const int e = errno;
    release(g);
    return set_error(ENGINE_ERR_IO, std::string("gguf_open: cannot open '") + path + "': " +
                                        std::strerror(e));
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
    release(g);
    return set_error(ENGINE_ERR_FORMAT, std::string("gguf: '") + path +
                                            "' is too small to be a GGUF file");
  }
  g->size = static_cast<uint64_t>(st.st_size);
  void* m = mmap(nullptr, static_cast<size_t>(g->size), PROT_READ, MAP_PRIVATE, g->fd, 0);
  if (m == MAP_FAILED) {
    const int e = errno;
    release(g);
    return set_error(ENGINE_ERR_IO, std::string("gguf_open: cannot map '") + path + "': " +
                                        std::strerror(e));
  }
  g->map = m;
  const int rc = parse(g);
  if (rc != ENGINE_OK) {
    release(g);
    return rc;
  }
  *out = g;
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_gguf_close(engine_gguf_t* g) {
  B200_ENTRY_BEGIN
  if (g != nullptr) release(g);
  return ENGINE_OK;
  B200_ENTRY_END
}

int engine_gguf_version(const engine_gguf_t* g, int32_t* version, uint64_t* alignment) {
  B200_REQUIRE(g != nullptr, "gguf_version: null handle");
  if (version) *version = g->version;
  if (alignment) *alignment = g->alignment;
  return ENGINE_OK;
}

int engine_gguf_tensor_count(const engine_gguf_t* g, int64_t* n) {
  B200_REQUIRE(g != nullptr && n != nullptr, "gguf_tensor_count: null pointer");
  *n = static_cast<int64_t>(g->tensors.size());
  return ENGINE_OK;
}

int engine_gguf_tensor(const engine_gguf_t* g, int64_t index, engine_gguf_tensor_t* out) {
  B200_REQUIRE(g != nullptr && out != nullptr, "gguf_tensor: null pointer");
  B200_REQUIRE(index >= 0 && index < static_cast<int64_t>(g->tensors.size()),
               "gguf_tensor: index out of range");
  const GTensor& t = g->tensors[static_cast<size_t>(index)];
  out->name = t.name.c_str();
  out->type = t.type;
  out->n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) out->dims[d] = t.dims[d];
  out->offset = t.offset;
  out->nbytes = t.nbytes;
  out->data = static_cast<const uint8_t*>(g->map) + t.offset;
  return ENGINE_OK;
}

int engine_gguf_find_tensor(const engine_gguf_t* g, const char* name, int64_t* index) {
  B200_REQUIRE(g != nullptr && name != nullptr && index != nullptr,
               "gguf_find_tensor: null pointer");
  auto it = g->tensor_index.find(name);
  if (it == g->tensor_index.end())
    return set_error(ENGINE_ERR_INVALID, std::string("gguf_find_tensor: no tensor '") + name + "'");
  *index = static_cast<int64_t>(it->second);
  return ENGINE_OK;
}

int engine_gguf_meta_count(const engine_gguf_t* g, int64_t* n) {
  B200_REQUIRE(g != nullptr && n != nullptr, "gguf_meta_count: null pointer");
  *n = static_cast<int64_t>(g->meta.size());
  return ENGINE_OK;
}

int engine_gguf_meta_entry(const engine_gguf_t* g, int64_t index, const char** key,
                           int32_t* type, int32_t* elem_type, uint64_t* count) {
  B200_REQUIRE(g != nullptr, "gguf_meta_entry: null handle");
  B200_REQUIRE(index >= 0 && index < static_cast<int64_t>(g->meta.size()),
               "gguf_meta_entry: index out of range");
  const Meta& m = g->meta[static_cast<size_t>(index)];
  if (key) *key = m.key.c_str();
  if (type) *type = m.type;
  if (elem_type) *elem_type = m.elem_type;
  if (count) *count = m.count;
  return ENGINE_OK;
}

int engine_gguf_meta_int(const engine_gguf_t* g, const char* key, int64_t* v) {
  B200_REQUIRE(g != nullptr && v != nullptr, "gguf_meta_int: null pointer");
  const Meta* m = find_meta(g, key);
  if (m == nullptr)
    return set_error(ENGINE_ERR_INVALID, std::string("gguf_meta_int: no key '") + (key ? key : "") + "'");
  if (!m->is_int)
    return set_error(ENGINE_ERR_INVALID, "gguf_meta_int: '" + m->key + "' is not an integer");
  if (m->u64_big)
    return set_error(ENGINE_ERR_INVALID, "gguf_meta_int: '" + m->key + "' exceeds int64");
  *v = m->i;
  return ENGINE_OK;
}

int engine_gguf_meta_float(const engine_gguf_t* g, const char* key, double* v) {
  B200_REQUIRE(g != nullptr && v != nullptr, "gguf_meta_float: null pointer");
  const Meta* m = find_meta(g, key);
  if (m == nullptr)
    return set_error(ENGINE_ERR_INVALID, std::string("gguf_meta_float: no key '") + (key ? key : "") + "'");
  if (!m->is_float)
    return set_error(ENGINE_ERR_INVALID, "gguf_meta_float: '" + m->key + "' is not a float");
  *v = m->f;
  return ENGINE_OK;
}

int engine_gguf_meta_string(const engine_gguf_t* g, const char* key, const char** s,
                            uint64_t* len) {
  B200_REQUIRE(g != nullptr && s != nullptr, "gguf_meta_string: null pointer");
  const Meta* m = find_meta(g, key);
  if (m == nullptr)
    return set_error(ENGINE_ERR_INVALID, std::string("gguf_meta_string: no key '") + (key ? key : "") + "'");
  if (m->type != ENGINE_GGUF_STRING)
    return set_error(ENGINE_ERR_INVALID, "gguf_meta_string: '" + m->key + "' is not a string");
  *s = m->s.c_str();
  if (len) *len = m->s.size();
  return ENGINE_OK;
}

int engine_gguf_load_tensor(engine_gguf_t* g, int64_t index, void* payload,
                            engine_half_t* scales, void* staging, engine_stream_t stream) {
  B200_ENTRY_BEGIN
  B200_REQUIRE(g != nullptr, "gguf_load_tensor: null handle");
  B200_REQUIRE(index >= 0 && index < static_cast<int64_t>(g->tensors.size()),
               "gguf_load_tensor: index out of range");
  const GTensor& t = g->tensors[static_cast<size_t>(index)];
  const bool quant = t.type == ENGINE_GGML_Q8_0 || t.type == ENGINE_GGML_Q4_0;
  const bool plain =
      t.type == ENGINE_GGML_F32 || t.type == ENGINE_GGML_F16 || t.type == ENGINE_GGML_BF16;
  if (!quant && !plain)
    return set_error(ENGINE_ERR_UNSUPPORTED,
                     "gguf_load_tensor: tensor '" + t.name + "' has GGML type " +
                         std::to_string(t.type) +
                         "; the device layouts cover F32, F16, BF16, Q8_0 and Q4_0");
  B200_REQUIRE(payload != nullptr, "gguf_load_tensor: null device pointer");
  if (quant) {
    B200_REQUIRE(scales != nullptr && staging != nullptr, "gguf_load_tensor: null device pointer");
  }
  if (t.nbytes == 0) return ENGINE_OK;
  auto st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  B200_CUDA(cudaGetDevice(&dev));
  if (g->ev[0] != nullptr && g->dev != dev) {  // events belong to one device
    for (int b = 0; b < 2; ++b) {
      B200_CUDA(cudaEventSynchronize(g->ev[b]));
      cudaEventDestroy(g->ev[b]);
      g->ev[b] = nullptr;
    }
  }
  for (int b = 0; b < 2; ++b) {
    if (g->pin[b] == nullptr) B200_CUDA(cudaHostAlloc(&g->pin[b], kChunk, cudaHostAllocPortable));
    if (g->ev[b] == nullptr) B200_CUDA(cudaEventCreateWithFlags(&g->ev[b], cudaEventDisableTiming));
  }
  g->dev = dev;
  // Two pinned buffers: while one chunk's DMA runs, the next chunk is copied
  // out of the mapping (page-cache reads) into the other buffer.
  const uint8_t* src = static_cast<const uint8_t*>(g->map) + t.offset;
  uint8_t* dst = static_cast<uint8_t*>(quant ? staging : payload);
  int b = 0;
  for (uint64_t off = 0; off < t.nbytes; off += kChunk, b ^= 1) {
    const size_t n = static_cast<size_t>(t.nbytes - off < kChunk ? t.nbytes - off : kChunk);
    B200_CUDA(cudaEventSynchronize(g->ev[b]));  // the DMA that last read this buffer is done
    std::memcpy(g->pin[b], src + off, n);
    B200_CUDA(cudaMemcpyAsync(dst + off, g->pin[b], n, cudaMemcpyHostToDevice, st));
    B200_CUDA(cudaEventRecord(g->ev[b], st));
  }
  if (quant) {
    int64_t rows = 1;
    for (int d = 1; d < t.n_dims; ++d) rows *= t.dims[d];
    return engine_cuda_quant_repack(t.type == ENGINE_GGML_Q8_0 ? ENGINE_Q8_0 : ENGINE_Q4_0,
                                    staging, payload, scales, rows, t.dims[0], stream);
  }
  return ENGINE_OK;
  B200_ENTRY_END
}

}  // extern "C"
