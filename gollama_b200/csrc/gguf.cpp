// GGUF files (pkg/gguf/reader.go, pkg/gguf/format.go), host side.
//
// The reader maps the file read-only and parses what gguf.Reader parses
// (reader.go:63-207): the header (magic "GGUF", version 2 or 3, tensor and
// metadata counts), every metadata key/value (all thirteen value types,
// arrays of any of them, nested arrays included), every tensor's name,
// dimensions (GGUF order, innermost first), type and data offset, and the
// start of the tensor data: the end of the tensor infos rounded up to
// `general.alignment` when that key holds a uint32, else 32 (:112-121).  As in
// the reference a later duplicate key or tensor name replaces the earlier one
// in lookups.  Tensor sizes follow TensorInfo.SizeBytes (format.go:171-177):
// whole blocks of GetTypeInfo's geometry (:117-149), unknown types 4 bytes per
// element.
//
// Unlike the reference, which indexes the mapped bytes without bounds checks
// on scalar fields, every read is checked: a truncated or inconsistent file is
// an error (GLC_ERR_IO), never a crash.
//
// Device side: glc_gguf_tensor_upload copies a tensor's raw bytes (quantized
// blocks as stored) to device memory, where glc_linear_bwd_dx_q takes them
// directly; glc_gguf_tensor_load is loadTensor (pkg/model/transformer.go:
// 285-303): the bytes to the device, then the device Dequantize.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "glc_internal.h"

namespace glc {
namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint64_t kDefaultAlignment = 32;
enum : uint32_t {
  T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64, T_COUNT
};

int fail_io(const std::string& msg) {
  host_error() = msg;
  return GLC_ERR_IO;
}
int fail_arg(const std::string& msg) {
  host_error() = msg;
  return GLC_ERR_INVALID;
}

// GetTypeInfo (format.go:117-149): elements per block and bytes per block.
void type_info(uint32_t t, uint64_t* block, uint64_t* bytes) {
  switch (t) {
    case 0: *block = 1; *bytes = 4; return;      // F32
    case 1: *block = 1; *bytes = 2; return;      // F16
    case 2: *block = 32; *bytes = 18; return;    // Q4_0
    case 3: *block = 32; *bytes = 20; return;    // Q4_1
    case 6: *block = 32; *bytes = 22; return;    // Q5_0
    case 7: *block = 32; *bytes = 24; return;    // Q5_1
    case 8: *block = 32; *bytes = 34; return;    // Q8_0
    case 9: *block = 32; *bytes = 36; return;    // Q8_1
    case 10: *block = 256; *bytes = 84; return;  // Q2_K
    case 11: *block = 256; *bytes = 110; return; // Q3_K
    case 12: *block = 256; *bytes = 144; return; // Q4_K
    case 13: *block = 256; *bytes = 176; return; // Q5_K
    case 14: *block = 256; *bytes = 210; return; // Q6_K
    case 15: *block = 256; *bytes = 292; return; // Q8_K
    case 30: *block = 1; *bytes = 2; return;     // BF16
    default: *block = 1; *bytes = 4; return;
  }
}

}  // namespace

struct GgufValue {
  uint32_t type = 0;
  uint64_t u = 0;  // unsigned integers and bool
  int64_t i = 0;   // signed integers
  double f = 0.0;  // float32 (exactly) and float64
  std::string s;
  uint32_t elem_type = 0;  // arrays
  std::vector<GgufValue> arr;
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t elements() const {  // NumElements (format.go:159-168)
    if (dims.empty()) return 0;
    uint64_t n = 1;
    for (uint64_t d : dims) n *= d;
    return n;
  }
  uint64_t size_bytes() const {  // SizeBytes (format.go:171-177)
    uint64_t block, bytes;
    type_info(type, &block, &bytes);
    return (elements() + block - 1) / block * bytes;
  }
};

}  // namespace glc

struct glc_gguf {
  int fd = -1;
  const uint8_t* data = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t n_tensors = 0, n_kv = 0, data_offset = 0;
  std::vector<std::pair<std::string, glc::GgufValue>> meta;
  std::unordered_map<std::string, size_t> meta_index;
  std::vector<glc::GgufTensor> tensors;
  std::unordered_map<std::string, size_t> tensor_index;
  ~glc_gguf() {
    if (data) munmap(const_cast<uint8_t*>(data), size);
    if (fd >= 0) close(fd);
  }
};

namespace glc {
namespace {

// Bounds-checked little-endian cursor over the mapped file.
struct Cursor {
  const uint8_t* p;
  size_t size, off = 0;
  bool have(uint64_t n) const { return n <= size - off; }
  bool u32(uint32_t* v) {
    if (!have(4)) return false;
    *v = 0;
    for (int k = 0; k < 4; ++k) *v |= static_cast<uint32_t>(p[off + k]) << (8 * k);
    off += 4;
    return true;
  }
  bool u64(uint64_t* v) {
    if (!have(8)) return false;
    *v = 0;
    for (int k = 0; k < 8; ++k) *v |= static_cast<uint64_t>(p[off + k]) << (8 * k);
    off += 8;
    return true;
  }
  bool bytes(void* dst, size_t n) {
    if (!have(n)) return false;
    std::memcpy(dst, p + off, n);
    off += n;
    return true;
  }
  // readString (reader.go:211-228): u64 length, then the bytes
  bool str(std::string* s) {
    uint64_t n;
    if (!u64(&n) || !have(n)) return false;
    s->assign(reinterpret_cast<const char*>(p + off), static_cast<size_t>(n));
    off += static_cast<size_t>(n);
    return true;
  }
};

// Smallest encoding of one value of a type (bounds the element count of an
// array against the bytes left, so a corrupt count cannot allocate wildly).
uint64_t min_bytes(uint32_t t) {
  switch (t) {
    case T_U8: case T_I8: case T_BOOL: return 1;
    case T_U16: case T_I16: return 2;
    case T_U32: case T_I32: case T_F32: return 4;
    case T_U64: case T_I64: case T_F64: case T_STRING: return 8;
    case T_ARRAY: return 12;
    default: return 1;
  }
}

// readValue (reader.go:231-296).
int read_value(Cursor& c, uint32_t type, GgufValue* v, int depth) {
  v->type = type;
  switch (type) {
    case T_U8: case T_I8: case T_BOOL: {
      uint8_t b;
      if (!c.bytes(&b, 1)) return fail_io("gguf: unexpected end of file in a metadata value");
      v->u = b;
      v->i = static_cast<int8_t>(b);
      if (type == T_BOOL) v->u = b != 0;
      return GLC_OK;
    }
    case T_U16: case T_I16: {
      uint8_t b[2];
      if (!c.bytes(b, 2)) return fail_io("gguf: unexpected end of file in a metadata value");
      v->u = static_cast<uint64_t>(b[0] | (b[1] << 8));
      v->i = static_cast<int16_t>(v->u);
      return GLC_OK;
    }
    case T_U32: case T_I32: case T_F32: {
      uint32_t x;
      if (!c.u32(&x)) return fail_io("gguf: unexpected end of file in a metadata value");
      v->u = x;
      v->i = static_cast<int32_t>(x);
      float f;
      std::memcpy(&f, &x, 4);
      v->f = f;
      return GLC_OK;
    }
    case T_U64: case T_I64: case T_F64: {
      uint64_t x;
      if (!c.u64(&x)) return fail_io("gguf: unexpected end of file in a metadata value");
      v->u = x;
      v->i = static_cast<int64_t>(x);
      std::memcpy(&v->f, &x, 8);
      return GLC_OK;
    }
    case T_STRING:
      if (!c.str(&v->s)) return fail_io("gguf: unexpected end of file in a string");
      return GLC_OK;
    case T_ARRAY: {
      if (depth > 16) return fail_io("gguf: arrays nested too deeply");
      uint32_t et;
      uint64_t n;
      if (!c.u32(&et) || !c.u64(&n)) return fail_io("gguf: unexpected end of file in an array header");
      if (et >= T_COUNT) return fail_io("gguf: unknown metadata value type " + std::to_string(et));
      if (n > (c.size - c.off) / min_bytes(et)) return fail_io("gguf: array longer than the file");
      v->elem_type = et;
      v->arr.resize(static_cast<size_t>(n));
      for (uint64_t k = 0; k < n; ++k) {
        int rc = read_value(c, et, &v->arr[static_cast<size_t>(k)], depth + 1);
        if (rc) return rc;
      }
      return GLC_OK;
    }
    default:
      return fail_io("gguf: unknown metadata value type " + std::to_string(type));
  }
}

// parse (reader.go:63-123), parseMetadata (:126-153), parseTensorInfo (:156-207).
int parse(glc_gguf* g) {
  if (g->size < 24) return fail_io("gguf: file too small to be valid GGUF");
  Cursor c{g->data, g->size};
  uint32_t magic;
  c.u32(&magic);
  if (magic != kMagic) return fail_io("gguf: invalid magic number");
  c.u32(&g->version);
  if (g->version < 2 || g->version > 3)
    return fail_io("gguf: unsupported GGUF version " + std::to_string(g->version));
  c.u64(&g->n_tensors);
  c.u64(&g->n_kv);
  // every entry takes at least 12 (key/value) or 24 (tensor info) bytes
  if (g->n_kv > g->size / 12 || g->n_tensors > g->size / 24)
    return fail_io("gguf: more entries than the file can hold");
  g->meta.reserve(static_cast<size_t>(g->n_kv));
  for (uint64_t k = 0; k < g->n_kv; ++k) {
    std::string key;
    uint32_t type;
    if (!c.str(&key) || !c.u32(&type)) return fail_io("gguf: unexpected end of file in a metadata key");
    GgufValue v;
    int rc = read_value(c, type, &v, 0);
    if (rc) return rc;
    g->meta_index[key] = g->meta.size();
    g->meta.emplace_back(std::move(key), std::move(v));
  }
  g->tensors.resize(static_cast<size_t>(g->n_tensors));
  for (uint64_t k = 0; k < g->n_tensors; ++k) {
    GgufTensor& t = g->tensors[static_cast<size_t>(k)];
    uint32_t nd;
    if (!c.str(&t.name) || !c.u32(&nd)) return fail_io("gguf: unexpected end of file in a tensor info");
    if (!c.have(static_cast<uint64_t>(nd) * 8)) return fail_io("gguf: unexpected end of file in tensor dimensions");
    t.dims.resize(nd);
    uint64_t count = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      c.u64(&t.dims[d]);
      if (t.dims[d] != 0 && count > UINT64_MAX / t.dims[d] / 4)
        return fail_io("gguf: dimensions of tensor '" + t.name + "' overflow");
      count *= t.dims[d];
    }
    if (!c.u32(&t.type) || !c.u64(&t.offset)) return fail_io("gguf: unexpected end of file in a tensor info");
    g->tensor_index[t.name] = static_cast<size_t>(k);
  }
  uint64_t align = kDefaultAlignment;
  auto it = g->meta_index.find("general.alignment");
  if (it != g->meta_index.end() && g->meta[it->second].second.type == T_U32) {
    align = g->meta[it->second].second.u;
    if (align == 0) return fail_io("gguf: general.alignment is 0");
  }
  g->data_offset = c.off;
  if (g->data_offset % align) g->data_offset += align - g->data_offset % align;
  return GLC_OK;
}

const GgufValue* element(const glc_gguf* g, int64_t i, uint64_t elem) {
  if (!g || i < 0 || static_cast<uint64_t>(i) >= g->meta.size()) return nullptr;
  const GgufValue& v = g->meta[static_cast<size_t>(i)].second;
  if (v.type != T_ARRAY) return elem == 0 ? &v : nullptr;
  return elem < v.arr.size() ? &v.arr[static_cast<size_t>(elem)] : nullptr;
}

int copy_string(const std::string& s, char* buf, size_t cap, size_t* len) {
  if (len) *len = s.size();
  if (buf && cap) {
    const size_t k = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), k);
    buf[k] = 0;
  }
  return GLC_OK;
}

}  // namespace
}  // namespace glc

extern "C" {

int glc_gguf_open(const char* path, glc_gguf** out) {
  if (!path || !out) return glc::fail_arg("gguf: bad arguments");
  *out = nullptr;
  auto* g = new glc_gguf();
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    delete g;
    return glc::fail_io(std::string("gguf: cannot open ") + path + ": " + std::strerror(errno));
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0) {
    delete g;
    return glc::fail_io(std::string("gguf: cannot stat ") + path);
  }
  g->size = static_cast<size_t>(st.st_size);
  if (g->size >= 24) {
    void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
      delete g;
      return glc::fail_io(std::string("gguf: cannot map ") + path);
    }
    g->data = static_cast<const uint8_t*>(m);
  }
  int rc = glc::parse(g);
  if (rc) {
    delete g;
    return rc;
  }
  *out = g;
  return GLC_OK;
}

int glc_gguf_close(glc_gguf* g) {
  if (!g) return GLC_ERR_INVALID;
  delete g;
  return GLC_OK;
}

int glc_gguf_header(glc_gguf* g, uint32_t* version, uint64_t* n_tensors, uint64_t* n_kv, uint64_t* data_offset) {
  if (!g) return glc::fail_arg("gguf: null reader");
  if (version) *version = g->version;
  if (n_tensors) *n_tensors = g->n_tensors;
  if (n_kv) *n_kv = g->n_kv;
  if (data_offset) *data_offset = g->data_offset;
  return GLC_OK;
}

int glc_gguf_meta_find(glc_gguf* g, const char* key, int64_t* index) {
  if (!g || !key || !index) return glc::fail_arg("gguf: bad arguments");
  auto it = g->meta_index.find(key);
  *index = it == g->meta_index.end() ? -1 : static_cast<int64_t>(it->second);
  return GLC_OK;
}

int glc_gguf_meta_key(glc_gguf* g, int64_t i, char* buf, size_t cap, size_t* len) {
  if (!g || i < 0 || static_cast<uint64_t>(i) >= g->meta.size()) return glc::fail_arg("gguf: no such metadata entry");
  return glc::copy_string(g->meta[static_cast<size_t>(i)].first, buf, cap, len);
}

int glc_gguf_meta_type(glc_gguf* g, int64_t i, int* type, int* elem_type, uint64_t* count) {
  if (!g || i < 0 || static_cast<uint64_t>(i) >= g->meta.size()) return glc::fail_arg("gguf: no such metadata entry");
  const glc::GgufValue* v = &g->meta[static_cast<size_t>(i)].second;
  if (type) *type = static_cast<int>(v->type);
  if (elem_type) *elem_type = v->type == glc::T_ARRAY ? static_cast<int>(v->elem_type) : -1;
  if (count) *count = v->type == glc::T_ARRAY ? v->arr.size() : 1;
  return GLC_OK;
}

int glc_gguf_meta_number(glc_gguf* g, int64_t i, uint64_t elem, int64_t* as_int, uint64_t* as_uint,
                         double* as_double) {
  const glc::GgufValue* v = glc::element(g, i, elem);
  if (!v || v->type == glc::T_STRING || v->type == glc::T_ARRAY)
    return glc::fail_arg("gguf: not a numeric metadata value");
  if (as_int) *as_int = v->i;
  if (as_uint) *as_uint = v->u;
  if (as_double) *as_double = v->f;
  return GLC_OK;
}

int glc_gguf_meta_string(glc_gguf* g, int64_t i, uint64_t elem, char* buf, size_t cap, size_t* len) {
  const glc::GgufValue* v = glc::element(g, i, elem);
  if (!v || v->type != glc::T_STRING) return glc::fail_arg("gguf: not a string metadata value");
  return glc::copy_string(v->s, buf, cap, len);
}

int glc_gguf_tensor_find(glc_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return glc::fail_arg("gguf: bad arguments");
  auto it = g->tensor_index.find(name);
  *index = it == g->tensor_index.end() ? -1 : static_cast<int64_t>(it->second);
  return GLC_OK;
}

int glc_gguf_tensor_info(glc_gguf* g, int64_t i, char* name, size_t name_cap, size_t* name_len, int* type,
                         int* ndims, uint64_t* dims, int dims_cap, uint64_t* offset, uint64_t* nbytes) {
  if (!g || i < 0 || static_cast<uint64_t>(i) >= g->tensors.size()) return glc::fail_arg("gguf: no such tensor");
  const glc::GgufTensor& t = g->tensors[static_cast<size_t>(i)];
  glc::copy_string(t.name, name, name_cap, name_len);
  if (type) *type = static_cast<int>(t.type);
  if (ndims) *ndims = static_cast<int>(t.dims.size());
  for (int d = 0; dims && d < dims_cap && d < static_cast<int>(t.dims.size()); ++d) dims[d] = t.dims[d];
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.size_bytes();
  return GLC_OK;
}

// GetTensorData (reader.go:407-424): the tensor's bytes inside the mapping.
int glc_gguf_tensor_data(glc_gguf* g, int64_t i, const void** data, uint64_t* nbytes) {
  if (!g || !data || i < 0 || static_cast<uint64_t>(i) >= g->tensors.size())
    return glc::fail_arg("gguf: no such tensor");
  const glc::GgufTensor& t = g->tensors[static_cast<size_t>(i)];
  const uint64_t size = t.size_bytes();
  if (t.offset > g->size || g->data_offset > g->size - t.offset || size > g->size - g->data_offset - t.offset)
    return glc::fail_io("gguf: tensor data extends beyond file: " + t.name);
  *data = g->data + g->data_offset + t.offset;
  if (nbytes) *nbytes = size;
  return GLC_OK;
}

int glc_gguf_tensor_upload(glc_ctx* ctx, glc_gguf* g, int64_t i, void* dev, uint64_t cap) {
  if (!ctx || !dev) return GLC_ERR_INVALID;
  glc::Context* c = reinterpret_cast<glc::Context*>(ctx);
  const void* src = nullptr;
  uint64_t n = 0;
  int rc = glc_gguf_tensor_data(g, i, &src, &n);
  if (rc) return c->fail(rc, glc::host_error());
  if (n > cap) return c->fail(GLC_ERR_INVALID, "gguf_tensor_upload: destination smaller than the tensor");
  cudaError_t e = cudaMemcpyAsync(dev, src, static_cast<size_t>(n), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? GLC_OK : c->fail_cuda(e, "gguf_tensor_upload");
}

int glc_gguf_tensor_load(glc_ctx* ctx, glc_gguf* g, int64_t i, float* dev, int64_t n) {
  if (!ctx || !dev) return GLC_ERR_INVALID;
  glc::Context* c = reinterpret_cast<glc::Context*>(ctx);
  if (!g || i < 0 || static_cast<uint64_t>(i) >= g->tensors.size())
    return c->fail(GLC_ERR_INVALID, "gguf_tensor_load: no such tensor");
  const glc::GgufTensor& t = g->tensors[static_cast<size_t>(i)];
  if (n < 0 || static_cast<uint64_t>(n) != t.elements())
    return c->fail(GLC_ERR_INVALID, "gguf_tensor_load: n is not the tensor's element count");
  const void* src = nullptr;
  uint64_t nbytes = 0;
  int rc = glc_gguf_tensor_data(g, i, &src, &nbytes);
  if (rc) return c->fail(rc, glc::host_error());
  void* ws = nullptr;
  rc = c->workspace(static_cast<size_t>(nbytes), &ws);
  if (rc) return rc;
  cudaError_t e = cudaMemcpyAsync(ws, src, static_cast<size_t>(nbytes), cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "gguf_tensor_load: copy");
  rc = glc_dequantize(ctx, static_cast<int>(t.type), ws, dev, static_cast<size_t>(n));
  if (rc) return rc;
  e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? GLC_OK : c->fail_cuda(e, "gguf_tensor_load");
}

}  // extern "C"
