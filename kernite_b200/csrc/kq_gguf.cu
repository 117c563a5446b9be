// kq_gguf.cu -- a reader for GGUF model files (host code only): the data format on the input
// side of the matvec. It maps the file, walks the header, the metadata and the tensor table with
// every length checked against the file's size, and hands out each tensor's name, GGML type,
// dimensions and bytes in place. A GGUF file stores a k-quant matrix exactly as kq_matvec takes
// it: ne0 = k elements per row (k/256 super-blocks), ne1 = rows, rows back to back.
//
// The format (GGUF v2/v3, little-endian) is the GGML project's public file format, which
// fxeqxmulfx/kernite does not read: "GGUF" magic, u32 version, u64 tensor count, u64 metadata
// count; metadata pairs (string key, u32 value type, value; arrays carry an element type and a
// count); per tensor a string name, u32 dimension count, u64 dimensions, u32 GGML type and a u64
// offset into the data section, which starts at the next multiple of general.alignment (default
// 32) after the table. Strings are a u64 length and that many bytes.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "kq_internal.h"

struct kq_gguf {
  int fd = -1;
  const uint8_t* base = nullptr;
  uint64_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_start = 0;
  struct Meta {
    uint32_t type = 0;  // value type; for arrays, 9
    uint64_t u = 0;     // integer and bool values (signed ones sign-extended)
    double f = 0.0;     // float values
    std::string s;      // string values
  };
  std::map<std::string, Meta> meta;
  struct Tensor {
    std::string name;
    uint32_t type = 0, n_dims = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t offset = 0, nbytes = 0;
  };
  std::vector<Tensor> tensors;
};

namespace kq {
namespace {

const char* kCall = "kq_gguf_open";

// (elements per block, bytes per block) of the GGML types whose size this reader knows
bool type_size(uint32_t type, uint64_t& block, uint64_t& bytes) {
  switch (type) {
    case 0: block = 1; bytes = 4; return true;      // F32
    case 1: block = 1; bytes = 2; return true;      // F16
    case 2: block = 32; bytes = 18; return true;    // Q4_0
    case 3: block = 32; bytes = 20; return true;    // Q4_1
    case 6: block = 32; bytes = 22; return true;    // Q5_0
    case 7: block = 32; bytes = 24; return true;    // Q5_1
    case 8: block = 32; bytes = 34; return true;    // Q8_0
    case 10: block = 256; bytes = 84; return true;  // Q2_K
    case 11: block = 256; bytes = 110; return true; // Q3_K
    case 12: block = 256; bytes = 144; return true; // Q4_K
    case 13: block = 256; bytes = 176; return true; // Q5_K
    case 14: block = 256; bytes = 210; return true; // Q6_K
    case 15: block = 256; bytes = 292; return true; // Q8_K
    case 24: block = 1; bytes = 1; return true;     // I8
    case 25: block = 1; bytes = 2; return true;     // I16
    case 26: block = 1; bytes = 4; return true;     // I32
    case 27: block = 1; bytes = 8; return true;     // I64
    case 28: block = 1; bytes = 8; return true;     // F64
    case 30: block = 1; bytes = 2; return true;     // BF16
    default: return false;
  }
}

// A bounds-checked cursor over the mapped file.
struct Cursor {
  const uint8_t* p;
  uint64_t size, at = 0;
  std::string err;
  bool need(uint64_t n, const char* what) {
    if (!err.empty()) return false;
    if (n > size - at) {
      err = std::string("truncated file: ") + what + " at byte " + std::to_string(at) +
            " needs " + std::to_string(n) + " bytes, " + std::to_string(size - at) + " left";
      return false;
    }
    return true;
  }
  template <typename T>
  bool get(T& v, const char* what) {
    if (!need(sizeof(T), what)) return false;
    std::memcpy(&v, p + at, sizeof(T));
    at += sizeof(T);
    return true;
  }
  bool str(std::string& s, const char* what) {
    uint64_t n = 0;
    if (!get(n, what) || !need(n, what)) return false;
    s.assign(reinterpret_cast<const char*>(p + at), n);
    at += n;
    return true;
  }
  bool skip(uint64_t n, const char* what) {
    if (!need(n, what)) return false;
    at += n;
    return true;
  }
};

// Bytes of one scalar metadata value of type t (0 for strings and arrays, 0xff.. if unknown).
uint64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;   // u8, i8, bool
    case 2: case 3: return 2;           // u16, i16
    case 4: case 5: case 6: return 4;   // u32, i32, f32
    case 10: case 11: case 12: return 8;  // u64, i64, f64
    case 8: case 9: return 0;           // string, array
    default: return ~uint64_t(0);
  }
}

bool read_scalar(Cursor& c, uint32_t t, kq_gguf::Meta& m) {
  switch (t) {
    case 0: { uint8_t v; if (!c.get(v, "u8 value")) return false; m.u = v; return true; }
    case 1: { int8_t v; if (!c.get(v, "i8 value")) return false; m.u = uint64_t(int64_t(v)); return true; }
    case 2: { uint16_t v; if (!c.get(v, "u16 value")) return false; m.u = v; return true; }
    case 3: { int16_t v; if (!c.get(v, "i16 value")) return false; m.u = uint64_t(int64_t(v)); return true; }
    case 4: { uint32_t v; if (!c.get(v, "u32 value")) return false; m.u = v; return true; }
    case 5: { int32_t v; if (!c.get(v, "i32 value")) return false; m.u = uint64_t(int64_t(v)); return true; }
    case 6: { float v; if (!c.get(v, "f32 value")) return false; m.f = v; return true; }
    case 7: { uint8_t v; if (!c.get(v, "bool value")) return false; m.u = v != 0; return true; }
    case 8: return c.str(m.s, "string value");
    case 10: { uint64_t v; if (!c.get(v, "u64 value")) return false; m.u = v; return true; }
    case 11: { int64_t v; if (!c.get(v, "i64 value")) return false; m.u = uint64_t(v); return true; }
    case 12: { double v; if (!c.get(v, "f64 value")) return false; m.f = v; return true; }
    default:
      c.err = "unknown metadata value type " + std::to_string(t) + " at byte " + std::to_string(c.at);
      return false;
  }
}

int parse(kq_gguf* g) {
  Cursor c{g->base, g->size};
  uint32_t magic = 0;
  if (!c.get(magic, "magic") || magic != 0x46554747u)  // "GGUF"
    return fail(KQ_E_INVALID, kCall, c.err.empty() ? "not a GGUF file (bad magic)" : c.err);
  if (!c.get(g->version, "version")) return fail(KQ_E_INVALID, kCall, c.err);
  if (g->version < 2 || g->version > 3)
    return fail(KQ_E_UNSUPPORTED, kCall, "GGUF version " + std::to_string(g->version) +
                                             " (this reader takes 2 and 3)");
  uint64_t n_tensors = 0, n_meta = 0;
  if (!c.get(n_tensors, "tensor count") || !c.get(n_meta, "metadata count"))
    return fail(KQ_E_INVALID, kCall, c.err);
  // every entry takes at least 8 bytes, which bounds the counts by the file's size
  if (n_tensors > g->size / 8 || n_meta > g->size / 8)
    return fail(KQ_E_INVALID, kCall, "tensor or metadata count larger than the file");
  for (uint64_t i = 0; i < n_meta; ++i) {
    std::string key;
    uint32_t t = 0;
    if (!c.str(key, "metadata key") || !c.get(t, "metadata type"))
      return fail(KQ_E_INVALID, kCall, c.err);
    kq_gguf::Meta m;
    m.type = t;
    if (t == 9) {  // array: element type, count, elements (kept as type and count)
      uint32_t et = 0;
      uint64_t n = 0;
      if (!c.get(et, "array type") || !c.get(n, "array count"))
        return fail(KQ_E_INVALID, kCall, c.err);
      m.u = n;
      const uint64_t eb = scalar_bytes(et);
      if (eb == ~uint64_t(0) || et == 9)
        return fail(KQ_E_INVALID, kCall, "array of type " + std::to_string(et) + " in " + key);
      if (eb) {
        if (n > (g->size - c.at) / eb) return fail(KQ_E_INVALID, kCall, "truncated array " + key);
        c.skip(n * eb, "array");
      } else {  // strings
        for (uint64_t j = 0; j < n; ++j) {
          std::string s;
          if (!c.str(s, "array string")) return fail(KQ_E_INVALID, kCall, c.err);
        }
      }
    } else if (!read_scalar(c, t, m)) {
      return fail(KQ_E_INVALID, kCall, c.err + " (key " + key + ")");
    }
    g->meta[key] = m;
  }
  const auto al = g->meta.find("general.alignment");
  if (al != g->meta.end()) {
    if (al->second.type != 4 || al->second.u == 0)
      return fail(KQ_E_INVALID, kCall, "general.alignment must be a nonzero u32");
    g->alignment = al->second.u;
  }
  g->tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    kq_gguf::Tensor& t = g->tensors[i];
    if (!c.str(t.name, "tensor name") || !c.get(t.n_dims, "dimension count"))
      return fail(KQ_E_INVALID, kCall, c.err);
    if (t.n_dims < 1 || t.n_dims > 4)
      return fail(KQ_E_INVALID, kCall, "tensor " + t.name + " has " + std::to_string(t.n_dims) +
                                           " dimensions (1..4)");
    for (uint32_t d = 0; d < t.n_dims; ++d)
      if (!c.get(t.dims[d], "dimension")) return fail(KQ_E_INVALID, kCall, c.err);
    if (!c.get(t.type, "tensor type") || !c.get(t.offset, "tensor offset"))
      return fail(KQ_E_INVALID, kCall, c.err);
  }
  g->data_start = (c.at + g->alignment - 1) / g->alignment * g->alignment;
  for (kq_gguf::Tensor& t : g->tensors) {
    uint64_t block = 0, bytes = 0;
    if (!type_size(t.type, block, bytes)) continue;  // nbytes stays 0: size unknown here
    if (t.dims[0] % block)
      return fail(KQ_E_INVALID, kCall, "tensor " + t.name + ": " + std::to_string(t.dims[0]) +
                                           " elements per row, not whole blocks of " +
                                           std::to_string(block));
    uint64_t n = t.dims[0] / block * bytes;
    for (int d = 1; d < 4; ++d) {
      if (t.dims[d] && n > ~uint64_t(0) / t.dims[d])
        return fail(KQ_E_INVALID, kCall, "tensor " + t.name + " size overflows");
      n *= t.dims[d];
    }
    t.nbytes = n;
    if (t.offset % g->alignment || t.offset > g->size || g->data_start > g->size - t.offset ||
        n > g->size - g->data_start - t.offset)
      return fail(KQ_E_INVALID, kCall, "tensor " + t.name + " (offset " +
                                           std::to_string(t.offset) + ", " + std::to_string(n) +
                                           " bytes) lies outside the file's data section");
  }
  return KQ_OK;
}

void gguf_release(kq_gguf* g) {
  if (g->base) munmap(const_cast<uint8_t*>(g->base), g->size);
  if (g->fd >= 0) close(g->fd);
  delete g;
}

void gguf_describe(const kq_gguf* g, const kq_gguf::Tensor& t, kq_gguf_tensor* out) {
  out->name = t.name.c_str();
  out->type = t.type;
  out->n_dims = t.n_dims;
  for (int d = 0; d < 4; ++d) out->dims[d] = t.dims[d];
  out->offset = g->data_start + t.offset;
  out->nbytes = t.nbytes;
  out->data = g->base + g->data_start + t.offset;
}

}  // namespace
}  // namespace kq

using kq::fail;

extern "C" {

int kq_gguf_open(const char* path, kq_gguf** out) {
  if (!path || !out) return fail(KQ_E_INVALID, kq::kCall, "null argument");
  *out = nullptr;
  kq_gguf* g = new kq_gguf;
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    const int e = errno;
    kq::gguf_release(g);
    return fail(KQ_E_INVALID, kq::kCall, std::string(path) + ": " + std::strerror(e));
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0 || st.st_size < 24) {
    kq::gguf_release(g);
    return fail(KQ_E_INVALID, kq::kCall, std::string(path) + ": not a GGUF file (too short)");
  }
  g->size = static_cast<uint64_t>(st.st_size);
  void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
  if (m == MAP_FAILED) {
    const int e = errno;
    g->size = 0;
    kq::gguf_release(g);
    return fail(KQ_E_INVALID, kq::kCall, std::string(path) + ": mmap: " + std::strerror(e));
  }
  g->base = static_cast<const uint8_t*>(m);
  const int rc = kq::parse(g);
  if (rc != KQ_OK) {
    kq::gguf_release(g);
    return rc;
  }
  *out = g;
  return KQ_OK;
}

int kq_gguf_close(kq_gguf* g) {
  if (g) kq::gguf_release(g);
  return KQ_OK;
}

uint64_t kq_gguf_tensor_count(const kq_gguf* g) { return g ? g->tensors.size() : 0; }

int kq_gguf_tensor_at(const kq_gguf* g, uint64_t i, kq_gguf_tensor* out) {
  if (!g || !out) return fail(KQ_E_INVALID, "kq_gguf_tensor_at", "null argument");
  if (i >= g->tensors.size())
    return fail(KQ_E_INVALID, "kq_gguf_tensor_at",
                "index " + std::to_string(i) + " of " + std::to_string(g->tensors.size()));
  kq::gguf_describe(g, g->tensors[i], out);
  return KQ_OK;
}

int kq_gguf_find(const kq_gguf* g, const char* name, kq_gguf_tensor* out) {
  if (!g || !name || !out) return fail(KQ_E_INVALID, "kq_gguf_find", "null argument");
  for (const kq_gguf::Tensor& t : g->tensors)
    if (t.name == name) {
      kq::gguf_describe(g, t, out);
      return KQ_OK;
    }
  return fail(KQ_E_INVALID, "kq_gguf_find", std::string("no tensor named ") + name);
}

int kq_gguf_meta_int(const kq_gguf* g, const char* key, int64_t* out) {
  if (!g || !key || !out) return fail(KQ_E_INVALID, "kq_gguf_meta_int", "null argument");
  const auto it = g->meta.find(key);
  if (it == g->meta.end())
    return fail(KQ_E_INVALID, "kq_gguf_meta_int", std::string("no metadata key ") + key);
  const uint32_t t = it->second.type;
  if (t == 6 || t == 8 || t == 9 || t == 12)
    return fail(KQ_E_INVALID, "kq_gguf_meta_int", std::string(key) + " is not an integer");
  *out = static_cast<int64_t>(it->second.u);
  return KQ_OK;
}

int kq_gguf_meta_str(const kq_gguf* g, const char* key, const char** out) {
  if (!g || !key || !out) return fail(KQ_E_INVALID, "kq_gguf_meta_str", "null argument");
  const auto it = g->meta.find(key);
  if (it == g->meta.end() || it->second.type != 8)
    return fail(KQ_E_INVALID, "kq_gguf_meta_str", std::string("no string metadata ") + key);
  *out = it->second.s.c_str();
  return KQ_OK;
}

}  // extern "C"
