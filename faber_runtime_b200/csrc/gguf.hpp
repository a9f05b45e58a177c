// gguf.hpp — fail-closed GGUF v3 container reader (host code).
//
// The reference admits exactly one pinned file (src/gguf.rs:581-812:
// SHA-256, size, 37 keys, 290 tensors). This reader keeps that function's
// structural checks and drops the pin, so any llama-architecture GGUF v3 file
// can be parsed:
//   * magic "GGUF" and version 3;
//   * the KV and tensor counts are bounded by the bytes that remain before
//     anything is reserved for them;
//   * keys, strings and tensor names are length-capped and valid UTF-8; keys
//     and tensor names are unique; BOOL values are 0 or 1; arrays hold
//     scalars or strings (no nested arrays);
//   * tensors have 1..4 dimensions, each >= 1, with overflow-checked element
//     and byte counts; the dtype is one of the admitted GGML types and the
//     element count is a whole number of its blocks;
//   * offsets are aligned (general.alignment, default 32), sequential and
//     non-overlapping in table order (src/gguf.rs:707-735), and the data
//     region ends inside the buffer.
// The first violated check throws (INVALID_ARGUMENT) with its kind in the
// message, named after the reference's AdmissionError variants
// (src/gguf.rs:229-325). The reader keeps offsets only: the caller owns the
// bytes, and a tensor's data is bytes[offset, offset + nbytes).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <set>
#include <string>
#include <vector>

#include "common.cuh"

namespace faber {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint32_t kGgufVersion = 3;
constexpr uint64_t kGgufDefaultAlignment = 32;
constexpr uint64_t kGgufMaxKey = 1024;
constexpr uint64_t kGgufMaxString = 16u << 20;
constexpr uint64_t kGgufMaxName = 1024;
constexpr uint32_t kGgufMaxDims = 4;

// GGUF metadata value types (GGUF v3 specification).
enum GgufValueType : uint32_t {
  GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5,
  GGUF_F32 = 6, GGUF_BOOL = 7, GGUF_STRING = 8, GGUF_ARRAY = 9, GGUF_U64 = 10, GGUF_I64 = 11,
  GGUF_F64 = 12
};

// Admitted GGML tensor types: the reference's closed set (src/gguf.rs:124-192)
// plus F16; block elements and bytes per block.
inline bool ggml_geometry(uint32_t t, uint64_t& elems, uint64_t& bytes) {
  switch (t) {
    case 0: elems = 1; bytes = 4; return true;      // F32
    case 1: elems = 1; bytes = 2; return true;      // F16
    case 6: elems = 32; bytes = 22; return true;    // Q5_0
    case 8: elems = 32; bytes = 34; return true;    // Q8_0
    case 12: elems = 256; bytes = 144; return true; // Q4_K
    case 14: elems = 256; bytes = 210; return true; // Q6_K
    default: return false;
  }
}

struct GgufKv {
  std::string key;
  uint32_t type = 0;        // GgufValueType
  uint32_t arr_type = 0;    // element type of an array
  uint64_t arr_count = 0;
  uint64_t payload = 0;     // buffer offset of an array's first element
  uint64_t u = 0;           // unsigned integer / bool value
  int64_t i = 0;            // signed integer value
  double f = 0.0;           // float value
  std::string s;            // string value
};

struct GgufTensor {
  std::string name;
  uint32_t type = 0;
  uint32_t n_dims = 0;
  uint64_t dims[kGgufMaxDims] = {1, 1, 1, 1};  // GGML order: dims[0] is the contiguous one
  uint64_t elements = 0, nbytes = 0;
  uint64_t rel_offset = 0;  // inside the data region
  uint64_t offset = 0;      // inside the buffer
};

struct GgufFile {
  uint32_t version = 0;
  uint64_t alignment = kGgufDefaultAlignment;
  uint64_t data_offset = 0, data_len = 0;
  std::vector<GgufKv> kv;
  std::vector<GgufTensor> tensors;
  const GgufKv* find(const std::string& key) const {
    for (const GgufKv& k : kv)
      if (k.key == key) return &k;
    return nullptr;
  }
};

[[noreturn]] inline void gguf_fail(const std::string& kind, const std::string& detail) {
  throw Error(FABER_STATUS_INVALID_ARGUMENT, "GGUF " + kind + ": " + detail);
}

inline bool valid_utf8(const uint8_t* p, uint64_t n) {
  uint64_t i = 0;
  while (i < n) {
    const uint8_t c = p[i];
    uint64_t len;
    uint32_t cp;
    if (c < 0x80) { ++i; continue; }
    if ((c & 0xE0) == 0xC0) { len = 2; cp = c & 0x1F; }
    else if ((c & 0xF0) == 0xE0) { len = 3; cp = c & 0x0F; }
    else if ((c & 0xF8) == 0xF0) { len = 4; cp = c & 0x07; }
    else return false;
    if (i + len > n) return false;
    for (uint64_t k = 1; k < len; ++k) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    // overlong forms, surrogates and values past U+10FFFF are not UTF-8
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) ||
        (cp >= 0xD800 && cp <= 0xDFFF) || cp > 0x10FFFF)
      return false;
    i += len;
  }
  return true;
}

class GgufCursor {
 public:
  GgufCursor(const uint8_t* b, uint64_t n) : b_(b), n_(n) {}
  uint64_t pos() const { return pos_; }
  uint64_t left() const { return n_ - pos_; }
  const uint8_t* take(uint64_t k) {
    if (k > left())
      gguf_fail("TruncatedFile", "needed " + std::to_string(pos_ + k) + " bytes, available " +
                                     std::to_string(n_));
    const uint8_t* p = b_ + pos_;
    pos_ += k;
    return p;
  }
  template <class T>
  T read() {
    T v;
    std::memcpy(&v, take(sizeof(T)), sizeof(T));  // little-endian host
    return v;
  }
  std::string str(uint64_t cap, const char* kind, const std::string& ctx) {
    const uint64_t len = read<uint64_t>();
    if (len > cap) gguf_fail(kind, ctx + " is " + std::to_string(len) + " bytes, ceiling " + std::to_string(cap));
    const uint8_t* p = take(len);
    if (!valid_utf8(p, len)) gguf_fail("InvalidUtf8", ctx);
    return std::string(reinterpret_cast<const char*>(p), len);
  }

 private:
  const uint8_t* b_;
  uint64_t n_;
  uint64_t pos_ = 0;
};

inline uint64_t gguf_scalar_bytes(uint32_t t) {
  switch (t) {
    case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
    case GGUF_U16: case GGUF_I16: return 2;
    case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
    case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
    default: return 0;
  }
}

// One scalar of type t into kv (u / i / f), BOOL checked.
inline void gguf_scalar(GgufCursor& c, uint32_t t, GgufKv& kv) {
  switch (t) {
    case GGUF_U8: kv.u = c.read<uint8_t>(); kv.i = (int64_t)kv.u; break;
    case GGUF_I8: kv.i = c.read<int8_t>(); break;
    case GGUF_U16: kv.u = c.read<uint16_t>(); kv.i = (int64_t)kv.u; break;
    case GGUF_I16: kv.i = c.read<int16_t>(); break;
    case GGUF_U32: kv.u = c.read<uint32_t>(); kv.i = (int64_t)kv.u; break;
    case GGUF_I32: kv.i = c.read<int32_t>(); break;
    case GGUF_U64: kv.u = c.read<uint64_t>(); kv.i = (int64_t)kv.u; break;
    case GGUF_I64: kv.i = c.read<int64_t>(); break;
    case GGUF_F32: kv.f = c.read<float>(); break;
    case GGUF_F64: kv.f = c.read<double>(); break;
    case GGUF_BOOL: {
      const uint8_t v = c.read<uint8_t>();
      if (v > 1) gguf_fail("MalformedBool", kv.key + " holds " + std::to_string(v));
      kv.u = v;
      kv.i = v;
      break;
    }
    default: gguf_fail("MetadataValueMismatch", kv.key + ": unknown value type " + std::to_string(t));
  }
}

inline uint64_t gguf_align_up(uint64_t v, uint64_t a, const std::string& ctx) {
  if (v > UINT64_MAX - (a - 1)) gguf_fail("ArithmeticOverflow", ctx);
  return (v + a - 1) & ~(a - 1);
}

inline GgufFile gguf_parse(const uint8_t* bytes, uint64_t len) {
  GgufFile f;
  GgufCursor c(bytes, len);
  const uint32_t magic = c.read<uint32_t>();
  if (magic != kGgufMagic) gguf_fail("InvalidMagic", "0x" + [&] {
      char b[16];
      std::snprintf(b, sizeof b, "%08x", magic);
      return std::string(b);
    }());
  f.version = c.read<uint32_t>();
  if (f.version != kGgufVersion) gguf_fail("UnsupportedVersion", std::to_string(f.version));
  const uint64_t n_tensors = c.read<uint64_t>();
  const uint64_t n_kv = c.read<uint64_t>();
  // every KV takes at least 8 (key length) + 4 (type) + 1 bytes, every tensor
  // info at least 8 + 4 + 8 + 4 + 8: counts past that cannot be real
  if (n_kv > c.left() / 13)
    gguf_fail("MetadataKvCountMismatch", std::to_string(n_kv) + " KVs cannot fit in " +
                                             std::to_string(c.left()) + " bytes");
  if (n_tensors > c.left() / 32)
    gguf_fail("TensorCountMismatch", std::to_string(n_tensors) + " tensors cannot fit in " +
                                         std::to_string(c.left()) + " bytes");
  std::set<std::string> keys;
  f.kv.reserve(n_kv);
  for (uint64_t k = 0; k < n_kv; ++k) {
    GgufKv kv;
    kv.key = c.str(kGgufMaxKey, "KeyTooLong", "key");
    if (!keys.insert(kv.key).second) gguf_fail("DuplicateMetadataKey", kv.key);
    kv.type = c.read<uint32_t>();
    if (kv.type == GGUF_STRING) {
      kv.s = c.str(kGgufMaxString, "StringTooLong", kv.key);
    } else if (kv.type == GGUF_ARRAY) {
      kv.arr_type = c.read<uint32_t>();
      kv.arr_count = c.read<uint64_t>();
      kv.payload = c.pos();
      if (kv.arr_type == GGUF_STRING) {
        if (kv.arr_count > c.left() / 8)
          gguf_fail("TokenizerArrayCountMismatch", kv.key + ": " + std::to_string(kv.arr_count) +
                                                       " strings cannot fit");
        for (uint64_t e = 0; e < kv.arr_count; ++e) c.str(kGgufMaxString, "StringTooLong", kv.key);
      } else {
        const uint64_t es = gguf_scalar_bytes(kv.arr_type);
        if (es == 0)
          gguf_fail("MetadataValueMismatch", kv.key + ": array of value type " + std::to_string(kv.arr_type));
        if (kv.arr_count > c.left() / es)
          gguf_fail("TruncatedFile", kv.key + ": " + std::to_string(kv.arr_count) + " elements cannot fit");
        if (kv.arr_type == GGUF_BOOL) {
          const uint8_t* p = c.take(kv.arr_count);
          for (uint64_t e = 0; e < kv.arr_count; ++e)
            if (p[e] > 1) gguf_fail("MalformedBool", kv.key + "[" + std::to_string(e) + "]");
        } else {
          c.take(kv.arr_count * es);
        }
      }
    } else {
      gguf_scalar(c, kv.type, kv);
    }
    f.kv.push_back(std::move(kv));
  }
  if (const GgufKv* a = f.find("general.alignment")) {
    if (a->type != GGUF_U32 || a->u == 0 || (a->u & (a->u - 1)) != 0)
      gguf_fail("MetadataValueMismatch", "general.alignment must be a power-of-two UINT32");
    f.alignment = a->u;
  }
  std::set<std::string> names;
  f.tensors.reserve(n_tensors);
  uint64_t prev_end = 0, total = 0;
  for (uint64_t k = 0; k < n_tensors; ++k) {
    GgufTensor t;
    t.name = c.str(kGgufMaxName, "TensorNameTooLong", "tensor name");
    if (!names.insert(t.name).second) gguf_fail("DuplicateTensorName", t.name);
    t.n_dims = c.read<uint32_t>();
    if (t.n_dims == 0 || t.n_dims > kGgufMaxDims)
      gguf_fail("TensorDimCountMismatch", t.name + " has " + std::to_string(t.n_dims) + " dimensions");
    t.elements = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      t.dims[d] = c.read<uint64_t>();
      if (t.dims[d] == 0) gguf_fail("TensorDimTooLarge", t.name + " has a zero dimension");
      if (t.elements > UINT64_MAX / t.dims[d]) gguf_fail("ArithmeticOverflow", "dimensions of " + t.name);
      t.elements *= t.dims[d];
    }
    t.type = c.read<uint32_t>();
    uint64_t be = 0, bb = 0;
    if (!ggml_geometry(t.type, be, bb))
      gguf_fail("UnknownDtype", t.name + " has dtype " + std::to_string(t.type));
    t.rel_offset = c.read<uint64_t>();
    if (t.rel_offset % f.alignment != 0)
      gguf_fail("MisalignedTensorOffset", t.name + " at " + std::to_string(t.rel_offset));
    if (t.elements % be != 0)
      gguf_fail("TensorElementsNotBlockAligned", t.name + ": " + std::to_string(t.elements) +
                                                     " elements, blocks of " + std::to_string(be));
    // the innermost dimension holds whole blocks (a row never splits a block)
    if (t.dims[0] % be != 0)
      gguf_fail("TensorElementsNotBlockAligned", t.name + ": rows of " + std::to_string(t.dims[0]));
    const uint64_t blocks = t.elements / be;
    if (blocks > UINT64_MAX / bb) gguf_fail("ArithmeticOverflow", "byte length of " + t.name);
    t.nbytes = blocks * bb;
    if (t.rel_offset > UINT64_MAX - t.nbytes) gguf_fail("ArithmeticOverflow", "byte-range end of " + t.name);
    if (t.rel_offset < prev_end)
      gguf_fail("OverlappingTensorRanges", t.name + " at " + std::to_string(t.rel_offset) +
                                               ", previous range ends at " + std::to_string(prev_end));
    const uint64_t expect = gguf_align_up(prev_end, f.alignment, "tensor offsets");
    if (t.rel_offset != expect)
      gguf_fail("NonSequentialTensorOffsets", t.name + " at " + std::to_string(t.rel_offset) +
                                                  ", expected " + std::to_string(expect));
    prev_end = t.rel_offset + t.nbytes;
    if (total > UINT64_MAX - t.nbytes) gguf_fail("ArithmeticOverflow", "total tensor-data length");
    total += t.nbytes;
    f.tensors.push_back(std::move(t));
  }
  f.data_offset = gguf_align_up(c.pos(), f.alignment, "tensor-data region start");
  f.data_len = prev_end;
  if (f.data_offset > len || f.data_len > len - f.data_offset)
    gguf_fail("TruncatedTensorData", "data ends at " + std::to_string(f.data_offset) + " + " +
                                         std::to_string(f.data_len) + ", buffer holds " + std::to_string(len));
  for (GgufTensor& t : f.tensors) t.offset = f.data_offset + t.rel_offset;
  return f;
}

}  // namespace faber
