// safetensors.cu — host-side reader of the safetensors weight container, so a
// caller can map a checkpoint shard and move its tensors (affine-u4 packed
// weights, bf16 scales / biases / norm gains) to the device with this library
// alone. Host code only.
//
// Reference: src/format/safetensor.rs:1-91 (layout [u64 LE header length]
// [JSON header][tensor bytes], data_offsets relative to the end of the
// header, keys starting with "__" skipped) and the dtype names of
// src/format/dtype.rs:17-31. The reference panics on a malformed file; here
// every problem is a LISA_EINVAL from lisa_attn_st_open.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "../../include/lisa_attn.h"

namespace {

struct StTensor {
  std::string name;
  int dtype;
  std::vector<uint64_t> shape;
  uint64_t off;  // from the start of the data region
  uint64_t len;
};

// Minimal JSON reader for the header: objects, arrays, strings, numbers,
// true / false / null. Returns false on any syntax error.
struct Json {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool lit(const char* s) {
    const size_t n = strlen(s);
    if ((size_t)(e - p) < n || memcmp(p, s, n) != 0) return false;
    p += n;
    return true;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) return false;
        switch (*p) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (e - p < 5) return false;
            unsigned v = 0;
            for (int i = 1; i <= 4; ++i) {
              const char c = p[i];
              v <<= 4;
              if (c >= '0' && c <= '9') v |= c - '0';
              else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
              else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
              else return false;
            }
            p += 4;
            if (v < 0x80) out += (char)v;  // names are ASCII in practice; keep the rest as UTF-8
            else if (v < 0x800) { out += (char)(0xC0 | (v >> 6)); out += (char)(0x80 | (v & 0x3F)); }
            else { out += (char)(0xE0 | (v >> 12)); out += (char)(0x80 | ((v >> 6) & 0x3F)); out += (char)(0x80 | (v & 0x3F)); }
            break;
          }
          default: return false;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool uint(uint64_t& v) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return false;
    v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p - '0');
      if (v > (UINT64_MAX - d) / 10) return false;
      v = v * 10 + d;
      ++p;
    }
    return true;
  }
  bool skip() {  // any value
    ws();
    if (p >= e) return false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      ws();
      if (p < e && *p == close) { ++p; return true; }
      while (true) {
        if (obj) {
          std::string k;
          if (!str(k)) return false;
          ws();
          if (p >= e || *p != ':') return false;
          ++p;
        }
        if (!skip()) return false;
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == close) { ++p; return true; }
        return false;
      }
    }
    if (lit("true") || lit("false") || lit("null")) return true;
    // number
    const char* s = p;
    while (p < e && (strchr("+-0123456789.eE", *p) != nullptr)) ++p;
    return p > s;
  }
  bool uint_array(std::vector<uint64_t>& out) {
    ws();
    if (p >= e || *p != '[') return false;
    ++p;
    out.clear();
    ws();
    if (p < e && *p == ']') { ++p; return true; }
    while (true) {
      uint64_t v;
      if (!uint(v)) return false;
      out.push_back(v);
      ws();
      if (p < e && *p == ',') { ++p; continue; }
      if (p < e && *p == ']') { ++p; return true; }
      return false;
    }
  }
};

int dtype_code(const std::string& n) {
  static const char* names[] = {"BOOL", "U8", "U16", "I16", "F16", "BF16", "U32", "I32", "F32", "U64", "F64"};
  for (int i = 0; i < 11; ++i)
    if (n == names[i]) return i;
  return -1;
}

const uint64_t kElemBytes[] = {1, 1, 2, 2, 2, 2, 4, 4, 4, 8, 8};

// One tensor entry {"dtype":..., "shape":[...], "data_offsets":[a, b]}.
bool parse_entry(Json& j, StTensor& t) {
  j.ws();
  if (j.p >= j.e || *j.p != '{') return false;
  ++j.p;
  bool have_dtype = false, have_shape = false, have_off = false;
  j.ws();
  if (j.p < j.e && *j.p == '}') return false;
  while (true) {
    std::string key;
    if (!j.str(key)) return false;
    j.ws();
    if (j.p >= j.e || *j.p != ':') return false;
    ++j.p;
    if (key == "dtype") {
      std::string d;
      if (!j.str(d)) return false;
      t.dtype = dtype_code(d);
      if (t.dtype < 0) return false;
      have_dtype = true;
    } else if (key == "shape") {
      if (!j.uint_array(t.shape)) return false;
      have_shape = true;
    } else if (key == "data_offsets") {
      std::vector<uint64_t> o;
      if (!j.uint_array(o) || o.size() != 2 || o[1] < o[0]) return false;
      t.off = o[0];
      t.len = o[1] - o[0];
      have_off = true;
    } else if (!j.skip()) {
      return false;
    }
    j.ws();
    if (j.p < j.e && *j.p == ',') { ++j.p; continue; }
    if (j.p < j.e && *j.p == '}') { ++j.p; break; }
    return false;
  }
  return have_dtype && have_shape && have_off;
}

}  // namespace

struct lisa_attn_shard {
  void* map = nullptr;
  size_t map_bytes = 0;
  uint64_t data_start = 0;
  uint64_t data_len = 0;
  std::vector<StTensor> tensors;
};

#pragma GCC visibility push(default)
extern "C" {

int lisa_attn_st_open(const char* path, lisa_attn_shard** out) {
  if (!path || !out) return LISA_EINVAL;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return LISA_EINVAL;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    close(fd);
    return LISA_EINVAL;
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return LISA_EINVAL;
  lisa_attn_shard* s = new lisa_attn_shard();
  s->map = m;
  s->map_bytes = (size_t)st.st_size;
  const uint8_t* b = static_cast<const uint8_t*>(m);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
  bool ok = hlen <= s->map_bytes - 8;
  if (ok) {
    s->data_start = 8 + hlen;
    s->data_len = s->map_bytes - s->data_start;
    Json j{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hlen)};
    j.ws();
    ok = j.p < j.e && *j.p == '{';
    if (ok) {
      ++j.p;
      j.ws();
      if (j.p < j.e && *j.p == '}') {
        ++j.p;
      } else {
        while (ok) {
          std::string name;
          ok = j.str(name);
          if (!ok) break;
          j.ws();
          ok = j.p < j.e && *j.p == ':';
          if (!ok) break;
          ++j.p;
          if (name.compare(0, 2, "__") == 0) {
            ok = j.skip();  // __metadata__ and other top-level keys
          } else {
            StTensor t;
            ok = parse_entry(j, t);
            if (ok) {
              t.name = name;
              uint64_t elems = 1;
              for (uint64_t d : t.shape) elems *= d;
              // the byte range lies inside the data region and fits the shape
              ok = t.off + t.len <= s->data_len && t.len == elems * kElemBytes[t.dtype];
              if (ok) s->tensors.push_back(t);
            }
          }
          if (!ok) break;
          j.ws();
          if (j.p < j.e && *j.p == ',') { ++j.p; continue; }
          ok = j.p < j.e && *j.p == '}';
          break;
        }
      }
    }
  }
  if (!ok) {
    munmap(s->map, s->map_bytes);
    delete s;
    return LISA_EINVAL;
  }
  *out = s;
  return LISA_OK;
}

int lisa_attn_st_close(lisa_attn_shard* s) {
  if (!s) return LISA_EINVAL;
  munmap(s->map, s->map_bytes);
  delete s;
  return LISA_OK;
}

int lisa_attn_st_count(const lisa_attn_shard* s) { return s ? (int)s->tensors.size() : LISA_EINVAL; }

int lisa_attn_st_find(const lisa_attn_shard* s, const char* name) {
  if (!s || !name) return LISA_EINVAL;
  for (size_t i = 0; i < s->tensors.size(); ++i)
    if (s->tensors[i].name == name) return (int)i;
  return LISA_EINVAL;
}

int lisa_attn_st_info(const lisa_attn_shard* s, int index, char* name, size_t name_bytes, int* dtype,
                      uint64_t* shape, int max_dims, int* ndim, uint64_t* data_offset, uint64_t* nbytes) {
  if (!s || index < 0 || index >= (int)s->tensors.size()) return LISA_EINVAL;
  const StTensor& t = s->tensors[index];
  if (name && name_bytes) {
    const size_t n = t.name.size() < name_bytes - 1 ? t.name.size() : name_bytes - 1;
    memcpy(name, t.name.data(), n);
    name[n] = 0;
  }
  if (dtype) *dtype = t.dtype;
  if (ndim) *ndim = (int)t.shape.size();
  if (shape)
    for (int i = 0; i < max_dims && i < (int)t.shape.size(); ++i) shape[i] = t.shape[i];
  if (data_offset) *data_offset = t.off;
  if (nbytes) *nbytes = t.len;
  return LISA_OK;
}

int lisa_attn_st_host_ptr(const lisa_attn_shard* s, int index, const void** ptr) {
  if (!s || !ptr || index < 0 || index >= (int)s->tensors.size()) return LISA_EINVAL;
  *ptr = static_cast<const uint8_t*>(s->map) + s->data_start + s->tensors[index].off;
  return LISA_OK;
}

int lisa_attn_st_upload(const lisa_attn_shard* s, int index, void* dst, size_t dst_bytes, void* stream) {
  if (!s || !dst || index < 0 || index >= (int)s->tensors.size()) return LISA_EINVAL;
  const StTensor& t = s->tensors[index];
  if (dst_bytes < t.len) return LISA_EINVAL;
  const void* src = static_cast<const uint8_t*>(s->map) + s->data_start + t.off;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // pageable source: the copy is staged by the driver; synchronise so the
  // mapping may be closed as soon as this returns
  if (cudaMemcpyAsync(dst, src, t.len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return LISA_ECUDA;
  return LISA_OK;
}

}  // extern "C"
#pragma GCC visibility pop
