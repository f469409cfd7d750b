#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <memory>

#include "common.h"

namespace mx {
namespace {

// A minimal JSON reader: just enough for a safetensors header (objects,
// arrays, strings, integers; no floats, booleans or nulls are needed, but they
// are accepted and ignored).
struct Json {
  enum Kind { Null, Num, Str, Arr, Obj } kind = Null;
  int64_t num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
};

struct Parser {
  const char* p;
  const char* e;
  std::string where;

  [[noreturn]] void fail(const char* what) {
    throw Error(where + ": malformed safetensors header (" + what + ")", MX_E_IO);
  }
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  std::string string() {
    if (p >= e || *p != '"') fail("expected a string");
    ++p;
    std::string s;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        ++p;
        if (p >= e) fail("bad escape");
        char c = *p++;
        switch (c) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {
            if (e - p < 4) fail("bad \\u escape");
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else fail("bad \\u escape");
            }
            if (v < 0x80) s += char(v);
            else if (v < 0x800) { s += char(0xC0 | (v >> 6)); s += char(0x80 | (v & 0x3F)); }
            else { s += char(0xE0 | (v >> 12)); s += char(0x80 | ((v >> 6) & 0x3F)); s += char(0x80 | (v & 0x3F)); }
            break;
          }
          default: s += c;
        }
      } else {
        s += *p++;
      }
    }
    if (p >= e) fail("unterminated string");
    ++p;
    return s;
  }
  Json value() {
    ws();
    if (p >= e) fail("unexpected end");
    Json j;
    if (*p == '{') {
      j.kind = Json::Obj;
      ++p;
      ws();
      if (p < e && *p == '}') { ++p; return j; }
      for (;;) {
        ws();
        std::string k = string();
        ws();
        if (p >= e || *p != ':') fail("expected ':'");
        ++p;
        j.obj.emplace_back(std::move(k), value());
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == '}') { ++p; break; }
        fail("expected ',' or '}'");
      }
    } else if (*p == '[') {
      j.kind = Json::Arr;
      ++p;
      ws();
      if (p < e && *p == ']') { ++p; return j; }
      for (;;) {
        j.arr.push_back(value());
        ws();
        if (p < e && *p == ',') { ++p; continue; }
        if (p < e && *p == ']') { ++p; break; }
        fail("expected ',' or ']'");
      }
    } else if (*p == '"') {
      j.kind = Json::Str;
      j.str = string();
    } else if (*p == '-' || (*p >= '0' && *p <= '9')) {
      j.kind = Json::Num;
      bool neg = *p == '-';
      if (neg) ++p;
      int64_t v = 0;
      while (p < e && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
      // a fraction or exponent is not part of this format; skip it
      while (p < e && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' || (*p >= '0' && *p <= '9'))) ++p;
      j.num = neg ? -v : v;
    } else if (e - p >= 4 && (!strncmp(p, "true", 4) || !strncmp(p, "null", 4))) {
      p += 4;
    } else if (e - p >= 5 && !strncmp(p, "false", 5)) {
      p += 5;
    } else {
      fail("unexpected character");
    }
    return j;
  }
};

float half_to_float(uint16_t h) {
  uint32_t s = (h >> 15) & 1, ex = (h >> 10) & 0x1F, m = h & 0x3FF;
  uint32_t bits;
  if (ex == 0) {
    if (m == 0) {
      bits = s << 31;
    } else {  // subnormal: renormalise
      int e2 = -1;
      do { m <<= 1; ++e2; } while (!(m & 0x400));
      m &= 0x3FF;
      bits = (s << 31) | uint32_t(127 - 15 - e2) << 23 | (m << 13);
    }
  } else if (ex == 31) {
    bits = (s << 31) | 0x7F800000u | (m << 13);
  } else {
    bits = (s << 31) | (ex - 15 + 127) << 23 | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

}  // namespace

SafeTensors::SafeTensors(const std::string& path) : path_(path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error(path + ": " + strerror(errno), MX_E_IO);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw Error(path + ": stat failed", MX_E_IO);
  }
  map_len_ = size_t(st.st_size);
  if (map_len_ < 8) {
    ::close(fd);
    throw Error(path + ": too short to be a safetensors file", MX_E_IO);
  }
  map_ = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw Error(path + ": mmap failed", MX_E_IO);
  }
  const uint8_t* b = static_cast<const uint8_t*>(map_);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
  if (hlen > map_len_ - 8) {
    munmap(map_, map_len_);
    map_ = nullptr;
    throw Error(path + ": header length runs past the end of the file", MX_E_IO);
  }
  data_ = b + 8 + hlen;
  data_len_ = map_len_ - 8 - hlen;
  Parser ps{reinterpret_cast<const char*>(b + 8), reinterpret_cast<const char*>(b + 8 + hlen), path};
  Json root;
  try {
    root = ps.value();
  } catch (...) {
    munmap(map_, map_len_);
    map_ = nullptr;
    throw;
  }
  if (root.kind != Json::Obj) {
    munmap(map_, map_len_);
    map_ = nullptr;
    throw Error(path + ": header is not a JSON object", MX_E_IO);
  }
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      for (auto& m : kv.second.obj)
        if (m.second.kind == Json::Str) metadata_[m.first] = m.second.str;
      continue;
    }
    TensorInfo t;
    for (auto& f : kv.second.obj) {
      if (f.first == "dtype") t.dtype = f.second.str;
      else if (f.first == "shape")
        for (auto& d : f.second.arr) t.shape.push_back(d.num);
      else if (f.first == "data_offsets" && f.second.arr.size() == 2) {
        t.begin = uint64_t(f.second.arr[0].num);
        t.end = uint64_t(f.second.arr[1].num);
      }
    }
    if (t.end < t.begin || t.end > data_len_) {
      munmap(map_, map_len_);
      map_ = nullptr;
      throw Error(path + ": tensor " + kv.first + " runs past the end of the file", MX_E_IO);
    }
    tensors_[kv.first] = std::move(t);
  }
}

SafeTensors::~SafeTensors() {
  if (map_) munmap(map_, map_len_);
}

const TensorInfo& SafeTensors::info(const std::string& name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw Error(path_ + ": no tensor named " + name, MX_E_IO);
  return it->second;
}

std::vector<float> SafeTensors::f32(const std::string& name) const {
  const TensorInfo& t = info(name);
  int64_t n = t.numel();
  std::vector<float> out(static_cast<size_t>(n));
  const uint8_t* src = data_ + t.begin;
  size_t bytes = t.end - t.begin;
  auto need = [&](size_t esz) {
    if (bytes != size_t(n) * esz)
      throw Error(fmt("%s: tensor %s holds %zu bytes, its shape needs %zu", path_.c_str(), name.c_str(), bytes,
                      size_t(n) * esz),
                  MX_E_IO);
  };
  if (t.dtype == "F32") {
    need(4);
    memcpy(out.data(), src, bytes);
  } else if (t.dtype == "F16") {
    need(2);
    for (int64_t i = 0; i < n; ++i) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      out[i] = half_to_float(h);
    }
  } else if (t.dtype == "BF16") {
    need(2);
    for (int64_t i = 0; i < n; ++i) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      uint32_t bits = uint32_t(h) << 16;
      memcpy(&out[i], &bits, 4);
    }
  } else if (t.dtype == "F64") {
    need(8);
    for (int64_t i = 0; i < n; ++i) {
      double d;
      memcpy(&d, src + 8 * i, 8);
      out[i] = float(d);
    }
  } else {
    throw Error(path_ + ": tensor " + name + " has dtype " + t.dtype + ", not a float type", MX_E_IO);
  }
  return out;
}

}  // namespace mx
