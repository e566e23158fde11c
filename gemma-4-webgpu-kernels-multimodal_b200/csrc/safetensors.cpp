#include "safetensors.h"

#include <ctype.h>
#include <fcntl.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace g4m {

namespace {

// Just enough JSON for a safetensors header: objects, arrays, strings,
// numbers and literals.
struct Json {
  const char* p;
  const char* e;
  void ws() {
    while (p < e && isspace((unsigned char)*p)) ++p;
  }
  bool lit(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) {
        ++p;
        char c = *p++;
        if (c == 'u') {
          if (e - p < 4) return false;
          unsigned v = (unsigned)strtoul(std::string(p, p + 4).c_str(), nullptr, 16);
          p += 4;
          if (v < 0x80) out.push_back((char)v);
          else if (v < 0x800) {
            out.push_back((char)(0xC0 | (v >> 6)));
            out.push_back((char)(0x80 | (v & 0x3F)));
          } else {
            out.push_back((char)(0xE0 | (v >> 12)));
            out.push_back((char)(0x80 | ((v >> 6) & 0x3F)));
            out.push_back((char)(0x80 | (v & 0x3F)));
          }
        } else {
          out.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c == 'r' ? '\r' : c == 'b' ? '\b' : c == 'f' ? '\f' : c);
        }
      } else {
        out.push_back(*p++);
      }
    }
    if (p >= e) return false;
    ++p;
    return true;
  }
  bool num(double& v) {
    ws();
    char* end = nullptr;
    std::string tmp(p, (size_t)((e - p) < 64 ? (e - p) : 64));
    v = strtod(tmp.c_str(), &end);
    if (end == tmp.c_str()) return false;
    p += (end - tmp.c_str());
    return true;
  }
  bool skip() {
    ws();
    if (p >= e) return false;
    if (*p == '"') {
      std::string s;
      return str(s);
    }
    if (*p == '{') {
      ++p;
      if (lit('}')) return true;
      do {
        std::string k;
        if (!str(k) || !lit(':') || !skip()) return false;
      } while (lit(','));
      return lit('}');
    }
    if (*p == '[') {
      ++p;
      if (lit(']')) return true;
      do {
        if (!skip()) return false;
      } while (lit(','));
      return lit(']');
    }
    if (!strncmp(p, "true", 4) && e - p >= 4) { p += 4; return true; }
    if (!strncmp(p, "false", 5) && e - p >= 5) { p += 5; return true; }
    if (!strncmp(p, "null", 4) && e - p >= 4) { p += 4; return true; }
    double v;
    return num(v);
  }
  bool int_array(std::vector<int64_t>& out) {
    out.clear();
    if (!lit('[')) return false;
    if (lit(']')) return true;
    do {
      double v;
      if (!num(v)) return false;
      out.push_back((int64_t)v);
    } while (lit(','));
    return lit(']');
  }
};

}  // namespace

SafeTensors::~SafeTensors() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

bool SafeTensors::open(const std::string& path, std::string& err) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    err = "cannot open safetensors file: " + path;
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    ::close(fd);
    err = "safetensors file too small: " + path;
    return false;
  }
  size_ = (size_t)st.st_size;
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) {
    err = "cannot map safetensors file: " + path;
    return false;
  }
  base_ = (const uint8_t*)m;
  uint64_t hlen;
  memcpy(&hlen, base_, 8);
  if (hlen > 100ull * 1024 * 1024 || 8 + hlen > size_) {
    err = "safetensors header length out of range";
    return false;
  }
  data_off_ = 8 + hlen;
  Json j{(const char*)base_ + 8, (const char*)base_ + 8 + hlen};
  if (!j.lit('{')) {
    err = "safetensors header is not a JSON object";
    return false;
  }
  if (!j.lit('}')) {
    do {
      std::string name;
      if (!j.str(name) || !j.lit(':')) {
        err = "malformed safetensors header";
        return false;
      }
      if (name == "__metadata__") {
        if (!j.skip()) {
          err = "malformed safetensors metadata";
          return false;
        }
        continue;
      }
      TensorInfo ti;
      if (!j.lit('{')) {
        err = "malformed tensor entry: " + name;
        return false;
      }
      do {
        std::string key;
        if (!j.str(key) || !j.lit(':')) {
          err = "malformed tensor entry: " + name;
          return false;
        }
        if (key == "dtype") {
          if (!j.str(ti.dtype)) return (err = "bad dtype: " + name, false);
        } else if (key == "shape") {
          if (!j.int_array(ti.shape)) return (err = "bad shape: " + name, false);
        } else if (key == "data_offsets") {
          std::vector<int64_t> o;
          if (!j.int_array(o) || o.size() != 2) return (err = "bad data_offsets: " + name, false);
          ti.begin = (uint64_t)o[0];
          ti.end = (uint64_t)o[1];
        } else if (!j.skip()) {
          err = "malformed tensor entry: " + name;
          return false;
        }
      } while (j.lit(','));
      if (!j.lit('}')) {
        err = "malformed tensor entry: " + name;
        return false;
      }
      if (ti.end < ti.begin || data_off_ + ti.end > size_) {
        err = "tensor data out of file bounds: " + name;
        return false;
      }
      t_[name] = ti;
    } while (j.lit(','));
    if (!j.lit('}')) {
      err = "malformed safetensors header end";
      return false;
    }
  }
  return true;
}

const TensorInfo* SafeTensors::find(const std::string& name) const {
  auto it = t_.find(name);
  return it == t_.end() ? nullptr : &it->second;
}

std::string shape_str(const TensorInfo& t) {
  std::string s = t.dtype + " [";
  for (size_t i = 0; i < t.shape.size(); ++i) {
    if (i) s += ", ";
    s += std::to_string(t.shape[i]);
  }
  return s + "]";
}

}  // namespace g4m
