// safetensors.hpp -- reads one tensor's entry from a .safetensors header (host code).
//
// File layout (the format Envision reads in src/safetensor.pas:466-513): an 8-byte little-endian
// header length n, n bytes of JSON mapping tensor names to {"dtype", "shape", "data_offsets"}
// (an optional "__metadata__" entry carries no offsets), then the raw little-endian data;
// data_offsets are relative to the end of the header.
#pragma once
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

namespace envg_st {

struct TensorInfo {
  std::string dtype;           // "BF16", "F16", "F32", ...
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;  // byte offsets relative to the data section
  int64_t data_start = 0;      // absolute file offset of the data section (8 + header length)
};

// Minimal JSON scanner for the header: strings (with escapes), numbers, arrays, objects.
class Scanner {
 public:
  Scanner(const char* p, const char* e) : p_(p), e_(e) {}
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool eat(char c) {
    ws();
    if (p_ < e_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  bool string(std::string* out) {
    ws();
    if (p_ >= e_ || *p_ != '"') return false;
    ++p_;
    std::string s;
    while (p_ < e_ && *p_ != '"') {
      if (*p_ == '\\' && p_ + 1 < e_) {
        ++p_;
        switch (*p_) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u':  // keep \uXXXX as written (names are ASCII in practice)
            s += "\\u";
            break;
          default: s += *p_;
        }
        ++p_;
      } else {
        s += *p_++;
      }
    }
    if (p_ >= e_) return false;
    ++p_;
    if (out) *out = s;
    return true;
  }
  bool integer(int64_t* out) {
    ws();
    const char* b = p_;
    if (p_ < e_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
    if (p_ == b) return false;
    *out = strtoll(std::string(b, p_).c_str(), nullptr, 10);
    return true;
  }
  bool int_array(std::vector<int64_t>* out) {
    if (!eat('[')) return false;
    out->clear();
    if (eat(']')) return true;
    do {
      int64_t v;
      if (!integer(&v)) return false;
      out->push_back(v);
    } while (eat(','));
    return eat(']');
  }
  // Skips any JSON value.
  bool skip() {
    ws();
    if (p_ >= e_) return false;
    if (*p_ == '"') return string(nullptr);
    if (*p_ == '{' || *p_ == '[') {
      const char open = *p_, close = open == '{' ? '}' : ']';
      ++p_;
      if (eat(close)) return true;
      do {
        if (open == '{') {
          if (!string(nullptr) || !eat(':')) return false;
        }
        if (!skip()) return false;
      } while (eat(','));
      return eat(close);
    }
    while (p_ < e_ && *p_ != ',' && *p_ != '}' && *p_ != ']' && *p_ != ' ' && *p_ != '\n') ++p_;
    return true;
  }

 private:
  const char* p_;
  const char* e_;
};

// Looks `name` up in the header of the file at `path`.  Returns an empty string on success, or
// the reason it failed.
inline std::string find_tensor(const char* path, const char* name, TensorInfo* info) {
  FILE* f = fopen(path, "rb");
  if (!f) return std::string("cannot open ") + path;
  uint64_t n = 0;
  if (fread(&n, 8, 1, f) != 1) {
    fclose(f);
    return "file too short for a safetensors header";
  }
  fseek(f, 0, SEEK_END);
  const long long fsize = ftell(f);
  if (n == 0 || (long long)n > fsize - 8) {
    fclose(f);
    return "invalid safetensors header length";
  }
  std::vector<char> hdr(n);
  fseek(f, 8, SEEK_SET);
  const size_t got = fread(hdr.data(), 1, n, f);
  fclose(f);
  if (got != n) return "truncated safetensors header";
  Scanner sc(hdr.data(), hdr.data() + n);
  if (!sc.eat('{')) return "header is not a JSON object";
  if (sc.eat('}')) return std::string("tensor not found: ") + name;
  do {
    std::string key;
    if (!sc.string(&key) || !sc.eat(':')) return "malformed header";
    if (key != name) {
      if (!sc.skip()) return "malformed header";
      continue;
    }
    if (!sc.eat('{')) return "tensor entry is not an object";
    bool have_dtype = false, have_shape = false, have_off = false;
    if (!sc.eat('}')) {
      do {
        std::string field;
        if (!sc.string(&field) || !sc.eat(':')) return "malformed tensor entry";
        if (field == "dtype") {
          have_dtype = sc.string(&info->dtype);
          if (!have_dtype) return "bad dtype";
        } else if (field == "shape") {
          have_shape = sc.int_array(&info->shape);
          if (!have_shape) return "bad shape";
        } else if (field == "data_offsets") {
          std::vector<int64_t> o;
          if (!sc.int_array(&o) || o.size() != 2) return "bad data_offsets";
          info->begin = o[0];
          info->end = o[1];
          have_off = true;
        } else if (!sc.skip()) {
          return "malformed tensor entry";
        }
      } while (sc.eat(','));
      if (!sc.eat('}')) return "malformed tensor entry";
    }
    if (!have_dtype || !have_off) return "tensor entry lacks dtype or data_offsets";
    if (!have_shape) info->shape.clear();
    info->data_start = 8 + (int64_t)n;
    if (info->begin < 0 || info->end < info->begin || info->data_start + info->end > fsize)
      return "tensor data outside the file";
    return "";
  } while (sc.eat(','));
  return std::string("tensor not found: ") + name;
}

inline int64_t dtype_bytes(const std::string& dt) {
  if (dt == "BF16" || dt == "F16") return 2;
  if (dt == "F32") return 4;
  return 0;
}

}  // namespace envg_st
