// Host-side file I/O for the runtime: a minimal JSON reader (configs and safetensors
// headers, the role of the reference's src/core/json.cpp) and an mmap safetensors
// reader that hands out raw tensor bytes (the reference's src/core/weights.cpp reads
// the same files but converts every tensor to an fp32 host copy; here the bytes are
// uploaded to the device in their stored dtype).
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace wc {

struct JsonValue {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<JsonValue> arr;
  std::map<std::string, JsonValue> obj;

  bool has(const std::string& k) const { return kind == Obj && obj.count(k) && obj.at(k).kind != Null; }
  const JsonValue& at(const std::string& k) const {
    if (kind != Obj || !obj.count(k)) throw std::runtime_error("missing key '" + k + "'");
    return obj.at(k);
  }
  double number_or(const std::string& k, double d) const { return has(k) ? at(k).num : d; }
  bool bool_or(const std::string& k, bool d) const { return has(k) ? at(k).b : d; }
  std::string str_or(const std::string& k, const std::string& d) const { return has(k) ? at(k).str : d; }
};

class JsonReader {
 public:
  explicit JsonReader(const std::string& s) : s_(s) {}
  JsonValue parse() {
    JsonValue v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;

  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool eat(const char* lit) {
    const size_t n = std::strlen(lit);
    if (s_.compare(i_, n, lit) == 0) {
      i_ += n;
      return true;
    }
    return false;
  }
  JsonValue value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    JsonValue v;
    const char c = s_[i_];
    if (c == '{') {
      v.kind = JsonValue::Obj;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (true) {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected key");
        std::string k = string_lit();
        ws();
        if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
        ++i_;
        v.obj[k] = value();
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == '}') {
          ++i_;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = JsonValue::Arr;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == ']') {
          ++i_;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = JsonValue::Str;
      v.str = string_lit();
      return v;
    }
    if (eat("true")) {
      v.kind = JsonValue::Bool;
      v.b = true;
      return v;
    }
    if (eat("false")) {
      v.kind = JsonValue::Bool;
      return v;
    }
    if (eat("null")) return v;
    // number
    const size_t st = i_;
    while (i_ < s_.size() && (std::strchr("+-0123456789.eE", s_[i_]) != nullptr)) ++i_;
    if (st == i_) fail("unexpected character");
    v.kind = JsonValue::Num;
    v.num = std::stod(s_.substr(st, i_ - st));
    return v;
  }
  std::string string_lit() {
    ++i_;  // opening quote
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) fail("bad escape");
        const char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i_ + 4 > s_.size()) fail("bad \\u escape");
            const unsigned cp = unsigned(std::stoul(s_.substr(i_, 4), nullptr, 16));
            i_ += 4;
            if (cp < 0x80) out += char(cp);
            else if (cp < 0x800) {
              out += char(0xC0 | (cp >> 6));
              out += char(0x80 | (cp & 0x3F));
            } else {
              out += char(0xE0 | (cp >> 12));
              out += char(0x80 | ((cp >> 6) & 0x3F));
              out += char(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    ++i_;
    return out;
  }
};

inline JsonValue json_parse(const std::string& s) { return JsonReader(s).parse(); }

inline std::string read_file(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot read " + path);
  std::string out;
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) out.append(buf, n);
  std::fclose(f);
  return out;
}

struct TensorView {
  std::string dtype;            // "F32" | "BF16" | "F16"
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

class SafetensorsFile {
 public:
  explicit SafetensorsFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("cannot open " + path);
    struct stat st {};
    if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
    size_ = size_t(st.st_size);
    if (size_ < 8) throw std::runtime_error("truncated safetensors file " + path);
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) throw std::runtime_error("mmap failed for " + path);
    base_ = static_cast<const uint8_t*>(m);
    try {
      parse(path);
    } catch (...) {  // the destructor does not run for a throwing constructor
      munmap(const_cast<uint8_t*>(base_), size_);
      ::close(fd_);
      base_ = nullptr;
      fd_ = -1;
      throw;
    }
  }
  ~SafetensorsFile() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    if (fd_ >= 0) ::close(fd_);
  }
  SafetensorsFile(const SafetensorsFile&) = delete;
  SafetensorsFile& operator=(const SafetensorsFile&) = delete;
  const std::map<std::string, TensorView>& tensors() const { return tensors_; }

 private:
  void parse(const std::string& path) {
    uint64_t hlen = 0;
    std::memcpy(&hlen, base_, 8);
    if (hlen > size_ - 8) throw std::runtime_error("corrupt safetensors header length in " + path);
    const std::string header(reinterpret_cast<const char*>(base_ + 8), size_t(hlen));
    const JsonValue h = json_parse(header);
    if (h.kind != JsonValue::Obj) throw std::runtime_error("corrupt safetensors header in " + path);
    const uint8_t* data = base_ + 8 + hlen;
    const size_t data_size = size_ - 8 - hlen;
    for (auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      TensorView t;
      t.dtype = kv.second.at("dtype").str;
      for (auto& s : kv.second.at("shape").arr) t.shape.push_back(int64_t(s.num));
      const auto& off = kv.second.at("data_offsets").arr;
      if (off.size() != 2) throw std::runtime_error("bad data_offsets for " + kv.first);
      const size_t b = size_t(off[0].num), e = size_t(off[1].num);
      if (b > e || e > data_size) throw std::runtime_error("data_offsets out of range for " + kv.first);
      t.data = data + b;
      t.bytes = e - b;
      tensors_[kv.first] = t;
    }
  }

  int fd_ = -1;
  size_t size_ = 0;
  const uint8_t* base_ = nullptr;
  std::map<std::string, TensorView> tensors_;
};

}  // namespace wc
