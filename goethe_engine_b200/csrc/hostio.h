// Host-side readers used by gc_open: a small JSON parser (manifest.json) and a GGUF v2/v3 reader (tensor table,
// metadata, memory-mapped tensor data). Plain C++17, no dependencies.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace gck {

// ---------------------------------------------------------------------------------------------------- JSON
struct Json {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  const Json *get(const std::string &k) const {
    if (kind != Obj) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
  double num_or(const std::string &k, double d) const {
    const Json *j = get(k);
    return j && j->kind == Num ? j->num : d;
  }
  std::string str_or(const std::string &k, const std::string &d) const {
    const Json *j = get(k);
    return j && j->kind == Str ? j->str : d;
  }
};

class JsonParser {
 public:
  explicit JsonParser(const std::string &s) : s_(s) {}
  Json parse() {
    Json j = value();
    ws();
    if (i_ != s_.size()) throw std::runtime_error("trailing characters in JSON");
    return j;
  }

 private:
  const std::string &s_;
  size_t i_ = 0;
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) i_++;
  }
  char peek() {
    ws();
    if (i_ >= s_.size()) throw std::runtime_error("unexpected end of JSON");
    return s_[i_];
  }
  void expect(char c) {
    if (peek() != c) throw std::runtime_error(std::string("JSON: expected ") + c);
    i_++;
  }
  std::string string() {
    expect('"');
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) break;
        char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            unsigned cp = std::stoul(s_.substr(i_, 4), nullptr, 16);
            i_ += 4;
            if (cp < 0x80) out += static_cast<char>(cp);
            else if (cp < 0x800) { out += static_cast<char>(0xc0 | (cp >> 6)); out += static_cast<char>(0x80 | (cp & 63)); }
            else { out += static_cast<char>(0xe0 | (cp >> 12)); out += static_cast<char>(0x80 | ((cp >> 6) & 63)); out += static_cast<char>(0x80 | (cp & 63)); }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) throw std::runtime_error("unterminated JSON string");
    i_++;
    return out;
  }
  Json value() {
    Json j;
    char c = peek();
    if (c == '{') {
      i_++;
      j.kind = Json::Obj;
      if (peek() == '}') { i_++; return j; }
      while (true) {
        std::string k = string();
        expect(':');
        j.obj[k] = value();
        char d = peek();
        i_++;
        if (d == '}') break;
        if (d != ',') throw std::runtime_error("JSON: expected , or }");
      }
    } else if (c == '[') {
      i_++;
      j.kind = Json::Arr;
      if (peek() == ']') { i_++; return j; }
      while (true) {
        j.arr.push_back(value());
        char d = peek();
        i_++;
        if (d == ']') break;
        if (d != ',') throw std::runtime_error("JSON: expected , or ]");
      }
    } else if (c == '"') {
      j.kind = Json::Str;
      j.str = string();
    } else if (s_.compare(i_, 4, "true") == 0) {
      j.kind = Json::Bool; j.b = true; i_ += 4;
    } else if (s_.compare(i_, 5, "false") == 0) {
      j.kind = Json::Bool; i_ += 5;
    } else if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
    } else {
      size_t k = i_;
      while (k < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[k])) || s_[k] == '-' || s_[k] == '+' ||
                               s_[k] == '.' || s_[k] == 'e' || s_[k] == 'E'))
        k++;
      if (k == i_) throw std::runtime_error("JSON: bad value");
      j.kind = Json::Num;
      j.num = std::strtod(s_.substr(i_, k - i_).c_str(), nullptr);
      i_ = k;
    }
    return j;
  }
};

// ---------------------------------------------------------------------------------------------------- GGUF
struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;   // ggml order: dims[0] = row length
  uint32_t type = 0;
  const uint8_t *data = nullptr;
  size_t bytes = 0;
};

struct GgufMeta {
  int kind = 0;           // 0 int, 1 float, 2 string, 3 other
  long long i = 0;
  double f = 0;
  std::string s;
};

class GgufFile {
 public:
  std::map<std::string, GgufMeta> meta;
  std::map<std::string, GgufTensor> tensors;

  explicit GgufFile(const std::string &path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error(path + ": cannot open");
    struct stat st;
    if (fstat(fd_, &st) != 0) throw std::runtime_error(path + ": cannot stat");
    size_ = static_cast<size_t>(st.st_size);
    map_ = static_cast<uint8_t *>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
    if (map_ == MAP_FAILED) { map_ = nullptr; throw std::runtime_error(path + ": cannot map"); }
    parse();
  }
  ~GgufFile() {
    if (map_) munmap(map_, size_);
    if (fd_ >= 0) ::close(fd_);
  }
  GgufFile(const GgufFile &) = delete;
  GgufFile &operator=(const GgufFile &) = delete;

 private:
  std::string path_;
  int fd_ = -1;
  uint8_t *map_ = nullptr;
  size_t size_ = 0, pos_ = 0;

  void need(size_t n) {
    if (pos_ + n > size_) throw std::runtime_error(path_ + ": truncated GGUF header");
  }
  template <typename T>
  T rd() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, map_ + pos_, sizeof(T));
    pos_ += sizeof(T);
    return v;
  }
  std::string rstr() {
    uint64_t n = rd<uint64_t>();
    need(n);
    std::string s(reinterpret_cast<const char *>(map_ + pos_), n);
    pos_ += n;
    return s;
  }
  GgufMeta rval(uint32_t t) {
    GgufMeta m;
    switch (t) {
      case 0: m.i = rd<uint8_t>(); break;
      case 1: m.i = rd<int8_t>(); break;
      case 2: m.i = rd<uint16_t>(); break;
      case 3: m.i = rd<int16_t>(); break;
      case 4: m.i = rd<uint32_t>(); break;
      case 5: m.i = rd<int32_t>(); break;
      case 6: m.kind = 1; m.f = rd<float>(); break;
      case 7: m.i = rd<uint8_t>(); break;
      case 8: m.kind = 2; m.s = rstr(); break;
      case 9: {
        uint32_t et = rd<uint32_t>();
        uint64_t n = rd<uint64_t>();
        for (uint64_t k = 0; k < n; k++) rval(et);
        m.kind = 3;
        break;
      }
      case 10: m.i = static_cast<long long>(rd<uint64_t>()); break;
      case 11: m.i = rd<int64_t>(); break;
      case 12: m.kind = 1; m.f = rd<double>(); break;
      default: throw std::runtime_error(path_ + ": unknown GGUF metadata type");
    }
    if (m.kind == 0) m.f = static_cast<double>(m.i);
    if (m.kind == 1) m.i = static_cast<long long>(m.f);
    return m;
  }
  static size_t tensor_bytes(uint32_t type, const std::vector<uint64_t> &dims) {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    switch (type) {
      case 0: return n * 4;
      case 1: return n * 2;
      case 8: return n / 32 * 34;
      case 12: return n / 256 * 144;
      default: return 0;   // a type this library does not read: size unknown, only an error if it is used
    }
  }
  void parse() {
    if (size_ < 4 || std::memcmp(map_, "GGUF", 4) != 0) throw std::runtime_error(path_ + ": not a GGUF file");
    pos_ = 4;
    uint32_t ver = rd<uint32_t>();
    if (ver != 2 && ver != 3) throw std::runtime_error(path_ + ": unsupported GGUF version");
    uint64_t nt = rd<uint64_t>(), nkv = rd<uint64_t>();
    for (uint64_t k = 0; k < nkv; k++) {
      std::string key = rstr();
      meta[key] = rval(rd<uint32_t>());
    }
    std::vector<std::pair<GgufTensor, uint64_t>> infos;
    for (uint64_t k = 0; k < nt; k++) {
      GgufTensor t;
      t.name = rstr();
      uint32_t nd = rd<uint32_t>();
      if (nd > 8) throw std::runtime_error(path_ + ": tensor rank");
      for (uint32_t d = 0; d < nd; d++) t.dims.push_back(rd<uint64_t>());
      t.type = rd<uint32_t>();
      uint64_t off = rd<uint64_t>();
      infos.emplace_back(t, off);
    }
    size_t align = 32;
    auto a = meta.find("general.alignment");
    if (a != meta.end() && a->second.i > 0) align = static_cast<size_t>(a->second.i);
    size_t base = (pos_ + align - 1) / align * align;
    for (auto &p : infos) {
      GgufTensor t = p.first;
      t.bytes = tensor_bytes(t.type, t.dims);
      if (base + p.second + t.bytes > size_) throw std::runtime_error(path_ + ": tensor " + t.name + " past the end");
      t.data = map_ + base + p.second;
      tensors[t.name] = t;
    }
  }
};

}  // namespace gck
