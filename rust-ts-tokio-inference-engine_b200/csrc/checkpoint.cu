// safetensors reader (host only): an 8-byte little-endian header length, a
// JSON header {name: {"dtype", "shape", "data_offsets": [begin, end]}, ...,
// "__metadata__": {...}}, then the data block the offsets index.
#include "checkpoint.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>

namespace qwen {

namespace {

// A minimal JSON value: enough for safetensors headers.
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  double num = 0;
  bool b = false;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const {
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  Json parse_document() {
    Json v = value(0);
    ws();
    if (p_ != end_) fail("trailing bytes after the header object");
    return v;
  }

 private:
  [[noreturn]] void fail(const char* what) { throw std::invalid_argument(std::string("safetensors header: ") + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool eat(char c) {
    ws();
    if (p_ < end_ && *p_ == c) {
      ++p_;
      return true;
    }
    return false;
  }
  Json value(int depth) {
    if (depth > 16) fail("nesting too deep");
    ws();
    if (p_ >= end_) fail("unexpected end");
    Json v;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.kind = Json::Object;
      if (eat('}')) return v;
      do {
        ws();
        std::string k = string();
        if (!eat(':')) fail("expected ':'");
        for (const auto& kv : v.obj)
          if (kv.first == k) fail("duplicate key");
        v.obj.emplace_back(std::move(k), value(depth + 1));
      } while (eat(','));
      if (!eat('}')) fail("expected '}'");
    } else if (c == '[') {
      ++p_;
      v.kind = Json::Array;
      if (eat(']')) return v;
      do v.arr.push_back(value(depth + 1));
      while (eat(','));
      if (!eat(']')) fail("expected ']'");
    } else if (c == '"') {
      v.kind = Json::String;
      v.str = string();
    } else if (c == 't' || c == 'f' || c == 'n') {
      const char* words[] = {"true", "false", "null"};
      for (const char* w : words) {
        const size_t n = std::strlen(w);
        if (size_t(end_ - p_) >= n && std::strncmp(p_, w, n) == 0) {
          p_ += n;
          v.kind = w[0] == 'n' ? Json::Null : Json::Bool;
          v.b = w[0] == 't';
          return v;
        }
      }
      fail("bad literal");
    } else {
      v.kind = Json::Number;
      const char* s = p_;
      if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
      bool digits = false;
      while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' ||
                           *p_ == '+')) {
        digits |= (*p_ >= '0' && *p_ <= '9');
        ++p_;
      }
      if (!digits) fail("bad number");
      v.num = std::strtod(std::string(s, p_).c_str(), nullptr);
    }
    return v;
  }
  std::string string() {
    if (p_ >= end_ || *p_ != '"') fail("expected a string");
    ++p_;
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= end_) fail("bad escape");
        const char e = *p_++;
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {  // tensor names are ASCII; keep BMP code points as UTF-8
            if (end_ - p_ < 4) fail("bad unicode escape");
            const unsigned cp = unsigned(std::stoul(std::string(p_, p_ + 4), nullptr, 16));
            p_ += 4;
            if (cp < 0x80) out += char(cp);
            else if (cp < 0x800) { out += char(0xC0 | (cp >> 6)); out += char(0x80 | (cp & 0x3F)); }
            else { out += char(0xE0 | (cp >> 12)); out += char(0x80 | ((cp >> 6) & 0x3F)); out += char(0x80 | (cp & 0x3F)); }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p_ >= end_) fail("unterminated string");
    ++p_;
    return out;
  }
  const char* p_;
  const char* end_;
};

struct FileCloser {
  void operator()(FILE* f) const {
    if (f) std::fclose(f);
  }
};

}  // namespace

double HostTensor::at(size_t i) const {
  switch (dtype) {
    case kF32: {
      float f;
      std::memcpy(&f, bytes.data() + 4 * i, 4);
      return f;
    }
    case kF16: {
      uint16_t h;
      std::memcpy(&h, bytes.data() + 2 * i, 2);
      return double(__half2float(__ushort_as_half(h)));
    }
    case kBF16: {
      uint16_t h;
      std::memcpy(&h, bytes.data() + 2 * i, 2);
      const uint32_t u = uint32_t(h) << 16;
      float f;
      std::memcpy(&f, &u, 4);
      return f;
    }
    default:
      throw std::invalid_argument("checkpoint tensor is not floating point");
  }
}

bool load_safetensors(const std::string& path, std::map<std::string, HostTensor>& out) {
  std::unique_ptr<FILE, FileCloser> f(std::fopen(path.c_str(), "rb"));
  if (!f) throw std::invalid_argument("cannot open safetensors shard: " + path);
  if (std::fseek(f.get(), 0, SEEK_END) != 0) throw std::runtime_error("safetensors shard is not seekable");
  const long long size = std::ftell(f.get());
  std::rewind(f.get());
  uint8_t len_bytes[8];
  if (size < 8 || std::fread(len_bytes, 1, 8, f.get()) != 8) throw std::invalid_argument("safetensors header size");
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | len_bytes[i];
  if (hlen < 2 || hlen > (uint64_t(8) << 20) || hlen + 8 > uint64_t(size))
    throw std::invalid_argument("safetensors header size");
  std::string header(hlen, '\0');
  if (std::fread(header.data(), 1, hlen, f.get()) != hlen) throw std::invalid_argument("safetensors header truncated");
  const Json doc = Parser(header.data(), header.size()).parse_document();
  if (doc.kind != Json::Object) throw std::invalid_argument("safetensors header: not an object");
  const uint64_t data_bytes = uint64_t(size) - 8 - hlen;
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  bool shifted_norms = false;
  std::map<std::string, HostTensor> fresh;
  for (const auto& kv : doc.obj) {
    const std::string& name = kv.first;
    if (name == "__metadata__") continue;
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* sh = t.get("shape");
    const Json* of = t.get("data_offsets");
    if (t.kind != Json::Object || !dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !of ||
        of->kind != Json::Array || of->arr.size() != 2)
      throw std::invalid_argument("safetensors tensor entry: " + name);
    HostTensor h;
    size_t item = 0;
    if (dt->str == "F32") h.dtype = kF32, item = 4;
    else if (dt->str == "I32") h.dtype = kI32, item = 4;
    else if (dt->str == "U32") h.dtype = kU32, item = 4;
    else if (dt->str == "F16") h.dtype = kF16, item = 2;
    else if (dt->str == "BF16") h.dtype = kBF16, item = 2;
    else throw std::invalid_argument("unsupported parameter dtype: " + name);
    if (sh->arr.empty() || sh->arr.size() > 4) throw std::invalid_argument("parameter shape bounds: " + name);
    uint64_t bytes = item;
    for (const Json& d : sh->arr) {
      if (d.kind != Json::Number || d.num < 1 || d.num > 1e12 || d.num != double(int64_t(d.num)))
        throw std::invalid_argument("parameter shape bounds: " + name);
      h.shape.push_back(int64_t(d.num));
      bytes *= uint64_t(d.num);
      if (bytes > (uint64_t(64) << 30)) throw std::invalid_argument("parameter size overflow: " + name);
    }
    const double b0 = of->arr[0].num, b1 = of->arr[1].num;
    if (of->arr[0].kind != Json::Number || of->arr[1].kind != Json::Number || b0 < 0 || b1 < b0 ||
        uint64_t(b1) - uint64_t(b0) != bytes || uint64_t(b1) > data_bytes)
      throw std::invalid_argument("parameter offsets outside shard: " + name);
    ranges.emplace_back(uint64_t(b0), uint64_t(b1));
    if (out.count(name) || fresh.count(name)) throw std::invalid_argument("duplicate native parameter: " + name);
    h.bytes.resize(bytes);
    if (std::fseek(f.get(), long(8 + hlen + uint64_t(b0)), SEEK_SET) != 0 ||
        (bytes && std::fread(h.bytes.data(), 1, bytes, f.get()) != bytes))
      throw std::runtime_error("safetensors data truncated: " + name);
    const bool conv_hf = name.size() >= 13 && name.compare(name.size() - 13, 13, "conv1d.weight") == 0 &&
                         h.shape.back() != 1;
    if (name.find("mtp.") != std::string::npos || conv_hf) shifted_norms = true;
    fresh.emplace(name, std::move(h));
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); ++i)
    if (ranges[i - 1].second > ranges[i].first) throw std::invalid_argument("overlapping parameter offsets");
  for (auto& kv : fresh) out.emplace(kv.first, std::move(kv.second));
  return shifted_norms;
}

}  // namespace qwen
