// RFC 8259 JSON for the host-side readers of libdsb.so (checkpoint headers,
// config.json, the safetensors index, tokenizer.json): recursive descent
// over untrusted input with bounded nesting; objects keep their keys in file
// order and a repeated key is an error; integers that fit int64 stay exact.
// Also the thread-local message of the host-only C ABI calls.

#pragma once

#include <algorithm>
#include <charconv>
#include <cstdint>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace dsb {

// This thread's last error message of a host-only subsystem of the C ABI
// (each has its own: dsb_checkpoint_error, dsb_tokenizer_error).
enum HostChannel { kHostCheckpoint = 0, kHostTokenizer = 1 };
// Record `msg` on `channel` and return `code`.
int host_fail(int code, std::string msg, HostChannel channel = kHostCheckpoint);
const char* host_error(HostChannel channel = kHostCheckpoint);

struct Json {
  enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  int64_t i = 0;
  double d = 0.0;
  std::string s;
  std::vector<Json> a;
  std::vector<std::pair<std::string, Json>> o;

  const Json* get(const char* key) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : o)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  bool is_number() const { return kind == Int || kind == Num; }
};

// RFC 8259 JSON, recursive descent; objects keep their keys in file order and
// a repeated key is an error.
class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}

  bool parse(Json* out, std::string* err) {
    ws();
    if (!value(out, 0)) {
      *err = err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      *err = "trailing characters after the JSON value";
      return false;
    }
    return true;
  }

 private:
  static constexpr int kMaxDepth = 64;
  const char* p_;
  const char* end_;
  std::string err_;

  bool error(const char* what) {
    err_ = what;
    return false;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = std::strlen(w);
    if ((size_t)(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void put_utf8(std::string* s, uint32_t cp) {
    if (cp < 0x80) {
      s->push_back((char)cp);
    } else if (cp < 0x800) {
      s->push_back((char)(0xC0 | (cp >> 6)));
      s->push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      s->push_back((char)(0xE0 | (cp >> 12)));
      s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      s->push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      s->push_back((char)(0xF0 | (cp >> 18)));
      s->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      s->push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(uint32_t* v) {
    if (end_ - p_ < 4) return false;
    uint32_t x = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p_++;
      x <<= 4;
      if (c >= '0' && c <= '9') x |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') x |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') x |= (uint32_t)(c - 'A' + 10);
      else return false;
    }
    *v = x;
    return true;
  }
  bool string(std::string* out) {
    ++p_;  // opening quote
    while (true) {
      if (p_ >= end_) return error("unterminated string");
      const char c = *p_++;
      if (c == '"') return true;
      if ((unsigned char)c < 0x20) return error("control character in string");
      if (c != '\\') {
        out->push_back(c);
        continue;
      }
      if (p_ >= end_) return error("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': out->push_back('"'); break;
        case '\\': out->push_back('\\'); break;
        case '/': out->push_back('/'); break;
        case 'b': out->push_back('\b'); break;
        case 'f': out->push_back('\f'); break;
        case 'n': out->push_back('\n'); break;
        case 'r': out->push_back('\r'); break;
        case 't': out->push_back('\t'); break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(&cp)) return error("bad \\u escape");
          if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: needs its low half
            uint32_t lo = 0;
            if (!lit("\\u") || !hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return error("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return error("unpaired surrogate");
          }
          put_utf8(out, cp);
          break;
        }
        default: return error("bad escape");
      }
    }
  }
  bool number(Json* out) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return error("bad number");
    if (*p_ == '0') ++p_;
    else
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    bool integral = true;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return error("bad number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return error("bad number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (integral) {
      int64_t v = 0;
      const auto r = std::from_chars(s, p_, v);
      if (r.ec == std::errc() && r.ptr == p_) {
        out->kind = Json::Int;
        out->i = v;
        out->d = (double)v;
        return true;
      }
    }
    double v = 0.0;
    const auto r = std::from_chars(s, p_, v);
    if (r.ec != std::errc() || r.ptr != p_) return error("number out of range");
    out->kind = Json::Num;
    out->d = v;
    return true;
  }
  // No key twice: pairwise for small objects, sorted for large ones (a
  // tokenizer vocabulary or a weight map has 1e5 keys).
  static bool unique_keys(const Json& obj) {
    const size_t n = obj.o.size();
    if (n <= 16) {
      for (size_t i = 0; i < n; ++i)
        for (size_t j = i + 1; j < n; ++j)
          if (obj.o[i].first == obj.o[j].first) return false;
      return true;
    }
    std::vector<const std::string*> keys(n);
    for (size_t i = 0; i < n; ++i) keys[i] = &obj.o[i].first;
    std::sort(keys.begin(), keys.end(), [](const std::string* a, const std::string* b) { return *a < *b; });
    for (size_t i = 1; i < n; ++i)
      if (*keys[i] == *keys[i - 1]) return false;
    return true;
  }
  bool value(Json* out, int depth) {
    if (depth > kMaxDepth) return error("JSON nested too deeply");
    if (p_ >= end_) return error("unexpected end of JSON");
    const char c = *p_;
    if (c == '{') {
      ++p_;
      out->kind = Json::Obj;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        if (p_ >= end_ || *p_ != '"') return error("expected a key");
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return error("expected ':'");
        ++p_;
        ws();
        out->o.emplace_back(std::move(key), Json());
        if (!value(&out->o.back().second, depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return unique_keys(*out) ? true : error("repeated key in object");
        }
        return error("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      out->kind = Json::Arr;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (true) {
        ws();
        out->a.emplace_back();
        if (!value(&out->a.back(), depth + 1)) return false;
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return error("expected ',' or ']'");
      }
    }
    if (c == '"') {
      out->kind = Json::Str;
      return string(&out->s);
    }
    if (lit("true")) {
      out->kind = Json::Bool;
      out->b = true;
      return true;
    }
    if (lit("false")) {
      out->kind = Json::Bool;
      return true;
    }
    if (lit("null")) return true;
    return number(out);
  }
};

inline bool parse_json(const char* p, size_t n, Json* out, std::string* err) {
  return JsonParser(p, n).parse(out, err);
}

}  // namespace dsb
