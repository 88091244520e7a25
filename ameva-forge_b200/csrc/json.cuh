// Minimal JSON reader for the graph front-end: a DOM of null / bool / number /
// string / array / object values, parsed from a NUL-terminated UTF-8 text.
// Strict RFC 8259 grammar (no comments, no trailing commas), nesting capped at
// 64 levels, object keys kept in document order.  Host code only.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace fg {
namespace json {

struct Value {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  const Value *find(const char *key) const {
    for (const auto &kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

struct ParseError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Parser {
 public:
  explicit Parser(const char *s) : p_(s) {}
  // key_check(key) is called for every object key; it may throw to reject one.
  template <class KeyCheck>
  Value parse(KeyCheck key_check) {
    Value v = value(key_check, 0);
    ws();
    if (*p_) fail("trailing characters");
    return v;
  }

 private:
  const char *p_;

  [[noreturn]] void fail(const char *what) { throw ParseError(what); }
  void ws() {
    while (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r') ++p_;
  }
  bool lit(const char *w) {
    const size_t n = std::strlen(w);
    if (std::strncmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void put_utf8(std::string &o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i, ++p_) {
      const char c = *p_;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    if (*p_ != '"') fail("expected string");
    ++p_;
    std::string o;
    for (;;) {
      const unsigned char c = (unsigned char)*p_;
      if (c == 0) fail("unterminated string");
      if (c < 0x20) fail("control character in string");
      ++p_;
      if (c == '"') return o;
      if (c != '\\') {
        o += (char)c;
        continue;
      }
      const char e = *p_++;
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (p_[0] != '\\' || p_[1] != 'u') fail("lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            fail("lone surrogate");
          }
          put_utf8(o, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
  }
  double number() {
    const char *s = p_;
    if (*p_ == '-') ++p_;
    if (*p_ == '0') {
      ++p_;
    } else if (*p_ >= '1' && *p_ <= '9') {
      while (*p_ >= '0' && *p_ <= '9') ++p_;
    } else {
      fail("bad number");
    }
    if (*p_ == '.') {
      ++p_;
      if (!(*p_ >= '0' && *p_ <= '9')) fail("bad fraction");
      while (*p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (*p_ == 'e' || *p_ == 'E') {
      ++p_;
      if (*p_ == '+' || *p_ == '-') ++p_;
      if (!(*p_ >= '0' && *p_ <= '9')) fail("bad exponent");
      while (*p_ >= '0' && *p_ <= '9') ++p_;
    }
    return std::strtod(std::string(s, p_).c_str(), nullptr);
  }
  template <class KeyCheck>
  Value value(KeyCheck &key_check, int depth) {
    if (depth > 64) fail("nesting too deep");
    ws();
    Value v;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v.kind = Value::OBJ;
      ws();
      if (*p_ == '}') {
        ++p_;
        return v;
      }
      for (;;) {
        ws();
        std::string k = string();
        key_check(k);
        ws();
        if (*p_ != ':') fail("expected ':'");
        ++p_;
        v.obj.emplace_back(std::move(k), value(key_check, depth + 1));
        ws();
        if (*p_ == ',') {
          ++p_;
          continue;
        }
        if (*p_ == '}') {
          ++p_;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      v.kind = Value::ARR;
      ws();
      if (*p_ == ']') {
        ++p_;
        return v;
      }
      for (;;) {
        v.arr.push_back(value(key_check, depth + 1));
        ws();
        if (*p_ == ',') {
          ++p_;
          continue;
        }
        if (*p_ == ']') {
          ++p_;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Value::STR;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Value::BOOL;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Value::BOOL;
      return v;
    }
    if (lit("null")) return v;
    v.kind = Value::NUM;
    v.num = number();
    return v;
  }
};

}  // namespace json
}  // namespace fg
