// json.h -- a small JSON reader for the model loaders (config.json, the
// SafeTensors header and shard index).  RFC 8259 values; numbers keep both
// their double value (strtod, as serde_json then casts to f32) and, for
// integers, their exact unsigned 64-bit value.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

namespace lrs {

struct JValue {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0.0;
  bool is_uint = false;  // a non-negative integer literal that fits 64 bits
  uint64_t u = 0;
  std::string s;
  std::vector<JValue> arr;
  std::vector<std::pair<std::string, JValue>> obj;

  const JValue* get(const std::string& key) const {
    if (kind != Obj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}

  // Parses one value that must span the whole input (whitespace aside).
  bool parse(JValue* out, std::string* err) {
    skip();
    if (!value(out, 0)) {
      *err = err_.empty() ? "invalid JSON" : err_;
      return false;
    }
    skip();
    if (p_ != end_) {
      *err = "trailing characters after the JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  void skip() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
  }
  bool fail(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  bool lit(const char* w) {
    const char* q = p_;
    for (; *w; w++, q++)
      if (q >= end_ || *q != *w) return fail("invalid literal");
    p_ = q;
    return true;
  }
  static int hexv(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
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
    if (end_ - p_ < 4) return fail("truncated \\u escape");
    *v = 0;
    for (int i = 0; i < 4; i++) {
      const int h = hexv(p_[i]);
      if (h < 0) return fail("invalid \\u escape");
      *v = (*v << 4) | (uint32_t)h;
    }
    p_ += 4;
    return true;
  }
  bool string(std::string* s) {
    p_++;  // opening quote
    while (true) {
      if (p_ >= end_) return fail("unterminated string");
      const char c = *p_++;
      if (c == '"') return true;
      if ((unsigned char)c < 0x20) return fail("control character in string");
      if (c != '\\') {
        s->push_back(c);
        continue;
      }
      if (p_ >= end_) return fail("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            uint32_t lo;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate");
            p_ += 2;
            if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return fail("invalid surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            return fail("lone surrogate");
          }
          put_utf8(s, cp);
          break;
        }
        default:
          return fail("invalid escape");
      }
    }
  }
  bool number(JValue* v) {
    const char* q = p_;
    if (q < end_ && *q == '-') q++;
    if (q >= end_ || *q < '0' || *q > '9') return fail("invalid number");
    if (*q == '0') {
      q++;
    } else {
      while (q < end_ && *q >= '0' && *q <= '9') q++;
    }
    bool integral = true;
    if (q < end_ && *q == '.') {
      integral = false;
      q++;
      if (q >= end_ || *q < '0' || *q > '9') return fail("invalid number");
      while (q < end_ && *q >= '0' && *q <= '9') q++;
    }
    if (q < end_ && (*q == 'e' || *q == 'E')) {
      integral = false;
      q++;
      if (q < end_ && (*q == '+' || *q == '-')) q++;
      if (q >= end_ || *q < '0' || *q > '9') return fail("invalid number");
      while (q < end_ && *q >= '0' && *q <= '9') q++;
    }
    const std::string text(p_, q);
    v->kind = JValue::Num;
    v->num = strtod(text.c_str(), nullptr);
    if (integral && text[0] != '-') {
      uint64_t u = 0;
      bool fits = true;
      for (char c : text) {
        const uint64_t d = (uint64_t)(c - '0');
        if (u > (UINT64_MAX - d) / 10) {
          fits = false;
          break;
        }
        u = u * 10 + d;
      }
      v->is_uint = fits;
      v->u = u;
    }
    p_ = q;
    return true;
  }
  bool value(JValue* v, int depth) {
    if (depth > 128) return fail("JSON nested too deeply");
    if (p_ >= end_) return fail("unexpected end of JSON");
    switch (*p_) {
      case 'n': v->kind = JValue::Null; return lit("null");
      case 't': v->kind = JValue::Bool; v->b = true; return lit("true");
      case 'f': v->kind = JValue::Bool; v->b = false; return lit("false");
      case '"': v->kind = JValue::Str; return string(&v->s);
      case '[': {
        v->kind = JValue::Arr;
        p_++;
        skip();
        if (p_ < end_ && *p_ == ']') {
          p_++;
          return true;
        }
        while (true) {
          v->arr.emplace_back();
          skip();
          if (!value(&v->arr.back(), depth + 1)) return false;
          skip();
          if (p_ >= end_) return fail("unterminated array");
          if (*p_ == ',') {
            p_++;
            continue;
          }
          if (*p_ == ']') {
            p_++;
            return true;
          }
          return fail("expected ',' or ']'");
        }
      }
      case '{': {
        v->kind = JValue::Obj;
        p_++;
        skip();
        if (p_ < end_ && *p_ == '}') {
          p_++;
          return true;
        }
        while (true) {
          skip();
          if (p_ >= end_ || *p_ != '"') return fail("expected a key string");
          std::string key;
          if (!string(&key)) return false;
          skip();
          if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
          p_++;
          skip();
          v->obj.emplace_back(std::move(key), JValue{});
          if (!value(&v->obj.back().second, depth + 1)) return false;
          skip();
          if (p_ >= end_) return fail("unterminated object");
          if (*p_ == ',') {
            p_++;
            continue;
          }
          if (*p_ == '}') {
            p_++;
            return true;
          }
          return fail("expected ',' or '}'");
        }
      }
      default:
        return number(v);
    }
  }
};

}  // namespace lrs
