// Minimal JSON reader for the checkpoint configs and the safetensors header.
// Supports objects, arrays, strings (with \uXXXX escapes), numbers, true/false/null.
#pragma once
#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace j1rt {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;  // String: the text; Number: the literal as written
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // insertion order kept

  const Json* get(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  bool is_num() const { return kind == Number; }
  bool is_str() const { return kind == String; }
  bool is_bool() const { return kind == Bool; }
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}
  bool parse(Json& out, std::string& err) {
    bool ok = value(out, 0);
    skip();
    if (ok && p_ != end_) ok = fail("trailing characters");
    if (!ok) err = err_;
    return ok;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  bool fail(const char* m) {
    err_ = m;
    return false;
  }
  void skip() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    size_t n = 0;
    while (s[n]) ++n;
    if (static_cast<size_t>(end_ - p_) < n) return false;
    for (size_t i = 0; i < n; ++i)
      if (p_[i] != s[i]) return false;
    p_ += n;
    return true;
  }
  static void utf8(std::string& o, uint32_t c) {
    if (c < 0x80) {
      o += static_cast<char>(c);
    } else if (c < 0x800) {
      o += static_cast<char>(0xC0 | (c >> 6));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      o += static_cast<char>(0xE0 | (c >> 12));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    } else {
      o += static_cast<char>(0xF0 | (c >> 18));
      o += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
      o += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      o += static_cast<char>(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t& v) {
    if (end_ - p_ < 4) return false;
    v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else return false;
    }
    return true;
  }
  bool string(std::string& o) {
    ++p_;  // opening quote
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') {
        o += c;
        continue;
      }
      if (p_ >= end_) return fail("bad escape");
      char e = *p_++;
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
          uint32_t v;
          if (!hex4(v)) return fail("bad \\u escape");
          if (v >= 0xD800 && v < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            uint32_t lo;
            if (!hex4(lo)) return fail("bad surrogate");
            v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(o, v);
          break;
        }
        default:
          return fail("bad escape");
      }
    }
    if (p_ >= end_) return fail("unterminated string");
    ++p_;
    return true;
  }
  bool value(Json& out, int depth) {
    if (depth > 64) return fail("nesting too deep");
    skip();
    if (p_ >= end_) return fail("unexpected end");
    char c = *p_;
    if (c == '{') {
      out.kind = Json::Object;
      ++p_;
      skip();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      while (true) {
        skip();
        if (p_ >= end_ || *p_ != '"') return fail("expected key");
        std::string key;
        if (!string(key)) return false;
        skip();
        if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        out.obj.emplace_back(std::move(key), Json());
        if (!value(out.obj.back().second, depth + 1)) return false;
        skip();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      out.kind = Json::Array;
      ++p_;
      skip();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      while (true) {
        out.arr.emplace_back();
        if (!value(out.arr.back(), depth + 1)) return false;
        skip();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      out.kind = Json::String;
      return string(out.str);
    }
    if (lit("true")) {
      out.kind = Json::Bool;
      out.b = true;
      return true;
    }
    if (lit("false")) {
      out.kind = Json::Bool;
      out.b = false;
      return true;
    }
    if (lit("null")) {
      out.kind = Json::Null;
      return true;
    }
    if (c == '-' || (c >= '0' && c <= '9')) {
      std::string tok;
      while (p_ < end_ && (std::isdigit(static_cast<unsigned char>(*p_)) || *p_ == '-' || *p_ == '+' ||
                           *p_ == '.' || *p_ == 'e' || *p_ == 'E'))
        tok += *p_++;
      char* e = nullptr;
      out.kind = Json::Number;
      out.num = std::strtod(tok.c_str(), &e);
      if (!e || *e) return fail("bad number");
      out.str = tok;  // the literal as written (integers beyond double precision, int vs float)
      return true;
    }
    return fail("unexpected character");
  }
};

inline bool parse_json(const std::string& text, Json& out, std::string& err) {
  JsonParser p(text.data(), text.size());
  return p.parse(out, err);
}

}  // namespace j1rt
