// Minimal JSON reader for Program files (src/program.ts:150-165): objects,
// arrays, strings, numbers (as double), true/false/null. Throws
// std::runtime_error with the byte offset on malformed input.
#pragma once
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace wgx {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  const Value *get(const std::string &k) const {
    for (auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  bool has(const std::string &k) const { return get(k) != nullptr; }
};

class Parser {
 public:
  Parser(const char *s, size_t n) : s_(s), n_(n) {}
  Value parse() {
    Value v = value();
    ws();
    if (i_ != n_) err("trailing characters");
    return v;
  }

 private:
  const char *s_;
  size_t n_, i_ = 0;
  [[noreturn]] void err(const char *m) {
    throw std::runtime_error(std::string("program JSON: ") + m + " at byte " + std::to_string(i_));
  }
  void ws() {
    while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool lit(const char *w) {
    size_t k = 0;
    while (w[k]) {
      if (i_ + k >= n_ || s_[i_ + k] != w[k]) return false;
      ++k;
    }
    i_ += k;
    return true;
  }
  Value value() {
    ws();
    if (i_ >= n_) err("unexpected end");
    char c = s_[i_];
    Value v;
    if (c == '{') {
      v.kind = Value::Object;
      ++i_;
      ws();
      if (i_ < n_ && s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (true) {
        ws();
        if (i_ >= n_ || s_[i_] != '"') err("expected key");
        std::string k = string();
        ws();
        if (i_ >= n_ || s_[i_] != ':') err("expected ':'");
        ++i_;
        v.obj.emplace_back(std::move(k), value());
        ws();
        if (i_ < n_ && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < n_ && s_[i_] == '}') {
          ++i_;
          return v;
        }
        err("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Value::Array;
      ++i_;
      ws();
      if (i_ < n_ && s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (i_ < n_ && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < n_ && s_[i_] == ']') {
          ++i_;
          return v;
        }
        err("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Value::String;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Value::Bool;
      return v;
    }
    if (lit("null")) return v;
    // number
    const char *start = s_ + i_;
    char *end = nullptr;
    std::string tmp(start, std::min<size_t>(n_ - i_, 64));
    double d = std::strtod(tmp.c_str(), &end);
    if (end == tmp.c_str()) err("bad value");
    i_ += size_t(end - tmp.c_str());
    v.kind = Value::Number;
    v.num = d;
    return v;
  }
  std::string string() {
    ++i_;  // opening quote
    std::string out;
    while (i_ < n_ && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= n_) err("bad escape");
        char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i_ + 4 > n_) err("bad unicode escape");
            unsigned cp = std::stoul(std::string(s_ + i_, 4), nullptr, 16);
            i_ += 4;
            if (cp < 0x80) {
              out += char(cp);
            } else if (cp < 0x800) {
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
    if (i_ >= n_) err("unterminated string");
    ++i_;
    return out;
  }
};

inline Value parse(const char *s, size_t n) { return Parser(s, n).parse(); }

}  // namespace json
}  // namespace wgx
