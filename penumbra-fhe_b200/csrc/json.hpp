// json.hpp -- a small JSON reader for the IR wire format (model.fhe files).
//
// The reference reads the same files with serde_json (runtime/src/ir.rs:169-180).  Integers stay
// exact 64-bit values (weights, biases and LUT entries are integers in the IR); errors carry the
// byte offset.
#pragma once
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace pnb {
namespace json {

struct Value {
  enum Kind { Null, Bool, Int, Float, String, Array, Object } kind = Null;
  bool b = false;
  int64_t i = 0;
  bool i_unsigned_overflow = false;  // integer literal above INT64_MAX (kept in u)
  uint64_t u = 0;
  double f = 0;
  std::string s;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  const Value* get(const std::string& key) const {
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  bool is_int() const { return kind == Int; }
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), n_(n) {}

  Value parse() {
    Value v = value();
    ws();
    if (pos_ != n_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  size_t n_;
  size_t pos_ = 0;

  [[noreturn]] void fail(const char* what) const {
    throw std::runtime_error(std::string("JSON parse error at byte ") + std::to_string(pos_) +
                             ": " + what);
  }
  void ws() {
    while (pos_ < n_ && (p_[pos_] == ' ' || p_[pos_] == '\n' || p_[pos_] == '\t' ||
                         p_[pos_] == '\r'))
      ++pos_;
  }
  char peek() {
    ws();
    if (pos_ >= n_) fail("unexpected end of input");
    return p_[pos_];
  }
  void expect(char c) {
    if (peek() != c) fail((std::string("expected '") + c + "'").c_str());
    ++pos_;
  }
  bool lit(const char* w) {
    size_t k = 0;
    while (w[k]) {
      if (pos_ + k >= n_ || p_[pos_ + k] != w[k]) return false;
      ++k;
    }
    pos_ += k;
    return true;
  }

  Value value() {
    char c = peek();
    Value v;
    if (c == '{') {
      ++pos_;
      v.kind = Value::Object;
      if (peek() == '}') { ++pos_; return v; }
      for (;;) {
        if (peek() != '"') fail("expected object key");
        std::string k = str();
        expect(':');
        v.obj.emplace_back(std::move(k), value());
        char d = peek();
        ++pos_;
        if (d == '}') break;
        if (d != ',') fail("expected ',' or '}'");
      }
    } else if (c == '[') {
      ++pos_;
      v.kind = Value::Array;
      if (peek() == ']') { ++pos_; return v; }
      for (;;) {
        v.arr.push_back(value());
        char d = peek();
        ++pos_;
        if (d == ']') break;
        if (d != ',') fail("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = Value::String;
      v.s = str();
    } else if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = Value::Bool;
    } else if (lit("null")) {
      v.kind = Value::Null;
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      number(v);
    } else {
      fail("unexpected character");
    }
    return v;
  }

  std::string str() {
    expect('"');
    std::string out;
    while (pos_ < n_ && p_[pos_] != '"') {
      char c = p_[pos_++];
      if (c == '\\') {
        if (pos_ >= n_) fail("bad escape");
        char e = p_[pos_++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (pos_ + 4 > n_) fail("bad \\u escape");
            unsigned cp = std::strtoul(std::string(p_ + pos_, 4).c_str(), nullptr, 16);
            pos_ += 4;
            if (cp < 0x80) {
              out += (char)cp;
            } else if (cp < 0x800) {
              out += (char)(0xC0 | (cp >> 6));
              out += (char)(0x80 | (cp & 0x3F));
            } else {
              out += (char)(0xE0 | (cp >> 12));
              out += (char)(0x80 | ((cp >> 6) & 0x3F));
              out += (char)(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (pos_ >= n_) fail("unterminated string");
    ++pos_;
    return out;
  }

  void number(Value& v) {
    size_t start = pos_;
    bool neg = false;
    if (p_[pos_] == '-') { neg = true; ++pos_; }
    bool integral = true;
    while (pos_ < n_ && ((p_[pos_] >= '0' && p_[pos_] <= '9') || p_[pos_] == '.' ||
                         p_[pos_] == 'e' || p_[pos_] == 'E' || p_[pos_] == '+' ||
                         p_[pos_] == '-')) {
      if (p_[pos_] == '.' || p_[pos_] == 'e' || p_[pos_] == 'E') integral = false;
      ++pos_;
    }
    std::string tok(p_ + start, pos_ - start);
    if (integral) {
      v.kind = Value::Int;
      errno = 0;
      if (neg) {
        v.i = std::strtoll(tok.c_str(), nullptr, 10);
        if (errno) fail("integer out of range");
      } else {
        unsigned long long u = std::strtoull(tok.c_str(), nullptr, 10);
        if (errno) fail("integer out of range");
        v.u = u;
        if (u > (unsigned long long)INT64_MAX) v.i_unsigned_overflow = true;
        else v.i = (int64_t)u;
      }
    } else {
      v.kind = Value::Float;
      v.f = std::strtod(tok.c_str(), nullptr);
    }
  }
};

inline Value parse(const char* p, size_t n) { return Parser(p, n).parse(); }

}  // namespace json
}  // namespace pnb
