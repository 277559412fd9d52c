// A small JSON reader for manifest.json and hobson_config.json (objects keep their key order).
#pragma once
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace sd {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  const Value* get(const std::string& k) const {
    if (kind != Object) return nullptr;
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  const Value& at(const std::string& k) const {
    const Value* v = get(k);
    if (!v) throw std::runtime_error("missing key " + k);
    return *v;
  }
  bool is_null() const { return kind == Null; }
  double number(double dflt = 0.0) const { return kind == Number ? num : (kind == Bool ? (b ? 1.0 : 0.0) : dflt); }
  long long integer(long long dflt = 0) const { return kind == Number ? (long long)num : dflt; }
  bool boolean(bool dflt = false) const { return kind == Bool ? b : dflt; }
};

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Value parse() {
    Value v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;

  [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("json: ") + what + " at " + std::to_string(i_)); }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
  }
  bool lit(const char* w) {
    size_t n = strlen(w);
    if (s_.compare(i_, n, w) == 0) {
      i_ += n;
      return true;
    }
    return false;
  }
  static void utf8(std::string& out, unsigned cp) {
    if (cp < 0x80) out += (char)cp;
    else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
    else if (cp < 0x10000) { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
    else { out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 0x3F)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
  }
  unsigned hex4() {
    if (i_ + 4 > s_.size()) fail("bad escape");
    unsigned v = (unsigned)strtoul(s_.substr(i_, 4).c_str(), nullptr, 16);
    i_ += 4;
    return v;
  }
  std::string string() {
    if (s_[i_] != '"') fail("expected string");
    i_++;
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c != '\\') { out += c; continue; }
      if (i_ >= s_.size()) fail("bad escape");
      char e = s_[i_++];
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
          unsigned cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && i_ + 6 <= s_.size() && s_[i_] == '\\' && s_[i_ + 1] == 'u') {
            i_ += 2;
            unsigned lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    i_++;
    return out;
  }
  Value value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    Value v;
    char c = s_[i_];
    if (c == '{') {
      v.kind = Value::Object;
      i_++;
      ws();
      if (s_[i_] == '}') { i_++; return v; }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (s_[i_] != ':') fail("expected ':'");
        i_++;
        Value x = value();
        bool replaced = false;
        for (auto& kv : v.obj)
          if (kv.first == k) { kv.second = std::move(x); replaced = true; break; }
        if (!replaced) v.obj.emplace_back(std::move(k), std::move(x));
        ws();
        if (s_[i_] == ',') { i_++; continue; }
        if (s_[i_] == '}') { i_++; break; }
        fail("expected ',' or '}'");
      }
    } else if (c == '[') {
      v.kind = Value::Array;
      i_++;
      ws();
      if (s_[i_] == ']') { i_++; return v; }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (s_[i_] == ',') { i_++; continue; }
        if (s_[i_] == ']') { i_++; break; }
        fail("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = Value::String;
      v.str = string();
    } else if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = Value::Bool;
    } else if (lit("null")) {
      v.kind = Value::Null;
    } else {
      char* end = nullptr;
      v.num = strtod(s_.c_str() + i_, &end);
      if (end == s_.c_str() + i_) fail("bad value");
      v.kind = Value::Number;
      i_ = end - s_.c_str();
    }
    return v;
  }
};

inline Value parse(const std::string& s) { return Parser(s).parse(); }

}  // namespace json
}  // namespace sd
