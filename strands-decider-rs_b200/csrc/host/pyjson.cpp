#include "pyjson.h"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

#include "unicode.h"

namespace sd {
namespace pj {
namespace {

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Value parse() {
    ws();
    Value v = value(0);
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;

  [[noreturn]] void fail(const std::string& what) {
    throw std::runtime_error("JSON: " + what + " at byte " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) i_++;
  }
  bool lit(const char* w) {
    const size_t n = strlen(w);
    if (s_.compare(i_, n, w) == 0) {
      i_ += n;
      return true;
    }
    return false;
  }
  Value value(int depth) {
    if (depth > 128) fail("nesting too deep");
    if (i_ >= s_.size()) fail("unexpected end");
    const char c = s_[i_];
    if (c == '{') {
      i_++;
      Value v = Value::object();
      ws();
      if (i_ < s_.size() && s_[i_] == '}') {
        i_++;
        return v;
      }
      while (true) {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected a key");
        std::string k = string();
        ws();
        if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
        i_++;
        ws();
        v.set(k, value(depth + 1));  // a repeated key keeps its first position, the last value
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          i_++;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == '}') {
          i_++;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      i_++;
      Value v = Value::array();
      ws();
      if (i_ < s_.size() && s_[i_] == ']') {
        i_++;
        return v;
      }
      while (true) {
        ws();
        v.arr.push_back(value(depth + 1));
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          i_++;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == ']') {
          i_++;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') return Value::str(string());
    if (lit("true")) return Value::boolean(true);
    if (lit("false")) return Value::boolean(false);
    if (lit("null")) return Value();
    return number();
  }
  uint32_t hex4() {
    if (i_ + 4 > s_.size()) fail("bad \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; k++) {
      const char c = s_[i_++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    i_++;  // '"'
    std::string out;
    while (true) {
      if (i_ >= s_.size()) fail("unterminated string");
      const unsigned char c = (unsigned char)s_[i_++];
      if (c == '"') break;
      if (c < 0x20) fail("control character in string");
      if (c != '\\') {
        out += (char)c;
        continue;
      }
      if (i_ >= s_.size()) fail("bad escape");
      const char e = s_[i_++];
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
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            if (i_ + 2 > s_.size() || s_[i_] != '\\' || s_[i_ + 1] != 'u') fail("lone leading surrogate");
            i_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo > 0xDFFF) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
            fail("lone trailing surrogate");
          }
          uni::append(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    std::vector<uint32_t> tmp;
    if (!uni::decode(out, tmp)) fail("string is not UTF-8");
    return out;
  }
  Value number() {
    const size_t st = i_;
    bool is_float = false;
    if (i_ < s_.size() && s_[i_] == '-') i_++;
    if (i_ >= s_.size() || !isdigit((unsigned char)s_[i_])) fail("expected a value");
    if (s_[i_] == '0') {
      i_++;
    } else {
      while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
    }
    if (i_ < s_.size() && s_[i_] == '.') {
      is_float = true;
      i_++;
      if (i_ >= s_.size() || !isdigit((unsigned char)s_[i_])) fail("bad number");
      while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
    }
    if (i_ < s_.size() && (s_[i_] == 'e' || s_[i_] == 'E')) {
      is_float = true;
      i_++;
      if (i_ < s_.size() && (s_[i_] == '+' || s_[i_] == '-')) i_++;
      if (i_ >= s_.size() || !isdigit((unsigned char)s_[i_])) fail("bad number");
      while (i_ < s_.size() && isdigit((unsigned char)s_[i_])) i_++;
    }
    const std::string lit = s_.substr(st, i_ - st);
    if (!is_float) {
      errno = 0;
      char* end = nullptr;
      const long long v = strtoll(lit.c_str(), &end, 10);
      if (errno == 0 && end && *end == 0) return Value::integer(v);
    }
    const double d = strtod(lit.c_str(), nullptr);
    if (!std::isfinite(d)) fail("number out of range");
    return Value::num(d);
  }
};

void dump_py(const Value& v, int level, std::string& out) {
  auto pad = [&](int n) { out.append(2 * n, ' '); };
  switch (v.kind) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Int: out += std::to_string(v.i); break;
    case Value::Float: out += py_float(v.f); break;
    case Value::String: quote(out, v.s); break;
    case Value::Array:
      if (v.arr.empty()) {
        out += "[]";
        break;
      }
      out += "[";
      for (size_t k = 0; k < v.arr.size(); k++) {
        out += k == 0 ? "\n" : ",\n";
        pad(level + 1);
        dump_py(v.arr[k], level + 1, out);
      }
      out += "\n";
      pad(level);
      out += "]";
      break;
    case Value::Object:
      if (v.obj.empty()) {
        out += "{}";
        break;
      }
      out += "{";
      for (size_t k = 0; k < v.obj.size(); k++) {
        out += k == 0 ? "\n" : ",\n";
        pad(level + 1);
        quote(out, v.obj[k].first);
        out += ": ";
        dump_py(v.obj[k].second, level + 1, out);
      }
      out += "\n";
      pad(level);
      out += "}";
      break;
  }
}

void dump(const Value& v, std::string& out) {
  switch (v.kind) {
    case Value::Null: out += "null"; break;
    case Value::Bool: out += v.b ? "true" : "false"; break;
    case Value::Int: out += std::to_string(v.i); break;
    case Value::Float: out += std::isfinite(v.f) ? py_float(v.f) : "null"; break;
    case Value::String: quote(out, v.s); break;
    case Value::Array:
      out += "[";
      for (size_t k = 0; k < v.arr.size(); k++) {
        if (k) out += ",";
        dump(v.arr[k], out);
      }
      out += "]";
      break;
    case Value::Object:
      out += "{";
      for (size_t k = 0; k < v.obj.size(); k++) {
        if (k) out += ",";
        quote(out, v.obj[k].first);
        out += ":";
        dump(v.obj[k].second, out);
      }
      out += "}";
      break;
  }
}

}  // namespace

Value parse(const std::string& text) { return Parser(text).parse(); }

void quote(std::string& out, const std::string& s) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += (char)c;
        }
    }
  }
  out += '"';
}

// Python's repr(float): the shortest digit string that reads back as the same double (tried with
// 1..17 significant digits), written as Python does: positional for decimal exponents -4 .. 15,
// otherwise d.ddde+XX.
std::string py_float(double x) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x > 0 ? "Infinity" : "-Infinity";
  if (x == 0.0) return std::signbit(x) ? "-0.0" : "0.0";
  char buf[40];
  int prec = 1;
  for (; prec <= 17; prec++) {
    snprintf(buf, sizeof buf, "%.*e", prec - 1, x);
    if (strtod(buf, nullptr) == x) break;
  }
  // buf: [-]d.ddde[+-]XX
  std::string s(buf);
  std::string sign;
  if (s[0] == '-') sign = "-", s = s.substr(1);
  const size_t e = s.find('e');
  std::string mant = s.substr(0, e);
  const int exp10 = atoi(s.c_str() + e + 1);
  std::string digits;
  for (char c : mant)
    if (c != '.') digits += c;
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int n = (int)digits.size();
  const int point = exp10 + 1;  // digits before the decimal point
  std::string body;
  if (point <= -4 || point > 16) {
    body = digits.substr(0, 1);
    if (n > 1) body += "." + digits.substr(1);
    char eb[16];
    snprintf(eb, sizeof eb, "e%c%02d", point - 1 >= 0 ? '+' : '-', std::abs(point - 1));
    body += eb;
  } else if (point <= 0) {
    body = "0." + std::string(-point, '0') + digits;
  } else if (point >= n) {
    body = digits + std::string(point - n, '0') + ".0";
  } else {
    body = digits.substr(0, point) + "." + digits.substr(point);
  }
  return sign + body;
}

std::string dumps_py(const Value& v) {
  std::string out;
  dump_py(v, 0, out);
  return out;
}

std::string dumps(const Value& v) {
  std::string out;
  dump(v, out);
  return out;
}

}  // namespace pj
}  // namespace sd
