// JSON for the host code: values keep object key order and tell integers from floats, as the
// reference's serde_json (`preserve_order`, `Cargo.toml:27`) does; `dumps_py` writes Python's
// json.dumps(v, indent=2, ensure_ascii=False) with repr() floats (src/prompt.rs:309-372), and
// `dumps` compact JSON for responses.
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace sd {
namespace pj {

struct Value {
  enum Kind { Null, Bool, Int, Float, String, Array, Object } kind = Null;
  bool b = false;
  long long i = 0;  // Int (also u64 values up to 2^63 - 1; larger integers are Float, as serde_json)
  double f = 0.0;
  std::string s;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  static Value str(std::string v) {
    Value x;
    x.kind = String;
    x.s = std::move(v);
    return x;
  }
  static Value num(double v) {
    Value x;
    x.kind = Float;
    x.f = v;
    return x;
  }
  static Value integer(long long v) {
    Value x;
    x.kind = Int;
    x.i = v;
    return x;
  }
  static Value boolean(bool v) {
    Value x;
    x.kind = Bool;
    x.b = v;
    return x;
  }
  static Value object() {
    Value x;
    x.kind = Object;
    return x;
  }
  static Value array() {
    Value x;
    x.kind = Array;
    return x;
  }
  const Value* get(const std::string& k) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  void set(const std::string& k, Value v) {  // insert or replace, keeping the first position
    for (auto& kv : obj)
      if (kv.first == k) {
        kv.second = std::move(v);
        return;
      }
    obj.emplace_back(k, std::move(v));
  }
  bool is_content() const { return kind == String || kind == Array || kind == Object; }
  bool is_number() const { return kind == Int || kind == Float; }
  double as_double() const { return kind == Int ? (double)i : f; }
};

Value parse(const std::string& text);  // throws std::runtime_error with a message
std::string py_float(double x);        // Python repr(float)
std::string dumps_py(const Value& v);  // json.dumps(v, indent=2, ensure_ascii=False)
std::string dumps(const Value& v);     // compact
void quote(std::string& out, const std::string& s);  // a JSON string literal, non-ASCII kept

}  // namespace pj
}  // namespace sd
