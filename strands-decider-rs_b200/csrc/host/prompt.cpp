#include "prompt.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>

#include "unicode.h"

namespace sd {
namespace prompt {
namespace {

[[noreturn]] void fail(const std::string& m) { throw std::runtime_error(m); }

// Python's str.strip() (whitespace: str.isspace)
std::string py_strip(const std::string& s) {
  std::vector<uint32_t> cps;
  if (!uni::decode(s, cps)) return s;
  size_t a = 0, b = cps.size();
  while (a < b && uni::py_space(cps[a])) a++;
  while (b > a && uni::py_space(cps[b - 1])) b--;
  return uni::encode(std::vector<uint32_t>(cps.begin() + a, cps.begin() + b));
}

// " ".join(s.split()): runs of Python whitespace collapsed to one space, ends trimmed
std::string py_collapse(const std::string& s) {
  std::vector<uint32_t> cps;
  if (!uni::decode(s, cps)) return s;
  std::string out;
  bool in_word = false, any = false;
  for (uint32_t c : cps) {
    if (uni::py_space(c)) {
      in_word = false;
      continue;
    }
    if (!in_word && any) out += ' ';
    uni::append(out, c);
    in_word = any = true;
  }
  return out;
}

// Python's round(x, 4) as the reference computes it (src/prompt.rs:222-225): the 4-decimal string
double round4(double x) {
  char buf[64];
  snprintf(buf, sizeof buf, "%.4f", x);
  return strtod(buf, nullptr);
}

double choice_confidence(const std::vector<double>& p) {  // derive_confidence (src/prompt.rs:227-235)
  const double n = (double)p.size();
  if (p.size() <= 1) return 1.0;
  double mx = p[0];
  for (double x : p) mx = std::max(mx, x);
  return std::min(std::max((n * mx - 1.0) / (n - 1.0), 0.0), 1.0);
}

double score_confidence(std::vector<double> p, double smoothing) {  // derive_score_confidence (:237-256)
  const size_t n = p.size();
  if (n <= 1) return 1.0;
  double total = 0.0;
  for (double x : p) total += x;
  if (total <= 0.0) return 0.0;
  for (double& x : p) x /= total;
  double mean = 0.0;
  for (size_t i = 0; i < n; i++) mean += (double)i * p[i];
  double var = 0.0;
  for (size_t i = 0; i < n; i++) var += p[i] * ((double)i - mean) * ((double)i - mean);
  const double sigma = std::sqrt(var);
  const double mx = ((double)n - 1.0) / 2.0;
  const double floor = smoothing > 0.0 ? std::sqrt(smoothing) : 0.0;
  if (mx <= floor) return sigma <= floor ? 1.0 : 0.0;
  return std::min(std::max((mx - sigma) / (mx - floor), 0.0), 1.0);
}

const char* header(Kind k) {
  switch (k) {
    case Kind::Noul: return "Decide whether the statement is true of the state.";
    case Kind::Choice: return "Select exactly one option.";
    default: return "Rate the state against the ordered levels below (lowest first).";
  }
}

}  // namespace

const char* kind_name(Kind k) { return k == Kind::Noul ? "noul" : (k == Kind::Choice ? "choice" : "score"); }

Question Question::noul(pj::Value instructions) {
  Question q;
  q.kind = Kind::Noul;
  q.instructions = std::move(instructions);
  q.options = {{"false", pj::Value::str("the statement does not hold for this state")},
               {"true", pj::Value::str("the statement holds for this state")}};
  return q;
}

void Question::validate() const {
  if (!instructions.is_content()) fail("question instructions must be a string, object or array");
  for (const auto& o : options)
    if (o.second.kind != pj::Value::Null && !o.second.is_content()) fail("option descriptions must be strings, objects, arrays or null");
  const size_t n = options.size();
  switch (kind) {
    case Kind::Noul:
      if (n != 2 || options[0].first != "false" || options[1].first != "true") fail("noul options must be false, true");
      break;
    case Kind::Choice:
      if (n < 2 || n > 255) fail("choice requires between 2 and 255 options");
      for (size_t i = 1; i < n; i++)
        for (size_t j = 0; j < i; j++)
          if (options[j].first == options[i].first) fail("choice options must be unique");
      break;
    case Kind::Score:
      if (n < 2 || n > 10) fail("score requires between 2 and 10 levels");
      for (const auto& o : options)
        if (o.second.kind != pj::Value::String) fail("score levels must be strings");
      break;
  }
}

Question Question::from_json(const pj::Value& v) {
  if (v.kind != pj::Value::Object) fail("a question must be an object");
  const pj::Value* criteria = v.get("criteria");
  if (criteria && criteria->kind == pj::Value::Null) criteria = nullptr;
  auto noul_keys = [](const pj::Value* c) {
    for (const auto& kv : c->obj)
      if (kv.first != "true" && kv.first != "false") return false;
    return true;
  };
  Kind kind;
  const pj::Value* t = v.get("type");
  if (t) {
    if (t->kind == pj::Value::String && t->s == "noul") kind = Kind::Noul;
    else if (t->kind == pj::Value::String && t->s == "choice") kind = Kind::Choice;
    else if (t->kind == pj::Value::String && t->s == "score") kind = Kind::Score;
    else fail("question type must be noul, choice or score");
  } else if (!criteria) {
    kind = Kind::Noul;
  } else if (criteria->kind == pj::Value::Array) {
    kind = Kind::Score;
  } else if (criteria->kind == pj::Value::Object && noul_keys(criteria)) {
    kind = Kind::Noul;
  } else {
    kind = Kind::Choice;
  }
  const pj::Value* ins = v.get("instructions");
  pj::Value instructions = ins ? *ins : pj::Value();
  Question q;
  switch (kind) {
    case Kind::Noul:
      if (!criteria) {
        q = Question::noul(instructions);
      } else if (criteria->kind == pj::Value::Object && noul_keys(criteria)) {
        q = Question::noul(instructions);
        for (auto& o : q.options)
          if (const pj::Value* d = criteria->get(o.first)) o.second = *d;
      } else {
        fail("noul criteria keys must be a subset of {'true', 'false'}");
      }
      break;
    case Kind::Choice:
      if (!criteria || criteria->kind != pj::Value::Object) fail("choice criteria must map option names to descriptions");
      q.kind = Kind::Choice;
      q.instructions = instructions;
      for (const auto& kv : criteria->obj) q.options.emplace_back(kv.first, kv.second);
      break;
    case Kind::Score: {
      bool ok = criteria && criteria->kind == pj::Value::Array;
      if (ok)
        for (const auto& c : criteria->arr) ok = ok && c.kind == pj::Value::String;
      if (!ok) fail("score criteria must be a list of level descriptions");
      q.kind = Kind::Score;
      q.instructions = instructions;
      for (size_t i = 0; i < criteria->arr.size(); i++) q.options.emplace_back(std::to_string(i), criteria->arr[i]);
      break;
    }
  }
  q.validate();
  return q;
}

std::string render_content(const pj::Value& v) {  // src/prompt.rs:159-165
  if (v.kind == pj::Value::Null) return "";
  if (v.kind == pj::Value::String) return py_strip(v.s);
  return pj::dumps_py(v);
}

std::string render_state(const pj::Value& state) { return "<state>\n" + render_content(state) + "\n</state>\n"; }

Rendered render_question(const Question& q) {  // src/prompt.rs:171-200
  Rendered r;
  r.kind = q.kind;
  std::string text = std::string("<question type=\"") + kind_name(q.kind) + "\">\n" + header(q.kind) + "\n" +
                     uni::nfc(render_content(q.instructions)) + "\n<options>\n";
  for (size_t i = 0; i < q.options.size(); i++) {
    const std::string d = py_collapse(render_content(q.options[i].second));
    std::string line = std::to_string(i + 1) + ". " + uni::nfc(q.options[i].first);
    if (!d.empty()) line += " \xE2\x80\x94 " + uni::nfc(d);  // " — "
    r.spans.emplace_back((uint32_t)text.size(), (uint32_t)(text.size() + line.size()));
    text += line + "\n";
    r.labels.push_back(q.options[i].first);
    r.descriptions.push_back(render_content(q.options[i].second));
  }
  text += "</options>\n</question>\n<answer>";
  r.text = std::move(text);
  return r;
}

std::vector<size_t> option_token_index(const std::vector<std::pair<uint32_t, uint32_t>>& offsets,
                                       const std::vector<std::pair<uint32_t, uint32_t>>& spans) {
  std::vector<size_t> out;
  for (const auto& sp : spans) {
    long idx = -1;
    for (long i = (long)offsets.size() - 1; i >= 0; i--) {
      const auto& o = offsets[i];
      if (o.second > o.first && o.first >= sp.first && o.second <= sp.second) {
        idx = i;
        break;
      }
    }
    if (idx < 0)
      fail("option span (" + std::to_string(sp.first) + "," + std::to_string(sp.second) +
           ") has no tokens left; the prompt was truncated through its option list");
    out.push_back((size_t)idx);
  }
  return out;
}

pj::Value to_answer(const Rendered& rq, const std::vector<double>& p, double smoothing) {  // src/prompt.rs:258-296
  pj::Value a = pj::Value::object();
  a.set("type", pj::Value::str(kind_name(rq.kind)));
  if (rq.kind == Kind::Noul) {
    size_t t = 0;
    for (size_t i = 0; i < rq.labels.size(); i++)
      if (rq.labels[i] == "true") t = i;
    a.set("noul", pj::Value::num(round4(p[t])));
    return a;
  }
  pj::Value probs = pj::Value::object();
  for (size_t i = 0; i < rq.labels.size(); i++) probs.set(rq.labels[i], pj::Value::num(round4(p[i])));
  if (rq.kind == Kind::Choice) {
    size_t best = 0;
    for (size_t i = 0; i < p.size(); i++)
      if (p[i] > p[best]) best = i;
    a.set("choice", pj::Value::str(rq.labels[best]));
    a.set("probabilities", probs);
    a.set("confidence", pj::Value::num(round4(choice_confidence(p))));
    return a;
  }
  double s = 0.0;
  for (size_t i = 0; i < p.size(); i++) s += (double)i * p[i];
  a.set("score", pj::Value::num(round4(s)));
  pj::Value legend = pj::Value::object();
  for (size_t i = 0; i < rq.labels.size(); i++) legend.set(rq.labels[i], pj::Value::str(rq.descriptions[i]));
  a.set("legend", legend);
  a.set("probabilities", probs);
  a.set("confidence", pj::Value::num(round4(score_confidence(p, smoothing))));
  return a;
}

}  // namespace prompt
}  // namespace sd
