#include "tokenizer.h"

#include <algorithm>
#include <queue>
#include <stdexcept>
#include <tuple>

#include "pyjson.h"
#include "unicode.h"

namespace sd {
namespace {

// Printable stand-ins for the 256 byte values, as byte-level BPE vocabularies are written
// (src/tokenizer.rs:67-81).
std::vector<uint32_t> byte_chars() {
  std::vector<uint32_t> out(256);
  uint32_t n = 0;
  for (uint32_t b = 0; b < 256; b++) {
    const bool printable = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    out[b] = printable ? b : 255 + (++n);
  }
  return out;
}

[[noreturn]] void unsupported(const std::string& what) { throw std::runtime_error("tokenizer.json: unsupported " + what); }

bool is(const pj::Value* v, const char* s) { return v && v->kind == pj::Value::String && v->s == s; }
bool is_false(const pj::Value* v) { return v && v->kind == pj::Value::Bool && !v->b; }
bool truthy(const pj::Value* v) { return v && v->kind == pj::Value::Bool && v->b; }

}  // namespace

std::unique_ptr<Tokenizer> Tokenizer::from_json(const std::string& text) {
  pj::Value f;
  try {
    f = pj::parse(text);
  } catch (const std::exception& e) {
    throw std::runtime_error(std::string("tokenizer.json: ") + e.what());
  }
  const pj::Value* norm = f.get("normalizer");
  if (norm && norm->kind != pj::Value::Null && !(norm->kind == pj::Value::Object && norm->obj.size() == 1 && is(norm->get("type"), "NFC")))
    unsupported("normalizer");
  const pj::Value* p = f.get("pre_tokenizer");
  const pj::Value* pts = p ? p->get("pretokenizers") : nullptr;
  const bool ok = p && is(p->get("type"), "Sequence") && pts && pts->kind == pj::Value::Array && pts->arr.size() == 2;
  const pj::Value* split = ok ? &pts->arr[0] : nullptr;
  const pj::Value* bl = ok ? &pts->arr[1] : nullptr;
  const pj::Value* pat = (ok && split->get("pattern")) ? split->get("pattern")->get("Regex") : nullptr;
  if (!(ok && is(split->get("type"), "Split") && is(split->get("behavior"), "Isolated") && is_false(split->get("invert")) && pat &&
        pat->kind == pj::Value::String && is(bl->get("type"), "ByteLevel") && is_false(bl->get("add_prefix_space")) &&
        is_false(bl->get("use_regex"))))
    unsupported("pre_tokenizer");
  const pj::Value* m = f.get("model");
  if (!m || !is(m->get("type"), "BPE") || truthy(m->get("byte_fallback")) || truthy(m->get("ignore_merges"))) unsupported("model");
  std::unique_ptr<Tokenizer> t(new Tokenizer());
  const pj::Value* added = f.get("added_tokens");
  if (added && added->kind == pj::Value::Array)
    for (const pj::Value& a : added->arr) {
      if (truthy(a.get("single_word")) || truthy(a.get("lstrip")) || truthy(a.get("rstrip")) || truthy(a.get("normalized")))
        unsupported("added token options");
      const pj::Value* c = a.get("content");
      const pj::Value* id = a.get("id");
      if (!c || c->kind != pj::Value::String || !id || id->kind != pj::Value::Int) unsupported("added token");
      t->added_.emplace_back(c->s, (uint32_t)id->i);
    }
  std::stable_sort(t->added_.begin(), t->added_.end(), [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
  const pj::Value* vocab = m->get("vocab");
  if (!vocab || vocab->kind != pj::Value::Object) unsupported("model");
  std::unordered_map<std::string, uint32_t> v;
  v.reserve(vocab->obj.size() * 2);
  for (const auto& kv : vocab->obj) v[kv.first] = (uint32_t)kv.second.i;
  const std::vector<uint32_t> chars = byte_chars();
  t->byte_id_.resize(256);
  for (int b = 0; b < 256; b++) {
    std::string s;
    uni::append(s, chars[b]);
    auto it = v.find(s);
    if (it == v.end()) unsupported("vocabulary (missing a byte)");
    t->byte_id_[b] = it->second;
  }
  const pj::Value* merges = m->get("merges");
  if (merges && merges->kind == pj::Value::Array) {
    uint32_t rank = 0;
    for (const pj::Value& mg : merges->arr) {
      std::string a, b;
      if (mg.kind == pj::Value::Array && mg.arr.size() == 2 && mg.arr[0].kind == pj::Value::String && mg.arr[1].kind == pj::Value::String) {
        a = mg.arr[0].s, b = mg.arr[1].s;
      } else if (mg.kind == pj::Value::String) {
        const size_t sp = mg.s.find(' ');
        if (sp == std::string::npos) unsupported("merge");
        a = mg.s.substr(0, sp), b = mg.s.substr(sp + 1);
      } else {
        unsupported("merge");
      }
      auto ia = v.find(a), ib = v.find(b), iab = v.find(a + b);
      if (ia == v.end() || ib == v.end() || iab == v.end()) unsupported("merge (token not in vocabulary)");
      const uint64_t key = ((uint64_t)ia->second << 32) | ib->second;
      t->merges_[key] = {rank, iab->second};  // a pair listed twice keeps its last rank, as the reference's map insert
      rank++;
    }
  }
  try {
    t->split_.reset(new Regex(pat->s));
  } catch (const std::exception& e) {
    throw std::runtime_error(std::string("tokenizer.json: pre-tokenizer regex: ") + e.what());
  }
  return t;
}

Encoding Tokenizer::encode(const std::string& text) const {
  std::vector<uint32_t> check;
  if (!uni::decode(text, check)) throw std::runtime_error("text is not UTF-8");
  Encoding enc;
  uint32_t base = 0;
  size_t pos = 0;  // byte position in text
  while (pos < text.size()) {
    // the leftmost added token (the longest one there), at a character boundary
    size_t gap = text.size();
    const std::pair<std::string, uint32_t>* special = nullptr;
    if (!added_.empty())
      for (size_t i = pos; i < text.size(); i++) {
        if (((unsigned char)text[i] & 0xC0) == 0x80) continue;
        for (const auto& a : added_)
          if (text.compare(i, a.first.size(), a.first) == 0) {
            gap = i, special = &a;
            break;
          }
        if (special) break;
      }
    const std::string segment = uni::nfc(text.substr(pos, gap - pos));
    encode_segment(segment, base, enc);
    base += (uint32_t)segment.size();
    if (!special) break;
    enc.ids.push_back(special->second);
    enc.offsets.emplace_back(base, base + (uint32_t)special->first.size());
    base += (uint32_t)special->first.size();
    pos = gap + special->first.size();
  }
  return enc;
}

void Tokenizer::encode_segment(const std::string& s, uint32_t base, Encoding& enc) const {
  std::vector<uint32_t> cps;
  std::vector<size_t> cb;
  uni::decode(s, cps, &cb);
  size_t last = 0;
  for (const auto& mt : split_->find_all(cps)) {
    const size_t st = cb[mt.first], en = cb[mt.second];
    if (st > last) bpe(s, last, st, base, enc);
    if (en > st) bpe(s, st, en, base, enc);
    last = en;
  }
  if (last < s.size()) bpe(s, last, s.size(), base, enc);
}

void Tokenizer::bpe(const std::string& b, size_t from, size_t to, uint32_t base, Encoding& enc) const {
  const int n = (int)(to - from);
  std::vector<uint32_t> ids(n);
  std::vector<int> len(n, 1), prev(n), next(n);
  for (int i = 0; i < n; i++) {
    ids[i] = byte_id_[(unsigned char)b[from + i]];
    prev[i] = i - 1;
    next[i] = i + 1 < n ? i + 1 : -1;
  }
  // (rank, position, merged id): lowest rank first, then leftmost
  using E = std::tuple<uint32_t, int, uint32_t>;
  std::priority_queue<E, std::vector<E>, std::greater<E>> q;
  auto lookup = [&](uint32_t a, uint32_t c) -> const std::pair<uint32_t, uint32_t>* {
    auto it = merges_.find(((uint64_t)a << 32) | c);
    return it == merges_.end() ? nullptr : &it->second;
  };
  for (int i = 0; i + 1 < n; i++)
    if (auto mg = lookup(ids[i], ids[i + 1])) q.emplace(mg->first, i, mg->second);
  while (!q.empty()) {
    const auto [rank, pos, new_id] = q.top();
    q.pop();
    const int nx = next[pos];
    if (len[pos] == 0 || nx == -1) continue;
    auto mg = lookup(ids[pos], ids[nx]);
    if (!mg || mg->second != new_id) continue;
    ids[pos] = new_id;
    len[pos] += len[nx];
    next[pos] = next[nx];
    len[nx] = 0;
    const int after = next[pos];
    if (after != -1) prev[after] = pos;
    const int pv = prev[pos];
    if (pv != -1)
      if (auto m2 = lookup(ids[pv], new_id)) q.emplace(m2->first, pv, m2->second);
    if (after != -1)
      if (auto m2 = lookup(new_id, ids[after])) q.emplace(m2->first, pos, m2->second);
  }
  for (int i = 0; i < n; i++) {
    if (len[i] == 0) continue;
    size_t lo = from + i, hi = from + i + len[i];
    while (lo > 0 && ((unsigned char)b[lo] & 0xC0) == 0x80) lo--;
    while (hi < b.size() && ((unsigned char)b[hi] & 0xC0) == 0x80) hi++;
    enc.ids.push_back(ids[i]);
    enc.offsets.emplace_back(base + (uint32_t)lo, base + (uint32_t)hi);
  }
}

}  // namespace sd
