// The Decider (the reference's src/lib.rs:100-209) in C++ over the engine's C ABI: tokenizer, prompt,
// torso (sd_forward / sd_forward_fork), pointer head, answers. Exposed as sd_decider_* (JSON request in,
// the System One response body out), plus the tokenizer and prompt rendering on their own.
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>
#include <atomic>

#include "prompt.h"
#include "pyjson.h"
#include "sd_b200.h"
#include "tokenizer.h"
#include "unicode.h"

namespace {

thread_local std::string g_host_error;

constexpr size_t kMaxBatch = 32;  // questions per fork; the reference's MAX_BATCH (src/lib.rs:107-108)

int host_fail(std::string* slot, const std::string& msg) {
  if (slot) *slot = msg;
  g_host_error = msg;
  return SD_ERR_INVALID;
}

// fn(i) for i in [0, n) on up to `threads` host threads (0: one per hardware thread, at most 16);
// fn must not throw.
template <class F>
void parallel_for(size_t n, int threads, F&& fn) {
  size_t t = threads > 0 ? (size_t)threads : std::min<size_t>(16, std::max(1u, std::thread::hardware_concurrency()));
  t = std::min(t, n);
  if (t <= 1) {
    for (size_t i = 0; i < n; i++) fn(i);
    return;
  }
  std::atomic<size_t> next{0};
  auto work = [&]() {
    for (size_t i; (i = next.fetch_add(1)) < n;) fn(i);
  };
  std::vector<std::thread> pool;
  for (size_t k = 1; k < t; k++) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
}

bool read_file(const std::string& path, std::string& out, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = path + ": cannot open";
    return false;
  }
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

char* dup_string(const std::string& s) {
  char* p = static_cast<char*>(malloc(s.size() + 1));
  if (p) memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

struct Config {  // hobson_config.json (src/lib.rs:89-98)
  size_t max_length = 0;
  double temperature = 1.0;
  std::map<std::string, double> temperature_by_kind;
  double ordinal_smoothing = 0.0;
};

}  // namespace

struct sd_tokenizer {
  std::unique_ptr<sd::Tokenizer> tok;
};

struct sd_decider {
  sd_engine* engine = nullptr;
  sd_head* head = nullptr;
  std::unique_ptr<sd::Tokenizer> tok;
  Config cfg;
  std::string err;

  ~sd_decider() {
    sd_head_free(head);
    sd_engine_destroy(engine);
  }

  double temperature(sd::prompt::Kind k) const {
    auto it = cfg.temperature_by_kind.find(sd::prompt::kind_name(k));
    return it == cfg.temperature_by_kind.end() ? cfg.temperature : it->second;
  }

  // A request ready for the torso: its questions rendered, the state and the questions tokenized,
  // the option tokens located (the part of `Decider::run`, src/lib.rs:156-184, before the forwards).
  struct Prepared {
    std::vector<std::pair<std::string, sd::prompt::Question>> named;
    std::vector<sd::prompt::Rendered> rendered;
    sd::Encoding st;
    std::vector<sd::Encoding> qs;
    std::vector<std::vector<size_t>> options;
  };

  Prepared prepare(const sd::pj::Value& state, const std::vector<std::pair<std::string, sd::prompt::Question>>& named) const {
    using namespace sd;
    if (!state.is_content()) throw std::runtime_error("state must be a string, object or array");
    if (named.empty()) throw std::runtime_error("ask at least one question");
    for (const auto& q : named) q.second.validate();
    Prepared p;
    p.named = named;
    for (const auto& q : named) p.rendered.push_back(prompt::render_question(q.second));
    p.st = tok->encode(prompt::render_state(state));
    size_t longest = 0;
    for (const auto& r : p.rendered) {
      p.qs.push_back(tok->encode(r.text));
      longest = std::max(longest, p.qs.back().ids.size());
    }
    const size_t ns = p.st.ids.size();
    if (ns + longest > cfg.max_length)
      throw std::runtime_error("prompt of " + std::to_string(ns + longest) + " tokens (" + std::to_string(ns) + " state + " +
                               std::to_string(longest) + " question) exceeds the context window of " +
                               std::to_string(cfg.max_length) + " tokens");
    for (size_t i = 0; i < p.qs.size(); i++) p.options.push_back(prompt::option_token_index(p.qs[i].offsets, p.rendered[i].spans));
    return p;
  }

  // The pointer head over question i's hidden rows (its options', then its last token's).
  std::vector<double> head_probs(const Prepared& p, size_t i, const float* hidden, size_t nrows) const {
    std::vector<double> probs(nrows - 1);
    if (sd_head_probs(head, hidden, (int32_t)nrows, sd_engine_hidden_size(engine), temperature(p.rendered[i].kind),
                      probs.data()) != SD_OK)
      throw std::runtime_error(sd_last_error());
    return probs;
  }

  // `Response::to_json` (src/lib.rs:78-87) from each question's probabilities; usage as the official
  // engine counts it: chunks of questions, each with the state once.
  sd::pj::Value respond(const Prepared& p, const std::vector<std::vector<double>>& probs) const {
    using namespace sd;
    pj::Value answers = pj::Value::object();
    for (size_t i = 0; i < p.qs.size(); i++)
      answers.set(p.named[i].first, prompt::to_answer(p.rendered[i], probs[i], cfg.ordinal_smoothing));
    size_t input_tokens = 0;
    for (size_t c = 0; c < p.qs.size(); c += kMaxBatch) {
      const size_t e = std::min(p.qs.size(), c + kMaxBatch);
      input_tokens += p.st.ids.size();
      for (size_t i = c; i < e; i++) input_tokens += p.qs[i].ids.size();
    }
    pj::Value usage = pj::Value::object();
    usage.set("input_tokens", pj::Value::integer((long long)input_tokens));
    usage.set("output_tokens", pj::Value::integer((long long)p.named.size()));
    pj::Value resp = pj::Value::object();
    resp.set("model", pj::Value::str("strands-decider-rs-0.1.0"));
    resp.set("answers", answers);
    resp.set("usage", usage);
    return resp;
  }

  void check(int rc) const {
    if (rc != SD_OK) throw std::runtime_error(sd_engine_last_error(engine));
  }

  // Whether a request fits one tree pass (at most 65536 tokens and 4096 sequences per pass).
  static bool fits_tree(const Prepared& p) {
    size_t tokens = p.st.ids.size();
    for (const auto& q : p.qs) tokens += q.ids.size();
    return tokens <= 65536 && p.qs.size() < 4096;
  }

  // `Decider::run` (src/lib.rs:156-208): the answers, in question order, and the usage count.
  sd::pj::Value run(const sd::pj::Value& state, const std::vector<std::pair<std::string, sd::prompt::Question>>& named) {
    const Prepared p = prepare(state, named);
    const size_t ns = p.st.ids.size();
    const int d = sd_engine_hidden_size(engine);
    std::vector<std::vector<double>> probs(p.qs.size());
    if (p.qs.size() == 1) {
      std::vector<uint32_t> ids(p.st.ids);
      ids.insert(ids.end(), p.qs[0].ids.begin(), p.qs[0].ids.end());
      std::vector<int32_t> rows;
      for (size_t o : p.options[0]) rows.push_back((int32_t)(ns + o));
      rows.push_back((int32_t)ids.size() - 1);
      std::vector<float> hidden(rows.size() * (size_t)d);
      check(sd_forward(engine, ids.data(), (int32_t)ids.size(), rows.data(), (int32_t)rows.size(), nullptr, 0, hidden.data(),
                       nullptr, nullptr));
      probs[0] = head_probs(p, 0, hidden.data(), rows.size());
    } else if (fits_tree(p)) {
      // the state and every question in one packed pass, each question continuing the state
      std::vector<uint32_t> ids(p.st.ids);
      std::vector<int32_t> lens{(int32_t)ns}, parent{-1}, rows, nrows{0};
      for (size_t i = 0; i < p.qs.size(); i++) {
        ids.insert(ids.end(), p.qs[i].ids.begin(), p.qs[i].ids.end());
        lens.push_back((int32_t)p.qs[i].ids.size());
        parent.push_back(0);
        for (size_t o : p.options[i]) rows.push_back((int32_t)o);
        rows.push_back((int32_t)p.qs[i].ids.size() - 1);
        nrows.push_back((int32_t)p.options[i].size() + 1);
      }
      std::vector<float> hidden(rows.size() * (size_t)d);
      check(sd_forward_tree(engine, nullptr, parent.data(), ids.data(), lens.data(), (int32_t)lens.size(), rows.data(),
                            nrows.data(), hidden.data()));
      size_t at = 0;
      for (size_t i = 0; i < p.qs.size(); i++) {
        probs[i] = head_probs(p, i, hidden.data() + at * d, (size_t)nrows[i + 1]);
        at += nrows[i + 1];
      }
    } else {
      sd_snapshot* prefix = nullptr;
      check(sd_forward(engine, p.st.ids.data(), (int32_t)ns, nullptr, 0, nullptr, 1, nullptr, &prefix, nullptr));
      try {
        for (size_t c = 0; c < p.qs.size(); c += kMaxBatch) {
          const size_t e = std::min(p.qs.size(), c + kMaxBatch);
          std::vector<uint32_t> ids;
          std::vector<int32_t> lens, rows, nrows;
          for (size_t i = c; i < e; i++) {
            ids.insert(ids.end(), p.qs[i].ids.begin(), p.qs[i].ids.end());
            lens.push_back((int32_t)p.qs[i].ids.size());
            for (size_t o : p.options[i]) rows.push_back((int32_t)o);
            rows.push_back((int32_t)p.qs[i].ids.size() - 1);
            nrows.push_back((int32_t)p.options[i].size() + 1);
          }
          std::vector<float> hidden(rows.size() * (size_t)d);
          check(sd_forward_fork(engine, prefix, ids.data(), lens.data(), (int32_t)lens.size(), rows.data(), nrows.data(),
                                hidden.data(), nullptr));
          size_t at = 0;
          for (size_t i = c; i < e; i++) {
            probs[i] = head_probs(p, i, hidden.data() + at * d, (size_t)nrows[i - c]);
            at += nrows[i - c];
          }
        }
      } catch (...) {
        sd_snapshot_free(prefix);
        throw;
      }
      sd_snapshot_free(prefix);
    }
    return respond(p, probs);
  }

  // Many requests at once, as a server answers concurrent ones: whole requests in packed tree passes
  // (sd_forward_tree_probs: each request's state, or with a single question state and question
  // together as `Decider::run` does, then its questions continuing it in the same pass), with the
  // pointer head on the GPU. A request too long for one pass takes two: its state kept as a snapshot
  // (sd_forward_batch), then its questions continuing it in packed forks (sd_forward_fork_multi_probs).
  // Each request's answers equal its own `run` up to f32 summation order. out[i]: the response, or {"error": message} for a request that
  // failed (invalid, too long, or a failed pass of the torso).
  std::vector<sd::pj::Value> run_batch(const std::vector<const sd::pj::Value*>& states,
                                       const std::vector<std::vector<std::pair<std::string, sd::prompt::Question>>>& named,
                                       std::vector<std::string> errors) {
    using namespace sd;
    constexpr size_t kPassTokens = 65536, kPassSeqs = 4096;  // the packed passes' limits
    const size_t n = states.size();
    const int d = sd_engine_hidden_size(engine);
    std::vector<Prepared> prep(n);
    std::vector<std::vector<std::vector<double>>> probs(n);
    std::vector<sd_snapshot*> snaps(n, nullptr);
    // rendering and tokenizing, request by request on the host threads (the tokenizer is read-only)
    parallel_for(n, 0, [&](size_t r) {
      if (!errors[r].empty()) return;
      try {
        prep[r] = prepare(*states[r], named[r]);
        probs[r].resize(prep[r].qs.size());
      } catch (const std::exception& e) {
        errors[r] = e.what();
      }
    });
    auto fail_all = [&](const std::vector<size_t>& group, const std::string& msg) {
      for (size_t r : group) errors[r] = msg;
    };
    // tree passes: whole requests, as many as one pass holds
    {
      std::vector<size_t> group;
      size_t tokens = 0, seqs = 0;
      auto flush = [&]() {
        if (group.empty()) return;
        std::vector<uint32_t> ids;
        std::vector<int32_t> lens, parent, rows, nrows;
        std::vector<double> temps;
        std::vector<std::pair<size_t, size_t>> asked;  // (request, question) of each sequence with rows
        for (size_t r : group) {
          const Prepared& p = prep[r];
          const size_t ns = p.st.ids.size();
          const int32_t root = (int32_t)lens.size();
          ids.insert(ids.end(), p.st.ids.begin(), p.st.ids.end());
          parent.push_back(-1);
          if (p.qs.size() == 1) {
            ids.insert(ids.end(), p.qs[0].ids.begin(), p.qs[0].ids.end());
            for (size_t o : p.options[0]) rows.push_back((int32_t)(ns + o));
            rows.push_back((int32_t)(ns + p.qs[0].ids.size()) - 1);
            nrows.push_back((int32_t)p.options[0].size() + 1);
            lens.push_back((int32_t)(ns + p.qs[0].ids.size()));
            temps.push_back(temperature(p.rendered[0].kind));
            asked.emplace_back(r, 0);
            continue;
          }
          lens.push_back((int32_t)ns);
          nrows.push_back(0);
          temps.push_back(1.0);
          for (size_t i = 0; i < p.qs.size(); i++) {
            ids.insert(ids.end(), p.qs[i].ids.begin(), p.qs[i].ids.end());
            lens.push_back((int32_t)p.qs[i].ids.size());
            parent.push_back(root);
            for (size_t o : p.options[i]) rows.push_back((int32_t)o);
            rows.push_back((int32_t)p.qs[i].ids.size() - 1);
            nrows.push_back((int32_t)p.options[i].size() + 1);
            temps.push_back(temperature(p.rendered[i].kind));
            asked.emplace_back(r, i);
          }
        }
        std::vector<double> all(rows.size() - asked.size());
        const int rc = sd_forward_tree_probs(engine, nullptr, parent.data(), ids.data(), lens.data(), (int32_t)lens.size(),
                                             rows.data(), nrows.data(), head, temps.data(), all.data());
        if (rc != SD_OK) {
          fail_all(group, sd_engine_last_error(engine));
        } else {
          size_t at = 0;
          for (const auto& rq : asked) {
            const size_t k = prep[rq.first].options[rq.second].size();
            probs[rq.first][rq.second].assign(all.begin() + at, all.begin() + at + k);
            at += k;
          }
        }
        group.clear();
        tokens = seqs = 0;
      };
      for (size_t r = 0; r < n; r++) {
        if (!errors[r].empty() || !fits_tree(prep[r])) continue;
        const Prepared& p = prep[r];
        size_t len = p.st.ids.size();
        for (const auto& q : p.qs) len += q.ids.size();
        const size_t ns = p.qs.size() == 1 ? 1 : 1 + p.qs.size();
        if (tokens + len > kPassTokens || seqs + ns > kPassSeqs) flush();
        group.push_back(r);
        tokens += len;
        seqs += ns;
      }
      flush();
    }
    // requests too long for one tree pass. pass 1: one sequence per request
    {
      std::vector<size_t> group;
      size_t tokens = 0;
      auto flush = [&]() {
        if (group.empty()) return;
        std::vector<uint32_t> ids;
        std::vector<int32_t> lens, rows, nrows;
        for (size_t r : group) {
          const Prepared& p = prep[r];
          const size_t ns = p.st.ids.size();
          ids.insert(ids.end(), p.st.ids.begin(), p.st.ids.end());
          if (p.qs.size() == 1) {
            ids.insert(ids.end(), p.qs[0].ids.begin(), p.qs[0].ids.end());
            for (size_t o : p.options[0]) rows.push_back((int32_t)(ns + o));
            rows.push_back((int32_t)(ns + p.qs[0].ids.size()) - 1);
            nrows.push_back((int32_t)p.options[0].size() + 1);
            lens.push_back((int32_t)(ns + p.qs[0].ids.size()));
          } else {
            nrows.push_back(0);
            lens.push_back((int32_t)ns);
          }
        }
        std::vector<float> hidden(rows.size() * (size_t)d);
        std::vector<sd_snapshot*> out(group.size(), nullptr);
        const int rc = sd_forward_batch(engine, nullptr, ids.data(), lens.data(), (int32_t)lens.size(), rows.data(), nrows.data(),
                                        1, hidden.data(), out.data(), nullptr);
        if (rc != SD_OK) {
          fail_all(group, sd_engine_last_error(engine));
        } else {
          size_t at = 0;
          for (size_t g = 0; g < group.size(); g++) {
            const size_t r = group[g];
            if (prep[r].qs.size() == 1) {
              sd_snapshot_free(out[g]);
              try {
                probs[r][0] = head_probs(prep[r], 0, hidden.data() + at * d, (size_t)nrows[g]);
              } catch (const std::exception& e) {
                errors[r] = e.what();
              }
              at += nrows[g];
            } else {
              snaps[r] = out[g];
            }
          }
        }
        group.clear();
        tokens = 0;
      };
      for (size_t r = 0; r < n; r++) {
        if (!errors[r].empty() || fits_tree(prep[r])) continue;
        const Prepared& p = prep[r];
        const size_t len = p.st.ids.size() + (p.qs.size() == 1 ? p.qs[0].ids.size() : 0);
        if (tokens + len > kPassTokens || group.size() == kPassSeqs) flush();
        group.push_back(r);
        tokens += len;
      }
      flush();
    }
    // pass 2: every question of the requests with several, each continuing its request's snapshot
    {
      std::vector<std::pair<size_t, size_t>> group;  // (request, question)
      size_t tokens = 0;
      auto flush = [&]() {
        if (group.empty()) return;
        std::vector<const sd_snapshot*> caches;
        std::vector<uint32_t> ids;
        std::vector<int32_t> lens, rows, nrows;
        std::vector<double> temps;
        for (const auto& rq : group) {
          const Prepared& p = prep[rq.first];
          const Encoding& q = p.qs[rq.second];
          caches.push_back(snaps[rq.first]);
          ids.insert(ids.end(), q.ids.begin(), q.ids.end());
          lens.push_back((int32_t)q.ids.size());
          for (size_t o : p.options[rq.second]) rows.push_back((int32_t)o);
          rows.push_back((int32_t)q.ids.size() - 1);
          nrows.push_back((int32_t)p.options[rq.second].size() + 1);
          temps.push_back(temperature(p.rendered[rq.second].kind));
        }
        // the fork and the pointer head on the GPU: only the probabilities come back
        std::vector<double> all(rows.size() - group.size());
        const int rc = sd_forward_fork_multi_probs(engine, caches.data(), ids.data(), lens.data(), (int32_t)lens.size(),
                                                   rows.data(), nrows.data(), head, temps.data(), all.data());
        size_t at = 0;
        for (size_t g = 0; g < group.size(); g++) {
          const size_t r = group[g].first;
          if (rc != SD_OK) {
            errors[r] = sd_engine_last_error(engine);
          } else if (errors[r].empty()) {
            probs[r][group[g].second].assign(all.begin() + at, all.begin() + at + nrows[g] - 1);
          }
          at += nrows[g] - 1;
        }
        group.clear();
        tokens = 0;
      };
      for (size_t r = 0; r < n; r++) {
        if (!snaps[r]) continue;
        for (size_t i = 0; i < prep[r].qs.size(); i++) {
          const size_t len = prep[r].qs[i].ids.size();
          if (tokens + len > kPassTokens || group.size() == kPassSeqs) flush();
          group.emplace_back(r, i);
          tokens += len;
        }
      }
      flush();
    }
    for (sd_snapshot* s : snaps) sd_snapshot_free(s);
    std::vector<pj::Value> out(n);
    for (size_t r = 0; r < n; r++) {
      if (errors[r].empty()) {
        out[r] = respond(prep[r], probs[r]);
      } else {
        out[r] = pj::Value::object();
        out[r].set("error", pj::Value::str(errors[r]));
      }
    }
    return out;
  }
};

extern "C" {

const char* sd_host_last_error(void) { return g_host_error.c_str(); }

void sd_string_free(char* s) { free(s); }

int sd_tokenizer_load(const char* path, sd_tokenizer** out) {
  if (!path || !out) return host_fail(nullptr, "sd_tokenizer_load: null argument");
  std::string text, err;
  if (!read_file(path, text, err)) return host_fail(nullptr, err);
  try {
    auto t = new sd_tokenizer();
    t->tok = sd::Tokenizer::from_json(text);
    *out = t;
    return SD_OK;
  } catch (const std::exception& e) {
    return host_fail(nullptr, e.what());
  }
}

void sd_tokenizer_free(sd_tokenizer* t) { delete t; }

int sd_tokenizer_encode(const sd_tokenizer* t, const char* text, size_t len, uint32_t* ids, uint32_t* offsets, int64_t cap,
                        int64_t* n_out) {
  if (!t || (!text && len) || !n_out) return host_fail(nullptr, "sd_tokenizer_encode: null argument");
  try {
    const sd::Encoding enc = t->tok->encode(std::string(text ? text : "", len));
    *n_out = (int64_t)enc.ids.size();
    for (int64_t i = 0; i < (int64_t)enc.ids.size() && i < cap; i++) {
      if (ids) ids[i] = enc.ids[i];
      if (offsets) offsets[2 * i] = enc.offsets[i].first, offsets[2 * i + 1] = enc.offsets[i].second;
    }
    return SD_OK;
  } catch (const std::exception& e) {
    return host_fail(nullptr, e.what());
  }
}

int sd_tokenizer_encode_batch(const sd_tokenizer* t, const char* const* texts, const size_t* lens, int64_t n, int32_t threads,
                              uint32_t* ids, uint32_t* offsets, int64_t cap, int64_t* counts) {
  if (!t || n < 0 || (n > 0 && (!texts || !lens || !counts)))
    return host_fail(nullptr, "sd_tokenizer_encode_batch: null argument");
  for (int64_t i = 0; i < n; i++)
    if (!texts[i] && lens[i]) return host_fail(nullptr, "sd_tokenizer_encode_batch: null text");
  std::vector<sd::Encoding> enc((size_t)n);
  std::vector<std::string> errs((size_t)n);
  parallel_for((size_t)n, threads, [&](size_t i) {
    try {
      enc[i] = t->tok->encode(std::string(texts[i] ? texts[i] : "", lens[i]));
    } catch (const std::exception& e) {
      errs[i] = e.what();
    }
  });
  for (int64_t i = 0; i < n; i++)
    if (!errs[i].empty()) return host_fail(nullptr, "text " + std::to_string(i) + ": " + errs[i]);
  int64_t at = 0;
  for (int64_t i = 0; i < n; i++) {
    counts[i] = (int64_t)enc[i].ids.size();
    for (size_t k = 0; k < enc[i].ids.size() && at < cap; k++, at++) {
      if (ids) ids[at] = enc[i].ids[k];
      if (offsets) offsets[2 * at] = enc[i].offsets[k].first, offsets[2 * at + 1] = enc[i].offsets[k].second;
    }
  }
  return SD_OK;
}

int sd_prompt_render(const char* request_json, char** out_json) {
  if (!request_json || !out_json) return host_fail(nullptr, "sd_prompt_render: null argument");
  try {
    using namespace sd;
    const pj::Value req = pj::parse(request_json);
    const pj::Value* state = req.get("state");
    const pj::Value* qs = req.get("questions");
    pj::Value out = pj::Value::object();
    out.set("state", pj::Value::str(prompt::render_state(state ? *state : pj::Value())));
    pj::Value arr = pj::Value::array();
    if (qs && qs->kind == pj::Value::Array)
      for (const pj::Value& q : qs->arr) {
        const prompt::Rendered r = prompt::render_question(prompt::Question::from_json(q));
        pj::Value o = pj::Value::object();
        o.set("text", pj::Value::str(r.text));
        pj::Value spans = pj::Value::array();
        for (const auto& sp : r.spans) {
          pj::Value p = pj::Value::array();
          p.arr.push_back(pj::Value::integer(sp.first));
          p.arr.push_back(pj::Value::integer(sp.second));
          spans.arr.push_back(p);
        }
        o.set("spans", spans);
        arr.arr.push_back(o);
      }
    out.set("questions", arr);
    *out_json = dup_string(pj::dumps(out));
    return SD_OK;
  } catch (const std::exception& e) {
    return host_fail(nullptr, e.what());
  }
}

int sd_decider_load(const char* model_dir, int device, sd_decider** out) {
  if (!model_dir || !out) return host_fail(nullptr, "sd_decider_load: null argument");
  const std::string dir(model_dir);
  std::unique_ptr<sd_decider> d(new sd_decider());
  std::string text, err;
  if (!read_file(dir + "/tokenizer.json", text, err)) return host_fail(nullptr, err);
  try {
    d->tok = sd::Tokenizer::from_json(text);
  } catch (const std::exception& e) {
    return host_fail(nullptr, e.what());
  }
  int rc = sd_engine_create(model_dir, device, &d->engine);
  if (rc != SD_OK) return host_fail(nullptr, sd_last_error()), rc;
  rc = sd_head_load((dir + "/head.safetensors").c_str(), &d->head);
  if (rc != SD_OK) return host_fail(nullptr, sd_last_error()), rc;
  if (!read_file(dir + "/hobson_config.json", text, err)) return host_fail(nullptr, err);
  try {
    const sd::pj::Value c = sd::pj::parse(text);
    const sd::pj::Value* ml = c.get("max_length");
    const sd::pj::Value* t = c.get("temperature");
    if (!ml || ml->kind != sd::pj::Value::Int || ml->i < 0) throw std::runtime_error("missing or bad field `max_length`");
    if (!t || !t->is_number()) throw std::runtime_error("missing or bad field `temperature`");
    d->cfg.max_length = (size_t)ml->i;
    d->cfg.temperature = t->as_double();
    if (const sd::pj::Value* tk = c.get("temperature_by_kind")) {
      if (tk->kind != sd::pj::Value::Object) throw std::runtime_error("bad field `temperature_by_kind`");
      for (const auto& kv : tk->obj) {
        if (!kv.second.is_number()) throw std::runtime_error("bad field `temperature_by_kind`");
        d->cfg.temperature_by_kind[kv.first] = kv.second.as_double();
      }
    }
    if (const sd::pj::Value* os = c.get("ordinal_smoothing")) {
      if (!os->is_number()) throw std::runtime_error("bad field `ordinal_smoothing`");
      d->cfg.ordinal_smoothing = os->as_double();
    }
  } catch (const std::exception& e) {
    return host_fail(nullptr, std::string("hobson_config.json: ") + e.what());
  }
  *out = d.release();
  return SD_OK;
}

void sd_decider_free(sd_decider* d) { delete d; }

// `Request::from_json` (src/lib.rs:46-63): the state, and the questions in order.
static const sd::pj::Value* parse_request(const sd::pj::Value& req,
                                          std::vector<std::pair<std::string, sd::prompt::Question>>& named) {
  using namespace sd;
  const pj::Value* state = req.kind == pj::Value::Object ? req.get("state") : nullptr;
  if (!state || !state->is_content()) throw std::runtime_error("state must be a string, object or array");
  const pj::Value* images = req.get("images");
  if (images && images->kind == pj::Value::Array && !images->arr.empty())
    throw std::runtime_error("this engine has no vision tower; images are not supported");
  const pj::Value* qs = req.get("questions");
  if (!qs || qs->kind != pj::Value::Object || qs->obj.empty()) throw std::runtime_error("questions must be a non-empty object");
  for (const auto& kv : qs->obj) {
    try {
      named.emplace_back(kv.first, prompt::Question::from_json(kv.second));
    } catch (const std::exception& e) {
      throw std::runtime_error("question " + kv.first + ": " + e.what());
    }
  }
  return state;
}

const char* sd_decider_last_error(const sd_decider* d) { return d ? d->err.c_str() : g_host_error.c_str(); }

int sd_decider_ask_all(sd_decider* d, const char* request_json, char** response_json) {
  if (!d || !request_json || !response_json) return host_fail(d ? &d->err : nullptr, "sd_decider_ask_all: null argument");
  *response_json = nullptr;
  try {
    using namespace sd;
    const pj::Value req = pj::parse(request_json);
    std::vector<std::pair<std::string, prompt::Question>> named;
    const pj::Value* state = parse_request(req, named);
    *response_json = dup_string(pj::dumps(d->run(*state, named)));
    return SD_OK;
  } catch (const std::exception& e) {
    return host_fail(&d->err, e.what());
  }
}

int sd_decider_ask_batch(sd_decider* d, const char* requests_json, char** responses_json) {
  if (!d || !requests_json || !responses_json)
    return host_fail(d ? &d->err : nullptr, "sd_decider_ask_batch: null argument");
  *responses_json = nullptr;
  try {
    using namespace sd;
    const pj::Value reqs = pj::parse(requests_json);
    if (reqs.kind != pj::Value::Array) throw std::runtime_error("requests must be a JSON array");
    const size_t n = reqs.arr.size();
    std::vector<const pj::Value*> states(n, nullptr);
    std::vector<std::vector<std::pair<std::string, prompt::Question>>> named(n);
    std::vector<std::string> errors(n);
    for (size_t r = 0; r < n; r++) {
      try {
        states[r] = parse_request(reqs.arr[r], named[r]);
      } catch (const std::exception& e) {
        errors[r] = e.what();
      }
    }
    pj::Value out = pj::Value::array();
    for (auto& v : d->run_batch(states, named, errors)) out.arr.push_back(std::move(v));
    *responses_json = dup_string(pj::dumps(out));
    return SD_OK;
  } catch (const std::exception& e) {
    return host_fail(&d->err, e.what());
  }
}

}  // extern "C"
