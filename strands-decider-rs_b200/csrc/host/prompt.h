// Prompt rendering and answer reading (the reference's src/prompt.rs): Question (:28-140), render_content /
// render_state / render_question (:159-200), option_token_index (:203-213), to_answer and
// Answer::to_json (:215-296).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "pyjson.h"

namespace sd {
namespace prompt {

enum class Kind { Noul, Choice, Score };
const char* kind_name(Kind k);

struct Question {
  Kind kind = Kind::Noul;
  pj::Value instructions;
  std::vector<std::pair<std::string, pj::Value>> options;  // (label, description; Null: none)

  static Question noul(pj::Value instructions);
  void validate() const;                       // throws std::runtime_error with the schema's message
  static Question from_json(const pj::Value& v);  // the System One form {"type", "instructions", "criteria"}
};

struct Rendered {
  std::string text;
  Kind kind = Kind::Noul;
  std::vector<std::string> labels;
  std::vector<std::string> descriptions;
  std::vector<std::pair<uint32_t, uint32_t>> spans;  // UTF-8 byte ranges of each option's line in text
};

std::string render_content(const pj::Value& v);
std::string render_state(const pj::Value& state);
Rendered render_question(const Question& q);
// The last token inside each option's line; throws when a line has none (the prompt was cut).
std::vector<size_t> option_token_index(const std::vector<std::pair<uint32_t, uint32_t>>& offsets,
                                       const std::vector<std::pair<uint32_t, uint32_t>>& spans);
// The answer as `Answer::to_json` writes it, from the head's probabilities over the options.
pj::Value to_answer(const Rendered& rq, const std::vector<double>& probs, double ordinal_smoothing);

}  // namespace prompt
}  // namespace sd
