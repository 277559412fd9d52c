// A small backtracking regular-expression matcher over code points, for the tokenizer's pre-tokenizer
// pattern (the reference compiles the pattern of its tokenizer.json with fancy-regex,
// src/tokenizer.rs:129). Leftmost match, alternatives in order, greedy or lazy quantifiers with
// backtracking (Perl semantics). Supported: literals, `.`, classes `[...]` (ranges, negation,
// escapes), \p{..}/\P{..} general categories (L, Lu, ..., Z, Zs, ...), \s \S (White_Space), \d \D,
// \w \W, \r \n \t \f \v \xHH \x{H..} \uHHHH, groups `(...)` `(?:...)` `(?i:...)` `(?i)`, lookahead
// `(?=...)` `(?!...)`, `^` `$`, quantifiers `? * + {n} {n,} {n,m}` and their lazy forms. Anything else
// is a compile error.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace sd {

class Regex {
 public:
  struct Node;
  explicit Regex(const std::string& pattern);  // throws std::runtime_error on syntax it does not support
  ~Regex();
  // Successive non-overlapping leftmost matches in s, as [begin, end) code-point indices.
  std::vector<std::pair<size_t, size_t>> find_all(const std::vector<uint32_t>& s) const;

 private:
  std::unique_ptr<Node> root_;
};

}  // namespace sd
