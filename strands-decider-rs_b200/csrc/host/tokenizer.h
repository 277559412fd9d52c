// Byte-level BPE from a tokenizer.json, encode direction only (the reference's src/tokenizer.rs:14-246):
// added tokens matched leftmost-longest first (:157-165), NFC per segment between them (:135-155),
// the Split pre-tokenizer regex with its gaps encoded as their own pieces (:167-181), lowest-rank
// merge first with leftmost tie-break (:185-232), and byte offsets into the normalized text that widen
// a partial character to the whole character (:233-244).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "regex.h"

namespace sd {

struct Encoding {
  std::vector<uint32_t> ids;
  std::vector<std::pair<uint32_t, uint32_t>> offsets;  // byte ranges in the NFC text
};

class Tokenizer {
 public:
  // `Tokenizer::from_json` (src/tokenizer.rs:84-131), with its checks on the file shape; throws
  // std::runtime_error.
  static std::unique_ptr<Tokenizer> from_json(const std::string& text);
  // `Tokenizer::encode` (src/tokenizer.rs:135-155); text must be UTF-8 (throws otherwise).
  Encoding encode(const std::string& text) const;

 private:
  std::vector<uint32_t> byte_id_;                                      // 256 entries
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges_;  // (a << 32 | b) -> (rank, id)
  std::vector<std::pair<std::string, uint32_t>> added_;                // longest (UTF-8 bytes) first
  std::unique_ptr<Regex> split_;

  void encode_segment(const std::string& seg, uint32_t base, Encoding& enc) const;
  void bpe(const std::string& b, size_t from, size_t to, uint32_t base, Encoding& enc) const;
};

}  // namespace sd
