// Unicode support for the host code (tokenizer, prompt): UTF-8 conversion, general categories,
// whitespace classes, simple case mappings and NFC, from tables generated out of Python's
// unicodedata (unicode_tables.inc, gen_unicode.py).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace sd {
namespace uni {

// UTF-8 -> code points; false on malformed input. `byte_at` (optional) receives the byte offset of
// each code point, plus the total length at the end.
bool decode(const std::string& s, std::vector<uint32_t>& out, std::vector<size_t>* byte_at = nullptr);
std::string encode(const std::vector<uint32_t>& cps);
void append(std::string& out, uint32_t cp);

// General category: two-letter name ("Lu", "Nd", ...; "Cn" when unassigned) and its major class
// letter ('L', 'M', 'N', 'P', 'S', 'Z', 'C').
const char* category(uint32_t cp);
char major(uint32_t cp);
int combining_class(uint32_t cp);

bool white_space(uint32_t cp);  // the White_Space property (regex \s)
bool py_space(uint32_t cp);     // Python's str.isspace (str.strip, str.split)
uint32_t to_lower(uint32_t cp);  // simple (one code point) mappings
uint32_t to_upper(uint32_t cp);

// Normalization Form C.
std::vector<uint32_t> nfc(const std::vector<uint32_t>& cps);
std::string nfc(const std::string& s);  // s must be valid UTF-8

const char* version();

}  // namespace uni
}  // namespace sd
