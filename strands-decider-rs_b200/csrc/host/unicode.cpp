// Unicode tables and NFC (UAX #15: full canonical decomposition, canonical ordering, canonical
// composition; Hangul syllables algorithmically).
#include "unicode.h"

#include <algorithm>

namespace sd {
namespace uni {
namespace {

struct CatRange {
  uint32_t lo, hi;
  uint8_t v;
};
struct Decomp {
  uint32_t cp, off, n;
};
struct Compose {
  uint32_t a, b, c;
};
struct CaseMap {
  uint32_t from, to;
};

#include "unicode_tables.inc"

constexpr uint32_t SBase = 0xAC00, LBase = 0x1100, VBase = 0x1161, TBase = 0x11A7;
constexpr uint32_t LCount = 19, VCount = 21, TCount = 28, NCount = VCount * TCount, SCount = LCount * NCount;

template <size_t N>
int range_value(const CatRange (&t)[N], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (t[mid].hi < cp) lo = mid + 1;
    else hi = mid;
  }
  return (lo < N && t[lo].lo <= cp && cp <= t[lo].hi) ? t[lo].v : 0;
}

template <size_t N>
uint32_t case_map(const CaseMap (&t)[N], uint32_t cp) {
  const CaseMap* e = std::lower_bound(t, t + N, cp, [](const CaseMap& m, uint32_t x) { return m.from < x; });
  return (e != t + N && e->from == cp) ? e->to : cp;
}

const Decomp* find_decomp(uint32_t cp) {
  constexpr size_t N = sizeof(kDecomp) / sizeof(kDecomp[0]);
  const Decomp* e = std::lower_bound(kDecomp, kDecomp + N, cp, [](const Decomp& d, uint32_t x) { return d.cp < x; });
  return (e != kDecomp + N && e->cp == cp) ? e : nullptr;
}

uint32_t compose_pair(uint32_t a, uint32_t b) {
  if (a >= LBase && a < LBase + LCount && b >= VBase && b < VBase + VCount)
    return SBase + ((a - LBase) * VCount + (b - VBase)) * TCount;
  if (a >= SBase && a < SBase + SCount && (a - SBase) % TCount == 0 && b > TBase && b < TBase + TCount)
    return a + (b - TBase);
  constexpr size_t N = sizeof(kCompose) / sizeof(kCompose[0]);
  const Compose* e = std::lower_bound(kCompose, kCompose + N, std::make_pair(a, b), [](const Compose& c, std::pair<uint32_t, uint32_t> x) {
    return c.a < x.first || (c.a == x.first && c.b < x.second);
  });
  return (e != kCompose + N && e->a == a && e->b == b) ? e->c : 0;
}

}  // namespace

const char* version() { return SD_UNICODE_VERSION; }

bool decode(const std::string& s, std::vector<uint32_t>& out, std::vector<size_t>* byte_at) {
  out.clear();
  if (byte_at) byte_at->clear();
  const size_t n = s.size();
  size_t i = 0;
  while (i < n) {
    const unsigned char c = (unsigned char)s[i];
    uint32_t cp;
    size_t len;
    if (c < 0x80) cp = c, len = 1;
    else if ((c & 0xE0) == 0xC0) cp = c & 0x1F, len = 2;
    else if ((c & 0xF0) == 0xE0) cp = c & 0x0F, len = 3;
    else if ((c & 0xF8) == 0xF0) cp = c & 0x07, len = 4;
    else return false;
    if (i + len > n) return false;
    for (size_t k = 1; k < len; k++) {
      const unsigned char cc = (unsigned char)s[i + k];
      if ((cc & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (cc & 0x3F);
    }
    // overlong forms, surrogates and values past U+10FFFF are not UTF-8
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF ||
        (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    if (byte_at) byte_at->push_back(i);
    out.push_back(cp);
    i += len;
  }
  if (byte_at) byte_at->push_back(n);
  return true;
}

void append(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += (char)cp;
  } else if (cp < 0x800) {
    out += (char)(0xC0 | (cp >> 6));
    out += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += (char)(0xE0 | (cp >> 12));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  } else {
    out += (char)(0xF0 | (cp >> 18));
    out += (char)(0x80 | ((cp >> 12) & 0x3F));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  }
}

std::string encode(const std::vector<uint32_t>& cps) {
  std::string out;
  out.reserve(cps.size());
  for (uint32_t cp : cps) append(out, cp);
  return out;
}

const char* category(uint32_t cp) { return kCatNames[range_value(kCats, cp)]; }
char major(uint32_t cp) { return category(cp)[0]; }
int combining_class(uint32_t cp) { return range_value(kCcc, cp); }

bool white_space(uint32_t cp) {
  return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 || (cp >= 0x2000 && cp <= 0x200A) ||
         cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F || cp == 0x3000;
}

bool py_space(uint32_t cp) {
  constexpr size_t N = sizeof(kPySpace) / sizeof(kPySpace[0]);
  return std::binary_search(kPySpace, kPySpace + N, cp);
}

uint32_t to_lower(uint32_t cp) { return case_map(kLower, cp); }
uint32_t to_upper(uint32_t cp) { return case_map(kUpper, cp); }

std::vector<uint32_t> nfc(const std::vector<uint32_t>& in) {
  // 1. full canonical decomposition
  std::vector<uint32_t> d;
  d.reserve(in.size() + 8);
  for (uint32_t cp : in) {
    if (cp >= SBase && cp < SBase + SCount) {
      const uint32_t s = cp - SBase;
      d.push_back(LBase + s / NCount);
      d.push_back(VBase + (s % NCount) / TCount);
      if (s % TCount) d.push_back(TBase + s % TCount);
    } else if (const Decomp* e = find_decomp(cp)) {
      d.insert(d.end(), kDecompData + e->off, kDecompData + e->off + e->n);
    } else {
      d.push_back(cp);
    }
  }
  // 2. canonical ordering: stable sort of each run of non-starters by combining class
  std::vector<int> cc(d.size());
  for (size_t i = 0; i < d.size(); i++) cc[i] = combining_class(d[i]);
  for (size_t i = 0; i < d.size();) {
    if (cc[i] == 0) {
      i++;
      continue;
    }
    size_t j = i;
    while (j < d.size() && cc[j] != 0) j++;
    for (size_t a = i + 1; a < j; a++)  // insertion sort (runs are short), stable
      for (size_t b = a; b > i && cc[b - 1] > cc[b]; b--) std::swap(cc[b - 1], cc[b]), std::swap(d[b - 1], d[b]);
    i = j;
  }
  // 3. canonical composition
  std::vector<uint32_t> out;
  out.reserve(d.size());
  long starter = -1;  // index in out of the last starter
  int last_cc = -1;   // class of the last character after the starter (-1: none, adjacent)
  for (size_t i = 0; i < d.size(); i++) {
    const uint32_t ch = d[i];
    const int c = cc[i];
    if (starter >= 0 && (last_cc == -1 || (last_cc != 0 && last_cc < c))) {
      const uint32_t comp = compose_pair(out[starter], ch);
      if (comp) {
        out[starter] = comp;
        continue;
      }
    }
    if (c == 0) {
      starter = (long)out.size();
      last_cc = -1;
    } else {
      last_cc = c;
    }
    out.push_back(ch);
  }
  return out;
}

std::string nfc(const std::string& s) {
  std::vector<uint32_t> cps;
  if (!decode(s, cps)) return s;
  bool ascii = true;
  for (uint32_t cp : cps) ascii = ascii && cp < 0x80;
  return ascii ? s : encode(nfc(cps));
}

}  // namespace uni
}  // namespace sd
