// Backtracking matcher: the pattern is parsed into a tree; matching is continuation-passing (each
// node calls the rest of the match with the position it reached, and backtracks when that fails).
// A repeat of one character class is matched iteratively (longest run first, then shorter), so long
// runs such as a whitespace block do not recurse per character.
#include "regex.h"

#include <functional>
#include <stdexcept>

#include "unicode.h"

namespace sd {

struct Regex::Node {
  enum Kind { Char, Class, Any, Seq, Alt, Repeat, Look, Bol, Eol } kind;
  // Char
  uint32_t cp = 0;
  bool icase = false;
  // Class: items are code-point ranges or categories; matches when any item does, xor negate
  struct Item {
    enum { Range, Cat, Major, Space, Digit, Word } type;
    uint32_t lo = 0, hi = 0;
    std::string cat;
    bool neg = false;  // \P{..}, \S, \D, \W inside a class
  };
  std::vector<Item> items;
  bool negate = false;
  // Seq, Alt, Repeat (child[0]), Look (child[0])
  std::vector<std::unique_ptr<Node>> child;
  int min = 0, max = -1;  // Repeat; max -1: unbounded
  bool greedy = true;
  bool look_neg = false;  // Look: (?!...)

  explicit Node(Kind k) : kind(k) {}

  bool single() const { return kind == Char || kind == Class || kind == Any; }

  static bool item_match(const Item& it, uint32_t c) {
    bool r = false;
    switch (it.type) {
      case Item::Range: r = c >= it.lo && c <= it.hi; break;
      case Item::Cat: r = it.cat == uni::category(c); break;
      case Item::Major: r = uni::major(c) == it.cat[0]; break;
      case Item::Space: r = uni::white_space(c); break;
      case Item::Digit: r = std::string(uni::category(c)) == "Nd"; break;
      case Item::Word: {
        const char* g = uni::category(c);
        r = g[0] == 'L' || g[0] == 'M' || (g[0] == 'N' && g[1] == 'd') || (g[0] == 'P' && g[1] == 'c') || c == 0x200C || c == 0x200D;
        break;
      }
    }
    return r != it.neg;
  }

  bool match1(uint32_t c) const {
    switch (kind) {
      case Char:
        if (c == cp) return true;
        return icase && uni::to_lower(uni::to_upper(c)) == uni::to_lower(uni::to_upper(cp));
      case Any: return c != '\n';
      case Class: {
        bool m = false;
        for (const Item& it : items)
          if (item_match(it, c) || (icase && (item_match(it, uni::to_lower(c)) || item_match(it, uni::to_upper(c))))) {
            m = true;
            break;
          }
        return m != negate;
      }
      default: return false;
    }
  }
};

namespace {

using Node = Regex::Node;
using Ptr = std::unique_ptr<Node>;

class Parser {
 public:
  explicit Parser(const std::string& p) {
    if (!uni::decode(p, s_)) throw std::runtime_error("pattern is not UTF-8");
  }
  Ptr parse() {
    Ptr n = alt();
    if (i_ != s_.size()) fail("unbalanced ')'");
    return n;
  }

 private:
  std::vector<uint32_t> s_;
  size_t i_ = 0;
  bool icase_ = false;

  [[noreturn]] void fail(const std::string& what) { throw std::runtime_error("regex: " + what + " at " + std::to_string(i_)); }
  bool eof() const { return i_ >= s_.size(); }
  uint32_t peek() const { return s_[i_]; }
  bool take(uint32_t c) {
    if (!eof() && s_[i_] == c) {
      i_++;
      return true;
    }
    return false;
  }

  // an inline (?i) lasts to the end of the enclosing group, later alternatives included
  Ptr alt() {
    const bool saved = icase_;
    std::vector<Ptr> opts;
    opts.push_back(seq());
    while (take('|')) opts.push_back(seq());
    icase_ = saved;
    if (opts.size() == 1) return std::move(opts[0]);
    Ptr n(new Node(Node::Alt));
    n->child = std::move(opts);
    return n;
  }

  Ptr seq() {
    Ptr n(new Node(Node::Seq));
    while (!eof() && peek() != '|' && peek() != ')') {
      Ptr a = atom();
      if (!a) continue;  // a flag group such as (?i)
      a = quantified(std::move(a));
      n->child.push_back(std::move(a));
    }
    return n;
  }

  Ptr quantified(Ptr a) {
    while (!eof()) {
      int mn, mx;
      const uint32_t c = peek();
      if (c == '?') mn = 0, mx = 1;
      else if (c == '*') mn = 0, mx = -1;
      else if (c == '+') mn = 1, mx = -1;
      else if (c == '{' && brace(mn, mx)) {
      } else break;
      if (c != '{') i_++;
      Ptr r(new Node(Node::Repeat));
      r->min = mn, r->max = mx;
      r->greedy = !take('?');
      if (take('+')) fail("possessive quantifiers are not supported");
      r->child.push_back(std::move(a));
      a = std::move(r);
    }
    return a;
  }

  // {n}, {n,}, {n,m}; leaves i_ unchanged (and returns false) when this is not a quantifier
  bool brace(int& mn, int& mx) {
    size_t j = i_ + 1;
    auto num = [&](int& v) {
      size_t k = j;
      v = 0;
      while (j < s_.size() && s_[j] >= '0' && s_[j] <= '9') v = v * 10 + (int)(s_[j++] - '0');
      return j > k;
    };
    if (!num(mn)) return false;
    mx = mn;
    if (j < s_.size() && s_[j] == ',') {
      j++;
      if (!num(mx)) mx = -1;
    }
    if (j >= s_.size() || s_[j] != '}') return false;
    i_ = j + 1;
    return true;
  }

  Ptr atom() {
    const uint32_t c = s_[i_++];
    switch (c) {
      case '(': return group();
      case '[': return cls();
      case '.': return Ptr(new Node(Node::Any));
      case '^': return Ptr(new Node(Node::Bol));
      case '$': return Ptr(new Node(Node::Eol));
      case '\\': return escape();
      case '*': case '+': case '?': fail("nothing to repeat");
      default: {
        Ptr n(new Node(Node::Char));
        n->cp = c;
        n->icase = icase_;
        return n;
      }
    }
  }

  Ptr group() {
    if (take('?')) {
      if (eof()) fail("bad group");
      if (take(':')) return closed(alt());
      if (peek() == '=' || peek() == '!') {
        const bool neg = s_[i_++] == '!';
        Ptr n(new Node(Node::Look));
        n->look_neg = neg;
        n->child.push_back(alt());
        if (!take(')')) fail("missing ')'");
        return n;
      }
      // flags: (?i) or (?i:...)
      bool on = false;
      while (!eof() && peek() == 'i') on = true, i_++;
      if (!on) fail("unsupported group");
      if (take(')')) {
        icase_ = true;
        return nullptr;
      }
      if (!take(':')) fail("unsupported group flags");
      const bool saved = icase_;
      icase_ = true;
      Ptr n = alt();
      icase_ = saved;
      return closed(std::move(n));
    }
    return closed(alt());  // capturing group: the matcher only reports whole matches
  }

  Ptr closed(Ptr n) {
    if (!take(')')) fail("missing ')'");
    return n;
  }

  uint32_t hex(int digits) {  // digits < 0: braced
    uint32_t v = 0;
    int n = 0;
    const bool braced = digits < 0 && take('{');
    while (!eof() && (braced || n < digits)) {
      const uint32_t c = peek();
      int d;
      if (c >= '0' && c <= '9') d = c - '0';
      else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
      else break;
      v = v * 16 + d, n++, i_++;
    }
    if (braced && !take('}')) fail("bad \\x{..}");
    if (n == 0 || (!braced && digits > 0 && n != digits)) fail("bad hex escape");
    return v;
  }

  // an escape: a class item, or a literal code point (item.type == Range with lo == hi)
  Node::Item escape_item() {
    if (eof()) fail("trailing '\\'");
    const uint32_t c = s_[i_++];
    Node::Item it;
    it.type = Node::Item::Range;
    switch (c) {
      case 'p': case 'P': {
        std::string name;
        if (take('{')) {
          while (!eof() && peek() != '}') name += (char)s_[i_++];
          if (!take('}')) fail("bad \\p{..}");
        } else {
          if (eof()) fail("bad \\p");
          name = (char)s_[i_++];
        }
        static const char* majors = "LMNPSZC";
        if (name.size() == 1 && std::string(majors).find(name[0]) != std::string::npos) it.type = Node::Item::Major;
        else if (name.size() == 2 && std::string(majors).find(name[0]) != std::string::npos) it.type = Node::Item::Cat;
        else fail("unsupported property \\p{" + name + "}");
        it.cat = name;
        it.neg = c == 'P';
        return it;
      }
      case 's': case 'S': it.type = Node::Item::Space, it.neg = c == 'S'; return it;
      case 'd': case 'D': it.type = Node::Item::Digit, it.neg = c == 'D'; return it;
      case 'w': case 'W': it.type = Node::Item::Word, it.neg = c == 'W'; return it;
      case 'n': it.lo = it.hi = '\n'; return it;
      case 'r': it.lo = it.hi = '\r'; return it;
      case 't': it.lo = it.hi = '\t'; return it;
      case 'f': it.lo = it.hi = '\f'; return it;
      case 'v': it.lo = it.hi = '\v'; return it;
      case 'x': it.lo = it.hi = (!eof() && peek() == '{') ? hex(-1) : hex(2); return it;
      case 'u': it.lo = it.hi = hex(4); return it;
      default:
        if ((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9'))
          fail(std::string("unsupported escape \\") + (char)c);
        it.lo = it.hi = c;  // escaped punctuation
        return it;
    }
  }

  Ptr escape() {
    Node::Item it = escape_item();
    if (it.type == Node::Item::Range) {
      Ptr n(new Node(Node::Char));
      n->cp = it.lo;
      n->icase = icase_;
      return n;
    }
    Ptr n(new Node(Node::Class));
    n->items.push_back(it);
    n->icase = icase_;
    return n;
  }

  Ptr cls() {
    Ptr n(new Node(Node::Class));
    n->icase = icase_;
    n->negate = take('^');
    bool first = true;
    while (true) {
      if (eof()) fail("unterminated class");
      if (peek() == ']' && !first) {
        i_++;
        break;
      }
      first = false;
      Node::Item it;
      if (take('\\')) {
        it = escape_item();
      } else {
        if (peek() == '[') fail("nested classes are not supported");
        it.type = Node::Item::Range;
        it.lo = it.hi = s_[i_++];
      }
      // a range a-b (a literal on both sides)
      if (it.type == Node::Item::Range && i_ + 1 < s_.size() && peek() == '-' && s_[i_ + 1] != ']') {
        i_++;
        Node::Item hi;
        if (take('\\')) hi = escape_item();
        else hi.type = Node::Item::Range, hi.lo = hi.hi = s_[i_++];
        if (hi.type != Node::Item::Range || hi.lo < it.lo) fail("bad class range");
        it.hi = hi.lo;
      }
      n->items.push_back(it);
    }
    return n;
  }
};

using Cont = std::function<bool(size_t)>;

bool m(const Node* n, const std::vector<uint32_t>& s, size_t i, const Cont& k);

bool seq_from(const Node* n, size_t j, const std::vector<uint32_t>& s, size_t i, const Cont& k) {
  if (j == n->child.size()) return k(i);
  return m(n->child[j].get(), s, i, [&](size_t p) { return seq_from(n, j + 1, s, p, k); });
}

bool rep(const Node* n, int count, const std::vector<uint32_t>& s, size_t i, const Cont& k) {
  const Node* c = n->child[0].get();
  const bool more = n->max < 0 || count < n->max;
  auto again = [&](size_t p) { return p != i && rep(n, count + 1, s, p, k); };  // an empty pass ends the loop
  if (n->greedy) {
    if (more && m(c, s, i, again)) return true;
    return count >= n->min && k(i);
  }
  if (count >= n->min && k(i)) return true;
  return more && m(c, s, i, again);
}

bool m(const Node* n, const std::vector<uint32_t>& s, size_t i, const Cont& k) {
  switch (n->kind) {
    case Node::Char:
    case Node::Class:
    case Node::Any: return i < s.size() && n->match1(s[i]) && k(i + 1);
    case Node::Seq: return seq_from(n, 0, s, i, k);
    case Node::Alt:
      for (const auto& c : n->child)
        if (m(c.get(), s, i, k)) return true;
      return false;
    case Node::Repeat: {
      const Node* c = n->child[0].get();
      if (c->single()) {  // iterative: the longest run first (greedy) or the shortest (lazy)
        size_t run = 0;
        const size_t cap = n->max < 0 ? s.size() - i : std::min<size_t>(s.size() - i, (size_t)n->max);
        while (run < cap && c->match1(s[i + run])) run++;
        if ((int)run < n->min) return false;
        if (n->greedy) {
          for (size_t r = run + 1; r-- > (size_t)n->min;)
            if (k(i + r)) return true;
        } else {
          for (size_t r = n->min; r <= run; r++)
            if (k(i + r)) return true;
        }
        return false;
      }
      return rep(n, 0, s, i, k);
    }
    case Node::Look: {
      const bool found = m(n->child[0].get(), s, i, [](size_t) { return true; });
      return found != n->look_neg && k(i);
    }
    case Node::Bol: return i == 0 && k(i);
    case Node::Eol: return i == s.size() && k(i);
  }
  return false;
}

}  // namespace

Regex::Regex(const std::string& pattern) { root_ = Parser(pattern).parse(); }
Regex::~Regex() = default;

std::vector<std::pair<size_t, size_t>> Regex::find_all(const std::vector<uint32_t>& s) const {
  std::vector<std::pair<size_t, size_t>> out;
  size_t i = 0;
  while (i <= s.size()) {
    size_t end = 0;
    bool found = false;
    size_t st = i;
    for (; st <= s.size(); st++)
      if (m(root_.get(), s, st, [&](size_t p) { end = p; return true; })) {
        found = true;
        break;
      }
    if (!found) break;
    out.emplace_back(st, end);
    i = end > st ? end : st + 1;  // after an empty match, search on from the next character
  }
  return out;
}

}  // namespace sd
