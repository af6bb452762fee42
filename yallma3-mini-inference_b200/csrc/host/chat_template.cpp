// Renderer for the Jinja subset chat templates use. The reference renders
// tokenizer.chat_template with minijinja 2.20.0 (Cargo.lock) at its default
// settings (tokenizer.rs:408-430); this file follows minijinja's semantics:
//  * template text: no trim_blocks / lstrip_blocks; a single trailing newline
//    of the source is dropped; `{%-`, `-%}`, `{{-`, `-}}`, `{#-`, `-#}` strip
//    the neighbouring Unicode White_Space; `+` markers are accepted (no-ops);
//  * undefined values (lenient): print as empty text, iterate as empty, are
//    false, compare equal to undefined only; attribute or item access on them,
//    calling them and arithmetic on them are errors;
//  * values print as minijinja prints them (true / false / none);
//  * strings, lists and maps have no Python-style methods (`.strip()` and the
//    like need minijinja-contrib's pycompat, which the reference does not use);
//    attribute access on a map is key lookup;
//  * a `{% set %}` inside a for loop lives in the loop's one frame: it is
//    visible in later iterations and gone after the loop.
// Statements: for (name or name tuple targets, an `if` filter, else), if /
// elif / else, set (name, namespace attribute). Expressions: string (with
// \n \t \r \b \f \\ \' \" \/ \uXXXX escapes), integer, boolean, none, list,
// tuple and map literals; names, attributes, subscripts, slices with steps,
// calls of range / namespace / dict; operators `if else`, or, and, not,
// comparisons, in, not in, + - * // % ** ~, unary minus; filters and tests as
// listed in apply_filter / run_test; raw blocks. Floats, macros, call /
// filter / with blocks, includes and the remaining builtin filters give
// YL_ERR_UNSUPPORTED.
#include "chat_template.h"

#include <pthread.h>

#include <algorithm>
#include <cctype>
#include <climits>
#include <cstring>
#include <new>
#include <stdexcept>
#include <unordered_map>

#include "common.h"
#include "tokenizer.h"

namespace yl {

struct TplError : std::runtime_error {
  int code;
  TplError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

namespace {

[[noreturn]] void bad(const std::string& m) { throw TplError(YL_ERR_FORMAT, m); }
[[noreturn]] void unsup(const std::string& m) { throw TplError(YL_ERR_UNSUPPORTED, m + " (not supported)"); }

// ------------------------------------------------------------------ values --

struct Val;
using ValList = std::vector<Val>;
using ValMap = std::vector<std::pair<std::string, Val>>;  // insertion order, unique keys

struct Val {
  enum Kind { UNDEF, NONE, BOOL, INT, STR, LIST, MAP } k = UNDEF;
  enum Tag { PLAIN, NAMESPACE, LOOP } tag = PLAIN;
  bool b = false;
  int64_t i = 0;
  std::string s;
  std::shared_ptr<ValList> l;
  std::shared_ptr<ValMap> m;
};

Val v_none() { Val v; v.k = Val::NONE; return v; }
Val v_bool(bool b) { Val v; v.k = Val::BOOL; v.b = b; return v; }
Val v_int(int64_t i) { Val v; v.k = Val::INT; v.i = i; return v; }
Val v_str(std::string s) { Val v; v.k = Val::STR; v.s = std::move(s); return v; }
Val v_list(ValList l = {}) { Val v; v.k = Val::LIST; v.l = std::make_shared<ValList>(std::move(l)); return v; }
Val v_map(ValMap m = {}) { Val v; v.k = Val::MAP; v.m = std::make_shared<ValMap>(std::move(m)); return v; }

const char* kind_name(const Val& v) {
  static const char* n[] = {"undefined", "none", "bool", "number", "string", "sequence", "map"};
  return n[v.k];
}

const Val* map_find(const ValMap& m, const std::string& key) {
  for (const auto& kv : m)
    if (kv.first == key) return &kv.second;
  return nullptr;
}
void map_put(ValMap* m, const std::string& key, Val v) {
  for (auto& kv : *m)
    if (kv.first == key) { kv.second = std::move(v); return; }
  m->push_back({key, std::move(v)});
}

// byte offsets of the code points of a (valid UTF-8) string, plus its size
std::vector<size_t> cp_offsets(const std::string& s) {
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  if (!utf8_code_points(s, &cps, &offs)) bad("text is not UTF-8");
  return offs;
}
ValList chars_of(const std::string& s) {
  const std::vector<size_t> o = cp_offsets(s);
  ValList out;
  for (size_t k = 0; k + 1 < o.size(); ++k) out.push_back(v_str(s.substr(o[k], o[k + 1] - o[k])));
  return out;
}

std::string trim_ws(const std::string& s, bool left, bool right) {
  std::vector<uint32_t> cps;
  std::vector<size_t> o;
  if (!utf8_code_points(s, &cps, &o)) bad("text is not UTF-8");
  size_t a = 0, b = cps.size();
  while (left && a < b && is_white_space(cps[a])) ++a;
  while (right && b > a && is_white_space(cps[b - 1])) --b;
  return s.substr(o[a], o[b] - o[a]);
}

std::string to_text(const Val& v) {
  switch (v.k) {
    case Val::UNDEF: return "";
    case Val::NONE: return "none";
    case Val::BOOL: return v.b ? "true" : "false";
    case Val::INT: return std::to_string(v.i);
    case Val::STR: return v.s;
    default: unsup(std::string("printing a ") + kind_name(v));
  }
}

bool truthy(const Val& v) {
  switch (v.k) {
    case Val::BOOL: return v.b;
    case Val::INT: return v.i != 0;
    case Val::STR: return !v.s.empty();
    case Val::LIST: return !v.l->empty();
    case Val::MAP: return !v.m->empty();
    default: return false;
  }
}

bool is_num(const Val& v) { return v.k == Val::INT || v.k == Val::BOOL; }
int64_t num(const Val& v) { return v.k == Val::INT ? v.i : (int64_t)v.b; }

bool equal(const Val& a, const Val& b) {
  if (is_num(a) && is_num(b)) return num(a) == num(b);
  if (a.k != b.k) return false;
  switch (a.k) {
    case Val::UNDEF: case Val::NONE: return true;
    case Val::STR: return a.s == b.s;
    case Val::LIST:
      if (a.l->size() != b.l->size()) return false;
      for (size_t q = 0; q < a.l->size(); ++q)
        if (!equal((*a.l)[q], (*b.l)[q])) return false;
      return true;
    case Val::MAP:
      if (a.tag == Val::NAMESPACE || b.tag == Val::NAMESPACE) return a.m == b.m;
      if (a.m->size() != b.m->size()) return false;
      for (const auto& kv : *a.m) {
        const Val* o = map_find(*b.m, kv.first);
        if (!o || !equal(kv.second, *o)) return false;
      }
      return true;
    default: return false;
  }
}

// <0, 0, >0 for numbers and for strings (UTF-8 byte order is code point order)
int order(const Val& a, const Val& b) {
  if (is_num(a) && is_num(b)) return num(a) < num(b) ? -1 : num(a) > num(b) ? 1 : 0;
  if (a.k == Val::STR && b.k == Val::STR) return a.s.compare(b.s) < 0 ? -1 : a.s == b.s ? 0 : 1;
  bad(std::string("cannot compare ") + kind_name(a) + " with " + kind_name(b));
}

bool contains(const Val& hay, const Val& needle) {
  switch (hay.k) {
    case Val::STR:
      if (needle.k != Val::STR) bad("'in <string>' needs a string on the left");
      return hay.s.find(needle.s) != std::string::npos;
    case Val::LIST:
      for (const Val& x : *hay.l)
        if (equal(x, needle)) return true;
      return false;
    case Val::MAP: return needle.k == Val::STR && map_find(*hay.m, needle.s) != nullptr;
    case Val::UNDEF: return false;
    default: bad(std::string("cannot test membership in a ") + kind_name(hay));
  }
}

ValList iterate(const Val& v) {
  switch (v.k) {
    case Val::UNDEF: return {};
    case Val::LIST: return *v.l;
    case Val::STR: return chars_of(v.s);
    case Val::MAP: {
      ValList keys;
      for (const auto& kv : *v.m) keys.push_back(v_str(kv.first));
      return keys;
    }
    default: bad(std::string("a ") + kind_name(v) + " is not iterable");
  }
}

// --------------------------------------------------------- expression AST --

struct Expr;
using ExprP = std::shared_ptr<Expr>;
struct Expr {
  enum Kind { CONST, NAME, LIST, MAP, ATTR, ITEM, SLICE, CALL, FILTER, TEST, NOT, NEG, BIN, COND } k;
  Val c;                                          // CONST
  std::string name;                               // NAME, ATTR, FILTER, TEST, BIN operator
  std::vector<ExprP> a;                           // operand(s), then positional arguments
  std::vector<std::pair<std::string, ExprP>> kw;  // keyword arguments
  bool neg = false;                               // TEST: `is not`
};
ExprP mk(Expr::Kind k) {
  auto e = std::make_shared<Expr>();
  e->k = k;
  return e;
}

struct Tk {
  enum K { NAME, STR, INT, OP, END } k = END;
  std::string v;
  int64_t i = 0;
};

void put_cp(uint32_t cp, std::string* s) {
  if (cp < 0x80) {
    *s += (char)cp;
  } else if (cp < 0x800) {
    *s += (char)(0xC0 | (cp >> 6));
    *s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    *s += (char)(0xE0 | (cp >> 12));
    *s += (char)(0x80 | ((cp >> 6) & 0x3F));
    *s += (char)(0x80 | (cp & 0x3F));
  } else {
    *s += (char)(0xF0 | (cp >> 18));
    *s += (char)(0x80 | ((cp >> 12) & 0x3F));
    *s += (char)(0x80 | ((cp >> 6) & 0x3F));
    *s += (char)(0x80 | (cp & 0x3F));
  }
}

// one string literal starting at s[p] (a quote); returns the index after it
size_t lex_string(const std::string& s, size_t p, std::string* out) {
  const char q = s[p];
  size_t k = p + 1;
  auto hex4 = [&](size_t at) {
    if (at + 4 > s.size()) bad("truncated \\u escape");
    uint32_t v = 0;
    for (size_t j = at; j < at + 4; ++j) {
      const char c = s[j];
      if (!isxdigit((unsigned char)c)) bad("bad \\u escape");
      v = v * 16 + (uint32_t)(isdigit((unsigned char)c) ? c - '0' : (tolower(c) - 'a' + 10));
    }
    return v;
  };
  for (; k < s.size() && s[k] != q; ++k) {
    if (s[k] != '\\') { *out += s[k]; continue; }
    if (++k >= s.size()) break;
    switch (s[k]) {
      case 'n': *out += '\n'; break;
      case 't': *out += '\t'; break;
      case 'r': *out += '\r'; break;
      case 'b': *out += '\b'; break;
      case 'f': *out += '\f'; break;
      case '\\': case '\'': case '"': case '/': *out += s[k]; break;
      case 'u': {
        uint32_t cp = hex4(k + 1);
        k += 4;
        if (cp >= 0xD800 && cp < 0xDC00) {  // a surrogate pair: \uD8xx\uDCxx
          if (k + 2 >= s.size() || s[k + 1] != '\\' || s[k + 2] != 'u') bad("unpaired surrogate in \\u escape");
          const uint32_t lo = hex4(k + 3);
          if (lo < 0xDC00 || lo > 0xDFFF) bad("unpaired surrogate in \\u escape");
          cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          k += 6;
        } else if (cp >= 0xDC00 && cp < 0xE000) {
          bad("unpaired surrogate in \\u escape");
        }
        put_cp(cp, out);
        break;
      }
      default: bad(std::string("invalid escape \\") + s[k]);
    }
  }
  if (k >= s.size()) bad("unterminated string literal");
  return k + 1;
}

std::vector<Tk> lex(const std::string& s) {
  std::vector<Tk> out;
  size_t p = 0;
  while (p < s.size()) {
    const unsigned char c = (unsigned char)s[p];
    if (c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v') { ++p; continue; }
    Tk t;
    if (isalpha(c) || c == '_') {
      size_t q = p;
      while (q < s.size() && (isalnum((unsigned char)s[q]) || s[q] == '_')) ++q;
      t.k = Tk::NAME;
      t.v = s.substr(p, q - p);
      p = q;
    } else if (isdigit(c)) {
      size_t q = p;
      int64_t v = 0;
      for (; q < s.size() && (isdigit((unsigned char)s[q]) || s[q] == '_'); ++q) {
        if (s[q] == '_') continue;
        if (v > (INT64_MAX - (s[q] - '0')) / 10) unsup("an integer literal beyond 64 bits");
        v = v * 10 + (s[q] - '0');
      }
      if (q + 1 < s.size() && (s[q] == '.' || s[q] == 'e' || s[q] == 'E') &&
          (isdigit((unsigned char)s[q + 1]) || s[q + 1] == '-' || s[q + 1] == '+'))
        unsup("floating-point literals");
      t.k = Tk::INT;
      t.i = v;
      p = q;
    } else if (c == '\'' || c == '"') {
      t.k = Tk::STR;
      p = lex_string(s, p, &t.v);
    } else {
      static const char* two[] = {"==", "!=", "<=", ">=", "//", "**"};
      t.k = Tk::OP;
      for (const char* o : two)
        if (s.compare(p, 2, o) == 0) t.v = o;
      if (t.v.empty()) {
        if (c == 0 || !strchr("+-*/%~<>=()[]{},.:|", (char)c)) bad(std::string("unexpected character '") + (char)c + "'");
        t.v = std::string(1, (char)c);
      }
      p += t.v.size();
    }
    out.push_back(std::move(t));
  }
  out.push_back(Tk{});
  return out;
}

// Jinja's expression grammar, loosest binding first: `x if c else y`, or,
// and, not, comparisons / in / not in, + -, ~, * / // %, **, unary minus,
// then a primary with its postfix subscripts and calls, filters and tests.
// Nesting limits keep the recursive parser, evaluator and block runner
// within about 1 MiB of stack whatever the template holds (they run on a
// thread of their own with 8 MiB, run_on_own_stack).
constexpr int kMaxNest = 500;     // nested sub-expressions (a parenthesised level counts two)
constexpr int kMaxEval = 1000;    // expression tree depth when evaluated (long filter or operator chains)
constexpr int kMaxBlocks = 200;   // nested for / if blocks

class Parser {
 public:
  explicit Parser(std::vector<Tk> t) : t_(std::move(t)) {}
  ExprP expr() { return cond_(); }
  ExprP or_expr() { return or_(); }
  bool at_end() const { return t_[p_].k == Tk::END; }
  bool kw(const char* w, size_t ahead = 0) const {
    const Tk& x = peek(ahead);
    return x.k == Tk::NAME && x.v == w;
  }
  bool op(const char* o) const { return t_[p_].k == Tk::OP && t_[p_].v == o; }
  const Tk& peek(size_t ahead = 0) const { return t_[std::min(p_ + ahead, t_.size() - 1)]; }
  void skip() { ++p_; }
  std::string name() {
    if (peek().k != Tk::NAME) bad("expected a name");
    return t_[p_++].v;
  }
  void expect(const char* o) {
    if (!op(o)) bad(std::string("expected '") + o + "'");
    ++p_;
  }
  void end() {
    if (!at_end()) bad("unexpected '" + (peek().k == Tk::INT ? std::to_string(peek().i) : peek().v) + "'");
  }

 private:
  std::vector<Tk> t_;
  size_t p_ = 0;
  int depth_ = 0;
  struct Nest {
    int* d;
    explicit Nest(int* depth) : d(depth) {
      if (++*d > kMaxNest) bad("expression nested too deeply");
    }
    ~Nest() { --*d; }
  };

  ExprP bin(const std::string& o, ExprP l, ExprP r) {
    auto e = mk(Expr::BIN);
    e->name = o;
    e->a = {std::move(l), std::move(r)};
    return e;
  }
  ExprP cond_() {
    Nest guard(&depth_);
    ExprP e = or_();
    while (kw("if")) {
      ++p_;
      auto c = mk(Expr::COND);
      ExprP test = or_();
      ExprP alt;
      if (kw("else")) { ++p_; alt = cond_(); }
      c->a = {std::move(test), std::move(e), std::move(alt)};
      e = c;
    }
    return e;
  }
  ExprP or_() {
    ExprP e = and_();
    while (kw("or")) { ++p_; e = bin("or", e, and_()); }
    return e;
  }
  ExprP and_() {
    ExprP e = not_();
    while (kw("and")) { ++p_; e = bin("and", e, not_()); }
    return e;
  }
  ExprP not_() {
    if (kw("not")) {
      Nest guard(&depth_);
      ++p_;
      auto e = mk(Expr::NOT);
      e->a = {not_()};
      return e;
    }
    return compare_();
  }
  ExprP compare_() {
    ExprP e = math1_();
    for (;;) {
      std::string o;
      if (op("==") || op("!=") || op("<") || op(">") || op("<=") || op(">=")) o = t_[p_++].v;
      else if (kw("in")) { ++p_; o = "in"; }
      else if (kw("not") && kw("in", 1)) { p_ += 2; o = "not in"; }
      else return e;
      e = bin(o, e, math1_());
    }
  }
  ExprP math1_() {
    ExprP e = concat_();
    while (op("+") || op("-")) { const std::string o = t_[p_++].v; e = bin(o, e, concat_()); }
    return e;
  }
  ExprP concat_() {
    ExprP e = math2_();
    while (op("~")) { ++p_; e = bin("~", e, math2_()); }
    return e;
  }
  ExprP math2_() {
    ExprP e = pow_();
    while (op("*") || op("/") || op("//") || op("%")) { const std::string o = t_[p_++].v; e = bin(o, e, pow_()); }
    return e;
  }
  ExprP pow_() {
    ExprP e = unary_(true);
    while (op("**")) { ++p_; e = bin("**", e, unary_(true)); }
    return e;
  }
  ExprP unary_(bool with_filter) {
    Nest guard(&depth_);
    ExprP e;
    if (op("-")) {
      ++p_;
      e = mk(Expr::NEG);
      e->a = {unary_(false)};
    } else if (op("+")) {
      ++p_;
      e = unary_(false);
    } else {
      e = primary_();
    }
    e = postfix_(e);
    if (with_filter) e = filters_(e);
    return e;
  }
  ExprP primary_() {
    const Tk& k = peek();
    if (k.k == Tk::NAME) {
      ++p_;
      auto e = mk(Expr::CONST);
      if (k.v == "true" || k.v == "True") e->c = v_bool(true);
      else if (k.v == "false" || k.v == "False") e->c = v_bool(false);
      else if (k.v == "none" || k.v == "None") e->c = v_none();
      else { e->k = Expr::NAME; e->name = k.v; }
      return e;
    }
    if (k.k == Tk::STR) {
      std::string s;
      while (peek().k == Tk::STR) s += t_[p_++].v;  // adjacent literals concatenate
      auto e = mk(Expr::CONST);
      e->c = v_str(s);
      return e;
    }
    if (k.k == Tk::INT) {
      ++p_;
      auto e = mk(Expr::CONST);
      e->c = v_int(k.i);
      return e;
    }
    if (op("(")) {
      ++p_;
      if (op(")")) { ++p_; return mk(Expr::LIST); }  // ()
      ExprP e = cond_();
      if (op(",")) {  // a tuple, a list here
        auto l = mk(Expr::LIST);
        l->a.push_back(e);
        while (op(",")) {
          ++p_;
          if (op(")")) break;
          l->a.push_back(cond_());
        }
        e = l;
      }
      expect(")");
      return e;
    }
    if (op("[")) {
      ++p_;
      auto l = mk(Expr::LIST);
      while (!op("]")) {
        l->a.push_back(cond_());
        if (!op(",")) break;
        ++p_;
      }
      expect("]");
      return l;
    }
    if (op("{")) {
      ++p_;
      auto m = mk(Expr::MAP);
      while (!op("}")) {
        m->a.push_back(cond_());
        expect(":");
        m->a.push_back(cond_());
        if (!op(",")) break;
        ++p_;
      }
      expect("}");
      return m;
    }
    if (k.k == Tk::END) bad("unexpected end of expression");
    bad("unexpected '" + k.v + "'");
  }
  void call_args_(Expr* e) {  // after '('
    while (!op(")")) {
      if (peek().k == Tk::NAME && peek(1).k == Tk::OP && peek(1).v == "=") {
        const std::string n = t_[p_].v;
        p_ += 2;
        e->kw.push_back({n, cond_()});
      } else {
        if (!e->kw.empty()) bad("positional argument after a keyword argument");
        e->a.push_back(cond_());
      }
      if (!op(",")) break;
      ++p_;
    }
    expect(")");
  }
  ExprP postfix_(ExprP e) {
    for (;;) {
      if (op(".")) {
        ++p_;
        if (peek().k == Tk::NAME) {
          auto n = mk(Expr::ATTR);
          n->name = t_[p_++].v;
          n->a = {e};
          e = n;
        } else if (peek().k == Tk::INT) {
          auto n = mk(Expr::ITEM);
          auto idx = mk(Expr::CONST);
          idx->c = v_int(t_[p_++].i);
          n->a = {e, idx};
          e = n;
        } else {
          bad("expected a name after '.'");
        }
      } else if (op("[")) {
        ++p_;
        ExprP lo, hi, step;
        bool slice = false;
        if (!op(":")) lo = cond_();
        if (op(":")) {
          slice = true;
          ++p_;
          if (!op("]") && !op(":")) hi = cond_();
          if (op(":")) {
            ++p_;
            if (!op("]")) step = cond_();
          }
        }
        if (op(",")) unsup("tuple subscripts");
        expect("]");
        auto n = mk(slice ? Expr::SLICE : Expr::ITEM);
        n->a = slice ? std::vector<ExprP>{e, lo, hi, step} : std::vector<ExprP>{e, lo};
        e = n;
      } else if (op("(")) {
        ++p_;
        auto n = mk(Expr::CALL);
        n->a = {e};
        call_args_(n.get());
        e = n;
      } else {
        return e;
      }
    }
  }
  ExprP filters_(ExprP e) {
    for (;;) {
      if (op("|")) {
        ++p_;
        auto n = mk(Expr::FILTER);
        n->name = name();
        n->a = {e};
        if (op("(")) { ++p_; call_args_(n.get()); }
        e = n;
      } else if (kw("is")) {
        ++p_;
        auto n = mk(Expr::TEST);
        if (kw("not")) { ++p_; n->neg = true; }
        n->name = name();
        n->a = {e};
        if (op("(")) {
          ++p_;
          call_args_(n.get());
        } else if ((peek().k == Tk::NAME && !kw("else") && !kw("or") && !kw("and")) || peek().k == Tk::STR ||
                   peek().k == Tk::INT || op("[") || op("{")) {
          if (kw("is")) bad("tests cannot be chained with 'is'");
          n->a.push_back(postfix_(primary_()));  // `is divisibleby 3`, `is equalto 'x'`
        }
        e = n;
      } else if (op("(")) {
        ++p_;
        auto n = mk(Expr::CALL);
        n->a = {e};
        call_args_(n.get());
        e = n;
      } else {
        return e;
      }
    }
  }
};

// ---------------------------------------------------------- template AST --

struct Node;
using NodeP = std::shared_ptr<Node>;
using Body = std::vector<NodeP>;
struct Node {
  enum Kind { TEXT, OUT, FOR, IF, SET, SET_ATTR } k;
  std::string text;                              // TEXT
  ExprP e;                                       // OUT; SET value; FOR iterable
  std::vector<std::string> targets;              // FOR targets; SET {name}; SET_ATTR {name, attribute}
  ExprP filter;                                  // FOR ... if filter
  Body body, else_body;                          // FOR
  std::vector<std::pair<ExprP, Body>> branches;  // IF (a null condition: else)
};

struct Piece {
  enum Kind { TEXT, VAR, STMT } k;
  std::string s;
};

// Splits template source into text, {{ }} and {% %} pieces (comments
// dropped), applying the whitespace-control markers.
std::vector<Piece> split_template(std::string src) {
  if (src.size() >= 2 && src.compare(src.size() - 2, 2, "\r\n") == 0) src.resize(src.size() - 2);
  else if (!src.empty() && src.back() == '\n') src.pop_back();
  std::vector<Piece> out;
  size_t p = 0;
  bool lstrip_next = false;
  for (;;) {
    size_t open = p;
    for (;; ++open) {
      open = src.find('{', open);
      if (open == std::string::npos || open + 1 >= src.size()) { open = std::string::npos; break; }
      const char c = src[open + 1];
      if (c == '{' || c == '%' || c == '#') break;
    }
    std::string text = src.substr(p, (open == std::string::npos ? src.size() : open) - p);
    if (lstrip_next) text = trim_ws(text, true, false);
    lstrip_next = false;
    if (open == std::string::npos) {
      if (!text.empty()) out.push_back({Piece::TEXT, text});
      return out;
    }
    const char kind = src[open + 1];
    size_t j = open + 2;
    if (j < src.size() && src[j] == '-') { text = trim_ws(text, false, true); ++j; }
    else if (j < src.size() && src[j] == '+') ++j;
    if (!text.empty()) out.push_back({Piece::TEXT, text});
    size_t end;
    if (kind == '#') {
      end = src.find("#}", j);
      if (end == std::string::npos) bad("unterminated comment");
    } else {  // the closing delimiter, outside string literals
      const char* close = kind == '{' ? "}}" : "%}";
      end = j;
      for (;;) {
        if (end >= src.size()) bad(kind == '{' ? "unterminated '{{'" : "unterminated '{%'");
        if (src[end] == '\'' || src[end] == '"') {
          std::string ignored;
          end = lex_string(src, end, &ignored);
          continue;
        }
        if (src.compare(end, 2, close) == 0) break;
        ++end;
      }
    }
    std::string inner = src.substr(j, end - j);
    if (!inner.empty() && inner.back() == '-') { inner.pop_back(); lstrip_next = true; }
    else if (!inner.empty() && inner.back() == '+') inner.pop_back();
    p = end + 2;
    if (kind == '%' && trim_ws(inner, true, true) == "raw") {
      // {% raw %}: the text up to the next {% endraw %} is literal
      size_t e = p, e_end = std::string::npos;
      bool e_lstrip = false, e_rstrip = false;
      while ((e = src.find("{%", e)) != std::string::npos) {
        size_t k = e + 2;
        const bool ls = k < src.size() && src[k] == '-';
        if (k < src.size() && (src[k] == '-' || src[k] == '+')) ++k;
        const size_t c = src.find("%}", k);
        if (c == std::string::npos) break;
        std::string w = src.substr(k, c - k);
        const bool rs = !w.empty() && w.back() == '-';
        if (!w.empty() && (w.back() == '-' || w.back() == '+')) w.pop_back();
        if (trim_ws(w, true, true) == "endraw") {
          e_end = c + 2;
          e_lstrip = ls;
          e_rstrip = rs;
          break;
        }
        e += 2;
      }
      if (e_end == std::string::npos) bad("missing endraw");
      std::string body = src.substr(p, e - p);
      if (lstrip_next) body = trim_ws(body, true, false);
      if (e_lstrip) body = trim_ws(body, false, true);
      if (!body.empty()) out.push_back({Piece::TEXT, body});
      lstrip_next = e_rstrip;
      p = e_end;
      continue;
    }
    if (kind == '{') out.push_back({Piece::VAR, inner});
    else if (kind == '%') out.push_back({Piece::STMT, inner});
  }
}

// Parses pieces from ps[*i] into *body until one of `stops`; returns the stop
// keyword met ("" at the end of the pieces) and hands its statement's parser
// to *stop_p.
std::string parse_body(const std::vector<Piece>& ps, size_t* i, const std::vector<std::string>& stops, Body* body,
                       std::unique_ptr<Parser>* stop_p, int depth = 0) {
  if (depth > kMaxBlocks) bad("blocks nested too deeply");
  static const char* kUnsupported[] = {"macro", "endmacro", "call", "endcall", "filter", "endfilter", "with",
                                       "endwith", "include", "import", "from", "extends", "block",
                                       "endblock", "autoescape", "endautoescape", "do", "break", "continue",
                                       "endset"};
  while (*i < ps.size()) {
    const Piece& pc = ps[(*i)++];
    if (pc.k == Piece::TEXT) {
      auto n = std::make_shared<Node>();
      n->k = Node::TEXT;
      n->text = pc.s;
      body->push_back(n);
      continue;
    }
    auto owned = std::make_unique<Parser>(lex(pc.s));
    Parser& P = *owned;
    if (pc.k == Piece::VAR) {
      auto n = std::make_shared<Node>();
      n->k = Node::OUT;
      n->e = P.expr();
      P.end();
      body->push_back(n);
      continue;
    }
    const std::string word = P.name();
    for (const auto& s : stops)
      if (word == s) {
        if (stop_p) *stop_p = std::move(owned);
        else P.end();
        return word;
      }
    auto n = std::make_shared<Node>();
    if (word == "for") {
      n->k = Node::FOR;
      n->targets.push_back(P.name());
      while (P.op(",")) { P.skip(); n->targets.push_back(P.name()); }
      if (!P.kw("in")) bad("expected 'in' in a for statement");
      P.skip();
      n->e = P.or_expr();
      if (P.kw("if")) { P.skip(); n->filter = P.expr(); }
      if (P.kw("recursive")) unsup("recursive loops");
      P.end();
      const std::string w = parse_body(ps, i, {"endfor", "else"}, &n->body, nullptr, depth + 1);
      if (w.empty()) bad("missing endfor");
      if (w == "else" && parse_body(ps, i, {"endfor"}, &n->else_body, nullptr, depth + 1) != "endfor")
        bad("missing endfor");
    } else if (word == "if") {
      n->k = Node::IF;
      ExprP cond = P.expr();
      P.end();
      for (;;) {
        Body b;
        std::unique_ptr<Parser> sp;
        const std::string w = parse_body(ps, i, {"elif", "else", "endif"}, &b, &sp, depth + 1);
        if (w.empty()) bad("missing endif");
        n->branches.push_back({cond, std::move(b)});
        if (w == "endif") { sp->end(); break; }
        if (w == "elif") { cond = sp->expr(); sp->end(); continue; }
        sp->end();
        Body eb;
        if (parse_body(ps, i, {"endif"}, &eb, nullptr, depth + 1) != "endif") bad("missing endif");
        n->branches.push_back({nullptr, std::move(eb)});
        break;
      }
    } else if (word == "set") {
      const std::string target = P.name();
      if (P.op(".")) {
        P.skip();
        n->k = Node::SET_ATTR;
        n->targets = {target, P.name()};
      } else {
        n->k = Node::SET;
        n->targets = {target};
      }
      if (P.op(",")) unsup("set with several targets");
      if (P.at_end()) unsup("block set");
      P.expect("=");
      n->e = P.expr();
      P.end();
    } else {
      for (const char* u : kUnsupported)
        if (word == u) unsup("the '" + word + "' statement");
      if (word == "endfor" || word == "endif" || word == "elif" || word == "else") bad("unexpected '" + word + "'");
      bad("unknown statement '" + word + "'");
    }
    body->push_back(n);
  }
  return "";
}

// -------------------------------------------------------------- evaluation --

struct Ctx {
  std::vector<std::unordered_map<std::string, Val>> frames;
  int depth = 0;  // eval recursion
  Val lookup(const std::string& n) const {
    for (auto it = frames.rbegin(); it != frames.rend(); ++it) {
      auto f = it->find(n);
      if (f != it->end()) return f->second;
    }
    return Val();
  }
};

Val eval(const Expr& e, Ctx& c);
bool run_test(const std::string& name, const Val& v, const std::vector<Val>& args);

Val get_attr(const Val& v, const std::string& name) {
  if (v.k == Val::UNDEF) bad("attribute '" + name + "' of an undefined value");
  if (v.k == Val::MAP) {
    const Val* r = map_find(*v.m, name);
    return r ? *r : Val();
  }
  return Val();
}

Val get_item(const Val& v, const Val& key) {
  if (v.k == Val::UNDEF) bad("subscript of an undefined value");
  if (v.k == Val::MAP) {
    if (key.k != Val::STR) return Val();
    const Val* r = map_find(*v.m, key.s);
    return r ? *r : Val();
  }
  if ((v.k == Val::LIST || v.k == Val::STR) && key.k == Val::INT) {
    if (v.k == Val::LIST) {
      const int64_t n = (int64_t)v.l->size(), q = key.i < 0 ? key.i + n : key.i;
      return q >= 0 && q < n ? (*v.l)[q] : Val();
    }
    const std::vector<size_t> o = cp_offsets(v.s);
    const int64_t n = (int64_t)o.size() - 1, q = key.i < 0 ? key.i + n : key.i;
    return q >= 0 && q < n ? v_str(v.s.substr(o[q], o[q + 1] - o[q])) : Val();
  }
  return Val();
}

Val slice(const Val& v, const Val* lo, const Val* hi, const Val* st) {
  if (v.k == Val::UNDEF) bad("slice of an undefined value");
  if (v.k != Val::LIST && v.k != Val::STR) bad(std::string("cannot slice a ") + kind_name(v));
  const ValList items = v.k == Val::LIST ? *v.l : chars_of(v.s);
  const int64_t n = (int64_t)items.size();
  auto as_int = [](const Val* x) -> const Val* {
    if (x && x->k != Val::NONE && x->k != Val::UNDEF && x->k != Val::INT) bad("slice bounds must be integers");
    return x && x->k == Val::INT ? x : nullptr;
  };
  const Val *a = as_int(lo), *b = as_int(hi), *s = as_int(st);
  const int64_t step = s ? s->i : 1;
  if (step == 0) bad("slice step cannot be zero");
  const int64_t lower = step > 0 ? 0 : -1, upper = step > 0 ? n : n - 1;  // Python's slice.indices
  auto norm = [&](const Val* x, int64_t dflt) {
    if (!x) return dflt;
    const int64_t q = x->i < 0 ? x->i + n : x->i;
    return q < lower ? lower : q > upper ? upper : q;
  };
  const int64_t from = norm(a, step > 0 ? lower : upper), to = norm(b, step > 0 ? upper : lower);
  ValList out;
  for (int64_t q = from; step > 0 ? q < to : q > to; q += step) out.push_back(items[q]);
  if (v.k == Val::LIST) return v_list(std::move(out));
  std::string r;
  for (const Val& x : out) r += x.s;
  return v_str(r);
}

std::string case_map(const std::string& s, int mode) {  // 0 lower, 1 upper, 2 capitalize
  for (unsigned char ch : s)
    if (ch >= 0x80) unsup("case mapping of non-ASCII text");
  std::string r = s;
  for (size_t q = 0; q < r.size(); ++q) {
    const bool up = mode == 1 || (mode == 2 && q == 0);
    r[q] = up ? (char)toupper((unsigned char)r[q]) : (char)tolower((unsigned char)r[q]);
  }
  return r;
}

void no_overflow(bool overflow) {
  if (overflow) bad("integer overflow");
}

Val arith(const std::string& o, const Val& l, const Val& r) {
  if (l.k == Val::UNDEF || r.k == Val::UNDEF) bad("undefined value in '" + o + "'");
  if (o == "/") unsup("true division (floating point)");
  if (o == "+") {
    if (l.k == Val::STR && r.k == Val::STR) return v_str(l.s + r.s);
    if (l.k == Val::LIST && r.k == Val::LIST) {
      ValList x = *l.l;
      x.insert(x.end(), r.l->begin(), r.l->end());
      return v_list(std::move(x));
    }
  }
  if (o == "*" && ((l.k == Val::STR && r.k == Val::INT) || (l.k == Val::INT && r.k == Val::STR))) {
    const std::string& s = l.k == Val::STR ? l.s : r.s;
    const int64_t n = l.k == Val::INT ? l.i : r.i;
    if (n > 0 && s.size() * (uint64_t)n > (64u << 20)) bad("string repetition too large");
    std::string out;
    for (int64_t q = 0; q < n; ++q) out += s;
    return v_str(out);
  }
  if (l.k != Val::INT || r.k != Val::INT) bad("'" + o + "' on " + kind_name(l) + " and " + kind_name(r));
  const int64_t a = l.i, b = r.i;
  int64_t v;
  if (o == "+") { no_overflow(__builtin_add_overflow(a, b, &v)); return v_int(v); }
  if (o == "-") { no_overflow(__builtin_sub_overflow(a, b, &v)); return v_int(v); }
  if (o == "*") { no_overflow(__builtin_mul_overflow(a, b, &v)); return v_int(v); }
  if (o == "//" || o == "%") {
    if (b == 0) bad("division by zero");
    if (a == INT64_MIN && b == -1) bad("integer overflow");
    int64_t q = a / b, m = a % b;
    if (m != 0 && ((m < 0) != (b < 0))) { --q; m += b; }  // floor division, Python's sign rule
    return v_int(o == "//" ? q : m);
  }
  if (o == "**") {
    if (b < 0) unsup("negative powers (floating point)");
    int64_t acc = 1;
    for (int64_t q = 0; q < b && acc != 0; ++q) {
      no_overflow(__builtin_mul_overflow(acc, a, &v));
      acc = v;
    }
    return v_int(acc);
  }
  bad("unknown operator " + o);
}

// minijinja builtin filters this renderer does not implement
const char* kKnownFilters[] = {"attr", "batch", "bool", "dictsort", "escape", "e", "float", "format", "groupby",
                               "indent", "int", "lines", "max", "min", "pprint", "round", "slice", "sort", "split",
                               "sum", "title", "tojson", "unique", "urlencode", "wordcount", "chain", "zip"};

Val apply_filter(const std::string& f, const Val& v, const std::vector<Val>& args,
                 const std::vector<std::pair<std::string, Val>>& kw) {
  auto arg = [&](size_t q, const char* key) -> const Val* {
    if (q < args.size()) return &args[q];
    for (const auto& x : kw)
      if (x.first == key) return &x.second;
    return nullptr;
  };
  if (f == "trim") {
    const Val* chars = arg(0, "chars");
    if (!chars || chars->k == Val::NONE || chars->k == Val::UNDEF) return v_str(trim_ws(to_text(v), true, true));
    const ValList cs = chars_of(to_text(*chars)), all = chars_of(to_text(v));
    auto in_set = [&](const Val& ch) {
      for (const Val& x : cs)
        if (x.s == ch.s) return true;
      return false;
    };
    size_t a = 0, b = all.size();
    while (a < b && in_set(all[a])) ++a;
    while (b > a && in_set(all[b - 1])) --b;
    std::string r;
    for (size_t q = a; q < b; ++q) r += all[q].s;
    return v_str(r);
  }
  if (f == "length" || f == "count") {
    if (v.k == Val::STR) return v_int((int64_t)cp_offsets(v.s).size() - 1);
    if (v.k == Val::LIST) return v_int((int64_t)v.l->size());
    if (v.k == Val::MAP) return v_int((int64_t)v.m->size());
    bad(std::string("length of a ") + kind_name(v));
  }
  if (f == "lower") return v_str(case_map(to_text(v), 0));
  if (f == "upper") return v_str(case_map(to_text(v), 1));
  if (f == "capitalize") return v_str(case_map(to_text(v), 2));
  if (f == "string") return v.k == Val::STR ? v : v_str(to_text(v));
  if (f == "safe") return v;
  if (f == "default" || f == "d") {
    const Val* dv = arg(0, "default_value");
    const Val* bo = arg(1, "boolean");
    const bool use = v.k == Val::UNDEF || (bo && truthy(*bo) && !truthy(v));
    return use ? (dv ? *dv : v_str("")) : v;
  }
  if (f == "first" || f == "last") {
    if (v.k == Val::UNDEF) return Val();
    if (v.k != Val::LIST && v.k != Val::STR) bad(f + " of a " + kind_name(v));
    const ValList items = v.k == Val::LIST ? *v.l : chars_of(v.s);
    if (items.empty()) return Val();
    return f == "first" ? items.front() : items.back();
  }
  if (f == "join") {
    const Val* sep = arg(0, "d");
    if (arg(1, "attribute")) unsup("join with an attribute");
    const std::string d = sep ? to_text(*sep) : "";
    std::string r;
    bool first = true;
    for (const Val& x : iterate(v)) {
      if (!first) r += d;
      r += to_text(x);
      first = false;
    }
    return v_str(r);
  }
  if (f == "list") return v_list(iterate(v));
  if (f == "reverse") {
    if (v.k != Val::LIST && v.k != Val::STR) bad(std::string("reverse of a ") + kind_name(v));
    ValList items = v.k == Val::LIST ? *v.l : chars_of(v.s);
    std::reverse(items.begin(), items.end());
    if (v.k == Val::LIST) return v_list(std::move(items));
    std::string r;
    for (const Val& x : items) r += x.s;
    return v_str(r);
  }
  if (f == "replace") {
    const Val *from = arg(0, "old"), *to = arg(1, "new");
    if (!from || !to) bad("replace needs two arguments");
    if (arg(2, "count")) unsup("replace with a count");
    const std::string s = to_text(v), a = to_text(*from), b = to_text(*to);
    if (a.empty()) unsup("replace of the empty string");
    std::string r;
    size_t q = 0;
    for (size_t h; (h = s.find(a, q)) != std::string::npos; q = h + a.size()) r += s.substr(q, h - q) + b;
    return v_str(r + s.substr(q));
  }
  if (f == "abs") {
    if (v.k != Val::INT) bad(std::string("abs of a ") + kind_name(v));
    if (v.i == INT64_MIN) bad("integer overflow");
    return v_int(v.i < 0 ? -v.i : v.i);
  }
  if (f == "items") {
    if (v.k == Val::UNDEF) return v_list();
    if (v.k != Val::MAP) bad(std::string("items of a ") + kind_name(v));
    ValList out;
    for (const auto& kv : *v.m) out.push_back(v_list({v_str(kv.first), kv.second}));
    return v_list(std::move(out));
  }
  if (f == "select" || f == "reject" || f == "selectattr" || f == "rejectattr") {
    const bool attr = f == "selectattr" || f == "rejectattr", keep = f == "select" || f == "selectattr";
    if (!kw.empty()) unsup(f + " with keyword arguments");
    size_t q = 0;
    std::string attr_name;
    if (attr) {
      if (args.empty()) bad(f + " needs an attribute name");
      attr_name = to_text(args[q++]);
    }
    std::string test;
    if (q < args.size()) test = to_text(args[q++]);
    const std::vector<Val> targs(args.begin() + (ptrdiff_t)q, args.end());
    ValList out;
    for (const Val& x : iterate(v)) {
      const Val probe = attr ? get_attr(x, attr_name) : x;
      const bool hit = test.empty() ? truthy(probe) : run_test(test, probe, targs);
      if (hit == keep) out.push_back(x);
    }
    return v_list(std::move(out));
  }
  if (f == "map") {
    for (const auto& x : kw)
      if (x.first != "attribute" && x.first != "default") unsup("map with keyword " + x.first);
    ValList out;
    const Val* at = nullptr;
    const Val* dflt = nullptr;
    for (const auto& x : kw) (x.first == "attribute" ? at : dflt) = &x.second;
    if (at) {
      for (const Val& x : iterate(v)) {
        Val r = get_attr(x, to_text(*at));
        out.push_back(r.k == Val::UNDEF && dflt ? *dflt : r);
      }
      return v_list(std::move(out));
    }
    if (args.empty()) bad("map needs a filter name or attribute=");
    const std::string fn = to_text(args[0]);
    const std::vector<Val> fargs(args.begin() + 1, args.end());
    for (const Val& x : iterate(v)) out.push_back(apply_filter(fn, x, fargs, {}));
    return v_list(std::move(out));
  }
  for (const char* k : kKnownFilters)
    if (f == k) unsup("the '" + f + "' filter");
  bad("unknown filter '" + f + "'");
}

bool run_test(const std::string& t, const Val& v, const std::vector<Val>& args) {
  auto need = [&](size_t n) {
    if (args.size() != n) bad("test '" + t + "' takes " + std::to_string(n) + " argument(s)");
  };
  if (t == "defined") return v.k != Val::UNDEF;
  if (t == "undefined") return v.k == Val::UNDEF;
  if (t == "none") return v.k == Val::NONE;
  if (t == "boolean") return v.k == Val::BOOL;
  if (t == "true") return v.k == Val::BOOL && v.b;
  if (t == "false") return v.k == Val::BOOL && !v.b;
  if (t == "integer" || t == "number") return v.k == Val::INT;
  if (t == "float") return false;
  if (t == "string") return v.k == Val::STR;
  if (t == "mapping") return v.k == Val::MAP;
  if (t == "sequence") return v.k == Val::LIST;
  if (t == "iterable") return v.k == Val::LIST || v.k == Val::STR || v.k == Val::MAP;
  if (t == "odd" || t == "even") {
    if (v.k != Val::INT) bad("test '" + t + "' of a " + kind_name(v));
    return (v.i % 2 != 0) == (t == "odd");
  }
  if (t == "divisibleby") {
    need(1);
    if (v.k != Val::INT || args[0].k != Val::INT) bad("divisibleby needs numbers");
    if (args[0].i == 0) bad("division by zero");
    return v.i % args[0].i == 0;
  }
  if (t == "eq" || t == "equalto" || t == "==") { need(1); return equal(v, args[0]); }
  if (t == "ne" || t == "!=") { need(1); return !equal(v, args[0]); }
  if (t == "lt" || t == "lessthan" || t == "<") { need(1); return order(v, args[0]) < 0; }
  if (t == "le" || t == "<=") { need(1); return order(v, args[0]) <= 0; }
  if (t == "gt" || t == "greaterthan" || t == ">") { need(1); return order(v, args[0]) > 0; }
  if (t == "ge" || t == ">=") { need(1); return order(v, args[0]) >= 0; }
  if (t == "in") { need(1); return contains(args[0], v); }
  if (t == "startingwith" || t == "endingwith") {
    need(1);
    if (v.k != Val::STR || args[0].k != Val::STR) return false;
    const std::string& s = v.s;
    const std::string& x = args[0].s;
    if (x.size() > s.size()) return false;
    return t == "startingwith" ? s.compare(0, x.size(), x) == 0 : s.compare(s.size() - x.size(), x.size(), x) == 0;
  }
  static const char* known[] = {"sameas", "lower", "upper", "safe", "escaped", "filter", "test"};
  for (const char* k : known)
    if (t == k) unsup("the '" + t + "' test");
  bad("unknown test '" + t + "'");
}

Val call(const Expr& e, Ctx& c) {
  const Expr& f = *e.a[0];
  std::vector<Val> args;
  for (size_t q = 1; q < e.a.size(); ++q) args.push_back(eval(*e.a[q], c));
  std::vector<std::pair<std::string, Val>> kw;
  for (const auto& x : e.kw) kw.push_back({x.first, eval(*x.second, c)});
  if (f.k == Expr::ATTR) {
    const Val obj = eval(*f.a[0], c);
    if (obj.k == Val::UNDEF) bad("method '" + f.name + "' of an undefined value");
    if (obj.tag == Val::LOOP && f.name == "cycle") {  // the argument at index0 modulo their count
      if (args.empty()) bad("loop.cycle needs arguments");
      return args[(size_t)map_find(*obj.m, "index0")->i % args.size()];
    }
    if (obj.tag == Val::LOOP && f.name == "changed") unsup("loop.changed");
    bad(std::string("unknown method ") + kind_name(obj) + "." + f.name + "()");
  }
  if (f.k == Expr::NAME && c.lookup(f.name).k == Val::UNDEF) {
    if (f.name == "range") {
      for (const Val& a : args)
        if (a.k != Val::INT) bad("range needs integers");
      if (args.empty() || args.size() > 3 || !kw.empty()) bad("range takes 1 to 3 arguments");
      const int64_t lo = args.size() > 1 ? args[0].i : 0, hi = args.size() > 1 ? args[1].i : args[0].i;
      const int64_t step = args.size() > 2 ? args[2].i : 1;
      if (step == 0) bad("range step cannot be zero");
      ValList out;
      for (int64_t q = lo; step > 0 ? q < hi : q > hi; q += step) {
        if (out.size() >= 100000) bad("range has too many elements");
        out.push_back(v_int(q));
      }
      return v_list(std::move(out));
    }
    if (f.name == "namespace" || f.name == "dict") {
      Val m = v_map();
      if (f.name == "namespace") m.tag = Val::NAMESPACE;
      for (const Val& a : args) {
        if (a.k != Val::MAP) bad(f.name + "() takes keyword arguments or a map");
        for (const auto& kv : *a.m) map_put(m.m.get(), kv.first, kv.second);
      }
      for (const auto& kv : kw) map_put(m.m.get(), kv.first, kv.second);
      return m;
    }
    if (f.name == "debug" || f.name == "cycler" || f.name == "joiner" || f.name == "lipsum")
      unsup("the '" + f.name + "' function");
    bad("unknown function '" + f.name + "'");
  }
  bad("value is not callable");
}

Val eval_node(const Expr& e, Ctx& c);

Val eval(const Expr& e, Ctx& c) {
  if (++c.depth > kMaxEval) bad("expression too deep to evaluate");
  Val v = eval_node(e, c);
  --c.depth;
  return v;
}

Val eval_node(const Expr& e, Ctx& c) {
  switch (e.k) {
    case Expr::CONST: return e.c;
    case Expr::NAME: return c.lookup(e.name);
    case Expr::LIST: {
      ValList l;
      for (const ExprP& x : e.a) l.push_back(eval(*x, c));
      return v_list(std::move(l));
    }
    case Expr::MAP: {
      Val m = v_map();
      for (size_t q = 0; q + 1 < e.a.size(); q += 2) {
        const Val key = eval(*e.a[q], c);
        if (key.k != Val::STR) unsup("map keys other than strings");
        map_put(m.m.get(), key.s, eval(*e.a[q + 1], c));
      }
      return m;
    }
    case Expr::ATTR: return get_attr(eval(*e.a[0], c), e.name);
    case Expr::ITEM: {
      const Val obj = eval(*e.a[0], c);
      return get_item(obj, eval(*e.a[1], c));
    }
    case Expr::SLICE: {
      const Val obj = eval(*e.a[0], c);
      Val b[3];
      const Val* p[3] = {nullptr, nullptr, nullptr};
      for (int q = 0; q < 3; ++q)
        if (e.a[q + 1]) { b[q] = eval(*e.a[q + 1], c); p[q] = &b[q]; }
      return slice(obj, p[0], p[1], p[2]);
    }
    case Expr::CALL: return call(e, c);
    case Expr::FILTER: {
      const Val v = eval(*e.a[0], c);
      std::vector<Val> args;
      for (size_t q = 1; q < e.a.size(); ++q) args.push_back(eval(*e.a[q], c));
      std::vector<std::pair<std::string, Val>> kw;
      for (const auto& x : e.kw) kw.push_back({x.first, eval(*x.second, c)});
      return apply_filter(e.name, v, args, kw);
    }
    case Expr::TEST: {
      const Val v = eval(*e.a[0], c);
      std::vector<Val> args;
      for (size_t q = 1; q < e.a.size(); ++q) args.push_back(eval(*e.a[q], c));
      if (!e.kw.empty()) unsup("tests with keyword arguments");
      return v_bool(run_test(e.name, v, args) != e.neg);
    }
    case Expr::NOT: return v_bool(!truthy(eval(*e.a[0], c)));
    case Expr::NEG: {
      const Val v = eval(*e.a[0], c);
      if (v.k != Val::INT) bad(std::string("unary minus of a ") + kind_name(v));
      if (v.i == INT64_MIN) bad("integer overflow");
      return v_int(-v.i);
    }
    case Expr::COND: return truthy(eval(*e.a[0], c)) ? eval(*e.a[1], c) : (e.a[2] ? eval(*e.a[2], c) : Val());
    case Expr::BIN: {
      const std::string& o = e.name;
      if (o == "and") {
        Val l = eval(*e.a[0], c);
        return truthy(l) ? eval(*e.a[1], c) : l;
      }
      if (o == "or") {
        Val l = eval(*e.a[0], c);
        return truthy(l) ? l : eval(*e.a[1], c);
      }
      const Val l = eval(*e.a[0], c), r = eval(*e.a[1], c);
      if (o == "~") return v_str(to_text(l) + to_text(r));
      if (o == "==") return v_bool(equal(l, r));
      if (o == "!=") return v_bool(!equal(l, r));
      if (o == "<") return v_bool(order(l, r) < 0);
      if (o == ">") return v_bool(order(l, r) > 0);
      if (o == "<=") return v_bool(order(l, r) <= 0);
      if (o == ">=") return v_bool(order(l, r) >= 0);
      if (o == "in") return v_bool(contains(r, l));
      if (o == "not in") return v_bool(!contains(r, l));
      return arith(o, l, r);
    }
  }
  return Val();
}

void bind(Ctx& c, const std::vector<std::string>& targets, const Val& item) {
  if (targets.size() == 1) {
    c.frames.back()[targets[0]] = item;
    return;
  }
  if (item.k != Val::LIST || item.l->size() != targets.size())
    bad(std::string("cannot unpack a ") + kind_name(item) + " into " + std::to_string(targets.size()) + " names");
  for (size_t q = 0; q < targets.size(); ++q) c.frames.back()[targets[q]] = (*item.l)[q];
}

void exec(const Body& body, Ctx& c, std::string* out) {
  for (const NodeP& np : body) {
    const Node& n = *np;
    switch (n.k) {
      case Node::TEXT: *out += n.text; break;
      case Node::OUT: *out += to_text(eval(*n.e, c)); break;
      case Node::SET: c.frames.back()[n.targets[0]] = eval(*n.e, c); break;
      case Node::SET_ATTR: {
        const Val ns = c.lookup(n.targets[0]);
        if (ns.k != Val::MAP || ns.tag != Val::NAMESPACE) bad("can only assign attributes of a namespace");
        map_put(ns.m.get(), n.targets[1], eval(*n.e, c));
        break;
      }
      case Node::IF:
        for (const auto& br : n.branches)
          if (!br.first || truthy(eval(*br.first, c))) {
            exec(br.second, c, out);
            break;
          }
        break;
      case Node::FOR: {
        ValList items = iterate(eval(*n.e, c));
        if (n.filter) {
          ValList kept;
          c.frames.emplace_back();
          for (const Val& x : items) {
            bind(c, n.targets, x);
            if (truthy(eval(*n.filter, c))) kept.push_back(x);
          }
          c.frames.pop_back();
          items.swap(kept);
        }
        if (items.empty()) {
          exec(n.else_body, c, out);
          break;
        }
        const int64_t depth = 1;  // loop.depth counts recursive-loop levels; a nested loop is not one
        const int64_t len = (int64_t)items.size();
        c.frames.emplace_back();  // one frame for the whole loop
        for (int64_t q = 0; q < len; ++q) {
          bind(c, n.targets, items[q]);
          Val loop = v_map({{"index", v_int(q + 1)},
                            {"index0", v_int(q)},
                            {"revindex", v_int(len - q)},
                            {"revindex0", v_int(len - q - 1)},
                            {"first", v_bool(q == 0)},
                            {"last", v_bool(q == len - 1)},
                            {"length", v_int(len)},
                            {"previtem", q > 0 ? items[q - 1] : Val()},
                            {"nextitem", q + 1 < len ? items[q + 1] : Val()},
                            {"depth", v_int(depth)},
                            {"depth0", v_int(depth - 1)}});
          loop.tag = Val::LOOP;
          c.frames.back()["loop"] = loop;
          exec(n.body, c, out);
        }
        c.frames.pop_back();
        break;
      }
    }
  }
}

}  // namespace

struct ChatTemplate {
  Body body;
};

namespace {

// Runs body (which throws TplError / bad_alloc on failure) on a thread with
// an 8 MiB stack, so the nesting limits above hold whatever stack the
// caller's thread has, and reports the outcome on the caller's thread (the
// last-error message is thread-local).
template <class Body>
int run_on_own_stack(Body&& body) {
  struct Job {
    Body* body = nullptr;
    int code = YL_OK;
    std::string msg;
  } job;
  job.body = &body;
  auto work = [](void* p) -> void* {
    Job* j = static_cast<Job*>(p);
    try {
      (*j->body)();
    } catch (const TplError& e) {
      j->code = e.code;
      j->msg = std::string("chat template: ") + e.what();
    } catch (const std::bad_alloc&) {
      j->code = YL_ERR_OOM;
      j->msg = "chat template: out of memory";
    }
    return nullptr;
  };
  pthread_attr_t attr;
  pthread_t th;
  bool started = pthread_attr_init(&attr) == 0;
  if (started) {
    started = pthread_attr_setstacksize(&attr, 8u << 20) == 0 && pthread_create(&th, &attr, work, &job) == 0;
    pthread_attr_destroy(&attr);
  }
  if (!started) return fail(YL_ERR_OOM, "chat template: cannot start the rendering thread");
  pthread_join(th, nullptr);
  return job.code == YL_OK ? YL_OK : fail(job.code, job.msg);
}

}  // namespace

int chat_template_parse(const std::string& src, std::shared_ptr<const ChatTemplate>* out) {
  std::vector<uint32_t> cps;
  if (!utf8_code_points(src, &cps, nullptr)) return fail(YL_ERR_FORMAT, "chat template: not UTF-8");
  auto t = std::make_shared<ChatTemplate>();
  const int rc = run_on_own_stack([&] {
    const std::vector<Piece> ps = split_template(src);
    size_t i = 0;
    parse_body(ps, &i, {}, &t->body, nullptr);
  });
  if (rc == YL_OK) *out = t;
  return rc;
}

int chat_template_render(const ChatTemplate& t, const ChatMessages& messages, bool add_generation_prompt,
                         std::string* out) {
  for (const auto& m : messages) {
    std::vector<uint32_t> cps;
    if (!utf8_code_points(m.first, &cps, nullptr) || !utf8_code_points(m.second, &cps, nullptr))
      return fail(YL_ERR_ARG, "chat message is not UTF-8");
  }
  std::string r;
  const int rc = run_on_own_stack([&] {
    ValList msgs;
    for (const auto& m : messages)  // serde_json's map keeps its keys sorted: content before role
      msgs.push_back(v_map({{"content", v_str(m.second)}, {"role", v_str(m.first)}}));
    Ctx c;
    c.frames.emplace_back();
    c.frames.back()["messages"] = v_list(std::move(msgs));
    c.frames.back()["add_generation_prompt"] = v_bool(add_generation_prompt);
    exec(t.body, c, &r);
  });
  if (rc == YL_OK) *out = std::move(r);
  return rc;
}

}  // namespace yl
