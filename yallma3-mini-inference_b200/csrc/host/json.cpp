// Recursive-descent JSON reader (RFC 8259): objects, arrays, strings with
// escapes (\uXXXX and surrogate pairs to UTF-8), numbers, literals.
#include "json.h"

#include <cstdlib>
#include <cstring>

namespace yl {

const Json* Json::get(const std::string& key) const {
  if (kind != OBJ) return nullptr;
  const Json* hit = nullptr;  // a repeated key: the last one wins, as in serde_json
  for (const auto& kv : obj)
    if (kv.first == key) hit = &kv.second;
  return hit;
}

bool Json::as_u64(uint64_t* out) const {
  if (kind != NUM || !is_u64) return false;
  *out = u;
  return true;
}

bool Json::as_f64(double* out) const {
  if (kind != NUM) return false;
  *out = num;
  return true;
}

const std::string* Json::as_str() const { return kind == STR ? &str : nullptr; }

namespace {

struct Parser {
  const char* p;
  size_t n, i = 0;
  std::string err;
  int depth = 0;

  bool fail(const char* what) {
    if (err.empty()) err = std::string(what) + " at byte " + std::to_string(i);
    return false;
  }
  void ws() {
    while (i < n && (p[i] == ' ' || p[i] == '\t' || p[i] == '\n' || p[i] == '\r')) ++i;
  }
  bool lit(const char* w) {
    const size_t k = strlen(w);
    if (n - i < k || memcmp(p + i, w, k) != 0) return fail("bad literal");
    i += k;
    return true;
  }
  static void utf8(uint32_t c, std::string* s) {
    if (c < 0x80) {
      s->push_back((char)c);
    } else if (c < 0x800) {
      s->push_back((char)(0xC0 | (c >> 6)));
      s->push_back((char)(0x80 | (c & 0x3F)));
    } else if (c < 0x10000) {
      s->push_back((char)(0xE0 | (c >> 12)));
      s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      s->push_back((char)(0x80 | (c & 0x3F)));
    } else {
      s->push_back((char)(0xF0 | (c >> 18)));
      s->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
      s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
      s->push_back((char)(0x80 | (c & 0x3F)));
    }
  }
  bool hex4(uint32_t* out) {
    if (n - i < 4) return fail("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = p[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    *out = v;
    return true;
  }
  bool string(std::string* s) {
    if (i >= n || p[i] != '"') return fail("expected string");
    ++i;
    while (true) {
      if (i >= n) return fail("unterminated string");
      const unsigned char c = (unsigned char)p[i++];
      if (c == '"') return true;
      if (c < 0x20) return fail("control character in string");
      if (c != '\\') {
        s->push_back((char)c);
        continue;
      }
      if (i >= n) return fail("unterminated escape");
      const char e = p[i++];
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t c1;
          if (!hex4(&c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // high surrogate: a low one must follow
            uint32_t c2;
            if (n - i < 2 || p[i] != '\\' || p[i + 1] != 'u') return fail("lone surrogate");
            i += 2;
            if (!hex4(&c2)) return false;
            if (c2 < 0xDC00 || c2 >= 0xE000) return fail("bad surrogate pair");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          } else if (c1 >= 0xDC00 && c1 < 0xE000) {
            return fail("lone surrogate");
          }
          utf8(c1, s);
          break;
        }
        default: return fail("bad escape");
      }
    }
  }
  bool number(Json* v) {
    const size_t b = i;
    bool integer = true, neg = false;
    if (i < n && p[i] == '-') { neg = true; ++i; }
    if (i >= n || !(p[i] >= '0' && p[i] <= '9')) return fail("bad number");
    if (p[i] == '0') ++i;
    else while (i < n && p[i] >= '0' && p[i] <= '9') ++i;
    if (i < n && p[i] == '.') {
      integer = false;
      ++i;
      if (i >= n || !(p[i] >= '0' && p[i] <= '9')) return fail("bad fraction");
      while (i < n && p[i] >= '0' && p[i] <= '9') ++i;
    }
    if (i < n && (p[i] == 'e' || p[i] == 'E')) {
      integer = false;
      ++i;
      if (i < n && (p[i] == '+' || p[i] == '-')) ++i;
      if (i >= n || !(p[i] >= '0' && p[i] <= '9')) return fail("bad exponent");
      while (i < n && p[i] >= '0' && p[i] <= '9') ++i;
    }
    const std::string tok(p + b, i - b);
    v->kind = Json::NUM;
    v->num = strtod(tok.c_str(), nullptr);  // correctly rounded
    if (integer && !neg) {
      uint64_t u = 0;
      bool fits = true;
      for (char c : tok) {
        const uint64_t d = (uint64_t)(c - '0');
        if (u > (UINT64_MAX - d) / 10) { fits = false; break; }
        u = u * 10 + d;
      }
      v->is_u64 = fits;
      v->u = fits ? u : 0;
    }
    return true;
  }
  bool value(Json* v) {
    ws();
    if (i >= n) return fail("unexpected end");
    if (++depth > 64) return fail("nesting too deep");
    bool ok = true;
    const char c = p[i];
    if (c == '{') {
      v->kind = Json::OBJ;
      ++i;
      ws();
      if (i < n && p[i] == '}') {
        ++i;
      } else {
        while (ok) {
          ws();
          std::pair<std::string, Json> kv;
          if (!(ok = string(&kv.first))) break;
          ws();
          if (i >= n || p[i] != ':') { ok = fail("expected ':'"); break; }
          ++i;
          if (!(ok = value(&kv.second))) break;
          v->obj.push_back(std::move(kv));
          ws();
          if (i < n && p[i] == ',') { ++i; continue; }
          if (i < n && p[i] == '}') { ++i; break; }
          ok = fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      v->kind = Json::ARR;
      ++i;
      ws();
      if (i < n && p[i] == ']') {
        ++i;
      } else {
        while (ok) {
          Json e;
          if (!(ok = value(&e))) break;
          v->arr.push_back(std::move(e));
          ws();
          if (i < n && p[i] == ',') { ++i; continue; }
          if (i < n && p[i] == ']') { ++i; break; }
          ok = fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      v->kind = Json::STR;
      ok = string(&v->str);
    } else if (c == 't') {
      v->kind = Json::BOOL;
      v->b = true;
      ok = lit("true");
    } else if (c == 'f') {
      v->kind = Json::BOOL;
      ok = lit("false");
    } else if (c == 'n') {
      ok = lit("null");
    } else {
      ok = number(v);
    }
    --depth;
    return ok;
  }
};

}  // namespace

bool json_parse(const char* text, size_t n, Json* out, std::string* err) {
  Parser ps;
  ps.p = text;
  ps.n = n;
  *out = Json();
  bool ok = ps.value(out);
  if (ok) {
    ps.ws();
    if (ps.i != n) ok = ps.fail("trailing characters");
  }
  if (!ok && err) *err = ps.err;
  return ok;
}

}  // namespace yl
