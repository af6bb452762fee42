// Byte-level BPE tokenizer of the reference (tokenizer.rs), restated in C++
// for the generation entry points. Same vocabulary tables, merge scores,
// pre-tokenizer split, greedy best-pair merge loop and byte-level decode.
#include "tokenizer.h"

#include <algorithm>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <sstream>

#include "chat_template.h"
#include "common.h"
#include "json.h"
#include "unicode_tables.h"
#include "upload.h"

namespace yl {

namespace {

// ---------------------------------------------------------------- UTF-8 --

void put_utf8(uint32_t cp, std::string* s) {
  if (cp < 0x80) {
    s->push_back((char)cp);
  } else if (cp < 0x800) {
    s->push_back((char)(0xC0 | (cp >> 6)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    s->push_back((char)(0xE0 | (cp >> 12)));
    s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    s->push_back((char)(0xF0 | (cp >> 18)));
    s->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  }
}

// Length of the well-formed UTF-8 sequence at s[i] (Unicode Table 3-7), or,
// when it is ill-formed, -(length of its maximal subpart) (at least 1): the
// unit String::from_utf8_lossy replaces with one U+FFFD.
int utf8_seq(const unsigned char* s, size_t n, size_t i, uint32_t* cp) {
  const unsigned b0 = s[i];
  if (b0 < 0x80) { *cp = b0; return 1; }
  int len;
  unsigned lo = 0x80, hi = 0xBF;
  if (b0 >= 0xC2 && b0 <= 0xDF) len = 2;
  else if (b0 == 0xE0) { len = 3; lo = 0xA0; }
  else if (b0 >= 0xE1 && b0 <= 0xEC) len = 3;
  else if (b0 == 0xED) { len = 3; hi = 0x9F; }
  else if (b0 >= 0xEE && b0 <= 0xEF) len = 3;
  else if (b0 == 0xF0) { len = 4; lo = 0x90; }
  else if (b0 >= 0xF1 && b0 <= 0xF3) len = 4;
  else if (b0 == 0xF4) { len = 4; hi = 0x8F; }
  else return -1;
  uint32_t v = len == 2 ? (b0 & 0x1F) : len == 3 ? (b0 & 0x0F) : (b0 & 0x07);
  for (int k = 1; k < len; ++k) {
    if (i + k >= n) return -k;
    const unsigned b = s[i + k];
    const unsigned l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
    if (b < l || b > h) return -k;
    v = (v << 6) | (b & 0x3F);
  }
  *cp = v;
  return len;
}

bool utf8_decode(const std::string& s, std::vector<uint32_t>* cps, std::vector<size_t>* offs) {
  const unsigned char* p = (const unsigned char*)s.data();
  for (size_t i = 0; i < s.size();) {
    uint32_t cp;
    const int l = utf8_seq(p, s.size(), i, &cp);
    if (l < 0) return false;
    cps->push_back(cp);
    if (offs) offs->push_back(i);
    i += (size_t)l;
  }
  if (offs) offs->push_back(s.size());
  return true;
}

std::string utf8_lossy(const std::string& b) {
  std::string out;
  const unsigned char* p = (const unsigned char*)b.data();
  for (size_t i = 0; i < b.size();) {
    uint32_t cp;
    const int l = utf8_seq(p, b.size(), i, &cp);
    if (l > 0) {
      out.append(b, i, (size_t)l);
      i += (size_t)l;
    } else {
      out += "\xEF\xBF\xBD";
      i += (size_t)(-l);
    }
  }
  return out;
}

// -------------------------------------------------- character classes --

bool in_ranges(const uint32_t (*r)[2], unsigned n, uint32_t cp) {
  unsigned lo = 0, hi = n;
  while (lo < hi) {
    const unsigned mid = (lo + hi) / 2;
    if (cp < r[mid][0]) hi = mid;
    else if (cp > r[mid][1]) lo = mid + 1;
    else return true;
  }
  return false;
}
enum { C_SPACE, C_LETTER, C_NUMBER, C_OTHER };
int char_class(uint32_t cp) {
  if (in_ranges(kUniSpace, kUniSpace_N, cp)) return C_SPACE;
  if (in_ranges(kUniLetter, kUniLetter_N, cp)) return C_LETTER;
  if (in_ranges(kUniNumber, kUniNumber_N, cp)) return C_NUMBER;
  return C_OTHER;
}

// Length (in code points) of the leftmost-first match of the GPT-2 pattern
//   '(?:[sdmt]|ll|ve|re)| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+
// (tokenizer.rs:28-30) at cps[i]. Every character belongs to one of the
// classes the last four alternatives take, so some alternative always
// matches and the matches tile the text.
size_t gpt2_match(const std::vector<uint32_t>& cps, const std::vector<int>& cls, size_t i) {
  const size_t n = cps.size();
  if (cps[i] == '\'' && i + 1 < n) {
    const uint32_t c1 = cps[i + 1];
    if (c1 == 's' || c1 == 'd' || c1 == 'm' || c1 == 't') return 2;
    if (i + 2 < n) {
      const uint32_t c2 = cps[i + 2];
      if ((c1 == 'l' && c2 == 'l') || (c1 == 'v' && c2 == 'e') || (c1 == 'r' && c2 == 'e')) return 3;
    }
  }
  for (int want : {C_LETTER, C_NUMBER, C_OTHER}) {
    // ' ?X+': the optional space is taken when a run follows it
    size_t j = i;
    if (cps[j] == ' ' && j + 1 < n && cls[j + 1] == want) ++j;
    if (cls[j] != want) continue;
    while (j < n && cls[j] == want) ++j;
    return j - i;
  }
  size_t j = i;  // \s+
  while (j < n && cls[j] == C_SPACE) ++j;
  return j - i;
}

// ------------------------------------------------------------- tables --

// bytes_to_unicode of GPT-2 (tokenizer.rs:55-76): printable bytes map to
// themselves, the others to 256 + n in byte order.
void gpt2_byte_table(uint32_t table[256]) {
  bool direct[256] = {};
  for (int b = '!'; b <= '~'; ++b) direct[b] = true;
  for (int b = 0xA1; b <= 0xAC; ++b) direct[b] = true;
  for (int b = 0xAE; b <= 0xFF; ++b) direct[b] = true;
  uint32_t n = 0;
  for (int b = 0; b < 256; ++b) table[b] = direct[b] ? (uint32_t)b : 256 + n++;
}

void finish_tables(Tokenizer* t, bool byte_level) {
  t->index.clear();
  t->index.reserve(t->vocab.size() * 2);
  for (uint32_t i = 0; i < t->vocab.size(); ++i) t->index[t->vocab[i]] = i;  // the last equal text wins
  // encode_template_output's map of the entries containing '<' (tokenizer.rs:439-444; a later equal text
  // replaces an earlier one); only those that start with '<' can match at a '<'
  t->lt_index.clear();
  t->lt_max_len = 0;
  for (uint32_t i = 0; i < t->vocab.size(); ++i)
    if (!t->vocab[i].empty() && t->vocab[i][0] == '<') {
      t->lt_index[t->vocab[i]] = i;
      t->lt_max_len = std::max(t->lt_max_len, t->vocab[i].size());
    }
  t->byte_level = byte_level;
  if (!byte_level) {  // tokenizer.bin: byte b is token b + 3 (tokenizer.rs:255)
    for (int b = 0; b < 256; ++b) t->byte_to_token[b] = (uint32_t)b + 3;
    t->token_to_byte.clear();
    t->char_to_byte.clear();
    return;
  }
  uint32_t table[256];
  gpt2_byte_table(table);
  t->token_to_byte.assign(std::max<size_t>(t->vocab.size(), 256), -1);
  t->char_to_byte.clear();
  for (int b = 0; b < 256; ++b) {
    t->char_to_byte[table[b]] = (uint8_t)b;
    std::string c;
    put_utf8(table[b], &c);
    auto it = t->index.find(c);
    t->byte_to_token[b] = it == t->index.end() ? 0u : it->second;
    if (it != t->index.end()) t->token_to_byte[it->second] = (int16_t)b;
  }
}

// merges rank -> score (tokenizer.rs:80-91, :158-169): the merged text's
// token scores merges.len() - i, a later merge of the same text overwriting
void merge_scores(Tokenizer* t, const std::vector<std::string>& merges) {
  t->scores.assign(t->vocab.size(), 0.0f);
  std::unordered_map<std::string, uint32_t> idx;
  idx.reserve(t->vocab.size() * 2);
  for (uint32_t i = 0; i < t->vocab.size(); ++i) idx[t->vocab[i]] = i;
  for (size_t i = 0; i < merges.size(); ++i) {
    const size_t sp = merges[i].find(' ');
    if (sp == std::string::npos) continue;
    const std::string merged = merges[i].substr(0, sp) + merges[i].substr(sp + 1);
    auto it = idx.find(merged);
    if (it != idx.end()) t->scores[it->second] = (float)(merges.size() - i);
  }
}

// Tokenizer::bpe_merge (tokenizer.rs:306-336): repeatedly merge the adjacent
// pair whose concatenation is the best-scoring vocabulary entry (the first
// such pair on ties), until no pair is in the vocabulary.
void bpe_merge(const Tokenizer& t, std::vector<uint32_t>* toks) {
  std::string buf;
  for (;;) {
    float best = -1e10f;
    uint32_t best_id = 0;
    long best_idx = -1;
    for (size_t i = 0; i + 1 < toks->size(); ++i) {
      buf = t.vocab[(*toks)[i]];
      buf += t.vocab[(*toks)[i + 1]];
      auto it = t.index.find(buf);
      if (it != t.index.end() && t.scores[it->second] > best) {
        best = t.scores[it->second];
        best_id = it->second;
        best_idx = (long)i;
      }
    }
    if (best_idx < 0) break;
    (*toks)[best_idx] = best_id;
    toks->erase(toks->begin() + best_idx + 1);
  }
}

void byte_encode(const Tokenizer& t, const char* s, size_t n, std::vector<uint32_t>* out) {
  for (size_t i = 0; i < n; ++i) out->push_back(t.byte_to_token[(unsigned char)s[i]]);
}

// ---------------------------------------------------------- loaders --

uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

// The tokenizer keys of a GGUF v3 file's metadata (transformer_llama_gguf.rs:581-641).
int load_gguf_tok(const std::string& path, Tokenizer* t) {
  Mapped mp;
  int rc = map_file(path.c_str(), &mp);
  if (rc) return rc;
  const uint8_t* p = mp.data();
  const size_t size = mp.size;
  size_t off = 0;
  bool ok = true;
  auto rd = [&](size_t k) -> uint64_t {
    if (off + k > size) { ok = false; return 0; }
    uint64_t v = 0;
    memcpy(&v, p + off, k);
    off += k;
    return v;
  };
  auto str = [&]() -> std::string {
    const uint64_t n = rd(8);
    if (!ok || n > size - off) { ok = false; return std::string(); }  // (off + n could wrap)
    std::string s((const char*)p + off, n);
    off += n;
    return s;
  };
  if (rd(4) != 0x46554747u) return fail(YL_ERR_FORMAT, "Not a GGUF file (bad magic)");
  if (rd(4) != 3) return fail(YL_ERR_FORMAT, "Only GGUF version 3 is supported");
  rd(8);
  const uint64_t n_kv = rd(8);
  std::vector<std::string> tokens, merges;
  bool have_tokens = false;
  bool have_bos = false, have_eos = false;
  uint64_t bos = 128000, eos = 128009;
  std::string pre = "default";
  bool add_bos = true, add_space = false;
  std::string tmpl;
  bool have_tmpl = false;
  // scalar of type ty, as u64/i64/f64/bool/string
  std::function<void(uint32_t, int, uint64_t*, std::string*, bool*)> skip;
  skip = [&](uint32_t ty, int depth, uint64_t* u, std::string* s, bool* integral) {
    if (integral) *integral = false;
    switch (ty) {
      case 0: case 1: case 7: { uint64_t v = rd(1); if (u) *u = ty == 1 ? (uint64_t)(int64_t)(int8_t)v : v; break; }
      case 2: case 3: { uint64_t v = rd(2); if (u) *u = ty == 3 ? (uint64_t)(int64_t)(int16_t)v : v; break; }
      case 4: case 5: {
        uint64_t v = rd(4);
        if (u) *u = ty == 5 ? (uint64_t)(int64_t)(int32_t)v : v;
        if (integral) *integral = true;
        break;
      }
      case 6: rd(4); break;
      case 8: { std::string v = str(); if (s) *s = std::move(v); break; }
      case 9: {
        const uint32_t et = (uint32_t)rd(4);
        const uint64_t n = rd(8);
        if (depth > 1) { ok = false; break; }
        for (uint64_t k = 0; k < n && ok; ++k) skip(et, depth + 1, nullptr, nullptr, nullptr);
        break;
      }
      case 10: case 11: { uint64_t v = rd(8); if (u) *u = v; if (integral) *integral = true; break; }
      case 12: rd(8); break;
      default: ok = false;
    }
  };
  for (uint64_t i = 0; i < n_kv && ok; ++i) {
    const std::string key = str();
    const uint32_t ty = (uint32_t)rd(4);
    if ((key == "tokenizer.ggml.tokens" || key == "tokenizer.ggml.merges") && ty == 9) {
      const uint32_t et = (uint32_t)rd(4);
      const uint64_t n = rd(8);
      if (et != 8) return fail(YL_ERR_FORMAT, key + " elements are not strings");
      std::vector<std::string>& dst = key == "tokenizer.ggml.tokens" ? tokens : merges;
      if (n > size) return fail(YL_ERR_FORMAT, "truncated GGUF metadata");
      dst.reserve(n);
      for (uint64_t k = 0; k < n && ok; ++k) dst.push_back(str());
      if (key == "tokenizer.ggml.tokens") have_tokens = true;
      continue;
    }
    uint64_t u = 0;
    std::string s;
    bool integral = false;
    skip(ty, 0, &u, &s, &integral);
    if (key == "tokenizer.ggml.bos_token_id" && integral) { bos = u; have_bos = true; }
    else if (key == "tokenizer.ggml.eos_token_id" && integral) { eos = u; have_eos = true; }
    else if (key == "tokenizer.ggml.pre" && ty == 8) pre = s;
    else if (key == "tokenizer.ggml.add_bos_token" && ty == 7) add_bos = u != 0;
    else if (key == "tokenizer.ggml.add_space_prefix" && ty == 7) add_space = u != 0;
    else if (key == "tokenizer.chat_template" && ty == 8) { tmpl = s; have_tmpl = true; }
  }
  (void)have_bos;
  (void)have_eos;
  if (!ok) return fail(YL_ERR_FORMAT, "truncated GGUF metadata");
  if (!have_tokens) return fail(YL_ERR_FORMAT, "tokenizer.ggml.tokens not found");
  tokenizer_from_parts(t, std::move(tokens), merges, (uint32_t)bos, (uint32_t)eos, pre, add_bos, add_space);
  t->has_template = have_tmpl;
  t->chat_template = tmpl;
  if (have_tmpl) {  // set_chat_template (tokenizer.rs:408-416) parses it at load
    t->tmpl_rc = chat_template_parse(tmpl, &t->tmpl);
    if (t->tmpl_rc) t->tmpl_err = yl_last_error();
  }
  return YL_OK;
}

bool read_all(const std::string& path, std::string* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::stringstream ss;
  ss << f.rdbuf();
  *out = ss.str();
  return true;
}

// Tokenizer::from_json (tokenizer.rs:134-217)
int load_json_tok(const std::string& path, Tokenizer* t) {
  std::string text;
  if (!read_all(path, &text)) return fail(YL_ERR_IO, "cannot read " + path);
  Json root;
  std::string err;
  if (!json_parse(text.data(), text.size(), &root, &err)) return fail(YL_ERR_FORMAT, "tokenizer.json: " + err);
  const Json* model = root.get("model");
  const Json* vocab = model ? model->get("vocab") : nullptr;
  const Json* added = root.get("added_tokens");
  const Json* merges = model ? model->get("merges") : nullptr;
  if (!vocab || vocab->kind != Json::OBJ || !added || added->kind != Json::ARR || !merges || merges->kind != Json::ARR)
    return fail(YL_ERR_FORMAT, "tokenizer.json: model.vocab, model.merges or added_tokens missing");
  // serde_json's map iterates keys in sorted order; a later duplicate key replaces an earlier one
  std::map<std::string, uint64_t> vmap;
  uint64_t max_id = 0;
  for (const auto& kv : vocab->obj) {
    uint64_t id;
    if (!kv.second.as_u64(&id)) return fail(YL_ERR_FORMAT, "tokenizer.json: vocabulary id is not an integer");
    vmap[kv.first] = id;
  }
  for (const auto& kv : vmap) max_id = std::max(max_id, kv.second);
  for (const Json& a : added->arr) {
    const Json* id = a.get("id");
    uint64_t v;
    if (!id || !id->as_u64(&v) || !a.get("content") || !a.get("content")->as_str())
      return fail(YL_ERR_FORMAT, "tokenizer.json: bad added token");
    max_id = std::max(max_id, v);
  }
  if (max_id > (1u << 24)) return fail(YL_ERR_FORMAT, "tokenizer.json: token id too large");
  std::vector<std::string> v((size_t)max_id + 1);
  for (const auto& kv : vmap) v[kv.second] = kv.first;
  uint32_t bos = 128000u, eos = 128009u;
  for (const Json& a : added->arr) {
    uint64_t id;
    a.get("id")->as_u64(&id);
    const std::string& c = *a.get("content")->as_str();
    v[id] = c;
  }
  for (const Json& a : added->arr) {
    uint64_t id;
    a.get("id")->as_u64(&id);
    const std::string& c = *a.get("content")->as_str();
    if (c == "<|begin_of_text|>") bos = (uint32_t)id;
    if (c == "<|end_of_text|>" || c == "<|eot_id|>") eos = (uint32_t)id;
  }
  std::vector<std::string> ms;
  for (const Json& m : merges->arr) {
    if (!m.as_str()) return fail(YL_ERR_UNSUPPORTED, "tokenizer.json: merges must be strings \"a b\"");
    ms.push_back(*m.as_str());
  }
  tokenizer_from_parts(t, std::move(v), ms, bos, eos, "default", true, false);
  return YL_OK;
}

// Tokenizer::new (tokenizer.rs:219-262): the lm.rs tokenizer.bin
int load_bin_tok(const std::string& path, Tokenizer* t) {
  std::string d;
  if (!read_all(path, &d)) return fail(YL_ERR_IO, "cannot read " + path);
  const uint8_t* p = (const uint8_t*)d.data();
  if (d.size() < 16) return fail(YL_ERR_FORMAT, "tokenizer.bin is shorter than its 16-byte header");
  const uint32_t n = rd32(p);
  t->bos = rd32(p + 8);
  t->eos = rd32(p + 12);
  size_t off = 16;
  t->vocab.clear();
  t->scores.clear();
  for (uint32_t i = 0; i < n; ++i) {
    if (off + 8 > d.size()) return fail(YL_ERR_FORMAT, "tokenizer.bin is truncated");
    float sc;
    memcpy(&sc, p + off, 4);
    const uint32_t len = rd32(p + off + 4);
    off += 8;
    if (off + len > d.size()) return fail(YL_ERR_FORMAT, "tokenizer.bin is truncated");
    std::string s(d, off, len);
    std::vector<uint32_t> cps;
    if (!utf8_decode(s, &cps, nullptr)) return fail(YL_ERR_FORMAT, "tokenizer.bin: token is not UTF-8");
    t->vocab.push_back(std::move(s));
    t->scores.push_back(sc);
    off += len;
  }
  t->pre = "default";
  t->add_bos_token = true;
  t->add_space_prefix = false;
  finish_tables(t, false);
  return YL_OK;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}
std::string dir_of(const std::string& p) {
  const size_t k = p.find_last_of('/');
  return k == std::string::npos ? std::string(".") : p.substr(0, k);
}
bool exists(const std::string& p) {
  std::ifstream f(p, std::ios::binary);
  return (bool)f;
}

}  // namespace

bool utf8_code_points(const std::string& s, std::vector<uint32_t>* cps, std::vector<size_t>* offs) {
  return utf8_decode(s, cps, offs);
}
bool is_white_space(uint32_t cp) { return in_ranges(kUniSpace, kUniSpace_N, cp); }

void tokenizer_from_parts(Tokenizer* t, std::vector<std::string> vocab, const std::vector<std::string>& merges,
                          uint32_t bos, uint32_t eos, const std::string& pre, bool add_bos, bool add_space_prefix) {
  t->vocab = std::move(vocab);
  merge_scores(t, merges);
  t->bos = bos;
  t->eos = eos;
  t->pre = pre;
  t->add_bos_token = add_bos;
  t->add_space_prefix = add_space_prefix;
  finish_tables(t, true);
}

int tokenizer_load(const std::string& path, std::unique_ptr<Tokenizer>* out) {
  std::unique_ptr<Tokenizer> t(new Tokenizer());
  int rc;
  if (ends_with(path, ".gguf")) {
    rc = load_gguf_tok(path, t.get());
  } else if (ends_with(path, ".safetensors")) {
    // transformer_llama_st.rs:340-349: tokenizer.json, else tokenizer.bin
    const std::string d = dir_of(path);
    rc = exists(d + "/tokenizer.json") ? load_json_tok(d + "/tokenizer.json", t.get())
                                       : load_bin_tok(d + "/tokenizer.bin", t.get());
  } else if (ends_with(path, ".lmrs")) {
    rc = load_bin_tok(dir_of(path) + "/tokenizer.bin", t.get());  // transformer_llama_lmrs.rs:66
  } else {
    rc = fail(YL_ERR_UNSUPPORTED, "Unsupported model extension for path: " + path);
  }
  if (rc) return rc;
  *out = std::move(t);
  return YL_OK;
}

int tok_encode(const Tokenizer& t, const std::string& text, bool bos, bool eos, std::vector<uint32_t>* out) {
  if (text.empty()) return fail(YL_ERR_ARG, "Text to encode should not be empty");
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  if (!utf8_decode(text, &cps, &offs)) return fail(YL_ERR_ARG, "text is not valid UTF-8");
  out->clear();
  if (bos) out->push_back(t.bos);
  if (t.pre == "gpt2" || t.pre == "smollm") {
    std::string s = text;
    if (t.add_space_prefix && s[0] != ' ') {
      s = " " + s;
      cps.insert(cps.begin(), (uint32_t)' ');
      for (size_t& o : offs) ++o;
      offs.insert(offs.begin(), 0);
    }
    std::vector<int> cls(cps.size());
    for (size_t i = 0; i < cps.size(); ++i) cls[i] = char_class(cps[i]);
    std::vector<uint32_t> seg;
    for (size_t i = 0; i < cps.size();) {
      const size_t len = gpt2_match(cps, cls, i);
      seg.clear();
      byte_encode(t, s.data() + offs[i], offs[i + len] - offs[i], &seg);
      bpe_merge(t, &seg);
      out->insert(out->end(), seg.begin(), seg.end());
      i += len;
    }
  } else {
    std::vector<uint32_t> toks;
    if (t.byte_level) {
      byte_encode(t, text.data(), text.size(), &toks);
    } else {
      for (size_t i = 0; i < cps.size(); ++i) {
        const std::string c = text.substr(offs[i], offs[i + 1] - offs[i]);
        auto it = t.index.find(c);
        if (it != t.index.end()) toks.push_back(it->second);
        else
          for (unsigned char b : c) toks.push_back((uint32_t)b + 3);
      }
    }
    bpe_merge(t, &toks);
    out->insert(out->end(), toks.begin(), toks.end());
  }
  if (eos) out->push_back(t.eos);
  return YL_OK;
}

std::string tok_decode(const Tokenizer& t, const uint32_t* ids, size_t n) {
  const size_t V = t.vocab.size();
  if (!t.byte_level) {
    std::string s;
    for (size_t i = 0; i < n; ++i)
      if (ids[i] < V) s += t.vocab[ids[i]];
    return s;
  }
  std::string bytes;
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  for (size_t i = 0; i < n; ++i) {
    const uint32_t id = ids[i];
    if (id < t.token_to_byte.size() && t.token_to_byte[id] >= 0) {
      bytes.push_back((char)(uint8_t)t.token_to_byte[id]);
    } else if (id < V) {
      const std::string& s = t.vocab[id];
      cps.clear();
      offs.clear();
      utf8_decode(s, &cps, &offs);  // vocabulary entries are UTF-8 (checked at load for tokenizer.bin)
      for (size_t k = 0; k < cps.size(); ++k) {
        auto it = t.char_to_byte.find(cps[k]);
        if (it != t.char_to_byte.end()) bytes.push_back((char)it->second);
        else bytes.append(s, offs[k], offs[k + 1] - offs[k]);
      }
    }
  }
  return utf8_lossy(bytes);
}

namespace {
// encode_wrap_n_header (tokenizer.rs:268-297)
int wrap_n_header(const Tokenizer& t, const std::string& text, const std::string& header, bool wrap,
                  std::vector<uint32_t>* out) {
  std::vector<uint32_t> e;
  int rc;
  if (!t.has_llama_tokens()) {
    if (wrap && t.add_bos_token) out->push_back(t.bos);
    if (!text.empty()) {
      if ((rc = tok_encode(t, text, false, false, &e))) return rc;
      out->insert(out->end(), e.begin(), e.end());
    }
    return YL_OK;
  }
  if (wrap) out->push_back(128000u);
  if (!header.empty()) {
    out->push_back(128006u);
    if ((rc = tok_encode(t, header, false, false, &e))) return rc;
    out->insert(out->end(), e.begin(), e.end());
    out->push_back(128007u);
    out->push_back(271u);
  }
  if (!text.empty()) {
    if ((rc = tok_encode(t, text, false, false, &e))) return rc;
    out->insert(out->end(), e.begin(), e.end());
  }
  if (wrap) {
    out->push_back(271u);
    out->push_back(128009u);
  }
  return YL_OK;
}
}  // namespace

int tok_encode_template_output(const Tokenizer& t, const std::string& text, std::vector<uint32_t>* out) {
  out->clear();
  std::vector<uint32_t> e;
  size_t pos = 0;
  while (pos < text.size()) {
    if (text[pos] == '<') {  // the longest entry that matches here (one text per length can)
      bool hit = false;
      for (size_t len = std::min(t.lt_max_len, text.size() - pos); len > 0 && !hit; --len) {
        auto it = t.lt_index.find(text.substr(pos, len));
        if (it != t.lt_index.end()) {
          out->push_back(it->second);
          pos += len;
          hit = true;
        }
      }
      if (hit) continue;
    }
    const size_t start = pos++;
    while (pos < text.size() && text[pos] != '<') ++pos;
    const int rc = tok_encode(t, text.substr(start, pos - start), false, false, &e);
    if (rc) return rc;
    out->insert(out->end(), e.begin(), e.end());
  }
  return YL_OK;
}

int tok_render_chat(const Tokenizer& t, const std::vector<std::pair<std::string, std::string>>& messages,
                    bool add_generation_prompt, std::vector<uint32_t>* out) {
  out->clear();
  if (!t.has_template) return YL_OK;
  if (!t.tmpl) return fail(t.tmpl_rc, t.tmpl_err);
  std::string text;
  const int rc = chat_template_render(*t.tmpl, messages, add_generation_prompt, &text);
  if (rc) return rc;
  if (text.empty()) return YL_OK;
  return tok_encode_template_output(t, text, out);
}

int tok_encode_wrap_n_header(const Tokenizer& t, const std::string& text, const std::string& header, bool wrap,
                             std::vector<uint32_t>* out) {
  out->clear();
  return wrap_n_header(t, text, header, wrap, out);
}

int tok_set_chat_template(Tokenizer* t, const std::string& tmpl) {
  std::shared_ptr<const ChatTemplate> ct;
  const int rc = chat_template_parse(tmpl, &ct);
  if (rc) return rc;  // the reference panics here; the tokenizer is left as it was
  t->has_template = true;
  t->chat_template = tmpl;
  t->tmpl = ct;
  t->tmpl_rc = 0;
  t->tmpl_err.clear();
  return YL_OK;
}

int tok_apply_system_template(const Tokenizer& t, const std::string& system, std::vector<uint32_t>* out) {
  out->clear();
  if (t.has_template) return tok_render_chat(t, {{"system", system}}, false, out);
  if (t.has_llama_tokens()) return wrap_n_header(t, system, "system", true, out);
  if (system.empty()) return YL_OK;
  return tok_encode(t, system, false, false, out);
}

int tok_apply_turn_template(const Tokenizer& t, const std::string& user, bool add_empty_assistant,
                            std::vector<uint32_t>* out) {
  out->clear();
  int rc;
  if (t.has_template) {
    std::vector<std::pair<std::string, std::string>> msgs = {{"user", user}};
    if (add_empty_assistant) msgs.push_back({"assistant", ""});
    if ((rc = tok_render_chat(t, msgs, add_empty_assistant, out))) return rc;
    if (add_empty_assistant && !out->empty() && out->back() == 128009u) out->pop_back();  // Tokenizer::EOT
    return YL_OK;
  }
  std::vector<uint32_t> e;
  if (t.has_llama_tokens()) {
    std::vector<uint32_t> uid, aid;
    if ((rc = tok_encode(t, "user", false, false, &uid))) return rc;
    if ((rc = tok_encode(t, "assistant", false, false, &aid))) return rc;
    if (uid.size() != 1 || aid.size() != 1)
      return fail(YL_ERR_FORMAT, "expected 'user' and 'assistant' to be single tokens");
    out->insert(out->end(), {128006u, uid[0], 128007u, 271u});
    if ((rc = wrap_n_header(t, user, "", false, out))) return rc;
    out->push_back(128009u);
    if (add_empty_assistant) out->insert(out->end(), {128006u, aid[0], 128007u, 271u});
    return YL_OK;
  }
  if (t.add_bos_token) out->push_back(t.bos);
  if ((rc = tok_encode(t, user, false, false, &e))) return rc;
  out->insert(out->end(), e.begin(), e.end());
  return YL_OK;
}

int tok_chat_prompt(const Tokenizer& t, const std::string& system, const std::string& user,
                    std::vector<uint32_t>* out) {
  out->clear();
  int rc;
  std::vector<uint32_t> e;
  if (t.has_template) {  // main.rs:149-153: [BOS] instead of the system template
    if (t.add_bos_token) out->push_back(t.bos);
    if (!system.empty()) {
      if ((rc = tok_apply_system_template(t, system, &e))) return rc;
      out->insert(out->end(), e.begin(), e.end());
    }
  } else if ((rc = tok_apply_system_template(t, system, out))) {
    return rc;
  }
  if ((rc = tok_apply_turn_template(t, user, true, &e))) return rc;  // main.rs:173
  out->insert(out->end(), e.begin(), e.end());
  return YL_OK;
}

}  // namespace yl
