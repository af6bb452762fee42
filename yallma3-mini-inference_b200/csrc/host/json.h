// A small JSON reader for the files the safetensors loader reads
// (config.json, the safetensors header, tokenizer.json's added tokens).
// Values keep what the loader's accessors need: numbers as double and, for
// non-negative integer literals, also as an exact uint64 (serde_json's
// as_u64 answers only for those).
#pragma once
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace yl {

struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ };
  Kind kind = NUL;
  bool b = false;
  double num = 0.0;
  bool is_u64 = false;  // a non-negative integer literal that fits uint64
  uint64_t u = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  // member of an object (nullptr when absent or not an object)
  const Json* get(const std::string& key) const;
  // serde_json-style accessors: false when the value has another type
  bool as_u64(uint64_t* out) const;
  bool as_f64(double* out) const;
  const std::string* as_str() const;
};

// Parses text[0, n) as one JSON value (surrounding whitespace allowed).
// On failure returns false with a message naming the byte offset.
bool json_parse(const char* text, size_t n, Json* out, std::string* err);

}  // namespace yl
