// Host-side tokenizer of the generation entry points (infer_ffi): the
// reference's byte-level BPE tokenizer (tokenizer.rs), loaded from the same
// files as the model: GGUF metadata (Tokenizer::from_gguf_parts,
// tokenizer.rs:78-132), tokenizer.json (from_json, :134-217) or tokenizer.bin
// (new, :219-262).
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace yl {

struct Tokenizer {
  std::vector<std::string> vocab;
  std::vector<float> scores;
  // text -> id as the reference's binary search over the text-sorted
  // vocabulary finds it: a stable sort keeps equal texts in id order and the
  // search settles on the last of them, i.e. the highest id
  std::unordered_map<std::string, uint32_t> index;
  bool byte_level = true;
  uint32_t byte_to_token[256] = {};
  std::vector<int16_t> token_to_byte;              // byte a token stands for, -1 if none
  std::unordered_map<uint32_t, uint8_t> char_to_byte;  // GPT-2 byte-table code point -> byte
  uint32_t bos = 0, eos = 0;
  std::string pre = "default";
  bool add_bos_token = true, add_space_prefix = false;
  bool has_template = false;  // a Jinja chat template was found (kept, not rendered)
  std::string chat_template;

  bool has_llama_tokens() const { return vocab.size() > 128009; }  // tokenizer.rs:264-266
};

// Loads the tokenizer that belongs to a model file: its GGUF metadata, or
// tokenizer.json / tokenizer.bin beside a .safetensors file, or tokenizer.bin
// beside a .lmrs file (the files the reference's loaders read).
int tokenizer_load(const std::string& model_path, std::unique_ptr<Tokenizer>* out);
// Builds the tokenizer from GGUF-style parts (tokenizer.rs:78-132).
void tokenizer_from_parts(Tokenizer* t, std::vector<std::string> vocab, const std::vector<std::string>& merges,
                          uint32_t bos, uint32_t eos, const std::string& pre, bool add_bos, bool add_space_prefix);

// Tokenizer::encode (tokenizer.rs:338-392). The text must be non-empty valid
// UTF-8 (the reference asserts non-empty; a Rust &str is always UTF-8).
int tok_encode(const Tokenizer& t, const std::string& text, bool bos, bool eos, std::vector<uint32_t>* out);
// Tokenizer::decode (tokenizer.rs:523-551), String::from_utf8_lossy included.
std::string tok_decode(const Tokenizer& t, const uint32_t* ids, size_t n);
// The prompt of one fresh conversation as the reference's console builds it
// (main.rs:149-153 and :177): the system template of an empty system prompt,
// then the user turn with an empty assistant header (tokenizer.rs:453-521,
// the no-template branches). Jinja templates are not rendered: a tokenizer
// that carries one is prompted with the same built-in format.
int tok_chat_prompt(const Tokenizer& t, const std::string& system, const std::string& user,
                    std::vector<uint32_t>* out);

}  // namespace yl

// C-ABI handle (include/yallma3.h): owns one tokenizer.
struct yl_tokenizer {
  yl::Tokenizer t;
};
