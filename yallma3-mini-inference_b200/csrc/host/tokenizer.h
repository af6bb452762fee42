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
#include <utility>
#include <vector>

namespace yl {

struct ChatTemplate;

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
  bool has_template = false;  // the GGUF metadata held tokenizer.chat_template
  std::string chat_template;
  std::shared_ptr<const ChatTemplate> tmpl;  // the parsed template (null if it did not parse)
  int tmpl_rc = 0;                           // why it did not parse
  std::string tmpl_err;
  // vocabulary entries that start with '<' -> the highest id of that text,
  // and their longest length in bytes (encode_template_output)
  std::unordered_map<std::string, uint32_t> lt_index;
  size_t lt_max_len = 0;

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
// Tokenizer::render_chat_template (tokenizer.rs:418-436): the chat template
// rendered with {messages, add_generation_prompt}, then encoded as
// encode_template_output does (:438-473). No template: an empty result.
int tok_render_chat(const Tokenizer& t, const std::vector<std::pair<std::string, std::string>>& messages,
                    bool add_generation_prompt, std::vector<uint32_t>* out);
// encode_template_output (tokenizer.rs:438-473): at each '<' the longest
// vocabulary entry that matches there becomes one id; the text up to the next
// '<' goes through encode(text, false, false).
int tok_encode_template_output(const Tokenizer& t, const std::string& text, std::vector<uint32_t>* out);
// Tokenizer::encode_wrap_n_header (tokenizer.rs:277-297).
int tok_encode_wrap_n_header(const Tokenizer& t, const std::string& text, const std::string& header, bool wrap,
                             std::vector<uint32_t>* out);
// Tokenizer::set_chat_template (tokenizer.rs:408-416): parses and installs a
// template; on a parse error the tokenizer is left unchanged (the reference
// panics).
int tok_set_chat_template(Tokenizer* t, const std::string& tmpl);
// Tokenizer::apply_system_template (tokenizer.rs:477-495).
int tok_apply_system_template(const Tokenizer& t, const std::string& system, std::vector<uint32_t>* out);
// Tokenizer::apply_turn_template (tokenizer.rs:497-539).
int tok_apply_turn_template(const Tokenizer& t, const std::string& user, bool add_empty_assistant,
                            std::vector<uint32_t>* out);
// The prompt of one fresh conversation as the reference's console builds it.
// Without a chat template (main.rs:149-153, :177): apply_system_template of
// the system prompt, then apply_turn_template(user, true), no-template
// branches (tokenizer.rs:475-521). With one: [BOS] when add_bos_token
// (main.rs:149-153), the rendered system turn when a system prompt is given
// (apply_system_template, tokenizer.rs:476-482), then the rendered user turn
// with an empty assistant message and add_generation_prompt, less a trailing
// <|eot_id|> (apply_turn_template, tokenizer.rs:496-508).
int tok_chat_prompt(const Tokenizer& t, const std::string& system, const std::string& user,
                    std::vector<uint32_t>* out);

// UTF-8 helpers shared with the chat-template renderer: the code points of s
// (false if s is not well-formed UTF-8) with their byte offsets plus s.size(),
// and the Unicode White_Space property.
bool utf8_code_points(const std::string& s, std::vector<uint32_t>* cps, std::vector<size_t>* offs);
bool is_white_space(uint32_t cp);

}  // namespace yl

// C-ABI handle (include/yallma3.h): owns one tokenizer.
struct yl_tokenizer {
  yl::Tokenizer t;
};
