// Chat templates: the Jinja text a GGUF file carries in tokenizer.chat_template,
// rendered the way the reference renders it (tokenizer.rs:408-436: a
// minijinja Environment with default settings, the context
// {messages: [{role, content}, ...], add_generation_prompt}).
#pragma once
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace yl {

struct ChatTemplate;                                                   // a parsed template
using ChatMessages = std::vector<std::pair<std::string, std::string>>;  // (role, content)

// Both calls run on an internal thread with an 8 MiB stack (the caller's
// stack size does not matter) and bound nesting: more than ~250 nested
// parentheses, expressions deeper than 1000 nodes or blocks nested more than
// 200 deep give YL_ERR_FORMAT; YL_ERR_OOM if the thread cannot start.

// Parses a template (Environment::add_template_owned, tokenizer.rs:411-413).
// YL_ERR_FORMAT for a syntax error (where minijinja rejects the template),
// YL_ERR_UNSUPPORTED for a statement this renderer does not implement.
int chat_template_parse(const std::string& src, std::shared_ptr<const ChatTemplate>* out);

// Template::render of the reference's context (tokenizer.rs:421-428).
// YL_ERR_FORMAT where minijinja fails the render (an undefined value under
// attribute access or arithmetic, an unknown filter, test, function or
// method, a type error); YL_ERR_UNSUPPORTED for an expression this renderer
// does not implement; YL_ERR_ARG for a message that is not UTF-8.
int chat_template_render(const ChatTemplate& t, const ChatMessages& messages, bool add_generation_prompt,
                         std::string* out);

}  // namespace yl
