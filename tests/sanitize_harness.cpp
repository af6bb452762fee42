// Host-only harness for tests/test_host_sanitizers.py: the chat-template
// renderer and the tokenizer of the product library, compiled with
// AddressSanitizer and UBSan, run over inputs the test writes.
//   sanitize_harness templates <file>            templates separated by "\n<<<SEP>>>\n"
//   sanitize_harness tokenizer <gguf> <file>     texts separated by byte 0x01
//   sanitize_harness load <file>                 model paths, one per line: tokenizer_load
//                                                 (errors expected), then one encode
//   sanitize_harness json <file>                 JSON documents separated by byte 0x01
#include <cstdio>
#include <cstring>
#include <exception>
#include <fstream>
#include <memory>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "../yallma3-mini-inference_b200/csrc/host/chat_template.h"
#include "../yallma3-mini-inference_b200/csrc/host/json.h"
#include "../yallma3-mini-inference_b200/csrc/host/tokenizer.h"

namespace yl {
static std::string g_err;
void set_error(const std::string& m) { g_err = m; }
int fail(int code, const std::string& m) {
  g_err = m;
  return code;
}
}  // namespace yl
extern "C" const char* yl_last_error(void) { return yl::g_err.c_str(); }

static std::string read_file(const char* path) {
  std::ifstream f(path, std::ios::binary);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

static std::vector<std::string> split(const std::string& all, const std::string& sep) {
  std::vector<std::string> out;
  size_t p = 0;
  for (;;) {
    const size_t q = all.find(sep, p);
    out.push_back(all.substr(p, q == std::string::npos ? std::string::npos : q - p));
    if (q == std::string::npos) return out;
    p = q + sep.size();
  }
}

int main(int argc, char** argv) {
  if (argc >= 3 && !strcmp(argv[1], "templates")) {
    const yl::ChatMessages msgs = {{"system", "  sys a \n"}, {"user", "Hi there <|x|> \xC3\xA9"}, {"assistant", ""}};
    int n = 0, rendered = 0;
    for (const std::string& t : split(read_file(argv[2]), "\n<<<SEP>>>\n")) {
      std::shared_ptr<const yl::ChatTemplate> ct;
      if (yl::chat_template_parse(t, &ct) == 0) {
        std::string out;
        for (int gen = 0; gen < 2; ++gen) rendered += yl::chat_template_render(*ct, msgs, gen != 0, &out) == 0;
      }
      ++n;
    }
    printf("templates %d rendered %d\n", n, rendered);
    return 0;
  }
  if (argc >= 4 && !strcmp(argv[1], "tokenizer")) {
    std::unique_ptr<yl::Tokenizer> t;
    if (yl::tokenizer_load(argv[2], &t)) {
      printf("load failed: %s\n", yl::g_err.c_str());
      return 1;
    }
    std::mt19937 rng(3);
    int n = 0, ok = 0;
    for (const std::string& s : split(read_file(argv[3]), std::string(1, '\x01'))) {
      std::vector<uint32_t> ids;
      if (!s.empty()) {
        ok += yl::tok_encode(*t, s, true, true, &ids) == 0;
        ok += yl::tok_chat_prompt(*t, n % 3 ? "" : "be brief", s, &ids) == 0;
      }
      std::vector<uint32_t> rnd(1 + rng() % 40);
      for (auto& x : rnd) x = rng() % (uint32_t)(t->vocab.size() + 20);  // some ids out of range
      ok += !yl::tok_decode(*t, rnd.data(), rnd.size()).empty();
      ++n;
    }
    printf("texts %d ok %d\n", n, ok);
    return 0;
  }
  if (argc >= 3 && !strcmp(argv[1], "load")) {
    int n = 0, loaded = 0;
    for (const std::string& path : split(read_file(argv[2]), "\n")) {
      if (path.empty()) continue;
      std::unique_ptr<yl::Tokenizer> t;
      ++n;
      try {
        if (yl::tokenizer_load(path, &t) != 0) continue;
      } catch (const std::exception& e) {
        printf("exception escaped tokenizer_load (%s): %s\n", e.what(), path.c_str());
        return 3;
      } catch (...) {
        printf("exception escaped tokenizer_load: %s\n", path.c_str());
        return 3;
      }
      ++loaded;
      std::vector<uint32_t> ids;
      yl::tok_encode(*t, "hello world, it's 3.14", true, false, &ids);
      yl::tok_chat_prompt(*t, "", "hi", &ids);
      if (!ids.empty()) yl::tok_decode(*t, ids.data(), ids.size());
    }
    printf("files %d loaded %d\n", n, loaded);
    return 0;
  }
  if (argc >= 3 && !strcmp(argv[1], "json")) {
    int n = 0, parsed = 0;
    for (const std::string& doc : split(read_file(argv[2]), std::string(1, '\x01'))) {
      yl::Json j;
      std::string err;
      parsed += yl::json_parse(doc.data(), doc.size(), &j, &err);
      ++n;
    }
    printf("documents %d parsed %d\n", n, parsed);
    return 0;
  }
  fprintf(stderr, "usage: sanitize_harness templates <file> | tokenizer <gguf> <file> | load <file> | json <file>\n");
  return 2;
}
