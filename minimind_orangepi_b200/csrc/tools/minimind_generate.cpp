// minimind_generate: the reference CLI (src/csrc/tools/minimind_generate.cpp)
// on the CUDA decode path. Same flags (--model --prompt --tokens
// --max-new-tokens --stream) and the same stdout lines
// ("prompt_tokens: ...", "token: N" when streaming, "generated_tokens: ...").
// Without a runtime model directory it falls back to the reference's toy
// model, whose shapes the CUDA kernels do not support: that case exits with an
// error instead of computing on the CPU.
#include "language_model.h"
#include "runtime_loader.h"
#include "tokenizer.h"

#include <cstdlib>
#include <exception>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

namespace {

std::string arg_value(int argc, char** argv, const std::string& name, const std::string& fallback) {
  for (int i = 1; i + 1 < argc; ++i)
    if (argv[i] == name) return argv[i + 1];
  return fallback;
}

bool has_arg(int argc, char** argv, const std::string& name) {
  for (int i = 1; i < argc; ++i)
    if (argv[i] == name) return true;
  return false;
}

std::vector<int32_t> parse_ids(const std::string& s) {
  std::vector<int32_t> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ','))
    if (!item.empty()) out.push_back(static_cast<int32_t>(std::strtol(item.c_str(), nullptr, 10)));
  return out;
}

std::vector<int32_t> prompt_ids(const std::string& prompt, const std::string& explicit_ids,
                                const minimind::model::LanguageModel& model) {
  auto ids = explicit_ids.empty() ? std::vector<int32_t>{} : parse_ids(explicit_ids);
  if (ids.empty()) {
    ids = minimind::ByteTokenizer().encode(prompt);
    for (auto& t : ids) t = t % static_cast<int32_t>(model.config().vocab_size);
  }
  if (ids.empty()) ids.push_back(model.config().bos_token_id);
  for (int32_t t : ids)
    if (t < 0 || t >= model.config().vocab_size) throw std::out_of_range("input token id is out of vocabulary range");
  return ids;
}

}  // namespace

int main(int argc, char** argv) try {
  const std::string prompt = arg_value(argc, argv, "--prompt", "MiniMind");
  const std::string tokens = arg_value(argc, argv, "--tokens", "");
  const std::string model_dir = arg_value(argc, argv, "--model", "");
  const int64_t max_new = std::strtoll(arg_value(argc, argv, "--max-new-tokens", "8").c_str(), nullptr, 10);
  const bool stream = has_arg(argc, argv, "--stream");

  auto model = (!model_dir.empty() && minimind::model::has_runtime_language_model(model_dir))
                   ? minimind::model::load_runtime_language_model(model_dir)
                   : minimind::model::make_toy_language_model();
  const auto ids = prompt_ids(prompt, tokens, model);
  std::cout << "prompt_tokens:";
  for (int32_t t : ids) std::cout << ' ' << t;
  std::cout << '\n';

  std::vector<int32_t> generated;
  if (stream) {
    std::cout << std::flush;
    model.generate_stream(ids, max_new, [&generated](int32_t t) {
      generated.push_back(t);
      std::cout << "token: " << t << '\n' << std::flush;
    });
  } else {
    generated = model.generate(ids, max_new);
  }
  std::cout << "generated_tokens:";
  for (int32_t t : generated) std::cout << ' ' << t;
  std::cout << '\n' << std::flush;
  return 0;
} catch (const std::exception& e) {
  std::cerr << "minimind_generate: " << e.what() << '\n';
  return 1;
}
