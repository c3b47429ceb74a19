// bench_decode: the reference decode benchmark (bench/bench_decode.cpp) on the
// CUDA path. Same flags (--model --prompt --input-tokens --tokens --warmup) and
// the same key=value output; prefill is the prompt fed through the device
// decode step (the reference's device prefill is not part of this path), and
// the decode loop is timed exactly as the reference does: decode_steps =
// generated - 1. Extension: --batch B decodes B independent copies of the
// prompt together through LanguageModel::forward_next_tokens and reports the
// aggregate rate.
#include "language_model.h"
#include "runtime_loader.h"
#include "tokenizer.h"

#include <algorithm>
#include <chrono>
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

int64_t int_arg(int argc, char** argv, const std::string& name, int64_t fallback) {
  const std::string v = arg_value(argc, argv, name, "");
  return v.empty() ? fallback : std::strtoll(v.c_str(), nullptr, 10);
}

std::vector<int32_t> parse_ids(const std::string& s) {
  std::vector<int32_t> out;
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ','))
    if (!item.empty()) out.push_back(static_cast<int32_t>(std::strtol(item.c_str(), nullptr, 10)));
  return out;
}

struct Timing {
  double prefill_s = 0, decode_s = 0;
  int64_t prefill_tokens = 0, decode_steps = 0, generated = 0;
};

Timing run(const minimind::model::LanguageModel& model, const std::vector<int32_t>& ids, int64_t decode_tokens,
           int batch) {
  using clock = std::chrono::steady_clock;
  std::vector<minimind::model::DecoderState> states(static_cast<std::size_t>(batch));
  std::vector<minimind::model::DecoderState*> ptrs;
  for (auto& s : states) {
    s = model.make_state();
    ptrs.push_back(&s);
  }
  Timing t;
  const auto p0 = clock::now();
  std::vector<int32_t> next(static_cast<std::size_t>(batch));
  for (int32_t tok : ids) next = model.forward_next_tokens(std::vector<int32_t>(static_cast<std::size_t>(batch), tok), ptrs);
  const auto p1 = clock::now();
  for (int64_t i = 0; i + 1 < decode_tokens; ++i) next = model.forward_next_tokens(next, ptrs);
  const auto p2 = clock::now();
  t.prefill_s = std::chrono::duration<double>(p1 - p0).count();
  t.decode_s = std::chrono::duration<double>(p2 - p1).count();
  t.prefill_tokens = static_cast<int64_t>(ids.size());
  t.decode_steps = std::max<int64_t>(0, decode_tokens - 1);
  t.generated = decode_tokens;
  return t;
}

}  // namespace

int main(int argc, char** argv) try {
  const std::string model_dir = arg_value(argc, argv, "--model", "");
  const std::string prompt = arg_value(argc, argv, "--prompt", "hello");
  const std::string explicit_ids = arg_value(argc, argv, "--input-tokens", "");
  const int64_t decode_tokens = int_arg(argc, argv, "--tokens", 16);
  const int64_t warmup = int_arg(argc, argv, "--warmup", 1);
  const int batch = static_cast<int>(int_arg(argc, argv, "--batch", 1));

  auto model = (!model_dir.empty() && minimind::model::has_runtime_language_model(model_dir))
                   ? minimind::model::load_runtime_language_model(model_dir)
                   : minimind::model::make_toy_language_model();
  auto ids = explicit_ids.empty() ? std::vector<int32_t>{} : parse_ids(explicit_ids);
  if (ids.empty()) {
    ids = minimind::ByteTokenizer().encode(prompt);
    for (auto& t : ids) t = t % static_cast<int32_t>(model.config().vocab_size);
  }
  if (ids.empty()) ids.push_back(model.config().bos_token_id);

  for (int64_t i = 0; i < warmup; ++i) (void)run(model, ids, decode_tokens, batch);
  const Timing t = run(model, ids, decode_tokens, batch);
  const double dtps = t.decode_steps == 0 || t.decode_s == 0 ? 0.0 : double(t.decode_steps) * batch / t.decode_s;
  const double ptps = t.prefill_tokens == 0 || t.prefill_s == 0 ? 0.0 : double(t.prefill_tokens) * batch / t.prefill_s;
  std::cout << "prompt_tokens=" << ids.size() << '\n';
  std::cout << "generated_tokens=" << t.generated << '\n';
  std::cout << "prefill_tokens=" << t.prefill_tokens << '\n';
  std::cout << "prefill_seconds=" << t.prefill_s << '\n';
  std::cout << "prefill_tokens_per_second=" << ptps << '\n';
  std::cout << "decode_steps=" << t.decode_steps << '\n';
  std::cout << "decode_seconds=" << t.decode_s << '\n';
  std::cout << "decode_tokens_per_second=" << dtps << '\n';
  if (batch != 1) std::cout << "batch=" << batch << '\n';
  return 0;
} catch (const std::exception& e) {
  std::cerr << "bench_decode: " << e.what() << '\n';
  return 1;
}
