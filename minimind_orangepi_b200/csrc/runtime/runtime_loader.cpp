#include "runtime_loader.h"

#include <cctype>
#include <filesystem>
#include <fstream>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace minimind::model {

namespace {

std::string trim(const std::string& s) {
  std::size_t b = 0, e = s.size();
  while (b < e && std::isspace(static_cast<unsigned char>(s[b]))) ++b;
  while (e > b && std::isspace(static_cast<unsigned char>(s[e - 1]))) --e;
  return s.substr(b, e - b);
}

std::unordered_map<std::string, std::string> read_key_values(const std::filesystem::path& path) {
  std::ifstream in(path);
  if (!in) throw std::runtime_error("failed to open runtime config: " + path.string());
  std::unordered_map<std::string, std::string> kv;
  std::string line;
  while (std::getline(in, line)) {
    line = trim(line);
    if (line.empty() || line[0] == '#') continue;
    const auto eq = line.find('=');
    if (eq == std::string::npos) throw std::runtime_error("invalid runtime config line: " + line);
    kv[trim(line.substr(0, eq))] = trim(line.substr(eq + 1));
  }
  return kv;
}

}  // namespace

MiniMindConfig load_runtime_config(const std::string& model_dir) {
  const auto kv = read_key_values(std::filesystem::path(model_dir) / "minimind_runtime_config.txt");
  const auto i64 = [&](const char* k, int64_t d) {
    const auto it = kv.find(k);
    return it == kv.end() ? d : static_cast<int64_t>(std::stoll(it->second));
  };
  const auto boolean = [&](const char* k, bool d) {
    const auto it = kv.find(k);
    return it == kv.end() ? d : (it->second == "1" || it->second == "true" || it->second == "True");
  };
  const auto f32 = [&](const char* k, float d) {
    const auto it = kv.find(k);
    return it == kv.end() ? d : std::stof(it->second);
  };
  MiniMindConfig c = default_minimind_config();
  c.hidden_size = i64("hidden_size", c.hidden_size);
  c.num_hidden_layers = i64("num_hidden_layers", c.num_hidden_layers);
  c.use_moe = boolean("use_moe", false);
  c.vocab_size = i64("vocab_size", c.vocab_size);
  c.num_attention_heads = i64("num_attention_heads", c.num_attention_heads);
  c.num_key_value_heads = i64("num_key_value_heads", c.num_key_value_heads);
  c.head_dim = i64("head_dim", c.hidden_size / c.num_attention_heads);
  c.intermediate_size = i64("intermediate_size", c.intermediate_size);
  c.max_position_embeddings = i64("max_position_embeddings", c.max_position_embeddings);
  c.tie_word_embeddings = boolean("tie_word_embeddings", c.tie_word_embeddings);
  c.num_experts = i64("num_experts", c.num_experts);
  c.num_experts_per_tok = i64("num_experts_per_tok", c.num_experts_per_tok);
  c.moe_intermediate_size = i64("moe_intermediate_size", c.intermediate_size);
  c.rms_norm_eps = f32("rms_norm_eps", c.rms_norm_eps);
  c.rope_theta = f32("rope_theta", c.rope_theta);
  return c;
}

bool has_runtime_language_model(const std::string& model_dir) {
  const std::filesystem::path dir(model_dir);
  return std::filesystem::exists(dir / "minimind_runtime_config.txt") && std::filesystem::exists(dir / "weights.bin");
}

LanguageModel load_runtime_language_model(const std::string& model_dir) {
  MiniMindConfig c = load_runtime_config(model_dir);
  return LanguageModel(std::move(c), (std::filesystem::path(model_dir) / "weights.bin").string());
}

}  // namespace minimind::model
