#include "config.h"

#include <cmath>

namespace minimind::model {

MiniMindConfig default_minimind_config() {
  MiniMindConfig c;
  c.head_dim = c.hidden_size / c.num_attention_heads;
  c.intermediate_size = static_cast<int64_t>(std::ceil(static_cast<double>(c.hidden_size) * M_PI / 64.0)) * 64;
  c.moe_intermediate_size = c.intermediate_size;
  return c;
}

std::vector<std::string> validate_config(const MiniMindConfig& c) {
  std::vector<std::string> errors;
  const auto positive = [&](int64_t v, const char* name) {
    if (v <= 0) errors.push_back(std::string(name) + " must be positive");
  };
  positive(c.hidden_size, "hidden_size");
  positive(c.num_hidden_layers, "num_hidden_layers");
  positive(c.vocab_size, "vocab_size");
  positive(c.num_attention_heads, "num_attention_heads");
  positive(c.num_key_value_heads, "num_key_value_heads");
  positive(c.head_dim, "head_dim");
  positive(c.intermediate_size, "intermediate_size");
  positive(c.max_position_embeddings, "max_position_embeddings");
  const bool heads_ok = c.hidden_size > 0 && c.num_attention_heads > 0;
  if (heads_ok && c.hidden_size % c.num_attention_heads != 0)
    errors.push_back("hidden_size must be divisible by num_attention_heads");
  if (heads_ok && c.head_dim != c.hidden_size / c.num_attention_heads)
    errors.push_back("head_dim must equal hidden_size / num_attention_heads");
  if (c.num_attention_heads > 0 && c.num_key_value_heads > 0 && c.num_attention_heads % c.num_key_value_heads != 0)
    errors.push_back("num_attention_heads must be divisible by num_key_value_heads");
  if (c.rope_theta <= 0.0F) errors.push_back("rope_theta must be positive");
  if (c.rms_norm_eps <= 0.0F) errors.push_back("rms_norm_eps must be positive");
  if (c.hidden_act != "silu") errors.push_back("only silu hidden_act is currently supported");
  if (c.use_moe) {
    positive(c.num_experts, "num_experts");
    positive(c.num_experts_per_tok, "num_experts_per_tok");
    positive(c.moe_intermediate_size, "moe_intermediate_size");
    if (c.num_experts_per_tok != 1) errors.push_back("only top-1 MoE routing is currently planned");
    if (c.num_experts_per_tok > c.num_experts) errors.push_back("num_experts_per_tok cannot exceed num_experts");
  }
  if (c.rope_scaling.enabled) {
    if (c.rope_scaling.type != "yarn") errors.push_back("only yarn rope scaling is supported");
    if (c.rope_scaling.factor <= 1.0F) errors.push_back("rope scaling factor must be greater than 1");
    if (c.rope_scaling.original_max_position_embeddings <= 0)
      errors.push_back("rope scaling original_max_position_embeddings must be positive");
  }
  return errors;
}

}  // namespace minimind::model
