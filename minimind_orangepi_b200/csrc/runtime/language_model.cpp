// LanguageModel over the C ABI. Follows the control flow of the reference
// (src/csrc/models/minimind/language_model.cpp) — validation, state handling,
// greedy generation with EOS stop — while every forward step is one
// mmc_decode_step on the GPU.
#include "language_model.h"

#include "minimind_cuda.h"

#include <algorithm>
#include <cstdlib>
#include <filesystem>
#include <stdexcept>
#include <string>
#include <utility>

namespace minimind::model {

namespace {

void mmc_check(int code) {
  if (code == MMC_OK) return;
  const std::string msg = mmc_last_error();
  if (code == MMC_ERR_INVALID) throw std::invalid_argument(msg);
  if (code == MMC_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
  throw std::runtime_error(msg);
}

void require_size(const std::vector<float>& v, int64_t expected, const char* name) {
  if (static_cast<int64_t>(v.size()) != expected) throw std::invalid_argument(std::string(name) + " has invalid size");
}

mmc_model_desc describe(const MiniMindConfig& c) {
  mmc_model_desc d{};
  d.hidden_size = c.hidden_size;
  d.num_hidden_layers = c.num_hidden_layers;
  d.num_attention_heads = c.num_attention_heads;
  d.num_key_value_heads = c.num_key_value_heads;
  d.head_dim = c.head_dim;
  d.intermediate_size = c.intermediate_size;
  d.vocab_size = c.vocab_size;
  d.max_position_embeddings = c.max_position_embeddings;
  d.rms_norm_eps = c.rms_norm_eps;
  d.rope_theta = c.rope_theta;
  return d;
}

// generate_stream runs at least this many decode steps on the streamed graph
// loop; shorter runs are not worth capturing a graph for
constexpr int64_t kStreamMinSteps = 8;

int64_t env_i64(const char* name, int64_t fallback) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::strtoll(v, nullptr, 10) : fallback;
}

}  // namespace

RuntimeOptions RuntimeOptions::from_env() {
  RuntimeOptions o;
  o.device = static_cast<int>(env_i64("MINIMIND_DEVICE", o.device));
  o.kv_tokens = env_i64("MINIMIND_KV_TOKENS", o.kv_tokens);
  o.max_batch = static_cast<int>(env_i64("MINIMIND_MAX_BATCH", o.max_batch));
  o.max_seqs = std::max(o.max_seqs, o.max_batch);
  return o;
}

// Owns the CUDA context (weights on the device, page pool, scratch).
class DeviceModel {
 public:
  DeviceModel(const MiniMindConfig& config, const DenseModelWeights* weights, const std::string& weights_bin,
              const RuntimeOptions& o) {
    const mmc_model_desc d = describe(config);
    mmc_check(mmc_create(&d, o.device, &ctx_));
    try {
      if (config.use_moe) {
        if (weights != nullptr) throw std::invalid_argument("MoE models load on the device from weights.bin");
        mmc_check(mmc_configure_moe(ctx_, static_cast<int32_t>(config.num_experts), config.moe_intermediate_size));
      }
      if (weights != nullptr) {
        std::vector<const float*> ptrs;
        std::vector<int64_t> counts;
        auto add = [&](const std::vector<float>& v) {
          ptrs.push_back(v.data());
          counts.push_back(static_cast<int64_t>(v.size()));
        };
        add(weights->embed_tokens);
        add(weights->final_norm);
        add(weights->lm_head);
        for (const auto& l : weights->layers) {
          for (const auto* v : {&l.input_norm, &l.post_attention_norm, &l.q_norm, &l.k_norm, &l.q_proj, &l.k_proj,
                                &l.v_proj, &l.o_proj, &l.gate_proj, &l.up_proj, &l.down_proj})
            add(*v);
        }
        mmc_check(mmc_load_weights(ctx_, ptrs.data(), counts.data(), static_cast<int32_t>(ptrs.size())));
      } else {
        // a packed cache next to weights.bin (DecodeEngine(packed_cache=True)
        // or mmc_save_packed writes it) skips the fp32 read and re-pack when
        // it is at least as new as weights.bin
        namespace fs = std::filesystem;
        const fs::path cache = fs::path(weights_bin).parent_path() / "weights.mmcpk";
        std::error_code ec;
        const bool fresh = fs::exists(cache, ec) &&
                           fs::last_write_time(cache, ec) >= fs::last_write_time(fs::path(weights_bin), ec) && !ec;
        if (!fresh || mmc_load_packed(ctx_, cache.c_str()) != MMC_OK)
          mmc_check(mmc_load_weights_file(ctx_, weights_bin.c_str()));
      }
      const int64_t pages = std::max<int64_t>(1, (o.kv_tokens + 63) / 64) + o.max_seqs;
      mmc_check(mmc_kv_init(ctx_, pages, o.max_seqs, o.max_batch));
    } catch (...) {
      mmc_destroy(ctx_);
      throw;
    }
  }
  ~DeviceModel() { mmc_destroy(ctx_); }
  DeviceModel(const DeviceModel&) = delete;
  DeviceModel& operator=(const DeviceModel&) = delete;
  mmc_ctx* ctx() const { return ctx_; }

 private:
  mmc_ctx* ctx_ = nullptr;
};

// One open device sequence; closing it returns its pages to the pool.
class DeviceSequence {
 public:
  DeviceSequence(std::shared_ptr<DeviceModel> model, int64_t reserve) : model_(std::move(model)) {
    mmc_check(mmc_seq_open(model_->ctx(), reserve, &id_));
  }
  ~DeviceSequence() { mmc_seq_close(model_->ctx(), id_); }
  DeviceSequence(const DeviceSequence&) = delete;
  DeviceSequence& operator=(const DeviceSequence&) = delete;
  int32_t id() const { return id_; }
  const DeviceModel* owner() const { return model_.get(); }

 private:
  std::shared_ptr<DeviceModel> model_;
  int32_t id_ = -1;
};

LanguageModel::LanguageModel(MiniMindConfig config, DenseModelWeights weights, RuntimeOptions options)
    : config_(std::move(config)), weights_(std::move(weights)), options_(options) {
  const auto errors = validate_config(config_);
  if (!errors.empty()) throw std::invalid_argument("invalid MiniMind config: " + errors.front());
  require_size(weights_.embed_tokens, config_.vocab_size * config_.hidden_size, "embed_tokens");
  require_size(weights_.final_norm, config_.hidden_size, "final_norm");
  require_size(weights_.lm_head, config_.vocab_size * config_.hidden_size, "lm_head");
  if (static_cast<int64_t>(weights_.layers.size()) != config_.num_hidden_layers)
    throw std::invalid_argument("layer weight count does not match config");
}

LanguageModel::LanguageModel(MiniMindConfig config, std::string weights_bin, RuntimeOptions options)
    : config_(std::move(config)), weights_bin_(std::move(weights_bin)), options_(options) {
  const auto errors = validate_config(config_);
  if (!errors.empty()) throw std::invalid_argument("invalid MiniMind config: " + errors.front());
}

DeviceModel& LanguageModel::device() const {
  if (!device_) {
    device_ = std::make_shared<DeviceModel>(config_, weights_bin_.empty() ? &weights_ : nullptr, weights_bin_,
                                            options_);
    if (weights_bin_.empty()) {
      // the fp32 host copy is no longer needed once the device holds the weights
      weights_ = DenseModelWeights{};
    }
  }
  return *device_;
}

void LanguageModel::bind(DecoderState& state) const {
  const DeviceModel& model = device();  // creates the context on first use
  if (!state.device || state.device->owner() != &model) {
    if (state.position != 0) throw std::invalid_argument("decoder state belongs to another model");
    state.device = std::make_shared<DeviceSequence>(device_, 64);
  }
}

DecoderState LanguageModel::make_state() const {
  DecoderState s;
  s.layers.resize(static_cast<std::size_t>(config_.num_hidden_layers));
  return s;
}

std::vector<float> LanguageModel::forward_token(int32_t token, DecoderState& state) const {
  if (token < 0 || token >= config_.vocab_size) throw std::out_of_range("token id out of vocabulary range");
  bind(state);
  const int32_t seq = state.device->id();
  int32_t next = 0;
  std::vector<float> logits(static_cast<std::size_t>(config_.vocab_size));
  mmc_check(mmc_decode_step(device_->ctx(), 1, &seq, &token, &next, logits.data()));
  state.position += 1;
  for (auto& l : state.layers) l.tokens += 1;
  return logits;
}

int32_t LanguageModel::forward_next_token(int32_t token, DecoderState& state) const {
  if (token < 0 || token >= config_.vocab_size) throw std::out_of_range("token id out of vocabulary range");
  bind(state);
  const int32_t seq = state.device->id();
  int32_t next = 0;
  mmc_check(mmc_decode_step(device_->ctx(), 1, &seq, &token, &next, nullptr));
  state.position += 1;
  for (auto& l : state.layers) l.tokens += 1;
  return next;
}

std::vector<int32_t> LanguageModel::forward_next_tokens(const std::vector<int32_t>& tokens,
                                                        const std::vector<DecoderState*>& states) const {
  if (tokens.size() != states.size() || tokens.empty())
    throw std::invalid_argument("tokens and states must be non-empty and of equal length");
  std::vector<int32_t> seqs(tokens.size()), next(tokens.size());
  for (std::size_t i = 0; i < tokens.size(); ++i) {
    if (tokens[i] < 0 || tokens[i] >= config_.vocab_size) throw std::out_of_range("token id out of vocabulary range");
    bind(*states[i]);
    seqs[i] = states[i]->device->id();
  }
  mmc_check(mmc_decode_step(device_->ctx(), static_cast<int32_t>(tokens.size()), seqs.data(), tokens.data(),
                            next.data(), nullptr));
  for (auto* s : states) {
    s->position += 1;
    for (auto& l : s->layers) l.tokens += 1;
  }
  return next;
}

// language_model.cpp:334-366 (prefill_next_token_device on the device build):
// the whole prompt in batched passes on the device (mmc_prefill), then the
// greedy token after its last position.
int32_t LanguageModel::prefill_next_token(const std::vector<int32_t>& prompt_tokens, DecoderState& state) const {
  if (prompt_tokens.empty()) throw std::invalid_argument("prompt_tokens cannot be empty");
  for (int32_t t : prompt_tokens)
    if (t < 0 || t >= config_.vocab_size) throw std::out_of_range("token id out of vocabulary range");
  bind(state);
  const int32_t seq = state.device->id();
  const int32_t n = static_cast<int32_t>(prompt_tokens.size());
  int32_t next = 0;
  mmc_check(mmc_prefill(device_->ctx(), 1, &seq, &n, prompt_tokens.data(), &next));
  state.position += n;
  for (auto& l : state.layers) l.tokens += n;
  return next;
}

void LanguageModel::generate_stream(const std::vector<int32_t>& prompt_tokens, int64_t max_new_tokens,
                                    const std::function<void(int32_t)>& on_token) const {
  if (prompt_tokens.empty()) throw std::invalid_argument("prompt_tokens cannot be empty");
  if (max_new_tokens < 0) throw std::invalid_argument("max_new_tokens cannot be negative");
  DecoderState state = make_state();
  int32_t next = prefill_next_token(prompt_tokens, state);
  const int64_t steps = max_new_tokens - 1;  // decode steps after the prompt's token
  if (steps < kStreamMinSteps) {
    for (int64_t i = 0; i < max_new_tokens; ++i) {
      on_token(next);
      if (next == config_.eos_token_id || i + 1 == max_new_tokens) break;
      next = forward_next_token(next, state);
    }
    return;
  }
  // Longer runs stay on the captured device loop: the graph feeds each
  // step's token to the next on the device, and every step's token reaches
  // the host through mapped pinned memory as soon as that step finishes, so the
  // callback sees tokens while later steps are already running.
  mmc_ctx* ctx = device_->ctx();
  const int32_t seq = state.device->id();
  mmc_check(mmc_seq_reserve(ctx, seq, state.position + steps + 1));
  mmc_check(mmc_graph_build(ctx, 1, &seq));
  mmc_check(mmc_graph_set_tokens(ctx, &next));
  mmc_check(mmc_graph_stream_start(ctx, static_cast<int32_t>(steps)));
  for (int64_t i = 0; i < max_new_tokens; ++i) {
    on_token(next);
    if (next == config_.eos_token_id || i + 1 == max_new_tokens) break;
    mmc_check(mmc_graph_stream_next(ctx, &next));
  }
  mmc_check(mmc_graph_stream_stop(ctx));
}

std::vector<int32_t> LanguageModel::generate(const std::vector<int32_t>& prompt_tokens, int64_t max_new_tokens) const {
  std::vector<int32_t> out;
  out.reserve(static_cast<std::size_t>(std::max<int64_t>(max_new_tokens, 0)));
  generate_stream(prompt_tokens, max_new_tokens, [&out](int32_t t) { out.push_back(t); });
  return out;
}

int32_t argmax_token(const std::vector<float>& logits) {
  if (logits.empty()) throw std::invalid_argument("logits cannot be empty");
  return static_cast<int32_t>(std::distance(logits.begin(), std::max_element(logits.begin(), logits.end())));
}

// The reference's toy model (hidden 4, head_dim 2). It validates as a config,
// but its shapes are below the CUDA kernels' minimum (hidden % 64, head_dim in
// {16..128}), so its first forward call throws std::invalid_argument.
LanguageModel make_toy_language_model() {
  MiniMindConfig c;
  c.hidden_size = 4;
  c.num_hidden_layers = 1;
  c.vocab_size = 8;
  c.num_attention_heads = 2;
  c.num_key_value_heads = 1;
  c.head_dim = 2;
  c.intermediate_size = 8;
  c.max_position_embeddings = 16;
  c.rope_theta = 10000.0F;
  c.tie_word_embeddings = false;
  c.moe_intermediate_size = 8;
  DenseModelWeights w;
  w.embed_tokens.assign(32, 0.0F);
  for (int i = 1; i <= 4; ++i) w.embed_tokens[static_cast<std::size_t>(i * 4 + i - 1)] = 1.0F;
  w.final_norm.assign(4, 1.0F);
  w.lm_head.assign(32, 0.0F);
  DenseLayerWeights l;
  l.input_norm.assign(4, 1.0F);
  l.post_attention_norm.assign(4, 1.0F);
  l.q_norm.assign(2, 1.0F);
  l.k_norm.assign(2, 1.0F);
  l.q_proj.assign(16, 0.0F);
  l.k_proj.assign(8, 0.0F);
  l.v_proj.assign(8, 0.0F);
  l.o_proj.assign(16, 0.0F);
  l.gate_proj.assign(32, 0.0F);
  l.up_proj.assign(32, 0.0F);
  l.down_proj.assign(32, 0.0F);
  w.layers.push_back(std::move(l));
  return LanguageModel(c, std::move(w));
}

}  // namespace minimind::model
