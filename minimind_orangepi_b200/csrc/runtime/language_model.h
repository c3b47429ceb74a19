// LanguageModel: the reference's model API (src/csrc/models/minimind/
// language_model.h:13-53) with every decode step running on a B200 through
// libminimind_cuda.so. There is no CPU fallback: construction succeeds for any
// valid config, and the first forward call fails with std::invalid_argument if
// the shape is outside what the CUDA kernels support (see mmc_create).
#pragma once

#include "decoder_layer.h"

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

namespace minimind::model {

class DeviceModel;
class DeviceSequence;

struct DenseModelWeights {
  std::vector<float> embed_tokens;
  std::vector<DenseLayerWeights> layers;
  std::vector<float> final_norm;
  std::vector<float> lm_head;
};

struct DecoderState {
  std::vector<LayerKvCache> layers;
  int64_t position = 0;
  std::shared_ptr<DeviceSequence> device;  // opened on the first forward call
};

// Device-side sizing. Environment overrides: MINIMIND_DEVICE,
// MINIMIND_KV_TOKENS (page-pool capacity in positions), MINIMIND_MAX_BATCH.
struct RuntimeOptions {
  int device = 0;
  int64_t kv_tokens = 65536;
  int max_seqs = 64;
  int max_batch = 64;
  static RuntimeOptions from_env();
};

class LanguageModel {
 public:
  LanguageModel(MiniMindConfig config, DenseModelWeights weights, RuntimeOptions options = RuntimeOptions::from_env());
  // Weights streamed to the device straight from a weights.bin file.
  LanguageModel(MiniMindConfig config, std::string weights_bin, RuntimeOptions options = RuntimeOptions::from_env());

  const MiniMindConfig& config() const noexcept { return config_; }
  DecoderState make_state() const;
  std::vector<float> forward_token(int32_t token, DecoderState& state) const;
  int32_t forward_next_token(int32_t token, DecoderState& state) const;
  // Batched decode: one step for several independent sequences at once.
  std::vector<int32_t> forward_next_tokens(const std::vector<int32_t>& tokens,
                                           const std::vector<DecoderState*>& states) const;
  int32_t prefill_next_token(const std::vector<int32_t>& prompt_tokens, DecoderState& state) const;
  void generate_stream(const std::vector<int32_t>& prompt_tokens,
                       int64_t max_new_tokens,
                       const std::function<void(int32_t)>& on_token) const;
  std::vector<int32_t> generate(const std::vector<int32_t>& prompt_tokens, int64_t max_new_tokens) const;

 private:
  DeviceModel& device() const;
  void bind(DecoderState& state) const;

  MiniMindConfig config_;
  mutable DenseModelWeights weights_;  // released once uploaded
  std::string weights_bin_;
  RuntimeOptions options_;
  mutable std::shared_ptr<DeviceModel> device_;
};

LanguageModel make_toy_language_model();
int32_t argmax_token(const std::vector<float>& logits);

}  // namespace minimind::model
