// Loads a runtime model directory (minimind_runtime_config.txt + weights.bin),
// the on-disk format of the reference runtime
// (src/csrc/models/minimind/runtime_loader.h:9-12).
#pragma once

#include "language_model.h"

#include <string>

namespace minimind::model {

// Same keys and fallbacks as the reference's config_from_file
// (runtime_loader.cpp:71-88), plus two optional keys the reference ignores:
// rms_norm_eps and rope_theta (defaults 1e-6 / 1e6 as in config.h:36-37).
MiniMindConfig load_runtime_config(const std::string& model_dir);
// The weights are streamed from weights.bin straight to the GPU on first use.
LanguageModel load_runtime_language_model(const std::string& model_dir);
bool has_runtime_language_model(const std::string& model_dir);

}  // namespace minimind::model
