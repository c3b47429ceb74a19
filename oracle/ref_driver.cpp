// TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product library.
//
// C driver around the reference's own fp32 CPU decode path, built by
// oracle/build_ref.sh from the reference sources into oracle/_ref/. It exists
// so tests, smoke() and bench.py's CPU baseline can call the *reference code*
// (LanguageModel::forward_token / forward_next_token, language_model.cpp:297-333)
// on the same weights.bin the CUDA path loads.
//
// Why a driver of our own: the reference's weight reader is file-local
// (runtime_loader.cpp:121-167) and its config reader never reads rms_norm_eps or
// rope_theta (runtime_loader.cpp:71-88), so the reference always runs with the
// struct defaults eps=1e-6, theta=1e6 (config.h:36-37). The driver re-reads the
// same two files with the same key set and tensor order and lets the caller pin
// eps/theta explicitly, then constructs the reference LanguageModel.
#include "language_model.h"

#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace mm = minimind::model;

namespace {

thread_local std::string g_error;

std::string trim(const std::string& s) {
  std::size_t b = 0, e = s.size();
  while (b < e && std::isspace(static_cast<unsigned char>(s[b]))) ++b;
  while (e > b && std::isspace(static_cast<unsigned char>(s[e - 1]))) --e;
  return s.substr(b, e - b);
}

std::map<std::string, std::string> read_kv(const std::string& path) {
  std::ifstream in(path);
  if (!in) throw std::runtime_error("failed to open runtime config: " + path);
  std::map<std::string, std::string> kv;
  std::string line;
  while (std::getline(in, line)) {
    line = trim(line);
    if (line.empty() || line[0] == '#') continue;
    auto eq = line.find('=');
    if (eq == std::string::npos) throw std::runtime_error("invalid runtime config line: " + line);
    kv[trim(line.substr(0, eq))] = trim(line.substr(eq + 1));
  }
  return kv;
}

int64_t geti(const std::map<std::string, std::string>& kv, const char* k, int64_t d) {
  auto it = kv.find(k);
  return it == kv.end() ? d : std::stoll(it->second);
}
bool getb(const std::map<std::string, std::string>& kv, const char* k, bool d) {
  auto it = kv.find(k);
  return it == kv.end() ? d : (it->second == "1" || it->second == "true" || it->second == "True");
}

std::vector<float> read_tensor(std::ifstream& in, const std::string& name) {
  uint64_t n = 0;
  in.read(reinterpret_cast<char*>(&n), 8);
  std::string got(n, '\0');
  in.read(got.data(), static_cast<std::streamsize>(n));
  if (!in || got != name) throw std::runtime_error("expected tensor " + name + ", got " + got);
  uint64_t count = 0;
  in.read(reinterpret_cast<char*>(&count), 8);
  std::vector<float> v(count);
  in.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * 4));
  if (!in) throw std::runtime_error("failed to read " + name);
  return v;
}

struct RefModel {
  mm::LanguageModel model;
};

}  // namespace

extern "C" {

const char* mmref_last_error() { return g_error.c_str(); }

// eps/theta <= 0 keep the reference defaults (1e-6 / 1e6).
void* mmref_load(const char* model_dir, float eps, float theta) {
  try {
    const std::string dir(model_dir);
    auto kv = read_kv(dir + "/minimind_runtime_config.txt");
    mm::MiniMindConfig c = mm::default_minimind_config();
    c.hidden_size = geti(kv, "hidden_size", c.hidden_size);
    c.num_hidden_layers = geti(kv, "num_hidden_layers", c.num_hidden_layers);
    c.use_moe = getb(kv, "use_moe", false);
    c.vocab_size = geti(kv, "vocab_size", c.vocab_size);
    c.num_attention_heads = geti(kv, "num_attention_heads", c.num_attention_heads);
    c.num_key_value_heads = geti(kv, "num_key_value_heads", c.num_key_value_heads);
    c.head_dim = geti(kv, "head_dim", c.hidden_size / c.num_attention_heads);
    c.intermediate_size = geti(kv, "intermediate_size", c.intermediate_size);
    c.max_position_embeddings = geti(kv, "max_position_embeddings", c.max_position_embeddings);
    c.tie_word_embeddings = getb(kv, "tie_word_embeddings", c.tie_word_embeddings);
    c.num_experts = geti(kv, "num_experts", c.num_experts);
    c.num_experts_per_tok = geti(kv, "num_experts_per_tok", c.num_experts_per_tok);
    c.moe_intermediate_size = geti(kv, "moe_intermediate_size", c.intermediate_size);
    if (eps > 0.0F) c.rms_norm_eps = eps;
    if (theta > 0.0F) c.rope_theta = theta;

    std::ifstream in(dir + "/weights.bin", std::ios::binary);
    if (!in) throw std::runtime_error("failed to open runtime weights");
    char magic[8];
    in.read(magic, 8);
    if (!in || std::memcmp(magic, "MMRTW001", 8) != 0) throw std::runtime_error("unsupported runtime weight format");
    mm::DenseModelWeights w;
    w.embed_tokens = read_tensor(in, "model.embed_tokens.weight");
    w.final_norm = read_tensor(in, "model.norm.weight");
    w.lm_head = read_tensor(in, "lm_head.weight");
    for (int64_t l = 0; l < c.num_hidden_layers; ++l) {
      const std::string p = "model.layers." + std::to_string(l) + ".";
      mm::DenseLayerWeights lw;
      lw.input_norm = read_tensor(in, p + "input_layernorm.weight");
      lw.post_attention_norm = read_tensor(in, p + "post_attention_layernorm.weight");
      lw.q_norm = read_tensor(in, p + "self_attn.q_norm.weight");
      lw.k_norm = read_tensor(in, p + "self_attn.k_norm.weight");
      lw.q_proj = read_tensor(in, p + "self_attn.q_proj.weight");
      lw.k_proj = read_tensor(in, p + "self_attn.k_proj.weight");
      lw.v_proj = read_tensor(in, p + "self_attn.v_proj.weight");
      lw.o_proj = read_tensor(in, p + "self_attn.o_proj.weight");
      if (c.use_moe) {  // tensor order of runtime_loader.cpp:148-158
        lw.moe_gate = read_tensor(in, p + "mlp.gate.weight");
        for (int64_t e = 0; e < c.num_experts; ++e) {
          const std::string ep = p + "mlp.experts." + std::to_string(e) + ".";
          mm::ExpertWeights ew;
          ew.gate_proj = read_tensor(in, ep + "gate_proj.weight");
          ew.up_proj = read_tensor(in, ep + "up_proj.weight");
          ew.down_proj = read_tensor(in, ep + "down_proj.weight");
          lw.experts.push_back(std::move(ew));
        }
      } else {
        lw.gate_proj = read_tensor(in, p + "mlp.gate_proj.weight");
        lw.up_proj = read_tensor(in, p + "mlp.up_proj.weight");
        lw.down_proj = read_tensor(in, p + "mlp.down_proj.weight");
      }
      w.layers.push_back(std::move(lw));
    }
    return new RefModel{mm::LanguageModel(c, std::move(w))};
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void* mmref_toy_model() {
  try {
    return new RefModel{mm::make_toy_language_model()};
  } catch (const std::exception& e) {
    g_error = e.what();
    return nullptr;
  }
}

void mmref_free(void* m) { delete static_cast<RefModel*>(m); }

void* mmref_state_new(void* m) {
  return new mm::DecoderState(static_cast<RefModel*>(m)->model.make_state());
}
void mmref_state_free(void* s) { delete static_cast<mm::DecoderState*>(s); }
int64_t mmref_position(void* s) { return static_cast<mm::DecoderState*>(s)->position; }

// Reference LanguageModel::forward_token: fp32 logits [vocab]; returns the
// reference argmax_token of them (first maximum), or -1 on error.
int32_t mmref_forward_token(void* m, void* s, int32_t token, float* logits) {
  try {
    auto out = static_cast<RefModel*>(m)->model.forward_token(token, *static_cast<mm::DecoderState*>(s));
    if (logits) std::memcpy(logits, out.data(), out.size() * sizeof(float));
    return mm::argmax_token(out);
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

// Reference LanguageModel::forward_next_token (the timed CPU hot path).
int32_t mmref_forward_next_token(void* m, void* s, int32_t token) {
  try {
    return static_cast<RefModel*>(m)->model.forward_next_token(token, *static_cast<mm::DecoderState*>(s));
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

// Reference LanguageModel::generate (greedy, EOS stop). out must hold max_new.
int64_t mmref_generate(void* m, const int32_t* prompt, int64_t n_prompt, int64_t max_new, int32_t* out) {
  try {
    std::vector<int32_t> p(prompt, prompt + n_prompt);
    auto g = static_cast<RefModel*>(m)->model.generate(p, max_new);
    std::memcpy(out, g.data(), g.size() * sizeof(int32_t));
    return static_cast<int64_t>(g.size());
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

// Benchmark helper: give a fresh state `ctx` cached positions of seeded
// synthetic K/V so the timed CPU decode steps run at the workload's context
// length without an O(ctx) token-by-token prompt pass first. Only the timing
// sample uses this; parity runs always build the cache through forward_token.
int mmref_fill_context(void* m, void* s, int64_t ctx, uint64_t seed) {
  try {
    const auto& c = static_cast<RefModel*>(m)->model.config();
    auto* st = static_cast<mm::DecoderState*>(s);
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> dist(0.0F, 1.0F);
    const std::size_t n = static_cast<std::size_t>(ctx * c.num_key_value_heads * c.head_dim);
    for (auto& layer : st->layers) {
      layer.keys.resize(n);
      layer.values.resize(n);
      for (auto& v : layer.keys) v = dist(rng);
      for (auto& v : layer.values) v = dist(rng);
      layer.tokens = ctx;
    }
    st->position = ctx;
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return -1;
  }
}

}  // extern "C"
