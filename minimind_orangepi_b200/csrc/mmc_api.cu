// libminimind_cuda.so: context, weights, paged KV cache and the decode step
// behind the C ABI declared in include/minimind_cuda.h.
//
// One decode step for B rows is a fixed chain of kernels on one stream
// (6 per layer + 1; 6 per layer + 2 on the tensor-core path), every launch after the first carrying programmatic
// stream serialization so each kernel's weight / KV-page prefetch overlaps its
// predecessor:
//   per layer: qkv projection (RMSNorm prologue; layer 0 gathers the embedding)
//              -> fused attention (q/k norm, RoPE, KV append, flash-decode)
//              -> o projection (+ residual)
//              -> gate/up projection (RMSNorm prologue, SiLU*mul epilogue)
//              -> down projection (+ residual)
//   lm_head projection (final RMSNorm prologue, argmax epilogue; writes the
//   next tokens back into the token buffer and advances the positions)
// B <= 4 uses the CUDA-core projections (gemv.cu), larger batches the
// tensor-core ones (gemm_tc.cu). The chain can be captured once as a CUDA
// graph and replayed with the tokens fed back on the device.
#include "../../include/minimind_cuda.h"
#include "kernels/kernels.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace {

thread_local std::string g_error;

struct MmcError : std::runtime_error {
  int code;
  MmcError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const std::string& msg) { throw MmcError(code, msg); }

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(MMC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return MMC_OK;
  } catch (const MmcError& e) {
    g_error = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_error = "host allocation failed";
    return MMC_ERR_CUDA;
  } catch (const std::exception& e) {
    g_error = e.what();
    return MMC_ERR_CUDA;
  }
}

template <typename T>
T* dalloc(size_t count, const char* what) {
  void* p = nullptr;
  ck(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)), what);
  ck(cudaMemset(p, 0, std::max<size_t>(count, 1) * sizeof(T)), what);
  return static_cast<T*>(p);
}

constexpr int kMaxParts = 8;
// batches of up to this many rows run as one persistent launch per step
constexpr int kStepMaxRows = mmc::kStepGroupRows * mmc::kStepMaxGroups;

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

struct Layer {
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  __half *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  __half* router = nullptr;                 // MoE: [experts][H] (post-attention norm folded in)
  std::vector<__half*> egu, edown;          // MoE: per expert [2 MI][H] (interleaved, folded), [H][MI]
  // the same dense projections in fragment order for the persistent step
  __half *qkv_f = nullptr, *o_f = nullptr, *gu_f = nullptr, *down_f = nullptr;
  // the same in the small-batch (skinny.cu) fragment order
  __half *qkv_s = nullptr, *o_s = nullptr, *gu_s = nullptr, *down_s = nullptr;
};

}  // namespace

// pinned ring slots of the streamed graph loop (steps in flight ahead of the
// host's reads)
constexpr int kRingSlots = 32;

struct mmc_ctx {
  mmc_model_desc d{};
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  // parts 1.. of a split batch run on their own streams, forked from and
  // joined back into the launch stream
  cudaStream_t part_stream[kMaxParts - 1] = {};
  cudaEvent_t fork_ev = nullptr, join_ev[kMaxParts - 1] = {};
  int split_parts = 4;  // large batches run as this many concurrent parts
  int moe_experts = 0;    // > 0: top-1 MoE MLP (mmc_configure_moe)
  int64_t moe_inter = 0;
  int* expert_ids = nullptr;  // [max_batch] routed expert per row
  std::vector<void*> allocs;

  // weights
  bool loaded = false;
  float* embed = nullptr;
  __half* lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<Layer> layers;
  float *rope_cos = nullptr, *rope_sin = nullptr;

  // KV cache
  bool kv_ready = false;
  __half* kv_pool = nullptr;
  int64_t n_pages = 0, page_halves = 0;
  int max_seqs = 0, max_pages = 0, max_batch = 0;
  int* d_block_table = nullptr;
  int* d_seq_pos = nullptr;
  std::vector<int> h_block_table;
  std::vector<int64_t> h_pos;
  std::vector<int> h_pages;  // pages reserved per sequence
  std::vector<char> h_open;
  std::vector<int> free_pages;

  // per-step scratch (sized for max_batch)
  float *hidden = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
  __half *h16 = nullptr, *attn16 = nullptr, *act16 = nullptr;  // tensor-core path activations
  __half* q16 = nullptr;  // normalised + rotated q heads, [max_batch][nq][hd]
  int *tokens = nullptr, *slots = nullptr, *next = nullptr;
  int* row_off = nullptr;  // [max_batch] prompt-pass position offsets
  int* attn_order = nullptr;  // [max_batch] per batch part: its rows, longest attention work items first
  int* h_order = nullptr;     // pinned staging of attn_order
  void* argmax_part = nullptr;
  unsigned* argmax_counter = nullptr;
  float* attn_part = nullptr;
  unsigned* attn_counters = nullptr;
  unsigned* attn_work = nullptr;  // [parts][layers][4] attention work-queue words
  int decode_split_k = env_int("MMC_DECODE_SPLIT_K", 1);
  int decode_split_k_alone = env_int("MMC_DECODE_SPLIT_K_ALONE", 4);
  unsigned* chain_sync = nullptr;  // [parts][chain_sync_words(max_batch)] projection-chain queues
  int chain_words = 0;
  bool mlp_chain = false;  // MMC_MLP_CHAIN at creation
  bool attn_fused = true;  // MMC_ATTN_FUSED at creation: q/k prep inside the decode attention launch
  float* ss = nullptr;  // [max_batch][ceil(H / 128)] residual-row sums of squares (folded RMSNorm)
  // persistent step (batches of up to kStepMaxRows rows, dense models)
  bool persistent = false;  // MMC_PERSISTENT at creation (default off: measured slower than the chain)
  bool skinny = true;       // MMC_SKINNY at creation: small batches on the skinny.cu projections
  int attn_merge_tail = -1;  // MMC_ATTN_MERGE_TAIL at creation (-1: by batch size)
  int skinny_min_rows = env_int("MMC_SKINNY_MIN_ROWS", 2);  // smallest batch on them (1 row: gemv measured faster)
  __half* lm_s = nullptr;   // lm_head in the skinny fragment order
  int ss_cap = 0;           // sums-of-squares slots per row (the larger of the two paths' producers)
  int part_cap = 0;         // argmax partial slots per row
  __half* lm_f = nullptr;
  float* step_ssp = nullptr;       // [rows][H / 16]
  float* step_part = nullptr;      // [rows][nkv][max_pages][rep][hd + 2]
  unsigned* step_arrive = nullptr; // [rows][nkv]
  void* step_lm_part = nullptr;    // [groups][V / 16][32] (value, index)
  unsigned* step_sync = nullptr;   // kStepSyncWords
  bool step_trace_on = false;      // MMC_STEP_TRACE at creation
  unsigned long long* step_trace = nullptr;
  int64_t step_trace_cap = 0;
  int step_trace_tasks = 0;
  int* err = nullptr;
  int* h_stage = nullptr;  // pinned: [2][max_batch] ints
  int max_splits_cap = 64;
  std::vector<int> async_slots;  // slot list currently in `slots` (empty: unknown); uploads are skipped when equal
  int64_t hist_host = 0;         // host copy of the history counter: replays since its last reset

  // graph loop
  cudaGraphExec_t graph = nullptr;
  int graph_batch = 0;
  std::vector<int> graph_slots;
  int* hist = nullptr;
  int* hist_step = nullptr;
  int hist_cap = 0;
  int64_t graph_cap_tokens = 0;  // positions the captured split plan covers

  // streamed graph loop: each replay is followed by an async copy of its
  // tokens (and the device error word) into a pinned ring slot and an event
  int* h_ring = nullptr;  // pinned [kRingSlots]: the device error word, copied after every 8th streamed step
  int* h_hist = nullptr;  // host view of `hist` (mapped pinned memory the token sink writes directly)
  cudaEvent_t ring_ev[kRingSlots] = {};
  int64_t st_total = 0, st_enqueued = 0, st_consumed = 0;

  template <typename T>
  T* alloc(size_t n, const char* what) {
    T* p = dalloc<T>(n, what);
    allocs.push_back(p);
    return p;
  }
  int q_size() const { return int(d.num_attention_heads * d.head_dim); }
  int kv_size() const { return int(d.num_key_value_heads * d.head_dim); }
  int rep() const { return int(d.num_attention_heads / d.num_key_value_heads); }
};

namespace {

constexpr int mmc_kernel_kinds = 7;

void use_device(const mmc_ctx* c) { ck(cudaSetDevice(c->device), "cudaSetDevice"); }

// Host -> device copy ordered on the context's stream and complete on return.
// (A plain cudaMemcpy from pageable memory may return before its DMA lands and
// is not ordered with work on the context's non-blocking stream.)
void upload(const mmc_ctx* c, void* dst, const void* src, size_t bytes, const char* what) {
  ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream), what);
  ck(cudaStreamSynchronize(c->stream), what);
}

void require(bool ok, int code, const std::string& msg) {
  if (!ok) fail(code, msg);
}

const char* device_error_text(int e) {
  return e == mmc::kDevWaitTimeout     ? "a bounded wait timed out"
         : e == mmc::kDevBadToken      ? "token id out of vocabulary range"
         : e == mmc::kDevNoPage        ? "KV position not backed by a reserved page"
         : e == mmc::kDevPositionLimit ? "position exceeds max_position_embeddings"
                                       : "unknown";
}

// Raises MMC_ERR_DEVICE (and clears the word) if the device error word `e`,
// already read back, is set.
void raise_device_error(mmc_ctx* c, int e) {
  if (e != 0) {
    ck(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream), "clear device error word");
    ck(cudaStreamSynchronize(c->stream), "clear device error word");
    fail(MMC_ERR_DEVICE, std::string("device error: ") + device_error_text(e) + " (code " + std::to_string(e) + ")");
  }
}

void check_device_error(mmc_ctx* c) {
  int e = 0;
  ck(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
  raise_device_error(c, e);
}

// Split size for the attention kernel: enough CTAs to cover the SMs a few
// times over, at most `max_splits_cap` splits per sequence, and at least
// kMinSplitPages pages per split. (Measured on B200, MiniMind2, 1..128 rows x
// 200..3000 positions, forcing every split size from 2 to 48 pages: this rule
// is within 3 % of the best size on average; one-page splits, the previous
// rule at small batches, spent more on their merges than the extra CTAs
// gained: 32 rows at 1100 positions 657 -> 559 us per step.)
constexpr int64_t kMinSplitPages = 8;
int plan_split_raw(int64_t total_pages, int64_t nkv, int num_sms, int cap, int64_t max_ctx, int* max_splits) {
  const int64_t pages = std::max<int64_t>(1, (max_ctx + mmc::kPageTokens - 1) / mmc::kPageTokens);
  // work items per persistent attention CTA (2 per SM): enough that the
  // queue's tail is short, few enough that per-item merging stays cheap
  static const int items_per_cta = [] {
    const char* e = std::getenv("MMC_ATTN_ITEMS_PER_CTA");
    const int v = e ? std::atoi(e) : 1;
    return v > 0 ? v : 1;
  }();
  int64_t sp = std::max<int64_t>(1, total_pages * nkv / (int64_t(items_per_cta) * 2 * num_sms));
  sp = std::max<int64_t>(sp, std::min<int64_t>(kMinSplitPages, pages));
  sp = std::max<int64_t>(sp, (pages + cap - 1) / cap);
  sp = std::min<int64_t>(sp, pages);
  *max_splits = int((pages + sp - 1) / sp);
  return int(sp * mmc::kPageTokens);
}

int plan_split(const mmc_ctx* c, int64_t total_pages, int64_t max_ctx, int* max_splits) {
  return plan_split_raw(total_pages, c->d.num_key_value_heads, c->num_sms, c->max_splits_cap, max_ctx, max_splits);
}


struct StepIO {
  int B = 0;
  const int* slots = nullptr;
  int* tokens = nullptr;
  int* next_out = nullptr;
  float* logits = nullptr;
  int* hist = nullptr;
  int* hist_step = nullptr;
  int hist_cap = 0;
  int hist_stride = 0;  // row stride of the history (the whole graph batch)
  int split_tokens = 64;
  int max_splits = 1;
  int64_t total_pages = 1, max_ctx = 1;  // attention plan inputs (whole batch)
  int attn_ctas_per_sm = 2;  // persistent attention CTAs per SM (1 when concurrent batch parts share the GPU)
  const int* row_off = nullptr;  // prompt pass: per-row position offsets (positions advanced by the host)
  const int* order = nullptr;    // [B] device: per batch part, the part's rows in attention work-queue order
  bool alone = true;  // the batch runs as one part (nothing concurrent competes for the SMs)
  int row0 = 0;  // first scratch row of this part of the batch
  int part = 0;  // 0 .. kMaxParts-1: which counter region this part uses
};

// Batches of up to kGemvMaxBatch rows use the CUDA-core projections with
// fused RMSNorm prologues; larger batches the tensor-core projections with the
// RMSNorms folded across kernels. Both run 6 kernels per layer.
constexpr int kGemvMaxBatch = 4;
bool use_skinny(const mmc_ctx* c, int B);
// the CUDA-core projections serve batches of up to kGemvMaxBatch rows that
// the skinny projections do not take
bool use_gemv(const mmc_ctx* c, int B) { return B <= kGemvMaxBatch && !use_skinny(c, B); }
enum Kind { kKindQkv = 0, kKindAttn = 1, kKindO = 2, kKindGateUp = 3, kKindDown = 4, kKindLm = 5, kKindNorm = 6 };

// With MMC_MLP_CHAIN=1 (read when a context is created) the tensor-core path
// runs o / gate-up / down as one persistent launch per layer (mlp_chain.cu).
// Measured on B200 it is faster than the three launches when timed alone, but
// slower inside the decode-step graph at config 4 (its CTAs wait on stage
// dependencies while holding shared memory the concurrent batch parts need),
// so it is off by default.
bool use_mlp_chain(const mmc_ctx* c) { return c->mlp_chain; }

// `alone`: the batch runs as one part (the decode attention then folds the
// q/k prep into its own launch; concurrent parts keep the separate prep
// launch, measured faster there)
int kernels_per_step(const mmc_ctx* c, int B, bool alone = true) {
  const int L = int(c->d.num_hidden_layers);
  if (c->attn_fused && alone) {  // attention is one launch (q/k prep fused in)
    if (c->moe_experts > 0) {
      const int per = 4 + 2 * c->moe_experts;
      return use_gemv(c, B) ? per * L + 1 : per * L + 2;
    }
    if (use_gemv(c, B)) return 5 * L + 1;
    return (use_mlp_chain(c) ? 3 : 5) * L + 2;
  }
  // attention is two launches; the tensor-core path adds the layer-0
  // embedding gather (its RMSNorms are folded into the projections)
  if (c->moe_experts > 0) {  // o, router and gate/up + down per expert replace the dense MLP
    const int per = 5 + 2 * c->moe_experts;
    return use_gemv(c, B) ? per * L + 1 : per * L + 2;
  }
  if (use_gemv(c, B)) return 6 * L + 1;
  return (use_mlp_chain(c) ? 4 : 6) * L + 2;
}

// persistent CTAs of one projection-chain launch (MMC_CHAIN_CTAS)
int chain_ctas(const mmc_ctx* c) {
  static const int v = env_int("MMC_CHAIN_CTAS", 0);
  return v > 0 ? v : c->num_sms;
}

// Batches of 5..kSkinnyMaxBatch rows of a dense model run their projections on
// skinny.cu when the context packed its weights for it and every projection
// fits the kernel at this batch size.
bool use_skinny(const mmc_ctx* c, int B) {
  if (c->lm_s == nullptr || B < c->skinny_min_rows || B > mmc::kSkinnyMaxBatch || use_mlp_chain(c) ||
      c->moe_experts > 0)
    return false;
  const auto& d = c->d;
  const int H = int(d.hidden_size), I = int(d.intermediate_size), Q = int(c->q_size());
  const int NQKV = Q + 2 * int(c->kv_size()), V = int(d.vocab_size);
  auto ok = [&](int N, int K) { return mmc::skinny_supported(N, K, B, c->num_sms); };
  return ok(NQKV, H) && ok(H, Q) && ok(2 * I, H) && ok(H, I) && ok(V, H);
}

void launch_proj(mmc_ctx* c, int pro, int epi, const mmc::ProjArgs& a, cudaStream_t s, bool pdl) {
  ck(mmc::launch_gemv(pro, epi, a, c->num_sms, s, pdl), "projection launch");
}

// `ev` (optional, kernels_per_step + 1 events): recorded before every launch
// and after the last one, with programmatic overlap disabled, so the gaps are
// per-kernel device durations; `kinds` receives each launch's Kind.
void enqueue_step(mmc_ctx* c, const StepIO& io, cudaStream_t s, cudaEvent_t* ev = nullptr,
                  std::vector<int>* kinds = nullptr) {
  const auto& d = c->d;
  const int H = int(d.hidden_size), I = int(d.intermediate_size), Q = c->q_size(), KV = c->kv_size();
  const int NQKV = Q + 2 * KV;
  // per-row scratch of this part of the batch (rows row0 .. row0 + B)
  const size_t r0 = size_t(io.row0);
  float* const hidden = c->hidden + r0 * H;
  float* const qkv = c->qkv + r0 * NQKV;
  float* const attn = c->attn + r0 * Q;
  const size_t IA = size_t(std::max<int64_t>(I, c->moe_inter));  // activation row capacity (dense or expert)
  float* const act = c->act + r0 * IA;
  __half* const h16 = c->h16 + r0 * H;
  __half* const attn16 = c->attn16 + r0 * Q;
  __half* const act16 = c->act16 + r0 * IA;
  float* const attn_part = c->attn_part + r0 * size_t(d.num_key_value_heads) * c->max_splits_cap * c->rep() *
                                                size_t(d.head_dim + 2);
  unsigned* const attn_counters = c->attn_counters + r0 * size_t(d.num_key_value_heads);
  void* const argmax_part = static_cast<uint8_t*>(c->argmax_part) + r0 * size_t(c->part_cap) * 8;
  unsigned* const argmax_counter = c->argmax_counter + size_t(io.part) * size_t(c->max_batch + 2);
  int* const expert_ids = c->expert_ids + r0;  // MoE: routed expert per row
  // concurrent batch parts keep the tcgen05 projections: skinny CTAs of 64
  // rows hold up to 192 KB of shared memory, which the parts' kernels then
  // cannot share an SM with (config 4, 256 rows as 4 parts x 64: 1.93 vs
  // 1.49 ms per step measured on B200)
  const bool sk = io.alone && use_skinny(c, io.B);
  const bool tc = !use_gemv(c, io.B);
  int evi = 0;
  bool first = true;
  // returns whether this launch may use programmatic overlap
  auto mark = [&](Kind k) {
    if (ev) ck(cudaEventRecord(ev[evi++], s), "event record");
    if (kinds) kinds->push_back(k);
    const bool pdl = !first && ev == nullptr;
    first = false;
    return pdl;
  };
  // tensor-core path: h16 holds the fp16 residual rows, ss their per-M-tile
  // sums of squares; each RMSNorm is the norm weight folded into the next
  // projection's W and a 1/rms scale in its epilogue.
  float* const ss = c->ss + r0 * size_t(c->ss_cap);
  auto embed_rows = [&] {
    mmc::EmbedArgs e;
    e.embed = c->embed;
    e.tokens = io.tokens;
    e.vocab = int(d.vocab_size);
    e.hidden = hidden;
    e.h16 = h16;
    e.ss = ss;
    e.B = io.B;
    e.H = H;
    e.err = c->err;
    const bool pdl = mark(kKindNorm);
    ck(mmc::launch_embed_rows(e, s, pdl), "embedding launch");
  };
  // sums-of-squares partials per row left by the last producer of the
  // residual rows (the embedding gather, or a skinny residual projection)
  int ss_parts = int((H + 127) / 128);
  auto skproj = [&](Kind k, int epi, const __half* Wf, int N, int K, const __half* X, float* out, __half* out16,
                    int ldo, bool normed) {
    mmc::SkinnyArgs t;
    t.Wf = Wf;
    t.X = X;
    t.N = N;
    t.K = K;
    t.B = io.B;
    t.out = out;
    t.out16 = out16;
    t.ldo = ldo;
    if (normed) {
      t.ss_in = ss;
      t.ss_parts = ss_parts;
      t.eps = d.rms_norm_eps;
    }
    if (epi == mmc::kEpiResid) {
      t.h16_out = h16;
      t.ss_out = ss;
    }
    t.err = c->err;
    const bool pdl = mark(k);
    ck(mmc::launch_skinny(epi, t, c->num_sms, s, pdl), "skinny projection launch");
    if (epi == mmc::kEpiResid) ss_parts = mmc::skinny_grid(N, c->num_sms);
  };
  // normed: the input is the residual stream (scale by 1/rms); resid: update
  // the residual stream and emit its fp16 copy and sums of squares
  auto tcproj = [&](Kind k, int epi, const __half* W, int N, int K, const __half* X, float* out, __half* out16,
                    int ldo, bool normed, const int* row_sel = nullptr, int row_sel_val = 0) {
    mmc::TcArgs t;
    t.row_sel = row_sel;
    t.row_sel_val = row_sel_val;
    // Split-K (thread-block clusters) spreads a projection's weight tiles over
    // more SMs. Measured on B200: it wins for a batch that runs alone (few CTAs
    // per projection: 0.99 -> 0.87 ms/step at 32 sequences) and loses when
    // concurrent batch parts already fill the GPU. MMC_DECODE_SPLIT_K /
    // MMC_DECODE_SPLIT_K_ALONE cap the splits for the two cases.
    t.max_splits = io.alone ? c->decode_split_k_alone : c->decode_split_k;
    t.split_bn = 16;
    if (normed) {
      t.ss_in = ss;
      t.eps = d.rms_norm_eps;
    }
    if (epi == mmc::kEpiResid) {
      t.h16_out = h16;
      t.ss_out = ss;
    }
    t.W = W;
    t.X = X;
    t.N = N;
    t.K = K;
    t.B = io.B;
    t.out = out;
    t.out16 = out16;
    t.ldo = ldo;
    t.err = c->err;
    const bool pdl = mark(k);
    ck(mmc::launch_gemm_tc(epi, t, s, pdl), "tensor-core projection launch");
  };
  for (int l = 0; l < int(d.num_hidden_layers); ++l) {
    const Layer& L = c->layers[l];
    // ---- q|k|v projection
    if (sk) {
      if (l == 0) embed_rows();
      skproj(kKindQkv, mmc::kEpiStore, L.qkv_s, NQKV, H, h16, qkv, nullptr, NQKV, true);
    } else if (tc) {
      if (l == 0) embed_rows();
      tcproj(kKindQkv, mmc::kEpiStore, L.qkv, NQKV, H, h16, qkv, nullptr, NQKV, true);
    } else {
      mmc::ProjArgs p;
      p.B = io.B;
      p.err = c->err;
      p.W = L.qkv;
      p.N = NQKV;
      p.K = H;
      p.in = hidden;
      p.eps = d.rms_norm_eps;
      p.out = qkv;
      p.ldo = NQKV;
      if (l == 0) {
        p.embed = c->embed;
        p.vocab = int(d.vocab_size);
        p.tokens = io.tokens;
        p.hidden = hidden;
      }
      const bool pdl = mark(kKindQkv);
      launch_proj(c, l == 0 ? mmc::kProEmbedNorm : mmc::kProNorm, mmc::kEpiStore, p, s, pdl);
    }
    // ---- attention
    mmc::AttnArgs a;
    a.qkv = qkv;
    a.ld_qkv = NQKV;
    a.q_norm = L.q_norm;
    a.k_norm = L.k_norm;
    a.rope_cos = c->rope_cos;
    a.rope_sin = c->rope_sin;
    a.max_pos = int(d.max_position_embeddings);
    a.eps = d.rms_norm_eps;
    a.kv_pool = c->kv_pool;
    a.layer = l;
    a.layers = int(d.num_hidden_layers);
    a.block_table = c->d_block_table;
    a.max_pages = c->max_pages;
    a.seq_pos = c->d_seq_pos;
    a.row_off = io.row_off;
    a.order = io.order ? io.order + io.row0 : nullptr;
    // decode steps of a batch running alone: q/k prep inside the attention kernel
    a.fused = io.row_off == nullptr && c->attn_fused && io.alone;
    a.slots = io.slots;
    a.B = io.B;
    a.nq = int(d.num_attention_heads);
    a.nkv = int(d.num_key_value_heads);
    a.hd = int(d.head_dim);
    a.split_tokens = io.split_tokens;
    a.max_splits = io.max_splits;
    a.out = tc ? nullptr : attn;
    a.out16 = tc ? attn16 : nullptr;
    a.part = attn_part;
    a.counters = attn_counters;
    // one set of queue words per (batch part, layer); each launch clears the
    // previous layer's set, which has completed by then (it is 4 launches back
    // in the part's chain)
    {
      const int L = int(d.num_hidden_layers);
      a.work = c->attn_work + 4 * (size_t(io.part) * L + l);
      if (L > 1) a.work_prev = c->attn_work + 4 * (size_t(io.part) * L + (l + L - 1) % L);
    }
    // split merges (measured on B200): inline by the last split below 48 rows
    // (batch 1 at 128..1152 positions: 290 vs 306 us per step), from the tail
    // queue from 48 rows up, where CTAs hold several items (64 rows: 0.861 vs
    // 0.894 ms, 128 rows: 1.157 vs 1.207 ms)
    a.merge_tail = c->attn_merge_tail >= 0 ? c->attn_merge_tail : (io.B >= 48 ? 1 : 0);
    a.q16 = c->q16 + r0 * Q;
    a.ctas_per_sm = io.attn_ctas_per_sm;
    a.err = c->err;
    {
      const bool pdl = mark(kKindAttn);
      ck(mmc::launch_attention(a, s, pdl), "attention launch");
    }
    if (sk) {
      skproj(kKindO, mmc::kEpiResid, L.o_s, H, Q, attn16, hidden, nullptr, H, false);
      skproj(kKindGateUp, mmc::kEpiSwiglu, L.gu_s, 2 * I, H, h16, nullptr, act16, I, true);
      skproj(kKindDown, mmc::kEpiResid, L.down_s, H, I, act16, hidden, nullptr, H, false);
      continue;
    }
    if (tc) {
      if (c->moe_experts > 0) {
        tcproj(kKindO, mmc::kEpiResid, L.o, H, Q, attn16, hidden, nullptr, H, false);
        // top-1 MoE (decoder_layer.cpp:370-389): router argmax -> expert id per
        // row, then every expert's gate/up + down over the batch with the
        // residual update committed only for the rows routed to it
        mmc::TcArgs r;
        r.W = L.router;
        r.X = h16;
        r.N = c->moe_experts;
        r.K = H;
        r.B = io.B;
        r.ss_in = ss;
        r.eps = d.rms_norm_eps;
        r.argmax_part = argmax_part;
        r.counter = argmax_counter;
        r.sink.tokens = expert_ids;
        r.err = c->err;
        {
          const bool pdl = mark(kKindGateUp);
          ck(mmc::launch_gemm_tc(mmc::kEpiArgmax, r, s, pdl), "router launch");
        }
        const int MI = int(c->moe_inter);
        for (int e = 0; e < c->moe_experts; ++e) {
          tcproj(kKindGateUp, mmc::kEpiSwiglu, L.egu[e], 2 * MI, H, h16, nullptr, act16, MI, true);
          tcproj(kKindDown, mmc::kEpiResid, L.edown[e], H, MI, act16, hidden, nullptr, H, false, expert_ids, e);
        }
      } else if (use_mlp_chain(c)) {
        mmc::ChainArgs ch;
        ch.Wo = L.o;
        ch.Wgu = L.gu;
        ch.Wdown = L.down;
        ch.attn16 = attn16;
        ch.hidden = hidden;
        ch.h16 = h16;
        ch.ss = ss;
        ch.act16 = act16;
        ch.N[0] = H, ch.K[0] = Q;
        ch.N[1] = 2 * I, ch.K[1] = H;
        ch.N[2] = H, ch.K[2] = I;
        ch.B = io.B;
        ch.eps = d.rms_norm_eps;
        ch.sync = c->chain_sync + size_t(io.part) * c->chain_words;
        ch.err = c->err;
        const bool pdl = mark(kKindO);
        ck(mmc::launch_mlp_chain(ch, chain_ctas(c), s, pdl), "projection chain launch");
      } else {
        tcproj(kKindO, mmc::kEpiResid, L.o, H, Q, attn16, hidden, nullptr, H, false);
        tcproj(kKindGateUp, mmc::kEpiSwiglu, L.gu, 2 * I, H, h16, nullptr, act16, I, true);
        tcproj(kKindDown, mmc::kEpiResid, L.down, H, I, act16, hidden, nullptr, H, false);
      }
      continue;
    }
    // ---- o projection + residual
    mmc::ProjArgs o;
    o.B = io.B;
    o.err = c->err;
    o.W = L.o;
    o.N = H;
    o.K = Q;
    o.in = attn;
    o.out = hidden;
    o.ldo = H;
    {
      const bool pdl = mark(kKindO);
      launch_proj(c, mmc::kProPlain, mmc::kEpiResid, o, s, pdl);
    }
    if (c->moe_experts > 0) {
      // top-1 MoE: router argmax per row, then each expert masked to its rows
      mmc::ProjArgs r;
      r.B = io.B;
      r.err = c->err;
      r.W = L.router;
      r.N = c->moe_experts;
      r.K = H;
      r.in = hidden;
      r.eps = d.rms_norm_eps;
      r.argmax_part = argmax_part;
      r.counter = argmax_counter;
      r.sink.tokens = expert_ids;
      {
        const bool pdl = mark(kKindGateUp);
        launch_proj(c, mmc::kProNormFinal, mmc::kEpiArgmax, r, s, pdl);
      }
      const int MI = int(c->moe_inter);
      for (int e = 0; e < c->moe_experts; ++e) {
        mmc::ProjArgs eg;
        eg.B = io.B;
        eg.err = c->err;
        eg.W = L.egu[e];
        eg.N = 2 * MI;
        eg.K = H;
        eg.in = hidden;
        eg.eps = d.rms_norm_eps;
        eg.out = act;
        eg.ldo = MI;
        {
          const bool pdl = mark(kKindGateUp);
          launch_proj(c, mmc::kProNorm, mmc::kEpiSwiglu, eg, s, pdl);
        }
        mmc::ProjArgs ed;
        ed.B = io.B;
        ed.err = c->err;
        ed.W = L.edown[e];
        ed.N = H;
        ed.K = MI;
        ed.in = act;
        ed.out = hidden;
        ed.ldo = H;
        ed.row_sel = expert_ids;
        ed.row_sel_val = e;
        {
          const bool pdl = mark(kKindDown);
          launch_proj(c, mmc::kProPlain, mmc::kEpiResid, ed, s, pdl);
        }
      }
      continue;
    }
    // ---- gate/up + SiLU*mul
    mmc::ProjArgs gu;
    gu.B = io.B;
    gu.err = c->err;
    gu.W = L.gu;
    gu.N = 2 * I;
    gu.K = H;
    gu.in = hidden;
    gu.eps = d.rms_norm_eps;
    gu.out = act;
    gu.ldo = I;
    {
      const bool pdl = mark(kKindGateUp);
      launch_proj(c, mmc::kProNorm, mmc::kEpiSwiglu, gu, s, pdl);
    }
    // ---- down + residual
    mmc::ProjArgs dn;
    dn.B = io.B;
    dn.err = c->err;
    dn.W = L.down;
    dn.N = H;
    dn.K = I;
    dn.in = act;
    dn.out = hidden;
    dn.ldo = H;
    {
      const bool pdl = mark(kKindDown);
      launch_proj(c, mmc::kProPlain, mmc::kEpiResid, dn, s, pdl);
    }
  }
  // ---- final norm + lm_head + argmax (next tokens, positions, history)
  mmc::TokenSink sink;
  sink.tokens = io.tokens;
  sink.next_out = io.next_out;
  sink.seq_pos = io.row_off ? nullptr : c->d_seq_pos;
  sink.slots = io.slots;
  sink.hist = io.hist;
  sink.hist_step = io.hist_step;
  sink.hist_cap = io.hist_cap;
  sink.hist_stride = io.hist_stride > 0 ? io.hist_stride : io.B;
  if (sk) {
    mmc::SkinnyArgs t;
    t.Wf = c->lm_s;
    t.X = h16;
    t.N = int(d.vocab_size);
    t.K = H;
    t.B = io.B;
    t.ss_in = ss;
    t.ss_parts = ss_parts;
    t.eps = d.rms_norm_eps;
    t.logits = io.logits;
    t.argmax_part = argmax_part;
    t.counter = argmax_counter;
    t.sink = sink;
    t.err = c->err;
    const bool pdl = mark(kKindLm);
    ck(mmc::launch_skinny(mmc::kEpiArgmax, t, c->num_sms, s, pdl), "lm_head launch");
  } else if (tc) {
    mmc::TcArgs t;
    t.W = c->lm_head;
    t.X = h16;
    t.N = int(d.vocab_size);
    t.K = H;
    t.B = io.B;
    t.ss_in = ss;
    t.eps = d.rms_norm_eps;
    t.logits = io.logits;
    t.argmax_part = argmax_part;
    t.counter = argmax_counter;
    t.sink = sink;
    t.err = c->err;
    const bool pdl = mark(kKindLm);
    ck(mmc::launch_gemm_tc(mmc::kEpiArgmax, t, s, pdl), "lm_head launch");
  } else {
    mmc::ProjArgs lm;
    lm.B = io.B;
    lm.err = c->err;
    lm.W = c->lm_head;
    lm.N = int(d.vocab_size);
    lm.K = H;
    lm.in = hidden;
    lm.eps = d.rms_norm_eps;
    lm.logits = io.logits;
    lm.argmax_part = argmax_part;
    lm.counter = argmax_counter;
    lm.sink = sink;
    const bool pdl = mark(kKindLm);
    launch_proj(c, mmc::kProNormFinal, mmc::kEpiArgmax, lm, s, pdl);
  }
  if (ev) ck(cudaEventRecord(ev[evi++], s), "event record");
}

// Batches of at least 2 * kSplitMinRows rows on the tensor-core path run as
// split_parts independent parts on their own streams (parallel branches of the
// captured graph): sequences never interact, so one part's latency-bound
// projections overlap another part's HBM-bound attention.
constexpr int kSplitMinRows = 64;

int attn_ctas_split() {
  static const int v = [] {
    const char* e = std::getenv("MMC_ATTN_CTAS_SPLIT");
    const int x = e ? std::atoi(e) : 1;
    return x > 0 ? x : 1;
  }();
  return v;
}

// number of concurrent parts a batch of B rows runs as (1: not split)
int batch_parts(const mmc_ctx* c, int B) {
  // below 256 rows one part with the fused attention measured faster on B200
  // (128 rows: 1.17 ms/step as one part, 1.27 as two)
  if (B < 4 * kSplitMinRows) return 1;
  int p = std::min(c->split_parts, kMaxParts);
  while (p > 1 && B < p * kSplitMinRows) --p;
  return std::max(p, 1);
}

// rows of part i of a B-row batch cut into p parts: cuts at B * i / p rounded
// down to 16 rows, so with B >= p * kSplitMinRows every part has >= 48 rows
void part_rows(int B, int p, int i, int* r0, int* n) {
  auto cut = [&](int j) { return j >= p ? B : int(int64_t(B) * j / p) / 16 * 16; };
  *r0 = cut(i);
  *n = cut(i + 1) - *r0;
}

// Attention work-queue order (a scheduling hint; any permutation gives the
// same results): per batch part, its rows sorted by the size of their work
// items (pages per split under the part's split plan), longest first, so the
// persistent attention kernel hands out the long items before the short ones
// and its tail is short. Fills host[0, B) with part-relative row indices.
// With `whole`, the batch is one part (a step enqueued without splitting).
void fill_attn_order(const mmc_ctx* c, const StepIO& io, const int32_t* seq_ids, int* host, bool whole = false) {
  const int P = whole ? 1 : batch_parts(c, io.B);
  for (int i = 0; i < P; ++i) {
    int r0 = 0, n = io.B;
    if (P > 1) part_rows(io.B, P, i, &r0, &n);
    int max_splits = 1;
    const int64_t part_pages = P > 1 ? std::max<int64_t>(1, io.total_pages * n / io.B) : io.total_pages;
    const int split_pages = plan_split(c, part_pages, io.max_ctx, &max_splits) / mmc::kPageTokens;
    std::vector<std::pair<int64_t, int>> key(static_cast<size_t>(n));
    for (int b = 0; b < n; ++b) {
      const int64_t pages = (c->h_pos[seq_ids[r0 + b]] + 1 + mmc::kPageTokens - 1) / mmc::kPageTokens;
      const int64_t splits = (pages + split_pages - 1) / split_pages;
      key[size_t(b)] = {-((pages + splits - 1) / splits), b};
    }
    std::stable_sort(key.begin(), key.end());
    for (int b = 0; b < n; ++b) host[r0 + b] = key[size_t(b)].second;
  }
}

bool use_step(const mmc_ctx* c, const StepIO& io) {
  return c->lm_f != nullptr && c->step_sync != nullptr && io.B <= kStepMaxRows && io.row_off == nullptr;
}

// The whole decode step as one persistent launch (step_kernel.cu).
void enqueue_persistent(mmc_ctx* c, const StepIO& io, cudaStream_t s) {
  const auto& d = c->d;
  mmc::StepArgs a;
  for (int l = 0; l < int(d.num_hidden_layers); ++l) {
    const Layer& L = c->layers[l];
    a.layer[l].qkv = L.qkv_f;
    a.layer[l].o = L.o_f;
    a.layer[l].gu = L.gu_f;
    a.layer[l].down = L.down_f;
    a.layer[l].q_norm = L.q_norm;
    a.layer[l].k_norm = L.k_norm;
  }
  a.lm = c->lm_f;
  a.embed = c->embed;
  a.rope_cos = c->rope_cos;
  a.rope_sin = c->rope_sin;
  a.kv_pool = c->kv_pool;
  a.block_table = c->d_block_table;
  a.max_pages = c->max_pages;
  a.n_pages = int(c->n_pages);
  a.seq_pos = c->d_seq_pos;
  a.slots = io.slots;
  a.tokens = io.tokens;
  a.next_out = io.next_out;
  a.logits = io.logits;
  a.hist = io.hist;
  a.hist_step = io.hist_step;
  a.hist_cap = io.hist_cap;
  a.hist_stride = io.hist_stride > 0 ? io.hist_stride : io.B;
  a.B = io.B;
  a.H = int(d.hidden_size);
  a.NQKV = c->q_size() + 2 * c->kv_size();
  a.I = int(d.intermediate_size);
  a.V = int(d.vocab_size);
  a.L = int(d.num_hidden_layers);
  a.nq = int(d.num_attention_heads);
  a.nkv = int(d.num_key_value_heads);
  a.hd = int(d.head_dim);
  a.max_pos = int(d.max_position_embeddings);
  a.eps = d.rms_norm_eps;
  a.h = c->hidden;
  a.h16 = c->h16;
  a.ssp = c->step_ssp;
  a.qkv = c->qkv;
  a.attn16 = c->attn16;
  a.act16 = c->act16;
  a.part = c->step_part;
  a.arrive = c->step_arrive;
  a.lm_part = c->step_lm_part;
  a.sync = c->step_sync;
  a.err = c->err;
  mmc::step_plan(a, io.max_ctx, c->num_sms);
  require(a.s_max <= c->max_pages, MMC_ERR_INVALID, "persistent step split plan exceeds its partial buffer");
  if (c->step_trace_on) {  // debug: per-task timestamps of the last step (mmc_debug_step_trace)
    if (c->step_trace_cap < int64_t(a.total_tasks)) {
      c->step_trace_cap = int64_t(a.total_tasks);
      c->step_trace = c->alloc<unsigned long long>(size_t(c->step_trace_cap) * 8, "step trace");
    }
    a.trace = c->step_trace;
    c->step_trace_tasks = a.total_tasks;
  }
  ck(mmc::launch_step(a, c->num_sms, s), "persistent step launch");
}

void enqueue_batch(mmc_ctx* c, const StepIO& io, cudaStream_t s) {
  if (use_step(c, io)) {
    enqueue_persistent(c, io, s);
    return;
  }
  const int64_t total_pages = io.total_pages, max_ctx = io.max_ctx;
  const int P = batch_parts(c, io.B);
  if (P == 1) {
    enqueue_step(c, io, s);
    return;
  }
  ck(cudaEventRecord(c->fork_ev, s), "fork");
  for (int i = 0; i < P; ++i) {
    int r0, n;
    part_rows(io.B, P, i, &r0, &n);
    StepIO a = io;
    a.B = n;
    a.row0 = io.row0 + r0;
    a.part = i;
    a.alone = false;
    a.slots = io.slots + r0;
    if (io.row_off) a.row_off = io.row_off + r0;
    a.tokens = io.tokens + r0;
    if (io.next_out) a.next_out = io.next_out + r0;
    if (io.logits) a.logits = io.logits + size_t(r0) * c->d.vocab_size;
    if (io.hist) a.hist = io.hist + r0;
    if (io.hist_step) a.hist_step = io.hist_step + i;
    a.hist_stride = io.B;
    a.attn_ctas_per_sm = attn_ctas_split();
    // each part plans its own attention split over its share of the pages
    a.split_tokens = plan_split(c, std::max<int64_t>(1, total_pages * n / io.B), max_ctx, &a.max_splits);
    cudaStream_t ps = s;
    if (i > 0) {
      ps = c->part_stream[i - 1];
      ck(cudaStreamWaitEvent(ps, c->fork_ev, 0), "fork");
    }
    enqueue_step(c, a, ps);
  }
  for (int i = 1; i < P; ++i) {
    ck(cudaEventRecord(c->join_ev[i - 1], c->part_stream[i - 1]), "join");
    ck(cudaStreamWaitEvent(s, c->join_ev[i - 1], 0), "join");
  }
}

// Positions the captured / planned attention split covers for every part.
int64_t plan_cap_tokens(const mmc_ctx* c, const StepIO& io) {
  const int64_t total_pages = io.total_pages, max_ctx = io.max_ctx;
  const int P = batch_parts(c, io.B);
  if (P == 1) return int64_t(io.max_splits) * io.split_tokens;
  int64_t cap = INT64_MAX;
  for (int i = 0; i < P; ++i) {
    int r0, n, ms = 1;
    part_rows(io.B, P, i, &r0, &n);
    const int st = plan_split(c, std::max<int64_t>(1, total_pages * n / io.B), max_ctx, &ms);
    cap = std::min(cap, int64_t(ms) * st);
  }
  return cap;
}

void require_ready(const mmc_ctx* c) {
  require(c != nullptr, MMC_ERR_INVALID, "null context");
  require(c->loaded, MMC_ERR_STATE, "weights are not loaded");
  require(c->kv_ready, MMC_ERR_STATE, "KV cache is not initialised (mmc_kv_init)");
}

void check_seq(const mmc_ctx* c, int32_t seq) {
  require(seq >= 0 && seq < c->max_seqs && c->h_open[seq], MMC_ERR_INVALID, "invalid sequence id");
}

void reserve_pages(mmc_ctx* c, int32_t seq, int64_t tokens) {
  require(tokens <= c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE,
          "reservation exceeds max_position_embeddings");
  const int need = int((tokens + mmc::kPageTokens - 1) / mmc::kPageTokens);
  require(need <= c->max_pages, MMC_ERR_INVALID, "reservation exceeds the per-sequence page table");
  int have = c->h_pages[seq];
  if (need <= have) return;
  require(int64_t(c->free_pages.size()) >= need - have, MMC_ERR_NO_PAGES, "KV page pool exhausted");
  for (; have < need; ++have) {
    c->h_block_table[size_t(seq) * c->max_pages + have] = c->free_pages.back();
    c->free_pages.pop_back();
  }
  const int old = c->h_pages[seq];
  c->h_pages[seq] = need;
  upload(c, c->d_block_table + size_t(seq) * c->max_pages + old,
         c->h_block_table.data() + size_t(seq) * c->max_pages + old, sizeof(int) * (need - old), "block table upload");
}

void stream_drain(mmc_ctx* c);

// Host-side checks shared by the eager step entry points; returns the plan.
// An eager step ends a streamed graph run that is still in progress.
StepIO plan_step(mmc_ctx* c, int32_t batch, const int32_t* seq_ids, bool auto_reserve) {
  stream_drain(c);
  require_ready(c);
  require(batch >= 1 && batch <= c->max_batch, MMC_ERR_INVALID, "batch outside [1, max_batch]");
  require(seq_ids != nullptr, MMC_ERR_INVALID, "null seq_ids");
  std::vector<char> seen(c->max_seqs, 0);
  int64_t total_pages = 0, max_ctx = 1;
  for (int b = 0; b < batch; ++b) {
    const int32_t s = seq_ids[b];
    check_seq(c, s);
    require(!seen[s], MMC_ERR_INVALID, "a sequence appears twice in one batch");
    seen[s] = 1;
    const int64_t ctx = c->h_pos[s] + 1;
    require(ctx <= c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE, "position exceeds max_position_embeddings");
    if (auto_reserve) reserve_pages(c, s, ctx);
    require(int64_t(c->h_pages[s]) * mmc::kPageTokens >= ctx, MMC_ERR_NO_PAGES, "sequence has no page for this position");
    total_pages += (ctx + mmc::kPageTokens - 1) / mmc::kPageTokens;
    max_ctx = std::max(max_ctx, ctx);
  }
  StepIO io;
  io.B = batch;
  io.split_tokens = plan_split(c, total_pages, max_ctx, &io.max_splits);
  io.total_pages = total_pages;
  io.max_ctx = max_ctx;
  return io;
}

std::vector<float> rope_table(int64_t max_pos, int64_t hd, float theta, bool want_sin) {
  // decoder_layer.cpp:97-122: inv_freq = 1 / theta^(2d/hd), angle = pos * inv_freq,
  // evaluated in fp32 with the same float math calls so the table is bit-equal.
  const int64_t half = hd / 2;
  std::vector<float> t(size_t(max_pos * half));
  for (int64_t p = 0; p < max_pos; ++p)
    for (int64_t j = 0; j < half; ++j) {
      const float inv_freq = 1.0F / std::pow(theta, static_cast<float>(j * 2) / static_cast<float>(hd));
      const float angle = static_cast<float>(p) * inv_freq;
      t[size_t(p * half + j)] = want_sin ? std::sin(angle) : std::cos(angle);
    }
  return t;
}

const char* tensor_suffix(int i) {
  static const char* names[] = {"input_layernorm.weight",    "post_attention_layernorm.weight",
                                "self_attn.q_norm.weight",   "self_attn.k_norm.weight",
                                "self_attn.q_proj.weight",   "self_attn.k_proj.weight",
                                "self_attn.v_proj.weight",   "self_attn.o_proj.weight",
                                "mlp.gate_proj.weight",      "mlp.up_proj.weight",
                                "mlp.down_proj.weight"};
  return names[i];
}

// tensors per layer in weights.bin: 8 attention/norm tensors, then the MLP --
// dense gate/up/down, or (MoE, runtime_loader.cpp:148-158) the router and
// each expert's gate/up/down
int layer_tensors(const mmc_ctx* c) { return c->moe_experts > 0 ? 9 + 3 * c->moe_experts : 11; }
int tensor_total(const mmc_ctx* c) { return 3 + layer_tensors(c) * int(c->d.num_hidden_layers); }

// expected element count of tensor i in weights.bin order
int64_t expected_count(const mmc_ctx* c, int i) {
  const auto& d = c->d;
  const int64_t H = d.hidden_size, V = d.vocab_size, Q = d.num_attention_heads * d.head_dim,
                KV = d.num_key_value_heads * d.head_dim, I = d.intermediate_size, HD = d.head_dim;
  if (i == 0 || i == 2) return V * H;
  if (i == 1) return H;
  const int j = (i - 3) % layer_tensors(c);
  const int64_t counts[11] = {H, H, HD, HD, Q * H, KV * H, KV * H, H * Q, I * H, I * H, H * I};
  if (j < 8 || c->moe_experts == 0) return counts[j];
  if (j == 8) return int64_t(c->moe_experts) * H;
  return (j - 9) % 3 == 2 ? H * c->moe_inter : c->moe_inter * H;
}

std::string tensor_name(const mmc_ctx* c, int i) {
  if (i == 0) return "model.embed_tokens.weight";
  if (i == 1) return "model.norm.weight";
  if (i == 2) return "lm_head.weight";
  const int lt = layer_tensors(c), j = (i - 3) % lt;
  const std::string p = "model.layers." + std::to_string((i - 3) / lt) + ".";
  if (j < 8 || c->moe_experts == 0) return p + tensor_suffix(j);
  if (j == 8) return p + "mlp.gate.weight";
  static const char* part[3] = {"gate_proj.weight", "up_proj.weight", "down_proj.weight"};
  return p + "mlp.experts." + std::to_string((j - 9) / 3) + "." + part[(j - 9) % 3];
}

void finish_load(mmc_ctx* c);

// Whether the model's shapes fit the persistent step kernel (step_kernel.cu).
bool step_shape_ok(const mmc_ctx* c) {
  const auto& d = c->d;
  const int64_t Q = c->q_size(), NQKV = Q + 2 * c->kv_size();
  return d.num_hidden_layers <= mmc::kStepMaxLayers && (d.head_dim == 64 || d.head_dim == 96 || d.head_dim == 128) &&
         c->rep() <= 6 && d.hidden_size % 16 == 0 && NQKV % 16 == 0 && d.vocab_size % 16 == 0 &&
         d.hidden_size <= mmc::kStepMaxK && d.intermediate_size <= mmc::kStepMaxK && Q <= mmc::kStepMaxK;
}

// Whether every dense projection has a skinny.cu form (16-row tiles, 32-column
// blocks).
bool skinny_shape_ok(const mmc_ctx* c) {
  const auto& d = c->d;
  const int H = int(d.hidden_size), I = int(d.intermediate_size), Q = int(c->q_size());
  const int NQKV = Q + 2 * int(c->kv_size()), V = int(d.vocab_size);
  auto ok = [&](int N, int K) { return mmc::skinny_supported(N, K, 1, c->num_sms); };
  return ok(NQKV, H) && ok(H, Q) && ok(2 * I, H) && ok(H, I) && ok(V, H);
}

// Every packed weight buffer of a loaded context, in the order of the packed
// cache file: (device pointer slot, bytes). With allocate, the buffers are
// allocated first (loading a cache).
std::vector<std::pair<void**, size_t>> packed_buffers(mmc_ctx* c, bool allocate) {
  const auto& d = c->d;
  const size_t H = size_t(d.hidden_size), V = size_t(d.vocab_size), Q = size_t(c->q_size()),
               KV = size_t(c->kv_size()), I = size_t(d.intermediate_size), HD = size_t(d.head_dim);
  std::vector<std::pair<void**, size_t>> out;
  auto add = [&](auto** slot, size_t elems) {
    using T = std::remove_pointer_t<std::remove_reference_t<decltype(*slot)>>;
    if (allocate) *slot = c->alloc<T>(elems, "packed weights");
    out.emplace_back(reinterpret_cast<void**>(slot), elems * sizeof(T));
  };
  if (allocate) c->layers.assign(size_t(d.num_hidden_layers), Layer{});
  add(&c->embed, V * H);
  add(&c->final_norm, H);
  add(&c->lm_head, V * H);
  for (auto& L : c->layers) {
    add(&L.in_norm, H);
    add(&L.post_norm, H);
    add(&L.q_norm, HD);
    add(&L.k_norm, HD);
    add(&L.qkv, (Q + 2 * KV) * H);
    add(&L.o, H * Q);
    if (c->moe_experts > 0) {
      const size_t E = size_t(c->moe_experts), MI = size_t(c->moe_inter);
      add(&L.router, E * H);
      if (allocate) {
        L.egu.assign(E, nullptr);
        L.edown.assign(E, nullptr);
      }
      for (size_t e = 0; e < E; ++e) {
        add(&L.egu[e], 2 * MI * H);
        add(&L.edown[e], H * MI);
      }
    } else {
      add(&L.gu, 2 * I * H);
      add(&L.down, H * I);
    }
  }
  return out;
}

// Packed cache header: magic, packing layout version, the model description.
constexpr char kPackedMagic[8] = {'M', 'M', 'C', 'P', 'K', '0', '0', '1'};
constexpr uint32_t kPackedLayout = 2;  // rows fp16 RNE, norms folded, gate/up interleaved by 8, MoE fields

// Upload all tensors; `get(i, staging)` fills host fp32 tensor i.
template <typename Getter>
void upload_weights(mmc_ctx* c, Getter&& get) {
  const auto& d = c->d;
  const int64_t H = d.hidden_size, V = d.vocab_size, Q = c->q_size(), KV = c->kv_size(), I = d.intermediate_size;
  const int n = tensor_total(c);
  int64_t max_count = 0;
  for (int i = 0; i < n; ++i) max_count = std::max(max_count, expected_count(c, i));
  float* stage_d = nullptr;
  ck(cudaMalloc(&stage_d, size_t(max_count) * 4 * 2), "weight staging");
  std::unique_ptr<float, void (*)(float*)> guard(stage_d, [](float* p) { cudaFree(p); });
  float* stage_d2 = stage_d + max_count;
  std::vector<float> host, host2;
  auto put = [&](int i, float* dst_d) {
    get(i, host);
    upload(c, dst_d, host.data(), host.size() * 4, "weight upload");
  };
  c->embed = c->alloc<float>(size_t(V * H), "embed");
  put(0, c->embed);
  c->final_norm = c->alloc<float>(size_t(H), "final_norm");
  put(1, c->final_norm);
  c->lm_head = c->alloc<__half>(size_t(V * H), "lm_head");
  put(2, stage_d);
  ck(mmc::launch_pack_rows(stage_d, c->lm_head, V, H, c->stream, c->final_norm), "pack lm_head");
  ck(cudaStreamSynchronize(c->stream), "pack");
  c->layers.assign(size_t(d.num_hidden_layers), Layer{});
  for (int l = 0; l < int(d.num_hidden_layers); ++l) {
    Layer& L = c->layers[l];
    const int base = 3 + layer_tensors(c) * l;
    L.in_norm = c->alloc<float>(size_t(H), "norm");
    put(base + 0, L.in_norm);
    L.post_norm = c->alloc<float>(size_t(H), "norm");
    put(base + 1, L.post_norm);
    L.q_norm = c->alloc<float>(size_t(d.head_dim), "norm");
    put(base + 2, L.q_norm);
    L.k_norm = c->alloc<float>(size_t(d.head_dim), "norm");
    put(base + 3, L.k_norm);
    // fused [q; k; v] rows, language_model.cpp:95-119
    L.qkv = c->alloc<__half>(size_t((Q + 2 * KV) * H), "qkv");
    put(base + 4, stage_d);
    ck(mmc::launch_pack_rows(stage_d, L.qkv, Q, H, c->stream, L.in_norm), "pack q");
    ck(cudaStreamSynchronize(c->stream), "pack");
    put(base + 5, stage_d);
    ck(mmc::launch_pack_rows(stage_d, L.qkv + Q * H, KV, H, c->stream, L.in_norm), "pack k");
    ck(cudaStreamSynchronize(c->stream), "pack");
    put(base + 6, stage_d);
    ck(mmc::launch_pack_rows(stage_d, L.qkv + (Q + KV) * H, KV, H, c->stream, L.in_norm), "pack v");
    ck(cudaStreamSynchronize(c->stream), "pack");
    L.o = c->alloc<__half>(size_t(H * Q), "o");
    put(base + 7, stage_d);
    ck(mmc::launch_pack_rows(stage_d, L.o, H, Q, c->stream), "pack o");
    ck(cudaStreamSynchronize(c->stream), "pack");
    if (c->moe_experts > 0) {
      // router rows and each expert's gate/up + down, packed like the dense MLP
      // (the post-attention norm folded into the router and gate/up columns)
      const int64_t E = c->moe_experts, MI = c->moe_inter;
      L.router = c->alloc<__half>(size_t(E * H), "router");
      put(base + 8, stage_d);
      ck(mmc::launch_pack_rows(stage_d, L.router, E, H, c->stream, L.post_norm), "pack router");
      ck(cudaStreamSynchronize(c->stream), "pack");
      L.egu.assign(size_t(E), nullptr);
      L.edown.assign(size_t(E), nullptr);
      for (int64_t e = 0; e < E; ++e) {
        L.egu[e] = c->alloc<__half>(size_t(2 * MI * H), "expert gate_up");
        put(base + 9 + 3 * int(e), stage_d);
        put(base + 10 + 3 * int(e), stage_d2);
        ck(mmc::launch_pack_gate_up(stage_d, stage_d2, L.egu[e], MI, H, c->stream, L.post_norm), "pack expert");
        ck(cudaStreamSynchronize(c->stream), "pack");
        L.edown[e] = c->alloc<__half>(size_t(H * MI), "expert down");
        put(base + 11 + 3 * int(e), stage_d);
        ck(mmc::launch_pack_rows(stage_d, L.edown[e], H, MI, c->stream), "pack expert down");
        ck(cudaStreamSynchronize(c->stream), "pack");
      }
    } else {
      L.gu = c->alloc<__half>(size_t(2 * I * H), "gate_up");
      put(base + 8, stage_d);
      put(base + 9, stage_d2);
      ck(mmc::launch_pack_gate_up(stage_d, stage_d2, L.gu, I, H, c->stream, L.post_norm), "pack gate_up");
      ck(cudaStreamSynchronize(c->stream), "pack");
      L.down = c->alloc<__half>(size_t(H * I), "down");
      put(base + 10, stage_d);
      ck(mmc::launch_pack_rows(stage_d, L.down, H, I, c->stream), "pack down");
      ck(cudaStreamSynchronize(c->stream), "pack");
    }
  }
  finish_load(c);
}

// RoPE tables and the loaded flag (after the weight buffers are filled).
void finish_load(mmc_ctx* c) {
  const auto& d = c->d;
  if (c->persistent && c->moe_experts == 0 && step_shape_ok(c)) {
    const int64_t H = d.hidden_size, I = d.intermediate_size, Q = c->q_size(), NQKV = Q + 2 * c->kv_size();
    auto frag = [&](const __half* src, int64_t N, int64_t K) {
      __half* dst = c->alloc<__half>(size_t(N * K), "fragment-order weights");
      ck(mmc::launch_pack_fragments(src, dst, N, K, c->stream), "fragment packing");
      return dst;
    };
    for (auto& L : c->layers) {
      L.qkv_f = frag(L.qkv, NQKV, H);
      L.o_f = frag(L.o, H, Q);
      L.gu_f = frag(L.gu, 2 * I, H);
      L.down_f = frag(L.down, H, I);
    }
    c->lm_f = frag(c->lm_head, d.vocab_size, H);
  }
  if (c->skinny && c->moe_experts == 0 && skinny_shape_ok(c)) {
    const int64_t H = d.hidden_size, I = d.intermediate_size, Q = c->q_size(), NQKV = Q + 2 * c->kv_size();
    auto pack = [&](const __half* src, int64_t N, int64_t K) {
      __half* dst = c->alloc<__half>(size_t(N * K), "skinny fragment-order weights");
      ck(mmc::launch_pack_skinny(src, dst, N, K, c->stream), "skinny packing");
      return dst;
    };
    for (auto& L : c->layers) {
      L.qkv_s = pack(L.qkv, NQKV, H);
      L.o_s = pack(L.o, H, Q);
      L.gu_s = pack(L.gu, 2 * I, H);
      L.down_s = pack(L.down, H, I);
    }
    c->lm_s = pack(c->lm_head, d.vocab_size, H);
  }
  const auto cos_t = rope_table(d.max_position_embeddings, d.head_dim, d.rope_theta, false);
  const auto sin_t = rope_table(d.max_position_embeddings, d.head_dim, d.rope_theta, true);
  c->rope_cos = c->alloc<float>(cos_t.size(), "rope");
  c->rope_sin = c->alloc<float>(sin_t.size(), "rope");
  upload(c, c->rope_cos, cos_t.data(), cos_t.size() * 4, "rope upload");
  upload(c, c->rope_sin, sin_t.data(), sin_t.size() * 4, "rope upload");
  ck(cudaDeviceSynchronize(), "weight upload");
  c->loaded = true;
}

// Ends a streamed run: waits for the replays already enqueued (their steps
// happened: positions were advanced when they were enqueued).
void stream_drain(mmc_ctx* c) {
  if (c->st_enqueued > c->st_consumed) ck(cudaStreamSynchronize(c->stream), "stream drain");
  c->st_total = c->st_enqueued = c->st_consumed = 0;
}

void drop_graph(mmc_ctx* c) {
  if (c->st_total > 0) cudaStreamSynchronize(c->stream);
  c->st_total = c->st_enqueued = c->st_consumed = 0;
  if (c->graph) cudaGraphExecDestroy(c->graph);
  c->graph = nullptr;
  c->graph_batch = 0;
  c->graph_slots.clear();
}

}  // namespace

void mmc_set_last_error(const std::string& msg) { g_error = msg; }

extern "C" {

const char* mmc_last_error(void) { return g_error.c_str(); }
int mmc_abi_version(void) { return 1; }

int mmc_create(const mmc_model_desc* desc, int device, mmc_ctx** out) {
  return guarded([&] {
    require(desc && out, MMC_ERR_INVALID, "null argument");
    const mmc_model_desc& d = *desc;
    require(d.hidden_size > 0 && d.num_hidden_layers > 0 && d.num_attention_heads > 0 &&
                d.num_key_value_heads > 0 && d.head_dim > 0 && d.intermediate_size > 0 && d.vocab_size > 0 &&
                d.max_position_embeddings > 0,
            MMC_ERR_INVALID, "model dimensions must be positive");
    require(d.num_attention_heads % d.num_key_value_heads == 0, MMC_ERR_INVALID,
            "num_attention_heads must be divisible by num_key_value_heads");
    require(d.num_attention_heads / d.num_key_value_heads <= 8, MMC_ERR_INVALID,
            "at most 8 query heads per kv head are supported");
    require(d.head_dim == 16 || d.head_dim == 32 || d.head_dim == 64 || d.head_dim == 96 || d.head_dim == 128,
            MMC_ERR_INVALID, "head_dim must be one of 16, 32, 64, 96, 128");
    require(d.hidden_size % 64 == 0 && d.intermediate_size % 64 == 0 &&
                (d.num_attention_heads * d.head_dim) % 64 == 0,
            MMC_ERR_INVALID, "hidden_size, intermediate_size and heads*head_dim must be multiples of 64");
    require(d.rms_norm_eps > 0.f && d.rope_theta > 0.f, MMC_ERR_INVALID, "eps and theta must be positive");
    auto c = std::make_unique<mmc_ctx>();
    c->d = d;
    c->device = device;
    ck(cudaSetDevice(device), "cudaSetDevice");
    int major = 0;
    ck(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device), "device query");
    require(major == 10, MMC_ERR_CUDA, "libminimind_cuda is built for sm_100a (B200) only");
    ck(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device), "device query");
    ck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
    for (int i = 0; i < kMaxParts - 1; ++i) {
      ck(cudaStreamCreateWithFlags(&c->part_stream[i], cudaStreamNonBlocking), "stream");
      ck(cudaEventCreateWithFlags(&c->join_ev[i], cudaEventDisableTiming), "event");
    }
    ck(cudaEventCreateWithFlags(&c->fork_ev, cudaEventDisableTiming), "event");
    c->split_parts = std::max(1, std::min(kMaxParts, env_int("MMC_SPLIT_BATCH", 4)));
    c->mlp_chain = env_int("MMC_MLP_CHAIN", 0) != 0;
    c->persistent = env_int("MMC_PERSISTENT", 0) != 0;
    c->attn_fused = env_int("MMC_ATTN_FUSED", 1) != 0;
    c->skinny = env_int("MMC_SKINNY", 1) != 0;
    c->attn_merge_tail = env_int("MMC_ATTN_MERGE_TAIL", -1);
    c->step_trace_on = env_int("MMC_STEP_TRACE", 0) != 0;
    ck(mmc::step_init_attributes(), "persistent step attributes");
    ck(mmc::gemv_init_attributes(), "gemv attributes");
    ck(mmc::skinny_init_attributes(), "skinny projection attributes");
    ck(mmc::gemm_tc_init_attributes(), "tensor-core projection attributes");
    ck(mmc::mlp_chain_init_attributes(), "projection chain attributes");
    ck(mmc::attention_init_attributes(), "attention attributes");
    c->err = c->alloc<int>(1, "error word");
    ck(cudaDeviceSynchronize(), "context init");
    *out = c.release();
  });
}

void mmc_destroy(mmc_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  drop_graph(c);
  for (void* p : c->allocs) cudaFree(p);
  if (c->h_stage) cudaFreeHost(c->h_stage);
  if (c->h_order) cudaFreeHost(c->h_order);
  if (c->h_ring) cudaFreeHost(c->h_ring);
  if (c->h_hist) cudaFreeHost(c->h_hist);
  for (auto e : c->ring_ev)
    if (e) cudaEventDestroy(e);
  for (auto ps : c->part_stream)
    if (ps) cudaStreamSynchronize(ps);
  if (c->stream) cudaStreamDestroy(c->stream);
  for (auto ps : c->part_stream)
    if (ps) cudaStreamDestroy(ps);
  if (c->fork_ev) cudaEventDestroy(c->fork_ev);
  for (auto e : c->join_ev)
    if (e) cudaEventDestroy(e);
  delete c;
}

int mmc_load_weights(mmc_ctx* c, const float* const* tensors, const int64_t* counts, int32_t n) {
  return guarded([&] {
    require(c && tensors && counts, MMC_ERR_INVALID, "null argument");
    require(!c->loaded, MMC_ERR_STATE, "weights already loaded");
    use_device(c);
    const int expect = tensor_total(c);
    require(n == expect, MMC_ERR_INVALID, "expected " + std::to_string(expect) + " tensors in weights.bin order");
    for (int i = 0; i < n; ++i)
      require(counts[i] == expected_count(c, i) && tensors[i], MMC_ERR_INVALID,
              tensor_name(c, i) + " has invalid size");
    upload_weights(c, [&](int i, std::vector<float>& h) { h.assign(tensors[i], tensors[i] + counts[i]); });
  });
}

int mmc_load_weights_file(mmc_ctx* c, const char* path) {
  return guarded([&] {
    require(c && path, MMC_ERR_INVALID, "null argument");
    require(!c->loaded, MMC_ERR_STATE, "weights already loaded");
    use_device(c);
    std::ifstream in(path, std::ios::binary);
    require(bool(in), MMC_ERR_IO, std::string("failed to open runtime weights: ") + path);
    char magic[8] = {};
    in.read(magic, 8);
    require(bool(in) && std::memcmp(magic, "MMRTW001", 8) == 0, MMC_ERR_IO, "unsupported runtime weight format");
    int next = 0;
    upload_weights(c, [&](int i, std::vector<float>& h) {
      require(i == next++, MMC_ERR_STATE, "weights must be read in file order");
      uint64_t len = 0;
      in.read(reinterpret_cast<char*>(&len), 8);
      require(bool(in) && len < 4096, MMC_ERR_IO, "failed to read tensor name");
      std::string name(len, '\0');
      in.read(name.data(), std::streamsize(len));
      const std::string want = tensor_name(c, i);
      require(bool(in) && name == want, MMC_ERR_IO, "expected tensor " + want + ", got " + name);
      uint64_t count = 0;
      in.read(reinterpret_cast<char*>(&count), 8);
      require(bool(in) && int64_t(count) == expected_count(c, i), MMC_ERR_IO, want + " has invalid size");
      h.resize(count);
      in.read(reinterpret_cast<char*>(h.data()), std::streamsize(count * 4));
      require(bool(in), MMC_ERR_IO, "failed to read " + want);
    });
  });
}

int mmc_configure_moe(mmc_ctx* c, int32_t num_experts, int64_t moe_intermediate_size) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    require(!c->loaded && !c->kv_ready, MMC_ERR_STATE, "configure MoE before loading weights and the KV cache");
    require(num_experts >= 1 && num_experts <= 64, MMC_ERR_INVALID, "num_experts outside [1, 64]");
    require(moe_intermediate_size > 0 && moe_intermediate_size % 64 == 0, MMC_ERR_INVALID,
            "moe_intermediate_size must be a positive multiple of 64");
    c->moe_experts = num_experts;
    c->moe_inter = moe_intermediate_size;
    c->mlp_chain = false;  // the projection chain covers the dense MLP only
  });
}

int mmc_save_packed(mmc_ctx* c, const char* path) {
  return guarded([&] {
    require(c && path, MMC_ERR_INVALID, "null argument");
    require(c->loaded, MMC_ERR_STATE, "weights are not loaded");
    use_device(c);
    const std::string tmp = std::string(path) + ".tmp";
    {
      std::ofstream out(tmp, std::ios::binary | std::ios::trunc);
      require(bool(out), MMC_ERR_IO, "failed to create " + tmp);
      out.write(kPackedMagic, 8);
      out.write(reinterpret_cast<const char*>(&kPackedLayout), 4);
      out.write(reinterpret_cast<const char*>(&c->d), sizeof(mmc_model_desc));
      const int64_t moe[2] = {c->moe_experts, c->moe_inter};
      out.write(reinterpret_cast<const char*>(moe), sizeof(moe));
      std::vector<char> host;
      for (auto& [slot, bytes] : packed_buffers(c, false)) {
        host.resize(bytes);
        ck(cudaMemcpy(host.data(), *slot, bytes, cudaMemcpyDeviceToHost), "D2H packed weights");
        const uint64_t n = bytes;
        out.write(reinterpret_cast<const char*>(&n), 8);
        out.write(host.data(), std::streamsize(bytes));
      }
      require(bool(out), MMC_ERR_IO, "failed to write " + tmp);
    }
    require(std::rename(tmp.c_str(), path) == 0, MMC_ERR_IO, std::string("failed to rename to ") + path);
  });
}

int mmc_load_packed(mmc_ctx* c, const char* path) {
  return guarded([&] {
    require(c && path, MMC_ERR_INVALID, "null argument");
    require(!c->loaded, MMC_ERR_STATE, "weights already loaded");
    use_device(c);
    std::ifstream in(path, std::ios::binary);
    require(bool(in), MMC_ERR_IO, std::string("failed to open packed weights: ") + path);
    char magic[8] = {};
    uint32_t layout = 0;
    mmc_model_desc d{};
    in.read(magic, 8);
    in.read(reinterpret_cast<char*>(&layout), 4);
    in.read(reinterpret_cast<char*>(&d), sizeof(d));
    int64_t moe[2] = {0, 0};
    in.read(reinterpret_cast<char*>(moe), sizeof(moe));
    require(bool(in) && std::memcmp(magic, kPackedMagic, 8) == 0 && layout == kPackedLayout, MMC_ERR_IO,
            "not a packed weight cache of this library version");
    require(std::memcmp(&d, &c->d, sizeof(d)) == 0 && moe[0] == c->moe_experts && moe[1] == c->moe_inter,
            MMC_ERR_INVALID, "packed weights were made for another model");
    // read everything before allocating, so a short file leaves the context unloaded
    c->layers.assign(size_t(c->d.num_hidden_layers), Layer{});
    auto slots = packed_buffers(c, false);  // sizes only (pointers not yet allocated)
    std::vector<std::vector<char>> host;
    for (auto& [slot, bytes] : slots) {
      uint64_t n = 0;
      in.read(reinterpret_cast<char*>(&n), 8);
      require(bool(in) && n == bytes, MMC_ERR_IO, "packed weight cache is truncated or corrupt");
      host.emplace_back(bytes);
      in.read(host.back().data(), std::streamsize(bytes));
      require(bool(in), MMC_ERR_IO, "packed weight cache is truncated");
    }
    auto dev = packed_buffers(c, true);
    for (size_t i = 0; i < dev.size(); ++i) upload(c, *dev[i].first, host[i].data(), dev[i].second, "packed upload");
    finish_load(c);
  });
}

int mmc_kv_page_bytes(const mmc_ctx* c, int64_t* bytes) {
  return guarded([&] {
    require(c && bytes, MMC_ERR_INVALID, "null argument");
    *bytes = c->d.num_hidden_layers * 2 * c->d.num_key_value_heads * mmc::kPageTokens * c->d.head_dim * 2;
  });
}

int mmc_kv_init(mmc_ctx* c, int64_t n_pages, int32_t max_seqs, int32_t max_batch) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    require(!c->kv_ready, MMC_ERR_STATE, "KV cache already initialised");
    require(n_pages > 0 && n_pages < (int64_t(1) << 31) && max_seqs > 0 && max_batch > 0, MMC_ERR_INVALID,
            "n_pages, max_seqs and max_batch must be positive");
    use_device(c);
    const auto& d = c->d;
    c->page_halves = d.num_hidden_layers * 2 * d.num_key_value_heads * mmc::kPageTokens * d.head_dim;
    c->n_pages = n_pages;
    c->max_seqs = max_seqs;
    c->max_batch = max_batch;
    c->max_pages = int((d.max_position_embeddings + mmc::kPageTokens - 1) / mmc::kPageTokens);
    c->kv_pool = c->alloc<__half>(size_t(n_pages) * c->page_halves, "KV page pool");
    c->d_block_table = c->alloc<int>(size_t(max_seqs) * c->max_pages, "block table");
    c->d_seq_pos = c->alloc<int>(size_t(max_seqs), "positions");
    c->h_block_table.assign(size_t(max_seqs) * c->max_pages, -1);
    upload(c, c->d_block_table, c->h_block_table.data(), c->h_block_table.size() * 4, "block table init");
    c->h_pos.assign(size_t(max_seqs), 0);
    c->h_pages.assign(size_t(max_seqs), 0);
    c->h_open.assign(size_t(max_seqs), 0);
    c->free_pages.resize(size_t(n_pages));
    for (int64_t i = 0; i < n_pages; ++i) c->free_pages[size_t(i)] = int(n_pages - 1 - i);
    const int H = int(d.hidden_size), I = int(d.intermediate_size), Q = c->q_size(), KV = c->kv_size();
    const int V = int(d.vocab_size);
    c->hidden = c->alloc<float>(size_t(max_batch) * H, "hidden");
    c->qkv = c->alloc<float>(size_t(max_batch) * (Q + 2 * KV), "qkv");
    c->attn = c->alloc<float>(size_t(max_batch) * Q, "attn");
    const int64_t IA = std::max<int64_t>(I, c->moe_inter);  // MLP activation width (dense or expert)
    c->act = c->alloc<float>(size_t(max_batch) * IA, "act");
    c->expert_ids = c->alloc<int>(size_t(max_batch), "routed experts");
    c->h16 = c->alloc<__half>(size_t(max_batch) * H, "residual rows fp16");
    c->attn16 = c->alloc<__half>(size_t(max_batch) * Q, "attention output fp16");
    c->act16 = c->alloc<__half>(size_t(max_batch) * IA, "act fp16");
    c->q16 = c->alloc<__half>(size_t(max_batch) * Q, "q fp16");
    c->logits = c->alloc<float>(size_t(max_batch) * V, "logits");
    c->tokens = c->alloc<int>(size_t(max_batch), "tokens");
    c->slots = c->alloc<int>(size_t(max_batch), "slots");
    c->next = c->alloc<int>(size_t(max_batch), "next");
    c->row_off = c->alloc<int>(size_t(max_batch), "prompt row offsets");
    c->attn_order = c->alloc<int>(size_t(max_batch), "attention row order");
    ck(cudaMallocHost(&c->h_order, sizeof(int) * size_t(max_batch)), "pinned attention row order");
    size_t part_bytes = 0;
    for (int b = 1; b <= std::min(max_batch, 4); ++b)
      part_bytes = std::max(part_bytes, mmc::gemv_argmax_part_bytes(V, H, b, c->num_sms));
    part_bytes = std::max(part_bytes, mmc::tc_argmax_part_bytes(V, max_batch));
    c->part_cap = int(std::max<int64_t>((V + 127) / 128, mmc::skinny_grid(int(V), c->num_sms)));
    part_bytes = std::max(part_bytes, size_t(max_batch) * c->part_cap * 8);
    c->argmax_part = c->alloc<uint8_t>(part_bytes, "argmax partials");
    c->argmax_counter = c->alloc<unsigned>(kMaxParts * (size_t(max_batch) + 2), "argmax counters (per batch part)");
    c->attn_part = c->alloc<float>(
        mmc::attn_part_floats(max_batch, int(d.num_key_value_heads), c->max_splits_cap, c->rep(), int(d.head_dim)),
        "attention partials");
    c->attn_counters = c->alloc<unsigned>(size_t(max_batch) * d.num_key_value_heads, "attention counters");
    c->attn_work = c->alloc<unsigned>(4 * size_t(kMaxParts) * d.num_hidden_layers,
                                      "attention work queues (per batch part and layer)");
    c->chain_words = mmc::chain_sync_words(max_batch);
    c->chain_sync = c->alloc<unsigned>(size_t(kMaxParts) * c->chain_words, "projection-chain queues (per batch part)");
    c->ss_cap = int(std::max<int64_t>((H + 127) / 128, mmc::skinny_grid(int(H), c->num_sms)));
    c->ss = c->alloc<float>(size_t(max_batch) * c->ss_cap, "residual sums of squares");
    if (c->lm_f != nullptr) {  // persistent step scratch (its batches have at most kStepMaxRows rows)
      const size_t rows = size_t(std::min(max_batch, kStepMaxRows));
      c->step_ssp = c->alloc<float>(rows * (H / 16), "step sums of squares");
      c->step_part = c->alloc<float>(rows * d.num_key_value_heads * size_t(c->max_pages) * c->rep() *
                                         size_t(d.head_dim + 2),
                                     "step attention partials");
      c->step_arrive = c->alloc<unsigned>(rows * d.num_key_value_heads, "step job arrivals");
      c->step_lm_part = c->alloc<uint8_t>(size_t(mmc::kStepMaxGroups) * (V / 16) * mmc::kStepGroupRows * 8,
                                          "step argmax partials");
      c->step_sync = c->alloc<unsigned>(mmc::kStepSyncWords, "step counters");
    }
    ck(cudaMallocHost(&c->h_stage, sizeof(int) * 4 * size_t(max_batch)), "pinned staging");
    ck(cudaDeviceSynchronize(), "KV init");
    c->kv_ready = true;
  });
}

int mmc_seq_open(mmc_ctx* c, int64_t reserve_tokens, int32_t* seq_out) {
  return guarded([&] {
    require(c && seq_out, MMC_ERR_INVALID, "null argument");
    require(c->kv_ready, MMC_ERR_STATE, "KV cache is not initialised (mmc_kv_init)");
    use_device(c);
    int s = -1;
    for (int i = 0; i < c->max_seqs; ++i)
      if (!c->h_open[i]) {
        s = i;
        break;
      }
    require(s >= 0, MMC_ERR_NO_PAGES, "all sequence slots are in use");
    c->h_open[s] = 1;
    c->h_pos[s] = 0;
    c->h_pages[s] = 0;
    const int zero = 0;
    upload(c, c->d_seq_pos + s, &zero, sizeof(int), "position reset");
    try {
      reserve_pages(c, s, std::max<int64_t>(reserve_tokens, 1));
    } catch (...) {
      c->h_open[s] = 0;
      throw;
    }
    *seq_out = s;
  });
}

int mmc_seq_reserve(mmc_ctx* c, int32_t seq, int64_t tokens) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    check_seq(c, seq);
    reserve_pages(c, seq, tokens);
  });
}

int mmc_seq_close(mmc_ctx* c, int32_t seq) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    check_seq(c, seq);
    ck(cudaStreamSynchronize(c->stream), "drain before close");
    for (int p = 0; p < c->h_pages[seq]; ++p) {
      int& e = c->h_block_table[size_t(seq) * c->max_pages + p];
      c->free_pages.push_back(e);
      e = -1;
    }
    if (c->h_pages[seq] > 0)
      upload(c, c->d_block_table + size_t(seq) * c->max_pages, c->h_block_table.data() + size_t(seq) * c->max_pages,
             sizeof(int) * c->h_pages[seq], "block table upload");
    c->h_pages[seq] = 0;
    c->h_open[seq] = 0;
    c->h_pos[seq] = 0;
    if (std::find(c->graph_slots.begin(), c->graph_slots.end(), seq) != c->graph_slots.end()) drop_graph(c);
  });
}

int mmc_seq_position(const mmc_ctx* c, int32_t seq, int64_t* pos) {
  return guarded([&] {
    require(c && pos, MMC_ERR_INVALID, "null argument");
    check_seq(c, seq);
    *pos = c->h_pos[seq];
  });
}

int mmc_debug_read_kv(mmc_ctx* c, int32_t seq, int32_t layer, float* keys, float* values) {
  return guarded([&] {
    require(c && keys && values, MMC_ERR_INVALID, "null argument");
    require_ready(c);
    use_device(c);
    check_seq(c, seq);
    require(layer >= 0 && layer < c->d.num_hidden_layers, MMC_ERR_INVALID, "layer out of range");
    ck(cudaStreamSynchronize(c->stream), "sync");
    const int hd = int(c->d.head_dim), nkv = int(c->d.num_key_value_heads), cpr = hd / 8;
    const int64_t tile = int64_t(mmc::kPageTokens) * hd;
    std::vector<__half> slab(static_cast<size_t>(tile));
    const int64_t n = c->h_pos[seq];
    for (int64_t p0 = 0; p0 < n; p0 += mmc::kPageTokens) {
      const int page = c->h_block_table[size_t(seq) * c->max_pages + p0 / mmc::kPageTokens];
      for (int kv = 0; kv < 2; ++kv)
        for (int h = 0; h < nkv; ++h) {
          const size_t off = ((((size_t)page * c->d.num_hidden_layers + layer) * 2 + kv) * nkv + h) * size_t(tile);
          ck(cudaMemcpy(slab.data(), c->kv_pool + off, size_t(tile) * 2, cudaMemcpyDeviceToHost), "read page");
          for (int r = 0; r < mmc::kPageTokens && p0 + r < n; ++r)
            for (int ch = 0; ch < cpr; ++ch)
              for (int e = 0; e < 8; ++e) {
                const __half v = slab[size_t(mmc_kv_row_offset(hd, r, ch) + e)];
                float* dst = kv ? values : keys;
                dst[size_t(((p0 + r) * nkv + h) * hd + ch * 8 + e)] = __half2float(v);
              }
        }
    }
  });
}

int mmc_debug_fill_kv(mmc_ctx* c, int32_t seq, int64_t n_tokens, uint32_t seed) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    require_ready(c);
    use_device(c);
    check_seq(c, seq);
    require(c->h_pos[seq] == 0, MMC_ERR_STATE, "fill needs an empty sequence");
    require(n_tokens >= 0 && n_tokens < c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE,
            "n_tokens outside [0, max_position_embeddings)");
    reserve_pages(c, seq, std::max<int64_t>(n_tokens + 1, 1));
    if (n_tokens > 0)
      ck(mmc::launch_fill_kv(c->kv_pool, c->d_block_table + size_t(seq) * c->max_pages, int(n_tokens),
                             c->page_halves, int(c->d.head_dim), seed, c->stream),
         "fill launch");
    const int pos = int(n_tokens);
    upload(c, c->d_seq_pos + seq, &pos, sizeof(int), "position");
    c->h_pos[seq] = n_tokens;
  });
}

int mmc_debug_scratch(mmc_ctx* c, int32_t which, float* host, int64_t count) {
  return guarded([&] {
    require(c && host && count >= 0, MMC_ERR_INVALID, "null argument");
    require_ready(c);
    use_device(c);
    const float* src = which == 0 ? c->hidden : which == 1 ? c->qkv : which == 2 ? c->attn : which == 3 ? c->act : nullptr;
    require(src != nullptr, MMC_ERR_INVALID, "unknown scratch buffer");
    const int64_t cap = int64_t(c->max_batch) * (which == 0 ? c->d.hidden_size : which == 1 ? c->q_size() + 2 * c->kv_size()
                                                  : which == 2 ? c->q_size() : c->d.intermediate_size);
    require(count <= cap, MMC_ERR_INVALID, "count exceeds the buffer");
    ck(cudaStreamSynchronize(c->stream), "sync");
    ck(cudaMemcpy(host, src, size_t(count) * 4, cudaMemcpyDeviceToHost), "scratch read");
  });
}

int mmc_debug_step_trace(mmc_ctx* c, uint64_t* host, int64_t max_tasks, int64_t* n_tasks) {
  return guarded([&] {
    require(c && host && n_tasks, MMC_ERR_INVALID, "null argument");
    require(c->step_trace != nullptr, MMC_ERR_STATE, "no step trace (MMC_STEP_TRACE=1 at creation)");
    use_device(c);
    ck(cudaStreamSynchronize(c->stream), "sync");
    const int64_t n = std::min<int64_t>(max_tasks, c->step_trace_tasks);
    ck(cudaMemcpy(host, c->step_trace, size_t(n) * 8 * 8, cudaMemcpyDeviceToHost), "trace read");
    *n_tasks = c->step_trace_tasks;
  });
}

int mmc_decode_step(mmc_ctx* c, int32_t batch, const int32_t* seq_ids, const int32_t* tokens, int32_t* next_tokens,
                    float* logits_host) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    require(tokens && next_tokens, MMC_ERR_INVALID, "null argument");
    StepIO io = plan_step(c, batch, seq_ids, /*auto_reserve=*/true);
    for (int b = 0; b < batch; ++b)
      require(tokens[b] >= 0 && tokens[b] < c->d.vocab_size, MMC_ERR_OUT_OF_RANGE,
              "token id out of vocabulary range");
    const bool use_graph = c->graph && !logits_host && batch == c->graph_batch &&
                           std::equal(seq_ids, seq_ids + batch, c->graph_slots.begin()) &&
                           std::all_of(seq_ids, seq_ids + batch,
                                       [&](int32_t q) { return c->h_pos[q] + 1 <= c->graph_cap_tokens; });
    // host staging: [slots][tokens][error word]; the slot list is uploaded only
    // when `slots` holds another one
    std::memcpy(c->h_stage + batch, tokens, sizeof(int) * batch);
    if (c->async_slots.size() != size_t(batch) || !std::equal(seq_ids, seq_ids + batch, c->async_slots.begin())) {
      std::memcpy(c->h_stage, seq_ids, sizeof(int) * batch);
      ck(cudaMemcpyAsync(c->slots, c->h_stage, sizeof(int) * batch, cudaMemcpyHostToDevice, c->stream), "H2D slots");
      c->async_slots.assign(seq_ids, seq_ids + batch);
    }
    ck(cudaMemcpyAsync(c->tokens, c->h_stage + batch, sizeof(int) * batch, cudaMemcpyHostToDevice, c->stream),
       "H2D tokens");
    io.slots = c->slots;
    io.tokens = c->tokens;
    io.logits = logits_host ? c->logits : nullptr;
    if (!use_graph && !use_step(c, io) && env_int("MMC_ATTN_ORDER", 1) != 0) {
      fill_attn_order(c, io, seq_ids, c->h_order);
      ck(cudaMemcpyAsync(c->attn_order, c->h_order, sizeof(int) * batch, cudaMemcpyHostToDevice, c->stream),
         "H2D attention order");
      io.order = c->attn_order;
    }
    // a graph replay's argmax epilogue writes the next tokens into the mapped
    // history as well: only the device error word is copied back
    const int* next_host = c->h_stage + 2 * batch;
    if (use_graph) {
      ck(cudaGraphLaunch(c->graph, c->stream), "graph launch");
      next_host = c->h_hist + size_t(c->hist_host % c->hist_cap) * c->graph_batch;
      ++c->hist_host;
    } else {
      enqueue_batch(c, io, c->stream);
      ck(cudaMemcpyAsync(c->h_stage + 2 * batch, c->tokens, sizeof(int) * batch, cudaMemcpyDeviceToHost, c->stream),
         "D2H next tokens");
    }
    // the device error word rides along (one synchronisation per step)
    ck(cudaMemcpyAsync(c->h_stage + 3 * batch, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream),
       "D2H error word");
    if (logits_host)
      ck(cudaMemcpyAsync(logits_host, c->logits, sizeof(float) * batch * c->d.vocab_size, cudaMemcpyDeviceToHost,
                         c->stream),
         "D2H logits");
    ck(cudaStreamSynchronize(c->stream), "decode step");
    raise_device_error(c, c->h_stage[3 * batch]);
    std::memcpy(next_tokens, next_host, sizeof(int) * batch);
    for (int b = 0; b < batch; ++b) c->h_pos[seq_ids[b]] += 1;
  });
}

int mmc_prefill(mmc_ctx* c, int32_t n_seqs, const int32_t* seq_ids, const int32_t* prompt_lens, const int32_t* tokens,
                int32_t* next_tokens) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    require_ready(c);
    require(n_seqs >= 1 && seq_ids && prompt_lens && tokens && next_tokens, MMC_ERR_INVALID, "null argument");
    stream_drain(c);
    // validate everything before anything runs
    int64_t total = 0;
    std::vector<char> seen(c->max_seqs, 0);
    for (int i = 0; i < n_seqs; ++i) {
      const int32_t s = seq_ids[i];
      check_seq(c, s);
      require(!seen[s], MMC_ERR_INVALID, "a sequence appears twice in one prompt pass");
      seen[s] = 1;
      require(prompt_lens[i] >= 1, MMC_ERR_INVALID, "empty prompt");
      require(c->h_pos[s] + prompt_lens[i] <= c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE,
              "prompt exceeds max_position_embeddings");
      total += prompt_lens[i];
    }
    for (int64_t t = 0; t < total; ++t)
      require(tokens[t] >= 0 && tokens[t] < c->d.vocab_size, MMC_ERR_OUT_OF_RANGE, "token id out of vocabulary range");
    for (int i = 0; i < n_seqs; ++i) reserve_pages(c, seq_ids[i], c->h_pos[seq_ids[i]] + prompt_lens[i]);

    // rows in prompt order, packed into passes of at most max_batch rows; a
    // row's position is its sequence's position at the start of the pass
    // plus its offset among that sequence's rows in the pass
    const int cap = c->max_batch;
    int* h_slots = c->h_stage;
    int* h_tok = c->h_stage + cap;
    int* h_off = c->h_stage + 2 * cap;
    int* h_next = c->h_stage + 3 * cap;
    int si = 0, ti = 0;  // next sequence / its next prompt token
    int64_t consumed = 0;
    while (consumed < total) {
      int rows = 0;
      std::vector<std::pair<int, int>> last_rows;  // (sequence index, row) of prompts that end in this pass
      std::vector<std::pair<int32_t, int>> advanced;  // (sequence, rows in this pass)
      int64_t total_pages = 0, max_ctx = 1;
      int64_t tok_base = 0;
      for (int i = 0; i < si; ++i) tok_base += prompt_lens[i];
      while (rows < cap && si < n_seqs) {
        const int32_t s = seq_ids[si];
        const int take = std::min(cap - rows, prompt_lens[si] - ti);
        for (int k = 0; k < take; ++k) {
          h_slots[rows + k] = s;
          h_tok[rows + k] = tokens[tok_base + ti + k];
          h_off[rows + k] = k;
          const int64_t ctx = c->h_pos[s] + k + 1;
          total_pages += (ctx + mmc::kPageTokens - 1) / mmc::kPageTokens;
          max_ctx = std::max(max_ctx, ctx);
        }
        advanced.emplace_back(s, take);
        rows += take;
        ti += take;
        if (ti == prompt_lens[si]) {
          last_rows.emplace_back(si, rows - 1);
          tok_base += prompt_lens[si];
          ++si;
          ti = 0;
        }
      }
      ck(cudaMemcpyAsync(c->slots, h_slots, sizeof(int) * rows, cudaMemcpyHostToDevice, c->stream), "H2D slots");
      ck(cudaMemcpyAsync(c->tokens, h_tok, sizeof(int) * rows, cudaMemcpyHostToDevice, c->stream), "H2D tokens");
      ck(cudaMemcpyAsync(c->row_off, h_off, sizeof(int) * rows, cudaMemcpyHostToDevice, c->stream), "H2D offsets");
      c->async_slots.clear();
      StepIO io;
      io.B = rows;
      io.split_tokens = plan_split(c, total_pages, max_ctx, &io.max_splits);
      io.total_pages = total_pages;
      io.max_ctx = max_ctx;
      io.slots = c->slots;
      io.tokens = c->tokens;
      io.row_off = c->row_off;
      enqueue_batch(c, io, c->stream);
      ck(cudaMemcpyAsync(h_next, c->tokens, sizeof(int) * rows, cudaMemcpyDeviceToHost, c->stream), "D2H tokens");
      ck(cudaStreamSynchronize(c->stream), "prompt pass");
      check_device_error(c);
      for (const auto& [i, r] : last_rows) next_tokens[i] = h_next[r];
      // advance the positions (host and device) by the rows each sequence had
      for (const auto& [s, n] : advanced) {
        c->h_pos[s] += n;
        const int v = int(c->h_pos[s]);
        upload(c, c->d_seq_pos + s, &v, sizeof(int), "position update");
      }
      consumed += rows;
    }
  });
}

int mmc_profile_step(mmc_ctx* c, int32_t batch, const int32_t* seq_ids, const int32_t* tokens, int32_t* next_tokens,
                     float* kind_ms, int32_t* kind_launches) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    require(tokens && next_tokens && kind_ms && kind_launches, MMC_ERR_INVALID, "null argument");
    StepIO io = plan_step(c, batch, seq_ids, /*auto_reserve=*/true);
    for (int b = 0; b < batch; ++b)
      require(tokens[b] >= 0 && tokens[b] < c->d.vocab_size, MMC_ERR_OUT_OF_RANGE,
              "token id out of vocabulary range");
    upload(c, c->slots, seq_ids, sizeof(int) * batch, "H2D slots");
    upload(c, c->tokens, tokens, sizeof(int) * batch, "H2D tokens");
    c->async_slots.clear();
    io.slots = c->slots;
    io.tokens = c->tokens;
    if (env_int("MMC_ATTN_ORDER", 1) != 0) {  // the profiled step runs the batch as one part
      fill_attn_order(c, io, seq_ids, c->h_order, /*whole=*/true);
      upload(c, c->attn_order, c->h_order, sizeof(int) * batch, "attention order");
      io.order = c->attn_order;
    }
    const int n = kernels_per_step(c, batch);
    std::vector<cudaEvent_t> ev(size_t(n) + 1);
    std::vector<int> kinds;
    for (auto& e : ev) ck(cudaEventCreate(&e), "event create");
    try {
      // hold the stream while the host enqueues the step, so the event gaps
      // measure device time rather than host launch latency
      ck(mmc::launch_hold(uint64_t(n) * 20000ull, c->stream), "hold launch");
      enqueue_step(c, io, c->stream, ev.data(), &kinds);
      ck(cudaStreamSynchronize(c->stream), "profiled step");
      check_device_error(c);
      for (int k = 0; k < mmc_kernel_kinds; ++k) {
        kind_ms[k] = 0.f;
        kind_launches[k] = 0;
      }
      for (int i = 0; i < int(kinds.size()); ++i) {
        float ms = 0.f;
        ck(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "event time");
        const int kind = kinds[size_t(i)];
        kind_ms[kind] += ms;
        kind_launches[kind] += 1;
      }
    } catch (...) {
      for (auto& e : ev) cudaEventDestroy(e);
      throw;
    }
    for (auto& e : ev) cudaEventDestroy(e);
    ck(cudaMemcpy(next_tokens, c->tokens, sizeof(int) * batch, cudaMemcpyDeviceToHost), "D2H next tokens");
    for (int b = 0; b < batch; ++b) c->h_pos[seq_ids[b]] += 1;
  });
}

int mmc_decode_step_async(mmc_ctx* c, int32_t batch, const int32_t* seq_ids, const int32_t* d_tokens,
                          int32_t* d_next, float* d_logits, void* stream) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    require(d_tokens && d_next, MMC_ERR_INVALID, "null argument");
    StepIO io = plan_step(c, batch, seq_ids, /*auto_reserve=*/true);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (c->async_slots.size() != size_t(batch) || !std::equal(seq_ids, seq_ids + batch, c->async_slots.begin())) {
      // the slot list changes rarely: upload it synchronously and remember it
      ck(cudaStreamSynchronize(s), "drain before slot upload");
      upload(c, c->slots, seq_ids, sizeof(int) * batch, "H2D slots");
      c->async_slots.assign(seq_ids, seq_ids + batch);
    }
    ck(cudaMemcpyAsync(c->tokens, d_tokens, sizeof(int) * batch, cudaMemcpyDeviceToDevice, s), "tokens");
    io.slots = c->slots;
    io.tokens = c->tokens;
    io.next_out = d_next;
    io.logits = d_logits;
    enqueue_batch(c, io, s);
    for (int b = 0; b < batch; ++b) c->h_pos[seq_ids[b]] += 1;
  });
}

int mmc_graph_build(mmc_ctx* c, int32_t batch, const int32_t* seq_ids) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    require_ready(c);
    require(batch >= 1 && batch <= c->max_batch && seq_ids, MMC_ERR_INVALID, "bad batch");
    drop_graph(c);
    int64_t total_pages = 0, cap = 1;
    for (int b = 0; b < batch; ++b) {
      check_seq(c, seq_ids[b]);
      const int64_t tok = int64_t(c->h_pages[seq_ids[b]]) * mmc::kPageTokens;
      total_pages += c->h_pages[seq_ids[b]];
      cap = std::max(cap, tok);
    }
    // validation of duplicates etc.
    (void)plan_step(c, batch, seq_ids, false);
    StepIO io;
    io.B = batch;
    io.split_tokens = plan_split(c, total_pages, cap, &io.max_splits);
    io.total_pages = total_pages;
    io.max_ctx = cap;
    if (!c->hist) {
      // the history lives in mapped pinned host memory: the lm_head argmax
      // epilogue writes each step's tokens straight to the host, so a
      // streamed run needs no copy between graph replays
      c->hist_cap = 8192;
      ck(cudaHostAlloc(reinterpret_cast<void**>(&c->h_hist), sizeof(int) * size_t(c->hist_cap) * c->max_batch,
                       cudaHostAllocMapped),
         "token history (mapped)");
      ck(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->hist), c->h_hist, 0), "token history device view");
      c->hist_step = c->alloc<int>(kMaxParts, "history counters (per batch part)");
    }
    upload(c, c->slots, seq_ids, sizeof(int) * batch, "slots");
    c->async_slots.clear();
    io.slots = c->slots;
    io.tokens = c->tokens;
    io.hist = c->hist;
    io.hist_step = c->hist_step;
    io.hist_cap = c->hist_cap;
    if (!use_step(c, io) && env_int("MMC_ATTN_ORDER", 1) != 0) {  // read by the captured attention launches
      fill_attn_order(c, io, seq_ids, c->h_order);
      upload(c, c->attn_order, c->h_order, sizeof(int) * batch, "attention order");
      io.order = c->attn_order;
    }
    cudaGraph_t g = nullptr;
    ck(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      enqueue_batch(c, io, c->stream);
    } catch (...) {
      cudaStreamEndCapture(c->stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    ck(cudaStreamEndCapture(c->stream, &g), "end capture");
    cudaError_t e = cudaGraphInstantiate(&c->graph, g, 0);
    cudaGraphDestroy(g);
    ck(e, "graph instantiate");
    c->graph_batch = batch;
    c->graph_slots.assign(seq_ids, seq_ids + batch);
    c->async_slots.assign(seq_ids, seq_ids + batch);  // uploaded above
    ck(cudaMemsetAsync(c->hist_step, 0, kMaxParts * sizeof(int), c->stream), "history reset");
    c->hist_host = 0;
    c->graph_cap_tokens = plan_cap_tokens(c, io);
  });
}

int mmc_graph_set_tokens(mmc_ctx* c, const int32_t* tokens) {
  return guarded([&] {
    require(c && tokens && c->graph, MMC_ERR_STATE, "no graph built");
    use_device(c);
    for (int b = 0; b < c->graph_batch; ++b)
      require(tokens[b] >= 0 && tokens[b] < c->d.vocab_size, MMC_ERR_OUT_OF_RANGE, "token id out of vocabulary range");
    upload(c, c->slots, c->graph_slots.data(), sizeof(int) * c->graph_batch, "slots");
    c->async_slots = c->graph_slots;
    upload(c, c->tokens, tokens, sizeof(int) * c->graph_batch, "tokens");
  });
}

int mmc_graph_run(mmc_ctx* c, int32_t n_steps, void* stream) {
  return guarded([&] {
    require(c && c->graph, MMC_ERR_STATE, "no graph built");
    use_device(c);
    require(n_steps >= 0 && n_steps <= c->hist_cap, MMC_ERR_INVALID, "n_steps outside [0, 8192]");
    stream_drain(c);
    for (int s : c->graph_slots) {
      require(c->h_pos[s] + n_steps <= int64_t(c->h_pages[s]) * mmc::kPageTokens, MMC_ERR_NO_PAGES,
              "graph run needs more reserved KV pages (mmc_seq_reserve)");
      require(c->h_pos[s] + n_steps <= c->graph_cap_tokens, MMC_ERR_STATE,
              "graph run goes past the positions the graph was built for (rebuild it)");
      require(c->h_pos[s] + n_steps <= c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE,
              "position exceeds max_position_embeddings");
    }
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    ck(cudaMemsetAsync(c->hist_step, 0, kMaxParts * sizeof(int), st), "history reset");
    for (int i = 0; i < n_steps; ++i) ck(cudaGraphLaunch(c->graph, st), "graph launch");
    c->hist_host = n_steps;
    for (int s : c->graph_slots) c->h_pos[s] += n_steps;
  });
}

int mmc_graph_stream_start(mmc_ctx* c, int32_t n_steps) {
  return guarded([&] {
    require(c && c->graph, MMC_ERR_STATE, "no graph built");
    use_device(c);
    require(n_steps >= 1, MMC_ERR_INVALID, "n_steps must be positive");
    stream_drain(c);
    for (int s : c->graph_slots) {
      require(c->h_pos[s] + n_steps <= int64_t(c->h_pages[s]) * mmc::kPageTokens, MMC_ERR_NO_PAGES,
              "streamed run needs more reserved KV pages (mmc_seq_reserve)");
      require(c->h_pos[s] + n_steps <= c->graph_cap_tokens, MMC_ERR_STATE,
              "streamed run goes past the positions the graph was built for (rebuild it)");
      require(c->h_pos[s] + n_steps <= c->d.max_position_embeddings, MMC_ERR_OUT_OF_RANGE,
              "position exceeds max_position_embeddings");
    }
    if (!c->h_ring) {
      ck(cudaHostAlloc(reinterpret_cast<void**>(&c->h_ring), sizeof(int) * kRingSlots, cudaHostAllocDefault),
         "pinned error words");
      for (auto& e : c->ring_ev) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "ring event");
    }
    ck(cudaMemsetAsync(c->hist_step, 0, kMaxParts * sizeof(int), c->stream), "history reset");
    c->hist_host = 0;
    c->st_total = n_steps;
  });
}

namespace {
// keep up to kRingSlots replays in flight ahead of the host's reads (each
// replay's tokens land in the mapped history; an event marks its end, and
// every 8th replay also copies the device error word); positions advance as
// each replay is enqueued
void stream_top_up(mmc_ctx* c) {
  while (c->st_enqueued < c->st_total && c->st_enqueued < c->st_consumed + kRingSlots) {
    const int slot = int(c->st_enqueued % kRingSlots);
    ck(cudaGraphLaunch(c->graph, c->stream), "graph launch");
    ++c->hist_host;
    c->h_ring[slot] = 0;
    if (c->st_enqueued % 8 == 7 || c->st_enqueued + 1 == c->st_total)
      ck(cudaMemcpyAsync(c->h_ring + slot, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream), "D2H error word");
    ck(cudaEventRecord(c->ring_ev[slot], c->stream), "ring event");
    for (int s : c->graph_slots) c->h_pos[s] += 1;
    ++c->st_enqueued;
  }
}
}  // namespace

int mmc_graph_stream_next(mmc_ctx* c, int32_t* tokens) {
  return guarded([&] {
    require(c && tokens, MMC_ERR_INVALID, "null argument");
    require(c->graph && c->st_consumed < c->st_total, MMC_ERR_STATE, "no streamed step left (mmc_graph_stream_start)");
    use_device(c);
    stream_top_up(c);
    const int slot = int(c->st_consumed % kRingSlots);
    ck(cudaEventSynchronize(c->ring_ev[slot]), "streamed step");
    const int B = c->graph_batch;
    if (c->h_ring[slot] != 0) {
      const int e = c->h_ring[slot];
      stream_drain(c);
      raise_device_error(c, e);
    }
    const int* row = c->h_hist + size_t(c->st_consumed % c->hist_cap) * B;
    std::memcpy(tokens, row, sizeof(int) * B);
    ++c->st_consumed;
    if (c->st_consumed == c->st_total) c->st_total = c->st_enqueued = c->st_consumed = 0;
    else stream_top_up(c);
  });
}

int mmc_graph_stream_stop(mmc_ctx* c) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    stream_drain(c);
    check_device_error(c);
  });
}

int mmc_graph_tokens(mmc_ctx* c, int32_t n_steps, int32_t* tokens) {
  return guarded([&] {
    require(c && c->graph && tokens, MMC_ERR_STATE, "no graph built");
    use_device(c);
    require(n_steps >= 0 && n_steps <= c->hist_cap, MMC_ERR_INVALID, "n_steps out of range");
    ck(cudaStreamSynchronize(c->stream), "sync");
    ck(cudaDeviceSynchronize(), "sync");
    check_device_error(c);
    std::memcpy(tokens, c->h_hist, sizeof(int) * size_t(n_steps) * c->graph_batch);
  });
}

int mmc_synchronize(mmc_ctx* c) {
  return guarded([&] {
    require(c != nullptr, MMC_ERR_INVALID, "null context");
    use_device(c);
    ck(cudaStreamSynchronize(c->stream), "sync");
    check_device_error(c);
  });
}

int mmc_kernels_per_step(const mmc_ctx* c, int32_t batch, int32_t* k) {
  return guarded([&] {
    require(c && k, MMC_ERR_INVALID, "null argument");
    require(batch >= 1, MMC_ERR_INVALID, "bad batch");
    if (c->lm_f != nullptr && c->step_sync != nullptr && batch <= kStepMaxRows) {  // the persistent step
      *k = 1;
      return;
    }
    // a batch that runs as concurrent parts launches each part's chain
    const int P = use_gemv(c, batch) ? 1 : batch_parts(c, batch);
    int total = 0;
    for (int i = 0; i < P; ++i) {
      int r0 = 0, n = batch;
      if (P > 1) part_rows(batch, P, i, &r0, &n);
      total += kernels_per_step(c, n, P == 1);
    }
    *k = total;
  });
}

// ------------------------------------------------------------- single ops

namespace {
// first bytes of an attention-op workspace: error word at 0, work queue at 16
constexpr size_t kOpAttnHeader = 256;
void op_init_attributes() {
  static thread_local int done_dev = -1;
  int dev = 0;
  ck(cudaGetDevice(&dev), "device");
  if (done_dev == dev) return;
  ck(mmc::gemv_init_attributes(), "attributes");
  ck(mmc::gemm_tc_init_attributes(), "attributes");
  ck(mmc::attention_init_attributes(), "attributes");
  done_dev = dev;
}
int current_sms() {
  int dev = 0, sms = 148;
  ck(cudaGetDevice(&dev), "device");
  ck(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "device query");
  return sms;
}
}  // namespace

int mmc_op_projection(int32_t batch, int32_t n, int32_t k, const void* w, const void* x, float* y, void* stream) {
  return guarded([&] {
    require(batch >= 1 && n > 0 && k > 0 && w && x && y, MMC_ERR_INVALID, "bad projection arguments");
    require(batch <= kGemvMaxBatch ? k % 8 == 0 : k % 64 == 0, MMC_ERR_INVALID,
            "k must be a multiple of 8 (batch <= 4) or 64 (batch > 4)");
    op_init_attributes();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (batch <= kGemvMaxBatch) {
      mmc::ProjArgs a;
      a.W = static_cast<const __half*>(w);
      a.N = n;
      a.K = k;
      a.B = batch;
      a.in = static_cast<const float*>(x);
      a.out = y;
      a.ldo = n;
      ck(mmc::launch_gemv(mmc::kProPlain, mmc::kEpiStore, a, current_sms(), s, false), "projection launch");
    } else {
      mmc::TcArgs t;
      t.W = static_cast<const __half*>(w);
      t.X = static_cast<const __half*>(x);
      t.N = n;
      t.K = k;
      t.B = batch;
      t.out = y;
      t.ldo = n;
      ck(mmc::launch_gemm_tc(mmc::kEpiStore, t, s, false), "projection launch");
    }
  });
}

int mmc_op_lm_head_argmax_workspace_size(int32_t batch, int32_t n, int32_t k, size_t* bytes) {
  return guarded([&] {
    require(batch >= 1 && n > 0 && k > 0 && bytes, MMC_ERR_INVALID, "bad arguments");
    const size_t part = batch <= kGemvMaxBatch ? mmc::gemv_argmax_part_bytes(n, k, batch, current_sms())
                                               : mmc::tc_argmax_part_bytes(n, batch);
    // partials | counters | token buffer
    *bytes = (part + 255) / 256 * 256 + size_t(mmc::tc_counter_words(n, batch) + 2) * 4 + size_t(batch) * 4 + 256;
  });
}

int mmc_op_lm_head_argmax(int32_t batch, int32_t n, int32_t k, const void* w, const void* x, float* logits,
                          int32_t* next, void* ws, size_t ws_bytes, void* stream) {
  return guarded([&] {
    size_t need = 0;
    if (mmc_op_lm_head_argmax_workspace_size(batch, n, k, &need) != MMC_OK) fail(MMC_ERR_INVALID, g_error);
    require(w && x && next && ws && ws_bytes >= need, MMC_ERR_INVALID, "bad arguments or workspace too small");
    require(batch <= kGemvMaxBatch ? k % 8 == 0 : k % 64 == 0, MMC_ERR_INVALID,
            "k must be a multiple of 8 (batch <= 4) or 64 (batch > 4)");
    op_init_attributes();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t part = batch <= kGemvMaxBatch ? mmc::gemv_argmax_part_bytes(n, k, batch, current_sms())
                                               : mmc::tc_argmax_part_bytes(n, batch);
    uint8_t* base = static_cast<uint8_t*>(ws);
    const size_t words = size_t(mmc::tc_counter_words(n, batch) + 2);
    unsigned* counters = reinterpret_cast<unsigned*>(base + (part + 255) / 256 * 256);
    int* tok = reinterpret_cast<int*>(counters + words);
    ck(cudaMemsetAsync(counters, 0, words * 4, s), "counter reset");
    mmc::TokenSink sink;
    sink.tokens = tok;
    sink.next_out = next;
    if (batch <= kGemvMaxBatch) {
      mmc::ProjArgs a;
      a.W = static_cast<const __half*>(w);
      a.N = n;
      a.K = k;
      a.B = batch;
      a.in = static_cast<const float*>(x);
      a.logits = logits;
      a.argmax_part = base;
      a.counter = counters;
      a.sink = sink;
      ck(mmc::launch_gemv(mmc::kProPlain, mmc::kEpiArgmax, a, current_sms(), s, false), "lm_head launch");
    } else {
      mmc::TcArgs t;
      t.W = static_cast<const __half*>(w);
      t.X = static_cast<const __half*>(x);
      t.N = n;
      t.K = k;
      t.B = batch;
      t.logits = logits;
      t.argmax_part = base;
      t.counter = counters;
      t.sink = sink;
      ck(mmc::launch_gemm_tc(mmc::kEpiArgmax, t, s, false), "lm_head launch");
    }
  });
}

int mmc_op_attention_workspace_size(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t max_ctx,
                                    size_t* bytes) {
  return guarded([&] {
    require(batch >= 1 && nkv >= 1 && nq % nkv == 0 && hd > 0 && max_ctx >= 1 && bytes, MMC_ERR_INVALID,
            "bad arguments");
    const int splits = std::min(64, (max_ctx + mmc::kPageTokens - 1) / mmc::kPageTokens);
    // header (error word, work queue) | arrival counters | split partials | q heads (fp16)
    *bytes = kOpAttnHeader + (size_t(batch) * nkv * 4 + 255) / 256 * 256 +
             (mmc::attn_part_floats(batch, nkv, splits, nq / nkv, hd) * 4 + 255) / 256 * 256 +
             size_t(batch) * nq * hd * 2;
  });
}

int mmc_op_attention(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t layer, int32_t layers,
                     const float* qkv, const float* q_norm, const float* k_norm, const float* rope_cos,
                     const float* rope_sin, int32_t max_pos, float eps, void* kv_pool, const int32_t* block_table,
                     int32_t max_pages, const int32_t* seq_pos, const int32_t* slots, int32_t max_ctx, float* out,
                     void* ws, size_t ws_bytes, void* stream) {
  return guarded([&] {
    size_t need = 0;
    if (mmc_op_attention_workspace_size(batch, nq, nkv, hd, max_ctx, &need) != MMC_OK) fail(MMC_ERR_INVALID, g_error);
    require(ws && ws_bytes >= need, MMC_ERR_INVALID, "workspace too small");
    op_init_attributes();
    // same split planner as the decode step; at most 64 splits, so the
    // workspace size above stays an upper bound
    const int64_t pages = (max_ctx + mmc::kPageTokens - 1) / mmc::kPageTokens;
    int max_splits = 1;
    const int split_tokens = plan_split_raw(int64_t(batch) * pages, nkv, current_sms(), 64, max_ctx, &max_splits);
    mmc::AttnArgs a;
    a.qkv = qkv;
    a.ld_qkv = (nq + 2 * nkv) * hd;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.rope_cos = rope_cos;
    a.rope_sin = rope_sin;
    a.max_pos = max_pos;
    a.eps = eps;
    a.kv_pool = static_cast<__half*>(kv_pool);
    a.layer = layer;
    a.layers = layers;
    a.block_table = block_table;
    a.max_pages = max_pages;
    a.seq_pos = seq_pos;
    a.slots = slots;
    a.B = batch;
    a.nq = nq;
    a.nkv = nkv;
    a.hd = hd;
    a.split_tokens = split_tokens;
    a.max_splits = max_splits;
    a.out = out;
    uint8_t* base = static_cast<uint8_t*>(ws);
    // workspace layout as sized by mmc_op_attention_workspace_size; the error
    // word is the first int, where mmc_op_attention_status reads it
    const int splits_ws = int(std::min<int64_t>(64, pages));
    const size_t cbytes = (size_t(batch) * nkv * 4 + 255) / 256 * 256;
    const size_t pbytes = (mmc::attn_part_floats(batch, nkv, splits_ws, nq / nkv, hd) * 4 + 255) / 256 * 256;
    a.err = reinterpret_cast<int*>(base);
    a.work = reinterpret_cast<unsigned*>(base + 16);
    a.counters = reinterpret_cast<unsigned*>(base + kOpAttnHeader);
    a.part = reinterpret_cast<float*>(base + kOpAttnHeader + cbytes);
    a.q16 = reinterpret_cast<__half*>(base + kOpAttnHeader + cbytes + pbytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ck(cudaMemsetAsync(base, 0, kOpAttnHeader + size_t(batch) * nkv * 4, s), "counter reset");
    ck(mmc::launch_attention(a, s, false), "attention launch");
  });
}

int mmc_op_attention_status(const void* ws, void* stream) {
  return guarded([&] {
    require(ws != nullptr, MMC_ERR_INVALID, "null workspace");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int e = 0;
    ck(cudaMemcpyAsync(&e, ws, sizeof(int), cudaMemcpyDeviceToHost, s), "read attention error word");
    ck(cudaStreamSynchronize(s), "read attention error word");
    if (e != 0) {
      ck(cudaMemsetAsync(const_cast<void*>(ws), 0, sizeof(int), s), "clear attention error word");
      ck(cudaStreamSynchronize(s), "clear attention error word");
      fail(MMC_ERR_DEVICE, std::string("device error: ") + device_error_text(e) + " (code " + std::to_string(e) + ")");
    }
  });
}

int64_t mmc_kv_row_offset(int32_t hd, int32_t row, int32_t chunk) {
  const int cpr = hd / 8;
  const int x = (cpr % 8 == 0) ? (row & 7) : ((cpr % 4 == 0) ? ((row >> 1) & 3) : ((row >> 2) & 1));
  return int64_t(row) * hd + int64_t(chunk ^ x) * 8;
}

}  // extern "C"
