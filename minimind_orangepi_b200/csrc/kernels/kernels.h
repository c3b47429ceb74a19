// Host-side launch interface of the decode kernels. No torch types; plain
// device pointers. All launches go on the caller's stream and, when `pdl` is
// set, carry programmatic stream serialization so a kernel's weight prefetch
// overlaps the tail of the kernel before it.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmc {

// Error codes a kernel can leave in the context's device error word.
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,    // a bounded mbarrier wait gave up
  kDevBadToken = 2,       // token id outside [0, vocab)
  kDevNoPage = 3,         // KV position not backed by a reserved page
  kDevPositionLimit = 4,  // position >= max_position_embeddings
};

// Prologue: how a projection kernel builds its input rows x[b][0..K).
enum Prologue : int {
  kProPlain = 0,      // x = in[b]                              (fp32 activations)
  kProNorm = 1,       // x = in[b] * rs (w folded into W)       decoder_layer.cpp:32-42
  kProNormFinal = 2,  // final norm, same form                  language_model.cpp:24-38
  kProEmbedNorm = 3,  // in[b] = embed[token[b]] (also written to `hidden`), then kProNorm
};

// Epilogue: what a projection kernel does with y[b][n] = W[n] . x[b].
enum Epilogue : int {
  kEpiStore = 0,   // out[b][n] = y
  kEpiResid = 1,   // out[b][n] += y               (residual stream, fp32)
  kEpiSwiglu = 2,  // out[b][i] = silu(gate_i) * up_i   (gate/up rows interleaved by 8)
  kEpiArgmax = 3,  // next token = first argmax_n y (optionally logits[b][n] = y)
};

// Per-step bookkeeping the lm_head argmax epilogue updates once the next
// token is known (device-resident decode loop).
struct TokenSink {
  int* tokens = nullptr;          // [B] in: this step's tokens; out: next tokens (feedback)
  int* next_out = nullptr;        // [B] optional copy of the next tokens
  int* seq_pos = nullptr;         // [max_seqs] position (cached tokens) per sequence slot, += 1
  const int* slots = nullptr;     // [B] sequence slot of each batch row
  int* hist = nullptr;            // optional [hist_cap][B] token history
  int* hist_step = nullptr;       // device counter of history rows written
  int hist_cap = 0;
  int hist_stride = 0;            // elements between history rows
};

struct ProjArgs {
  const __half* W = nullptr;  // [N][K] row-major fp16
  int N = 0, K = 0, B = 0;
  // prologue
  const float* in = nullptr;  // [B][K] fp32 (hidden / activations)
  float eps = 0.f;  // RMSNorm prologues (x * rs; the norm weight is folded into W)
  const float* embed = nullptr;  // [vocab][K] fp32
  int vocab = 0;
  const int* tokens = nullptr;
  float* hidden = nullptr;  // kProEmbedNorm writes the embedding rows here
  // epilogue
  float* out = nullptr;  // [B][ldo]
  int ldo = 0;
  const int* row_sel = nullptr;  // kEpiResid: update only rows b with row_sel[b] == row_sel_val (MoE)
  int row_sel_val = 0;
  float* logits = nullptr;  // kEpiArgmax: optional [B][N]
  void* argmax_part = nullptr;  // kEpiArgmax scratch: [B][grid] (value, index)
  unsigned* counter = nullptr;  // kEpiArgmax: zero-initialised arrival counter
  TokenSink sink;
  int* err = nullptr;
};

// CUDA-core projection for small batches (B <= 4): each CTA bulk-copies its
// contiguous weight slab into shared memory before waiting on the previous
// kernel, then computes all B rows from shared memory.
int gemv_rows_per_cta(int N, int K, int epi, int num_sms);
size_t gemv_smem_bytes(int rows_per_cta, int K, int B);
size_t gemv_argmax_part_bytes(int N, int K, int B, int num_sms);
cudaError_t launch_gemv(int pro, int epi, const ProjArgs& a, int num_sms, cudaStream_t stream, bool pdl);
cudaError_t gemv_init_attributes();

// Tensor-core projection for batches B > 4 (tcgen05.mma, fp16 operands, fp32
// accumulate in TMEM): weight rows on the UMMA M side, batch rows on N.
struct TcArgs {
  CUtensorMap map_w;  // filled by launch_gemm_tc (TMA descriptors of W and X)
  CUtensorMap map_x;
  const __half* W = nullptr;  // [N][K] fp16
  const __half* X = nullptr;  // [B][K] fp16 activations
  int N = 0, K = 0, B = 0;
  float* out = nullptr;     // kEpiStore / kEpiResid: [B][ldo] fp32
  __half* out16 = nullptr;  // kEpiSwiglu: [B][ldo] fp16
  int ldo = 0;
  float* logits = nullptr;       // kEpiArgmax: optional [B][N]
  void* argmax_part = nullptr;   // kEpiArgmax: [B][ceil(N/128)] (value, index)
  unsigned* counter = nullptr;   // kEpiArgmax: tc_counter_words zeroed words
  TokenSink sink;
  int* err = nullptr;
  // split-K: gridDim.z = splits CTAs of one tile form a thread-block cluster
  // and reduce their accumulators over distributed shared memory (fixed order)
  int splits = 1;      // set by the launcher
  int max_splits = 8;  // caller's cap (1: never split)
  int split_bn = 0;    // batch tile when splitting (0: the planner's default)
  // RMSNorm folded across kernels (the norm weight is folded into W's
  // columns at load time): a consumer with ss_in scales its outputs by
  // rs[b] = 1 / sqrt(sum_m ss_in[b][m] / K + eps), m < ceil(K / 128); a
  // kEpiResid producer writes the fp16 copy of the updated residual rows
  // (h16_out, [B][N]) and its per-M-tile sums of squares
  // (ss_out[b][blockIdx.x], stride ceil(N / 128)).
  const float* ss_in = nullptr;
  float eps = 0.f;
  __half* h16_out = nullptr;
  float* ss_out = nullptr;
  const int* row_sel = nullptr;  // kEpiResid: update only rows b with row_sel[b] == row_sel_val (MoE)
  int row_sel_val = 0;
};
// Small-batch projection (5..64 rows) on mma.sync (skinny.cu): weights in
// the skinny fragment order (launch_pack_skinny), each CTA owning T 16-row
// tiles over the full K; inputs, outputs and the folded RMSNorm as TcArgs,
// except that sums of squares are per CTA: a consumer reads ss_parts partials
// per row (ss_in[b * ss_parts + m]); a kEpiResid producer writes
// skinny_grid(N) of them (ss_out[b * grid + blockIdx.x]).
constexpr int kSkinnyMaxBatch = 64;
constexpr int kSkinnyMaxSmem = 200 * 1024;
struct SkinnyArgs {
  const __half* Wf = nullptr;  // [N / 16 tiles][K / 32 blocks][2 steps][32 lanes][8 halves]
  const __half* X = nullptr;   // [B][K] fp16
  int N = 0, K = 0, B = 0;
  int T = 1;  // tiles per CTA (set by the launcher)
  float* out = nullptr;     // kEpiStore / kEpiResid: [B][ldo] fp32
  __half* out16 = nullptr;  // kEpiSwiglu: [B][ldo] fp16
  int ldo = 0;
  const float* ss_in = nullptr;
  int ss_parts = 0;
  float eps = 0.f;
  __half* h16_out = nullptr;  // kEpiResid: [B][N] fp16 copy of the updated rows
  float* ss_out = nullptr;
  const int* row_sel = nullptr;
  int row_sel_val = 0;
  float* logits = nullptr;       // kEpiArgmax: optional [B][N]
  void* argmax_part = nullptr;   // kEpiArgmax: [B][grid] (value, index)
  unsigned* counter = nullptr;   // kEpiArgmax: one zeroed, self-resetting word
  TokenSink sink;
  int* err = nullptr;
};
int skinny_tiles_per_cta(int N, int num_sms);
int skinny_grid(int N, int num_sms);
size_t skinny_smem_bytes(int N, int K, int B, int num_sms);
bool skinny_supported(int N, int K, int B, int num_sms);
cudaError_t skinny_init_attributes();
cudaError_t launch_skinny(int epi, const SkinnyArgs& a, int num_sms, cudaStream_t stream, bool pdl);
cudaError_t launch_pack_skinny(const __half* src, __half* dst, int64_t N, int64_t K, cudaStream_t s);

int tc_batch_tile(int N, int B);
// split-K factor the launcher uses for this projection (1 = none)
// (environment overrides MMC_TC_SPLIT, MMC_TC_SPLIT_BN, MMC_TC_SPLIT_TARGET)
int tc_split_k(const TcArgs& a, int epi);
size_t tc_argmax_part_bytes(int N, int B);
int tc_counter_words(int N, int B);
cudaError_t launch_gemm_tc(int epi, const TcArgs& a, cudaStream_t stream, bool pdl);
cudaError_t gemm_tc_init_attributes();

// Back half of a decoder layer on the tensor-core path as one persistent
// launch (o projection + residual, gate/up + SwiGLU with the folded
// post-attention norm, down projection + residual), tasks in dependency order
// from an atomic queue (mlp_chain.cu).
struct ChainArgs {
  CUtensorMap map_w[3];  // filled by launch_mlp_chain
  CUtensorMap map_x[3];
  const __half* Wo = nullptr;     // [H][Q]
  const __half* Wgu = nullptr;    // [2I][H], gate/up interleaved by 8 rows, post-attention norm folded in
  const __half* Wdown = nullptr;  // [H][I]
  const __half* attn16 = nullptr;  // [B][Q] attention output
  float* hidden = nullptr;  // [B][H] residual stream (updated twice)
  __half* h16 = nullptr;    // [B][H] fp16 residual rows (written twice)
  float* ss = nullptr;      // [B][H / 128] sums of squares (written twice)
  __half* act16 = nullptr;  // [B][I]
  int N[3] = {0, 0, 0}, K[3] = {0, 0, 0};  // o: H x Q, gate/up: 2I x H, down: H x I
  int B = 0;
  float eps = 0.f;
  unsigned* sync = nullptr;  // chain_sync_words(B) zeroed words, self-resetting
  int* err = nullptr;
  int m_tiles[3] = {0, 0, 0}, n_tiles = 0;  // set by the launcher
};
int chain_sync_words(int B);
cudaError_t launch_mlp_chain(const ChainArgs& a, int max_ctas, cudaStream_t stream, bool pdl);
cudaError_t mlp_chain_init_attributes();

// Layer-0 input of the tensor-core path: gathers embedding rows into the
// residual stream, its fp16 copy and the sums of squares the first
// projection's folded RMSNorm needs.
struct EmbedArgs {
  const float* embed = nullptr;  // [vocab][H]
  const int* tokens = nullptr;
  int vocab = 0;
  float* hidden = nullptr;   // [B][H]
  __half* h16 = nullptr;     // [B][H]
  float* ss = nullptr;       // [B][ceil(H / 128)]: slot 0 = sum of squares, others 0
  int B = 0, H = 0;
  int* err = nullptr;
};
cudaError_t launch_embed_rows(const EmbedArgs& a, cudaStream_t stream, bool pdl);

// Fused decode attention: q/k per-head RMSNorm + rotate-half RoPE and K/V
// append into the paged cache (prep launch), then split-KV GQA flash-decode
// over the cache with split combine (persistent launch). Two launches per layer.
struct AttnArgs {
  const float* qkv = nullptr;  // [B][(nq + 2 nkv) * hd] raw projections (fp32)
  int ld_qkv = 0;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  const float* rope_cos = nullptr;  // [max_pos][hd/2]
  const float* rope_sin = nullptr;
  int max_pos = 0;
  float eps = 0.f;
  __half* kv_pool = nullptr;  // pages [n_pages][layers][2][nkv][page][hd] (fp16, swizzled rows)
  int layer = 0, layers = 0;
  const int* block_table = nullptr;  // [max_seqs][max_pages]
  int max_pages = 0;
  const int* seq_pos = nullptr;  // [max_seqs] tokens cached before this step
  const int* slots = nullptr;    // [B]
  const int* row_off = nullptr;  // optional [B]: row b sits at seq_pos[slots[b]] + row_off[b] (prompt pass)
  const int* order = nullptr;    // optional [B]: work-queue order of the rows (longest work items first)
  // fused (decode steps: one row per sequence): the attention kernel does the
  // q/k RMSNorm + RoPE and the K/V append itself from the raw projections, and
  // the prep launch is skipped (a prompt pass, whose rows read each other's
  // appended rows, keeps the prep launch)
  int fused = 0;
  int B = 0, nq = 0, nkv = 0, hd = 0;
  int split_tokens = 0;  // multiple of the page size
  int max_splits = 0;    // grid.x
  float* out = nullptr;     // [B][nq * hd] fp32, or
  __half* out16 = nullptr;  // [B][nq * hd] fp16 when set (tensor-core path)
  float* part = nullptr;  // [B][nkv][max_splits][rep][hd + 2] split partials
  unsigned* counters = nullptr;  // [B][nkv], zero-initialised, self-resetting
  unsigned* work = nullptr;      // [3] work-queue head, exit count, merge-queue head; zeroed
  // split merges: 0 = the split that finishes last merges its (row, kv head)
  // at once; 1 = splits only announce their partials and the merges run from
  // a tail queue once the work queue drains (keeps CTAs streaming pages when
  // they hold several items)
  int merge_tail = 0;
  // optional [3]: the work words of an earlier launch that has completed (the
  // previous layer's attention of the same batch part), which this launch
  // clears; without it the last CTA of this launch clears its own words
  unsigned* work_prev = nullptr;
  __half* q16 = nullptr;         // [B][nq][hd] fp16 normalised + rotated q (written by the prep launch)
  int ctas_per_sm = 0;           // persistent grid size per SM (0: 2)
  int* err = nullptr;
};
constexpr int kPageTokens = 64;
size_t attn_part_floats(int B, int nkv, int max_splits, int rep, int hd);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t stream, bool pdl);
cudaError_t attention_init_attributes();

// Persistent decode step for small batches (step_kernel.cu): the whole step --
// embedding gather, every layer's q|k|v projection, q/k norm + RoPE + KV
// append + split-KV attention, o projection, gate/up + SwiGLU, down
// projection, and lm_head + argmax -- as ONE cooperative launch of one CTA per
// SM. The rows run as independent groups of up to 32; the step is a list of
// tasks (stage, group, tile) dealt round-robin to the CTAs, each task waiting
// on a per-(group, stage) completion counter instead of a kernel boundary,
// while a producer warp per CTA prefetches the weight tiles and KV pages of
// the CTA's next tasks into a shared-memory ring.
constexpr int kStepGroupRows = 32;
constexpr int kStepMaxGroups = 2;
constexpr int kStepRingBytes = 136 * 1024;  // per-CTA prefetch ring
constexpr int kStepMaxLayers = 32;
constexpr int kStepMaxStages = 2 + 5 * kStepMaxLayers;
constexpr int kStepSyncWords = 1024;
constexpr int kStepMaxK = 2048;  // longest input row the step supports
struct StepLayer {
  const __half* qkv = nullptr;   // fragment order (launch_pack_fragments) of the fused [q; k; v] rows
  const __half* o = nullptr;
  const __half* gu = nullptr;    // gate/up interleaved by 8 rows
  const __half* down = nullptr;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
};
struct StepArgs {
  StepLayer layer[kStepMaxLayers];
  const __half* lm = nullptr;  // fragment order, final norm folded in
  const float* embed = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  __half* kv_pool = nullptr;
  const int* block_table = nullptr;
  int max_pages = 0;
  int n_pages = 0;  // pages in the pool (page ids from the block table are checked against it)
  int* seq_pos = nullptr;
  const int* slots = nullptr;
  int* tokens = nullptr;    // [B] in: this step's tokens, out: next tokens
  int* next_out = nullptr;  // optional [B]
  float* logits = nullptr;  // optional [B][V]
  int* hist = nullptr;
  int* hist_step = nullptr;
  int hist_cap = 0, hist_stride = 0;
  int B = 0, H = 0, NQKV = 0, I = 0, V = 0, L = 0, nq = 0, nkv = 0, hd = 0, max_pos = 0;
  float eps = 0.f;
  // scratch
  float* h = nullptr;       // [B][H] residual stream
  __half* h16 = nullptr;    // [B][H]
  float* ssp = nullptr;     // [B][H / 16] sums of squares of 16-column chunks of h
  float* qkv = nullptr;     // [B][NQKV] raw projections (scaled by 1/rms)
  __half* attn16 = nullptr; // [B][nq * hd]
  __half* act16 = nullptr;  // [B][I]
  float* part = nullptr;    // [B][nkv][s_max][rep][hd + 2] attention job partials
  unsigned* arrive = nullptr;  // [B][nkv] job arrival counters (self-resetting)
  void* lm_part = nullptr;     // [groups][lm tasks][kStepGroupRows] (value, index)
  unsigned* sync = nullptr;    // kStepSyncWords zeroed words (self-resetting)
  // attention: pages per chunk (one ring entry), jobs per (row, kv head), chunks per job
  int split_pages = 1, s_max = 1, job_chunks = 1;
  int groups = 0, stages = 0, total_tasks = 0;
  int tiles[8] = {0};  // 16-row weight tiles per task, by task type (set by step_plan)
  int tasks[8] = {0};  // tile groups per stage, by task type (set by step_plan)
  int offs[kStepMaxStages * kStepMaxGroups + 1];  // first task of (stage, group), set by step_plan
  unsigned long long* trace = nullptr;  // optional [total_tasks][8] timestamps (ns), see mmc_debug_step_trace
  int* err = nullptr;
};
// attention pages per chunk the ring can hold for head_dim hd
int step_max_split_pages(int hd);
// fills the attention plan (from the longest context the step may see), groups and the task table
void step_plan(StepArgs& a, int64_t max_ctx_tokens, int num_sms);
cudaError_t launch_step(const StepArgs& a, int num_sms, cudaStream_t stream);
cudaError_t step_init_attributes();
// fragment order of a row-major fp16 [N][K] matrix (N % 16 == 0, K % 16 == 0):
// per 16-row tile, per 16-column step, the 32 lanes' m16n8k16 A fragments (16 B each)
cudaError_t launch_pack_fragments(const __half* src, __half* dst, int64_t N, int64_t K, cudaStream_t s);

// Weight packing: fp32 source rows -> fp16 destination rows (RNE), with an
// optional gate/up interleave by blocks of 8 rows.
// col_scale (optional, [cols]): folded RMSNorm weight, W[n][k] * col_scale[k]
cudaError_t launch_pack_rows(const float* src, __half* dst, int64_t rows, int64_t cols, cudaStream_t s,
                             const float* col_scale = nullptr);
cudaError_t launch_hold(uint64_t ns, cudaStream_t s);
cudaError_t launch_fill_kv(__half* pool, const int* pages, int n_tokens, int64_t page_halves, int row_halves,
                           uint32_t seed, cudaStream_t s);
cudaError_t launch_pack_gate_up(const float* gate, const float* up, __half* dst, int64_t inter, int64_t cols,
                                cudaStream_t s, const float* col_scale = nullptr);

}  // namespace mmc
