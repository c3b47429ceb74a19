/*
 * minimind_cuda.h — C ABI of the B200 decode engine (libminimind_cuda.so).
 *
 * This is the boundary that replaces the reference's device plumbing for the
 * single-token decode step of lvyufeng/minimind-orangepi. In the reference the
 * C++ runtime reaches the device through CANN: the AscendRuntime singleton and
 * DeviceBuffer/DeviceTensor/DeviceMatrix types (ascend_matmul.h:17-109) and the
 * two-phase aclnn custom ops (aclnnMiniMindXxxGetWorkspaceSize +
 * aclnnMiniMindXxx, e.g. ascend_custom_ops.cpp:875-883), wrapped by the
 * `device_*` functions of ascend_custom_ops.h:70-161. Here the runtime calls
 * the plain-C functions below instead: no C++ or torch types cross the
 * boundary, only pointers, sizes and status codes.
 *
 * Conventions
 *   - Every function returns an mmc_status (0 = success). On failure a
 *     thread-local message is available from mmc_last_error(). Nothing throws
 *     across the ABI. The C++ runtime maps MMC_ERR_INVALID to
 *     std::invalid_argument, MMC_ERR_OUT_OF_RANGE to std::out_of_range and the
 *     rest to std::runtime_error, the exception types the reference raises
 *     (language_model.cpp:17-21, :67-77; ascend_matmul.cpp:94-104).
 *   - There is no CPU fallback. Every compute entry point runs CUDA kernels
 *     built for sm_100a or fails with MMC_ERR_CUDA.
 *   - One context per GPU; a context is used by one host thread at a time.
 *   - "host" arguments are ordinary host memory; "d_" arguments are device
 *     pointers on the context's GPU. `stream` arguments are cudaStream_t
 *     passed as void* (NULL = the context's own stream).
 */
#ifndef MINIMIND_CUDA_H
#define MINIMIND_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MMC_EXPORT __attribute__((visibility("default")))
#else
#define MMC_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mmc_status {
  MMC_OK = 0,
  MMC_ERR_INVALID = 1,      /* bad shape / argument / sequence id */
  MMC_ERR_OUT_OF_RANGE = 2, /* token id outside [0, vocab) or position past max_position_embeddings */
  MMC_ERR_CUDA = 3,         /* a CUDA runtime call failed */
  MMC_ERR_NO_PAGES = 4,     /* the KV page pool is exhausted */
  MMC_ERR_DEVICE = 5,       /* a kernel reported an error (bounded wait timed out, missing page, ...) */
  MMC_ERR_STATE = 6,        /* call order violated (weights not loaded, KV not initialised, ...) */
  MMC_ERR_IO = 7            /* weights.bin missing / truncated / wrong format */
} mmc_status;

/* Model shape. Mirrors MiniMindConfig (config.h:21-45) for the dense decoder;
 * rms_norm_eps / rope_theta are explicit because the reference runtime config
 * does not carry them (runtime_loader.cpp:71-88). */
typedef struct mmc_model_desc {
  int64_t hidden_size;
  int64_t num_hidden_layers;
  int64_t num_attention_heads;
  int64_t num_key_value_heads;
  int64_t head_dim;
  int64_t intermediate_size;
  int64_t vocab_size;
  int64_t max_position_embeddings;
  float rms_norm_eps;
  float rope_theta;
} mmc_model_desc;

typedef struct mmc_ctx mmc_ctx;

/* Thread-local text of the last failure on this thread. */
MMC_EXPORT const char* mmc_last_error(void);
MMC_EXPORT int mmc_abi_version(void);

/* ------------------------------------------------------------- lifecycle */

/* Replaces the lazy AscendRuntime bring-up (ascend_matmul.cpp:176-221) and
 * validate_config's device limits (config.cpp:15-78): checks the shape
 * (hidden % 64, head_dim in {16,32,64,96,128}, heads % kv_heads, q heads per
 * kv head <= 8, intermediate % 64), selects `device` and creates the context's
 * stream. */
MMC_EXPORT int mmc_create(const mmc_model_desc* desc, int device, mmc_ctx** out);
MMC_EXPORT void mmc_destroy(mmc_ctx* ctx);

/* Replaces LanguageModel::ascend_weights() (language_model.cpp:273-288) and
 * upload_ascend_layer_weights (language_model.cpp:169-200): `tensors[i]` are
 * host fp32 arrays in weights.bin order (runtime_loader.cpp:121-167:
 * embed_tokens, norm, lm_head, then per layer input_layernorm,
 * post_attention_layernorm, q_norm, k_norm, q, k, v, o, gate, up, down) with
 * `counts[i]` elements each. Projections are packed to fp16 on the device; the
 * embedding and norm weights stay fp32. */
MMC_EXPORT int mmc_load_weights(mmc_ctx* ctx, const float* const* tensors, const int64_t* counts, int32_t n_tensors);
/* Same, streaming straight from a weights.bin file (MMRTW001). */
MMC_EXPORT int mmc_load_weights_file(mmc_ctx* ctx, const char* weights_bin_path);

/* ------------------------------------------------------------- KV cache */

/* Bytes of one KV page (64 positions x all layers x K,V x kv heads x head_dim, fp16). */
MMC_EXPORT int mmc_kv_page_bytes(const mmc_ctx* ctx, int64_t* bytes);
/* Replaces ensure_attention_cache (ascend_custom_ops.cpp:126-139; contiguous
 * [cap][kv_heads][head_dim] per layer, cap = max(tokens, 2048), regrown
 * without copy): allocates a pool of `n_pages` pages shared by up to
 * `max_seqs` sequences and scratch for batches of up to `max_batch` rows. */
MMC_EXPORT int mmc_kv_init(mmc_ctx* ctx, int64_t n_pages, int32_t max_seqs, int32_t max_batch);
/* A sequence is the device side of one DecoderState (language_model.h:22-25).
 * `reserve_tokens` positions are backed by pages up front (more are taken on
 * demand by mmc_decode_step). */
MMC_EXPORT int mmc_seq_open(mmc_ctx* ctx, int64_t reserve_tokens, int32_t* seq_out);
MMC_EXPORT int mmc_seq_reserve(mmc_ctx* ctx, int32_t seq, int64_t tokens);
MMC_EXPORT int mmc_seq_close(mmc_ctx* ctx, int32_t seq);
/* DecoderState::position: tokens already cached for the sequence. */
MMC_EXPORT int mmc_seq_position(const mmc_ctx* ctx, int32_t seq, int64_t* position);
/* Test helper: copy the cached K and V of one layer to host fp32 arrays laid
 * out like the reference CPU cache LayerKvCache::keys/values
 * ([position][kv_head][head_dim], decoder_layer.h:40-48). */
MMC_EXPORT int mmc_debug_read_kv(mmc_ctx* ctx, int32_t seq, int32_t layer, float* keys_host, float* values_host);

/* Benchmark helper: mark the first `n_tokens` positions of an empty sequence
 * as cached and fill them with seeded pseudo-random fp16 K/V (all layers), so
 * decode steps can be timed at a long context without an O(n) prompt pass.
 * Decode cost does not depend on the cached values. */
MMC_EXPORT int mmc_debug_fill_kv(mmc_ctx* ctx, int32_t seq, int64_t n_tokens, uint32_t seed);

/* Test helper: copy a per-step scratch buffer of the last step to host fp32:
 * which = 0 residual stream [batch][hidden], 1 raw q|k|v projections
 * [batch][(nq + 2 nkv) * hd], 2 attention output [batch][nq * hd],
 * 3 SiLU*mul activations [batch][intermediate]. `count` floats are copied. */
MMC_EXPORT int mmc_debug_scratch(mmc_ctx* ctx, int32_t which, float* host, int64_t count);

/* Debug helper for the persistent step (MMC_PERSISTENT=1, batches of up to 64 rows): with
 * MMC_STEP_TRACE=1 set when the context was created, each step records per
 * task global-timer nanoseconds (CTA, start, dependencies met, computed,
 * signalled, three unused); this copies the last step's records ([n][8]
 * uint64) to host memory and reports the step's task count. */
MMC_EXPORT int mmc_debug_step_trace(mmc_ctx* ctx, uint64_t* host, int64_t max_tasks, int64_t* n_tasks);

/* ------------------------------------------------------------- decode */

/* One greedy decode step for `batch` sequences — the batched form of
 * LanguageModel::forward_next_token (language_model.cpp:310-333):
 * embedding -> layers -> final norm -> lm_head -> argmax (first maximum).
 * Host buffers; synchronous. `logits_host` (optional, [batch][vocab]) receives
 * the fp32 logits like LanguageModel::forward_token (language_model.cpp:297-308).
 * Each sequence's position advances by one. When a graph was built for
 * exactly this list of sequences (mmc_graph_build) and no logits are asked
 * for, the step replays that graph instead of launching kernel by kernel.
 * A token outside the vocabulary
 * fails with MMC_ERR_OUT_OF_RANGE before anything runs (embedding_row,
 * language_model.cpp:67-77). */
MMC_EXPORT int mmc_decode_step(mmc_ctx* ctx, int32_t batch, const int32_t* seq_ids, const int32_t* tokens,
                    int32_t* next_tokens, float* logits_host);

/* Top-1 mixture-of-experts MLP (the reference's use_moe path,
 * decoder_layer.cpp:370-389, tensors in runtime_loader.cpp:148-158 order):
 * call after mmc_create and before loading weights. Each layer's MLP becomes
 * a router projection (num_experts rows; the first maximum picks the expert,
 * no gate weighting) followed by the chosen expert's gate/up + SwiGLU + down.
 * moe_intermediate_size must be a multiple of 64. */
MMC_EXPORT int mmc_configure_moe(mmc_ctx* ctx, int32_t num_experts, int64_t moe_intermediate_size);

/* Packed-weight cache (the runtime-format fast path): mmc_save_packed writes
 * the loaded context's device weights (fp16 rows with the RMSNorm weights
 * folded in, interleaved gate/up, fp32 embedding and norms) to `path`;
 * mmc_load_packed fills an unloaded context from such a file instead of
 * reading and re-packing weights.bin (runtime_loader.cpp:110-167 reads fp32
 * and the device path re-packs on every load, ascend_matmul.cpp:285-305). The
 * file records the model description and the packing layout; a mismatch is
 * MMC_ERR_INVALID / MMC_ERR_IO and leaves the context unloaded. */
MMC_EXPORT int mmc_save_packed(mmc_ctx* ctx, const char* path);
MMC_EXPORT int mmc_load_packed(mmc_ctx* ctx, const char* path);

/* Prompt pass on the device (replaces the token-by-token prompt loop of
 * LanguageModel::generate_stream, language_model.cpp:368-396, and plays the
 * role of prefill_next_token_device, language_model.cpp:229-251): feeds
 * prompt_lens[i] tokens to each sequence seq_ids[i] (tokens concatenated in
 * sequence order) in batched passes of up to max_batch rows, one row per
 * prompt position. Each row attends causally to its sequence's cache up to
 * its own position; every row's K/V is appended and the positions advance by
 * the prompt lengths. next_tokens[i] receives the greedy token after sequence
 * i's last prompt token (what the last mmc_decode_step of a token-by-token
 * prompt would return). Pages are reserved as needed. Synchronous. */
MMC_EXPORT int mmc_prefill(mmc_ctx* ctx, int32_t n_seqs, const int32_t* seq_ids, const int32_t* prompt_lens,
                           const int32_t* tokens, int32_t* next_tokens);

/* One decode step like mmc_decode_step, with a CUDA event between every two
 * kernels (programmatic overlap off) so each kernel's device time is
 * measured. kind_ms[7] / kind_launches[7] receive the summed milliseconds and
 * launch counts per kernel kind: 0 qkv projection, 1 attention (q/k prep +
 * attention), 2 o projection, 3 gate/up projection, 4 down projection,
 * 5 lm_head + argmax, 6 embedding gather (batches above 4). */
MMC_EXPORT int mmc_profile_step(mmc_ctx* ctx, int32_t batch, const int32_t* seq_ids, const int32_t* tokens,
                                int32_t* next_tokens, float* kind_ms, int32_t* kind_launches);

/* Same step, asynchronous on `stream`, with the tokens in device memory
 * (`d_tokens` read, `d_next` written, `d_logits` optional). Sequence ids are
 * host memory (the host tracks positions and pages). */
MMC_EXPORT int mmc_decode_step_async(mmc_ctx* ctx, int32_t batch, const int32_t* seq_ids, const int32_t* d_tokens,
                          int32_t* d_next, float* d_logits, void* stream);

/* Device-resident greedy loop. mmc_graph_build captures one full decode step
 * for this batch composition as a CUDA graph whose next tokens feed the
 * following step's embedding on the device. mmc_graph_run replays it
 * `n_steps` times (positions advance, pages must already be reserved) and
 * records every step's tokens in mapped pinned host memory; mmc_graph_tokens
 * waits for the stream and copies them out ([n_steps][batch]). */
MMC_EXPORT int mmc_graph_build(mmc_ctx* ctx, int32_t batch, const int32_t* seq_ids);
MMC_EXPORT int mmc_graph_set_tokens(mmc_ctx* ctx, const int32_t* tokens_host);
MMC_EXPORT int mmc_graph_run(mmc_ctx* ctx, int32_t n_steps, void* stream);
MMC_EXPORT int mmc_graph_tokens(mmc_ctx* ctx, int32_t n_steps, int32_t* tokens_host);

/* Streaming on the device-resident loop (replaces the per-token callback
 * loop of LanguageModel::generate_stream, language_model.cpp:368-396, whose
 * tokens the CLI prints as they come, minimind_generate.cpp:95-100):
 * mmc_graph_stream_start arms `n_steps` replays of the graph built by
 * mmc_graph_build (tokens set by mmc_graph_set_tokens); each
 * mmc_graph_stream_next returns the next step's tokens ([batch], host
 * memory) as soon as that step has finished on the device, while up to 32
 * later replays are already queued behind it. The lm_head epilogue writes
 * each step's tokens straight into mapped pinned host memory (a ring of 8192
 * steps), so nothing but the replays runs on the stream and the loop keeps
 * running on the device between reads. The device error word is copied back
 * after every 8th replay and after the last one: a device-side error is
 * reported by the next call of mmc_graph_stream_next that reaches such a
 * replay (tokens of up to 7 steps before it may come from the failed steps),
 * and always by the final one. A position advances when its replay is queued;
 * mmc_graph_stream_stop (or any other step, prompt pass or graph call) waits
 * for the queued replays and ends the run early, e.g. at an end-of-sequence
 * token. */
MMC_EXPORT int mmc_graph_stream_start(mmc_ctx* ctx, int32_t n_steps);
MMC_EXPORT int mmc_graph_stream_next(mmc_ctx* ctx, int32_t* tokens_host);
MMC_EXPORT int mmc_graph_stream_stop(mmc_ctx* ctx);

/* Wait for the context's stream and report any device-side error. */
MMC_EXPORT int mmc_synchronize(mmc_ctx* ctx);
/* Number of kernels one decode step launches for a batch of `batch` rows:
 * 1 for batches of up to 64 rows on dense models when the context was
 * created with MMC_PERSISTENT=1 (the persistent step: the whole step is one
 * cooperative launch); otherwise 5 per layer + 1 for batch 1 (and for 2..4
 * rows when the model's shapes do not fit the small-batch projections), 5 per
 * layer + 2 for a larger batch that runs as one part (below 256 rows), and
 * 6 per layer + 2 for each of the concurrent parts of a batch of 256+ rows (up
 * to 4 parts of >= 64 rows; the parts keep the separate q/k prep launch); one
 * more per layer when the context was created with MMC_ATTN_FUSED=0. */
MMC_EXPORT int mmc_kernels_per_step(const mmc_ctx* ctx, int32_t batch, int32_t* kernels);

/* ------------------------------------------------------------- single ops
 * Operator-level entry points with the two-phase shape of the reference's
 * aclnn ops (aclnnXxxGetWorkspaceSize, then the launch with a caller-provided
 * workspace): used by the per-kernel parity tests and the kernel sweep. All
 * pointers are device pointers; launches are asynchronous on `stream`. */

/* y[b][n] = sum_k W[n][k] x[b][k]; W fp16 [N][K] row-major, y fp32.
 * x is fp32 [batch][k] when batch <= 4 (CUDA-core path) and fp16 when
 * batch > 4 (tcgen05 tensor-core path). Replaces device_matmul
 * (ascend_matmul.cpp:385-410). No workspace. */
MMC_EXPORT int mmc_op_projection(int32_t batch, int32_t n, int32_t k, const void* d_w_fp16, const void* d_x, float* d_y,
                      void* stream);
/* Fused lm_head GEMV + argmax: logits (optional) and the first-maximum index
 * per row (x typed as for mmc_op_projection). Replaces device_matmul_argmax
 * (ascend_matmul.cpp:467-497). */
MMC_EXPORT int mmc_op_lm_head_argmax_workspace_size(int32_t batch, int32_t n, int32_t k, size_t* bytes);
MMC_EXPORT int mmc_op_lm_head_argmax(int32_t batch, int32_t n, int32_t k, const void* d_w_fp16, const void* d_x,
                          float* d_logits, int32_t* d_next, void* d_workspace, size_t workspace_bytes, void* stream);
/* Fused q/k RMSNorm + RoPE + K/V append + GQA decode attention for one layer
 * over a paged cache. Replaces device_decode_qkv_postprocess +
 * device_attention_from_cache (ascend_custom_ops.cpp:825-916).
 *   d_qkv      [batch][(nq + 2 nkv) * hd] fp32 raw projections
 *   d_kv_pool  pages [n_pages][layers][2][nkv][64][hd] fp16 (rows swizzled,
 *              see mmc_kv_row_offset)
 *   d_block_table [max_seqs][max_pages] int32, d_seq_pos [max_seqs] int32
 *              (positions BEFORE this token; not modified), d_slots [batch]
 *   d_rope_cos/sin [max_pos][hd/2] fp32, d_out [batch][nq * hd] fp32 */
MMC_EXPORT int mmc_op_attention_workspace_size(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t max_ctx,
                                    size_t* bytes);
MMC_EXPORT int mmc_op_attention(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t layer, int32_t layers,
                     const float* d_qkv, const float* d_q_norm, const float* d_k_norm, const float* d_rope_cos,
                     const float* d_rope_sin, int32_t max_pos, float eps, void* d_kv_pool,
                     const int32_t* d_block_table, int32_t max_pages, const int32_t* d_seq_pos,
                     const int32_t* d_slots, int32_t max_ctx, float* d_out, void* d_workspace,
                     size_t workspace_bytes, void* stream);
/* Reports a device-side error of the last mmc_op_attention launched with the
 * workspace `d_workspace` on `stream`: waits for the stream, reads the
 * kernel's error word (the first int of the workspace) and returns
 * MMC_ERR_DEVICE with the reason (KV position without a page in the block
 * table, position past max_pos, a bounded wait that ran out) if it is set,
 * clearing it. mmc_op_attention itself stays asynchronous and does not read
 * it. Replaces the error checks after aclnn launches (check_acl,
 * ascend_custom_ops.cpp:875-883). */
MMC_EXPORT int mmc_op_attention_status(const void* d_workspace, void* stream);
/* mmc_op_attention without a workspace argument, for callers that cannot
 * allocate device memory where they run (a custom allocator's own hooks, a
 * loop with a no-allocation rule, hosts that own all device memory). No
 * counterpart in the reference. The scratch is a fixed 16 MiB array inside the
 * library that every GPU loading it keeps until exit; sizes needing more
 * scratch than that (see mmc_op_attention_workspace_size) fail with
 * MMC_ERR_INVALID. The first call on a device looks up the array's address
 * with that device current (make it before any stream capture); with lazy
 * module loading that first call may also allocate the array's backing, so
 * warm up once (or set CUDA_MODULE_LOADING=EAGER) before a region where
 * allocation is forbidden. The cached address belongs to the device's primary
 * context: do not call after cudaDeviceReset. The array is shared by all
 * calls: calls that overlap on the GPU race. The call waits for its kernel and
 * returns MMC_ERR_DEVICE if the kernel reported an error. Allocates nothing
 * after the first call. */
MMC_EXPORT int mmc_op_attention_noalloc(int32_t batch, int32_t nq, int32_t nkv, int32_t hd, int32_t layer,
                                        int32_t layers, const float* d_qkv, const float* d_q_norm,
                                        const float* d_k_norm, const float* d_rope_cos, const float* d_rope_sin,
                                        int32_t max_pos, float eps, void* d_kv_pool, const int32_t* d_block_table,
                                        int32_t max_pages, const int32_t* d_seq_pos, const int32_t* d_slots,
                                        int32_t max_ctx, float* d_out, void* stream);
/* Element offset (in halves) of (row, 16-byte chunk) inside one 64 x hd page
 * slab: the cache's swizzled row layout, for tools that read pages directly. */
MMC_EXPORT int64_t mmc_kv_row_offset(int32_t hd, int32_t row, int32_t chunk);

#ifdef __cplusplus
}
#endif

#endif /* MINIMIND_CUDA_H */
