// Fused decode attention over a paged fp16 KV cache: two launches per layer.
//
// Replaces, for one decoder layer, the reference's
//   mini_mind_decode_qkv_postprocess (per-head q/k RMSNorm + RoPE + K/V append,
//     op_kernel/mini_mind_decode_qkv_postprocess.cpp:54-177; CPU form
//     decoder_layer.cpp:342-359)                          -> qk_prep_kernel
//   mini_mind_attention (GQA softmax(q.K/sqrt(d)).V over the cache,
//     op_kernel/mini_mind_attention.cpp:41-91; CPU form decoder_layer.cpp:184-234)
//                                                          -> attention_kernel
//
// qk_prep_kernel (one CTA per batch row and kv head) normalises and rotates the
// group's q heads into an fp16 buffer and appends the new token's K/V row to
// the cache page.
//
// attention_kernel is persistent (about two CTAs per SM). Work items are
// (batch row, kv head, split of the context), taken from an atomic queue by a
// dedicated producer warp that streams each item's 64-position pages -- K and V
// slabs, one contiguous 64 x hd fp16 block each, plus the item's q heads on its
// first page -- by bulk async copies into a ring of stages (full/empty
// mbarriers, per-stage item metadata in shared memory). Four consumer warps
// take 16 positions of each page:
//   S^T[16 tok x 8 heads] = K[16 x hd] . Q^T     (mma m16n8k16, heads on N)
//   online softmax per head (exp2 domain)
//   P^T -> B fragment by movmatrix (8x8 transpose in registers)
//   O^T[hd x 8 heads] += V^T[hd x 16 tok] . P^T  (ldmatrix.trans for V^T)
// The GQA group's q heads sit on the mma N dimension, so one K/V read serves
// all of them. At an item's last page the consumers merge their warps and
// either write the output or a split partial; the partials of a (row, kv
// head) are merged by the split that arrives last at its counter
// (self-resetting), or -- AttnArgs::merge_tail, for batches where CTAs hold
// several items -- from a tail queue once the work queue drains. The queue
// words of one launch are cleared by a later launch (AttnArgs::work_prev), so
// no CTA ends with an atomic. The producer never waits on the consumers
// except for a free stage, so copies stay in flight across item boundaries.
//
// Rows inside a page are stored with a 16-byte-chunk XOR swizzle (common.cuh
// swz_chunk) so the flat page copy lands in shared memory already
// conflict-free for ldmatrix; the append writes the same layout.

#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

// 4 consumer warps of 16 positions each (8 warps of 8 positions is the other
// supported split: more page throughput per CTA at long contexts, but slower
// for the batched decode step at ~1-2 K positions, where two CTAs per SM and
// the 4-stage ring matter more).
#ifndef MMC_ATTN_STAGES
#define MMC_ATTN_STAGES 3  // ring stages for head_dim <= 96 (build-time tuning knob)
#endif
constexpr int kConsumerWarps = 4;
constexpr int kTokPerWarp = 64 / kConsumerWarps;
constexpr int kAttnThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kMaxRep = 8;  // q heads per kv head carried on the mma N dimension

template <int HD>
struct AttnCfg {
  static constexpr int CPR = HD / 8;                     // 16-byte chunks per row
  static constexpr int TILE = kPageTokens * HD;          // halves per K (or V) page slab
  static constexpr int NST = HD <= 96 ? MMC_ATTN_STAGES : 3;  // ring stages
  static constexpr int KC = HD / 16;                     // k-chunks (S) == m-tiles (O)
  static constexpr size_t STAGE_BYTES = size_t(2) * TILE * 2;
  static constexpr size_t RING_BYTES = NST * STAGE_BYTES;
  // per stage: the group's q heads; after the ring: warp partials [warps][rep][HD + 2]
  // per stage: the group's fp16 q heads (prepared by qk_prep_kernel), or,
  // fused, the raw fp32 q heads and the raw k and v of the group's kv head,
  // then the item's RoPE cos / sin rows (HD / 2 each) and the q / k norm
  // weights (HD each)
  __host__ __device__ static size_t q_bytes(int rep, bool fused) {
    return fused ? size_t(rep + 5) * HD * 4 : size_t(rep) * HD * 2;
  }
  __host__ __device__ static size_t comb_floats(int rep) { return size_t(kConsumerWarps) * rep * (HD + 2); }
  // fused: the item's normalised + rotated q heads and new k, v rows (fp16)
  __host__ __device__ static size_t prep_bytes(int rep, bool fused) { return fused ? size_t(rep + 2) * HD * 2 : 0; }
  __host__ __device__ static size_t smem(int rep, bool fused) {
    return RING_BYTES + NST * q_bytes(rep, fused) + comb_floats(rep) * 4 + prep_bytes(rep, fused);
  }
};

__device__ __forceinline__ size_t page_slab(int page, int layer, int layers, int kv, int nkv, int h, int tile) {
  return ((((size_t)page * layers + layer) * 2 + kv) * nkv + h) * (size_t)tile;
}

// per-head RMSNorm (decoder_layer.cpp:32-42) + rotate-half RoPE
// (decoder_layer.cpp:139-152) of one head by one warp; result rounded to fp16.
template <int HD>
__device__ __forceinline__ void norm_rope_head(const float* src, const float* w, const float* cos_r,
                                               const float* sin_r, float eps, __half* dst, int lane) {
  constexpr int HALF = HD / 2;
  constexpr int PER = (HALF + 31) / 32;
  float first[PER], second[PER];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int d = lane + 32 * j;
    first[j] = d < HALF ? src[d] : 0.f;
    second[j] = d < HALF ? src[d + HALF] : 0.f;
    ss += first[j] * first[j] + second[j] * second[j];
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / float(HD) + eps);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int d = lane + 32 * j;
    if (d < HALF) {
      const float f = first[j] * (scale * w[d]);
      const float s = second[j] * (scale * w[d + HALF]);
      const float c = cos_r[d], sn = sin_r[d];
      dst[d] = __float2half_rn(f * c - s * sn);
      dst[d + HALF] = __float2half_rn(s * c + f * sn);
    }
  }
}

struct StageMeta {
  int b, h, split, tok_begin, tok_end, nch, nsplits, chunk;  // chunk < 0: end of this CTA's stream
  int pos;   // the row's current position (ctx - 1)
  int page;  // the page this stage holds
};

// Work item w (split-major numbering). A sequence of P cached pages is cut into
// n = ceil(P / split_pages) splits of equal size (ceil(P / n) pages), so no
// split is a short remainder.
__device__ __forceinline__ bool decode_item(const AttnArgs& a, int w, StageMeta& m) {
  const int per_split = a.B * a.nkv;
  m.split = w / per_split;
  const int bh = w % per_split;
  m.b = a.order ? a.order[bh / a.nkv] : bh / a.nkv;
  if (m.b < 0 || m.b >= a.B) {  // a corrupt order entry: record it, skip the item
    set_error(a.err, kDevPositionLimit);
    return false;
  }
  m.h = bh % a.nkv;
  const int ctx = a.seq_pos[a.slots[m.b]] + (a.row_off ? a.row_off[m.b] : 0) + 1;
  m.pos = ctx - 1;
  if (a.fused && (ctx > a.max_pos || (ctx - 1) / kPageTokens >= a.max_pages)) {
    set_error(a.err, kDevPositionLimit);
    return false;
  }
  const int pages = (ctx + kPageTokens - 1) / kPageTokens;
  const int split_pages = a.split_tokens / kPageTokens;
  m.nsplits = (pages + split_pages - 1) / split_pages;
  if (m.split >= m.nsplits) return false;
  const int per = (pages + m.nsplits - 1) / m.nsplits;
  m.tok_begin = m.split * per * kPageTokens;
  if (m.tok_begin >= ctx) return false;
  m.tok_end = min(ctx, m.tok_begin + per * kPageTokens);
  m.nch = (m.tok_end - m.tok_begin + kPageTokens - 1) / kPageTokens;
  return true;
}


__device__ __forceinline__ void red_add_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

template <int HD>
__global__ void __launch_bounds__(128) qk_prep_kernel(AttnArgs a) {
  using C = AttnCfg<HD>;
  __shared__ __align__(16) __half kv_new[2][HD];
  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rep = a.nq / a.nkv;
  pdl_wait();
  pdl_launch_dependents();
  const int slot = a.slots[b];
  const int pos = a.seq_pos[slot] + (a.row_off ? a.row_off[b] : 0);
  if (pos >= a.max_pos || pos / kPageTokens >= a.max_pages) {
    if (tid == 0) set_error(a.err, kDevPositionLimit);
    return;
  }
  const float* row = a.qkv + (size_t)b * a.ld_qkv;
  const float* cos_r = a.rope_cos + (size_t)pos * (HD / 2);
  const float* sin_r = a.rope_sin + (size_t)pos * (HD / 2);
  for (int j = warp; j < rep + 2; j += 4) {
    if (j < rep) {
      norm_rope_head<HD>(row + (size_t)(h * rep + j) * HD, a.q_norm, cos_r, sin_r, a.eps,
                         a.q16 + ((size_t)b * a.nq + h * rep + j) * HD, lane);
    } else if (j == rep) {
      norm_rope_head<HD>(row + (size_t)(a.nq + h) * HD, a.k_norm, cos_r, sin_r, a.eps, kv_new[0], lane);
    } else {
      const float* v = row + (size_t)(a.nq + a.nkv + h) * HD;
      for (int d = lane; d < HD; d += 32) kv_new[1][d] = __float2half_rn(v[d]);
    }
  }
  __syncthreads();
  if (tid < 2 * C::CPR) {
    const int kv = tid / C::CPR, c = tid % C::CPR;
    const int page = a.block_table[(size_t)slot * a.max_pages + pos / kPageTokens];
    if (page < 0) {
      set_error(a.err, kDevNoPage);
      return;
    }
    const int r = pos % kPageTokens;
    __half* dst = a.kv_pool + page_slab(page, a.layer, a.layers, kv, a.nkv, h, C::TILE) + (size_t)r * HD +
                  swz_chunk(r, c, C::CPR) * 8;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&kv_new[kv][c * 8]);
  }
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 3) attention_kernel(AttnArgs a) {
  using C = AttnCfg<HD>;
  extern __shared__ __align__(128) uint8_t smem[];
  __half* ring = reinterpret_cast<__half*>(smem);
  const int rep = a.nq / a.nkv;
  __half* qring = reinterpret_cast<__half*>(smem + C::RING_BYTES);                        // [NST][rep][HD]
  float* comb = reinterpret_cast<float*>(smem + C::RING_BYTES + C::NST * C::q_bytes(rep, a.fused));  // [warps][rep][HD+2]
  __half* prep = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(comb) + C::comb_floats(rep) * 4);  // [rep+2][HD]
  const size_t qstride = C::q_bytes(rep, a.fused) / 2;  // halves per q stage
  __shared__ __align__(8) uint64_t full_bar[C::NST];
  __shared__ __align__(8) uint64_t empty_bar[C::NST];
  __shared__ StageMeta meta[C::NST];
  __shared__ int merge_last, merge_task, merge_ok;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int total_items = a.max_splits * a.B * a.nkv;

  // the queue words of an earlier launch that has completed (the previous
  // layer's attention of this batch part): cleared here for its next use
  if (a.work_prev != nullptr && blockIdx.x == 0 && tid == 0) {
    a.work_prev[0] = 0u;
    a.work_prev[1] = 0u;
    a.work_prev[2] = 0u;
  }
  if (tid == 0) {
    for (int s = 0; s < C::NST; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ======================================================= producer warp
    // The whole warp runs the producer: lane 0 issues the copies, all lanes
    // hold 32 page-table entries of the current item (one load round trip
    // per 32 pages), and the next work item is taken from the queue and
    // decoded right after the current item's first page is issued, while the
    // ring is full -- so item boundaries cost the consumers nothing.
    auto fetch = [&](StageMeta& m) -> bool {  // warp-uniform
      while (true) {
        int w = 0;
        if (lane == 0) w = int(atomicAdd(&a.work[0], 1u));
        w = __shfl_sync(0xffffffffu, w, 0);
        if (w >= total_items) return false;
        if (!decode_item(a, w, m)) continue;
        if (m.nsplits > a.max_splits) {
          if (lane == 0) set_error(a.err, kDevPositionLimit);
          continue;
        }
        return true;
      }
    };
    auto load_pages = [&](const StageMeta& m, int block) {  // entries [block*32, block*32+32) of the item
      const int pidx = m.tok_begin / kPageTokens + block * 32 + lane;
      const int slot = a.slots[m.b];
      return (block * 32 + lane < m.nch && pidx < a.max_pages) ? a.block_table[(size_t)slot * a.max_pages + pidx]
                                                              : -1;
    };
    // The first item and its page-table entries depend only on the work
    // queue, positions and block tables (stable during the step), so they are
    // fetched before waiting on qk_prep_kernel, whose q heads and appended
    // K/V rows the page copies below read.
    StageMeta cur{}, nxt{};
    bool have_cur = fetch(cur), have_nxt = false, nxt_decoded = false;
    int cur_pages = have_cur ? load_pages(cur, 0) : -1, nxt_pages = -1;
    // Fused, the cached pages do not depend on the previous kernel (the
    // current position's row is patched in by the consumers): the first
    // item's pages go out before the dependency wait, and only its raw q/k/v
    // copy waits for the q|k|v projection to finish.
    bool waited = !a.fused;
    if (waited) {
      pdl_wait();
      pdl_launch_dependents();
    }
    int def_stage = -1;  // stage whose raw q/k/v copy waits for the dependency
    StageMeta def_item{};
    auto issue_raw = [&](int st, const StageMeta& it) {  // lane 0
      float* raw = reinterpret_cast<float*>(qring + (size_t)st * qstride);
      const float* row = a.qkv + (size_t)it.b * a.ld_qkv;
      bulk_g2s(raw, row + (size_t)it.h * rep * HD, uint32_t(rep * HD * 4), &full_bar[st]);
      if (it.tok_end == it.pos + 1) {
        bulk_g2s(raw + rep * HD, row + (size_t)(a.nq + it.h) * HD, uint32_t(HD * 4), &full_bar[st]);
        bulk_g2s(raw + (rep + 1) * HD, row + (size_t)(a.nq + a.nkv + it.h) * HD, uint32_t(HD * 4), &full_bar[st]);
      }
    };
    auto finish_wait = [&]() {  // whole warp
      if (waited) return;
      pdl_wait();
      pdl_launch_dependents();
      waited = true;
      if (lane == 0 && def_stage >= 0) issue_raw(def_stage, def_item);
      __syncwarp();
    };
    int chunk = 0;
    bool done = !have_cur;
    for (int c = 0;; ++c) {
      const int s = c % C::NST;
      if (c >= C::NST) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(&empty_bar[s], ((c / C::NST) - 1) & 1, a.err);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) done = true;
      }
      if (!done && chunk >= cur.nch) {  // current item exhausted: move to the next
        if (!nxt_decoded) {
          have_nxt = fetch(nxt);
          nxt_pages = have_nxt ? load_pages(nxt, 0) : -1;
        }
        nxt_decoded = false;
        if (!have_nxt) {
          done = true;
        } else {
          cur = nxt;
          cur_pages = nxt_pages;
          chunk = 0;
        }
      }
      int page = -1;
      if (!done) {
        if (chunk > 0 && (chunk & 31) == 0) cur_pages = load_pages(cur, chunk >> 5);
        page = __shfl_sync(0xffffffffu, cur_pages, chunk & 31);
        if (page < 0) {
          if (lane == 0) set_error(a.err, kDevNoPage);
          done = true;
        }
      }
      if (done) {
        if (lane == 0) {
          meta[s].chunk = -1;
          mbar_arrive_expect_tx(&full_bar[s], 0);
        }
        break;
      }
      if (lane == 0) {
        StageMeta m = cur;
        m.chunk = chunk;
        m.page = page;
        meta[s] = m;
        const bool first = chunk == 0;
        const bool last_split = cur.tok_end == cur.pos + 1;
        // fused: raw q heads, plus raw k and v for the split holding the current position
        const uint32_t qbytes = a.fused ? uint32_t((rep + (last_split ? 2 : 0)) * HD * 4) : uint32_t(rep * HD * 2);
        // fused: the item's RoPE rows and norm weights ride along (they do not
        // depend on the previous kernel, so they go out at once)
        const uint32_t aux = (first && a.fused) ? uint32_t(3 * HD * 4) : 0u;
        mbar_arrive_expect_tx(&full_bar[s], uint32_t(C::STAGE_BYTES) + (first ? qbytes : 0u) + aux);
        __half* dst = ring + (size_t)s * 2 * C::TILE;
        bulk_g2s(dst, a.kv_pool + page_slab(page, a.layer, a.layers, 0, a.nkv, cur.h, C::TILE), C::TILE * 2,
                 &full_bar[s]);
        bulk_g2s(dst + C::TILE, a.kv_pool + page_slab(page, a.layer, a.layers, 1, a.nkv, cur.h, C::TILE),
                 C::TILE * 2, &full_bar[s]);
        if (first && a.fused) {
          float* ax = reinterpret_cast<float*>(qring + (size_t)s * qstride) + (rep + 2) * HD;
          bulk_g2s(ax, a.rope_cos + (size_t)cur.pos * (HD / 2), uint32_t(HD / 2 * 4), &full_bar[s]);
          bulk_g2s(ax + HD / 2, a.rope_sin + (size_t)cur.pos * (HD / 2), uint32_t(HD / 2 * 4), &full_bar[s]);
          bulk_g2s(ax + HD, a.q_norm, uint32_t(HD * 4), &full_bar[s]);
          bulk_g2s(ax + 2 * HD, a.k_norm, uint32_t(HD * 4), &full_bar[s]);
          if (waited) {
            issue_raw(s, cur);
          } else {
            def_stage = s;
            def_item = cur;
          }
        } else if (first) {
          bulk_g2s(qring + (size_t)s * qstride, a.q16 + ((size_t)cur.b * a.nq + cur.h * rep) * HD, qbytes,
                   &full_bar[s]);
        }
      }
      __syncwarp();
      ++chunk;
      if (chunk == 1 && !nxt_decoded) {  // ring is full: look ahead to the next item now
        have_nxt = fetch(nxt);
        nxt_pages = have_nxt ? load_pages(nxt, 0) : -1;
        nxt_decoded = true;
      }
      // the ring is full or the first item's pages are all out: now wait
      if (!waited && (c + 1 >= C::NST || chunk >= cur.nch)) finish_wait();
    }
    finish_wait();
    __syncwarp();
  } else {
    // ====================================================== consumer warps
    pdl_wait();
    pdl_launch_dependents();
    const int g = lane >> 2, t = lane & 3;
    const float sl2 = 1.4426950408889634f / sqrtf(float(HD));
    const int r0 = warp * kTokPerWarp;
    const size_t pstride = (size_t)rep * (HD + 2);
    StageMeta it{};
    uint32_t qb0[C::KC], qb1[C::KC];
    float mA = -1e30f, mB = -1e30f, lA = 0.f, lB = 0.f;
    float o[C::KC][4];
    for (int c = 0;; ++c) {
      const int s = c % C::NST;
      if (!mbar_wait_bounded(&full_bar[s], (c / C::NST) & 1, a.err)) break;
      const StageMeta m = meta[s];
      if (m.chunk < 0) break;
      const __half* kt = ring + (size_t)s * 2 * C::TILE;
      const __half* vt = kt + C::TILE;
      if (m.chunk == 0) {  // a new item: its q heads arrived with this page
        it = m;
        const __half* qs = qring + (size_t)s * qstride;
        if (a.fused) {
          // q/k per-head RMSNorm + RoPE (decoder_layer.cpp:342-359) from the raw
          // projections in this stage: q heads for the item, and the new k and
          // v rows when the item holds the current position. (Every warp has
          // its previous item's q in registers: the merge synchronised them.)
          const float* raw = reinterpret_cast<const float*>(qs);
          const float* cos_r = raw + (rep + 2) * HD;  // copied with the page
          const float* sin_r = cos_r + HD / 2;
          const float* qn = cos_r + HD;
          const float* kn = cos_r + 2 * HD;
          for (int j = warp; j < rep; j += kConsumerWarps)
            norm_rope_head<HD>(raw + j * HD, qn, cos_r, sin_r, a.eps, prep + j * HD, lane);
          if (it.tok_end == it.pos + 1) {
            if (warp == 0) norm_rope_head<HD>(raw + rep * HD, kn, cos_r, sin_r, a.eps, prep + rep * HD, lane);
            if (warp == 1)
              for (int d = lane; d < HD; d += 32) prep[(rep + 1) * HD + d] = __float2half_rn(raw[(rep + 1) * HD + d]);
          }
          consumer_sync();
          qs = prep;
        }
#pragma unroll
        for (int kc = 0; kc < C::KC; ++kc) {
          qb0[kc] = g < rep ? *reinterpret_cast<const uint32_t*>(qs + g * HD + 16 * kc + 2 * t) : 0u;
          qb1[kc] = g < rep ? *reinterpret_cast<const uint32_t*>(qs + g * HD + 16 * kc + 8 + 2 * t) : 0u;
        }
        mA = mB = -1e30f;
        lA = lB = 0.f;
#pragma unroll
        for (int mt = 0; mt < C::KC; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
      }
      if (a.fused && m.chunk == it.nch - 1 && it.tok_end == it.pos + 1) {
        // the new K/V row: into this stage's copy of the current page (the
        // copy predates it) and into the cache for later steps (the K/V
        // append of the reference, decoder_layer.cpp:355-359)
        const int r = it.pos % kPageTokens;
        if (tid < 2 * C::CPR) {
          const int kv = tid / C::CPR, ch = tid % C::CPR;
          const uint4 v = *reinterpret_cast<const uint4*>(prep + (rep + kv) * HD + ch * 8);
          __half* sp = ring + (size_t)s * 2 * C::TILE + kv * C::TILE + r * HD + swz_chunk(r, ch, C::CPR) * 8;
          *reinterpret_cast<uint4*>(sp) = v;
          __half* gp = a.kv_pool + page_slab(m.page, a.layer, a.layers, kv, a.nkv, it.h, C::TILE) + (size_t)r * HD +
                       swz_chunk(r, ch, C::CPR) * 8;
          *reinterpret_cast<uint4*>(gp) = v;
        }
        consumer_sync();
      }
      const int tok0 = it.tok_begin + m.chunk * kPageTokens + r0;
      if (tok0 < it.tok_end) {
        // ---- S^T = K . Q^T over this warp's positions (rows 8-15 of the
        //      m16 tile repeat rows 0-7 when a warp owns 8 positions; masked)
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kc = 0; kc < C::KC; ++kc) {
          const int rr = r0 + (kTokPerWarp == 16 ? ((lane >> 3) & 1) * 8 : 0) + (lane & 7);
          const int chn = 2 * kc + (lane >> 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(smem_u32(kt + rr * HD + swz_chunk(rr, chn, C::CPR) * 8), a0, a1, a2, a3);
          mma16816(sc, a0, a1, a2, a3, qb0[kc], qb1[kc]);
        }
        const bool v0 = tok0 + g < it.tok_end, v1 = kTokPerWarp == 16 && tok0 + g + 8 < it.tok_end;
        const float sA0 = v0 ? sc[0] * sl2 : -INFINITY, sB0 = v0 ? sc[1] * sl2 : -INFINITY;
        const float sA1 = v1 ? sc[2] * sl2 : -INFINITY, sB1 = v1 ? sc[3] * sl2 : -INFINITY;
        float mxA = fmaxf(sA0, sA1), mxB = fmaxf(sB0, sB1);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, off));
          mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, off));
        }
        const float nA = fmaxf(mA, mxA), nB = fmaxf(mB, mxB);
        const float alA = exp2f(mA - nA), alB = exp2f(mB - nB);
        mA = nA;
        mB = nB;
        const float pA0 = exp2f(sA0 - nA), pB0 = exp2f(sB0 - nB);
        const float pA1 = exp2f(sA1 - nA), pB1 = exp2f(sB1 - nB);
        lA = lA * alA + pA0 + pA1;
        lB = lB * alB + pB0 + pB1;
#pragma unroll
        for (int mt = 0; mt < C::KC; ++mt) {
          o[mt][0] *= alA;
          o[mt][1] *= alB;
          o[mt][2] *= alA;
          o[mt][3] *= alB;
        }
        // ---- P^T as the B operand: transpose the two 8x8 halves in registers
        const uint32_t pb0 = movmatrix_t(pack_half2(pA0, pB0));
        const uint32_t pb1 = movmatrix_t(pack_half2(pA1, pB1));
        // ---- O^T += V^T . P^T
#pragma unroll
        for (int mt = 0; mt < C::KC; ++mt) {
          const int rr = r0 + (kTokPerWarp == 16 ? ((lane >> 4) & 1) * 8 : 0) + (lane & 7);
          const int chn = 2 * mt + ((lane >> 3) & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(smem_u32(vt + rr * HD + swz_chunk(rr, chn, C::CPR) * 8), a0, a1, a2, a3);
          mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);  // this warp is done with the stage
      if (m.chunk != it.nch - 1) continue;

      // ---------------------------------------------- item done: merge warps
      float lAr = lA, lBr = lB;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        lAr += __shfl_xor_sync(0xffffffffu, lAr, off);
        lBr += __shfl_xor_sync(0xffffffffu, lBr, off);
      }
      {
        float* cw = comb + (size_t)warp * rep * (HD + 2);
        const int hA = 2 * t, hB = 2 * t + 1;
        if (hA < rep) {
#pragma unroll
          for (int mt = 0; mt < C::KC; ++mt) {
            cw[hA * (HD + 2) + 16 * mt + g] = o[mt][0];
            cw[hA * (HD + 2) + 16 * mt + g + 8] = o[mt][2];
          }
          if (g == 0) {
            cw[hA * (HD + 2) + HD] = mA;
            cw[hA * (HD + 2) + HD + 1] = lAr;
          }
        }
        if (hB < rep) {
#pragma unroll
          for (int mt = 0; mt < C::KC; ++mt) {
            cw[hB * (HD + 2) + 16 * mt + g] = o[mt][1];
            cw[hB * (HD + 2) + 16 * mt + g + 8] = o[mt][3];
          }
          if (g == 0) {
            cw[hB * (HD + 2) + HD] = mB;
            cw[hB * (HD + 2) + HD + 1] = lBr;
          }
        }
      }
      consumer_sync();
      float* part_bh = a.part + ((size_t)it.b * a.nkv + it.h) * a.max_splits * pstride;
      const size_t out_off = (size_t)it.b * a.nq * HD + (size_t)it.h * rep * HD;
      auto put_out = [&](int idx, float v) {
        if (a.out16) a.out16[out_off + idx] = __float2half_rn(v);
        else a.out[out_off + idx] = v;
      };
      for (int i = tid; i < rep * HD; i += kConsumerWarps * 32) {
        const int j = i / HD, d = i % HD;
        float M = -1e30f;
        for (int w4 = 0; w4 < kConsumerWarps; ++w4) M = fmaxf(M, comb[(w4 * rep + j) * (HD + 2) + HD]);
        float L = 0.f, O = 0.f;
        for (int w4 = 0; w4 < kConsumerWarps; ++w4) {
          const float* cw = comb + (w4 * rep + j) * (HD + 2);
          const float f = exp2f(cw[HD] - M);
          L += cw[HD + 1] * f;
          O += cw[d] * f;
        }
        if (it.nsplits == 1) {
          put_out(j * HD + d, O / L);
        } else {
          float* pp = part_bh + it.split * pstride + j * (HD + 2);
          pp[d] = O;
          if (d == 0) {
            pp[HD] = M;
            pp[HD + 1] = L;
          }
        }
      }
      consumer_sync();  // partials / outputs stored; comb is reused by the next item
      if (it.nsplits <= 1) continue;
      if (a.merge_tail) {
        // announce the partial without waiting: the merges run from the tail
        // queue below, off the page stream's critical path
        if (tid == 0) red_add_release_gpu(&a.counters[(size_t)it.b * a.nkv + it.h], 1u);
        continue;
      }
      // the split that finishes last merges the (row, kv head)'s partials:
      // no split waits for another
      if (tid == 0) {
        unsigned* cnt = &a.counters[(size_t)it.b * a.nkv + it.h];
        __threadfence();
        merge_last = atom_add_acq_rel_gpu(cnt, 1u) == unsigned(it.nsplits - 1);
        if (merge_last) *cnt = 0u;  // every split has arrived: reset for the next launch
      }
      consumer_sync();
      if (!merge_last) continue;
      {
        // stage the split partials in shared memory (independent coalesced
        // loads), then merge from there
        const int n = it.nsplits * int(pstride);
        const bool staged = n <= int(C::comb_floats(rep));
        if (staged) {
          for (int i = tid; i < n; i += kConsumerWarps * 32) comb[i] = __ldcg(part_bh + i);
          consumer_sync();
        }
        const float* src = staged ? comb : part_bh;
        for (int i = tid; i < rep * HD; i += kConsumerWarps * 32) {
          const int j = i / HD, d = i % HD;
          float M = -1e30f;
          for (int sp = 0; sp < it.nsplits; ++sp) M = fmaxf(M, src[sp * pstride + j * (HD + 2) + HD]);
          float L = 0.f, O = 0.f;
          for (int sp = 0; sp < it.nsplits; ++sp) {
            const float* pp = src + sp * pstride + j * (HD + 2);
            const float f = exp2f(pp[HD] - M);
            L += pp[HD + 1] * f;
            O += (staged ? pp[d] : __ldcg(pp + d)) * f;
          }
          put_out(j * HD + d, O / L);
        }
        consumer_sync();  // comb is reused by the next item
      }
    }

    // ---------------------------------------------- tail: merge split items
    // (merge_tail) Once the work queue is empty every item is held by a
    // running CTA, so waiting here for a (row, kv head)'s splits cannot
    // deadlock. Tasks come from a second queue; each waits (bounded) for its
    // pair's split count, merges the partials and clears the count.
    const int pairs = a.merge_tail ? a.B * a.nkv : 0;
    for (;;) {
      if (pairs == 0) break;
      if (tid == 0) merge_task = int(atomicAdd(&a.work[2], 1u));
      consumer_sync();
      const int task = merge_task;
      consumer_sync();  // everyone has read merge_task before it is rewritten
      if (task >= pairs) break;
      const int b = task / a.nkv, h = task % a.nkv;
      const int ctx = a.seq_pos[a.slots[b]] + (a.row_off ? a.row_off[b] : 0) + 1;
      const int pages = (ctx + kPageTokens - 1) / kPageTokens;
      const int split_pages = a.split_tokens / kPageTokens;
      const int nsplits = (pages + split_pages - 1) / split_pages;
      if (nsplits <= 1 || nsplits > a.max_splits) continue;
      unsigned* cnt = &a.counters[(size_t)b * a.nkv + h];
      if (tid == 0) {
        merge_ok = 1;
        if (ld_acquire_gpu(cnt) < unsigned(nsplits)) {
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_gpu(cnt) < unsigned(nsplits)) {
            if (global_timer_ns() - t0 > 2000000000ull) {
              set_error(a.err, kDevWaitTimeout);
              merge_ok = 0;
              break;
            }
            __nanosleep(64);
          }
        }
      }
      consumer_sync();
      if (merge_ok) {
        float* part_bh = a.part + ((size_t)b * a.nkv + h) * a.max_splits * pstride;
        const size_t out_off = (size_t)b * a.nq * HD + (size_t)h * rep * HD;
        const int n = nsplits * int(pstride);
        const bool staged = n <= int(C::comb_floats(rep));
        if (staged) {
          for (int i = tid; i < n; i += kConsumerWarps * 32) comb[i] = __ldcg(part_bh + i);
          consumer_sync();
        }
        const float* src = staged ? comb : part_bh;
        for (int i = tid; i < rep * HD; i += kConsumerWarps * 32) {
          const int j = i / HD, d = i % HD;
          float M = -1e30f;
          for (int sp = 0; sp < nsplits; ++sp) M = fmaxf(M, src[sp * pstride + j * (HD + 2) + HD]);
          float L = 0.f, O = 0.f;
          for (int sp = 0; sp < nsplits; ++sp) {
            const float* pp = src + sp * pstride + j * (HD + 2);
            const float f = exp2f(pp[HD] - M);
            L += pp[HD + 1] * f;
            O += (staged ? pp[d] : __ldcg(pp + d)) * f;
          }
          if (a.out16) a.out16[out_off + j * HD + d] = __float2half_rn(O / L);
          else a.out[out_off + j * HD + d] = O / L;
        }
        if (tid == 0) *cnt = 0u;
      }
      consumer_sync();  // comb is reused by the next task
    }
  }

  // ---- queue reset: without a later launch that clears them, the last CTA
  //      to leave clears the work counters
  if (a.work_prev != nullptr) return;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&a.work[1], 1u) == gridDim.x - 1) {
      a.work[0] = 0u;
      a.work[1] = 0u;
      a.work[2] = 0u;
    }
  }
}

template <int HD>
cudaError_t launch_hd(const AttnArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t prep = {};
  prep.gridDim = dim3(a.nkv, a.B);
  prep.blockDim = dim3(128);
  prep.stream = s;
  prep.attrs = attr;
  prep.numAttrs = pdl ? 1 : 0;
  if (!a.fused) {
    const cudaError_t e = cudaLaunchKernelEx(&prep, qk_prep_kernel<HD>, a);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  const int items = a.max_splits * a.nkv * a.B;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int per_sm = a.ctas_per_sm > 0 ? a.ctas_per_sm : 2;
  cfg.gridDim = dim3(items < per_sm * sms ? items : per_sm * sms);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = AttnCfg<HD>::smem(a.nq / a.nkv, a.fused != 0);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl || !a.fused) ? 1 : 0;  // unfused: always overlaps qk_prep_kernel's tail
  return cudaLaunchKernelEx(&cfg, attention_kernel<HD>, a);
}

template <int HD>
cudaError_t attr_hd() {
  const cudaError_t e = set_kernel_smem(qk_prep_kernel<HD>, 0);
  const cudaError_t e2 = set_kernel_smem(attention_kernel<HD>, int(AttnCfg<HD>::smem(kMaxRep, true)));
  return e != cudaSuccess ? e : e2;
}

}  // namespace

size_t attn_part_floats(int B, int nkv, int max_splits, int rep, int hd) {
  return size_t(B) * nkv * max_splits * rep * (hd + 2);
}

cudaError_t attention_init_attributes() {
  cudaError_t e = cudaSuccess, r;
  if ((r = attr_hd<16>()) != cudaSuccess) e = r;
  if ((r = attr_hd<32>()) != cudaSuccess) e = r;
  if ((r = attr_hd<64>()) != cudaSuccess) e = r;
  if ((r = attr_hd<96>()) != cudaSuccess) e = r;
  if ((r = attr_hd<128>()) != cudaSuccess) e = r;
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
  if (a.nkv <= 0 || a.nq % a.nkv != 0 || a.nq / a.nkv > kMaxRep || a.split_tokens % kPageTokens != 0 ||
      a.max_splits <= 0 || a.B <= 0 || a.work == nullptr || (a.q16 == nullptr && !a.fused) ||
      (a.fused && a.row_off != nullptr))
    return cudaErrorInvalidValue;
  switch (a.hd) {
    case 16: return launch_hd<16>(a, s, pdl);
    case 32: return launch_hd<32>(a, s, pdl);
    case 64: return launch_hd<64>(a, s, pdl);
    case 96: return launch_hd<96>(a, s, pdl);
    case 128: return launch_hd<128>(a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mmc
