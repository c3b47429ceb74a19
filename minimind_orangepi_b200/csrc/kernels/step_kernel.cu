// Persistent decode step for small batches: one cooperative launch per step.
//
// The chained form of the step (6 launches per layer) pays a kernel boundary
// between every two dependent operations; at a few rows each launch does ~1 us
// of work behind several us of dependency latency. Here the whole step -- the
// operations of the reference's forward_next_token (language_model.cpp:310-333
// -> decoder_layer.cpp:312-407) -- runs as one grid of one CTA per SM that
// lives for the whole step.
//
// Work list. The batch rows form independent groups of up to 32 rows. Per
// group the step is a chain of stages: EMB (embedding gather), then per layer
// QKV, ATTN, O, GU, DOWN, then LM. Each stage is cut into tasks:
//   EMB   one task per row
//   QKV/O/GU/DOWN/LM  one or two 16-row weight tiles x a block of the group's
//         rows (32, or 16 when the input rows are longer than 1024), on
//         mma.sync m16n8k16 with the weights as the A operand; epilogues:
//         store (QKV), residual + fp16 copy + sums of squares (O, DOWN),
//         SiLU*mul of the interleaved gate/up rows (GU), logits + first
//         maximum per tile (LM; the group's last LM task reduces them and
//         writes the next tokens, positions and token history)
//   ATTN  (row, kv head, job): q RMSNorm + RoPE of the kv head's q heads from
//         the raw projection, the new K/V row (the job holding the current
//         position also appends it to the cache), online-softmax attention over
//         the job's chunks of 64-position pages, streamed through the ring and
//         carried across chunks; the last job of a (row, kv head) to finish
//         merges the jobs' partials
// Tasks are numbered stage-major, group-minor, and CTA c runs tasks c, c + G,
// c + 2G, ... in order. A task waits until its group's previous stage has
// completed (a release/acquire counter per (group, stage)); every task waits
// only on tasks with smaller numbers and all CTAs are resident (cooperative
// launch), so the smallest unfinished task can always run.
//
// Data movement. Nothing a task reads from HBM depends on the step's
// arithmetic except its small input rows: a producer warp per CTA walks the
// CTA's task list ahead of the eight compute warps and bulk-copies weight
// tiles and (past-position) KV pages into a shared-memory ring as soon as the
// ring has room, so HBM streams the step's bytes behind the dependency chain.
// Weights are stored in HBM in "fragment" order (per 16-row tile and
// 16-column step, the 32 lanes' m16n8k16 A fragments): one contiguous copy
// lands a tile that each lane reads with one 16-byte shared load per k-step.
// Input rows are copied into a padded shared buffer after the wait.
//
// RMSNorm is folded as on the tensor-core path: norm weights are folded into
// the consuming projection's columns at load time; producers of the residual
// stream write per-16-column sums of squares, consumers scale their outputs by
// 1/rms. Every wait is bounded (about 2 s): on timeout the kernel records an
// error, raises an abort flag every waiter checks, and all CTAs return.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

constexpr int kThreads = 256;              // compute warps
constexpr int kWarps = kThreads / 32;
constexpr int kBlock = kThreads + 32;      // + the producer warp
constexpr int kSlots = 8;                  // ring entries in flight per CTA
constexpr int kRingBytes = kStepRingBytes;
constexpr int kXHalves = kStepGroupRows * 1032;  // input rows: 32 x (1024 + 8) or 16 x (2048 + 8) halves
constexpr int kXBytes = kXHalves * 2;
constexpr int kRedBytes = kWarps * kStepGroupRows * 16 * 4;  // one 16 x 32 partial tile per warp
constexpr int kYsumBytes = 2 * kStepGroupRows * 16 * 4;      // SwiGLU / argmax staging (2 tiles)
constexpr size_t kSmemBytes = size_t(kRingBytes) + kXBytes + kRedBytes + kYsumBytes + 128 /* align */;
constexpr int kMaxRows = kStepGroupRows * kStepMaxGroups;

enum TaskType : int { kEmb = 0, kQkv = 1, kAttn = 2, kO = 3, kGu = 4, kDown = 5, kLm = 6 };

// sync words: done[group][stage] | lm arrivals[group] | groups done | exits | abort
__device__ __forceinline__ unsigned* done_word(const StepArgs& a, int g, int st) {
  return a.sync + g * kStepMaxStages + st;
}
__device__ __forceinline__ unsigned* lm_arrive_word(const StepArgs& a, int g) {
  return a.sync + kStepMaxGroups * kStepMaxStages + g;
}
__device__ __forceinline__ unsigned* groups_done_word(const StepArgs& a) {
  return a.sync + kStepMaxGroups * kStepMaxStages + kStepMaxGroups;
}
__device__ __forceinline__ unsigned* exit_word(const StepArgs& a) { return groups_done_word(a) + 1; }
__device__ __forceinline__ unsigned* abort_word(const StepArgs& a) { return groups_done_word(a) + 2; }

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned* p) {
  unsigned v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void red_release(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// barrier of the eight compute warps (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// Self-checks of the indices the kernel derives (each records a distinct
// code in the error word and the access is skipped).
#define STEP_CHECK(cond, id) ((cond) ? true : (set_error(a.err, 100 + (id)), false))

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return (v > bv) || (v == bv && i < bi); }

struct Shared {
  uint64_t slot_bar[kSlots];
  uint64_t x_bar;
  int slot_off[kSlots];                 // written by the producer before it arms the slot
  unsigned long long slot_end[kSlots];  // producer only
  bool slot_armed[kSlots];              // producer: the slot's last entry copies bytes
  unsigned slot_par;                    // at exit: the phases the unconsumed slots expect
  volatile int consumed;                // ring entries the compute warps have finished
  volatile int abort;
  int produced;                         // ring entries the producer issued (exit drain)
  int signal, last, first_unconsumed;
  float rs[kStepGroupRows];
  int row_slot[kMaxRows];  // per batch row: sequence slot and cached positions (fixed during the step)
  int row_pos[kMaxRows];
};

struct Task {
  int type, layer, st, g, i;
  int rows;        // rows of the group
  int tg, r0, nr;  // projections: tile group, first row of the row block, rows in it
};

__device__ __forceinline__ int group_rows(const StepArgs& a, int g) {
  const int r = a.B - g * kStepGroupRows;
  return r < kStepGroupRows ? r : kStepGroupRows;
}
__device__ __forceinline__ bool is_gemm(int type) { return type != kEmb && type != kAttn; }
__device__ __forceinline__ int gemm_k(const StepArgs& a, int type) {
  return type == kO ? a.nq * a.hd : type == kDown ? a.I : a.H;
}
__device__ __forceinline__ int gemm_rows(const StepArgs& a, int type) {
  return type == kQkv ? a.NQKV : type == kGu ? 2 * a.I : type == kLm ? a.V : a.H;
}
// rows of a projection task's row block: the input rows must fit the shared buffer
__device__ __forceinline__ int block_rows(const StepArgs& a, int type) {
  return gemm_k(a, type) + 8 <= kXHalves / kStepGroupRows ? kStepGroupRows : kStepGroupRows / 2;
}
__device__ __forceinline__ int row_blocks(const StepArgs& a, int type, int rows) {
  const int rb = block_rows(a, type);
  return (rows + rb - 1) / rb;
}

__device__ __forceinline__ Task decode_task(const StepArgs& a, const int* offs, int t) {
  int lo = 0, hi = a.stages * a.groups;  // the last (stage, group) whose first task is <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= t) lo = mid;
    else hi = mid;
  }
  Task k;
  k.st = lo / a.groups;
  k.g = lo % a.groups;
  k.i = t - offs[lo];
  k.rows = group_rows(a, k.g);
  if (k.st == 0) {
    k.type = kEmb;
    k.layer = 0;
  } else if (k.st == a.stages - 1) {
    k.type = kLm;
    k.layer = a.L;
  } else {
    k.type = kQkv + (k.st - 1) % 5;
    k.layer = (k.st - 1) / 5;
  }
  k.tg = k.r0 = k.nr = 0;
  if (is_gemm(k.type)) {
    const int nrb = row_blocks(a, k.type, k.rows), rb = block_rows(a, k.type);
    k.tg = k.i / nrb;
    k.r0 = (k.i % nrb) * rb;
    k.nr = min(rb, k.rows - k.r0);
  }
  return k;
}

// completions of stage type `type` a group of `rows` rows reaches
__device__ __forceinline__ unsigned stage_need(const StepArgs& a, int type, int rows) {
  switch (type) {
    case kEmb: return unsigned(rows);
    case kAttn: return unsigned(rows * a.nkv);
    default: return unsigned(a.tasks[type] * row_blocks(a, type, rows));
  }
}

__device__ __forceinline__ const __half* gemm_w(const StepArgs& a, const Task& k) {
  const StepLayer& l = a.layer[k.layer < kStepMaxLayers ? k.layer : 0];
  switch (k.type) {
    case kQkv: return l.qkv;
    case kO: return l.o;
    case kGu: return l.gu;
    case kDown: return l.down;
    default: return a.lm;
  }
}
__device__ __forceinline__ const __half* gemm_x(const StepArgs& a, int type) {
  return type == kO ? a.attn16 : type == kDown ? a.act16 : a.h16;
}
// 16-row tiles of task k (the last tile group of a stage may have fewer)
__device__ __forceinline__ int gemm_tiles(const StepArgs& a, const Task& k) {
  const int T = a.tiles[k.type], total = gemm_rows(a, k.type) / 16;
  const int left = total - k.tg * T;
  return left < T ? left : T;
}

__device__ __forceinline__ size_t page_slab(int page, int layer, int layers, int kv, int nkv, int h, int tile) {
  return ((((size_t)page * layers + layer) * 2 + kv) * nkv + h) * (size_t)tile;
}

// Attention job geometry. A (row, kv head) pair's context is cut into chunks
// of split_pages 64-position pages (one ring entry each); its chunks are
// dealt to s_max jobs of job_chunks consecutive chunks. A job streams its
// chunks through the ring and carries the online softmax across them; jobs
// of the same pair write partials that the last one to finish merges.
struct AttnGeo {
  int b, h, s, slot, pos, pages, c0, c1, p0, p1, nsplits;
  bool valid, last;
};
__device__ __forceinline__ AttnGeo attn_geo(const StepArgs& a, const Shared& sh, const Task& k) {
  AttnGeo q;
  const int per_row = a.nkv * a.s_max;
  const int bl = k.i / per_row;
  q.h = (k.i % per_row) / a.s_max;
  q.s = k.i % a.s_max;
  q.b = k.g * kStepGroupRows + bl;
  q.slot = sh.row_slot[q.b];
  q.pos = sh.row_pos[q.b];
  q.pages = q.pos / kPageTokens + 1;
  q.valid = q.last = false;
  q.c0 = q.c1 = q.p0 = q.p1 = q.nsplits = 0;
  if (q.pos < 0 || q.pos >= a.max_pos || q.pages > a.max_pages) return q;  // the host never lets this happen
  const int nch = (q.pages + a.split_pages - 1) / a.split_pages;
  q.nsplits = (nch + a.job_chunks - 1) / a.job_chunks;
  q.c0 = q.s * a.job_chunks;
  q.c1 = min(nch, q.c0 + a.job_chunks);
  q.valid = q.c0 < nch;
  q.p0 = q.c0 * a.split_pages;
  q.p1 = min(q.pages, q.c1 * a.split_pages);
  q.last = q.valid && q.p1 == q.pages;
  return q;
}
// ring entries of a task: one per attention chunk, else one
__device__ __forceinline__ int task_entries(const Task& k, const AttnGeo& g) {
  return (k.type == kAttn && g.valid) ? g.c1 - g.c0 : 1;
}
// pages of entry ce of an attention job
__device__ __forceinline__ void chunk_pages(const StepArgs& a, const AttnGeo& g, int ce, int* p0, int* p1) {
  *p0 = g.p0 + ce * a.split_pages;
  *p1 = min(g.p1, *p0 + a.split_pages);
}
// bytes entry ce of a task prefetches into the ring (0: none)
__device__ __forceinline__ int entry_bytes(const StepArgs& a, const Task& k, const AttnGeo& geo, int ce) {
  if (is_gemm(k.type)) return gemm_tiles(a, k) * 16 * gemm_k(a, k.type) * 2;
  if (k.type == kAttn && geo.valid) {
    int p0, p1;
    chunk_pages(a, geo, ce, &p0, &p1);
    return (p1 - p0) * 2 * kPageTokens * a.hd * 2;
  }
  return 0;
}

// producer warp: issue the copies of entry ce of a task into `dst` (lane 0
// issues; the lanes look up up to 32 page-table entries at once)
__device__ void issue_prefetch(const StepArgs& a, const Task& k, const AttnGeo& geo, int ce, uint8_t* dst, int bytes,
                               uint64_t* bar, int lane) {
  if (is_gemm(k.type)) {
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, uint32_t(bytes));
      const int K = gemm_k(a, k.type);
      bulk_g2s(dst, gemm_w(a, k) + size_t(k.tg) * a.tiles[k.type] * 16 * K, uint32_t(bytes), bar);
    }
    return;
  }
  const int tile = kPageTokens * a.hd;
  int p0, p1;
  chunk_pages(a, geo, ce, &p0, &p1);
  const int np = p1 - p0;
  int my_page = -1;
  if (lane < np) my_page = __ldcg(a.block_table + (size_t)geo.slot * a.max_pages + p0 + lane);
  if (lane < np && (my_page < 0 || my_page >= a.n_pages)) {  // unreserved (or corrupt) entry: skip the copy
    set_error(a.err, kDevNoPage);
    my_page = -1;
  }
  if (lane == 0) mbar_arrive_expect_tx(bar, uint32_t(bytes));
  int missing = 0;
  for (int p = 0; p < np; ++p) {
    const int page = __shfl_sync(0xffffffffu, my_page, p);
    if (lane != 0) continue;
    __half* d = reinterpret_cast<__half*>(dst) + size_t(p) * 2 * tile;
    if (page >= 0) {
      bulk_g2s(d, a.kv_pool + page_slab(page, k.layer, a.L, 0, a.nkv, geo.h, tile), uint32_t(tile * 2), bar);
      bulk_g2s(d + tile, a.kv_pool + page_slab(page, k.layer, a.L, 1, a.nkv, geo.h, tile), uint32_t(tile * 2), bar);
    } else {
      missing += tile * 4;
    }
  }
  // an unreserved page (recorded above) still owes its transaction bytes
  if (lane == 0 && missing > 0)
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(uint32_t(missing))
                 : "memory");
}

// compute thread: bounded wait on a copy; on timeout the error is recorded
// and the run aborts after this task (the task still runs to its end on
// whatever the buffer holds, so that every compute thread reaches the same
// barriers)
__device__ __forceinline__ void wait_bar(uint64_t* bar, unsigned par, const StepArgs& a, Shared& sh) {
  if (!mbar_wait_bounded(bar, par, a.err)) {
    sh.abort = 1;
    atomicExch(abort_word(a), 1u);
  }
}

// 1/rms of the block's input rows from the per-16-column sums of squares
// (8 threads per row)
__device__ __forceinline__ void compute_rs(const StepArgs& a, const Task& k, Shared& sh) {
  const int tid = threadIdx.x;
  const int col = tid >> 3, j = tid & 7;
  const int P = a.H / 16;
  float s = 0.f;
  if (col < k.nr) {
    const float* p = a.ssp + size_t(k.g * kStepGroupRows + k.r0 + col) * P;
    for (int c = j; c < P; c += 8) s += __ldcg(p + c);
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (j == 0) sh.rs[col] = col < k.nr ? 1.0f / sqrtf(s / float(a.H) + a.eps) : 1.f;
}

// warp 0 of the compute warps: copy the block's input rows into the shared
// buffer, one bulk copy per lane (lane 0 arms the barrier with the total)
__device__ __forceinline__ void issue_x_warp(const StepArgs& a, const Task& k, Shared& sh, __half* xs, int lane) {
  const int K = gemm_k(a, k.type), XS = K + 8;
  const __half* x = gemm_x(a, k.type) + size_t(k.g * kStepGroupRows + k.r0) * K;
  if (lane == 0) mbar_arrive_expect_tx(&sh.x_bar, uint32_t(k.nr * K * 2));
  __syncwarp();
  if (lane < k.nr) {
    fence_proxy_async_global();  // the rows were written (generic proxy) by other CTAs
    if (STEP_CHECK(k.g * kStepGroupRows + k.r0 + lane < a.B && k.nr * XS <= kXHalves, 12))
      bulk_g2s(xs + lane * XS, x + size_t(lane) * K, uint32_t(K * 2), &sh.x_bar);
  }
}

// ------------------------------------------------------------ projection tasks
// T (1 or 2) 16-row weight tiles x up to 32 input rows. Warp w works on tile
// w % T and every (8 / T)-th 16-column step of it; the partial tiles meet in
// shared memory.
__device__ void gemm_task(const StepArgs& a, const Task& k, Shared& sh, const uint8_t* ring, __half* xs, float* red,
                          float* ysum, int slot, unsigned& par, unsigned& xpar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = gemm_k(a, k.type), XS = K + 8, nk = K / 16;
  const int T = gemm_tiles(a, k);
  const int tile0 = k.tg * a.tiles[k.type];
  const bool normed = k.type == kQkv || k.type == kGu || k.type == kLm;
  const bool resid = k.type == kO || k.type == kDown;
  const int nout = T * 16 * kStepGroupRows;  // (tile, col, row) outputs
  const int b0 = k.g * kStepGroupRows + k.r0;
  // residual values of this thread's outputs, loaded while the inputs land
  float hv[4] = {0.f, 0.f, 0.f, 0.f};
  if (resid) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int idx = tid + m * kThreads;
      const int tt = idx >> 9, col = (idx >> 4) & 31, row = idx & 15;
      if (idx < nout && col < k.nr) hv[m] = __ldcg(a.h + size_t(b0 + col) * a.H + (tile0 + tt) * 16 + row);
    }
  }
  if (normed) compute_rs(a, k, sh);

  const int nt = (k.nr + 7) >> 3;
  const int my_tile = warp % T, slice = warp / T, nslices = (kWarps - my_tile + T - 1) / T;
  float acc[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  const int xr = (lane & 7) + ((lane >> 4) & 1) * 8;
  const uint32_t xbase = smem_u32(xs + xr * XS + ((lane >> 3) & 1) * 8);
  const uint32_t xbase2 = xbase + uint32_t(16 * XS * 2);
  wait_bar(&sh.slot_bar[slot], (par >> slot) & 1u, a, sh);
  par ^= 1u << slot;
  const uint4* wf = reinterpret_cast<const uint4*>(ring + sh.slot_off[slot]) + size_t(my_tile) * nk * 32;
  {
    AttnGeo none{};
    const int bytes = entry_bytes(a, k, none, 0);
    if (!STEP_CHECK(sh.slot_off[slot] >= 0 && sh.slot_off[slot] + bytes <= kRingBytes &&
                        (my_tile + 1) * nk * 32 * 16 <= bytes && XS * 2 * (nt > 2 ? 32 : 16) <= kXBytes,
                    14))
      wf = reinterpret_cast<const uint4*>(ring);
  }
  wait_bar(&sh.x_bar, xpar & 1u, a, sh);
  xpar ^= 1u;
  // two k-steps per iteration: both steps' loads before their mma
  int kk = slice;
  for (; kk + nslices < nk; kk += 2 * nslices) {
    const uint4 w0 = wf[kk * 32 + lane], w1 = wf[(kk + nslices) * 32 + lane];
    uint32_t p0, p1, p2, p3, q0, q1, q2, q3;
    ldsm_x4(xbase + uint32_t(kk * 32), p0, p1, p2, p3);
    ldsm_x4(xbase + uint32_t((kk + nslices) * 32), q0, q1, q2, q3);
    mma16816(acc[0], w0.x, w0.y, w0.z, w0.w, p0, p1);
    if (nt > 1) mma16816(acc[1], w0.x, w0.y, w0.z, w0.w, p2, p3);
    mma16816(acc[0], w1.x, w1.y, w1.z, w1.w, q0, q1);
    if (nt > 1) mma16816(acc[1], w1.x, w1.y, w1.z, w1.w, q2, q3);
    if (nt > 2) {
      ldsm_x4(xbase2 + uint32_t(kk * 32), p0, p1, p2, p3);
      ldsm_x4(xbase2 + uint32_t((kk + nslices) * 32), q0, q1, q2, q3);
      mma16816(acc[2], w0.x, w0.y, w0.z, w0.w, p0, p1);
      if (nt > 3) mma16816(acc[3], w0.x, w0.y, w0.z, w0.w, p2, p3);
      mma16816(acc[2], w1.x, w1.y, w1.z, w1.w, q0, q1);
      if (nt > 3) mma16816(acc[3], w1.x, w1.y, w1.z, w1.w, q2, q3);
    }
  }
  if (kk < nk) {
    const uint4 w0 = wf[kk * 32 + lane];
    uint32_t p0, p1, p2, p3;
    ldsm_x4(xbase + uint32_t(kk * 32), p0, p1, p2, p3);
    mma16816(acc[0], w0.x, w0.y, w0.z, w0.w, p0, p1);
    if (nt > 1) mma16816(acc[1], w0.x, w0.y, w0.z, w0.w, p2, p3);
    if (nt > 2) {
      ldsm_x4(xbase2 + uint32_t(kk * 32), p0, p1, p2, p3);
      mma16816(acc[2], w0.x, w0.y, w0.z, w0.w, p0, p1);
      if (nt > 3) mma16816(acc[3], w0.x, w0.y, w0.z, w0.w, p2, p3);
    }
  }
  // partial tiles: red[warp][col][row]
  {
    const int g = lane >> 2, t = lane & 3;
    float* rw = red + warp * (kStepGroupRows * 16);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int c = n * 8 + 2 * t;
      rw[c * 16 + g] = acc[n][0];
      rw[(c + 1) * 16 + g] = acc[n][1];
      rw[c * 16 + g + 8] = acc[n][2];
      rw[(c + 1) * 16 + g + 8] = acc[n][3];
    }
  }
  csync();
  ArgBest* best = reinterpret_cast<ArgBest*>(ysum);  // LM: [T][32] per-tile column maxima
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int idx = tid + m * kThreads;
    const bool live = idx < nout;
    const int tt = idx >> 9, col = (idx >> 4) & 31, row = idx & 15;
    float y = 0.f;
    if (live)
      for (int w = tt; w < kWarps; w += T) y += red[w * (kStepGroupRows * 16) + col * 16 + row];
    const bool ok = live && col < k.nr;
    const int b = b0 + col;
    const int n = (tile0 + tt) * 16 + row;
    if (normed) y *= sh.rs[col];
    if (k.type == kQkv) {
      if (ok && STEP_CHECK(b < a.B && n < a.NQKV, 2)) a.qkv[size_t(b) * a.NQKV + n] = y;
    } else if (resid) {
      float hn = 0.f;
      if (ok && STEP_CHECK(b < a.B && n < a.H && tile0 + tt < a.H / 16, 3)) {
        const size_t i2 = size_t(b) * a.H + n;
        hn = hv[m] + y;
        a.h[i2] = hn;
        a.h16[i2] = __float2half_rn(hn);
      }
      float sq = hn * hn;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if (ok && row == 0) a.ssp[size_t(b) * (a.H / 16) + tile0 + tt] = sq;
    } else if (k.type == kGu) {
      if (live) ysum[idx] = y;
    } else {  // kLm: logits and this tile's first maximum per row
      if (ok && a.logits && STEP_CHECK(b < a.B && n < a.V, 9)) a.logits[size_t(b) * a.V + n] = y;
      float bv = ok ? y : -INFINITY;
      int bi = ok ? n : 0x7fffffff;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (live && row == 0) best[tt * kStepGroupRows + col] = {bv, bi};
    }
  }
  if (k.type == kGu) {  // gate rows 0-7 and up rows 8-15 of each tile
    csync();
    for (int idx = tid; idx < T * 8 * kStepGroupRows; idx += kThreads) {
      const int tt = idx / (8 * kStepGroupRows), rem = idx % (8 * kStepGroupRows);
      const int col = rem / 8, row = rem % 8;
      if (col < k.nr && STEP_CHECK(b0 + col < a.B && (tile0 + tt) * 8 + row < a.I, 4)) {
        const float gv = ysum[(tt * kStepGroupRows + col) * 16 + row];
        const float uv = ysum[(tt * kStepGroupRows + col) * 16 + row + 8];
        a.act16[size_t(b0 + col) * a.I + (tile0 + tt) * 8 + row] = __float2half_rn((gv / (1.0f + expf(-gv))) * uv);
      }
    }
  } else if (k.type == kLm) {
    csync();
    if (tid < k.nr) {
      ArgBest bb = best[tid];
      for (int tt = 1; tt < T; ++tt)
        if (better(best[tt * kStepGroupRows + tid].v, best[tt * kStepGroupRows + tid].i, bb.v, bb.i))
          bb = best[tt * kStepGroupRows + tid];
      ArgBest* part = reinterpret_cast<ArgBest*>(a.lm_part);
      if (STEP_CHECK(k.g < kStepMaxGroups && k.tg < a.tasks[kLm] && k.r0 + tid < kStepGroupRows, 8))
        part[(size_t(k.g) * a.tasks[kLm] + k.tg) * kStepGroupRows + k.r0 + tid] = bb;
    }
  }
}

// last LM task of a group: argmax over the per-tile partials, next tokens,
// positions, token history
__device__ void lm_finish(const StepArgs& a, const Shared& sh, const Task& k) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nlm = a.tasks[kLm];
  const ArgBest* part = reinterpret_cast<const ArgBest*>(a.lm_part) + size_t(k.g) * nlm * kStepGroupRows;
  for (int bl = warp; bl < k.rows; bl += kWarps) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < nlm; c += 32) {
      const float v = __ldcg(&part[size_t(c) * kStepGroupRows + bl].v);
      const int i = __ldcg(&part[size_t(c) * kStepGroupRows + bl].i);
      if (better(v, i, bv, bi)) {
        bv = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      const int b = k.g * kStepGroupRows + bl;
      const int next = (bi >= 0 && bi < a.V) ? bi : 0;
      a.tokens[b] = next;
      if (a.next_out) a.next_out[b] = next;
      a.seq_pos[sh.row_slot[b]] = sh.row_pos[b] + 1;
      if (a.hist) {
        const int step = *(volatile int*)a.hist_step;
        a.hist[size_t(step % a.hist_cap) * a.hist_stride + b] = next;  // a ring
      }
    }
  }
}

// ------------------------------------------------------------ EMB task
__device__ void emb_task(const StepArgs& a, const Task& k) {
  const int tid = threadIdx.x;
  const int b = k.g * kStepGroupRows + k.i;
  int tok = __ldcg(a.tokens + b);
  if (tok < 0 || tok >= a.V) {
    if (tid == 0) set_error(a.err, kDevBadToken);
    tok = 0;
  }
  const float* src = a.embed + size_t(tok) * a.H;
  for (int e0 = 0; e0 < a.H; e0 += kThreads) {
    const int e = e0 + tid;
    float x = 0.f;
    if (e < a.H) {
      x = src[e];
      a.h[size_t(b) * a.H + e] = x;
      a.h16[size_t(b) * a.H + e] = __float2half_rn(x);
    }
    float sq = x * x;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (e < a.H && (e & 15) == 0) a.ssp[size_t(b) * (a.H / 16) + e / 16] = sq;
  }
}

// ------------------------------------------------------------ ATTN task
// per-head RMSNorm (decoder_layer.cpp:32-42) + rotate-half RoPE
// (decoder_layer.cpp:139-152) of one head by one warp, fp16 result
template <int HD>
__device__ __forceinline__ void norm_rope(const float* src, const float* w, const float* cos_r, const float* sin_r,
                                          float eps, __half* dst, int lane) {
  constexpr int HALF = HD / 2;
  constexpr int PER = (HALF + 31) / 32;
  float f[PER], s2[PER];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int d = lane + 32 * j;
    f[j] = d < HALF ? __ldcg(src + d) : 0.f;
    s2[j] = d < HALF ? __ldcg(src + d + HALF) : 0.f;
    ss += f[j] * f[j] + s2[j] * s2[j];
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / float(HD) + eps);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int d = lane + 32 * j;
    if (d < HALF) {
      const float x1 = f[j] * (scale * w[d]);
      const float x2 = s2[j] * (scale * w[d + HALF]);
      const float c = cos_r[d], sn = sin_r[d];
      dst[d] = __float2half_rn(x1 * c - x2 * sn);
      dst[d + HALF] = __float2half_rn(x2 * c + x1 * sn);
    }
  }
}

template <int HD>
__device__ void attn_task(const StepArgs& a, const Task& k, Shared& sh, const uint8_t* ring, uint8_t* scratch,
                          int e0, unsigned& par) {
  constexpr int CPR = HD / 8, TILE = kPageTokens * HD, KC = HD / 16;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const AttnGeo q = attn_geo(a, sh, k);
  if (!q.valid) return;
  const int rep = a.nq / a.nkv;
  const StepLayer& L = a.layer[k.layer];
  __half* q_s = reinterpret_cast<__half*>(scratch);                 // [8][HD]
  __half* kvn = q_s + 8 * HD;                                         // [2][HD]
  float* comb = reinterpret_cast<float*>(scratch + (8 + 2) * HD * 2);  // [warps][rep][HD + 2]
  const float* row = a.qkv + size_t(q.b) * a.NQKV;
  const float* cos_r = a.rope_cos + size_t(q.pos) * (HD / 2);
  const float* sin_r = a.rope_sin + size_t(q.pos) * (HD / 2);
  if (warp < rep) {
    norm_rope<HD>(row + size_t(q.h * rep + warp) * HD, L.q_norm, cos_r, sin_r, a.eps, q_s + warp * HD, lane);
  } else {
    for (int d = lane; d < HD; d += 32) q_s[warp * HD + d] = __float2half_rn(0.f);
  }
  if (q.last) {
    if (warp == 6) norm_rope<HD>(row + size_t(a.nq + q.h) * HD, L.k_norm, cos_r, sin_r, a.eps, kvn, lane);
    if (warp == 7)
      for (int d = lane; d < HD; d += 32)
        kvn[HD + d] = __float2half_rn(__ldcg(row + size_t(a.nq + a.nkv + q.h) * HD + d));
  }
  csync();
  const int ctx = q.pos + 1;
  const int g = lane >> 2, t = lane & 3;
  const float sl2 = 1.4426950408889634f / sqrtf(float(HD));
  uint32_t qb0[KC], qb1[KC];
#pragma unroll
  for (int kc = 0; kc < KC; ++kc) {
    qb0[kc] = *reinterpret_cast<const uint32_t*>(q_s + g * HD + 16 * kc + 2 * t);
    qb1[kc] = *reinterpret_cast<const uint32_t*>(q_s + g * HD + 16 * kc + 8 + 2 * t);
  }
  float mA = -1e30f, mB = -1e30f, lA = 0.f, lB = 0.f;
  float o[KC][4];
#pragma unroll
  for (int mt = 0; mt < KC; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  // ---- the job's chunks, one ring entry each, softmax state carried across
  const int nch = q.c1 - q.c0;
  for (int ce = 0; ce < nch; ++ce) {
    const int slot = (e0 + ce) % kSlots;
    int cp0, cp1;
    chunk_pages(a, q, ce, &cp0, &cp1);
    wait_bar(&sh.slot_bar[slot], (par >> slot) & 1u, a, sh);
    par ^= 1u << slot;
    __half* pages = const_cast<__half*>(reinterpret_cast<const __half*>(ring + sh.slot_off[slot]));
    if (!STEP_CHECK(sh.slot_off[slot] >= 0 && sh.slot_off[slot] + (cp1 - cp0) * 4 * TILE <= kRingBytes &&
                        cp1 > cp0 && cp1 - cp0 <= a.split_pages,
                    1))
      pages = reinterpret_cast<__half*>(const_cast<uint8_t*>(ring));
    if (q.last && cp1 == q.pages) {
      // the new K/V row: into the shared copy of the current page and into
      // the cache (after the page copy has landed, so the two never overlap)
      const int r = q.pos % kPageTokens;
      if (tid < 2 * CPR) {
        const int kv = tid / CPR, c = tid % CPR;
        const uint4 v = *reinterpret_cast<const uint4*>(kvn + kv * HD + c * 8);
        __half* sp = pages + size_t(cp1 - 1 - cp0) * 2 * TILE + kv * TILE + r * HD + swz_chunk(r, c, CPR) * 8;
        *reinterpret_cast<uint4*>(sp) = v;
        const int page = __ldcg(a.block_table + (size_t)q.slot * a.max_pages + q.pos / kPageTokens);
        if (page >= 0 && page < a.n_pages) {
          __half* gp =
              a.kv_pool + page_slab(page, k.layer, a.L, kv, a.nkv, q.h, TILE) + r * HD + swz_chunk(r, c, CPR) * 8;
          *reinterpret_cast<uint4*>(gp) = v;
        }
      }
      csync();
    }
    // per warp: 16-position units of the chunk's pages
    const int tok_begin = cp0 * kPageTokens, tok_end = min(ctx, cp1 * kPageTokens);
    const int units = (cp1 - cp0) * 4;
    for (int u = warp; u < units; u += kWarps) {
      const int pi = u >> 2, r0 = (u & 3) * 16;
      const int tok0 = tok_begin + pi * kPageTokens + r0;
      if (tok0 >= tok_end) continue;
      const __half* kt = pages + size_t(pi) * 2 * TILE;
      const __half* vt = kt + TILE;
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        const int rr = r0 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int chn = 2 * kc + (lane >> 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(smem_u32(kt + rr * HD + swz_chunk(rr, chn, CPR) * 8), a0, a1, a2, a3);
        mma16816(sc, a0, a1, a2, a3, qb0[kc], qb1[kc]);
      }
      const bool v0 = tok0 + g < tok_end, v1 = tok0 + g + 8 < tok_end;
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
      for (int mt = 0; mt < KC; ++mt) {
        o[mt][0] *= alA;
        o[mt][1] *= alB;
        o[mt][2] *= alA;
        o[mt][3] *= alB;
      }
      const uint32_t pb0 = movmatrix_t(pack_half2(pA0, pB0));
      const uint32_t pb1 = movmatrix_t(pack_half2(pA1, pB1));
#pragma unroll
      for (int mt = 0; mt < KC; ++mt) {
        const int rr = r0 + ((lane >> 4) & 1) * 8 + (lane & 7);
        const int chn = 2 * mt + ((lane >> 3) & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(smem_u32(vt + rr * HD + swz_chunk(rr, chn, CPR) * 8), a0, a1, a2, a3);
        mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
    // the chunk's ring entry is free once every warp is done with it
    csync();
    if (tid == 0) sh.consumed = e0 + ce + 1;
  }

  // ---- merge the warps: comb[warp][head][HD + 2] = (O, m, l)
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
      for (int mt = 0; mt < KC; ++mt) {
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
      for (int mt = 0; mt < KC; ++mt) {
        cw[hB * (HD + 2) + 16 * mt + g] = o[mt][1];
        cw[hB * (HD + 2) + 16 * mt + g + 8] = o[mt][3];
      }
      if (g == 0) {
        cw[hB * (HD + 2) + HD] = mB;
        cw[hB * (HD + 2) + HD + 1] = lBr;
      }
    }
  }
  csync();
  const size_t pstride = size_t(rep) * (HD + 2);
  const size_t out_off = size_t(q.b) * a.nq * HD + size_t(q.h) * rep * HD;
  float* part_bh = a.part + (size_t(q.b) * a.nkv + q.h) * a.s_max * pstride;
  for (int i = tid; i < rep * HD; i += kThreads) {
    const int j = i / HD, d = i % HD;
    float M = -1e30f;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, comb[(w * rep + j) * (HD + 2) + HD]);
    float Ls = 0.f, O = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float* cw = comb + (w * rep + j) * (HD + 2);
      const float f = exp2f(cw[HD] - M);
      Ls += cw[HD + 1] * f;
      O += cw[d] * f;
    }
    if (!STEP_CHECK(q.b < a.B && q.h < a.nkv && q.s < a.s_max && j < rep, 5)) continue;
    if (q.nsplits == 1) {
      a.attn16[out_off + i] = __float2half_rn(O / Ls);
    } else {
      float* pp = part_bh + q.s * pstride + j * (HD + 2);
      pp[d] = O;
      if (d == 0) {
        pp[HD] = M;
        pp[HD + 1] = Ls;
      }
    }
  }
  if (q.nsplits == 1) {
    if (tid == 0) sh.signal = 1;
    return;
  }
  // ---- the last job of this (row, kv head) to finish merges all jobs
  csync();
  if (tid == 0) {
    unsigned* cnt = a.arrive + size_t(q.b) * a.nkv + q.h;
    const unsigned prev = atom_add_acq_rel(cnt, 1u);
    sh.last = prev == unsigned(q.nsplits - 1);
    if (sh.last) *cnt = 0u;
  }
  csync();
  if (!sh.last) return;
  for (int i = tid; i < rep * HD; i += kThreads) {
    const int j = i / HD, d = i % HD;
    float M = -1e30f;
    for (int sp = 0; sp < q.nsplits; ++sp) M = fmaxf(M, __ldcg(part_bh + sp * pstride + j * (HD + 2) + HD));
    float Ls = 0.f, O = 0.f;
    for (int sp = 0; sp < q.nsplits; ++sp) {
      const float* pp = part_bh + sp * pstride + j * (HD + 2);
      const float f = exp2f(__ldcg(pp + HD) - M);
      Ls += __ldcg(pp + HD + 1) * f;
      O += __ldcg(pp + d) * f;
    }
    a.attn16[out_off + i] = __float2half_rn(O / Ls);
  }
  if (tid == 0) sh.signal = 1;
}

// ------------------------------------------------------------ the kernel
template <int HD>
__global__ void __launch_bounds__(kBlock, 1) step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* ring = base;
  __half* xs = reinterpret_cast<__half*>(base + kRingBytes);
  float* red = reinterpret_cast<float*>(base + kRingBytes + kXBytes);
  float* ysum = reinterpret_cast<float*>(base + kRingBytes + kXBytes + kRedBytes);
  __shared__ Shared sh;
  __shared__ int offs[kStepMaxStages * kStepMaxGroups + 1];

  const int tid = threadIdx.x, lane = tid & 31;
  const int n_offs = a.stages * a.groups + 1;
  for (int i = tid; i < n_offs; i += kBlock) offs[i] = a.offs[i];
  for (int b = tid; b < a.B; b += kBlock) {  // slots and positions are fixed until the step's end
    const int s = __ldcg(a.slots + b);
    sh.row_slot[b] = s;
    sh.row_pos[b] = __ldcg(a.seq_pos + s);
  }
  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sh.slot_bar[s], 1);
      sh.slot_armed[s] = false;
    }
    mbar_init(&sh.x_bar, 1);
    fence_mbar_init();
    sh.slot_par = 0u;
    sh.abort = 0;
    sh.consumed = 0;
    sh.produced = 0;
    sh.first_unconsumed = 0;
  }
  __syncthreads();
  const unsigned* abort_p = abort_word(a);
  const int G = int(gridDim.x);

  if (tid >= kThreads) {
    // ================================================= producer warp
    // walks this CTA's tasks (and their ring entries) ahead of the compute
    // warps: an entry may be issued once its slot's previous entry has been
    // consumed and the ring has room for it
    unsigned long long alloc = 0ull;
    int e = 0;
    bool ok = true;
    for (int jp = 0; ok; ++jp) {
      const int t = blockIdx.x + jp * G;
      if (t >= a.total_tasks) break;
      const Task k = decode_task(a, offs, t);
      AttnGeo geo{};
      if (k.type == kAttn) geo = attn_geo(a, sh, k);
      const int ne = task_entries(k, geo);
      for (int ce = 0; ce < ne; ++ce, ++e) {
        const int bytes = entry_bytes(a, k, geo, ce);
        const int s = e % kSlots;
        unsigned long long p = alloc;
        const uint64_t t0 = global_timer_ns();
        while (true) {
          const int done = sh.consumed;
          if (sh.abort) {
            ok = false;
            break;
          }
          if (e - done < kSlots) {
            if (bytes == 0) break;
            // live data occupies [free_pos, alloc) of the ring's linear address
            // space (nothing when every issued entry has been consumed)
            const unsigned long long free_pos = done > 0 ? sh.slot_end[(done - 1) % kSlots] : 0ull;
            p = alloc;
            const unsigned long long off = p % kRingBytes;
            if (off + bytes > kRingBytes) p += kRingBytes - off;  // no region wraps around the end
            const unsigned long long live_start = free_pos >= alloc ? p : free_pos;
            if (p + bytes - live_start <= kRingBytes) break;
          }
          if (ld_volatile(abort_p) != 0u || global_timer_ns() - t0 > 2000000000ull) {
            if (lane == 0) set_error(a.err, kDevWaitTimeout);
            ok = false;
            break;
          }
          __nanosleep(32);
        }
        if (!ok) break;
        if (bytes > kRingBytes || int(p % kRingBytes) + bytes > kRingBytes) {  // never: the plan caps entries
          if (lane == 0) set_error(a.err, kDevWaitTimeout);
          ok = false;
          break;
        }
        if (bytes > 0) {
          if (lane == 0) sh.slot_off[s] = int(p % kRingBytes);
          __syncwarp();
          issue_prefetch(a, k, geo, ce, ring + (p % kRingBytes), bytes, &sh.slot_bar[s], lane);
          alloc = p + bytes;
        }
        if (lane == 0) {
          sh.slot_end[s] = alloc;
          sh.slot_armed[s] = bytes > 0;
        }
        __syncwarp();
      }
    }
    if (lane == 0) sh.produced = e;
  } else {
    // ================================================= compute warps
    unsigned par = 0u, xpar = 0u;  // mbarrier phases each compute thread expects next
    int e = 0;                      // ring entries consumed
    for (int j = 0;; ++j) {
      const int t = blockIdx.x + j * G;
      if (t >= a.total_tasks) break;
      const Task k = decode_task(a, offs, t);
      if (tid == 0) {
        if (a.trace) {
          a.trace[size_t(t) * 8] = blockIdx.x;
          a.trace[size_t(t) * 8 + 1] = global_timer_ns();
        }
        if (k.st > 0) {  // the group's previous stage must be complete
          const int prev = k.st == 1 ? kEmb : (k.type == kLm || k.type == kQkv ? kDown : k.type - 1);
          const unsigned need = stage_need(a, prev, k.rows);
          const unsigned* w = done_word(a, k.g, k.st - 1);
          if (ld_acquire(w) < need) {
            const uint64_t t0 = global_timer_ns();
            while (ld_acquire(w) < need) {
              if (ld_volatile(abort_p) != 0u) {
                sh.abort = 1;
                break;
              }
              if (global_timer_ns() - t0 > 2000000000ull) {
                set_error(a.err, kDevWaitTimeout);
                atomicExch(abort_word(a), 1u);
                sh.abort = 1;
                break;
              }
            }
          }
        }
      }
      if (warp_id() == 0) {  // the block's input rows, one copy per lane, once lane 0 saw them complete
        __syncwarp();
        if (!sh.abort && is_gemm(k.type)) issue_x_warp(a, k, sh, xs, lane);
      }
      if (tid == 0 && a.trace) a.trace[size_t(t) * 8 + 2] = global_timer_ns();
      csync();
      if (sh.abort) break;
      if (tid == 0) sh.signal = 0;  // (the previous task's signaller has read it: it passed the barrier above)
      AttnGeo geo{};
      if (k.type == kAttn) geo = attn_geo(a, sh, k);
      const int ne = task_entries(k, geo);
      switch (k.type) {
        case kEmb: emb_task(a, k); break;
        case kAttn: attn_task<HD>(a, k, sh, ring, reinterpret_cast<uint8_t*>(xs), e, par); break;
        default: gemm_task(a, k, sh, ring, xs, red, ysum, e % kSlots, par, xpar); break;
      }
      e += ne;
      csync();
      if (tid == 0) {
        if (a.trace) a.trace[size_t(t) * 8 + 3] = global_timer_ns();
        sh.consumed = e;  // the task's ring entries are free again
        if (k.type == kLm)
          sh.last = atom_add_acq_rel(lm_arrive_word(a, k.g), 1u) ==
                    unsigned(a.tasks[kLm] * row_blocks(a, kLm, k.rows) - 1);
      }
      // completion: every stage but ATTN counts each task; ATTN counts a
      // (row, kv head) when its output row is final. Another thread than the
      // one that starts the next task signals, so the two overlap.
      if (tid == 32 && k.type != kLm && (k.type != kAttn || sh.signal)) {
        red_release(done_word(a, k.g, k.st), 1u);
        if (a.trace) a.trace[size_t(t) * 8 + 4] = global_timer_ns();
      }
      if (k.type == kLm) {
        csync();
        if (sh.last) {
          lm_finish(a, sh, k);
          csync();
          if (tid == 0) {
            *lm_arrive_word(a, k.g) = 0u;
            if (atom_add_acq_rel(groups_done_word(a), 1u) == unsigned(a.groups - 1)) {
              *groups_done_word(a) = 0u;
              if (a.hist_step) *a.hist_step += 1;
            }
          }
        }
      }
    }
    if (tid == 0) {
      sh.first_unconsumed = e;
      sh.slot_par = par;      // the phases its slots expect
      sh.consumed = 1 << 30;  // releases a producer still waiting for room
    }
  }
  __syncthreads();
  if (tid == 0) {
    // ring entries an aborted run never consumed must land before the CTA
    // exits (bounded: a copy that never completes is already an error). The
    // unconsumed entries hold distinct slots; the armed ones copy bytes.
    for (int ee = sh.first_unconsumed; ee < sh.produced; ++ee) {
      const int s = ee % kSlots;
      if (sh.slot_armed[s]) mbar_wait_bounded(&sh.slot_bar[s], (sh.slot_par >> s) & 1u, a.err);
    }
    // every CTA has finished its tasks once the exit count is full: the last
    // one resets the step's counters for the next launch
    if (atom_add_acq_rel(exit_word(a), 1u) == gridDim.x - 1) {
      for (int g = 0; g < a.groups; ++g) {
        for (int st = 0; st < a.stages; ++st) *done_word(a, g, st) = 0u;
        *lm_arrive_word(a, g) = 0u;
      }
      *groups_done_word(a) = 0u;
      *abort_word(a) = 0u;
      __threadfence();
      *exit_word(a) = 0u;
    }
  }
}

__global__ void pack_fragments_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int64_t N, int64_t K) {
  const int64_t total = N * K;
  for (int64_t o = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; o < total; o += int64_t(gridDim.x) * blockDim.x) {
    const int64_t tile = o / (16 * K), rem = o % (16 * K);
    const int64_t kk = rem / 256, w = rem % 256;
    const int lane = int(w / 8), jx = int(w % 8);
    const int g = lane >> 2, t = lane & 3;
    const int reg = jx >> 1, hi = jx & 1;
    const int row = g + ((reg & 1) ? 8 : 0);
    const int col = 2 * t + hi + ((reg & 2) ? 8 : 0);
    dst[o] = src[(tile * 16 + row) * K + kk * 16 + col];
  }
}

template <int HD>
cudaError_t attr_step() {
  return set_kernel_smem(step_kernel<HD>, int(kSmemBytes));
}

template <int HD>
cudaError_t launch_hd(const StepArgs& a, int num_sms, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kBlock);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel<HD>, a);
}

}  // namespace

int step_max_split_pages(int hd) {
  const int page_bytes = 2 * kPageTokens * hd * 2;
  const int p = (kRingBytes * 5 / 8) / page_bytes;
  return p < 1 ? 1 : (p > 8 ? 8 : p);
}

void step_plan(StepArgs& a, int64_t max_ctx_tokens, int num_sms) {
  a.groups = (a.B + kStepGroupRows - 1) / kStepGroupRows;
  a.stages = 2 + 5 * a.L;
  const int64_t max_pages = (max_ctx_tokens + kPageTokens - 1) / kPageTokens;
  // projections: tiles per task so that a stage has at most about one task
  // per CTA, at most two tiles (the epilogue's staging) and half the ring
  const int rows_of[8] = {0, a.NQKV, 0, a.H, 2 * a.I, a.H, a.V, 0};
  const int k_of[8] = {0, a.H, 0, a.nq * a.hd, a.H, a.I, a.H, 0};
  for (int type = kQkv; type <= kLm; ++type) {
    if (type == kAttn) continue;
    const int tiles = rows_of[type] / 16;
    int T = (tiles * a.groups + num_sms - 1) / num_sms;
    const int cap = std::max(1, (kRingBytes / 2) / (16 * k_of[type] * 2));
    T = std::max(1, std::min(T, std::min(cap, 2)));
    a.tiles[type] = T;
    a.tasks[type] = (tiles + T - 1) / T;
  }
  // attention: chunks of up to `cap` pages (one ring entry each); each
  // (row, kv head) pair's chunks are dealt to s_max jobs of at most four
  // consecutive chunks, so that all groups' jobs cover about one CTA each
  const int cap = step_max_split_pages(a.hd);
  const int rows = std::max(1, std::min(a.B, kStepGroupRows));
  const int64_t pairs = int64_t(rows) * a.nkv * a.groups;
  const int64_t units = max_pages * pairs;  // page-units of the whole step's attention
  int sp = int((units + num_sms - 1) / num_sms);  // pages per CTA if spread evenly
  sp = sp < 1 ? 1 : (sp > cap ? cap : sp);
  a.split_pages = sp;
  const int nch = int((max_pages + sp - 1) / sp);  // chunks of the longest context
  int parts = int(std::max<int64_t>(1, num_sms / pairs));
  parts = std::min(parts, nch);
  int jc = (nch + parts - 1) / parts;
  jc = std::min(jc, 4);  // a job's chunks never reuse a ring slot
  a.job_chunks = jc;
  a.s_max = (nch + jc - 1) / jc;
  int t = 0;
  for (int st = 0; st < a.stages; ++st) {
    const int type = st == 0 ? kEmb : (st == a.stages - 1 ? kLm : kQkv + (st - 1) % 5);
    for (int g = 0; g < a.groups; ++g) {
      const int grows = std::min(kStepGroupRows, a.B - g * kStepGroupRows);
      a.offs[st * a.groups + g] = t;
      if (type == kEmb) {
        t += grows;
      } else if (type == kAttn) {
        t += grows * a.nkv * a.s_max;
      } else {  // tile groups x row blocks (16-row blocks when the input rows exceed 1024)
        const int rb = k_of[type] + 8 <= kXHalves / kStepGroupRows ? kStepGroupRows : kStepGroupRows / 2;
        t += a.tasks[type] * ((grows + rb - 1) / rb);
      }
    }
  }
  a.offs[a.stages * a.groups] = t;
  a.total_tasks = t;
}

cudaError_t step_init_attributes() {
  cudaError_t e = cudaSuccess, r;
  if ((r = attr_step<64>()) != cudaSuccess) e = r;
  if ((r = attr_step<96>()) != cudaSuccess) e = r;
  if ((r = attr_step<128>()) != cudaSuccess) e = r;
  return e;
}

cudaError_t launch_step(const StepArgs& a, int num_sms, cudaStream_t s) {
  if (a.B < 1 || a.B > kStepGroupRows * kStepMaxGroups || a.L > kStepMaxLayers || a.nq % a.nkv != 0 ||
      a.nq / a.nkv > 6 || a.H % 16 != 0 || a.NQKV % 16 != 0 || (2 * a.I) % 16 != 0 || a.V % 16 != 0 ||
      a.H > kStepMaxK || a.I > kStepMaxK || a.nq * a.hd > kStepMaxK || a.total_tasks <= 0 || a.sync == nullptr)
    return cudaErrorInvalidValue;
  switch (a.hd) {
    case 64: return launch_hd<64>(a, num_sms, s);
    case 96: return launch_hd<96>(a, num_sms, s);
    case 128: return launch_hd<128>(a, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pack_fragments(const __half* src, __half* dst, int64_t N, int64_t K, cudaStream_t s) {
  if (N % 16 != 0 || K % 16 != 0) return cudaErrorInvalidValue;
  pack_fragments_kernel<<<1184, 256, 0, s>>>(src, dst, N, K);
  return cudaGetLastError();
}

}  // namespace mmc
