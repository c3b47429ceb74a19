// One persistent tensor-core kernel for the back half of a decoder layer on
// the batched path (reference: decoder_layer.cpp:362-405, o_proj + residual,
// post-attention RMSNorm, gate/up + SwiGLU, down_proj + residual):
//
//   stage 0  hidden += attn16 . Wo^T         (+ fp16 rows, sums of squares)
//   stage 1  act16 = silu(g) * u, [g|u] = (h16 . Wgu^T) / rms  (norm folded into Wgu)
//   stage 2  hidden += act16 . Wdown^T       (+ fp16 rows, sums of squares)
//
// The tasks -- (stage, 128-row weight tile m, 16-row batch tile n) -- are
// numbered stage by stage and taken from one atomic queue, so every task a
// CTA waits for was claimed earlier by a running CTA and makes progress
// without waiting on anything later: the kernel cannot deadlock. A task of
// stage s reads the batch tile n that stage s-1 produced; it waits (bounded,
// acquire) until all stage s-1 tiles of n have been published (release), so
// one launch replaces three dependent launches and their ramps. Weight tiles
// need no dependency: the producer issues a task's first weight stages
// before it waits, and the first task's before griddepcontrol.wait.
//
// Warp roles (192 threads): warps 0-3 epilogue (warp w reads TMEM lanes
// 32w..32w+31), warp 4 lane 0 TMA producer and task scheduler, warp 5 TMEM
// allocation + lane 0 MMA issuer. Two TMEM accumulators let one task's
// epilogue overlap the next task's MMAs. The producer hands task ids to the
// MMA and epilogue warps through a 4-slot mailbox (mbarriers). Every wait is
// bounded (2 s) and reports through the error word.
#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace mmc {
namespace {

constexpr int CBN = 16;  // batch rows per task
constexpr int kChainThreads = 192;
constexpr int kChainStages = 4;
constexpr int kMailbox = 4;
constexpr int A_BYTES = UM * BK * 2, B_BYTES = CBN * BK * 2, ST_BYTES = A_BYTES + B_BYTES;

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// generic-proxy writes of this thread become visible to later async-proxy
// (TMA) reads of global memory, and vice versa
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Bounded spin until *p >= want (acquire). false: timed out (error recorded).
__device__ __forceinline__ bool wait_count(const unsigned* p, unsigned want, int* err) {
  if (ld_acquire(p) >= want) return true;
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire(p) < want) {
    if (global_timer_ns() - t0 > 2000000000ull) {
      set_error(err, kDevWaitTimeout);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

struct TaskInfo {
  int s, m, n, kt;  // stage, weight tile, batch tile, 64-wide k-steps
};

__device__ __forceinline__ TaskInfo decode_task(const ChainArgs& a, int t) {
  TaskInfo ti;
  const int nt = a.n_tiles;
  int base = 0;
  ti.s = 2;
  for (int s = 0; s < 3; ++s) {
    const int cnt = a.m_tiles[s] * nt;
    if (t < base + cnt) {
      ti.s = s;
      break;
    }
    base += cnt;
  }
  const int idx = t - base;
  ti.n = idx / a.m_tiles[ti.s];  // batch-tile major: tile 0's work finishes first
  ti.m = idx % a.m_tiles[ti.s];
  ti.kt = a.K[ti.s] / BK;
  return ti;
}

__global__ void __launch_bounds__(kChainThreads, 1) mlp_chain_kernel(const __grid_constant__ ChainArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[kChainStages], empty_bar[kChainStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2];
  __shared__ __align__(8) uint64_t box_full[kMailbox], box_empty[kMailbox];
  __shared__ int box[kMailbox];
  __shared__ uint32_t tmem_base_s;
  __shared__ float rs_s[CBN];
  __shared__ float ssw_s[4][CBN];
  __shared__ bool last_cta;
  __shared__ int abort_s, epi_task;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int total = (a.m_tiles[0] + a.m_tiles[1] + a.m_tiles[2]) * a.n_tiles;

  if (tid == 0) {
    abort_s = 0;
    for (int i = 0; i < kChainStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    for (int i = 0; i < kMailbox; ++i) {
      mbar_init(&box_full[i], 1);
      mbar_init(&box_empty[i], 5);  // MMA issuer + 4 epilogue warps
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(32u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 4) {
    // ============================================ producer + task scheduler
    // A timed-out dependency wait records the error and the pipeline carries
    // on with whatever the activations hold, so every stage's copies complete
    // and nothing is left in flight; a timed-out mailbox or ring wait stops
    // the scheduler (the other roles then stop on their own bounded waits).
    if (lane == 0) {
      bool waited_pdl = false;
      uint32_t g = 0;  // k-steps issued so far (ring position)
      for (int q = 0;; ++q) {
        const int b = q % kMailbox;
        bool ok = abort_s == 0;
        if (ok && q >= kMailbox) ok = mbar_wait_bounded(&box_empty[b], ((q / kMailbox) - 1) & 1, a.err);
        int t = ok ? int(atomicAdd(&a.sync[0], 1u)) : total;
        if (t >= total) t = -1;
        box[b] = t;
        mbar_arrive(&box_full[b]);
        if (t < 0) {
          if (!ok) abort_s = 1;
          break;
        }
        const TaskInfo ti = decode_task(a, t);
        const CUtensorMap* mw = &a.map_w[ti.s];
        const CUtensorMap* mx = &a.map_x[ti.s];
        // weight tiles of the first ring-full of k-steps go out before the
        // dependency wait, their activation tiles after it
        const int pre = ti.kt < kChainStages ? ti.kt : kChainStages;
        bool ring_ok = true;
        for (int kt = 0; kt < ti.kt && ring_ok; ++kt) {
          const uint32_t gi = g + kt, st = gi % kChainStages;
          if (kt == pre) {  // (only reached when kt > ring depth) handled in the loop below
            break;
          }
          if (gi >= kChainStages) ring_ok = mbar_wait_bounded(&empty_bar[st], ((gi / kChainStages) - 1) & 1, a.err);
          if (!ring_ok) break;
          mbar_arrive_expect_tx(&full_bar[st], uint32_t(ST_BYTES));
          tma_load_2d(smem + st * ST_BYTES, mw, kt * BK, ti.m * UM, &full_bar[st]);
        }
        if (!waited_pdl) {  // stage-0 inputs come from the previous kernel
          pdl_wait();
          waited_pdl = true;
        }
        if (!ring_ok) {
          abort_s = 1;
          break;  // stages already armed still get their weight bytes; the MMA issuer times out
        }
        if (ti.s > 0) {
          wait_count(&a.sync[2 + (ti.s - 1) * a.n_tiles + ti.n], unsigned(a.m_tiles[ti.s - 1]), a.err);
          fence_proxy_async_global();
        }
        for (int kt = 0; kt < pre; ++kt) {
          const uint32_t st = (g + kt) % kChainStages;
          tma_load_2d(smem + st * ST_BYTES + A_BYTES, mx, kt * BK, ti.n * CBN, &full_bar[st]);
        }
        for (int kt = pre; kt < ti.kt; ++kt) {
          const uint32_t gi = g + kt, st = gi % kChainStages;
          if (!mbar_wait_bounded(&empty_bar[st], ((gi / kChainStages) - 1) & 1, a.err)) {
            ring_ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[st], uint32_t(ST_BYTES));
          tma_load_2d(smem + st * ST_BYTES, mw, kt * BK, ti.m * UM, &full_bar[st]);
          tma_load_2d(smem + st * ST_BYTES + A_BYTES, mx, kt * BK, ti.n * CBN, &full_bar[st]);
        }
        g += uint32_t(ti.kt);
        if (!ring_ok) {
          abort_s = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ===================================================== MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16<CBN>();
      uint32_t g = 0;
      for (int q = 0;; ++q) {
        const int b = q % kMailbox;
        if (!mbar_wait_bounded(&box_full[b], (q / kMailbox) & 1, a.err)) break;
        const int t = box[b];
        mbar_arrive(&box_empty[b]);
        if (t < 0) break;
        const TaskInfo ti = decode_task(a, t);
        const int acc = q & 1;
        bool ok = q < 2 || mbar_wait_bounded(&acc_empty[acc], ((q / 2) - 1) & 1, a.err);
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * CBN);
        for (int kt = 0; kt < ti.kt && ok; ++kt, ++g) {
          const uint32_t st = g % kChainStages;
          if (!mbar_wait_bounded(&full_bar[st], (g / kChainStages) & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t as = smem_u32(smem + st * ST_BYTES), bs = as + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, sw128_desc(as + k * 32), sw128_desc(bs + k * 32), idesc, (kt | k) != 0);
          umma_commit(&empty_bar[st]);
        }
        umma_commit(&acc_full[acc]);  // the epilogue is released either way
        if (!ok) {
          abort_s = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ==================================================== epilogue warps
    // Waits are done by thread 0 and broadcast through shared memory, so the
    // four warps always take the same path through the named barriers.
    pdl_wait();
    pdl_launch_dependents();
    const int row_in_tile = warp * 32 + lane;
    for (int q = 0;; ++q) {
      const int b = q % kMailbox;
      if (tid == 0) {
        const bool ok = mbar_wait_bounded(&box_full[b], (q / kMailbox) & 1, a.err);
        epi_task = ok ? box[b] : -1;
      }
      epi_sync();
      const int t = epi_task;
      if (lane == 0) mbar_arrive(&box_empty[b]);
      if (t < 0) break;
      const TaskInfo ti = decode_task(a, t);
      const int acc = q & 1;
      const int n0 = ti.n * CBN, row = ti.m * UM + row_in_tile;
      const int N = a.N[ti.s];
      if (ti.s == 1 && tid < CBN) {
        // folded post-attention RMSNorm of the stage-0 output rows
        float r = 1.f;
        if (n0 + tid < a.B) {
          wait_count(&a.sync[2 + ti.n], unsigned(a.m_tiles[0]), a.err);  // already satisfied: orders the reads
          const int parts = (a.K[1] + UM - 1) / UM;
          float ss = 0.f;
          for (int m = 0; m < parts; ++m) ss += __ldcg(a.ss + size_t(n0 + tid) * parts + m);
          r = 1.0f / sqrtf(ss / float(a.K[1]) + a.eps);
        }
        rs_s[tid] = r;
      } else if (ti.s == 2 && tid == 0) {
        // the residual rows were last written by stage 0 (ordered through stage 1)
        wait_count(&a.sync[2 + a.n_tiles + ti.n], unsigned(a.m_tiles[1]), a.err);
      }
      if (tid == 0) mbar_wait_bounded(&acc_full[acc], (q / 2) & 1, a.err);
      epi_sync();
      tc_fence_after();
      float v[16];
      tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(acc * CBN), v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);  // accumulator free for the task after next
      if (ti.s == 1) {
        // gate rows 16j..16j+7 and up rows 16j+8..16j+15 sit 8 lanes apart
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = v[j] * rs_s[j];
          const float up = __shfl_down_sync(0xffffffffu, x, 8);
          const int bb = n0 + j;
          if ((lane & 8) == 0 && row < N && bb < a.B) {
            const int i = (row >> 4) * 8 + (row & 7);
            a.act16[size_t(bb) * (N / 2) + i] = __float2half_rn((x / (1.0f + expf(-x))) * up);
          }
        }
      } else {
        const int H = N;
        float nv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int bb = n0 + j;
          nv[j] = (row < H && bb < a.B) ? __ldcg(a.hidden + size_t(bb) * H + row) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int bb = n0 + j;
          if (row < H && bb < a.B) {
            nv[j] += v[j];
            a.hidden[size_t(bb) * H + row] = nv[j];
            a.h16[size_t(bb) * H + row] = __float2half_rn(nv[j]);
          } else {
            nv[j] = 0.f;
          }
        }
        float sq[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) sq[j] = nv[j] * nv[j];
        const float tot = colsum16(sq, lane);
        const int cj = colsum16_col(lane);
        if ((lane & 1) == 0) ssw_s[warp][cj] = tot;
        epi_sync();
        if (tid < CBN && n0 + tid < a.B) {
          const int parts = (H + UM - 1) / UM;
          a.ss[size_t(n0 + tid) * parts + ti.m] = ssw_s[0][tid] + ssw_s[1][tid] + ssw_s[2][tid] + ssw_s[3][tid];
        }
      }
      // publish this tile to the next stage's TMA reads (other CTAs)
      __threadfence();
      fence_proxy_async_global();
      epi_sync();
      if (tid == 0 && ti.s < 2) red_release_add(&a.sync[2 + ti.s * a.n_tiles + ti.n], 1u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc<32>(tmem);
  // the last CTA to leave resets the queue and the stage counters
  if (tid == 0) {
    __threadfence();
    last_cta = atomicAdd(&a.sync[1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last_cta) {
    __threadfence();
    for (int i = tid; i < 2 + 2 * a.n_tiles; i += kChainThreads) a.sync[i] = 0u;
  }
}

}  // namespace

int chain_sync_words(int B) { return 2 + 2 * ((B + CBN - 1) / CBN); }

cudaError_t mlp_chain_init_attributes() {
  return set_kernel_smem(mlp_chain_kernel, kChainStages * ST_BYTES + 1024);
}

cudaError_t launch_mlp_chain(const ChainArgs& a_in, int max_ctas, cudaStream_t s, bool pdl) {
  ChainArgs a = a_in;
  if (a.B < 1 || a.sync == nullptr) return cudaErrorInvalidValue;
  for (int i = 0; i < 3; ++i)
    if (a.K[i] % BK != 0 || a.N[i] <= 0) return cudaErrorInvalidValue;
  if (a.N[1] % 16 != 0 || a.N[0] != a.N[2] || a.K[1] != a.N[0] || a.K[2] * 2 != a.N[1]) return cudaErrorInvalidValue;
  a.n_tiles = (a.B + CBN - 1) / CBN;
  for (int i = 0; i < 3; ++i) a.m_tiles[i] = (a.N[i] + UM - 1) / UM;
  cudaError_t e;
  if ((e = tc_make_map(&a.map_w[0], a.Wo, a.N[0], a.K[0], UM)) != cudaSuccess) return e;
  if ((e = tc_make_map(&a.map_w[1], a.Wgu, a.N[1], a.K[1], UM)) != cudaSuccess) return e;
  if ((e = tc_make_map(&a.map_w[2], a.Wdown, a.N[2], a.K[2], UM)) != cudaSuccess) return e;
  if ((e = tc_make_map(&a.map_x[0], a.attn16, a.B, a.K[0], CBN)) != cudaSuccess) return e;
  if ((e = tc_make_map(&a.map_x[1], a.h16, a.B, a.K[1], CBN)) != cudaSuccess) return e;
  if ((e = tc_make_map(&a.map_x[2], a.act16, a.B, a.K[2], CBN)) != cudaSuccess) return e;
  const int tasks = (a.m_tiles[0] + a.m_tiles[1] + a.m_tiles[2]) * a.n_tiles;
  const int gu_tasks = a.m_tiles[1] * a.n_tiles;
  int grid = gu_tasks < max_ctas ? gu_tasks : max_ctas;
  if (grid > tasks) grid = tasks;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kChainThreads);
  cfg.dynamicSmemBytes = kChainStages * ST_BYTES + 1024;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, mlp_chain_kernel, a);
}

}  // namespace mmc
