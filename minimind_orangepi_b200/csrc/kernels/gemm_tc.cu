// Batched projections (B > 4) on the 5th-generation tensor cores (tcgen05).
//
// Y^T[n][b] = W[n][:] . X[b][:]: the weight rows are the UMMA M side (128 per
// CTA), the batch rows the N side (BN per CTA), K runs in 64-element steps.
// Operands are fp16 in HBM/L2 (W packed at load time, X written fp16 by the
// producer kernel). Warp-specialised pipeline, no block-wide barrier in the K
// loop:
//   warp 0 / lane 0  TMA producer: 2-D tensor-map loads (128-byte swizzle, the
//                    canonical UMMA K-major SW128 layout) into a ring of
//                    stages; full[s] completes on the transaction bytes; the
//                    first stages' weight tiles are issued before
//                    griddepcontrol.wait;
//   warp 1 / lane 0  MMA issuer: waits full[s], issues tcgen05.mma (fp32
//                    accumulate in TMEM), commits empty[s] to free the stage
//                    and finally `done`;
//   all 4 warps      epilogue: tcgen05.ld of the accumulator (warp w owns TMEM
//                    lanes 32w..32w+31 = weight rows) fused with the store /
//                    residual add / SiLU*mul / argmax of the decode step.
//
// RMSNorm is carried across kernels instead of run as its own pass: the norm
// weight is folded into the consuming projection's W at load time, a residual
// epilogue writes the fp16 residual rows plus one sum of squares per (row,
// M-tile), and the consumer scales its outputs by 1/rms (computed by the
// otherwise idle warps 2-3 during the K loop).
//
// Split-K (projections with fewer tiles than SMs): the k-splits of one tile
// run as a thread-block cluster; each parks its accumulator in its stage ring
// and the ranks reduce disjoint column slices over distributed shared memory
// in rank order, so results do not depend on scheduling.
//
// Every wait is bounded (2 s): on timeout the kernel records an error, frees
// its TMEM and returns.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace mmc {
namespace {

constexpr int kThreads = 128;
// Stage ring depth per batch tile: at most ~96-144 KB of tiles, so that a CTA
// of this kernel can share an SM with an attention CTA (about 110 KB) when the
// parts of a split batch run concurrently. (Measured on B200: a fifth stage
// for small batch tiles, or an L2 prefetch of the later weight tiles, made
// the decode step slower.)
#ifndef MMC_TC_SMALL_STAGES
#define MMC_TC_SMALL_STAGES 3  // ring stages for batch tiles <= 32 (build-time tuning knob)
#endif
template <int BN>
constexpr int stages_for() {
  return BN >= 256 ? 3 : BN <= 32 ? MMC_TC_SMALL_STAGES : 4;
}

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return (v > bv) || (v == bv && i < bi); }


template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads) gemm_tc_kernel(const __grid_constant__ TcArgs a) {
  constexpr int NSTAGE = stages_for<BN>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-align the stage ring (SWIZZLE_128B atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = UM * BK * 2, B_BYTES = BN * BK * 2, ST_BYTES = A_BYTES + B_BYTES;
  __shared__ __align__(8) uint64_t full_bar[8];
  __shared__ __align__(8) uint64_t empty_bar[8];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ ArgBest best_s[EPI == kEpiArgmax ? 4 : 1][BN];
  __shared__ float rs_s[BN];
  __shared__ float ssw_s[EPI == kEpiResid ? 4 : 1][BN];
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * UM, n0 = blockIdx.y * BN;
  // split-K: blockIdx.z takes k-steps [kbase, kbase + KT) of the K / 64 total
  const int KT_all = a.K / BK, S = gridDim.z, kz = blockIdx.z;
  const int kbase = int((long long)kz * KT_all / S);
  const int KT = int((long long)(kz + 1) * KT_all / S) - kbase;
  const int pre = KT < NSTAGE ? KT : NSTAGE;

  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    fence_mbar_init();
    // weight tiles do not depend on the previous kernel: start them now
    for (int s = 0; s < pre; ++s) {
      mbar_arrive_expect_tx(&full_bar[s], uint32_t(ST_BYTES));
      tma_load_2d(smem + s * ST_BYTES, &a.map_w, (kbase + s) * BK, m0, &full_bar[s]);
    }
  }
  __syncthreads();
  pdl_wait();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(uint32_t(BN < 32 ? 32 : BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      for (int s = 0; s < pre; ++s)
        tma_load_2d(smem + s * ST_BYTES + A_BYTES, &a.map_x, (kbase + s) * BK, n0, &full_bar[s]);
      for (int kt = pre; kt < KT; ++kt) {
        const int s = kt % NSTAGE;
        if (!mbar_wait_bounded(&empty_bar[s], ((kt / NSTAGE) - 1) & 1, a.err)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], uint32_t(ST_BYTES));
        tma_load_2d(smem + s * ST_BYTES, &a.map_w, (kbase + kt) * BK, m0, &full_bar[s]);
        tma_load_2d(smem + s * ST_BYTES + A_BYTES, &a.map_x, (kbase + kt) * BK, n0, &full_bar[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = idesc_f16<BN>();
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % NSTAGE;
        if (!mbar_wait_bounded(&full_bar[s], (kt / NSTAGE) & 1, a.err)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t as = smem_u32(smem + s * ST_BYTES);
        const uint32_t bs = as + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16(tmem, sw128_desc(as + k * 32), sw128_desc(bs + k * 32), idesc, (kt | k) != 0);
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&done_bar);  // arrives once every MMA above has completed
    }
    __syncwarp();
  } else {
    // warps 2-3, idle during the K loop: the folded RMSNorm's per-column
    // 1/rms of the input (sums of squares from the producer of X) and the
    // zeroed per-warp sums of squares of a residual epilogue
    const int t = tid - 64;
    if (a.ss_in != nullptr) {
      const int parts = (a.K + UM - 1) / UM;
      for (int c = t; c < BN; c += 64) {
        float r = 1.f;
        if (n0 + c < a.B) {
          float ss = 0.f;
          for (int m = 0; m < parts; ++m) ss += a.ss_in[size_t(n0 + c) * parts + m];
          r = 1.0f / sqrtf(ss / float(a.K) + a.eps);
        }
        rs_s[c] = r;
      }
    }
    if (EPI == kEpiResid)
      for (int c = t; c < 4 * BN; c += 64) (&ssw_s[0][0])[c] = 0.f;
  }
  if (!mbar_wait_bounded(&done_bar, 0, a.err)) abort_flag = 1;
  tc_fence_after();
  __syncthreads();

  const int row = m0 + warp * 32 + lane;  // this thread's weight row
  const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);

  const bool want_ss = EPI == kEpiResid && a.ss_out != nullptr;

  // Epilogue of NC batch columns c0 .. c0 + NC (values v of this thread's
  // row); all lanes of the warp take part. Global loads are issued for all
  // columns before any cross-lane reduction.
  auto epi_cols = [&](int c0, int nc, float* v) {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (a.ss_in != nullptr && j < nc) v[j] *= rs_s[c0 + j];
    if (EPI == kEpiStore) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = n0 + c0 + j;
        if (j < nc && row < a.N && b < a.B) a.out[size_t(b) * a.ldo + row] = v[j];
      }
    } else if (EPI == kEpiResid) {
      // row_sel (MoE): only rows routed to expert row_sel_val are updated
      bool upd[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = n0 + c0 + j;
        upd[j] = j < nc && row < a.N && b < a.B && (a.row_sel == nullptr || a.row_sel[b] == a.row_sel_val);
      }
      float nv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = n0 + c0 + j;
        nv[j] = upd[j] ? a.out[size_t(b) * a.ldo + row] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = n0 + c0 + j;
        if (upd[j]) {
          nv[j] += v[j];
          a.out[size_t(b) * a.ldo + row] = nv[j];
          if (a.h16_out) a.h16_out[size_t(b) * a.N + row] = __float2half_rn(nv[j]);
        }
      }
      if (want_ss) {
        float sq[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) sq[j] = j < nc ? nv[j] * nv[j] : 0.f;
        const float tot = colsum16(sq, lane);
        const int cj = colsum16_col(lane);
        if ((lane & 1) == 0 && cj < nc) ssw_s[warp][c0 + cj] = tot;
      }
    } else if (EPI == kEpiSwiglu) {
      // gate rows 16j..16j+7 and up rows 16j+8..16j+15 sit 8 lanes apart
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j >= nc) continue;
        const float up = __shfl_down_sync(0xffffffffu, v[j], 8);
        const int b = n0 + c0 + j;
        if ((lane & 8) == 0 && row < a.N && b < a.B) {
          const float g = v[j];
          const int i = (row >> 4) * 8 + (row & 7);
          a.out16[size_t(b) * a.ldo + i] = __float2half_rn((g / (1.0f + expf(-g))) * up);
        }
      }
    } else {  // argmax over this CTA's rows, per batch column
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j >= nc) continue;
        const int b = n0 + c0 + j;
        if (a.logits && row < a.N && b < a.B) a.logits[size_t(b) * a.N + row] = v[j];
        float bv = row < a.N ? v[j] : -INFINITY;
        int bi = row < a.N ? row : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) best_s[warp][c0 + j] = {bv, bi};
      }
    }
  };

  int c_lo = 0, c_hi = BN;  // batch columns this CTA finishes
  if (S == 1) {
    if (!abort_flag) {
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 16) {
        float v[16];
        tmem_ld16(trow + cc, v);
        epi_cols(cc, 16, v);
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc<BN>(tmem);
  } else {
    // split-K cluster: every CTA parks its fp32 accumulator in its (now idle)
    // stage ring as [column][row]; CTA rank r then sums column slice r over
    // all ranks in rank order through distributed shared memory.
    float* red = reinterpret_cast<float*>(smem);
    if (!abort_flag) {
#pragma unroll 1
      for (int cc = 0; cc < BN; cc += 16) {
        float v[16];
        tmem_ld16(trow + cc, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) red[(cc + j) * UM + warp * 32 + lane] = v[j];
      }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc<BN>(tmem);
    cluster_sync();
    const int rank = int(cluster_ctarank());
    c_lo = rank * BN / S;
    c_hi = (rank + 1) * BN / S;
    if (!abort_flag) {
      const uint32_t local = smem_u32(red) + uint32_t(warp * 32 + lane) * 4u;
      for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
        const int nc = c_hi - c0 < 16 ? c_hi - c0 : 16;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.f;
        for (int q = 0; q < S; ++q) {
          const uint32_t peer = map_dsmem(local + uint32_t(c0 * UM) * 4u, uint32_t(q));
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < nc) v[j] += ld_dsmem_f32(peer + uint32_t(j * UM) * 4u);
        }
        epi_cols(c0, nc, v);
      }
    }
    cluster_sync();  // peers' rings stay alive until every rank has read them
  }
  if (abort_flag) return;
  if (want_ss) {
    __syncthreads();
    for (int c = c_lo + tid; c < c_hi; c += kThreads)
      if (n0 + c < a.B && (a.row_sel == nullptr || a.row_sel[n0 + c] == a.row_sel_val))
        a.ss_out[size_t(n0 + c) * gridDim.x + blockIdx.x] = ssw_s[0][c] + ssw_s[1][c] + ssw_s[2][c] + ssw_s[3][c];
  }
  if (EPI != kEpiArgmax) return;

  ArgBest* part = reinterpret_cast<ArgBest*>(a.argmax_part);
  // every batch column of the tile (BN may exceed the thread count)
  for (int c = tid; c < BN && n0 + c < a.B; c += kThreads) {
    ArgBest bb = {-INFINITY, 0x7fffffff};
    for (int w = 0; w < 4; ++w)
      if (better(best_s[w][c].v, best_s[w][c].i, bb.v, bb.i)) bb = best_s[w][c];
    part[size_t(n0 + c) * gridDim.x + blockIdx.x] = bb;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&a.counter[blockIdx.y], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int r = warp; r < BN; r += 4) {
    const int b = n0 + r;
    if (b >= a.B) break;
    ArgBest bb = {-INFINITY, 0x7fffffff};
    for (int c = lane; c < int(gridDim.x); c += 32) {
      const float qv = __ldcg(&part[size_t(b) * gridDim.x + c].v);
      const int qi = __ldcg(&part[size_t(b) * gridDim.x + c].i);
      if (better(qv, qi, bb.v, bb.i)) bb = {qv, qi};
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
      if (better(ov, oi, bb.v, bb.i)) bb = {ov, oi};
    }
    if (lane == 0) {
      const int next = (bb.i >= 0 && bb.i < a.N) ? bb.i : 0;
      const TokenSink& s = a.sink;
      s.tokens[b] = next;
      if (s.next_out) s.next_out[b] = next;
      if (s.seq_pos) s.seq_pos[s.slots[b]] += 1;
      if (s.hist) {
        const int step = *s.hist_step;
        s.hist[(step % s.hist_cap) * s.hist_stride + b] = next;  // a ring
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    a.counter[blockIdx.y] = 0u;
    if (a.sink.hist_step) {
      const unsigned done = atomicAdd(&a.counter[gridDim.y], 1u);
      if (done == gridDim.y - 1) {
        a.counter[gridDim.y] = 0u;
        __threadfence();
        *a.sink.hist_step += 1;
      }
    }
  }
}

// Layer-0 rows of the tensor-core path: embedding gather into the residual
// stream and its fp16 copy, plus the row's sum of squares for the folded
// RMSNorm of the first projection (slot 0; the other M-tile slots are 0).
__global__ void __launch_bounds__(256) embed_rows_kernel(EmbedArgs a) {
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  int tok = a.tokens[b];
  if (tok < 0 || tok >= a.vocab) {
    set_error(a.err, kDevBadToken);
    tok = 0;
  }
  const float* src = a.embed + size_t(tok) * a.H;
  float ss = 0.f;
  for (int k = tid * 4; k < a.H; k += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(src + k);
    *reinterpret_cast<float4*>(a.hidden + size_t(b) * a.H + k) = v;
    uint2 h;
    h.x = pack_half2(v.x, v.y);
    h.y = pack_half2(v.z, v.w);
    *reinterpret_cast<uint2*>(a.h16 + size_t(b) * a.H + k) = h;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  const int parts = (a.H + UM - 1) / UM;
  if (tid < parts) {
    float tot = 0.f;
    if (tid == 0)
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += red[w];
    a.ss[size_t(b) * parts + tid] = tot;
  }
}

template <int BN>
constexpr size_t tc_smem() {
  return size_t(stages_for<BN>()) * (UM * BK * 2 + BN * BK * 2) + 1024;
}

template <int BN, int EPI>
cudaError_t launch_bn(const TcArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + UM - 1) / UM, (a.B + BN - 1) / BN, a.splits > 1 ? a.splits : 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = tc_smem<BN>();
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (a.splits > 1) {  // the k-splits of one tile form a cluster
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = unsigned(a.splits);
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI>, a);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D fp16 [rows][K] row-major tensor, boxes of 64 (K) x box_rows, 128-byte
// swizzle (the UMMA SW128 K-major layout); rows past `rows` read as zero.
cudaError_t make_map(CUtensorMap* m, const __half* base, int rows, int K, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  const cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

// Split-K plan for projections whose (M-tile x batch-tile) grid leaves SMs
// idle: a batch tile of up to 32 rows and enough k-splits (each at least two
// 64-wide k-steps, at most 8: one portable cluster) to reach about one CTA
// per SM. Returns the split count (1: no split) and sets *bn.
int split_plan(const TcArgs& a, int epi, int* bn) {
  *bn = tc_batch_tile(a.N, a.B);
  static const int enabled = env_int("MMC_TC_SPLIT", 1);
  static const int target = env_int("MMC_TC_SPLIT_TARGET", 148);
  static const int bn_cap = env_int("MMC_TC_SPLIT_BN", 32);
  if (!enabled || epi == kEpiArgmax || a.max_splits < 2) return 1;
  const int mt = (a.N + UM - 1) / UM, KT = a.K / BK;
  if (mt * ((a.B + *bn - 1) / *bn) >= target || KT < 4) return 1;
  const int cap = a.split_bn > 0 ? a.split_bn : bn_cap;
  int b = 16;
  while (b < cap && b < a.B) b *= 2;
  const int tiles = mt * ((a.B + b - 1) / b);
  const int S = std::min(std::min(KT / 2, std::min(a.max_splits, 8)), (target + tiles - 1) / tiles);
  if (S < 2) return 1;
  *bn = b;
  return S;
}

template <int EPI>
cudaError_t launch_epi(const TcArgs& a_in, cudaStream_t s, bool pdl) {
  TcArgs a = a_in;
  int bn = 16;
  a.splits = split_plan(a_in, EPI, &bn);
  cudaError_t e = make_map(&a.map_w, a.W, a.N, a.K, UM);
  if (e != cudaSuccess) return e;
  e = make_map(&a.map_x, a.X, a.B, a.K, bn);
  if (e != cudaSuccess) return e;
  switch (bn) {
    case 16: return launch_bn<16, EPI>(a, s, pdl);
    case 32: return launch_bn<32, EPI>(a, s, pdl);
    case 64: return launch_bn<64, EPI>(a, s, pdl);
    case 128: return launch_bn<128, EPI>(a, s, pdl);
    default: return launch_bn<256, EPI>(a, s, pdl);
  }
}

template <int BN>
cudaError_t attrs_bn() {
  cudaError_t e = cudaSuccess, r;
  const int bytes = int(tc_smem<BN>());
  if ((r = set_kernel_smem(gemm_tc_kernel<BN, kEpiStore>, bytes)) !=
      cudaSuccess)
    e = r;
  if ((r = set_kernel_smem(gemm_tc_kernel<BN, kEpiResid>, bytes)) !=
      cudaSuccess)
    e = r;
  if ((r = set_kernel_smem(gemm_tc_kernel<BN, kEpiSwiglu>, bytes)) != cudaSuccess)
    e = r;
  if ((r = set_kernel_smem(gemm_tc_kernel<BN, kEpiArgmax>, bytes)) != cudaSuccess)
    e = r;
  return e;
}

}  // namespace

cudaError_t tc_make_map(CUtensorMap* m, const __half* base, int rows, int K, int box_rows) {
  return make_map(m, base, rows, K, box_rows);
}

int tc_split_k(const TcArgs& a, int epi) {
  int bn;
  return split_plan(a, epi, &bn);
}

// Batch tile: the largest of {256,128,64,32} that still gives every SM work,
// else 32 (small problems are latency-bound; more CTAs help).
int tc_batch_tile(int N, int B) {
  const int mt = (N + UM - 1) / UM;
  for (int bn : {256, 128, 64, 32}) {
    if (bn > 2 * B) continue;
    if (mt * ((B + bn - 1) / bn) >= 148) return bn;
  }
  return 16;
}

size_t tc_argmax_part_bytes(int N, int B) { return size_t(B) * ((N + UM - 1) / UM) * sizeof(ArgBest); }
int tc_counter_words(int N, int B) { return (B + 15) / 16 + 2; }

cudaError_t gemm_tc_init_attributes() {
  cudaError_t e1 = attrs_bn<32>(), e2 = attrs_bn<64>(), e3 = attrs_bn<128>(), e4 = attrs_bn<256>();
  cudaError_t e5 = attrs_bn<16>();
  if (e5 == cudaSuccess) e5 = set_kernel_smem(embed_rows_kernel, 0);
  return e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3 != cudaSuccess ? e3 : e4 != cudaSuccess ? e4 : e5;
}

cudaError_t launch_gemm_tc(int epi, const TcArgs& a, cudaStream_t s, bool pdl) {
  if (a.B < 1 || a.K % BK != 0 || a.N <= 0 || a.K <= 0) return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu && a.N % 16 != 0) return cudaErrorInvalidValue;
  switch (epi) {
    case kEpiStore: return launch_epi<kEpiStore>(a, s, pdl);
    case kEpiResid: return launch_epi<kEpiResid>(a, s, pdl);
    case kEpiSwiglu: return launch_epi<kEpiSwiglu>(a, s, pdl);
    case kEpiArgmax: return launch_epi<kEpiArgmax>(a, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_embed_rows(const EmbedArgs& a, cudaStream_t s, bool pdl) {
  if (a.H % 4 != 0 || a.B < 1 || (a.H + UM - 1) / UM > 256) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, embed_rows_kernel, a);
}

}  // namespace mmc
