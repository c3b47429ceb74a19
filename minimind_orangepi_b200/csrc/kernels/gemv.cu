// Small-batch projections (B <= 4) on CUDA cores, weights streamed once.
//
// Replaces the reference's per-projection Cube matvec (aclnnMm,
// ascend_matmul.cpp:385-410) and the separate RMSNorm / add / SwiGLU / ArgMax
// ops around it (ascend_custom_ops.cpp:535-604, ascend_matmul.cpp:467-497) with
// one kernel per projection:
//   * each CTA owns a contiguous slab of weight rows (rows are contiguous in
//     the [N][K] layout) and pulls it into shared memory with ONE bulk async
//     copy issued before griddepcontrol.wait, so the HBM read overlaps the
//     previous kernel;
//   * the input rows are rebuilt in the prologue (RMSNorm / embedding gather
//     fused), the dot products run in fp32 from shared memory, and the
//     epilogue fuses the residual add, SiLU*mul or the argmax.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace mmc {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct ArgBest {
  float v;
  int i;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  // first maximum wins (std::max_element); NaN never wins
  return (v > bv) || (v == bv && i < bi);
}

__device__ __forceinline__ void finalize_token(const TokenSink& s, int B, int b, int next) {
  s.tokens[b] = next;
  if (s.next_out) s.next_out[b] = next;
  if (s.seq_pos) s.seq_pos[s.slots[b]] += 1;
  if (s.hist) {
    const int step = *s.hist_step;
    s.hist[(step % s.hist_cap) * s.hist_stride + b] = next;  // a ring
  }
}

__device__ __forceinline__ size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int NB, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(ProjArgs a, int rows_per_cta) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[kWarps][2][NB];
  __shared__ float rs[NB];
  __shared__ ArgBest best_s[kWarps][NB];
  __shared__ int abort_flag;
  __shared__ bool is_last;

  const int K = a.K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.x * rows_per_cta;
  const int rows = min(rows_per_cta, a.N - row0);
  __half* w_s = reinterpret_cast<__half*>(smem);
  float* x_s = reinterpret_cast<float*>(smem + align_up(size_t(rows_per_cta) * K * 2, 128));

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    // Weights do not depend on the previous kernel: fetch before the wait.
    const uint32_t bytes = uint32_t(rows) * uint32_t(K) * 2u;
    mbar_arrive_expect_tx(&bar, bytes);
    const __half* src = a.W + size_t(row0) * K;
    // a single bulk copy moves at most 2^20-16 bytes per instruction on some
    // parts; split defensively into 64 KB pieces.
    uint32_t off = 0;
    while (off < bytes) {
      const uint32_t n = min(bytes - off, 65536u);
      bulk_g2s(reinterpret_cast<uint8_t*>(w_s) + off, reinterpret_cast<const uint8_t*>(src) + off, n, &bar);
      off += n;
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  // ---------------------------------------------------------------- prologue
  // All rows' loads are issued before any is used (one L2 round trip for the
  // whole batch instead of one per row).
  const int B = a.B;
  const float* srcs[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    srcs[b] = a.in + size_t(b) * K;
    if (PRO == kProEmbedNorm && b < B) {
      int tok = a.tokens[b];
      if (tok < 0 || tok >= a.vocab) {
        set_error(a.err, kDevBadToken);
        tok = 0;
      }
      srcs[b] = a.embed + size_t(tok) * K;
    }
  }
  float ssb[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) ssb[b] = 0.f;
  for (int k = tid * 4; k < K; k += kThreads * 4) {
    float4 v[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b)
      v[b] = b < B ? *reinterpret_cast<const float4*>(srcs[b] + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      *reinterpret_cast<float4*>(x_s + b * K + k) = v[b];
      if (PRO == kProEmbedNorm && blockIdx.x == 0 && b < B)
        *reinterpret_cast<float4*>(a.hidden + size_t(b) * K + k) = v[b];
      ssb[b] += v[b].x * v[b].x + v[b].y * v[b].y + v[b].z * v[b].z + v[b].w * v[b].w;
    }
  }
  if (PRO != kProPlain) {
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float ss = warp_sum(ssb[b]);
      if (lane == 0) red[warp][0][b] = ss;
    }
  }
  if (PRO != kProPlain) {
    __syncthreads();
    if (tid < NB) {
      float s = 0.f;
      for (int w = 0; w < kWarps; ++w) s += red[w][0][tid];
      rs[tid] = 1.0f / sqrtf(s / float(K) + a.eps);
    }
    __syncthreads();
    for (int b = 0; b < B; ++b) {
      float* xb = x_s + b * K;
      const float r = rs[b];
      // the norm weight is folded into W's columns at load time
      for (int k = tid; k < K; k += kThreads) xb[k] *= r;
    }
  }
  __syncthreads();

  // wait for the weight slab (bounded)
  if (!mbar_wait_bounded(&bar, 0, a.err)) abort_flag = 1;
  __syncthreads();
  if (abort_flag) return;

  // ---------------------------------------------------------------- compute
  const int npairs = (rows + 1) / 2;
  int ksl = 1;
  if (npairs < kWarps) {
    ksl = kWarps / npairs;
    ksl = ksl >= 8 ? 8 : (ksl >= 4 ? 4 : (ksl >= 2 ? 2 : 1));
  }
  const int nvec = K / 8;
  ArgBest best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = {-INFINITY, 0x7fffffff};

  auto pair_rows = [&](int p, int& r0, int& r1) {
    if (EPI == kEpiSwiglu) {
      r0 = (p >> 3) * 16 + (p & 7);
      r1 = r0 + 8;
    } else {
      r0 = 2 * p;
      r1 = 2 * p + 1;
    }
  };

  auto dot_pair = [&](int r0, int r1, int s, int nsl, float* acc0, float* acc1) {
#pragma unroll
    for (int b = 0; b < NB; ++b) acc0[b] = acc1[b] = 0.f;
    const bool has1 = r1 < rows;
    const __half* w0 = w_s + size_t(r0) * K;
    const __half* w1 = w_s + size_t(has1 ? r1 : r0) * K;
    for (int v = lane + 32 * s; v < nvec; v += 32 * nsl) {
      const uint4 u0 = *reinterpret_cast<const uint4*>(w0 + v * 8);
      const uint4 u1 = *reinterpret_cast<const uint4*>(w1 + v * 8);
      const __half2* h0 = reinterpret_cast<const __half2*>(&u0);
      const __half2* h1 = reinterpret_cast<const __half2*>(&u1);
      float f0[8], f1[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 p0 = __half22float2(h0[j]);
        const float2 p1 = __half22float2(h1[j]);
        f0[2 * j] = p0.x;
        f0[2 * j + 1] = p0.y;
        f1[2 * j] = p1.x;
        f1[2 * j + 1] = p1.y;
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const float4 xa = *reinterpret_cast<const float4*>(x_s + b * K + v * 8);
        const float4 xb = *reinterpret_cast<const float4*>(x_s + b * K + v * 8 + 4);
        const float xs[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc0[b] = fmaf(f0[j], xs[j], acc0[b]);
          acc1[b] = fmaf(f1[j], xs[j], acc1[b]);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      acc0[b] = warp_sum(acc0[b]);
      acc1[b] = warp_sum(acc1[b]);
    }
  };

  auto epilogue = [&](int r0, int r1, const float* acc0, const float* acc1) {
    const bool has1 = r1 < rows;
    const int g0 = row0 + r0, g1 = row0 + r1;
    if (EPI == kEpiResid) {
      // residual add: every row's loads first (one round trip), then the stores
      bool upd[NB];
      float o0[NB], o1[NB];
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        upd[b] = b < B && (a.row_sel == nullptr || a.row_sel[b] == a.row_sel_val);  // MoE: rows routed here
        o0[b] = upd[b] ? a.out[size_t(b) * a.ldo + g0] : 0.f;
        o1[b] = upd[b] && has1 ? a.out[size_t(b) * a.ldo + g1] : 0.f;
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (!upd[b]) continue;
        a.out[size_t(b) * a.ldo + g0] = o0[b] + acc0[b];
        if (has1) a.out[size_t(b) * a.ldo + g1] = o1[b] + acc1[b];
      }
      return;
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (b >= B) break;
      if (EPI == kEpiStore) {
        a.out[size_t(b) * a.ldo + g0] = acc0[b];
        if (has1) a.out[size_t(b) * a.ldo + g1] = acc1[b];
      } else if (EPI == kEpiResid) {
        // the read-modify-writes of all rows are done in one pass above
      } else if (EPI == kEpiSwiglu) {
        const float g = acc0[b];
        const int i = (g0 >> 4) * 8 + (g0 & 7);
        a.out[size_t(b) * a.ldo + i] = (g / (1.0f + expf(-g))) * acc1[b];
      } else {  // argmax
        if (a.logits) {
          a.logits[size_t(b) * a.N + g0] = acc0[b];
          if (has1) a.logits[size_t(b) * a.N + g1] = acc1[b];
        }
        if (better(acc0[b], g0, best[b].v, best[b].i)) best[b] = {acc0[b], g0};
        if (has1 && better(acc1[b], g1, best[b].v, best[b].i)) best[b] = {acc1[b], g1};
      }
    }
  };

  float acc0[NB], acc1[NB];
  if (ksl == 1) {
    for (int p = warp; p < npairs; p += kWarps) {
      int r0, r1;
      pair_rows(p, r0, r1);
      dot_pair(r0, r1, 0, 1, acc0, acc1);
      if (lane == 0) epilogue(r0, r1, acc0, acc1);
    }
  } else {
    const int p = warp / ksl, s = warp % ksl;
    int r0 = 0, r1 = 0;
    if (p < npairs) {
      pair_rows(p, r0, r1);
      dot_pair(r0, r1, s, ksl, acc0, acc1);
      if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          red[warp][0][b] = acc0[b];
          red[warp][1][b] = acc1[b];
        }
      }
    }
    __syncthreads();
    if (p < npairs && s == 0 && lane == 0) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float t0 = 0.f, t1 = 0.f;
        for (int j = 0; j < ksl; ++j) {
          t0 += red[warp + j][0][b];
          t1 += red[warp + j][1][b];
        }
        acc0[b] = t0;
        acc1[b] = t1;
      }
      epilogue(r0, r1, acc0, acc1);
    }
  }

  if (EPI != kEpiArgmax) return;

  // ------------------------------------------------ argmax: CTA, then grid
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < NB; ++b) best_s[warp][b] = best[b];
  }
  __syncthreads();
  ArgBest* part = reinterpret_cast<ArgBest*>(a.argmax_part);
  if (tid < B) {
    ArgBest bb = {-INFINITY, 0x7fffffff};
    for (int w = 0; w < kWarps; ++w)
      if (better(best_s[w][tid].v, best_s[w][tid].i, bb.v, bb.i)) bb = best_s[w][tid];
    part[size_t(tid) * gridDim.x + blockIdx.x] = bb;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int b = warp; b < B; b += kWarps) {
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
      int next = bb.i;
      if (next < 0 || next >= a.N) next = 0;  // all-NaN row
      finalize_token(a.sink, B, b, next);
    }
  }
  __syncthreads();
  if (tid == 0) {
    if (a.sink.hist_step) *a.sink.hist_step += 1;
    *a.counter = 0u;
  }
}

template <int NB, int PRO, int EPI>
cudaError_t set_attr() {
  return set_kernel_smem(gemv_kernel<NB, PRO, EPI>, 200 * 1024);
}

template <int NB>
cudaError_t set_attrs_nb() {
  cudaError_t e = cudaSuccess;
  cudaError_t r;
#define MMC_ATTR(P, E) \
  if ((r = set_attr<NB, P, E>()) != cudaSuccess) e = r;
  MMC_ATTR(kProPlain, kEpiStore)
  MMC_ATTR(kProNorm, kEpiStore)
  MMC_ATTR(kProEmbedNorm, kEpiStore)
  MMC_ATTR(kProPlain, kEpiResid)
  MMC_ATTR(kProNorm, kEpiSwiglu)
  MMC_ATTR(kProNormFinal, kEpiArgmax)
  MMC_ATTR(kProPlain, kEpiArgmax)
#undef MMC_ATTR
  return e;
}

template <int NB, int PRO, int EPI>
cudaError_t launch_t(const ProjArgs& a, int rpc, int grid, size_t smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<NB, PRO, EPI>, a, rpc);
}

template <int NB>
cudaError_t dispatch_nb(int pro, int epi, const ProjArgs& a, int rpc, int grid, size_t smem, cudaStream_t s,
                        bool pdl) {
#define MMC_CASE(P, E) \
  if (pro == P && epi == E) return launch_t<NB, P, E>(a, rpc, grid, smem, s, pdl);
  MMC_CASE(kProPlain, kEpiStore)
  MMC_CASE(kProNorm, kEpiStore)
  MMC_CASE(kProEmbedNorm, kEpiStore)
  MMC_CASE(kProPlain, kEpiResid)
  MMC_CASE(kProNorm, kEpiSwiglu)
  MMC_CASE(kProNormFinal, kEpiArgmax)
  MMC_CASE(kProPlain, kEpiArgmax)
#undef MMC_CASE
  return cudaErrorInvalidValue;
}

}  // namespace

int gemv_rows_per_cta(int N, int K, int epi, int num_sms) {
  const int gran = epi == kEpiSwiglu ? 16 : 2;
  int rpc = (N + num_sms - 1) / num_sms;
  rpc = (rpc + gran - 1) / gran * gran;
  // keep the slab <= 96 KB so two kernels' CTAs can share an SM under PDL
  while (rpc > gran && size_t(rpc) * K * 2 > 96 * 1024) rpc -= gran;
  return std::max(rpc, gran);
}

size_t gemv_smem_bytes(int rpc, int K, int B) {
  const int nb = B <= 1 ? 1 : (B <= 2 ? 2 : 4);
  return (size_t(rpc) * K * 2 + 127) / 128 * 128 + size_t(nb) * K * 4;
}

size_t gemv_argmax_part_bytes(int N, int K, int B, int num_sms) {
  const int rpc = gemv_rows_per_cta(N, K, kEpiArgmax, num_sms);
  const int grid = (N + rpc - 1) / rpc;
  return size_t(B) * grid * sizeof(ArgBest);
}

cudaError_t gemv_init_attributes() {
  cudaError_t e1 = set_attrs_nb<1>(), e2 = set_attrs_nb<2>(), e4 = set_attrs_nb<4>();
  return e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e4);
}

cudaError_t launch_gemv(int pro, int epi, const ProjArgs& a, int num_sms, cudaStream_t s, bool pdl) {
  if (a.B < 1 || a.B > 4 || a.K % 8 != 0 || a.N <= 0) return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu && a.N % 16 != 0) return cudaErrorInvalidValue;
  const int rpc = gemv_rows_per_cta(a.N, a.K, epi, num_sms);
  const int grid = (a.N + rpc - 1) / rpc;
  const size_t smem = gemv_smem_bytes(rpc, a.K, a.B);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (a.B == 1) return dispatch_nb<1>(pro, epi, a, rpc, grid, smem, s, pdl);
  if (a.B == 2) return dispatch_nb<2>(pro, epi, a, rpc, grid, smem, s, pdl);
  return dispatch_nb<4>(pro, epi, a, rpc, grid, smem, s, pdl);
}

}  // namespace mmc
