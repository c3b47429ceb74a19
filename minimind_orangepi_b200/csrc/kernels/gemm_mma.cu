// Batched projections (B > 4) on tensor cores: Y^T[n][b] = W[n][:] . X[b][:]^T.
//
// Same contract as the small-batch projection (gemv.cu) — fused RMSNorm /
// embedding prologue and store / residual / SiLU*mul / argmax epilogues — but
// the dot products run as mma.sync m16n8k16 (fp16 x fp16 -> fp32) with the
// weight rows on M and the batch on N, so each weight byte fetched serves the
// whole batch tile. Weight tiles arrive by cp.async into an XOR-swizzled
// 3-stage ring (issued before griddepcontrol.wait); activation tiles are read
// as fp32, normalised and rounded to fp16 on the way into shared memory.
//
// CTA tile 64 weight rows x BN batch rows x 64-deep k steps, 4 warps, each
// warp 16 rows x BN.
#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

constexpr int kThreads = 128;
constexpr int BM = 64;
constexpr int BK = 64;
constexpr int NSTAGE = 3;

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return (v > bv) || (v == bv && i < bi); }

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}

// byte offset of (row, 16B chunk) inside a [rows][64 halves] swizzled tile
__device__ __forceinline__ int tile_off(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

template <int BN, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads) gemm_kernel(ProjArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int W_BYTES = BM * BK * 2, X_BYTES = BN * BK * 2, ST_BYTES = W_BYTES + X_BYTES;
  constexpr int NT = BN / 8;               // n-tiles per warp
  constexpr int XV = BN * BK / 4 / kThreads;  // float4 loads per thread per k-tile
  __shared__ float rs[BN];
  __shared__ const float* src_row[BN];
  __shared__ ArgBest best_s[4][BN];
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int K = a.K, KT = K / BK;

  auto issue_w = [&](int kt) {
    uint8_t* ws = smem + (kt % NSTAGE) * ST_BYTES;
#pragma unroll
    for (int i = 0; i < (BM * BK / 8) / kThreads; ++i) {
      const int idx = tid + i * kThreads;
      const int r = idx >> 3, c = idx & 7;
      const bool ok = m0 + r < a.N;
      const __half* src = a.W + size_t(ok ? m0 + r : 0) * K + kt * BK + c * 8;
      cp_async16_zfill(ws + tile_off(r, c), src, ok);
    }
  };
  // weight tiles do not depend on the previous kernel
#pragma unroll
  for (int s = 0; s < NSTAGE - 1; ++s) {
    if (s < KT) issue_w(s);
    cp_async_commit();
  }
  pdl_wait();
  pdl_launch_dependents();

  // ------------------------------------------------ prologue: row sources, norms
  if (tid < BN) {
    const int b = n0 + tid;
    const float* p = nullptr;
    if (b < a.B) {
      if (PRO == kProEmbedNorm) {
        int tok = a.tokens[b];
        if (tok < 0 || tok >= a.vocab) {
          set_error(a.err, kDevBadToken);
          tok = 0;
        }
        p = a.embed + size_t(tok) * K;
      } else {
        p = a.in + size_t(b) * K;
      }
    }
    src_row[tid] = p;
  }
  __syncthreads();
  if (PRO != kProPlain) {
    for (int r = warp; r < BN; r += 4) {
      const float* p = src_row[r];
      float ss = 0.f;
      if (p) {
        for (int k = lane * 4; k < K; k += 128) {
          const float4 v = *reinterpret_cast<const float4*>(p + k);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) rs[r] = p ? 1.0f / sqrtf(ss / float(K) + a.eps) : 0.f;
    }
    __syncthreads();
  }

  float4 xr[XV];
  auto load_x = [&](int kt) {
#pragma unroll
    for (int i = 0; i < XV; ++i) {
      const int idx = tid + i * kThreads;
      const int r = idx / (BK / 4), c4 = idx % (BK / 4);
      const float* p = src_row[r];
      xr[i] = p ? *reinterpret_cast<const float4*>(p + kt * BK + c4 * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_x = [&](int kt) {
    uint8_t* xs = smem + (kt % NSTAGE) * ST_BYTES + W_BYTES;
#pragma unroll
    for (int i = 0; i < XV; ++i) {
      const int idx = tid + i * kThreads;
      const int r = idx / (BK / 4), c4 = idx % (BK / 4);
      const int k = kt * BK + c4 * 4;
      float4 v = xr[i];
      if (PRO == kProEmbedNorm && blockIdx.x == 0 && src_row[r])
        *reinterpret_cast<float4*>(a.hidden + size_t(n0 + r) * K + k) = v;
      if (PRO != kProPlain) {
        const float s = rs[r];
        const float4 w = *reinterpret_cast<const float4*>(a.norm_w + k);
        if (PRO == kProNormFinal) {
          v = make_float4((v.x * s) * w.x, (v.y * s) * w.y, (v.z * s) * w.z, (v.w * s) * w.w);
        } else {
          v = make_float4(v.x * (s * w.x), v.y * (s * w.y), v.z * (s * w.z), v.w * (s * w.w));
        }
      }
      uint2 hv;
      hv.x = pack_half2(v.x, v.y);
      hv.y = pack_half2(v.z, v.w);
      *reinterpret_cast<uint2*>(xs + tile_off(r, c4 >> 1) + (c4 & 1) * 8) = hv;
    }
  };

#pragma unroll
  for (int s = 0; s < NSTAGE - 1; ++s) {
    if (s < KT) {
      load_x(s);
      store_x(s);
    }
  }

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  for (int kt = 0; kt < KT; ++kt) {
    cp_async_wait<NSTAGE - 2>();
    __syncthreads();
    const int pf = kt + NSTAGE - 1;
    if (pf < KT) {
      issue_w(pf);
      load_x(pf);
    }
    cp_async_commit();

    const uint8_t* ws = smem + (kt % NSTAGE) * ST_BYTES;
    const uint8_t* xs = ws + W_BYTES;
#pragma unroll
    for (int ks = 0; ks < BK / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int c = 2 * ks + (lane >> 4);
        ldsm_x4(smem_u32(ws + tile_off(r, c)), a0, a1, a2, a3);
      }
#pragma unroll
      for (int jp = 0; jp < NT / 2; ++jp) {
        const int r = 16 * jp + ((lane >> 4) & 1) * 8 + (lane & 7);
        const int c = 2 * ks + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(xs + tile_off(r, c)), b0, b1, b2, b3);
        mma16816(acc[2 * jp], a0, a1, a2, a3, b0, b1);
        mma16816(acc[2 * jp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    if (pf < KT) store_x(pf);
  }
  cp_async_wait<0>();

  // ------------------------------------------------------------ epilogue
  const int rA = m0 + warp * 16 + g, rB = rA + 8;
  ArgBest bst[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = n0 + 8 * j + 2 * t + e;
      const float vA = acc[j][e], vB = acc[j][2 + e];
      bst[j][e] = {-INFINITY, 0x7fffffff};
      if (col >= a.B) continue;
      if (EPI == kEpiStore) {
        if (rA < a.N) a.out[size_t(col) * a.ldo + rA] = vA;
        if (rB < a.N) a.out[size_t(col) * a.ldo + rB] = vB;
      } else if (EPI == kEpiResid) {
        if (rA < a.N) a.out[size_t(col) * a.ldo + rA] += vA;
        if (rB < a.N) a.out[size_t(col) * a.ldo + rB] += vB;
      } else if (EPI == kEpiSwiglu) {
        if (rA < a.N) {
          const int i = (rA >> 4) * 8 + (rA & 7);
          a.out[size_t(col) * a.ldo + i] = (vA / (1.0f + expf(-vA))) * vB;
        }
      } else {
        if (a.logits) {
          if (rA < a.N) a.logits[size_t(col) * a.N + rA] = vA;
          if (rB < a.N) a.logits[size_t(col) * a.N + rB] = vB;
        }
        ArgBest bb = {-INFINITY, 0x7fffffff};
        if (rA < a.N && better(vA, rA, bb.v, bb.i)) bb = {vA, rA};
        if (rB < a.N && better(vB, rB, bb.v, bb.i)) bb = {vB, rB};
        bst[j][e] = bb;
      }
    }
  }
  if (EPI != kEpiArgmax) return;

#pragma unroll
  for (int j = 0; j < NT; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      ArgBest bb = bst[j][e];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bb.v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bb.i, o);
        if (better(ov, oi, bb.v, bb.i)) bb = {ov, oi};
      }
      if (g == 0) best_s[warp][8 * j + 2 * t + e] = bb;
    }
  }
  __syncthreads();
  ArgBest* part = reinterpret_cast<ArgBest*>(a.argmax_part);
  if (tid < BN && n0 + tid < a.B) {
    ArgBest bb = {-INFINITY, 0x7fffffff};
    for (int w = 0; w < 4; ++w)
      if (better(best_s[w][tid].v, best_s[w][tid].i, bb.v, bb.i)) bb = best_s[w][tid];
    part[size_t(n0 + tid) * gridDim.x + blockIdx.x] = bb;
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
        if (step < s.hist_cap) s.hist[step * a.B + b] = next;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    a.counter[blockIdx.y] = 0u;
    // the history row counter advances once per step: the batch tile that
    // finishes last among all tiles bumps it (second-level counter).
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

template <int BN>
constexpr size_t smem_bytes() {
  return size_t(NSTAGE) * (BM * BK * 2 + BN * BK * 2);
}

template <int BN, int PRO, int EPI>
cudaError_t launch_t(const ProjArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + BM - 1) / BM, (a.B + BN - 1) / BN);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes<BN>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, gemm_kernel<BN, PRO, EPI>, a);
}

template <int BN>
cudaError_t dispatch(int pro, int epi, const ProjArgs& a, cudaStream_t s, bool pdl) {
#define MMC_CASE(P, E) \
  if (pro == P && epi == E) return launch_t<BN, P, E>(a, s, pdl);
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

template <int BN>
cudaError_t attrs_bn() {
  cudaError_t e = cudaSuccess, r;
#define MMC_ATTR(P, E)                                                                                  \
  if ((r = cudaFuncSetAttribute(gemm_kernel<BN, P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                int(smem_bytes<BN>()))) != cudaSuccess)                               \
    e = r;
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

}  // namespace

size_t gemm_argmax_part_bytes(int N, int B) { return size_t(B) * ((N + BM - 1) / BM) * sizeof(ArgBest); }

cudaError_t gemm_init_attributes() {
  cudaError_t e1 = attrs_bn<16>(), e2 = attrs_bn<32>(), e3 = attrs_bn<64>();
  return e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3);
}

// The argmax epilogue needs a.counter to hold gridDim.y + 1 zeroed words.
cudaError_t launch_gemm(int pro, int epi, const ProjArgs& a, cudaStream_t s, bool pdl) {
  if (a.B < 1 || a.K % BK != 0 || a.N <= 0) return cudaErrorInvalidValue;
  if (epi == kEpiSwiglu && a.N % 16 != 0) return cudaErrorInvalidValue;
  if (a.B <= 16) return dispatch<16>(pro, epi, a, s, pdl);
  if (a.B <= 32) return dispatch<32>(pro, epi, a, s, pdl);
  return dispatch<64>(pro, epi, a, s, pdl);
}

}  // namespace mmc
