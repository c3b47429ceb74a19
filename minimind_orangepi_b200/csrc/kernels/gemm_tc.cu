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
// Every wait is bounded (2 s): on timeout the kernel records an error, frees
// its TMEM and returns.
#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

constexpr int kThreads = 128;
constexpr int UM = 128;       // UMMA M (weight rows per CTA)
constexpr int BK = 64;        // K per stage (one 128-byte swizzle atom of fp16)
// Stage ring depth per batch tile: at most ~96-144 KB of tiles, so a CTA of
// this kernel can share an SM with an attention CTA (about 110 KB) when the
// two halves of a split batch run concurrently.
template <int BN>
constexpr int stages_for() {
  return BN >= 256 ? 3 : 4;
}

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return (v > bv) || (v == bv && i < bi); }


// K-major SWIZZLE_128B shared-memory matrix descriptor (tile base 1024-aligned):
// start>>4 | LBO (16 B)>>4 << 16 | SBO (1024 B)>>4 << 32 | version 1 << 46 | layout 2 << 61
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}

// instruction descriptor, kind::f16: fp32 accumulate, fp16 A/B, both K-major
template <int BN>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(UM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

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
  __shared__ ArgBest best_s[4][BN];
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * UM, n0 = blockIdx.y * BN;
  const int KT = a.K / BK;
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
      tma_load_2d(smem + s * ST_BYTES, &a.map_w, s * BK, m0, &full_bar[s]);
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
      for (int s = 0; s < pre; ++s) tma_load_2d(smem + s * ST_BYTES + A_BYTES, &a.map_x, s * BK, n0, &full_bar[s]);
      for (int kt = pre; kt < KT; ++kt) {
        const int s = kt % NSTAGE;
        if (!mbar_wait_bounded(&empty_bar[s], ((kt / NSTAGE) - 1) & 1, a.err)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], uint32_t(ST_BYTES));
        tma_load_2d(smem + s * ST_BYTES, &a.map_w, kt * BK, m0, &full_bar[s]);
        tma_load_2d(smem + s * ST_BYTES + A_BYTES, &a.map_x, kt * BK, n0, &full_bar[s]);
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
  }
  if (!mbar_wait_bounded(&done_bar, 0, a.err)) abort_flag = 1;
  tc_fence_after();
  __syncthreads();

  ArgBest bst[BN / 16 > 0 ? BN / 16 : 1];
  if (!abort_flag) {
    const int row = m0 + warp * 32 + lane;  // this thread's weight row
    const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
#pragma unroll 1
    for (int cc = 0; cc < BN; cc += 16) {
      float v[16];
      tmem_ld16(trow + cc, v);
      if (EPI == kEpiStore || EPI == kEpiResid) {
        if (row < a.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = n0 + cc + j;
            if (b < a.B) {
              float* o = a.out + size_t(b) * a.ldo + row;
              if (EPI == kEpiResid) *o += v[j];
              else *o = v[j];
            }
          }
        }
      } else if (EPI == kEpiSwiglu) {
        // gate rows 16j..16j+7 and up rows 16j+8..16j+15 sit 8 lanes apart
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float up = __shfl_down_sync(0xffffffffu, v[j], 8);
          const int b = n0 + cc + j;
          if ((lane & 8) == 0 && row < a.N && b < a.B) {
            const float g = v[j];
            const int i = (row >> 4) * 8 + (row & 7);
            a.out16[size_t(b) * a.ldo + i] = __float2half_rn((g / (1.0f + expf(-g))) * up);
          }
        }
      } else {  // argmax over this CTA's rows, per batch column
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int b = n0 + cc + j;
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
          if (lane == 0) best_s[warp][cc + j] = {bv, bi};
        }
      }
    }
  }
  (void)bst;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(uint32_t(BN < 32 ? 32 : BN))
                 : "memory");
  }
  if (EPI != kEpiArgmax || abort_flag) return;

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
        if (step < s.hist_cap) s.hist[step * s.hist_stride + b] = next;
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

// RMSNorm of each batch row to fp16 (the tensor-core projections' input).
// kEmbed: row = embed[token[b]], also written to hidden[b] (layer 0).
template <bool kEmbed, bool kFinal>
__global__ void __launch_bounds__(256) rmsnorm_f16_kernel(NormArgs a) {
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const float* src = a.hidden + size_t(b) * a.H;
  float* const hidden_w = a.hidden_out;
  if (kEmbed) {
    int tok = a.tokens[b];
    if (tok < 0 || tok >= a.vocab) {
      set_error(a.err, kDevBadToken);
      tok = 0;
    }
    src = a.embed + size_t(tok) * a.H;
  }
  float ss = 0.f;
  for (int k = tid * 4; k < a.H; k += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(src + k);
    if (kEmbed) *reinterpret_cast<float4*>(hidden_w + size_t(b) * a.H + k) = v;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float rs = 1.0f / sqrtf(tot / float(a.H) + a.eps);
  for (int k = tid * 4; k < a.H; k += 1024) {
    const float4 v = *reinterpret_cast<const float4*>(src + k);
    const float4 w = *reinterpret_cast<const float4*>(a.w + k);
    float4 o;
    if (kFinal) o = make_float4((v.x * rs) * w.x, (v.y * rs) * w.y, (v.z * rs) * w.z, (v.w * rs) * w.w);
    else o = make_float4(v.x * (rs * w.x), v.y * (rs * w.y), v.z * (rs * w.z), v.w * (rs * w.w));
    uint2 h;
    h.x = pack_half2(o.x, o.y);
    h.y = pack_half2(o.z, o.w);
    *reinterpret_cast<uint2*>(a.out + size_t(b) * a.H + k) = h;
  }
}

template <int BN>
constexpr size_t tc_smem() {
  return size_t(stages_for<BN>()) * (UM * BK * 2 + BN * BK * 2) + 1024;
}

template <int BN, int EPI>
cudaError_t launch_bn(const TcArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + UM - 1) / UM, (a.B + BN - 1) / BN);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = tc_smem<BN>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
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

template <int EPI>
cudaError_t launch_epi(const TcArgs& a_in, cudaStream_t s, bool pdl) {
  const int bn = tc_batch_tile(a_in.N, a_in.B);
  TcArgs a = a_in;
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
  if ((r = cudaFuncSetAttribute(gemm_tc_kernel<BN, kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)) !=
      cudaSuccess)
    e = r;
  if ((r = cudaFuncSetAttribute(gemm_tc_kernel<BN, kEpiResid>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)) !=
      cudaSuccess)
    e = r;
  if ((r = cudaFuncSetAttribute(gemm_tc_kernel<BN, kEpiSwiglu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                bytes)) != cudaSuccess)
    e = r;
  if ((r = cudaFuncSetAttribute(gemm_tc_kernel<BN, kEpiArgmax>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                bytes)) != cudaSuccess)
    e = r;
  return e;
}

}  // namespace

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

cudaError_t launch_rmsnorm_f16(const NormArgs& a, bool embed, bool final_norm, cudaStream_t s, bool pdl) {
  if (a.H % 4 != 0 || a.B < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (embed) return cudaLaunchKernelEx(&cfg, rmsnorm_f16_kernel<true, false>, a);
  if (final_norm) return cudaLaunchKernelEx(&cfg, rmsnorm_f16_kernel<false, true>, a);
  return cudaLaunchKernelEx(&cfg, rmsnorm_f16_kernel<false, false>, a);
}

}  // namespace mmc
