// Fused decode attention over a paged fp16 KV cache.
//
// Replaces, for one decoder layer, the reference's
//   mini_mind_decode_qkv_postprocess (per-head q/k RMSNorm + RoPE + K/V append,
//     op_kernel/mini_mind_decode_qkv_postprocess.cpp:54-177; CPU form
//     decoder_layer.cpp:342-359) and
//   mini_mind_attention (GQA softmax(q.K/sqrt(d)).V over the cache,
//     op_kernel/mini_mind_attention.cpp:41-91; CPU form decoder_layer.cpp:184-234)
// with one launch.
//
// Grid (split, kv_head, batch_row); 4 warps per CTA. A CTA walks its split of
// the sequence one 64-token page at a time: each page's K and V slabs (one
// contiguous 64 x hd fp16 block each) arrive by bulk async copy into a
// multi-stage shared-memory ring, issued before griddepcontrol.wait because
// cached positions never depend on the projection kernel in front of it.
// Each warp owns 16 tokens of a page:
//   S^T[16 tok x 8 heads] = K[16 x hd] . Q^T     (mma m16n8k16, heads on N)
//   online softmax per head (exp2 domain)
//   P^T -> B fragment by movmatrix (8x8 transpose in registers)
//   O^T[hd x 8 heads] += V^T[hd x 16 tok] . P^T  (ldmatrix.trans for V^T)
// The q heads of the GQA group sit on the mma N dimension, so one K/V read
// serves all of them. Warps, then splits, are merged with the usual
// (max, sum, acc) rescaling; the last CTA of a (row, kv_head) merges the splits
// (arrival counter, self-resetting).
//
// Rows inside a page are stored with a 16-byte-chunk XOR swizzle (common.cuh
// swz_chunk) so the flat page copy lands in shared memory already
// conflict-free for ldmatrix; the append writes the same layout.
#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxRep = 8;  // q heads per kv head carried on the mma N dimension

template <int HD>
struct AttnCfg {
  static constexpr int CPR = HD / 8;                     // 16-byte chunks per row
  static constexpr int TILE = kPageTokens * HD;          // halves per K (or V) page slab
  static constexpr int NST = HD <= 96 ? 4 : 3;           // ring stages
  static constexpr int KC = HD / 16;                     // k-chunks (S) == m-tiles (O)
  static constexpr size_t STAGE_BYTES = size_t(2) * TILE * 2;
  static constexpr size_t RING_BYTES = NST * STAGE_BYTES;
  static constexpr size_t COMB_FLOATS = 4 * kMaxRep * (HD + 2);
  static constexpr size_t SMEM = RING_BYTES + COMB_FLOATS * 4 + kMaxRep * HD * 2 + 2 * HD * 2;
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

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnArgs a) {
  using C = AttnCfg<HD>;
  extern __shared__ __align__(128) uint8_t smem[];
  __half* ring = reinterpret_cast<__half*>(smem);
  float* comb = reinterpret_cast<float*>(smem + C::RING_BYTES);  // [4 warps][8 heads][HD + 2]
  __half* q_s = reinterpret_cast<__half*>(comb + C::COMB_FLOATS);  // [8][HD]
  __half* kv_new = q_s + kMaxRep * HD;                             // [2][HD]
  __shared__ __align__(8) uint64_t bars[C::NST];
  __shared__ int abort_flag;
  __shared__ bool is_last;

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int rep = a.nq / a.nkv;

  // Cached positions and the page table were settled before the kernel in
  // front of this one started (see the file comment), so read them pre-wait.
  const int slot = a.slots[b];
  const int pos = a.seq_pos[slot];
  const int ctx = pos + 1;
  const int tok_begin = split * a.split_tokens;
  if (tok_begin >= ctx) {
    pdl_wait();
    pdl_launch_dependents();
    return;
  }
  const int tok_end = min(ctx, tok_begin + a.split_tokens);
  const int nsplits = (ctx + a.split_tokens - 1) / a.split_tokens;
  const int n_chunks = (tok_end - tok_begin + kPageTokens - 1) / kPageTokens;
  const bool owns_tail = tok_end == ctx;
  const int* bt = a.block_table + (size_t)slot * a.max_pages;

  if (tid == 0) {
    abort_flag = 0;
    if (pos >= a.max_pos || nsplits > a.max_splits) {
      set_error(a.err, kDevPositionLimit);
      abort_flag = 1;
    }
    for (int s = 0; s < C::NST; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (abort_flag) {
    pdl_wait();
    pdl_launch_dependents();
    return;
  }

  auto issue = [&](int c) {  // thread 0 only
    const int stage = c % C::NST;
    const int pidx = tok_begin / kPageTokens + c;
    const int page = pidx < a.max_pages ? bt[pidx] : -1;
    __half* dst = ring + (size_t)stage * 2 * C::TILE;
    if (page < 0) {
      set_error(a.err, kDevNoPage);
      abort_flag = 1;
      // complete the phase without data so waiters do not hang
      mbar_arrive_expect_tx(&bars[stage], 0);
      return;
    }
    mbar_arrive_expect_tx(&bars[stage], uint32_t(C::STAGE_BYTES));
    bulk_g2s(dst, a.kv_pool + page_slab(page, a.layer, a.layers, 0, a.nkv, h, C::TILE), C::TILE * 2, &bars[stage]);
    bulk_g2s(dst + C::TILE, a.kv_pool + page_slab(page, a.layer, a.layers, 1, a.nkv, h, C::TILE), C::TILE * 2,
             &bars[stage]);
  };
  if (tid == 0) {
    for (int c = 0; c < min(C::NST, n_chunks); ++c) issue(c);
  }

  pdl_wait();
  pdl_launch_dependents();

  // ------------------------------------------- q (and tail k/v) post-process
  const float* row = a.qkv + (size_t)b * a.ld_qkv;
  const float* cos_r = a.rope_cos + (size_t)pos * (HD / 2);
  const float* sin_r = a.rope_sin + (size_t)pos * (HD / 2);
  for (int j = warp; j < kMaxRep; j += 4) {
    if (j < rep) {
      norm_rope_head<HD>(row + (size_t)(h * rep + j) * HD, a.q_norm, cos_r, sin_r, a.eps, q_s + j * HD, lane);
    } else {
      for (int d = lane; d < HD; d += 32) q_s[j * HD + d] = __float2half_rn(0.f);
    }
  }
  const int tail_row = pos % kPageTokens;
  if (owns_tail) {
    if (warp == 0) {
      norm_rope_head<HD>(row + (size_t)(a.nq + h) * HD, a.k_norm, cos_r, sin_r, a.eps, kv_new, lane);
    } else if (warp == 1) {
      const float* v = row + (size_t)(a.nq + a.nkv + h) * HD;
      for (int d = lane; d < HD; d += 32) kv_new[HD + d] = __float2half_rn(v[d]);
    }
  }
  __syncthreads();
  if (owns_tail && tid < 2 * C::CPR) {
    // append the new K/V row into the cache page (swizzled row layout)
    const int kv = tid / C::CPR, c = tid % C::CPR;
    const int page = bt[pos / kPageTokens];
    if (page >= 0) {
      __half* dst = a.kv_pool + page_slab(page, a.layer, a.layers, kv, a.nkv, h, C::TILE) + (size_t)tail_row * HD +
                    swz_chunk(tail_row, c, C::CPR) * 8;
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(kv_new + kv * HD + c * 8);
    }
  }

  // Q^T as the B operand of S^T = K . Q^T: b0 = Q[g][16kc + 2t..], b1 = +8
  uint32_t qb0[C::KC], qb1[C::KC];
#pragma unroll
  for (int kc = 0; kc < C::KC; ++kc) {
    qb0[kc] = *reinterpret_cast<const uint32_t*>(q_s + g * HD + 16 * kc + 2 * t);
    qb1[kc] = *reinterpret_cast<const uint32_t*>(q_s + g * HD + 16 * kc + 8 + 2 * t);
  }

  const float sl2 = 1.4426950408889634f / sqrtf(float(HD));
  float mA = -1e30f, mB = -1e30f, lA = 0.f, lB = 0.f;
  float o[C::KC][4];
#pragma unroll
  for (int mt = 0; mt < C::KC; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  const int r0 = warp * 16;
  for (int c = 0; c < n_chunks; ++c) {
    const int stage = c % C::NST;
    const uint32_t parity = (c / C::NST) & 1;
    if (!mbar_wait_bounded(&bars[stage], parity, a.err)) abort_flag = 1;
    __half* kt = ring + (size_t)stage * 2 * C::TILE;
    __half* vt = kt + C::TILE;
    const bool tail_chunk = owns_tail && c == n_chunks - 1;
    if (tail_chunk) {
      __syncthreads();
      if (tid < 2 * C::CPR) {
        const int kv = tid / C::CPR, cc = tid % C::CPR;
        __half* dst = (kv ? vt : kt) + tail_row * HD + swz_chunk(tail_row, cc, C::CPR) * 8;
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(kv_new + kv * HD + cc * 8);
      }
    }
    __syncthreads();
    if (abort_flag) return;

    const int tok0 = tok_begin + c * kPageTokens + r0;
    if (tok0 < tok_end) {
      // ---- S^T = K . Q^T over this warp's 16 tokens
      float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kc = 0; kc < C::KC; ++kc) {
        const int rr = r0 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int ch = 2 * kc + (lane >> 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(smem_u32(kt + rr * HD + swz_chunk(rr, ch, C::CPR) * 8), a0, a1, a2, a3);
        mma16816(s, a0, a1, a2, a3, qb0[kc], qb1[kc]);
      }
      const bool v0 = tok0 + g < tok_end, v1 = tok0 + g + 8 < tok_end;
      const float sA0 = v0 ? s[0] * sl2 : -INFINITY, sB0 = v0 ? s[1] * sl2 : -INFINITY;
      const float sA1 = v1 ? s[2] * sl2 : -INFINITY, sB1 = v1 ? s[3] * sl2 : -INFINITY;
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
        const int rr = r0 + ((lane >> 4) & 1) * 8 + (lane & 7);
        const int ch = 2 * mt + ((lane >> 3) & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(smem_u32(vt + rr * HD + swz_chunk(rr, ch, C::CPR) * 8), a0, a1, a2, a3);
        mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && c + C::NST < n_chunks) {
      fence_proxy_async_smem();
      issue(c + C::NST);
    }
  }

  // ------------------------------------------------- merge the 4 warps
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, off);
    lB += __shfl_xor_sync(0xffffffffu, lB, off);
  }
  {
    float* cw = comb + (size_t)warp * kMaxRep * (HD + 2);
    const int hA = 2 * t, hB = 2 * t + 1;
#pragma unroll
    for (int mt = 0; mt < C::KC; ++mt) {
      cw[hA * (HD + 2) + 16 * mt + g] = o[mt][0];
      cw[hB * (HD + 2) + 16 * mt + g] = o[mt][1];
      cw[hA * (HD + 2) + 16 * mt + g + 8] = o[mt][2];
      cw[hB * (HD + 2) + 16 * mt + g + 8] = o[mt][3];
    }
    if (g == 0) {
      cw[hA * (HD + 2) + HD] = mA;
      cw[hA * (HD + 2) + HD + 1] = lA;
      cw[hB * (HD + 2) + HD] = mB;
      cw[hB * (HD + 2) + HD + 1] = lB;
    }
  }
  __syncthreads();

  const size_t pstride = (size_t)rep * (HD + 2);
  float* part_bh = a.part + ((size_t)b * a.nkv + h) * a.max_splits * pstride;
  const size_t out_off = (size_t)b * a.nq * HD + (size_t)h * rep * HD;
  auto put_out = [&](int idx, float v) {
    if (a.out16) a.out16[out_off + idx] = __float2half_rn(v);
    else a.out[out_off + idx] = v;
  };
  for (int i = tid; i < rep * HD; i += kAttnThreads) {
    const int j = i / HD, d = i % HD;
    float M = -1e30f;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, comb[(w * kMaxRep + j) * (HD + 2) + HD]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float* cw = comb + (w * kMaxRep + j) * (HD + 2);
      const float f = exp2f(cw[HD] - M);
      L += cw[HD + 1] * f;
      O += cw[d] * f;
    }
    if (nsplits == 1) {
      put_out(j * HD + d, O / L);
    } else {
      float* p = part_bh + split * pstride + j * (HD + 2);
      p[d] = O;
      if (d == 0) {
        p[HD] = M;
        p[HD + 1] = L;
      }
    }
  }
  if (nsplits == 1) return;

  // ---------------------------------------------- merge splits (last CTA)
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&a.counters[(size_t)b * a.nkv + h], 1u) == unsigned(nsplits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int i = tid; i < rep * HD; i += kAttnThreads) {
    const int j = i / HD, d = i % HD;
    float M = -1e30f;
    for (int s = 0; s < nsplits; ++s) M = fmaxf(M, __ldcg(part_bh + s * pstride + j * (HD + 2) + HD));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nsplits; ++s) {
      const float* p = part_bh + s * pstride + j * (HD + 2);
      const float f = exp2f(__ldcg(p + HD) - M);
      L += __ldcg(p + HD + 1) * f;
      O += __ldcg(p + d) * f;
    }
    put_out(j * HD + d, O / L);
  }
  if (tid == 0) a.counters[(size_t)b * a.nkv + h] = 0u;
}

template <int HD>
cudaError_t launch_hd(const AttnArgs& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.max_splits, a.nkv, a.B);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = AttnCfg<HD>::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, attention_kernel<HD>, a);
}

template <int HD>
cudaError_t attr_hd() {
  return cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(AttnCfg<HD>::SMEM));
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
      a.max_splits <= 0 || a.B <= 0)
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
