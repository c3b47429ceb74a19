// Projections of small decode batches (5..64 rows) on mma.sync tensor cores,
// one kernel per projection with no split-K and no cross-CTA reduction.
//
// Replaces, for these batch sizes, the reference's per-projection Cube matvec
// (aclnnMm, ascend_matmul.cpp:385-410) and the RMSNorm / residual add /
// SwiGLU / ArgMax ops around it (ascend_custom_ops.cpp:535-604,
// ascend_matmul.cpp:467-497), in the data layout of the tensor-core path
// (fp16 input rows; the RMSNorm weight folded into W, the 1/rms applied in
// the epilogue from the producer's per-CTA sums of squares).
//
// At a few dozen rows a projection is a few microseconds of latency around a
// ~1 us weight read, so the kernel is laid out to keep the part after the
// dependency wait short:
//   * each CTA owns T 16-row weight tiles over the full K and bulk-copies them
//     (stored in HBM in the CTA's fragment order) into shared memory with one
//     copy issued before griddepcontrol.wait, so the weight read overlaps the
//     previous kernel;
//   * after the wait every thread issues its 16-byte cp.async copies of the
//     input rows at once (one L2 round trip for the whole [B][K] input), and
//     the 1/rms partial sums are loaded in parallel with them;
//   * warp w multiplies tile w % T over K-range w / T with m16n8k16 (weights
//     the A operand, batch rows on N), then the warps' partial tiles are summed
//     in shared memory in a fixed order and the epilogue (store / residual +
//     fp16 copy + sums of squares / SiLU*mul / argmax) writes the outputs.
// The tensor-core path's tcgen05 kernel (gemm_tc.cu) carries weights on the
// 128-row UMMA M side, which at 768-row projections leaves 6 tiles and needs
// split-K clusters to spread over the SMs; 16-row mma.sync tiles give every
// CTA its full K instead.
//
// K order. Within each 32-column block the reduction order is permuted so
// that one 16-byte load of an input row feeds two k16 steps: lane (g, t)
// holds row g's columns 8t..8t+7, of which 8t+4s+{0,1} / 8t+4s+{2,3} are the
// B fragment's k = 2t+{0,1} / 2t+8+{0,1} of step s; the weights are packed
// with the same map (launch_pack_skinny), so the products are unchanged and
// only the fp32 summation order differs from a plain k loop.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace mmc {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSsSlots = 5;  // sums-of-squares partials per row: at most 32 * kSsSlots

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return (v > bv) || (v == bv && i < bi); }

// 16-byte async copy; src_bytes = 0 fills the destination with zeros
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// Input rows larger than kXWhole bytes are staged in chunks of at most
// kXChunk bytes through two buffers (the next chunk's copies in flight while
// the warps multiply the current one).
constexpr int kXWhole = 128 * 1024;
constexpr int kXChunk = 64 * 1024;

struct SkLayout {
  size_t w_bytes, x_bytes, red_bytes, stash_bytes, total;
  int cb;  // 32-column blocks per input chunk (nb when staged whole)
};
// rows of the cross-warp partial tiles are padded by 8 floats so that the
// float2 stores of one warp hit distinct banks
__host__ __device__ constexpr int red_ld(int NT) { return NT * 8 + 8; }
__host__ __device__ inline SkLayout sk_layout(int T, int K, int NT) {
  SkLayout s;
  const int nb = K / 32;
  s.w_bytes = size_t(T) * nb * 1024;
  const int per_block = NT * 512;
  s.cb = nb * per_block <= kXWhole ? nb : kXChunk / per_block;
  s.x_bytes = size_t(s.cb < nb ? 2 : 1) * s.cb * per_block;
  s.red_bytes = size_t(kWarps) * 16 * red_ld(NT) * 4;
  s.stash_bytes = size_t(NT) * 8 * T * 16 * 4;
  // red aliases the input stage, the epilogue stash the weight slab (both
  // dead by then)
  const size_t a = s.w_bytes > s.stash_bytes ? s.w_bytes : s.stash_bytes;
  const size_t b = s.x_bytes > s.red_bytes ? s.x_bytes : s.red_bytes;
  s.w_bytes = (a + 127) / 128 * 128;
  s.total = s.w_bytes + b;
  return s;
}

template <int NT, int EPI>
__global__ void __launch_bounds__(kThreads, 2) skinny_kernel(const SkinnyArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t wbar;
  __shared__ float rs_s[64];
  __shared__ int abort_flag;
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, K = a.K, B = a.B;
  const int nb = K / 32;
  const int tiles_total = a.N / 16;
  const int tile0 = blockIdx.x * T;
  const int my_tiles = min(T, tiles_total - tile0);
  const SkLayout L = sk_layout(T, K, NT);
  uint8_t* w_s = smem;
  uint8_t* x_s = smem + L.w_bytes;
  float* red = reinterpret_cast<float*>(x_s);    // after the MMAs
  float* stash = reinterpret_cast<float*>(w_s);  // after the MMAs

  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&wbar, 1);
    fence_mbar_init();
    // the weight tiles do not depend on the previous kernel: copy them now
    const uint32_t bytes = uint32_t(my_tiles) * uint32_t(nb) * 1024u;
    mbar_arrive_expect_tx(&wbar, bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.Wf) + size_t(tile0) * nb * 1024;
    for (uint32_t off = 0; off < bytes; off += 65536u)
      bulk_g2s(w_s + off, src + off, min(bytes - off, 65536u), &wbar);
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();

  // ---- input rows: [block][n-tile][lane] 16-byte pieces, zero past row B,
  //      chunk c (blocks [c * cb, c * cb + cb)) into buffer c & 1
  const int cb = L.cb, nchunks = (nb + cb - 1) / cb;
  const size_t xbuf = size_t(cb) * NT * 512;
  auto stage = [&](int c) {
    const int blk0 = c * cb, nblk = min(cb, nb - blk0);
    uint8_t* dst = x_s + (c & 1) * xbuf;
    for (int i = tid; i < NT * nblk * 32; i += kThreads) {
      const int ln = i & 31, j = (i >> 5) % NT, blk = blk0 + (i >> 5) / NT;
      const int row = 8 * j + (ln >> 2);
      const __half* src = a.X + size_t(row < B ? row : 0) * K + blk * 32 + 8 * (ln & 3);
      cp_async16_zfill(dst + size_t(i) * 16, src, row < B ? 16u : 0u);
    }
  };
  stage(0);
  cp_async_commit();
  // ---- folded RMSNorm: 1/rms per batch row from the producer's partial
  //      sums (warp w takes rows w, w + 8, ...; every load is issued before
  //      any is summed, so this costs one L2 round trip)
  if (a.ss_in != nullptr) {
    float v[8][kSsSlots];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int b = warp + kWarps * q;
#pragma unroll
      for (int h = 0; h < kSsSlots; ++h) {
        const int m = lane + 32 * h;
        v[q][h] = (b < B && m < a.ss_parts) ? a.ss_in[size_t(b) * a.ss_parts + m] : 0.f;
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float ss = 0.f;
#pragma unroll
      for (int h = 0; h < kSsSlots; ++h) ss += v[q][h];
      ss = warp_sum(ss);
      const int b = warp + kWarps * q;
      if (lane == 0 && b < B) rs_s[b] = 1.0f / sqrtf(ss / float(K) + a.eps);
    }
  }
  if (!mbar_wait_bounded(&wbar, 0, a.err)) abort_flag = 1;

  // ---- warp w: tile w % T, K-range part w / T of every chunk
  const int kparts = kWarps / T;
  const int tw = warp % T, kp = warp / T;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) {
      stage(c + 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (!abort_flag && tw < my_tiles) {
      const int blk0 = c * cb, nblk = min(cb, nb - blk0);
      const int b0 = kp * nblk / kparts, b1 = (kp + 1) * nblk / kparts;
      const uint8_t* wt = w_s + size_t(tw) * nb * 1024 + size_t(blk0) * 1024 + lane * 16;
      const uint8_t* xt = x_s + (c & 1) * xbuf + lane * 16;
#pragma unroll 2
      for (int blk = b0; blk < b1; ++blk) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(wt + size_t(blk) * 1024);
        const uint4 w1 = *reinterpret_cast<const uint4*>(wt + size_t(blk) * 1024 + 512);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint4 x = *reinterpret_cast<const uint4*>(xt + (size_t(blk) * NT + j) * 512);
          mma16816(acc[j], w0.x, w0.y, w0.z, w0.w, x.x, x.y);
          mma16816(acc[j], w1.x, w1.y, w1.z, w1.w, x.z, x.w);
        }
      }
    }
    if (c + 1 < nchunks) __syncthreads();  // buffer c & 1 is restaged two chunks later
  }
  __syncthreads();  // every warp is done with the input stage and the weight slab
  constexpr int ld = red_ld(NT);
  {
    // partial tile of this warp: red[warp][16 rows][ld]
    const int g = lane >> 2, t = lane & 3;
    float* rw = red + size_t(warp) * 16 * ld;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      *reinterpret_cast<float2*>(rw + g * ld + 8 * j + 2 * t) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(rw + (g + 8) * ld + 8 * j + 2 * t) = make_float2(acc[j][2], acc[j][3]);
    }
  }
  __syncthreads();
  if (abort_flag) return;

  // ---- epilogue: element (tile tt, row r, batch column b), rows fastest
  auto value = [&](int tt, int r, int b) {
    float v = 0.f;
    for (int p = 0; p < kparts; ++p) v += red[(size_t(p * T + tt) * 16 + r) * ld + b];
    return a.ss_in != nullptr ? v * rs_s[b] : v;
  };
  if (EPI == kEpiStore) {
    for (int i = tid; i < my_tiles * 16 * B; i += kThreads) {
      const int r = i & 15, b = (i >> 4) % B, tt = (i >> 4) / B;
      a.out[size_t(b) * a.ldo + (tile0 + tt) * 16 + r] = value(tt, r, b);
    }
    return;
  }
  if (EPI == kEpiSwiglu) {
    // gate rows 0-7 and up rows 8-15 of every tile (interleaved by 8 at load)
    for (int i = tid; i < my_tiles * 8 * B; i += kThreads) {
      const int r = i & 7, b = (i >> 3) % B, tt = (i >> 3) / B;
      const float gt = value(tt, r, b), up = value(tt, r + 8, b);
      a.out16[size_t(b) * a.ldo + (tile0 + tt) * 8 + r] = __float2half_rn((gt / (1.0f + expf(-gt))) * up);
    }
    return;
  }
  const int rows = my_tiles * 16;
  if (EPI == kEpiResid) {
    for (int i = tid; i < rows * B; i += kThreads) {
      const int rr = i % rows, b = i / rows;
      const int row = tile0 * 16 + rr;
      const bool upd = a.row_sel == nullptr || a.row_sel[b] == a.row_sel_val;
      float nv = 0.f;
      if (upd) {
        nv = a.out[size_t(b) * a.ldo + row] + value(rr >> 4, rr & 15, b);
        a.out[size_t(b) * a.ldo + row] = nv;
        if (a.h16_out) a.h16_out[size_t(b) * a.N + row] = __float2half_rn(nv);
      }
      stash[size_t(b) * rows + rr] = nv * nv;
    }
    if (a.ss_out == nullptr) return;
    __syncthreads();
    if (tid < B && (a.row_sel == nullptr || a.row_sel[tid] == a.row_sel_val)) {
      float s = 0.f;
      for (int rr = 0; rr < rows; ++rr) s += stash[size_t(tid) * rows + rr];
      a.ss_out[size_t(tid) * gridDim.x + blockIdx.x] = s;
    }
    return;
  }

  // ---- argmax (lm_head): logits, first maximum per batch row over the CTA's
  //      rows, then over the CTAs (the last CTA to arrive)
  for (int i = tid; i < rows * B; i += kThreads) {
    const int rr = i % rows, b = i / rows;
    const float v = value(rr >> 4, rr & 15, b);
    if (a.logits) a.logits[size_t(b) * a.N + tile0 * 16 + rr] = v;
    stash[size_t(b) * rows + rr] = v;
  }
  __syncthreads();
  ArgBest* part = reinterpret_cast<ArgBest*>(a.argmax_part);
  if (tid < B) {
    ArgBest bb = {-INFINITY, 0x7fffffff};
    for (int rr = 0; rr < rows; ++rr) {
      const float v = stash[size_t(tid) * rows + rr];
      if (better(v, tile0 * 16 + rr, bb.v, bb.i)) bb = {v, tile0 * 16 + rr};
    }
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
      const int next = (bb.i >= 0 && bb.i < a.N) ? bb.i : 0;  // all-NaN row: token 0
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
    if (a.sink.hist_step) *a.sink.hist_step += 1;
    *a.counter = 0u;
  }
}

// dst[tile][block][step][lane][8 halves]: lane (g, t), step s, register q
// (a0..a3 = rows g / g+8 x low / high column pair), half e of the pair:
// row g + 8 * (q & 1), column block * 32 + 8t + 4s + 2 * (q >> 1) + e
__global__ void pack_skinny_kernel(const __half* __restrict__ src, __half* __restrict__ dst, int64_t N, int64_t K) {
  const int64_t total = N * K;
  for (int64_t o = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; o < total; o += int64_t(gridDim.x) * blockDim.x) {
    const int64_t tile = o / (16 * K), rem = o % (16 * K);
    const int64_t blk = rem / 512;
    const int w = int(rem % 512);
    const int s = w / 256, ln = (w % 256) / 8, e8 = w % 8;
    const int g = ln >> 2, t = ln & 3, q = e8 >> 1, e = e8 & 1;
    const int64_t row = tile * 16 + g + 8 * (q & 1);
    const int64_t col = blk * 32 + 8 * t + 4 * s + 2 * (q >> 1) + e;
    dst[o] = src[row * K + col];
  }
}

template <int NT, int EPI>
cudaError_t launch_nt(const SkinnyArgs& a, size_t smem, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  const int tiles = a.N / 16;
  cfg.gridDim = dim3((tiles + a.T - 1) / a.T);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, skinny_kernel<NT, EPI>, a);
}

int nt_of(int B) {
  const int nt = (B + 7) / 8;
  return nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8;
}

template <int EPI>
cudaError_t launch_epi(const SkinnyArgs& a, size_t smem, cudaStream_t s, bool pdl) {
  switch (nt_of(a.B)) {
    case 1: return launch_nt<1, EPI>(a, smem, s, pdl);
    case 2: return launch_nt<2, EPI>(a, smem, s, pdl);
    case 4: return launch_nt<4, EPI>(a, smem, s, pdl);
    default: return launch_nt<8, EPI>(a, smem, s, pdl);
  }
}

template <int NT>
cudaError_t attrs_nt() {
  cudaError_t e = cudaSuccess, r;
  const int bytes = kSkinnyMaxSmem;
  if ((r = set_kernel_smem(skinny_kernel<NT, kEpiStore>, bytes)) != cudaSuccess) e = r;
  if ((r = set_kernel_smem(skinny_kernel<NT, kEpiResid>, bytes)) != cudaSuccess) e = r;
  if ((r = set_kernel_smem(skinny_kernel<NT, kEpiSwiglu>, bytes)) != cudaSuccess) e = r;
  if ((r = set_kernel_smem(skinny_kernel<NT, kEpiArgmax>, bytes)) != cudaSuccess) e = r;
  return e;
}

}  // namespace

int skinny_tiles_per_cta(int N, int num_sms) {
  const int tiles = N / 16;
  for (int T : {1, 2, 4, 8})
    if ((tiles + T - 1) / T <= num_sms) return T;
  return 8;
}

int skinny_grid(int N, int num_sms) {
  const int T = skinny_tiles_per_cta(N, num_sms);
  return (N / 16 + T - 1) / T;
}

size_t skinny_smem_bytes(int N, int K, int B, int num_sms) {
  return sk_layout(skinny_tiles_per_cta(N, num_sms), K, nt_of(B)).total;
}

bool skinny_supported(int N, int K, int B, int num_sms) {
  return B >= 1 && B <= kSkinnyMaxBatch && N >= 16 && N % 16 == 0 && K % 32 == 0 && K >= 32 &&
         skinny_grid(N, num_sms) <= 32 * kSsSlots && skinny_smem_bytes(N, K, B, num_sms) <= size_t(kSkinnyMaxSmem);
}

cudaError_t skinny_init_attributes() {
  cudaError_t e1 = attrs_nt<1>(), e2 = attrs_nt<2>(), e4 = attrs_nt<4>(), e8 = attrs_nt<8>();
  return e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e4 != cudaSuccess ? e4 : e8;
}

cudaError_t launch_skinny(int epi, const SkinnyArgs& a_in, int num_sms, cudaStream_t s, bool pdl) {
  if (!skinny_supported(a_in.N, a_in.K, a_in.B, num_sms) || a_in.Wf == nullptr || a_in.X == nullptr)
    return cudaErrorInvalidValue;
  if (a_in.ss_in != nullptr && (a_in.ss_parts <= 0 || a_in.ss_parts > 32 * kSsSlots)) return cudaErrorInvalidValue;
  if (epi == kEpiArgmax && (a_in.argmax_part == nullptr || a_in.counter == nullptr)) return cudaErrorInvalidValue;
  SkinnyArgs a = a_in;
  a.T = skinny_tiles_per_cta(a.N, num_sms);
  const size_t smem = sk_layout(a.T, a.K, nt_of(a.B)).total;
  switch (epi) {
    case kEpiStore: return launch_epi<kEpiStore>(a, smem, s, pdl);
    case kEpiResid: return launch_epi<kEpiResid>(a, smem, s, pdl);
    case kEpiSwiglu: return launch_epi<kEpiSwiglu>(a, smem, s, pdl);
    case kEpiArgmax: return launch_epi<kEpiArgmax>(a, smem, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pack_skinny(const __half* src, __half* dst, int64_t N, int64_t K, cudaStream_t s) {
  if (N % 16 != 0 || K % 32 != 0) return cudaErrorInvalidValue;
  pack_skinny_kernel<<<1184, 256, 0, s>>>(src, dst, N, K);
  return cudaGetLastError();
}

}  // namespace mmc
