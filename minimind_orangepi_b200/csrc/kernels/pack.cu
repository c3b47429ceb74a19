// Weight packing at load time: fp32 rows from weights.bin -> fp16 rows in HBM.
//
// The reference packs its device weights transposed ([K][N]) for the Cube
// unit and rounds half away from zero (ascend_matmul.cpp:28-61, 285-305). Here
// rows stay row-major [N][K] — a decode projection streams each weight row once
// and contiguous rows give contiguous slabs — and rounding is IEEE
// round-to-nearest-even (__float2half_rn).
//
// gate/up are fused like the reference's gate_up_proj (language_model.cpp:95-119)
// but interleaved in blocks of 8 rows: packed rows [16j, 16j+8) are gate rows
// [8j, 8j+8) and packed rows [16j+8, 16j+16) the matching up rows, so the
// SiLU*mul epilogue finds gate_i and up_i 8 rows apart inside one 16-row tile.
//
// A projection that reads an RMSNorm output gets the norm weight folded into
// its columns (W'[n][k] = W[n][k] * w[k], rounded once): the decode kernels then
// only scale by the per-row 1/rms, which lets the tensor-core path carry the
// norm across kernels without a normalisation pass.
#include "kernels.h"

namespace mmc {
namespace {

__global__ void pack_rows_kernel(const float* __restrict__ src, __half* __restrict__ dst, int64_t n, int64_t cols,
                                 const float* __restrict__ col_scale) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __float2half_rn(col_scale ? src[i] * col_scale[i % cols] : src[i]);
}

__global__ void pack_gate_up_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                    __half* __restrict__ dst, int64_t inter, int64_t cols,
                                    const float* __restrict__ col_scale) {
  const int64_t n = 2 * inter * cols;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t prow = i / cols, c = i % cols;
    const int64_t blk = prow / 16, r = prow % 16;
    const int64_t src_row = blk * 8 + (r & 7);
    const float* s = r < 8 ? gate : up;
    const float v = s[src_row * cols + c];
    dst[i] = __float2half_rn(col_scale ? v * col_scale[c] : v);
  }
}

// Seeded pseudo-random fp16 values in [-2, 2) for positions [0, n) of one
// sequence's pages (all layers, K and V). A 32-bit integer hash of the element
// index gives reproducible contents.
__global__ void fill_kv_kernel(__half* pool, const int* pages, int n_tokens, int64_t page_halves, int row_halves,
                               uint32_t seed) {
  const int64_t total = int64_t((n_tokens + 63) / 64) * page_halves;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int p = int(i / page_halves);
    const int64_t off = i % page_halves;
    const int row = int((off / row_halves) % 64);
    if (p * 64 + row >= n_tokens) continue;
    uint32_t x = uint32_t(i) * 0x9E3779B9u ^ seed;
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    const float v = float(x & 0xFFFF) * (4.0f / 65536.0f) - 2.0f;
    pool[int64_t(pages[p]) * page_halves + off] = __float2half_rn(v);
  }
}

// Keeps the GPU busy for about `ns` nanoseconds (bounded by the global timer)
// so that host-side enqueueing finishes before timed work starts.
__global__ void hold_kernel(uint64_t ns) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  uint64_t t = t0;
  while (t - t0 < ns) {
    __nanosleep(1000);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  }
}

}  // namespace

cudaError_t launch_hold(uint64_t ns, cudaStream_t s) {
  if (ns > 100000000ull) ns = 100000000ull;  // at most 0.1 s
  hold_kernel<<<1, 1, 0, s>>>(ns);
  return cudaGetLastError();
}

cudaError_t launch_fill_kv(__half* pool, const int* pages, int n_tokens, int64_t page_halves, int row_halves,
                           uint32_t seed, cudaStream_t s) {
  fill_kv_kernel<<<592, 256, 0, s>>>(pool, pages, n_tokens, page_halves, row_halves, seed);
  return cudaGetLastError();
}

cudaError_t launch_pack_rows(const float* src, __half* dst, int64_t rows, int64_t cols, cudaStream_t s,
                             const float* col_scale) {
  pack_rows_kernel<<<1184, 256, 0, s>>>(src, dst, rows * cols, cols, col_scale);
  return cudaGetLastError();
}

cudaError_t launch_pack_gate_up(const float* gate, const float* up, __half* dst, int64_t inter, int64_t cols,
                                cudaStream_t s, const float* col_scale) {
  if (inter % 8 != 0) return cudaErrorInvalidValue;
  pack_gate_up_kernel<<<1184, 256, 0, s>>>(gate, up, dst, inter, cols, col_scale);
  return cudaGetLastError();
}

}  // namespace mmc
