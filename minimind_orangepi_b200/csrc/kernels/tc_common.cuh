// tcgen05 / TMA building blocks shared by the tensor-core projection kernels
// (gemm_tc.cu, mlp_chain.cu): UMMA shared-memory and instruction descriptors,
// MMA issue and commit, TMEM load / dealloc, 2-D TMA tile loads, and a warp
// column-sum helper for epilogues.
#pragma once

#include "common.cuh"

namespace mmc {

constexpr int UM = 128;  // UMMA M (weight rows per CTA)
constexpr int BK = 64;   // K per stage (one 128-byte swizzle atom of fp16)

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
// Column sums of a 32-row x 16-column block held one row per lane (x[16]):
// a reduce-scatter butterfly (8 + 4 + 2 + 1 shuffles) leaves each lane pair
// with one column, one more shuffle completes it. Returns the sum of column
// colsum16_col(lane) (the same in both lanes of a pair); x is clobbered.
__device__ __forceinline__ int colsum16_col(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
__device__ __forceinline__ float colsum16(float* x, int lane) {
#pragma unroll
  for (int o = 16, n = 8; o >= 2; o >>= 1, n >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = hi ? x[i] : x[i + n];
      const float keep = hi ? x[i + n] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return x[0] + __shfl_xor_sync(0xffffffffu, x[0], 1);
}

template <int COLS>
__device__ __forceinline__ void tmem_dealloc(uint32_t tmem) {
  tc_fence_after();
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(COLS < 32 ? 32 : COLS))
               : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cta address -> the same offset in cluster CTA `rank`'s shared memory
__device__ __forceinline__ uint32_t map_dsmem(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

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


// tensor map of a row-major fp16 [rows][K] matrix, 64 x box_rows boxes, 128-byte swizzle
cudaError_t tc_make_map(CUtensorMap* m, const __half* base, int rows, int K, int box_rows);

}  // namespace mmc
