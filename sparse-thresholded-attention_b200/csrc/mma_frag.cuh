// Warp-level m16n8k16 bf16 fragments (ldmatrix + mma.sync), used by the gather-attend and
// PQ-Stream kernels for their per-tile (16 query rows x 64 slot) products.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace sta {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// C (16x8 fp32) += A (16x16 bf16, row) * B (16x8 bf16, col)
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// split two fp32 values into packed hi and lo bf16 pairs
__device__ __forceinline__ void pack_split(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(x0, __bfloat162float(h0)));
  const __nv_bfloat16 l1 = __float2bfloat16_rn(__fsub_rn(x1, __bfloat162float(h1)));
  __nv_bfloat162 H, L;
  H.x = h0;
  H.y = h1;
  L.x = l0;
  L.y = l1;
  hi = *reinterpret_cast<uint32_t*>(&H);
  lo = *reinterpret_cast<uint32_t*>(&L);
}

}  // namespace sta

namespace sta {

// x ~= sum_i piece_i, each piece a bf16 (NP = 1: plain rounding, 2: hi + lo, 3: hi + mid + lo).
// Every residual is formed exactly in fp32, so NP pieces keep ~8*NP significant bits.
template <int NP>
__device__ __forceinline__ void split_pieces(float x, __nv_bfloat16 (&o)[NP]) {
  float r = x;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    o[i] = __float2bfloat16_rn(r);
    r = __fsub_rn(r, __bfloat162float(o[i]));
  }
}

// two fp32 values -> NP packed bf16x2 pieces
template <int NP>
__device__ __forceinline__ void pack_pieces(float x0, float x1, uint32_t (&o)[NP]) {
  __nv_bfloat16 a[NP], b[NP];
  split_pieces<NP>(x0, a);
  split_pieces<NP>(x1, b);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    __nv_bfloat162 v;
    v.x = a[i];
    v.y = b[i];
    o[i] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// C += sum over piece pairs (pa, pb) with pa + pb < NP of A_pa * B_pb, smallest terms first.
// NP = 2 gives the 3-product "3xBF16" form, NP = 3 the 6-product fp32-accurate form.
template <int NP>
__device__ __forceinline__ void mma_pieces(float (&c)[4], const uint32_t (&a)[NP][4],
                                           const uint32_t (&b)[NP][2]) {
#pragma unroll
  for (int s = NP - 1; s >= 0; --s) {
#pragma unroll
    for (int pa = s; pa >= 0; --pa) {
      const int pb = s - pa;
      mma_bf16(c, a[pa], b[pb][0], b[pb][1]);
    }
  }
}

}  // namespace sta
