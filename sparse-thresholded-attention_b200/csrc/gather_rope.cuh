// Row gather + RoPE helpers shared by the attend and PQ-Stream kernels: vectorised loads of 8
// elements, rotation of 8 frequency pairs (direct sincos or an exact cos/sin table), split into
// bf16 pieces, and 16-byte copies of pre-rotated rows.
#pragma once

#include "common.cuh"
#include "mma_frag.cuh"

namespace sta {

// 8 consecutive elements as fp32
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// Rotate 8 frequency pairs (f0..f0+7 with partners f0+HALF..) of one row and store the NP-piece
// split into a padded smem row set (plane stride `plane`, row pointer `dst`).
// Position `pos` as an index of the cos/sin table (entries at i / R), or -1 when the table does
// not hold it.  Entries are formed from the exact float i / R with the same fp32 expression as
// the direct path, so a hit is bit-identical to recomputing.
__device__ __forceinline__ int64_t table_index(float pos, float R, int64_t len) {
  if (len <= 0) return -1;
  const float fi = pos * R;  // exact: R is +-1 or a power of two
  if (!(fi >= 0.f) || fi != floorf(fi) || fi >= (float)len) return -1;
  return (int64_t)fi;
}

template <int NP, int HALF, typename TV>
__device__ __forceinline__ void rotate8(const TV* src, bool valid, int f0, float pos,
                                        const float* inv_freq, float rope_scale,
                                        __nv_bfloat16* dst, int plane,
                                        const float2* tab = nullptr, int64_t ti = -1) {
  float x1[8], x2[8];
  if (valid) {
    load8(src + f0, x1);
    load8(src + f0 + HALF, x2);
  } else {
#pragma unroll
    for (int u = 0; u < 8; ++u) x1[u] = x2[u] = 0.f;
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    float r1, r2;
    if (ti >= 0) {
      const float2 cs = __ldg(tab + ti * HALF + f0 + u);
      r1 = __fsub_rn(__fmul_rn(x1[u], cs.x), __fmul_rn(x2[u], cs.y));
      r2 = __fadd_rn(__fmul_rn(x2[u], cs.x), __fmul_rn(x1[u], cs.y));
    } else {
      const float ang = __fmul_rn(pos, __ldg(inv_freq + f0 + u));
      rope_pair(x1[u], x2[u], ang, rope_scale, r1, r2);
    }
    __nv_bfloat16 a[NP], b[NP];
    split_pieces<NP>(r1, a);
    split_pieces<NP>(r2, b);
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      dst[j * plane + f0 + u] = a[j];
      dst[j * plane + f0 + u + HALF] = b[j];
    }
  }
}

// copy 8 pre-rotated bf16 (hi and lo) of both halves of a row
template <int HALF>
__device__ __forceinline__ void copy_rotated(const __nv_bfloat16* hi, const __nv_bfloat16* lo,
                                             int f0, __nv_bfloat16* dst, int plane) {
  *reinterpret_cast<uint4*>(dst + f0) = *reinterpret_cast<const uint4*>(hi + f0);
  *reinterpret_cast<uint4*>(dst + f0 + HALF) = *reinterpret_cast<const uint4*>(hi + f0 + HALF);
  *reinterpret_cast<uint4*>(dst + plane + f0) = *reinterpret_cast<const uint4*>(lo + f0);
  *reinterpret_cast<uint4*>(dst + plane + f0 + HALF) = *reinterpret_cast<const uint4*>(lo + f0 + HALF);
}

template <typename TV>
__device__ __forceinline__ float ldf(const TV* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}


}  // namespace sta
