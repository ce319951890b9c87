// RoPE prologue of the selection geometry: rotate raw Q or K rows at their (scaled) positions
// and store the fp32 result as a (hi, lo) pair of bf16 tensors, the operand format of the
// 3xBF16 tensor-core score products.
//
// Reference behaviour (shared_selection_triton_exact_2.py:79-86 for Q, :97-104 for K): the
// reference re-derives RoPE(K) for every (query tile, key block) pair in both passes, i.e.
// O(N^2 D) trigonometry.  The selection geometry does not depend on the query tile, so here
// every row is rotated exactly once (O(N D)) and the passes become plain contractions.
#include "common.cuh"
#include "gather_rope.cuh"
#include "sta_internal.h"

namespace sta {

template <typename T>
__device__ __forceinline__ float load_f(const T* p);
template <>
__device__ __forceinline__ float load_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// Position id of row n: linear n (mode 0) or one of the Dual Chunk Attention position sets of
// ChunkLlama's rotary tables (dca_kernel.py:194-231, chunk_len L = chunk_size s - local window):
// mode 1 keys and same-chunk queries n mod L; mode 2 queries against the previous chunk
// min(L + n mod L, s); mode 3 queries against older chunks min(2L - 1, s).
__device__ __forceinline__ int64_t position_id(int64_t n, int mode, int64_t L, int64_t s) {
  if (mode == 1) return n % L;
  if (mode == 2) return min(L + n % L, s);
  if (mode == 3) return min(2 * L - 1, s);
  return n;
}

// One thread per (row, frequency pair).  x is (rows = heads*N, D) with element strides
// (stride_h, stride_n); last dim contiguous; row n sits at position pos0 + n.
// Angle = (float(position_id) * pos_scale) * inv_freq.
template <typename T>
__global__ void rope_split_kernel(const T* __restrict__ x, int64_t heads, int64_t N, int D,
                                  int64_t stride_h, int64_t stride_n,
                                  const float* __restrict__ inv_freq, float pos_scale,
                                  float rope_scale, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo, int mode, int64_t dca_L,
                                  int64_t dca_s, int64_t pos0) {
  const int half = D >> 1;
  const int64_t total = heads * N * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int f = (int)(i % half);
    const int64_t row = i / half;
    const int64_t n = row % N;
    const int64_t h = row / N;
    const T* src = x + h * stride_h + n * stride_n;
    const float x1 = load_f(src + f);
    const float x2 = load_f(src + f + half);
    const float pid = (float)position_id(pos0 + n, mode, dca_L, dca_s);
    const float ang = __fmul_rn(__fmul_rn(pid, pos_scale), __ldg(inv_freq + f));
    float r1, r2;
    rope_pair(x1, x2, ang, rope_scale, r1, r2);
    __nv_bfloat16 h1, l1, h2, l2;
    split_bf16(r1, h1, l1);
    split_bf16(r2, h2, l2);
    const int64_t o = row * D;
    hi[o + f] = h1;
    lo[o + f] = l1;
    hi[o + f + half] = h2;
    lo[o + f + half] = l2;
  }
}

// Vectorised form: one thread per (row, 8 consecutive frequency pairs): 16-byte loads of the
// 8 first-half and 8 second-half elements, cos / sin from the exact table of the geometry when
// the row's position lies on it (bit-identical to evaluating them), 16-byte stores of the hi /
// lo pieces.  Same arithmetic per element as rope_split_kernel.
template <typename T>
__global__ void rope_split8_kernel(const T* __restrict__ x, int64_t heads, int64_t N, int D,
                                   int64_t stride_h, int64_t stride_n,
                                   const float* __restrict__ inv_freq, float pos_scale,
                                   float rope_scale, __nv_bfloat16* __restrict__ hi,
                                   __nv_bfloat16* __restrict__ lo, int mode, int64_t dca_L,
                                   int64_t dca_s, int64_t pos0, const float2* __restrict__ tab,
                                   float tab_R, int64_t tab_len) {
  const int half = D >> 1;
  const int groups = half >> 3;
  const int64_t total = heads * N * groups;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int f0 = (int)(i % groups) * 8;
    const int64_t row = i / groups;
    const int64_t n = row % N;
    const int64_t h = row / N;
    const T* src = x + h * stride_h + n * stride_n;
    float x1[8], x2[8];
    load8(src + f0, x1);
    load8(src + f0 + half, x2);
    const float pos = __fmul_rn((float)position_id(pos0 + n, mode, dca_L, dca_s), pos_scale);
    const int64_t ti = table_index(pos, tab_R, tab_len);
    __align__(16) __nv_bfloat16 h1[8], l1[8], h2[8], l2[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float r1, r2;
      if (ti >= 0) {
        const float2 cs = __ldg(tab + ti * half + f0 + u);
        r1 = __fsub_rn(__fmul_rn(x1[u], cs.x), __fmul_rn(x2[u], cs.y));
        r2 = __fadd_rn(__fmul_rn(x2[u], cs.x), __fmul_rn(x1[u], cs.y));
      } else {
        const float ang = __fmul_rn(pos, __ldg(inv_freq + f0 + u));
        rope_pair(x1[u], x2[u], ang, rope_scale, r1, r2);
      }
      split_bf16(r1, h1[u], l1[u]);
      split_bf16(r2, h2[u], l2[u]);
    }
    const int64_t o = row * D;
    *reinterpret_cast<uint4*>(hi + o + f0) = *reinterpret_cast<const uint4*>(h1);
    *reinterpret_cast<uint4*>(lo + o + f0) = *reinterpret_cast<const uint4*>(l1);
    *reinterpret_cast<uint4*>(hi + o + f0 + half) = *reinterpret_cast<const uint4*>(h2);
    *reinterpret_cast<uint4*>(lo + o + f0 + half) = *reinterpret_cast<const uint4*>(l2);
  }
}

int launch_rope_split(const void* x, int dtype, int64_t heads, int64_t N, int D,
                      int64_t stride_h, int64_t stride_n, const float* inv_freq,
                      float pos_scale, float rope_scale, void* hi, void* lo,
                      cudaStream_t stream, int mode, int64_t dca_L, int64_t dca_s,
                      int64_t pos0, const void* tab, float tab_R, int64_t tab_len) {
  const int64_t total = heads * N * (D / 2);
  if (total == 0) return 0;
  const int threads = 256;
  const int64_t es = dtype == STA_DTYPE_F32 ? 4 : 2;
  const bool vec = (D % 16) == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(stride_h * es) |
                     (uintptr_t)(stride_n * es) | reinterpret_cast<uintptr_t>(hi) |
                     reinterpret_cast<uintptr_t>(lo)) & 15u) == 0;
  if (vec) {
    int64_t blocks = (total / 8 + threads - 1) / threads;
    if (blocks > 148 * 32) blocks = 148 * 32;
    const float2* t2 = static_cast<const float2*>(tab);
    const int64_t tl = tab ? tab_len : 0;
    if (dtype == STA_DTYPE_F32)
      rope_split8_kernel<float><<<(unsigned)blocks, threads, 0, stream>>>(
          static_cast<const float*>(x), heads, N, D, stride_h, stride_n, inv_freq, pos_scale,
          rope_scale, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), mode,
          dca_L, dca_s, pos0, t2, tab_R, tl);
    else
      rope_split8_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x), heads, N, D, stride_h, stride_n, inv_freq,
          pos_scale, rope_scale, static_cast<__nv_bfloat16*>(hi),
          static_cast<__nv_bfloat16*>(lo), mode, dca_L, dca_s, pos0, t2, tab_R, tl);
    return cudaGetLastError() == cudaSuccess ? 0 : STA_ERR_CUDA;
  }
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (dtype == STA_DTYPE_F32) {
    rope_split_kernel<float><<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const float*>(x), heads, N, D, stride_h, stride_n, inv_freq, pos_scale,
        rope_scale, static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), mode, dca_L,
        dca_s, pos0);
  } else {
    rope_split_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), heads, N, D, stride_h, stride_n, inv_freq,
        pos_scale, rope_scale, static_cast<__nv_bfloat16*>(hi),
        static_cast<__nv_bfloat16*>(lo), mode, dca_L, dca_s, pos0);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : STA_ERR_CUDA;
}

// (cos, sin) * rope_scale at positions i / R, formed exactly like the direct RoPE path
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int half, float rope_scale,
                                  float R, int64_t len, float2* __restrict__ out) {
  const int64_t total = len * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int f = (int)(i % half);
    const float pos = (float)(i / half) / R;
    const float ang = __fmul_rn(pos, __ldg(inv_freq + f));
    float s, c;
    sincosf(ang, &s, &c);
    out[i] = make_float2(__fmul_rn(c, rope_scale), __fmul_rn(s, rope_scale));
  }
}

int launch_rope_table(const float* inv_freq, int D, float rope_scale, float R, int64_t len,
                      void* out, cudaStream_t stream) {
  const int64_t total = len * (D / 2);
  if (total <= 0) return 0;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  rope_table_kernel<<<(unsigned)blocks, 256, 0, stream>>>(inv_freq, D / 2, rope_scale, R, len,
                                                          static_cast<float2*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : STA_ERR_CUDA;
}

}  // namespace sta
