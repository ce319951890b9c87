// Gather + repositioned attention over the selected key slots (Kernel C / C').
//
// Reference: _gather_attn_kernel, shared_selection_triton_exact_2.py:146-225 and
// _gather_attn_pq_kernel, shared_selection_triton_perquery.py:226-312.  Per (head, tile):
//   Q rotated at newpos_q (one position per query), K slot rows gathered by idx and rotated at
//   newpos_k, s = (Qr . Kr) * sm_scale, keep = causal-by-original-position & valid [& mask bit],
//   online softmax over 64-slot blocks with the reference's -inf guard, P rounded to the value
//   dtype before the PV product, out = acc / l.
// Differences in execution only: the slot loop stops at the tile's kept size instead of
// sweeping all k_max slots (padding slots contribute exactly nothing), QK uses the 3xBF16 split
// (fp32-accurate) and an fp32 V uses the split for PV too.
#include "common.cuh"
#include "mma_frag.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int BK = 64;

struct AttendP {
  const void* q;
  int64_t qsh, qsn;
  const void* k;
  int64_t ksh, ksn;
  const void* v;
  int64_t vsh, vsn;
  void* out;
  int64_t BH, N, nt;
  int H, Hkv;
  int k_max;
  const int32_t* idx;
  const float* npk;
  const float* npq;
  const int32_t* mask;
  const int32_t* kept;
  const float* inv_freq;
  float rope_scale, sm_scale;
};

template <typename TV>
__device__ __forceinline__ float ldf(const TV* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <int D, int T, bool F32>
__global__ void __launch_bounds__(T * 2)
gather_attend_kernel(const AttendP p) {
  using TV = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int NW = T / 16;
  constexpr int NTH = NW * 32;
  constexpr int LD = D + 8;  // padded smem row (bf16 elements)
  constexpr int HALF = D / 2;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQh = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sQl = sQh + T * LD;
  __nv_bfloat16* sKh = sQl + T * LD;
  __nv_bfloat16* sKl = sKh + BK * LD;
  __nv_bfloat16* sVh = sKl + BK * LD;
  __nv_bfloat16* sVl = sVh + BK * LD;  // used when F32
  int* sIdx = reinterpret_cast<int*>(sVl + (F32 ? BK * LD : 0));
  float* sNpk = reinterpret_cast<float*>(sIdx + BK);
  int* sMask = reinterpret_cast<int*>(sNpk + BK);

  const int t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int64_t N = p.N;
  const int64_t kvh = (bh / p.H) * p.Hkv + (bh % p.H) / (p.H / p.Hkv);
  const TV* qg = static_cast<const TV*>(p.q) + bh * p.qsh;
  const TV* kg = static_cast<const TV*>(p.k) + kvh * p.ksh;
  const TV* vg = static_cast<const TV*>(p.v) + kvh * p.vsh;
  const int64_t row_base = (bh * p.nt + t);
  const int32_t* idx_row = p.idx + row_base * p.k_max;
  const float* npk_row = p.npk + row_base * p.k_max;
  const float* npq_row = p.npq + row_base * T;
  const int32_t* mask_row = p.mask ? p.mask + row_base * p.k_max : nullptr;

  // ---- Q prologue: rotate at newpos_q, split, stage, load A fragments
  for (int it = tid; it < T * HALF; it += NTH) {
    const int r = it / HALF, f = it % HALF;
    const int64_t qp = (int64_t)t * T + r;
    float x1 = 0.f, x2 = 0.f;
    if (qp < N) {
      x1 = ldf(qg + qp * p.qsn + f);
      x2 = ldf(qg + qp * p.qsn + f + HALF);
    }
    const float ang = __fmul_rn(npq_row[r], __ldg(p.inv_freq + f));
    float r1, r2;
    rope_pair(x1, x2, ang, p.rope_scale, r1, r2);
    __nv_bfloat16 h1, l1, h2, l2;
    split_bf16(r1, h1, l1);
    split_bf16(r2, h2, l2);
    sQh[r * LD + f] = h1;
    sQl[r * LD + f] = l1;
    sQh[r * LD + f + HALF] = h2;
    sQl[r * LD + f + HALF] = l2;
  }
  __syncthreads();
  uint32_t qa_h[D / 16][4], qa_l[D / 16][4];
  {
    const int mi = lane >> 3;
    const int r = warp * 16 + (lane & 7) + (mi & 1) * 8;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int col = ks * 16 + (mi >> 1) * 8;
      ldsm_x4(smem_u32(sQh + r * LD + col), qa_h[ks][0], qa_h[ks][1], qa_h[ks][2], qa_h[ks][3]);
      ldsm_x4(smem_u32(sQl + r * LD + col), qa_l[ks][0], qa_l[ks][1], qa_l[ks][2], qa_l[ks][3]);
    }
  }

  const int ra = warp * 16 + g, rb = ra + 8;  // tile-local rows of this thread
  const int64_t qpa = (int64_t)t * T + ra, qpb = (int64_t)t * T + rb;
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  int nslots = p.k_max;
  if (p.kept) {
    const int ks = p.kept[row_base];
    nslots = ks < p.k_max ? ks : p.k_max;
  }
  for (int s0 = 0; s0 < nslots; s0 += BK) {
    __syncthreads();
    for (int i = tid; i < BK; i += NTH) {
      const int slot = s0 + i;
      int id = (int)N;
      float np = 0.f;
      int mk = -1;
      if (slot < p.k_max) {
        id = idx_row[slot];
        if (id < N) np = npk_row[slot];
        if (mask_row) mk = mask_row[slot];
      }
      sIdx[i] = id;
      sNpk[i] = np;
      sMask[i] = mk;
    }
    __syncthreads();
    // gather + rotate K, gather V
    for (int it = tid; it < BK * HALF; it += NTH) {
      const int i = it / HALF, f = it % HALF;
      const int id = sIdx[i];
      float x1 = 0.f, x2 = 0.f;
      if (id < N) {
        x1 = ldf(kg + (int64_t)id * p.ksn + f);
        x2 = ldf(kg + (int64_t)id * p.ksn + f + HALF);
      }
      const float ang = __fmul_rn(sNpk[i], __ldg(p.inv_freq + f));
      float r1, r2;
      rope_pair(x1, x2, ang, p.rope_scale, r1, r2);
      __nv_bfloat16 h1, l1, h2, l2;
      split_bf16(r1, h1, l1);
      split_bf16(r2, h2, l2);
      sKh[i * LD + f] = h1;
      sKl[i * LD + f] = l1;
      sKh[i * LD + f + HALF] = h2;
      sKl[i * LD + f + HALF] = l2;
    }
    for (int it = tid; it < BK * D; it += NTH) {
      const int i = it / D, d = it % D;
      const int id = sIdx[i];
      const float x = id < N ? ldf(vg + (int64_t)id * p.vsn + d) : 0.f;
      if (F32) {
        __nv_bfloat16 h, l;
        split_bf16(x, h, l);
        sVh[i * LD + d] = h;
        sVl[i * LD + d] = l;
      } else {
        sVh[i * LD + d] = __float2bfloat16_rn(x);
      }
    }
    __syncthreads();

    float s[BK / 8][4];
#pragma unroll
    for (int i = 0; i < BK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    {
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
        for (int np2 = 0; np2 < BK / 16; ++np2) {
          const int row = (2 * np2 + (mi >> 1)) * 8 + rr;
          const int col = ks * 16 + (mi & 1) * 8;
          uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
          ldsm_x4(smem_u32(sKh + row * LD + col), h0, h1, h2, h3);
          ldsm_x4(smem_u32(sKl + row * LD + col), l0, l1, l2, l3);
          mma_bf16(s[2 * np2], qa_h[ks], h0, h1);
          mma_bf16(s[2 * np2], qa_h[ks], l0, l1);
          mma_bf16(s[2 * np2], qa_l[ks], h0, h1);
          mma_bf16(s[2 * np2 + 1], qa_h[ks], h2, h3);
          mma_bf16(s[2 * np2 + 1], qa_h[ks], l2, l3);
          mma_bf16(s[2 * np2 + 1], qa_l[ks], h2, h3);
        }
      }
    }
    // scale + mask, row max
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BK / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = nt * 8 + 2 * c4 + (e & 1);
        const int row = e < 2 ? ra : rb;
        const int64_t qp = e < 2 ? qpa : qpb;
        const int id = sIdx[col];
        const bool keep = id < N && qp >= id && ((sMask[col] >> row) & 1);
        const float v = keep ? __fmul_rn(s[nt][e], p.sm_scale) : -INFINITY;
        s[nt][e] = v;
        if (e < 2) mxA = fmaxf(mxA, v);
        else mxB = fmaxf(mxB, v);
      }
    }
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
    const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
    const float msA = mnA == -INFINITY ? 0.f : mnA;
    const float msB = mnB == -INFINITY ? 0.f : mnB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int nt = 0; nt < BK / 8; ++nt) {
      s[nt][0] = expf(__fsub_rn(s[nt][0], msA));
      s[nt][1] = expf(__fsub_rn(s[nt][1], msA));
      s[nt][2] = expf(__fsub_rn(s[nt][2], msB));
      s[nt][3] = expf(__fsub_rn(s[nt][3], msB));
      sumA += s[nt][0] + s[nt][1];
      sumB += s[nt][2] + s[nt][3];
    }
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
    sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
    sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
    const float alA = expf(__fsub_rn(mA, msA)), alB = expf(__fsub_rn(mB, msB));
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alA;
      o[i][1] *= alA;
      o[i][2] *= alB;
      o[i][3] *= alB;
    }
    mA = mnA;
    mB = mnB;
    // PV
    {
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        uint32_t ph[4], pl[4];
        if (F32) {
          pack_split(s[2 * kk][0], s[2 * kk][1], ph[0], pl[0]);
          pack_split(s[2 * kk][2], s[2 * kk][3], ph[1], pl[1]);
          pack_split(s[2 * kk + 1][0], s[2 * kk + 1][1], ph[2], pl[2]);
          pack_split(s[2 * kk + 1][2], s[2 * kk + 1][3], ph[3], pl[3]);
        } else {
          ph[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
          ph[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
          ph[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
          ph[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
        }
        const int row = kk * 16 + rr + (mi & 1) * 8;
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          const int col = (2 * dp + (mi >> 1)) * 8;
          uint32_t v0, v1, v2, v3;
          ldsm_x4_t(smem_u32(sVh + row * LD + col), v0, v1, v2, v3);
          mma_bf16(o[2 * dp], ph, v0, v1);
          mma_bf16(o[2 * dp + 1], ph, v2, v3);
          if (F32) {
            uint32_t w0, w1, w2, w3;
            ldsm_x4_t(smem_u32(sVl + row * LD + col), w0, w1, w2, w3);
            mma_bf16(o[2 * dp], ph, w0, w1);
            mma_bf16(o[2 * dp + 1], ph, w2, w3);
            mma_bf16(o[2 * dp], pl, v0, v1);
            mma_bf16(o[2 * dp + 1], pl, v2, v3);
          }
        }
      }
    }
  }

  // ---- epilogue
  TV* og = static_cast<TV*>(p.out) + bh * N * D;
  const float iA = 1.f / lA, iB = 1.f / lB;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int col = dt * 8 + 2 * c4;
    if (qpa < N) {
      if (F32) {
        reinterpret_cast<float2*>(og + qpa * D + col)[0] = make_float2(o[dt][0] / lA, o[dt][1] / lA);
      } else {
        reinterpret_cast<__nv_bfloat162*>(og + qpa * D + col)[0] =
            __floats2bfloat162_rn(o[dt][0] / lA, o[dt][1] / lA);
      }
    }
    if (qpb < N) {
      if (F32) {
        reinterpret_cast<float2*>(og + qpb * D + col)[0] = make_float2(o[dt][2] / lB, o[dt][3] / lB);
      } else {
        reinterpret_cast<__nv_bfloat162*>(og + qpb * D + col)[0] =
            __floats2bfloat162_rn(o[dt][2] / lB, o[dt][3] / lB);
      }
    }
  }
  (void)iA;
  (void)iB;
}

template <int D, int T, bool F32>
int launch_one(const AttendP& p, cudaStream_t stream) {
  constexpr int LD = D + 8;
  const size_t smem = (size_t)(2 * T * LD + 2 * BK * LD + (F32 ? 2 : 1) * BK * LD) * 2 + 3 * BK * 4;
  auto kern = gather_attend_kernel<D, T, F32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  dim3 grid((unsigned)p.nt, (unsigned)p.BH);
  kern<<<grid, T * 2, smem, stream>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace

int launch_gather_attend(const sta_attend_args* a, cudaStream_t stream) {
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->idx || !a->newpos_k || !a->newpos_q ||
      !a->inv_freq)
    return fail(STA_ERR_ARG, "sta_gather_attend: null pointer");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_gather_attend: d must be 64 or 128");
  if (a->tile != 32 && a->tile != 64) return fail(STA_ERR_UNSUPPORTED, "sta_gather_attend: tile must be 32 or 64");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_gather_attend: bad head counts");
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  AttendP p;
  p.q = a->q; p.qsh = a->q_stride_h; p.qsn = a->q_stride_n;
  p.k = a->k; p.ksh = a->k_stride_h; p.ksn = a->k_stride_n;
  p.v = a->v; p.vsh = a->v_stride_h; p.vsn = a->v_stride_n;
  p.out = a->out;
  p.BH = a->batch * a->n_heads;
  p.N = a->n;
  p.nt = (a->n + a->tile - 1) / a->tile;
  p.H = (int)a->n_heads;
  p.Hkv = (int)a->n_kv_heads;
  p.k_max = a->k_max;
  p.idx = a->idx;
  p.npk = a->newpos_k;
  p.npq = a->newpos_q;
  p.mask = a->mask;
  p.kept = a->kept_size;
  p.inv_freq = a->inv_freq;
  p.rope_scale = a->rope_scale;
  p.sm_scale = a->sm_scale;
  if (p.BH > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_gather_attend: too many heads");
  const bool f32 = a->dtype == STA_DTYPE_F32;
  if (a->d == 128) {
    if (a->tile == 64) return f32 ? launch_one<128, 64, true>(p, stream) : launch_one<128, 64, false>(p, stream);
    return f32 ? launch_one<128, 32, true>(p, stream) : launch_one<128, 32, false>(p, stream);
  }
  if (a->tile == 64) return f32 ? launch_one<64, 64, true>(p, stream) : launch_one<64, 64, false>(p, stream);
  return f32 ? launch_one<64, 32, true>(p, stream) : launch_one<64, 32, false>(p, stream);
}

}  // namespace sta
