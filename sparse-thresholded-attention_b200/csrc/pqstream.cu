// PQ-Stream, pass 2: per-query threshold selection with streamed block positions, fused with
// the attention over the kept keys.
//
// Reference: _pqstream_kernel, pqstream_kernel.py:174-368 (pass 2 is :251-358).  Pass 1 (exact
// row max under the selection geometry) is sta_select(max_only=1) on the tensor cores; this
// kernel reads its row maxima.  Per (head, 32-query tile), key blocks of block_n are visited in
// DESCENDING order; for each block:
//   s_sel = (Qsel . Ksel) * sm_scale   (selection geometry, pre-rotated hi/lo operands)
//   keep  = (s_sel >= m - tau | forced) & causal & row < N & key < N
//   c_i   = sum_j keep ; adv = max_i c_i (or the block's occupied slot count, ADV_FULL)
//   if adv > 0 (or skipping disabled): keys rotated with base RoPE at npk = -(d + o_j),
//     o_j = hi_t - j, queries at npq = qpos - P_top; online softmax + PV; d += adv.
// Outputs: out, span (= final d), kept (per-query kept count), blocks, skipped.
#include "common.cuh"
#include "mma_frag.cuh"
#include "gather_rope.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int T = 32;      // query tile (fixed by the reference's bit packing convention)
constexpr int NW = 2;      // warps (16 query rows each)
constexpr int NTH = 64;

struct PQSP {
  const void* q;
  int64_t qsh, qsn;
  const void* k;
  int64_t ksh, ksn;
  const void* v;
  int64_t vsh, vsn;
  void* out;
  int64_t BH, N, nt;
  int64_t qbase, Nq;  // queries: positions qbase .. N-1, held as rows 0 .. Nq-1
  int H, Hkv;
  const __nv_bfloat16 *qh, *ql, *kh, *kl;
  const float* row_max;
  const float* tau;
  int n_global, n_local;
  const float* inv_freq_c;
  float sm_scale;
  int adv_full, use_skip;
  const float2* rtab;
  float rtab_R;
  int64_t rtab_len;
  float* span;
  int32_t* kept;
  float* blocks;
  float* skipped;
};

template <typename TV>
__device__ __forceinline__ float ldv(const TV* p);
template <>
__device__ __forceinline__ float ldv<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldv<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// s (16 rows of this warp x BN keys) = sum of piece products of A [NP][T][LD] and B [NP][BN][LD]
template <int D, int BN, int NP>
__device__ __forceinline__ void score_tile(const __nv_bfloat16* sA, const __nv_bfloat16* sB,
                                           float (&s)[BN / 8][4]) {
  constexpr int LD = D + 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    uint32_t a[NP][4];
    const int ar = warp * 16 + rr + (mi & 1) * 8;
    const int ac = ks * 16 + (mi >> 1) * 8;
#pragma unroll
    for (int j = 0; j < NP; ++j)
      ldsm_x4(smem_u32(sA + (j * T + ar) * LD + ac), a[j][0], a[j][1], a[j][2], a[j][3]);
#pragma unroll
    for (int np2 = 0; np2 < BN / 16; ++np2) {
      const int row = (2 * np2 + (mi >> 1)) * 8 + rr;
      const int col = ks * 16 + (mi & 1) * 8;
      uint32_t b0[NP][2], b1[NP][2];
#pragma unroll
      for (int j = 0; j < NP; ++j)
        ldsm_x4(smem_u32(sB + (j * BN + row) * LD + col), b0[j][0], b0[j][1], b1[j][0], b1[j][1]);
      mma_pieces<NP>(s[2 * np2], a, b0);
      mma_pieces<NP>(s[2 * np2 + 1], a, b1);
    }
  }
}

template <int D, int BN, bool F32>
__global__ void __launch_bounds__(NTH) pqstream_kernel(const PQSP p) {
  using TV = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int LD = D + 8;
  constexpr int HALF = D / 2;
  constexpr int NQ = F32 ? 3 : 2;  // pieces of the attend-geometry Q / K
  constexpr int NV = F32 ? 3 : 1;  // pieces of P / V
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQs = reinterpret_cast<__nv_bfloat16*>(smem);  // [2][T][LD] select geometry
  __nv_bfloat16* sQa = sQs + 2 * T * LD;                         // [NQ][T][LD] attend geometry
  __nv_bfloat16* sKs = sQa + NQ * T * LD;                        // [2][BN][LD]
  __nv_bfloat16* sKa = sKs + 2 * BN * LD;                        // [NQ][BN][LD]
  __nv_bfloat16* sV = sKa + NQ * BN * LD;                        // [NV][BN][LD]
  __shared__ int s_cmax[NW];

  const int t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int64_t N = p.N;
  const int64_t kvh = (bh / p.H) * p.Hkv + (bh % p.H) / (p.H / p.Hkv);
  const TV* qg = static_cast<const TV*>(p.q) + bh * p.qsh;
  const TV* kg = static_cast<const TV*>(p.k) + kvh * p.ksh;
  const TV* vg = static_cast<const TV*>(p.v) + kvh * p.vsh;
  const __nv_bfloat16* qhg = p.qh + bh * p.Nq * D;
  const __nv_bfloat16* qlg = p.ql + bh * p.Nq * D;
  const __nv_bfloat16* khg = p.kh + kvh * N * D;
  const __nv_bfloat16* klg = p.kl + kvh * N * D;

  const int64_t tstart = p.qbase + (int64_t)t * T;  // absolute position of the tile's first query
  const int64_t P_top = min(tstart + T - 1, N - 1);
  const int64_t hi = P_top + 1;
  const int nblk = (int)((hi + BN - 1) / BN);
  const float tau = __ldg(p.tau + (bh % p.H));
  const int64_t loc_lo = tstart - p.n_local + 1, loc_hi = tstart + T - 1;

  // ---- prologue: Q in both geometries
  for (int it = tid; it < T * D; it += NTH) {
    const int r = it / D, d = it % D;
    const int64_t qp = tstart + r;
    const int64_t ql = qp - p.qbase;
    __nv_bfloat16 zh = __float2bfloat16_rn(0.f);
    sQs[r * LD + d] = qp < N ? qhg[ql * D + d] : zh;
    sQs[(T + r) * LD + d] = qp < N ? qlg[ql * D + d] : zh;
  }
  for (int it = tid; it < T * HALF; it += NTH) {
    const int r = it / HALF, f = it % HALF;
    const int64_t qp = tstart + r;
    float x1 = 0.f, x2 = 0.f;
    if (qp < N) {
      x1 = ldv(qg + (qp - p.qbase) * p.qsn + f);
      x2 = ldv(qg + (qp - p.qbase) * p.qsn + f + HALF);
    }
    const float npq = (float)(qp - P_top);
    float r1, r2;
    const int64_t ti = table_index(npq, p.rtab_R, p.rtab_len);
    if (ti >= 0) {
      const float2 cs = __ldg(p.rtab + ti * HALF + f);
      r1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
      r2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
    } else {
      const float ang = __fmul_rn(npq, __ldg(p.inv_freq_c + f));
      rope_pair(x1, x2, ang, 1.f, r1, r2);
    }
    __nv_bfloat16 a[NQ], b[NQ];
    split_pieces<NQ>(r1, a);
    split_pieces<NQ>(r2, b);
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
      sQa[(j * T + r) * LD + f] = a[j];
      sQa[(j * T + r) * LD + f + HALF] = b[j];
    }
  }

  const int ra = warp * 16 + g, rb = ra + 8;
  const int64_t qpa = tstart + ra, qpb = tstart + rb;
  const bool okA = qpa < N, okB = qpb < N;
  const int64_t ra_l = qpa - p.qbase, rb_l = qpb - p.qbase;  // slab rows
  const float thrA = okA ? __fsub_rn(p.row_max[bh * p.Nq + ra_l], tau) : INFINITY;
  const float thrB = okB ? __fsub_rn(p.row_max[bh * p.Nq + rb_l], tau) : INFINITY;

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  int keptA = 0, keptB = 0;
  float dpos = 0.f;
  int n_used = 0;

  for (int tb = 0; tb < nblk; ++tb) {
    const int64_t sn = (int64_t)(nblk - 1 - tb) * BN;
    const int64_t hi_t = min(P_top, sn + BN - 1);
    __syncthreads();
    // phase 1: selection-geometry K (hi/lo) of the block
    for (int it = tid; it < BN * (D / 8); it += NTH) {
      const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
      const int64_t j = sn + i;
      uint4 h = make_uint4(0u, 0u, 0u, 0u), l = h;
      if (j < N) {
        h = *reinterpret_cast<const uint4*>(khg + j * D + d0);
        l = *reinterpret_cast<const uint4*>(klg + j * D + d0);
      }
      *reinterpret_cast<uint4*>(sKs + i * LD + d0) = h;
      *reinterpret_cast<uint4*>(sKs + (BN + i) * LD + d0) = l;
    }
    __syncthreads();

    // selection scores and keep mask
    float s[BN / 8][4];
    score_tile<D, BN, 2>(sQs, sKs, s);
    uint32_t keepbits[BN / 8];
    int cA = 0, cB = 0;
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
      uint32_t kb = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t j = sn + nt * 8 + 2 * c4 + (e & 1);
        const int64_t qp = e < 2 ? qpa : qpb;
        const bool rok = e < 2 ? okA : okB;
        const float thr = e < 2 ? thrA : thrB;
        const bool forced = j < p.n_global || (j >= loc_lo && j <= loc_hi);
        const float sc = __fmul_rn(s[nt][e], p.sm_scale);
        const bool keep = (sc >= thr || forced) && qp >= j && rok && j < N;
        kb |= (keep ? 1u : 0u) << e;
        if (keep) {
          if (e < 2) ++cA;
          else ++cB;
        }
      }
      keepbits[nt] = kb;
    }
    cA += __shfl_xor_sync(0xffffffffu, cA, 1);
    cA += __shfl_xor_sync(0xffffffffu, cA, 2);
    cB += __shfl_xor_sync(0xffffffffu, cB, 1);
    cB += __shfl_xor_sync(0xffffffffu, cB, 2);
    int cm = max(cA, cB);
#pragma unroll
    for (int o2 = 4; o2 < 32; o2 <<= 1) cm = max(cm, __shfl_xor_sync(0xffffffffu, cm, o2));
    if (lane == 0) s_cmax[warp] = cm;
    __syncthreads();
    int cmax = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) cmax = max(cmax, s_cmax[w]);
    const float adv = p.adv_full ? (float)(hi_t - sn + 1) : (float)cmax;
    if (p.use_skip && !(adv > 0.f)) continue;

    // phase 2 (used blocks only): raw K rotated at the streamed positions, and V
    for (int it = tid; it < BN * (HALF / 8); it += NTH) {
      const int i = it / (HALF / 8), f0 = (it % (HALF / 8)) * 8;
      const int64_t j = sn + i;
      const float npk = -__fadd_rn(dpos, (float)(hi_t - j));
      rotate8<NQ, HALF>(kg + (j < N ? j : 0) * p.ksn, j < N, f0, npk, p.inv_freq_c, 1.f,
                        sKa + i * LD, BN * LD, p.rtab, table_index(npk, p.rtab_R, p.rtab_len));
    }
    for (int it = tid; it < BN * (D / 8); it += NTH) {
      const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
      const int64_t j = sn + i;
      __nv_bfloat16* dst = sV + i * LD + d0;
      if (!F32) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (j < N) u = *reinterpret_cast<const uint4*>(vg + j * p.vsn + d0);
        *reinterpret_cast<uint4*>(dst) = u;
      } else {
        float x[8];
        if (j < N) {
          load8(vg + j * p.vsn + d0, x);
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u) x[u] = 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          __nv_bfloat16 pc[NV];
          split_pieces<NV>(x[u], pc);
#pragma unroll
          for (int q2 = 0; q2 < NV; ++q2) dst[q2 * BN * LD + u] = pc[q2];
        }
      }
    }
    __syncthreads();

    // attend scores at the streamed positions
    score_tile<D, BN, NQ>(sQa, sKa, s);
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool keep = (keepbits[nt] >> e) & 1u;
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
    for (int nt = 0; nt < BN / 8; ++nt) {
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
    {
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t pp[NV][4];
        {
          uint32_t x0[NV], x1[NV], x2[NV], x3[NV];
          pack_pieces<NV>(s[2 * kk][0], s[2 * kk][1], x0);
          pack_pieces<NV>(s[2 * kk][2], s[2 * kk][3], x1);
          pack_pieces<NV>(s[2 * kk + 1][0], s[2 * kk + 1][1], x2);
          pack_pieces<NV>(s[2 * kk + 1][2], s[2 * kk + 1][3], x3);
#pragma unroll
          for (int j = 0; j < NV; ++j) {
            pp[j][0] = x0[j];
            pp[j][1] = x1[j];
            pp[j][2] = x2[j];
            pp[j][3] = x3[j];
          }
        }
        const int row = kk * 16 + rr + (mi & 1) * 8;
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          const int col = (2 * dp + (mi >> 1)) * 8;
          uint32_t v0[NV][2], v1[NV][2];
#pragma unroll
          for (int j = 0; j < NV; ++j)
            ldsm_x4_t(smem_u32(sV + (j * BN + row) * LD + col), v0[j][0], v0[j][1], v1[j][0], v1[j][1]);
          mma_pieces<NV>(o[2 * dp], pp, v0);
          mma_pieces<NV>(o[2 * dp + 1], pp, v1);
        }
      }
    }
    keptA += cA;
    keptB += cB;
    dpos = __fadd_rn(dpos, adv);
    ++n_used;
  }

  TV* og = static_cast<TV*>(p.out) + bh * p.Nq * D;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int col = dt * 8 + 2 * c4;
    if (okA) {
      if (F32)
        reinterpret_cast<float2*>(og + ra_l * D + col)[0] = make_float2(o[dt][0] / lA, o[dt][1] / lA);
      else
        reinterpret_cast<__nv_bfloat162*>(og + ra_l * D + col)[0] =
            __floats2bfloat162_rn(o[dt][0] / lA, o[dt][1] / lA);
    }
    if (okB) {
      if (F32)
        reinterpret_cast<float2*>(og + rb_l * D + col)[0] = make_float2(o[dt][2] / lB, o[dt][3] / lB);
      else
        reinterpret_cast<__nv_bfloat162*>(og + rb_l * D + col)[0] =
            __floats2bfloat162_rn(o[dt][2] / lB, o[dt][3] / lB);
    }
  }
  if (c4 == 0) {
    if (okA) p.kept[bh * p.Nq + ra_l] = keptA;
    if (okB) p.kept[bh * p.Nq + rb_l] = keptB;
  }
  if (tid == 0) {
    const int64_t o2 = bh * p.nt + t;
    p.span[o2] = dpos;
    p.blocks[o2] = (float)nblk;
    p.skipped[o2] = (float)(nblk - n_used);
  }
}

template <int D, int BN, bool F32>
int launch_one(const PQSP& p, cudaStream_t stream) {
  constexpr int LD = D + 8;
  constexpr int NQ = F32 ? 3 : 2, NV = F32 ? 3 : 1;
  const size_t smem = (size_t)((2 + NQ) * T * LD + (2 + NQ + NV) * BN * LD) * 2;
  auto kern = pqstream_kernel<D, BN, F32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  dim3 grid((unsigned)p.nt, (unsigned)p.BH);
  kern<<<grid, NTH, smem, stream>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace

int launch_pqstream(const sta_pqstream_args* a, cudaStream_t stream) {
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->q_hi || !a->q_lo || !a->k_hi || !a->k_lo ||
      !a->row_max || !a->tau || !a->inv_freq_c || !a->span || !a->kept || !a->blocks || !a->skipped)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: null pointer");
  if (a->tile != 32) return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: tile must be 32");
  if (a->block_n != 32 && a->block_n != 64)
    return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: block_n must be 32 or 64");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: d must be 64 or 128");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: bad head counts");
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  {
    const int64_t es = a->dtype == STA_DTYPE_F32 ? 4 : 2;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                         reinterpret_cast<uintptr_t>(a->v);
    const int64_t st = (a->q_stride_h | a->q_stride_n | a->k_stride_h | a->k_stride_n |
                        a->v_stride_h | a->v_stride_n) * es;
    if ((al & 15u) || (st & 15))
      return fail(STA_ERR_UNSUPPORTED,
                  "sta_pqstream_attend: q/k/v rows must start on 16-byte boundaries");
  }
  PQSP p;
  p.q = a->q; p.qsh = a->q_stride_h; p.qsn = a->q_stride_n;
  p.k = a->k; p.ksh = a->k_stride_h; p.ksn = a->k_stride_n;
  p.v = a->v; p.vsh = a->v_stride_h; p.vsn = a->v_stride_n;
  p.out = a->out;
  p.BH = a->batch * a->n_heads;
  p.N = a->n;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: q_pos_base outside [0, n)");
  p.qbase = a->q_pos_base;
  p.Nq = a->n - a->q_pos_base;
  p.nt = (p.Nq + T - 1) / T;
  p.H = (int)a->n_heads;
  p.Hkv = (int)a->n_kv_heads;
  p.qh = static_cast<const __nv_bfloat16*>(a->q_hi);
  p.ql = static_cast<const __nv_bfloat16*>(a->q_lo);
  p.kh = static_cast<const __nv_bfloat16*>(a->k_hi);
  p.kl = static_cast<const __nv_bfloat16*>(a->k_lo);
  p.row_max = a->row_max;
  p.tau = a->tau;
  p.n_global = a->n_global;
  p.n_local = a->n_local;
  p.inv_freq_c = a->inv_freq_c;
  p.sm_scale = a->sm_scale;
  p.adv_full = a->pos_advance == STA_ADV_FULL;
  p.use_skip = a->use_skip;
  p.rtab = static_cast<const float2*>(a->rope_table);
  p.rtab_R = a->rope_table_R;
  p.rtab_len = a->rope_table ? a->rope_table_len : 0;
  p.span = a->span;
  p.kept = a->kept;
  p.blocks = a->blocks;
  p.skipped = a->skipped;
  if (p.BH > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: too many heads");
  const bool f32 = a->dtype == STA_DTYPE_F32;
  if (a->d == 128) {
    if (a->block_n == 64) return f32 ? launch_one<128, 64, true>(p, stream) : launch_one<128, 64, false>(p, stream);
    return f32 ? launch_one<128, 32, true>(p, stream) : launch_one<128, 32, false>(p, stream);
  }
  if (a->block_n == 64) return f32 ? launch_one<64, 64, true>(p, stream) : launch_one<64, 64, false>(p, stream);
  return f32 ? launch_one<64, 32, true>(p, stream) : launch_one<64, 32, false>(p, stream);
}

}  // namespace sta
