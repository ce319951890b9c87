// PQ-Stream, pass 2: streamed block positions and the attention over the kept keys.
//
// Reference: _pqstream_kernel, pqstream_kernel.py:174-368 (pass 2 is :251-358).  The reference
// rescores every causal key block of every 32-query tile inside the streaming loop.  Here the
// keep decisions come from the tensor-core Kernel A (sta_select, 2 passes, per-query keep bits
// of each (tile, key) -- the same exact-max threshold test), and this kernel only streams:
// per (head, 32-query tile), key blocks of block_n are taken in DESCENDING order and
//   keep  = (bit | forced) & causal & row < N & key < N
//   c_i   = sum_j keep ; adv = max_i c_i (or the block's occupied slot count, ADV_FULL)
//   d_b   = sum of adv over the blocks above b (exact: integers in fp32)
// then the blocks holding any kept key are attended in the same order: keys rotated with base
// RoPE at npk = -(d_b + o_j), o_j = hi_t - j, queries at npq = qpos - P_top; online softmax +
// PV.  Blocks without kept keys change no softmax state, so visiting only the blocks with keeps
// is exact; the skip rule (adv == 0) only decides the `skipped` statistic and d.
// Outputs: out, span (= final d), kept (per-query kept count), blocks, skipped.
#include "common.cuh"
#include "mma_frag.cuh"
#include "gather_rope.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int T = 32;      // query tile (fixed by the reference's bit packing convention)
constexpr int NW = 4;      // warps: two pairs, each pair covers the tile's 32 rows (16 per warp)
constexpr int NTH = NW * 32;
constexpr int SP = 32;     // key slots a warp pair scores per batch
constexpr int SB = 2 * SP; // key slots per batch

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
  const uint32_t* bits;
  int64_t head_stride;       // compact bits
  const uint8_t* bmax;
  int64_t bmax_stride;       // compact block maxima (entries of 32 keys)
  const int32_t* row_count;
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
                                           float (&s)[BN / 8][4], int warp) {
  constexpr int LD = D + 8;
  const int lane = threadIdx.x & 31;
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

// exclusive prefix sum over the CTA's NTH threads (2 warps); total returned in `total`
__device__ __forceinline__ int cta_excl_sum(int x, int* sh, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sh[w] = inc;
  __syncthreads();
  int base = 0;
  total = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    if (i < w) base += sh[i];
    total += sh[i];
  }
  __syncthreads();
  return base + inc - x;
}

template <int D, int BN, bool F32>
__global__ void __launch_bounds__(NTH) pqstream_kernel(const PQSP p) {
  using TV = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int LD = D + 8;
  constexpr int HALF = D / 2;
  constexpr int NQ = F32 ? 3 : 2;  // pieces of the attend-geometry Q / K
  constexpr int NV = F32 ? 3 : 1;  // pieces of P / V
  constexpr int KBUF = NQ * SP * LD, VBUF = NV * SP * LD;
  constexpr int NH = BN / 32;      // 32-key words per block
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQa = reinterpret_cast<__nv_bfloat16*>(smem);   // [NQ][T][LD]
  __nv_bfloat16* sKa = sQa + NQ * T * LD;                         // [2 pairs][NQ][SP][LD]
  __nv_bfloat16* sV = sKa + 2 * KBUF;                             // [2 pairs][NV][SP][LD]
  int* s_fcm = reinterpret_cast<int*>(sV + 2 * VBUF);             // forced blocks' max_i c_i
  __shared__ int s_list[NTH];            // blocks with keeps of the current chunk (descending)
  __shared__ float s_dl[NTH];            // their streamed offset d
  __shared__ uint32_t s_bm[NTH][NH];     // their keys kept by some query (bit per key)
  __shared__ int s_bo[NTH];              // exclusive prefix of their kept-key counts
  __shared__ int s_sj[SB];               // pending slots: key, position, per-query keep bits
  __shared__ float s_sp[SB];
  __shared__ uint32_t s_scw[SB];
  __shared__ int s_extra[T];
  __shared__ int s_red[NW];
  __shared__ float s_ml[T][2];

  const int t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pair = warp >> 1, rw = warp & 1;
  const int g = lane >> 2, c4 = lane & 3;
  const int64_t N = p.N;
  const int64_t kvh = (bh / p.H) * p.Hkv + (bh % p.H) / (p.H / p.Hkv);
  const TV* qg = static_cast<const TV*>(p.q) + bh * p.qsh;
  const TV* kg = static_cast<const TV*>(p.k) + kvh * p.ksh;
  const TV* vg = static_cast<const TV*>(p.v) + kvh * p.vsh;

  const int64_t tstart = p.qbase + (int64_t)t * T;  // absolute position of the tile's first query
  const int64_t P_top = min(tstart + T - 1, N - 1);
  const int64_t hi = P_top + 1;
  const int nblk = (int)((hi + BN - 1) / BN);
  const int nrows = (int)(hi - tstart);
  const uint32_t rowvalid = nrows >= 32 ? 0xffffffffu : ((1u << nrows) - 1u);
  const int64_t loc_lo = tstart - p.n_local + 1, loc_hi = tstart + T - 1;
  const uint32_t* bits_row = p.bits + bh * p.head_stride + tri_tile_offset(t, T, p.qbase);
  const uint8_t* bmax_row = p.bmax + bh * p.bmax_stride + tri_tile_offset(t, 1, p.qbase / 32);

  // keep bits (bit r = query row r) of key j: Kernel A's threshold decisions OR the forced keys
  // (global prefix, local window), restricted to causal, real rows
  auto forced_rows = [&](int64_t j) -> uint32_t {
    if (!(j < p.n_global || (j >= loc_lo && j <= loc_hi))) return 0u;
    const int64_t dl = j - tstart;
    const uint32_t causal = dl <= 0 ? 0xffffffffu : (dl >= 32 ? 0u : ~((1u << dl) - 1u));
    return causal & rowvalid;
  };
  auto keep_word = [&](int64_t j) -> uint32_t {
    return (j <= P_top ? __ldg(bits_row + j) : 0u) | forced_rows(j);
  };
  // forced blocks: [0, ng_blk) and [lb0, nblk); slot f of s_fcm
  const int ng_blk = (int)min((int64_t)nblk, ((int64_t)max(p.n_global, 0) + BN - 1) / BN);
  const int lb0 = (int)min((int64_t)nblk, (loc_lo > 0 ? loc_lo : 0) / BN);
  const int nf_g = min(ng_blk, lb0);
  const int nfs = nf_g + (nblk - lb0);

  // ---- phase 1: exact max_i c_i of the forced blocks (Kernel A's keeps OR the forced keys)
  for (int i = tid; i < T; i += NTH) s_extra[i] = 0;
  __syncthreads();
  int extra = 0;  // lane r: forced keys of row r that Kernel A's threshold did not keep
  for (int f = warp; f < nfs; f += NW) {
    const int b = f < nf_g ? f : lb0 + (f - nf_g);
    int cf = 0, cn = 0;
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const int64_t j = (int64_t)b * BN + h * 32 + lane;
      const uint32_t w = j <= P_top ? bits_row[j] : 0u;
      cn += __popc(transpose32(w));
      cf += __popc(transpose32(w | forced_rows(j)));
    }
    extra += cf - cn;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) cf = max(cf, __shfl_xor_sync(0xffffffffu, cf, o));
    if (lane == 0) s_fcm[f] = cf;
  }
  atomicAdd(&s_extra[lane], extra);

  // ---- Q at the streamed query positions (attend geometry)
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
    __nv_bfloat16 a[NQ], b2[NQ];
    split_pieces<NQ>(r1, a);
    split_pieces<NQ>(r2, b2);
#pragma unroll
    for (int j = 0; j < NQ; ++j) {
      sQa[(j * T + r) * LD + f] = a[j];
      sQa[(j * T + r) * LD + f + HALF] = b2[j];
    }
  }
  __syncthreads();

  const int ra = rw * 16 + g, rb = ra + 8;  // tile rows of this thread's fragments
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  __nv_bfloat16* myK = sKa + pair * KBUF;
  __nv_bfloat16* myV = sV + pair * VBUF;

  // attend one batch of SB pending slots (fewer at the end: the rest are padding, masked):
  // every thread stages rotated K / V, then pair p scores slots [SP*p, SP*p + SP) for all rows
  auto attend_batch = [&](int nb) {
    if (!F32) {
      // V rows need no transform: asynchronous copies overlap the K rotations below
      for (int it = tid; it < SB * (D / 8); it += NTH) {
        const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
        const int64_t j = i < nb ? s_sj[i] : 0;
        cp_async16(sV + (i / SP) * VBUF + (i % SP) * LD + d0, vg + j * p.vsn + d0, i < nb ? 16 : 0);
      }
    }
    for (int it = tid; it < SB * (HALF / 8); it += NTH) {
      const int i = it / (HALF / 8), f0 = (it % (HALF / 8)) * 8;
      const int64_t j = i < nb ? s_sj[i] : 0;
      const float npk = i < nb ? s_sp[i] : 0.f;
      __nv_bfloat16* dst = sKa + (i / SP) * KBUF + (i % SP) * LD;
      rotate8<NQ, HALF>(kg + j * p.ksn, i < nb, f0, npk, p.inv_freq_c, 1.f, dst, SP * LD, p.rtab,
                        table_index(npk, p.rtab_R, p.rtab_len));
    }
    for (int it = tid; F32 && it < SB * (D / 8); it += NTH) {
      const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
      const int64_t j = i < nb ? s_sj[i] : 0;
      __nv_bfloat16* dst = sV + (i / SP) * VBUF + (i % SP) * LD + d0;
      {
        float x[8];
        if (i < nb) {
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
          for (int q2 = 0; q2 < NV; ++q2) dst[q2 * SP * LD + u] = pc[q2];
        }
      }
    }
    if (!F32) cp_async_wait_all();
    __syncthreads();
    float s[SP / 8][4];
    score_tile<D, SP, NQ>(sQa, myK, s, rw);
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < SP / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = nt * 8 + 2 * c4 + (e & 1);
        const int row = e < 2 ? ra : rb;
        const int si = pair * SP + col;
        const bool keep = si < nb && ((s_scw[si] >> row) & 1u);
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
    for (int nt = 0; nt < SP / 8; ++nt) {
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
      for (int kk = 0; kk < SP / 16; ++kk) {
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
            ldsm_x4_t(smem_u32(myV + (j * SP + row) * LD + col), v0[j][0], v0[j][1], v1[j][0], v1[j][1]);
          mma_pieces<NV>(o[2 * dp], pp, v0);
          mma_pieces<NV>(o[2 * dp + 1], pp, v1);
        }
      }
    }
    __syncthreads();  // buffers and pending slots free again
  };

  // ---- phase 2: descending blocks, NTH per chunk: streamed offsets d, the blocks with keeps,
  // their kept keys in (block, key) order appended to the pending slots, SB slots attended at a
  // time
  int carry_d = 0, n_pos = 0, n_pend = 0;
  for (int c0 = 0; c0 < nblk; c0 += NTH) {
    const int tb = c0 + tid;
    int adv = 0, use = 0, b = 0;
    if (tb < nblk) {
      b = nblk - 1 - tb;
      int cm;
      if (b < nf_g) cm = s_fcm[b];
      else if (b >= lb0) cm = s_fcm[nf_g + (b - lb0)];
      else cm = __ldg(bmax_row + (int64_t)b * (BN / 32));
      const int64_t sn = (int64_t)b * BN;
      const int64_t hi_t = min(P_top, sn + BN - 1);
      adv = p.adv_full ? (int)(hi_t - sn + 1) : cm;
      use = cm > 0;
      n_pos += adv > 0;
    }
    int tot_d, n_use;
    const int ed = cta_excl_sum(adv, s_red, tot_d);
    const int eu = cta_excl_sum(use, s_red, n_use);
    if (use) {
      s_list[eu] = b;
      s_dl[eu] = (float)(carry_d + ed);
    }
    carry_d += tot_d;
    __syncthreads();
    // keys of each listed block kept by some query
    for (int li = warp; li < n_use; li += NW) {
      const int64_t sn = (int64_t)s_list[li] * BN;
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        const uint32_t m = __ballot_sync(0xffffffffu, keep_word(sn + h * 32 + lane) != 0u);
        if (lane == 0) s_bm[li][h] = m;
      }
    }
    __syncthreads();
    int cnt = 0;
    if (tid < n_use) {
#pragma unroll
      for (int h = 0; h < NH; ++h) cnt += __popc(s_bm[tid][h]);
    }
    int n_slots;
    const int off = cta_excl_sum(cnt, s_red, n_slots);
    if (tid < n_use) s_bo[tid] = off;
    __syncthreads();
    for (int s0 = 0; s0 < n_slots;) {
      const int take = min(SB - n_pend, n_slots - s0);
      for (int i = tid; i < take; i += NTH) {
        const int gi = s0 + i;
        int lo = 0, hi2 = n_use - 1;  // last listed block with s_bo <= gi
        while (lo < hi2) {
          const int mid = (lo + hi2 + 1) >> 1;
          if (s_bo[mid] <= gi) lo = mid;
          else hi2 = mid - 1;
        }
        int k = gi - s_bo[lo], kb = 0;
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const uint32_t m = s_bm[lo][h];
          const int c = __popc(m);
          if (k >= 0 && k < c) kb = h * 32 + (int)__fns(m, 0, k + 1);
          k -= c;
        }
        const int64_t sn = (int64_t)s_list[lo] * BN;
        const int64_t j = sn + kb;
        const int64_t hi_t = min(P_top, sn + BN - 1);
        s_sj[n_pend + i] = (int)j;
        s_sp[n_pend + i] = -__fadd_rn(s_dl[lo], (float)(hi_t - j));
        s_scw[n_pend + i] = keep_word(j);
      }
      n_pend += take;
      s0 += take;
      __syncthreads();
      if (n_pend == SB) {
        attend_batch(SB);
        n_pend = 0;
      }
    }
  }
  if (n_pend > 0) attend_batch(n_pend);
  int n_adv;
  {
    int tot;
    cta_excl_sum(n_pos, s_red, tot);
    n_adv = tot;
  }

  // ---- merge the two pairs' softmax states (pair 1 -> shared memory -> pair 0)
  float* s_o = reinterpret_cast<float*>(sKa);  // the K buffers are free now
  __syncthreads();
  if (pair == 1) {
    float* dst = s_o + (size_t)(rw * 32 + lane) * (D / 2);
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[i * 4 + e] = o[i][e];
  }
  __syncthreads();
  if (pair == 1 && c4 == 0) {
    s_ml[ra][0] = mA;
    s_ml[ra][1] = lA;
    s_ml[rb][0] = mB;
    s_ml[rb][1] = lB;
  }
  __syncthreads();
  if (pair == 0) {
    const float* src = s_o + (size_t)(rw * 32 + lane) * (D / 2);
    const float m1A = s_ml[ra][0], l1A = s_ml[ra][1], m1B = s_ml[rb][0], l1B = s_ml[rb][1];
    const float MA = fmaxf(mA, m1A), MB = fmaxf(mB, m1B);
    const float a0A = mA == -INFINITY ? 0.f : expf(__fsub_rn(mA, MA));
    const float a1A = m1A == -INFINITY ? 0.f : expf(__fsub_rn(m1A, MA));
    const float a0B = mB == -INFINITY ? 0.f : expf(__fsub_rn(mB, MB));
    const float a1B = m1B == -INFINITY ? 0.f : expf(__fsub_rn(m1B, MB));
    lA = lA * a0A + l1A * a1A;
    lB = lB * a0B + l1B * a1B;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] = o[i][0] * a0A + src[i * 4 + 0] * a1A;
      o[i][1] = o[i][1] * a0A + src[i * 4 + 1] * a1A;
      o[i][2] = o[i][2] * a0B + src[i * 4 + 2] * a1B;
      o[i][3] = o[i][3] * a0B + src[i * 4 + 3] * a1B;
    }
  }
  const int64_t qpa = tstart + ra, qpb = tstart + rb;
  const bool okA = qpa < N && pair == 0, okB = qpb < N && pair == 0;
  const int64_t ra_l = qpa - p.qbase, rb_l = qpb - p.qbase;  // slab rows
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
  // kept keys per query: Kernel A's count plus the forced keys its threshold did not keep
  if (c4 == 0) {
    if (okA) p.kept[bh * p.Nq + ra_l] = p.row_count[bh * p.Nq + ra_l] + s_extra[ra];
    if (okB) p.kept[bh * p.Nq + rb_l] = p.row_count[bh * p.Nq + rb_l] + s_extra[rb];
  }
  if (tid == 0) {
    const int64_t o2 = bh * p.nt + t;
    p.span[o2] = (float)carry_d;
    p.blocks[o2] = (float)nblk;
    p.skipped[o2] = (float)(p.use_skip ? nblk - n_adv : 0);
  }
}

template <int D, int BN, bool F32>
int launch_one(const PQSP& p, cudaStream_t stream) {
  constexpr int LD = D + 8;
  constexpr int NQ = F32 ? 3 : 2, NV = F32 ? 3 : 1;
  // forced blocks per tile: the global prefix and the local window (+ its partial blocks)
  const int64_t ng = (int64_t)(p.n_global > 0 ? p.n_global : 0);
  const int64_t nl = (int64_t)(p.n_local > 0 ? p.n_local : 0);
  const int64_t nfs_cap = (ng + BN - 1) / BN + (nl + T + BN - 1) / BN + 2;
  const size_t smem = (size_t)(NQ * T + 2 * (NQ + NV) * SP) * LD * 2 + (size_t)nfs_cap * 4;
  if (smem > 200 * 1024)
    return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: n_global / n_local too large");
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
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->bits || !a->block_max || !a->row_count ||
      !a->inv_freq_c || !a->span || !a->kept || !a->blocks || !a->skipped)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: null pointer");
  if (a->tile != 32) return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: tile must be 32");
  if (a->block_n != 32 && a->block_n != 64)
    return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: block_n must be 32 or 64");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_pqstream_attend: d must be 64 or 128");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: bad head counts");
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n || a->q_pos_base % 32)
    return fail(STA_ERR_ARG, "sta_pqstream_attend: q_pos_base must be a multiple of 32 in [0, n)");
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
  p.qbase = a->q_pos_base;
  p.Nq = a->n - a->q_pos_base;
  p.nt = (p.Nq + T - 1) / T;
  p.H = (int)a->n_heads;
  p.Hkv = (int)a->n_kv_heads;
  p.bits = a->bits;
  p.head_stride = tri_head_stride(a->n, T, a->q_pos_base);
  p.bmax = a->block_max;
  p.bmax_stride = tri_head_stride((a->n + 31) / 32, 1, a->q_pos_base / 32);
  p.row_count = a->row_count;
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
