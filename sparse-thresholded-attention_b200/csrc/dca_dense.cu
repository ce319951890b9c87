// Dense Dual Chunk Attention prefill as one fused tcgen05 attention kernel.
//
// Reference: dca_forward, dca_kernel.py:447-487 (prefill, q_len > 1).  Per query segment of
// chunk_len L queries it runs three attention blocks -- intra (same chunk, causal), succ (the
// previous chunk) and inter (older chunks), each with its own query rotation against keys
// rotated at cyclic positions j mod L (ChunkLlama tables, :194-231) -- and merges them by
// log-sum-exp (_merge_lse, :352-366).  The merge is one softmax over all causal keys, so here
// every query row runs ONE online softmax over all its causal 128-key blocks, each block scored
// with the query plane of its chunk relation (intra / succ / inter), which is the same plane
// rule as the thresholded DCA selection (q_plane below).  chunk_size == 0 gives plain causal
// attention with RoPE at the true positions.
//
// Per CTA (persistent, one per SM, longest-first over items of 128 query rows of one q head):
//   warps 0-7  softmax: two warps per TMEM lane quadrant share each query row (TMEM lane r),
//              64 S columns each.  Per key block: read S from TMEM, mask, the row max of both
//              halves (shared memory), running max in the log2 domain, lazy rescale of O (only when
//              the max grows by more than 2^8, after the previous P.V has completed), P = 2^(x-m)
//              written back into the same TMEM columns as bf16 (hi, and lo for fp32 inputs),
//              row sum in fp32; at the item's end O / l to global memory;
//   warp 8     TMA producer: the item's query plane (single buffer, reloaded on a plane change),
//              K blocks and V^T blocks through two rings;
//   warp 9     MMA issuer (one thread): S = Q.K^T (M128 N128 K16, smem operands) into one of
//              three TMEM slots, then O += P.V with P read from TMEM (the A operand) and V^T
//              from shared memory; S of block g+1 is issued before P.V of block g so the
//              softmax of one block overlaps the tensor work of the next.
// Numerics: scores from the fp32-rotated rows split into hi / lo bf16 pieces, three products
// (~2^-16 relative: a single bf16 product of the rounded rows, as flash-attention on bf16 rows
// computes it, moves outputs by up to ~5e-2 on these inputs).  P.V: bf16 inputs multiply P
// rounded to bf16 by V (bf16, exact), as the reference does; fp32 inputs split P and V into
// hi / lo pieces as well (three products).
// Every wait is bounded; on expiry the kernel records STA_ERR_TIMEOUT and unwinds.
#include <cstdio>

#include "common.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int BM = 128;           // query rows per item == TMEM lanes
constexpr int BN = 128;           // keys per block == MMA N of S
constexpr int NS = 3;             // S / P slots (128 TMEM columns each)
constexpr int OCOL = NS * BN;     // O accumulator columns [384, 384 + D)
constexpr int kChunk = 128 * 128; // one 128-row x 64-bf16 swizzled chunk (16 KB)
constexpr int kSP = 2;            // softmax warps per TMEM lane quadrant
constexpr int kSoftmax = 4 * kSP; // softmax warps (warps 0 .. kSoftmax-1)

template <int D, bool F32>
struct DCfg {
  static constexpr int NC = D / 64;                   // 64-column chunks of a row of Q / K
  static constexpr int NPV = F32 ? 2 : 1;             // bf16 pieces of P and V^T
  static constexpr int Q_BYTES = 2 * NC * kChunk;     // Q hi + lo
  static constexpr int K_STAGE = 2 * NC * kChunk;     // one 128-key block, hi + lo
  static constexpr int VT_CHUNK = D * 128;            // D rows (d) x 64 keys, swizzled
  static constexpr int V_STAGE = NPV * 2 * VT_CHUNK;  // one 128-key block of V^T, all pieces
  static constexpr int NSK = F32 ? 1 : 2;
  static constexpr int NSV = 1;
  // + barriers (< 256 B) and the softmax parts' row exchange (kSP x 128 floats)
  static constexpr int SMEM = 1024 + Q_BYTES + NSK * K_STAGE + NSV * V_STAGE + 256 + kSP * 512;
  static constexpr int kThreads = (kSoftmax + 2) * 32;
};

struct DParams {
  int64_t BH;
  int H, Hkv;
  int64_t N;         // keys
  int64_t Nq;        // query rows held (positions qbase .. N-1)
  int64_t qbase;     // multiple of 128
  int qb0, nqb;
  int64_t dca_L;     // chunk_len (multiple of 128), 0: plain causal
  float c_log2;      // sm_scale * log2(e)
  void* out;         // (BH, Nq, D) in the input dtype
  int out_f32;
  int* err;
  uint64_t limit_ns;
};

__device__ __forceinline__ int dplane(const DParams& p, int qb, int kb) {
  if (p.dca_L <= 0) return 0;
  const int64_t rel = ((int64_t)qb * BM) / p.dca_L - ((int64_t)kb * BN) / p.dca_L;
  return rel <= 0 ? 0 : (rel == 1 ? 1 : 2);
}

// Longest-first: the largest query blocks of every head first.
__device__ __forceinline__ void ditem(int64_t w, const DParams& p, int64_t& bh, int& qb,
                                      int64_t& kvh) {
  qb = p.nqb - 1 - (int)(w / p.BH) + p.qb0;
  bh = w % p.BH;
  const int G = p.H / p.Hkv;
  kvh = (bh / p.H) * p.Hkv + (bh % p.H) / G;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a -> low half, b -> high half
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D, bool F32>
__global__ void __launch_bounds__((kSoftmax + 2) * 32, 1)
dca_dense_kernel(const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
                 const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
                 const __grid_constant__ CUtensorMap tm_vhi, const __grid_constant__ CUtensorMap tm_vlo,
                 const DParams p) {
  using C = DCfg<D, F32>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = sQ + C::Q_BYTES;
  uint8_t* sV = sK + C::NSK * C::K_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + C::NSV * C::V_STAGE);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + C::NSK;
  uint64_t* v_full = k_empty + C::NSK;
  uint64_t* v_empty = v_full + C::NSV;
  uint64_t* s_full = v_empty + C::NSV;   // [NS] S of a block in its slot
  uint64_t* p_full = s_full + NS;        // [NS] P written (all softmax threads)
  uint64_t* pv_done = p_full + NS;       // [NS] P.V of the slot's block completed
  uint64_t* o_free = pv_done + NS;       // O read out (all softmax threads)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(o_free + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::NSK; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int s = 0; s < C::NSV; ++s) {
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(s_full + s, 1);
      mbar_init(p_full + s, kSoftmax * 32);
      mbar_init(pv_done + s, 1);
    }
    mbar_init(o_free, kSoftmax * 32);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 0) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int64_t total = p.BH * (int64_t)p.nqb;

  if (warp == kSoftmax) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_qhi);
      prefetch_tmap(&tm_khi);
      prefetch_tmap(&tm_vhi);
      uint32_t kc = 0, vc = 0, qloads = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; w < total && ok; w += gridDim.x) {
        int64_t bh, kvh;
        int qb;
        ditem(w, p, bh, qb, kvh);
        int cur = -1;
        for (int kb = 0; kb <= qb && ok; ++kb) {
          const int plane = dplane(p, qb, kb);
          if (plane != cur) {
            if (qloads > 0 && !mbar_wait(q_empty, (qloads - 1) & 1, s_abort, p.err, kErrTimeoutQ,
                                         p.limit_ns)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(q_full, C::Q_BYTES);
            const int z = (int)(plane * p.BH + bh);
            const int qrow = (qb - p.qb0) * BM;
            for (int c = 0; c < C::NC; ++c) {
              tma_load_3d(sQ + c * kChunk, &tm_qhi, q_full, c * 64, qrow, z);
              tma_load_3d(sQ + (C::NC + c) * kChunk, &tm_qlo, q_full, c * 64, qrow, z);
            }
            ++qloads;
            cur = plane;
          }
          {  // K block
            const uint32_t s = kc % C::NSK, r = kc / C::NSK;
            if (r > 0 && !mbar_wait(k_empty + s, (r - 1) & 1, s_abort, p.err, kErrTimeoutEmpty,
                                    p.limit_ns)) {
              ok = false;
              break;
            }
            uint8_t* st = sK + s * C::K_STAGE;
            mbar_arrive_expect_tx(k_full + s, C::K_STAGE);
            for (int c = 0; c < C::NC; ++c) {
              tma_load_3d(st + c * kChunk, &tm_khi, k_full + s, c * 64, kb * BN, (int)kvh);
              tma_load_3d(st + (C::NC + c) * kChunk, &tm_klo, k_full + s, c * 64, kb * BN, (int)kvh);
            }
            ++kc;
          }
          {  // V^T block: two 64-key chunks of D rows
            const uint32_t s = vc % C::NSV, r = vc / C::NSV;
            if (r > 0 && !mbar_wait(v_empty + s, (r - 1) & 1, s_abort, p.err, kErrTimeoutEmpty,
                                    p.limit_ns)) {
              ok = false;
              break;
            }
            uint8_t* st = sV + s * C::V_STAGE;
            mbar_arrive_expect_tx(v_full + s, C::V_STAGE);
            for (int c2 = 0; c2 < 2; ++c2) {
              tma_load_3d(st + c2 * C::VT_CHUNK, &tm_vhi, v_full + s, kb * BN + c2 * 64, 0, (int)kvh);
              if (F32) tma_load_3d(st + (2 + c2) * C::VT_CHUNK, &tm_vlo, v_full + s, kb * BN + c2 * 64, 0, (int)kvh);
            }
            ++vc;
          }
        }
      }
    }
  } else if (warp == kSoftmax + 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BM, BN);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BM, D);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      uint32_t kc = 0, vc = 0, qloads = 0, g = 0, it = 0;
      bool ok = true;
      // P.V of block gp (first block of item `item`: overwrite O once the previous item's O has
      // been read out)
      auto issue_pv = [&](uint32_t gp, bool first, uint32_t item) -> bool {
        if (first && item > 0 &&
            !mbar_wait(o_free, (item - 1) & 1, s_abort, p.err, kErrTimeoutAcc, p.limit_ns))
          return false;
        const uint32_t slot = gp % NS;
        if (!mbar_wait(p_full + slot, (gp / NS) & 1, s_abort, p.err, kErrTimeoutAcc, p.limit_ns))
          return false;
        const uint32_t s = vc % C::NSV, r = vc / C::NSV;
        if (!mbar_wait(v_full + s, r & 1, s_abort, p.err, kErrTimeoutK, p.limit_ns)) return false;
        tc_fence_after();
        const uint32_t st = v_addr + s * C::V_STAGE;
        const uint32_t a0 = tmem_base + slot * BN;
        uint32_t acc = first ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16 keys per MMA
          const uint32_t voff = (kk >> 2) * C::VT_CHUNK + (kk & 3) * 32;
          const uint64_t vh = sw128_kmajor_desc(st + voff);
          umma_bf16_ts(tmem_base + OCOL, a0 + kk * 8, vh, idesc_o, acc);
          acc = 1;
          if (F32) {
            const uint64_t vl = sw128_kmajor_desc(st + 2 * C::VT_CHUNK + voff);
            umma_bf16_ts(tmem_base + OCOL, a0 + 64 + kk * 8, vh, idesc_o, 1);  // P lo . V hi
            umma_bf16_ts(tmem_base + OCOL, a0 + kk * 8, vl, idesc_o, 1);       // P hi . V lo
          }
        }
        umma_commit(v_empty + s);
        umma_commit(pv_done + slot);
        ++vc;
        return true;
      };
      bool pend = false;  // P.V of block pend_g (item pend_item) not issued yet
      bool pend_first = false;
      uint32_t pend_g = 0, pend_item = 0;
      for (int64_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
        int64_t bh, kvh;
        int qb;
        ditem(w, p, bh, qb, kvh);
        int cur = -1;
        for (int kb = 0; kb <= qb; ++kb, ++g) {
          const int plane = dplane(p, qb, kb);
          if (plane != cur) {
            if (qloads > 0) umma_commit(q_empty);  // the resident plane is free once read
            if (!mbar_wait(q_full, qloads & 1, s_abort, p.err, kErrTimeoutQ, p.limit_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            ++qloads;
            cur = plane;
          }
          // S of block g into slot g % NS once the P.V that last read that slot has completed
          const uint32_t slot = g % NS;
          if (g >= NS && !mbar_wait(pv_done + slot, ((g / NS) - 1) & 1, s_abort, p.err,
                                    kErrTimeoutAcc, p.limit_ns)) {
            ok = false;
            break;
          }
          const uint32_t s = kc % C::NSK, r = kc / C::NSK;
          if (!mbar_wait(k_full + s, r & 1, s_abort, p.err, kErrTimeoutK, p.limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = k_addr + s * C::K_STAGE;
          const uint32_t d_s = tmem_base + slot * BN;
          uint32_t acc = 0;
#pragma unroll
          for (int c = 0; c < C::NC; ++c) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t off = c * kChunk + kk * 32;
              const uint64_t qh = sw128_kmajor_desc(q_addr + off);
              const uint64_t kh = sw128_kmajor_desc(st + off);
              const uint64_t ql = sw128_kmajor_desc(q_addr + C::NC * kChunk + off);
              const uint64_t kl = sw128_kmajor_desc(st + C::NC * kChunk + off);
              umma_bf16(d_s, qh, kh, idesc_s, acc);
              acc = 1;
              umma_bf16(d_s, ql, kh, idesc_s, 1);
              umma_bf16(d_s, qh, kl, idesc_s, 1);
            }
          }
          umma_commit(k_empty + s);
          umma_commit(s_full + slot);
          ++kc;
          // then P.V of the previous block: the softmax of block g overlaps it
          if (pend && !issue_pv(pend_g, pend_first, pend_item)) {
            ok = false;
            break;
          }
          pend = true;
          pend_g = g;
          pend_first = (kb == 0);
          pend_item = it;
        }
      }
      if (ok && pend) issue_pv(pend_g, pend_first, pend_item);
    }
  } else {
    // -------------------------------------------------------------- softmax / epilogue
    // kSP warps per TMEM lane quadrant share each row: warp (quad, part) handles the row's
    // columns [part * BN / kSP, +BN / kSP) of S and the O columns of chunks c with
    // c % kSP == part.  Row maxima and sums of the parts meet in shared memory behind the
    // quadrant's named barrier (id 1 + quad).  After a failed wait a warp keeps walking the
    // schedule without touching TMEM, so every warp still reaches every barrier.
    const int quad = warp & 3;
    const int part = warp >> 2;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(quad * 32) << 16);
    constexpr int CW = BN / kSP;  // S columns per warp
    float* s_x = reinterpret_cast<float*>(s_tmem + 4);  // [kSP][128] partial max / sum
    uint32_t g = 0;
    bool ok = true;
    auto quad_sync = [&]() { named_bar_sync(1 + quad, kSP * 32); };
    for (int64_t w = blockIdx.x; w < total; w += gridDim.x) {
      int64_t bh, kvh;
      int qb;
      ditem(w, p, bh, qb, kvh);
      const int64_t qp = (int64_t)qb * BM + row;
      const bool row_ok = qp < p.N;
      float m_used = -INFINITY, l = 0.f;
      for (int kb = 0; kb <= qb; ++kb, ++g) {
        const uint32_t slot = g % NS;
        int bad = 0;
        if (ok && lane == 0) bad = !mbar_wait(s_full + slot, (g / NS) & 1, s_abort, p.err,
                                               kErrTimeoutAcc, p.limit_ns);
        if (__shfl_sync(0xffffffffu, bad, 0)) ok = false;
        float x[CW];
        const int64_t kbase = (int64_t)kb * BN + part * CW;
        float mx = -INFINITY;
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < CW / 32; ++c) {
            float v[32];
            tmem_ld32(lane_addr + slot * BN + part * CW + c * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) x[c * 32 + j] = v[j];
          }
          if (kb == qb || !row_ok) {  // the diagonal block (or a row past the end): mask
            const int64_t lim = row_ok ? qp - kbase : -1;  // keys j <= lim are causal
#pragma unroll
            for (int j = 0; j < CW; ++j) {
              x[j] = (j <= lim) ? x[j] * p.c_log2 : -INFINITY;
              mx = fmaxf(mx, x[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < CW; ++j) {
              x[j] *= p.c_log2;
              mx = fmaxf(mx, x[j]);
            }
          }
        }
        // the row max over all parts
        s_x[part * 128 + row] = mx;
        quad_sync();
#pragma unroll
        for (int q2 = 0; q2 < kSP; ++q2) mx = fmaxf(mx, s_x[q2 * 128 + row]);
        quad_sync();
        if (!ok) continue;
        // Lazy rescale: only when some row's max grew by more than 2^8.  The TMEM accesses are
        // warp-collective, so the decision is taken per warp (the parts of a quadrant see the
        // same row maxima and decide alike): every row then moves to its own new max (factor
        // <= 1; 0 for a row without earlier contributions).
        const float m_new = fmaxf(m_used, mx);
        const bool want = mx > m_used + 8.f;
        if (kb == 0) {
          m_used = m_new;
        } else if (__any_sync(0xffffffffu, want)) {
          // O holds the blocks so far at m_used: rescale once the last P.V has landed
          const uint32_t gp = g - 1;
          int bad2 = 0;
          if (lane == 0) bad2 = !mbar_wait(pv_done + gp % NS, (gp / NS) & 1, s_abort, p.err,
                                            kErrTimeoutAcc, p.limit_ns);
          if (__shfl_sync(0xffffffffu, bad2, 0)) {
            ok = false;
            continue;
          }
          tc_fence_after();
          const float f = m_used > -INFINITY ? exp2f(m_used - m_new) : 0.f;
#pragma unroll
          for (int c = part; c < D / 32; c += kSP) {
            float v[32];
            tmem_ld32(lane_addr + OCOL + c * 32, v);
            tmem_wait_ld();
            uint32_t u[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) u[j] = __float_as_uint(v[j] * f);
            tmem_st32(lane_addr + OCOL + c * 32, u);
          }
          l *= f;
          m_used = m_new;
        }
        // P = 2^(x - m_used) as bf16 pairs (key 2w in the low half of column w), 64 keys per
        // store; fp32 inputs also store the residual lo pieces 64 columns further
        float bsum = 0.f;
#pragma unroll
        for (int h = 0; h < CW / 64; ++h) {
          uint32_t ph[32], pl[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float xa = x[64 * h + 2 * j], xb = x[64 * h + 2 * j + 1];
            // m_used is finite for every row with a causal key; 2^(-inf) = 0 for masked keys
            const float a = row_ok ? exp2f(xa - m_used) : 0.f;
            const float b = row_ok ? exp2f(xb - m_used) : 0.f;
            bsum += a + b;
            ph[j] = pack_bf16(a, b);
            if (F32) {
              const __nv_bfloat162 hv = *reinterpret_cast<const __nv_bfloat162*>(&ph[j]);
              pl[j] = pack_bf16(a - __low2float(hv), b - __high2float(hv));
            }
          }
          const uint32_t pc = slot * BN + (part * CW) / 2 + 32 * h;
          tmem_st32(lane_addr + pc, ph);
          if (F32) tmem_st32(lane_addr + pc + 64, pl);
        }
        l += bsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full + slot);
      }
      // item end: the row sum over the parts, O after the last P.V divided by it
      s_x[part * 128 + row] = l;
      quad_sync();
      float lt = 0.f;
#pragma unroll
      for (int q2 = 0; q2 < kSP; ++q2) lt += s_x[q2 * 128 + row];
      quad_sync();
      if (ok) {
        const uint32_t gp = g - 1;
        int bad = 0;
        if (lane == 0) bad = !mbar_wait(pv_done + gp % NS, (gp / NS) & 1, s_abort, p.err,
                                         kErrTimeoutAcc, p.limit_ns);
        if (__shfl_sync(0xffffffffu, bad, 0)) ok = false;
      }
      if (ok) {
        tc_fence_after();
        const float inv = (row_ok && lt > 0.f) ? 1.f / lt : 0.f;
        const int64_t orow = bh * p.Nq + (qp - p.qbase);
#pragma unroll
        for (int c = part; c < D / 32; c += kSP) {
          float v[32];
          tmem_ld32(lane_addr + OCOL + c * 32, v);
          tmem_wait_ld();
          if (row_ok) {
            if (p.out_f32) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + orow * D + c * 32);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(v[4 * j] * inv, v[4 * j + 1] * inv, v[4 * j + 2] * inv,
                                     v[4 * j + 3] * inv);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + orow * D + c * 32);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                dst[j] = make_uint4(pack_bf16(v[8 * j] * inv, v[8 * j + 1] * inv),
                                    pack_bf16(v[8 * j + 2] * inv, v[8 * j + 3] * inv),
                                    pack_bf16(v[8 * j + 4] * inv, v[8 * j + 5] * inv),
                                    pack_bf16(v[8 * j + 6] * inv, v[8 * j + 7] * inv));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(o_free);
      }
    }
  }

  // -------------------------------------------------------------- teardown
  if (*s_abort) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, 512);
}

}  // namespace
}  // namespace sta

namespace sta {
namespace {

// V (heads, n, d) -> V^T (heads, d, npad) bf16 hi [, lo], keys n .. npad-1 zero: the B operand
// of P.V wants the keys contiguous.  32 x 32 tiles through shared memory, coalesced both ways.
template <typename T>
__global__ void vt_kernel(const T* __restrict__ v, int64_t n, int d, int64_t sh, int64_t sn,
                          __nv_bfloat16* __restrict__ vh, __nv_bfloat16* __restrict__ vl,
                          int64_t npad) {
  __shared__ float tile[32][33];
  const int64_t h = blockIdx.z;
  const int64_t j0 = (int64_t)blockIdx.x * 32;
  const int d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    const int64_t j = j0 + r;
    float x = 0.f;
    if (j < n) {
      const T* src = v + h * sh + j * sn + d0 + tx;
      if constexpr (sizeof(T) == 4) x = *reinterpret_cast<const float*>(src);
      else x = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(src));
    }
    tile[r][tx] = x;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const float x = tile[tx][r];  // key j0 + tx, column d0 + r
    const int64_t o = (h * d + d0 + r) * npad + j0 + tx;
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    vh[o] = hi;
    if (vl) vl[o] = __float2bfloat16_rn(x - __bfloat162float(hi));
  }
}

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

#define STA_CHECK_RC(x)            \
  do {                             \
    const int _r = (x);            \
    if (_r != STA_OK) return _r;   \
  } while (0)

struct DLayout {
  size_t qh, ql, kh, kl, vh, vl, total;
  int64_t npad, planes;
};

DLayout dca_layout(const sta_dca_args* a) {
  DLayout L{};
  const bool f32 = a->dtype == STA_DTYPE_F32;
  const int64_t BH = a->n_heads, BHk = a->n_kv_heads;  // one batch element at a time
  const int64_t Nq = a->n - a->q_pos_base, D = a->d;
  L.planes = a->chunk_size > 0 ? 3 : 1;
  L.npad = (a->n + 63) / 64 * 64;
  size_t o = 0;
  auto take = [&](size_t b) { const size_t r = o; o += al256(b); return r; };
  // the RoPE prologue always writes both pieces; bf16 inputs read only the hi ones
  L.qh = take((size_t)L.planes * BH * Nq * D * 2);
  L.ql = take((size_t)L.planes * BH * Nq * D * 2);
  L.kh = take((size_t)BHk * a->n * D * 2);
  L.kl = take((size_t)BHk * a->n * D * 2);
  L.vh = take((size_t)BHk * D * L.npad * 2);
  L.vl = f32 ? take((size_t)BHk * D * L.npad * 2) : 0;
  L.total = o;
  return L;
}

int dca_check(const sta_dca_args* a) {
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->inv_freq)
    return fail(STA_ERR_ARG, "sta_dca_forward: null pointer");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_dca_forward: head_dim must be 64 or 128");
  if (a->dtype != STA_DTYPE_F32 && a->dtype != STA_DTYPE_BF16)
    return fail(STA_ERR_UNSUPPORTED, "sta_dca_forward: dtype must be f32 or bf16");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_dca_forward: n_heads must be a positive multiple of n_kv_heads");
  if (a->q_pos_base < 0 || (a->n > 0 && a->q_pos_base >= a->n) || a->q_pos_base % BM)
    return fail(STA_ERR_UNSUPPORTED, "sta_dca_forward: q_pos_base must be a multiple of 128 below n");
  if (a->chunk_size > 0) {
    const int64_t L = (int64_t)a->chunk_size - a->local_window;
    if (a->local_window <= 0 || L <= 0 || L % 128)
      return fail(STA_ERR_UNSUPPORTED,
                  "sta_dca_forward: needs 0 < local_window < chunk_size and chunk_size - local_window a multiple of 128");
  }
  if (a->n > ((int64_t)1 << 30)) return fail(STA_ERR_UNSUPPORTED, "sta_dca_forward: n too large");
  return STA_OK;
}

template <int D, bool F32>
cudaError_t launch_dca_kernel(const CUtensorMap* m, const DParams& p, int grid, cudaStream_t st) {
  using C = DCfg<D, F32>;
  cudaError_t e = cudaFuncSetAttribute(dca_dense_kernel<D, F32>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dca_dense_kernel<D, F32><<<grid, C::kThreads, C::SMEM, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], p);
  return cudaGetLastError();
}

}  // namespace
}  // namespace sta

extern "C" {

size_t sta_dca_workspace_bytes(const sta_dca_args* a) {
  if (sta::dca_check(a) != STA_OK) return 0;
  return sta::dca_layout(a).total;
}

int sta_dca_forward(const sta_dca_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sta;
  const int rc = dca_check(a);
  if (rc != STA_OK) return rc;
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  const DLayout L = dca_layout(a);
  if (!workspace || workspace_bytes < L.total) return fail(STA_ERR_WORKSPACE, "sta_dca_forward: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  const bool f32 = a->dtype == STA_DTYPE_F32;
  const int64_t es = f32 ? 4 : 2;
  const int64_t H = a->n_heads, Hk = a->n_kv_heads, N = a->n, D = a->d;
  const int64_t qbase = a->q_pos_base, Nq = N - qbase;
  const int64_t dL = a->chunk_size > 0 ? (int64_t)a->chunk_size - a->local_window : 0;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  for (int64_t b = 0; b < a->batch; ++b) {
    const uint8_t* q = static_cast<const uint8_t*>(a->q) + b * H * a->q_stride_h * es;
    const uint8_t* k = static_cast<const uint8_t*>(a->k) + b * Hk * a->k_stride_h * es;
    const uint8_t* v = static_cast<const uint8_t*>(a->v) + b * Hk * a->v_stride_h * es;
    uint8_t* out = static_cast<uint8_t*>(a->out) + b * H * Nq * D * es;
    // query planes and keys of the geometry (DCA position roles, or linear positions)
    if (dL > 0) {
      const size_t plane = (size_t)H * Nq * D * 2;
      for (int role = 1; role <= 3; ++role)
        STA_CHECK_RC(launch_rope_split(q, a->dtype, H, Nq, (int)D, a->q_stride_h, a->q_stride_n,
                                       a->inv_freq, 1.0f, a->rope_scale,
                                       w + L.qh + (role - 1) * plane, w + L.ql + (role - 1) * plane,
                                       st, role, dL, a->chunk_size, qbase));
      STA_CHECK_RC(launch_rope_split(k, a->dtype, Hk, N, (int)D, a->k_stride_h, a->k_stride_n,
                                     a->inv_freq, 1.0f, a->rope_scale, w + L.kh, w + L.kl, st, 1,
                                     dL, a->chunk_size, 0));
    } else {
      STA_CHECK_RC(launch_rope_split(q, a->dtype, H, Nq, (int)D, a->q_stride_h, a->q_stride_n,
                                     a->inv_freq, 1.0f, a->rope_scale, w + L.qh, w + L.ql, st, 0,
                                     0, 0, qbase));
      STA_CHECK_RC(launch_rope_split(k, a->dtype, Hk, N, (int)D, a->k_stride_h, a->k_stride_n,
                                     a->inv_freq, 1.0f, a->rope_scale, w + L.kh, w + L.kl, st, 0,
                                     0, 0, 0));
    }
    {
      dim3 grid((unsigned)(L.npad / 32), (unsigned)(D / 32), (unsigned)Hk), blk(32, 8);
      __nv_bfloat16* vh = reinterpret_cast<__nv_bfloat16*>(w + L.vh);
      __nv_bfloat16* vl = f32 ? reinterpret_cast<__nv_bfloat16*>(w + L.vl) : nullptr;
      if (f32)
        vt_kernel<float><<<grid, blk, 0, st>>>(static_cast<const float*>((const void*)v), N, (int)D,
                                               a->v_stride_h, a->v_stride_n, vh, vl, L.npad);
      else
        vt_kernel<__nv_bfloat16><<<grid, blk, 0, st>>>(
            static_cast<const __nv_bfloat16*>((const void*)v), N, (int)D, a->v_stride_h,
            a->v_stride_n, vh, vl, L.npad);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
    }
    CUtensorMap m[6];
    void* qlo_map = w + L.ql;
    void* klo_map = w + L.kl;
    void* vlo_map = f32 ? (void*)(w + L.vl) : (void*)(w + L.vh);
    bool okm = make_tmap_bf16_3d(&m[0], w + L.qh, D, Nq, L.planes * H, 64, BM) &&
               make_tmap_bf16_3d(&m[1], qlo_map, D, Nq, L.planes * H, 64, BM) &&
               make_tmap_bf16_3d(&m[2], w + L.kh, D, N, Hk, 64, BN) &&
               make_tmap_bf16_3d(&m[3], klo_map, D, N, Hk, 64, BN) &&
               make_tmap_bf16_3d(&m[4], w + L.vh, L.npad, D, Hk, 64, (uint32_t)D) &&
               make_tmap_bf16_3d(&m[5], vlo_map, L.npad, D, Hk, 64, (uint32_t)D);
    if (!okm) return fail(STA_ERR_CUDA, "sta_dca_forward: cuTensorMapEncodeTiled failed");
    DParams p{};
    p.BH = H;
    p.H = (int)H;
    p.Hkv = (int)Hk;
    p.N = N;
    p.Nq = Nq;
    p.qbase = qbase;
    p.qb0 = (int)(qbase / BM);
    p.nqb = (int)((Nq + BM - 1) / BM);
    p.dca_L = dL;
    p.c_log2 = a->sm_scale * 1.4426950408889634f;
    p.out = out;
    p.out_f32 = f32 ? 1 : 0;
    p.err = device_error_word();
    p.limit_ns = 4000000000ull;
    const int64_t total = H * p.nqb;
    const int grid = (int)(total < nsm ? total : nsm);
    cudaError_t e;
    if (D == 128) e = f32 ? launch_dca_kernel<128, true>(m, p, grid, st) : launch_dca_kernel<128, false>(m, p, grid, st);
    else e = f32 ? launch_dca_kernel<64, true>(m, p, grid, st) : launch_dca_kernel<64, false>(m, p, grid, st);
    if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  }
  return STA_OK;
}

}  // extern "C"
