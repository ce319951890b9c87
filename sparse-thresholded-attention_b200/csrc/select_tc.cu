// Exact-max two-pass selection (Kernel A) on 5th-generation tensor cores.
//
// Reference: _select_vote_kernel, shared_selection_triton_exact_2.py:50-140 (votes, row
// counts, margin / expmass weighted votes) and _select_bits_kernel,
// shared_selection_triton_perquery.py:119-218 (packed per-query keep bits, tile 32).
//
// Work item: 128 consecutive query rows of one q head (query block qb), against all causal
// 256-key blocks [0, ceil((qb+1)*128 / 256) * 256).  Pass 1 sweeps the blocks for the exact row max m_i; pass 2
// sweeps them again and evaluates keep = s >= m_i - tau_h & causal & row < N per (query, key).
//
// Scores are s = (Qr . Kr) * sm_scale with Qr / Kr the fp32 rotated rows, formed as three
// bf16 tcgen05 products (hi*hi + hi*lo + lo*hi, fp32 accumulation in TMEM); both passes issue
// the identical instruction sequence, so pass 2 reproduces pass 1's scores bit for bit.
//
// Roles (576 threads, one CTA per SM, persistent over a longest-first static schedule):
//   warps 0-15 epilogue: warps w, w+4, w+8, w+12 share TMEM lane quadrant w%4 (rows
//              32(w%4)..+31) and split each block's 256 columns; row max in pass 1;
//              keep / warp-ballot votes / per-query bits / weighted votes in pass 2;
//   warp 16    TMA producer (Q tile once per item, K blocks through an NSTAGE smem ring);
//   warp 17    MMA issuer (one thread), M=128 N=256 K=16, 2 TMEM accumulator slots of 256
//              columns; the K ring holds one bf16 piece (hi or lo) of a key block per stage.
// All waits are bounded; on expiry the kernel records STA_ERR_TIMEOUT and unwinds.
#include <cuda_fp16.h>
#include "common.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int BM = 128;       // query rows per item == TMEM lanes
constexpr int BN = 256;       // keys per block == MMA N
constexpr int NACC = 2;       // accumulator slots (2 x 256 fp32 columns = all 512 TMEM columns)
#ifndef STA_SELECT_PREFETCH_PARTS
#define STA_SELECT_PREFETCH_PARTS 2
#endif
#ifndef STA_SELECT_EPI_WARPS
#define STA_SELECT_EPI_WARPS 16
#endif
constexpr int kEpi = STA_SELECT_EPI_WARPS * 32;  // epilogue threads: kParts warps per TMEM lane
constexpr int kParts = kEpi / 128;               // quadrant, each taking BN / kParts columns
constexpr int kChunks = BN / 32 / kParts;        // 32-column chunks per warp and key block
constexpr int kThreads = kEpi + 64;
constexpr int kTileBytes = BM * 128;   // 128 query rows x 64 bf16 (one 128-byte swizzle chunk)
constexpr int kKTileBytes = BN * 128;  // 256 key rows x 64 bf16

template <int D>
struct Cfg {
  static constexpr int NC = D / 64;
  static constexpr int Q_BYTES = 2 * NC * kTileBytes;
  // one stage holds ONE bf16 piece (hi or lo) of a 256-key block; a block uses two stages
  static constexpr int STAGE_BYTES = NC * kKTileBytes;
  static constexpr int NSTAGE = (D == 64) ? 4 : 2;
  static constexpr int RED_WORDS = 2 * 4 * BN;   // [buffer][quadrant][column]
  static constexpr int HIST_WORDS = 2 * 65;     // per-tile vote histograms of an item (T 64 / 128)
  static constexpr int SMEM = 1024 + Q_BYTES + NSTAGE * STAGE_BYTES + 2 * RED_WORDS * 4 + 2 * kEpi * 4 +
                              HIST_WORDS * 4 + 512;
};

struct Params {
  int64_t BH;
  int H, Hkv;
  int64_t N;            // keys (= last query position + 1)
  int64_t Nq;           // query rows held by Q (positions qbase .. N-1)
  int64_t qbase;        // absolute position of query row 0 (multiple of BM)
  int qb0;              // qbase / BM
  int T;
  int nqb;              // local query blocks
  int npass;
  int wmode;
  float sm_scale;
  const float* tau;
  uint8_t* votes;
  float* wvotes;
  uint32_t* bits;
  float* row_max;
  int32_t* row_count;
  int* err;
  int64_t head_stride;  // compact per-head stride
  int64_t dca_L;        // > 0: Dual Chunk Attention selection geometry, chunk_len (multiple of 256)
  uint8_t* block_max;   // PQ-Stream block maxima (tile 32) or null
  int bmax_bn;
  int64_t bmax_head_stride;
  uint64_t limit_ns;    // bound of every mbarrier wait
  uint32_t* vote_hist;  // (BH, nt local, T + 1) nonzero-vote histograms (T 64 / 128) or null
  // screened scoring (SCR kernels): canonical bf16 pieces for exact recomputation, per-row
  // query norms and per-32-key-chunk key norm maxima of the fp16 screening operands
  const __nv_bfloat16 *qh, *ql, *kh, *kl;
  const float2* qnorm;  // (BH, Nq): ||q16||, ||q' - q16|| (max over DCA planes)
  const float2* knorm;  // (BHk): max ||k16||, max ||k' - k16|| over the head's keys
  int64_t nkc;          // 32-key chunks per kv head
};

// Which rotated Q plane scores key block kb of query block qb: 0 = plain (or same DCA chunk),
// 1 = the previous DCA chunk, 2 = older DCA chunks.
__device__ __forceinline__ int q_plane(const Params& p, int qb, int kb) {
  if (p.dca_L <= 0) return 0;
  const int64_t rel = ((int64_t)qb * BM) / p.dca_L - ((int64_t)kb * BN) / p.dca_L;
  return rel <= 0 ? 0 : (rel == 1 ? 1 : 2);
}

// lane l receives sum over the warp's lanes of v[l] (fixed butterfly order, 31 shuffles)
__device__ __forceinline__ float transpose_reduce32(float (&v)[32]) {
  const int l = lane_id();
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool up = (l & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = up ? v[i] : v[i + s];
      const float keep = up ? v[i + s] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// Smallest fp32 x with fl(x * sm) >= thr (sm > 0).  fl(x * sm) is non-decreasing in x, so
// "fl(acc * sm) >= thr" is exactly "acc >= x": the keep test can run on raw accumulators.
__device__ __forceinline__ float raw_threshold(float thr, float sm) {
  if (!(thr > -INFINITY)) return -INFINITY;
  if (thr == INFINITY) return INFINITY;
  float x = __fdiv_rn(thr, sm);
  for (int i = 0; i < 8 && __fmul_rn(x, sm) >= thr; ++i) x = nextafterf(x, -INFINITY);
  for (int i = 0; i < 16 && __fmul_rn(x, sm) < thr; ++i) x = nextafterf(x, INFINITY);
  return x;
}

// Canonical exact score of one (query row, key) pair in raw accumulator units: the three
// products hi*hi + hi*lo + lo*hi of the bf16 pieces, lane l taking dims [l*E, l*E+E) in a
// fixed FMA order and a xor butterfly summing the lanes (every lane ends with the identical
// value).  Every pass that needs an exact score calls this, so they agree bit for bit.
template <int D>
__device__ __forceinline__ float exact_score(const __nv_bfloat16* qh, const __nv_bfloat16* ql,
                                             const __nv_bfloat16* kh, const __nv_bfloat16* kl) {
  constexpr int E = D / 32;
  const int l = lane_id();
  __nv_bfloat16 a[E], b[E], c[E], d[E];
  if constexpr (E == 4) {
    *reinterpret_cast<uint2*>(a) = __ldg(reinterpret_cast<const uint2*>(qh) + l);
    *reinterpret_cast<uint2*>(b) = __ldg(reinterpret_cast<const uint2*>(ql) + l);
    *reinterpret_cast<uint2*>(c) = __ldg(reinterpret_cast<const uint2*>(kh) + l);
    *reinterpret_cast<uint2*>(d) = __ldg(reinterpret_cast<const uint2*>(kl) + l);
  } else {
    *reinterpret_cast<uint32_t*>(a) = __ldg(reinterpret_cast<const unsigned int*>(qh) + l);
    *reinterpret_cast<uint32_t*>(b) = __ldg(reinterpret_cast<const unsigned int*>(ql) + l);
    *reinterpret_cast<uint32_t*>(c) = __ldg(reinterpret_cast<const unsigned int*>(kh) + l);
    *reinterpret_cast<uint32_t*>(d) = __ldg(reinterpret_cast<const unsigned int*>(kl) + l);
  }
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float x = __bfloat162float(a[e]), y = __bfloat162float(b[e]);
    const float u = __bfloat162float(c[e]), w = __bfloat162float(d[e]);
    acc = __fmaf_rn(x, u, acc);
    acc = __fmaf_rn(x, w, acc);
    acc = __fmaf_rn(y, u, acc);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  return acc;
}

// Warp-collective exact scoring of the pairs (this lane's query row, key j) for the bits j of
// pend; q* point at the warp's first query row, k* at the chunk's first key.  MAX: returns the
// max of x and the exact scores; otherwise returns (as float bits) the bits whose exact score
// reaches x (the raw threshold).  Out of line: it runs for few chunks, and keeping its
// registers out of the epilogue's hot loop avoids spills there.
template <int D, bool MAX>
__device__ __noinline__ float resolve_pairs(uint32_t pend, float x, const __nv_bfloat16* qh,
                                            const __nv_bfloat16* ql, const __nv_bfloat16* kh,
                                            const __nv_bfloat16* kl) {
  const int lane = lane_id();
  float mx = x;
  uint32_t res = 0;
  for (;;) {
    uint32_t lanes = __ballot_sync(0xffffffffu, pend != 0u);
    if (!lanes) break;
    const int myj = pend ? __ffs(pend) - 1 : 0;
    while (lanes) {
      const int src = __ffs(lanes) - 1;
      lanes &= lanes - 1;
      const int j = __shfl_sync(0xffffffffu, myj, src);
      const float sc = exact_score<D>(qh + (int64_t)src * D, ql + (int64_t)src * D,
                                      kh + (int64_t)j * D, kl + (int64_t)j * D);
      if (lane == src) {
        if (MAX) mx = fmaxf(mx, sc);
        else if (sc >= x) res |= 1u << j;
      }
    }
    if (pend) pend &= pend - 1u;
  }
  return MAX ? mx : __uint_as_float(res);
}

// Upper bound of |screened score - canonical score| for a query row with fp16-operand norms
// (qa, qr) against a key chunk with (ka, kr):  q' = q16 + rq, k' = k16 + rk gives
// q'.k' - q16.k16 = q16.rk + rq.k16 + rq.rk (Cauchy-Schwarz per term); the 2^-13 |q16||k16|
// slack covers the dropped lo*lo product (<= 2^-16), fp32 accumulation of the tensor-core sum
// (<= 128 * 2^-24) and of the canonical FMA chain (<= 384 * 2^-24), all relative to |q||k|.
__device__ __forceinline__ float screen_bound(float qa, float qr, float ka, float kr) {
  return __fmaf_ru(qa, kr, __fmaf_ru(qr, ka, __fmaf_ru(qr, kr, __fmul_ru(1.220703125e-4f, __fmul_ru(qa, ka)))));
}

// first canonical query row (q_hi / q_lo row index) of an epilogue warp's 32 rows
__device__ __forceinline__ int64_t qrow_of(const Params& p, int qb, int kb, int64_t bh, int quad) {
  return ((int64_t)q_plane(p, qb, kb) * p.BH + bh) * p.Nq + ((int64_t)qb * BM - p.qbase) + quad * 32;
}

__device__ __forceinline__ void decode_item(int64_t w, const Params& p, int64_t& bh, int& qb,
                                            int64_t& kvh) {
  qb = p.nqb - 1 - (int)(w / p.BH) + p.qb0;  // absolute query block
  bh = w % p.BH;
  const int G = p.H / p.Hkv;
  kvh = (bh / p.H) * p.Hkv + (bh % p.H) / G;
}

template <int D, bool SCR>
__global__ void __launch_bounds__(kThreads, 1)
select_kernel(const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
              const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
              const Params p) {
  using C = Cfg<D>;
  // screened: one fp16 operand piece per block and three passes (screened max, exact max of
  // the candidates, votes); exact: two bf16 pieces, three products, two passes
  constexpr int kPieces = SCR ? 1 : 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = base + C::Q_BYTES;
  uint32_t* s_vote = reinterpret_cast<uint32_t*>(sK + C::NSTAGE * C::STAGE_BYTES);
  float* s_w = reinterpret_cast<float*>(s_vote + C::RED_WORDS);
  float* s_rowx = s_w + C::RED_WORDS;                                  // [kParts][128 rows]
  int* s_rowc = reinterpret_cast<int*>(s_rowx + kEpi);                  // [kParts][128 rows]
  uint32_t* s_hist = reinterpret_cast<uint32_t*>(s_rowc + kEpi);       // [BM / T][T + 1]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_hist + C::HIST_WORDS);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_empty = k_full + C::NSTAGE;
  uint64_t* acc_full = k_empty + C::NSTAGE;
  uint64_t* acc_empty = acc_full + NACC;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acc_empty + NACC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(acc_full + a, 1);
      mbar_init(acc_empty + a, kEpi);
    }
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

  if (warp == kEpi / 32) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_qhi);
      prefetch_tmap(&tm_qlo);
      prefetch_tmap(&tm_khi);
      prefetch_tmap(&tm_klo);
      uint32_t kc = 0, qloads = 0;
      int it = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
        int64_t bh, kvh;
        int qb;
        decode_item(w, p, bh, qb, kvh);
        const int nb = qb / 2 + 1;  // 256-key blocks covering the item's causal keys
        int cur = -1;               // Q plane resident in smem
        for (int pass = 0; pass < p.npass && ok; ++pass) {
          for (int kb = 0; kb < nb && ok; ++kb) {
            const int plane = q_plane(p, qb, kb);
            if (plane != cur) {
              if (qloads > 0 &&
                  !mbar_wait(q_empty, (qloads - 1) & 1, s_abort, p.err, kErrTimeoutQ, p.limit_ns)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(q_full, SCR ? C::Q_BYTES / 2 : C::Q_BYTES);
              const int z = (int)(plane * p.BH + bh);
              for (int c = 0; c < C::NC; ++c) {
                const int qrow = (qb - p.qb0) * BM;  // local row in the Q slab
                tma_load_3d(sQ + c * kTileBytes, &tm_qhi, q_full, c * 64, qrow, z);
                if (!SCR) tma_load_3d(sQ + (C::NC + c) * kTileBytes, &tm_qlo, q_full, c * 64, qrow, z);
              }
              ++qloads;
              cur = plane;
            }
            for (int piece = 0; piece < kPieces; ++piece, ++kc) {  // hi piece, then lo piece
              const uint32_t s = kc % C::NSTAGE, r = kc / C::NSTAGE;
              if (r > 0 && !mbar_wait(k_empty + s, (r - 1) & 1, s_abort, p.err, kErrTimeoutEmpty, p.limit_ns)) {
                ok = false;
                break;
              }
              uint8_t* st = sK + s * C::STAGE_BYTES;
              const CUtensorMap* tm = piece == 0 ? &tm_khi : &tm_klo;
              mbar_arrive_expect_tx(k_full + s, C::STAGE_BYTES);
              for (int c = 0; c < C::NC; ++c)
                tma_load_3d(st + c * kKTileBytes, tm, k_full + s, c * 64, kb * BN, (int)kvh);
            }
          }
        }
      }
    }
  } else if (warp == kEpi / 32 + 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = SCR ? idesc_f16_f32(BM, BN) : idesc_bf16_f32(BM, BN);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      uint32_t kc = 0, ac = 0, qloads = 0;
      int it = 0;
      bool ok = true;
      for (int64_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
        int64_t bh, kvh;
        int qb;
        decode_item(w, p, bh, qb, kvh);
        const int nb = qb / 2 + 1;
        int cur = -1;
        for (int pass = 0; pass < p.npass && ok; ++pass) {
          for (int kb = 0; kb < nb; ++kb, ++ac) {
            const int plane = q_plane(p, qb, kb);
            if (plane != cur) {
              // the resident Q tile is released once every MMA issued so far has completed
              if (qloads > 0) umma_commit(q_empty);
              if (!mbar_wait(q_full, qloads & 1, s_abort, p.err, kErrTimeoutQ, p.limit_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              ++qloads;
              cur = plane;
            }
            const uint32_t slot = ac % NACC, use = ac / NACC;
            if (use > 0 && !mbar_wait(acc_empty + slot, (use - 1) & 1, s_abort, p.err,
                                      kErrTimeoutAcc, p.limit_ns)) {
              ok = false;
              break;
            }
            const uint32_t d_tmem = tmem_base + slot * BN;
            uint32_t acc = 0;
            // piece 0 (K hi): Qhi.Khi + Qlo.Khi ; piece 1 (K lo): Qhi.Klo.  Screened: the one
            // fp16 product Q16.K16
            for (int piece = 0; piece < kPieces; ++piece, ++kc) {
              const uint32_t s = kc % C::NSTAGE, r = kc / C::NSTAGE;
              if (!mbar_wait(k_full + s, r & 1, s_abort, p.err, kErrTimeoutK, p.limit_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t st = k_addr + s * C::STAGE_BYTES;
#pragma unroll
              for (int c = 0; c < C::NC; ++c) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  const uint32_t qoff = c * kTileBytes + kk * 32;
                  const uint64_t qh = sw128_kmajor_desc(q_addr + qoff);
                  const uint64_t kd = sw128_kmajor_desc(st + c * kKTileBytes + kk * 32);
                  umma_bf16(d_tmem, qh, kd, idesc, acc);
                  acc = 1;
                  if (!SCR && piece == 0) {
                    const uint64_t ql = sw128_kmajor_desc(q_addr + C::NC * kTileBytes + qoff);
                    umma_bf16(d_tmem, ql, kd, idesc, 1);
                  }
                }
              }
              umma_commit(k_empty + s);
            }
            if (!ok) break;
            umma_commit(acc_full + slot);
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Thread r owns accumulator row r.  Scores are compared in raw accumulator units against a
    // per-row threshold derived exactly (see raw_threshold), so no per-element scaling is
    // needed for the keep decision.
    // Exact kernels: pass 0 keeps the raw row max, pass 1 votes.
    // Screened kernels (SCR): the accumulator holds the fp16 product s16 = Q16.K16, within
    // Bc = screen_bound(row norms, the kv head's maximum key norms) of the canonical score.
    // Pass 0: max16 = max of s16, so the exact max is >= max16 - Bc.  Pass 1: every key with
    // s16 >= max16 - 2 Bc is scored exactly (exact_score); their max is the exact row max.
    // Pass 2: s16 > thr + Bc keeps, s16 < thr - Bc drops, the keys in between are scored exactly.
    constexpr int kVotePass = SCR ? 2 : 1;
    const int quad = warp & 3;             // TMEM lane quadrant
    const int part = warp >> 2;            // which kChunks of the block's eight 32-column chunks
    const int row = quad * 32 + lane;
    const int64_t nt = (p.N + p.T - 1) / p.T;
    const int quads_per_tile = p.T / 32;
    const int max_pass = SCR ? 1 : 0;      // the pass after which the exact row max is known
    uint32_t ac = 0;
    int rb = 0;
    bool ok = true;
    // After a failed wait (ok == false) a warp keeps walking the same schedule without touching
    // TMEM or memory, so every epilogue warp still reaches every named barrier.
    for (int64_t w = blockIdx.x; w < total; w += gridDim.x) {
      int64_t bh, kvh;
      int qb;
      decode_item(w, p, bh, qb, kvh);
      const int64_t q0 = (int64_t)qb * BM;
      const int64_t qp = q0 + row;
      const bool row_ok = qp < p.N;
      const float tau_h = __ldg(p.tau + (bh % p.H));
      const int nb = qb / 2 + 1;
      float mraw = -INFINITY, m = -INFINITY, thr = -INFINITY, thr_raw = INFINITY;
      float thr_pad = 0.f;
      float Bc = 0.f;  // screen bound of this row against every key of the head (SCR)
      if (SCR && row_ok) {
        const float2 qn = __ldg(p.qnorm + bh * p.Nq + (qp - p.qbase));
        const float2 kn = __ldg(p.knorm + kvh);
        Bc = screen_bound(qn.x, qn.y, kn.x, kn.y);
      }
      float cthr = -INFINITY, hi_thr = INFINITY, lo_thr = INFINITY;
      int cnt = 0;
      for (int pass = 0; pass < p.npass; ++pass) {
        if (pass == kVotePass) {
          if (p.vote_hist && p.T != 32) {
            // this thread's bin of its tile's histogram (ordered before the first atomics by the
            // tile's combine barrier)
            const int g = quad / quads_per_tile;
            const int ti = (part * quads_per_tile + quad % quads_per_tile) * 32 + lane;
            if (ti <= p.T) s_hist[g * (p.T + 1) + ti] = 0u;
          }
          thr = __fsub_rn(m, tau_h);
          thr_raw = row_ok ? raw_threshold(thr, p.sm_scale) : INFINITY;
          // covers the rounding of thr_raw +- Bc
          thr_pad = fabsf(thr_raw) < INFINITY ? 1.9073486e-6f * fabsf(thr_raw) : 0.f;
          hi_thr = __fadd_ru(__fadd_ru(thr_raw, Bc), thr_pad);
          lo_thr = __fsub_rd(__fsub_rd(thr_raw, Bc), thr_pad);
        }
        for (int kb = 0; kb < nb; ++kb, ++ac) {
          const uint32_t slot = ac % NACC, use = ac / NACC;
          int bad = 0;
          if (ok && lane == 0) bad = !mbar_wait(acc_full + slot, use & 1, s_abort, p.err, kErrTimeoutAcc, p.limit_ns);
          if (__shfl_sync(0xffffffffu, bad, 0)) ok = false;
          if (ok) {
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + slot * BN;
            // with 8 epilogue warps the next chunk's load is kept in flight (vn); with 16 the
            // other warps of the quadrant hide its latency and the registers go to occupancy
            constexpr bool kPrefetch = kParts <= STA_SELECT_PREFETCH_PARTS;
            float v[32], vn[32];  // vn unused (eliminated) without prefetch
            tmem_ld32(taddr + part * (BN / kParts), v);
            tmem_wait_ld();
            int rc_even = 0;  // kept count of the previous (even) chunk, for 64-key blocks
#pragma unroll 1
            for (int cc = 0; cc < kChunks; ++cc) {
              const int ch = part * kChunks + cc;
              if constexpr (kPrefetch) {
                if (cc + 1 < kChunks) tmem_ld32(taddr + (ch + 1) * 32, vn);  // next chunk in flight
              } else if (cc > 0) {
                tmem_ld32(taddr + ch * 32, v);
                tmem_wait_ld();
              }
              const int64_t kbase = (int64_t)kb * BN + ch * 32;
              // causal mask of this row over the chunk's 32 keys (all ones off the diagonal)
              const int64_t lim = qp - kbase;
              const uint32_t cmask = lim >= 31 ? 0xffffffffu : (lim < 0 ? 0u : ((2u << lim) - 1u));
              if (pass == 0) {
                float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                if (cmask == 0xffffffffu) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) m4[j & 3] = fmaxf(m4[j & 3], v[j]);
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    m4[j & 3] = fmaxf(m4[j & 3], ((cmask >> j) & 1u) ? v[j] : -INFINITY);
                }
                const float cm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
                mraw = fmaxf(mraw, cm);
              } else if (SCR && pass == 1) {
                // candidates: s16 >= (max16 - Bc) - Bc; most chunks have none (chunk max first)
                float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int j = 0; j < 32; ++j) m4[j & 3] = fmaxf(m4[j & 3], v[j]);
                uint32_t cand = 0;
                if (fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) >= cthr) {
#pragma unroll
                  for (int j = 0; j < 32; ++j) cand |= (v[j] >= cthr ? 1u : 0u) << j;
                }
                cand &= cmask;
                if (!row_ok) cand = 0;
                if (__any_sync(0xffffffffu, cand != 0u)) {
                  const int64_t qo = qrow_of(p, qb, kb, bh, quad) * D, ko = (kvh * p.N + kbase) * D;
                  mraw = resolve_pairs<D, true>(cand, mraw, p.qh + qo, p.ql + qo, p.kh + ko, p.kl + ko);
                }
              } else {
                uint32_t word;
                if constexpr (SCR) {
                  const float hi = hi_thr, lo = lo_thr;
                  uint32_t k4[4] = {0u, 0u, 0u, 0u}, b4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    k4[j & 3] |= (v[j] > hi ? 1u : 0u) << j;
                    b4[j & 3] |= (v[j] >= lo ? 1u : 0u) << j;
                  }
                  word = (k4[0] | k4[1]) | (k4[2] | k4[3]);
                  uint32_t band = ((b4[0] | b4[1]) | (b4[2] | b4[3])) & ~word & cmask;
                  if (!row_ok) band = 0;
                  if (__any_sync(0xffffffffu, band != 0u)) {
                    const int64_t qo = qrow_of(p, qb, kb, bh, quad) * D, ko = (kvh * p.N + kbase) * D;
                    word |= __float_as_uint(resolve_pairs<D, false>(band, thr_raw, p.qh + qo, p.ql + qo,
                                                                    p.kh + ko, p.kl + ko));
                  }
                } else {
                  uint32_t w4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                  for (int j = 0; j < 32; ++j) w4[j & 3] |= (v[j] >= thr_raw ? 1u : 0u) << j;
                  word = (w4[0] | w4[1]) | (w4[2] | w4[3]);
                }
                word &= cmask;
                if (!row_ok) word = 0;
                cnt += __popc(word);
                const uint32_t colw = transpose32(word);  // lane j: keep bits of column j, bit r = row r
                float myw = 0.f;
                // weighted votes only where some row of the warp keeps a key of this chunk (the
                // kept sets are sparse: most chunks have none, and their sums are exactly 0)
                if (!SCR && p.wmode != 0 && __any_sync(0xffffffffu, word != 0u)) {
                  // v is not read again for this chunk: reuse it for the per-key weights
#pragma unroll
                  for (int j = 0; j < 32; ++j) {
                    const float sc = __fmul_rn(v[j], p.sm_scale);
                    const float c = p.wmode == 1 ? __fsub_rn(sc, thr) : expf(__fsub_rn(sc, m));
                    v[j] = ((word >> j) & 1u) ? c : 0.f;
                  }
                  myw = transpose_reduce32(v);
                }
                if (p.T == 32) {
                  // a 32-query tile is exactly this warp's 32 rows: lane j already holds the
                  // tile's votes / bits / weighted vote of key kbase + j -- store them directly
                  const int64_t tg = q0 / 32 + quad;
                  const int64_t kj = kbase + lane;
                  if (tg < nt && kj < min((tg + 1) * 32, p.N)) {
                    const int64_t off =
                        bh * p.head_stride + tri_tile_offset(tg - p.qbase / 32, 32, p.qbase) + kj;
                    if (p.votes) p.votes[off] = (uint8_t)__popc(colw);
                    if (p.wmode != 0 && p.wvotes) p.wvotes[off] = myw;
                    if (p.bits) p.bits[off] = colw;
                  }
                  if (p.block_max) {
                    // PQ-Stream: max over the tile's rows of the kept count of each key block
                    // (32 keys, or 64 = this chunk and the previous one of the same warp)
                    int c = __popc(word);
                    const bool wide = p.bmax_bn == 64;
                    if (wide && !(cc & 1)) {
                      rc_even = c;
                    } else {
                      if (wide) c += rc_even;
#pragma unroll
                      for (int o = 16; o >= 1; o >>= 1) c = max(c, __shfl_xor_sync(0xffffffffu, c, o));
                      const int64_t kb0 = wide ? kbase - 32 : kbase;
                      if (lane == 0 && tg < nt && kb0 < min((tg + 1) * 32, p.N))
                        p.block_max[bh * p.bmax_head_stride +
                                    tri_tile_offset(tg - p.qbase / 32, 1, p.qbase / 32) + kb0 / 32] =
                            (uint8_t)c;
                    }
                  }
                } else {
                  const int o = rb * (4 * BN) + quad * BN + ch * 32 + lane;
                  s_vote[o] = __popc(colw);
                  s_w[o] = myw;
                }
              }
              if constexpr (kPrefetch) {
                if (cc + 1 < kChunks) {
                  tmem_wait_ld();
#pragma unroll
                  for (int j = 0; j < 32; ++j) v[j] = vn[j];
                }
              }
            }
            tc_fence_before();
            mbar_arrive(acc_empty + slot);
          }  // ok
          if (pass == kVotePass && p.T != 32) {
            // combine the quadrants of each query tile and store compact votes / wvotes: the
            // warps of one tile's quadrants meet at their own barrier (ids 4, 5)
            const int g = quad / quads_per_tile;                 // == tile of the item
            named_bar_sync(4 + g, quads_per_tile * kParts * 32);
            const int64_t tg = q0 / p.T + g;
            // the tile's quads_per_tile * kParts warps cover the block's columns (one pass with
            // 16 epilogue warps and 64-query tiles)
            for (int col = (part * quads_per_tile + quad % quads_per_tile) * 32 + lane; col < BN;
                 col += quads_per_tile * kParts * 32) {
              const int64_t kj = (int64_t)kb * BN + col;
              if (!(ok && tg < nt && kj < min((tg + 1) * (int64_t)p.T, p.N))) continue;
              uint32_t vs = 0;
              float wsum = 0.f;
              for (int qq = g * quads_per_tile; qq < (g + 1) * quads_per_tile; ++qq) {
                const int o = rb * (4 * BN) + qq * BN + col;
                vs += s_vote[o];
                wsum += s_w[o];
              }
              const int64_t off =
                  bh * p.head_stride + tri_tile_offset(tg - p.qbase / p.T, p.T, p.qbase) + kj;
              if (p.votes) p.votes[off] = (uint8_t)vs;
              if (p.wmode != 0 && p.wvotes) p.wvotes[off] = wsum;
              if (p.vote_hist && vs) atomicAdd(&s_hist[g * (p.T + 1) + vs], 1u);
            }
            rb ^= 1;
          }
        }
        if (SCR && pass == 0) {
          // screened max of the row: max16 - Bc bounds the exact max from below, so a key can
          // be the exact max only if s16 >= max16 - 2 Bc
          s_rowx[part * 128 + row] = mraw;
          named_bar_sync(3, kEpi);
          float mh = -INFINITY;
#pragma unroll
          for (int q2 = 0; q2 < kParts; ++q2) mh = fmaxf(mh, s_rowx[q2 * 128 + row]);
          named_bar_sync(3, kEpi);
          cthr = __fsub_rd(__fsub_rd(mh, Bc), Bc);
          mraw = -INFINITY;  // pass 1 collects the exact max
        }
        if (pass == max_pass) {
          // the column parts of each row meet: exact row max, then scale once
          s_rowx[part * 128 + row] = mraw;
          named_bar_sync(3, kEpi);
#pragma unroll
          for (int q2 = 0; q2 < kParts; ++q2) mraw = fmaxf(mraw, s_rowx[q2 * 128 + row]);
          named_bar_sync(3, kEpi);
          m = __fmul_rn(mraw, p.sm_scale);  // scaling is monotone: max commutes with it
        }
      }
      s_rowc[part * 128 + row] = cnt;
      named_bar_sync(3, kEpi);
      cnt = 0;
#pragma unroll
      for (int q2 = 0; q2 < kParts; ++q2) cnt += s_rowc[q2 * 128 + row];
      named_bar_sync(3, kEpi);
      if (ok && part == 0 && row_ok) {
        if (p.row_max) p.row_max[bh * p.Nq + (qp - p.qbase)] = m;
        if (p.row_count && p.npass > kVotePass) p.row_count[bh * p.Nq + (qp - p.qbase)] = cnt;
      }
      if (p.vote_hist && p.T != 32 && p.npass > kVotePass) {
        // the same thread that zeroed a bin flushes it (the barrier above ordered the atomics)
        const int g = quad / quads_per_tile;
        const int ti = (part * quads_per_tile + quad % quads_per_tile) * 32 + lane;
        const int64_t tg = q0 / p.T + g;
        if (ok && ti <= p.T && tg < nt)
          p.vote_hist[(bh * ((p.Nq + p.T - 1) / p.T) + (tg - p.qbase / p.T)) * (p.T + 1) + ti] =
              s_hist[g * (p.T + 1) + ti];
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  if (*s_abort) {
    // let in-flight asynchronous copies / MMAs drain before the CTA releases its resources
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, 512);
}

// Screening operands of the screened select kernel: q16 = fp16(q_hi + q_lo) (saturated to
// the fp16 range; the residual then only widens the bound), the row norms ||q16|| and
// ||q' - q16|| (max over the DCA planes), k16 likewise and per kv head the maxima of the key
// norms (kn zeroed by the caller).  One warp per query row (all planes) or per 32-key chunk;
// lane l owns dims [l*E, l*E+E).
template <int D>
__global__ void __launch_bounds__(256)
select_prep_kernel(const __nv_bfloat16* __restrict__ qh, const __nv_bfloat16* __restrict__ ql,
                   int64_t qrows, int qplanes, const __nv_bfloat16* __restrict__ kh,
                   const __nv_bfloat16* __restrict__ kl, int64_t BHk, int64_t N, int64_t nkc,
                   __half* __restrict__ q16, __half* __restrict__ k16, float2* __restrict__ qn,
                   float2* __restrict__ kn) {
  constexpr int E = D / 32;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int l = threadIdx.x & 31;
  // squared norms of the fp16 part and of the residual of one row, summed over the warp
  auto row = [&](const __nv_bfloat16* h, const __nv_bfloat16* lo, __half* o, float& na, float& nr) {
    __nv_bfloat16 a[E], b[E];
    __half c[E];
    if constexpr (E == 4) {
      *reinterpret_cast<uint2*>(a) = *reinterpret_cast<const uint2*>(h + l * E);
      *reinterpret_cast<uint2*>(b) = *reinterpret_cast<const uint2*>(lo + l * E);
    } else {
      *reinterpret_cast<uint32_t*>(a) = *reinterpret_cast<const uint32_t*>(h + l * E);
      *reinterpret_cast<uint32_t*>(b) = *reinterpret_cast<const uint32_t*>(lo + l * E);
    }
    float sa = 0.f, sr = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float x = __fadd_rn(__bfloat162float(a[e]), __bfloat162float(b[e]));  // exact
      const float xs = fminf(fmaxf(x, -65504.f), 65504.f);
      c[e] = __float2half_rn(xs);
      const float f = __half2float(c[e]);
      const float r = __fsub_rn(x, f);
      sa = __fmaf_ru(f, f, sa);
      sr = __fmaf_ru(r, r, sr);
    }
    if constexpr (E == 4) *reinterpret_cast<uint2*>(o + l * E) = *reinterpret_cast<uint2*>(c);
    else *reinterpret_cast<uint32_t*>(o + l * E) = *reinterpret_cast<uint32_t*>(c);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      sa = __fadd_ru(sa, __shfl_xor_sync(0xffffffffu, sa, off));
      sr = __fadd_ru(sr, __shfl_xor_sync(0xffffffffu, sr, off));
    }
    na = __fsqrt_ru(sa);
    nr = __fsqrt_ru(sr);
  };
  if (gw < qrows) {
    float ma = 0.f, mr = 0.f;
    for (int pl = 0; pl < qplanes; ++pl) {
      const int64_t o = ((int64_t)pl * qrows + gw) * D;
      float na, nr;
      row(qh + o, ql + o, q16 + o, na, nr);
      ma = fmaxf(ma, na);
      mr = fmaxf(mr, nr);
    }
    if (l == 0) qn[gw] = make_float2(ma, mr);
  } else if (gw < qrows + BHk * nkc) {
    const int64_t c = gw - qrows, h = c / nkc, j0 = (c % nkc) * 32;
    float ma = 0.f, mr = 0.f;
    for (int64_t j = j0; j < j0 + 32 && j < N; ++j) {
      const int64_t o = (h * N + j) * D;
      float na, nr;
      row(kh + o, kl + o, k16 + o, na, nr);
      ma = fmaxf(ma, na);
      mr = fmaxf(mr, nr);
    }
    if (l == 0) {  // norms are >= 0: their bit patterns order like the values
      atomicMax(reinterpret_cast<int*>(&kn[h].x), __float_as_int(ma));
      atomicMax(reinterpret_cast<int*>(&kn[h].y), __float_as_int(mr));
    }
  }
}

struct ScreenLayout {
  size_t q16, k16, qn, kn, total;
};

ScreenLayout screen_layout(const sta_select_args* a) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int64_t qplanes = a->dca_chunk_len > 0 ? 3 : 1;
  const int64_t nq = a->n - a->q_pos_base;
  const int64_t BH = a->batch * a->n_heads, BHk = a->batch * a->n_kv_heads;
  ScreenLayout L{};
  size_t o = 0;
  L.q16 = o; o += al((size_t)qplanes * BH * nq * a->d * 2);
  L.k16 = o; o += al((size_t)BHk * a->n * a->d * 2);
  L.qn = o; o += al((size_t)BH * nq * 8);
  L.kn = o; o += al((size_t)BHk * 8);
  L.total = o;
  return L;
}

}  // namespace

size_t select_screen_bytes(const sta_select_args* a) {
  if (!a || a->n <= 0 || a->batch <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 ||
      (a->d != 64 && a->d != 128) || a->q_pos_base < 0 || a->q_pos_base >= a->n)
    return 0;
  return screen_layout(a).total;
}

int launch_select(const sta_select_args* a, cudaStream_t stream) {
  if (!a || !a->q_hi || !a->q_lo || !a->k_hi || !a->k_lo || !a->tau)
    return fail(STA_ERR_ARG, "sta_select: null pointer");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_select: d must be 64 or 128");
  if (a->tile != 32 && a->tile != 64 && a->tile != 128)
    return fail(STA_ERR_UNSUPPORTED, "sta_select: tile must be 32, 64 or 128");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_select: n_heads must be a positive multiple of n_kv_heads");
  if (a->bits && a->tile != 32) return fail(STA_ERR_UNSUPPORTED, "sta_select: bits need tile 32");
  if (a->wmode != 0 && !a->wvotes && !a->max_only)
    return fail(STA_ERR_ARG, "sta_select: weighted mode needs wvotes");
  if (a->n <= 0 || a->batch <= 0) return 0;
  if (a->n > (int64_t)1 << 30) return fail(STA_ERR_UNSUPPORTED, "sta_select: n too large");
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n || a->q_pos_base % BM)
    return fail(STA_ERR_UNSUPPORTED, "sta_select: q_pos_base must be a multiple of 128 below n");
  const int64_t nq = a->n - a->q_pos_base;

  const int64_t BH = a->batch * a->n_heads;
  const int64_t BHk = a->batch * a->n_kv_heads;
  CUtensorMap m_qhi, m_qlo, m_khi, m_klo;
  const int64_t qplanes = a->dca_chunk_len > 0 ? 3 : 1;  // DCA: intra / previous / older chunk Q
  bool okm = make_tmap_bf16_3d(&m_qhi, a->q_hi, a->d, nq, qplanes * BH, 64, BM) &&
             make_tmap_bf16_3d(&m_qlo, a->q_lo, a->d, nq, qplanes * BH, 64, BM) &&
             make_tmap_bf16_3d(&m_khi, a->k_hi, a->d, a->n, BHk, 64, BN) &&
             make_tmap_bf16_3d(&m_klo, a->k_lo, a->d, a->n, BHk, 64, BN);
  if (!okm) return fail(STA_ERR_CUDA, "sta_select: cuTensorMapEncodeTiled failed");

  Params p;
  p.BH = BH;
  p.H = (int)a->n_heads;
  p.Hkv = (int)a->n_kv_heads;
  p.N = a->n;
  p.Nq = nq;
  p.qbase = a->q_pos_base;
  p.qb0 = (int)(a->q_pos_base / BM);
  p.T = a->tile;
  p.nqb = (int)((nq + BM - 1) / BM);
  p.npass = a->max_only ? 1 : 2;
  p.wmode = a->max_only ? 0 : a->wmode;
  p.sm_scale = a->sm_scale;
  p.tau = a->tau;
  p.votes = a->max_only ? nullptr : a->votes;
  p.wvotes = a->max_only ? nullptr : a->wvotes;
  p.bits = a->max_only ? nullptr : a->bits;
  p.row_max = a->row_max;
  p.row_count = a->row_count;
  p.err = device_error_word();
  p.head_stride = tri_head_stride(a->n, a->tile, a->q_pos_base);
  p.dca_L = a->dca_chunk_len;
  p.block_max = a->max_only ? nullptr : a->block_max;
  p.bmax_bn = a->block_max_bn;
  p.bmax_head_stride = tri_head_stride((a->n + 31) / 32, 1, a->q_pos_base / 32);
  p.limit_ns = a->wait_limit_ns > 0 ? a->wait_limit_ns : 4000000000ull;
  p.vote_hist = (a->max_only || !a->votes || a->tile == 32) ? nullptr : a->vote_hist;
  if (p.block_max && (a->tile != 32 || (p.bmax_bn != 32 && p.bmax_bn != 64)))
    return fail(STA_ERR_UNSUPPORTED, "sta_select: block_max needs tile 32 and block_max_bn 32 or 64");
  if (p.dca_L > 0 && (p.dca_L % BN)) return fail(STA_ERR_UNSUPPORTED, "sta_select: DCA chunk_len must be a multiple of 256");

  // Screened scoring needs the caller's scratch and plain (unweighted) votes: weighted votes
  // use the score of every kept key, which the exact three-product kernel provides.
  const bool scr = a->screen_ws != nullptr && p.wmode == 0;
  CUtensorMap m_q16, m_k16;
  if (scr) {
    const ScreenLayout SL = screen_layout(a);
    uint8_t* ws = static_cast<uint8_t*>(a->screen_ws);
    if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
      return fail(STA_ERR_ARG, "sta_select: screen_ws must be 256-byte aligned");
    __half* q16 = reinterpret_cast<__half*>(ws + SL.q16);
    __half* k16 = reinterpret_cast<__half*>(ws + SL.k16);
    p.qh = static_cast<const __nv_bfloat16*>(a->q_hi);
    p.ql = static_cast<const __nv_bfloat16*>(a->q_lo);
    p.kh = static_cast<const __nv_bfloat16*>(a->k_hi);
    p.kl = static_cast<const __nv_bfloat16*>(a->k_lo);
    p.qnorm = reinterpret_cast<const float2*>(ws + SL.qn);
    p.knorm = reinterpret_cast<const float2*>(ws + SL.kn);
    p.nkc = (a->n + 31) / 32;
    if (!make_tmap_bf16_3d(&m_q16, q16, a->d, nq, qplanes * BH, 64, BM) ||
        !make_tmap_bf16_3d(&m_k16, k16, a->d, a->n, BHk, 64, BN))
      return fail(STA_ERR_CUDA, "sta_select: cuTensorMapEncodeTiled failed");
    const int64_t warps = BH * nq + BHk * p.nkc;
    cudaMemsetAsync(ws + SL.kn, 0, (size_t)BHk * 8, stream);
    const int64_t blocks = (warps + 7) / 8;
    if (a->d == 128)
      select_prep_kernel<128><<<(unsigned)blocks, 256, 0, stream>>>(
          p.qh, p.ql, BH * nq, (int)qplanes, p.kh, p.kl, BHk, a->n, p.nkc, q16, k16,
          reinterpret_cast<float2*>(ws + SL.qn), reinterpret_cast<float2*>(ws + SL.kn));
    else
      select_prep_kernel<64><<<(unsigned)blocks, 256, 0, stream>>>(
          p.qh, p.ql, BH * nq, (int)qplanes, p.kh, p.kl, BHk, a->n, p.nkc, q16, k16,
          reinterpret_cast<float2*>(ws + SL.qn), reinterpret_cast<float2*>(ws + SL.kn));
    p.npass = a->max_only ? 2 : 3;
  }

  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t total = BH * p.nqb;
  const int grid = (int)(total < nsm ? total : nsm);
  cudaError_t e;
  auto run = [&](auto kern, int smem) {
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (r == cudaSuccess) {
      if (scr) kern<<<grid, kThreads, smem, stream>>>(m_q16, m_qlo, m_k16, m_klo, p);
      else kern<<<grid, kThreads, smem, stream>>>(m_qhi, m_qlo, m_khi, m_klo, p);
    }
    return r;
  };
  if (a->d == 128) e = scr ? run(select_kernel<128, true>, Cfg<128>::SMEM) : run(select_kernel<128, false>, Cfg<128>::SMEM);
  else e = scr ? run(select_kernel<64, true>, Cfg<64>::SMEM) : run(select_kernel<64, false>, Cfg<64>::SMEM);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  return STA_OK;
}

}  // namespace sta
