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
#include "common.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int BM = 128;       // query rows per item == TMEM lanes
constexpr int BN = 256;       // keys per block == MMA N
constexpr int NACC = 2;       // accumulator slots (2 x 256 fp32 columns = all 512 TMEM columns)
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
  static constexpr int SMEM = 1024 + Q_BYTES + NSTAGE * STAGE_BYTES + 2 * RED_WORDS * 4 + 2 * kEpi * 4 + 512;
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

__device__ __forceinline__ void decode_item(int64_t w, const Params& p, int64_t& bh, int& qb,
                                            int64_t& kvh) {
  qb = p.nqb - 1 - (int)(w / p.BH) + p.qb0;  // absolute query block
  bh = w % p.BH;
  const int G = p.H / p.Hkv;
  kvh = (bh / p.H) * p.Hkv + (bh % p.H) / G;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
select_kernel(const __grid_constant__ CUtensorMap tm_qhi, const __grid_constant__ CUtensorMap tm_qlo,
              const __grid_constant__ CUtensorMap tm_khi, const __grid_constant__ CUtensorMap tm_klo,
              const Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = base + C::Q_BYTES;
  uint32_t* s_vote = reinterpret_cast<uint32_t*>(sK + C::NSTAGE * C::STAGE_BYTES);
  float* s_w = reinterpret_cast<float*>(s_vote + C::RED_WORDS);
  float* s_rowx = s_w + C::RED_WORDS;                                  // [kParts][128 rows]
  int* s_rowc = reinterpret_cast<int*>(s_rowx + kEpi);                  // [kParts][128 rows]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_rowc + kEpi);
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
              mbar_arrive_expect_tx(q_full, C::Q_BYTES);
              const int z = (int)(plane * p.BH + bh);
              for (int c = 0; c < C::NC; ++c) {
                const int qrow = (qb - p.qb0) * BM;  // local row in the Q slab
                tma_load_3d(sQ + c * kTileBytes, &tm_qhi, q_full, c * 64, qrow, z);
                tma_load_3d(sQ + (C::NC + c) * kTileBytes, &tm_qlo, q_full, c * 64, qrow, z);
              }
              ++qloads;
              cur = plane;
            }
            for (int piece = 0; piece < 2; ++piece, ++kc) {  // hi piece, then lo piece
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
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
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
            // piece 0 (K hi): Qhi.Khi + Qlo.Khi ; piece 1 (K lo): Qhi.Klo
            for (int piece = 0; piece < 2; ++piece, ++kc) {
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
                  if (piece == 0) {
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
    // needed for the keep decision; pass 1 keeps the raw row max and scales it once.
    const int quad = warp & 3;             // TMEM lane quadrant
    const int part = warp >> 2;            // which kChunks of the block's eight 32-column chunks
    const int row = quad * 32 + lane;
    const int64_t nt = (p.N + p.T - 1) / p.T;
    const int quads_per_tile = p.T / 32;
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
      int cnt = 0;
      for (int pass = 0; pass < p.npass; ++pass) {
        if (pass == 1) {
          thr = __fsub_rn(m, tau_h);
          thr_raw = row_ok ? raw_threshold(thr, p.sm_scale) : INFINITY;
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
            constexpr bool kPrefetch = kParts <= 2;
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
                mraw = fmaxf(mraw, fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
              } else {
                uint32_t w4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                for (int j = 0; j < 32; ++j) w4[j & 3] |= (v[j] >= thr_raw ? 1u : 0u) << j;
                uint32_t word = ((w4[0] | w4[1]) | (w4[2] | w4[3])) & cmask;
                if (!row_ok) word = 0;
                cnt += __popc(word);
                const uint32_t colw = transpose32(word);  // lane j: keep bits of column j, bit r = row r
                float myw = 0.f;
                // weighted votes only where some row of the warp keeps a key of this chunk (the
                // kept sets are sparse: most chunks have none, and their sums are exactly 0)
                if (p.wmode != 0 && __any_sync(0xffffffffu, word != 0u)) {
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
          if (pass == 1 && p.T != 32) {
            // combine the quadrants of each query tile and store compact votes / wvotes: the
            // warps of one tile's quadrants meet at their own barrier (ids 4, 5)
            const int g = quad / quads_per_tile;                 // == tile of the item
            named_bar_sync(4 + g, quads_per_tile * kParts * 32);
            const int col = (part * quads_per_tile + quad % quads_per_tile) * 32 + lane;
            const int64_t tg = q0 / p.T + g;
            const int64_t kj = (int64_t)kb * BN + col;
            if (ok && col < BN && tg < nt && kj < min((tg + 1) * (int64_t)p.T, p.N)) {
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
            }
            rb ^= 1;
          }
        }
        if (pass == 0) {
          // the two column halves of each row meet: exact row max, then scale once
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
        if (p.row_count && p.npass == 2) p.row_count[bh * p.Nq + (qp - p.qbase)] = cnt;
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

}  // namespace

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
  if (p.block_max && (a->tile != 32 || (p.bmax_bn != 32 && p.bmax_bn != 64)))
    return fail(STA_ERR_UNSUPPORTED, "sta_select: block_max needs tile 32 and block_max_bn 32 or 64");
  if (p.dca_L > 0 && (p.dca_L % BN)) return fail(STA_ERR_UNSUPPORTED, "sta_select: DCA chunk_len must be a multiple of 256");

  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t total = BH * p.nqb;
  const int grid = (int)(total < nsm ? total : nsm);
  cudaError_t e;
  if (a->d == 128) {
    e = cudaFuncSetAttribute(select_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<128>::SMEM);
    if (e == cudaSuccess)
      select_kernel<128><<<grid, kThreads, Cfg<128>::SMEM, stream>>>(m_qhi, m_qlo, m_khi, m_klo, p);
  } else {
    e = cudaFuncSetAttribute(select_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg<64>::SMEM);
    if (e == cudaSuccess)
      select_kernel<64><<<grid, kThreads, Cfg<64>::SMEM, stream>>>(m_qhi, m_qlo, m_khi, m_klo, p);
  }
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  return STA_OK;
}

}  // namespace sta
