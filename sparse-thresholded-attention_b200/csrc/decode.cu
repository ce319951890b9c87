// Decode: one query per head against the KV cache (per-query selection + attention).
//
// Reference (torch paths the reference's hooks run by default at decode):
//   PI      _decode_build_sets + _decode_attend_torch, shared_selection_triton_exact.py:464-560
//   RANK    _decode_build_sets_pq + _decode_attend_torch_pq,
//           shared_selection_triton_perquery.py:652-740
//   STREAM  _decode_build_sets_pqs + _decode_attend_torch, pqstream_kernel.py:694-795
//   CHUNK   _decode_build_sets_chunk + _decode_attend_torch_pq,
//           shared_selection_triton_chunked.py:412-483
// and the score kernels _decode_select_kernel (shared_selection_triton_exact.py:211-247 and
// siblings).  Three launches:
//   decode_score_kernel   one warp per key, all q heads of its kv head: raw K row read once
//                         (coalesced), rotated at j * pos_scale_a (cos/sin table or sincosf),
//                         dotted with each rotated query -> scores (heads, m) fp32;
//   decode_select_kernel  one CTA per q head: exact max, threshold, optional top-pct, forced
//                         keys, k_max cap by score (radix order statistic over order-preserving
//                         integer keys), positions (PI cummax / dense rank / streamed), compaction;
//   decode_attend_kernel  one CTA per q head: each warp streams slots (rotate K at its new
//                         position, dot, online softmax, PV), warps merged at the end.
// The decode step reads the cache once for the scores (HBM-bound) and at most k_max rows again.
#include <float.h>

#include <type_traits>

#include "common.cuh"
#include "gather_rope.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int kScoreThreads = 256;  // 8 warps, one key per warp at a time
constexpr int kKeysPerCta = 64;
constexpr int kSelThreads = 1024;
constexpr int kItems = 4;           // consecutive keys per thread per scan chunk
constexpr int kAttThreads = 1024;  // 32 warps stream the slots of one q head

struct DecP {
  const void* q;
  int64_t qsh;
  const void* k;
  int64_t ksh, ksn;
  const void* v;
  int64_t vsh, vsn;
  void* out;
  int64_t BH, H, Hkv, G, m, q_pos;
  const float* tau;
  const float* ia;
  float psa, rsa;
  const float* ic;
  float psc, rsc;
  float sm;
  int mode, n_global, n_local, k_max, bn;
  int C, n_chunk, mean_agg, weighted;  // CHUNK
  float pct;
  int64_t cap, nblk;
  const float2* ta;
  float ta_R;
  int64_t ta_len;
  const float2* tc;
  float tc_R;
  int64_t tc_len;
  float* scores;
  int32_t* idx;
  float* npk;
  float* npq;
  int32_t* kept;
  int32_t* usize;
  float* dblk;
  float* crank;     // CHUNK: (BH, nC) chunk rank values
  uint8_t* cflag;   // CHUNK: (BH, nC) bit0 candidate, bit1 forced, bit2 selected
  int64_t nC;
};

template <typename TV>
__device__ __forceinline__ float ldf(const TV* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// (cos, sin) * rope_scale at position pos, frequency f: table when the position lies on it
__device__ __forceinline__ void cos_sin(float pos, int f, const float* inv_freq, float rope_scale,
                                        const float2* tab, float R, int64_t len, int half,
                                        float& c, float& s) {
  const int64_t ti = table_index(pos, R, len);
  if (ti >= 0) {
    const float2 cs = __ldg(tab + ti * half + f);
    c = cs.x;
    s = cs.y;
  } else {
    const float ang = __fmul_rn(pos, __ldg(inv_freq + f));
    sincosf(ang, &s, &c);
    c = __fmul_rn(c, rope_scale);
    s = __fmul_rn(s, rope_scale);
  }
}

// Lane l of a warp holds EL = D/32 elements of a row: dims f0 .. f0+EL-1 of the first half
// (l < 16) or of the second half (l >= 16), f0 = (l % 16) * EL; the rotation partner of a first-
// half dim is lane l ^ 16.  Rotates the lane's elements at `pos`.
template <int D>
__device__ __forceinline__ void rotate_lane(float (&x)[D / 32], float pos, const float* inv_freq,
                                            float rope_scale, const float2* tab, float R,
                                            int64_t len) {
  constexpr int EL = D / 32, HALF = D / 2;
  const int lane = threadIdx.x & 31;
  const bool first = lane < 16;
  const int f0 = (lane & 15) * EL;
#pragma unroll
  for (int i = 0; i < EL; ++i) {
    const float par = __shfl_xor_sync(0xffffffffu, x[i], 16);
    float c, s;
    cos_sin(pos, f0 + i, inv_freq, rope_scale, tab, R, len, HALF, c, s);
    const float x1 = first ? x[i] : par, x2 = first ? par : x[i];
    x[i] = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))
                 : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
}

template <int D>
__device__ __forceinline__ int lane_dim(int i) {
  constexpr int EL = D / 32, HALF = D / 2;
  const int lane = threadIdx.x & 31;
  return (lane < 16 ? 0 : HALF) + (lane & 15) * EL + i;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ---- scores -------------------------------------------------------------------------------
template <int D, typename TV>
__global__ void __launch_bounds__(kScoreThreads) decode_score_kernel(const DecP p) {
  constexpr int EL = D / 32, HALF = D / 2;
  extern __shared__ float s_q[];  // [G][D] queries rotated at q_pos * pos_scale_a
  const int64_t kvh = blockIdx.y;
  const int64_t b = kvh / p.Hkv;
  const int64_t bh0 = b * p.H + (kvh % p.Hkv) * p.G;
  const int tid = threadIdx.x, warp = tid >> 5;
  const float qpos = __fmul_rn((float)p.q_pos, p.psa);
  for (int it = tid; it < p.G * HALF; it += kScoreThreads) {
    const int g = it / HALF, f = it % HALF;
    const TV* qr = static_cast<const TV*>(p.q) + (bh0 + g) * p.qsh;
    const float x1 = ldf(qr + f), x2 = ldf(qr + f + HALF);
    float c, s;
    cos_sin(qpos, f, p.ia, p.rsa, p.ta, p.ta_R, p.ta_len, HALF, c, s);
    s_q[g * D + f] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    s_q[g * D + f + HALF] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  __syncthreads();
  const TV* kg = static_cast<const TV*>(p.k) + kvh * p.ksh;
  const int64_t j0 = (int64_t)blockIdx.x * kKeysPerCta;
  for (int kk = warp; kk < kKeysPerCta; kk += kScoreThreads / 32) {
    const int64_t j = j0 + kk;
    if (j >= p.m) break;
    float x[EL];
#pragma unroll
    for (int i = 0; i < EL; ++i) x[i] = ldf(kg + j * p.ksn + lane_dim<D>(i));
    rotate_lane<D>(x, __fmul_rn((float)j, p.psa), p.ia, p.rsa, p.ta, p.ta_R, p.ta_len);
    for (int g = 0; g < p.G; ++g) {
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < EL; ++i) part = fmaf(s_q[g * D + lane_dim<D>(i)], x[i], part);
      const float sc = warp_sum(part);
      if ((threadIdx.x & 31) == 0) p.scores[(bh0 + g) * p.m + j] = __fmul_rn(sc, p.sm);
    }
  }
}

// ---- selection ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t okey(float f) {  // order-preserving unsigned key
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float okey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int NT>
__device__ __forceinline__ int blk_excl_sum(int x, int* sh, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    int s = lane < NT / 32 ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < NT / 32) sh[lane] = s;
  }
  __syncthreads();
  const int base = w > 0 ? sh[w - 1] : 0;
  total = sh[NT / 32 - 1];
  __syncthreads();
  return base + inc - x;
}

template <int NT>
__device__ __forceinline__ float blk_excl_max(float x, float* sh, float& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = fmaxf(inc, y);
  }
  float ex = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) ex = -INFINITY;
  if (lane == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    float s = lane < NT / 32 ? sh[lane] : -INFINITY;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s = fmaxf(s, y);
    }
    if (lane < NT / 32) sh[lane] = s;
  }
  __syncthreads();
  const float base = w > 0 ? sh[w - 1] : -INFINITY;
  total = sh[NT / 32 - 1];
  __syncthreads();
  return fmaxf(base, ex);
}

template <int NT>
__device__ __forceinline__ int blk_sum(int x, int* sh) {
  int t;
  blk_excl_sum<NT>(x, sh, t);
  return t;
}

// k-th largest score (k >= 1, at most the population) among keys passing `filt`: 4 rounds of
// 8-bit radix selection over the order-preserving keys.  Returns the value and the number of
// filtered keys strictly greater.
template <typename F>
__device__ void kth_largest(const float* sc, int64_t m, int64_t k, F filt, uint32_t* hist,
                            float& value, int64_t& n_greater) {
  __shared__ uint32_t s_prefix;
  __shared__ int64_t s_k, s_gt;
  if (threadIdx.x == 0) {
    s_prefix = 0u;
    s_k = k;
    s_gt = 0;
  }
  uint32_t mask = 0u;
  for (int round = 0; round < 4; ++round) {
    const int shift = 24 - 8 * round;
    for (int i = threadIdx.x; i < 256; i += kSelThreads) hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int64_t j = threadIdx.x; j < m; j += kSelThreads) {
      if (!filt(j)) continue;
      const uint32_t key = okey(sc[j]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t kk = s_k, cum = 0;
      int d;
      for (d = 255; d > 0; --d) {
        if (cum + (int64_t)hist[d] >= kk) break;
        cum += hist[d];
      }
      s_gt += cum;
      s_k = kk - cum;
      s_prefix = prefix | ((uint32_t)d << shift);
    }
    __syncthreads();
    mask |= 255u << shift;
  }
  value = okey_inv(s_prefix);
  n_greater = s_gt;
  __syncthreads();
}

__global__ void __launch_bounds__(kSelThreads) decode_select_kernel(const DecP p) {
  const int64_t bh = blockIdx.x;
  const int64_t h = bh % p.H;
  const int tid = threadIdx.x;
  const int64_t m = p.m, qpos = p.q_pos;
  const float* sc = p.scores + bh * m;
  __shared__ int sh_i[32];
  __shared__ float sh_f[32];
  __shared__ uint32_t hist[256];

  // exact max, threshold
  float mx = -INFINITY;
  for (int64_t j = tid; j < m; j += kSelThreads) mx = fmaxf(mx, sc[j]);
  float tot;
  blk_excl_max<kSelThreads>(mx, sh_f, tot);
  const float thr = __fsub_rn(tot, __ldg(p.tau + h));
  const int64_t loc_lo = qpos - p.n_local + 1 > 0 ? qpos - p.n_local + 1 : 0;
  auto forced = [&](int64_t j) { return j < p.n_global || (j >= loc_lo && j <= qpos) || j == qpos; };
  int np = 0;
  for (int64_t j = tid; j < m; j += kSelThreads) np += sc[j] >= thr;
  const int64_t n_pass = blk_sum<kSelThreads>(np, sh_i);

  // optional top-pct of the passers (PI), tie-inclusive
  float cut_p = -INFINITY;
  if (p.mode == STA_DECODE_PI && p.pct < 100.f && n_pass > 0) {
    float bf = ceilf(__fmul_rn((float)((double)p.pct / 100.0), (float)n_pass));
    const int64_t bud = bf < 1.f ? 1 : (int64_t)bf;
    int64_t gt;
    kth_largest(sc, m, bud, [&](int64_t j) { return sc[j] >= thr; }, hist, cut_p, gt);
  }
  auto keep = [&](int64_t j) { return sc[j] >= thr && sc[j] >= cut_p; };
  int nc = 0, nf = 0;
  for (int64_t j = tid; j < m; j += kSelThreads) {
    const bool f = forced(j);
    nf += f;
    nc += f || keep(j);
  }
  const int64_t count = blk_sum<kSelThreads>(nc, sh_i);
  const int64_t n_forced = blk_sum<kSelThreads>(nf, sh_i);

  // k_max cap by score
  const bool over = (p.mode == STA_DECODE_PI || p.mode == STA_DECODE_RANK) && count > p.k_max;
  bool cap_none = false;  // over and no budget: forced keys only
  float cut_c = -INFINITY;
  int64_t need_eq = 0;
  if (over) {
    const int64_t bud = p.k_max - n_forced;
    if (bud <= 0) {
      cap_none = true;
    } else {
      int64_t gt;
      kth_largest(sc, m, bud, [&](int64_t j) { return keep(j) && !forced(j); }, hist, cut_c, gt);
      need_eq = bud - gt;  // RANK: exact budget, ties to the lowest key indices
    }
  }

  // CHUNK: rank chunks by the passers' summed (or mean) exp(s - m) / keep count; forced chunks
  // (global prefix, local window) plus the top n_chunk others, ties to the lowest chunk index
  float* crank = p.crank ? p.crank + bh * p.nC : nullptr;
  uint8_t* cflag = p.cflag ? p.cflag + bh * p.nC : nullptr;
  if (p.mode == STA_DECODE_CHUNK) {
    const int64_t C = p.C;
    const int64_t gch = ((int64_t)max(p.n_global, 0) + C - 1) / C;
    const int64_t lo_c = loc_lo / C, hi_c = qpos / C;
    int ncand = 0;
    for (int64_t c = tid; c < p.nC; c += kSelThreads) {
      float mass = 0.f;
      int cnt = 0;
      const int64_t e = min((c + 1) * C, m);
      for (int64_t j = c * C; j < e; ++j) {
        if (sc[j] >= thr) {
          mass = __fadd_rn(mass, p.weighted ? expf(__fsub_rn(sc[j], tot)) : 1.f);
          ++cnt;
        }
      }
      if (p.mean_agg) mass = __fdiv_rn(mass, (float)(cnt > 1 ? cnt : 1));
      const bool visible = c * C <= qpos;
      const bool fc = (c < gch || (c >= lo_c && c <= hi_c)) && visible;
      crank[c] = mass;
      cflag[c] = fc ? 2 : (visible ? 1 : 0);
      ncand += !fc && visible;
    }
    const int64_t n_cand = blk_sum<kSelThreads>(ncand, sh_i);  // (syncs: the arrays are visible)
    const int64_t n_take = p.n_chunk < p.nC ? p.n_chunk : p.nC;
    const bool all = n_cand <= n_take;
    float cut = 0.f;
    int64_t need = 0;
    if (!all && n_take > 0) {
      int64_t gt;
      kth_largest(crank, p.nC, n_take, [&](int64_t c) { return cflag[c] == 1; }, hist, cut, gt);
      need = n_take - gt;
    }
    int64_t tie_carry = 0;
    for (int64_t c0 = 0; c0 < p.nC; c0 += kSelThreads) {
      const int64_t c = c0 + tid;
      int tie = 0;
      bool sel = false;
      if (c < p.nC) {
        const uint8_t f = cflag[c];
        if (f == 2) sel = true;
        else if (f == 1 && n_take > 0) {
          if (all || crank[c] > cut) sel = true;
          else if (crank[c] == cut) tie = 1;
        }
      }
      int tt;
      const int tr = blk_excl_sum<kSelThreads>(tie, sh_i, tt);
      if (tie && tie_carry + tr < need) sel = true;
      if (c < p.nC && sel) cflag[c] |= 4;
      tie_carry += tt;
    }
    __syncthreads();
  }

  // streamed offsets: d_b = kept keys in the blocks after b (nearer the query)
  float* dblk = p.dblk ? p.dblk + bh * p.nblk : nullptr;
  auto base_final = [&](int64_t j) { return forced(j) || keep(j); };
  if (p.mode == STA_DECODE_STREAM) {
    for (int64_t b = tid; b < p.nblk; b += kSelThreads) {
      int c = 0;
      const int64_t e = min((b + 1) * (int64_t)p.bn, m);
      for (int64_t j = b * p.bn; j < e; ++j) c += base_final(j);
      dblk[b] = (float)c;
    }
    __syncthreads();
    // exclusive suffix sums over the blocks (descending order), in chunks of the CTA
    int64_t carry = 0;
    for (int64_t c0 = 0; c0 < p.nblk; c0 += kSelThreads) {
      const int64_t r = c0 + tid;                // r-th block from the top
      const int64_t b = p.nblk - 1 - r;
      const int c = r < p.nblk ? (int)dblk[b] : 0;
      int t;
      const int ex = blk_excl_sum<kSelThreads>(c, sh_i, t);
      if (r < p.nblk) dblk[b] = (float)(carry + ex);
      carry += t;
      __syncthreads();
    }
  }

  // compaction: ranks (prefix count), positions, slots in key order
  int32_t* idx_row = p.idx + bh * p.cap;
  float* npk_row = p.npk + bh * p.cap;
  int64_t carry = 0, tie_carry = 0;
  float cm_carry = -INFINITY;
  for (int64_t c0 = 0; c0 < m; c0 += (int64_t)kSelThreads * kItems) {
    const int64_t j0 = c0 + (int64_t)tid * kItems;
    uint32_t flags = 0, tie = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= m) continue;
      bool f;
      if (p.mode == STA_DECODE_CHUNK) {
        f = (cflag[j / p.C] & 4) || j == qpos;
      } else if (!over) {
        f = base_final(j);
      } else if (forced(j)) {
        f = true;
      } else if (cap_none || !keep(j)) {
        f = false;
      } else if (p.mode == STA_DECODE_PI) {
        f = sc[j] >= cut_c;                    // tie-inclusive (exact.py:517-519)
      } else {
        f = sc[j] > cut_c;
        if (sc[j] == cut_c) tie |= 1u << i;
      }
      flags |= (f ? 1u : 0u) << i;
    }
    if (over && p.mode == STA_DECODE_RANK) {
      int tt;
      const int tb = blk_excl_sum<kSelThreads>(__popc(tie), sh_i, tt);
#pragma unroll
      for (int i = 0; i < kItems; ++i)
        if ((tie >> i) & 1u)
          if (tie_carry + tb + __popc(tie & ((1u << i) - 1u)) < need_eq) flags |= 1u << i;
      tie_carry += tt;
    }
    int total;
    const int base = blk_excl_sum<kSelThreads>(__popc(flags), sh_i, total);
    float rank0f[kItems], cr[kItems];
    float tmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t before = carry + base + __popc(flags & ((1u << i) - 1u));
      const bool f = (flags >> i) & 1u;
      rank0f[i] = (float)(before + (f ? 1 : 0) - 1);
      cr[i] = f ? __fsub_rn(__fmul_rn((float)(j0 + i), p.psc), rank0f[i]) : -INFINITY;
      tmax = fmaxf(tmax, cr[i]);
    }
    float run = -INFINITY;
    if (p.mode == STA_DECODE_PI) {
      float bmax;
      const float ex = blk_excl_max<kSelThreads>(tmax, sh_f, bmax);
      run = fmaxf(cm_carry, ex);
      cm_carry = fmaxf(cm_carry, bmax);
    }
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= m) break;
      const bool f = (flags >> i) & 1u;
      float np2;
      if (p.mode == STA_DECODE_PI) {
        run = fmaxf(run, cr[i]);
        np2 = __fadd_rn(rank0f[i], run);
      } else if (p.mode == STA_DECODE_RANK || p.mode == STA_DECODE_CHUNK) {
        np2 = rank0f[i];
      } else {
        const int64_t b = j / p.bn;
        const int64_t hi_b = min(qpos, b * p.bn + p.bn - 1);
        np2 = -__fadd_rn(dblk[b], (float)(hi_b - j));
      }
      const int64_t rk = (int64_t)rank0f[i];
      if (f && rk < p.cap) {
        idx_row[rk] = (int32_t)j;
        npk_row[rk] = np2;
      }
      if (j == qpos) p.npq[bh] = p.mode == STA_DECODE_STREAM ? 0.f : np2;
    }
    carry += total;
  }
  __syncthreads();
  for (int64_t s = carry + tid; s < p.cap; s += kSelThreads) {
    idx_row[s] = (int32_t)m;
    npk_row[s] = 0.f;
  }
  if (tid == 0) {
    p.kept[bh] = (int32_t)carry;
    if (p.usize) p.usize[bh] = (int32_t)n_pass;
  }
}

// ---- attention ----------------------------------------------------------------------------
template <int D, typename TV>
__global__ void __launch_bounds__(kAttThreads) decode_attend_kernel(const DecP p) {
  constexpr int EL = D / 32, HALF = D / 2, NWA = kAttThreads / 32;
  __shared__ float s_q[D];
  __shared__ float s_m[NWA], s_l[NWA];
  __shared__ float s_acc[NWA][D];
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t kvh = b * p.Hkv + h / p.G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float qp = p.npq[bh];
  for (int f = tid; f < HALF; f += kAttThreads) {
    const TV* qr = static_cast<const TV*>(p.q) + bh * p.qsh;
    const float x1 = ldf(qr + f), x2 = ldf(qr + f + HALF);
    float c, s;
    cos_sin(qp, f, p.ic, p.rsc, p.tc, p.tc_R, p.tc_len, HALF, c, s);
    s_q[f] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    s_q[f + HALF] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  }
  __syncthreads();
  float qv[EL];
#pragma unroll
  for (int i = 0; i < EL; ++i) qv[i] = s_q[lane_dim<D>(i)];
  const TV* kg = static_cast<const TV*>(p.k) + kvh * p.ksh;
  const TV* vg = static_cast<const TV*>(p.v) + kvh * p.vsh;
  const int32_t* idx_row = p.idx + bh * p.cap;
  const float* npk_row = p.npk + bh * p.cap;
  const int64_t ns = min((int64_t)p.kept[bh], p.cap);
  float mr = -INFINITY, l = 0.f, acc[EL];
#pragma unroll
  for (int i = 0; i < EL; ++i) acc[i] = 0.f;
  for (int64_t sl = warp; sl < ns; sl += NWA) {
    const int64_t j = idx_row[sl];
    float x[EL], vv[EL];
#pragma unroll
    for (int i = 0; i < EL; ++i) {
      x[i] = ldf(kg + j * p.ksn + lane_dim<D>(i));
      vv[i] = ldf(vg + j * p.vsn + lane_dim<D>(i));
    }
    rotate_lane<D>(x, npk_row[sl], p.ic, p.rsc, p.tc, p.tc_R, p.tc_len);
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < EL; ++i) part = fmaf(qv[i], x[i], part);
    const float s = __fmul_rn(warp_sum(part), p.sm);
    const float mn = fmaxf(mr, s);
    const float a = expf(__fsub_rn(mr, mn));  // 0 while nothing was seen (mr = -inf)
    const float e = expf(__fsub_rn(s, mn));
    l = l * a + e;
#pragma unroll
    for (int i = 0; i < EL; ++i) acc[i] = acc[i] * a + e * vv[i];
    mr = mn;
  }
  if (lane == 0) {
    s_m[warp] = mr;
    s_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < EL; ++i) s_acc[warp][lane_dim<D>(i)] = acc[i];
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < NWA; ++w) M = fmaxf(M, s_m[w]);
  for (int d = tid; d < D; d += kAttThreads) {
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < NWA; ++w) {
      const float a = s_m[w] == -INFINITY ? 0.f : expf(__fsub_rn(s_m[w], M));
      L += s_l[w] * a;
      o += s_acc[w][d] * a;
    }
    const float r = o / L;
    if (std::is_same<TV, float>::value)
      static_cast<float*>(p.out)[bh * D + d] = r;
    else
      static_cast<__nv_bfloat16*>(p.out)[bh * D + d] = __float2bfloat16_rn(r);
  }
}

struct DecLayout {
  size_t scores, idx, npk, npq, kept, usize, dblk, crank, cflag, total;
  int64_t cap, nblk, nC;
};

inline size_t al(size_t x) { return (x + 255) & ~size_t(255); }

DecLayout dec_layout(const sta_decode_args* a) {
  DecLayout L{};
  const int64_t BH = a->batch * a->n_heads;
  L.cap = a->mode == STA_DECODE_STREAM ? a->m : a->k_max;
  L.nblk = a->mode == STA_DECODE_STREAM ? (a->m + a->block_n - 1) / a->block_n : 0;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t r = o;
    o += al(bytes);
    return r;
  };
  L.scores = take((size_t)BH * a->m * 4);
  L.idx = take((size_t)BH * L.cap * 4);
  L.npk = take((size_t)BH * L.cap * 4);
  L.npq = take((size_t)BH * 4);
  L.kept = take((size_t)BH * 4);
  L.usize = take((size_t)BH * 4);
  L.dblk = take((size_t)BH * (L.nblk > 0 ? L.nblk : 1) * 4);
  L.nC = a->mode == STA_DECODE_CHUNK ? (a->m + a->chunk_size - 1) / a->chunk_size : 0;
  L.crank = take((size_t)BH * (L.nC > 0 ? L.nC : 1) * 4);
  L.cflag = take((size_t)BH * (L.nC > 0 ? L.nC : 1));
  L.total = o;
  return L;
}

int dec_check(const sta_decode_args* a) {
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->tau || !a->inv_freq_a || !a->inv_freq_c)
    return fail(STA_ERR_ARG, "sta_decode: null pointer");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "sta_decode: d must be 64 or 128");
  if (a->dtype != STA_DTYPE_F32 && a->dtype != STA_DTYPE_BF16)
    return fail(STA_ERR_UNSUPPORTED, "sta_decode: dtype must be f32 or bf16");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads || a->batch <= 0)
    return fail(STA_ERR_ARG, "sta_decode: bad head counts");
  if (a->m <= 0) return fail(STA_ERR_ARG, "sta_decode: empty cache");
  if (a->mode < STA_DECODE_PI || a->mode > STA_DECODE_CHUNK)
    return fail(STA_ERR_ARG, "sta_decode: mode");
  if (a->mode != STA_DECODE_STREAM && a->k_max <= 0) return fail(STA_ERR_ARG, "sta_decode: k_max");
  if (a->mode == STA_DECODE_CHUNK && (a->chunk_size <= 0 || a->n_chunk < 0))
    return fail(STA_ERR_ARG, "sta_decode: chunk_size / n_chunk");
  if (a->mode == STA_DECODE_STREAM && a->block_n <= 0) return fail(STA_ERR_ARG, "sta_decode: block_n");
  if (a->n_kv_heads > 65535 || a->m > ((int64_t)1 << 31) - 1)
    return fail(STA_ERR_UNSUPPORTED, "sta_decode: too many kv heads / keys");
  return STA_OK;
}

template <int D, typename TV>
int dec_launch(const DecP& p, cudaStream_t st) {
  const dim3 g1((unsigned)((p.m + kKeysPerCta - 1) / kKeysPerCta), (unsigned)(p.BH / p.G));
  const size_t sm1 = (size_t)p.G * D * 4;
  if (sm1 > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(decode_score_kernel<D, TV>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
    if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  }
  decode_score_kernel<D, TV><<<g1, kScoreThreads, sm1, st>>>(p);
  decode_select_kernel<<<(unsigned)p.BH, kSelThreads, 0, st>>>(p);
  decode_attend_kernel<D, TV><<<(unsigned)p.BH, kAttThreads, 0, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace

size_t decode_workspace_bytes(const sta_decode_args* a) {
  if (dec_check(a) != STA_OK) return 0;
  return dec_layout(a).total;
}

int decode_forward(const sta_decode_args* a, void* ws, size_t ws_len, cudaStream_t st) {
  const int rc = dec_check(a);
  if (rc != STA_OK) return rc;
  const DecLayout L = dec_layout(a);
  if (!ws || ws_len < L.total) return fail(STA_ERR_WORKSPACE, "sta_decode: workspace too small");
  uint8_t* w = static_cast<uint8_t*>(ws);
  DecP p;
  p.q = a->q; p.qsh = a->q_stride_h;
  p.k = a->k; p.ksh = a->k_stride_h; p.ksn = a->k_stride_n;
  p.v = a->v; p.vsh = a->v_stride_h; p.vsn = a->v_stride_n;
  p.out = a->out;
  p.BH = a->batch * a->n_heads;
  p.H = a->n_heads;
  p.Hkv = a->n_kv_heads;
  p.G = a->n_heads / a->n_kv_heads;
  p.m = a->m;
  p.q_pos = a->m - 1;
  p.tau = a->tau;
  p.ia = a->inv_freq_a; p.psa = a->pos_scale_a; p.rsa = a->rope_scale_a;
  p.ic = a->inv_freq_c; p.psc = a->pos_scale_c; p.rsc = a->rope_scale_c;
  p.sm = a->sm_scale;
  p.mode = a->mode;
  p.n_global = a->n_global;
  p.n_local = a->n_local;
  p.k_max = a->k_max;
  p.bn = a->block_n > 0 ? a->block_n : 32;
  p.pct = a->pct_decode;
  p.cap = L.cap;
  p.nblk = L.nblk;
  p.ta = static_cast<const float2*>(a->rope_table_a);
  p.ta_R = a->rope_table_a_R;
  p.ta_len = a->rope_table_a ? a->rope_table_a_len : 0;
  p.tc = static_cast<const float2*>(a->rope_table_c);
  p.tc_R = a->rope_table_c_R;
  p.tc_len = a->rope_table_c ? a->rope_table_c_len : 0;
  p.scores = reinterpret_cast<float*>(w + L.scores);
  p.idx = a->idx_out ? a->idx_out : reinterpret_cast<int32_t*>(w + L.idx);
  p.npk = a->newpos_k_out ? a->newpos_k_out : reinterpret_cast<float*>(w + L.npk);
  p.npq = a->newpos_q_out ? a->newpos_q_out : reinterpret_cast<float*>(w + L.npq);
  p.kept = a->kept_out ? a->kept_out : reinterpret_cast<int32_t*>(w + L.kept);
  p.usize = a->usize_out ? a->usize_out : reinterpret_cast<int32_t*>(w + L.usize);
  p.dblk = L.nblk > 0 ? reinterpret_cast<float*>(w + L.dblk) : nullptr;
  p.C = a->chunk_size > 0 ? a->chunk_size : 16;
  p.n_chunk = a->n_chunk;
  p.mean_agg = a->chunk_agg == 1;
  p.weighted = a->select_score != STA_SCORE_FREQ;
  p.nC = L.nC;
  p.crank = L.nC > 0 ? reinterpret_cast<float*>(w + L.crank) : nullptr;
  p.cflag = L.nC > 0 ? w + L.cflag : nullptr;
  const bool f32 = a->dtype == STA_DTYPE_F32;
  if (a->d == 128) return f32 ? dec_launch<128, float>(p, st) : dec_launch<128, __nv_bfloat16>(p, st);
  return f32 ? dec_launch<64, float>(p, st) : dec_launch<64, __nv_bfloat16>(p, st);
}

}  // namespace sta
