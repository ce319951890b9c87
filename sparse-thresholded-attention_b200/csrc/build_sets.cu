// Device-side key-set construction (one CTA per (head, query tile)).
//
// sta_build_sets    <- _build_sets, shared_selection_triton_exact_2.py:277-426
//                      (sort form: shared_selection_triton_exact.py:253-370)
// sta_build_sets_pq <- _build_sets_pq, shared_selection_triton_perquery.py:363-453
//
// The reference runs these as torch ops over dense (H, nt, N) tensors (topk / sort / cumsum /
// cummax / scatter, plus host syncs).  Here each tile is one CTA that streams its compact vote
// row (only the tile's causal keys j < hi_t exist) from HBM/L2:
//   * order statistic of the tie-inclusive top-pct cut: a (tile+1)-bin vote histogram for
//     frequency ranking, an exact 4 x 8-bit radix select over the fp32 rank bits otherwise;
//   * the 30 -> 25 -> 20 fallback needs only |shared| (from the histogram / select) and the
//     handful of forced keys that are not shared;
//   * one block-wide pass with a prefix count (ranks) and a prefix max (the PI cummax) writes
//     idx / newpos_k / newpos_q directly in slot order.
// All rank / position arithmetic is fp32 with explicit rounding, matching torch bit for bit.
#include <float.h>

#include "common.cuh"
#include "sta_internal.h"

namespace sta {

namespace {

constexpr int kBT = 256;          // threads per CTA
constexpr int kItems = 8;         // consecutive keys per thread per scan chunk
constexpr int kChunk = kBT * kItems;

struct SetRow {
  const uint8_t* v;     // compact votes of this (head, tile)
  const float* w;       // compact weighted votes (or null)
  const uint32_t* b;    // compact bits (or null)
  int64_t hi;           // causal key count of the tile
};

__device__ __forceinline__ float rank_value(const SetRow& r, int64_t j, bool weighted) {
  if (j >= r.hi) return 0.f;
  const float vf = (float)r.v[j];
  if (!weighted) return vf;
  return __fadd_rn(r.w[j], __fmul_rn(1e-6f, vf));
}

// ---- block scans (256 threads) ----------------------------------------------------------
__device__ __forceinline__ int block_excl_sum(int x, int* sh, int& total) {
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
    int s = lane < (kBT / 32) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < (kBT / 32)) sh[lane] = s;
  }
  __syncthreads();
  const int base = (w > 0 ? sh[w - 1] : 0);
  total = sh[kBT / 32 - 1];
  __syncthreads();
  return base + inc - x;
}

__device__ __forceinline__ float block_excl_max(float x, float* sh, float& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = fmaxf(inc, y);
  }
  // exclusive within warp
  float ex = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) ex = -INFINITY;
  if (lane == 31) sh[w] = inc;
  __syncthreads();
  if (w == 0) {
    float s = lane < (kBT / 32) ? sh[lane] : -INFINITY;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s = fmaxf(s, y);
    }
    if (lane < (kBT / 32)) sh[lane] = s;
  }
  __syncthreads();
  const float base = (w > 0 ? sh[w - 1] : -INFINITY);
  total = sh[kBT / 32 - 1];
  __syncthreads();
  return fmaxf(base, ex);
}

__device__ __forceinline__ int block_sum(int x, int* sh) {
  int total;
  block_excl_sum(x, sh, total);
  return total;
}

// ---- forced keys: glob [0, gend) U local [lstart, lend] -----------------------------------
struct Forced {
  int64_t gend, lstart, lend;  // local range clipped to [0, N-1], lstart may be > lend (empty)
  __device__ __forceinline__ bool has(int64_t j) const {
    return j < gend || (j >= lstart && j <= lend);
  }
  __device__ __forceinline__ int64_t count() const {
    const int64_t ls = lstart > gend ? lstart : gend;
    return gend + (lend >= ls ? lend - ls + 1 : 0);
  }
  // i-th forced key in ascending order, i < count()
  __device__ __forceinline__ int64_t at(int64_t i) const {
    if (i < gend) return i;
    const int64_t ls = lstart > gend ? lstart : gend;
    return ls + (i - gend);
  }
};

__device__ __forceinline__ Forced make_forced(int64_t N, int64_t tstart, int T, int n_global,
                                              int n_local) {
  Forced f;
  f.gend = n_global < N ? n_global : N;
  if (f.gend < 0) f.gend = 0;
  int64_t lo = tstart - n_local + 1;
  int64_t hi = tstart + T - 1;
  if (lo < 0) lo = 0;
  if (hi > N - 1) hi = N - 1;
  f.lstart = lo;
  f.lend = hi;
  return f;
}

// ---- exact k-th largest (k >= 1) of the rank values of all N keys (keys >= hi are 0) ------
// 4 rounds of 8-bit radix selection over the fp32 bit patterns (all rank values are >= +0,
// so unsigned order == float order).  Only keys passing `filter` take part (cand_only: PQ
// candidates = union minus forced).  Returns the value bits and the number of keys strictly
// greater / equal.
__device__ void radix_kth_largest(const SetRow& r, int64_t N, bool weighted, int64_t k,
                                  bool cand_only, const Forced& F, uint32_t* hist,
                                  uint32_t& out_bits, int64_t& n_greater, int64_t& n_equal) {
  __shared__ uint32_t s_prefix, s_digit;
  __shared__ int64_t s_k, s_gt, s_eq;
  if (threadIdx.x == 0) {
    s_prefix = 0u;
    s_k = k;
    s_gt = 0;
  }
  uint32_t mask = 0u;
  for (int round = 0; round < 4; ++round) {
    const int shift = 24 - 8 * round;
    for (int i = threadIdx.x; i < 256; i += kBT) hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    auto count = [&](int64_t j) {
      const uint32_t key = __float_as_uint(rank_value(r, j, weighted));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    };
    if (cand_only && (reinterpret_cast<uintptr_t>(r.v) & 7u) == 0) {
      // candidates have a nonzero vote: 8 votes per load, four loads in flight, all-zero
      // words skipped (the union is sparse)
      const int64_t nw = r.hi / 8;
      const uint2* vw = reinterpret_cast<const uint2*>(r.v);
      for (int64_t w0 = threadIdx.x; w0 < nw; w0 += 4 * kBT) {
        uint2 u4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int64_t w = w0 + (int64_t)q * kBT;
          u4[q] = w < nw ? vw[w] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint2 u = u4[q];
          if ((u.x | u.y) == 0u) continue;
          const int64_t jb = (w0 + (int64_t)q * kBT) * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t j = jb + i;
            if ((((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 255u) && !F.has(j)) count(j);
          }
        }
      }
      for (int64_t j = nw * 8 + threadIdx.x; j < r.hi; j += kBT)
        if (r.v[j] != 0 && !F.has(j)) count(j);
    } else {
      for (int64_t j = threadIdx.x; j < r.hi; j += kBT) {
        if (cand_only && (r.v[j] == 0 || F.has(j))) continue;
        count(j);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      // keys at or beyond hi: value +0 (never candidates in cand_only mode)
      if (!cand_only && prefix == 0u && N > r.hi) hist[0] += (uint32_t)(N - r.hi);
      int64_t kk = s_k, cum = 0;
      int d = 0;
      for (d = 255; d >= 0; --d) {
        if (cum + (int64_t)hist[d] >= kk) break;
        cum += hist[d];
      }
      if (d < 0) d = 0;  // k larger than the population: caller guarantees this cannot happen
      s_digit = (uint32_t)d;
      s_gt += cum;
      s_k = kk - cum;
      s_prefix = prefix | ((uint32_t)d << shift);
      s_eq = hist[d];
    }
    __syncthreads();
    mask |= 255u << shift;
  }
  out_bits = s_prefix;
  n_greater = s_gt;
  n_equal = s_eq;
  __syncthreads();
}

// ---- shared-path selection ------------------------------------------------------------------
struct BuildP {
  const uint8_t* votes;
  const float* wvotes;
  int64_t BH, N, nt, head_stride, qbase;
  int T, k_max, n_global, n_local;
  int nsteps;
  int steps[3];
  int start_pct;
  float pos_scale;
  int weighted;
  int measure;
  int32_t* idx;
  float* newpos_k;
  float* newpos_q;
  int32_t* shared_size;
  int32_t* kept_size;
  int32_t* chosen;
  uint8_t* overflow;
  int32_t* kpct_meas;
  uint8_t* overflow20;
  const uint32_t* vote_hist;
};

__global__ void __launch_bounds__(kBT) build_sets_kernel(const BuildP p) {
  const int64_t t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x;
  const int64_t N = p.N;
  const int T = p.T;
  const int64_t tstart = p.qbase + t * T;  // absolute position of the tile's first query
  SetRow r;
  const int64_t off = bh * p.head_stride + tri_tile_offset(t, T, p.qbase);
  r.v = p.votes + off;
  r.w = p.weighted ? p.wvotes + off : nullptr;
  r.b = nullptr;
  r.hi = min(tstart + T, N);
  const bool weighted = p.weighted != 0;
  const Forced F = make_forced(N, tstart, T, p.n_global, p.n_local);
  const int64_t n_forced = F.count();

  __shared__ uint32_t hist[256];
  __shared__ int sh_i[32];
  __shared__ float sh_f[32];
  __shared__ int64_t s_usize;
  __shared__ uint32_t s_cut;
  __shared__ int64_t s_ge;

  // ---- union size and (frequency ranking) vote histogram over bins 0..T: from the select
  // kernel's histograms when given, else one pass over the votes
  const uint32_t* vh = (!weighted && p.vote_hist) ? p.vote_hist + (bh * p.nt + t) * (T + 1) : nullptr;
  for (int i = tid; i < 256; i += kBT) hist[i] = (vh && i >= 1 && i <= T) ? vh[i] : 0u;
  __syncthreads();
  int nz = 0;
  int64_t j_tail = vh ? r.hi : 0;
  if (vh) {
    for (int i = tid; i <= T; i += kBT)
      if (i >= 1) nz += (int)hist[i];
  } else if ((reinterpret_cast<uintptr_t>(r.v) & 7u) == 0) {
    // 8 votes per load, four loads in flight per thread; most keys have none, so all-zero
    // words are skipped
    const int64_t nw = r.hi / 8;
    const uint2* vw = reinterpret_cast<const uint2*>(r.v);
    for (int64_t w0 = tid; w0 < nw; w0 += 4 * kBT) {
      uint2 u4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t w = w0 + (int64_t)q * kBT;
        u4[q] = w < nw ? vw[w] : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint2 u = u4[q];
        if ((u.x | u.y) == 0u) continue;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t v = ((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 255u;
          if (v) {
            ++nz;
            if (!weighted) atomicAdd(&hist[v], 1u);
          }
        }
      }
    }
    j_tail = nw * 8;
  }
  for (int64_t j = j_tail + tid; j < r.hi; j += kBT) {
    const uint32_t v = r.v[j];
    if (v) {
      ++nz;
      if (!weighted) atomicAdd(&hist[v], 1u);
    }
  }
  const int usize_i = block_sum(nz, sh_i);
  if (tid == 0) {
    s_usize = usize_i;
    if (!weighted) hist[0] = (uint32_t)(N - usize_i);
  }
  __syncthreads();
  const int64_t usize = s_usize;

  // v_cut for budget b (b >= 1): returns bits of the cut value and |{j : rank >= cut}|
  auto cut_for_budget = [&](int64_t b, uint32_t& cut_bits, int64_t& n_ge) {
    if (!weighted) {
      __syncthreads();
      if (tid == 0) {
        int64_t cum = 0;
        int v;
        for (v = T; v > 0; --v) {
          cum += hist[v];
          if (cum >= b) break;
        }
        if (v == 0) cum += hist[0];
        s_cut = __float_as_uint((float)v);
        s_ge = cum;
      }
      __syncthreads();
      cut_bits = s_cut;
      n_ge = s_ge;
      __syncthreads();
    } else {
      int64_t gt, eq;
      radix_kth_largest(r, N, true, b, false, F, hist, cut_bits, gt, eq);
      n_ge = gt + eq;
    }
  };
  // forced keys whose rank value is below the cut
  auto forced_below = [&](uint32_t cut_bits) -> int64_t {
    const float cut = __uint_as_float(cut_bits);
    int c = 0;
    for (int64_t i = tid; i < n_forced; i += kBT) {
      const int64_t j = F.at(i);
      if (rank_value(r, j, weighted) < cut) ++c;
    }
    return block_sum(c, sh_i);
  };
  auto budget_of = [&](int pct) -> int64_t {
    const float b = ceilf(__fmul_rn((float)((double)pct / 100.0), (float)usize));
    return b < 1.f ? 1 : (int64_t)b;
  };

  // ---- 30 -> 25 -> 20 fallback (first percentage whose kept set fits k_max)
  bool resolved = false, orig_overflow = false, has_shared = true;
  int chosen = 0;
  uint32_t cut_bits = 0;
  int64_t n_shared = 0, n_kept = 0;
  for (int si = 0; si < p.nsteps; ++si) {
    const int pc = p.steps[si];
    uint32_t cb;
    int64_t nge;
    cut_for_budget(budget_of(pc), cb, nge);
    const int64_t nk = nge + forced_below(cb);
    if (pc == p.start_pct) orig_overflow = nk > p.k_max;
    cut_bits = cb;
    n_shared = nge;
    n_kept = nk;
    if (nk <= p.k_max) {
      resolved = true;
      chosen = pc;
      break;
    }
  }
  if (!resolved && p.start_pct == 0) {
    // reference: the unresolved set becomes the forced keys alone (exact_2.py:344-347)
    has_shared = false;
    n_shared = 0;
    n_kept = n_forced;
    orig_overflow = n_forced > p.k_max;
  }
  int kpct_meas = chosen;
  if (p.measure && !resolved) {
    for (int pc = p.steps[p.nsteps - 1] - 1; pc >= 1; --pc) {
      uint32_t cb;
      int64_t nge;
      cut_for_budget(budget_of(pc), cb, nge);
      const int64_t nk = nge + forced_below(cb);
      if (nk <= p.k_max) {
        kpct_meas = pc;
        break;
      }
    }
  }

  // ---- compaction pass: ranks (prefix count) + PI positions (prefix max) in key order
  const float cut = __uint_as_float(cut_bits);
  const int64_t E = (has_shared && cut_bits == 0u) ? N : (r.hi > F.gend ? r.hi : F.gend);
  const int64_t nt_row = (bh * p.nt + t);
  int32_t* idx_row = p.idx + nt_row * p.k_max;
  float* npk_row = p.newpos_k + nt_row * p.k_max;
  float* npq_row = p.newpos_q + nt_row * T;
  int64_t carry = 0;
  float cm_carry = -INFINITY;
  // pos_scale 1: j - rank0 never decreases along the kept keys (each gap adds >= 0), so the
  // running max at a kept key is its own j - rank0 and its position is exactly j -- no max scan.
  // (Positions of keys that are not kept are only read for the tile's queries, which the local
  // window keeps whenever n_local >= 1.)
  const bool identity = p.pos_scale == 1.f && p.n_local >= 1;
  // the thread's kItems consecutive votes packed in 8 bytes: one 8-byte load where aligned and
  // in range; the next chunk's word is loaded while the current chunk is scanned
  auto load_votes = [&](int64_t j0) -> uint2 {
    if (j0 + kItems <= r.hi && ((reinterpret_cast<uintptr_t>(r.v + j0) & 7u) == 0))
      return *reinterpret_cast<const uint2*>(r.v + j0);
    uint32_t x = 0u, y = 0u;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const uint32_t b = j0 + i < r.hi ? (uint32_t)r.v[j0 + i] : 0u;
      if (i < 4) x |= b << (8 * i);
      else y |= b << (8 * (i - 4));
    }
    return make_uint2(x, y);
  };
  uint2 u_next = load_votes((int64_t)tid * kItems);
  for (int64_t c0 = 0; c0 < E; c0 += kChunk) {
    const int64_t j0 = c0 + (int64_t)tid * kItems;
    const uint2 u = u_next;
    if (c0 + kChunk < E) u_next = load_votes(j0 + kChunk);
    uint32_t vb[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) vb[i] = ((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 255u;
    uint32_t flags = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j < E) {
        const float rv = !weighted ? (float)vb[i]
                                   : (j < r.hi ? __fadd_rn(r.w[j], __fmul_rn(1e-6f, (float)vb[i])) : 0.f);
        const bool kept = (has_shared && rv >= cut) || F.has(j);
        flags |= (kept ? 1u : 0u) << i;
      }
    }
    int total;
    const int base = block_excl_sum(__popc(flags), sh_i, total);
    float rank0f[kItems], cr[kItems];
    float tmax = -INFINITY;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t before = carry + base + __popc(flags & ((1u << i) - 1u));
      const bool f = (flags >> i) & 1u;
      rank0f[i] = (float)(before + (f ? 1 : 0) - 1);
      const int64_t j = j0 + i;
      cr[i] = f ? __fsub_rn(__fmul_rn((float)j, p.pos_scale), rank0f[i]) : -INFINITY;
      tmax = fmaxf(tmax, cr[i]);
    }
    float run = cm_carry, bmax = -INFINITY;
    if (!identity) {
      const float excl = block_excl_max(tmax, sh_f, bmax);
      run = fmaxf(cm_carry, excl);
    }
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= E) break;
      run = fmaxf(run, cr[i]);
      const float np = identity ? (float)j : __fadd_rn(rank0f[i], run);
      const bool f = (flags >> i) & 1u;
      const int64_t rk = (int64_t)rank0f[i];
      if (f && rk < p.k_max) {
        idx_row[rk] = (int32_t)j;
        npk_row[rk] = np;
      }
      if (j >= tstart && j < tstart + T) npq_row[j - tstart] = np;
    }
    carry += total;
    cm_carry = fmaxf(cm_carry, bmax);
  }
  __syncthreads();
  // padded query rows of a ragged last tile read position N-1 (reference clamps qpos)
  if (tstart + T > N) {
    const float last = npq_row[N - 1 - tstart];
    for (int i = tid; i < T; i += kBT)
      if (tstart + i > N - 1) npq_row[i] = last;
  }
  for (int64_t s = carry + tid; s < p.k_max; s += kBT) {
    idx_row[s] = (int32_t)N;
    npk_row[s] = 0.f;
  }
  if (tid == 0) {
    const int64_t o = nt_row;
    p.shared_size[o] = (int32_t)n_shared;
    p.kept_size[o] = (int32_t)n_kept;
    p.chosen[o] = chosen;
    p.overflow[o] = orig_overflow ? 1 : 0;
    p.kpct_meas[o] = kpct_meas;
    p.overflow20[o] = (orig_overflow && !resolved) ? 1 : 0;
  }
}

// ---- PQ-Union selection -----------------------------------------------------------------------
struct BuildPQP {
  const uint8_t* votes;
  const float* wvotes;
  const uint32_t* bits;
  int64_t BH, N, nt, head_stride, qbase;
  int T, k_max, n_global, n_local;
  int weighted;
  int32_t* idx;
  float* newpos_k;
  float* newpos_q;
  int32_t* mask;
  int32_t* usize;
  int32_t* kept_size;
  uint8_t* overflow;
};

__global__ void __launch_bounds__(kBT) build_sets_pq_kernel(const BuildPQP p) {
  const int64_t t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x;
  const int64_t N = p.N;
  const int T = p.T;
  const int64_t tstart = p.qbase + t * T;  // absolute position of the tile's first query
  SetRow r;
  const int64_t off = bh * p.head_stride + tri_tile_offset(t, T, p.qbase);
  r.v = p.votes + off;
  r.w = p.weighted ? p.wvotes + off : nullptr;
  r.b = p.bits + off;
  r.hi = min(tstart + T, N);
  const bool weighted = p.weighted != 0;
  const Forced F = make_forced(N, tstart, T, p.n_global, p.n_local);
  const int64_t n_forced = F.count();

  __shared__ uint32_t hist[256];
  __shared__ int sh_i[32];

  int nu = 0, nfu = 0;
  if ((reinterpret_cast<uintptr_t>(r.v) & 7u) == 0) {
    // 8 votes per load, four loads in flight; the union is sparse, so only nonzero words are
    // looked at
    const int64_t nw = r.hi / 8;
    const uint2* vw = reinterpret_cast<const uint2*>(r.v);
    for (int64_t w0 = tid; w0 < nw; w0 += 4 * kBT) {
      uint2 u4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t w = w0 + (int64_t)q * kBT;
        u4[q] = w < nw ? vw[w] : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint2 u = u4[q];
        if ((u.x | u.y) == 0u) continue;
        const int64_t w = w0 + (int64_t)q * kBT;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 255u) {
            ++nu;
            if (F.has(w * 8 + i)) ++nfu;
          }
        }
      }
    }
    for (int64_t j = nw * 8 + tid; j < r.hi; j += kBT) {
      if (r.v[j]) {
        ++nu;
        if (F.has(j)) ++nfu;
      }
    }
  } else {
    for (int64_t j = tid; j < r.hi; j += kBT) {
      if (r.v[j]) {
        ++nu;
        if (F.has(j)) ++nfu;
      }
    }
  }
  const int64_t usize = block_sum(nu, sh_i);
  const int64_t forced_in_union = block_sum(nfu, sh_i);
  const int64_t kept_full = usize + n_forced - forced_in_union;
  const bool overflow = kept_full > p.k_max;

  // truncation: forced + the top b_eff candidates (union minus forced) by rank value
  int64_t b_eff = 0, need_eq = 0;
  float vb = INFINITY;
  if (overflow) {
    int64_t budget = p.k_max - n_forced;
    if (budget < 0) budget = 0;
    const int64_t ktop = p.k_max < N ? p.k_max : N;
    b_eff = budget < ktop ? budget : ktop;
    if (b_eff > 0) {
      uint32_t bits;
      int64_t gt, eq;
      radix_kth_largest(r, N, weighted, b_eff, true, F, hist, bits, gt, eq);
      vb = __uint_as_float(bits);
      need_eq = b_eff - gt;
    }
  }

  const int64_t E = r.hi > F.gend ? r.hi : F.gend;
  const int64_t nt_row = bh * p.nt + t;
  int32_t* idx_row = p.idx + nt_row * p.k_max;
  float* npk_row = p.newpos_k + nt_row * p.k_max;
  float* npq_row = p.newpos_q + nt_row * T;
  int32_t* mask_row = p.mask + nt_row * p.k_max;
  int64_t carry = 0, tie_carry = 0;
  // the thread's kItems consecutive votes packed in 8 bytes (one 8-byte load where aligned and
  // in range); the next chunk's word is loaded while the current chunk is processed
  auto load_votes = [&](int64_t j0) -> uint2 {
    if (j0 + kItems <= r.hi && ((reinterpret_cast<uintptr_t>(r.v + j0) & 7u) == 0))
      return *reinterpret_cast<const uint2*>(r.v + j0);
    uint32_t x = 0u, y = 0u;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const uint32_t b = j0 + i < r.hi ? (uint32_t)r.v[j0 + i] : 0u;
      if (i < 4) x |= b << (8 * i);
      else y |= b << (8 * (i - 4));
    }
    return make_uint2(x, y);
  };
  uint2 u_next = load_votes((int64_t)tid * kItems);
  for (int64_t c0 = 0; c0 < E; c0 += kChunk) {
    const int64_t j0 = c0 + (int64_t)tid * kItems;
    const uint2 u = u_next;
    if (c0 + kChunk < E) u_next = load_votes(j0 + kChunk);
    uint32_t vb8[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) vb8[i] = ((i < 4 ? u.x : u.y) >> (8 * (i & 3))) & 255u;
    uint32_t flags = 0, tie = 0, sure = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= E) continue;
      const bool forced = F.has(j);
      const bool uni = vb8[i] != 0;
      if (!overflow) {
        if (forced || uni) sure |= 1u << i;
      } else if (forced) {
        sure |= 1u << i;
      } else if (uni && b_eff > 0) {
        const float rv = rank_value(r, j, weighted);
        if (rv > vb) sure |= 1u << i;
        else if (rv == vb) tie |= 1u << i;
      }
    }
    // chunks without any kept key (most of them: the union is sparse) only advance
    const bool has_query = j0 < tstart + T && j0 + kItems > tstart;  // npq needs these ranks
    if (!__syncthreads_or((sure | tie) != 0u || has_query)) continue;
    if (overflow) {
      int tie_total;
      const int tie_base = block_excl_sum(__popc(tie), sh_i, tie_total);
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        if ((tie >> i) & 1u) {
          const int64_t tr = tie_carry + tie_base + __popc(tie & ((1u << i) - 1u));
          if (tr < need_eq) sure |= 1u << i;
        }
      }
      tie_carry += tie_total;
    }
    flags = sure;
    int total;
    const int base = block_excl_sum(__popc(flags), sh_i, total);
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= E) break;
      const bool f = (flags >> i) & 1u;
      const int64_t before = carry + base + __popc(flags & ((1u << i) - 1u));
      const int64_t rk = before + (f ? 1 : 0) - 1;
      if (f && rk < p.k_max) {
        idx_row[rk] = (int32_t)j;
        npk_row[rk] = (float)rk;
        mask_row[rk] = F.has(j) ? -1 : (j < r.hi ? (int32_t)r.b[j] : 0);
      }
      if (j >= tstart && j < tstart + T) npq_row[j - tstart] = (float)rk;
    }
    carry += total;
  }
  __syncthreads();
  if (tstart + T > N) {
    const float last = npq_row[N - 1 - tstart];
    for (int i = tid; i < T; i += kBT)
      if (tstart + i > N - 1) npq_row[i] = last;
  }
  for (int64_t s = carry + tid; s < p.k_max; s += kBT) {
    idx_row[s] = (int32_t)N;
    npk_row[s] = 0.f;
    mask_row[s] = 0;
  }
  if (tid == 0) {
    p.usize[nt_row] = (int32_t)usize;
    p.kept_size[nt_row] = (int32_t)carry;
    p.overflow[nt_row] = overflow ? 1 : 0;
  }
}

// ---- chunk_exact selection ----------------------------------------------------------------------
struct BuildChunkP {
  const uint8_t* votes;
  const float* wvotes;
  int64_t BH, N, nt, head_stride, qbase;
  int T, k_max, n_global, n_local, C, n_chunk, weighted, mean_agg;
  int32_t* idx;
  float* newpos_k;
  float* newpos_q;
  int32_t* mask;
  int32_t* usize;
  int32_t* kept_size;
};

// dynamic smem: mass[nC] floats, then flags[nC] bytes (bit0 candidate, bit1 forced, bit2 selected)
__global__ void __launch_bounds__(kBT) build_sets_chunk_kernel(const BuildChunkP p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  const int64_t t = blockIdx.x;
  const int64_t bh = blockIdx.y;
  const int tid = threadIdx.x;
  const int64_t N = p.N;
  const int T = p.T, C = p.C;
  const int64_t tstart = p.qbase + t * T;
  const int64_t nC = (N + C - 1) / C;
  float* mass = reinterpret_cast<float*>(dsm);
  uint8_t* flag = reinterpret_cast<uint8_t*>(mass + nC);
  const int64_t off = bh * p.head_stride + tri_tile_offset(t, T, p.qbase);
  const uint8_t* v = p.votes + off;
  const float* w = p.weighted ? p.wvotes + off : nullptr;
  const int64_t hi = min(tstart + T, N);      // causal keys of the tile (votes exist below)
  const int64_t last_q = hi - 1;
  const int64_t nvis = last_q / C + 1;        // chunks with c*C <= last_q
  const int64_t gch = (p.n_global + C - 1) / C;
  const int64_t lo_c = (tstart - p.n_local + 1 > 0 ? tstart - p.n_local + 1 : 0) / C;
  const int64_t hi_c = last_q / C;

  __shared__ int sh_i[32];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int64_t s_k, s_gt;

  // chunk masses: fp32 sum of the passers' rank values in key order (chunk_agg "mean" divides by
  // the passer count, at least 1), plus candidate / forced flags
  int nu = 0, ncand = 0;
  for (int64_t c = tid; c < nC; c += kBT) {
    float m = 0.f;
    int cnt = 0;
    uint8_t f = 0;
    if (c < nvis) {
      const int64_t j1 = min((c + 1) * C, hi);
      for (int64_t j = c * C; j < j1; ++j) {
        const uint32_t vv = v[j];
        if (vv) {
          m = __fadd_rn(m, p.weighted ? w[j] : (float)vv);
          ++cnt;
        }
      }
      if (p.mean_agg) m = __fdiv_rn(m, (float)(cnt > 1 ? cnt : 1));
      const bool forced = c < gch || (c >= lo_c && c <= hi_c);
      f = forced ? 2 : 1;
      if (!forced) ++ncand;
      nu += cnt;
    }
    mass[c] = m;
    flag[c] = f;
  }
  const int usize = block_sum(nu, sh_i);
  const int n_cand = block_sum(ncand, sh_i);
  const int64_t n_take = p.n_chunk < nC ? p.n_chunk : nC;

  // top n_take candidates by mass: exact radix select of the n_take-th largest, ties to the
  // lowest chunk index
  float cut = -1.f;
  int64_t need_eq = 0;
  const bool all = n_cand <= n_take;
  if (!all && n_take > 0) {
    if (tid == 0) {
      s_prefix = 0u;
      s_k = n_take;
      s_gt = 0;
    }
    uint32_t msk = 0u;
    for (int round = 0; round < 4; ++round) {
      const int shift = 24 - 8 * round;
      for (int i = tid; i < 256; i += kBT) hist[i] = 0u;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int64_t c = tid; c < nvis; c += kBT) {
        if (flag[c] != 1) continue;
        const uint32_t key = __float_as_uint(mass[c]);
        if ((key & msk) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
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
      msk |= 255u << shift;
    }
    cut = __uint_as_float(s_prefix);
    need_eq = n_take - s_gt;
  }
  __syncthreads();
  // mark selected chunks (candidates above the cut, the first need_eq at the cut, forced)
  {
    int64_t tie_carry = 0;
    for (int64_t c0 = 0; c0 < nvis; c0 += kBT) {
      const int64_t c = c0 + tid;
      int tie = 0;
      bool sel = false;
      if (c < nvis) {
        const uint8_t f = flag[c];
        if (f == 2) sel = true;
        else if (f == 1) {
          if (all && n_take > 0) sel = true;
          else if (!all && mass[c] > cut) sel = true;
          else if (!all && mass[c] == cut) tie = 1;
        }
      }
      int tie_total;
      const int tr = block_excl_sum(tie, sh_i, tie_total);
      if (tie && tie_carry + tr < need_eq) sel = true;
      if (c < nvis && sel) flag[c] |= 4;
      tie_carry += tie_total;
    }
  }
  __syncthreads();
  // keys of the selected chunks up to the tile's last query: dense ranks, compaction
  const int64_t nt_row = bh * p.nt + t;
  int32_t* idx_row = p.idx + nt_row * p.k_max;
  float* npk_row = p.newpos_k + nt_row * p.k_max;
  float* npq_row = p.newpos_q + nt_row * T;
  int32_t* mask_row = p.mask ? p.mask + nt_row * p.k_max : nullptr;
  const int64_t E = hi;  // keys 0..last_q
  int64_t carry = 0;
  for (int64_t c0 = 0; c0 < E; c0 += kChunk) {
    const int64_t j0 = c0 + (int64_t)tid * kItems;
    uint32_t flags = 0;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j < E && (flag[j / C] & 4)) flags |= 1u << i;
    }
    int total;
    const int base = block_excl_sum(__popc(flags), sh_i, total);
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t j = j0 + i;
      if (j >= E) break;
      const bool f = (flags >> i) & 1u;
      const int64_t rk = carry + base + __popc(flags & ((1u << i) - 1u)) + (f ? 1 : 0) - 1;
      if (f && rk < p.k_max) {
        idx_row[rk] = (int32_t)j;
        npk_row[rk] = (float)rk;
        if (mask_row) mask_row[rk] = -1;
      }
      if (j >= tstart && j < tstart + T) npq_row[j - tstart] = (float)rk;
    }
    carry += total;
  }
  __syncthreads();
  if (tstart + T > N) {
    const float last = npq_row[N - 1 - tstart];
    for (int i = tid; i < T; i += kBT)
      if (tstart + i > N - 1) npq_row[i] = last;
  }
  for (int64_t s2 = carry + tid; s2 < p.k_max; s2 += kBT) {
    idx_row[s2] = (int32_t)N;
    npk_row[s2] = 0.f;
    if (mask_row) mask_row[s2] = 0;
  }
  if (tid == 0) {
    p.usize[nt_row] = usize;
    p.kept_size[nt_row] = (int32_t)carry;
  }
}

}  // namespace

int launch_build_sets_chunk(const sta_build_chunk_args* a, cudaStream_t stream) {
  if (!a || !a->votes || !a->idx || !a->newpos_k || !a->newpos_q || !a->usize || !a->kept_size)
    return fail(STA_ERR_ARG, "sta_build_sets_chunk: null pointer");
  if (a->select_score != STA_SCORE_FREQ && !a->wvotes)
    return fail(STA_ERR_ARG, "sta_build_sets_chunk: weighted ranking needs wvotes");
  if (a->chunk_size <= 0 || a->n_chunk < 0 || a->k_max <= 0 || a->tile <= 0 || a->tile > 255)
    return fail(STA_ERR_ARG, "sta_build_sets_chunk: bad chunk_size / n_chunk / k_max / tile");
  if (a->n <= 0 || a->heads <= 0) return STA_OK;
  BuildChunkP p;
  p.votes = a->votes;
  p.wvotes = a->wvotes;
  p.BH = a->heads;
  p.N = a->n;
  p.T = a->tile;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n) return fail(STA_ERR_ARG, "q_pos_base outside [0, n)");
  p.qbase = a->q_pos_base;
  p.nt = (a->n - a->q_pos_base + a->tile - 1) / a->tile;
  p.head_stride = tri_head_stride(a->n, a->tile, a->q_pos_base);
  p.k_max = a->k_max;
  p.n_global = a->n_global;
  p.n_local = a->n_local;
  p.C = a->chunk_size;
  p.n_chunk = a->n_chunk;
  p.weighted = a->select_score != STA_SCORE_FREQ;
  p.mean_agg = a->chunk_agg == 1;
  p.idx = a->idx;
  p.newpos_k = a->newpos_k;
  p.newpos_q = a->newpos_q;
  p.mask = a->mask;
  p.usize = a->usize;
  p.kept_size = a->kept_size;
  const int64_t nC = (a->n + a->chunk_size - 1) / a->chunk_size;
  const size_t smem = (size_t)nC * 5 + 16;
  if (smem > 200 * 1024) return fail(STA_ERR_UNSUPPORTED, "sta_build_sets_chunk: too many chunks");
  if (p.nt > 0x7fffffff || p.BH > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_build_sets_chunk: grid");
  cudaError_t e = cudaFuncSetAttribute(build_sets_chunk_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  dim3 grid((unsigned)p.nt, (unsigned)p.BH);
  build_sets_chunk_kernel<<<grid, kBT, smem, stream>>>(p);
  e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

int launch_build_sets(const sta_build_args* a, cudaStream_t stream) {
  if (!a || !a->votes || !a->idx || !a->newpos_k || !a->newpos_q || !a->shared_size ||
      !a->kept_size || !a->chosen || !a->overflow || !a->kpct_meas || !a->overflow20)
    return fail(STA_ERR_ARG, "sta_build_sets: null pointer");
  if (a->select_score != STA_SCORE_FREQ && !a->wvotes)
    return fail(STA_ERR_ARG, "sta_build_sets: weighted ranking needs wvotes");
  if (a->tile <= 0 || a->tile > 255 || a->k_max <= 0)
    return fail(STA_ERR_UNSUPPORTED, "sta_build_sets: tile must be in [1, 255], k_max > 0");
  if (a->n <= 0 || a->heads <= 0) return STA_OK;
  BuildP p;
  p.votes = a->votes;
  p.wvotes = a->wvotes;
  p.BH = a->heads;
  p.N = a->n;
  p.T = a->tile;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n) return fail(STA_ERR_ARG, "q_pos_base outside [0, n)");
  p.qbase = a->q_pos_base;
  p.nt = (a->n - a->q_pos_base + a->tile - 1) / a->tile;
  p.head_stride = tri_head_stride(a->n, a->tile, a->q_pos_base);
  p.k_max = a->k_max;
  p.n_global = a->n_global;
  p.n_local = a->n_local;
  int start = (int)lrintf(a->pct);  // python round(): ties to even, as lrint in default mode
  if (start < 0) start = 0;
  p.start_pct = start;
  p.nsteps = 0;
  p.steps[p.nsteps++] = start;
  if (25 < start) p.steps[p.nsteps++] = 25;
  if (20 < start) p.steps[p.nsteps++] = 20;
  p.pos_scale = a->pos_scale;
  p.weighted = a->select_score != STA_SCORE_FREQ;
  p.measure = a->measure;
  p.idx = a->idx;
  p.newpos_k = a->newpos_k;
  p.newpos_q = a->newpos_q;
  p.shared_size = a->shared_size;
  p.kept_size = a->kept_size;
  p.chosen = a->chosen;
  p.overflow = a->overflow;
  p.kpct_meas = a->kpct_meas;
  p.vote_hist = a->vote_hist;
  p.overflow20 = a->overflow20;
  if (p.nt > 0x7fffffff || p.BH > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_build_sets: grid");
  dim3 grid((unsigned)p.nt, (unsigned)p.BH);
  build_sets_kernel<<<grid, kBT, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

int launch_build_sets_pq(const sta_build_pq_args* a, cudaStream_t stream) {
  if (!a || !a->votes || !a->bits || !a->idx || !a->newpos_k || !a->newpos_q || !a->mask ||
      !a->usize || !a->kept_size || !a->overflow)
    return fail(STA_ERR_ARG, "sta_build_sets_pq: null pointer");
  if (a->tile != 32) return fail(STA_ERR_UNSUPPORTED, "sta_build_sets_pq: tile must be 32");
  if (a->select_score != STA_SCORE_FREQ && !a->wvotes)
    return fail(STA_ERR_ARG, "sta_build_sets_pq: weighted ranking needs wvotes");
  if (a->n <= 0 || a->heads <= 0) return STA_OK;
  BuildPQP p;
  p.votes = a->votes;
  p.wvotes = a->wvotes;
  p.bits = a->bits;
  p.BH = a->heads;
  p.N = a->n;
  p.T = a->tile;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n) return fail(STA_ERR_ARG, "q_pos_base outside [0, n)");
  p.qbase = a->q_pos_base;
  p.nt = (a->n - a->q_pos_base + a->tile - 1) / a->tile;
  p.head_stride = tri_head_stride(a->n, a->tile, a->q_pos_base);
  p.k_max = a->k_max;
  p.n_global = a->n_global;
  p.n_local = a->n_local;
  p.weighted = a->select_score != STA_SCORE_FREQ;
  p.idx = a->idx;
  p.newpos_k = a->newpos_k;
  p.newpos_q = a->newpos_q;
  p.mask = a->mask;
  p.usize = a->usize;
  p.kept_size = a->kept_size;
  p.overflow = a->overflow;
  if (p.nt > 0x7fffffff || p.BH > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_build_sets_pq: grid");
  dim3 grid((unsigned)p.nt, (unsigned)p.BH);
  build_sets_pq_kernel<<<grid, kBT, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? STA_OK : fail(STA_ERR_CUDA, cudaGetErrorString(e));
}

}  // namespace sta
