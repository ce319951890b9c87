// Gather + repositioned attention over the selected key slots (Kernel C / C').
//
// Reference: _gather_attn_kernel, shared_selection_triton_exact_2.py:146-225 and
// _gather_attn_pq_kernel, shared_selection_triton_perquery.py:226-312.  Per (head, tile):
//   Q rotated at newpos_q (one position per query), K slot rows gathered by idx and rotated at
//   newpos_k, s = (Qr . Kr) * sm_scale, keep = causal-by-original-position & valid [& mask bit],
//   online softmax over 64-slot blocks with the reference's -inf guard, P rounded to the value
//   dtype before the PV product, out = acc / l.
// Differences in execution only: the slot loop stops at the tile's kept size instead of
// sweeping all k_max slots (padding slots contribute exactly nothing); QK runs on bf16 tensor
// cores with the rotated fp32 operands split into bf16 pieces (2 pieces / 3 products for bf16
// inputs, 3 pieces / 6 products -- fp32-accurate -- for fp32 inputs, where P and V are split
// the same way).
#include "common.cuh"
#include "mma_frag.cuh"
#include "gather_rope.cuh"
#include "sta_internal.h"

namespace sta {

namespace {


struct AttendP {
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
  int k_max;
  const int32_t* idx;
  const float* npk;
  const float* npq;
  const int32_t* mask;
  const int32_t* kept;
  const float* inv_freq;
  float rope_scale, sm_scale;
  const __nv_bfloat16 *qh, *ql, *kh, *kl;  // pre-rotated selection-geometry rows (or null)
  float ps_sel;
  int direct;                             // reuse pre-rotated rows where bit-identical
  const float2* rtab;                     // (cos, sin) * rope_scale at positions i / rtab_R
  float rtab_R;
  int64_t rtab_len;
};

// Roles: warps 0 .. T/16-1 consume (16 query rows each: QK, online softmax, PV); NPW producer
// warps gather the next slot block (idx / positions / mask, K rotated at its position or copied
// pre-rotated, V) into the other of two shared-memory stages, so loads and rotations overlap the
// tensor-core work.  Stage hand-off: named barriers FULL(s) (producers arrive, consumers wait)
// and EMPTY(s) (consumers arrive, producers wait).
constexpr int NPW = 4;
constexpr int kBarFull = 1, kBarEmpty = 3, kBarProd = 5;

template <int D, int T, bool F32>
struct AttCfg {
  static constexpr int BK = 32;              // slots per block (64 measured slower: 1 CTA / SM)
  static constexpr int LD = D + 8;           // padded smem row (bf16 elements)
  static constexpr int NQ = F32 ? 3 : 2;     // bf16 pieces of the rotated Q / K rows
  static constexpr int NV = F32 ? 3 : 1;     // pieces of P and V (1: P rounded to bf16)
  static constexpr int NCW = T / 16;         // consumer warps
  static constexpr int NTH = (NCW + NPW) * 32;
  static constexpr int KST = NQ * BK * LD;   // bf16 elements of one K stage
  static constexpr int VST = NV * BK * LD;
  static constexpr size_t SMEM = (size_t)(NQ * T * LD + 2 * (KST + VST)) * 2 + 2 * 3 * BK * 4;
};

template <int D, int T, bool F32>
__global__ void __launch_bounds__(AttCfg<D, T, F32>::NTH)
gather_attend_kernel(const AttendP p) {
  using C = AttCfg<D, T, F32>;
  using TV = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int BK = C::BK, LD = C::LD, NQ = C::NQ, NV = C::NV, NCW = C::NCW, NTH = C::NTH;
  constexpr int HALF = D / 2;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);   // [NQ][T][LD]
  __nv_bfloat16* sK = sQ + NQ * T * LD;                           // [2][NQ][BK][LD]
  __nv_bfloat16* sV = sK + 2 * C::KST;                            // [2][NV][BK][LD]
  int* sIdx = reinterpret_cast<int*>(sV + 2 * C::VST);            // [2][BK]
  float* sNpk = reinterpret_cast<float*>(sIdx + 2 * BK);          // [2][BK]
  int* sMask = reinterpret_cast<int*>(sNpk + 2 * BK);             // [2][BK]

  // grid (heads, tiles) with the tile index reversed: the last tiles of every head, which hold
  // the most kept slots, start first and the short early tiles fill the tail
  const int t = (int)(p.nt - 1 - blockIdx.y);
  const int64_t bh = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
  const bool use_mask = mask_row != nullptr;
  const bool direct = !F32 && p.direct;
  constexpr int C8 = HALF / 8;

  // ---- Q prologue (all warps): rotate at newpos_q (or reuse the pre-rotated row), split
  for (int it = tid; it < T * C8; it += NTH) {
    const int r = it / C8, f0 = (it % C8) * 8;
    const int64_t qp = p.qbase + (int64_t)t * T + r;  // absolute query position
    const int64_t ql = qp - p.qbase;                    // row in the Q slab
    const float pos = npq_row[r];
    __nv_bfloat16* dst = sQ + r * LD;
    if (direct && qp < N && pos == __fmul_rn((float)qp, p.ps_sel)) {
      copy_rotated<HALF>(p.qh + (bh * p.Nq + ql) * D, p.ql + (bh * p.Nq + ql) * D, f0, dst, T * LD);
    } else {
      rotate8<NQ, HALF>(qg + ql * p.qsn, qp < N, f0, pos, p.inv_freq, p.rope_scale, dst, T * LD,
                        p.rtab, table_index(pos, p.rtab_R, p.rtab_len));
    }
  }
  int nslots = p.k_max;
  if (p.kept) {
    const int ks = p.kept[row_base];
    nslots = ks < p.k_max ? ks : p.k_max;
  }
  const int nblocks = (nslots + BK - 1) / BK;
  __syncthreads();

  if (warp >= NCW) {
    // ================================================================ producers
    const int ptid = tid - NCW * 32;
    // slot metadata of the next block is fetched into registers while the current block's
    // rows are gathered, so each block pays one global round trip instead of two
    int nid = (int)N, nmk = -1;
    float nnp = 0.f;
    auto fetch = [&](int ib) {
      const int slot = ib * BK + ptid;
      nid = (int)N;
      nnp = 0.f;
      nmk = -1;
      if (ptid < BK && slot < p.k_max) {
        nid = idx_row[slot];
        nnp = npk_row[slot];
        if (use_mask) nmk = mask_row[slot];
      }
    };
    fetch(0);
    for (int ib = 0; ib < nblocks; ++ib) {
      const int st = ib & 1;
      if (ib >= 2) named_bar_sync(kBarEmpty + st, NTH);
      int* mIdx = sIdx + st * BK;
      float* mNpk = sNpk + st * BK;
      int* mMask = sMask + st * BK;
      if (ptid < BK) {
        mIdx[ptid] = nid;
        mNpk[ptid] = nid < N ? nnp : 0.f;
        mMask[ptid] = nmk;
      }
      named_bar_sync(kBarProd, NPW * 32);
      if (ib + 1 < nblocks) fetch(ib + 1);
      __nv_bfloat16* kdst = sK + st * C::KST;
      __nv_bfloat16* vdst = sV + st * C::VST;
      if (!F32) {
        // V rows need no transform: asynchronous copies overlap the K rotations below
        for (int it = ptid; it < BK * (D / 8); it += NPW * 32) {
          const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
          const int id = mIdx[i];
          cp_async16(vdst + i * LD + d0, vg + (int64_t)(id < N ? id : 0) * p.vsn + d0, id < N ? 16 : 0);
        }
      }
      for (int it = ptid; it < BK * C8; it += NPW * 32) {
        const int i = it / C8, f0 = (it % C8) * 8;
        const int id = mIdx[i];
        const float pos = mNpk[i];
        __nv_bfloat16* dst = kdst + i * LD;
        if (direct && id < N && pos == __fmul_rn((float)id, p.ps_sel)) {
          // the pre-rotated row is bit-identical: asynchronous copies of its hi / lo pieces
          const __nv_bfloat16* h = p.kh + (kvh * N + id) * D;
          const __nv_bfloat16* l = p.kl + (kvh * N + id) * D;
          cp_async16(dst + f0, h + f0, 16);
          cp_async16(dst + f0 + HALF, h + f0 + HALF, 16);
          cp_async16(dst + BK * LD + f0, l + f0, 16);
          cp_async16(dst + BK * LD + f0 + HALF, l + f0 + HALF, 16);
        } else {
          rotate8<NQ, HALF>(kg + (int64_t)(id < N ? id : 0) * p.ksn, id < N, f0, pos, p.inv_freq,
                            p.rope_scale, dst, BK * LD, p.rtab, table_index(pos, p.rtab_R, p.rtab_len));
        }
      }
      if (F32) {
        for (int it = ptid; it < BK * (D / 8); it += NPW * 32) {
          const int i = it / (D / 8), d0 = (it % (D / 8)) * 8;
          const int id = mIdx[i];
          __nv_bfloat16* dst = vdst + i * LD + d0;
          float x[8];
          if (id < N) {
            load8(vg + (int64_t)id * p.vsn + d0, x);
          } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = 0.f;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            __nv_bfloat16 a[NV];
            split_pieces<NV>(x[u], a);
#pragma unroll
            for (int j = 0; j < NV; ++j) dst[j * BK * LD + u] = a[j];
          }
        }
      } else {
        cp_async_wait_all();
      }
      named_bar_arrive(kBarFull + st, NTH);
    }
    return;
  }

  // ================================================================== consumers
  const int g = lane >> 2, c4 = lane & 3;
  const int mi = lane >> 3, rr = lane & 7;
  const int ra = warp * 16 + g, rb = ra + 8;  // tile-local rows of this thread
  const int64_t qpa = p.qbase + (int64_t)t * T + ra, qpb = p.qbase + (int64_t)t * T + rb;
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  for (int ib = 0; ib < nblocks; ++ib) {
    const int st = ib & 1;
    named_bar_sync(kBarFull + st, NTH);
    const __nv_bfloat16* cK = sK + st * C::KST;
    const __nv_bfloat16* cV = sV + st * C::VST;
    const int* cIdx = sIdx + st * BK;
    const int* cMask = sMask + st * BK;

    float s[BK / 8][4];
#pragma unroll
    for (int i = 0; i < BK / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[NQ][4];
      const int ar = warp * 16 + rr + (mi & 1) * 8;
      const int ac = ks * 16 + (mi >> 1) * 8;
#pragma unroll
      for (int j = 0; j < NQ; ++j)
        ldsm_x4(smem_u32(sQ + (j * T + ar) * LD + ac), a[j][0], a[j][1], a[j][2], a[j][3]);
#pragma unroll
      for (int np2 = 0; np2 < BK / 16; ++np2) {
        const int row = (2 * np2 + (mi >> 1)) * 8 + rr;
        const int col = ks * 16 + (mi & 1) * 8;
        uint32_t b0[NQ][2], b1[NQ][2];
#pragma unroll
        for (int j = 0; j < NQ; ++j)
          ldsm_x4(smem_u32(cK + (j * BK + row) * LD + col), b0[j][0], b0[j][1], b1[j][0], b1[j][1]);
        mma_pieces<NQ>(s[2 * np2], a, b0);
        mma_pieces<NQ>(s[2 * np2 + 1], a, b1);
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
        const int id = cIdx[col];
        const bool keep = id < N && qp >= id && (!use_mask || ((cMask[col] >> row) & 1));
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
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
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
          ldsm_x4_t(smem_u32(cV + (j * BK + row) * LD + col), v0[j][0], v0[j][1], v1[j][0], v1[j][1]);
        mma_pieces<NV>(o[2 * dp], pp, v0);
        mma_pieces<NV>(o[2 * dp + 1], pp, v1);
      }
    }
    if (ib + 2 < nblocks) named_bar_arrive(kBarEmpty + st, NTH);
  }

  // ---- epilogue
  TV* og = static_cast<TV*>(p.out) + bh * p.Nq * D;
  const int64_t ora = qpa - p.qbase, orb = qpb - p.qbase;  // rows of the output slab
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int col = dt * 8 + 2 * c4;
    if (qpa < N) {
      if (F32) {
        reinterpret_cast<float2*>(og + ora * D + col)[0] = make_float2(o[dt][0] / lA, o[dt][1] / lA);
      } else {
        reinterpret_cast<__nv_bfloat162*>(og + ora * D + col)[0] =
            __floats2bfloat162_rn(o[dt][0] / lA, o[dt][1] / lA);
      }
    }
    if (qpb < N) {
      if (F32) {
        reinterpret_cast<float2*>(og + orb * D + col)[0] = make_float2(o[dt][2] / lB, o[dt][3] / lB);
      } else {
        reinterpret_cast<__nv_bfloat162*>(og + orb * D + col)[0] =
            __floats2bfloat162_rn(o[dt][2] / lB, o[dt][3] / lB);
      }
    }
  }
}

template <int D, int T, bool F32>
int launch_one(const AttendP& p, cudaStream_t stream) {
  using C = AttCfg<D, T, F32>;
  auto kern = gather_attend_kernel<D, T, F32>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  dim3 grid((unsigned)p.BH, (unsigned)p.nt);
  kern<<<grid, C::NTH, C::SMEM, stream>>>(p);
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
  if (a->mask && a->tile != 32)
    return fail(STA_ERR_UNSUPPORTED, "sta_gather_attend: a per-query mask needs tile 32");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "sta_gather_attend: bad head counts");
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  {
    const int64_t es = a->dtype == STA_DTYPE_F32 ? 4 : 2;
    const uintptr_t al = reinterpret_cast<uintptr_t>(a->q) | reinterpret_cast<uintptr_t>(a->k) |
                         reinterpret_cast<uintptr_t>(a->v);
    const int64_t st = (a->q_stride_h | a->q_stride_n | a->k_stride_h | a->k_stride_n |
                        a->v_stride_h | a->v_stride_n) * es;
    if ((al & 15u) || (st & 15))
      return fail(STA_ERR_UNSUPPORTED,
                  "sta_gather_attend: q/k/v rows must start on 16-byte boundaries (pointers and "
                  "strides); pass contiguous or row-aligned views");
  }
  AttendP p;
  p.q = a->q; p.qsh = a->q_stride_h; p.qsn = a->q_stride_n;
  p.k = a->k; p.ksh = a->k_stride_h; p.ksn = a->k_stride_n;
  p.v = a->v; p.vsh = a->v_stride_h; p.vsn = a->v_stride_n;
  p.out = a->out;
  p.BH = a->batch * a->n_heads;
  p.N = a->n;
  if (a->q_pos_base < 0 || a->q_pos_base >= a->n)
    return fail(STA_ERR_ARG, "sta_gather_attend: q_pos_base outside [0, n)");
  p.qbase = a->q_pos_base;
  p.Nq = a->n - a->q_pos_base;
  p.nt = (p.Nq + a->tile - 1) / a->tile;
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
  p.qh = static_cast<const __nv_bfloat16*>(a->q_hi);
  p.ql = static_cast<const __nv_bfloat16*>(a->q_lo);
  p.kh = static_cast<const __nv_bfloat16*>(a->k_hi);
  p.kl = static_cast<const __nv_bfloat16*>(a->k_lo);
  p.ps_sel = a->pos_scale_sel;
  p.direct = a->same_geometry && a->q_hi && a->q_lo && a->k_hi && a->k_lo;
  p.rtab = static_cast<const float2*>(a->rope_table);
  p.rtab_R = a->rope_table_R;
  p.rtab_len = a->rope_table ? a->rope_table_len : 0;
  if (p.nt > 65535) return fail(STA_ERR_UNSUPPORTED, "sta_gather_attend: too many query tiles");
  const bool f32 = a->dtype == STA_DTYPE_F32;
  if (a->d == 128) {
    if (a->tile == 64) return f32 ? launch_one<128, 64, true>(p, stream) : launch_one<128, 64, false>(p, stream);
    return f32 ? launch_one<128, 32, true>(p, stream) : launch_one<128, 32, false>(p, stream);
  }
  if (a->tile == 64) return f32 ? launch_one<64, 64, true>(p, stream) : launch_one<64, 64, false>(p, stream);
  return f32 ? launch_one<64, 32, true>(p, stream) : launch_one<64, 32, false>(p, stream);
}

}  // namespace sta
