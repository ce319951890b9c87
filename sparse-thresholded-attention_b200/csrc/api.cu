// C ABI of libsta.so: argument checking, TMA descriptor encoding, workspace layout and the
// three prefill orchestrators (shared selection, PQ-Union, PQ-Stream).
//
// The orchestrators replace the reference's Python orchestration functions
// (shared_pi_attention, shared_selection_triton_exact_2.py:432-486 and the hybrid variant
// :450-510 of shared_selection_triton_hybrid_exact.py; shared_pq_attention,
// shared_selection_triton_perquery.py:459-525; pqstream_attention, pqstream_kernel.py:498-564)
// with a fixed sequence of device launches on the caller's stream and no host synchronisation.
// Scratch lives in a caller-provided workspace; when a cap is given, the op walks over groups of
// kv heads (every stage is independent per (batch, kv head)), reusing the same scratch.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "sta_internal.h"

namespace sta {

namespace {
thread_local char g_last_error[512] = "";

__device__ int g_device_error;  // bounded-wait failure code (0 = none)

int* g_err_ptr[64] = {nullptr};
}  // namespace

void set_error(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
}

int fail(int code, const char* msg) {
  set_error(msg);
  return code;
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

// ------------------------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed)
// ------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t d, uint64_t n,
                       uint64_t heads, uint32_t box_d, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  cuuint64_t dims[3] = {d, n, heads};
  cuuint64_t strides[2] = {d * 2, d * n * 2};
  cuuint32_t box[3] = {box_d, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------------------------------------
// workspace layout
// ------------------------------------------------------------------------------------------
namespace {

enum Variant { kShared = 0, kPQUnion = 1, kPQStream = 2, kChunk = 3 };

inline size_t al(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  int64_t c;          // kv heads per group
  size_t qh, ql, kh, kl, votes, wvotes, bits, idx, npk, npq, mask, rowcnt, bmax, rtab, stab, total;
  size_t scr, scr_len;  // screened-select scratch (0 length: exact three-product scoring)
  size_t vhist;         // per-tile vote histograms (shared path, frequency ranking) or 0
  float rtab_R, stab_R;
  int64_t rtab_len, stab_len;
  bool stab_shared;  // the selection table is the attend table
};

int64_t esize(int dt) { return dt == STA_DTYPE_F32 ? 4 : 2; }

// STA_SELECT_SCREEN=1 in the environment turns screened Kernel A scoring on in the forward
// entry points.  Off by default: on B200 the screened kernel's three epilogue passes cost more
// than the two products per pair it saves (cfg2: 23.7 ms vs 20.1 ms exact).
bool screen_enabled() {
  static const bool on = [] {
    const char* e = getenv("STA_SELECT_SCREEN");
    return e && e[0] == '1';
  }();
  return on;
}

Layout layout_for(const sta_forward_args* a, Variant v, int64_t c) {
  Layout L{};
  L.c = c;
  const int64_t G = a->n_heads / a->n_kv_heads;
  const int64_t qh = c * G;  // q heads in the group
  const int64_t N = a->n, D = a->d;
  const int64_t Nq = N - a->q_pos_base;  // query rows of the slab
  const int T = (v == kShared || v == kChunk) ? a->tile : 32;
  const int64_t nt = (Nq + T - 1) / T;
  const int64_t HS = tri_head_stride(N, T, a->q_pos_base);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t r = o;
    o += al(bytes);
    return r;
  };
  const int64_t qplanes = a->dca_chunk_size > 0 ? 3 : 1;
  L.qh = take(qplanes * qh * Nq * D * 2);
  L.ql = take(qplanes * qh * Nq * D * 2);
  L.kh = take(c * N * D * 2);
  L.kl = take(c * N * D * 2);
  if (v == kPQStream) {
    // Kernel A's keep bits, block maxima and per-query counts feed the streaming pass
    L.bits = take(qh * HS * 4);
    L.bmax = take(qh * tri_head_stride((N + 31) / 32, 1, a->q_pos_base / 32));
    L.rowcnt = take(qh * Nq * 4);
  } else {
    L.votes = take(qh * HS);
    if (a->select_score != STA_SCORE_FREQ) L.wvotes = take(qh * HS * 4);
    if (v == kPQUnion) L.bits = take(qh * HS * 4);
    L.idx = take(qh * nt * (int64_t)a->k_max * 4);
    L.npk = take(qh * nt * (int64_t)a->k_max * 4);
    L.npq = take(qh * nt * T * 4);
    if (v == kPQUnion) L.mask = take(qh * nt * (int64_t)a->k_max * 4);
    if (v == kShared && a->select_score == STA_SCORE_FREQ && T != 32)
      L.vhist = take(qh * nt * (T + 1) * 4);
  }
  // cos/sin table of the attend geometry: integer dense ranks (PQ-Union, chunk) or PI positions
  // at a power-of-two fraction (shared path with pos_scale_c in {1, 1/2, 1/4})
  L.rtab_R = 0.f;
  L.rtab_len = 0;
  if (v == kPQUnion || v == kChunk) {
    L.rtab_R = 1.f;
    L.rtab_len = (int64_t)a->k_max + 1;
  } else if (v == kPQStream) {
    L.rtab_R = -1.f;  // streamed positions -(d + o) are non-positive integers, |.| <= N
    L.rtab_len = N + 1;
  } else if (v == kShared) {
    for (int r = 1; r <= 4; r *= 2)
      if (a->pos_scale_c * (float)r == 1.f) {
        L.rtab_R = (float)r;
        L.rtab_len = N * r + 1;
      }
  }
  if (L.rtab_len > 0) L.rtab = take((size_t)L.rtab_len * (D / 2) * 8);
  // cos/sin table of the selection geometry for the RoPE prologue: positions j * pos_scale_a
  // (DCA position ids are integers), shared with the attend table when they coincide
  L.stab_R = 0.f;
  L.stab_len = 0;
  L.stab_shared = false;
  if (a->dca_chunk_size > 0) {
    L.stab_R = 1.f;
  } else {
    for (int r = 1; r <= 4; r *= 2)
      if (a->pos_scale_a * (float)r == 1.f) L.stab_R = (float)r;
  }
  if (L.stab_R > 0.f) {
    L.stab_len = N * (int64_t)L.stab_R + 1;
    if (v == kShared && a->same_geometry && a->dca_chunk_size <= 0 && L.rtab_R == L.stab_R &&
        a->rope_scale_a == a->rope_scale_c && L.rtab_len >= L.stab_len) {
      L.stab_shared = true;
      L.stab = L.rtab;
      L.stab_len = L.rtab_len;
    } else {
      L.stab = take((size_t)L.stab_len * (D / 2) * 8);
    }
  }
  // screened Kernel A scoring for unweighted selections (sta_select_args.screen_ws)
  if (screen_enabled() && (v == kPQStream || a->select_score == STA_SCORE_FREQ)) {
    sta_select_args s{};
    s.batch = 1;
    s.n_heads = qh;
    s.n_kv_heads = c;
    s.n = N;
    s.d = a->d;
    s.dca_chunk_len = a->dca_chunk_size > 0 ? 1 : 0;
    s.q_pos_base = a->q_pos_base;
    L.scr_len = select_screen_bytes(&s);
    if (L.scr_len > 0) L.scr = take(L.scr_len);
  }
  L.total = o;
  return L;
}

int64_t group_size(const sta_forward_args* a, Variant v) {
  const int64_t hk = a->n_kv_heads;
  if (a->max_workspace_bytes <= 0) return hk;
  const size_t per = layout_for(a, v, 1).total;
  int64_t c = (int64_t)(a->max_workspace_bytes / (int64_t)(per ? per : 1));
  if (c < 1) c = 1;
  if (c > hk) c = hk;
  while (hk % c) --c;  // equal groups
  return c;
}

int check_forward(const sta_forward_args* a, Variant v) {
  if (!a || !a->q || !a->k || !a->v || !a->out || !a->tau || !a->inv_freq_a || !a->inv_freq_c)
    return fail(STA_ERR_ARG, "forward: null pointer");
  if (a->d != 64 && a->d != 128) return fail(STA_ERR_UNSUPPORTED, "forward: head_dim must be 64 or 128");
  if (a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return fail(STA_ERR_ARG, "forward: n_heads must be a positive multiple of n_kv_heads");
  if (a->dtype != STA_DTYPE_F32 && a->dtype != STA_DTYPE_BF16)
    return fail(STA_ERR_UNSUPPORTED, "forward: dtype must be f32 or bf16");
  if ((v == kShared || v == kChunk) && a->tile != 32 && a->tile != 64)
    return fail(STA_ERR_UNSUPPORTED, "forward: tile must be 32 or 64");
  if ((v == kPQUnion || v == kPQStream) && a->tile != 32)
    return fail(STA_ERR_UNSUPPORTED, "forward: tile must be 32");
  if (v == kChunk) {
    if (a->chunk_size <= 0 || a->k_max % a->chunk_size || a->n_chunk <= 0)
      return fail(STA_ERR_ARG, "forward: chunk_exact needs chunk_size | k_max and n_chunk > 0");
    if (!(a->shared_size && a->kept_size))
      return fail(STA_ERR_ARG, "forward: chunk statistics outputs required");
  }
  if (v != kPQStream && a->k_max <= 0) return fail(STA_ERR_ARG, "forward: k_max must be > 0");
  if (a->q_pos_base < 0 || (a->n > 0 && a->q_pos_base >= a->n) || a->q_pos_base % 128)
    return fail(STA_ERR_UNSUPPORTED, "forward: q_pos_base must be a multiple of 128 below n");
  if (a->dca_chunk_size > 0) {
    const int64_t L = (int64_t)a->dca_chunk_size - a->dca_local_window;
    if (a->dca_local_window <= 0 || L <= 0 || L % 256)
      return fail(STA_ERR_UNSUPPORTED,
                  "forward: DCA needs 0 < local_window < chunk_size and chunk_size - local_window a multiple of 256");
    if (v == kPQStream) return fail(STA_ERR_UNSUPPORTED, "forward: DCA selection is not wired into PQ-Stream");
  }
  if (v == kShared && !(a->shared_size && a->kept_size && a->chosen && a->overflow &&
                        a->kpct_meas && a->overflow20))
    return fail(STA_ERR_ARG, "forward: shared statistics outputs required");
  if (v == kPQUnion && !(a->shared_size && a->kept_size && a->overflow))
    return fail(STA_ERR_ARG, "forward: PQ-Union statistics outputs required");
  if (v == kPQStream && !(a->span && a->kept_rows && a->blocks && a->skipped))
    return fail(STA_ERR_ARG, "forward: PQ-Stream statistics outputs required");
  return STA_OK;
}

size_t ws_bytes(const sta_forward_args* a, Variant v) {
  if (check_forward(a, v) != STA_OK) return 0;
  return layout_for(a, v, group_size(a, v)).total;
}

#define STA_TRY(x)                 \
  do {                             \
    const int _r = (x);            \
    if (_r != STA_OK) return _r;   \
  } while (0)

int run_forward(const sta_forward_args* a, Variant v, void* ws, size_t ws_len, cudaStream_t st) {
  STA_TRY(check_forward(a, v));
  if (a->n <= 0 || a->batch <= 0) return STA_OK;
  const int64_t c = group_size(a, v);
  const Layout L = layout_for(a, v, c);
  if (!ws || ws_len < L.total) return fail(STA_ERR_WORKSPACE, "forward: workspace too small");
  uint8_t* w = static_cast<uint8_t*>(ws);
  const int64_t H = a->n_heads, Hk = a->n_kv_heads, G = H / Hk, N = a->n;
  const int64_t qbase = a->q_pos_base, Nq = N - qbase;
  const int T = (v == kShared || v == kChunk) ? a->tile : 32;
  const int64_t nt = (Nq + T - 1) / T;
  const int64_t es = esize(a->dtype);
  const int64_t kmax = a->k_max;
  if (L.rtab_len > 0)
    STA_TRY(launch_rope_table(a->inv_freq_c, a->d, v == kShared ? a->rope_scale_c : 1.0f,
                              L.rtab_R, L.rtab_len, w + L.rtab, st));
  if (L.stab_len > 0 && !L.stab_shared)
    STA_TRY(launch_rope_table(a->inv_freq_a, a->d, a->rope_scale_a, L.stab_R, L.stab_len,
                              w + L.stab, st));
  const void* stab = L.stab_len > 0 ? w + L.stab : nullptr;
  for (int64_t b = 0; b < a->batch; ++b) {
    for (int64_t g0 = 0; g0 < Hk; g0 += c) {
      const int64_t h0 = b * H + g0 * G;   // first q head (flattened over batch)
      const int64_t k0 = b * Hk + g0;      // first kv head
      const int64_t qn = c * G;
      const uint8_t* q = static_cast<const uint8_t*>(a->q) + h0 * a->q_stride_h * es;
      const uint8_t* k = static_cast<const uint8_t*>(a->k) + k0 * a->k_stride_h * es;
      const uint8_t* vv = static_cast<const uint8_t*>(a->v) + k0 * a->v_stride_h * es;
      uint8_t* out = static_cast<uint8_t*>(a->out) + h0 * Nq * a->d * es;
      const float* tau = a->tau + g0 * G;
      auto mark = [&](int i) {
        if (a->stage_events) cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), st);
      };
      mark(0);
      const bool dca = a->dca_chunk_size > 0;
      const int64_t dL = dca ? (int64_t)a->dca_chunk_size - a->dca_local_window : 0;
      if (!dca) {
        STA_TRY(launch_rope_split(q, a->dtype, qn, Nq, a->d, a->q_stride_h, a->q_stride_n,
                                  a->inv_freq_a, a->pos_scale_a, a->rope_scale_a, w + L.qh,
                                  w + L.ql, st, 0, 0, 0, qbase, stab, L.stab_R, L.stab_len));
        STA_TRY(launch_rope_split(k, a->dtype, c, N, a->d, a->k_stride_h, a->k_stride_n,
                                  a->inv_freq_a, a->pos_scale_a, a->rope_scale_a, w + L.kh,
                                  w + L.kl, st, 0, 0, 0, 0, stab, L.stab_R, L.stab_len));
      } else {
        const size_t plane = (size_t)qn * Nq * a->d * 2;
        for (int role = 1; role <= 3; ++role)
          STA_TRY(launch_rope_split(q, a->dtype, qn, Nq, a->d, a->q_stride_h, a->q_stride_n,
                                    a->inv_freq_a, 1.0f, a->rope_scale_a,
                                    w + L.qh + (role - 1) * plane, w + L.ql + (role - 1) * plane,
                                    st, role, dL, a->dca_chunk_size, qbase, stab, L.stab_R,
                                    L.stab_len));
        STA_TRY(launch_rope_split(k, a->dtype, c, N, a->d, a->k_stride_h, a->k_stride_n,
                                  a->inv_freq_a, 1.0f, a->rope_scale_a, w + L.kh, w + L.kl, st,
                                  1, dL, a->dca_chunk_size, 0, stab, L.stab_R, L.stab_len));
      }
      sta_select_args s{};
      s.q_hi = w + L.qh;
      s.q_lo = w + L.ql;
      s.k_hi = w + L.kh;
      s.k_lo = w + L.kl;
      s.batch = 1;
      s.n_heads = qn;
      s.n_kv_heads = c;
      s.n = N;
      s.d = a->d;
      s.tile = T;
      s.sm_scale = a->sm_scale;
      s.tau = tau;
      s.dca_chunk_len = (int32_t)dL;
      s.q_pos_base = qbase;
      s.screen_ws = L.scr_len > 0 ? w + L.scr : nullptr;
      mark(1);
      if (v == kPQStream) {
        s.bits = reinterpret_cast<uint32_t*>(w + L.bits);
        s.block_max = w + L.bmax;
        s.block_max_bn = a->block_n;
        s.row_count = reinterpret_cast<int32_t*>(w + L.rowcnt);
        STA_TRY(launch_select(&s, st));
        mark(2);
        sta_pqstream_args pa{};
        pa.q = q; pa.q_stride_h = a->q_stride_h; pa.q_stride_n = a->q_stride_n;
        pa.k = k; pa.k_stride_h = a->k_stride_h; pa.k_stride_n = a->k_stride_n;
        pa.v = vv; pa.v_stride_h = a->v_stride_h; pa.v_stride_n = a->v_stride_n;
        pa.out = out;
        pa.dtype = a->dtype;
        pa.batch = 1;
        pa.n_heads = qn;
        pa.n_kv_heads = c;
        pa.n = N;
        pa.d = a->d;
        pa.tile = 32;
        pa.block_n = a->block_n;
        pa.bits = reinterpret_cast<uint32_t*>(w + L.bits);
        pa.block_max = w + L.bmax;
        pa.row_count = reinterpret_cast<int32_t*>(w + L.rowcnt);
        pa.n_global = a->n_global;
        pa.n_local = a->n_local;
        pa.inv_freq_c = a->inv_freq_c;
        pa.sm_scale = a->sm_scale;
        pa.pos_advance = a->pos_advance;
        pa.use_skip = a->use_skip;
        pa.rope_table = L.rtab_len > 0 ? w + L.rtab : nullptr;
        pa.rope_table_R = L.rtab_R;
        pa.rope_table_len = L.rtab_len;
        pa.span = a->span + h0 * nt;
        pa.kept = a->kept_rows + h0 * Nq;
        pa.q_pos_base = qbase;
        pa.blocks = a->blocks + h0 * nt;
        pa.skipped = a->skipped + h0 * nt;
        mark(3);
        STA_TRY(launch_pqstream(&pa, st));
        mark(4);
        continue;
      }
      s.wmode = a->select_score;
      s.votes = w + L.votes;
      s.wvotes = a->select_score != STA_SCORE_FREQ ? reinterpret_cast<float*>(w + L.wvotes) : nullptr;
      s.bits = v == kPQUnion ? reinterpret_cast<uint32_t*>(w + L.bits) : nullptr;
      s.vote_hist = L.vhist ? reinterpret_cast<uint32_t*>(w + L.vhist) : nullptr;
      STA_TRY(launch_select(&s, st));
      mark(2);
      int32_t* idx = a->idx_out ? a->idx_out + h0 * nt * kmax : reinterpret_cast<int32_t*>(w + L.idx);
      float* npk = a->newpos_k_out ? a->newpos_k_out + h0 * nt * kmax : reinterpret_cast<float*>(w + L.npk);
      float* npq = a->newpos_q_out ? a->newpos_q_out + h0 * nt * T : reinterpret_cast<float*>(w + L.npq);
      int32_t* mask = nullptr;
      if (v == kShared) {
        sta_build_args ba{};
        ba.votes = w + L.votes;
        ba.wvotes = s.wvotes;
        ba.vote_hist = s.vote_hist;
        ba.heads = qn;
        ba.n = N;
        ba.tile = T;
        ba.k_max = a->k_max;
        ba.n_global = a->n_global;
        ba.n_local = a->n_local;
        ba.pct = a->pct;
        ba.pos_scale = a->pos_scale_c;
        ba.select_score = a->select_score;
        ba.measure = a->measure;
        ba.idx = idx;
        ba.newpos_k = npk;
        ba.newpos_q = npq;
        ba.shared_size = a->shared_size + h0 * nt;
        ba.kept_size = a->kept_size + h0 * nt;
        ba.chosen = a->chosen + h0 * nt;
        ba.overflow = a->overflow + h0 * nt;
        ba.kpct_meas = a->kpct_meas + h0 * nt;
        ba.overflow20 = a->overflow20 + h0 * nt;
        ba.q_pos_base = qbase;
        STA_TRY(launch_build_sets(&ba, st));
      } else if (v == kChunk) {
        int32_t* cmask = a->mask_out ? a->mask_out + h0 * nt * kmax : nullptr;
        sta_build_chunk_args ba{};
        ba.votes = w + L.votes;
        ba.wvotes = s.wvotes;
        ba.heads = qn;
        ba.n = N;
        ba.tile = T;
        ba.k_max = a->k_max;
        ba.n_global = a->n_global;
        ba.n_local = a->n_local;
        ba.chunk_size = a->chunk_size;
        ba.n_chunk = a->n_chunk;
        ba.select_score = a->select_score;
        ba.chunk_agg = a->chunk_agg;
        ba.idx = idx;
        ba.newpos_k = npk;
        ba.newpos_q = npq;
        ba.mask = cmask;
        ba.usize = a->shared_size + h0 * nt;
        ba.kept_size = a->kept_size + h0 * nt;
        ba.q_pos_base = qbase;
        STA_TRY(launch_build_sets_chunk(&ba, st));
      } else {
        mask = a->mask_out ? a->mask_out + h0 * nt * kmax : reinterpret_cast<int32_t*>(w + L.mask);
        sta_build_pq_args ba{};
        ba.votes = w + L.votes;
        ba.wvotes = s.wvotes;
        ba.bits = reinterpret_cast<uint32_t*>(w + L.bits);
        ba.heads = qn;
        ba.n = N;
        ba.tile = 32;
        ba.k_max = a->k_max;
        ba.n_global = a->n_global;
        ba.n_local = a->n_local;
        ba.select_score = a->select_score;
        ba.idx = idx;
        ba.newpos_k = npk;
        ba.newpos_q = npq;
        ba.mask = mask;
        ba.usize = a->shared_size + h0 * nt;
        ba.kept_size = a->kept_size + h0 * nt;
        ba.overflow = a->overflow + h0 * nt;
        ba.q_pos_base = qbase;
        STA_TRY(launch_build_sets_pq(&ba, st));
      }
      mark(3);
      sta_attend_args ca{};
      ca.q = q; ca.q_stride_h = a->q_stride_h; ca.q_stride_n = a->q_stride_n;
      ca.k = k; ca.k_stride_h = a->k_stride_h; ca.k_stride_n = a->k_stride_n;
      ca.v = vv; ca.v_stride_h = a->v_stride_h; ca.v_stride_n = a->v_stride_n;
      ca.out = out;
      ca.dtype = a->dtype;
      ca.batch = 1;
      ca.n_heads = qn;
      ca.n_kv_heads = c;
      ca.n = N;
      ca.d = a->d;
      ca.tile = T;
      ca.k_max = a->k_max;
      ca.idx = idx;
      ca.newpos_k = npk;
      ca.newpos_q = npq;
      ca.mask = mask;
      ca.kept_size = a->kept_size + h0 * nt;
      ca.inv_freq = a->inv_freq_c;
      ca.rope_scale = v == kShared ? a->rope_scale_c : 1.0f;
      ca.sm_scale = a->sm_scale;
      ca.q_hi = w + L.qh;
      ca.q_lo = w + L.ql;
      ca.k_hi = w + L.kh;
      ca.k_lo = w + L.kl;
      ca.pos_scale_sel = a->pos_scale_a;
      ca.same_geometry = (v == kShared && a->same_geometry && !dca) ? 1 : 0;
      ca.rope_table = L.rtab_len > 0 ? w + L.rtab : nullptr;
      ca.rope_table_R = L.rtab_R;
      ca.rope_table_len = L.rtab_len;
      ca.q_pos_base = qbase;
      STA_TRY(launch_gather_attend(&ca, st));
      mark(4);
    }
  }
  return STA_OK;
}

}  // namespace
}  // namespace sta

// ==========================================================================================
// extern "C" entry points
// ==========================================================================================
using namespace sta;

extern "C" {

const char* sta_last_error(void) { return g_last_error; }

int sta_version(void) { return 5; }

int64_t sta_tri_head_stride(int64_t n, int32_t tile) { return tri_head_stride(n, tile); }

int64_t sta_tri_head_stride_q(int64_t n, int32_t tile, int64_t q_pos_base) {
  return tri_head_stride(n, tile, q_pos_base);
}

int sta_rope_split(const void* x, int32_t dtype, int64_t heads, int64_t n, int32_t d,
                   int64_t stride_h, int64_t stride_n, const float* inv_freq, float pos_scale,
                   float rope_scale, void* out_hi, void* out_lo, void* stream) {
  if (!x || !inv_freq || !out_hi || !out_lo) return fail(STA_ERR_ARG, "sta_rope_split: null pointer");
  if (d <= 0 || (d & 1)) return fail(STA_ERR_ARG, "sta_rope_split: d must be even");
  if (dtype != STA_DTYPE_F32 && dtype != STA_DTYPE_BF16)
    return fail(STA_ERR_UNSUPPORTED, "sta_rope_split: dtype");
  return launch_rope_split(x, dtype, heads, n, d, stride_h, stride_n, inv_freq, pos_scale,
                           rope_scale, out_hi, out_lo, static_cast<cudaStream_t>(stream));
}

int sta_rope_split_dca(const void* x, int32_t dtype, int64_t heads, int64_t n, int32_t d,
                       int64_t stride_h, int64_t stride_n, const float* inv_freq, float rope_scale,
                       int32_t chunk_size, int32_t local_window, int32_t role, void* out_hi,
                       void* out_lo, void* stream) {
  if (!x || !inv_freq || !out_hi || !out_lo) return fail(STA_ERR_ARG, "sta_rope_split_dca: null pointer");
  if (d <= 0 || (d & 1)) return fail(STA_ERR_ARG, "sta_rope_split_dca: d must be even");
  if (role < 0 || role > 3 || local_window <= 0 || chunk_size <= local_window)
    return fail(STA_ERR_ARG, "sta_rope_split_dca: bad role / chunk_size / local_window");
  if (dtype != STA_DTYPE_F32 && dtype != STA_DTYPE_BF16)
    return fail(STA_ERR_UNSUPPORTED, "sta_rope_split_dca: dtype");
  return launch_rope_split(x, dtype, heads, n, d, stride_h, stride_n, inv_freq, 1.0f, rope_scale,
                           out_hi, out_lo, static_cast<cudaStream_t>(stream), role,
                           (int64_t)chunk_size - local_window, chunk_size);
}

int sta_rope_table(const float* inv_freq, int32_t d, float rope_scale, float R, int64_t len,
                   void* out, void* stream) {
  if (!inv_freq || !out) return fail(STA_ERR_ARG, "sta_rope_table: null pointer");
  if (d <= 0 || (d & 1) || !(R == 1.f || R == 2.f || R == 4.f || R == -1.f))
    return fail(STA_ERR_ARG, "sta_rope_table: d even, R in {1, 2, 4, -1}");
  return launch_rope_table(inv_freq, d, rope_scale, R, len, out, static_cast<cudaStream_t>(stream));
}

int sta_select(const sta_select_args* a, void* stream) {
  return launch_select(a, static_cast<cudaStream_t>(stream));
}

size_t sta_select_screen_bytes(const sta_select_args* a) { return select_screen_bytes(a); }

int sta_build_sets(const sta_build_args* a, void* stream) {
  return launch_build_sets(a, static_cast<cudaStream_t>(stream));
}

int sta_build_sets_pq(const sta_build_pq_args* a, void* stream) {
  return launch_build_sets_pq(a, static_cast<cudaStream_t>(stream));
}

int sta_build_sets_chunk(const sta_build_chunk_args* a, void* stream) {
  return launch_build_sets_chunk(a, static_cast<cudaStream_t>(stream));
}

int sta_gather_attend(const sta_attend_args* a, void* stream) {
  return launch_gather_attend(a, static_cast<cudaStream_t>(stream));
}

int sta_pqstream_attend(const sta_pqstream_args* a, void* stream) {
  return launch_pqstream(a, static_cast<cudaStream_t>(stream));
}

size_t sta_shared_workspace_bytes(const sta_forward_args* a) { return ws_bytes(a, kShared); }
size_t sta_pq_union_workspace_bytes(const sta_forward_args* a) { return ws_bytes(a, kPQUnion); }
size_t sta_pq_stream_workspace_bytes(const sta_forward_args* a) { return ws_bytes(a, kPQStream); }
size_t sta_chunk_workspace_bytes(const sta_forward_args* a) { return ws_bytes(a, kChunk); }

int sta_chunk_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                      void* stream) {
  return run_forward(a, kChunk, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace sta {
int check_shared_forward(const sta_forward_args* a) { return check_forward(a, kShared); }
}  // namespace sta

extern "C" {

int sta_shared_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return run_forward(a, kShared, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int sta_pq_union_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return run_forward(a, kPQUnion, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int sta_pq_stream_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                          void* stream) {
  return run_forward(a, kPQStream, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

size_t sta_decode_workspace_bytes(const sta_decode_args* a) { return decode_workspace_bytes(a); }

int sta_decode_forward(const sta_decode_args* a, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return decode_forward(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int sta_device_error(void* stream, int32_t* code_out) {
  int* p = device_error_word();
  if (!p) return fail(STA_ERR_CUDA, "sta_device_error: symbol lookup failed");
  int host = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&host, p, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  if (code_out) *code_out = host;
  if (host != 0) {
    const int zero = 0;
    cudaMemcpyAsync(p, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
  }
  return host != 0 ? fail(STA_ERR_TIMEOUT, "a bounded device wait expired") : STA_OK;
}

}  // extern "C"
