/*
 * sta.h -- C ABI of the B200 (sm_100a) thresholded-attention prefill library (libsta.so).
 *
 * Plain pointers and sizes only: every pointer is a CUDA device pointer unless stated
 * otherwise, every stride is in ELEMENTS, the last (head_dim) dimension of every tensor is
 * contiguous.  `stream` is a cudaStream_t passed as void*.  Every entry point returns an int
 * status (STA_OK == 0); no C++ exception crosses this boundary.  sta_last_error() returns a
 * static description of the most recent failure of the calling thread.
 *
 * Tensor conventions follow the reference's call surfaces (Vihaan-Thaker/
 * Sparse-Thresholded-Attention): q (batch*n_heads, n, d), k / v (batch*n_kv_heads, n, d)
 * (GQA-native: q head h of batch b reads kv head b*n_kv_heads + h / (n_heads / n_kv_heads);
 * the reference instead receives repeat_kv-expanded k/v, which is n_kv_heads == n_heads).
 * Batch 1 is the reference's only case (assert Z == 1, shared_selection_triton_exact_2.py:444).
 *
 * Per-(head, tile) selection arrays (votes, wvotes, bits) are stored COMPACT: tile t of a
 * head holds only its causal keys j < hi_t = min((t+1)*tile, n), at offset
 * tile*t*(t+1)/2 inside the head, heads sta_tri_head_stride(n, tile) apart.
 */
#ifndef STA_H_
#define STA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define STA_OK 0
#define STA_ERR_ARG 1          /* bad argument (null pointer, inconsistent sizes)           */
#define STA_ERR_UNSUPPORTED 2  /* shape / option this build does not support                */
#define STA_ERR_CUDA 3         /* a CUDA runtime call or launch failed                      */
#define STA_ERR_TIMEOUT 4      /* a bounded device-side wait expired (kernel unwound)       */
#define STA_ERR_WORKSPACE 5    /* workspace too small                                       */

#define STA_DTYPE_F32 0
#define STA_DTYPE_BF16 1

#define STA_SCORE_FREQ 0     /* rank by vote frequency                   */
#define STA_SCORE_MARGIN 1   /* rank by summed margin s - (m - tau)      */
#define STA_SCORE_EXPMASS 2  /* rank by summed exp(s - m)                */

#define STA_ADV_MAX 0        /* PQ-Stream: d += max_i c_i                 */
#define STA_ADV_FULL 1       /* PQ-Stream: d += slots the block occupies  */

/* ---------------------------------------------------------------------------------------
 * Library
 * ------------------------------------------------------------------------------------- */
const char* sta_last_error(void);
/* ABI version: 5 (2: query slabs, PQ-Stream pass 2 on Kernel A keep bits, decode; 3: select wait
 * limit; 4: screened select scoring, sta_select_args.screen_ws; 5: vote histograms) */
int sta_version(void);
/* Number of elements of one head of a compact selection array. */
int64_t sta_tri_head_stride(int64_t n, int32_t tile);
/* Same for a query slab starting at q_pos_base: local tile t at offset
 * t*q_pos_base + tile*t*(t+1)/2, keys j < min(q_pos_base + (t+1)*tile, n). */
int64_t sta_tri_head_stride_q(int64_t n, int32_t tile, int64_t q_pos_base);

/* ---------------------------------------------------------------------------------------
 * Stage 0 -- RoPE prologue of the selection geometry.
 * Rotates raw rows (heads, n, d) at position float(i) * pos_scale with (inv_freq, rope_scale)
 * and writes the fp32 result split into two bf16 tensors hi + lo (heads, n, d), contiguous.
 * Replaces the per-block rotations inside Kernel A (shared_selection_triton_exact_2.py:79-104).
 * ------------------------------------------------------------------------------------- */
int sta_rope_split(const void* x, int32_t dtype, int64_t heads, int64_t n, int32_t d,
                   int64_t stride_h, int64_t stride_n, const float* inv_freq, float pos_scale,
                   float rope_scale, void* out_hi, void* out_lo, void* stream);

/* Dual Chunk Attention position ids (ChunkLlama rotary tables, dca_kernel.py:194-231):
 * chunk_len L = chunk_size - local_window; role 0 linear n, 1 keys and same-chunk queries
 * n mod L, 2 queries scoring the previous chunk min(L + n mod L, chunk_size), 3 queries scoring
 * older chunks min(2L - 1, chunk_size).  Otherwise as sta_rope_split (pos_scale 1). */
int sta_rope_split_dca(const void* x, int32_t dtype, int64_t heads, int64_t n, int32_t d,
                       int64_t stride_h, int64_t stride_n, const float* inv_freq, float rope_scale,
                       int32_t chunk_size, int32_t local_window, int32_t role, void* out_hi,
                       void* out_lo, void* stream);

/* cos/sin table of a RoPE geometry: out[i * d/2 + f] = (cos(a) * rope_scale, sin(a) * rope_scale)
 * with a = fl(fl(i / R) * inv_freq[f]) (float2 pairs, len * d/2 entries; R in {1, 2, 4, -1}). */
int sta_rope_table(const float* inv_freq, int32_t d, float rope_scale, float R, int64_t len,
                   void* out, void* stream);

/* ---------------------------------------------------------------------------------------
 * Stage 1 -- exact-max two-pass selection on tcgen05 tensor cores (Kernel A).
 * Replaces _select_vote_kernel (shared_selection_triton_exact_2.py:50-140) and
 * _select_bits_kernel (shared_selection_triton_perquery.py:119-218).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_select_args {
  const void* q_hi;        /* bf16 (batch*n_heads, n, d) rotated queries, hi part */
  const void* q_lo;        /*                                           lo part */
  const void* k_hi;        /* bf16 (batch*n_kv_heads, n, d) rotated keys */
  const void* k_lo;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t n;
  int32_t d;               /* 64 or 128 */
  int32_t tile;            /* 32, 64 or 128 */
  float sm_scale;
  int32_t wmode;           /* STA_SCORE_*: 0 = no weighted votes */
  const float* tau;        /* (n_heads,) threshold per q head */
  int32_t max_only;        /* 1: pass 1 only (row max), no votes */
  uint8_t* votes;          /* compact (batch*n_heads heads), or NULL */
  float* wvotes;           /* compact, required when wmode != 0 */
  uint32_t* bits;          /* compact per-query keep bits (tile == 32 only), or NULL */
  float* row_max;          /* (batch*n_heads, n) exact row max, or NULL */
  int32_t* row_count;      /* (batch*n_heads, n) kept keys per query, or NULL */
  /* > 0: Dual Chunk Attention selection geometry with this chunk length (multiple of 256);
   * q_hi / q_lo then hold 3 planes (3, batch*n_heads, n, d): queries rotated for keys of the
   * same chunk, of the previous chunk and of older chunks (sta_rope_split_dca roles 1, 2, 3) */
  int32_t dca_chunk_len;
  /* absolute position of the first query row (multiple of 128; 0 for a whole-sequence
   * prefill).  q_hi / q_lo then hold the n - q_pos_base rows q_pos_base..n-1, k holds all n
   * keys, and row_max / row_count are (batch*n_heads, n - q_pos_base); compact arrays use the
   * layout of sta_tri_head_stride_q */
  int64_t q_pos_base;
  /* optional (tile 32, 2 passes): per (tile, key block) the maximum over the tile's queries of
   * the number of kept keys in the block -- the PQ-Stream advance before forced keys.  Blocks
   * of block_max_bn (32 or 64) keys; tile t holds ceil(hi_t / 32) bytes at offset
   * t*(q_pos_base/32) + t*(t+1)/2, heads sta_tri_head_stride_q(ceil(n/32), 1, q_pos_base/32)
   * apart; a 64-key block's entry sits at its first 32-key index. */
  uint8_t* block_max;
  int32_t block_max_bn;
  /* bound of every device-side wait of the kernel in nanoseconds (0 = the default, 4 s).  On
   * expiry the kernel unwinds and sets the device error word read by sta_device_error; the
   * call itself has already returned STA_OK (launches are asynchronous).  Small values exist
   * to exercise that failure path in tests. */
  uint64_t wait_limit_ns;
  /* optional scratch of sta_select_screen_bytes(a) bytes (256-byte aligned) enabling screened
   * scoring for unweighted votes / bits / row maxima (wmode 0): every score is first formed as
   * ONE fp16 tensor-core product, and only the (query, key) pairs whose screened score lies
   * within a proven bound of the row max or of the threshold are scored exactly (the fixed-order
   * fp32 sum of the three bf16 piece products).  Results are those of exact scoring; NULL
   * scores every pair with three bf16 products.  Measured on B200 the exact kernel is the
   * faster one at the benchmark shapes (its per-block epilogue, not the tensor products, sets
   * the pace, and screening adds a third epilogue pass); the forward entry points use
   * screening only when STA_SELECT_SCREEN=1 is set in the environment. */
  void* screen_ws;
  /* optional (tile 64 or 128, votes): per (head, local tile) the histogram of the tile's
   * nonzero vote values, (batch*n_heads, nt, tile + 1) uint32, bin v = number of keys with
   * vote v (bin 0 is left 0).  sta_build_args.vote_hist consumes it. */
  uint32_t* vote_hist;
} sta_select_args;

int sta_select(const sta_select_args* a, void* stream);
/* Bytes of sta_select_args.screen_ws for these arguments (0 for invalid shapes). */
size_t sta_select_screen_bytes(const sta_select_args* a);

/* ---------------------------------------------------------------------------------------
 * Stage 2 -- device selection of the shared path (top pct% of the pooled set with the
 * 30 -> 25 -> 20 fallback, forced global/local keys, PI repositioning, compaction).
 * Replaces _build_sets (shared_selection_triton_exact_2.py:277-426; exact.py:253-370).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_build_args {
  const uint8_t* votes;    /* compact */
  const float* wvotes;     /* compact, used when select_score != FREQ */
  int64_t heads;           /* batch*n_heads */
  int64_t n;
  int32_t tile;
  int32_t k_max;
  int32_t n_global;
  int32_t n_local;
  float pct;
  float pos_scale;         /* PI compression of the attend geometry */
  int32_t select_score;    /* STA_SCORE_* */
  int32_t measure;         /* 1: refine kpct_meas below the floor percentage */
  int32_t* idx;            /* (heads, nt, k_max) kept key positions ascending, sentinel n */
  float* newpos_k;         /* (heads, nt, k_max) */
  float* newpos_q;         /* (heads, nt, tile) */
  int32_t* shared_size;    /* (heads, nt) */
  int32_t* kept_size;      /* (heads, nt) */
  int32_t* chosen;         /* (heads, nt) percentage that fit, 0 if none */
  uint8_t* overflow;       /* (heads, nt) top-pct set exceeded k_max */
  int32_t* kpct_meas;      /* (heads, nt) */
  uint8_t* overflow20;     /* (heads, nt) still over k_max at the floor percentage */
  int64_t q_pos_base;      /* first query position (the reference's q_pos_base, shared_selection_triton_exact_2.py:291);
                            * nt = ceil((n - q_pos_base) / tile) local tiles */
  /* optional (select_score FREQ): the vote histograms sta_select wrote (vote_hist); the union
   * size and the frequency order statistic then come from them instead of a pass over the
   * votes.  NULL: computed from the votes. */
  const uint32_t* vote_hist;
} sta_build_args;

int sta_build_sets(const sta_build_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * Stage 2' -- PQ-Union selection: full union + forced, expmass (or freq) truncation of last
 * resort, dense ranks, per-slot query bitmask.
 * Replaces _build_sets_pq (shared_selection_triton_perquery.py:363-453).  Ties at the
 * truncation cut keep the lowest key indices.
 * ------------------------------------------------------------------------------------- */
typedef struct sta_build_pq_args {
  const uint8_t* votes;
  const float* wvotes;
  const uint32_t* bits;
  int64_t heads;
  int64_t n;
  int32_t tile;            /* 32 */
  int32_t k_max;
  int32_t n_global;
  int32_t n_local;
  int32_t select_score;
  int32_t* idx;
  float* newpos_k;
  float* newpos_q;
  int32_t* mask;           /* (heads, nt, k_max) bit i = query row i attends; forced = -1 */
  int32_t* usize;
  int32_t* kept_size;
  uint8_t* overflow;
  int64_t q_pos_base;      /* as sta_build_args (shared_selection_triton_perquery.py:381) */
} sta_build_pq_args;

int sta_build_sets_pq(const sta_build_pq_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * Stage 2'' -- chunk_exact selection: per-chunk (chunk_size keys) sums of the tile's passer
 * rank values, the top n_chunk visible non-forced chunks (ties: lowest chunk index) plus the
 * forced global/local chunks, causal-edge trim, dense ranks, pooled mask (-1 on valid slots).
 * Replaces _build_sets_chunk (shared_selection_triton_chunked.py:149-243).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_build_chunk_args {
  const uint8_t* votes;
  const float* wvotes;     /* compact, used when select_score != FREQ */
  int64_t heads;
  int64_t n;
  int32_t tile;
  int32_t k_max;
  int32_t n_global;
  int32_t n_local;
  int32_t chunk_size;
  int32_t n_chunk;
  int32_t select_score;
  int32_t chunk_agg;       /* 0 = sum, 1 = mean over the chunk's passers */
  int32_t* idx;
  float* newpos_k;
  float* newpos_q;
  int32_t* mask;           /* optional (NULL): -1 on valid slots, 0 on padding */
  int32_t* usize;          /* (heads, nt) passers visible to the tile */
  int32_t* kept_size;      /* (heads, nt) */
  int64_t q_pos_base;      /* as sta_build_args */
} sta_build_chunk_args;

int sta_build_sets_chunk(const sta_build_chunk_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * Stage 3 -- gather + repositioned attention over the selected slots (Kernel C / C').
 * Replaces _gather_attn_kernel (shared_selection_triton_exact_2.py:146-225) and
 * _gather_attn_pq_kernel (shared_selection_triton_perquery.py:226-312).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_attend_args {
  const void* q; int64_t q_stride_h; int64_t q_stride_n;   /* raw (batch*n_heads, n, d) */
  const void* k; int64_t k_stride_h; int64_t k_stride_n;   /* raw (batch*n_kv_heads, n, d) */
  const void* v; int64_t v_stride_h; int64_t v_stride_n;
  void* out;               /* (batch*n_heads, n, d) contiguous, dtype */
  int32_t dtype;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t n;
  int32_t d;
  int32_t tile;            /* 32 or 64 */
  int32_t k_max;
  const int32_t* idx;
  const float* newpos_k;
  const float* newpos_q;
  const int32_t* mask;     /* NULL: every query attends every valid slot */
  const int32_t* kept_size;/* (heads, nt) or NULL: bounds the slot loop (result unchanged) */
  const float* inv_freq;   /* attend geometry */
  float rope_scale;
  float sm_scale;
  /* optional: selection-geometry rows pre-rotated by sta_rope_split (bf16 hi + lo, contiguous
   * (batch*n_heads | batch*n_kv_heads, n, d)).  When same_geometry != 0 (attend and selection
   * geometries share inv_freq and rope_scale) a query / slot whose position equals
   * fl(position_index * pos_scale_sel) is bit-identical to its pre-rotated row, which is then
   * copied instead of rotated again.  Ignored for fp32 inputs. */
  const void* q_hi; const void* q_lo; const void* k_hi; const void* k_lo;
  float pos_scale_sel;
  int32_t same_geometry;
  /* optional cos/sin table of the attend geometry (sta_rope_table): positions i / R for
   * 0 <= i < rope_table_len, (cos, sin) * rope_scale pairs; a slot whose position lies on it
   * reads the table instead of evaluating sincos (bit-identical) */
  const void* rope_table;
  float rope_table_R;
  int64_t rope_table_len;
  /* first query position: q / out / q_hi / q_lo hold rows q_pos_base..n-1 (n - q_pos_base
   * rows), k / v / k_hi / k_lo all n keys (the reference's q_pos_base, shared_selection_triton_exact_2.py:169) */
  int64_t q_pos_base;
} sta_attend_args;

int sta_gather_attend(const sta_attend_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * PQ-Stream pass 2 (streamed positions + attend over the kept keys, descending key blocks).
 * Together with sta_select (2 passes, tile 32, bits + block_max + row_count) this replaces
 * _pqstream_kernel (pqstream_kernel.py:174-368).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_pqstream_args {
  const void* q; int64_t q_stride_h; int64_t q_stride_n;
  const void* k; int64_t k_stride_h; int64_t k_stride_n;
  const void* v; int64_t v_stride_h; int64_t v_stride_n;
  void* out;
  int32_t dtype;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t n;
  int32_t d;
  int32_t tile;            /* 32 */
  int32_t block_n;         /* 32 or 64 */
  /* keep decisions of the selection geometry, from sta_select (2 passes, tile 32): */
  const uint32_t* bits;    /* compact per-query keep bits */
  const uint8_t* block_max;/* block maxima with block_max_bn == block_n */
  const int32_t* row_count;/* (batch*n_heads, n - q_pos_base) kept keys per query */
  int32_t n_global;
  int32_t n_local;
  const float* inv_freq_c; /* attend geometry: base RoPE, rope_scale 1 */
  float sm_scale;
  int32_t pos_advance;     /* STA_ADV_* */
  int32_t use_skip;
  /* optional cos/sin table of the attend geometry at positions -i (sta_rope_table, R = -1) */
  const void* rope_table;
  float rope_table_R;
  int64_t rope_table_len;
  float* span;             /* (heads, nt) */
  int32_t* kept;           /* (heads, n - q_pos_base) */
  float* blocks;           /* (heads, nt) */
  float* skipped;          /* (heads, nt) */
  int64_t q_pos_base;      /* as sta_attend_args */
} sta_pqstream_args;

int sta_pqstream_attend(const sta_pqstream_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * Orchestrators: the whole prefill op in one call (replaces shared_pi_attention of
 * shared_selection_triton_exact_2.py:432-486 / YaRN:442-496 / hybrid:450-510,
 * shared_pq_attention of shared_selection_triton_perquery.py:459-525 and
 * pqstream_attention of pqstream_kernel.py:498-564).  Scratch comes from `workspace`
 * (device memory, >= the size the matching *_workspace_bytes call reports).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_forward_args {
  /* inputs */
  const void* q; int64_t q_stride_h; int64_t q_stride_n;
  const void* k; int64_t k_stride_h; int64_t k_stride_n;
  const void* v; int64_t v_stride_h; int64_t v_stride_n;
  void* out;
  int32_t dtype;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t n;
  int32_t d;
  const float* tau;                 /* (n_heads,) */
  /* selection geometry (Kernel A) */
  const float* inv_freq_a; float pos_scale_a; float rope_scale_a;
  /* attend geometry (selection repositioning + Kernel C) */
  const float* inv_freq_c; float pos_scale_c; float rope_scale_c;
  float sm_scale;
  float pct;
  int32_t n_global;
  int32_t n_local;
  int32_t tile;
  int32_t k_max;
  int32_t select_score;
  int32_t measure;
  int32_t block_n;                  /* PQ-Stream key block */
  int32_t pos_advance;              /* PQ-Stream */
  int32_t use_skip;                 /* PQ-Stream */
  /* per-(head, tile) statistics (shared: shared_size, kept_size, chosen, overflow,
   * kpct_meas, overflow20; PQ-Union: usize -> shared_size, kept_size, overflow;
   * PQ-Stream: span, kept, blocks, skipped) */
  int32_t* shared_size;
  int32_t* kept_size;
  int32_t* chosen;
  uint8_t* overflow;
  int32_t* kpct_meas;
  uint8_t* overflow20;
  float* span;
  int32_t* kept_rows;
  float* blocks;
  float* skipped;
  /* optional copies of the intermediates (NULL = keep them in the workspace only) */
  int32_t* idx_out;
  float* newpos_k_out;
  float* newpos_q_out;
  int32_t* mask_out;
  /* scratch cap: the op runs over groups of kv heads so that its workspace stays below this
   * many bytes (0 = one group holding every kv head) */
  int64_t max_workspace_bytes;
  /* optional: 5 cudaEvent_t recorded on `stream` before the RoPE prologue, before Kernel A,
   * before the selection, before the attend kernel and at the end (NULL = none); with more
   * than one kv-head group they bracket the last group */
  void* const* stage_events;
  /* 1 when the selection and attend geometries share inv_freq and rope_scale (lets the attend
   * kernel reuse pre-rotated rows, see sta_attend_args) */
  int32_t same_geometry;
  /* chunk_exact only */
  int32_t chunk_size;
  int32_t n_chunk;
  int32_t chunk_agg;
  /* > 0: the selection geometry uses Dual Chunk Attention position ids (chunk_size s, local
   * window w, chunk_len s - w a multiple of 256) with inv_freq_a / rope_scale_a */
  int32_t dca_chunk_size;
  int32_t dca_local_window;
  /* > 0: query slab.  q / out hold the n - q_pos_base queries at positions q_pos_base..n-1
   * (multiple of 128), k / v the n keys 0..n-1; per-tile statistics cover the slab's
   * ceil((n - q_pos_base) / tile) tiles and PQ-Stream kept_rows its rows.  Every query tile's
   * result is independent of the other tiles, so a sequence split into slabs reproduces the
   * whole-sequence call exactly (single-sequence multi-GPU partition). */
  int64_t q_pos_base;
} sta_forward_args;

size_t sta_shared_workspace_bytes(const sta_forward_args* a);
int sta_shared_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                       void* stream);
size_t sta_pq_union_workspace_bytes(const sta_forward_args* a);
int sta_pq_union_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                         void* stream);
size_t sta_chunk_workspace_bytes(const sta_forward_args* a);
/* chunk_exact (shared_chunk_attention, shared_selection_triton_chunked.py:249-320); statistics:
 * shared_size <- usize, kept_size */
int sta_chunk_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                      void* stream);
size_t sta_pq_stream_workspace_bytes(const sta_forward_args* a);
int sta_pq_stream_forward(const sta_forward_args* a, void* workspace, size_t workspace_bytes,
                          void* stream);

/* ---------------------------------------------------------------------------------------
 * Dense Dual Chunk Attention prefill (replaces dca_forward's prefill, dca_kernel.py:447-487:
 * the intra / succ / inter flash-attention blocks and their log-sum-exp merge, :292-366).
 * Every query attends to all its causal keys; keys are rotated at j mod L (L = chunk_size -
 * local_window), a query at the intra position for keys of its own chunk, the succ position
 * min(L + i mod L, chunk_size) for the previous chunk and the inter position
 * min(2L - 1, chunk_size) for older chunks, cos / sin multiplied by rope_scale (ChunkLlama's
 * mscale); one softmax over all of them.  chunk_size == 0: plain causal attention with RoPE at
 * the true positions.  L must be a multiple of 128.  Scores: three bf16 products of hi / lo
 * pieces of the fp32-rotated rows; P.V: P rounded to bf16 times V for bf16 inputs (as the
 * reference), hi / lo pieces of P and V (three products) for f32 inputs.
 * q_pos_base (multiple of 128): q holds the queries at positions q_pos_base .. n-1, out
 * (batch*n_heads, n - q_pos_base, d); k / v hold keys 0 .. n-1 (a decode step is the last row
 * of the slab that holds it).
 * ------------------------------------------------------------------------------------- */
typedef struct sta_dca_args {
  const void* q; int64_t q_stride_h; int64_t q_stride_n;    /* (batch*n_heads, n - q_pos_base, d) */
  const void* k; int64_t k_stride_h; int64_t k_stride_n;    /* raw (batch*n_kv_heads, n, d) */
  const void* v; int64_t v_stride_h; int64_t v_stride_n;
  void* out;               /* (batch*n_heads, n - q_pos_base, d), dtype, contiguous */
  int32_t dtype;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t n;
  int32_t d;               /* 64 or 128 */
  const float* inv_freq;   /* (d/2,) */
  float rope_scale;        /* mscale on cos / sin */
  float sm_scale;
  int32_t chunk_size;      /* s; 0 = plain causal RoPE attention */
  int32_t local_window;    /* w */
  int64_t q_pos_base;
} sta_dca_args;

size_t sta_dca_workspace_bytes(const sta_dca_args* a);
int sta_dca_forward(const sta_dca_args* a, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * Allocation-free variant of sta_shared_forward.  No counterpart in the reference: it exists
 * for hosts that may not allocate device memory themselves (plugins whose runtime owns every
 * device allocation, code under a fixed pre-reserved memory budget).  Scratch comes from a
 * STA_STATIC_SCRATCH_BYTES array of device memory that the library holds on every GPU that
 * loads it, until the process exits; the call allocates nothing.  Larger problems run over
 * smaller groups of kv heads; if one kv head needs more than the array, the call returns
 * STA_ERR_WORKSPACE.  The first call on a device looks the array up (with that device
 * current) -- make it before any stream capture.  All calls share the array and it keeps the
 * last call's contents (the op reads no scratch before writing it); calls that overlap on the
 * GPU race on it.
 * ------------------------------------------------------------------------------------- */
#define STA_STATIC_SCRATCH_BYTES (64ull << 20)
int sta_shared_forward_static(const sta_forward_args* a, void* stream);

/* ---------------------------------------------------------------------------------------
 * Decode: one query per head against the KV cache (keys 0 .. m-1, the query at position m-1).
 * Replaces the per-query selection + attend of the reference's decode paths:
 *   STA_DECODE_PI     _decode_build_sets + _decode_attend_torch
 *                     (shared_selection_triton_exact.py:464-560): threshold keep, optional
 *                     top-pct_decode of the passers, forced global / local / self, k_max cap by
 *                     score (tie-inclusive cut), PI reposition with pos_scale_c;
 *   STA_DECODE_RANK   _decode_build_sets_pq + _decode_attend_torch_pq
 *                     (shared_selection_triton_perquery.py:652-740): full set, exact-budget cap
 *                     by score (ties: lowest key index), dense-rank positions;
 *   STA_DECODE_STREAM _decode_build_sets_pqs + _decode_attend_torch (pqstream_kernel.py:694-795):
 *                     full set, no cap, streamed positions over block_n blocks, query at 0;
 *   STA_DECODE_CHUNK  _decode_build_sets_chunk + _decode_attend_torch_pq
 *                     (shared_selection_triton_chunked.py:412-483): chunks of chunk_size keys
 *                     ranked by the summed (or mean) exp(s - m) / keep count of their passers,
 *                     forced chunks + the top n_chunk others (ties: lowest chunk), self, dense
 *                     ranks.
 * Scores use the selection geometry (inv_freq_a, pos_scale_a, rope_scale_a); the attention uses
 * (inv_freq_c, rope_scale_c) at the new positions; softmax and PV in fp32.
 * ------------------------------------------------------------------------------------- */
#define STA_DECODE_PI 0
#define STA_DECODE_RANK 1
#define STA_DECODE_STREAM 2
#define STA_DECODE_CHUNK 3

typedef struct sta_decode_args {
  const void* q; int64_t q_stride_h;                        /* (batch*n_heads, d) */
  const void* k; int64_t k_stride_h; int64_t k_stride_n;    /* raw cache (batch*n_kv_heads, m, d) */
  const void* v; int64_t v_stride_h; int64_t v_stride_n;
  void* out;               /* (batch*n_heads, d), dtype */
  int32_t dtype;
  int64_t batch;
  int64_t n_heads;
  int64_t n_kv_heads;
  int64_t m;               /* keys in the cache, the query's own included */
  int32_t d;               /* 64 or 128 */
  const float* tau;        /* (n_heads,) */
  const float* inv_freq_a; float pos_scale_a; float rope_scale_a;
  const float* inv_freq_c; float pos_scale_c; float rope_scale_c;
  float sm_scale;
  int32_t mode;            /* STA_DECODE_* */
  int32_t n_global;
  int32_t n_local;
  int32_t k_max;           /* slot cap (PI, RANK); ignored by STREAM (every kept key) */
  float pct_decode;        /* PI only: < 100 keeps the top pct of the threshold passers */
  int32_t block_n;         /* STREAM: key block */
  /* optional cos/sin tables (sta_rope_table) of the selection and attend geometries */
  const void* rope_table_a; float rope_table_a_R; int64_t rope_table_a_len;
  const void* rope_table_c; float rope_table_c_R; int64_t rope_table_c_len;
  /* optional outputs: the slot set (heads, cap) with cap = k_max (PI, RANK) or m (STREAM) */
  int32_t* idx_out;
  float* newpos_k_out;
  float* newpos_q_out;     /* (heads,) */
  int32_t* kept_out;       /* (heads,) size of the final set */
  int32_t* usize_out;      /* (heads,) threshold passers */
  /* CHUNK only */
  int32_t chunk_size;
  int32_t n_chunk;
  int32_t chunk_agg;       /* 0 = sum, 1 = mean */
  int32_t select_score;    /* STA_SCORE_FREQ ranks by keep count, otherwise by exp(s - m) */
} sta_decode_args;

size_t sta_decode_workspace_bytes(const sta_decode_args* a);
int sta_decode_forward(const sta_decode_args* a, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Error word of the bounded device waits on the current device (0 = none; 101-104 name the
 * wait of the selection kernel that expired).  Kernels report an expired wait only through
 * this word -- the launching call has already returned STA_OK -- so a C caller that needs to
 * know polls it after the stream's work: it synchronises `stream`, stores the word in
 * *code_out, clears it, and returns STA_ERR_TIMEOUT when it was set. */
int sta_device_error(void* stream, int32_t* code_out);

#ifdef __cplusplus
}
#endif

#endif /* STA_H_ */
