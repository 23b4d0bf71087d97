/*
 * lumen_cuda.h — C ABI of the B200 (sm_100a) TurboQuant KV cache.
 *
 * This is the drop-in boundary for the TurboQuant compressed-KV path of
 * rabbitson87/lumen-rs. Every entry point names the reference interface it
 * replaces (paths are inside that project):
 *   crates/lumen-core/src/compressor.rs        TurboQuantCompressor
 *   crates/lumen-core/src/{rotation,lloyd_max,qjl}.rs   table files
 *   crates/turboquant-cache/src/traits.rs      trait KVCache
 *   crates/turboquant-cache/src/simple.rs      SimpleCache
 *   crates/lumen-mlx/src/native_cache.rs       NativeRotatingKvCacheTurboQuant
 *   crates/lumen-mlx/src/turboquant.rs         turboquant_fused_attn
 *
 * Conventions
 *  - Every call returns an int status: LC_OK (0) or a negative LC_ERR_*.
 *    lc_last_error() returns a message for the last failure on this thread.
 *    No C++ exception crosses the ABI.
 *  - Plain pointers and sizes only. A data pointer may be host memory or
 *    device memory of the cache's device; the library tells them apart and
 *    stages host buffers itself. Caller buffers are borrowed for the call.
 *  - `stream` is a cudaStream_t passed as void*; NULL means the library's
 *    own (non-blocking) stream for that object; pass cudaStreamLegacy
 *    ((void*)0x1) for the legacy default stream. Calls that return host
 *    results synchronise.
 *  - A handle is thread-compatible, not thread-safe: one thread at a time,
 *    matching the reference's `&mut self`.
 */
#ifndef LUMEN_CUDA_H
#define LUMEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define LC_OK 0
#define LC_ERR_INVALID (-1)  /* bad argument, shape or handle */
#define LC_ERR_BITS (-2)     /* bit width outside the accepted range */
#define LC_ERR_REFUSED (-3)  /* rollback refused (native_cache.rs:304-335) */
#define LC_ERR_CUDA (-4)     /* CUDA runtime error */
#define LC_ERR_TIMEOUT (-5)  /* a bounded device wait ran out */
#define LC_ERR_NOMEM (-6)    /* page pool or device memory exhausted */
#define LC_ERR_IO (-7)       /* file I/O failure */
#define LC_ERR_MAGIC (-8)    /* table file with the wrong magic */
#define LC_ERR_STATE (-9)    /* call not valid in the handle's state */

/* Message for the last failing call on this thread ("" if none). */
const char* lc_last_error(void);

/* Element types of caller tensors. */
#define LC_F32 0
#define LC_BF16 1
#define LC_F16 2

/* ---- codec tables (one TurboQuantCompressor) --------------------------- */
typedef struct lc_codec lc_codec;

/* TurboQuantCompressor::new (compressor.rs:20-32): rotation from `seed`,
 * QJL projection from `seed + 1`, Lloyd-Max codebook with `lloyd_max_iter`
 * EM iterations. The rotation and projection come from this library's own
 * seeded generator (SplitMix64 + Box-Muller, then the reference's
 * Gram-Schmidt construction), not from Rust's StdRng: for the reference's
 * exact tables, load its files with lc_codec_from_files. bits: 1..8. */
int lc_codec_new(uint32_t bits, uint64_t qjl_m, uint64_t seed, uint64_t lloyd_max_iter,
                 uint64_t head_dim, lc_codec** out);

/* TurboQuantCompressor::from_files (compressor.rs:43-58): TQCB codebook
 * (lloyd_max.rs:187-213), TQRM rotation (rotation.rs:130-150) and TQJL
 * projection (qjl.rs:248-272) files. */
int lc_codec_from_files(const char* codebook_path, const char* rotation_path, const char* qjl_path,
                        lc_codec** out);

/* Same tables from host arrays: rotation [d*d] row-major f32, boundaries
 * [2^bits + 1] f64 (first -inf, last +inf), centroids [2^bits] f64, qjl
 * projection [m*d] row-major f32 (may be NULL when qjl_m == 0). */
int lc_codec_from_tables(uint64_t head_dim, uint32_t bits, uint64_t qjl_m, const float* rotation,
                         const double* boundaries, const double* centroids, const float* qjl_proj,
                         lc_codec** out);

/* RotationMatrix::save / LloydMaxCodebook::save / QJLProjector::save. */
int lc_codec_save(const lc_codec* c, const char* codebook_path, const char* rotation_path,
                  const char* qjl_path);

/* Copy the tables out (any pointer may be NULL). */
int lc_codec_tables(const lc_codec* c, float* rotation, double* boundaries, double* centroids,
                    float* qjl_proj);

/* head_dim, bits, qjl_m. */
int lc_codec_shape(const lc_codec* c, uint64_t* head_dim, uint32_t* bits, uint64_t* qjl_m);

void lc_codec_free(lc_codec* c);

/* ---- bit packing (bitpack.rs:11-52) ------------------------------------ */
/* packed_words(n, bits): u64 words for n codes, 64/bits codes per word. */
uint64_t lc_packed_words(uint64_t n, uint32_t bits);

/* ---- the cache --------------------------------------------------------- */
typedef struct lc_cache lc_cache;

/* Store flags. */
#define LC_STORE_K_QJL 1u /* keep the K stage-2 QJL bits + residual norm */
#define LC_STORE_V_QJL 2u /* keep the V stage-2 QJL bits + residual norm */
/* keep per-page key bounds for page-sparse decode (LC_SPARSE_PAGES): the
 * elementwise min and max of the dequantized rotated keys of every full
 * 64-token page, the PageDigest of native_cache.rs:350-365 over the codes */
#define LC_STORE_DIGEST 4u
/* store V un-rotated, the Qwen TurboQuant layout (qwen3_5_moe.rs:2774-2781:
 * V is Lloyd-Max quantized as it is, "so no un-rotation step is needed on
 * read"): the V codec's rotation is taken as the identity, so codes, sigma,
 * QJL bits and lc_fetch hold the un-rotated quantization, and decode writes
 * sum_t p_t v_t with no R^T. K stays rotated. Not recorded in LKV2 files:
 * load a snapshot into a cache created with the same flag. */
#define LC_STORE_V_UNROTATED 8u

typedef struct lc_cache_config {
  int32_t n_layers;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t max_seqs;  /* sequence slots 0..max_seqs-1 */
  int64_t max_pages; /* page pool size; a page holds 256 tokens of every kv head of one layer */
  int64_t max_pages_per_seq; /* block-table width per (sequence, layer) */
  uint32_t store_flags;      /* LC_STORE_* */
  int32_t device;            /* CUDA device ordinal */
  int32_t step_prealloc;     /* 1: S=1 updates write in place (LUMEN_NATIVE_KV_STEP_PREALLOC) */
  int32_t reserved;
  /* Per-layer ring geometry; NULL => every layer is full (append-only).
   * max_size 0 marks a full layer; otherwise the sliding window size, with
   * keep sink tokens (native_cache.rs:1541-1550: keep < max_size). */
  const int64_t* layer_max_size;
  const int64_t* layer_keep;
} lc_cache_config;

/* SimpleCache::new (simple.rs:60-74) generalised to many sequences and to
 * mlx-lm ring layers. k_codec and v_codec may be the same handle; both must
 * have head_dim == config->head_dim. The codecs are copied to the device. */
int lc_cache_create(const lc_cache_config* config, const lc_codec* k_codec, const lc_codec* v_codec,
                    lc_cache** out);
void lc_cache_destroy(lc_cache* cache);

/* KVCache::store (traits.rs:14, simple.rs:123-135) for one (seq, layer,
 * kv head): keys/values [n_tokens, head_dim] f32, compressed on the GPU.
 * Full layers only; heads of a layer may hold different lengths. */
int lc_store(lc_cache* cache, int32_t seq, int32_t layer, int32_t head, const float* keys,
             const float* values, int64_t n_tokens);

/* KVCache::attend_keys (traits.rs:19; compressor.rs:165-184): stage-1
 * scores of `query` [head_dim] f32 against every cached key of (seq,
 * layer, head). scores: n_scores >= lc_seq_len floats. */
int lc_attend_keys(lc_cache* cache, int32_t seq, int32_t layer, int32_t head, const float* query,
                   float* scores, int64_t n_scores);

/* KVCache::attend_values (traits.rs:24; simple.rs:76-99, 142-155):
 * sum_t w_t * R^T(c_t * sigma_t), weights with |w| < 1e-10 skipped.
 * out: head_dim floats. */
int lc_attend_values(lc_cache* cache, int32_t seq, int32_t layer, int32_t head, const float* weights,
                     int64_t n_weights, float* out);

/* TurboQuantCompressor::estimate_inner_products (compressor.rs:122-159):
 * the two-stage scores of `query` [head_dim] f32 against every cached key
 * of (seq, layer, head): stage 1 (as lc_attend_keys) plus the QJL
 * correction ||r|| * sqrt(pi/2) / sqrt(m) * sum_i sign_i (Phi query)_i
 * (qjl.rs:76-119; 0 when ||r|| < 1e-10), in the reference's f32 order.
 * Needs a cache created with LC_STORE_K_QJL (LC_ERR_STATE otherwise). */
int lc_attend_keys_qjl(lc_cache* cache, int32_t seq, int32_t layer, int32_t head, const float* query,
                       float* scores, int64_t n_scores);

/* KVCache::seq_len (traits.rs:27). Negative on error. */
int64_t lc_seq_len(const lc_cache* cache, int32_t seq, int32_t layer, int32_t head);

/* KVCache::clear (traits.rs:30): every sequence, every layer. */
int lc_clear(lc_cache* cache);

/* KVCache::truncate (traits.rs:36, simple.rs:174-185): cap every head of
 * (seq, layer) at n_keep tokens; no-op when already shorter. */
int lc_truncate(lc_cache* cache, int32_t seq, int32_t layer, int64_t n_keep);

/* Quantize-on-append + NativeRotatingKvCacheTurboQuant::update_and_fetch
 * (native_cache.rs:1756-1793; with LC_STORE_K_QJL set, update_and_fetch_qjl
 * :1805-1856). keys/values: [n_seqs, n_kv_heads, n_tokens, head_dim] of
 * `dtype`, un-rotated; the kernel rotates, normalises, quantizes, packs and
 * (if stored) computes the QJL bits exactly as compress_one
 * (compressor.rs:61-107). Every listed sequence advances by n_tokens. */
int lc_append(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
              const void* keys, const void* values, int32_t dtype, int64_t n_tokens, void* stream);

/* lc_append with RoPE applied to the keys first: the prefill-side fusion of
 * the TQ layers' encode (gemma4_moe.rs:4385-4432 rotates and quantizes K
 * after RoPE), here taking the projection outputs before RoPE. Token t of
 * sequence b sits at position p = (tokens the layer held before the call) +
 * t; pair i < rope_dims / 2 turns by p * rope_base^(-2i / rope_dims)
 * (angle in f64, cos and sin rounded to f32 on the host), pairs
 * (i, i + rope_dims / 2) or, with traditional != 0, (2i, 2i + 1); dims past
 * rope_dims are left as they are. Values are not rotated. The result equals
 * lc_append of the keys with that RoPE applied in f32. */
int lc_append_rope(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                   const void* keys, const void* values, int32_t dtype, int64_t n_tokens, int32_t rope_dims,
                   double rope_base, int32_t traditional, void* stream);

/* NativeRotatingKvCacheTurboQuant::truncate_to (native_cache.rs:1728-1746
 * -> ring_truncate :304-335): LC_ERR_REFUSED if target > offset or the ring
 * has rotated (offset > max_size). */
int lc_truncate_to(lc_cache* cache, int32_t seq, int32_t layer, int64_t target);

/* Prefix reuse through the block table: dst (emptied first) receives the
 * first prefix_len tokens of src in every layer by sharing src's pages
 * (copy-on-write); no data is copied. The reference shares prefixes only for
 * plain layers (native_cache.rs:459-527) and deep-clones TurboQuant layers
 * (:1581-1610); sharing is refused like a rollback when a ring has rotated. */
int lc_fork(lc_cache* cache, int32_t src_seq, int32_t dst_seq, int64_t prefix_len);

/* Drop every page of one sequence (all layers). */
int lc_release(lc_cache* cache, int32_t seq);

/* Ring counters of (seq, layer): offset (tokens ever pushed), idx (write
 * index), buf_len (backing buffer length, cached_len), view_len (tokens the
 * last update returned / decode attends). Any pointer may be NULL. */
int lc_ring_state(const lc_cache* cache, int32_t seq, int32_t layer, int64_t* offset, int64_t* idx,
                  int64_t* buf_len, int64_t* view_len);

/* What lc_fetch copies out. */
#define LC_FETCH_VIEW 0    /* the tokens update_and_fetch returned */
#define LC_FETCH_BACKING 1 /* the whole backing buffer (padding, stale slots) */

typedef struct lc_fetch_out {
  uint64_t* k_words;  /* [n_kv_heads, n, packed_words(d, k_bits)] */
  float* k_sigma;     /* [n_kv_heads, n] */
  uint64_t* v_words;  /* [n_kv_heads, n, packed_words(d, v_bits)] */
  float* v_sigma;     /* [n_kv_heads, n] */
  uint64_t* k_qjl;    /* [n_kv_heads, n, ceil(m/64)] (LC_STORE_K_QJL) */
  float* k_rnorm;     /* [n_kv_heads, n] */
  uint64_t* v_qjl;    /* [n_kv_heads, n, ceil(m/64)] (LC_STORE_V_QJL) */
  float* v_rnorm;     /* [n_kv_heads, n] */
} lc_fetch_out;

/* Copy (seq, layer)'s stored vectors to host buffers in the reference's
 * CompressedVector layout (config.rs:30-46): packed u64 code words, sigma,
 * QJL words, residual norm. NULL fields are skipped. *n_out gets n. */
int lc_fetch(lc_cache* cache, int32_t seq, int32_t layer, int32_t which, lc_fetch_out* out,
             int64_t max_tokens, int64_t* n_out);

/* ---- LKV2 snapshots (crates/lumen-mlx/src/kv_disk.rs) ----------------------
 * The reference's on-disk prompt-cache format (layout kv_disk.rs:285-323):
 * "LKV2", version 2, a JSON KvManifest with its CRC-32, then typed records
 * each with its CRC-32. A saved sequence has one LayerMeta per cache layer,
 * kind FullTurboquant or SlidingTurboquant, carrying offset, idx, keep,
 * max_size, bits (K; "v_bits" too when V differs) and qjl_m, and the arrays
 * of turboquant_meta (kv_disk.rs:2000-2024): keys_codes u8 [1,H,S,D],
 * keys_sigma f32 [1,H,S,1], values_codes, values_sigma, and with
 * LC_STORE_K_QJL keys_signs bf16 +-1 [1,H,S,m] and keys_residual_norm f32
 * [1,H,S,1]; with LC_STORE_V_QJL the V signs and residual norms follow in
 * slots 6 and 7. S is the ring's backing length, rows in backing order. */

/* Write sequence `seq`'s layers to `path` (written to path.tmp, then
 * renamed). model_fingerprint may be NULL (""); prefix_tokens are stored in
 * the manifest. LC_ERR_STATE for a layer filled by lc_store with per-head
 * lengths; LC_ERR_IO on a write failure. */
int lc_save_lkv2(lc_cache* cache, int32_t seq, const char* path, const char* model_fingerprint,
                 const uint32_t* prefix_tokens, int64_t n_prefix_tokens);

/* Replace sequence `seq`'s layers with the snapshot in `path`. Everything is
 * checked before the cache changes: LC_ERR_MAGIC (magic, version), LC_ERR_IO
 * (CRC mismatch, truncation, trailing bytes, record length != shape x dtype,
 * malformed manifest), LC_ERR_STATE (model_fingerprint given and different),
 * LC_ERR_BITS (bit widths), LC_ERR_INVALID (layer count, kind, max_size /
 * keep, shapes, codes out of range, signs not +-1, missing QJL arrays the
 * cache keeps), LC_ERR_NOMEM (not enough free pages). */
int lc_load_lkv2(lc_cache* cache, int32_t seq, const char* path, const char* model_fingerprint);

/* Read and check an LKV2 file on the host only (no device): layer count,
 * record count and the manifest's position. Same error codes as
 * lc_load_lkv2's file checks. */
int lc_lkv2_info(const char* path, int64_t* n_layers, int64_t* n_records, uint64_t* position);

/* Decode flags. */
#define LC_Q_ROTATED 1u   /* q is already R q (Gemma path); skip the rotation */
#define LC_OUT_ROTATED 2u /* leave the output in the rotated basis (R baked into Wo) */
/* Score every key with the two-stage estimate of estimate_inner_products
 * (compressor.rs:122-159): stage 1 plus the QJL stage-2 correction of the
 * stored K sign bits and residual norm. Needs a cache created with
 * LC_STORE_K_QJL (LC_ERR_STATE otherwise), qjl_m <= 256 and the un-rotated
 * query (with LC_Q_ROTATED: LC_ERR_INVALID). Not taken by
 * lc_decode_attn_noalloc (LC_ERR_INVALID). */
#define LC_QJL_SCORES 4u
/* Page-sparse decode (sdpa_page_sparse, native_attention.rs:217-329, on the
 * codes): once a sequence holds 16384 keys or more (SPARSE_DECODE_MIN_KEYS),
 * each (sequence, kv head) attends to the 64-token pages whose bound
 * sum_d max(q'_d max_d, q'_d min_d), maxed over its query heads, is largest,
 * plus the first page and the 4 most recent full pages and the undigested
 * tail: max(pages / 8, 64) pages in all (sparse_keep_pages). q' is the
 * rotated query; min and max come from the digest. Needs a cache created with
 * LC_STORE_DIGEST (LC_ERR_STATE), a full (non-sliding) layer and one of the
 * tensor-core geometries with GQA <= 4: 4-bit K/V at head_dim 128, or 3-bit
 * K / 2-bit V at head_dim 256 (LC_ERR_INVALID otherwise); not combined with
 * LC_QJL_SCORES. Below 16384 keys the decode is dense. */
#define LC_SPARSE_PAGES 8u

/* Decode attention over the compressed cache, one query token per
 * sequence: out = softmax(scale * q K_dq^T) V_dq for every query head, with
 * GQA (query head h reads kv head h / (n_q_heads / n_kv_heads)).
 * turboquant_fused_attn (turboquant.rs:887-923) / SimpleCache attend_keys +
 * softmax + attend_values. q, out: [n_seqs, n_q_heads, head_dim]. */
int lc_decode_attn(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                   const void* q, int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags,
                   void* out, int32_t out_dtype, void* stream);

/* Masked (causal) attention of a prefill chunk over the compressed cache:
 * the tq layers' prefill branch of gemma4_moe.rs:4636-4660 (queries against
 * the dequantized codes, causal mask, scale) computed on the codes. The
 * chunk's K/V must already be appended: q [n_q_tokens, n_q_heads, head_dim]
 * holds the queries of the last n_q_tokens tokens of (seq, layer)'s view, and
 * query i attends to the first view_len - n_q_tokens + i + 1 tokens. out has
 * q's shape. Flags as lc_decode_attn. LC_ERR_STATE on a sliding layer whose
 * ring has wrapped (its view is not in token order); LC_ERR_INVALID if
 * n_q_tokens exceeds the view. 4-bit K/V at head_dim 128 with GQA <= 8
 * (and no QJL / sparse flag) runs a tensor-core kernel that dequantizes each
 * key tile once for 128 (token, head) query rows; other geometries run the
 * split-K decode with one virtual sequence per query token, whose cost grows
 * as n_q_tokens x prefix. */
int lc_prefill_attn(lc_cache* cache, int32_t layer, int32_t seq, const void* q, int32_t q_dtype,
                    int32_t n_q_tokens, int32_t n_q_heads, float scale, uint32_t flags, void* out,
                    int32_t out_dtype, void* stream);

/* One decode step of a layer: NativeRotatingKvCacheTurboQuant::
 * update_and_fetch of each sequence's new token followed by
 * turboquant_fused_attn on the rotated query (gemma4_moe.rs:4245-4797), as
 * lc_append (keys / values [n_seqs, n_kv_heads, 1, head_dim]) then
 * lc_decode_attn. The queries are rotated by the launch that rotates and
 * quantizes the new keys, and the attention takes them rotated; results as
 * the two calls (same flags, including LC_OUT_ROTATED). */
int lc_decode_step(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
                   const void* values, int32_t kv_dtype, const void* q, int32_t q_dtype, int32_t n_q_heads,
                   float scale, uint32_t flags, void* out, int32_t out_dtype, void* stream);

/* lc_decode_step for the layers layer0 .. layer0 + n_layers - 1 of one
 * decode step, in order, from one call: the per-layer arrays are stacked
 * [n_layers][...] (keys / values [n_layers][n_seqs][n_kv_heads][1][head_dim],
 * q and out [n_layers][n_seqs][n_q_heads][head_dim]); results as n_layers
 * lc_decode_step calls. No counterpart in the reference, whose layer loop
 * (gemma4_moe.rs:4245-4797) makes the two calls per layer itself: this entry
 * takes the per-layer crossing of a foreign-function boundary out of a
 * caller's step, for callers (benchmarks, a replayed decode schedule) whose
 * layers' inputs are ready together. */
int lc_decode_step_layers(lc_cache* cache, int32_t layer0, int32_t n_layers, int32_t n_seqs,
                          const int32_t* seq_ids, const void* keys, const void* values, int32_t kv_dtype,
                          const void* q, int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, void* out,
                          int32_t out_dtype, void* stream);

/* Bytes of the fixed device scratch lc_decode_attn_noalloc uses, per device. */
#define LC_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* lc_decode_attn for callers that cannot allocate device memory while they
 * decode: an engine that reserved all free HBM for its own pool before its
 * serving loop (cudaMalloc then fails), or a loop that must not take the
 * device-wide synchronisation of cudaFree. No counterpart in the reference:
 * its decode runs inside MLX, which allocates per call.
 *
 * Same arguments, results and error codes as lc_decode_attn, except:
 *  - q and out must be device memory (LC_ERR_INVALID otherwise).
 *  - All scratch (rotated queries, split-K partials, per-call metadata) is a
 *    fixed device array of LC_NOALLOC_SCRATCH_BYTES (32 MiB) per device plus
 *    a fixed 1 MiB host staging array. A call that needs more returns
 *    LC_ERR_NOMEM, with the bytes needed in lc_last_error(). The need is
 *    about rows * head_dim * 6 + rows * splits * (head_dim + 2) * 4 bytes
 *    for rows = n_seqs * n_q_heads, where splits is the number of split-K
 *    partials per row (12 for 32 sequences x 8 kv heads at 8K tokens: about
 *    7 MB in all).
 *  - A successful call makes no cudaMalloc, cudaMallocHost or cudaFree and
 *    calls no allocating library routine.
 *  - The first call on a device sets the scratch up: with that device
 *    current it looks up the array's address (cudaGetSymbolAddress). Make
 *    that first call before any stream capture.
 *  - Every call on a device, from any cache, uses the same scratch: calls
 *    that overlap on the GPU (issued on different streams without ordering)
 *    race and return wrong results. Issue them on one stream, or order them.
 *    A NULL stream means the cache's own stream, which differs between
 *    caches: a caller with several caches on one device passes them one
 *    shared stream, or orders the calls itself.
 *  - The kernels it launches are not timed by lc_cache_timing. */
int lc_decode_attn_noalloc(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                           const void* q, int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags,
                           void* out, int32_t out_dtype, void* stream);

/* Same, but stop before normalisation and return the softmax partials of
 * the whole local context per (seq, q head): m (log2 domain, max of
 * scale*log2(e)*score), l (sum of 2^(s-m)), o [head_dim] (unnormalised, in
 * the rotated basis). For one context split by sequence across devices. */
int lc_decode_attn_partials(lc_cache* cache, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                            const void* q, int32_t q_dtype, int32_t n_q_heads, float scale,
                            uint32_t flags, float* m, float* l, float* o, void* stream);

/* Merge n_parts sets of partials [n_parts, n_rows] (m, l) and
 * [n_parts, n_rows, head_dim] (o) into out [n_rows, head_dim], un-rotating
 * with the cache's V rotation unless LC_OUT_ROTATED: the combine of partial
 * softmax states of native_quant_attention.rs:190-207, for one context split
 * by sequence (e.g. partials all-gathered from the ranks holding its
 * shards). Device inputs are read in place; with device inputs and output
 * the call is asynchronous on `stream`. */
int lc_merge_partials(lc_cache* cache, int32_t n_parts, int32_t n_rows, const float* m,
                      const float* l, const float* o, uint32_t flags, void* out, int32_t out_dtype,
                      void* stream);

/* ---- one context split by tokens over GPUs ------------------------------
 * The reference keeps a sequence on one device; its merge of partial
 * softmax states (native_quant_attention.rs:190-207) combines chunks of one
 * context. A group is the set of ranks (one process per GPU, one node)
 * that each hold a contiguous token shard of the same sequences in their
 * own cache: lc_decode_attn_split computes this rank's partials, exchanges
 * them with every rank and merges, with no host round trip. */
typedef struct lc_group lc_group;
#define LC_GROUP_ID_BYTES 128
/* Force the NCCL all-gather exchange instead of peer stores. */
#define LC_GROUP_NCCL 1u

/* A new group id (ncclGetUniqueId): made by one rank, sent to the others
 * by the caller (any side channel). */
int lc_group_id(uint8_t* id);

/* Collective: every rank of the group calls it with the same id, world,
 * max_rows and head_dim. max_rows bounds n_seqs * n_q_heads of a call.
 * The ranks map each other's exchange buffers (CUDA IPC) and exchange
 * partials by stores over NVLink with release flags; where that mapping
 * fails on any rank (or with LC_GROUP_NCCL) all ranks use an in-place
 * ncclAllGather instead. world <= 8. */
int lc_group_create(int32_t world, int32_t rank, const uint8_t* id, int32_t device, int32_t max_rows,
                    int32_t head_dim, uint32_t flags, lc_group** out);

/* world, rank, and 1 if the exchange uses peer stores (0: NCCL). */
int lc_group_info(const lc_group* group, int32_t* world, int32_t* rank, int32_t* peer_stores);

/* LC_ERR_TIMEOUT once an exchange's bounded wait for a peer's partials ran
 * out (a rank failed or stopped calling); its output rows were NaN and the
 * group takes no more calls. LC_OK otherwise. Reads a host word, no sync. */
int lc_group_status(const lc_group* group);

/* Local: waits for this device's work, unmaps the peers and frees. Peers
 * write into this rank's buffer, so every rank must be past its last
 * lc_decode_attn_split (a barrier of the caller's) before any destroys. */
int lc_group_destroy(lc_group* group);

/* lc_decode_attn over sequences whose tokens are split across the group's
 * ranks: seq_ids name this rank's shard slots in `cache`; every rank calls
 * it with the same layer, n_seqs, n_q_heads, scale, flags and queries (the
 * same q on every rank) in the same order. Each rank's out receives the
 * attention over the whole split context. Flags as lc_decode_attn except
 * LC_SPARSE_PAGES. LC_ERR_TIMEOUT if an earlier exchange of the group
 * timed out (lc_group_status). */
int lc_decode_attn_split(lc_cache* cache, lc_group* group, int32_t layer, int32_t n_seqs,
                         const int32_t* seq_ids, const void* q, int32_t q_dtype, int32_t n_q_heads,
                         float scale, uint32_t flags, void* out, int32_t out_dtype, void* stream);

/* Device id, stream and last-kernel count (kernels this library launched). */
int lc_cache_info(const lc_cache* cache, int32_t* device, void** stream, uint64_t* kernel_launches);

/* Per-kernel device time from CUDA events recorded on the launching stream
 * around the split-K attention kernel and the quantize-append kernel (and,
 * in other_ms, the query rotation and partial-merge kernels of decode).
 * mode 1: start recording (clears earlier records); mode 0: stop and
 * report; mode 2: report and keep recording. Reporting synchronises the
 * recorded events. Any output pointer may be NULL. */
int lc_cache_timing(lc_cache* cache, int32_t mode, double* decode_ms, uint64_t* decode_launches,
                    double* append_ms, uint64_t* append_launches, double* other_ms);

/* ---- the raw ring (native_cache.rs:65-335) ------------------------------
 * N parallel buffers of arbitrary row width moving in lockstep, with
 * mlx-lm RotatingKVCache semantics: the update path of
 * NativeRotatingKvCacheTurboQuant::update_and_fetch(_qjl) on pre-quantized
 * tuples, device-resident. */
typedef struct lc_ring lc_ring;

/* n_bufs buffers, row_bytes[i] bytes per (head, token) row. */
int lc_ring_create(int32_t n_heads, int64_t max_size, int64_t keep, int32_t n_bufs,
                   const int64_t* row_bytes, int32_t device, lc_ring** out);

/* ring_update (native_cache.rs:277-290): news[i] is [n_heads, n_tokens,
 * row_bytes[i]] (host or device). prealloc mirrors
 * LUMEN_NATIVE_KV_STEP_PREALLOC. */
int lc_ring_update(lc_ring* ring, const void* const* news, int64_t n_tokens, int32_t prealloc,
                   void* stream);

/* ring_truncate (native_cache.rs:304-335). */
int lc_ring_truncate_to(lc_ring* ring, int64_t target);

int lc_ring_counters(const lc_ring* ring, int64_t* offset, int64_t* idx, int64_t* buf_len,
                     int64_t* view_len);

/* Copy buffer `buf` ([n_heads, n, row_bytes]) to host: which =
 * LC_FETCH_VIEW (what the last update returned) or LC_FETCH_BACKING. Returns
 * n via *n_out; LC_ERR_STATE when the ring holds no buffers yet. */
int lc_ring_read(lc_ring* ring, int32_t buf, int32_t which, void* dst, int64_t dst_bytes,
                 int64_t* n_out);

/* NativeRotatingKvCacheTurboQuant::clear (native_cache.rs:1712-1721). */
int lc_ring_clear(lc_ring* ring);

/* deep_clone (native_cache.rs:1581-1610). */
int lc_ring_deep_clone(const lc_ring* ring, lc_ring** out);

void lc_ring_destroy(lc_ring* ring);

/* Library version string. */
const char* lc_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LUMEN_CUDA_H */
