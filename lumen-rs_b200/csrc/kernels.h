// Launchers for the sm_100a kernels (defined in the .cu files).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>
#include <vector>

#include "common.h"

namespace lc {

// ---- row copies between paged and linear spaces (ring_kernels.cu) --------
struct CopyRowsArgs {
  RowSpace src, dst;
  PageLayout layout;
  const int64_t* src_rows = nullptr;  // device: source row of dst row i; null -> src_begin + i
  int64_t src_begin = 0, dst_begin = 0, n = 0;
  int32_t zero = 0;           // write zeros instead of copying
  uint32_t role_mask = ~0u;   // roles to touch
};
void launch_copy_rows(const CopyRowsArgs& a, cudaStream_t s);

// ---- codec tables on the device ------------------------------------------
struct CodecDev {
  int32_t dim = 0, bits = 0, n_levels = 0, m = 0, words = 0, qwords = 0;
  const float* R = nullptr;     // [d][d] row-major (R[i][j])
  const float* RT = nullptr;    // [d][d] RT[j][i] = R[i][j]
  const float* PT = nullptr;    // [d][m] PT[j][r] = Phi[r][j]
  const float* thr = nullptr;   // [n-1] smallest f32 >= boundary[k], k = 1..n-1
  const float* cent = nullptr;  // [n] centroids as f32 (lloyd_max.rs:157-159)
};

// ---- quantize-append (append.cu) ------------------------------------------
// Vectors are enumerated (seq s, head hl, token t) over src[side]
// [n_seqs][h_in][n_tok][dim]; vector (s, hl, t) lands in page dst_page[s*n_tok+t],
// row dst_row[s*n_tok+t], head h_base + hl.
struct AppendArgs {
  CodecDev codec[2];
  const void* src[2] = {nullptr, nullptr};
  int32_t dtype = LC_F32;
  int32_t n_seqs = 0, h_in = 0, h_base = 0;
  int64_t n_tok = 0;
  const uint64_t* dst_page = nullptr;  // [n_seqs * n_tok] device, or null: h_page / h_row
  const int32_t* dst_row = nullptr;
  const uint64_t* h_page = nullptr;    // host copies passed in the launch parameters
  const int32_t* h_row = nullptr;      // (at most kAppendInline slots)
  PageLayout layout;
  int32_t role_words[2] = {-1, -1}, role_sigma[2] = {-1, -1};
  int32_t role_qjl[2] = {-1, -1}, role_rnorm[2] = {-1, -1};
  // RoPE on the K side before the rotation (lc_append_rope): per (sequence,
  // token) slot rope_half (cos, sin) f32 pairs; null: no RoPE
  const float* rope_cs = nullptr;
  int32_t rope_half = 0, rope_traditional = 0;
  // queries of the same decode step to rotate in this launch (lc_decode_step):
  // q_out[r][:] = R q[r][:] (K codec R, f32) for r < q_rows; null: none
  const void* q = nullptr;
  int32_t q_dtype = LC_F32, q_rows = 0;
  float* q_out = nullptr;
};
// Whether launch_append can rotate a decode step's queries in the same
// launch (warp kernel with the K rotation staged in shared memory).
bool append_rotates_queries(int64_t n_vec, int dim, int m_max, bool stage2);
// Appends of at most this many (sequence, token) slots pass their destinations
// in the launch parameters.
constexpr int kAppendInline = 64;
void launch_append(const AppendArgs& a, cudaStream_t s);
// Dynamic shared memory the append kernel needs for head_dim d and qjl m.
size_t append_smem_bytes(int d, int m);

// ---- prefill attention with K/V tile reuse (prefill.cu) ---------------------
// The last L tokens of one sequence's view (in token order) attend causally
// to the view: query token i (0-based in the chunk) sees keys 0 ..
// n_total - L + i. A CTA takes one kv head and a block of query tokens (all
// G heads of each); every 64-key tile is dequantized once into shared memory
// for its 128 query rows. 4-bit K and V, head_dim 128, G <= 8. One launch:
// the kernel rotates its queries and writes the normalised, un-rotated rows
// (token * hq + head) itself.
struct PrefillArgs {
  const uint64_t* table_row = nullptr;  // the sequence's block-table row (page addresses)
  int64_t n_total = 0;                  // tokens in the view
  int32_t L = 0, hkv = 0, hq = 0;
  int64_t off_kw = 0, off_vw = 0, off_ks = 0, off_vs = 0;  // PageLayout offsets
  const void* q = nullptr;  // [L][hq][128] raw queries (f32 / bf16 / f16)
  int32_t q_dtype = 0, q_rotated = 0;  // q_rotated: q is already R q
  float qscale = 1.0f;                 // scale * log2(e) / kalpha
  const float* kR = nullptr;           // K codec R (row-major): q' = R q
  const float* vRT = nullptr;          // V codec R^T (row-major); null leaves the output rotated
  const float* kcent = nullptr;        // [16]
  const float* vcent = nullptr;        // [16]
  float kalpha = 1.0f, valpha = 1.0f;
  // precise tiles: when max sigma_K of a tile x max ||q'|| of the block
  // exceeds pthr, the scores add the K table's residual products
  // (decode_klo_thr, as the decode kernels)
  float pthr = 3.0e38f;
  void* out = nullptr;  // [L][hq][128], out_dtype
  int32_t out_dtype = 0;
  float oscale = 1.0f;  // 1 / valpha
};
bool prefill_tiled_path(int dim, int kbits, int vbits, int G);
void launch_prefill_tiled(const PrefillArgs& a, cudaStream_t s);

// ---- decode attention (decode.cu) ------------------------------------------
struct DecodeArgs {
  const uint64_t* table = nullptr;  // block table: row seq_ids[b] holds the page addresses of sequence b
  int64_t table_stride = 0;         // u64 entries per table row
  const int64_t* seqinfo = nullptr; // [n_seqs][2]: (tokens to attend, table row)
  const int64_t* seg = nullptr;     // flat path: [n_seqs + 1] tile prefix over (seq, kv head)
  PageLayout layout;
  int32_t role_kw = 0, role_vw = 1, role_ks = 2, role_vs = 3;
  int32_t n_seqs = 0, hkv = 0, hq = 0, dim = 0;
  int32_t kbits = 4, vbits = 4;
  const float* q_rot = nullptr;   // [n_seqs][hq][dim] f32, rotated and scaled by scale*log2(e)
  // the tensor-core 3/2-bit kernel can read already-rotated raw queries
  // instead (q_rot then unused): q_raw [n_seqs][hq][dim] of q_raw_dtype, times
  // q_raw_scale
  const void* q_raw = nullptr;
  int32_t q_raw_dtype = 0;
  float q_raw_scale = 1.0f;
  // the tensor-core 3/2-bit kernel with one chunk per (sequence, kv head):
  // it writes the normalised rows itself, out = R^T (o / l) x fin_oscale in
  // fin_dtype (fin_R row-major R of the V codec; null leaves them rotated),
  // and no merge follows; null fin_out: partials as usual
  void* fin_out = nullptr;
  int32_t fin_dtype = 0;
  const float* fin_R = nullptr;
  float fin_oscale = 1.0f;
  const __half* q_h = nullptr;    // same in f16
  const float* kcent = nullptr;   // [2^kbits]
  const float* vcent = nullptr;   // [2^vbits]
  float kalpha = 1.0f, valpha = 1.0f;  // f16 table scales of the fast path
  // Fast path score precision: a tile adds the K table's f16 residuals
  // (alpha c_k - f16(alpha c_k)) to its scores when some token's sigma_K
  // exceeds klo_thr / ||q'|| (q' = the head group's scaled rotated queries)
  // and it lies within kLoTheta of the running max (decode_klo_thr).
  float klo_thr = 0.0f;
  float* part = nullptr;          // [n_seqs][hkv][max_slots][G][dim + 2]  (m, l, o...)
  // With seqinfo == nullptr the per-call arrays are host copies passed in the
  // launch parameters (decode_inline_fits): seqinfo, seg, cnt as above.
  const int64_t* h_seqinfo = nullptr;
  const int64_t* h_seg = nullptr;
  const int32_t* h_cnt = nullptr;
  // QJL stage-2 scores (generic path only): q_proj [n_seqs][hq][qjl_m] f32 =
  // (Phi q) * scale * log2(e); null: stage-1 scores.
  const float* q_proj = nullptr;
  int32_t role_kq = -1, role_kr = -1, qjl_m = 0;
  // page-sparse decode (flat pair path): logical -> physical tiles, see DecodeDev
  const int32_t* tile_map = nullptr;
  int32_t map_stride = 0;
  float qjl_c = 0.f;  // sqrt(pi/2) / sqrt(qjl_m)
};

// ---- page-sparse decode (sparse.cu) -----------------------------------------
constexpr int kDigestPage = 64;                          // DIGEST_PAGE (native_cache.rs:351)
constexpr int kGroupsPerPage = kPageTokens / kDigestPage;  // digest pages per cache page
constexpr int kSparseSink = 1, kSparseRecent = 4;        // SPARSE_SINK_PAGES / _RECENT_PAGES
constexpr int64_t kSparseMinKeys = 16384;                // SPARSE_DECODE_MIN_KEYS
constexpr int kTileTokens = 32;                          // tokens per decode tile
// pages kept of `pages` digested ones (sparse_keep_pages, native_attention.rs:327-329)
inline int64_t sparse_keep_pages(int64_t pages) { return std::max<int64_t>(pages / 8, 64); }

struct DigestDev {
  const uint64_t* pages;  // [items] page address of each 64-token page to digest
  const int32_t* row0;    // [items] its first row in the page (multiple of 64)
  const float* cent;      // K centroids (f32)
  int64_t off_kw, off_ks, off_dg, row_kw, row_dg;
  int32_t bits, dim;
};
void launch_digest(const DigestDev& a, int64_t n_items, int heads, cudaStream_t s);

struct SelectDev {
  const int64_t* seqinfo;  // [n_seqs][2] (tokens, table row), device
  const uint64_t* table;
  int64_t table_stride;
  const void* q;           // [n_seqs][hq][dim] queries as given (q_dtype)
  int32_t q_dtype, q_rotated;
  const float* RT;         // [dim][dim] R^T of the key codec
  int64_t off_dg, row_dg;
  int32_t n_seqs, hkv, hq, G, dim;
  int32_t npad;            // >= the most digested pages of any sequence
  int32_t map_stride;      // tiles per (sequence, kv head) row of tile_map
  int32_t* tile_map;       // [n_seqs * hkv][map_stride] logical -> physical tile
};
void launch_page_select(const SelectDev& a, cudaStream_t s);

// Largest qjl_m the decode's QJL scores take (8 projection rows per lane).
constexpr int kMaxQjlDecode = 256;

// q_proj[r][i] = qscale * sum_j Phi[i][j] q[r][j] (PT = Phi^T, [dim][m]).
void launch_project_q(const void* q, int32_t dtype, int32_t n_rows, int32_t dim, int32_t m, const float* PT,
                      float qscale, float* q_proj, cudaStream_t s);

// Per-call decode arrays that fit in the launch parameters.
constexpr int kInlineSeqs = 64;
constexpr int kInlineCnt = 1024;
inline bool decode_inline_fits(int n_seqs, int hkv) {
  return n_seqs <= kInlineSeqs && (int64_t)n_seqs * hkv <= kInlineCnt;
}

// How a decode call is split: the flat tile-balanced fast path (one partial
// slot per warp range touching a (seq, kv head)) or the chunked generic path
// (one slot per chunk of pages_per_chunk pages).
struct DecodePlan {
  bool flat = false;
  bool mma = false;  // chunked, on the tensor cores (decode_mma_path geometry)
  int32_t grid = 0;
  int64_t per_warp = 1, total_tiles = 0;
  int32_t max_slots = 1;
  int32_t pages_per_chunk = 4, n_chunks = 1;
  int32_t max_cta_segs = 0;  // flat: most (seq, kv head) segments one CTA touches
  std::vector<int64_t> seg;  // [n_seqs + 1]
  std::vector<int32_t> cnt;  // [n_seqs * hkv] slots used per (seq, kv head)
};
// generic_only: take the chunked generic path even where the fast path
// applies (QJL scores).
DecodePlan plan_decode(const std::vector<int64_t>& lens, int hkv, int hq, int dim, int kbits, int vbits,
                       bool generic_only = false);
int num_sms();
// The chunked geometry with a tensor-core kernel: 3-bit K, 2-bit V, head_dim
// 256, up to 4 query heads per kv head.
bool decode_mma_path(int dim, int kbits, int vbits, int G);

// q_rot[s][h][:] = (R q[s][h]) * qscale (R applied unless q_is_rotated)
void launch_rotate_q(const void* q, int32_t q_dtype, int32_t n_rows, int32_t dim, const float* R,
                     bool q_is_rotated, float qscale, float* q_rot, __half* q_h, cudaStream_t s);
void launch_decode_partials(const DecodeArgs& a, const DecodePlan& p, cudaStream_t s);

// One-launch decode for the flat path with G <= 4 when every CTA touches few
// enough segments (decode_fusable): the kernel rotates its queries, and the
// warp completing a (seq, kv head) merges its partials; the CTA then writes
// the un-rotated rows. Rows of sequences with no tokens are not written.
struct FusedArgs {
  const void* q = nullptr;       // [n_seqs][hq][dim] raw queries
  int32_t q_dtype = 0, q_rotated = 0;
  float qscale = 1.0f;           // scale * log2(e) / kalpha
  const float* qR = nullptr;     // K codec R (row-major)
  const float* vRT = nullptr;    // V codec R^T (row-major); null leaves the output rotated
  const int32_t* cnt = nullptr;  // [n_seqs * hkv] partial slots (plan.cnt on the device)
  int32_t* ctr = nullptr;        // [n_seqs * hkv] zero on entry; left zero
  void* out = nullptr;
  int32_t out_dtype = 0;
  float oscale = 1.0f;           // 1 / valpha
  // softmax partials instead of `out` (m [rows], l [rows], o [rows][dim],
  // rotated and unnormalised, back to back), for a split context's shard
  float* parts = nullptr;
  int32_t parts_rows = 0;
};
bool decode_fusable(const DecodePlan& p, int G);
void launch_decode_fused(const DecodeArgs& a, const DecodePlan& p, const FusedArgs& f, cudaStream_t s);

// ---- parity hooks of the KVCache trait (hooks.cu): bit-exact in the
// reference's f32 order ----
// scores[t] = (sum_j (Rq)_j * c[code_tj]) * sigma_t for t < n   (compressor.rs:165-184)
// estimate_inner_products: stage 1 + QJL stage 2 (pq_scratch: m floats).
void launch_attend_keys_qjl(const float* q, const CodecDev& kc, const uint64_t* pages, const PageLayout& L,
                            int role_kw, int role_ks, int role_kq, int role_kr, int head, int64_t n,
                            float* rq_scratch, float* pq_scratch, float* scores, cudaStream_t s);
void launch_attend_keys(const float* q, const CodecDev& kc, const uint64_t* pages, const PageLayout& L, int role_kw,
                        int role_ks, int head, int64_t n, float* rq_scratch, float* scores, cudaStream_t s);
// out[i] = sum_t sum_j R[j][i] * (c[code_tj] * (sigma_t * w_t)), |w_t| >= 1e-10   (simple.rs:76-99, 142-155)
void launch_attend_values(const float* w, const CodecDev& vc, const uint64_t* pages, const PageLayout& L,
                          int role_vw, int role_vs, int head, int64_t n, float* out, cudaStream_t s);
// Combine partial slots -> (m, l, o) per row and/or the normalised output
// out[rows][dim] (un-rotated with R^T unless R == null). Row r's slots are
// part + (((r / G) * max_slots + c) * G + r % G) * (dim + 2), c < cnt[r / G]
// (cnt == null: max_slots for every row).
void launch_merge(const float* part, const int32_t* cnt, int32_t G, int32_t max_slots, int32_t n_rows, int32_t dim,
                  const float* R, void* out, int32_t out_dtype, float* m_out, float* l_out, float* o_out,
                  float oscale, cudaStream_t s);
// Merge n_parts partials laid out as separate arrays m, l [n_parts][n_rows]
// and o [n_parts][n_rows][dim] (e.g. gathered from the ranks of a split
// sequence), un-rotating by R unless it is null.
void launch_merge_parts(const float* m, const float* l, const float* o, int32_t n_parts, int32_t n_rows, int32_t dim,
                        const float* R, void* out, int32_t out_dtype, cudaStream_t s);
bool decode_fast_path(int dim, int kbits, int vbits, int G);

// Score precision of the fast path's f16 K table. The table rounds alpha c_k
// by at most lo_max (CodecOnDevice::lo_max), so a score z_t (log2 units) is
// off by about sigma_t * ||q'|| * lo_max. A tile whose largest such figure
// exceeds kLoEta, and which holds a score within kLoTheta of its head's
// running max, also multiplies the f16 residual table (the rounding errors,
// scaled by 2^11) by q' on the tensor cores and adds it, which leaves the
// scores f32-accurate. kLoEta sits between the figures of q ~ N(0, 1/d) and
// of q ~ N(0, 1) at scale 1 (the reference's Gemma call, RMS-normalised q),
// about 1.5e-3 and 1.7e-2 for 4-bit codes with x8 outlier channels; tokens
// kLoTheta below the max weigh under 2^-20 of it.
constexpr float kLoEta = 2e-3f;
constexpr float kLoTheta = 20.0f;
inline float decode_klo_thr(float lo_max) { return lo_max > 0.0f ? kLoEta / lo_max : 3.0e38f; }

// ---- fixed scratch of lc_decode_attn_noalloc (noalloc.cu) -----------------
// plan_decode's partition written into caller arrays seg [n + 1] (flat path
// only) and cnt [n * hkv], with no allocation; p.seg / p.cnt stay empty.
void plan_decode_into(const int64_t* lens, int n, int hkv, int hq, int dim, int kbits, int vbits, DecodePlan& p,
                      int64_t* seg, int32_t* cnt);
// Host staging bytes of one lc_decode_attn_noalloc call.
constexpr size_t kNoallocHostBytes = size_t(1) << 20;
// Held for the whole host side of an lc_decode_attn_noalloc call; guards
// the staging array and the per-device set-up below.
std::mutex& noalloc_mutex();
uint8_t* noalloc_host_staging();
// Device address of the LC_NOALLOC_SCRATCH_BYTES array on `device`, which
// must be current; the first call per device looks it up
// (cudaGetSymbolAddress). Call with noalloc_mutex() held.
uint8_t* noalloc_device_scratch(int device);

}  // namespace lc
