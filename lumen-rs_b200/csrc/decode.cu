// Decode attention over the TurboQuant-compressed cache: one query token per
// sequence, split-K over the context (flash-decode), all in the rotated basis.
//
// score_t = sigma_K[t] * <R q, c[code_K(t)]>            (compressor.rs:165-184)
// out     = R^T sum_t softmax(scale*score)_t sigma_V[t] c[code_V(t)]
//                                                      (simple.rs:76-99, 142-155)
// The reference un-rotates every token (O(N d^2)); here the weighted sum is
// accumulated in the rotated basis and un-rotated once per query head.
//
// Kernels
//  k_rotate_q       q' = (R q) * scale * log2(e) / alpha_K, f32 + f16 copies.
//  k_decode_pair    4-bit K/V, d = 128, GQA <= 4: the hot path. Persistent:
//                   one CTA of 16 warps per SM. The (sequence, kv head,
//                   32-token tile) space is cut into equal contiguous ranges,
//                   one per warp, so ragged batches stay balanced; a warp
//                   writes one softmax partial per (sequence, kv head)
//                   segment it touches. Each warp streams its tiles through a
//                   2-stage cp.async ring (16-byte copies of the packed words
//                   and sigmas straight from the pages). Codes become
//                   mma.sync fragments through a byte -> half2 centroid-pair
//                   table kept once per lane (one byte permute forms the
//                   address); S^T = K_dq Q^T and O^T = V_dq^T P^T run as
//                   m16n8k16 f16 MMAs with f32 accumulation, the MMA's N
//                   columns being (query head, f16 hi / lo part) so the query
//                   and P are f32-accurate. Precise tiles add the K table's
//                   f16 residuals (kLoEta). The fused variant rotates the
//                   queries on the tensor cores, merges a segment's partials
//                   in its last-arriving warp and un-rotates the output in
//                   the same launch.
//  k_decode_flat    4-bit K/V, d = 128, GQA 5..8: the same partition and
//                   tiles, with the query heads filling the N columns and the
//                   query hi / lo parts as two MMAs.
//  k_decode_mma32   3-bit K / 2-bit V, d = 256, GQA <= 4 (config 2): chunked
//                   items, one-lane bulk copies into per-warp stages, 6-bit
//                   K pair tables and a byte-indexed V table on m16n8k16.
//                   With one chunk per (sequence, kv head) it normalises and
//                   un-rotates the rows itself (no merge launch).
//  k_decode_generic any other bit width / head_dim, and QJL scores:
//                   CUDA-core, chunked.
//  k_merge          combines the partials, normalises, un-rotates (R^T).
// Roofline: HBM. Algorithmic bytes per (token, kv head) = 8*words_K +
// 8*words_V + 8 (136 B for 4-bit d=128), read once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cfloat>
#include <cstring>
#include <type_traits>

#include "devutil.cuh"
#include "group.h"
#include "kernels.h"

namespace lc {

namespace {

// Lazy rescale threshold (log2 units): the running max only moves when a new
// score exceeds it by more than this, which bounds p by 2^kTau.
constexpr float kTau = 8.0f;

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == LC_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == LC_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// v[i] = element idx[i] of an f32 / bf16 / f16 array, as f32, where ok[i]
// (else 0). The dtype branch is taken once, so all N loads are in flight
// before the first conversion waits on one.
template <int N>
__device__ __forceinline__ void load_n_any(const void* p, int dtype, const int64_t (&idx)[N], const bool (&ok)[N],
                                           float (&v)[N]) {
  if (dtype == LC_F32) {
    const float* q = static_cast<const float*>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = ok[i] ? q[idx[i]] : 0.f;
  } else {
    const unsigned short* q = static_cast<const unsigned short*>(p);
    unsigned short r[N];
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = ok[i] ? q[idx[i]] : (unsigned short)0;
#pragma unroll
    for (int i = 0; i < N; ++i)
      v[i] = dtype == LC_BF16 ? __uint_as_float((uint32_t)r[i] << 16) : __half2float(__ushort_as_half(r[i]));
  }
}

// Raw bits of element idx[i] (f32, or bf16 / f16 in the low half) where
// ok[i], else 0; raw_as_float converts one. The loads do not wait.
template <int N>
__device__ __forceinline__ void load_n_raw(const void* p, int dtype, const int64_t (&idx)[N], const bool (&ok)[N],
                                           uint32_t (&r)[N]) {
  if (dtype == LC_F32) {
    const uint32_t* q = static_cast<const uint32_t*>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = ok[i] ? q[idx[i]] : 0u;
  } else {
    const unsigned short* q = static_cast<const unsigned short*>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = ok[i] ? (uint32_t)q[idx[i]] : 0u;
  }
}
__device__ __forceinline__ float raw_as_float(uint32_t r, int dtype) {
  if (dtype == LC_F32) return __uint_as_float(r);
  if (dtype == LC_BF16) return __uint_as_float(r << 16);
  return __half2float(__ushort_as_half((unsigned short)r));
}

__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == LC_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dtype == LC_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

// ---------------------------------------------------------------------------
// q' = R q * qscale for kRotRows rows per block: block (x, y) takes rows
// kRotRows x .. + kRotRows - 1 and output dims 64 y .. 64 y + 63. Its 256
// threads are 4 slices of 64: slice js sums j in [js D/4, (js + 1) D/4) for
// its output dim, reading R^T[j][i] straight from global memory (coalesced;
// R^T is L2-resident) and the rows from shared memory (broadcast); the four
// partial sums are added through shared memory. So a thread makes one round
// trip for the rows and one or two for R^T, and many SMs are busy at decode
// batch sizes, each reading only its columns of R^T.
// ---------------------------------------------------------------------------
constexpr int kRotRows = 8, kRotDims = 64, kRotSplit = 4;
// acc[r] += sum_{u < C} M[(j0 + u) * D + i] * x[r][j0 + u] for NR rows of x in
// shared memory (row stride D): the C loads of M are all in flight before the
// first multiply, one L2 round trip per call.
template <int C, int NR>
__device__ __forceinline__ void mat_chunk(const float* __restrict__ M, int D, int i, int j0, const float* x,
                                          float (&acc)[NR]) {
  float w[C];
#pragma unroll
  for (int u = 0; u < C; ++u) w[u] = __ldg(M + (int64_t)(j0 + u) * D + i);
#pragma unroll
  for (int u = 0; u < C; u += 4) {
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const float4 v = *reinterpret_cast<const float4*>(x + r * D + j0 + u);
      acc[r] = fmaf(w[u + 3], v.w, fmaf(w[u + 2], v.z, fmaf(w[u + 1], v.y, fmaf(w[u], v.x, acc[r]))));
    }
  }
}

// acc[r] += sum_j M[j * D + i] * x[r][j] over all j < D (D a multiple of 32).
template <int NR>
__device__ __forceinline__ void mat_col(const float* __restrict__ M, int D, int i, const float* x, float (&acc)[NR]) {
  int j0 = 0;
  for (; j0 + 64 <= D; j0 += 64) mat_chunk<64, NR>(M, D, i, j0, x, acc);
  if (j0 < D) mat_chunk<32, NR>(M, D, i, j0, x, acc);
}

__global__ void __launch_bounds__(kRotDims * kRotSplit) k_rotate_q(const void* q, int dtype, int n_rows, int D,
                                                                const float* RT, int rotated, float qscale,
                                                                float* q_rot, __half* q_h) {
  extern __shared__ __align__(16) float sq[];  // [kRotRows][D], then [kRotSplit][kRotRows][kRotDims]
  pdl_launch_dependents();
  pdl_wait();  // q may come from the previous kernel of the stream
  float* red = sq + kRotRows * D;
  const int il = threadIdx.x % kRotDims, js = threadIdx.x / kRotDims;
  const int i = blockIdx.y * kRotDims + il;
  const int r0 = blockIdx.x * kRotRows;
  // the kRotRows rows, 8 loads per thread in flight at a time
  for (int k0 = threadIdx.x; k0 < kRotRows * D; k0 += 8 * blockDim.x) {
    int64_t idx[8];
    bool ok[8];
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = k0 + u * blockDim.x;
      idx[u] = (int64_t)r0 * D + k;
      ok[u] = k < kRotRows * D && r0 + k / D < n_rows;
    }
    load_n_any(q, dtype, idx, ok, v);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = k0 + u * blockDim.x;
      if (k < kRotRows * D) sq[k] = v[u];
    }
  }
  __syncthreads();
  if (!rotated) {
    float acc[kRotRows];
#pragma unroll
    for (int r = 0; r < kRotRows; ++r) acc[r] = 0.0f;
    const int jl = D / kRotSplit, jb = js * jl;
    int j0 = jb;
    for (; j0 + 64 <= jb + jl; j0 += 64) mat_chunk<64, kRotRows>(RT, D, i, j0, sq, acc);
    for (; j0 + 16 <= jb + jl; j0 += 16) mat_chunk<16, kRotRows>(RT, D, i, j0, sq, acc);
#pragma unroll
    for (int r = 0; r < kRotRows; ++r) red[(js * kRotRows + r) * kRotDims + il] = acc[r];
  }
  __syncthreads();
  // rows js, js + 4 of this block's 64 dims: the four slices' sums in order
#pragma unroll
  for (int rr = 0; rr < kRotRows / kRotSplit; ++rr) {
    const int r = js + kRotSplit * rr;
    const int row = r0 + r;
    float v = sq[r * D + i];
    if (!rotated) {
      v = red[(0 * kRotRows + r) * kRotDims + il];
#pragma unroll
      for (int t = 1; t < kRotSplit; ++t) v += red[(t * kRotRows + r) * kRotDims + il];
    }
    if (row < n_rows) {
      const float o = v * qscale;
      q_rot[(int64_t)row * D + i] = o;
      q_h[(int64_t)row * D + i] = __float2half_rn(o);
    }
  }
}

// QJL projection of the query rows for stage-2 scores: one CTA per row,
// thread i computes q_proj[row][i] = qscale * sum_j PT[j][i] q[row][j].
__global__ void k_project_q(const void* q, int dtype, int dim, int m, const float* PT, float qscale,
                            float* q_proj) {
  extern __shared__ float sq[];
  const int64_t row = blockIdx.x;
  for (int j = threadIdx.x; j < dim; j += blockDim.x) sq[j] = load_any(q, dtype, row * dim + j);
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < dim; ++j) acc = fmaf(PT[(int64_t)j * m + i], sq[j], acc);
    q_proj[row * m + i] = acc * qscale;
  }
}

// Per-call arrays of small calls travel in the launch parameters
// (__grid_constant__): no host-to-device copy between kernels.
struct InlineMeta {
  int64_t seqinfo[2 * kInlineSeqs];
  int64_t seg[kInlineSeqs + 1];
  int32_t cnt[kInlineCnt];
};

struct DecodeDev {
  const uint64_t* table;
  int64_t table_stride;
  const int64_t* seqinfo;  // [n_seqs][2] (tokens, table row)
  const int64_t* seg;      // flat: [n_seqs + 1] first tile of sequence b (all kv heads)
  int64_t per_warp, total_tiles;
  int32_t max_slots;
  int64_t off_kw, off_vw, off_ks, off_vs;
  int32_t row_kw, row_vw;
  int32_t n_seqs, hkv, hq, dim, kbits, vbits, pages_per_chunk, n_chunks, G;
  int32_t gen_tt, gen_stage;  // generic path: tokens per staged tile, bytes per stage
  const float* q_rot;
  const __half* q_h;
  const float* kcent;
  const float* vcent;
  float kalpha, valpha;
  float klo_thr;  // precise-score threshold numerator (DecodeArgs::klo_thr)
  float* part;
  // fused path (k_decode_pair<G, true>)
  const void* q_in;
  int32_t q_dtype, q_rotated;
  float qscale;
  const float* qR;       // K codec R (row-major): q' = R q
  const float* vRT;      // V codec R^T (row-major): out = R^T o (null: leave rotated)
  const float* out_R;    // k_decode_mma32 single-chunk finish: V codec R (row-major), null: leave rotated
  const int32_t* cnt;    // [n_seqs * hkv] partial slots
  int32_t* ctr;          // [n_seqs * hkv] arrival counters, zero between launches
  void* out;
  int32_t out_dtype;
  float oscale;
  // fused path, partials instead of the output: per row r (of `parts_rows`)
  // m at parts[r], l at parts[parts_rows + r], o (rotated, unnormalised) at
  // parts[2 parts_rows + r * D]; null: write `out`
  float* parts;
  int32_t parts_rows;
  // QJL stage-2 scores (generic path): see DecodeArgs
  const float* q_proj;
  int64_t off_kq, off_kr;
  int32_t row_kq, qjl_m;
  float qjl_c;
  // page-sparse decode: logical tile j of segment (b, kvh) is physical tile
  // tile_map[(b * hkv + kvh) * map_stride + j] of the sequence (null: dense)
  const int32_t* tile_map;
  int32_t map_stride;
  InlineMeta meta;  // seqinfo / seg / cnt when those pointers are null
  __device__ __forceinline__ const int64_t* si() const { return seqinfo ? seqinfo : meta.seqinfo; }
  __device__ __forceinline__ const int64_t* sg() const { return seg ? seg : meta.seg; }
  __device__ __forceinline__ const int32_t* ct() const { return cnt ? cnt : meta.cnt; }
};

// ---------------------------------------------------------------------------
// Fast path: 4-bit K and V, head_dim 128, up to 8 query heads per kv head.
// A tile is 32 tokens of one (sequence, kv head); a page holds 8 tiles.
// ---------------------------------------------------------------------------
constexpr int kFlatWarps = 16;
constexpr int kTileTok = 32;
constexpr int kStages = 2;
constexpr int kStK = 0;                    // [32 rows][64 B] K words
constexpr int kStV = 2048;                 // [32 rows][64 B] V words, 16-B chunks XOR-swizzled by (row & 2)
constexpr int kStKs = 4096, kStVs = 4224;  // [32] sigma_K, sigma_V
constexpr int kStageBytes = 4352;
constexpr int kWarpBytes = kStages * kStageBytes;
constexpr int kLutBytes = 65536;  // [byte][64 slots] u32: K table in slots 0..31, V table in 32..63
// The table sits at a 64 KiB-aligned shared address so one byte permute forms
// a lookup address; warps' stages fill the space before and after it.
constexpr int kFlatSmem = kLutBytes + (kFlatWarps + 1) * kWarpBytes;



// Table lookup. addr = [lane*4 | byte k of x | table base bits 16..31]: the
// lane's own copy of the entry (bank = lane, conflict-free across the warp).
__device__ __forceinline__ uint32_t lut_k(uint32_t x, uint32_t lanebase, uint32_t k) {
  uint32_t v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(__byte_perm(x, lanebase, 0x7604u | (k << 4))));
  return v;
}
__device__ __forceinline__ uint32_t lut_v(uint32_t x, uint32_t lanebase, uint32_t k) {
  uint32_t v;
  asm("ld.shared.u32 %0, [%1+128];" : "=r"(v) : "r"(__byte_perm(x, lanebase, 0x7604u | (k << 4))));
  return v;
}





// Walks (sequence, kv head, tile) in flat order; nt = tiles per kv head of b.
struct Walk {
  int b, kvh, tile, nt;
};

__device__ __forceinline__ int tiles_of(const DecodeDev& a, int b) {
  return (int)((a.si()[2 * b] + kTileTok - 1) / kTileTok);
}

__device__ __forceinline__ Walk locate(const DecodeDev& a, int64_t x) {
  int lo = 0, hi = a.n_seqs - 1;  // last b with seg[b] <= x (a sequence with tiles)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.sg()[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  Walk w;
  w.b = lo;
  w.nt = tiles_of(a, lo);
  const int64_t off = x - a.sg()[lo];
  w.kvh = (int)(off / w.nt);
  w.tile = (int)(off % w.nt);
  return w;
}

// locate() by a whole warp: lanes test 32 candidate sequences per load
// (first block starts at stride 32 when there are more than 32 sequences),
// so the search costs one or two global round trips instead of log2(n).
__device__ __forceinline__ Walk locate_warp(const DecodeDev& a, int64_t x, int lane) {
  const int n = a.n_seqs;
  int base = 0;
  if (n > 32) {
    for (int k0 = 0; k0 * 32 < n; k0 += 32) {
      const int b = (k0 + lane) * 32;
      const unsigned m = __ballot_sync(0xffffffffu, b < n && a.sg()[b] <= x);
      if (m) base = (k0 + 31 - __clz((int)m)) * 32;
      if (m != 0xffffffffu) break;
    }
  }
  const int bl = base + lane;
  const int64_t sv = bl <= n ? a.sg()[bl] : INT64_MAX;
  const unsigned m = __ballot_sync(0xffffffffu, bl < n && sv <= x);
  const int k = 31 - __clz((int)m);  // seg[base] <= x, so m != 0
  const int64_t s0 = __shfl_sync(0xffffffffu, sv, k);
  const int64_t s1n = __shfl_sync(0xffffffffu, sv, (k + 1) & 31);
  const int64_t s1 = k < 31 ? s1n : a.sg()[base + 32];
  Walk w;
  w.b = base + k;
  w.nt = (int)((s1 - s0) / a.hkv);
  const int64_t off = x - s0;
  w.kvh = (int)(off / w.nt);
  w.tile = (int)(off % w.nt);
  return w;
}

__device__ __forceinline__ void step(const DecodeDev& a, Walk& w) {
  if (++w.tile < w.nt) return;
  w.tile = 0;
  if (++w.kvh < a.hkv) return;
  w.kvh = 0;
  do {
    ++w.b;
  } while (w.b < a.n_seqs && (w.nt = tiles_of(a, w.b)) == 0);
}

// Producer: issues the 16-byte copies of one tile into a stage; caches the
// page address (it changes every 8 tiles).
struct Producer {
  Walk w;
  const uint8_t* page;
  int page_b, page_kvh, page_idx;

  __device__ __forceinline__ void issue(const DecodeDev& a, uint32_t st, int lane) {
    const int pidx = w.tile >> 3;
    if (pidx != page_idx || w.b != page_b) {
      const uint64_t* trow = a.table + a.si()[2 * w.b + 1] * a.table_stride;
      page = reinterpret_cast<const uint8_t*>(__ldg(trow + pidx));
      page_idx = pidx;
      page_b = w.b;
    }
    const int64_t hr = (int64_t)w.kvh * kPageTokens + (w.tile & 7) * kTileTok;
    const uint8_t* k = page + a.off_kw + hr * 64;
    const uint8_t* v = page + a.off_vw + hr * 64;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = lane + 32 * q;  // 16-byte chunk: row c >> 2, part c & 3
      cp_async16(st + kStK + c * 16, k + c * 16);
      const int r = c >> 2;
      cp_async16(st + kStV + r * 64 + (((c & 3) ^ (r & 2)) << 4), v + c * 16);
    }
    if (lane < 8) cp_async16(st + kStKs + lane * 16, page + a.off_ks + hr * 4 + lane * 16);
    else if (lane < 16) cp_async16(st + kStVs + (lane - 8) * 16, page + a.off_vs + hr * 4 + (lane - 8) * 16);
  }
};

// Producer with the next page address loaded ahead: a switch to the
// following page of the same sequence, or to page 0 of the next kv head,
// finds its address already in a register instead of waiting on a global
// load.
struct PrefetchProducer {
  Walk w;
  const uint8_t* page;
  int page_b, page_idx;
  uint64_t next;  // address of page next_idx of sequence next_b
  int next_b, next_idx;
  // Page-sparse: lane j holds the physical tile (win_ph) and its page
  // address (win_pg) of logical tile win_t0 + j of segment win_seg, read
  // 32 tiles at a time; cur_ph is the current tile's.
  int win_seg, win_t0, win_ph, cur_ph;
  uint64_t win_pg;

  // Page address of the current tile (and the next page's, ahead). Called
  // on its own at kernel start so the first table read is in flight while
  // the prologue does other work. Page-sparse: the window of 32 tile-map
  // entries and their page addresses, refilled when the walk leaves it.
  template <bool SPARSE = false>
  __device__ __forceinline__ void lookup(const DecodeDev& a, int lane) {
    if constexpr (SPARSE) {
      const int seg = w.b * a.hkv + w.kvh;
      if (seg != win_seg || (unsigned)(w.tile - win_t0) >= 32u) {
        win_seg = seg;
        win_t0 = w.tile;
        const int t = w.tile + lane;
        win_ph = 0;
        win_pg = 0;
        if (t < w.nt) {
          win_ph = a.tile_map[(int64_t)seg * a.map_stride + t];
          win_pg = __ldg(a.table + a.si()[2 * w.b + 1] * a.table_stride + (win_ph >> 3));
        }
      }
      const int j = w.tile - win_t0;
      cur_ph = __shfl_sync(0xffffffffu, win_ph, j);
      page = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, win_pg, j));
    } else {
      const int pidx = w.tile >> 3;
      if (pidx != page_idx || w.b != page_b) {
        const uint64_t* trow = a.table + a.si()[2 * w.b + 1] * a.table_stride;
        page = reinterpret_cast<const uint8_t*>((w.b == next_b && pidx == next_idx) ? next : __ldg(trow + pidx));
        const int npages = (w.nt + 7) >> 3;
        next_b = w.b;
        next_idx = pidx + 1 < npages ? pidx + 1 : 0;
        next = __ldg(trow + next_idx);
        page_idx = pidx;
        page_b = w.b;
      }
    }
  }

  template <bool SPARSE = false>
  __device__ __forceinline__ void issue(const DecodeDev& a, uint32_t st, int lane) {
    lookup<SPARSE>(a, lane);
    const int64_t hr = (int64_t)w.kvh * kPageTokens + ((SPARSE ? cur_ph : w.tile) & 7) * kTileTok;
    // chunk c = lane + 32 q: row c >> 2 = lane / 4 + 8 q, part c & 3 = lane & 3;
    // the V swizzle (part ^ (row & 2)) depends on the lane only
    const uint8_t* k = page + a.off_kw + hr * 64 + lane * 16;
    const uint8_t* v = page + a.off_vw + hr * 64 + lane * 16;
    const uint32_t vdst = st + kStV + (lane >> 2) * 64 + (((lane & 3) ^ ((lane >> 2) & 2)) << 4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      cp_async16(st + kStK + lane * 16 + q * 512, k + q * 512);
      cp_async16(vdst + q * 512, v + q * 512);
    }
    if (lane < 16) {
      const bool kside = lane < 8;
      cp_async16(st + (kside ? kStKs : kStVs) + (lane & 7) * 16,
                 page + (kside ? a.off_ks : a.off_vs) + hr * 4 + (lane & 7) * 16);
    }
  }
};

// 16 tokens (rows r0..r0+15): S^T = K_dq (Q_hi + Q_lo)^T into sc, two MMAs
// per K fragment (the f16 value and residual of every query element).
__device__ __forceinline__ void qk16_hl(const uint8_t* st, int r0, int g, int t, uint32_t lanebase,
                                        const uint32_t (&qb)[8][2], const uint32_t (&ql)[8][2], float* sc) {
  const uint4 k0 = *reinterpret_cast<const uint4*>(st + kStK + (r0 + g) * 64 + 16 * t);
  const uint4 k1 = *reinterpret_cast<const uint4*>(st + kStK + (r0 + g + 8) * 64 + 16 * t);
  const uint32_t kx[4] = {k0.x, k0.y, k0.z, k0.w};
  const uint32_t ky[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t a0 = lut_k(kx[j], lanebase, 2 * h);
      const uint32_t a2 = lut_k(kx[j], lanebase, 2 * h + 1);
      const uint32_t a1 = lut_k(ky[j], lanebase, 2 * h);
      const uint32_t a3 = lut_k(ky[j], lanebase, 2 * h + 1);
      mma16816(sc, a0, a1, a2, a3, qb[2 * j + h][0], qb[2 * j + h][1]);
      mma16816(sc, a0, a1, a2, a3, ql[2 * j + h][0], ql[2 * j + h][1]);
    }
  }
}

// ---- K table residuals (f32-accurate scores) ----
// The f16 table holds alpha c_k rounded; its residuals r_k = alpha c_k -
// f16(alpha c_k) (exact in f32), scaled by 2^11 to stay normal f16 numbers,
// sit in a 16-entry table with one copy per lane: entry (code n, lane l) at
// byte n * 128 + l * 4, r_n in both f16 halves, so lookups are
// conflict-free. A tile that needs the precision multiplies the residuals of
// its codes by the same Q^T fragments and adds 2^-11 times the product.
constexpr float kLoScale = 2048.f, kLoUnscale = 1.f / 2048.f;
constexpr int kLoTabWords = 16 * 32;

// Entry idx (< 512) of the residual table: code idx / 32, lane idx % 32.
__device__ __forceinline__ void build_klo(uint32_t* tab, const DecodeDev& a, int idx) {
  const float x = a.kcent[idx >> 5] * a.kalpha;  // the f32 product the f16 table rounds
  const float r = (x - __half2float(__float2half_rn(x))) * kLoScale;
  tab[idx] = h2_as_u32(__floats2half2_rn(r, r));
}

// Residual pair of byte k of x (the two codes of one A-fragment register):
// low nibble -> low half, high nibble -> high half. lane4 = lane * 4.
__device__ __forceinline__ uint32_t klo_pair(const uint32_t* tab, uint32_t x, int k, uint32_t lane4) {
  auto off = [&](int p) {  // byte offset of the entry of the nibble at bit p
    const uint32_t v = p >= 7 ? (x >> (p - 7)) : (x << (7 - p));
    return (v & 0x780u) | lane4;
  };
  const char* base = reinterpret_cast<const char*>(tab);
  const uint32_t e0 = *reinterpret_cast<const uint32_t*>(base + off(8 * k));
  const uint32_t e1 = *reinterpret_cast<const uint32_t*>(base + off(8 * k + 4));
  return __byte_perm(e0, e1, 0x7610);
}

// 16 tokens (rows r0..r0+15): c += Kres Q^T with the K fragments of qk16_2.
// Not unrolled, one code word per row at a time: it runs inside the main
// loop with everything else live, and must not raise the loop's register
// demand (its tiles are the minority, and only in peaked regimes).
__device__ __forceinline__ void qk16_lo(const uint8_t* st, int r0, int g, int t, const uint32_t* tab,
                                        uint32_t lane4, const uint32_t (&qb)[8][2], float* c) {
  const uint32_t* kr0 = reinterpret_cast<const uint32_t*>(st + kStK + (r0 + g) * 64 + 16 * t);
  const uint32_t* kr1 = kr0 + 128;  // row + 8
#pragma unroll 1
  for (int j = 0; j < 4; ++j) {
    const uint32_t kx = kr0[j], ky = kr1[j];
    uint32_t b00, b01, b10, b11;  // qb[2j], qb[2j + 1], picked without dynamic indexing
    b00 = qb[0][0]; b01 = qb[0][1]; b10 = qb[1][0]; b11 = qb[1][1];
    if (j == 1) { b00 = qb[2][0]; b01 = qb[2][1]; b10 = qb[3][0]; b11 = qb[3][1]; }
    if (j == 2) { b00 = qb[4][0]; b01 = qb[4][1]; b10 = qb[5][0]; b11 = qb[5][1]; }
    if (j == 3) { b00 = qb[6][0]; b01 = qb[6][1]; b10 = qb[7][0]; b11 = qb[7][1]; }
    mma16816(c, klo_pair(tab, kx, 0, lane4), klo_pair(tab, ky, 0, lane4), klo_pair(tab, kx, 1, lane4),
             klo_pair(tab, ky, 1, lane4), b00, b01);
    mma16816(c, klo_pair(tab, kx, 2, lane4), klo_pair(tab, ky, 2, lane4), klo_pair(tab, kx, 3, lane4),
             klo_pair(tab, ky, 3, lane4), b10, b11);
  }
}

// 16 tokens (rows r0..r0+15): O^T += V_dq^T P^T for the hi and lo parts of P.
__device__ __forceinline__ void pv16(const uint8_t* st, int r0, int g, int t, uint32_t lanebase, uint32_t pb0,
                                     uint32_t pb1, uint32_t pc0, uint32_t pc1, float (&oacc)[8][4]) {
  // rows (tokens) t, t+8 (pair 0) and t+4, t+12 (pair 1); word g = dims 16g..16g+15
  auto vrow = [&](int r) -> uint2 {
    return *reinterpret_cast<const uint2*>(st + kStV + r * 64 + ((((g >> 1) ^ (r & 2))) << 4) + (g & 1) * 8);
  };
  const uint2 v0 = vrow(r0 + t), v1 = vrow(r0 + t + 8), v2 = vrow(r0 + t + 4), v3 = vrow(r0 + t + 12);
  uint32_t ev[2][2], od[2][2];
  const uint32_t A0[2] = {v0.x, v0.y}, B0[2] = {v1.x, v1.y};
  const uint32_t A1[2] = {v2.x, v2.y}, B1[2] = {v3.x, v3.y};
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    ev[0][hh] = (A0[hh] & 0x0F0F0F0Fu) | ((B0[hh] & 0x0F0F0F0Fu) << 4);
    od[0][hh] = ((A0[hh] >> 4) & 0x0F0F0F0Fu) | (B0[hh] & 0xF0F0F0F0u);
    ev[1][hh] = (A1[hh] & 0x0F0F0F0Fu) | ((B1[hh] & 0x0F0F0F0Fu) << 4);
    od[1][hh] = ((A1[hh] >> 4) & 0x0F0F0F0Fu) | (B1[hh] & 0xF0F0F0F0u);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int hh = i >> 2;
    const uint32_t k = (uint32_t)(i & 3);
    const uint32_t a0 = lut_v(ev[0][hh], lanebase, k);
    const uint32_t a1 = lut_v(od[0][hh], lanebase, k);
    const uint32_t a2 = lut_v(ev[1][hh], lanebase, k);
    const uint32_t a3 = lut_v(od[1][hh], lanebase, k);
    mma16816(oacc[i], a0, a1, a2, a3, pb0, pb1);
    mma16816(oacc[i], a0, a1, a2, a3, pc0, pc1);
  }
}

// p' = p * sigma_V for (token u, token u+8) of heads 2t and 2t+1 as f16 hi +
// lo pairs, moved into the P^T B fragments of head g: tokens (t, t+8) from
// lane (t, g/2) and (t+4, t+12) from lane (t+4, g/2).
__device__ __forceinline__ void p_frag(float p00, float p10, float p01, float p11, int g, int t, int G,
                                       uint32_t& pb0, uint32_t& pb1, uint32_t& pc0, uint32_t& pc1) {
  const __half2 h0h = __floats2half2_rn(p00, p10);  // head 2t
  const __half2 h1h = __floats2half2_rn(p01, p11);  // head 2t+1
  const float2 f0 = __half22float2(h0h), f1 = __half22float2(h1h);
  const uint32_t h0 = h2_as_u32(h0h), h1 = h2_as_u32(h1h);
  const uint32_t l0 = h2_as_u32(__floats2half2_rn(p00 - f0.x, p10 - f0.y));
  const uint32_t l1 = h2_as_u32(__floats2half2_rn(p01 - f1.x, p11 - f1.y));
  const int src0 = t * 4 + (g >> 1), src1 = (t + 4) * 4 + (g >> 1);
  const bool odd = g & 1;
  const uint32_t x00 = __shfl_sync(0xffffffffu, h0, src0), x01 = __shfl_sync(0xffffffffu, h1, src0);
  const uint32_t x10 = __shfl_sync(0xffffffffu, h0, src1), x11 = __shfl_sync(0xffffffffu, h1, src1);
  const uint32_t y00 = __shfl_sync(0xffffffffu, l0, src0), y01 = __shfl_sync(0xffffffffu, l1, src0);
  const uint32_t y10 = __shfl_sync(0xffffffffu, l0, src1), y11 = __shfl_sync(0xffffffffu, l1, src1);
  pb0 = odd ? x01 : x00;
  pb1 = odd ? x11 : x10;
  pc0 = odd ? y01 : y00;
  pc1 = odd ? y11 : y10;
  if (g >= G) pb0 = pb1 = pc0 = pc1 = 0u;
}

// ---------------------------------------------------------------------------
// Pair layout for G <= 4. The MMA's 8 columns carry (head, part) pairs,
// n = 2 * head + part: part 0 is the f16 value and part 1 its f16 residual,
// for q in S^T = K_dq Q^T and for p' in O^T = V_dq^T P^T. Adding the two
// columns back gives f32-accurate q and p' at no extra MMA, and lane (g, t)
// then owns head t: scores of tokens g, g + 8 (+16, +24) and output
// columns 2t, 2t + 1 (dims 16g .. 16g + 15).
// ---------------------------------------------------------------------------

// 16 tokens (rows r0..r0+15) into two independent accumulators (even and
// odd k steps), so consecutive MMAs do not wait on each other.
__device__ __forceinline__ void qk16_2(const uint8_t* st, int r0, int g, int t, uint32_t lanebase,
                                       const uint32_t (&qb)[8][2], float* c0, float* c1) {
  const uint4 k0 = *reinterpret_cast<const uint4*>(st + kStK + (r0 + g) * 64 + 16 * t);
  const uint4 k1 = *reinterpret_cast<const uint4*>(st + kStK + (r0 + g + 8) * 64 + 16 * t);
  const uint32_t kx[4] = {k0.x, k0.y, k0.z, k0.w};
  const uint32_t ky[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t a0 = lut_k(kx[j], lanebase, 2 * h);
      const uint32_t a2 = lut_k(kx[j], lanebase, 2 * h + 1);
      const uint32_t a1 = lut_k(ky[j], lanebase, 2 * h);
      const uint32_t a3 = lut_k(ky[j], lanebase, 2 * h + 1);
      mma16816(h ? c1 : c0, a0, a1, a2, a3, qb[2 * j + h][0], qb[2 * j + h][1]);
    }
  }
}

// 16 tokens (rows r0..r0+15): O^T += V_dq^T P^T, one MMA per dim tile.
// vl = the lane's constant part of its V row offsets (see pair_vlane).
template <int R0>
__device__ __forceinline__ void pv16_1(const uint8_t* st, uint32_t vl, uint32_t lanebase, uint32_t pb0, uint32_t pb1,
                                       float (&oacc)[8][4]) {
  const uint8_t* vb = st + kStV + vl + R0 * 64;
  const uint2 v0 = *reinterpret_cast<const uint2*>(vb);         // token t
  const uint2 v1 = *reinterpret_cast<const uint2*>(vb + 512);   // token t + 8
  const uint2 v2 = *reinterpret_cast<const uint2*>(vb + 256);   // token t + 4
  const uint2 v3 = *reinterpret_cast<const uint2*>(vb + 768);   // token t + 12
  uint32_t ev[2][2], od[2][2];
  const uint32_t A0[2] = {v0.x, v0.y}, B0[2] = {v1.x, v1.y};
  const uint32_t A1[2] = {v2.x, v2.y}, B1[2] = {v3.x, v3.y};
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    ev[0][hh] = (A0[hh] & 0x0F0F0F0Fu) | ((B0[hh] & 0x0F0F0F0Fu) << 4);
    od[0][hh] = ((A0[hh] >> 4) & 0x0F0F0F0Fu) | (B0[hh] & 0xF0F0F0F0u);
    ev[1][hh] = (A1[hh] & 0x0F0F0F0Fu) | ((B1[hh] & 0x0F0F0F0Fu) << 4);
    od[1][hh] = ((A1[hh] >> 4) & 0x0F0F0F0Fu) | (B1[hh] & 0xF0F0F0F0u);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int hh = i >> 2;
    const uint32_t k = (uint32_t)(i & 3);
    const uint32_t a0 = lut_v(ev[0][hh], lanebase, k);
    const uint32_t a1 = lut_v(od[0][hh], lanebase, k);
    const uint32_t a2 = lut_v(ev[1][hh], lanebase, k);
    const uint32_t a3 = lut_v(od[1][hh], lanebase, k);
    mma16816(oacc[i], a0, a1, a2, a3, pb0, pb1);
  }
}

// Lane (g, t)'s constant V offset within a stage: rows r0 + t + {0, 4, 8, 12}
// all have bit 1 equal to t's, so the XOR swizzle of the 16-byte chunk
// (g / 2) ^ (row & 2) is fixed per lane; 8-byte half g & 1.
__device__ __forceinline__ uint32_t pair_vlane(int g, int t) {
  return (uint32_t)(t * 64 + (((g >> 1) ^ (t & 2)) << 4) + (g & 1) * 8);
}

// Fused path: rows of query / output kept in shared memory per CTA. A CTA
// touches at most kFusedSegs (sequence, kv head) segments (plan_decode
// checks), i.e. kFusedSegs * G <= 32 rows.
constexpr int kFusedSegs = 8;
constexpr int kFusedRows = 32;
constexpr int kFusedSmem = kFlatSmem + kFusedRows * 128 * 4;

// Centroid-pair lookup table: lane l < 16 holds K centroid l, lane 16 + l V
// centroid l (scaled); entry (e, slot) = (c[e & 15], c[e >> 4]), slots 0..31
// K and 32..63 V.
__device__ __forceinline__ float lut_centroid(const DecodeDev& a, int lane) {
  return lane < 16 ? a.kcent[lane] * a.kalpha : a.vcent[lane - 16] * a.valpha;
}
// cl = lut_centroid(a, lane), read at kernel start (ahead of the tile traffic)
__device__ __forceinline__ void build_lut(uint8_t* lut, float cl) {
#pragma unroll
  for (int it = 0; it < 256 * 64 / (kFlatWarps * 32); ++it) {
    const int idx = threadIdx.x + it * kFlatWarps * 32;
    const int e = idx >> 6, vside = (idx & 63) >= 32 ? 16 : 0;
    const float lo = __shfl_sync(0xffffffffu, cl, vside + (e & 15));
    const float hi = __shfl_sync(0xffffffffu, cl, vside + (e >> 4));
    reinterpret_cast<uint32_t*>(lut)[idx] = h2_as_u32(__floats2half2_rn(lo, hi));
  }
}

// ---- rotations of the fused path on the tensor cores ----
// D[i][r] = sum_j M[i][j] x[r][j] for a 128 x 128 f32 matrix M and up to 32
// rows x: A = M (16-row blocks mi), B = x^T (8-row blocks ni), K = j. Both
// operands are split into f16 hi + lo parts and D = Mh xh + Mh xl + Ml xh is
// accumulated in f32 by m16n8k16 products: the dropped Ml xl term is 2^-22
// of the product. M is scaled by 2^8 before the split (its entries are at
// most 1 in magnitude) so its low parts stay normal f16 numbers; the
// caller scales D by 2^-8 (exact).
// K is permuted inside every 16-wide step so lane t owns physical columns
// 16 ks + 4t .. 4t + 3: logical k (2t, 2t+1) -> 4t + (0, 1) and (2t+8, 2t+9)
// -> 4t + (2, 3). Both operands then load as one float4 per lane.
// Rows x live in shared memory, row r at x + 128 r, column j stored at
// j ^ 16 (r & 1): the float4 reads of rows g = 2p, 2p + 1 (one quarter-warp)
// fall in distinct banks.
constexpr float kRotScale = 256.f, kRotUnscale = 1.f / 256.f;

__device__ __forceinline__ int rot_swz(int r, int j) { return r * 128 + (j ^ ((r & 1) << 4)); }

__device__ __forceinline__ void split_h2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 f = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(x - f.x, y - f.y));
}

// M staged in shared memory: row i at i * 512 bytes from the base, its
// 16-byte chunk c stored at c ^ 4 (i & 1), so the fragment reads of rows
// g = 2p, 2p + 1 (one quarter-warp) fall in distinct banks. Both live in
// the warps' second pipeline stages, eight rows per warp: the prologue's R
// (the second tile is issued after the rotation) and the epilogue's V R^T
// (free once the main loop is over).
__device__ __forceinline__ int m_chunk(int i, int c) { return (c ^ ((i & 1) << 2)) << 4; }
__device__ __forceinline__ uint8_t* m_row(uint8_t* smem, int n_before, uint32_t lut_off, int i) {
  const int wi = i >> 3;
  uint8_t* st = wi < n_before ? smem + wi * kWarpBytes : smem + lut_off + kLutBytes + (wi - n_before) * kWarpBytes;
  return st + kStageBytes + (i & 7) * 512;
}

// d = D[16 mi + (g, g + 8)][8 ni + (2t, 2t + 1)] * 2^8 for one (mi, ni) block:
// d[0] (g, 2t), d[1] (g, 2t + 1), d[2] (g + 8, 2t), d[3] (g + 8, 2t + 1).
// mrow(i) is row i of M in the staged layout.
template <class MRow>
__device__ __forceinline__ void rot_block(MRow mrow, int mi, const float* xs, int ni, int g, int t, float (&d)[4]) {
  float e[4] = {0.f, 0.f, 0.f, 0.f};
  d[0] = d[1] = d[2] = d[3] = 0.f;
  const int r = 8 * ni + g, i0 = 16 * mi + g;
  const uint8_t* m0 = mrow(i0);
  const uint8_t* m1 = mrow(i0 + 8);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const float4 xv = *reinterpret_cast<const float4*>(xs + rot_swz(r, 16 * ks + 4 * t));
    const float4 f0 = *reinterpret_cast<const float4*>(m0 + m_chunk(i0, 4 * ks + t));
    const float4 f1 = *reinterpret_cast<const float4*>(m1 + m_chunk(i0 + 8, 4 * ks + t));
    uint32_t bh0, bl0, bh1, bl1;
    split_h2(xv.x, xv.y, bh0, bl0);
    split_h2(xv.z, xv.w, bh1, bl1);
    uint32_t ah[4], al[4];
    split_h2(f0.x * kRotScale, f0.y * kRotScale, ah[0], al[0]);
    split_h2(f1.x * kRotScale, f1.y * kRotScale, ah[1], al[1]);
    split_h2(f0.z * kRotScale, f0.w * kRotScale, ah[2], al[2]);
    split_h2(f1.z * kRotScale, f1.w * kRotScale, ah[3], al[3]);
    mma16816(d, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
    mma16816(e, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
    mma16816(e, al[0], al[1], al[2], al[3], bh0, bh1);
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) d[c] += e[c];
}

// P^T B fragments of both 16-token halves through shared memory, in the
// stage's K area (read completely by then). Lane (g, t) holds p' of head t
// for tokens (g, g + 8) of half 0 (pa, pb) and of half 1 (pc, pd) and writes
// the f16 value and residual pairs; lane (g, t) then reads column g = (head
// g / 2, part g & 1) at token pairs t (b0) and t + 4 (b1). Word of (half,
// part, head, pair): half * 64 + part * 32 + head * 8 + (pair ^ 4 part), so
// both the writes and the reads of a warp hit 32 distinct banks.
__device__ __forceinline__ void p_exchange(const uint8_t* st, float pa, float pb_, float pc, float pd, int g, int t,
                                           int G, uint32_t (&pb)[2][2]) {
  uint32_t* ps = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(st) + kStK);
  const __half2 h0 = __floats2half2_rn(pa, pb_), h1 = __floats2half2_rn(pc, pd);
  const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
  const uint32_t l0 = h2_as_u32(__floats2half2_rn(pa - f0.x, pb_ - f0.y));
  const uint32_t l1 = h2_as_u32(__floats2half2_rn(pc - f1.x, pd - f1.y));
  __syncwarp();
  ps[t * 8 + g] = h2_as_u32(h0);
  ps[32 + t * 8 + (g ^ 4)] = l0;
  ps[64 + t * 8 + g] = h2_as_u32(h1);
  ps[96 + t * 8 + (g ^ 4)] = l1;
  __syncwarp();
  const int head = g >> 1, part = g & 1;
  const int base = part * 32 + head * 8, sw = part << 2;
  const bool live = head < G;
  pb[0][0] = live ? ps[base + (t ^ sw)] : 0u;
  pb[0][1] = live ? ps[base + ((t + 4) ^ sw)] : 0u;
  pb[1][0] = live ? ps[64 + base + (t ^ sw)] : 0u;
  pb[1][1] = live ? ps[64 + base + ((t + 4) ^ sw)] : 0u;
}

template <int G, bool FUSED, bool SPARSE = false>
__global__ void __launch_bounds__(kFlatWarps * 32, 1) k_decode_pair(const __grid_constant__ DecodeDev a) {
  static_assert(G >= 1 && G <= 4, "pair layout holds 4 heads");
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = 128;
  constexpr int PS = D + 2;
  const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t lut_off = (65536u - (s0 & 0xFFFFu)) & 0xFFFFu;
  const int n_before = (int)(lut_off / kWarpBytes);
  uint8_t* lut = smem + lut_off;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lanebase = ((s0 + lut_off) & 0xFFFF0000u) | ((uint32_t)lane << 2);
  const uint32_t vl = pair_vlane(g, t);
  if constexpr (FUSED) pdl_launch_dependents();
  // tile indices fit in 32 bits (plan_decode: total_tiles < 2^31)
  const int w = blockIdx.x * kFlatWarps + warp;
  const int pw = (int)a.per_warp;
  const int begin = w * pw;
  const int end = min(begin + pw, (int)a.total_tiles);
  uint8_t* stages = warp < n_before ? smem + warp * kWarpBytes
                                    : smem + lut_off + kLutBytes + (warp - n_before) * kWarpBytes;
  const uint32_t st0 = (uint32_t)__cvta_generic_to_shared(stages);

  PrefetchProducer pr;
  pr.page = nullptr;
  pr.page_b = -1;
  pr.page_idx = -1;
  pr.next = 0;
  pr.next_b = -1;
  pr.next_idx = -1;
  pr.win_seg = -1;
  pr.win_t0 = 0;
  float* qs = reinterpret_cast<float*>(smem + kFlatSmem);  // [kFusedRows][D]
  __shared__ int merged[kFusedSegs];
  __shared__ uint32_t s_klo[kLoTabWords];  // K table residuals (precise tiles)
  // first (sequence, kv head) segment of this CTA and its query-row count,
  // kept in shared memory (read once per segment; no register in the loop)
  __shared__ int cta_seg[2];
  const bool rot_q = FUSED && !a.q_rotated;
  const float cl = lut_centroid(a, lane);
  // fused: the K rotation R into the warps' second pipeline stages (free
  // until the second tile is issued after the prologue), before any tile
  // traffic; an L2 hit shared by all CTAs
  if constexpr (FUSED) {
    if (rot_q) {
#pragma unroll
      for (int it = 0; it < D * D / 4 / (kFlatWarps * 32); ++it) {
        const int k = threadIdx.x + it * kFlatWarps * 32;  // row k / 32, chunk k % 32
        const int i = k >> 5;
        cp_async16((uint32_t)__cvta_generic_to_shared(m_row(smem, n_before, lut_off, i)) + m_chunk(i, k & 31),
                   a.qR + 4 * k);
      }
    }
    cp_commit();
  }
  if (begin < end) {
    pr.w = locate_warp(a, begin, lane);
    // the block table is written by host copies only; a page-sparse tile
    // map by the selection kernel, so the fused kernel reads it after the wait
    if constexpr (!(FUSED && SPARSE)) pr.template lookup<SPARSE>(a, lane);
  }
  Walk cw = pr.w;
  // fused: this CTA's segments and their query-row count (host-written
  // arrays only, so before the wait)
  int sid0 = 0, nrows = 0;
  if constexpr (FUSED) {
    const int cb = blockIdx.x * kFlatWarps * pw;
    const int ce = min(cb + kFlatWarps * pw, (int)a.total_tiles);
    if (cb < ce) {
      const Walk f = locate_warp(a, cb, lane), e = locate_warp(a, ce - 1, lane);
      sid0 = f.b * a.hkv + f.kvh;
      nrows = (e.b * a.hkv + e.kvh - sid0 + 1) * G;
    }
    // the centroid-pair and residual tables from constants, while the reads
    // above are in flight (read only after the barrier that follows the
    // rotation)
    build_lut(lut, cl);
    build_klo(s_klo, a, threadIdx.x);
  }
  // fused: everything above reads constants (codec tables, launch
  // parameters, the block table); the queries, the cache pages, the arrival
  // counters and the partials come after the previous kernel has completed
  if constexpr (FUSED) pdl_wait();

  // fused: the query rows' raw loads go out first, then the first tile; the
  // conversion waits on the rows after both are in flight
  constexpr int QIT = kFusedRows * D / (kFlatWarps * 32);
  uint32_t qraw[QIT];
  if constexpr (FUSED) {
    int64_t qidx[QIT];
    bool qok[QIT];
#pragma unroll
    for (int it = 0; it < QIT; ++it) {
      const int k = threadIdx.x + it * kFlatWarps * 32;
      const int r = k >> 7, j = k & 127;
      const int sid = sid0 + r / G;
      qidx[it] = ((int64_t)(sid / a.hkv) * a.hq + (int64_t)(sid % a.hkv) * G + r % G) * D + j;
      qok[it] = r < nrows;
    }
    load_n_raw(a.q_in, a.q_dtype, qidx, qok, qraw);
  }

  // The first tiles. Fused: one now, the second after the prologue; a tile
  // takes longer to compute than the next one takes to arrive.
  constexpr int kFirstTiles = FUSED ? 1 : 2;
#pragma unroll
  for (int k = 0; k < kFirstTiles; ++k) {
    if (begin + k < end) {
      pr.template issue<SPARSE>(a, st0 + k * kStageBytes, lane);
      step(a, pr.w);
    }
    cp_commit();
  }

  // ---- fused: q' = R (q * qscale) into qs on the tensor cores; warp w
  // computes output dims 16 (w & 7) .. + 15 of row blocks (w >> 3) and
  // (w >> 3) + 2 ----
  if constexpr (FUSED) {
    const int nb = (nrows + 7) >> 3, mi = warp & 7, n0 = warp >> 3;
    if (threadIdx.x < kFusedSegs) merged[threadIdx.x] = 0;
    if (threadIdx.x == 0) {
      cta_seg[0] = sid0;
      cta_seg[1] = nrows;
    }
#pragma unroll
    for (int it = 0; it < QIT; ++it) {
      const int k = threadIdx.x + it * kFlatWarps * 32;
      const int r = k >> 7, j = k & 127;
      if (r < nb * 8) qs[rot_q ? rot_swz(r, j) : k] = raw_as_float(qraw[it], a.q_dtype) * a.qscale;
    }
    if (rot_q) {
      cp_wait_one();  // R has landed; the first tile may still be in flight
      __syncthreads();
      auto rrow = [&](int i) { return static_cast<const uint8_t*>(m_row(smem, n_before, lut_off, i)); };
      float d[2][4];
      if (n0 < nb) rot_block(rrow, mi, qs, n0, g, t, d[0]);
      if (n0 + 2 < nb) rot_block(rrow, mi, qs, n0 + 2, g, t, d[1]);
      __syncthreads();  // every warp has read R and q
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int ni = n0 + 2 * u;
        if (ni < nb) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int r = 8 * ni + 2 * t + (c & 1), i = 16 * mi + g + 8 * (c >> 1);
            if (r < nrows) qs[r * D + i] = d[u][c] * kRotUnscale;
          }
        }
      }
    }
  } else {
    build_lut(lut, cl);
    build_klo(s_klo, a, threadIdx.x);
  }
  __syncthreads();  // the table, and the fused q' rows
  if (!FUSED && begin >= end) return;  // no block-wide barrier after this point
  if constexpr (FUSED) {  // the second tile (over R, read by every warp by now)
    if (begin + 1 < end) {
      pr.template issue<SPARSE>(a, st0 + kStageBytes, lane);
      step(a, pr.w);
    }
    cp_commit();
  }

  int x = begin;
  while (x < end) {
    // ---- a new (sequence, kv head) segment ----
    const int b = cw.b, kvh = cw.kvh;
    const int n_valid = (int)a.si()[2 * b];
    const int seg_first = (int)a.sg()[b] + kvh * cw.nt;
    const int seg_end = min(end, seg_first + cw.nt);
    // B fragments of Q: column g = (head g/2, part g&1), dims 32t + 4s + {0,1} / {2,3}
    uint32_t qb[8][2];
    float ss = 0.f;
    {
      const int head = g >> 1;
      const bool lo = g & 1;
      const int hsel = head < G ? head : 0;
      const float* qrow = FUSED ? qs + ((b * a.hkv + kvh - cta_seg[0]) * G + hsel) * D + 32 * t
                                : a.q_rot + ((int64_t)b * a.hq + (int64_t)kvh * G + hsel) * D + 32 * t;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const float4 v = *reinterpret_cast<const float4*>(qrow + 4 * s);
        const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
        uint32_t r0 = h2_as_u32(h01), r1 = h2_as_u32(h23);
        if (lo) {
          const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
          r0 = h2_as_u32(__floats2half2_rn(v.x - f01.x, v.y - f01.y));
          r1 = h2_as_u32(__floats2half2_rn(v.z - f23.x, v.w - f23.y));
        }
        qb[s][0] = head < G ? r0 : 0u;
        qb[s][1] = head < G ? r1 : 0u;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
    }
    // precise tiles need sigma_K > lthr: ||q'|| of the group's largest row
    // (lanes t = 0..3 of head g / 2 hold its 128 dims)
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss = fmaxf(ss, __shfl_xor_sync(0xffffffffu, ss, 8));
    ss = fmaxf(ss, __shfl_xor_sync(0xffffffffu, ss, 16));
    const float lthr = a.klo_thr * rsqrtf(ss);
    float m = -INFINITY, l = 0.f;
    float oacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;

    auto tile = [&](auto masked) {
      constexpr bool MASKED = decltype(masked)::value;
      const int stage = (x - begin) & 1;
      const int tok = (x - seg_first) * kTileTok;
      const uint8_t* st = stages + stage * kStageBytes;
      float sa0[4] = {0.f, 0.f, 0.f, 0.f}, sa1[4] = {0.f, 0.f, 0.f, 0.f};
      float sb0[4] = {0.f, 0.f, 0.f, 0.f}, sb1[4] = {0.f, 0.f, 0.f, 0.f};
      qk16_2(st, 0, g, t, lanebase, qb, sa0, sa1);
      qk16_2(st, 16, g, t, lanebase, qb, sb0, sb1);
      const float* ks = reinterpret_cast<const float*>(st + kStKs);
      const float* vs = reinterpret_cast<const float*>(st + kStVs);
      // this lane: head t, tokens u0 = g, u1 = g + 8, u2 = 16 + g, u3 = 24 + g
      const bool ok0 = !MASKED || tok + g < n_valid, ok1 = !MASKED || tok + g + 8 < n_valid;
      const bool ok2 = !MASKED || tok + g + 16 < n_valid, ok3 = !MASKED || tok + g + 24 < n_valid;
      const float k0 = ks[g], k1 = ks[g + 8], k2 = ks[g + 16], k3 = ks[g + 24];
      float y0 = (sa0[0] + sa1[0]) + (sa0[1] + sa1[1]);
      float y1 = (sa0[2] + sa1[2]) + (sa0[3] + sa1[3]);
      float y2 = (sb0[0] + sb1[0]) + (sb0[1] + sb1[1]);
      float y3 = (sb0[2] + sb1[2]) + (sb0[3] + sb1[3]);
      // f32-accurate scores where the f16 table's rounding could move the
      // softmax: large sigma_K x ||q'||, and a score near the running max
      if (__any_sync(0xffffffffu, t < G && fmaxf(fmaxf(k0, k1), fmaxf(k2, k3)) > lthr)) {
        const float zm = fmaxf(fmaxf(ok0 ? y0 * k0 : -INFINITY, ok1 ? y1 * k1 : -INFINITY),
                               fmaxf(ok2 ? y2 * k2 : -INFINITY, ok3 ? y3 * k3 : -INFINITY));
        if (__any_sync(0xffffffffu, t < G && fmaxf(fmaxf(k0, k1), fmaxf(k2, k3)) > lthr && zm > m - kLoTheta)) {
          float la[4] = {0.f, 0.f, 0.f, 0.f};
          qk16_lo(st, 0, g, t, s_klo, lanebase & 0xFFu, qb, la);
          y0 = fmaf(la[0] + la[1], kLoUnscale, y0);
          y1 = fmaf(la[2] + la[3], kLoUnscale, y1);
          la[0] = la[1] = la[2] = la[3] = 0.f;
          qk16_lo(st, 16, g, t, s_klo, lanebase & 0xFFu, qb, la);
          y2 = fmaf(la[0] + la[1], kLoUnscale, y2);
          y3 = fmaf(la[2] + la[3], kLoUnscale, y3);
        }
      }
      const float z0 = y0 * k0, z1 = y1 * k1, z2 = y2 * k2, z3 = y3 * k3;
      const float s0_ = ok0 ? z0 : -INFINITY, s1_ = ok1 ? z1 : -INFINITY;
      const float s2_ = ok2 ? z2 : -INFINITY, s3_ = ok3 ? z3 : -INFINITY;
      // lazy rescale: the running max m moves only when some score exceeds it
      // by more than kTau, which a warp vote detects without the cross-lane
      // max; the reduction and rescale run only then
      float mx = fmaxf(fmaxf(s0_, s1_), fmaxf(s2_, s3_));
      if (__any_sync(0xffffffffu, mx > m + kTau)) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (mx > m + kTau) {
          const float al = ex2(m - mx);
          l *= al;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            oacc[i][0] *= al;
            oacc[i][1] *= al;
            oacc[i][2] *= al;
            oacc[i][3] *= al;
          }
          m = mx;
        }
      }
      const float p0 = ex2(s0_ - m), p1 = ex2(s1_ - m), p2 = ex2(s2_ - m), p3 = ex2(s3_ - m);
      l += (p0 + p1) + (p2 + p3);
      const float w0 = ok0 ? vs[g] : 0.f, w1 = ok1 ? vs[g + 8] : 0.f;
      const float w2 = ok2 ? vs[g + 16] : 0.f, w3 = ok3 ? vs[g + 24] : 0.f;
      // P^T fragments through shared memory (this stage's K bytes are spent)
      uint32_t pb[2][2];
      p_exchange(st, p0 * w0, p1 * w1, p2 * w2, p3 * w3, g, t, G, pb);
      pv16_1<0>(st, vl, lanebase, pb[0][0], pb[0][1], oacc);
      pv16_1<16>(st, vl, lanebase, pb[1][0], pb[1][1], oacc);
    };

    for (; x < seg_end; ++x) {
      cp_wait_one();
      __syncwarp();
      if ((x - seg_first) * kTileTok + kTileTok <= n_valid) tile(std::integral_constant<bool, false>());
      else tile(std::integral_constant<bool, true>());
      __syncwarp();
      if (x + kStages < end) {
        pr.template issue<SPARSE>(a, st0 + ((x - begin) & 1) * kStageBytes, lane);
        step(a, pr.w);
      }
      cp_commit();
    }
    // the next segment in flat order (kv heads of b, then sequences with tiles)
    if (++cw.kvh == a.hkv) {
      cw.kvh = 0;
      do {
        ++cw.b;
      } while (cw.b < a.n_seqs && (cw.nt = tiles_of(a, cw.b)) == 0);
    }
    // ---- flush the segment's partial: head t, dims 16g + 2i (+1) ----
    float L = l;
    L += __shfl_xor_sync(0xffffffffu, L, 4);
    L += __shfl_xor_sync(0xffffffffu, L, 8);
    L += __shfl_xor_sync(0xffffffffu, L, 16);
    if (t < G) {
      const int64_t slot = ((int64_t)b * a.hkv + kvh) * a.max_slots + (w - seg_first / pw);
      float* row = a.part + (slot * G + t) * PS;
      if (g == 0) {
        row[0] = m;
        row[1] = L;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float2*>(row + 2 + 16 * g + 2 * i) =
            make_float2(oacc[i][0] + oacc[i][1], oacc[i][2] + oacc[i][3]);
    }
    if constexpr (FUSED) {
      // Count this warp's slot of the segment; the warp that completes it
      // marks the segment for this CTA's epilogue to merge.
      __threadfence();
      __syncwarp();
      const int sid = b * a.hkv + kvh;
      int old = 0;
      if (lane == 0) old = atomicAdd(a.ctr + sid, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == a.ct()[sid] - 1 && lane == 0) {
        a.ctr[sid] = 0;  // zero again for the next launch
        merged[sid - cta_seg[0]] = 1;
      }
    }
  }
  cp_wait_all();
  if constexpr (FUSED) {
    // ---- epilogue: the whole CTA merges the segments its warps completed
    // (their q' rows in qs are no longer read) and writes them un-rotated ----
    __syncthreads();
    __shared__ int mrow[kFusedRows];  // rows of the merged segments, compacted
    __shared__ int n_mrows;
    if (threadIdx.x == 0) {
      int k = 0;
      for (int r = 0; r < cta_seg[1]; ++r)
        if (merged[r / G]) mrow[k++] = r;
      n_mrows = k;
    }
    __syncthreads();
    const int nm = n_mrows, sid0 = cta_seg[0];
    if (nm == 0) return;  // uniform over the CTA
    __threadfence();      // the other warps' partials, read below from L2
    // V's R^T rows into the second pipeline stages, free now
    if (a.vRT) {
#pragma unroll
      for (int it = 0; it < D * D / 4 / (kFlatWarps * 32); ++it) {
        const int k = threadIdx.x + it * kFlatWarps * 32;  // row k / 32, chunk k % 32
        const int i = k >> 5;
        cp_async16((uint32_t)__cvta_generic_to_shared(m_row(smem, n_before, lut_off, i)) + m_chunk(i, k & 31), a.vRT + 4 * k);
      }
    }
    cp_commit();
    // merge, warp per compacted row k: lane c holds (m, l) of slot c of a
    // group of 32; the o rows of the group's first kMergeAhead slots are
    // loaded with them (lane: dims 2 lane, 2 lane + 1, 64 + 2 lane, + 1), so
    // a row of up to kMergeAhead slots costs one round trip to L2. Groups
    // fold into (M, L, acc) with an online rescale.
    constexpr int kMergeAhead = 16;
    float* om = qs;  // [nm][D] over the q' rows (no longer read), rot_swz layout
    for (int k = warp; k < nm; k += kFlatWarps) {
      const int r = mrow[k];
      const int sid = sid0 + r / G;
      const int n = a.ct()[sid];
      const float* prow = a.part + ((int64_t)sid * a.max_slots * G + r % G) * PS;
      const int64_t cs = (int64_t)G * PS;
      float M = -INFINITY, L = 0.f;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c0 = 0; c0 < n; c0 += 32) {
        const int c = c0 + lane;
        const float mc = c < n ? __ldcg(prow + c * cs) : -INFINITY;
        const float lc = c < n ? __ldcg(prow + c * cs + 1) : 0.f;
        float2 ov[kMergeAhead][2];
#pragma unroll
        for (int j = 0; j < kMergeAhead; ++j) {
          const bool live = c0 + j < n;
          const float* po = prow + (c0 + j) * cs + 2 + 2 * lane;
          ov[j][0] = live ? __ldcg(reinterpret_cast<const float2*>(po)) : make_float2(0.f, 0.f);
          ov[j][1] = live ? __ldcg(reinterpret_cast<const float2*>(po + 64)) : make_float2(0.f, 0.f);
        }
        float Mg = mc;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Mg = fmaxf(Mg, __shfl_xor_sync(0xffffffffu, Mg, off));
        const float Mn = fmaxf(M, Mg);
        const float keep = M == -INFINITY ? 0.f : ex2(M - Mn);  // rescale of what was folded so far
        const float wc = mc == -INFINITY ? 0.f : ex2(mc - Mn);
        float Lg = wc * lc;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) Lg += __shfl_xor_sync(0xffffffffu, Lg, off);
        L = L * keep + Lg;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] *= keep;
#pragma unroll
        for (int j = 0; j < kMergeAhead; ++j) {
          const float wj = __shfl_sync(0xffffffffu, wc, j);
          acc[0] = fmaf(wj, ov[j][0].x, acc[0]);
          acc[1] = fmaf(wj, ov[j][0].y, acc[1]);
          acc[2] = fmaf(wj, ov[j][1].x, acc[2]);
          acc[3] = fmaf(wj, ov[j][1].y, acc[3]);
        }
        for (int j = kMergeAhead; j < 32 && c0 + j < n; ++j) {  // slots past the loaded ones
          const float wj = __shfl_sync(0xffffffffu, wc, j);
          const float* po = prow + (c0 + j) * cs + 2 + 2 * lane;
          const float2 o0 = __ldcg(reinterpret_cast<const float2*>(po));
          const float2 o1 = __ldcg(reinterpret_cast<const float2*>(po + 64));
          acc[0] = fmaf(wj, o0.x, acc[0]);
          acc[1] = fmaf(wj, o0.y, acc[1]);
          acc[2] = fmaf(wj, o1.x, acc[2]);
          acc[3] = fmaf(wj, o1.y, acc[3]);
        }
        M = Mn;
      }
      if (a.parts) {  // the row's softmax partials (a split context's shard)
        const int sid = sid0 + r / G;
        const int64_t orow = (int64_t)(sid / a.hkv) * a.hq + (int64_t)(sid % a.hkv) * G + r % G;
        float* po = a.parts + 2 * (int64_t)a.parts_rows + orow * D;
        *reinterpret_cast<float2*>(po + 2 * lane) = make_float2(acc[0] * a.oscale, acc[1] * a.oscale);
        *reinterpret_cast<float2*>(po + 64 + 2 * lane) = make_float2(acc[2] * a.oscale, acc[3] * a.oscale);
        if (lane == 0) {
          a.parts[orow] = M;
          a.parts[a.parts_rows + orow] = L;
        }
        continue;
      }
      const float li = L > 0.f ? a.oscale / L : 0.f;
      *reinterpret_cast<float2*>(om + rot_swz(k, 2 * lane)) = make_float2(acc[0] * li, acc[1] * li);
      *reinterpret_cast<float2*>(om + rot_swz(k, 64 + 2 * lane)) = make_float2(acc[2] * li, acc[3] * li);
    }
    cp_wait_all();
    if (a.parts) return;  // uniform over the CTA; no barrier follows
    __syncthreads();
    // out = R^T o on the tensor cores: warp w computes output dims 16 (w & 7)
    // .. + 15 of compacted row blocks (w >> 3) and (w >> 3) + 2
    auto out_at = [&](int k, int i, float v) {
      const int row = mrow[k];
      const int sid = sid0 + row / G;
      const int64_t orow = (int64_t)(sid / a.hkv) * a.hq + (int64_t)(sid % a.hkv) * G + row % G;
      store_any(a.out, a.out_dtype, orow * D + i, v);
    };
    if (a.vRT) {
      const int nb = (nm + 7) >> 3, mi = warp & 7, n0 = warp >> 3;
      if (n0 < nb) {
        auto vrow = [&](int i) { return static_cast<const uint8_t*>(m_row(smem, n_before, lut_off, i)); };
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ni = n0 + 2 * u;
          if (ni < nb) {
            float d[4];
            rot_block(vrow, mi, om, ni, g, t, d);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int k = 8 * ni + 2 * t + (c & 1), i = 16 * mi + g + 8 * (c >> 1);
              if (k < nm) out_at(k, i, d[c] * kRotUnscale);
            }
          }
        }
      }
    } else {
      for (int u = threadIdx.x; u < nm * D; u += kFlatWarps * 32) out_at(u >> 7, u & (D - 1), om[rot_swz(u >> 7, u & (D - 1))]);
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kFlatWarps * 32, 1) k_decode_flat(const __grid_constant__ DecodeDev a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int D = 128;
  constexpr int PS = D + 2;
  const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t lut_off = (65536u - (s0 & 0xFFFFu)) & 0xFFFFu;
  const int n_before = (int)(lut_off / kWarpBytes);
  uint8_t* lut = smem + lut_off;
  __shared__ uint32_t s_klo[kLoTabWords];  // K table residuals (precise tiles)
  build_klo(s_klo, a, threadIdx.x);

  for (int idx = threadIdx.x; idx < 256 * 64; idx += blockDim.x) {
    const int e = idx >> 6, slot = idx & 63;
    const float* cent = slot < 32 ? a.kcent : a.vcent;
    const float al = slot < 32 ? a.kalpha : a.valpha;
    reinterpret_cast<uint32_t*>(lut)[idx] = h2_as_u32(__floats2half2_rn(cent[e & 15] * al, cent[e >> 4] * al));
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  const uint32_t lanebase = ((s0 + lut_off) & 0xFFFF0000u) | ((uint32_t)lane << 2);
  const int64_t w = (int64_t)blockIdx.x * kFlatWarps + warp;
  const int64_t begin = w * a.per_warp;
  const int64_t end = min(begin + a.per_warp, a.total_tiles);
  if (begin >= end) return;
  uint8_t* stages = warp < n_before ? smem + warp * kWarpBytes
                                    : smem + lut_off + kLutBytes + (warp - n_before) * kWarpBytes;
  const uint32_t st0 = (uint32_t)__cvta_generic_to_shared(stages);

  Producer pr;
  pr.w = locate(a, begin);
  pr.page = nullptr;
  pr.page_b = -1;
  pr.page_idx = -1;
  Walk cw = pr.w;
#pragma unroll
  for (int s = 0; s < kStages; ++s) {
    if (begin + s < end) {
      pr.issue(a, st0 + s * kStageBytes, lane);
      step(a, pr.w);
    }
    cp_commit();
  }

  int64_t x = begin;
  while (x < end) {
    // ---- a new (sequence, kv head) segment ----
    const int b = cw.b, kvh = cw.kvh;
    const int n_valid = (int)a.si()[2 * b];
    const int64_t seg_first = a.sg()[b] + (int64_t)kvh * cw.nt;
    const int64_t seg_end = min(end, seg_first + cw.nt);
    const int64_t slot_base = ((int64_t)b * a.hkv + kvh) * a.max_slots + (w - seg_first / a.per_warp);
    // B fragments of Q (column g = head g): f16 values and residuals of the
    // f32 rotated query, dims 32t + 4j + {0,1} / {2,3}
    uint32_t qb[8][2], ql[8][2];
    float ss = 0.f;
    {
      const float* qrow = a.q_rot + ((int64_t)b * a.hq + (int64_t)kvh * G + (g < G ? g : 0)) * D + 32 * t;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(qrow + 4 * j);
        uint32_t h0, l0, h1, l1;
        split_h2(v.x, v.y, h0, l0);
        split_h2(v.z, v.w, h1, l1);
        qb[j][0] = g < G ? h0 : 0u;
        qb[j][1] = g < G ? h1 : 0u;
        ql[j][0] = g < G ? l0 : 0u;
        ql[j][1] = g < G ? l1 : 0u;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) ss = fmaxf(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float lthr = a.klo_thr * rsqrtf(ss);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float oacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;

    // One 32-token tile; MASKED only for a sequence's last, partial tile.
    auto tile = [&](auto masked) {
      constexpr bool MASKED = decltype(masked)::value;
      const int stage = (int)((x - begin) & 1);
      const int tok = cw.tile * kTileTok;
      const uint8_t* st = stages + stage * kStageBytes;
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      qk16_hl(st, 0, g, t, lanebase, qb, ql, sa);
      qk16_hl(st, 16, g, t, lanebase, qb, ql, sb);
      const float* ks = reinterpret_cast<const float*>(st + kStKs);
      const float* vs = reinterpret_cast<const float*>(st + kStVs);
      // tokens of this thread: u0 = g, u1 = g+8, u2 = 16+g, u3 = 24+g
      const bool ok0 = !MASKED || tok + g < n_valid, ok1 = !MASKED || tok + g + 8 < n_valid;
      const bool ok2 = !MASKED || tok + g + 16 < n_valid, ok3 = !MASKED || tok + g + 24 < n_valid;
      const float k0 = ks[g], k1 = ks[g + 8], k2 = ks[g + 16], k3 = ks[g + 24];
      // f32-accurate scores where the f16 table's rounding could move the
      // softmax (see k_decode_pair)
      const bool live0 = 2 * t < G, live1 = 2 * t + 1 < G;
      if (__any_sync(0xffffffffu, live0 && fmaxf(fmaxf(k0, k1), fmaxf(k2, k3)) > lthr)) {
        const float za = fmaxf(fmaxf(ok0 ? sa[0] * k0 : -INFINITY, ok1 ? sa[2] * k1 : -INFINITY),
                               fmaxf(ok2 ? sb[0] * k2 : -INFINITY, ok3 ? sb[2] * k3 : -INFINITY));
        const float zb = fmaxf(fmaxf(ok0 ? sa[1] * k0 : -INFINITY, ok1 ? sa[3] * k1 : -INFINITY),
                               fmaxf(ok2 ? sb[1] * k2 : -INFINITY, ok3 ? sb[3] * k3 : -INFINITY));
        const bool near = (live0 && za > m0 - kLoTheta) || (live1 && zb > m1 - kLoTheta);
        if (__any_sync(0xffffffffu, near && fmaxf(fmaxf(k0, k1), fmaxf(k2, k3)) > lthr)) {
          float la[4] = {0.f, 0.f, 0.f, 0.f}, lb[4] = {0.f, 0.f, 0.f, 0.f};
          qk16_lo(st, 0, g, t, s_klo, lane4, qb, la);
          qk16_lo(st, 16, g, t, s_klo, lane4, qb, lb);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            sa[e] = fmaf(la[e], kLoUnscale, sa[e]);
            sb[e] = fmaf(lb[e], kLoUnscale, sb[e]);
          }
        }
      }
      // s[u][e]: token u, head 2t+e (log2 domain)
      const float s00 = ok0 ? sa[0] * k0 : -INFINITY, s01 = ok0 ? sa[1] * k0 : -INFINITY;
      const float s10 = ok1 ? sa[2] * k1 : -INFINITY, s11 = ok1 ? sa[3] * k1 : -INFINITY;
      const float s20 = ok2 ? sb[0] * k2 : -INFINITY, s21 = ok2 ? sb[1] * k2 : -INFINITY;
      const float s30 = ok3 ? sb[2] * k3 : -INFINITY, s31 = ok3 ? sb[3] * k3 : -INFINITY;
      float mx0 = fmaxf(fmaxf(s00, s10), fmaxf(s20, s30));
      float mx1 = fmaxf(fmaxf(s01, s11), fmaxf(s21, s31));
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      if (mx0 > m0 + kTau) {
        const float al = ex2(m0 - mx0);
        l0 *= al;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          oacc[i][0] *= al;
          oacc[i][2] *= al;
        }
        m0 = mx0;
      }
      if (mx1 > m1 + kTau) {
        const float al = ex2(m1 - mx1);
        l1 *= al;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          oacc[i][1] *= al;
          oacc[i][3] *= al;
        }
        m1 = mx1;
      }
      const float p00 = ex2(s00 - m0), p10 = ex2(s10 - m0), p20 = ex2(s20 - m0), p30 = ex2(s30 - m0);
      const float p01 = ex2(s01 - m1), p11 = ex2(s11 - m1), p21 = ex2(s21 - m1), p31 = ex2(s31 - m1);
      l0 += (p00 + p10) + (p20 + p30);
      l1 += (p01 + p11) + (p21 + p31);
      const float w0 = ok0 ? vs[g] : 0.f, w1 = ok1 ? vs[g + 8] : 0.f;
      const float w2 = ok2 ? vs[g + 16] : 0.f, w3 = ok3 ? vs[g + 24] : 0.f;
      uint32_t pb0, pb1, pc0, pc1;
      p_frag(p00 * w0, p10 * w1, p01 * w0, p11 * w1, g, t, G, pb0, pb1, pc0, pc1);
      pv16(st, 0, g, t, lanebase, pb0, pb1, pc0, pc1, oacc);
      p_frag(p20 * w2, p30 * w3, p21 * w2, p31 * w3, g, t, G, pb0, pb1, pc0, pc1);
      pv16(st, 16, g, t, lanebase, pb0, pb1, pc0, pc1, oacc);
    };

    for (; x < seg_end; ++x) {
      cp_wait_one();
      __syncwarp();
      if (cw.tile * kTileTok + kTileTok <= n_valid) tile(std::integral_constant<bool, false>());
      else tile(std::integral_constant<bool, true>());
      // ---- refill this stage with tile x + kStages ----
      __syncwarp();
      if (x + kStages < end) {
        pr.issue(a, st0 + (int)((x - begin) & 1) * kStageBytes, lane);
        step(a, pr.w);
      }
      cp_commit();
      step(a, cw);
    }
    // ---- flush the segment's partial ----
    float L0 = l0, L1 = l1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      L0 += __shfl_xor_sync(0xffffffffu, L0, o);
      L1 += __shfl_xor_sync(0xffffffffu, L1, o);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hd = 2 * t + e;
      if (hd < G) {
        float* row = a.part + (slot_base * G + hd) * PS;
        if (g == 0) {
          row[0] = e ? m1 : m0;
          row[1] = e ? L1 : L0;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          row[2 + 16 * g + 2 * i] = oacc[i][e];
          row[2 + 16 * g + 2 * i + 1] = oacc[i][2 + e];
        }
      }
    }
  }
  cp_wait_all();
}

// ---------------------------------------------------------------------------
// Generic path: any bit width, head_dim = 32*KPL, GS query heads per CTA,
// chunks of pages_per_chunk pages; partial slot = chunk. The warps of a block
// take the chunk's tiles of gen_tt tokens (16 or 32) in turn, staged into shared
// memory by a per-warp cp.async double buffer: K words, V words, sigma_K,
// sigma_V of the tile are contiguous in the page, so a tile is three or four
// flat 16-byte copies. Lane l owns dims l + 32k: its word index and bit
// shift per dim are fixed for the kernel. Softmax uses the lazy rescale of
// the fast path (the running max moves only when a score exceeds it by more
// than kTau).
// ---------------------------------------------------------------------------
template <int KPL, int GS, bool QJL>
__global__ void __launch_bounds__(128) k_decode_generic(const __grid_constant__ DecodeDev a) {
  extern __shared__ __align__(16) float gsm[];
  constexpr int D = 32 * KPL;
  constexpr int PS = D + 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  float* kc = gsm;           // [256]
  float* vc = gsm + 256;     // [256]
  float* wpart = gsm + 512;  // [nw][GS][PS]
  uint8_t* stage0 = reinterpret_cast<uint8_t*>(gsm + 512 + nw * GS * PS) + (size_t)warp * 2 * a.gen_stage;
  const uint32_t st_s = (uint32_t)__cvta_generic_to_shared(stage0);
  for (int i = threadIdx.x; i < (1 << a.kbits); i += blockDim.x) kc[i] = a.kcent[i];
  for (int i = threadIdx.x; i < (1 << a.vbits); i += blockDim.x) vc[i] = a.vcent[i];
  __syncthreads();
  const int groups = a.G / GS;
  const int kcpw = 64 / a.kbits, vcpw = 64 / a.vbits;
  const uint64_t kmask = (1ull << a.kbits) - 1, vmask = (1ull << a.vbits) - 1;
  const int64_t total = (int64_t)a.n_seqs * a.hkv * groups * a.n_chunks;
  const int TT = a.gen_tt;
  const int kw_row = a.row_kw / 8, vw_row = a.row_vw / 8;  // u64 words per token row
  // stage: [TT][kw_row] K words | [TT][vw_row] V words | [TT] sigma_K | [TT] sigma_V
  const int kbytes = TT * a.row_kw, vbytes = TT * a.row_vw;
  // per dim: K word | K shift << 8 | V word << 16 | V shift << 24 (each < 256)
  uint32_t idx[KPL];
#pragma unroll
  for (int k = 0; k < KPL; ++k) {
    const int d = lane + 32 * k;
    idx[k] = (uint32_t)(d / kcpw) | ((uint32_t)((d % kcpw) * a.kbits) << 8) | ((uint32_t)(d / vcpw) << 16) |
             ((uint32_t)((d % vcpw) * a.vbits) << 24);
  }

  for (int64_t item = blockIdx.x; item < total; item += gridDim.x) {
    const int chunk = (int)(item % a.n_chunks);
    int64_t rest = item / a.n_chunks;
    const int grp = (int)(rest % groups);
    rest /= groups;
    const int kvh = (int)(rest % a.hkv);
    const int s = (int)(rest / a.hkv);
    const int64_t n_valid = a.si()[2 * s];
    const uint64_t* trow = a.table + a.si()[2 * s + 1] * a.table_stride;
    const int qh0 = kvh * a.G + grp * GS;

    float q[GS][KPL], o[GS][KPL], m[GS], l[GS];
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int k = 0; k < KPL; ++k) {
        q[g][k] = a.q_rot[((int64_t)s * a.hq + qh0 + g) * D + lane + 32 * k];
        o[g][k] = 0.f;
      }
    }
    // QJL: projection rows i = lane + 32 r of (Phi q) * qscale per head
    constexpr bool qjl = QJL;
    constexpr int MQ = QJL ? kMaxQjlDecode / 32 : 1;
    float pq[GS][MQ];
#pragma unroll
    for (int g = 0; g < GS; ++g)
#pragma unroll
      for (int r = 0; r < MQ; ++r) {
        const int i = lane + 32 * r;
        pq[g][r] = (qjl && i < a.qjl_m) ? a.q_proj[((int64_t)s * a.hq + qh0 + g) * a.qjl_m + i] : 0.f;
      }
    {
      // The chunk's 32- (or 16-) token tiles, strided over the warps: tile t
      // is rows (t % tpp) TT .. of page chunk * pages_per_chunk + t / tpp,
      // whose address lane t / tpp holds. Whole tiles are copied: rows past
      // n_valid exist in the page and are not used.
      const int64_t p0 = (int64_t)chunk * a.pages_per_chunk;
      const int64_t ctok = n_valid - p0 * kPageTokens;
      const int64_t cmax = (int64_t)a.pages_per_chunk * kPageTokens;
      const int chunk_tok = (int)(ctok <= 0 ? 0 : (ctok < cmax ? ctok : cmax));
      const int tpp = kPageTokens / TT;
      const int ctiles = (chunk_tok + TT - 1) / TT;
      const uint64_t my_page =
          lane < a.pages_per_chunk && (p0 + lane) * kPageTokens < n_valid ? trow[p0 + lane] : 0ull;
      auto page_of = [&](int t) {
        return reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, my_page, t / tpp));
      };
      auto issue = [&](int t, int stg) {
        const uint8_t* page = page_of(t);
        const uint8_t* kg = page + a.off_kw + (int64_t)kvh * kPageTokens * a.row_kw;
        const uint8_t* vg = page + a.off_vw + (int64_t)kvh * kPageTokens * a.row_vw;
        const uint8_t* ksg = page + a.off_ks + (int64_t)kvh * kPageTokens * 4;
        const uint8_t* vsg = page + a.off_vs + (int64_t)kvh * kPageTokens * 4;
        const uint32_t dst = st_s + stg * a.gen_stage;
        const int r0 = (t % tpp) * TT;
        for (int c = lane; c * 16 < kbytes; c += 32) cp_async16(dst + c * 16, kg + (int64_t)r0 * a.row_kw + c * 16);
        for (int c = lane; c * 16 < vbytes; c += 32)
          cp_async16(dst + kbytes + c * 16, vg + (int64_t)r0 * a.row_vw + c * 16);
        for (int c = lane; c * 16 < TT * 8; c += 32) {  // sigma_K then sigma_V, TT * 4 bytes each
          const bool kside = c * 16 < TT * 4;
          const int off = kside ? c * 16 : c * 16 - TT * 4;
          cp_async16(dst + kbytes + vbytes + c * 16, (kside ? ksg : vsg) + (int64_t)r0 * 4 + off);
        }
        cp_commit();
      };
      if (warp < ctiles) issue(warp, 0);
      for (int t = warp, it = 0; t < ctiles; t += nw, ++it) {
        if (t + nw < ctiles) {
          issue(t + nw, (it + 1) & 1);
          cp_wait_one();
        } else {
          cp_wait_all();
        }
        __syncwarp();
        const uint8_t* st = stage0 + (it & 1) * a.gen_stage;
        const uint64_t* kw = reinterpret_cast<const uint64_t*>(st);
        const uint64_t* vw = reinterpret_cast<const uint64_t*>(st + kbytes);
        const float* ks = reinterpret_cast<const float*>(st + kbytes + vbytes);
        const float* vs = ks + TT;
        const int tl = t % tpp;
        const uint8_t* page = page_of(t);
        const uint64_t* kq = qjl ? reinterpret_cast<const uint64_t*>(page + a.off_kq + (int64_t)kvh * kPageTokens * a.row_kq)
                                 : nullptr;
        const float* kr = qjl ? reinterpret_cast<const float*>(page + a.off_kr) + (int64_t)kvh * kPageTokens : nullptr;
        const int cnt = min(TT, chunk_tok - t * TT);
        for (int tt = 0; tt < cnt; ++tt) {
          float part[GS];
#pragma unroll
          for (int g = 0; g < GS; ++g) part[g] = 0.f;
          float vv[KPL];
#pragma unroll
          for (int k = 0; k < KPL; ++k) {
            const uint64_t wk = kw[tt * kw_row + (idx[k] & 0xFF)];
            const float c = kc[(wk >> ((idx[k] >> 8) & 0xFF)) & kmask];
#pragma unroll
            for (int g = 0; g < GS; ++g) part[g] = fmaf(q[g][k], c, part[g]);
            const uint64_t wv = vw[tt * vw_row + ((idx[k] >> 16) & 0xFF)];
            vv[k] = vc[(wv >> (idx[k] >> 24)) & vmask];
          }
          // QJL stage 2 (compressor.rs:148-155, qjl.rs:86-119):
          // ||r|| sqrt(pi/2)/sqrt(m) * sum_i sign_i (Phi q)_i, 0 when ||r|| < 1e-10
          float cr[GS];
#pragma unroll
          for (int g = 0; g < GS; ++g) cr[g] = 0.f;
          if constexpr (qjl) {
            const uint64_t* sw = kq + (int64_t)(tl * TT + tt) * (a.row_kq / 8);
#pragma unroll
            for (int r = 0; r < MQ; ++r) {
              const int i = lane + 32 * r;
              if (i < a.qjl_m) {
                const bool pos = (sw[i >> 6] >> (i & 63)) & 1ull;
#pragma unroll
                for (int g = 0; g < GS; ++g) cr[g] += pos ? pq[g][r] : -pq[g][r];
              }
            }
          }
#pragma unroll
          for (int g = 0; g < GS; ++g) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
              part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
              if (qjl) cr[g] += __shfl_xor_sync(0xffffffffu, cr[g], off);
            }
          }
          float rho = 0.f;
          if (qjl) {
            const float rn = kr[tl * TT + tt];
            rho = rn < 1e-10f ? 0.f : rn * a.qjl_c;
          }
          const float ksv = ks[tt], vsv = vs[tt];
#pragma unroll
          for (int g = 0; g < GS; ++g) {
            const float sc = fmaf(part[g], ksv, cr[g] * rho);
            if (sc > m[g] + kTau) {  // uniform over the warp
              const float al = ex2(m[g] - sc);
              l[g] *= al;
#pragma unroll
              for (int k = 0; k < KPL; ++k) o[g][k] *= al;
              m[g] = sc;
            }
            const float p = ex2(sc - m[g]);
            l[g] += p;
            const float pw2 = p * vsv;
#pragma unroll
            for (int k = 0; k < KPL; ++k) o[g][k] = fmaf(pw2, vv[k], o[g][k]);
          }
        }
        __syncwarp();  // the stage is refilled by the next issue
      }
    }
    float* wp = wpart + warp * GS * PS;
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      if (lane == 0) {
        wp[g * PS] = m[g];
        wp[g * PS + 1] = l[g];
      }
#pragma unroll
      for (int k = 0; k < KPL; ++k) wp[g * PS + 2 + lane + 32 * k] = o[g][k];
    }
    __syncthreads();
    for (int u = threadIdx.x; u < GS * PS; u += blockDim.x) {
      const int g = u / PS, k = u % PS;
      float M = -INFINITY;
      for (int w = 0; w < nw; ++w) M = fmaxf(M, wpart[(w * GS + g) * PS]);
      float val;
      if (k == 0) {
        val = M;
      } else {
        val = 0.f;
        for (int w = 0; w < nw; ++w) {
          const float mw = wpart[(w * GS + g) * PS];
          if (mw != -INFINITY) val += exp2f(mw - M) * wpart[(w * GS + g) * PS + k];
        }
      }
      const int64_t slot = ((int64_t)s * a.hkv + kvh) * a.max_slots + chunk;
      a.part[(slot * a.G + grp * GS + g) * PS + k] = val;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Merge: partial slots of row r = (group r / G, head r % G) at
//   part + ((group * max_slots + c) * G + r % G) * PS,  c < cnt[group]
// -> normalised (optionally un-rotated) output, and/or merged (m, l, o).
// ---------------------------------------------------------------------------

struct MergeDev {
  const float* part;    // packed slots, or null: the separate arrays below
  const float* m_in;    // [slots][n_rows]
  const float* l_in;    // [slots][n_rows]
  const float* o_in;    // [slots][n_rows][D]
  const int32_t* cnt;
  int32_t G, max_slots, n_rows, D;
  float oscale;
  const float* R;
  void* out;
  int32_t out_dtype;
  float* m_out;
  float* l_out;
  float* o_out;
  // separate arrays: floats between slots (0: n_rows for m / l, n_rows * D for o)
  int64_t pstride;
  // split exchange: wait (bounded) until wait_flags[0..wait_n) reach epoch;
  // on a timeout set *status and write NaN rows
  const uint32_t* wait_flags;
  int32_t wait_n;
  uint32_t epoch;
  uint32_t* status;
};

// Bounded acquire-wait of the split exchange: about 2^22 polls of at least
// 256 ns each (over a second) before it gives up.
constexpr uint32_t kSpinLimit = 1u << 22;
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp per row merges the row's split partials: lane c holds slot c's
// max and weight (32 slots at a time, shuffled to the warp as the slots are
// summed, four slots' loads in flight), each lane accumulating head_dim/32
// contiguous dims. The block then un-rotates its rows: thread i computes
// output dim i of 4 rows, reading R[j][i] straight from global memory
// (coalesced, L2-resident). W rows per block (a multiple of 4): 8, or 4 at
// head_dim >= 256, where fewer rows per block put more SMs to work.
template <int kMergeWarps>
__global__ void __launch_bounds__(kMergeWarps * 32, 1) k_merge(MergeDev a) {
  extern __shared__ __align__(16) float so[];  // [kMergeWarps][D]
  pdl_launch_dependents();
  pdl_wait();  // the partials come from the previous kernel
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = a.D;
  const int PS = D + 2;
  const int per = D / 32;  // dims per lane (even)
  const int row = blockIdx.x * kMergeWarps + warp;
  float* orow = so + warp * D;
  if (a.wait_flags) {  // peers' partials: every flag at this call's epoch
    __shared__ int s_late;
    if (threadIdx.x == 0) s_late = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < a.wait_n; i += blockDim.x) {
      uint32_t n = 0;
      while ((int32_t)(ld_acquire_sys(a.wait_flags + i) - a.epoch) < 0) {
        if (++n > kSpinLimit) {
          s_late = 1;
          break;
        }
        __nanosleep(256);
      }
    }
    __syncthreads();
    if (s_late) {
      if (threadIdx.x == 0) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(a.status), "r"(1u) : "memory");
      for (int u = threadIdx.x; u < kMergeWarps * D; u += blockDim.x) {
        const int rr = blockIdx.x * kMergeWarps + u / D;
        if (rr < a.n_rows && a.out) store_any(a.out, a.out_dtype, (int64_t)rr * D + u % D, __int_as_float(0x7fc00000));
      }
      return;
    }
  }
  if (row < a.n_rows) {
    const int64_t group = row / a.G;
    const int gh = row % a.G;
    const int n = a.cnt ? a.cnt[group] : a.max_slots;
    // slot c of this row: m at pm[c * ms], l at pl[c * ms], o at po + c * os
    const float *pm, *pl, *po;
    int64_t ms, os;
    if (a.part) {
      const float* p = a.part + (group * a.max_slots * a.G + gh) * PS;
      pm = p;
      pl = p + 1;
      po = p + 2;
      ms = os = (int64_t)a.G * PS;
    } else {
      pm = a.m_in + row;
      pl = a.l_in + row;
      po = a.o_in + (int64_t)row * D;
      ms = a.pstride ? a.pstride : a.n_rows;
      os = a.pstride ? a.pstride : (int64_t)a.n_rows * D;
    }
    float M = -INFINITY;
    for (int c = lane; c < n; c += 32) M = fmaxf(M, __ldcg(pm + c * ms));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
    float O[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) O[k] = 0.f;
    for (int c0 = 0; c0 < n; c0 += 32) {
      float wl = 0.f;
      if (c0 + lane < n) {
        const float mc = __ldcg(pm + (c0 + lane) * ms);
        wl = mc == -INFINITY ? 0.f : exp2f(mc - M);
        L += wl * __ldcg(pl + (c0 + lane) * ms);
      }
      const int nn = min(32, n - c0);
#pragma unroll 8
      for (int u = 0; u < nn; ++u) {
        const float w = __shfl_sync(0xffffffffu, wl, u);
        const float2* pc = reinterpret_cast<const float2*>(po + (c0 + u) * os + lane * per);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (2 * k < per) {
            const float2 v = __ldcg(pc + k);
            O[2 * k] = fmaf(w, v.x, O[2 * k]);
            O[2 * k + 1] = fmaf(w, v.y, O[2 * k + 1]);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k < per) {
        const float ov = O[k] * a.oscale;
        if (a.o_out) a.o_out[(int64_t)row * D + lane * per + k] = ov;
        orow[lane * per + k] = L > 0.f ? ov / L : 0.f;
      }
    }
    if (a.o_out && lane == 0) {
      a.m_out[row] = M;
      a.l_out[row] = L;
    }
  } else {
    for (int k = lane; k < D; k += 32) orow[k] = 0.f;
  }
  if (!a.out) return;
  __syncthreads();
  // out[row][i] = sum_j R[j][i] * o[row][j]
  const int r_lo = blockIdx.x * kMergeWarps;
  for (int u = threadIdx.x; u < (kMergeWarps / 4) * D; u += blockDim.x) {
    const int i = u % D, rs = (u / D) * 4;
    float acc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = a.R ? 0.f : so[(rs + r) * D + i];
    if (a.R) mat_col<4>(a.R, D, i, so + rs * D, acc);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rr = r_lo + rs + r;
      if (rr < a.n_rows) store_any(a.out, a.out_dtype, (int64_t)rr * D + i, acc[r]);
    }
  }
}


// ---------------------------------------------------------------------------
// 3-bit K / 2-bit V at head_dim 256 on the tensor cores (the sliding and
// global layers of the mixed-precision geometry). Same partition as the
// generic path: an item is (sequence, kv head, chunk of pages) with all
// G <= 4 query heads; the block's warps take the chunk's 16-token tiles in
// turn through a per-warp cp.async double buffer, and the block merges its
// warps' partials into the chunk's slot. One block per SM.
//
// QK^T (S^T = K_dq Q^T: 16 tokens x 8 columns, column n = (head n / 2, f16
// part n % 2) as in the pair layout of the 4-bit path). A K word holds 21
// 3-bit codes (bit 63 zero, bitpack.rs); codes are read in pairs, pair p at
// bits 6p..6p+5 (the 11th pair's second code is the zero bit). Lane t of an
// MMA owns word 4v + t of word group v: in k-step j of the group its slots
// t and t + 4 are pairs 2j and 2j + 1 of that word, so every shift is a
// compile-time constant. Groups 0..2 (words 0..11) take 6 k-steps each, word
// 12 (dims 252..255) one: 19 k-steps. A pair indexes a 64-entry table of f16
// pairs (alpha c_a, alpha c_b), one copy per lane; the query fragments hold
// zeros at the slots of pair 11, of bit 63 and past dim 255, so whatever the
// table returns there adds nothing.
//
// PV (O^T = V_dq^T P^T, 16 m-tiles of dims). A V u32 holds 16 2-bit codes.
// Two tokens' u32s interleave into nibbles (token a's code | token b's << 2),
// one word for the even dims and one for the odd; byte k of either indexes a
// 256-entry table of u32 pairs (its two nibbles dequantized as f16 pairs), so
// one PRMT-addressed 8-byte load feeds two m-tiles. M-tile i, row g is dim
// 16 g + i and row g + 8 is dim 128 + 16 g + i; the k columns are tokens
// (t, t + 8) and (t + 4, t + 12) as in the 4-bit path.
//
// Precise tiles (large sigma_K x ||q'||, see kLoEta): the K pass is run a
// second time over the residual table (alpha c - f16(alpha c)) x 2^11.
// Page-sparse calls pass a tile map: the items then cover the logical
// (chosen) tokens and each tile is fetched from its mapped place.
// ---------------------------------------------------------------------------
constexpr int kM3Warps = 12;
constexpr int kM3TT = 16;
constexpr int kM3KRow = 104, kM3VRow = 64;  // bytes per token: 13 K words, 8 V words
constexpr int kM3KWords = 13;
constexpr int kM3Stage = kM3TT * (kM3KRow + kM3VRow) + 2 * kM3TT * 4;  // 2816
constexpr int kM3Unit = 2 * kM3Stage;  // a warp's two stages
constexpr int kM3KSteps = 19;
constexpr int kM3D = 256, kM3PS = kM3D + 2;
// tables, contiguous from a 64 KiB-aligned shared address: V bytes (256 x 32
// lanes x 8 B), K pairs (64 x 32 x 4 B), K pair residuals (64 x 32 x 4 B)
constexpr int kM3TabK = 65536, kM3TabKLo = 65536 + 8192, kM3Tab = 65536 + 2 * 8192;
// units of kM3Unit bytes around the tables: one per warp (its stages, then
// its partial of the item), one for the query fragments and head norms
constexpr int kM3Units = kM3Warps + 1;
constexpr int kM3Smem = kM3Tab + (kM3Units + 1) * kM3Unit;
// the query unit: fragments, head norms [4], the warps' stage mbarriers [warps][2]
constexpr int kM3OffNorm = kM3KSteps * 32 * 8, kM3OffBar = kM3OffNorm + 16;
static_assert(kM3OffBar + kM3Warps * 16 <= kM3Unit, "query unit overflow");
static_assert(4 * kM3PS * 4 <= kM3Unit, "a warp partial fits its unit");

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
// address of the K table entry of the 6-bit field at bit s of x (s constant
// after unrolling): field << 7 | base (base: 8 KiB-aligned table | lane * 4)
__device__ __forceinline__ uint32_t m3_kaddr(uint64_t x, int s, uint32_t base) {
  const uint32_t f = s >= 7 ? (uint32_t)(x >> (s - 7)) : (uint32_t)x << (7 - s);
  return (f & (63u << 7)) | base;
}
// J k-steps of one word group: x0 / x1 the lane's word of its tokens of MMA
// rows g / g + 8
template <int J>
__device__ __forceinline__ void m3_group(uint64_t x0, uint64_t x1, uint32_t tab, uint32_t qf, float (&c)[4]) {
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const uint32_t a0 = lds32(m3_kaddr(x0, 12 * j, tab)), a1 = lds32(m3_kaddr(x1, 12 * j, tab));
    uint32_t a2 = 0u, a3 = 0u;
    if (j < 5) {
      a2 = lds32(m3_kaddr(x0, 12 * j + 6, tab));
      a3 = lds32(m3_kaddr(x1, 12 * j + 6, tab));
    }
    const uint2 b = lds64(qf + j * 256);
    mma16816(c, a0, a1, a2, a3, b.x, b.y);
  }
}
// S^T += Ktab(K) Q^T over the 19 k-steps; kb: the stage's K words, ra / rb
// the tile rows (tokens) of the lane's MMA rows g / g + 8
__device__ __forceinline__ void m3_qk(const uint64_t* kb, int ra, int rb, int t, uint32_t tab, uint32_t qf,
                                      float (&c)[4]) {
#pragma unroll 1
  for (int v = 0; v < 3; ++v)
    m3_group<6>(kb[ra * kM3KWords + 4 * v + t], kb[rb * kM3KWords + 4 * v + t], tab, qf + v * 6 * 256, c);
  // word 12 + t: lanes t > 0 read the next row's words (zero query slots)
  m3_group<1>(kb[ra * kM3KWords + 12 + t], kb[rb * kM3KWords + 12 + t], tab, qf + 18 * 256, c);
}

template <int G>
__global__ void __launch_bounds__(kM3Warps * 32, 1) k_decode_mma32(const __grid_constant__ DecodeDev a) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t tab_off = (65536u - (s0 & 0xFFFFu)) & 0xFFFFu;
  const int n_before = min((int)(tab_off / kM3Unit), kM3Units);
  auto unit = [&](int u) -> uint8_t* {
    return u < n_before ? smem + u * kM3Unit : smem + tab_off + kM3Tab + (u - n_before) * kM3Unit;
  };
  uint8_t* tab = smem + tab_off;
  const uint32_t tab_s = s0 + tab_off;  // 64 KiB-aligned
  {
    uint32_t* vt = reinterpret_cast<uint32_t*>(tab);
    for (int idx = threadIdx.x; idx < 256 * 64; idx += blockDim.x) {
      const int b = idx >> 6, n = (idx & 1) ? b >> 4 : b & 15;
      vt[idx] = h2_as_u32(__floats2half2_rn(a.vcent[n & 3] * a.valpha, a.vcent[n >> 2] * a.valpha));
    }
    uint32_t* kt = reinterpret_cast<uint32_t*>(tab + kM3TabK);
    uint32_t* kl = reinterpret_cast<uint32_t*>(tab + kM3TabKLo);
    for (int idx = threadIdx.x; idx < 64 * 32; idx += blockDim.x) {
      const int e = idx >> 5;
      const float x0 = a.kcent[e & 7] * a.kalpha, x1 = a.kcent[e >> 3] * a.kalpha;
      kt[idx] = h2_as_u32(__floats2half2_rn(x0, x1));
      kl[idx] = h2_as_u32(__floats2half2_rn((x0 - __half2float(__float2half_rn(x0))) * kLoScale,
                                            (x1 - __half2float(__float2half_rn(x1))) * kLoScale));
    }
  }
  const uint32_t vlane = tab_s | ((uint32_t)lane << 3);
  const uint32_t ktab_s = tab_s + kM3TabK + ((uint32_t)lane << 2);
  const uint32_t klo_s = tab_s + kM3TabKLo + ((uint32_t)lane << 2);
  uint8_t* qunit = unit(kM3Warps);
  uint32_t* qfrag = reinterpret_cast<uint32_t*>(qunit);
  float* qnorm = reinterpret_cast<float*>(qunit + kM3OffNorm);
  const uint32_t bar_s = (uint32_t)__cvta_generic_to_shared(qunit) + kM3OffBar + warp * 16;  // stage s: + 8 s
  // lanes whose query column holds no head (g >= 2G) read a live lane's
  // fragment: the same addresses, so the load takes no extra bank wavefront
  // (their score columns are not used)
  const uint32_t qf_s = (uint32_t)__cvta_generic_to_shared(qunit) + (((g < 2 * G ? g : g % (2 * G)) << 2) | t) * 8;
  uint8_t* wunit = unit(warp);
  const uint32_t st_s = (uint32_t)__cvta_generic_to_shared(wunit);
  if (lane == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 8, 1);
    mbar_init_fence();
  }
  uint32_t ring = 0, cons = 0;  // tiles this warp issued / computed: stage count & 1, phase (count >> 1) & 1
  bool err = false;             // a stage wait ran out: the warp's partials become NaN
  // the tables above are the codecs' constants; the rotated queries and the
  // pages may come from the previous kernels of the stream
  pdl_wait();

  const int64_t total = (int64_t)a.n_seqs * a.hkv * a.n_chunks;
  for (int64_t item = blockIdx.x; item < total; item += gridDim.x) {
    const int chunk = (int)(item % a.n_chunks);
    const int64_t rest = item / a.n_chunks;
    const int kvh = (int)(rest % a.hkv);
    const int sq = (int)(rest / a.hkv);
    const int64_t n_valid = a.si()[2 * sq];
    const uint64_t* trow = a.table + a.si()[2 * sq + 1] * a.table_stride;
    const int64_t qrow0 = ((int64_t)sq * a.hq + (int64_t)kvh * G) * kM3D;
    // q' of head h at dim d: the rotated f32 rows, or the caller's rotated
    // rows scaled here
    auto qv = [&](int h, int d) {
      return a.q_in ? load_any(a.q_in, a.q_dtype, qrow0 + h * kM3D + d) * a.qscale : a.q_rot[qrow0 + h * kM3D + d];
    };
    const int p0 = chunk * a.pages_per_chunk;
    const int64_t ctok = n_valid - (int64_t)p0 * kPageTokens;
    const int64_t cmax = (int64_t)a.pages_per_chunk * kPageTokens;
    const int chunk_tok = (int)(ctok <= 0 ? 0 : (ctok < cmax ? ctok : cmax));
    constexpr int tpp = kPageTokens / kM3TT;
    const int ctiles = (chunk_tok + kM3TT - 1) / kM3TT;
    const uint64_t my_page = lane < a.pages_per_chunk && (int64_t)(p0 + lane) * kPageTokens < n_valid ? trow[p0 + lane] : 0ull;
    auto my_page_of = [&](int i) { return __shfl_sync(0xffffffffu, my_page, i); };
    // a tile: K words, V words, sigma_K, sigma_V of 16 consecutive rows, four
    // contiguous runs of the page, copied by lane 0 into stage ring & 1
    auto issue = [&](int tl) {
      fence_proxy_async();  // the stage's earlier reads and P^T writes come first
      __syncwarp();
      const uint8_t* page = reinterpret_cast<const uint8_t*>(my_page_of(tl / tpp));
      int rt = tl % tpp;  // 16-token tile within the page
      if (a.tile_map) {
        // page-sparse: logical 16-token tile lt of the (sequence, kv head) is
        // half (lt & 1) of its mapped 32-token tile
        const int64_t lt = (int64_t)chunk * a.pages_per_chunk * tpp + tl;
        const int64_t p16 = 2 * (int64_t)a.tile_map[((int64_t)sq * a.hkv + kvh) * a.map_stride + (lt >> 1)] + (lt & 1);
        page = reinterpret_cast<const uint8_t*>(trow[p16 / tpp]);
        rt = (int)(p16 % tpp);
      }
      if (lane == 0) {
        const int64_t r0 = (int64_t)kvh * kPageTokens + rt * kM3TT;
        const uint32_t dst = st_s + (ring & 1) * kM3Stage, bar = bar_s + (ring & 1) * 8;
        mbar_expect_tx(bar, kM3Stage);
        bulk_g2s(dst, page + a.off_kw + r0 * kM3KRow, kM3TT * kM3KRow, bar);
        bulk_g2s(dst + kM3TT * kM3KRow, page + a.off_vw + r0 * kM3VRow, kM3TT * kM3VRow, bar);
        bulk_g2s(dst + kM3TT * (kM3KRow + kM3VRow), page + a.off_ks + r0 * 4, kM3TT * 4, bar);
        bulk_g2s(dst + kM3TT * (kM3KRow + kM3VRow + 4), page + a.off_vs + r0 * 4, kM3TT * 4, bar);
      }
      ++ring;
    };
    // MMA row g (g + 8) of S^T is tile row ra (rb): rows 4 (g & 3) + (g >> 2)
    // and 2 more, so that the four rows a half-warp reads K words of (104-byte
    // rows) start 32 bytes apart mod 128 and take distinct banks. PV's token
    // slots follow: lane t's k-slots 2t, 2t + 1 hold the pair a P^T writer
    // lane gw0 = t + 4 (t & 1) holds (rows 4t + (t & 1) and 2 more), slots
    // 2t + 8, 2t + 9 the pair of lane gw0 ^ 4.
    const int ra = 4 * (g & 3) + (g >> 2), rb = ra + 2;
    const int gw0 = t + 4 * (t & 1);
    // the first tile's copy runs while the block builds the query fragments
    if (warp < ctiles) issue(warp);
    // query fragments in slot order: k-step ks, lane (n, tt) holds column n
    // = (head n / 2, f16 part n % 2) at the pairs of slots tt and tt + 4
    for (int u = threadIdx.x; u < kM3KSteps * 32; u += blockDim.x) {
      const int ks = u >> 5, ln = u & 31, n = ln >> 2, tt = ln & 3;
      const int head = n >> 1, part = n & 1;
      const int v = ks < 18 ? ks / 6 : 3, j = ks < 18 ? ks % 6 : 0;
      const int w = 4 * v + tt;
      uint32_t bb[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float x[2] = {0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pos = 2 * (2 * j + h) + e, d = 21 * w + pos;
          if (head < G && pos < 21 && d < kM3D) x[e] = qv(head, d);
        }
        const __half2 hv = __floats2half2_rn(x[0], x[1]);
        const float2 f = __half22float2(hv);
        bb[h] = part ? h2_as_u32(__floats2half2_rn(x[0] - f.x, x[1] - f.y)) : h2_as_u32(hv);
      }
      qfrag[u * 2] = bb[0];
      qfrag[u * 2 + 1] = bb[1];
    }
    if (warp < G) {  // ||q'||^2 per head, for the precise-tile test
      float s2 = 0.f;
      for (int d = lane; d < kM3D; d += 32) {
        const float v = qv(warp, d);
        s2 = fmaf(v, v, s2);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      if (lane == 0) qnorm[warp] = s2;
    }
    __syncthreads();
    float qn2 = 0.f;
#pragma unroll
    for (int h = 0; h < G; ++h) qn2 = fmaxf(qn2, qnorm[h]);
    const float lthr = a.klo_thr * rsqrtf(qn2);

    float m = -INFINITY, l = 0.f;
    float oacc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
    for (int tl = warp; tl < ctiles; tl += kM3Warps) {
      if (tl + kM3Warps < ctiles) issue(tl + kM3Warps);
      const uint32_t stg = cons & 1;
      if (!mbar_wait(bar_s + stg * 8, (cons >> 1) & 1)) err = true;
      ++cons;
      __syncwarp();
      const uint8_t* st = wunit + stg * kM3Stage;
      const uint64_t* kb = reinterpret_cast<const uint64_t*>(st);
      const uint32_t* vb = reinterpret_cast<const uint32_t*>(st + kM3TT * kM3KRow);
      const float* ks = reinterpret_cast<const float*>(st + kM3TT * (kM3KRow + kM3VRow));
      const float* vs = ks + kM3TT;
      const int tok = tl * kM3TT;
      const bool ok0 = tok + ra < chunk_tok, ok1 = tok + rb < chunk_tok;
      // ---- S^T: lane (g, t) gets head t at tile rows ra and rb ----
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      m3_qk(kb, ra, rb, t, ktab_s, qf_s, c);
      float y0 = c[0] + c[1], y1 = c[2] + c[3];
      const float k0 = ks[ra], k1 = ks[rb];
      if (__any_sync(0xffffffffu, t < G && fmaxf(k0, k1) > lthr)) {
        const float zm = fmaxf(ok0 ? y0 * k0 : -INFINITY, ok1 ? y1 * k1 : -INFINITY);
        if (__any_sync(0xffffffffu, t < G && fmaxf(k0, k1) > lthr && zm > m - kLoTheta)) {
          float cl[4] = {0.f, 0.f, 0.f, 0.f};
          m3_qk(kb, ra, rb, t, klo_s, qf_s, cl);
          y0 = fmaf(cl[0] + cl[1], kLoUnscale, y0);
          y1 = fmaf(cl[2] + cl[3], kLoUnscale, y1);
        }
      }
      const float s0_ = ok0 ? y0 * k0 : -INFINITY, s1_ = ok1 ? y1 * k1 : -INFINITY;
      float mx = fmaxf(s0_, s1_);
      if (__any_sync(0xffffffffu, mx > m + kTau)) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (mx > m + kTau) {
          const float al = ex2(m - mx);
          l *= al;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            oacc[i][0] *= al;
            oacc[i][1] *= al;
            oacc[i][2] *= al;
            oacc[i][3] *= al;
          }
          m = mx;
        }
      }
      const float pp0 = ex2(s0_ - m), pp1 = ex2(s1_ - m);
      l += pp0 + pp1;
      // V words g and g + 8 of the token pairs (4t + (tp ^ (t & 1)), + 2)
      // for k-slot pair tp (the pairs of P^T lanes gw0, gw0 ^ 4), read
      // before the P^T exchange reuses the stage's K area. Index word
      // xv[tp][h][par], byte k: the token pair's nibble (a | b << 2) at dim
      // 4k + 2h + par of word g, then the same of word g + 8, so that one
      // 8-byte table entry is (row g, row g + 8) of an m-tile's A operand.
      uint32_t xv[2][2][2];
#pragma unroll
      for (int tp = 0; tp < 2; ++tp) {
        uint32_t ev[2], od[2];  // word g, word g + 8
#pragma unroll
        for (int wv = 0; wv < 2; ++wv) {
          const int rv = 4 * t + (tp ^ (t & 1));
          const uint32_t va = vb[rv * 16 + g + 8 * wv], vbb = vb[(rv + 2) * 16 + g + 8 * wv];
          ev[wv] = (va & 0x33333333u) | ((vbb & 0x33333333u) << 2);
          od[wv] = ((va >> 2) & 0x33333333u) | (vbb & 0xCCCCCCCCu);
        }
        xv[tp][0][0] = (ev[0] & 0x0F0F0F0Fu) | ((ev[1] & 0x0F0F0F0Fu) << 4);
        xv[tp][1][0] = ((ev[0] >> 4) & 0x0F0F0F0Fu) | (ev[1] & 0xF0F0F0F0u);
        xv[tp][0][1] = (od[0] & 0x0F0F0F0Fu) | ((od[1] & 0x0F0F0F0Fu) << 4);
        xv[tp][1][1] = ((od[0] >> 4) & 0x0F0F0F0Fu) | (od[1] & 0xF0F0F0F0u);
      }
      // P^T fragments: lane (g, t) holds p' of head t at tile rows ra, rb and
      // reads column g = (head g / 2, part g & 1) at the pairs of lanes gw0
      // and gw0 ^ 4 (the layout of p_exchange, one 16-token half)
      uint32_t pb0, pb1;
      {
        const float pa = ok0 ? pp0 * vs[ra] : 0.f, pz = ok1 ? pp1 * vs[rb] : 0.f;
        uint32_t* ps = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(st));
        const __half2 h0 = __floats2half2_rn(pa, pz);
        const float2 f0 = __half22float2(h0);
        const uint32_t l0 = h2_as_u32(__floats2half2_rn(pa - f0.x, pz - f0.y));
        __syncwarp();
        ps[t * 8 + g] = h2_as_u32(h0);
        ps[32 + t * 8 + (g ^ 4)] = l0;
        __syncwarp();
        const int head = g >> 1, part = g & 1;
        const int base = part * 32 + head * 8, sw = part << 2;
        pb0 = head < G ? ps[base + (gw0 ^ sw)] : 0u;
        pb1 = head < G ? ps[base + ((gw0 ^ 4) ^ sw)] : 0u;
      }
      // ---- O^T += V^T P^T: m-tile 4k + 2h + par ----
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int par = 0; par < 2; ++par) {
            const uint32_t sel = 0x7604u | ((uint32_t)k << 4);
            const uint2 r0 = lds64(__byte_perm(xv[0][h][par], vlane, sel));  // a0, a1
            const uint2 r1 = lds64(__byte_perm(xv[1][h][par], vlane, sel));  // a2, a3
            mma16816(oacc[4 * k + 2 * h + par], r0.x, r0.y, r1.x, r1.y, pb0, pb1);
          }
      __syncwarp();  // the stage is refilled by the next issue
    }
    // ---- the warp's partial of the chunk in its unit (its copies are done):
    // head t, dims 16 g + i (rows g) and 128 + 16 g + i (rows g + 8) ----
    float L = l;
    L += __shfl_xor_sync(0xffffffffu, L, 4);
    L += __shfl_xor_sync(0xffffffffu, L, 8);
    L += __shfl_xor_sync(0xffffffffu, L, 16);
    if (__any_sync(0xffffffffu, err)) L = __int_as_float(0x7fc00000);  // NaN: the merged row shows it
    __syncwarp();
    float* wp = reinterpret_cast<float*>(wunit) + (t < G ? t : 0) * kM3PS;
    if (t < G) {
      if (g == 0) {
        wp[0] = m;
        wp[1] = L;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        wp[2 + 16 * g + i] = oacc[i][0] + oacc[i][1];
        wp[2 + 128 + 16 * g + i] = oacc[i][2] + oacc[i][3];
      }
    }
    __syncthreads();
    // the chunk's slot; with one chunk per (sequence, kv head) it stays in
    // the query unit (its fragments are spent) for the finish below
    float* fin = reinterpret_cast<float*>(qunit);  // [G][kM3PS]
    for (int u = threadIdx.x; u < G * kM3PS; u += blockDim.x) {
      const int hd = u / kM3PS, k = u % kM3PS;
      float M = -INFINITY;
      for (int w2 = 0; w2 < kM3Warps; ++w2) M = fmaxf(M, reinterpret_cast<const float*>(unit(w2))[hd * kM3PS]);
      float val;
      if (k == 0) {
        val = M;
      } else {
        val = 0.f;
        for (int w2 = 0; w2 < kM3Warps; ++w2) {
          const float* wq = reinterpret_cast<const float*>(unit(w2)) + hd * kM3PS;
          if (wq[0] != -INFINITY) val += exp2f(wq[0] - M) * wq[k];
        }
      }
      if (a.out) {
        fin[hd * kM3PS + k] = val;
      } else {
        const int64_t slot = ((int64_t)sq * a.hkv + kvh) * a.max_slots + chunk;
        a.part[(slot * G + hd) * kM3PS + k] = val;
      }
    }
    __syncthreads();
    if (a.out) {
      // out = R^T (o / l) x oscale, as the merge kernel would write it (a NaN
      // l from a stage wait that ran out stays visible)
      float* so = reinterpret_cast<float*>(unit(0));  // [G][kM3D]: warp 0's partial was read above
      for (int u = threadIdx.x; u < G * kM3D; u += blockDim.x) {
        const int hd = u / kM3D;
        const float L = fin[hd * kM3PS + 1];
        so[u] = (L > 0.f || L != L) ? fin[hd * kM3PS + 2 + u % kM3D] * a.oscale / L : 0.f;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < kM3D; i += blockDim.x) {
        float acc[G];
#pragma unroll
        for (int r = 0; r < G; ++r) acc[r] = a.out_R ? 0.f : so[r * kM3D + i];
        if (a.out_R) mat_col<G>(a.out_R, kM3D, i, so, acc);
#pragma unroll
        for (int r = 0; r < G; ++r)
          store_any(a.out, a.out_dtype, ((int64_t)sq * a.hq + (int64_t)kvh * G + r) * kM3D + i, acc[r]);
      }
      __syncthreads();
    }
  }
  // after a wait that ran out, the copies may still be in flight: wait for
  // each stage's last phase (bounded) before the block's shared memory goes
  if (__any_sync(0xffffffffu, err)) {
    const uint32_t uses0 = (ring + 1) >> 1, uses1 = ring >> 1;
    if (uses0) mbar_wait(bar_s, (uses0 - 1) & 1);
    if (uses1) mbar_wait(bar_s + 8, (uses1 - 1) & 1);
  }
}

int g_num_sms = 0;

template <int G>
void launch_flat_g(const DecodeDev& d, int grid, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_flat<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFlatSmem));
    attr = true;
  }
  k_decode_flat<G><<<(unsigned)grid, kFlatWarps * 32, kFlatSmem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

template <int G, bool FUSED, bool SPARSE = false>
void launch_pair_g(const DecodeDev& d, int grid, cudaStream_t s) {
  constexpr int smem = FUSED ? kFusedSmem : kFlatSmem;
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_pair<G, FUSED, SPARSE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
  if constexpr (FUSED) {
    // programmatic serialization: the prologue overlaps the previous kernel's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kFlatWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    LC_CUDA(cudaLaunchKernelEx(&cfg, k_decode_pair<G, FUSED, SPARSE>, d));
  } else {
    k_decode_pair<G, FUSED, SPARSE><<<(unsigned)grid, kFlatWarps * 32, smem, s>>>(d);
    LC_CUDA(cudaGetLastError());
  }
}

template <int G>
void launch_mma32_g(const DecodeDev& d, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_mma32<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kM3Smem));
    attr = true;
  }
  const int64_t total = (int64_t)d.n_seqs * d.hkv * d.n_chunks;
  const int64_t grid = std::min<int64_t>((int64_t)num_sms(), total);
  if (grid <= 0) return;
  launch_pdl(k_decode_mma32<G>, dim3((unsigned)grid), dim3(kM3Warps * 32), kM3Smem, s, d);
}

template <int KPL, int GS, bool QJL>
void launch_generic_q(DecodeDev d, cudaStream_t s) {
  const int nw = 4;
  // 32-token tiles where a token's K + V words fit 256 bytes, else 16
  d.gen_tt = d.row_kw + d.row_vw <= 256 ? 32 : 16;
  d.gen_stage = d.gen_tt * (d.row_kw + d.row_vw) + 2 * d.gen_tt * 4;
  const size_t smem = (512 + (size_t)nw * GS * (32 * KPL + 2)) * sizeof(float) + (size_t)nw * 2 * d.gen_stage;
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_generic<KPL, GS, QJL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 227 * 1024));
    attr = true;
  }
  LC_REQUIRE(smem <= 227 * 1024, LC_ERR_INVALID, "decode: head_dim / bit widths too large for the generic path");
  int per_sm = 0;
  LC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_generic<KPL, GS, QJL>, nw * 32, smem));
  if (per_sm < 1) per_sm = 1;
  const int64_t total = (int64_t)d.n_seqs * d.hkv * (d.G / GS) * d.n_chunks;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > total) grid = total;
  k_decode_generic<KPL, GS, QJL><<<(unsigned)grid, nw * 32, smem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

template <int KPL, int GS>
void launch_generic_t(const DecodeDev& d, cudaStream_t s) {
  if (d.q_proj) return launch_generic_q<KPL, GS, true>(d, s);
  return launch_generic_q<KPL, GS, false>(d, s);
}

template <int KPL>
void launch_generic_k(const DecodeDev& d, cudaStream_t s) {
  if constexpr (KPL <= 8) {
    if (d.G % 4 == 0) return launch_generic_t<KPL, 4>(d, s);
  }
  if (d.G % 2 == 0) return launch_generic_t<KPL, 2>(d, s);
  return launch_generic_t<KPL, 1>(d, s);
}

}  // namespace

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

bool decode_fast_path(int dim, int kbits, int vbits, int G) {
  return dim == 128 && kbits == 4 && vbits == 4 && G >= 1 && G <= 8;
}

bool decode_mma_path(int dim, int kbits, int vbits, int G) {
  return dim == 256 && kbits == 3 && vbits == 2 && G >= 1 && G <= 4;
}

// Most (sequence, kv head) segments any CTA's tile range touches.
static int32_t max_cta_segments(const int64_t* seg, const int64_t* lens, int n, int hkv, int64_t total, int64_t pw,
                                int grid) {
  if (total <= 0) return 0;
  auto sid_of = [&](int64_t x) {
    int lo = 0, hi = n - 1;  // last b with seg[b] <= x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg[mid] <= x) lo = mid;
      else hi = mid - 1;
    }
    const int64_t nt = (lens[lo] + kTileTok - 1) / kTileTok;
    return (int64_t)lo * hkv + (x - seg[lo]) / nt;
  };
  int64_t mx = 0;
  const int64_t span = (int64_t)kFlatWarps * pw;
  for (int c = 0; c < grid; ++c) {
    const int64_t cb = (int64_t)c * span;
    if (cb >= total) break;
    const int64_t ce = std::min(cb + span, total) - 1;
    mx = std::max(mx, sid_of(ce) - sid_of(cb) + 1);
  }
  return (int32_t)mx;
}

// The partition of one decode call, written into seg [n + 1] (flat path) and
// cnt [n * hkv]; shared by plan_decode (vectors it owns) and
// plan_decode_into (caller arrays, no allocation).
static void plan_core(const int64_t* lens, int n, int hkv, int hq, int dim, int kbits, int vbits, bool generic_only,
                      DecodePlan& p, int64_t* seg, int32_t* cnt) {
  const int G = hq / hkv;
  for (int64_t i = 0; i < (int64_t)n * hkv; ++i) cnt[i] = 0;
  if (!generic_only && decode_fast_path(dim, kbits, vbits, G)) {
    p.flat = true;
    p.grid = num_sms();
    seg[0] = 0;
    for (int b = 0; b < n; ++b) seg[b + 1] = seg[b] + (int64_t)hkv * ((lens[b] + kTileTok - 1) / kTileTok);
    p.total_tiles = seg[n];
    const int64_t W = (int64_t)p.grid * kFlatWarps;
    p.per_warp = p.total_tiles > 0 ? (p.total_tiles + W - 1) / W : 1;
    int32_t mx = 1;
    for (int b = 0; b < n; ++b) {
      const int64_t nt = (lens[b] + kTileTok - 1) / kTileTok;
      if (nt == 0) continue;
      for (int h = 0; h < hkv; ++h) {
        const int64_t s0 = seg[b] + (int64_t)h * nt;
        const int32_t c = (int32_t)((s0 + nt - 1) / p.per_warp - s0 / p.per_warp + 1);
        cnt[(size_t)b * hkv + h] = c;
        mx = c > mx ? c : mx;
      }
    }
    p.max_slots = mx;
    p.max_cta_segs = max_cta_segments(seg, lens, n, hkv, p.total_tiles, p.per_warp, p.grid);
  } else {
    p.flat = false;
    p.mma = !generic_only && decode_mma_path(dim, kbits, vbits, G);
    int64_t mx = 0;
    for (int b = 0; b < n; ++b) mx = lens[b] > mx ? lens[b] : mx;
    const int64_t pages = (mx + kPageTokens - 1) / kPageTokens;
    int ppc = 4;
    if (p.mma) {
      // The tensor-core path (one block of 12 warps per SM, an item's
      // 16-token tiles dealt to the warps in rounds): the chunk of 1 .. 16
      // pages with the least modelled time, waves x (item set-up + rounds x
      // round), with a set-up of ~2.7 tile rounds (the query fragments, the
      // first tile's latency, the block merge; fitted to B200 timings of
      // 1024-token and 32K-token layers). Short layers get one item per
      // (sequence, kv head); long ones 16-page chunks.
      const int64_t sms = num_sms();
      double best = 0.0;
      for (int c = 16; c >= 1; c >>= 1) {
        const int64_t items = (int64_t)n * hkv * ((pages + c - 1) / c);
        const int64_t waves = (items + sms - 1) / sms;
        const int64_t rounds = (c * (kPageTokens / 16) + 11) / 12;
        const double t = (double)waves * (2.7 + (double)rounds);
        if (c == 16 || t < best) {
          best = t;
          ppc = c;
        }
      }
    } else {
      // 4 pages per chunk, or fewer when that leaves too few (sequence, kv
      // head, chunk) items to fill the GPU (short contexts, sliding windows)
      const int64_t want = 8LL * num_sms();
      while (ppc > 1 && (int64_t)n * hkv * ((pages + ppc - 1) / ppc) < want) ppc >>= 1;
    }
    p.pages_per_chunk = ppc;
    p.n_chunks = (int32_t)((pages + ppc - 1) / ppc > 0 ? (pages + ppc - 1) / ppc : 1);
    p.max_slots = p.n_chunks;
    for (int64_t i = 0; i < (int64_t)n * hkv; ++i) cnt[i] = p.n_chunks;
  }
}

DecodePlan plan_decode(const std::vector<int64_t>& lens, int hkv, int hq, int dim, int kbits, int vbits,
                       bool generic_only) {
  DecodePlan p;
  const int n = (int)lens.size();
  p.cnt.assign((size_t)n * hkv, 0);
  p.seg.assign(n + 1, 0);
  plan_core(lens.data(), n, hkv, hq, dim, kbits, vbits, generic_only, p, p.seg.data(), p.cnt.data());
  if (!p.flat) p.seg.clear();
  return p;
}

void plan_decode_into(const int64_t* lens, int n, int hkv, int hq, int dim, int kbits, int vbits, DecodePlan& p,
                      int64_t* seg, int32_t* cnt) {
  plan_core(lens, n, hkv, hq, dim, kbits, vbits, false, p, seg, cnt);
}

void launch_rotate_q(const void* q, int32_t q_dtype, int32_t n_rows, int32_t dim, const float* RT,
                     bool q_is_rotated, float qscale, float* q_rot, __half* q_h, cudaStream_t s) {
  if (n_rows <= 0) return;
  LC_REQUIRE(dim % 64 == 0, LC_ERR_INVALID, "decode: head_dim must be 64, 128, 256 or 512");
  const dim3 grid((unsigned)((n_rows + kRotRows - 1) / kRotRows), (unsigned)(dim / kRotDims));
  const size_t smem = ((size_t)kRotRows * dim + (size_t)kRotSplit * kRotRows * kRotDims) * sizeof(float);
  launch_pdl(k_rotate_q, grid, dim3(kRotDims * kRotSplit), smem, s, q, q_dtype, n_rows, dim, RT,
             q_is_rotated ? 1 : 0, qscale, q_rot, q_h);
  LC_CUDA(cudaGetLastError());
}

void launch_project_q(const void* q, int32_t dtype, int32_t n_rows, int32_t dim, int32_t m, const float* PT,
                      float qscale, float* q_proj, cudaStream_t s) {
  if (n_rows <= 0) return;
  k_project_q<<<n_rows, 128, (size_t)dim * sizeof(float), s>>>(q, dtype, dim, m, PT, qscale, q_proj);
  LC_CUDA(cudaGetLastError());
}

static DecodeDev make_dev(const DecodeArgs& a, const DecodePlan& p) {
  LC_REQUIRE(p.total_tiles < (int64_t(1) << 31) - (int64_t)kFlatWarps * 148 * 2, LC_ERR_INVALID,
             "decode call too large: split it (at most 2^31 tiles of 32 tokens x kv head)");
  DecodeDev d{};
  if (!a.seqinfo) {
    LC_REQUIRE(a.h_seqinfo && a.n_seqs <= kInlineSeqs && (int64_t)a.n_seqs * a.hkv <= kInlineCnt, LC_ERR_STATE,
               "inline decode metadata does not fit");
    std::memcpy(d.meta.seqinfo, a.h_seqinfo, (size_t)a.n_seqs * 2 * sizeof(int64_t));
    if (a.h_seg) std::memcpy(d.meta.seg, a.h_seg, (size_t)(a.n_seqs + 1) * sizeof(int64_t));
    if (a.h_cnt) std::memcpy(d.meta.cnt, a.h_cnt, (size_t)a.n_seqs * a.hkv * sizeof(int32_t));
  }
  d.table = a.table;
  d.table_stride = a.table_stride;
  d.seqinfo = a.seqinfo;
  d.seg = a.seg;
  d.per_warp = p.per_warp;
  d.total_tiles = p.total_tiles;
  d.max_slots = p.max_slots;
  d.off_kw = a.layout.off[a.role_kw];
  d.off_vw = a.layout.off[a.role_vw];
  d.off_ks = a.layout.off[a.role_ks];
  d.off_vs = a.layout.off[a.role_vs];
  d.row_kw = (int32_t)a.layout.row[a.role_kw];
  d.row_vw = (int32_t)a.layout.row[a.role_vw];
  d.n_seqs = a.n_seqs;
  d.hkv = a.hkv;
  d.hq = a.hq;
  d.dim = a.dim;
  d.kbits = a.kbits;
  d.vbits = a.vbits;
  d.pages_per_chunk = p.pages_per_chunk;
  d.n_chunks = p.n_chunks;
  d.G = a.hq / a.hkv;
  d.q_rot = a.q_rot;
  d.q_h = a.q_h;
  if (a.q_raw) {
    d.q_in = a.q_raw;
    d.q_dtype = a.q_raw_dtype;
    d.q_rotated = 1;
    d.qscale = a.q_raw_scale;
  }
  if (a.fin_out) {
    d.out = a.fin_out;
    d.out_dtype = a.fin_dtype;
    d.out_R = a.fin_R;
    d.oscale = a.fin_oscale;
  }
  d.kcent = a.kcent;
  d.vcent = a.vcent;
  d.kalpha = a.kalpha;
  d.valpha = a.valpha;
  d.klo_thr = a.klo_thr;
  d.part = a.part;
  d.tile_map = a.tile_map;
  d.map_stride = a.map_stride;
  d.q_proj = a.q_proj;
  if (a.q_proj) {
    LC_REQUIRE(!p.flat && a.qjl_m > 0 && a.qjl_m <= kMaxQjlDecode && a.role_kq >= 0 && a.role_kr >= 0,
               LC_ERR_STATE, "QJL scores need the generic path, 0 < qjl_m <= 256 and stored K QJL bits");
    d.off_kq = a.layout.off[a.role_kq];
    d.off_kr = a.layout.off[a.role_kr];
    d.row_kq = (int32_t)a.layout.row[a.role_kq];
    d.qjl_m = a.qjl_m;
    d.qjl_c = a.qjl_c;
  }
  return d;
}

void launch_decode_partials(const DecodeArgs& a, const DecodePlan& p, cudaStream_t s) {
  const DecodeDev d = make_dev(a, p);
  if (p.flat) {
    if (p.total_tiles == 0) return;
    if (d.tile_map) {  // page-sparse: pair geometry only (checked by the caller)
      LC_REQUIRE(d.G >= 1 && d.G <= 4, LC_ERR_INVALID, "page-sparse decode needs GQA <= 4");
      switch (d.G) {
        case 1: return launch_pair_g<1, false, true>(d, p.grid, s);
        case 2: return launch_pair_g<2, false, true>(d, p.grid, s);
        case 3: return launch_pair_g<3, false, true>(d, p.grid, s);
        default: return launch_pair_g<4, false, true>(d, p.grid, s);
      }
    }
    switch (d.G) {
      case 1: return launch_pair_g<1, false>(d, p.grid, s);
      case 2: return launch_pair_g<2, false>(d, p.grid, s);
      case 3: return launch_pair_g<3, false>(d, p.grid, s);
      case 4: return launch_pair_g<4, false>(d, p.grid, s);
      case 5: return launch_flat_g<5>(d, p.grid, s);
      case 6: return launch_flat_g<6>(d, p.grid, s);
      case 7: return launch_flat_g<7>(d, p.grid, s);
      default: return launch_flat_g<8>(d, p.grid, s);
    }
  }
  if (p.mma) {
    LC_REQUIRE(!d.q_proj && d.row_kw == kM3KRow && d.row_vw == kM3VRow, LC_ERR_STATE,
               "decode: the tensor-core 3/2-bit path takes calls without QJL");
    switch (d.G) {
      case 1: return launch_mma32_g<1>(d, s);
      case 2: return launch_mma32_g<2>(d, s);
      case 3: return launch_mma32_g<3>(d, s);
      default: return launch_mma32_g<4>(d, s);
    }
  }
  switch (a.dim) {
    case 64: return launch_generic_k<2>(d, s);
    case 128: return launch_generic_k<4>(d, s);
    case 256: return launch_generic_k<8>(d, s);
    case 512: return launch_generic_k<16>(d, s);
    default: LC_THROW(LC_ERR_INVALID, "decode: head_dim must be 64, 128, 256 or 512");
  }
}

bool decode_fusable(const DecodePlan& p, int G) {
  // segments of more than 64 slots (a long sequence over the whole grid)
  // merge faster in the wide merge kernel than in one warp per row in-kernel
  return p.flat && G >= 1 && G <= 4 && p.max_cta_segs <= kFusedSegs && p.max_slots <= 64;
}

void launch_decode_fused(const DecodeArgs& a, const DecodePlan& p, const FusedArgs& f, cudaStream_t s) {
  LC_REQUIRE(decode_fusable(p, a.hq / a.hkv), LC_ERR_STATE, "decode plan is not fusable");
  if (p.total_tiles == 0) return;
  DecodeDev d = make_dev(a, p);
  d.q_in = f.q;
  d.q_dtype = f.q_dtype;
  d.q_rotated = f.q_rotated;
  d.qscale = f.qscale;
  d.qR = f.qR;
  d.vRT = f.vRT;
  d.cnt = f.cnt;
  d.ctr = f.ctr;
  d.out = f.out;
  d.out_dtype = f.out_dtype;
  d.oscale = f.oscale;
  d.parts = f.parts;
  d.parts_rows = f.parts_rows;
  if (d.tile_map) {  // page-sparse
    switch (d.G) {
      case 1: return launch_pair_g<1, true, true>(d, p.grid, s);
      case 2: return launch_pair_g<2, true, true>(d, p.grid, s);
      case 3: return launch_pair_g<3, true, true>(d, p.grid, s);
      default: return launch_pair_g<4, true, true>(d, p.grid, s);
    }
  }
  switch (d.G) {
    case 1: return launch_pair_g<1, true>(d, p.grid, s);
    case 2: return launch_pair_g<2, true>(d, p.grid, s);
    case 3: return launch_pair_g<3, true>(d, p.grid, s);
    default: return launch_pair_g<4, true>(d, p.grid, s);
  }
}

// Merge of rows with many slots (one long sequence split over all warps of
// the grid: a few hundred slots per row, few rows): a block per row, its
// kMergeWideWarps warps taking slots w, w + warps, ...; each warp's (M, L, O)
// goes to shared memory and the block combines them, normalises and
// un-rotates the row. The slot order inside a sum differs from k_merge's,
// within f32 rounding.
constexpr int kMergeWideWarps = 16;
__global__ void __launch_bounds__(kMergeWideWarps * 32, 1) k_merge_wide(MergeDev a) {
  extern __shared__ __align__(16) float sw[];  // [warps][D] O, then [warps] M, [warps] L, then [D] the row
  pdl_launch_dependents();
  pdl_wait();  // the partials come from the previous kernel
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int D = a.D, PS = D + 2, per = D / 32;
  const int row = blockIdx.x;
  float* wo = sw + warp * D;
  float* wm = sw + kMergeWideWarps * D;
  float* wl = wm + kMergeWideWarps;
  float* orow = wl + kMergeWideWarps;
  const int64_t group = row / a.G;
  const int gh = row % a.G;
  const int n = a.cnt ? a.cnt[group] : a.max_slots;
  const float *pm, *pl, *po;
  int64_t ms, os;
  if (a.part) {
    const float* p = a.part + (group * a.max_slots * a.G + gh) * PS;
    pm = p;
    pl = p + 1;
    po = p + 2;
    ms = os = (int64_t)a.G * PS;
  } else {
    pm = a.m_in + row;
    pl = a.l_in + row;
    po = a.o_in + (int64_t)row * D;
    ms = a.pstride ? a.pstride : a.n_rows;
    os = a.pstride ? a.pstride : (int64_t)a.n_rows * D;
  }
  // this warp's slots: c = warp + kMergeWideWarps k
  float M = -INFINITY;
  for (int c = warp + kMergeWideWarps * lane; c < n; c += kMergeWideWarps * 32) M = fmaxf(M, __ldcg(pm + c * ms));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  float O[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) O[k] = 0.f;
  for (int c0 = warp; c0 < n; c0 += kMergeWideWarps * 32) {
    const int c = c0 + kMergeWideWarps * lane;
    float wgt = 0.f;
    if (c < n) {
      const float mc = __ldcg(pm + c * ms);
      wgt = mc == -INFINITY ? 0.f : exp2f(mc - M);
      L += wgt * __ldcg(pl + c * ms);
    }
    const int nn = min(32, (n - c0 + kMergeWideWarps - 1) / kMergeWideWarps);
#pragma unroll 4
    for (int u = 0; u < nn; ++u) {
      const float w = __shfl_sync(0xffffffffu, wgt, u);
      const float2* pc = reinterpret_cast<const float2*>(po + (int64_t)(c0 + kMergeWideWarps * u) * os + lane * per);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (2 * k < per) {
          const float2 v = __ldcg(pc + k);
          O[2 * k] = fmaf(w, v.x, O[2 * k]);
          O[2 * k + 1] = fmaf(w, v.y, O[2 * k + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < per) wo[lane * per + k] = O[k];
  if (lane == 0) {
    wm[warp] = M;
    wl[warp] = L;
  }
  __syncthreads();
  float Mt = -INFINITY;
#pragma unroll
  for (int w = 0; w < kMergeWideWarps; ++w) Mt = fmaxf(Mt, wm[w]);
  float Lt = 0.f;
#pragma unroll
  for (int w = 0; w < kMergeWideWarps; ++w)
    if (wm[w] != -INFINITY) Lt += exp2f(wm[w] - Mt) * wl[w];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWideWarps; ++w)
      if (wm[w] != -INFINITY) v += exp2f(wm[w] - Mt) * sw[w * D + i];
    const float ov = v * a.oscale;
    if (a.o_out) a.o_out[(int64_t)row * D + i] = ov;
    orow[i] = Lt > 0.f ? ov / Lt : 0.f;
  }
  if (a.o_out && threadIdx.x == 0) {
    a.m_out[row] = Mt;
    a.l_out[row] = Lt;
  }
  if (!a.out) return;
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float acc[1] = {a.R ? 0.f : orow[i]};
    if (a.R) mat_col<1>(a.R, D, i, orow, acc);
    store_any(a.out, a.out_dtype, (int64_t)row * D + i, acc[0]);
  }
}

template <int W>
static void launch_merge_w(const MergeDev& d, cudaStream_t s) {
  const int blocks = (d.n_rows + W - 1) / W;
  const size_t smem = (size_t)W * d.D * sizeof(float);
  launch_pdl(k_merge<W>, dim3(blocks), dim3(W * 32), smem, s, d);
  LC_CUDA(cudaGetLastError());
}

static void launch_merge_dev(const MergeDev& d, cudaStream_t s) {
  if (!d.wait_flags && d.max_slots > 64) {  // few rows of many slots: a block per row
    const size_t smem = ((size_t)kMergeWideWarps * d.D + 2 * kMergeWideWarps + d.D) * sizeof(float);
    launch_pdl(k_merge_wide, dim3((unsigned)d.n_rows), dim3(kMergeWideWarps * 32), smem, s, d);
    return;
  }
  if (d.D >= 256) launch_merge_w<4>(d, s);
  else launch_merge_w<8>(d, s);
}

void launch_merge(const float* part, const int32_t* cnt, int32_t G, int32_t max_slots, int32_t n_rows, int32_t dim,
                  const float* R, void* out, int32_t out_dtype, float* m_out, float* l_out, float* o_out,
                  float oscale, cudaStream_t s) {
  if (n_rows <= 0) return;
  MergeDev d{part, nullptr, nullptr, nullptr, cnt, G, max_slots, n_rows, dim, oscale, R, out, out_dtype, m_out, l_out,
             o_out, 0, nullptr, 0, 0u, nullptr};
  launch_merge_dev(d, s);
}

void launch_merge_parts(const float* m, const float* l, const float* o, int32_t n_parts, int32_t n_rows, int32_t dim,
                        const float* R, void* out, int32_t out_dtype, cudaStream_t s) {
  if (n_rows <= 0) return;
  MergeDev d{nullptr, m, l, o, nullptr, 1, n_parts, n_rows, dim, 1.0f, R, out, out_dtype, nullptr, nullptr, nullptr,
             0, nullptr, 0, 0u, nullptr};
  launch_merge_dev(d, s);
}

void launch_merge_split(const SplitCall& x, int32_t D, const float* R, void* out, int32_t out_dtype,
                        cudaStream_t s) {
  MergeDev d{nullptr, x.parts, x.parts + x.rows, x.parts + 2 * (int64_t)x.rows, nullptr, 1, x.world, x.rows, D, 1.0f,
             R, out, out_dtype, nullptr, nullptr, nullptr, x.block_stride, x.wait_flags, x.wait_n, x.epoch,
             x.status};
  launch_merge_dev(d, s);
}

}  // namespace lc
