// Quantize-on-append, strict mode: one fused kernel that rotates, normalises,
// quantizes, packs and (optionally) computes the QJL stage-2 bits of every
// appended K/V vector and writes them into the cache pages.
//
// Bit-identical to the reference CPU compressor
// (crates/lumen-core/src/compressor.rs:61-107): every f32 operation is an
// explicit round-to-nearest intrinsic (__fmul_rn/__fadd_rn/__fsub_rn/
// __fdiv_rn/__fsqrt_rn, never contracted into an FMA) and every sum runs in
// the reference's order:
//   rotated[i]   = sum_j R[i][j] * x[j]            j ascending (rotation.rs:91-99)
//   norm_sq      = sum_i rotated[i]^2              i ascending (compressor.rs:70)
//   scale        = sqrt(norm_sq / d)                            (:71)
//   code[i]      = #{k : !(rotated[i]*inv < t_k)}               (lloyd_max.rs:132-143)
//   recon[i]     = sum_j R[j][i] * (c[code_j]*scale) j ascending (rotation.rs:102-113)
//   rnorm        = sqrt(sum_i (x[i]-recon[i])^2)                (compressor.rs:87-93)
//   qjl bit r    = (sum_j Phi[r][j] * res[j]) >= 0              (qjl.rs:57-74)
// The f64 boundary compare is replaced by an f32 compare against
// t_k = the smallest f32 >= boundary_k, which gives the same answer for every
// f32 input (x < b <=> x < t_k; NaN falls through to the top code).
//
// Work split: a CTA of `dim` threads handles kNB vectors at a time; thread i
// owns output coordinate i of all kNB vectors (kNB independent dependency
// chains per thread), the per-vector sequential norms run one vector per
// thread. The path is bound by FP32 issue (about 2*d^2 + m*d non-fused
// multiply/add pairs per vector), not by HBM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "kernels.h"

namespace lc {

namespace {

constexpr int kNB = 8;  // vectors per CTA pass
// Appends of at most this many vectors per side take the warp-per-vector
// kernel (latency-bound decode steps); larger ones the table-in-smem kernel.
constexpr int64_t kSmallAppend = 16384;

struct AppendDev {
  CodecDev codec[2];
  const void* src[2];
  int32_t dtype, n_seqs, h_in, h_base;
  int64_t n_tok;
  const uint64_t* dst_page;  // or null: the inline copies below
  const int32_t* dst_row;
  int32_t heads;
  int64_t off[kMaxRoles];
  int64_t row[kMaxRoles];
  int32_t role_words[2], role_sigma[2], role_qjl[2], role_rnorm[2];
  // RoPE on the K side (lc_append_rope), see AppendArgs
  const float* rope_cs;
  int32_t rope_half, rope_traditional;
  // decode-step queries rotated in the same launch (grid row 2), see AppendArgs
  const void* q;
  int32_t q_dtype, q_rows;
  float* q_out;
  // small calls (decode steps): destinations in the launch parameters
  uint64_t ipage[kAppendInline];
  int32_t irow[kAppendInline];
  __device__ __forceinline__ uint64_t page_of(int64_t slot) const { return dst_page ? dst_page[slot] : ipage[slot]; }
  __device__ __forceinline__ int32_t row_of(int64_t slot) const { return dst_page ? dst_row[slot] : irow[slot]; }
};

// RoPE pair i of vector slot `slot` (sequence s, token t: slot = s * n_tok + t)
// in place: (x0, x1) -> (x0 c - x1 s, x0 s + x1 c), f32 round-to-nearest ops
// in that order; pairs (i, i + half) or, traditional, (2i, 2i + 1).
__device__ __forceinline__ void rope_pair(float* x, const AppendDev& a, int64_t slot, int i) {
  const int i0 = a.rope_traditional ? 2 * i : i;
  const int i1 = a.rope_traditional ? 2 * i + 1 : i + a.rope_half;
  const float* e = a.rope_cs + (slot * a.rope_half + i) * 2;
  const float c = e[0], sn = e[1];
  const float x0 = x[i0], x1 = x[i1];
  x[i0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
  x[i1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
}

__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t i) {
  if (dtype == LC_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == LC_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// x[v] = element idx[v] of an f32 / bf16 / f16 array where ok[v] (else 0);
// the dtype branch is taken once, so all N loads are in flight together.
template <int N>
__device__ __forceinline__ void load_n_elem(const void* p, int dtype, const int64_t (&idx)[N], const bool (&ok)[N],
                                            float (&x)[N]) {
  if (dtype == LC_F32) {
    const float* q = static_cast<const float*>(p);
#pragma unroll
    for (int v = 0; v < N; ++v) x[v] = ok[v] ? q[idx[v]] : 0.0f;
  } else {
    const unsigned short* q = static_cast<const unsigned short*>(p);
    unsigned short r[N];
#pragma unroll
    for (int v = 0; v < N; ++v) r[v] = ok[v] ? q[idx[v]] : (unsigned short)0;
#pragma unroll
    for (int v = 0; v < N; ++v)
      x[v] = dtype == LC_BF16 ? __uint_as_float((uint32_t)r[v] << 16) : __half2float(__ushort_as_half(r[v]));
  }
}

// acc[v] = fl(fl(acc[v] + fl(M[j][i] x_v[j])) ...) over j = 0 .. D-1 in order
// (round-to-nearest f32 products and sums, no contraction), M row-major with
// row stride ld, x_v = xs + v * D. Four j per step: x rows are read as float4.
template <int NB>
__device__ __forceinline__ void seq_matvec(const float* M, int ld, const float* xs, int D, int i, float (&acc)[NB]) {
#pragma unroll 2
  for (int j = 0; j < D; j += 4) {
    const float r0 = M[j * ld + i], r1 = M[(j + 1) * ld + i], r2 = M[(j + 2) * ld + i], r3 = M[(j + 3) * ld + i];
#pragma unroll
    for (int v = 0; v < NB; ++v) {
      const float4 x = *reinterpret_cast<const float4*>(xs + v * D + j);
      acc[v] = __fadd_rn(acc[v], __fmul_rn(r0, x.x));
      acc[v] = __fadd_rn(acc[v], __fmul_rn(r1, x.y));
      acc[v] = __fadd_rn(acc[v], __fmul_rn(r2, x.z));
      acc[v] = __fadd_rn(acc[v], __fmul_rn(r3, x.w));
    }
  }
}

// Shared memory of the batched kernel, per group: xs, ys, rs [kNB][D],
// vscale, vinv, vrn [kNB], qbits, codes.
struct GroupBufs {
  float *xs, *ys, *rs, *vscale, *vinv, *vrn;
  uint32_t* qbits;
  uint8_t* codes;
};

__device__ __forceinline__ size_t group_bytes(int D, int qw32) {
  return (size_t)(3 * kNB * D + 3 * kNB) * 4 + (size_t)kNB * (qw32 > 0 ? qw32 : 1) * 4 + (size_t)kNB * D;
}

// The codec tables (R^T; R and Phi^T for stage 2) are read through L1: one
// cached copy serves every CTA on the SM, so more CTAs fit than with a copy
// in each CTA's shared memory (397 M against 361 M vectors/s at d = 128).
__global__ void k_append_strict(const __grid_constant__ AppendDev a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int side = blockIdx.y;
  const CodecDev c = a.codec[side];
  const int D = c.dim;
  const int M = c.m;
  const bool stage2 = a.role_qjl[side] >= 0;
  const int grp = threadIdx.x / D;  // vector group inside the CTA
  const int i = threadIdx.x % D;    // output coordinate
  const int qw32 = (M + 31) / 32;
  const float* RT = c.RT;
  const float* R = c.R;
  const float* PT = c.PT;
  const size_t off = 0;
  uint8_t* gb = smem + off + group_bytes(D, qw32) * grp;
  float* xs = reinterpret_cast<float*>(gb);  // [kNB][D]
  float* ys = xs + kNB * D;                  // rotated, then dequantized*scale
  float* rs = ys + kNB * D;                  // residual
  float* vscale = rs + kNB * D;
  float* vinv = vscale + kNB;
  float* vrn = vinv + kNB;
  uint32_t* qbits = reinterpret_cast<uint32_t*>(vrn + kNB);                           // [kNB][qw32]
  uint8_t* codes = reinterpret_cast<uint8_t*>(qbits + kNB * (qw32 > 0 ? qw32 : 1));  // [kNB][D]

  const int64_t n_vec = (int64_t)a.n_seqs * a.h_in * a.n_tok;
  const void* src = a.src[side];
  const int groups = blockDim.x / D;
  // thresholds and centroids (bits <= 8) for the code search
  __shared__ float sthr[256], scent[256];
  for (int k = threadIdx.x; k < c.n_levels - 1; k += blockDim.x) sthr[k] = c.thr[k];
  for (int k = threadIdx.x; k < c.n_levels; k += blockDim.x) scent[k] = c.cent[k];
  __syncthreads();

  for (int64_t base = (int64_t)blockIdx.x * groups * kNB; base < n_vec; base += (int64_t)gridDim.x * groups * kNB) {
    const int64_t v0 = base + (int64_t)grp * kNB;
    const int nb = v0 < n_vec ? (int)(n_vec - v0 < kNB ? n_vec - v0 : kNB) : 0;
    // ---- load the batch (input layout [n_seqs][h_in][n_tok][D]) ----
    {
      int64_t idx[kNB];
      bool ok[kNB];
      float xv[kNB];
#pragma unroll
      for (int v = 0; v < kNB; ++v) {
        idx[v] = (v0 + v) * D + i;
        ok[v] = v < nb;
      }
      load_n_elem(src, a.dtype, idx, ok, xv);
#pragma unroll
      for (int v = 0; v < kNB; ++v) xs[v * D + i] = xv[v];
    }
    __syncthreads();
    if (side == 0 && a.rope_cs) {  // thread i rotates pair i of every vector
      if (i < a.rope_half)
        for (int v = 0; v < nb; ++v) {
          const int64_t vi = v0 + v;  // (s, hl, t) over [n_seqs][h_in][n_tok]
          const int64_t slot = (vi / ((int64_t)a.h_in * a.n_tok)) * a.n_tok + vi % a.n_tok;
          rope_pair(xs + v * D, a, slot, i);
        }
      __syncthreads();
    }

    // ---- rotated[i] = sum_j R[i][j] * x[j] (rotation.rs:91-99) ----
    float acc[kNB];
#pragma unroll
    for (int v = 0; v < kNB; ++v) acc[v] = -0.0f;
    seq_matvec(RT, D, xs, D, i, acc);
#pragma unroll
    for (int v = 0; v < kNB; ++v) ys[v * D + i] = acc[v];
    __syncthreads();

    // ---- scale = sqrt(norm_sq / d), one vector per thread (compressor.rs:70-71) ----
    if (i < kNB) {
      float s = -0.0f;
      for (int k = 0; k < D; ++k) {
        const float y = ys[i * D + k];
        s = __fadd_rn(s, __fmul_rn(y, y));
      }
      const float sc = __fsqrt_rn(__fdiv_rn(s, (float)D));
      vscale[i] = sc;
      vinv[i] = __fdiv_rn(1.0f, sc);
    }
    __syncthreads();

    // ---- codes and dequantized*scale (compressor.rs:73-83) ----
#pragma unroll
    for (int v = 0; v < kNB; ++v) {
      const float sc = vscale[v];
      int code = 0;
      if (!(sc < 1e-10f)) {
        // the count of thresholds t with !(yn < t) (lloyd_max.rs:132-143's
        // linear scan) by binary search: the thresholds ascend, so that
        // predicate holds on a prefix of them (on all of them for NaN)
        const float yn = __fmul_rn(ys[v * D + i], vinv[v]);
        for (int step = c.n_levels >> 1; step > 0; step >>= 1)
          if (!(yn < sthr[code + step - 1])) code += step;
      }
      codes[v * D + i] = (uint8_t)code;
      ys[v * D + i] = __fmul_rn(scent[code], sc);
    }
    __syncthreads();

    if (stage2) {
      // ---- recon[i] = sum_j R[j][i] * deq[j] (rotation.rs:102-113), residual ----
#pragma unroll
      for (int v = 0; v < kNB; ++v) acc[v] = 0.0f;
      seq_matvec(R, D, ys, D, i, acc);
#pragma unroll
      for (int v = 0; v < kNB; ++v) rs[v * D + i] = __fsub_rn(xs[v * D + i], acc[v]);
      __syncthreads();
      // ---- residual norm (compressor.rs:88-93) ----
      if (i < kNB) {
        float s = 0.0f;
        for (int k = 0; k < D; ++k) {
          const float r = rs[i * D + k];
          s = __fadd_rn(s, __fmul_rn(r, r));
        }
        vrn[i] = __fsqrt_rn(s);
      }
      // ---- QJL sign bits (qjl.rs:57-74) ----
      for (int rbase = 0; rbase < M; rbase += D) {
        const int r = rbase + i;
        float dot[kNB];
#pragma unroll
        for (int v = 0; v < kNB; ++v) dot[v] = -0.0f;
        if (r < M) seq_matvec(PT, M, rs, D, r, dot);
        for (int v = 0; v < kNB; ++v) {
          const bool bit = r < M && dot[v] >= 0.0f;
          const unsigned bal = __ballot_sync(0xffffffffu, bit);
          if ((i & 31) == 0) {
            const int wi = r >> 5;
            if (wi < qw32) qbits[v * qw32 + wi] = bal;
          }
        }
      }
    }
    __syncthreads();

    // ---- pack and write (bitpack.rs:17-30) ----
    const int cpw = 64 / c.bits;
    const int W = c.words;
    for (int u = i; u < nb * W; u += D) {
      const int v = u / W, w = u % W;
      uint64_t word = 0;
      for (int k = 0; k < cpw; ++k) {
        const int idx = w * cpw + k;
        if (idx < D) word |= (uint64_t)codes[v * D + idx] << (k * c.bits);
      }
      const int64_t g = v0 + v;
      const int64_t t = g % a.n_tok;
      const int64_t sh = g / a.n_tok;
      const int hl = (int)(sh % a.h_in);
      const int64_t s = sh / a.h_in;
      const int64_t slot = s * a.n_tok + t;
      uint8_t* page = reinterpret_cast<uint8_t*>(a.page_of(slot));
      const int64_t hr = (int64_t)(a.h_base + hl) * kPageTokens + a.row_of(slot);
      const int rw = a.role_words[side];
      reinterpret_cast<uint64_t*>(page + a.off[rw] + hr * a.row[rw])[w] = word;
    }
    for (int v = i; v < nb; v += D) {
      const int64_t g = v0 + v;
      const int64_t t = g % a.n_tok;
      const int64_t sh = g / a.n_tok;
      const int hl = (int)(sh % a.h_in);
      const int64_t s = sh / a.h_in;
      const int64_t slot = s * a.n_tok + t;
      uint8_t* page = reinterpret_cast<uint8_t*>(a.page_of(slot));
      const int64_t hr = (int64_t)(a.h_base + hl) * kPageTokens + a.row_of(slot);
      const int rsg = a.role_sigma[side];
      *reinterpret_cast<float*>(page + a.off[rsg] + hr * a.row[rsg]) = vscale[v];
      if (stage2) {
        const int rq = a.role_qjl[side], rr = a.role_rnorm[side];
        uint64_t* qdst = reinterpret_cast<uint64_t*>(page + a.off[rq] + hr * a.row[rq]);
        for (int w = 0; w < c.qwords; ++w) {
          const uint64_t lo = 2 * w < qw32 ? qbits[v * qw32 + 2 * w] : 0u;
          const uint64_t hi = 2 * w + 1 < qw32 ? qbits[v * qw32 + 2 * w + 1] : 0u;
          qdst[w] = lo | (hi << 32);
        }
        *reinterpret_cast<float*>(page + a.off[rr] + hr * a.row[rr]) = vrn[v];
      }
    }
    __syncthreads();
  }
}

// Small appends (decode steps: a few hundred vectors): one warp per vector so
// every vector's chains run concurrently, kWarpVecs vectors per CTA sharing the
// tables staged once in shared memory (TAB) or read through L1. Lane l owns
// outputs l, l+32, ...; sequential sums of squares are formed as exact
// products in parallel and added in order by lane 0 (the same f32 result
// as the reference's fold). Operation order as k_append_strict.
constexpr int kWarpVecs = 4;
constexpr int kQRows = 3;  // decode-step query rows per warp (grid row 2)
constexpr int kRtChunk = 32;  // rows of R^T per shared-memory chunk when R^T does not fit

__device__ __forceinline__ float seq_sum(const float* v, int n, float init) {
  float s = init;
#pragma unroll 8
  for (int k = 0; k < n; ++k) s = __fadd_rn(s, v[k]);
  return s;
}

// seq_sum over n (a multiple of 4) floats on a 16-byte boundary: the same
// ascending order, with the loads as 16-byte vectors issued ahead of the adds
__device__ __forceinline__ float seq_sum4(const float* v, int n, float init) {
  const float4* v4 = reinterpret_cast<const float4*>(v);
  float s = init;
#pragma unroll 8
  for (int k = 0; k < n / 4; ++k) {
    const float4 q = v4[k];
    s = __fadd_rn(s, q.x);
    s = __fadd_rn(s, q.y);
    s = __fadd_rn(s, q.z);
    s = __fadd_rn(s, q.w);
  }
  return s;
}

// the code of yn: the count of ascending thresholds t with !(yn < t)
// (lloyd_max.rs:132-143), by a binary search of log2(L) steps
template <int L>
__device__ __forceinline__ int tile_code(float yn, const float* thr) {
  int code = 0;
#pragma unroll
  for (int step = L >> 1; step > 0; step >>= 1)
    if (!(yn < thr[code + step - 1])) code += step;
  return code;
}
__device__ __forceinline__ int level_code(float yn, const float* thr, int n_levels) {
  switch (n_levels) {
    case 16: return tile_code<16>(yn, thr);
    case 8: return tile_code<8>(yn, thr);
    case 4: return tile_code<4>(yn, thr);
    default: {
      int code = 0;
      for (int step = n_levels >> 1; step > 0; step >>= 1)
        if (!(yn < thr[code + step - 1])) code += step;
      return code;
    }
  }
}

// n16 16-byte chunks global -> shared with cp.async, issued without waiting.
__device__ __forceinline__ void stage16(void* dst, const void* src, int n16) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const char* g = static_cast<const char*>(src);
  for (int k = threadIdx.x; k < n16; k += blockDim.x)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d + k * 16), "l"(g + (size_t)k * 16) : "memory");
}

// Programmatic dependent launch (sm_90+): see launch_warp_append. Both are
// no-ops for a kernel launched without the programmatic-serialization
// attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int R, bool TAB>  // R = head_dim / 32
__global__ void __launch_bounds__(kWarpVecs * 32, 1) k_append_warp(const __grid_constant__ AppendDev a) {
  constexpr int D = 32 * R;
  pdl_launch_dependents();
  extern __shared__ __align__(16) uint8_t smem[];
  const int side = blockIdx.y;  // 0 K, 1 V, 2 the step's queries (K's rotation)
  const int cs = side == 1 ? 1 : 0;
  const CodecDev& c = a.codec[cs];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool stage2 = a.role_qjl[cs] >= 0;
  const int M = c.m;
  const int n1 = c.n_levels - 1;
  // ---- shared: [thr 256][cent 256][per warp: x, y, r (D each), sq 16 u32, codes D][tables] ----
  float* sthr = reinterpret_cast<float*>(smem);
  float* scent = sthr + 256;
  uint8_t* wb = smem + 2048 + (size_t)warp * (3 * D * 4 + 64 + D);
  float* x = reinterpret_cast<float*>(wb);
  float* y = x + D;
  float* res = y + D;
  uint32_t* sq = reinterpret_cast<uint32_t*>(res + D);
  uint8_t* scode = reinterpret_cast<uint8_t*>(sq + 16);
  const float* RT = c.RT;
  const float* Rm = c.R;
  const float* PT = c.PT;
  {
    float* tab = reinterpret_cast<float*>(smem + 2048 + (size_t)kWarpVecs * (3 * D * 4 + 64 + D));
    for (int k = threadIdx.x; k < n1; k += blockDim.x) sthr[k] = c.thr[k];
    for (int k = threadIdx.x; k <= n1; k += blockDim.x) scent[k] = c.cent[k];
    if (TAB) {
      // all table copies in flight at once: one L2 round trip
      stage16(tab, c.RT, D * D / 4);
      RT = tab;
      if (stage2) {
        float* tr = tab + D * D;
        float* tp = tr + D * D;
        stage16(tr, c.R, D * D / 4);
        stage16(tp, c.PT, D * M / 4);
        Rm = tr;
        PT = tp;
      }
      asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
    }
  }
  // the tables above are the codecs' constants; the inputs and the pages
  // written below may belong to the previous kernel of the stream
  pdl_wait();
  __syncthreads();
  if (TAB && side == 2) {
    // q'[i] = sum_j R[i][j] q[j] for kQRows query rows per warp (plain f32
    // FMAs: the decode scores are not bit-exact work), rows in the warp's
    // x, y and res buffers, R^T from the staged table
    const int64_t r0 = ((int64_t)blockIdx.x * kWarpVecs + warp) * kQRows;
    float* rows[kQRows] = {x, y, res};
    bool live[kQRows];
#pragma unroll
    for (int k = 0; k < kQRows; ++k) {
      live[k] = r0 + k < a.q_rows;
      if (live[k]) {
#pragma unroll
        for (int r = 0; r < R; ++r) rows[k][lane + 32 * r] = load_elem(a.q, a.q_dtype, (r0 + k) * D + lane + 32 * r);
      }
    }
    __syncwarp();
    float qa[kQRows][R];
#pragma unroll
    for (int k = 0; k < kQRows; ++k)
#pragma unroll
      for (int r = 0; r < R; ++r) qa[k][r] = 0.f;
    // lane l owns outputs R l .. R l + R - 1 (d 64 / 128): one vector load
    // of R^T[j][R l ..] per j
    constexpr bool kQContig = R == 2 || R == 4;
#pragma unroll 4
    for (int j = 0; j < D; ++j) {
      float w[R];
      if constexpr (R == 4) {
        const float4 q = *reinterpret_cast<const float4*>(RT + j * D + 4 * lane);
        w[0] = q.x;
        w[1] = q.y;
        w[2] = q.z;
        w[3] = q.w;
      } else if constexpr (R == 2) {
        const float2 q = *reinterpret_cast<const float2*>(RT + j * D + 2 * lane);
        w[0] = q.x;
        w[1] = q.y;
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) w[r] = RT[j * D + lane + 32 * r];
      }
#pragma unroll
      for (int k = 0; k < kQRows; ++k) {
        const float qj = rows[k][j];
#pragma unroll
        for (int r = 0; r < R; ++r) qa[k][r] = fmaf(w[r], qj, qa[k][r]);
      }
    }
#pragma unroll
    for (int k = 0; k < kQRows; ++k)
      if (live[k]) {
#pragma unroll
        for (int r = 0; r < R; ++r) a.q_out[(r0 + k) * D + (kQContig ? R * lane + r : lane + 32 * r)] = qa[k][r];
      }
    return;  // TAB: no block-wide barrier after this point
  }
  if (!TAB && side == 2) {
    // the step's query rows with R^T streamed through shared memory in
    // chunks of kRtChunk rows (head_dim 256: R^T does not fit); plain f32
    // FMAs as in the staged case, outputs lane + 32 r
    const int64_t r0 = ((int64_t)blockIdx.x * kWarpVecs + warp) * kQRows;
    float* rows[kQRows] = {x, y, res};
    bool live[kQRows];
#pragma unroll
    for (int k = 0; k < kQRows; ++k) {
      live[k] = r0 + k < a.q_rows;
      if (live[k]) {
#pragma unroll
        for (int r = 0; r < R; ++r) rows[k][lane + 32 * r] = load_elem(a.q, a.q_dtype, (r0 + k) * D + lane + 32 * r);
      }
    }
    __syncwarp();
    float qa[kQRows][R];
#pragma unroll
    for (int k = 0; k < kQRows; ++k)
#pragma unroll
      for (int r = 0; r < R; ++r) qa[k][r] = 0.f;
    float* rbuf = reinterpret_cast<float*>(smem + 2048 + (size_t)kWarpVecs * (3 * D * 4 + 64 + D));
    constexpr int NC = D / kRtChunk;
    stage16(rbuf, c.RT, kRtChunk * D / 4);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int ch = 0; ch < NC; ++ch) {
      if (ch + 1 < NC) {
        stage16(rbuf + ((ch + 1) & 1) * kRtChunk * D, c.RT + (size_t)(ch + 1) * kRtChunk * D, kRtChunk * D / 4);
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;\n" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      }
      __syncthreads();
      const float* rt = rbuf + (ch & 1) * kRtChunk * D;
#pragma unroll 4
      for (int jj = 0; jj < kRtChunk; ++jj) {
        float w[R];
#pragma unroll
        for (int r = 0; r < R; ++r) w[r] = rt[jj * D + lane + 32 * r];
#pragma unroll
        for (int k = 0; k < kQRows; ++k) {
          const float qj = rows[k][ch * kRtChunk + jj];
#pragma unroll
          for (int r = 0; r < R; ++r) qa[k][r] = fmaf(w[r], qj, qa[k][r]);
        }
      }
      __syncthreads();  // the buffer is read before it is refilled
    }
#pragma unroll
    for (int k = 0; k < kQRows; ++k)
      if (live[k]) {
#pragma unroll
        for (int r = 0; r < R; ++r) a.q_out[(r0 + k) * D + lane + 32 * r] = qa[k][r];
      }
    return;  // no block-wide barrier after this point
  }
  const int64_t n_vec = (int64_t)a.n_seqs * a.h_in * a.n_tok;
  const int64_t v = (int64_t)blockIdx.x * kWarpVecs + warp;
  const bool active = v < n_vec;
  if (TAB && !active) return;  // TAB: no block-wide barrier after this point
  const void* src = a.src[side];
  if (active) {
#pragma unroll
    for (int r = 0; r < R; ++r) x[lane + 32 * r] = load_elem(src, a.dtype, v * D + lane + 32 * r);
    __syncwarp();
    if (side == 0 && a.rope_cs) {
      const int64_t slot = (v / ((int64_t)a.h_in * a.n_tok)) * a.n_tok + v % a.n_tok;
      for (int i = lane; i < a.rope_half; i += 32) rope_pair(x, a, slot, i);
      __syncwarp();
    }
  }
  // ---- rotated[i] = sum_j R[i][j] x[j] (rotation.rs:91-99) ----
  // With the table staged (d 64 / 128) lane l owns the R consecutive outputs
  // R l .. R l + R - 1 and reads its coefficients R^T[j][R l ..] as one
  // vector load per j; otherwise outputs l, l + 32, ... Every output's sum
  // runs j ascending either way.
  constexpr bool kContig = TAB && (R == 2 || R == 4);
  auto own = [&](int r) { return kContig ? R * lane + r : lane + 32 * r; };
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = -0.0f;
  if constexpr (kContig) {
#pragma unroll 8
    for (int j = 0; j < D; j += 4) {
      const float4 x4 = *reinterpret_cast<const float4*>(x + j);
      const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float w[R];
        if constexpr (R == 4) {
          const float4 q = *reinterpret_cast<const float4*>(RT + (j + jj) * D + 4 * lane);
          w[0] = q.x;
          w[1] = q.y;
          w[2] = q.z;
          w[3] = q.w;
        } else {
          const float2 q = *reinterpret_cast<const float2*>(RT + (j + jj) * D + 2 * lane);
          w[0] = q.x;
          w[1] = q.y;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(w[r], xs[jj]));
      }
    }
  } else if constexpr (TAB) {
#pragma unroll 4
    for (int j = 0; j < D; ++j) {
      const float xj = x[j];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(RT[j * D + lane + 32 * r], xj));
    }
  } else {
    // R^T does not fit: the block streams it through shared memory in
    // chunks of kRtChunk rows (double-buffered cp.async), each chunk read
    // by all of the block's vectors; the sum over j keeps its order
    float* rbuf = reinterpret_cast<float*>(smem + 2048 + (size_t)kWarpVecs * (3 * D * 4 + 64 + D));
    constexpr int NC = D / kRtChunk;
    stage16(rbuf, c.RT, kRtChunk * D / 4);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int ch = 0; ch < NC; ++ch) {
      if (ch + 1 < NC) {
        stage16(rbuf + ((ch + 1) & 1) * kRtChunk * D, c.RT + (size_t)(ch + 1) * kRtChunk * D, kRtChunk * D / 4);
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;\n" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
      }
      __syncthreads();
      const float* rt = rbuf + (ch & 1) * kRtChunk * D;
      if (active) {
#pragma unroll 4
        for (int jj = 0; jj < kRtChunk; ++jj) {
          const float xj = x[ch * kRtChunk + jj];
#pragma unroll
          for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(rt[jj * D + lane + 32 * r], xj));
        }
      }
      __syncthreads();  // the buffer is read before it is refilled
    }
    if (!active) return;  // no block-wide barrier after this point
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    y[own(r)] = acc[r];
    res[own(r)] = __fmul_rn(acc[r], acc[r]);
  }
  __syncwarp();
  // ---- scale (compressor.rs:70-71) ----
  float sc = 0.f, inv = 0.f;
  if (lane == 0) {
    sc = __fsqrt_rn(__fdiv_rn(seq_sum4(res, D, -0.0f), (float)D));
    inv = __fdiv_rn(1.0f, sc);
  }
  sc = __shfl_sync(0xffffffffu, sc, 0);
  inv = __shfl_sync(0xffffffffu, inv, 0);
  // the count of thresholds with !(yn < t): a binary search over the
  // ascending thresholds gives the same count
  uint32_t chunk = 0;  // kContig: the lane's R codes, c.bits each
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = own(r);
    int code = 0;
    if (!(sc < 1e-10f)) code = level_code(__fmul_rn(acc[r], inv), sthr, n1 + 1);
    scode[i] = (uint8_t)code;
    if constexpr (kContig) chunk |= (uint32_t)code << (c.bits * r);  // r bits <= 24
    y[i] = __fmul_rn(scent[code], sc);
  }
  __syncwarp();
  float rn = 0.f;
  if (stage2) {
    // ---- recon[i] = sum_j R[j][i] deq[j] (rotation.rs:102-113), residual, norm ----
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll 4
    for (int j = 0; j < D; ++j) {
      const float yj = y[j];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fadd_rn(acc[r], __fmul_rn(Rm[j * D + lane + 32 * r], yj));
    }
    float rr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rr[r] = __fsub_rn(x[lane + 32 * r], acc[r]);
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      y[lane + 32 * r] = rr[r];                       // residual
      res[lane + 32 * r] = __fmul_rn(rr[r], rr[r]);   // its squares
    }
    __syncwarp();
    if (lane == 0) rn = __fsqrt_rn(seq_sum(res, D, 0.0f));
    // ---- QJL sign bits (qjl.rs:57-74) ----
    for (int rb = 0; rb < M; rb += 32) {
      const int row = rb + lane;
      bool bit = false;
      if (row < M) {
        float dot = -0.0f;
#pragma unroll 4
        for (int j = 0; j < D; ++j) dot = __fadd_rn(dot, __fmul_rn(PT[j * M + row], y[j]));
        bit = dot >= 0.0f;
      }
      const unsigned bal = __ballot_sync(0xffffffffu, bit);
      if (lane == 0 && (rb >> 5) < 16) sq[rb >> 5] = bal;
    }
  }
  __syncwarp();
  // ---- pack and write (bitpack.rs:17-30) ----
  const int64_t t = v % a.n_tok;
  const int64_t sh = v / a.n_tok;
  const int hl = (int)(sh % a.h_in);
  const int64_t s = sh / a.h_in;
  const int64_t slot = s * a.n_tok + t;
  uint8_t* page = reinterpret_cast<uint8_t*>(a.page_of(slot));
  const int64_t hr = (int64_t)(a.h_base + hl) * kPageTokens + a.row_of(slot);
  const int cpw = 64 / c.bits;
  const int rw = a.role_words[side];
  uint64_t* wdst = reinterpret_cast<uint64_t*>(page + a.off[rw] + hr * a.row[rw]);
  if (kContig && (c.bits & (c.bits - 1)) == 0 && R * c.bits <= 32) {
    // lanes own R consecutive codes: a word is the chunks of 64 / (R bits)
    // neighbouring lanes, OR-combined by shuffles
    const int lpw = 64 / (R * c.bits);
    uint64_t word = (uint64_t)chunk << (R * c.bits * (lane & (lpw - 1)));
    for (int o = 1; o < lpw; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
    if ((lane & (lpw - 1)) == 0) wdst[lane / lpw] = word;
  } else {
    for (int w = lane; w < c.words; w += 32) {
      uint64_t word = 0;
      for (int k = 0; k < cpw; ++k) {
        const int idx = w * cpw + k;
        if (idx < D) word |= (uint64_t)scode[idx] << (k * c.bits);
      }
      wdst[w] = word;
    }
  }
  if (lane == 0) {
    const int rsg = a.role_sigma[side];
    *reinterpret_cast<float*>(page + a.off[rsg] + hr * a.row[rsg]) = sc;
    if (stage2) {
      const int rq = a.role_qjl[side], rrl = a.role_rnorm[side];
      uint64_t* qdst = reinterpret_cast<uint64_t*>(page + a.off[rq] + hr * a.row[rq]);
      const int qw32 = (M + 31) / 32;
      for (int w = 0; w < c.qwords; ++w) {
        const uint64_t lo = 2 * w < qw32 ? sq[2 * w] : 0u;
        const uint64_t hi = 2 * w + 1 < qw32 ? sq[2 * w + 1] : 0u;
        qdst[w] = lo | (hi << 32);
      }
      *reinterpret_cast<float*>(page + a.off[rrl] + hr * a.row[rrl]) = rn;
    }
  }
}

template <int R>
void launch_warp_append(const AppendDev& d, bool stage2, int M, int64_t n_vec, cudaStream_t s) {
  constexpr int D = 32 * R;
  const size_t base = 2048 + (size_t)kWarpVecs * (3 * D * 4 + 64 + D);
  const size_t tables = (size_t)D * D * 4 + (stage2 ? (size_t)(D * D + D * M) * 4 : 0);
  const bool tab = base + tables <= 200 * 1024;
  const size_t smem = base + (tab ? tables : (size_t)2 * kRtChunk * D * 4);
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_append_warp<R, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    LC_CUDA(cudaFuncSetAttribute(k_append_warp<R, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr = true;
  }
  // Programmatic serialization: the table staging overlaps the previous
  // kernel's tail (the kernel waits for it before touching inputs or pages).
  cudaLaunchConfig_t cfg = {};
  int64_t gx = (n_vec + kWarpVecs - 1) / kWarpVecs;
  if (d.q) gx = std::max<int64_t>(gx, (d.q_rows + kWarpVecs * kQRows - 1) / (kWarpVecs * kQRows));
  cfg.gridDim = dim3((unsigned)gx, d.q ? 3 : 2);
  cfg.blockDim = dim3(kWarpVecs * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (tab) LC_CUDA(cudaLaunchKernelEx(&cfg, k_append_warp<R, true>, d));
  else LC_CUDA(cudaLaunchKernelEx(&cfg, k_append_warp<R, false>, d));
}

// Large appends without QJL stage 2 at head_dim 64 / 128: a warp takes
// kTileVecs vectors at a time and lane l owns the R consecutive outputs
// R l .. R l + R - 1 of all of them (R = dim / 32). Per step j of the
// rotation's ascending sum a lane reads its R coefficients R^T[j][R l ..] as
// one vector load and each vector's x[j] as a broadcast, so a lane keeps
// kTileVecs x R independent chains and the loads are ~5 % of the f32 work
// (the batched kernel above reads one coefficient per output and chain).
// The sums run as paired f32 adds (add.rn.f32x2 on sm_100: two IEEE
// round-to-nearest additions per lane and issue slot) over output pairs
// (2m, 2m + 1); the products stay scalar round-to-nearest multiplies, since
// a paired multiply feeding a paired add is contracted into a fused
// multiply-add by the code generator even with explicit rounding (measured:
// most sums then differ in the last bit). That is 3 issue slots per 2 terms
// instead of 4. Every f32 operation and sum order is the strict one: the rotation sums j ascending from -0, the squares are formed in
// parallel and added in order i ascending by one lane per vector (rows
// padded to d + 4 floats, so the lanes' 16-byte reads fall in distinct
// banks), the codes are the threshold count, so codes and sigma are
// bit-identical to k_append_strict.
constexpr int kTileWarps = 32, kTileVecs = 4;

// per warp: x [NV][D] f32, squares [NV][D + 4] f32, codes [NV][D] u8
template <int R>
__host__ __device__ constexpr size_t tile_warp_bytes() {
  constexpr int D = 32 * R;
  return (size_t)kTileVecs * D * 4 + (size_t)kTileVecs * (D + 4) * 4 + (size_t)kTileVecs * D;
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}

template <int R, int L>
__device__ __forceinline__ void tile_codes(const float (&acc)[kTileVecs][R], const float* sc, const float* inv,
                                           const float* thr, int n_levels, uint8_t* codes, int lane) {
#pragma unroll
  for (int v = 0; v < kTileVecs; ++v) {
    const float scv = __shfl_sync(0xffffffffu, *sc, v), invv = __shfl_sync(0xffffffffu, *inv, v);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      int code = 0;
      if (!(scv < 1e-10f)) {
        const float yn = __fmul_rn(acc[v][r], invv);
        if constexpr (L > 0) {
          code = tile_code<L>(yn, thr);
        } else {
          for (int step = n_levels >> 1; step > 0; step >>= 1)
            if (!(yn < thr[code + step - 1])) code += step;
        }
      }
      codes[v * (32 * R) + R * lane + r] = (uint8_t)code;
    }
  }
}

template <int R>
__global__ void __launch_bounds__(kTileWarps * 32, 1) k_append_tile(const __grid_constant__ AppendDev a) {
  constexpr int D = 32 * R;
  constexpr int NV = kTileVecs;
  extern __shared__ __align__(16) uint8_t smem[];
  const int side = blockIdx.y;
  const CodecDev& c = a.codec[side];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* rt = reinterpret_cast<float*>(smem);  // R^T [D][D]
  float* sthr = rt + D * D;                    // [256]
  uint8_t* wb = smem + (size_t)D * D * 4 + 1024 + (size_t)warp * tile_warp_bytes<R>();
  float* x = reinterpret_cast<float*>(wb);                  // [NV][D]
  float* sq = x + NV * D;                                   // [NV][D + 4] squares (rows padded: lane v reads row v)
  uint8_t* codes = reinterpret_cast<uint8_t*>(sq + NV * (D + 4));  // [NV][D]
  stage16(rt, c.RT, D * D / 4);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
  for (int k = threadIdx.x; k < c.n_levels - 1; k += blockDim.x) sthr[k] = c.thr[k];
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  __syncthreads();

  const int64_t n_vec = (int64_t)a.n_seqs * a.h_in * a.n_tok;
  const void* src = a.src[side];
  const int cpw = 64 / c.bits, W = c.words;
  const int rw = a.role_words[side], rsg = a.role_sigma[side];
  const bool rope = side == 0 && a.rope_cs;
  for (int64_t v0 = ((int64_t)blockIdx.x * kTileWarps + warp) * NV; v0 < n_vec;
       v0 += (int64_t)gridDim.x * kTileWarps * NV) {
    const int nv = (int)(n_vec - v0 < NV ? n_vec - v0 : NV);
    // ---- load (input layout [n_seqs][h_in][n_tok][D]): lane l's R
    // consecutive elements of each vector as one vector load ----
    float e[NV][R];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int64_t base = (v0 + v) * D + R * lane;
      if (v >= nv) {
#pragma unroll
        for (int r = 0; r < R; ++r) e[v][r] = 0.0f;
      } else if (a.dtype == LC_F32) {
        const float* q = static_cast<const float*>(src) + base;
        if constexpr (R == 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(q);
          e[v][0] = t4.x;
          e[v][1] = t4.y;
          e[v][2] = t4.z;
          e[v][3] = t4.w;
        } else {
          const float2 t2 = *reinterpret_cast<const float2*>(q);
          e[v][0] = t2.x;
          e[v][1] = t2.y;
        }
      } else {
        const unsigned short* q = static_cast<const unsigned short*>(src) + base;
        uint32_t h[R / 2];
        if constexpr (R == 4) {
          const uint2 t2 = *reinterpret_cast<const uint2*>(q);
          h[0] = t2.x;
          h[1] = t2.y;
        } else {
          h[0] = *reinterpret_cast<const uint32_t*>(q);
        }
#pragma unroll
        for (int k = 0; k < R / 2; ++k) {
          const uint32_t lo = h[k] & 0xFFFFu, hi = h[k] >> 16;
          e[v][2 * k] =
              a.dtype == LC_BF16 ? __uint_as_float(lo << 16) : __half2float(__ushort_as_half((unsigned short)lo));
          e[v][2 * k + 1] =
              a.dtype == LC_BF16 ? __uint_as_float(hi << 16) : __half2float(__ushort_as_half((unsigned short)hi));
        }
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int r = 0; r < R; ++r) x[v * D + R * lane + r] = e[v][r];
    __syncwarp();
    if (rope) {  // RoPE on K before quantisation (pairs cross lanes)
      for (int v = 0; v < nv; ++v) {
        const int64_t vi = v0 + v;
        const int64_t slot = (vi / ((int64_t)a.h_in * a.n_tok)) * a.n_tok + vi % a.n_tok;
        for (int i = lane; i < a.rope_half; i += 32) rope_pair(x + v * D, a, slot, i);
      }
      __syncwarp();
    }
    // ---- rotated[i] = sum_j R[i][j] x[j], j ascending (rotation.rs:91-99),
    // on output pairs (R l + 2m, R l + 2m + 1) ----
    constexpr int RP = R / 2;
    constexpr uint64_t kNegZero2 = 0x8000000080000000ull;
    uint64_t acc2[NV][RP];
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int m = 0; m < RP; ++m) acc2[v][m] = kNegZero2;
#pragma unroll 1
    for (int j = 0; j < D; j += 4) {
      uint64_t w[4][RP];  // (R^T[j + jj][R l + 2m], R^T[j + jj][R l + 2m + 1])
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        if constexpr (R == 4) {
          const ulonglong2 q = *reinterpret_cast<const ulonglong2*>(rt + (j + jj) * D + 4 * lane);
          w[jj][0] = q.x;
          w[jj][1] = q.y;
        } else {
          w[jj][0] = *reinterpret_cast<const unsigned long long*>(rt + (j + jj) * D + 2 * lane);
        }
      }
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const float4 x4 = *reinterpret_cast<const float4*>(x + v * D + j);
        const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
          for (int m = 0; m < RP; ++m) {
            const float p0 = __fmul_rn(__uint_as_float((uint32_t)w[jj][m]), xs[jj]);
            const float p1 = __fmul_rn(__uint_as_float((uint32_t)(w[jj][m] >> 32)), xs[jj]);
            acc2[v][m] = f2_add(acc2[v][m], f2_pack(p0, p1));
          }
      }
    }
    float acc[NV][R];
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int m = 0; m < RP; ++m) {
        acc[v][2 * m] = __uint_as_float((uint32_t)acc2[v][m]);
        acc[v][2 * m + 1] = __uint_as_float((uint32_t)(acc2[v][m] >> 32));
      }
    // ---- scale = sqrt(norm_sq / d): squares in parallel, lane v adds vector
    // v's in order (compressor.rs:70-71) ----
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int r = 0; r < R; ++r) sq[v * (D + 4) + R * lane + r] = __fmul_rn(acc[v][r], acc[v][r]);
    __syncwarp();
    float sc = 0.f, inv = 0.f;
    if (lane < nv) {
      const float4* row = reinterpret_cast<const float4*>(sq + lane * (D + 4));
      float s2 = -0.0f;
#pragma unroll 4
      for (int k = 0; k < D / 4; ++k) {
        const float4 q4 = row[k];
        s2 = __fadd_rn(s2, q4.x);
        s2 = __fadd_rn(s2, q4.y);
        s2 = __fadd_rn(s2, q4.z);
        s2 = __fadd_rn(s2, q4.w);
      }
      sc = __fsqrt_rn(__fdiv_rn(s2, (float)D));
      inv = __fdiv_rn(1.0f, sc);
    }
    // ---- codes: the count of thresholds t with !(yn < t) (lloyd_max.rs:132-143),
    // by binary search over the ascending thresholds ----
    switch (c.n_levels) {
      case 16: tile_codes<R, 16>(acc, &sc, &inv, sthr, 16, codes, lane); break;
      case 8: tile_codes<R, 8>(acc, &sc, &inv, sthr, 8, codes, lane); break;
      case 4: tile_codes<R, 4>(acc, &sc, &inv, sthr, 4, codes, lane); break;
      default: tile_codes<R, 0>(acc, &sc, &inv, sthr, c.n_levels, codes, lane); break;
    }
    __syncwarp();
    // ---- pack and write (bitpack.rs:17-30): lane v finds vector v's page
    // row, the word writers take it by shuffle ----
    uint64_t pg = 0;
    int64_t hr = 0;
    // (sequence, head, token) of v0: lane 0 divides, lane v steps v tokens on
    int64_t t = 0, sq_i = 0;
    int hl = 0;
    if (lane == 0) {
      const int64_t sh = v0 / a.n_tok;
      t = v0 - sh * a.n_tok;
      hl = (int)(sh % a.h_in);
      sq_i = sh / a.h_in;
    }
    t = __shfl_sync(0xffffffffu, t, 0);
    hl = __shfl_sync(0xffffffffu, hl, 0);
    sq_i = __shfl_sync(0xffffffffu, sq_i, 0);
    if (lane < nv) {
      t += lane;
      while (t >= a.n_tok) {
        t -= a.n_tok;
        if (++hl == a.h_in) {
          hl = 0;
          ++sq_i;
        }
      }
      const int64_t slot = sq_i * a.n_tok + t;
      pg = a.page_of(slot);
      hr = (int64_t)(a.h_base + hl) * kPageTokens + a.row_of(slot);
      *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(pg) + a.off[rsg] + hr * a.row[rsg]) = sc;
    }
    for (int u0 = 0; u0 < nv * W; u0 += 32) {
      const int u = u0 + lane;
      const int v = u / W, w = u - v * W;
      const uint64_t pv = __shfl_sync(0xffffffffu, pg, v < NV ? v : 0);
      const int64_t hv = __shfl_sync(0xffffffffu, hr, v < NV ? v : 0);
      if (u < nv * W) {
        uint64_t word = 0;
        for (int k = 0; k < cpw; ++k) {
          const int idx = w * cpw + k;
          if (idx < D) word |= (uint64_t)codes[v * D + idx] << (k * c.bits);
        }
        reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(pv) + a.off[rw] + hv * a.row[rw])[w] = word;
      }
    }
    __syncwarp();  // x, sq and codes are refilled by the next batch
  }
}

template <int R>
void launch_tile_append(const AppendDev& d, int64_t n_vec, cudaStream_t s) {
  constexpr int D = 32 * R;
  const size_t smem = (size_t)D * D * 4 + 1024 + (size_t)kTileWarps * tile_warp_bytes<R>();
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_append_tile<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  const int64_t batches = (n_vec + (int64_t)kTileWarps * kTileVecs - 1) / ((int64_t)kTileWarps * kTileVecs);
  const int64_t grid = std::min<int64_t>(batches, num_sms());
  k_append_tile<R><<<dim3((unsigned)grid, 2), kTileWarps * 32, smem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

}  // namespace

bool append_rotates_queries(int64_t n_vec, int dim, int m_max, bool stage2) {
  if (n_vec > kSmallAppend || m_max > 512) return false;
  if (dim == 256) return true;  // the warp kernel streaming R^T (its query rows stream it too)
  if (!(dim == 64 || dim == 128)) return false;
  const size_t base = 2048 + (size_t)kWarpVecs * (3 * dim * 4 + 64 + dim);
  const size_t tables = (size_t)dim * dim * 4 + (stage2 ? (size_t)(dim * dim + dim * m_max) * 4 : 0);
  return base + tables <= 200 * 1024;  // the warp kernel with R^T staged (TAB)
}

size_t append_smem_bytes(int d, int m) {
  const int qw32 = (m + 31) / 32;
  return (size_t)(3 * kNB * d + 3 * kNB) * 4 + (size_t)kNB * (qw32 > 0 ? qw32 : 1) * 4 + (size_t)kNB * d;
}

void launch_append(const AppendArgs& a, cudaStream_t s) {
  const int64_t n_vec = (int64_t)a.n_seqs * a.h_in * a.n_tok;
  if (n_vec <= 0) return;
  AppendDev d{};
  d.codec[0] = a.codec[0];
  d.codec[1] = a.codec[1];
  d.src[0] = a.src[0];
  d.src[1] = a.src[1];
  d.dtype = a.dtype;
  d.n_seqs = a.n_seqs;
  d.h_in = a.h_in;
  d.h_base = a.h_base;
  d.n_tok = a.n_tok;
  d.dst_page = a.dst_page;
  d.dst_row = a.dst_row;
  d.rope_cs = a.rope_cs;
  d.rope_half = a.rope_half;
  d.rope_traditional = a.rope_traditional;
  if (!a.dst_page) {
    const int64_t slots = (int64_t)a.n_seqs * a.n_tok;
    LC_REQUIRE(a.h_page && a.h_row && slots <= kAppendInline, LC_ERR_STATE, "inline append metadata does not fit");
    for (int64_t i = 0; i < slots; ++i) {
      d.ipage[i] = a.h_page[i];
      d.irow[i] = a.h_row[i];
    }
  }
  d.heads = a.layout.heads;
  for (int r = 0; r < kMaxRoles; ++r) {
    d.off[r] = a.layout.off[r];
    d.row[r] = a.layout.row[r];
  }
  bool stage2 = false;
  for (int k = 0; k < 2; ++k) {
    d.role_words[k] = a.role_words[k];
    d.role_sigma[k] = a.role_sigma[k];
    d.role_qjl[k] = a.role_qjl[k];
    d.role_rnorm[k] = a.role_rnorm[k];
    stage2 = stage2 || a.role_qjl[k] >= 0;
  }
  const int D = a.codec[0].dim;
  const int M = a.codec[0].m > a.codec[1].m ? a.codec[0].m : a.codec[1].m;
  if (a.q) {
    LC_REQUIRE(append_rotates_queries(n_vec, D, M, stage2), LC_ERR_STATE, "append cannot rotate these queries");
    d.q = a.q;
    d.q_dtype = a.q_dtype;
    d.q_rows = a.q_rows;
    d.q_out = a.q_out;
  }
  if (n_vec <= kSmallAppend && M <= 512 && (D == 64 || D == 128 || D == 256)) {
    if (D == 64) launch_warp_append<2>(d, stage2, M, n_vec, s);
    else if (D == 128) launch_warp_append<4>(d, stage2, M, n_vec, s);
    else launch_warp_append<8>(d, stage2, M, n_vec, s);
    return;
  }
  // the tile kernel reads each lane's elements as one vector load: the
  // inputs must sit on 16-byte (f32) / 8-byte (bf16, f16) boundaries
  const uintptr_t in_align = a.dtype == LC_F32 ? 16 : 8;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.src[0]) | reinterpret_cast<uintptr_t>(a.src[1])) % in_align) == 0;
  if (!stage2 && !a.q && aligned && (D == 64 || D == 128) && a.codec[0].bits <= 8 && a.codec[1].bits <= 8 &&
      a.codec[0].dim == a.codec[1].dim) {
    if (D == 64) launch_tile_append<2>(d, n_vec, s);
    else launch_tile_append<4>(d, n_vec, s);
    return;
  }
  const int groups = D <= 256 ? 2 : 1;
  const size_t smem = groups * append_smem_bytes(D, M);
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_append_strict, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024));
    attr = true;
  }
  LC_REQUIRE(smem <= 220 * 1024, LC_ERR_INVALID, "append: head_dim too large for the batched kernel");
  const int64_t batches = (n_vec + (int64_t)groups * kNB - 1) / ((int64_t)groups * kNB);
  const int64_t max_blocks = (int64_t)num_sms() * 4;
  dim3 grid((unsigned)(batches < max_blocks ? batches : max_blocks), 2);
  k_append_strict<<<grid, D * groups, smem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
