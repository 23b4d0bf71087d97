// Causal prefill attention over the compressed cache with K/V tile reuse: the
// masked SDPA of a prefill chunk (gemma4_moe.rs:4636-4660: queries against
// the dequantized codes, causal mask, scale) computed on the codes, on the
// tensor cores.
//
// Work: a CTA takes one kv head and a block of query tokens with all G query
// heads of each: 128 rows (token, head) = 8 warps x 16, so the tokens per CTA
// are 128 / G. It walks the keys the block can see in 64-key tiles. Each tile
// is staged packed (cp.async double buffer: K words, V words, sigma_K,
// sigma_V, as the page holds them), dequantized ONCE into shared memory as
// f16 [key][dim] tiles (K, and V), and then read by all 8 warps with ldmatrix
// into m16n8k16 MMAs, flash-attention style:
//   S (16 rows x 64 keys) = Q K^T, scaled per key by sigma_K, causal mask;
//   online softmax in log2 units (rows' running max and sum);
//   O (16 rows x 128 dims) += (P sigma_V) V.
// Precision: P sigma_V goes to the MMA as one f16 (relative 2^-11 per term,
// an output error far inside the decode tolerance). Queries are split into
// f16 hi + lo parts (two QK MMAs): a single f16 query moves scores by about
// 2^-11 ||q'|| sigma_K / sqrt(d), visible in the tolerance once sigma_K
// ||q'|| reaches ~10, as in any realistic attention. The K centroids are
// single f16 values (relative ~1e-4); on tiles where sigma_K x ||q'|| makes
// that visible (PrefillArgs::pthr, the decode kernels' criterion) the scores
// add Q (alpha c - f16(alpha c)) x 2^11 from a second, residual K tile.
//
// One launch: the block also rotates its query rows (R q on the tensor cores,
// f16 hi / lo splits of both operands) and normalises and un-rotates its
// output rows (V's R^T, the same way) before writing them.
//
// Traffic: each key tile is read from HBM once per (kv head, query block)
// and stays in L2 (the whole view of a 16K-token prefix is 17.8 MB for 8 kv
// heads), so DRAM traffic is about view x 136 B per kv head, not L x view.
// The roofline is the tensor pipe: two QK and one PV m16n8k16 MMA per
// (16 rows x 8 keys x 16 dims) on the common path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "devutil.cuh"
#include "kernels.h"

namespace lc {

namespace {

constexpr int kPfWarps = 8, kPfRows = 16 * kPfWarps;
constexpr int kPfKeys = 64, kPfD = 128;
constexpr int kPfRowB = 64;  // bytes of 4-bit codes per key row
// packed stage: K words [64][64 B] | V words [64][64 B] | sigma_K [64] | sigma_V [64]
constexpr int kPfStVw = kPfKeys * kPfRowB, kPfStKs = 2 * kPfKeys * kPfRowB, kPfStVs = kPfStKs + kPfKeys * 4;
constexpr int kPfStage = kPfStVs + kPfKeys * 4;  // 8704
constexpr int kPfTile = kPfKeys * kPfD * 2;      // f16 [64 keys][128 dims]: 16 KB
// shared memory from a 64 KiB-aligned base: the centroid-pair table (256
// bytes x 64 slots of u32: K in slots 0..15, K residuals in 16..31, V in
// 32..63), then the K, K-residual and V tiles and the two stages
constexpr int kPfLut = 65536;
constexpr int kPfOffK = kPfLut, kPfOffKl = kPfOffK + kPfTile, kPfOffV = kPfOffKl + kPfTile;
constexpr int kPfOffSt = kPfOffV + kPfTile;
constexpr int kPfUsed = kPfOffSt + 2 * kPfStage;
constexpr int kPfSmem = kPfUsed + 65536 - 128;  // room to align the table (the base is 128-aligned)
static_assert(kPfSmem <= 227 * 1024, "prefill shared memory");

// byte offset of (key, 16-byte chunk c) in an f16 [64][128] tile: chunks
// XOR-swizzled by key & 7 so ldmatrix rows and the dequant stores spread
// over all banks
__device__ __forceinline__ uint32_t pf_swz(int key, int c) { return key * 256 + ((c ^ (key & 7)) << 4); }

// Dequantizes the staged tile's K (slots `ks`), optionally its K residuals,
// and V into the f16 tiles: thread i takes u32 words i, i + 256, ... of each
// (8 dims of one key: four table lookups, one 16-byte store).
__device__ __forceinline__ void pf_dequant(const uint8_t* st, uint32_t lut_s, uint32_t k_s, uint32_t kl_s, uint32_t v_s,
                                           bool lo) {
  const int lane = threadIdx.x & 31;
  const uint32_t kb = lut_s | ((uint32_t)(lane & 15) << 2);
  const uint32_t klb = lut_s | ((uint32_t)(16 + (lane & 15)) << 2);
  const uint32_t vb = lut_s | ((uint32_t)(32 + lane) << 2);
  const uint32_t* kw = reinterpret_cast<const uint32_t*>(st);
  const uint32_t* vw = reinterpret_cast<const uint32_t*>(st + kPfStVw);
  auto look = [](uint32_t x, uint32_t base, uint32_t k) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(__byte_perm(x, base, 0x7604u | (k << 4))));
    return v;
  };
  auto st4 = [](uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
  };
#pragma unroll
  for (int j = 0; j < kPfKeys * 16 / (kPfWarps * 32); ++j) {
    const int w = threadIdx.x + j * kPfWarps * 32;
    const int key = w >> 4, c = w & 15;
    const uint32_t off = pf_swz(key, c);
    const uint32_t x = kw[w], y = vw[w];
    st4(k_s + off, look(x, kb, 0), look(x, kb, 1), look(x, kb, 2), look(x, kb, 3));
    if (lo) st4(kl_s + off, look(x, klb, 0), look(x, klb, 1), look(x, klb, 2), look(x, klb, 3));
    st4(v_s + off, look(y, vb, 0), look(y, vb, 1), look(y, vb, 2), look(y, vb, 3));
  }
}

__device__ __forceinline__ void pf_split(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 f = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(x - f.x, y - f.y));
}

constexpr float kPfLoScale = 2048.f, kPfLoUnscale = 1.f / 2048.f;
constexpr float kPfRotScale = 256.f, kPfRotUnscale = 1.f / 256.f;

template <int G>
__global__ void __launch_bounds__(kPfWarps * 32, 1) k_prefill_tiled(const __grid_constant__ PrefillArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_cent[32];
  __shared__ float s_qn[kPfWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix and row of this lane's address
  const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t lut_s = (s0 + 65535u) & ~65535u;
  uint8_t* base = smem + (lut_s - s0);
  const uint32_t k_s = lut_s + kPfOffK, kl_s = lut_s + kPfOffKl, v_s = lut_s + kPfOffV, st_s = lut_s + kPfOffSt;
  const uint8_t* stage0 = base + kPfOffSt;

  constexpr int TPC = kPfRows / G;  // query tokens per block
  const int nqb = (a.L + TPC - 1) / TPC;
  const int qb = nqb - 1 - (int)(blockIdx.x / a.hkv);  // the blocks with the most keys first
  const int kvh = (int)(blockIdx.x % a.hkv);
  const int tok0 = qb * TPC;
  const int ntok = min(TPC, a.L - tok0);
  const int64_t P0 = a.n_total - a.L;
  const int64_t n_keys = P0 + tok0 + ntok;  // keys the block's last token sees
  const int ntiles = (int)((n_keys + kPfKeys - 1) / kPfKeys);

  // K / V packed tile kt (64 keys, a quarter page) into stage stg
  auto issue = [&](int kt, int stg) {
    const int64_t j0 = (int64_t)kt * kPfKeys;
    const uint8_t* page = reinterpret_cast<const uint8_t*>(a.table_row[j0 / kPageTokens]);
    const int64_t r0 = (int64_t)kvh * kPageTokens + j0 % kPageTokens;
    const uint32_t dst = st_s + stg * kPfStage;
    for (int c = threadIdx.x; c < kPfStage / 16; c += blockDim.x) {
      const int o = c * 16;
      const uint8_t* src = o < kPfStVw   ? page + a.off_kw + r0 * kPfRowB + o
                           : o < kPfStKs ? page + a.off_vw + r0 * kPfRowB + (o - kPfStVw)
                           : o < kPfStVs ? page + a.off_ks + r0 * 4 + (o - kPfStKs)
                                         : page + a.off_vs + r0 * 4 + (o - kPfStVs);
      cp_async16(dst + o, src);
    }
    cp_commit();
  };
  if (ntiles > 0) issue(0, 0);

  // ---- the warp's rows: R0 = 16 warp + g and R1 = R0 + 8, row R = (token
  // tok0 + R / G, head R % G of the group) ----
  const int R0 = warp * 16 + g, R1 = R0 + 8;
  const bool v0 = R0 < TPC * G && R0 / G < ntok, v1 = R1 < TPC * G && R1 / G < ntok;
  const int tk0 = tok0 + R0 / G, tk1 = tok0 + R1 / G;
  const int64_t row0 = (int64_t)tk0 * a.hq + kvh * G + R0 % G, row1 = (int64_t)tk1 * a.hq + kvh * G + R1 % G;

  // ---- q' = (R q) * qscale on the tensor cores, into the A fragments of
  // Q K^T (hi and lo parts). R, scaled by 2^8 so its f16 residuals stay
  // normal, is staged as f16 hi / lo [i][j] tiles in the table's space
  // (built afterwards); q rows are split as they load. D = q_hi R_hi +
  // q_hi R_lo + q_lo R_hi (the dropped lo lo term is 2^-22 of the product).
  // The rotation's accumulators (16 rows x 128 dims, n-tile j = dims 8j ..)
  // are exactly the A fragments of k-step kk = n-tiles 2kk, 2kk + 1. ----
  const uint32_t rh_s = lut_s, rl_s = lut_s + 32768;
  if (!a.q_rotated) {
    for (int u = threadIdx.x; u < kPfD * kPfD / 8; u += blockDim.x) {  // 8 elements per thread step
      const int i = u >> 4, c = u & 15;
      const float4 f0 = *reinterpret_cast<const float4*>(a.kR + i * kPfD + 8 * c);
      const float4 f1 = *reinterpret_cast<const float4*>(a.kR + i * kPfD + 8 * c + 4);
      uint32_t h[4], l[4];
      pf_split(f0.x * kPfRotScale, f0.y * kPfRotScale, h[0], l[0]);
      pf_split(f0.z * kPfRotScale, f0.w * kPfRotScale, h[1], l[1]);
      pf_split(f1.x * kPfRotScale, f1.y * kPfRotScale, h[2], l[2]);
      pf_split(f1.z * kPfRotScale, f1.w * kPfRotScale, h[3], l[3]);
      const uint32_t off = pf_swz(i, c);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(rh_s + off), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                   "r"(h[3])
                   : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(rl_s + off), "r"(l[0]), "r"(l[1]), "r"(l[2]),
                   "r"(l[3])
                   : "memory");
    }
  }
  if (threadIdx.x < 32) s_cent[threadIdx.x] = threadIdx.x < 16 ? a.kcent[threadIdx.x] * a.kalpha
                                                                : a.vcent[threadIdx.x - 16] * a.valpha;
  __syncthreads();
  uint32_t qh[8][4], ql[8][4];
  float qn0 = 0.f, qn1 = 0.f;
  {
    // raw q of rows R0 / R1 at dims (d, d + 1), times qscale
    auto qpair = [&](bool ok, int64_t row, int d) -> float2 {
      if (!ok) return make_float2(0.f, 0.f);
      const int64_t e = row * kPfD + d;
      float2 f;
      if (a.q_dtype == LC_F32) {
        f = *reinterpret_cast<const float2*>(static_cast<const float*>(a.q) + e);
      } else {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(a.q) + e);
        if (a.q_dtype == LC_BF16) {
          f = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
        } else {
          f = make_float2(__half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu))),
                          __half2float(__ushort_as_half((unsigned short)(w >> 16))));
        }
      }
      return make_float2(f.x * a.qscale, f.y * a.qscale);
    };
    if (a.q_rotated) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int d = 16 * kk + 8 * hh + 2 * t;
          const float2 x0 = qpair(v0, row0, d), x1 = qpair(v1, row1, d);
          pf_split(x0.x, x0.y, qh[kk][2 * hh], ql[kk][2 * hh]);
          pf_split(x1.x, x1.y, qh[kk][2 * hh + 1], ql[kk][2 * hh + 1]);
          qn0 = fmaf(x0.x, x0.x, fmaf(x0.y, x0.y, qn0));
          qn1 = fmaf(x1.x, x1.x, fmaf(x1.y, x1.y, qn1));
        }
    } else {
      float d[16][4];
#pragma unroll
      for (int j = 0; j < 16; ++j) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // k-step: dims 16 kk .. of q
        uint32_t ah[4], al[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int dd = 16 * kk + 8 * hh + 2 * t;
          const float2 x0 = qpair(v0, row0, dd), x1 = qpair(v1, row1, dd);
          pf_split(x0.x, x0.y, ah[2 * hh], al[2 * hh]);
          pf_split(x1.x, x1.y, ah[2 * hh + 1], al[2 * hh + 1]);
        }
#pragma unroll
        for (int np = 0; np < 8; ++np) {  // output dims 16 np ..
          uint32_t bh[4], bl[4];
          const uint32_t off = pf_swz(16 * np + (mi >> 1) * 8 + mr, 2 * kk + (mi & 1));
          ldsm_x4(rh_s + off, bh);
          ldsm_x4(rl_s + off, bl);
          mma16816(d[2 * np], ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
          mma16816(d[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bh[2], bh[3]);
          mma16816(d[2 * np], ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
          mma16816(d[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bl[2], bl[3]);
          mma16816(d[2 * np], al[0], al[1], al[2], al[3], bh[0], bh[1]);
          mma16816(d[2 * np + 1], al[0], al[1], al[2], al[3], bh[2], bh[3]);
        }
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float* e = d[2 * kk + hh];
          const float x00 = e[0] * kPfRotUnscale, x01 = e[1] * kPfRotUnscale;
          const float x10 = e[2] * kPfRotUnscale, x11 = e[3] * kPfRotUnscale;
          pf_split(x00, x01, qh[kk][2 * hh], ql[kk][2 * hh]);
          pf_split(x10, x11, qh[kk][2 * hh + 1], ql[kk][2 * hh + 1]);
          qn0 = fmaf(x00, x00, fmaf(x01, x01, qn0));
          qn1 = fmaf(x10, x10, fmaf(x11, x11, qn1));
        }
    }
  }
  // per row the four lanes' sums add; the block's largest row norm bounds all
  {
    float r0n = qn0 + __shfl_xor_sync(0xffffffffu, qn0, 1);
    r0n += __shfl_xor_sync(0xffffffffu, r0n, 2);
    float r1n = qn1 + __shfl_xor_sync(0xffffffffu, qn1, 1);
    r1n += __shfl_xor_sync(0xffffffffu, r1n, 2);
    float w = fmaxf(r0n, r1n);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) s_qn[warp] = w;
  }
  __syncthreads();  // the rotation's reads of R are done: the table replaces it

  // centroid-pair table: entry (byte b, slot) = (c[b & 15], c[b >> 4]) x alpha;
  // K in slots 0..15, K residuals x 2^11 in 16..31, V in 32..63
  {
    uint32_t* lut = reinterpret_cast<uint32_t*>(base);
    for (int idx = threadIdx.x; idx < 256 * 64; idx += blockDim.x) {
      const int b = idx >> 6, slot = idx & 63, off = slot < 32 ? 0 : 16;
      const float x0 = s_cent[off + (b & 15)], x1 = s_cent[off + (b >> 4)];
      lut[idx] = slot >= 16 && slot < 32
                     ? h2_as_u32(__floats2half2_rn((x0 - __half2float(__float2half_rn(x0))) * kPfLoScale,
                                                   (x1 - __half2float(__float2half_rn(x1))) * kPfLoScale))
                     : h2_as_u32(__floats2half2_rn(x0, x1));
    }
  }
  float qmax2 = 0.f;
#pragma unroll
  for (int w = 0; w < kPfWarps; ++w) qmax2 = fmaxf(qmax2, s_qn[w]);
  const float lthr = a.pthr * rsqrtf(fmaxf(qmax2, 1e-30f));  // sigma_K above this: precise tile

  // row key limits: row sees keys j <= P0 + token (-1: an unused row)
  const int64_t lim0 = v0 ? P0 + tk0 : -1, lim1 = v1 ? P0 + tk1 : -1;
  // (views stay below 2^31 tokens: the block table holds at most that many)
  const int64_t wlim = max(__reduce_max_sync(0xffffffffu, (int)lim0), __reduce_max_sync(0xffffffffu, (int)lim1));
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  for (int kt = 0; kt < ntiles; ++kt) {
    cp_wait_all();
    // tile kt is staged for all threads, and every warp is done with tile
    // kt - 1 (its f16 tiles and its stage's sigmas): tile kt + 1 may land there
    __syncthreads();
    if (kt + 1 < ntiles) issue(kt + 1, (kt + 1) & 1);
    const uint8_t* st = stage0 + (kt & 1) * kPfStage;
    const float* sk = reinterpret_cast<const float*>(st + kPfStKs);
    const float* sv = reinterpret_cast<const float*>(st + kPfStVs);
    const int64_t j0 = (int64_t)kt * kPfKeys;
    // precise tile: the largest sigma_K of the tile's keys (every warp finds the same)
    float smax = 0.f;
    if (j0 + lane < n_keys) smax = sk[lane];
    if (j0 + lane + 32 < n_keys) smax = fmaxf(smax, sk[lane + 32]);
    const bool lo = __any_sync(0xffffffffu, smax > lthr);
    pf_dequant(st, lut_s, k_s, kl_s, v_s, lo);
    __syncthreads();
    if (wlim < j0) continue;  // the warp's rows end before this tile (its last tiles)

    // ---- S = Q K^T: n-tile j = keys 8j .. 8j + 7 of the tile ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    // per k-step: the four B loads, then the eight hi and the eight lo MMAs,
    // so that MMAs on one accumulator stand eight apart
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t b[4][4];
#pragma unroll
      for (int np = 0; np < 4; ++np) ldsm_x4(k_s + pf_swz(16 * np + (mi >> 1) * 8 + mr, 2 * kk + (mi & 1)), b[np]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        mma16816(s[2 * np], qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b[np][0], b[np][1]);
        mma16816(s[2 * np + 1], qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b[np][2], b[np][3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        mma16816(s[2 * np], ql[kk][0], ql[kk][1], ql[kk][2], ql[kk][3], b[np][0], b[np][1]);
        mma16816(s[2 * np + 1], ql[kk][0], ql[kk][1], ql[kk][2], ql[kk][3], b[np][2], b[np][3]);
      }
    }
    if (lo) {  // + Q (K table residuals) x 2^-11, two n-tiles at a time
#pragma unroll 1
      for (int np = 0; np < 4; ++np) {
        float r0[4] = {0.f, 0.f, 0.f, 0.f}, r1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t b[4];
          ldsm_x4(kl_s + pf_swz(16 * np + (mi >> 1) * 8 + mr, 2 * kk + (mi & 1)), b);
          mma16816(r0, qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b[0], b[1]);
          mma16816(r1, qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b[2], b[3]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s[2 * np][e] = fmaf(r0[e], kPfLoUnscale, s[2 * np][e]);
          s[2 * np + 1][e] = fmaf(r1[e], kPfLoUnscale, s[2 * np + 1][e]);
        }
      }
    }
    // ---- scale by sigma_K, causal mask; lane (g, t) holds rows g (e 0, 1)
    // and g + 8 (e 2, 3) at keys 8j + 2t + (e & 1) ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kc = 8 * j + 2 * t + (e & 1);
        const int64_t key = j0 + kc;
        const bool ok = key <= (e < 2 ? lim0 : lim1);
        s[j][e] = ok ? s[j][e] * sk[kc] : -INFINITY;
        if (e < 2) mx0 = fmaxf(mx0, s[j][e]);
        else mx1 = fmaxf(mx1, s[j][e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // ---- online softmax (log2 units): rescale O and l when the max moves ----
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = mn0 == -INFINITY ? 1.f : ex2(m0 - mn0), al1 = mn1 == -INFINITY ? 1.f : ex2(m1 - mn1);
    const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
    m0 = mn0;
    m1 = mn1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    // ---- O += (P sigma_V) V: k-step kk = keys 16kk .. 16kk + 15, n-tile
    // j = dims 8j .. 8j + 7; the A fragments come from S's n-tiles 2kk, 2kk + 1 ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int j = 2 * kk + hh, kc = 8 * j + 2 * t;
        const float p00 = ex2(s[j][0] - mu0), p01 = ex2(s[j][1] - mu0);
        const float p10 = ex2(s[j][2] - mu1), p11 = ex2(s[j][3] - mu1);
        l0 += p00 + p01;
        l1 += p10 + p11;
        // keys past the view have p = 0; their sigma_V is not read into the product
        const float w0 = p00 == 0.f ? 0.f : p00 * sv[kc], w1 = p01 == 0.f ? 0.f : p01 * sv[kc + 1];
        const float w2 = p10 == 0.f ? 0.f : p10 * sv[kc], w3 = p11 == 0.f ? 0.f : p11 * sv[kc + 1];
        ph[2 * hh] = h2_as_u32(__floats2half2_rn(w0, w1));
        ph[2 * hh + 1] = h2_as_u32(__floats2half2_rn(w2, w3));
      }
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t b[4];
        ldsm_x4_t(v_s + pf_swz(16 * kk + (mi & 1) * 8 + mr, 2 * np + (mi >> 1)), b);
        mma16816(o[2 * np], ph[0], ph[1], ph[2], ph[3], b[0], b[1]);
        mma16816(o[2 * np + 1], ph[0], ph[1], ph[2], ph[3], b[2], b[3]);
      }
    }
  }

  // ---- the rows: O / l * oscale, un-rotated by V's R^T on the tensor cores
  // (out[i] = sum_j R[j][i] o[j]: A = the normalised O in its accumulator
  // layout, B = R^T [i][j] staged as f16 hi / lo tiles x 2^8 in the table's
  // space), written in the caller's dtype ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float n0 = l0 > 0.f ? a.oscale / l0 : 0.f, n1 = l1 > 0.f ? a.oscale / l1 : 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    o[j][0] *= n0;
    o[j][1] *= n0;
    o[j][2] *= n1;
    o[j][3] *= n1;
  }
  if (a.vRT) {
    __syncthreads();  // every warp is past its last tile: the table space is free
    for (int u = threadIdx.x; u < kPfD * kPfD / 8; u += blockDim.x) {
      const int i = u >> 4, c = u & 15;
      const float4 f0 = *reinterpret_cast<const float4*>(a.vRT + i * kPfD + 8 * c);
      const float4 f1 = *reinterpret_cast<const float4*>(a.vRT + i * kPfD + 8 * c + 4);
      uint32_t h[4], l[4];
      pf_split(f0.x * kPfRotScale, f0.y * kPfRotScale, h[0], l[0]);
      pf_split(f0.z * kPfRotScale, f0.w * kPfRotScale, h[1], l[1]);
      pf_split(f1.x * kPfRotScale, f1.y * kPfRotScale, h[2], l[2]);
      pf_split(f1.z * kPfRotScale, f1.w * kPfRotScale, h[3], l[3]);
      const uint32_t off = pf_swz(i, c);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(rh_s + off), "r"(h[0]), "r"(h[1]), "r"(h[2]),
                   "r"(h[3])
                   : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(rl_s + off), "r"(l[0]), "r"(l[1]), "r"(l[2]),
                   "r"(l[3])
                   : "memory");
    }
    __syncthreads();
    float d[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) d[j][0] = d[j][1] = d[j][2] = d[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {  // k-step: dims 16 kk .. of o
      uint32_t ah[4], al[4];
      pf_split(o[2 * kk][0], o[2 * kk][1], ah[0], al[0]);
      pf_split(o[2 * kk][2], o[2 * kk][3], ah[1], al[1]);
      pf_split(o[2 * kk + 1][0], o[2 * kk + 1][1], ah[2], al[2]);
      pf_split(o[2 * kk + 1][2], o[2 * kk + 1][3], ah[3], al[3]);
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        uint32_t bh[4], bl[4];
        const uint32_t off = pf_swz(16 * np + (mi >> 1) * 8 + mr, 2 * kk + (mi & 1));
        ldsm_x4(rh_s + off, bh);
        ldsm_x4(rl_s + off, bl);
        mma16816(d[2 * np], ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
        mma16816(d[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bh[2], bh[3]);
        mma16816(d[2 * np], ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
        mma16816(d[2 * np + 1], ah[0], ah[1], ah[2], ah[3], bl[2], bl[3]);
        mma16816(d[2 * np], al[0], al[1], al[2], al[3], bh[0], bh[1]);
        mma16816(d[2 * np + 1], al[0], al[1], al[2], al[3], bh[2], bh[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] = d[j][0] * kPfRotUnscale;
      o[j][1] = d[j][1] * kPfRotUnscale;
      o[j][2] = d[j][2] * kPfRotUnscale;
      o[j][3] = d[j][3] * kPfRotUnscale;
    }
  }
  auto put2 = [&](int64_t row, int dim, float x, float y) {
    const int64_t e = row * kPfD + dim;
    if (a.out_dtype == LC_F32) {
      *reinterpret_cast<float2*>(static_cast<float*>(a.out) + e) = make_float2(x, y);
    } else if (a.out_dtype == LC_BF16) {
      *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + e) = __floats2bfloat162_rn(x, y);
    } else {
      *reinterpret_cast<__half2*>(static_cast<__half*>(a.out) + e) = __floats2half2_rn(x, y);
    }
  };
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (v0) put2(row0, 8 * j + 2 * t, o[j][0], o[j][1]);
    if (v1) put2(row1, 8 * j + 2 * t, o[j][2], o[j][3]);
  }
}

template <int G>
void launch_pf_g(const PrefillArgs& a, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_prefill_tiled<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
    attr = true;
  }
  constexpr int TPC = kPfRows / G;
  const int64_t blocks = (int64_t)((a.L + TPC - 1) / TPC) * a.hkv;
  k_prefill_tiled<G><<<(unsigned)blocks, kPfWarps * 32, kPfSmem, s>>>(a);
  LC_CUDA(cudaGetLastError());
}

}  // namespace

bool prefill_tiled_path(int dim, int kbits, int vbits, int G) {
  return dim == kPfD && kbits == 4 && vbits == 4 && G >= 1 && G <= 8;
}

void launch_prefill_tiled(const PrefillArgs& a, cudaStream_t s) {
  LC_REQUIRE(a.L > 0 && a.L <= a.n_total && a.hkv > 0 && a.hq % a.hkv == 0, LC_ERR_INVALID, "prefill: bad geometry");
  switch (a.hq / a.hkv) {
    case 1: return launch_pf_g<1>(a, s);
    case 2: return launch_pf_g<2>(a, s);
    case 3: return launch_pf_g<3>(a, s);
    case 4: return launch_pf_g<4>(a, s);
    case 5: return launch_pf_g<5>(a, s);
    case 6: return launch_pf_g<6>(a, s);
    case 7: return launch_pf_g<7>(a, s);
    case 8: return launch_pf_g<8>(a, s);
    default: LC_THROW(LC_ERR_INVALID, "prefill: GQA group above 8");
  }
}

}  // namespace lc
