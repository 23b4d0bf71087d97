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
//  k_rotate_q      q' = (R q) * scale * log2(e), f32 + f16 copies
//  k_decode_mma    4-bit K/V, d = 128: the GQA tile on the tensor cores.
//                  Codes are dequantized straight into mma.sync fragments
//                  (a 256-entry byte -> half2 centroid-pair table in shared
//                  memory, one copy per lane so every lookup is
//                  bank-conflict-free); S^T = K_dq Q^T and O^T = V_dq^T P^T
//                  run as m16n8k16 f16 MMAs with f32 accumulation.
//  k_decode_generic any bit width / head_dim: CUDA-core fallback.
//  k_merge         combines the split-K partials, normalises, un-rotates.
// Streaming reads of the compressed pages are the roofline (HBM): per
// (token, kv head) 8*words_K + 8*words_V + 8 bytes.
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <cfloat>

#include "kernels.h"

namespace lc {

namespace {

constexpr float kLog2e = 1.4426950408889634f;
// Lazy rescale threshold (log2 units): the running max is only moved when a
// new score exceeds it by more than this, bounding p by 2^kTau.
constexpr float kTau = 8.0f;

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == LC_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == LC_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == LC_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dtype == LC_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

// ---------------------------------------------------------------------------
// q' = R q * qscale. Block: dim threads, 8 rows per block.
// ---------------------------------------------------------------------------
constexpr int kRotRows = 8;

__global__ void k_rotate_q(const void* q, int dtype, int n_rows, int D, const float* RT, int rotated,
                           float qscale, float* q_rot, __half* q_h) {
  extern __shared__ float sq[];  // [kRotRows][D]
  const int i = threadIdx.x;
  const int r0 = blockIdx.x * kRotRows;
  for (int r = 0; r < kRotRows; ++r)
    sq[r * D + i] = (r0 + r < n_rows) ? load_any(q, dtype, (int64_t)(r0 + r) * D + i) : 0.0f;
  __syncthreads();
  float acc[kRotRows];
  if (rotated) {
#pragma unroll
    for (int r = 0; r < kRotRows; ++r) acc[r] = sq[r * D + i];
  } else {
#pragma unroll
    for (int r = 0; r < kRotRows; ++r) acc[r] = 0.0f;
    for (int j = 0; j < D; ++j) {
      const float w = __ldg(RT + (int64_t)j * D + i);  // R[i][j]
#pragma unroll
      for (int r = 0; r < kRotRows; ++r) acc[r] = fmaf(w, sq[r * D + j], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < kRotRows; ++r) {
    if (r0 + r < n_rows) {
      const float v = acc[r] * qscale;
      q_rot[(int64_t)(r0 + r) * D + i] = v;
      q_h[(int64_t)(r0 + r) * D + i] = __float2half_rn(v);
    }
  }
}

struct DecodeDev {
  const uint64_t* table;
  int64_t table_stride;
  const int64_t* seqinfo;
  int64_t off_kw, off_vw, off_ks, off_vs;
  int32_t row_kw, row_vw;
  int32_t n_seqs, hkv, hq, dim, kbits, vbits, pages_per_chunk, n_chunks, G;
  const float* q_rot;
  const __half* q_h;
  const float* kcent;
  const float* vcent;
  float* part;
};

// ---------------------------------------------------------------------------
// Fast path: 4-bit K and V, head_dim 128, up to 8 query heads per kv head.
// CTA = 4 warps; a warp streams one page (256 tokens) in tiles of 16 tokens.
// ---------------------------------------------------------------------------
constexpr int kMmaWarps = 4;
constexpr int kLutBytes = 256 * 64 * 4;  // [byte][64 slots]: K table slots 0..31, V table 32..63

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Table lookup: byte k of x selects a half2 centroid pair; the lane's own
// copy (slot lane) keeps the 32 lookups of a warp in 32 distinct banks.
__device__ __forceinline__ uint32_t lut_get(const uint8_t* lut, uint32_t x, uint32_t laneword, uint32_t sel,
                                            int slot_off) {
  const uint32_t off = __byte_perm(x, laneword, sel);
  return *reinterpret_cast<const uint32_t*>(lut + slot_off + off);
}

template <int G>
__global__ void __launch_bounds__(kMmaWarps * 32) k_decode_mma(DecodeDev a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* lut = smem;
  float* wpart = reinterpret_cast<float*>(smem + kLutBytes);  // [kMmaWarps][G][130]
  constexpr int D = 128;
  constexpr int PS = D + 2;

  for (int idx = threadIdx.x; idx < 256 * 64; idx += blockDim.x) {
    const int e = idx >> 6, slot = idx & 63;
    const float* cent = slot < 32 ? a.kcent : a.vcent;
    reinterpret_cast<uint32_t*>(lut)[idx] = h2_as_u32(__floats2half2_rn(cent[e & 15], cent[e >> 4]));
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t laneword = (uint32_t)lane << 2;
  const int64_t total = (int64_t)a.n_seqs * a.hkv * a.n_chunks;

  for (int64_t item = blockIdx.x; item < total; item += gridDim.x) {
    const int chunk = (int)(item % a.n_chunks);
    const int64_t rest = item / a.n_chunks;
    const int kvh = (int)(rest % a.hkv);
    const int s = (int)(rest / a.hkv);
    const int64_t n_valid = a.seqinfo[2 * s];
    const uint64_t* trow = a.table + a.seqinfo[2 * s + 1] * a.table_stride;
    const int64_t page_idx = (int64_t)chunk * kMmaWarps + warp;
    const int64_t tok0 = page_idx * kPageTokens;

    // B fragments of Q^T: k-step st covers dims 32t + 4st + {0,1} and {2,3}.
    uint32_t qb[8][2];
    {
      const __half* qrow = a.q_h + ((int64_t)s * a.hq + (int64_t)kvh * G + (g < G ? g : 0)) * D;
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(qrow + 32 * t + 4 * st);
        qb[st][0] = g < G ? p[0] : 0u;
        qb[st][1] = g < G ? p[1] : 0u;
      }
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float oacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;

    if (tok0 < n_valid) {
      const uint8_t* page = reinterpret_cast<const uint8_t*>(trow[page_idx]);
      const uint8_t* kb = page + a.off_kw + (int64_t)kvh * kPageTokens * 64;
      const uint8_t* vb = page + a.off_vw + (int64_t)kvh * kPageTokens * 64;
      const float* ksg = reinterpret_cast<const float*>(page + a.off_ks) + (int64_t)kvh * kPageTokens;
      const float* vsg = reinterpret_cast<const float*>(page + a.off_vs) + (int64_t)kvh * kPageTokens;
      const int64_t rem = n_valid - tok0;
      const int ntiles = rem >= kPageTokens ? 16 : (int)((rem + 15) / 16);

      uint4 nk0, nk1;
      uint2 nv[4];
      float nks0, nks1, nvs0, nvs1;
      auto load_tile = [&](int tile) {
        const int r = tile * 16;
        nk0 = *reinterpret_cast<const uint4*>(kb + (r + g) * 64 + 16 * t);
        nk1 = *reinterpret_cast<const uint4*>(kb + (r + g + 8) * 64 + 16 * t);
        nv[0] = *reinterpret_cast<const uint2*>(vb + (r + t) * 64 + 8 * g);
        nv[1] = *reinterpret_cast<const uint2*>(vb + (r + t + 8) * 64 + 8 * g);
        nv[2] = *reinterpret_cast<const uint2*>(vb + (r + t + 4) * 64 + 8 * g);
        nv[3] = *reinterpret_cast<const uint2*>(vb + (r + t + 12) * 64 + 8 * g);
        nks0 = ksg[r + g];
        nks1 = ksg[r + g + 8];
        nvs0 = vsg[r + g];
        nvs1 = vsg[r + g + 8];
      };
      load_tile(0);
      for (int tile = 0; tile < ntiles; ++tile) {
        const uint4 k0 = nk0, k1 = nk1;
        const uint2 v0 = nv[0], v1 = nv[1], v2 = nv[2], v3 = nv[3];
        const float ks0 = nks0, ks1 = nks1, vs0 = nvs0, vs1 = nvs1;
        if (tile + 1 < ntiles) load_tile(tile + 1);

        // ---- S^T[16 tok x 8 heads] = K_dq Q^T ----
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t kx[4] = {k0.x, k0.y, k0.z, k0.w};
        const uint32_t ky[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t s0 = 0x5504u | ((2u * h) << 4), s1 = 0x5504u | ((2u * h + 1u) << 4);
            const uint32_t a0 = lut_get(lut, kx[j], laneword, s0, 0);
            const uint32_t a2 = lut_get(lut, kx[j], laneword, s1, 0);
            const uint32_t a1 = lut_get(lut, ky[j], laneword, s0, 0);
            const uint32_t a3 = lut_get(lut, ky[j], laneword, s1, 0);
            mma16816(sc, a0, a1, a2, a3, qb[2 * j + h][0], qb[2 * j + h][1]);
          }
        }
        // ---- online softmax (log2 domain) ----
        const int64_t tg = tok0 + tile * 16 + g;
        const bool ok0 = tg < n_valid, ok1 = tg + 8 < n_valid;
        const float s00 = ok0 ? sc[0] * ks0 : -INFINITY;  // token g,   head 2t
        const float s01 = ok0 ? sc[1] * ks0 : -INFINITY;  // token g,   head 2t+1
        const float s10 = ok1 ? sc[2] * ks1 : -INFINITY;  // token g+8, head 2t
        const float s11 = ok1 ? sc[3] * ks1 : -INFINITY;  // token g+8, head 2t+1
        float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        if (mx0 > m0 + kTau) {
          const float al = exp2f(m0 - mx0);
          l0 *= al;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            oacc[i][0] *= al;
            oacc[i][2] *= al;
          }
          m0 = mx0;
        }
        if (mx1 > m1 + kTau) {
          const float al = exp2f(m1 - mx1);
          l1 *= al;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            oacc[i][1] *= al;
            oacc[i][3] *= al;
          }
          m1 = mx1;
        }
        const float p00 = ok0 ? exp2f(s00 - m0) : 0.f, p10 = ok1 ? exp2f(s10 - m0) : 0.f;
        const float p01 = ok0 ? exp2f(s01 - m1) : 0.f, p11 = ok1 ? exp2f(s11 - m1) : 0.f;
        l0 += p00 + p10;
        l1 += p01 + p11;
        const float w0 = ok0 ? vs0 : 0.f, w1 = ok1 ? vs1 : 0.f;
        const uint32_t h0 = h2_as_u32(__floats2half2_rn(p00 * w0, p10 * w1));  // head 2t:   tokens g, g+8
        const uint32_t h1 = h2_as_u32(__floats2half2_rn(p01 * w0, p11 * w1));  // head 2t+1: tokens g, g+8
        // ---- transpose P into the B fragment of P^T: head g, tokens (t, t+8), (t+4, t+12) ----
        const int src0 = t * 4 + (g >> 1), src1 = (t + 4) * 4 + (g >> 1);
        const uint32_t r00 = __shfl_sync(0xffffffffu, h0, src0), r01 = __shfl_sync(0xffffffffu, h1, src0);
        const uint32_t r10 = __shfl_sync(0xffffffffu, h0, src1), r11 = __shfl_sync(0xffffffffu, h1, src1);
        uint32_t pb0 = (g & 1) ? r01 : r00, pb1 = (g & 1) ? r11 : r10;
        if (g >= G) pb0 = pb1 = 0u;
        // ---- O^T[128 dims x 8 heads] += V_dq^T P^T ----
        // pair 0 = tokens (t, t+8), pair 1 = tokens (t+4, t+12); word g = dims 16g..16g+15
        uint32_t ev[2][2], od[2][2];
        {
          const uint32_t A0[2] = {v0.x, v0.y}, B0[2] = {v1.x, v1.y};
          const uint32_t A1[2] = {v2.x, v2.y}, B1[2] = {v3.x, v3.y};
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            ev[0][hh] = (A0[hh] & 0x0F0F0F0Fu) | ((B0[hh] & 0x0F0F0F0Fu) << 4);
            od[0][hh] = ((A0[hh] >> 4) & 0x0F0F0F0Fu) | (B0[hh] & 0xF0F0F0F0u);
            ev[1][hh] = (A1[hh] & 0x0F0F0F0Fu) | ((B1[hh] & 0x0F0F0F0Fu) << 4);
            od[1][hh] = ((A1[hh] >> 4) & 0x0F0F0F0Fu) | (B1[hh] & 0xF0F0F0F0u);
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int hh = i >> 2;
          const uint32_t sel = 0x5504u | ((uint32_t)(i & 3) << 4);
          const uint32_t a0 = lut_get(lut, ev[0][hh], laneword, sel, 128);
          const uint32_t a1 = lut_get(lut, od[0][hh], laneword, sel, 128);
          const uint32_t a2 = lut_get(lut, ev[1][hh], laneword, sel, 128);
          const uint32_t a3 = lut_get(lut, od[1][hh], laneword, sel, 128);
          mma16816(oacc[i], a0, a1, a2, a3, pb0, pb1);
        }
      }
    }
    // ---- warp partial: reduce l over the 8 lanes sharing t ----
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    float* wp = wpart + warp * G * PS;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hd = 2 * t + e;
      if (hd < G) {
        float* row = wp + hd * PS;
        if (g == 0) {
          row[0] = e ? m1 : m0;
          row[1] = e ? l1 : l0;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          row[2 + 16 * g + 2 * i] = oacc[i][e];
          row[2 + 16 * g + 2 * i + 1] = oacc[i][2 + e];
        }
      }
    }
    __syncthreads();
    // ---- merge the CTA's warps and write the chunk partial ----
    for (int u = threadIdx.x; u < G * (D + 2); u += blockDim.x) {
      const int hd = u / (D + 2), k = u % (D + 2);
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, wpart[(w * G + hd) * PS]);
      float val;
      if (k == 0) {
        val = M;
      } else {
        val = 0.f;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) {
          const float mw = wpart[(w * G + hd) * PS];
          if (mw != -INFINITY) val += exp2f(mw - M) * wpart[(w * G + hd) * PS + k];
        }
      }
      const int64_t row = (int64_t)s * a.hq + (int64_t)kvh * G + hd;
      a.part[(row * a.n_chunks + chunk) * PS + k] = val;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Generic path: any bit width, head_dim = 32*KPL, GS query heads per CTA.
// ---------------------------------------------------------------------------
template <int KPL, int GS>
__global__ void __launch_bounds__(128) k_decode_generic(DecodeDev a) {
  extern __shared__ __align__(16) float gsm[];
  const int D = 32 * KPL;
  const int PS = D + 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  float* kc = gsm;             // [256]
  float* vc = gsm + 256;       // [256]
  float* wpart = gsm + 512;    // [nw][GS][PS]
  for (int i = threadIdx.x; i < (1 << a.kbits); i += blockDim.x) kc[i] = a.kcent[i];
  for (int i = threadIdx.x; i < (1 << a.vbits); i += blockDim.x) vc[i] = a.vcent[i];
  __syncthreads();
  const int groups = a.G / GS;
  const int kcpw = 64 / a.kbits, vcpw = 64 / a.vbits;
  const uint64_t kmask = (1ull << a.kbits) - 1, vmask = (1ull << a.vbits) - 1;
  const int64_t total = (int64_t)a.n_seqs * a.hkv * groups * a.n_chunks;

  for (int64_t item = blockIdx.x; item < total; item += gridDim.x) {
    const int chunk = (int)(item % a.n_chunks);
    int64_t rest = item / a.n_chunks;
    const int grp = (int)(rest % groups);
    rest /= groups;
    const int kvh = (int)(rest % a.hkv);
    const int s = (int)(rest / a.hkv);
    const int64_t n_valid = a.seqinfo[2 * s];
    const uint64_t* trow = a.table + a.seqinfo[2 * s + 1] * a.table_stride;
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
    for (int pw = warp; pw < a.pages_per_chunk; pw += nw) {
      const int64_t page_idx = (int64_t)chunk * a.pages_per_chunk + pw;
      const int64_t tok0 = page_idx * kPageTokens;
      if (tok0 >= n_valid) break;
      const uint8_t* page = reinterpret_cast<const uint8_t*>(trow[page_idx]);
      const uint64_t* kw = reinterpret_cast<const uint64_t*>(page + a.off_kw + (int64_t)kvh * kPageTokens * a.row_kw);
      const uint64_t* vw = reinterpret_cast<const uint64_t*>(page + a.off_vw + (int64_t)kvh * kPageTokens * a.row_vw);
      const float* ks = reinterpret_cast<const float*>(page + a.off_ks) + (int64_t)kvh * kPageTokens;
      const float* vs = reinterpret_cast<const float*>(page + a.off_vs) + (int64_t)kvh * kPageTokens;
      const int kw_row = a.row_kw / 8, vw_row = a.row_vw / 8;
      const int nt = (int)(n_valid - tok0 < kPageTokens ? n_valid - tok0 : kPageTokens);
      for (int tt = 0; tt < nt; ++tt) {
        float part[GS];
#pragma unroll
        for (int g = 0; g < GS; ++g) part[g] = 0.f;
        float vv[KPL];
#pragma unroll
        for (int k = 0; k < KPL; ++k) {
          const int d = lane + 32 * k;
          const uint64_t w = kw[(int64_t)tt * kw_row + d / kcpw];
          const float c = kc[(w >> ((d % kcpw) * a.kbits)) & kmask];
#pragma unroll
          for (int g = 0; g < GS; ++g) part[g] = fmaf(q[g][k], c, part[g]);
          const uint64_t wv = vw[(int64_t)tt * vw_row + d / vcpw];
          vv[k] = vc[(wv >> ((d % vcpw) * a.vbits)) & vmask];
        }
#pragma unroll
        for (int g = 0; g < GS; ++g) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) part[g] += __shfl_xor_sync(0xffffffffu, part[g], off);
        }
        const float ksg = ks[tt], vsg = vs[tt];
#pragma unroll
        for (int g = 0; g < GS; ++g) {
          const float sc = part[g] * ksg;
          const float mn = fmaxf(m[g], sc);
          const float al = exp2f(m[g] - mn);
          const float p = exp2f(sc - mn);
          l[g] = l[g] * al + p;
          const float pw2 = p * vsg;
#pragma unroll
          for (int k = 0; k < KPL; ++k) o[g][k] = fmaf(pw2, vv[k], o[g][k] * al);
          m[g] = mn;
        }
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
      const int64_t row = (int64_t)s * a.hq + qh0 + g;
      a.part[(row * a.n_chunks + chunk) * PS + k] = val;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Merge: rows of partials -> normalised (optionally un-rotated) output, or
// merged partials. Block: dim threads, kMergeRows rows per block.
// ---------------------------------------------------------------------------
constexpr int kMergeRows = 8;

struct MergeDev {
  const float* part;
  int64_t stride_row, stride_part;
  int32_t n_rows, n_parts, D;
  const float* R;
  void* out;
  int32_t out_dtype;
  float* m_out;
  float* l_out;
  float* o_out;
};

__global__ void k_merge(MergeDev a) {
  extern __shared__ float so[];  // [kMergeRows][D]
  const int i = threadIdx.x;
  const int r0 = blockIdx.x * kMergeRows;
  const int D = a.D;
  for (int r = 0; r < kMergeRows; ++r) {
    const int row = r0 + r;
    float val = 0.f;
    if (row < a.n_rows) {
      const float* p = a.part + (int64_t)row * a.stride_row;
      float M = -INFINITY;
      for (int c = 0; c < a.n_parts; ++c) M = fmaxf(M, p[(int64_t)c * a.stride_part]);
      float L = 0.f, O = 0.f;
      for (int c = 0; c < a.n_parts; ++c) {
        const float* pc = p + (int64_t)c * a.stride_part;
        if (pc[0] == -INFINITY) continue;
        const float w = exp2f(pc[0] - M);
        L += w * pc[1];
        O += w * pc[2 + i];
      }
      if (a.o_out) {
        a.o_out[(int64_t)row * D + i] = O;
        if (i == 0) {
          a.m_out[row] = M;
          a.l_out[row] = L;
        }
      }
      val = L > 0.f ? O / L : 0.f;
    }
    so[r * D + i] = val;
  }
  if (!a.out) return;
  __syncthreads();
  float acc[kMergeRows];
  if (a.R) {
#pragma unroll
    for (int r = 0; r < kMergeRows; ++r) acc[r] = 0.f;
    for (int j = 0; j < D; ++j) {
      const float w = __ldg(a.R + (int64_t)j * D + i);  // (R^T)[i][j] = R[j][i]
#pragma unroll
      for (int r = 0; r < kMergeRows; ++r) acc[r] = fmaf(w, so[r * D + j], acc[r]);
    }
  } else {
#pragma unroll
    for (int r = 0; r < kMergeRows; ++r) acc[r] = so[r * D + i];
  }
#pragma unroll
  for (int r = 0; r < kMergeRows; ++r)
    if (r0 + r < a.n_rows) store_any(a.out, a.out_dtype, (int64_t)(r0 + r) * D + i, acc[r]);
}

int g_num_sms = 0;

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

template <int G>
void launch_mma_g(const DecodeDev& d, cudaStream_t s) {
  const size_t smem = kLutBytes + (size_t)kMmaWarps * G * 130 * sizeof(float);
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_mma<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  int per_sm = 0;
  LC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mma<G>, kMmaWarps * 32, smem));
  if (per_sm < 1) per_sm = 1;
  const int64_t total = (int64_t)d.n_seqs * d.hkv * d.n_chunks;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > total) grid = total;
  k_decode_mma<G><<<(unsigned)grid, kMmaWarps * 32, smem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

template <int KPL, int GS>
void launch_generic_t(const DecodeDev& d, cudaStream_t s) {
  const int nw = 4;
  const size_t smem = (512 + (size_t)nw * GS * (32 * KPL + 2)) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_decode_generic<KPL, GS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
    attr = true;
  }
  int per_sm = 0;
  LC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_generic<KPL, GS>, nw * 32, smem));
  if (per_sm < 1) per_sm = 1;
  const int64_t total = (int64_t)d.n_seqs * d.hkv * (d.G / GS) * d.n_chunks;
  int64_t grid = (int64_t)num_sms() * per_sm;
  if (grid > total) grid = total;
  k_decode_generic<KPL, GS><<<(unsigned)grid, nw * 32, smem, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

template <int KPL>
void launch_generic_k(const DecodeDev& d, cudaStream_t s) {
  constexpr int cap = 32 / KPL > 0 ? 32 / KPL : 1;  // keep GS*KPL <= 32 registers per array
  if (cap >= 4 && d.G % 4 == 0) return launch_generic_t<KPL, 4>(d, s);
  if (cap >= 2 && d.G % 2 == 0) return launch_generic_t<KPL, 2>(d, s);
  return launch_generic_t<KPL, 1>(d, s);
}

}  // namespace

bool decode_fast_path(int dim, int kbits, int vbits, int G) {
  return dim == 128 && kbits == 4 && vbits == 4 && G >= 1 && G <= 8;
}

void launch_rotate_q(const void* q, int32_t q_dtype, int32_t n_rows, int32_t dim, const float* RT,
                     bool q_is_rotated, float qscale, float* q_rot, __half* q_h, cudaStream_t s) {
  if (n_rows <= 0) return;
  const int blocks = (n_rows + kRotRows - 1) / kRotRows;
  k_rotate_q<<<blocks, dim, kRotRows * dim * sizeof(float), s>>>(q, q_dtype, n_rows, dim, RT, q_is_rotated ? 1 : 0,
                                                                 qscale, q_rot, q_h);
  LC_CUDA(cudaGetLastError());
}

void launch_decode_partials(const DecodeArgs& a, cudaStream_t s) {
  DecodeDev d;
  d.table = a.table;
  d.table_stride = a.table_stride;
  d.seqinfo = a.seqinfo;
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
  d.pages_per_chunk = a.pages_per_chunk;
  d.n_chunks = a.n_chunks;
  d.G = a.hq / a.hkv;
  d.q_rot = a.q_rot;
  d.q_h = a.q_h;
  d.kcent = a.kcent;
  d.vcent = a.vcent;
  d.part = a.part;
  if (decode_fast_path(a.dim, a.kbits, a.vbits, d.G) && a.pages_per_chunk == kMmaWarps) {
    switch (d.G) {
      case 1: return launch_mma_g<1>(d, s);
      case 2: return launch_mma_g<2>(d, s);
      case 3: return launch_mma_g<3>(d, s);
      case 4: return launch_mma_g<4>(d, s);
      case 5: return launch_mma_g<5>(d, s);
      case 6: return launch_mma_g<6>(d, s);
      case 7: return launch_mma_g<7>(d, s);
      default: return launch_mma_g<8>(d, s);
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

void launch_merge(const float* part, int32_t n_rows, int32_t n_parts, int32_t dim, int64_t stride_row,
                  int64_t stride_part, const float* R, void* out, int32_t out_dtype, float* m_out, float* l_out,
                  float* o_out, cudaStream_t s) {
  if (n_rows <= 0) return;
  MergeDev d{part, stride_row, stride_part, n_rows, n_parts, dim, R, out, out_dtype, m_out, l_out, o_out};
  const int blocks = (n_rows + kMergeRows - 1) / kMergeRows;
  k_merge<<<blocks, dim, kMergeRows * dim * sizeof(float), s>>>(d);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
