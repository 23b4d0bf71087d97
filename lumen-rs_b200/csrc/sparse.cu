// Page-sparse decode over the codes (LC_STORE_DIGEST / LC_SPARSE_PAGES):
// the PageDigest of crates/lumen-mlx/src/native_cache.rs:350-445 and the page
// selection of sdpa_page_sparse (native_attention.rs:217-329), with the keys
// taken as the decode sees them: rotated and dequantized, c[code] * sigma.
//
//   k_digest4      min and max over each full 64-token page, per head and dim,
//                  into the page's digest role (64 rows of head_dim / 8 bytes:
//                  min[D] f32 then max[D] f32); 4-bit codes, head_dim 128
//   k_digest_gen   the same for other bit widths at head_dim 128 / 256
//   k_page_select  per (sequence, kv head): bound of every digested page
//                  = max over the head's query group of
//                    sum_d max(q'_d * max_d, q'_d * min_d),
//                  sink and recent pages pinned, the keep largest chosen; the
//                  chosen pages (ascending) and the undigested tail become a
//                  map from logical to physical 32-token tiles for the decode
#include <cuda_bf16.h>

#include <cfloat>

#include "kernels.h"

namespace lc {

namespace {

// The 4-bit, head_dim 128 digest (the page-sparse geometry): a warp per
// (page, head), 4 warps (heads) per block. Lane l reads word l % 8 of token
// rows l / 8, + 4, + 8, ... (each load instruction covers 4 whole 64-byte
// rows), keeps the min and max of its word's 16 dims, and the 4 lanes that
// share a word combine theirs at the end.
__global__ void __launch_bounds__(128) k_digest4(DigestDev a, int heads) {
  __shared__ float sc[16];
  if (threadIdx.x < 16) sc[threadIdx.x] = a.cent[threadIdx.x];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + warp;
  if (h >= heads) return;
  const uint8_t* page = reinterpret_cast<const uint8_t*>(a.pages[blockIdx.x]);
  const int64_t hr0 = (int64_t)h * kPageTokens + a.row0[blockIdx.x];
  const int lt = lane >> 3, lw = lane & 7;
  const uint8_t* kw = page + a.off_kw + (hr0 + lt) * 64 + lw * 8;
  const float* ks = reinterpret_cast<const float*>(page + a.off_ks) + hr0 + lt;
  float mn[16], mx[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    mn[k] = FLT_MAX;
    mx[k] = -FLT_MAX;
  }
#pragma unroll 1
  for (int t0 = 0; t0 < kDigestPage; t0 += 16) {
    uint2 w[4];
    float sg[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      w[u] = *reinterpret_cast<const uint2*>(kw + (int64_t)(t0 + 4 * u) * 64);
      sg[u] = ks[t0 + 4 * u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t half = k < 8 ? w[u].x : w[u].y;
        const float v = __fmul_rn(sc[(half >> (4 * (k & 7))) & 15u], sg[u]);
        mn[k] = fminf(mn[k], v);
        mx[k] = fmaxf(mx[k], v);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    mn[k] = fminf(mn[k], __shfl_xor_sync(0xffffffffu, mn[k], 8));
    mn[k] = fminf(mn[k], __shfl_xor_sync(0xffffffffu, mn[k], 16));
    mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 8));
    mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 16));
  }
  if (lt == 0) {
    float4* dg = reinterpret_cast<float4*>(const_cast<uint8_t*>(page) + a.off_dg + hr0 * a.row_dg);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      dg[4 * lw + k] = make_float4(mn[4 * k], mn[4 * k + 1], mn[4 * k + 2], mn[4 * k + 3]);
      dg[32 + 4 * lw + k] = make_float4(mx[4 * k], mx[4 * k + 1], mx[4 * k + 2], mx[4 * k + 3]);
    }
  }
}

// Any other bit width at head_dim 128 / 256 (the tensor-core geometries): a
// warp per (page, head), 4 warps (heads) per block; lane l owns dims
// l + 32 k, reads each token row's words through L1 and keeps the min and
// max of f32(c[code]) * sigma of its dims.
template <int D>
__global__ void __launch_bounds__(128) k_digest_gen(DigestDev a, int heads) {
  constexpr int KD = D / 32;
  __shared__ float sc[256];
  for (int k = threadIdx.x; k < (1 << a.bits); k += blockDim.x) sc[k] = a.cent[k];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + warp;
  if (h >= heads) return;
  const uint8_t* page = reinterpret_cast<const uint8_t*>(a.pages[blockIdx.x]);
  const int64_t hr0 = (int64_t)h * kPageTokens + a.row0[blockIdx.x];
  const int cpw = 64 / a.bits;
  const uint64_t cmask = (1ull << a.bits) - 1ull;
  int wi[KD], sh[KD];
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    const int d = lane + 32 * k;
    wi[k] = d / cpw;
    sh[k] = (d % cpw) * a.bits;
  }
  float mn[KD], mx[KD];
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    mn[k] = FLT_MAX;
    mx[k] = -FLT_MAX;
  }
  const float* ks = reinterpret_cast<const float*>(page + a.off_ks) + hr0;
#pragma unroll 2
  for (int t = 0; t < kDigestPage; ++t) {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(page + a.off_kw + (hr0 + t) * a.row_kw);
    const float sg = ks[t];
#pragma unroll
    for (int k = 0; k < KD; ++k) {
      const float v = __fmul_rn(sc[(w[wi[k]] >> sh[k]) & cmask], sg);
      mn[k] = fminf(mn[k], v);
      mx[k] = fmaxf(mx[k], v);
    }
  }
  float* dg = reinterpret_cast<float*>(const_cast<uint8_t*>(page) + a.off_dg + hr0 * a.row_dg);
#pragma unroll
  for (int k = 0; k < KD; ++k) {
    dg[lane + 32 * k] = mn[k];
    dg[D + lane + 32 * k] = mx[k];
  }
}

// Query element i of an f32 / bf16 / f16 array.
__device__ __forceinline__ float q_elem(const void* p, int dtype, int64_t i) {
  if (dtype == LC_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == LC_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// A bound as an unsigned key of the same order (-0 taken as +0); pinned
// pages take the largest key.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f == 0.f ? 0.f : f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
constexpr uint32_t kPinnedKey = 0xFFFFFFFFu;
constexpr int kSelThreads = 512;
constexpr int kSelStages = 4;  // digest ring stages (8 x head_dim bytes) per warp: 3 in flight ahead

__device__ __forceinline__ void sel_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void sel_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void sel_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// One CTA per (sequence, kv head), head_dim D = 128 or 256, G <= 4:
//   1. q' = R q for the G query heads (q as given unless already rotated),
//      split into its positive and negative parts: the bound of a page is
//      max_g sum_d (q'+_d max_d + q'-_d min_d), the same sum as
//      sum_d max(q'_d max_d, q'_d min_d) since max_d >= min_d;
//   2. bounds: a warp per page, its digest streamed into a per-warp ring
//      by cp.async 3 pages ahead; lane l takes dims l + 32 j, whose q'+ and
//      q'- for every head it keeps in registers;
//   3. the keep-th largest key by a 4-pass radix select over bytes, and how
//      many keys equal to it are taken (lowest pages first);
//   4. the chosen pages' tiles in ascending order (per-warp chunks with
//      prefix offsets), then the undigested tail.
// The decode that follows is launched programmatically: its prologue reads
// nothing this kernel writes and may start on SMs this grid has left.
template <int D>
__global__ void __launch_bounds__(kSelThreads, D == 128 ? 2 : 1) k_page_select(SelectDev a) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int NT = kSelThreads, KD = D / 32, PGF = 2 * D;  // dims per lane, digest floats per page
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.x / a.hkv, kvh = blockIdx.x % a.hkv;
  const int G = a.G, tid = threadIdx.x;
  const int64_t n = a.seqinfo[2 * b];
  const uint64_t* trow = a.table + a.seqinfo[2 * b + 1] * a.table_stride;
  const int P = (int)(n / kDigestPage);
  // pages kept: sparse_keep_pages, or all of them below the key threshold
  int keep = P / 8 > 64 ? P / 8 : 64;
  if (n < kSparseMinKeys || P <= keep) keep = P;
  int32_t* out = a.tile_map + (int64_t)blockIdx.x * a.map_stride;
  if (keep == P) {  // dense: the identity map over every tile
    const int t1 = (int)((n + kTileTokens - 1) / kTileTokens);
    for (int t = tid; t < t1; t += NT) out[t] = t;
    return;
  }
  float* qp = reinterpret_cast<float*>(sm);  // [G][D] positive part of q'
  float* qn = qp + G * D;                     // [G][D] negative part
  float* qx = qn + G * D;                     // [G][D] the queries as given
  float* ring = qx + G * D;                   // [warps][kSelStages][2 D] digest pages
  uint32_t* key = reinterpret_cast<uint32_t*>(ring + (kSelThreads / 32) * kSelStages * PGF);  // [npad]
  uint64_t* pg = reinterpret_cast<uint64_t*>(key + ((a.npad + 1) & ~1));  // [npad / 4] page addresses
  float* red = reinterpret_cast<float*>(pg + a.npad / kGroupsPerPage + 1);    // [4][G][D] rotation partials
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[2];

  const int64_t q0 = ((int64_t)b * a.hq + (int64_t)kvh * G) * D;
  for (int i = tid; i < G * D; i += NT) qx[i] = q_elem(a.q, a.q_dtype, q0 + i);
  for (int i = tid; i < (P + kGroupsPerPage - 1) / kGroupsPerPage; i += NT) pg[i] = trow[i];
  __syncthreads();

  // the first digest pages of every warp go out before the rotation
  const int lane = tid & 31, warp = tid >> 5;
  constexpr int NW = NT / 32;
  const int K = warp < P ? (P - warp + NW - 1) / NW : 0;  // pages of this warp: warp + 16 k
  float* wring = ring + warp * kSelStages * PGF;
  const uint32_t ring0 = (uint32_t)__cvta_generic_to_shared(wring);
  auto live_page = [&](int p) { return p >= kSparseSink && p < P - kSparseRecent; };
  auto issue = [&](int k) {
    const int p = warp + NW * k;
    if (k < K && live_page(p)) {
      const uint8_t* dg = reinterpret_cast<const uint8_t*>(pg[p / kGroupsPerPage]) + a.off_dg +
                          ((int64_t)kvh * kPageTokens + (p % kGroupsPerPage) * kDigestPage) * a.row_dg;
      const uint32_t dst = ring0 + (k % kSelStages) * PGF * 4;
#pragma unroll
      for (int o = 0; o < PGF * 4; o += 512) sel_cp16(dst + o + lane * 16, dg + o + lane * 16);
    }
  };
#pragma unroll
  for (int k = 0; k < kSelStages - 1; ++k) {
    issue(k);
    sel_commit();
  }

  // q'_i = sum_j R[i][j] q_j: thread t sums j in [32 (t / 128), + 32) for
  // output dim i = t % 128 of every head (its 32 loads of R^T in flight
  // together, coalesced); the 4 partial sums are added through shared memory
  constexpr int NS = NT / D, SL = D / NS;  // slices of the sum over j, and their length
  if (!a.q_rotated) {
    const int i = tid % D, js = tid / D;
    float sg4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c0 = 0; c0 < SL; c0 += 32) {
      float rv[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) rv[u] = a.RT[(SL * js + c0 + u) * D + i];
#pragma unroll
      for (int g = 0; g < 4; ++g)
        if (g < G) {
#pragma unroll
          for (int u = 0; u < 32; ++u) sg4[g] = fmaf(rv[u], qx[g * D + SL * js + c0 + u], sg4[g]);
        }
    }
    for (int g = 0; g < G; ++g) red[(js * G + g) * D + i] = sg4[g];
    __syncthreads();
  }
  for (int r = tid; r < G * D; r += NT) {
    float s = 0.f;
    if (a.q_rotated) {
      s = qx[r];
    } else if constexpr (NS == 4) {
      s = (red[r] + red[G * D + r]) + (red[2 * G * D + r] + red[3 * G * D + r]);
    } else {
#pragma unroll
      for (int k = 0; k < NS; ++k) s += red[k * G * D + r];
    }
    qp[r] = fmaxf(s, 0.f);
    qn[r] = fminf(s, 0.f);
  }
  __syncthreads();

  // bounds: a warp per page; each page's digest (min[D] then max[D], 8 D
  // bytes) streams into the warp's ring by cp.async, kSelStages - 1 pages
  // ahead; lane l takes dims l + 32 j, whose q'+ and q'- for every head stay
  // in registers for the whole loop
  float rp[4][KD], rn[4][KD];  // [head][j]
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int j = 0; j < KD; ++j) {
      const int gg = g < G ? g : 0;  // heads past G repeat head 0: the max is unchanged
      rp[g][j] = qp[gg * D + lane + 32 * j];
      rn[g][j] = qn[gg * D + lane + 32 * j];
    }
  const bool hi = (lane & 16) != 0, mid = (lane & 8) != 0;
  for (int k = 0; k < K; ++k) {
    issue(k + kSelStages - 1);  // into the stage read at k - 1
    sel_commit();
    sel_wait<kSelStages - 1>();  // page k has landed
    __syncwarp();
    const int p = warp + NW * k;
    if (live_page(p)) {
      const float* st = wring + (k % kSelStages) * PGF;
      float sg[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < KD; ++j) {
        const float mn = st[lane + 32 * j], mx = st[D + lane + 32 * j];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          sg[g] = fmaf(rp[g][j], mx, sg[g]);
          sg[g] = fmaf(rn[g][j], mn, sg[g]);
        }
      }
      // transposed reduction: lane bit 4 keeps heads {0,1} or {2,3}, bit 3
      // one of the pair; then the sum over the other lanes, the max over heads
      float a0 = hi ? sg[2] : sg[0], a1 = hi ? sg[3] : sg[1];
      a0 += __shfl_xor_sync(0xffffffffu, hi ? sg[0] : sg[2], 16);
      a1 += __shfl_xor_sync(0xffffffffu, hi ? sg[1] : sg[3], 16);
      float v = mid ? a1 : a0;
      v += __shfl_xor_sync(0xffffffffu, mid ? a0 : a1, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
      v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
      if (lane == 0) key[p] = order_key(v);
    } else if (lane == 0) {
      key[p] = kPinnedKey;
    }
    __syncwarp();  // the stage is read before it is refilled
  }
  sel_wait<0>();
  __syncthreads();
  // radix select: T = the keep-th largest key; need = how many keys equal
  // to T are taken. Warp 0 scans the 256 bins from the top, lane l owning
  // bins 255 - 8l .. 248 - 8l.
  uint32_t prefix = 0, pmask = 0, need = (uint32_t)keep;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    __syncthreads();
    for (int i0 = warp * 32; i0 < P; i0 += NT) {
      const int i = i0 + lane;
      const uint32_t k = i < P ? key[i] : 0u;
      const bool in = i < P && (k & pmask) == prefix;
      const unsigned act = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t bin = (k >> shift) & 255u;
        const unsigned peers = __match_any_sync(act, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
      }
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t h[8], sum = 0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        h[u] = hist[255 - 8 * lane - u];
        sum += h[u];
      }
      uint32_t inc = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += t;
      }
      uint32_t cum = inc - sum;
      if (cum < need && inc >= need) {  // the bin holding the need-th key is this lane's
        bool found = false;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (!found && cum + h[u] >= need) {
            sel[0] = (uint32_t)(255 - 8 * lane - u);
            sel[1] = need - cum;
            found = true;
          }
          cum += h[u];
        }
      }
    }
    __syncthreads();
    prefix |= sel[0] << shift;
    pmask |= 255u << shift;
    need = sel[1];
  }
  // the chosen pages (key > T, and the first `need` keys equal to T in page
  // order) in ascending order, 32 pages per warp chunk: chunk counts of
  // ties, then of chosen pages, each turned into offsets by warp 0 (the
  // ring area is free now)
  const uint32_t T = prefix;
  const int nch = (P + 31) >> 5;
  uint32_t* c_eq = reinterpret_cast<uint32_t*>(ring);  // [nch] ties, then their offsets
  uint32_t* c_on = c_eq + nch;                         // [nch] chosen, then their offsets
  auto scan = [&](uint32_t* c) {                       // exclusive prefix sum by warp 0
    uint32_t carry = 0;
    for (int c0 = 0; c0 < nch; c0 += 32) {
      const uint32_t v = c0 + lane < nch ? c[c0 + lane] : 0u;
      uint32_t inc = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += t;
      }
      if (c0 + lane < nch) c[c0 + lane] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
  };
  const unsigned below = (1u << lane) - 1u;
  for (int ch = warp; ch < nch; ch += NW) {
    const int p = 32 * ch + lane;
    const bool eq = p < P && key[p] == T;
    const unsigned em = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) c_eq[ch] = (uint32_t)__popc(em);
  }
  __syncthreads();
  if (warp == 0) scan(c_eq);
  __syncthreads();
  for (int ch = warp; ch < nch; ch += NW) {
    const int p = 32 * ch + lane;
    const uint32_t k = p < P ? key[p] : 0u;
    const bool eq = p < P && k == T;
    const unsigned em = __ballot_sync(0xffffffffu, eq);
    const bool on = p < P && (k > T || (eq && c_eq[ch] + (uint32_t)__popc(em & below) < need));
    const unsigned m = __ballot_sync(0xffffffffu, on);
    if (lane == 0) c_on[ch] = (uint32_t)__popc(m);
  }
  __syncthreads();
  if (warp == 0) scan(c_on);
  __syncthreads();
  for (int ch = warp; ch < nch; ch += NW) {
    const int p = 32 * ch + lane;
    const uint32_t k = p < P ? key[p] : 0u;
    const bool eq = p < P && k == T;
    const unsigned em = __ballot_sync(0xffffffffu, eq);
    const bool on = p < P && (k > T || (eq && c_eq[ch] + (uint32_t)__popc(em & below) < need));
    const unsigned m = __ballot_sync(0xffffffffu, on);
    if (on) {
      const int pos = (int)c_on[ch] + __popc(m & below);
      out[2 * pos] = 2 * p;  // rows of tile_map need not be 8-byte aligned
      out[2 * pos + 1] = 2 * p + 1;
    }
  }
  // the undigested tail, after the keep chosen pages: tiles from the first
  // token past the full pages
  const int t0 = 2 * P, t1 = (int)((n + kTileTokens - 1) / kTileTokens);
  for (int t = t0 + tid; t < t1; t += NT) out[2 * keep + (t - t0)] = t;
}

}  // namespace

void launch_digest(const DigestDev& a, int64_t n_items, int heads, cudaStream_t s) {
  if (n_items <= 0) return;
  // page-sparse decode takes the fast-path geometry only (lc_decode_attn
  // refuses the rest before digesting)
  const dim3 grid((unsigned)n_items, (unsigned)((heads + 3) / 4));
  if (a.bits == 4 && a.dim == 128 && a.row_kw == 64) k_digest4<<<grid, 128, 0, s>>>(a, heads);
  else if (a.dim == 128 && a.bits <= 8) k_digest_gen<128><<<grid, 128, 0, s>>>(a, heads);
  else if (a.dim == 256 && a.bits <= 8) k_digest_gen<256><<<grid, 128, 0, s>>>(a, heads);
  else LC_THROW(LC_ERR_INVALID, "page digest: head_dim 128 or 256");
  LC_CUDA(cudaGetLastError());
}

template <int D>
static void launch_select_d(const SelectDev& a, cudaStream_t s) {
  const size_t smem = (size_t)3 * a.G * D * 4 + (size_t)(kSelThreads / 32) * kSelStages * 2 * D * 4 +
                      (size_t)((a.npad + 1) & ~1) * 4 + (size_t)(a.npad / kGroupsPerPage + 1) * 8 +
                      (size_t)4 * a.G * D * 4;
  static size_t max_dyn = 0;  // 227 KB less the static histogram
  if (max_dyn == 0) {
    cudaFuncAttributes fa;
    LC_CUDA(cudaFuncGetAttributes(&fa, k_page_select<D>));
    max_dyn = 227 * 1024 - fa.sharedSizeBytes;
    LC_CUDA(cudaFuncSetAttribute(k_page_select<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dyn));
  }
  LC_REQUIRE(smem <= max_dyn, LC_ERR_INVALID, "page-sparse decode: too many pages for one selection block");
  k_page_select<D><<<(unsigned)(a.n_seqs * a.hkv), kSelThreads, smem, s>>>(a);
  LC_CUDA(cudaGetLastError());
}

void launch_page_select(const SelectDev& a, cudaStream_t s) {
  LC_REQUIRE((a.dim == 128 || a.dim == 256) && a.G >= 1 && a.G <= 4, LC_ERR_INVALID,
             "page-sparse decode: head_dim 128 or 256, GQA <= 4");
  if (a.dim == 128) launch_select_d<128>(a, s);
  else launch_select_d<256>(a, s);
}

}  // namespace lc
