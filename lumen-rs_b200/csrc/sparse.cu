// Page-sparse decode over the codes (LC_STORE_DIGEST / LC_SPARSE_PAGES):
// the PageDigest of crates/lumen-mlx/src/native_cache.rs:350-445 and the page
// selection of sdpa_page_sparse (native_attention.rs:217-329), with the keys
// taken as the decode sees them: rotated and dequantized, c[code] * sigma.
//
//   k_digest       min and max over each full 64-token page, per head and dim,
//                  into the page's digest role (64 rows of head_dim / 8 bytes:
//                  min[D] f32 then max[D] f32)
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

__device__ __forceinline__ int code_of(const uint64_t* words, int j, int bits) {
  const int cpw = 64 / bits;
  return (int)((words[j / cpw] >> ((j % cpw) * bits)) & ((1ull << bits) - 1));
}

// One CTA (head_dim threads) per (page group, head): item k of the list is
// page address pages[k], first row row0[k] (a multiple of 64) within it.
__global__ void k_digest(DigestDev a) {
  const int64_t item = blockIdx.x;
  const int h = blockIdx.y;
  const int d = threadIdx.x;
  const uint8_t* page = reinterpret_cast<const uint8_t*>(a.pages[item]);
  const int row0 = a.row0[item];
  float mn = FLT_MAX, mx = -FLT_MAX;
  for (int t = 0; t < kDigestPage; ++t) {
    const int64_t hr = (int64_t)h * kPageTokens + row0 + t;
    const uint64_t* words = reinterpret_cast<const uint64_t*>(page + a.off_kw + hr * a.row_kw);
    const float sigma = *reinterpret_cast<const float*>(page + a.off_ks + hr * 4);
    const float v = __fmul_rn(a.cent[code_of(words, d, a.bits)], sigma);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  float* dg = reinterpret_cast<float*>(const_cast<uint8_t*>(page) + a.off_dg +
                                       ((int64_t)h * kPageTokens + row0) * a.row_dg);
  dg[d] = mn;
  dg[a.dim + d] = mx;
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

// One CTA per (sequence, kv head), head_dim 128, G <= 4:
//   1. q' = R q for the G query heads (q as given unless already rotated),
//      split into its positive and negative parts: the bound of a page is
//      max_g sum_d (q'+_d max_d + q'-_d min_d), the same sum as
//      sum_d max(q'_d max_d, q'_d min_d) since max_d >= min_d;
//   2. bounds: 8 lanes per page (float4 columns 4c + 32j of min and max),
//      4 pages per warp pass;
//   3. the keep-th largest key by a 4-pass radix select over bytes, and how
//      many keys equal to it are taken (lowest pages first);
//   4. warp 0 writes the chosen pages' tiles in ascending order, then the
//      undigested tail.
// The decode that follows is launched programmatically: its prologue reads
// nothing this kernel writes and may start on SMs this grid has left.
__global__ void __launch_bounds__(kSelThreads, 2) k_page_select(SelectDev a) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int D = 128, NT = kSelThreads;
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
  uint32_t* key = reinterpret_cast<uint32_t*>(qx + G * D);                // [npad]
  uint64_t* pg = reinterpret_cast<uint64_t*>(key + ((a.npad + 1) & ~1));  // [npad / 4] page addresses
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[2];

  const int64_t q0 = ((int64_t)b * a.hq + (int64_t)kvh * G) * D;
  for (int i = tid; i < G * D; i += NT) qx[i] = q_elem(a.q, a.q_dtype, q0 + i);
  for (int i = tid; i < (P + kGroupsPerPage - 1) / kGroupsPerPage; i += NT) pg[i] = trow[i];
  __syncthreads();
  // q'_i = sum_j R[i][j] q_j: thread t takes output dim i = t % 128 of heads
  // t / 128, t / 128 + 4, ...; RT = R^T keeps each step's reads coalesced
  for (int r = tid; r < G * D; r += NT) {
    const int g = r / D, i = r % D;
    float s = 0.f;
    if (a.q_rotated) {
      s = qx[r];
    } else {
#pragma unroll 16
      for (int j = 0; j < D; ++j) s = fmaf(a.RT[j * D + i], qx[g * D + j], s);
    }
    qp[r] = fmaxf(s, 0.f);
    qn[r] = fminf(s, 0.f);
  }
  __syncthreads();

  const int lane = tid & 31, warp = tid >> 5;
  const int sub = lane >> 3, c = lane & 7;
  for (int p0 = warp * 4; p0 < P; p0 += (NT / 32) * 4) {
    const int p = p0 + sub;
    const bool live = p < P && p >= kSparseSink && p < P - kSparseRecent;
    const float4* dg =
        live ? reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(pg[p / kGroupsPerPage]) + a.off_dg +
                                               ((int64_t)kvh * kPageTokens + (p % kGroupsPerPage) * kDigestPage) *
                                                   a.row_dg)
             : nullptr;
    float4 mn[4], mx[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      mn[j] = live ? dg[c + 8 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
      mx[j] = live ? dg[D / 4 + c + 8 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float bound = -FLT_MAX;
    for (int g = 0; g < G; ++g) {
      const float4* p4 = reinterpret_cast<const float4*>(qp + g * D);
      const float4* n4 = reinterpret_cast<const float4*>(qn + g * D);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 u = p4[c + 8 * j], v = n4[c + 8 * j];
        s = fmaf(u.x, mx[j].x, s);
        s = fmaf(u.y, mx[j].y, s);
        s = fmaf(u.z, mx[j].z, s);
        s = fmaf(u.w, mx[j].w, s);
        s = fmaf(v.x, mn[j].x, s);
        s = fmaf(v.y, mn[j].y, s);
        s = fmaf(v.z, mn[j].z, s);
        s = fmaf(v.w, mn[j].w, s);
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      bound = fmaxf(bound, s);
    }
    if (c == 0 && p < P) key[p] = live ? order_key(bound) : kPinnedKey;
  }
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
  if (warp == 0) {
    const uint32_t T = prefix;
    int j = 0;             // chosen pages written so far
    uint32_t eq_seen = 0;  // keys equal to T met so far
    for (int p0 = 0; p0 < P; p0 += 32) {
      const int p = p0 + lane;
      const uint32_t k = p < P ? key[p] : 0u;
      const bool eq = p < P && k == T;
      const unsigned em = __ballot_sync(0xffffffffu, eq);
      const uint32_t eq_rank = eq_seen + (uint32_t)__popc(em & ((1u << lane) - 1u));
      const bool on = p < P && (k > T || (eq && eq_rank < need));
      const unsigned m = __ballot_sync(0xffffffffu, on);
      if (on) {
        const int pos = j + __popc(m & ((1u << lane) - 1u));
        out[2 * pos] = 2 * p;  // rows of tile_map need not be 8-byte aligned
        out[2 * pos + 1] = 2 * p + 1;
      }
      eq_seen += (uint32_t)__popc(em);
      j += __popc(m);
    }
    // the undigested tail: tiles from the first token past the full pages
    const int t0 = 2 * P, t1 = (int)((n + kTileTokens - 1) / kTileTokens);
    for (int t = t0 + lane; t < t1; t += 32) out[2 * j + (t - t0)] = t;
  }
}

}  // namespace

void launch_digest(const DigestDev& a, int64_t n_items, int heads, cudaStream_t s) {
  if (n_items <= 0) return;
  k_digest<<<dim3((unsigned)n_items, (unsigned)heads), a.dim, 0, s>>>(a);
  LC_CUDA(cudaGetLastError());
}

void launch_page_select(const SelectDev& a, cudaStream_t s) {
  LC_REQUIRE(a.dim == 128 && a.G >= 1 && a.G <= 4, LC_ERR_INVALID, "page-sparse decode: head_dim 128, GQA <= 4");
  const size_t smem = (size_t)3 * a.G * a.dim * 4 + (size_t)((a.npad + 1) & ~1) * 4 +
                      (size_t)(a.npad / kGroupsPerPage + 1) * 8;
  static size_t max_dyn = 0;  // 227 KB less the static histogram
  if (max_dyn == 0) {
    cudaFuncAttributes fa;
    LC_CUDA(cudaFuncGetAttributes(&fa, k_page_select));
    max_dyn = 227 * 1024 - fa.sharedSizeBytes;
    LC_CUDA(cudaFuncSetAttribute(k_page_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_dyn));
  }
  LC_REQUIRE(smem <= max_dyn, LC_ERR_INVALID, "page-sparse decode: too many pages for one selection block");
  k_page_select<<<(unsigned)(a.n_seqs * a.hkv), kSelThreads, smem, s>>>(a);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
