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

// Bitonic sort of n (a power of two) (key, index) pairs in shared memory:
// key descending, index ascending on equal keys.
__device__ void bitonic_desc(float* key, int32_t* idx, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;  // this block sorts descending when up
          const float ki = key[i], kj = key[j];
          const int32_t ii = idx[i], ij = idx[j];
          const bool i_first = ki > kj || (ki == kj && ii < ij);
          if (up ? !i_first : i_first) {
            key[i] = kj;
            key[j] = ki;
            idx[i] = ij;
            idx[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
}

__global__ void k_page_select(SelectDev a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int b = blockIdx.x / a.hkv, kvh = blockIdx.x % a.hkv;
  const int D = a.dim, G = a.G;
  float* qs = reinterpret_cast<float*>(sm);  // [G][D]
  float* key = qs + G * D;                    // [npad]
  int32_t* idx = reinterpret_cast<int32_t*>(key + a.npad);
  uint64_t* pg = reinterpret_cast<uint64_t*>(idx + a.npad);  // [npad / 4] page addresses
  const int64_t n = a.seqinfo[2 * b];
  const uint64_t* trow = a.table + a.seqinfo[2 * b + 1] * a.table_stride;
  const int P = (int)(n / kDigestPage);
  // pages kept: sparse_keep_pages, or all of them below the key threshold
  int keep = P / 8 > 64 ? P / 8 : 64;
  if (n < kSparseMinKeys || P <= keep) keep = P;
  int32_t* out = a.tile_map + (int64_t)blockIdx.x * a.map_stride;
  if (keep == P) {  // dense: the identity map over every tile
    const int t1 = (int)((n + kTileTokens - 1) / kTileTokens);
    for (int t = threadIdx.x; t < t1; t += blockDim.x) out[t] = t;
    return;
  }
  for (int i = threadIdx.x; i < G * D; i += blockDim.x)
    qs[i] = a.q_rot[((int64_t)b * a.hq + (int64_t)kvh * G) * D + i];
  for (int i = threadIdx.x; i < (P + kGroupsPerPage - 1) / kGroupsPerPage; i += blockDim.x) pg[i] = trow[i];
  __syncthreads();
  // bounds: a warp takes 4 pages per round trip; lane l holds dims l + 32 j
  // of each page's min and max, read once for all G query heads
  constexpr int kPer = 4, kDj = 4;  // pages per pass; dims per lane (head_dim 128)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int p0 = warp * kPer; p0 < a.npad; p0 += nw * kPer) {
    float mn[kPer][kDj], mx[kPer][kDj];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int p = p0 + u;
      const bool live = p < P && p >= kSparseSink && p < P - kSparseRecent;
      const float* dg = live ? reinterpret_cast<const float*>(
                                   reinterpret_cast<const uint8_t*>(pg[p / kGroupsPerPage]) + a.off_dg +
                                   ((int64_t)kvh * kPageTokens + (p % kGroupsPerPage) * kDigestPage) * a.row_dg)
                             : nullptr;
#pragma unroll
      for (int j = 0; j < kDj; ++j) {
        const int d = lane + 32 * j;
        mn[u][j] = live && d < D ? dg[d] : 0.f;
        mx[u][j] = live && d < D ? dg[D + d] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int p = p0 + u;
      float bound = -FLT_MAX;
      for (int g = 0; g < G; ++g) {
        float sacc = 0.f;
#pragma unroll
        for (int j = 0; j < kDj; ++j) {
          const int d = lane + 32 * j;
          const float q = d < D ? qs[g * D + d] : 0.f;
          sacc += q > 0.f ? q * mx[u][j] : q * mn[u][j];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, off);
        bound = fmaxf(bound, sacc);
      }
      if (p < P && (p < kSparseSink || p >= P - kSparseRecent)) bound = FLT_MAX;  // pinned
      if (p >= P) bound = -FLT_MAX;                                             // padding
      if (lane == 0 && p < a.npad) {
        key[p] = bound;
        idx[p] = p;
      }
    }
  }
  __syncthreads();
  bitonic_desc(key, idx, a.npad);
  // flag the keep chosen pages (key[] reused), then warp 0 compacts them in
  // ascending page order: ballot + popcount per 32 pages
  int32_t* flag = reinterpret_cast<int32_t*>(key);
  for (int i = threadIdx.x; i < a.npad; i += blockDim.x) flag[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < keep; i += blockDim.x) flag[idx[i]] = 1;
  __syncthreads();
  if (warp == 0) {
    int j = 0;  // chosen pages written so far
    for (int p0 = 0; p0 < P; p0 += 32) {
      const int p = p0 + lane;
      const bool on = p < P && flag[p];
      const unsigned m = __ballot_sync(0xffffffffu, on);
      if (on) {
        const int pos = j + __popc(m & ((1u << lane) - 1u));
        out[2 * pos] = 2 * p;
        out[2 * pos + 1] = 2 * p + 1;
      }
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
  LC_REQUIRE(a.dim <= 128, LC_ERR_INVALID, "page-sparse decode: head_dim <= 128");
  const size_t smem = (size_t)a.G * a.dim * 4 + (size_t)a.npad * 8 + (size_t)(a.npad / kGroupsPerPage + 1) * 8;
  static bool attr = false;
  if (!attr) {
    LC_CUDA(cudaFuncSetAttribute(k_page_select, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr = true;
  }
  LC_REQUIRE(smem <= 227 * 1024, LC_ERR_INVALID, "page-sparse decode: too many pages for one selection block");
  k_page_select<<<(unsigned)(a.n_seqs * a.hkv), 1024, smem, s>>>(a);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
