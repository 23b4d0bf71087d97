// The KVCache trait's per-head calls, computed on the GPU in the reference's
// exact f32 order (explicit round-to-nearest ops, sequential sums), so they
// agree bit-for-bit with turboquant-cache's SimpleCache:
//   attend_keys   -> estimate_inner_products_stage1 (compressor.rs:165-184)
//   attend_keys_qjl -> estimate_inner_products      (compressor.rs:122-159)
//   attend_values -> accumulate_weighted_value      (simple.rs:76-99, 142-155)
// These are parity hooks: one (layer, head) at a time, latency-bound. The
// throughput path is the fused split-K decode in decode.cu.
#include <cmath>

#include "kernels.h"

namespace lc {

namespace {

struct HookDev {
  CodecDev c;
  const uint64_t* pages;
  int64_t off_w, off_s;
  int64_t row_w;
  int head;
  int64_t n;
  // QJL stage 2 (attend_keys_qjl): sign words, residual norm
  int64_t off_q = 0, off_r = 0, row_q = 0;
  float sqrt_half_pi = 0.f, sqrt_m = 0.f;  // f32 sqrt(pi/2), sqrt(m), computed on the host
};

__device__ __forceinline__ int code_at(const uint64_t* words, int j, int bits) {
  const int cpw = 64 / bits;
  return (int)((words[j / cpw] >> ((j % cpw) * bits)) & ((1ull << bits) - 1));
}

__device__ __forceinline__ const uint8_t* row_ptr(const HookDev& h, int64_t off, int64_t row_bytes, int64_t t) {
  const uint8_t* page = reinterpret_cast<const uint8_t*>(h.pages[t >> 8]);
  return page + off + ((int64_t)h.head * kPageTokens + (t & 255)) * row_bytes;
}

// rq[i] = sum_j R[i][j] * q[j], j ascending, from -0.0 (rotation.rs:91-99).
__global__ void k_rotate_strict(const float* q, const float* RT, int D, float* rq) {
  const int i = threadIdx.x;
  float acc = -0.0f;
  for (int j = 0; j < D; ++j) acc = __fadd_rn(acc, __fmul_rn(RT[(int64_t)j * D + i], q[j]));
  rq[i] = acc;
}

// pq[r] = sum_j Phi[r][j] * q[j], j ascending, from -0.0 (qjl.rs:76-84).
__global__ void k_project_strict(const float* q, const float* PT, int D, int m, float* pq) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m) return;
  float acc = -0.0f;
  for (int j = 0; j < D; ++j) acc = __fadd_rn(acc, __fmul_rn(PT[(int64_t)j * m + r], q[j]));
  pq[r] = acc;
}

// estimate_inner_products (compressor.rs:122-159): the stage-1 score of
// k_attend_keys plus estimate_correction_from_projection (qjl.rs:86-119):
// sum over rows r ascending of sign_r * pq[r] from 0.0, times
// ||r|| * sqrt(pi/2) / sqrt(m); 0 when ||r|| < 1e-10.
__global__ void k_attend_keys_qjl(HookDev h, const float* rq, const float* pq, float* scores) {
  extern __shared__ float sm[];
  const int D = h.c.dim, m = h.c.m;
  float* srq = sm;
  float* spq = sm + D;
  for (int j = threadIdx.x; j < D; j += blockDim.x) srq[j] = rq[j];
  for (int r = threadIdx.x; r < m; r += blockDim.x) spq[r] = pq[r];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= h.n) return;
  const uint64_t* words = reinterpret_cast<const uint64_t*>(row_ptr(h, h.off_w, h.row_w, t));
  const float sigma = *reinterpret_cast<const float*>(row_ptr(h, h.off_s, 4, t));
  float acc = -0.0f;
  for (int j = 0; j < D; ++j) acc = __fadd_rn(acc, __fmul_rn(srq[j], h.c.cent[code_at(words, j, h.c.bits)]));
  const float stage1 = __fmul_rn(acc, sigma);
  const uint64_t* signs = reinterpret_cast<const uint64_t*>(row_ptr(h, h.off_q, h.row_q, t));
  const float rnorm = *reinterpret_cast<const float*>(row_ptr(h, h.off_r, 4, t));
  float stage2 = 0.0f;
  if (!(rnorm < 1e-10f)) {
    float sum = 0.0f;
    for (int r = 0; r < m; ++r) {
      const float sg = ((signs[r >> 6] >> (r & 63)) & 1ull) ? 1.0f : -1.0f;
      sum = __fadd_rn(sum, __fmul_rn(sg, spq[r]));
    }
    stage2 = __fmul_rn(__fdiv_rn(__fmul_rn(rnorm, h.sqrt_half_pi), h.sqrt_m), sum);
  }
  scores[t] = __fadd_rn(stage1, stage2);
}

__global__ void k_attend_keys(HookDev h, const float* rq, float* scores) {
  extern __shared__ float srq[];
  const int D = h.c.dim;
  for (int j = threadIdx.x; j < D; j += blockDim.x) srq[j] = rq[j];
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= h.n) return;
  const uint64_t* words = reinterpret_cast<const uint64_t*>(row_ptr(h, h.off_w, h.row_w, t));
  const float sigma = *reinterpret_cast<const float*>(row_ptr(h, h.off_s, 4, t));
  float acc = -0.0f;
  for (int j = 0; j < D; ++j) acc = __fadd_rn(acc, __fmul_rn(srq[j], h.c.cent[code_at(words, j, h.c.bits)]));
  scores[t] = __fmul_rn(acc, sigma);
}

// One CTA of D threads; token t's dequantized*scaled values are staged in
// shared memory by thread j, then thread i accumulates R[j][i]*y_j over j.
__global__ void k_attend_values(HookDev h, const float* w, float* out) {
  extern __shared__ float sy[];
  const int D = h.c.dim;
  const int i = threadIdx.x;
  float acc = 0.0f;
  for (int64_t t = 0; t < h.n; ++t) {
    const float wt = w[t];
    if (fabsf(wt) < 1e-10f) continue;  // uniform across the CTA
    const uint64_t* words = reinterpret_cast<const uint64_t*>(row_ptr(h, h.off_w, h.row_w, t));
    const float sigma = *reinterpret_cast<const float*>(row_ptr(h, h.off_s, 4, t));
    const float sc = __fmul_rn(sigma, wt);
    __syncthreads();
    sy[i] = __fmul_rn(h.c.cent[code_at(words, i, h.c.bits)], sc);
    __syncthreads();
    for (int j = 0; j < D; ++j) acc = __fadd_rn(acc, __fmul_rn(h.c.R[(int64_t)j * D + i], sy[j]));
  }
  out[i] = acc;
}

HookDev make_hook(const CodecDev& c, const uint64_t* pages, const PageLayout& L, int role_w, int role_s, int head,
                  int64_t n) {
  HookDev h;
  h.c = c;
  h.pages = pages;
  h.off_w = L.off[role_w];
  h.off_s = L.off[role_s];
  h.row_w = L.row[role_w];
  h.head = head;
  h.n = n;
  return h;
}

}  // namespace

void launch_attend_keys(const float* q, const CodecDev& kc, const uint64_t* pages, const PageLayout& L, int role_kw,
                        int role_ks, int head, int64_t n, float* rq_scratch, float* scores, cudaStream_t s) {
  k_rotate_strict<<<1, kc.dim, 0, s>>>(q, kc.RT, kc.dim, rq_scratch);
  LC_CUDA(cudaGetLastError());
  if (n <= 0) return;
  const HookDev h = make_hook(kc, pages, L, role_kw, role_ks, head, n);
  const int threads = 128;
  k_attend_keys<<<(unsigned)((n + threads - 1) / threads), threads, kc.dim * sizeof(float), s>>>(h, rq_scratch,
                                                                                                  scores);
  LC_CUDA(cudaGetLastError());
}

void launch_attend_keys_qjl(const float* q, const CodecDev& kc, const uint64_t* pages, const PageLayout& L,
                            int role_kw, int role_ks, int role_kq, int role_kr, int head, int64_t n,
                            float* rq_scratch, float* pq_scratch, float* scores, cudaStream_t s) {
  LC_REQUIRE(kc.m > 0 && kc.PT, LC_ERR_STATE, "codec has no QJL projection");
  k_rotate_strict<<<1, kc.dim, 0, s>>>(q, kc.RT, kc.dim, rq_scratch);
  LC_CUDA(cudaGetLastError());
  k_project_strict<<<(kc.m + 127) / 128, 128, 0, s>>>(q, kc.PT, kc.dim, kc.m, pq_scratch);
  LC_CUDA(cudaGetLastError());
  if (n <= 0) return;
  HookDev h = make_hook(kc, pages, L, role_kw, role_ks, head, n);
  h.off_q = L.off[role_kq];
  h.row_q = L.row[role_kq];
  h.off_r = L.off[role_kr];
  h.sqrt_half_pi = std::sqrt((float)1.5707963267948966);  // f32 FRAC_PI_2, then sqrt (qjl.rs:116)
  h.sqrt_m = std::sqrt((float)kc.m);
  const int threads = 128;
  k_attend_keys_qjl<<<(unsigned)((n + threads - 1) / threads), threads, (kc.dim + kc.m) * sizeof(float), s>>>(
      h, rq_scratch, pq_scratch, scores);
  LC_CUDA(cudaGetLastError());
}

void launch_attend_values(const float* w, const CodecDev& vc, const uint64_t* pages, const PageLayout& L,
                          int role_vw, int role_vs, int head, int64_t n, float* out, cudaStream_t s) {
  const HookDev h = make_hook(vc, pages, L, role_vw, role_vs, head, n);
  k_attend_values<<<1, vc.dim, vc.dim * sizeof(float), s>>>(h, w, out);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
