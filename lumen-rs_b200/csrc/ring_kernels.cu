// Row copies for the paged ring: grow (zero-fill), trim/reorder (gather),
// write of new rows from a linear staging buffer and read-back for fetch.
// Byte work, HBM-bound: one thread per 4-byte word of a (row, head, role).
#include "kernels.h"

namespace lc {

namespace {

struct CopyRowsDev {
  RowSpace src, dst;
  int32_t heads, n_roles;
  int64_t off[kMaxRoles];
  int64_t row[kMaxRoles];
  const int64_t* src_rows;
  int64_t src_begin, dst_begin, n;
  int32_t zero;
  uint32_t role_mask;
};

__device__ __forceinline__ uint8_t* row_addr(const RowSpace& sp, const CopyRowsDev& a, int role, int h,
                                             int64_t r) {
  if (sp.pages) {
    uint8_t* page = reinterpret_cast<uint8_t*>(sp.pages[r >> 8]);
    return page + a.off[role] + ((int64_t)h * kPageTokens + (r & 255)) * a.row[role];
  }
  return sp.linear + sp.lin_off[role] + ((int64_t)h * sp.lin_rows + r) * a.row[role];
}

// grid: x over (row i, head) pairs; y over roles. Each thread block-strides
// over the 4-byte words (or bytes for odd widths) of its rows.
__global__ void k_copy_rows(CopyRowsDev a) {
  const int role = blockIdx.y;
  if (!((a.role_mask >> role) & 1u)) return;
  const int64_t rb = a.row[role];
  const bool words = (rb & 3) == 0;
  const int64_t units = words ? rb / 4 : rb;
  const int64_t total = a.n * a.heads * units;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = u % units;
    const int64_t ih = u / units;
    const int h = (int)(ih % a.heads);
    const int64_t i = ih / a.heads;
    uint8_t* d = row_addr(a.dst, a, role, h, a.dst_begin + i);
    if (a.zero) {
      if (words) reinterpret_cast<uint32_t*>(d)[k] = 0u;
      else d[k] = 0;
      continue;
    }
    const int64_t sr = a.src_rows ? a.src_rows[i] : a.src_begin + i;
    const uint8_t* s = row_addr(a.src, a, role, h, sr);
    if (words) reinterpret_cast<uint32_t*>(d)[k] = reinterpret_cast<const uint32_t*>(s)[k];
    else d[k] = s[k];
  }
}

}  // namespace

void launch_copy_rows(const CopyRowsArgs& a, cudaStream_t s) {
  if (a.n <= 0) return;
  CopyRowsDev d;
  d.src = a.src;
  d.dst = a.dst;
  d.heads = a.layout.heads;
  d.n_roles = a.layout.n_roles;
  for (int r = 0; r < kMaxRoles; ++r) {
    d.off[r] = a.layout.off[r];
    d.row[r] = a.layout.row[r];
  }
  d.src_rows = a.src_rows;
  d.src_begin = a.src_begin;
  d.dst_begin = a.dst_begin;
  d.n = a.n;
  d.zero = a.zero;
  d.role_mask = a.role_mask;
  int64_t max_units = 0;
  for (int r = 0; r < d.n_roles; ++r) {
    int64_t u = (d.row[r] & 3) == 0 ? d.row[r] / 4 : d.row[r];
    max_units = max_units > u ? max_units : u;
  }
  int64_t total = a.n * d.heads * max_units;
  int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  dim3 grid((unsigned)blocks, (unsigned)d.n_roles);
  k_copy_rows<<<grid, threads, 0, s>>>(d);
  LC_CUDA(cudaGetLastError());
}

}  // namespace lc
