// Paged device storage and the mlx-lm rotating-ring bookkeeping over it.
//
// Every cache buffer is "logical rows" (tokens) of fixed width per (head,
// role). Logical row r lives in page pages[r / 256] at row r % 256. The
// ring semantics (grow by 256, one-time trim, wrap to `keep`, temporal
// reorder on multi-token updates, rollback refusals) are those of
// crates/lumen-mlx/src/native_cache.rs:65-335; only the placement of rows
// in memory differs (pages instead of one contiguous MLX array), which is
// invisible through fetch.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <set>
#include <vector>

#include "common.h"

namespace lc {

// Fixed-size pages from one device allocation, with reference counts so a
// page can be shared by several sequences (prefix reuse) and copied on the
// first write.
class PagePool {
 public:
  PagePool() = default;
  PagePool(const PagePool&) = delete;
  PagePool& operator=(const PagePool&) = delete;
  ~PagePool();
  void init(const PageLayout& layout, int64_t n_pages, int device, bool zero);
  int32_t alloc();
  void incref(int32_t p) { ref_[p]++; }
  void decref(int32_t p);
  int32_t refs(int32_t p) const { return ref_[p]; }
  uint64_t addr(int32_t p) const { return reinterpret_cast<uint64_t>(base_) + (uint64_t)p * layout_.page_bytes; }
  const PageLayout& layout() const { return layout_; }
  int64_t free_pages() const { return (int64_t)free_.size(); }
  int64_t capacity() const { return n_pages_; }

 private:
  PageLayout layout_;
  uint8_t* base_ = nullptr;
  int64_t n_pages_ = 0;
  std::vector<int32_t> free_;
  std::vector<int32_t> ref_;
};

// Pinned host + device bump arena for small per-call uploads (page address
// lists, row maps, write plans). Wrapping synchronises the streams that used
// it, so a pending copy never reads host bytes that were rewritten.
class UploadArena {
 public:
  ~UploadArena();
  void init(size_t bytes);
  // Copies `bytes` from `src` to the device on `stream`; returns the device address.
  void* put(const void* src, size_t bytes, cudaStream_t stream);
  template <class T>
  T* put_vec(const std::vector<T>& v, cudaStream_t s) {
    return static_cast<T*>(put(v.data(), v.size() * sizeof(T), s));
  }

 private:
  uint8_t* host_ = nullptr;
  uint8_t* dev_ = nullptr;
  size_t size_ = 0, pos_ = 0;
  std::set<cudaStream_t> used_;
};

// One ring: the reference's (offset, idx, max_size, keep) plus the page list
// standing in for the MLX arrays.
struct RingCore {
  int64_t max_size = 0, keep = 0;
  bool has = false;  // buffers exist (the reference's Option::Some)
  std::vector<int32_t> pages;
  int64_t buf_len = 0;   // logical backing length (cached_len)
  int64_t offset = 0;    // tokens ever pushed
  int64_t idx = 0;       // write index
  int64_t view_len = 0;  // rows the last update returned
};

// Device operations on rings that share one pool.
struct RingOps {
  PagePool* pool = nullptr;
  UploadArena* arena = nullptr;
  cudaStream_t stream = nullptr;
  uint64_t* launches = nullptr;  // kernel launch counter

  // ring_update (native_cache.rs:277-290) up to the write: grows, trims,
  // reorders as the reference does and returns the first logical row of the
  // S new tokens (rows [w, w+S) are private pages, ready to be written).
  int64_t prepare_update(RingCore& r, int64_t S, bool prealloc);
  // Upper bound on the fresh pages prepare_update(r, S, prealloc) can take.
  int64_t new_pages_bound(const RingCore& r, int64_t S, bool prealloc) const;
  // ring_truncate (native_cache.rs:304-335); false where the reference errs.
  bool truncate_to(RingCore& r, int64_t target);
  void clear(RingCore& r);
  // Device page addresses covering rows [0, rows).
  std::vector<uint64_t> page_addrs(const RingCore& r) const;
  // Copy-on-write every page touching rows [a, b).
  void make_private(RingCore& r, int64_t a, int64_t b);
  // Deep copy into fresh pages.
  RingCore deep_clone(const RingCore& r);
  // Share the first n rows of src (pages incref'd): counters = n.
  RingCore share_prefix(const RingCore& src, int64_t n);

 private:
  void resize_pages(RingCore& r, int64_t rows);
  void zero_rows(RingCore& r, int64_t a, int64_t b);
  // Rebuild r's buffer as rows src_rows (old logical indices), new length n_new >= src_rows.size().
  void regather(RingCore& r, const std::vector<int64_t>& src_rows, int64_t n_new);
};

// Linear staging of a ring's rows: role-major [role][head][n][row].
void read_rows(RingOps& ops, const RingCore& r, int64_t row_begin, int64_t n, uint8_t* dev_linear,
               const int64_t* lin_off);

}  // namespace lc
