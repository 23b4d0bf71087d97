// Page pool, upload arena and the ring bookkeeping (see ring.h), plus the
// lc_ring_* entry points: the reference's rotating buffers over raw rows.
#include "ring.h"

#include <algorithm>
#include <cstring>

#include "kernels.h"

namespace lc {

// ---------------------------------------------------------------- PagePool
PagePool::~PagePool() {
  if (base_) cudaFree(base_);
}

void PagePool::init(const PageLayout& layout, int64_t n_pages, int device, bool zero) {
  LC_REQUIRE(n_pages > 0 && n_pages < (1ll << 31), LC_ERR_INVALID, "page pool size out of range");
  layout_ = layout;
  n_pages_ = n_pages;
  LC_CUDA(cudaSetDevice(device));
  const size_t bytes = (size_t)n_pages * (size_t)layout.page_bytes;
  cudaError_t e = cudaMalloc(&base_, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    LC_THROW(LC_ERR_NOMEM, "page pool: cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  }
  if (zero) LC_CUDA(cudaMemset(base_, 0, bytes));
  free_.resize(n_pages);
  for (int64_t i = 0; i < n_pages; ++i) free_[i] = (int32_t)(n_pages - 1 - i);
  ref_.assign(n_pages, 0);
}

int32_t PagePool::alloc() {
  LC_REQUIRE(!free_.empty(), LC_ERR_NOMEM, "page pool exhausted");
  const int32_t p = free_.back();
  free_.pop_back();
  ref_[p] = 1;
  return p;
}

void PagePool::decref(int32_t p) {
  if (--ref_[p] == 0) free_.push_back(p);
}

// ------------------------------------------------------------- UploadArena
UploadArena::~UploadArena() {
  if (host_) cudaFreeHost(host_);
  if (dev_) cudaFree(dev_);
}

void UploadArena::init(size_t bytes) {
  size_ = bytes;
  LC_CUDA(cudaMallocHost(&host_, bytes));
  LC_CUDA(cudaMalloc(&dev_, bytes));
}

void* UploadArena::put(const void* src, size_t bytes, cudaStream_t stream) {
  const size_t need = (bytes + 255) & ~size_t(255);
  LC_REQUIRE(need <= size_, LC_ERR_NOMEM, "upload larger than the staging arena");
  if (pos_ + need > size_) {
    for (cudaStream_t s : used_) LC_CUDA(cudaStreamSynchronize(s));
    used_.clear();
    pos_ = 0;
  }
  if (bytes) std::memcpy(host_ + pos_, src, bytes);
  void* d = dev_ + pos_;
  if (bytes) LC_CUDA(cudaMemcpyAsync(d, host_ + pos_, bytes, cudaMemcpyHostToDevice, stream));
  used_.insert(stream);
  pos_ += need;
  return d;
}

// ------------------------------------------------------------------- RingOps
static inline int64_t pages_for(int64_t rows) { return (rows + kPageTokens - 1) / kPageTokens; }

std::vector<uint64_t> RingOps::page_addrs(const RingCore& r) const {
  std::vector<uint64_t> a(r.pages.size());
  for (size_t i = 0; i < r.pages.size(); ++i) a[i] = pool->addr(r.pages[i]);
  return a;
}

void RingOps::resize_pages(RingCore& r, int64_t rows) {
  const int64_t want = pages_for(rows);
  while ((int64_t)r.pages.size() > want) {
    pool->decref(r.pages.back());
    r.pages.pop_back();
  }
  while ((int64_t)r.pages.size() < want) r.pages.push_back(pool->alloc());
}

void RingOps::make_private(RingCore& r, int64_t a, int64_t b) {
  if (b <= a) return;
  const int64_t p0 = a / kPageTokens, p1 = std::min<int64_t>(pages_for(b), (int64_t)r.pages.size());
  for (int64_t p = p0; p < p1; ++p) {
    const int32_t old = r.pages[p];
    if (pool->refs(old) > 1) {
      const int32_t fresh = pool->alloc();
      LC_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(pool->addr(fresh)), reinterpret_cast<void*>(pool->addr(old)),
                              pool->layout().page_bytes, cudaMemcpyDeviceToDevice, stream));
      pool->decref(old);
      r.pages[p] = fresh;
    }
  }
}

void RingOps::zero_rows(RingCore& r, int64_t a, int64_t b) {
  if (b <= a) return;
  make_private(r, a, b);
  CopyRowsArgs c;
  c.layout = pool->layout();
  c.dst.pages = arena->put_vec(page_addrs(r), stream);
  c.dst_begin = a;
  c.n = b - a;
  c.zero = 1;
  launch_copy_rows(c, stream);
  if (launches) ++*launches;
}

void RingOps::regather(RingCore& r, const std::vector<int64_t>& src_rows, int64_t n_new) {
  RingCore fresh;
  const int64_t np = pages_for(n_new);
  for (int64_t i = 0; i < np; ++i) fresh.pages.push_back(pool->alloc());
  if (!src_rows.empty()) {
    CopyRowsArgs c;
    c.layout = pool->layout();
    c.src.pages = arena->put_vec(page_addrs(r), stream);
    c.dst.pages = arena->put_vec(page_addrs(fresh), stream);
    c.src_rows = arena->put_vec(src_rows, stream);
    c.dst_begin = 0;
    c.n = (int64_t)src_rows.size();
    launch_copy_rows(c, stream);
    if (launches) ++*launches;
  }
  for (int32_t p : r.pages) pool->decref(p);
  r.pages.swap(fresh.pages);
}

int64_t RingOps::prepare_update(RingCore& r, int64_t S, bool prealloc) {
  LC_REQUIRE(S >= 1, LC_ERR_INVALID, "update needs at least one token");
  if (S == 1 && prealloc) {
    // ---- ring_update_in_place (native_cache.rs:146-231) ----
    const int64_t prev = r.offset;
    const bool need_grow = !r.has || (prev >= r.buf_len && r.buf_len < r.max_size);
    if (need_grow) {
      LC_REQUIRE(prev <= r.max_size, LC_ERR_STATE, "ring grow past max_size");
      const int64_t n = std::min<int64_t>(kPageTokens, r.max_size - prev);
      const int64_t old = r.has ? r.buf_len : 0;
      resize_pages(r, old + n);
      zero_rows(r, old, old + n);
      r.buf_len = old + n;
      r.has = true;
      r.idx = prev;
    }
    if (r.buf_len > r.max_size) {
      const int64_t trim = r.buf_len - r.max_size;
      std::vector<int64_t> rows;
      rows.reserve(r.max_size);
      for (int64_t i = 0; i < r.keep; ++i) rows.push_back(i);
      for (int64_t i = trim + r.keep; i < r.buf_len; ++i) rows.push_back(i);
      regather(r, rows, (int64_t)rows.size());
      r.buf_len = (int64_t)rows.size();
      r.idx = r.max_size;
    }
    if (r.idx == r.max_size) r.idx = r.keep;
    const int64_t w = r.idx;
    make_private(r, w, w + 1);
    r.idx += 1;
    r.offset = prev + 1;
    r.view_len = r.offset >= r.max_size ? r.buf_len : r.offset;
    return w;
  }
  // ---- ring_update_concat / rotating_concat (native_cache.rs:86-125, 240-268) ----
  if (!r.has) {
    resize_pages(r, S);
    r.has = true;
    r.buf_len = S;
    r.offset += S;
    r.idx = S;
    r.view_len = S;
    return 0;
  }
  const int64_t buf = r.buf_len, idx = r.idx, offset = r.offset, keep = r.keep;
  std::vector<int64_t> ordered;
  bool identity = false;
  int64_t id_len = 0;
  if (idx == buf) {
    identity = true;
    id_len = buf;
  } else if (idx < offset) {
    for (int64_t i = 0; i < std::min(keep, buf); ++i) ordered.push_back(i);
    for (int64_t i = idx; i < buf; ++i) ordered.push_back(i);
    for (int64_t i = keep; i < idx; ++i) ordered.push_back(i);
  } else {
    identity = true;
    id_len = std::min(idx, buf);
  }
  if (identity) {
    ordered.resize(id_len);
    for (int64_t i = 0; i < id_len; ++i) ordered[i] = i;
  }
  const int64_t held = (int64_t)ordered.size();
  const int64_t trim = std::max<int64_t>(held + 1 - r.max_size, 0);
  if (trim > 0) {
    std::vector<int64_t> t;
    for (int64_t i = 0; i < std::min(keep, held); ++i) t.push_back(ordered[i]);
    for (int64_t i = trim + keep; i < held; ++i) t.push_back(ordered[i]);
    ordered.swap(t);
    identity = false;
  }
  const int64_t kept = (int64_t)ordered.size();
  const int64_t n_new = kept + S;
  if (identity) {
    resize_pages(r, n_new);
    make_private(r, kept, n_new);
  } else {
    regather(r, ordered, n_new);
  }
  r.buf_len = n_new;
  r.offset = offset + S;
  r.idx = n_new;
  r.view_len = n_new;
  return kept;
}

int64_t RingOps::new_pages_bound(const RingCore& r, int64_t S, bool prealloc) const {
  if (S == 1 && prealloc) {
    int64_t n = 1;  // copy-on-write of the written page
    int64_t buf = r.has ? r.buf_len : 0;
    if (!r.has || (r.offset >= buf && buf < r.max_size)) {
      n += 1;
      buf += std::min<int64_t>(kPageTokens, r.max_size - r.offset);
    }
    if (buf > r.max_size) n += pages_for(r.max_size);  // one-time trim regathers
    return n;
  }
  if (!r.has) return pages_for(S);
  // the same decisions prepare_update takes, without side effects
  const int64_t buf = r.buf_len, idx = r.idx, keep = r.keep;
  int64_t held;
  bool identity = true;
  if (idx == buf) {
    held = buf;
  } else if (idx < r.offset) {
    identity = false;
    held = std::min(keep, buf) + std::max<int64_t>(buf - idx, 0) + std::max<int64_t>(idx - keep, 0);
  } else {
    held = std::min(idx, buf);
  }
  const int64_t trim = std::max<int64_t>(held + 1 - r.max_size, 0);
  if (trim > 0) {
    identity = false;
    held = std::min(keep, held) + std::max<int64_t>(held - trim - keep, 0);
  }
  const int64_t n_new = held + S;
  if (identity) return std::max<int64_t>(pages_for(n_new) - (int64_t)r.pages.size(), 0) + 1;
  return pages_for(n_new);
}

bool RingOps::truncate_to(RingCore& r, int64_t target) {
  if (target > r.offset) return false;
  if (target == r.offset) return true;
  if (r.offset > r.max_size) return false;
  r.offset = target;
  r.idx = target;
  r.view_len = std::min(target, r.buf_len);
  return true;
}

void RingOps::clear(RingCore& r) {
  for (int32_t p : r.pages) pool->decref(p);
  r.pages.clear();
  r.has = false;
  r.buf_len = r.offset = r.idx = r.view_len = 0;
}

RingCore RingOps::deep_clone(const RingCore& r) {
  RingCore c = r;
  c.pages.clear();
  for (size_t i = 0; i < r.pages.size(); ++i) {
    const int32_t p = pool->alloc();
    LC_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(pool->addr(p)), reinterpret_cast<void*>(pool->addr(r.pages[i])),
                            pool->layout().page_bytes, cudaMemcpyDeviceToDevice, stream));
    c.pages.push_back(p);
  }
  return c;
}

RingCore RingOps::share_prefix(const RingCore& src, int64_t n) {
  RingCore c;
  c.max_size = src.max_size;
  c.keep = src.keep;
  if (n <= 0) return c;
  const int64_t np = pages_for(n);
  for (int64_t i = 0; i < np; ++i) {
    pool->incref(src.pages[i]);
    c.pages.push_back(src.pages[i]);
  }
  c.has = true;
  c.buf_len = n;
  c.offset = n;
  c.idx = n;
  c.view_len = n;
  return c;
}

void read_rows(RingOps& ops, const RingCore& r, int64_t row_begin, int64_t n, uint8_t* dev_linear,
               const int64_t* lin_off) {
  if (n <= 0) return;
  CopyRowsArgs c;
  c.layout = ops.pool->layout();
  c.src.pages = ops.arena->put_vec(ops.page_addrs(r), ops.stream);
  c.src_begin = row_begin;
  c.dst.linear = dev_linear;
  for (int k = 0; k < kMaxRoles; ++k) c.dst.lin_off[k] = lin_off[k];
  c.dst.lin_rows = n;
  c.n = n;
  launch_copy_rows(c, ops.stream);
  if (ops.launches) ++*ops.launches;
}

}  // namespace lc

// ================================================================ lc_ring ABI
using namespace lc;

struct lc_ring {
  int device = 0;
  cudaStream_t stream = nullptr;
  PagePool pool;
  UploadArena arena;
  RingCore core;
  RingOps ops;
  uint64_t launches = 0;
  std::vector<int64_t> row_bytes;
  int32_t heads = 0;
  uint8_t* stage = nullptr;  // device staging for updates / reads
  size_t stage_bytes = 0;

  void ensure_stage(size_t bytes) {
    if (bytes <= stage_bytes) return;
    if (stage) {
      LC_CUDA(cudaStreamSynchronize(stream));
      cudaFree(stage);
    }
    LC_CUDA(cudaMalloc(&stage, bytes));
    stage_bytes = bytes;
  }
  ~lc_ring() {
    if (stage) cudaFree(stage);
    if (stream) cudaStreamDestroy(stream);
  }
};

static int64_t ring_pool_pages(int64_t max_size) {
  // Enough for the largest buffer the plans build (a full window plus a chunk)
  // and a regather copy of it.
  const int64_t base = (max_size + kPageTokens - 1) / kPageTokens;
  return std::min<int64_t>(4 * base + 64, 1 << 16);
}

extern "C" {

int lc_ring_create(int32_t n_heads, int64_t max_size, int64_t keep, int32_t n_bufs, const int64_t* row_bytes,
                   int32_t device, lc_ring** out) {
  return abi_guard([&] {
    LC_REQUIRE(out, LC_ERR_INVALID, "null out");
    *out = nullptr;
    LC_REQUIRE(n_heads > 0 && n_bufs > 0 && n_bufs <= kMaxRoles && row_bytes, LC_ERR_INVALID, "bad ring shape");
    LC_REQUIRE(max_size > 0, LC_ERR_INVALID, "max_size must be > 0");
    LC_REQUIRE(keep >= 0 && keep < max_size, LC_ERR_INVALID, "keep must be < max_size");
    std::vector<int64_t> rows(row_bytes, row_bytes + n_bufs);
    for (int64_t rb : rows) LC_REQUIRE(rb > 0, LC_ERR_INVALID, "row_bytes must be > 0");
    auto* r = new lc_ring;
    try {
      r->device = device;
      LC_CUDA(cudaSetDevice(device));
      LC_CUDA(cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking));
      r->row_bytes = rows;
      r->heads = n_heads;
      r->pool.init(PageLayout::make(n_heads, rows), ring_pool_pages(max_size), device, false);
      r->arena.init(4 << 20);
      r->core.max_size = max_size;
      r->core.keep = keep;
      r->ops.pool = &r->pool;
      r->ops.arena = &r->arena;
      r->ops.stream = r->stream;
      r->ops.launches = &r->launches;
    } catch (...) {
      delete r;
      throw;
    }
    *out = r;
  });
}

int lc_ring_update(lc_ring* r, const void* const* news, int64_t n_tokens, int32_t prealloc, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(r && news && n_tokens > 0, LC_ERR_INVALID, "bad update arguments");
    LC_CUDA(cudaSetDevice(r->device));
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : r->stream;
    r->ops.stream = s;
    const PageLayout& L = r->pool.layout();
    const int64_t w = r->ops.prepare_update(r->core, n_tokens, prealloc != 0);
    // stage the new rows linearly [role][head][n][row], then scatter
    int64_t lin_off[kMaxRoles] = {};
    size_t total = 0;
    for (int k = 0; k < L.n_roles; ++k) {
      lin_off[k] = (int64_t)total;
      total += (size_t)L.heads * n_tokens * L.row[k];
      total = (total + 255) & ~size_t(255);
    }
    r->ensure_stage(total);
    for (int k = 0; k < L.n_roles; ++k) {
      LC_REQUIRE(news[k], LC_ERR_INVALID, "null buffer in update");
      const size_t bytes = (size_t)L.heads * n_tokens * L.row[k];
      LC_CUDA(cudaMemcpyAsync(r->stage + lin_off[k], news[k], bytes, cudaMemcpyDefault, s));
    }
    CopyRowsArgs c;
    c.layout = L;
    c.src.linear = r->stage;
    for (int k = 0; k < kMaxRoles; ++k) c.src.lin_off[k] = lin_off[k];
    c.src.lin_rows = n_tokens;
    c.src_begin = 0;
    c.dst.pages = r->arena.put_vec(r->ops.page_addrs(r->core), s);
    c.dst_begin = w;
    c.n = n_tokens;
    launch_copy_rows(c, s);
    ++r->launches;
    LC_CUDA(cudaStreamSynchronize(s));
    r->ops.stream = r->stream;
  });
}

int lc_ring_truncate_to(lc_ring* r, int64_t target) {
  return abi_guard([&] {
    LC_REQUIRE(r, LC_ERR_INVALID, "null ring");
    if (!r->ops.truncate_to(r->core, target)) {
      if (target > r->core.offset)
        LC_THROW(LC_ERR_REFUSED, "truncate_to: target " + std::to_string(target) + " > offset " +
                                     std::to_string(r->core.offset));
      LC_THROW(LC_ERR_REFUSED, "truncate_to: post-rotation rollback not supported (offset=" +
                                   std::to_string(r->core.offset) + " > max_size=" + std::to_string(r->core.max_size) +
                                   ")");
    }
  });
}

int lc_ring_counters(const lc_ring* r, int64_t* offset, int64_t* idx, int64_t* buf_len, int64_t* view_len) {
  return abi_guard([&] {
    LC_REQUIRE(r, LC_ERR_INVALID, "null ring");
    if (offset) *offset = r->core.offset;
    if (idx) *idx = r->core.idx;
    if (buf_len) *buf_len = r->core.has ? r->core.buf_len : 0;
    if (view_len) *view_len = r->core.view_len;
  });
}

int lc_ring_read(lc_ring* r, int32_t buf, int32_t which, void* dst, int64_t dst_bytes, int64_t* n_out) {
  return abi_guard([&] {
    LC_REQUIRE(r, LC_ERR_INVALID, "null ring");
    const PageLayout& L = r->pool.layout();
    LC_REQUIRE(buf >= 0 && buf < L.n_roles, LC_ERR_INVALID, "buffer index out of range");
    LC_REQUIRE(r->core.has, LC_ERR_STATE, "ring holds no buffers");
    LC_CUDA(cudaSetDevice(r->device));
    const int64_t n = which == LC_FETCH_BACKING ? r->core.buf_len : r->core.view_len;
    if (n_out) *n_out = n;
    const size_t bytes = (size_t)L.heads * n * L.row[buf];
    if (n == 0) return;
    LC_REQUIRE(dst && (int64_t)bytes <= dst_bytes, LC_ERR_INVALID, "destination too small");
    r->ensure_stage(bytes);
    int64_t lin_off[kMaxRoles] = {};
    CopyRowsArgs c;
    c.layout = L;
    c.src.pages = r->arena.put_vec(r->ops.page_addrs(r->core), r->stream);
    c.dst.linear = r->stage;
    for (int k = 0; k < kMaxRoles; ++k) c.dst.lin_off[k] = lin_off[k];
    c.dst.lin_rows = n;
    c.n = n;
    c.role_mask = 1u << buf;
    launch_copy_rows(c, r->stream);
    ++r->launches;
    LC_CUDA(cudaMemcpyAsync(dst, r->stage, bytes, cudaMemcpyDefault, r->stream));
    LC_CUDA(cudaStreamSynchronize(r->stream));
  });
}

int lc_ring_clear(lc_ring* r) {
  return abi_guard([&] {
    LC_REQUIRE(r, LC_ERR_INVALID, "null ring");
    r->ops.clear(r->core);
  });
}

int lc_ring_deep_clone(const lc_ring* r, lc_ring** out) {
  return abi_guard([&] {
    LC_REQUIRE(r && out, LC_ERR_INVALID, "null argument");
    *out = nullptr;
    lc_ring* c = nullptr;
    const int st = lc_ring_create(r->heads, r->core.max_size, r->core.keep, (int32_t)r->row_bytes.size(),
                                  r->row_bytes.data(), r->device, &c);
    if (st != LC_OK) LC_THROW(st, lc_last_error());
    try {
      // copy pages across pools (same layout)
      RingCore nc = r->core;
      nc.pages.clear();
      for (size_t i = 0; i < r->core.pages.size(); ++i) {
        const int32_t p = c->pool.alloc();
        LC_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(c->pool.addr(p)),
                                reinterpret_cast<void*>(r->pool.addr(r->core.pages[i])), r->pool.layout().page_bytes,
                                cudaMemcpyDeviceToDevice, c->stream));
        nc.pages.push_back(p);
      }
      c->core = nc;
      LC_CUDA(cudaStreamSynchronize(c->stream));
    } catch (...) {
      lc_ring_destroy(c);
      throw;
    }
    *out = c;
  });
}

void lc_ring_destroy(lc_ring* r) {
  if (!r) return;
  cudaSetDevice(r->device);
  if (r->stream) cudaStreamSynchronize(r->stream);
  delete r;
}

}  // extern "C"
