// lc_cache: the TurboQuant KV cache on one GPU.
//
// State per (sequence, layer) is one RingCore (the reference's
// NativeRotatingKvCacheTurboQuant bookkeeping, native_cache.rs:1517-1862)
// over pages of one shared pool. A page holds 256 tokens of every kv head
// of a layer for each role:
//   0 K code words  [H][256][words_K] u64     (bitpack.rs layout)
//   1 V code words  [H][256][words_V] u64
//   2 K sigma       [H][256] f32
//   3 V sigma       [H][256] f32
//   4 K QJL words   [H][256][ceil(m/64)] u64  (LC_STORE_K_QJL)
//   5 K residual    [H][256] f32
//   6 V QJL words, 7 V residual               (LC_STORE_V_QJL)
// Full layers (the reference's append-only TurboQuant layers, keep = 0) use
// an unbounded ring; sliding layers use (max_size, keep). Prefix reuse shares
// pages between sequences and copies a page on its first write.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <ctime>
#include <memory>

#include "codec.h"
#include "group.h"
#include "kernels.h"
#include "lkv2.h"
#include "ring.h"

namespace lc {

namespace {
constexpr int64_t kFullMax = int64_t(1) << 50;  // "never wraps"
constexpr int R_KW = 0, R_VW = 1, R_KS = 2, R_VS = 3, R_KQ = 4, R_KR = 5, R_VQ = 6, R_VR = 7;

struct SeqLayer {
  RingCore ring;
  std::vector<int64_t> head_len;  // non-empty: per-head lengths (KVCache::store on a full layer)
  bool dirty = true;              // device block-table row out of date
  int64_t digested = 0;           // 64-token pages whose digest is up to date (LC_STORE_DIGEST)
};

template <class T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  void ensure(size_t want, cudaStream_t s) {
    if (want <= n) return;
    if (p) {
      LC_CUDA(cudaStreamSynchronize(s));
      cudaFree(p);
      p = nullptr;
    }
    const size_t grow = std::max(want, n + n / 2);
    cudaError_t e = cudaMalloc(&p, grow * sizeof(T));
    if (e != cudaSuccess) {
      cudaGetLastError();
      n = 0;
      LC_THROW(LC_ERR_NOMEM, "scratch allocation failed");
    }
    n = grow;
  }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};
}  // namespace

}  // namespace lc

using namespace lc;

struct lc_cache {
  lc_cache_config cfg{};
  std::vector<int64_t> max_size, keep;
  Codec kc, vc;
  CodecOnDevice dk, dv;
  PageLayout layout;
  PagePool pool;
  UploadArena arena;
  RingOps ops;
  cudaStream_t stream = nullptr;
  uint64_t launches = 0;
  std::vector<SeqLayer> st;  // [seq * n_layers + layer]
  int32_t role_dg = -1;       // page digest role (LC_STORE_DIGEST)
  uint64_t* d_table = nullptr;  // [n_layers][max_seqs][max_pages_per_seq]
  cudaEvent_t ev_copy = nullptr;
  DevBuf<uint8_t> in_k, in_v, qbuf, outbuf, fetchbuf;
  DevBuf<float> q_rot, part, hook_a, hook_b, hook_c, q_proj, q_step;
  DevBuf<__half> q_h;
  DevBuf<int32_t> ctr;  // fused decode arrival counters (zero between launches)
  DevBuf<int32_t> tile_map;  // page-sparse decode: logical -> physical tiles
  std::vector<uint8_t> blob;  // host staging of one call's metadata
  // kernel timing (lc_cache_timing)
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> t_decode, t_append, t_other;

  cudaEvent_t take_event() {
    if (ev_used == ev_pool.size()) {
      cudaEvent_t e;
      LC_CUDA(cudaEventCreate(&e));
      ev_pool.push_back(e);
    }
    return ev_pool[ev_used++];
  }
  // Records an event pair around f() on stream s when timing is on.
  template <class F>
  void timed(std::vector<std::pair<cudaEvent_t, cudaEvent_t>>& rec, cudaStream_t s, F&& f) {
    if (!timing) {
      f();
      return;
    }
    cudaEvent_t a = take_event(), b = take_event();
    LC_CUDA(cudaEventRecord(a, s));
    f();
    LC_CUDA(cudaEventRecord(b, s));
    rec.emplace_back(a, b);
  }

  SeqLayer& at(int32_t seq, int32_t layer) { return st[(size_t)seq * cfg.n_layers + layer]; }
  const SeqLayer& at(int32_t seq, int32_t layer) const { return st[(size_t)seq * cfg.n_layers + layer]; }
  bool full(int32_t layer) const { return max_size[layer] >= kFullMax; }
  void check(int32_t seq, int32_t layer) const {
    LC_REQUIRE(seq >= 0 && seq < cfg.max_seqs, LC_ERR_INVALID, "sequence id out of range");
    LC_REQUIRE(layer >= 0 && layer < cfg.n_layers, LC_ERR_INVALID, "layer out of range");
  }
  uint64_t* table_row(int32_t seq, int32_t layer) const {
    return d_table + ((size_t)layer * cfg.max_seqs + seq) * cfg.max_pages_per_seq;
  }
  cudaStream_t pick(void* s) const { return s ? static_cast<cudaStream_t>(s) : stream; }
  // V's R (row-major) / R^T for the output's un-rotation, or null when the
  // caller keeps the output rotated or V is stored un-rotated
  bool out_unrotated(uint32_t flags) const {
    return (flags & LC_OUT_ROTATED) || (cfg.store_flags & LC_STORE_V_UNROTATED);
  }
  const float* v_R(uint32_t flags) const { return out_unrotated(flags) ? nullptr : dv.R; }
  const float* v_RT(uint32_t flags) const { return out_unrotated(flags) ? nullptr : dv.RTd; }

  // Device work on the cache is serialised across streams: before work on
  // `s`, wait for everything issued on the stream used last.
  cudaStream_t last = nullptr;
  cudaEvent_t ev_order = nullptr;
  void order(cudaStream_t s) {
    if (last && last != s) {
      LC_CUDA(cudaEventRecord(ev_order, last));
      LC_CUDA(cudaStreamWaitEvent(s, ev_order, 0));
    }
    last = s;
  }

  // Upload (seq, layer)'s page addresses if they changed.
  void sync_table(int32_t seq, int32_t layer, cudaStream_t s) {
    SeqLayer& sl = at(seq, layer);
    if (!sl.dirty) return;
    LC_REQUIRE((int64_t)sl.ring.pages.size() <= cfg.max_pages_per_seq, LC_ERR_NOMEM,
               "sequence longer than max_pages_per_seq pages");
    const std::vector<uint64_t> addrs = ops.page_addrs(sl.ring);
    if (!addrs.empty()) {
      void* src = arena.put(addrs.data(), addrs.size() * 8, s);
      LC_CUDA(cudaMemcpyAsync(table_row(seq, layer), src, addrs.size() * 8, cudaMemcpyDeviceToDevice, s));
    }
    sl.dirty = false;
  }

  // Device pointer for a caller buffer: device memory is used in place, host
  // memory is copied into `buf`.
  const void* stage_in(const void* p, size_t bytes, DevBuf<uint8_t>& buf, cudaStream_t s, bool& host) {
    host = !is_device_ptr(p);
    if (!host) return p;
    buf.ensure(bytes, s);
    LC_CUDA(cudaMemcpyAsync(buf.p, p, bytes, cudaMemcpyHostToDevice, s));
    return buf.p;
  }

  ~lc_cache() {
    if (last) cudaStreamSynchronize(last);
    if (stream) cudaStreamSynchronize(stream);
    if (ev_order) cudaEventDestroy(ev_order);
    for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
    if (d_table) cudaFree(d_table);
    if (ev_copy) cudaEventDestroy(ev_copy);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace {

size_t dtype_size(int32_t dt) {
  if (dt == LC_F32) return 4;
  if (dt == LC_BF16 || dt == LC_F16) return 2;
  LC_THROW(LC_ERR_INVALID, "unknown dtype");
}

// Build the quantize-append for rows already prepared in the rings.
// RoPE of lc_append_rope: positions, dims and table of one call.
struct RopeArgs {
  int32_t dims = 0;  // rotated leading dims (even, <= head_dim)
  double base = 10000.0;
  int32_t traditional = 0;
  std::vector<float> cs;  // [n_seqs * n_tok][dims / 2][cos, sin]
};

// A decode step's queries for the append launch to rotate (lc_decode_step).
struct StepQ {
  const void* q = nullptr;  // device rows [rows][head_dim]
  int32_t dtype = LC_F32, rows = 0;
  float* out = nullptr;     // device [rows][head_dim] f32: R q
};

void run_append(lc_cache* c, int32_t n_seqs, int32_t h_in, int32_t h_base, int64_t n_tok,
                const std::vector<uint64_t>& dst_page, const std::vector<int32_t>& dst_row, const void* k,
                const void* v, int32_t dtype, cudaStream_t s, const RopeArgs* rope = nullptr,
                const StepQ* sq = nullptr) {
  AppendArgs a;
  if (sq) {
    a.q = sq->q;
    a.q_dtype = sq->dtype;
    a.q_rows = sq->rows;
    a.q_out = sq->out;
  }
  if (rope) {
    a.rope_cs = static_cast<const float*>(c->arena.put(rope->cs.data(), rope->cs.size() * sizeof(float), s));
    a.rope_half = rope->dims / 2;
    a.rope_traditional = rope->traditional;
  }
  a.codec[0] = c->dk.view();
  a.codec[1] = c->dv.view();
  a.src[0] = k;
  a.src[1] = v;
  a.dtype = dtype;
  a.n_seqs = n_seqs;
  a.h_in = h_in;
  a.h_base = h_base;
  a.n_tok = n_tok;
  if ((int64_t)dst_page.size() <= kAppendInline) {  // decode steps: in the launch parameters
    a.h_page = dst_page.data();
    a.h_row = dst_row.data();
  } else {
    // one upload: [page addresses u64 | rows i32]
    const size_t n = dst_page.size();
    std::vector<uint8_t>& blob = c->blob;
    blob.resize(n * 12);
    std::memcpy(blob.data(), dst_page.data(), n * 8);
    std::memcpy(blob.data() + n * 8, dst_row.data(), n * 4);
    const uint8_t* d = static_cast<const uint8_t*>(c->arena.put(blob.data(), blob.size(), s));
    a.dst_page = reinterpret_cast<const uint64_t*>(d);
    a.dst_row = reinterpret_cast<const int32_t*>(d + n * 8);
  }
  a.layout = c->layout;
  a.role_words[0] = R_KW;
  a.role_words[1] = R_VW;
  a.role_sigma[0] = R_KS;
  a.role_sigma[1] = R_VS;
  if (c->cfg.store_flags & LC_STORE_K_QJL) {
    a.role_qjl[0] = R_KQ;
    a.role_rnorm[0] = R_KR;
  }
  if (c->cfg.store_flags & LC_STORE_V_QJL) {
    a.role_qjl[1] = R_VQ;
    a.role_rnorm[1] = R_VR;
  }
  c->timed(c->t_append, s, [&] { launch_append(a, s); });
  ++c->launches;
}

}  // namespace

extern "C" {

int lc_cache_create(const lc_cache_config* cfg, const lc_codec* kcodec, const lc_codec* vcodec, lc_cache** out) {
  return abi_guard([&] {
    LC_REQUIRE(cfg && kcodec && vcodec && out, LC_ERR_INVALID, "null argument");
    *out = nullptr;
    LC_REQUIRE(cfg->n_layers > 0 && cfg->n_kv_heads > 0 && cfg->max_seqs > 0 && cfg->max_pages > 0 &&
                   cfg->max_pages_per_seq > 0,
               LC_ERR_INVALID, "cache config sizes must be > 0");
    LC_REQUIRE((uint64_t)cfg->head_dim == kcodec->c.dim && (uint64_t)cfg->head_dim == vcodec->c.dim, LC_ERR_INVALID,
               "codec head_dim differs from config head_dim");
    LC_REQUIRE(kcodec->c.bits >= 2 && kcodec->c.bits <= 8 && vcodec->c.bits >= 2 && vcodec->c.bits <= 8,
               LC_ERR_BITS, "cache bits must be in [2, 8] (native_cache.rs:1546-1549)");
    if (cfg->store_flags & LC_STORE_K_QJL) LC_REQUIRE(kcodec->c.m > 0, LC_ERR_INVALID, "K QJL needs qjl_m > 0");
    if (cfg->store_flags & LC_STORE_V_QJL) LC_REQUIRE(vcodec->c.m > 0, LC_ERR_INVALID, "V QJL needs qjl_m > 0");
    std::unique_ptr<lc_cache> c(new lc_cache);
    c->cfg = *cfg;
    c->cfg.layer_max_size = nullptr;
    c->cfg.layer_keep = nullptr;
    for (int32_t l = 0; l < cfg->n_layers; ++l) {
      int64_t ms = cfg->layer_max_size ? cfg->layer_max_size[l] : 0;
      int64_t kp = cfg->layer_keep ? cfg->layer_keep[l] : 0;
      if (ms == 0) {
        ms = kFullMax;
        kp = 0;
      }
      LC_REQUIRE(ms > 0, LC_ERR_INVALID, "TurboQuant cache: max_size must be > 0");
      LC_REQUIRE(kp >= 0 && kp < ms, LC_ERR_INVALID, "TurboQuant cache: keep must be < max_size");
      c->max_size.push_back(ms);
      c->keep.push_back(kp);
    }
    c->kc = kcodec->c;
    c->vc = vcodec->c;
    if (cfg->store_flags & LC_STORE_V_UNROTATED) {  // V quantized as it is: R = I
      const size_t d = c->vc.dim;
      c->vc.R.assign(d * d, 0.0f);
      for (size_t i = 0; i < d; ++i) c->vc.R[i * d + i] = 1.0f;
    }
    LC_CUDA(cudaSetDevice(cfg->device));
    LC_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    LC_CUDA(cudaEventCreateWithFlags(&c->ev_copy, cudaEventDisableTiming));
    LC_CUDA(cudaEventCreateWithFlags(&c->ev_order, cudaEventDisableTiming));
    c->dk.upload(c->kc);
    c->dv.upload(c->vc);
    const int64_t H = cfg->n_kv_heads;
    std::vector<int64_t> rows = {(int64_t)c->kc.words() * 8, (int64_t)c->vc.words() * 8, 4, 4};
    if (cfg->store_flags & (LC_STORE_K_QJL | LC_STORE_V_QJL)) {
      rows.push_back((cfg->store_flags & LC_STORE_K_QJL) ? (int64_t)c->kc.qwords() * 8 : 8);
      rows.push_back(4);
    }
    if (cfg->store_flags & LC_STORE_V_QJL) {
      rows.push_back((int64_t)c->vc.qwords() * 8);
      rows.push_back(4);
    }
    if (cfg->store_flags & LC_STORE_DIGEST) {
      // 64 rows of head_dim / 8 bytes per 64-token page and head: min[D], max[D] f32
      LC_REQUIRE(cfg->head_dim % 64 == 0, LC_ERR_INVALID, "LC_STORE_DIGEST needs head_dim % 64 == 0");
      c->role_dg = (int32_t)rows.size();
      rows.push_back((int64_t)cfg->head_dim / 8);
    }
    c->layout = PageLayout::make((int32_t)H, rows);
    c->pool.init(c->layout, cfg->max_pages, cfg->device, true);
    c->arena.init(16 << 20);
    c->ops.pool = &c->pool;
    c->ops.arena = &c->arena;
    c->ops.stream = c->stream;
    c->ops.launches = &c->launches;
    c->st.resize((size_t)cfg->max_seqs * cfg->n_layers);
    for (int32_t s = 0; s < cfg->max_seqs; ++s)
      for (int32_t l = 0; l < cfg->n_layers; ++l) {
        c->at(s, l).ring.max_size = c->max_size[l];
        c->at(s, l).ring.keep = c->keep[l];
      }
    const size_t tbytes = (size_t)cfg->n_layers * cfg->max_seqs * cfg->max_pages_per_seq * 8;
    LC_CUDA(cudaMalloc(&c->d_table, tbytes));
    LC_CUDA(cudaMemset(c->d_table, 0, tbytes));
    *out = c.release();
  });
}

void lc_cache_destroy(lc_cache* c) {
  if (!c) return;
  cudaSetDevice(c->cfg.device);
  delete c;
}

int lc_cache_info(const lc_cache* c, int32_t* device, void** stream, uint64_t* kernel_launches) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    if (device) *device = c->cfg.device;
    if (stream) *stream = c->stream;
    if (kernel_launches) *kernel_launches = c->launches;
  });
}

int lc_cache_timing(lc_cache* c, int32_t mode, double* decode_ms, uint64_t* decode_launches, double* append_ms,
                    uint64_t* append_launches, double* other_ms) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    LC_REQUIRE(mode >= 0 && mode <= 2, LC_ERR_INVALID, "timing mode must be 0, 1 or 2");
    if (mode == 1) {
      c->t_decode.clear();
      c->t_append.clear();
      c->t_other.clear();
      c->ev_used = 0;
      c->timing = true;
      return;
    }
    auto sum = [](const std::vector<std::pair<cudaEvent_t, cudaEvent_t>>& v) {
      double ms = 0;
      for (const auto& p : v) {
        LC_CUDA(cudaEventSynchronize(p.second));
        float t = 0;
        LC_CUDA(cudaEventElapsedTime(&t, p.first, p.second));
        ms += t;
      }
      return ms;
    };
    if (decode_ms) *decode_ms = sum(c->t_decode);
    if (decode_launches) *decode_launches = c->t_decode.size();
    if (append_ms) *append_ms = sum(c->t_append);
    if (append_launches) *append_launches = c->t_append.size();
    if (other_ms) *other_ms = sum(c->t_other);
    if (mode == 0) c->timing = false;
  });
}

static void append_impl(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
                        const void* values, int32_t dtype, int64_t n_tokens, void* stream, RopeArgs* rope,
                        const StepQ* sq = nullptr) {
  {
    LC_REQUIRE(c && seq_ids && keys && values, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_seqs > 0 && n_tokens > 0, LC_ERR_INVALID, "n_seqs and n_tokens must be > 0");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->pick(stream);
    c->order(s);
    c->ops.stream = s;
    const size_t esz = dtype_size(dtype);
    const int32_t H = c->cfg.n_kv_heads;
    std::vector<uint64_t> dst_page((size_t)n_seqs * n_tokens);
    std::vector<int32_t> dst_row((size_t)n_seqs * n_tokens);
    // Validate everything and bound the pages this call may take before any
    // ring moves, so a refused call leaves the cache unchanged.
    int64_t need = 0;
    for (int32_t b = 0; b < n_seqs; ++b) {
      const int32_t seq = seq_ids[b];
      c->check(seq, layer);
      for (int32_t b2 = 0; b2 < b; ++b2) LC_REQUIRE(seq_ids[b2] != seq, LC_ERR_INVALID, "duplicate sequence id");
      const SeqLayer& sl = c->at(seq, layer);
      if (!sl.head_len.empty())
        for (int64_t hl : sl.head_len)
          LC_REQUIRE(hl == sl.head_len[0], LC_ERR_STATE, "heads of this layer hold different lengths");
      need += c->ops.new_pages_bound(sl.ring, n_tokens, c->cfg.step_prealloc != 0);
      const int64_t held = sl.ring.has ? std::max(sl.ring.buf_len, sl.ring.offset) : 0;
      const int64_t rows = std::min(held + std::max<int64_t>(n_tokens, kPageTokens), sl.ring.max_size - 1 + n_tokens);
      LC_REQUIRE((rows + kPageTokens - 1) / kPageTokens <= c->cfg.max_pages_per_seq, LC_ERR_NOMEM,
                 "append would exceed max_pages_per_seq pages for a sequence");
    }
    LC_REQUIRE(need <= c->pool.free_pages(), LC_ERR_NOMEM,
               "page pool too small for this append (" + std::to_string(c->pool.free_pages()) + " pages free)");
    if (rope) {
      // position of token t of sequence b: tokens the layer held before the
      // call + t; angle pos * base^(-2i/dims) in f64, cos and sin rounded to f32
      const int32_t half = rope->dims / 2;
      rope->cs.assign((size_t)n_seqs * n_tokens * half * 2, 0.f);
      for (int32_t b = 0; b < n_seqs; ++b) {
        const SeqLayer& sl = c->at(seq_ids[b], layer);
        const int64_t pos0 = sl.head_len.empty() ? sl.ring.offset : sl.head_len[0];
        for (int64_t t = 0; t < n_tokens; ++t)
          for (int32_t i = 0; i < half; ++i) {
            const double ang = (double)(pos0 + t) * std::pow(rope->base, -2.0 * i / rope->dims);
            float* e = &rope->cs[(((size_t)b * n_tokens + t) * half + i) * 2];
            e[0] = (float)std::cos(ang);
            e[1] = (float)std::sin(ang);
          }
      }
    }
    for (int32_t b = 0; b < n_seqs; ++b) {
      const int32_t seq = seq_ids[b];
      SeqLayer& sl = c->at(seq, layer);
      sl.head_len.clear();
      if (!c->full(layer)) sl.digested = 0;  // a ring may move or overwrite digested rows
      const std::vector<int32_t> before = sl.ring.pages;
      const int64_t w = c->ops.prepare_update(sl.ring, n_tokens, c->cfg.step_prealloc != 0);
      if (sl.ring.pages != before) sl.dirty = true;
      for (int64_t t = 0; t < n_tokens; ++t) {
        const int64_t r = w + t;
        dst_page[(size_t)b * n_tokens + t] = c->pool.addr(sl.ring.pages[r / kPageTokens]);
        dst_row[(size_t)b * n_tokens + t] = (int32_t)(r % kPageTokens);
      }
    }
    const size_t bytes = (size_t)n_seqs * H * n_tokens * c->cfg.head_dim * esz;
    bool hk = false, hv = false;
    const void* dk = c->stage_in(keys, bytes, c->in_k, s, hk);
    const void* dv = c->stage_in(values, bytes, c->in_v, s, hv);
    if (hk || hv) LC_CUDA(cudaEventRecord(c->ev_copy, s));
    run_append(c, n_seqs, H, 0, n_tokens, dst_page, dst_row, dk, dv, dtype, s, rope, sq);
    if (hk || hv) LC_CUDA(cudaEventSynchronize(c->ev_copy));
    c->ops.stream = c->stream;
  }
}

int lc_append(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
              const void* values, int32_t dtype, int64_t n_tokens, void* stream) {
  return abi_guard(
      [&] { append_impl(c, layer, n_seqs, seq_ids, keys, values, dtype, n_tokens, stream, nullptr); });
}

int lc_append_rope(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
                   const void* values, int32_t dtype, int64_t n_tokens, int32_t rope_dims, double rope_base,
                   int32_t traditional, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    LC_REQUIRE(rope_dims > 0 && rope_dims % 2 == 0 && rope_dims <= c->cfg.head_dim, LC_ERR_INVALID,
               "rope_dims must be even and in [2, head_dim]");
    LC_REQUIRE(rope_base > 0.0, LC_ERR_INVALID, "rope_base must be > 0");
    RopeArgs r;
    r.dims = rope_dims;
    r.base = rope_base;
    r.traditional = traditional ? 1 : 0;
    append_impl(c, layer, n_seqs, seq_ids, keys, values, dtype, n_tokens, stream, &r);
  });
}

int lc_store(lc_cache* c, int32_t seq, int32_t layer, int32_t head, const float* keys, const float* values,
             int64_t n_tokens) {
  return abi_guard([&] {
    LC_REQUIRE(c && keys && values, LC_ERR_INVALID, "null argument");
    c->check(seq, layer);
    LC_REQUIRE(head >= 0 && head < c->cfg.n_kv_heads, LC_ERR_INVALID, "head out of range");
    LC_REQUIRE(c->full(layer), LC_ERR_STATE, "store() is for full layers; sliding layers use lc_append");
    if (n_tokens <= 0) return;
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    c->ops.stream = s;
    SeqLayer& sl = c->at(seq, layer);
    if (sl.head_len.empty()) sl.head_len.assign(c->cfg.n_kv_heads, sl.ring.offset);
    const int64_t start = sl.head_len[head];
    const int64_t end = start + n_tokens;
    const int64_t new_len = std::max(sl.ring.offset, end);
    // Full layer kept as an exact-size buffer holding the longest head.
    if (!sl.ring.has || new_len > sl.ring.buf_len) {
      const int64_t need = (new_len + kPageTokens - 1) / kPageTokens;
      while ((int64_t)sl.ring.pages.size() < need) sl.ring.pages.push_back(c->pool.alloc());
      sl.ring.has = true;
      sl.ring.buf_len = new_len;
    }
    c->ops.make_private(sl.ring, start, end);
    sl.ring.offset = new_len;
    sl.ring.idx = new_len;
    sl.ring.view_len = new_len;
    sl.head_len[head] = end;
    sl.dirty = true;
    sl.digested = 0;
    std::vector<uint64_t> dst_page(n_tokens);
    std::vector<int32_t> dst_row(n_tokens);
    for (int64_t t = 0; t < n_tokens; ++t) {
      const int64_t r = start + t;
      dst_page[t] = c->pool.addr(sl.ring.pages[r / kPageTokens]);
      dst_row[t] = (int32_t)(r % kPageTokens);
    }
    const size_t bytes = (size_t)n_tokens * c->cfg.head_dim * 4;
    bool hk = false, hv = false;
    const void* dk = c->stage_in(keys, bytes, c->in_k, s, hk);
    const void* dv = c->stage_in(values, bytes, c->in_v, s, hv);
    run_append(c, 1, 1, head, n_tokens, dst_page, dst_row, dk, dv, LC_F32, s);
    LC_CUDA(cudaStreamSynchronize(s));
  });
}

int64_t lc_seq_len(const lc_cache* c, int32_t seq, int32_t layer, int32_t head) {
  int64_t r = -1;
  const int st = abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    c->check(seq, layer);
    LC_REQUIRE(head >= 0 && head < c->cfg.n_kv_heads, LC_ERR_INVALID, "head out of range");
    const SeqLayer& sl = c->at(seq, layer);
    r = sl.head_len.empty() ? sl.ring.view_len : sl.head_len[head];
  });
  return st == LC_OK ? r : (int64_t)st;
}

int lc_attend_keys(lc_cache* c, int32_t seq, int32_t layer, int32_t head, const float* query, float* scores,
                   int64_t n_scores) {
  return abi_guard([&] {
    LC_REQUIRE(c && query && scores, LC_ERR_INVALID, "null argument");
    c->check(seq, layer);
    LC_REQUIRE(head >= 0 && head < c->cfg.n_kv_heads, LC_ERR_INVALID, "head out of range");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    const SeqLayer& sl = c->at(seq, layer);
    const int64_t n = sl.head_len.empty() ? sl.ring.view_len : sl.head_len[head];
    LC_REQUIRE(n_scores >= n, LC_ERR_INVALID, "scores buffer too small");
    const int D = c->cfg.head_dim;
    c->hook_a.ensure(D, s);
    c->hook_b.ensure(D, s);
    c->hook_c.ensure(std::max<int64_t>(n, 1), s);
    bool hq = false;
    DevBuf<uint8_t> tmp;
    const float* dq = static_cast<const float*>(c->stage_in(query, D * 4, c->qbuf, s, hq));
    const uint64_t* pages = c->arena.put_vec(c->ops.page_addrs(sl.ring), s);
    launch_attend_keys(dq, c->dk.view(), pages, c->layout, R_KW, R_KS, head, n, c->hook_b.p, c->hook_c.p, s);
    c->launches += 2;
    LC_CUDA(cudaMemcpyAsync(scores, c->hook_c.p, n * 4, cudaMemcpyDefault, s));
    LC_CUDA(cudaStreamSynchronize(s));
  });
}

int lc_attend_keys_qjl(lc_cache* c, int32_t seq, int32_t layer, int32_t head, const float* query, float* scores,
                       int64_t n_scores) {
  return abi_guard([&] {
    LC_REQUIRE(c && query && scores, LC_ERR_INVALID, "null argument");
    c->check(seq, layer);
    LC_REQUIRE(head >= 0 && head < c->cfg.n_kv_heads, LC_ERR_INVALID, "head out of range");
    LC_REQUIRE(c->cfg.store_flags & LC_STORE_K_QJL, LC_ERR_STATE, "cache does not keep the K QJL bits");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    const SeqLayer& sl = c->at(seq, layer);
    const int64_t n = sl.head_len.empty() ? sl.ring.view_len : sl.head_len[head];
    LC_REQUIRE(n_scores >= n, LC_ERR_INVALID, "scores buffer too small");
    const int D = c->cfg.head_dim;
    c->hook_a.ensure(D, s);
    c->hook_b.ensure((size_t)D + c->kc.m, s);
    c->hook_c.ensure(std::max<int64_t>(n, 1), s);
    bool hq = false;
    const float* dq = static_cast<const float*>(c->stage_in(query, D * 4, c->qbuf, s, hq));
    const uint64_t* pages = c->arena.put_vec(c->ops.page_addrs(sl.ring), s);
    launch_attend_keys_qjl(dq, c->dk.view(), pages, c->layout, R_KW, R_KS, R_KQ, R_KR, head, n, c->hook_b.p,
                           c->hook_b.p + D, c->hook_c.p, s);
    c->launches += 3;
    LC_CUDA(cudaMemcpyAsync(scores, c->hook_c.p, n * 4, cudaMemcpyDefault, s));
    LC_CUDA(cudaStreamSynchronize(s));
  });
}

int lc_attend_values(lc_cache* c, int32_t seq, int32_t layer, int32_t head, const float* weights, int64_t n_weights,
                     float* out) {
  return abi_guard([&] {
    LC_REQUIRE(c && out && (weights || n_weights == 0), LC_ERR_INVALID, "null argument");
    c->check(seq, layer);
    LC_REQUIRE(head >= 0 && head < c->cfg.n_kv_heads, LC_ERR_INVALID, "head out of range");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    const SeqLayer& sl = c->at(seq, layer);
    const int64_t n = sl.head_len.empty() ? sl.ring.view_len : sl.head_len[head];
    LC_REQUIRE(n_weights == n, LC_ERR_INVALID, "weights length differs from seq_len");
    const int D = c->cfg.head_dim;
    c->hook_a.ensure(D, s);
    bool hw = false;
    const float* dw = n > 0 ? static_cast<const float*>(c->stage_in(weights, n * 4, c->qbuf, s, hw)) : nullptr;
    const uint64_t* pages = c->arena.put_vec(c->ops.page_addrs(sl.ring), s);
    launch_attend_values(dw, c->dv.view(), pages, c->layout, R_VW, R_VS, head, n, c->hook_a.p, s);
    ++c->launches;
    LC_CUDA(cudaMemcpyAsync(out, c->hook_a.p, D * 4, cudaMemcpyDefault, s));
    LC_CUDA(cudaStreamSynchronize(s));
  });
}

int lc_clear(lc_cache* c) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    if (c->last) LC_CUDA(cudaStreamSynchronize(c->last));
    LC_CUDA(cudaStreamSynchronize(c->stream));
    for (auto& sl : c->st) {
      c->ops.clear(sl.ring);
      sl.head_len.clear();
      sl.dirty = true;
      sl.digested = 0;
    }
  });
}

// ---- LKV2 snapshots (kv_disk.rs) --------------------------------------------
// One LayerMeta per cache layer, kind FullTurboquant (unbounded ring) or
// SlidingTurboquant, with the ring bookkeeping (offset, idx, keep,
// max_size) and the arrays of turboquant_meta (kv_disk.rs:2000-2024):
//   0 keys_codes u8 [1, H, S, D]        1 keys_sigma f32 [1, H, S, 1]
//   2 values_codes u8 [1, H, S, D]      3 values_sigma f32 [1, H, S, 1]
//   4 keys_signs bf16 +-1 [1, H, S, m]  5 keys_residual_norm f32 [1, H, S, 1]
// (4, 5 when the cache keeps the K QJL bits), S = the ring's backing length,
// rows in backing order. When the cache keeps the V QJL bits they follow in
// slots 6, 7 (values_signs, values_residual_norm); the reference's reader
// uses slots 0-5 only. Codes are unpacked to one byte each and QJL bits to
// +-1, as the reference's MLX arrays hold them. Pages move as whole page
// images, one copy each way per page.
namespace {

constexpr uint16_t kBf16One = 0x3F80, kBf16MinusOne = 0xBF80;

struct LayerRecs {
  int64_t S = 0;
  const Lkv2Record* r[8] = {};
};

// Byte offset of (role, head, row-in-page) in a page image.
inline size_t img_at(const PageLayout& L, int role, int h, int t) {
  return (size_t)(L.off[role] + ((int64_t)h * kPageTokens + t) * L.row[role]);
}

}  // namespace

int lc_save_lkv2(lc_cache* c, int32_t seq, const char* path, const char* model_fingerprint,
                 const uint32_t* prefix_tokens, int64_t n_prefix_tokens) {
  return abi_guard([&] {
    LC_REQUIRE(c && path, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_prefix_tokens >= 0 && (n_prefix_tokens == 0 || prefix_tokens), LC_ERR_INVALID, "bad prefix tokens");
    c->check(seq, 0);
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    LC_CUDA(cudaStreamSynchronize(s));
    const int H = c->cfg.n_kv_heads, D = c->cfg.head_dim;
    const int kb = (int)c->kc.bits, vb = (int)c->vc.bits;
    const bool kq = c->cfg.store_flags & LC_STORE_K_QJL, vq = c->cfg.store_flags & LC_STORE_V_QJL;
    const int mk = (int)c->kc.m, mv = (int)c->vc.m;
    const PageLayout& PL = c->layout;
    Lkv2Manifest man;
    man.model_fingerprint = model_fingerprint ? model_fingerprint : "";
    man.created_at_unix = (uint64_t)std::time(nullptr);
    man.prefix_tokens.assign(prefix_tokens, prefix_tokens + n_prefix_tokens);
    man.is_deep = true;
    std::vector<Lkv2Record> recs;
    std::vector<uint8_t> img((size_t)PL.page_bytes);
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      const SeqLayer& sl = c->at(seq, l);
      LC_REQUIRE(sl.head_len.empty(), LC_ERR_STATE,
                 "LKV2: a layer holds per-head lengths (KVCache::store); only ring layers are saved");
      const RingCore& r = sl.ring;
      Lkv2Layer L;
      L.kind = c->full(l) ? "FullTurboquant" : "SlidingTurboquant";
      L.offset = (uint64_t)r.offset;
      L.max_size = c->max_size[l];
      L.keep = c->keep[l];
      L.idx = r.idx;
      L.bits = kb;
      L.qjl_m = kq ? mk : -1;
      L.v_bits = vb != kb ? vb : -1;
      man.position = std::max<uint64_t>(man.position, (uint64_t)r.offset);
      const int64_t S = r.has ? r.buf_len : 0;
      if (S == 0) {
        L.arrays.assign(vq ? 8 : 6, -1);
        man.layers.push_back(L);
        continue;
      }
      const int32_t S32 = (int32_t)S;
      const size_t first = recs.size();
      auto add = [&](uint8_t dt, std::vector<int32_t> shape) {
        L.arrays.push_back((int64_t)recs.size());
        recs.emplace_back();
        Lkv2Record& rec = recs.back();
        rec.dtype = dt;
        rec.shape = std::move(shape);
        rec.data.assign((size_t)(rec.elems() * lkv2_elem_size(dt)), 0);
      };
      add(kLkvU8, {1, H, S32, D});
      add(kLkvF32, {1, H, S32, 1});
      add(kLkvU8, {1, H, S32, D});
      add(kLkvF32, {1, H, S32, 1});
      if (kq) {
        add(kLkvBF16, {1, H, S32, mk});
        add(kLkvF32, {1, H, S32, 1});
      } else {
        L.arrays.push_back(-1);
        L.arrays.push_back(-1);
      }
      if (vq) {
        add(kLkvBF16, {1, H, S32, mv});
        add(kLkvF32, {1, H, S32, 1});
      }
      Lkv2Record* kc_ = &recs[first];
      Lkv2Record* ks_ = kc_ + 1;
      Lkv2Record* vc_ = kc_ + 2;
      Lkv2Record* vs_ = kc_ + 3;
      Lkv2Record* kg_ = kq ? kc_ + 4 : nullptr;
      Lkv2Record* kr_ = kq ? kc_ + 5 : nullptr;
      Lkv2Record* vg_ = vq ? kc_ + (kq ? 6 : 4) : nullptr;
      Lkv2Record* vr_ = vq ? vg_ + 1 : nullptr;
      auto codes = [&](const uint8_t* words, int bits, uint8_t* out) {
        const int cpw = 64 / bits;
        const uint64_t mask = (1ull << bits) - 1;
        for (int j = 0; j < D; ++j) {
          uint64_t w;
          std::memcpy(&w, words + (size_t)(j / cpw) * 8, 8);
          out[j] = (uint8_t)((w >> ((j % cpw) * bits)) & mask);
        }
      };
      auto signs = [&](const uint8_t* words, int m, uint8_t* out) {
        for (int i = 0; i < m; ++i) {
          uint64_t w;
          std::memcpy(&w, words + (size_t)(i / 64) * 8, 8);
          const uint16_t v = ((w >> (i % 64)) & 1ull) ? kBf16One : kBf16MinusOne;
          std::memcpy(out + 2 * (size_t)i, &v, 2);
        }
      };
      for (size_t p = 0; (int64_t)(p * kPageTokens) < S; ++p) {
        LC_CUDA(cudaMemcpy(img.data(), reinterpret_cast<const void*>(c->pool.addr(r.pages[p])), img.size(),
                           cudaMemcpyDeviceToHost));
        const int nt = (int)std::min<int64_t>(kPageTokens, S - (int64_t)p * kPageTokens);
        for (int h = 0; h < H; ++h)
          for (int t = 0; t < nt; ++t) {
            const size_t row = (size_t)h * S + p * kPageTokens + t;  // [1][H][S] index
            codes(&img[img_at(PL, R_KW, h, t)], kb, &kc_->data[row * D]);
            codes(&img[img_at(PL, R_VW, h, t)], vb, &vc_->data[row * D]);
            std::memcpy(&ks_->data[row * 4], &img[img_at(PL, R_KS, h, t)], 4);
            std::memcpy(&vs_->data[row * 4], &img[img_at(PL, R_VS, h, t)], 4);
            if (kq) {
              signs(&img[img_at(PL, R_KQ, h, t)], mk, &kg_->data[row * mk * 2]);
              std::memcpy(&kr_->data[row * 4], &img[img_at(PL, R_KR, h, t)], 4);
            }
            if (vq) {
              signs(&img[img_at(PL, R_VQ, h, t)], mv, &vg_->data[row * mv * 2]);
              std::memcpy(&vr_->data[row * 4], &img[img_at(PL, R_VR, h, t)], 4);
            }
          }
      }
      man.layers.push_back(L);
    }
    lkv2_write(path, man, recs);
  });
}

int lc_load_lkv2(lc_cache* c, int32_t seq, const char* path, const char* model_fingerprint) {
  return abi_guard([&] {
    LC_REQUIRE(c && path, LC_ERR_INVALID, "null argument");
    c->check(seq, 0);
    Lkv2Manifest man;
    std::vector<Lkv2Record> recs;
    lkv2_read(path, man, recs);
    if (model_fingerprint)
      LC_REQUIRE(man.model_fingerprint == model_fingerprint, LC_ERR_STATE, "LKV2: model fingerprint differs");
    const int H = c->cfg.n_kv_heads, D = c->cfg.head_dim;
    const int kb = (int)c->kc.bits, vb = (int)c->vc.bits;
    const bool kq = c->cfg.store_flags & LC_STORE_K_QJL, vq = c->cfg.store_flags & LC_STORE_V_QJL;
    const int mk = (int)c->kc.m, mv = (int)c->vc.m;
    LC_REQUIRE((int64_t)man.layers.size() == c->cfg.n_layers, LC_ERR_INVALID,
               "LKV2: layer count differs from the cache");
    // ---- validate everything before the cache changes ----
    std::vector<LayerRecs> plan(c->cfg.n_layers);
    int64_t pages_needed = 0;
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      const Lkv2Layer& L = man.layers[l];
      const std::string where = "LKV2 layer " + std::to_string(l) + ": ";
      LC_REQUIRE(L.kind == "FullTurboquant" || L.kind == "SlidingTurboquant", LC_ERR_INVALID,
                 where + "not a TurboQuant layer (" + L.kind + ")");
      LC_REQUIRE(L.max_size == c->max_size[l] && L.keep == c->keep[l], LC_ERR_INVALID,
                 where + "max_size / keep differ from the cache's layer");
      LC_REQUIRE(L.bits == kb && (L.v_bits >= 0 ? L.v_bits : L.bits) == vb, LC_ERR_BITS,
                 where + "bit widths differ from the cache's codecs");
      LC_REQUIRE(L.idx >= 0, LC_ERR_INVALID, where + "missing idx");
      auto slot = [&](size_t i) -> const Lkv2Record* {
        if (i >= L.arrays.size() || L.arrays[i] < 0) return nullptr;
        LC_REQUIRE(L.arrays[i] < (int64_t)recs.size(), LC_ERR_INVALID, where + "array index out of range");
        return &recs[(size_t)L.arrays[i]];
      };
      LayerRecs& P = plan[l];
      for (int i = 0; i < 8; ++i) P.r[i] = slot((size_t)i);
      if (!P.r[0]) {
        LC_REQUIRE(!P.r[1] && !P.r[2] && !P.r[3] && L.offset == 0, LC_ERR_INVALID, where + "keys_codes missing");
        continue;
      }
      const Lkv2Record& k0 = *P.r[0];
      LC_REQUIRE(k0.shape.size() == 4 && k0.shape[0] == 1 && k0.shape[1] == H && k0.shape[3] == D, LC_ERR_INVALID,
                 where + "keys_codes shape is not [1, n_kv_heads, S, head_dim]");
      const int32_t S = k0.shape[2];
      auto want = [&](const Lkv2Record* r, uint8_t dt, int32_t last, const char* what) {
        LC_REQUIRE(r && r->dtype == dt && r->shape == std::vector<int32_t>({1, H, S, last}), LC_ERR_INVALID,
                   where + what + " missing or of the wrong dtype/shape");
      };
      want(P.r[0], kLkvU8, D, "keys_codes");
      want(P.r[1], kLkvF32, 1, "keys_sigma");
      want(P.r[2], kLkvU8, D, "values_codes");
      want(P.r[3], kLkvF32, 1, "values_sigma");
      if (kq) {
        LC_REQUIRE(L.qjl_m == mk, LC_ERR_INVALID, where + "qjl_m differs from the K codec's");
        want(P.r[4], kLkvBF16, mk, "keys_signs");
        want(P.r[5], kLkvF32, 1, "keys_residual_norm");
      }
      if (vq) {
        want(P.r[6], kLkvBF16, mv, "values_signs");
        want(P.r[7], kLkvF32, 1, "values_residual_norm");
      }
      LC_REQUIRE((int64_t)S <= (int64_t)c->cfg.max_pages_per_seq * kPageTokens, LC_ERR_NOMEM,
                 where + "more rows than max_pages_per_seq holds");
      LC_REQUIRE(L.idx <= S, LC_ERR_INVALID, where + "idx beyond the buffer");
      LC_REQUIRE((int64_t)L.offset >= L.max_size || (int64_t)L.offset <= S, LC_ERR_INVALID,
                 where + "offset beyond the buffer of a ring that has not wrapped");
      for (uint8_t v : P.r[0]->data) LC_REQUIRE(v < (1u << kb), LC_ERR_INVALID, where + "K code out of range");
      for (uint8_t v : P.r[2]->data) LC_REQUIRE(v < (1u << vb), LC_ERR_INVALID, where + "V code out of range");
      for (int i : {4, 6}) {
        if (!((i == 4 && kq) || (i == 6 && vq))) continue;
        const std::vector<uint8_t>& d = P.r[i]->data;
        for (size_t k = 0; k < d.size(); k += 2) {
          const uint16_t v = (uint16_t)(d[k] | (d[k + 1] << 8));
          LC_REQUIRE(v == kBf16One || v == kBf16MinusOne, LC_ERR_INVALID, where + "QJL sign not +-1");
        }
      }
      P.S = S;
      pages_needed += (S + kPageTokens - 1) / kPageTokens;
    }
    LC_REQUIRE(pages_needed <= c->pool.free_pages(), LC_ERR_NOMEM, "LKV2: page pool too small for the snapshot");
    // ---- apply: fresh private pages per layer ----
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    LC_CUDA(cudaStreamSynchronize(s));
    const PageLayout& PL = c->layout;
    std::vector<uint8_t> img((size_t)PL.page_bytes);
    auto pack = [&](const uint8_t* codes, int bits, uint8_t* words) {
      const int cpw = 64 / bits;
      const int nw = (D + cpw - 1) / cpw;
      for (int w = 0; w < nw; ++w) {
        uint64_t v = 0;
        for (int k = 0; k < cpw && w * cpw + k < D; ++k) v |= (uint64_t)codes[w * cpw + k] << (k * bits);
        std::memcpy(words + 8 * (size_t)w, &v, 8);
      }
    };
    auto unsigns = [&](const uint8_t* pm, int m, uint8_t* words) {
      const int nw = (m + 63) / 64;
      for (int w = 0; w < nw; ++w) {
        uint64_t v = 0;
        for (int i = w * 64; i < std::min(m, w * 64 + 64); ++i)
          if (pm[2 * (size_t)i + 1] == 0x3F) v |= 1ull << (i % 64);  // +1 (0x3F80) -> bit set
        std::memcpy(words + 8 * (size_t)w, &v, 8);
      }
    };
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      SeqLayer& sl = c->at(seq, l);
      c->ops.clear(sl.ring);
      sl.head_len.clear();
      sl.dirty = true;
      sl.digested = 0;
      const Lkv2Layer& L = man.layers[l];
      const LayerRecs& P = plan[l];
      RingCore& r = sl.ring;
      r.max_size = c->max_size[l];
      r.keep = c->keep[l];
      if (P.S == 0) continue;
      const int64_t S = P.S;
      try {
        for (int64_t p = 0; p * kPageTokens < S; ++p) {
          std::fill(img.begin(), img.end(), 0);
          const int nt = (int)std::min<int64_t>(kPageTokens, S - p * kPageTokens);
          for (int h = 0; h < H; ++h)
            for (int t = 0; t < nt; ++t) {
              const size_t row = (size_t)h * S + p * kPageTokens + t;
              pack(&P.r[0]->data[row * D], kb, &img[img_at(PL, R_KW, h, t)]);
              pack(&P.r[2]->data[row * D], vb, &img[img_at(PL, R_VW, h, t)]);
              std::memcpy(&img[img_at(PL, R_KS, h, t)], &P.r[1]->data[row * 4], 4);
              std::memcpy(&img[img_at(PL, R_VS, h, t)], &P.r[3]->data[row * 4], 4);
              if (kq) {
                unsigns(&P.r[4]->data[row * mk * 2], mk, &img[img_at(PL, R_KQ, h, t)]);
                std::memcpy(&img[img_at(PL, R_KR, h, t)], &P.r[5]->data[row * 4], 4);
              }
              if (vq) {
                unsigns(&P.r[6]->data[row * mv * 2], mv, &img[img_at(PL, R_VQ, h, t)]);
                std::memcpy(&img[img_at(PL, R_VR, h, t)], &P.r[7]->data[row * 4], 4);
              }
            }
          const int32_t pg = c->pool.alloc();
          r.pages.push_back(pg);
          LC_CUDA(cudaMemcpy(reinterpret_cast<void*>(c->pool.addr(pg)), img.data(), img.size(),
                             cudaMemcpyHostToDevice));
        }
      } catch (...) {
        c->ops.clear(r);
        throw;
      }
      r.has = true;
      r.buf_len = S;
      r.offset = (int64_t)L.offset;
      r.idx = L.idx;
      r.view_len = r.offset >= r.max_size ? S : r.offset;
    }
  });
}

int lc_lkv2_info(const char* path, int64_t* n_layers, int64_t* n_records, uint64_t* position) {
  return abi_guard([&] {
    LC_REQUIRE(path, LC_ERR_INVALID, "null path");
    Lkv2Manifest man;
    std::vector<Lkv2Record> recs;
    lkv2_read(path, man, recs);
    if (n_layers) *n_layers = (int64_t)man.layers.size();
    if (n_records) *n_records = (int64_t)recs.size();
    if (position) *position = man.position;
  });
}

int lc_release(lc_cache* c, int32_t seq) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      c->check(seq, l);
      SeqLayer& sl = c->at(seq, l);
      c->ops.clear(sl.ring);
      sl.head_len.clear();
      sl.dirty = true;
      sl.digested = 0;
    }
  });
}

int lc_truncate(lc_cache* c, int32_t seq, int32_t layer, int64_t n_keep) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    c->check(seq, layer);
    LC_REQUIRE(n_keep >= 0, LC_ERR_INVALID, "n_keep must be >= 0");
    SeqLayer& sl = c->at(seq, layer);
    if (!sl.head_len.empty()) {
      int64_t mx = 0;
      for (auto& hl : sl.head_len) {
        hl = std::min(hl, n_keep);
        mx = std::max(mx, hl);
      }
      sl.ring.offset = sl.ring.idx = sl.ring.view_len = mx;
      sl.dirty = true;
      sl.digested = 0;
      return;
    }
    if (sl.ring.offset <= n_keep) return;
    if (!c->ops.truncate_to(sl.ring, n_keep))
      LC_THROW(LC_ERR_REFUSED, "truncate: post-rotation rollback not supported");
    sl.dirty = true;
    sl.digested = 0;
  });
}

int lc_truncate_to(lc_cache* c, int32_t seq, int32_t layer, int64_t target) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    c->check(seq, layer);
    SeqLayer& sl = c->at(seq, layer);
    LC_REQUIRE(sl.head_len.empty(), LC_ERR_STATE, "truncate_to on a layer filled per head; use lc_truncate");
    if (!c->ops.truncate_to(sl.ring, target)) {
      if (target > sl.ring.offset)
        LC_THROW(LC_ERR_REFUSED, "truncate_to: target " + std::to_string(target) + " > offset " +
                                     std::to_string(sl.ring.offset));
      LC_THROW(LC_ERR_REFUSED, "truncate_to: post-rotation rollback not supported (offset=" +
                                   std::to_string(sl.ring.offset) + " > max_size=" +
                                   std::to_string(sl.ring.max_size) + ")");
    }
    sl.dirty = true;
    sl.digested = 0;
  });
}

int lc_fork(lc_cache* c, int32_t src, int32_t dst, int64_t prefix_len) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    LC_REQUIRE(src != dst, LC_ERR_INVALID, "fork onto itself");
    LC_REQUIRE(prefix_len >= 0, LC_ERR_INVALID, "prefix_len must be >= 0");
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      c->check(src, l);
      c->check(dst, l);
      const SeqLayer& s = c->at(src, l);
      int64_t avail = s.ring.offset;
      if (!s.head_len.empty()) avail = *std::min_element(s.head_len.begin(), s.head_len.end());
      LC_REQUIRE(prefix_len <= avail && prefix_len <= (s.ring.has ? s.ring.buf_len : 0), LC_ERR_REFUSED,
                 "fork: prefix longer than the source holds");
      LC_REQUIRE(s.ring.offset <= s.ring.max_size, LC_ERR_REFUSED, "fork: source ring has rotated");
    }
    for (int32_t l = 0; l < c->cfg.n_layers; ++l) {
      SeqLayer& d = c->at(dst, l);
      c->ops.clear(d.ring);
      d.head_len.clear();
      d.digested = 0;
      d.ring = c->ops.share_prefix(c->at(src, l).ring, prefix_len);
      d.ring.max_size = c->max_size[l];
      d.ring.keep = c->keep[l];
      d.dirty = true;
    }
  });
}

int lc_ring_state(const lc_cache* c, int32_t seq, int32_t layer, int64_t* offset, int64_t* idx, int64_t* buf_len,
                  int64_t* view_len) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    c->check(seq, layer);
    const SeqLayer& sl = c->at(seq, layer);
    if (offset) *offset = sl.ring.offset;
    if (idx) *idx = sl.ring.idx;
    if (buf_len) *buf_len = sl.ring.has ? sl.ring.buf_len : 0;
    if (view_len) *view_len = sl.ring.view_len;
  });
}

int lc_fetch(lc_cache* c, int32_t seq, int32_t layer, int32_t which, lc_fetch_out* out, int64_t max_tokens,
             int64_t* n_out) {
  return abi_guard([&] {
    LC_REQUIRE(c && out, LC_ERR_INVALID, "null argument");
    c->check(seq, layer);
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->stream;
    c->order(s);
    const SeqLayer& sl = c->at(seq, layer);
    const int64_t n = which == LC_FETCH_BACKING ? (sl.ring.has ? sl.ring.buf_len : 0) : sl.ring.view_len;
    if (n_out) *n_out = n;
    LC_REQUIRE(n <= max_tokens, LC_ERR_INVALID, "max_tokens smaller than the stored length");
    if (n == 0) return;
    const PageLayout& L = c->layout;
    int64_t lin_off[kMaxRoles] = {};
    size_t total = 0;
    for (int k = 0; k < L.n_roles; ++k) {
      lin_off[k] = (int64_t)total;
      total += (size_t)L.heads * n * L.row[k];
      total = (total + 255) & ~size_t(255);
    }
    c->fetchbuf.ensure(total, s);
    c->ops.stream = s;
    read_rows(c->ops, sl.ring, 0, n, c->fetchbuf.p, lin_off);
    void* dsts[kMaxRoles] = {out->k_words, out->v_words, out->k_sigma, out->v_sigma, nullptr, nullptr, nullptr,
                             nullptr};
    if (c->cfg.store_flags & (LC_STORE_K_QJL | LC_STORE_V_QJL)) {
      if (c->cfg.store_flags & LC_STORE_K_QJL) {
        dsts[R_KQ] = out->k_qjl;
        dsts[R_KR] = out->k_rnorm;
      }
      if (c->cfg.store_flags & LC_STORE_V_QJL) {
        dsts[R_VQ] = out->v_qjl;
        dsts[R_VR] = out->v_rnorm;
      }
    }
    for (int k = 0; k < L.n_roles; ++k) {
      if (!dsts[k]) continue;
      LC_CUDA(cudaMemcpyAsync(dsts[k], c->fetchbuf.p + lin_off[k], (size_t)L.heads * n * L.row[k], cudaMemcpyDefault,
                              s));
    }
    LC_CUDA(cudaStreamSynchronize(s));
  });
}

struct DecodeRun {
  int32_t rows = 0, G = 1, max_slots = 1;
  const int32_t* cnt = nullptr;
  float oscale = 1.0f;  // 1 / V table scale of the fast path
  bool host_q = false;  // q was staged from host memory
  bool fused = false;   // the output is written: no merge launch needed
};

// fused_out: device output of a full attention call (lc_decode_attn), which
// the one-launch kernel writes when the plan allows; null for partials.
// Prefill attention (lc_prefill_attn): the n_seqs "sequences" are the last
// n_seqs tokens of sequence `seq`, query b attending to the first
// view_len - n_seqs + b + 1 tokens (causal). They share the sequence's block
// table row, so the split-K decode runs unchanged.
struct PrefillView {
  int32_t seq;
};

static DecodeRun decode_common(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* q,
                               int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, cudaStream_t s,
                               void* fused_out = nullptr, int32_t out_dtype = LC_F32,
                               const PrefillView* prefill = nullptr, float* fused_parts = nullptr) {
  LC_REQUIRE(c && (seq_ids || prefill) && q, LC_ERR_INVALID, "null argument");
  LC_REQUIRE(n_seqs > 0, LC_ERR_INVALID, "n_seqs must be > 0");
  const int32_t hkv = c->cfg.n_kv_heads;
  LC_REQUIRE(n_q_heads > 0 && n_q_heads % hkv == 0, LC_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads");
  const int32_t D = c->cfg.head_dim;
  LC_CUDA(cudaSetDevice(c->cfg.device));
  c->order(s);
  c->ops.stream = s;
  std::vector<int64_t> info((size_t)n_seqs * 2), lens(n_seqs);
  for (int32_t b = 0; b < n_seqs; ++b) {
    const int32_t seq = prefill ? prefill->seq : seq_ids[b];
    c->check(seq, layer);
    SeqLayer& sl = c->at(seq, layer);
    int64_t n = sl.ring.view_len;
    if (!sl.head_len.empty()) {
      for (int64_t hl : sl.head_len)
        LC_REQUIRE(hl == sl.head_len[0], LC_ERR_STATE, "heads of this layer hold different lengths");
      n = sl.head_len[0];
    }
    if (prefill) {
      // the view must be in token order: a ring that has wrapped holds its
      // window in rotated order (the window mask would need the positions)
      LC_REQUIRE(sl.head_len.empty() ? sl.ring.offset <= sl.ring.max_size : true, LC_ERR_STATE,
                 "prefill attention over a ring that has wrapped is not supported");
      LC_REQUIRE(n >= n_seqs, LC_ERR_INVALID, "prefill: more query tokens than the sequence holds");
      n = n - n_seqs + b + 1;
    }
    if (!prefill || b == 0) c->sync_table(seq, layer, s);
    info[2 * b] = n;
    info[2 * b + 1] = (int64_t)layer * c->cfg.max_seqs + seq;
    lens[b] = n;
  }
  const bool qjl = (flags & LC_QJL_SCORES) != 0;
  if (qjl) {
    LC_REQUIRE(c->cfg.store_flags & LC_STORE_K_QJL, LC_ERR_STATE, "QJL scores: cache does not keep the K QJL bits");
    LC_REQUIRE(!(flags & LC_Q_ROTATED), LC_ERR_INVALID, "QJL scores need the un-rotated query");
    LC_REQUIRE(c->kc.m > 0 && c->kc.m <= (uint64_t)kMaxQjlDecode, LC_ERR_INVALID,
               "QJL scores: qjl_m must be in [1, 256]");
  }
  // ---- page-sparse decode: digest new pages, then decode logical lengths
  // (the chosen pages and the tail) through a tile map ----
  const bool sparse = (flags & LC_SPARSE_PAGES) != 0;
  std::vector<int64_t> real_info;
  int32_t map_stride = 0;
  int32_t npad = 1;  // the most full pages of any sequence
  if (sparse) {
    LC_REQUIRE(c->role_dg >= 0, LC_ERR_STATE, "page-sparse decode: cache created without LC_STORE_DIGEST");
    LC_REQUIRE(!qjl && !prefill, LC_ERR_INVALID, "page-sparse decode: not with QJL scores or prefill attention");
    LC_REQUIRE(c->full(layer), LC_ERR_INVALID, "page-sparse decode: full (non-sliding) layers only");
    const int G = n_q_heads / hkv;
    LC_REQUIRE(((decode_fast_path(D, (int)c->kc.bits, (int)c->vc.bits, G) && G <= 4) ||
                decode_mma_path(D, (int)c->kc.bits, (int)c->vc.bits, G)),
               LC_ERR_INVALID,
               "page-sparse decode: the tensor-core geometries only (4-bit K/V at head_dim 128, or 3-bit K / "
               "2-bit V at head_dim 256; GQA <= 4)");
    real_info = info;
    std::vector<uint64_t> dpages;
    std::vector<int32_t> drows;
    for (int32_t b = 0; b < n_seqs; ++b) {
      SeqLayer& sl = c->at(seq_ids[b], layer);
      LC_REQUIRE(sl.head_len.empty(), LC_ERR_STATE, "page-sparse decode: layer filled per head");
      const int64_t n = lens[b], P = n / kDigestPage;
      for (int64_t g = sl.digested; g < P; ++g) {  // pages filled since the last digest
        dpages.push_back(c->pool.addr(sl.ring.pages[g / kGroupsPerPage]));
        drows.push_back((int32_t)((g % kGroupsPerPage) * kDigestPage));
      }
      sl.digested = std::max<int64_t>(sl.digested, P);
      int64_t keep = sparse_keep_pages(P);
      if (n < kSparseMinKeys || P <= keep) keep = P;  // dense
      const int64_t logical = keep * kDigestPage + (n - P * kDigestPage);
      lens[b] = logical;
      info[2 * b] = logical;
      map_stride = std::max<int32_t>(map_stride, (int32_t)((logical + kTileTokens - 1) / kTileTokens));
      npad = std::max<int32_t>(npad, (int32_t)P);
    }
    if (!dpages.empty()) {
      const size_t k = dpages.size();
      c->blob.resize(k * 12);
      std::memcpy(c->blob.data(), dpages.data(), k * 8);
      std::memcpy(c->blob.data() + k * 8, drows.data(), k * 4);
      const uint8_t* d = static_cast<const uint8_t*>(c->arena.put(c->blob.data(), c->blob.size(), s));
      DigestDev dg;
      dg.pages = reinterpret_cast<const uint64_t*>(d);
      dg.row0 = reinterpret_cast<const int32_t*>(d + k * 8);
      dg.cent = c->dk.cent_d;
      dg.off_kw = c->layout.off[R_KW];
      dg.off_ks = c->layout.off[R_KS];
      dg.off_dg = c->layout.off[c->role_dg];
      dg.row_kw = c->layout.row[R_KW];
      dg.row_dg = c->layout.row[c->role_dg];
      dg.bits = (int32_t)c->kc.bits;
      dg.dim = D;
      c->timed(c->t_other, s, [&] { launch_digest(dg, (int64_t)k, hkv, s); });
      ++c->launches;
    }
  }
  const DecodePlan plan = plan_decode(lens, hkv, n_q_heads, D, (int)c->kc.bits, (int)c->vc.bits, qjl);
  bool fused = (fused_out || fused_parts) && decode_fusable(plan, n_q_heads / hkv);
  if (fused_parts)  // empty sequences' partial rows (m = -inf) come from the split path's merge
    for (int32_t b = 0; b < n_seqs; ++b) fused = fused && lens[b] > 0;
  // The one-launch path of small calls passes its arrays in the launch
  // parameters; otherwise one upload: [seqinfo i64 | seg i64 | cnt i32].
  const bool inl = fused && decode_inline_fits(n_seqs, hkv);
  const int64_t* dinfo = nullptr;
  const int64_t* dseg = nullptr;
  const int32_t* dcnt = nullptr;
  if (!inl) {
    const size_t b_info = info.size() * 8, b_seg = plan.flat ? plan.seg.size() * 8 : 0, b_cnt = plan.cnt.size() * 4;
    c->blob.resize(b_info + b_seg + b_cnt);
    std::memcpy(c->blob.data(), info.data(), b_info);
    if (b_seg) std::memcpy(c->blob.data() + b_info, plan.seg.data(), b_seg);
    std::memcpy(c->blob.data() + b_info + b_seg, plan.cnt.data(), b_cnt);
    const uint8_t* dblob = static_cast<const uint8_t*>(c->arena.put(c->blob.data(), c->blob.size(), s));
    dinfo = reinterpret_cast<const int64_t*>(dblob);
    dseg = plan.flat ? reinterpret_cast<const int64_t*>(dblob + b_info) : nullptr;
    dcnt = reinterpret_cast<const int32_t*>(dblob + b_info + b_seg);
  }
  const int64_t rows = (int64_t)n_seqs * n_q_heads;
  bool hq = false;
  const void* dq = c->stage_in(q, (size_t)rows * D * dtype_size(q_dtype), c->qbuf, s, hq);
  const float kalpha = (plan.flat || plan.mma) ? c->dk.alpha : 1.0f,
              valpha = (plan.flat || plan.mma) ? c->dv.alpha : 1.0f;
  const float qscale = scale * 1.4426950408889634f / kalpha;
  // the 3/2-bit tensor-core kernel takes rotated queries as given (scaled as
  // it reads them), so a decode step's rotated rows need no launch here
  const bool raw_q = plan.mma && (flags & LC_Q_ROTATED) && !qjl && !sparse;
  if (!fused && !raw_q) {
    c->q_rot.ensure((size_t)rows * D, s);
    c->q_h.ensure((size_t)rows * D, s);
    c->timed(c->t_other, s, [&] {
      launch_rotate_q(dq, q_dtype, (int32_t)rows, D, c->dk.RTd, (flags & LC_Q_ROTATED) != 0, qscale, c->q_rot.p,
                      c->q_h.p, s);
    });
    ++c->launches;
  }
  if (qjl) {
    c->q_proj.ensure((size_t)rows * c->kc.m, s);
    c->timed(c->t_other, s, [&] {
      launch_project_q(dq, q_dtype, (int32_t)rows, D, (int32_t)c->kc.m, c->dk.PTd, qscale, c->q_proj.p, s);
    });
    ++c->launches;
  }
  if (sparse) {  // choose the pages (the select kernel rotates the queries itself)
    c->tile_map.ensure((size_t)n_seqs * hkv * std::max(map_stride, 1), s);
    SelectDev sd;
    sd.seqinfo = c->arena.put_vec(real_info, s);
    sd.table = c->d_table;
    sd.table_stride = c->cfg.max_pages_per_seq;
    sd.q = dq;
    sd.q_dtype = q_dtype;
    sd.q_rotated = (flags & LC_Q_ROTATED) ? 1 : 0;
    sd.RT = c->dk.RTd;
    sd.off_dg = c->layout.off[c->role_dg];
    sd.row_dg = c->layout.row[c->role_dg];
    sd.n_seqs = n_seqs;
    sd.hkv = hkv;
    sd.hq = n_q_heads;
    sd.G = n_q_heads / hkv;
    sd.dim = D;
    sd.npad = npad;
    sd.map_stride = map_stride;
    sd.tile_map = c->tile_map.p;
    c->timed(c->t_other, s, [&] { launch_page_select(sd, s); });
    ++c->launches;
  }
  c->part.ensure((size_t)rows * plan.max_slots * (D + 2), s);
  DecodeArgs a;
  a.table = c->d_table;
  a.table_stride = c->cfg.max_pages_per_seq;
  a.seqinfo = dinfo;
  a.seg = dseg;
  if (inl) {
    a.h_seqinfo = info.data();
    a.h_seg = plan.seg.data();
    a.h_cnt = plan.cnt.data();
  }
  a.layout = c->layout;
  a.role_kw = R_KW;
  a.role_vw = R_VW;
  a.role_ks = R_KS;
  a.role_vs = R_VS;
  a.n_seqs = n_seqs;
  a.hkv = hkv;
  a.hq = n_q_heads;
  a.dim = D;
  a.kbits = (int)c->kc.bits;
  a.vbits = (int)c->vc.bits;
  a.q_rot = c->q_rot.p;
  a.q_h = c->q_h.p;
  if (raw_q) {
    a.q_raw = dq;
    a.q_raw_dtype = q_dtype;
    a.q_raw_scale = qscale;
  }
  a.kcent = c->dk.cent_d;
  a.vcent = c->dv.cent_d;
  a.kalpha = kalpha;
  a.valpha = valpha;
  a.klo_thr = decode_klo_thr(c->dk.lo_max);
  a.part = c->part.p;
  if (sparse) {
    a.tile_map = c->tile_map.p;
    a.map_stride = map_stride;
  }
  // one chunk per (sequence, kv head) on the 3/2-bit tensor-core path (short
  // and sliding layers): the kernel finishes the rows, no merge launch
  const bool mma_fin = !fused && plan.mma && plan.n_chunks == 1 && fused_out && !fused_parts;
  if (mma_fin) {
    a.fin_out = fused_out;
    a.fin_dtype = out_dtype;
    a.fin_R = c->v_R(flags);
    a.fin_oscale = 1.0f / valpha;
  }
  if (qjl) {
    a.q_proj = c->q_proj.p;
    a.role_kq = R_KQ;
    a.role_kr = R_KR;
    a.qjl_m = (int32_t)c->kc.m;
    a.qjl_c = std::sqrt((float)1.5707963267948966) / std::sqrt((float)c->kc.m);
  }
  if (fused) {
    const size_t nctr = (size_t)n_seqs * hkv, before = c->ctr.n;
    c->ctr.ensure(nctr, s);
    if (c->ctr.n != before) LC_CUDA(cudaMemsetAsync(c->ctr.p, 0, c->ctr.n * sizeof(int32_t), s));
    const size_t esz = dtype_size(out_dtype);
    for (int32_t b = 0; b < n_seqs && fused_out; ++b)  // rows of empty sequences are zero
      if (lens[b] == 0)
        LC_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(fused_out) + (size_t)b * n_q_heads * D * esz, 0,
                                (size_t)n_q_heads * D * esz, s));
    FusedArgs f;
    f.q = dq;
    f.q_dtype = q_dtype;
    f.q_rotated = (flags & LC_Q_ROTATED) ? 1 : 0;
    f.qscale = qscale;
    f.qR = c->dk.R;
    f.vRT = c->v_RT(flags);
    f.cnt = dcnt;
    f.ctr = c->ctr.p;
    f.out = fused_out;
    f.out_dtype = out_dtype;
    f.oscale = 1.0f / valpha;
    if (fused_parts) {
      f.parts = fused_parts;
      f.parts_rows = (int32_t)rows;
      f.vRT = nullptr;
    }
    c->timed(c->t_decode, s, [&] { launch_decode_fused(a, plan, f, s); });
  } else {
    c->timed(c->t_decode, s, [&] { launch_decode_partials(a, plan, s); });
  }
  ++c->launches;
  if (hq) LC_CUDA(cudaEventRecord(c->ev_copy, s));
  DecodeRun r;
  r.fused = fused || mma_fin;
  r.rows = (int32_t)rows;
  r.G = n_q_heads / hkv;
  r.max_slots = plan.max_slots;
  r.cnt = dcnt;
  r.oscale = 1.0f / valpha;
  r.host_q = hq;
  return r;
}

// lc_prefill_attn on the tensor cores (prefill.cu) where the geometry has
// the tiled kernel (4-bit K and V, head_dim 128, GQA <= 8) and no QJL or
// page-sparse scores are asked for: one launch rotates the chunk's queries,
// attends and writes the normalised, un-rotated rows into `dout`. Returns false (nothing issued) for other calls,
// which take the split-K decode with one virtual sequence per query token.
static bool prefill_tiled(lc_cache* c, int32_t layer, int32_t seq, const void* q, int32_t q_dtype, int32_t L,
                          int32_t n_q_heads, float scale, uint32_t flags, void* dout, int32_t out_dtype,
                          cudaStream_t s, bool& host_q) {
  const int32_t hkv = c->cfg.n_kv_heads, D = c->cfg.head_dim;
  if (flags & (LC_QJL_SCORES | LC_SPARSE_PAGES)) return false;
  // the kernel writes output pairs as 8-byte (f32) / 4-byte (bf16, f16) stores
  if (reinterpret_cast<uintptr_t>(dout) % (out_dtype == LC_F32 ? 8 : 4) != 0) return false;
  if (n_q_heads % hkv != 0 || !prefill_tiled_path(D, (int)c->kc.bits, (int)c->vc.bits, n_q_heads / hkv)) return false;
  c->check(seq, layer);
  SeqLayer& sl = c->at(seq, layer);
  int64_t n = sl.ring.view_len;
  if (!sl.head_len.empty()) {
    for (int64_t hl : sl.head_len)
      LC_REQUIRE(hl == sl.head_len[0], LC_ERR_STATE, "heads of this layer hold different lengths");
    n = sl.head_len[0];
  }
  LC_REQUIRE(sl.head_len.empty() ? sl.ring.offset <= sl.ring.max_size : true, LC_ERR_STATE,
             "prefill attention over a ring that has wrapped is not supported");
  LC_REQUIRE(n >= L, LC_ERR_INVALID, "prefill: more query tokens than the sequence holds");
  c->order(s);
  c->ops.stream = s;
  c->sync_table(seq, layer, s);
  const int64_t rows = (int64_t)L * n_q_heads;
  const size_t qbytes = (size_t)rows * D * dtype_size(q_dtype);
  const void* dq = c->stage_in(q, qbytes, c->qbuf, s, host_q);
  // the kernel reads query pairs as 8-byte (f32) / 4-byte (bf16, f16) loads
  if (reinterpret_cast<uintptr_t>(dq) % (q_dtype == LC_F32 ? 8 : 4) != 0) {
    c->qbuf.ensure(qbytes, s);
    LC_CUDA(cudaMemcpyAsync(c->qbuf.p, dq, qbytes, cudaMemcpyDeviceToDevice, s));
    dq = c->qbuf.p;
  }
  PrefillArgs a;
  a.table_row = c->table_row(seq, layer);
  a.n_total = n;
  a.L = L;
  a.hkv = hkv;
  a.hq = n_q_heads;
  a.off_kw = c->layout.off[R_KW];
  a.off_vw = c->layout.off[R_VW];
  a.off_ks = c->layout.off[R_KS];
  a.off_vs = c->layout.off[R_VS];
  a.q = dq;
  a.q_dtype = q_dtype;
  a.q_rotated = (flags & LC_Q_ROTATED) ? 1 : 0;
  a.qscale = scale * 1.4426950408889634f / c->dk.alpha;
  a.kR = c->dk.R;
  a.vRT = c->v_RT(flags);
  a.kcent = c->dk.cent_d;
  a.vcent = c->dv.cent_d;
  a.kalpha = c->dk.alpha;
  a.valpha = c->dv.alpha;
  a.pthr = decode_klo_thr(c->dk.lo_max);
  a.out = dout;
  a.out_dtype = out_dtype;
  a.oscale = 1.0f / c->dv.alpha;
  c->timed(c->t_decode, s, [&] { launch_prefill_tiled(a, s); });
  if (host_q) LC_CUDA(cudaEventRecord(c->ev_copy, s));
  ++c->launches;
  return true;
}

// lc_decode_attn and lc_prefill_attn: decode, merge if the one-launch path
// was not taken, copy a host output back.
static void attn_call(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const PrefillView* prefill,
                      const void* q, int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, void* out,
                      int32_t out_dtype, void* stream) {
  LC_REQUIRE(out, LC_ERR_INVALID, "null out");
  cudaStream_t s = c ? c->pick(stream) : nullptr;
  LC_REQUIRE(c && n_q_heads > 0 && n_seqs > 0, LC_ERR_INVALID, "bad decode arguments");
  LC_CUDA(cudaSetDevice(c->cfg.device));
  const int32_t D = c->cfg.head_dim;
  const int64_t rows = (int64_t)n_seqs * n_q_heads;
  const size_t obytes = (size_t)rows * D * dtype_size(out_dtype);
  const bool host_out = !is_device_ptr(out);
  void* dout = out;
  if (host_out) {
    c->outbuf.ensure(obytes, s);
    dout = c->outbuf.p;
  }
  bool tiled_host_q = false;
  if (prefill && prefill_tiled(c, layer, prefill->seq, q, q_dtype, n_seqs, n_q_heads, scale, flags, dout, out_dtype, s,
                               tiled_host_q)) {
    if (host_out) {
      LC_CUDA(cudaMemcpyAsync(out, dout, obytes, cudaMemcpyDeviceToHost, s));
      LC_CUDA(cudaStreamSynchronize(s));
    } else if (tiled_host_q) {
      LC_CUDA(cudaEventSynchronize(c->ev_copy));
    }
    return;
  }
  const DecodeRun run =
      decode_common(c, layer, n_seqs, seq_ids, q, q_dtype, n_q_heads, scale, flags, s, dout, out_dtype, prefill);
  if (!run.fused) {
    c->timed(c->t_other, s, [&] {
      launch_merge(c->part.p, run.cnt, run.G, run.max_slots, (int32_t)rows, D,
                   c->v_R(flags), dout, out_dtype, nullptr, nullptr, nullptr,
                   run.oscale, s);
    });
    ++c->launches;
  }
  if (host_out) {
    LC_CUDA(cudaMemcpyAsync(out, dout, obytes, cudaMemcpyDeviceToHost, s));
    LC_CUDA(cudaStreamSynchronize(s));
  } else if (run.host_q) {
    LC_CUDA(cudaEventSynchronize(c->ev_copy));
  }
}

int lc_prefill_attn(lc_cache* c, int32_t layer, int32_t seq, const void* q, int32_t q_dtype, int32_t n_q_tokens,
                    int32_t n_q_heads, float scale, uint32_t flags, void* out, int32_t out_dtype, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null cache");
    const PrefillView pv{seq};
    attn_call(c, layer, n_q_tokens, nullptr, &pv, q, q_dtype, n_q_heads, scale, flags, out, out_dtype, stream);
  });
}

int lc_decode_attn(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* q,
                   int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, void* out, int32_t out_dtype,
                   void* stream) {
  return abi_guard([&] {
    attn_call(c, layer, n_seqs, seq_ids, nullptr, q, q_dtype, n_q_heads, scale, flags, out, out_dtype, stream);
  });
}

// One decode step of a layer: append each sequence's new token, then attend
// (the reference's update_and_fetch followed by turboquant_fused_attn on the
// rotated query, gemma4_moe.rs:4245-4797). The queries are rotated by the
// same launch that rotates and quantizes the new keys, so the attention
// kernel takes them rotated and skips its own rotation. The caller holds
// abi_guard.
static void decode_step_impl(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
                             const void* values, int32_t kv_dtype, const void* q, int32_t q_dtype, int32_t n_q_heads,
                             float scale, uint32_t flags, void* out, int32_t out_dtype, void* stream) {
  LC_REQUIRE(c && seq_ids && keys && values && q && out, LC_ERR_INVALID, "null argument");
  LC_REQUIRE(n_seqs > 0 && n_q_heads > 0, LC_ERR_INVALID, "bad decode arguments");
  dtype_size(q_dtype);
  LC_CUDA(cudaSetDevice(c->cfg.device));
  cudaStream_t s = c->pick(stream);
  const int32_t D = c->cfg.head_dim, H = c->cfg.n_kv_heads;
  const bool stage2 = (c->cfg.store_flags & (LC_STORE_K_QJL | LC_STORE_V_QJL)) != 0;
  const int m_max = (int)std::max(c->kc.m, c->vc.m);
  const bool rot = !(flags & (LC_Q_ROTATED | LC_QJL_SCORES)) &&
                   append_rotates_queries((int64_t)n_seqs * H, D, m_max, stage2);
  if (!rot) {
    append_impl(c, layer, n_seqs, seq_ids, keys, values, kv_dtype, 1, stream, nullptr);
    attn_call(c, layer, n_seqs, seq_ids, nullptr, q, q_dtype, n_q_heads, scale, flags, out, out_dtype, stream);
    return;
  }
  const int64_t rows = (int64_t)n_seqs * n_q_heads;
  c->order(s);
  bool hq = false;
  const void* dq = c->stage_in(q, (size_t)rows * D * dtype_size(q_dtype), c->qbuf, s, hq);
  c->q_step.ensure((size_t)rows * D, s);
  StepQ sq;
  sq.q = dq;
  sq.dtype = q_dtype;
  sq.rows = (int32_t)rows;
  sq.out = c->q_step.p;
  append_impl(c, layer, n_seqs, seq_ids, keys, values, kv_dtype, 1, stream, nullptr, &sq);
  attn_call(c, layer, n_seqs, seq_ids, nullptr, c->q_step.p, LC_F32, n_q_heads, scale, flags | LC_Q_ROTATED, out,
            out_dtype, stream);
  if (hq) LC_CUDA(cudaStreamSynchronize(s));  // the staged queries are read before the host reuses them
}

int lc_decode_step(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* keys,
                   const void* values, int32_t kv_dtype, const void* q, int32_t q_dtype, int32_t n_q_heads,
                   float scale, uint32_t flags, void* out, int32_t out_dtype, void* stream) {
  return abi_guard([&] {
    decode_step_impl(c, layer, n_seqs, seq_ids, keys, values, kv_dtype, q, q_dtype, n_q_heads, scale, flags, out,
                     out_dtype, stream);
  });
}

int lc_decode_step_layers(lc_cache* c, int32_t layer0, int32_t n_layers, int32_t n_seqs, const int32_t* seq_ids,
                          const void* keys, const void* values, int32_t kv_dtype, const void* q, int32_t q_dtype,
                          int32_t n_q_heads, float scale, uint32_t flags, void* out, int32_t out_dtype,
                          void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c && seq_ids && keys && values && q && out, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_layers > 0 && layer0 >= 0 && layer0 + n_layers <= c->cfg.n_layers, LC_ERR_INVALID,
               "layers out of range");
    LC_REQUIRE(n_seqs > 0 && n_q_heads > 0, LC_ERR_INVALID, "bad decode arguments");
    const size_t D = (size_t)c->cfg.head_dim;
    const size_t kv_stride = (size_t)n_seqs * c->cfg.n_kv_heads * D * dtype_size(kv_dtype);
    const size_t q_stride = (size_t)n_seqs * n_q_heads * D * dtype_size(q_dtype);
    const size_t o_stride = (size_t)n_seqs * n_q_heads * D * dtype_size(out_dtype);
    for (int32_t i = 0; i < n_layers; ++i)
      decode_step_impl(c, layer0 + i, n_seqs, seq_ids, static_cast<const uint8_t*>(keys) + i * kv_stride,
                       static_cast<const uint8_t*>(values) + i * kv_stride,
                       kv_dtype, static_cast<const uint8_t*>(q) + i * q_stride, q_dtype, n_q_heads, scale, flags,
                       static_cast<uint8_t*>(out) + i * o_stride, out_dtype, stream);
  });
}

int lc_decode_attn_partials(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* q,
                            int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, float* m, float* l,
                            float* o, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(m && l && o, LC_ERR_INVALID, "null output");
    cudaStream_t s = c ? c->pick(stream) : nullptr;
    const DecodeRun run = decode_common(c, layer, n_seqs, seq_ids, q, q_dtype, n_q_heads, scale, flags, s);
    const int32_t D = c->cfg.head_dim;
    const int64_t rows = run.rows;
    const bool dev = is_device_ptr(m) && is_device_ptr(l) && is_device_ptr(o);
    float *dm = m, *dl = l, *dov = o;
    if (!dev) {
      c->outbuf.ensure((size_t)rows * (D + 2) * 4, s);
      dm = reinterpret_cast<float*>(c->outbuf.p);
      dl = dm + rows;
      dov = dl + rows;
    }
    launch_merge(c->part.p, run.cnt, run.G, run.max_slots, (int32_t)rows, D, nullptr, nullptr, LC_F32, dm, dl, dov,
                 run.oscale, s);
    ++c->launches;
    if (!dev) {
      LC_CUDA(cudaMemcpyAsync(m, dm, rows * 4, cudaMemcpyDefault, s));
      LC_CUDA(cudaMemcpyAsync(l, dl, rows * 4, cudaMemcpyDefault, s));
      LC_CUDA(cudaMemcpyAsync(o, dov, (size_t)rows * D * 4, cudaMemcpyDefault, s));
      LC_CUDA(cudaStreamSynchronize(s));
    } else if (run.host_q) {
      LC_CUDA(cudaEventSynchronize(c->ev_copy));
    }
  });
}

int lc_merge_partials(lc_cache* c, int32_t n_parts, int32_t n_rows, const float* m, const float* l, const float* o,
                      uint32_t flags, void* out, int32_t out_dtype, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c && m && l && o && out, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_parts > 0 && n_rows > 0, LC_ERR_INVALID, "n_parts and n_rows must be > 0");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    cudaStream_t s = c->pick(stream);
    c->order(s);
    const int32_t D = c->cfg.head_dim;
    const size_t nml = (size_t)n_parts * n_rows, no = nml * D;
    // device inputs are read in place; host inputs are staged as [m | l | o]
    const bool dev = is_device_ptr(m) && is_device_ptr(l) && is_device_ptr(o);
    const float *dm = m, *dl = l, *dov = o;
    if (!dev) {
      c->part.ensure(2 * nml + no, s);
      float* base = c->part.p;
      LC_CUDA(cudaMemcpyAsync(base, m, nml * 4, cudaMemcpyDefault, s));
      LC_CUDA(cudaMemcpyAsync(base + nml, l, nml * 4, cudaMemcpyDefault, s));
      LC_CUDA(cudaMemcpyAsync(base + 2 * nml, o, no * 4, cudaMemcpyDefault, s));
      dm = base;
      dl = base + nml;
      dov = base + 2 * nml;
    }
    const size_t obytes = (size_t)n_rows * D * dtype_size(out_dtype);
    const bool host_out = !is_device_ptr(out);
    void* dout = out;
    if (host_out) {
      c->outbuf.ensure(obytes, s);
      dout = c->outbuf.p;
    }
    launch_merge_parts(dm, dl, dov, n_parts, n_rows, D, c->v_R(flags), dout, out_dtype,
                       s);
    ++c->launches;
    if (host_out) LC_CUDA(cudaMemcpyAsync(out, dout, obytes, cudaMemcpyDeviceToHost, s));
    if (host_out || !dev) LC_CUDA(cudaStreamSynchronize(s));
  });
}

// One long context split by tokens over the ranks of a group: this rank's
// partials of its shard (the decode kernels plus the slot merge, written
// straight into its block of the group's exchange buffer), the exchange,
// then the merge of all ranks' partials (native_quant_attention.rs:190-207)
// and the un-rotation, all on the stream.
int lc_decode_attn_split(lc_cache* c, lc_group* g, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                         const void* q, int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, void* out,
                         int32_t out_dtype, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c && g && out, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_seqs > 0 && n_q_heads > 0, LC_ERR_INVALID, "bad decode arguments");
    LC_REQUIRE(!(flags & LC_SPARSE_PAGES), LC_ERR_INVALID, "lc_decode_attn_split does not take LC_SPARSE_PAGES");
    LC_CUDA(cudaSetDevice(c->cfg.device));
    const int32_t D = c->cfg.head_dim;
    const int64_t rows = (int64_t)n_seqs * n_q_heads;
    LC_REQUIRE(rows <= INT32_MAX, LC_ERR_INVALID, "too many rows");
    const SplitCall x = group_begin(g, c->cfg.device, D, (int32_t)rows);
    cudaStream_t s = c->pick(stream);
    // the one-launch decode writes the shard's partials into this rank's
    // block when it applies; else the split-K slots are merged into it
    const DecodeRun run =
        decode_common(c, layer, n_seqs, seq_ids, q, q_dtype, n_q_heads, scale, flags, s, nullptr, LC_F32, nullptr,
                      x.block);
    if (!run.fused) {
      launch_merge(c->part.p, run.cnt, run.G, run.max_slots, (int32_t)rows, D, nullptr, nullptr, LC_F32, x.block,
                   x.block + rows, x.block + 2 * rows, run.oscale, s);
      ++c->launches;
    }
    group_exchange(g, x, s);
    const size_t obytes = (size_t)rows * D * dtype_size(out_dtype);
    const bool host_out = !is_device_ptr(out);
    void* dout = out;
    if (host_out) {
      c->outbuf.ensure(obytes, s);
      dout = c->outbuf.p;
    }
    launch_merge_split(x, D, c->v_R(flags), dout, out_dtype, s);
    ++c->launches;
    if (host_out) {
      LC_CUDA(cudaMemcpyAsync(out, dout, obytes, cudaMemcpyDeviceToHost, s));
      LC_CUDA(cudaStreamSynchronize(s));
    } else if (run.host_q) {
      LC_CUDA(cudaEventSynchronize(c->ev_copy));
    }
  });
}

// lc_decode_attn with every byte of scratch taken from fixed arrays
// (noalloc.cu): for callers that cannot allocate device memory while they
// decode. The work is lc_decode_attn's (query rotation, split-K partials,
// merge); only where the scratch and the per-call metadata live differs.
// Every slot the merge reads is written by the partials kernel first, so
// nothing in the scratch has to start at zero.
int lc_decode_attn_noalloc(lc_cache* c, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, const void* q,
                           int32_t q_dtype, int32_t n_q_heads, float scale, uint32_t flags, void* out,
                           int32_t out_dtype, void* stream) {
  return abi_guard([&] {
    LC_REQUIRE(c && seq_ids && q && out, LC_ERR_INVALID, "null argument");
    LC_REQUIRE(n_seqs > 0, LC_ERR_INVALID, "n_seqs must be > 0");
    const int32_t hkv = c->cfg.n_kv_heads, D = c->cfg.head_dim;
    LC_REQUIRE(n_q_heads > 0 && n_q_heads % hkv == 0, LC_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads");
    dtype_size(q_dtype);
    dtype_size(out_dtype);
    LC_CUDA(cudaSetDevice(c->cfg.device));
    LC_REQUIRE(is_device_ptr(q) && is_device_ptr(out), LC_ERR_INVALID,
               "lc_decode_attn_noalloc needs q and out in device memory");
    LC_REQUIRE(!(flags & (LC_QJL_SCORES | LC_SPARSE_PAGES)), LC_ERR_INVALID,
               "lc_decode_attn_noalloc does not take LC_QJL_SCORES or LC_SPARSE_PAGES");
    std::lock_guard<std::mutex> lock(noalloc_mutex());
    uint8_t* const dscr = noalloc_device_scratch(c->cfg.device);
    uint8_t* const hst = noalloc_host_staging();
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };

    // host staging: [seqinfo i64 2n | lens i64 n | seg i64 n+1 | cnt i32 n*hkv] then dirty table rows
    const size_t b_info = (size_t)n_seqs * 16, b_lens = (size_t)n_seqs * 8, b_seg = (size_t)(n_seqs + 1) * 8,
                 b_cnt = (size_t)n_seqs * hkv * 4;
    const size_t b_meta = b_info + b_lens + b_seg + b_cnt;
    LC_REQUIRE(b_meta <= kNoallocHostBytes, LC_ERR_NOMEM,
               "lc_decode_attn_noalloc: " + std::to_string(b_meta) + " bytes of metadata exceed the fixed " +
                   std::to_string(kNoallocHostBytes) + "-byte host staging");
    int64_t* info = reinterpret_cast<int64_t*>(hst);
    int64_t* lens = reinterpret_cast<int64_t*>(hst + b_info);
    int64_t* seg = reinterpret_cast<int64_t*>(hst + b_info + b_lens);
    int32_t* cnt = reinterpret_cast<int32_t*>(hst + b_info + b_lens + b_seg);
    size_t host_used = up(b_meta);
    for (int32_t b = 0; b < n_seqs; ++b) {
      const int32_t seq = seq_ids[b];
      c->check(seq, layer);
      const SeqLayer& sl = c->at(seq, layer);
      int64_t n = sl.ring.view_len;
      if (!sl.head_len.empty()) {
        for (int64_t hl : sl.head_len)
          LC_REQUIRE(hl == sl.head_len[0], LC_ERR_STATE, "heads of this layer hold different lengths");
        n = sl.head_len[0];
      }
      LC_REQUIRE((int64_t)sl.ring.pages.size() <= c->cfg.max_pages_per_seq, LC_ERR_NOMEM,
                 "sequence longer than max_pages_per_seq pages");
      if (sl.dirty) host_used += up(sl.ring.pages.size() * 8);
      info[2 * b] = n;
      info[2 * b + 1] = (int64_t)layer * c->cfg.max_seqs + seq;
      lens[b] = n;
    }
    LC_REQUIRE(host_used <= kNoallocHostBytes, LC_ERR_NOMEM,
               "lc_decode_attn_noalloc: " + std::to_string(host_used) + " bytes of metadata and block-table rows " +
                   "exceed the fixed " + std::to_string(kNoallocHostBytes) + "-byte host staging");
    DecodePlan plan;
    plan_decode_into(lens, n_seqs, hkv, n_q_heads, D, (int)c->kc.bits, (int)c->vc.bits, plan, seg, cnt);

    // device scratch: [seqinfo | seg | cnt] [q_rot f32 rows*D] [q_h f16 rows*D] [partials f32 rows*slots*(D+2)]
    const int64_t rows = (int64_t)n_seqs * n_q_heads;
    const size_t d_meta = up(b_info + b_seg + b_cnt), d_qrot = up((size_t)rows * D * 4), d_qh = up((size_t)rows * D * 2),
                 d_part = up((size_t)rows * plan.max_slots * (D + 2) * 4);
    const size_t need = d_meta + d_qrot + d_qh + d_part;
    LC_REQUIRE(need <= (size_t)LC_NOALLOC_SCRATCH_BYTES, LC_ERR_NOMEM,
               "lc_decode_attn_noalloc: this call needs " + std::to_string(need) +
                   " bytes of scratch; the fixed maximum is " + std::to_string((size_t)LC_NOALLOC_SCRATCH_BYTES) +
                   " (LC_NOALLOC_SCRATCH_BYTES); split the batch or use lc_decode_attn");

    // Checks done: from here on only device work is issued.
    cudaStream_t s = c->pick(stream);
    c->order(s);
    size_t hoff = up(b_meta);
    for (int32_t b = 0; b < n_seqs; ++b) {
      SeqLayer& sl = c->at(seq_ids[b], layer);
      if (!sl.dirty) continue;
      const size_t np = sl.ring.pages.size();
      uint64_t* addrs = reinterpret_cast<uint64_t*>(hst + hoff);
      for (size_t i = 0; i < np; ++i) addrs[i] = c->pool.addr(sl.ring.pages[i]);
      if (np) LC_CUDA(cudaMemcpyAsync(c->table_row(seq_ids[b], layer), addrs, np * 8, cudaMemcpyHostToDevice, s));
      hoff += up(np * 8);
      sl.dirty = false;
    }
    // one metadata copy, laid out [seqinfo | seg | cnt] on the device
    uint8_t* const dmeta = dscr;
    LC_CUDA(cudaMemcpyAsync(dmeta, info, b_info, cudaMemcpyHostToDevice, s));
    LC_CUDA(cudaMemcpyAsync(dmeta + b_info, seg, b_seg + b_cnt, cudaMemcpyHostToDevice, s));
    const int64_t* dinfo = reinterpret_cast<const int64_t*>(dmeta);
    const int64_t* dseg = plan.flat ? reinterpret_cast<const int64_t*>(dmeta + b_info) : nullptr;
    const int32_t* dcnt = reinterpret_cast<const int32_t*>(dmeta + b_info + b_seg);
    float* const q_rot = reinterpret_cast<float*>(dscr + d_meta);
    __half* const q_h = reinterpret_cast<__half*>(dscr + d_meta + d_qrot);
    float* const part = reinterpret_cast<float*>(dscr + d_meta + d_qrot + d_qh);

    const float kalpha = (plan.flat || plan.mma) ? c->dk.alpha : 1.0f,
              valpha = (plan.flat || plan.mma) ? c->dv.alpha : 1.0f;
    launch_rotate_q(q, q_dtype, (int32_t)rows, D, c->dk.RTd, (flags & LC_Q_ROTATED) != 0,
                    scale * 1.4426950408889634f / kalpha, q_rot, q_h, s);
    ++c->launches;
    DecodeArgs a;
    a.table = c->d_table;
    a.table_stride = c->cfg.max_pages_per_seq;
    a.seqinfo = dinfo;
    a.seg = dseg;
    a.layout = c->layout;
    a.role_kw = R_KW;
    a.role_vw = R_VW;
    a.role_ks = R_KS;
    a.role_vs = R_VS;
    a.n_seqs = n_seqs;
    a.hkv = hkv;
    a.hq = n_q_heads;
    a.dim = D;
    a.kbits = (int)c->kc.bits;
    a.vbits = (int)c->vc.bits;
    a.q_rot = q_rot;
    a.q_h = q_h;
    a.kcent = c->dk.cent_d;
    a.vcent = c->dv.cent_d;
    a.kalpha = kalpha;
    a.valpha = valpha;
    a.klo_thr = decode_klo_thr(c->dk.lo_max);
    a.part = part;
    launch_decode_partials(a, plan, s);
    ++c->launches;
    launch_merge(part, dcnt, n_q_heads / hkv, plan.max_slots, (int32_t)rows, D,
                 c->v_R(flags), out, out_dtype, nullptr, nullptr, nullptr,
                 1.0f / valpha, s);
    ++c->launches;
  });
}

}  // extern "C"
