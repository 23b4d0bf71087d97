// ABI plumbing: error strings, pointer classification, codec handles.
#include <cstring>
#include <string>

#include "codec.h"

namespace lc {

namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

bool is_device_ptr(const void* p) {
  if (!p) return false;
  cudaPointerAttributes at;
  const cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace lc

using namespace lc;

extern "C" {

const char* lc_last_error(void) { return g_last_error.c_str(); }

const char* lc_version(void) { return "lumen-cuda 0.1.0 (sm_100a)"; }

uint64_t lc_packed_words(uint64_t n, uint32_t bits) {
  if (bits == 0 || bits > 64) return 0;
  const uint64_t cpw = 64 / bits;
  return (n + cpw - 1) / cpw;
}

int lc_codec_new(uint32_t bits, uint64_t qjl_m, uint64_t seed, uint64_t lloyd_max_iter, uint64_t head_dim,
                 lc_codec** out) {
  return abi_guard([&] {
    LC_REQUIRE(out, LC_ERR_INVALID, "null out");
    *out = nullptr;
    auto* h = new lc_codec;
    try {
      h->c = Codec::generate(bits, qjl_m, seed, lloyd_max_iter, head_dim);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int lc_codec_from_files(const char* codebook_path, const char* rotation_path, const char* qjl_path, lc_codec** out) {
  return abi_guard([&] {
    LC_REQUIRE(out, LC_ERR_INVALID, "null out");
    *out = nullptr;
    auto* h = new lc_codec;
    try {
      h->c = Codec::from_files(codebook_path, rotation_path, qjl_path);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int lc_codec_from_tables(uint64_t head_dim, uint32_t bits, uint64_t qjl_m, const float* rotation,
                         const double* boundaries, const double* centroids, const float* qjl_proj, lc_codec** out) {
  return abi_guard([&] {
    LC_REQUIRE(out, LC_ERR_INVALID, "null out");
    *out = nullptr;
    auto* h = new lc_codec;
    try {
      h->c = Codec::from_tables(head_dim, bits, qjl_m, rotation, boundaries, centroids, qjl_proj);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int lc_codec_save(const lc_codec* c, const char* codebook_path, const char* rotation_path, const char* qjl_path) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null codec");
    c->c.save(codebook_path, rotation_path, qjl_path);
  });
}

int lc_codec_tables(const lc_codec* c, float* rotation, double* boundaries, double* centroids, float* qjl_proj) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null codec");
    if (rotation) std::memcpy(rotation, c->c.R.data(), c->c.R.size() * 4);
    if (boundaries) std::memcpy(boundaries, c->c.bounds.data(), c->c.bounds.size() * 8);
    if (centroids) std::memcpy(centroids, c->c.cents.data(), c->c.cents.size() * 8);
    if (qjl_proj && !c->c.P.empty()) std::memcpy(qjl_proj, c->c.P.data(), c->c.P.size() * 4);
  });
}

int lc_codec_shape(const lc_codec* c, uint64_t* head_dim, uint32_t* bits, uint64_t* qjl_m) {
  return abi_guard([&] {
    LC_REQUIRE(c, LC_ERR_INVALID, "null codec");
    if (head_dim) *head_dim = c->c.dim;
    if (bits) *bits = c->c.bits;
    if (qjl_m) *qjl_m = c->c.m;
  });
}

void lc_codec_free(lc_codec* c) { delete c; }

}  // extern "C"
