// Shared host-side definitions: status handling, page layout, device tables.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "lumen_cuda.h"

namespace lc {

// Thrown inside the library, turned into a status + lc_last_error() message
// at the ABI boundary (abi_guard). Never crosses the C ABI.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);

#define LC_THROW(code, msg) throw ::lc::Error((code), (msg))
#define LC_REQUIRE(cond, code, msg)   \
  do {                                \
    if (!(cond)) LC_THROW(code, msg); \
  } while (0)
#define LC_CUDA(call)                                                                      \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      LC_THROW(LC_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));          \
  } while (0)

template <class F>
int abi_guard(F&& f) {
  try {
    f();
    return LC_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return LC_ERR_NOMEM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return LC_ERR_INVALID;
  }
}

// Tokens per page: the reference's KV_CACHE_STEP (native_cache.rs:37), the
// ring's growth quantum and the block-table granularity.
constexpr int kPageTokens = 256;
constexpr int kMaxRoles = 9;

// A page holds kPageTokens rows of every head for each role (buffer), role
// regions back to back: role r, head h, row t lives at
//   page + off[r] + (h * kPageTokens + t) * row[r].
struct PageLayout {
  int32_t heads = 0;
  int32_t n_roles = 0;
  int64_t off[kMaxRoles] = {};
  int64_t row[kMaxRoles] = {};
  int64_t page_bytes = 0;

  static PageLayout make(int32_t heads, const std::vector<int64_t>& rows) {
    PageLayout L;
    L.heads = heads;
    L.n_roles = (int32_t)rows.size();
    int64_t o = 0;
    for (size_t r = 0; r < rows.size(); ++r) {
      L.off[r] = o;
      L.row[r] = rows[r];
      o += (int64_t)heads * kPageTokens * rows[r];
      o = (o + 255) & ~int64_t(255);
    }
    L.page_bytes = o;
    return L;
  }
};

// Where rows live for a device copy: paged (logical row r in page
// pages[r / 256]) or linear ([role][head][lin_rows][row] at base + lin_off).
struct RowSpace {
  const uint64_t* pages = nullptr;  // device array of page base addresses
  uint8_t* linear = nullptr;
  int64_t lin_off[kMaxRoles] = {};
  int64_t lin_rows = 0;
};

bool is_device_ptr(const void* p);

}  // namespace lc
