// Fixed scratch of lc_decode_attn_noalloc.
//
// lc_decode_attn grows its scratch (rotated queries, split-K partials) with
// cudaMalloc when a call needs more than the last one. Some callers cannot
// allocate device memory while they decode: an engine that reserved all
// free HBM for its own page pool before its serving loop (cudaMalloc then
// fails), or a loop that must not take the device-wide synchronisation of
// cudaFree. lc_decode_attn_noalloc takes its device scratch from the
// file-scope array below instead, and its host staging from a file-scope
// host array, so a successful call allocates nothing.
//
// Set-up: the first call on a device, with that device current, looks up
// the array's device address with cudaGetSymbolAddress (which also loads
// this module on the device). Make that first call before any stream
// capture. Every call on a device shares the one array: calls that overlap
// on the GPU race.
#include <mutex>

#include "kernels.h"
#include "lumen_cuda.h"

static __device__ __align__(256) uint8_t lc_noalloc_scratch[LC_NOALLOC_SCRATCH_BYTES];

namespace lc {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_dev_addr[kMaxDevices] = {};
alignas(256) uint8_t g_host_staging[kNoallocHostBytes];
}  // namespace

std::mutex& noalloc_mutex() { return g_mu; }

uint8_t* noalloc_host_staging() { return g_host_staging; }

uint8_t* noalloc_device_scratch(int device) {
  LC_REQUIRE(device >= 0 && device < kMaxDevices, LC_ERR_INVALID, "device id out of range for the fixed scratch");
  if (!g_dev_addr[device]) {
    int cur = -1;
    LC_CUDA(cudaGetDevice(&cur));
    LC_REQUIRE(cur == device, LC_ERR_STATE, "fixed-scratch set-up needs its device current");
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, lc_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      LC_THROW(LC_ERR_CUDA, std::string("cudaGetSymbolAddress(fixed scratch): ") + cudaGetErrorString(e));
    }
    LC_REQUIRE(p != nullptr && (reinterpret_cast<uintptr_t>(p) & 255) == 0, LC_ERR_CUDA,
               "fixed scratch address is null or not 256-byte aligned");
    g_dev_addr[device] = static_cast<uint8_t*>(p);
  }
  return g_dev_addr[device];
}

}  // namespace lc
