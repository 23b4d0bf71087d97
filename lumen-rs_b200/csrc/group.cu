// Sequence-split groups (lc_group_*): the exchange of softmax partials
// between the ranks that hold the token shards of one long context.
//
// Every rank owns one exchange buffer on its GPU: two parities of
// [world][block] f32 partials blocks, then a flag array [world][kPushCtas].
// Call e (epoch e, parity e & 1) runs on every rank as
//   partials -> this rank's block        (the decode kernels + slot merge)
//   k_split_push                         (peer stores of the block into every
//                                         rank's buffer over NVLink, then a
//                                         release store of flag[rank][cta] = e
//                                         on every rank)
//   merge (k_merge)                      (acquire-waits until all world x
//                                         kPushCtas flags reach e, bounded,
//                                         then merges the world blocks)
// The peers' buffers are mapped with CUDA IPC; the handles travel through
// one NCCL all-gather at creation. Two parities suffice: a rank reaches call
// e + 2's push only after its call e + 1 merge saw every rank's e + 1 flag,
// and each rank raises that flag only after its own call e merge is done
// (stream order), so no rank can still be reading the parity being
// overwritten. When the buffers cannot be mapped (or LC_GROUP_NCCL asks),
// the exchange is one in-place ncclAllGather on the same layout instead.
//
// A bounded wait that runs out sets a word in mapped host memory; the
// merge then writes NaN rows, and the group's next call (lc_group_status)
// reports LC_ERR_TIMEOUT. No wait spins forever.
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "group.h"
#include "kernels.h"

namespace lc {
namespace {

constexpr int kMaxGroup = 8;
constexpr int kPushCtas = 8;

struct PushArgs {
  const float* src;             // this rank's block (local)
  float* dst[kMaxGroup];        // rank r's copy of this rank's block (null: this rank)
  uint32_t* flag[kMaxGroup];    // rank r's flag[this rank][0..kPushCtas)
  int32_t world;
  int64_t n4;                   // float4s to copy
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA c copies its share of the block to every other rank (16-byte peer
// stores), fences at system scope, and the CTA's first `world` threads then
// raise flag[rank][c] = epoch on every rank.
__global__ void __launch_bounds__(256) k_split_push(PushArgs a) {
  const int64_t per = (a.n4 + kPushCtas - 1) / kPushCtas;
  const int64_t i0 = blockIdx.x * per, i1 = min(a.n4, i0 + per);
  const float4* s = reinterpret_cast<const float4*>(a.src);
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const float4 v = s[i];
#pragma unroll
    for (int r = 0; r < kMaxGroup; ++r)
      if (r < a.world && a.dst[r]) reinterpret_cast<float4*>(a.dst[r])[i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.world) st_release_sys(a.flag[threadIdx.x] + blockIdx.x, a.epoch);
}

void nccl_check(ncclResult_t r, const char* what) {
  LC_REQUIRE(r == ncclSuccess, LC_ERR_CUDA, std::string(what) + ": " + ncclGetErrorString(r));
}

}  // namespace
}  // namespace lc

using namespace lc;

struct lc_group {
  int32_t world = 1, rank = 0, device = 0, max_rows = 0, head_dim = 0;
  bool p2p = false;
  ncclComm_t comm = nullptr;
  int64_t block = 0;           // floats between ranks' blocks
  float* buf = nullptr;        // [2][world][block] then flags
  uint32_t* flags = nullptr;   // [world][kPushCtas], in buf's allocation
  float* peer_buf[kMaxGroup] = {};
  uint32_t epoch = 0;
  uint32_t* status_h = nullptr;  // mapped pinned word
  uint32_t* status_d = nullptr;

  float* parts(float* base, int parity) const { return base + (int64_t)parity * world * block; }
  uint32_t* flags_of(float* base) const {
    return reinterpret_cast<uint32_t*>(base + (int64_t)2 * world * block);
  }
  ~lc_group() {
    for (int r = 0; r < kMaxGroup; ++r)
      if (peer_buf[r] && peer_buf[r] != buf) cudaIpcCloseMemHandle(peer_buf[r]);
    if (comm) ncclCommDestroy(comm);
    if (buf) cudaFree(buf);
    if (status_h) cudaFreeHost(status_h);
  }
};

namespace lc {

SplitCall group_begin(lc_group* g, int32_t device, int32_t head_dim, int32_t rows) {
  LC_REQUIRE(g, LC_ERR_INVALID, "null group");
  LC_REQUIRE(device == g->device, LC_ERR_INVALID, "the group lives on another device than the cache");
  LC_REQUIRE(head_dim == g->head_dim, LC_ERR_INVALID, "the group was created for another head_dim");
  LC_REQUIRE(rows > 0 && rows <= g->max_rows, LC_ERR_INVALID,
             "rows (n_seqs * n_q_heads) exceed the group's max_rows");
  LC_REQUIRE(*(volatile uint32_t*)g->status_h == 0, LC_ERR_TIMEOUT,
             "an earlier exchange timed out waiting for a peer's partials; the group is unusable");
  SplitCall x;
  x.epoch = ++g->epoch;
  float* base = g->parts(g->buf, (int)(x.epoch & 1));
  x.parts = base;
  x.block = base + (int64_t)g->rank * g->block;
  x.block_stride = g->block;
  x.world = g->world;
  x.rank = g->rank;
  x.rows = rows;
  if (g->p2p) {
    x.wait_flags = g->flags;
    x.wait_n = g->world * kPushCtas;
    x.status = g->status_d;
  }
  return x;
}

void group_exchange(lc_group* g, const SplitCall& x, cudaStream_t s) {
  if (g->world == 1) return;
  const int parity = (int)(x.epoch & 1);
  if (g->p2p) {
    PushArgs a{};
    a.src = x.block;
    a.world = g->world;
    a.n4 = ((int64_t)x.rows * (g->head_dim + 2) + 3) / 4;
    a.epoch = x.epoch;
    for (int r = 0; r < g->world; ++r) {
      a.dst[r] = r == g->rank ? nullptr : g->parts(g->peer_buf[r], parity) + (int64_t)g->rank * g->block;
      a.flag[r] = g->flags_of(g->peer_buf[r]) + (int64_t)g->rank * kPushCtas;
    }
    k_split_push<<<kPushCtas, 256, 0, s>>>(a);
    LC_CUDA(cudaGetLastError());
  } else {
    nccl_check(ncclAllGather(x.block, const_cast<float*>(x.parts), (size_t)g->block, ncclFloat, g->comm, s),
               "ncclAllGather");
  }
}

}  // namespace lc

extern "C" {

int lc_group_id(uint8_t* id) {
  return abi_guard([&] {
    LC_REQUIRE(id, LC_ERR_INVALID, "null id");
    static_assert(sizeof(ncclUniqueId) == LC_GROUP_ID_BYTES, "ncclUniqueId size");
    ncclUniqueId u;
    nccl_check(ncclGetUniqueId(&u), "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof(u));
  });
}

int lc_group_create(int32_t world, int32_t rank, const uint8_t* id, int32_t device, int32_t max_rows,
                    int32_t head_dim, uint32_t flags, lc_group** out) {
  return abi_guard([&] {
    LC_REQUIRE(out && id, LC_ERR_INVALID, "null argument");
    *out = nullptr;
    LC_REQUIRE(world >= 1 && world <= kMaxGroup, LC_ERR_INVALID, "world must be 1..8 (one node)");
    LC_REQUIRE(rank >= 0 && rank < world, LC_ERR_INVALID, "rank must be in [0, world)");
    LC_REQUIRE(max_rows > 0 && (head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512),
               LC_ERR_INVALID, "max_rows must be > 0 and head_dim 64, 128, 256 or 512");
    LC_CUDA(cudaSetDevice(device));
    auto* g = new lc_group;
    try {
      g->world = world;
      g->rank = rank;
      g->device = device;
      g->max_rows = max_rows;
      g->head_dim = head_dim;
      g->block = ((int64_t)max_rows * (head_dim + 2) + 63) & ~int64_t(63);
      ncclUniqueId u;
      std::memcpy(&u, id, sizeof(u));
      nccl_check(ncclCommInitRank(&g->comm, world, u, rank), "ncclCommInitRank");
      if (world > 1) {  // peer stores write blocks of this size into every rank's buffer
        int64_t hv[2] = {g->block, -g->block};
        int64_t* dv = nullptr;
        LC_CUDA(cudaMalloc(&dv, sizeof(hv)));
        LC_CUDA(cudaMemcpy(dv, hv, sizeof(hv), cudaMemcpyHostToDevice));
        const ncclResult_t r = ncclAllReduce(dv, dv, 2, ncclInt64, ncclMin, g->comm, nullptr);
        const cudaError_t e = cudaMemcpy(hv, dv, sizeof(hv), cudaMemcpyDeviceToHost);
        cudaFree(dv);
        nccl_check(r, "ncclAllReduce (group shape)");
        LC_CUDA(e);
        LC_REQUIRE(hv[0] == g->block && -hv[1] == g->block, LC_ERR_INVALID,
                   "every rank must create the group with the same max_rows and head_dim");
      }
      const size_t bytes = (size_t)2 * world * g->block * 4 + (size_t)world * kPushCtas * 4;
      LC_CUDA(cudaMalloc(&g->buf, bytes));
      LC_CUDA(cudaMemset(g->buf, 0, bytes));
      g->flags = g->flags_of(g->buf);
      LC_CUDA(cudaHostAlloc(&g->status_h, sizeof(uint32_t), cudaHostAllocMapped));
      *g->status_h = 0;
      LC_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&g->status_d), g->status_h, 0));
      LC_CUDA(cudaDeviceSynchronize());
      for (int r = 0; r < kMaxGroup; ++r) g->peer_buf[r] = nullptr;
      g->peer_buf[rank] = g->buf;
      if (world > 1 && !(flags & LC_GROUP_NCCL)) {
        // exchange IPC handles, map the peers' buffers; every rank learns
        // whether all of them succeeded, so all take the same exchange
        cudaIpcMemHandle_t h;
        int ok = cudaIpcGetMemHandle(&h, g->buf) == cudaSuccess ? 1 : 0;
        cudaGetLastError();
        std::vector<uint8_t> hs((size_t)world * sizeof(h));
        uint8_t* dh = nullptr;
        int* dok = nullptr;
        LC_CUDA(cudaMalloc(&dh, hs.size()));
        LC_CUDA(cudaMalloc(&dok, sizeof(int)));
        LC_CUDA(cudaMemcpy(dh + (size_t)rank * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice));
        nccl_check(ncclAllGather(dh + (size_t)rank * sizeof(h), dh, sizeof(h), ncclUint8, g->comm, nullptr),
                   "ncclAllGather (IPC handles)");
        LC_CUDA(cudaMemcpy(hs.data(), dh, hs.size(), cudaMemcpyDeviceToHost));
        for (int r = 0; r < world && ok; ++r) {
          if (r == rank) continue;
          cudaIpcMemHandle_t hr;
          std::memcpy(&hr, hs.data() + (size_t)r * sizeof(h), sizeof(h));
          void* p = nullptr;
          if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess) {
            g->peer_buf[r] = static_cast<float*>(p);
          } else {
            cudaGetLastError();
            ok = 0;
          }
        }
        LC_CUDA(cudaMemcpy(dok, &ok, sizeof(int), cudaMemcpyHostToDevice));
        nccl_check(ncclAllReduce(dok, dok, 1, ncclInt32, ncclMin, g->comm, nullptr), "ncclAllReduce (IPC check)");
        LC_CUDA(cudaMemcpy(&ok, dok, sizeof(int), cudaMemcpyDeviceToHost));
        cudaFree(dh);
        cudaFree(dok);
        g->p2p = ok == 1;
        if (!g->p2p) {
          for (int r = 0; r < world; ++r) {
            if (r != rank && g->peer_buf[r]) cudaIpcCloseMemHandle(g->peer_buf[r]);
            if (r != rank) g->peer_buf[r] = nullptr;
          }
        }
      }
    } catch (...) {
      delete g;
      throw;
    }
    *out = g;
  });
}

int lc_group_info(const lc_group* g, int32_t* world, int32_t* rank, int32_t* peer_stores) {
  return abi_guard([&] {
    LC_REQUIRE(g, LC_ERR_INVALID, "null group");
    if (world) *world = g->world;
    if (rank) *rank = g->rank;
    if (peer_stores) *peer_stores = g->p2p ? 1 : 0;
  });
}

int lc_group_status(const lc_group* g) {
  return abi_guard([&] {
    LC_REQUIRE(g, LC_ERR_INVALID, "null group");
    LC_REQUIRE(*(volatile uint32_t*)g->status_h == 0, LC_ERR_TIMEOUT,
               "an exchange timed out waiting for a peer's partials");
  });
}

int lc_group_destroy(lc_group* g) {
  return abi_guard([&] {
    if (!g) return;
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    delete g;
  });
}

}  // extern "C"
