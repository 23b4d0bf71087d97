// The sequence-split group behind lc_decode_attn_split: the ranks holding
// the token shards of one long context exchange their softmax partials
// (m, l, o) every call, then each merges them.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

struct lc_group;

namespace lc {

// One call's view of the group's exchange buffers. Every rank's partials
// block is [m: rows][l: rows][o: rows * head_dim] f32, and the blocks of
// ranks 0..world-1 sit block_stride floats apart in `parts` (this device's
// memory). `block` is this rank's block inside `parts`, where its partials
// are written.
struct SplitCall {
  float* block = nullptr;
  const float* parts = nullptr;
  int64_t block_stride = 0;
  int32_t world = 1, rank = 0, rows = 0;
  // peer-store exchange: the merge waits until every flag reaches `epoch`
  const uint32_t* wait_flags = nullptr;
  int32_t wait_n = 0;
  uint32_t epoch = 0;
  uint32_t* status = nullptr;  // mapped host word: set when a wait ran out
};

// Checks the group against the call (device, head_dim, rows) and returns
// the buffers of the next exchange.
SplitCall group_begin(lc_group* g, int32_t device, int32_t head_dim, int32_t rows);
// Moves this rank's block to every rank: peer stores over NVLink plus
// release flags, or one in-place NCCL all-gather.
void group_exchange(lc_group* g, const SplitCall& x, cudaStream_t s);

// Merge of the world partials of a split call into out [rows][head_dim]
// (un-rotated by R unless null), after the flag wait when x.wait_flags is
// set (decode.cu).
void launch_merge_split(const SplitCall& x, int32_t D, const float* R, void* out, int32_t out_dtype,
                        cudaStream_t s);

}  // namespace lc
