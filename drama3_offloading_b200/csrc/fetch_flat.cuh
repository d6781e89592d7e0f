// The flat multi-buffer fetch shared by the fetch launch (fetch.cu) and the
// fetch + gate/up overlap launch (moe.cu): the bytes of every queued job
// (missed expert) in every buffer form one range of 16-byte vectors that the
// fetching CTAs stride over in chunks of kFetchThreads * kFetchUnroll vectors
// (16 KiB), four 16-byte loads of mapped host memory in flight per thread.
#pragma once

#include "d3_common.cuh"

namespace d3 {

struct FetchParams {
  const uint4* host[D3_MAX_BUFFERS];
  uint4* cache[D3_MAX_BUFFERS];
  int64_t vecs[D3_MAX_BUFFERS];   // 16-byte vectors per expert, per buffer
  int64_t vec_total;              // sum over buffers
  int32_t nbuf;
  const int32_t* fetch_slot;
  const int32_t* fetch_expert;
  const int32_t* nmiss;
};

constexpr int kFetchThreads = 256;
constexpr int kFetchUnroll = 4;

// Resolve launch for one layer (fetch.cu), with `zero` [nzero] int64 cleared
// by the same launch; fills *fp for a fetch of the queued jobs.  launch =
// false only validates the descriptor and fills *fp (the jobs queued by an
// earlier allocator launch).
int resolve_for_fetch(const d3_layer_cache* L, const void* ids, int32_t ids_bytes, int32_t k,
                      int64_t* zero, int32_t nzero, cudaStream_t st, FetchParams* fp,
                      int64_t* expert_bytes, bool launch = true);

}  // namespace d3
