// Expert-parallel dispatch/combine around the expert GEMM (resident config:
// experts sharded evenly over the ranks, tokens exchanged by all-to-all).
//
// No counterpart exists in the reference (it has no multi-GPU code); this is
// the B200 configuration BASELINE configs[4] asks for.  The exchange uses a
// STATIC per-destination capacity `cap` so every buffer shape -- and hence the
// NCCL all-to-all sizes -- is fixed and the whole step can be captured into a
// CUDA graph with no host sync:
//
//   pack:     pair (t, k) with expert e goes to rank d = e / experts_per_rank,
//             row d*cap + j of the send buffer (j = its rank among the pairs
//             to d, in pair order -- stable, deterministic); the row carries
//             x[t] and the local expert id e - d*experts_per_rank; unused rows
//             carry id -1 (the GEMM skips them).  src_slot[t,k] remembers the
//             row.
//   (all-to-all: the row block for rank d lands at rank d)
//   GEMM:     each received row is one (token, expert) pair, topk = 1
//   (all-to-all back)
//   combine:  out[t] (+)= sum_k w[t,k] * ret[src_slot[t,k]]  (fixed k order)
#include "d3_common.cuh"

#include <cuda_bf16.h>

namespace d3 {

constexpr int kEpMaxRanks = 64;

struct EpPackParams {
  const int32_t* ids; int T, topk, n_ranks, epr, cap;
  int32_t* send_eid;     // [n_ranks * cap]
  int32_t* src_slot;     // [T * topk]
  int32_t* overflow;     // device word: pairs dropped for lack of capacity
};

// One warp walks the pairs in order 32 at a time (stable ranks per
// destination); then the block marks the unused rows.
__global__ void __launch_bounds__(256) ep_plan_kernel(EpPackParams p) {
  __shared__ int cursor[kEpMaxRanks];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31;
  for (int d = tid; d < p.n_ranks; d += blockDim.x) cursor[d] = 0;
  __syncthreads();
  const int P = p.T * p.topk;
  if (tid < 32) {
    for (int b0 = 0; b0 < P; b0 += 32) {
      const int i = b0 + lane;
      const int e = i < P ? p.ids[i] : -1;
      const int d = (e >= 0 && e < p.n_ranks * p.epr) ? e / p.epr : -1;
      const unsigned m = __match_any_sync(0xffffffffu, d);
      const int leader = __ffs(m) - 1;
      const int rank = __popc(m & ((1u << lane) - 1));
      int base = 0;
      if (lane == leader && d >= 0) {
        base = cursor[d];
        cursor[d] = base + __popc(m);
      }
      base = __shfl_sync(0xffffffffu, base, leader);
      if (i < P) {
        int slot = -1;
        if (d >= 0) {
          const int j = base + rank;
          if (j < p.cap) {
            slot = d * p.cap + j;
            p.send_eid[slot] = e - d * p.epr;
          } else {
            atomicAdd(p.overflow, 1);
          }
        }
        p.src_slot[i] = slot;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int d = 0; d < p.n_ranks; ++d)
    for (int j = cursor[d] + tid; j < p.cap; j += blockDim.x) p.send_eid[d * p.cap + j] = -1;
}

// One CTA per pair: copy x[t] into its send row.
// src_slot is written by the overlapping plan launch: no __restrict__ (no
// non-coherent reads of it).
__global__ void __launch_bounds__(128) ep_copy_kernel(const __nv_bfloat16* x,
                                                      const int32_t* src_slot, int topk, int H,
                                                      __nv_bfloat16* __restrict__ send_x) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const int slot = src_slot[i];
  if (slot < 0) return;
  const int t = i / topk;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  uint4* dst = reinterpret_cast<uint4*>(send_x + (size_t)slot * H);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
}

// One thread per 4 columns of a token: out[t] = bf16([out[t] +] sum_k w[t,k] *
// ret[src_slot[t,k]]), k in order.  With wait_flags set (NVLink return), one
// warp of every CTA first waits for every serving rank's return epoch; the
// CTA barrier after it orders all of the CTA's reads of ret after the acquire
// (ret is written by other GPUs: no read-only-path loads).
__global__ void ep_combine_kernel(const __nv_bfloat16* ret, const int32_t* __restrict__ src_slot,
                                  const void* __restrict__ weights, int weights_f32, int T,
                                  int topk, int H, int accumulate,
                                  __nv_bfloat16* __restrict__ out, const long long* wait_flags,
                                  int wait_n, const long long* wait_epoch, int* err, int code,
                                  unsigned long long budget_ns) {
  pdl_trigger();
  pdl_wait();
  if (wait_flags) {
    if (threadIdx.x < 32 && !warp_wait_epochs(wait_flags, wait_n, *wait_epoch, budget_ns) &&
        threadIdx.x == 0)
      atomicCAS(err, 0, code);
    __syncthreads();
  }
  const int t = blockIdx.y;
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= T || j >= H) return;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (accumulate) {
    const uint2 raw = *reinterpret_cast<const uint2*>(out + (size_t)t * H + j);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = __bfloat162float(b[q]);
  }
  for (int k = 0; k < topk; ++k) {
    const int slot = src_slot[t * topk + k];
    if (slot < 0) continue;
    const float wk = weights_f32 ? static_cast<const float*>(weights)[t * topk + k]
                                 : __bfloat162float(
                                       static_cast<const __nv_bfloat16*>(weights)[t * topk + k]);
    const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(ret + (size_t)slot * H + j));
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = fmaf(wk, __bfloat162float(b[q]), acc[q]);
  }
  __nv_bfloat16 o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = __float2bfloat16_rn(acc[q]);
  *reinterpret_cast<uint2*>(out + (size_t)t * H + j) = *reinterpret_cast<uint2*>(o);
}

}  // namespace d3

using namespace d3;

extern "C" {

int d3_ep_dispatch_pack(const void* x, const int32_t* ids, int32_t T, int32_t topk, int32_t H,
                        int32_t n_ranks, int32_t experts_per_rank, int32_t cap, void* send_x,
                        int32_t* send_eid, int32_t* src_slot, int32_t* overflow,
                        d3_stream_t stream) {
  D3_CHECK_ARG(x && ids && send_x && send_eid && src_slot && overflow,
               "d3_ep_dispatch_pack: null pointer");
  D3_CHECK_ARG(T >= 1 && topk >= 1 && topk <= 64 && (long)T * topk <= 65536,
               "T, topk out of range");
  D3_CHECK_ARG(H >= 8 && H % 8 == 0, "H must be a positive multiple of 8");
  if (n_ranks < 1 || n_ranks > kEpMaxRanks)
    return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, %d]", kEpMaxRanks);
  D3_CHECK_ARG(experts_per_rank >= 1 && cap >= 1, "experts_per_rank and cap must be >= 1");
  if (!aligned16(x) || !aligned16(send_x))
    return fail(D3_ERR_MISALIGNED, "x and send_x must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  EpPackParams p{ids, T, topk, n_ranks, experts_per_rank, cap, send_eid, src_slot, overflow};
  // first launch of the call: an ordinary stream dependent of the caller's work
  D3_CUDA_TRY(launch_k(ep_plan_kernel, dim3(1), dim3(256), 0, st, false, p), "ep_plan_kernel");
  D3_CUDA_TRY(launch_k(ep_copy_kernel, dim3((unsigned)(T * topk)), dim3(128), 0, st, pdl,
                       static_cast<const __nv_bfloat16*>(x), (const int32_t*)src_slot, topk, H,
                       static_cast<__nv_bfloat16*>(send_x)),
              "ep_copy_kernel");
  return D3_OK;
}

static int ep_combine(const void* ret, const int32_t* src_slot, const void* weights,
                      int32_t weights_f32, int32_t T, int32_t topk, int32_t H, void* out,
                      int32_t accumulate, const int64_t* wait_flags, int32_t wait_n,
                      const int64_t* epoch, int32_t* err_word, int32_t code, int64_t budget_ns,
                      d3_stream_t stream) {
  D3_CHECK_ARG(ret && src_slot && weights && out, "d3_ep_combine: null pointer");
  D3_CHECK_ARG(T >= 1 && topk >= 1 && H >= 4 && H % 4 == 0, "bad shape");
  if (!aligned16(ret) || !aligned16(out)) return fail(D3_ERR_MISALIGNED, "ret/out not aligned");
  const dim3 grid((unsigned)((H / 4 + 127) / 128), (unsigned)T);
  D3_CUDA_TRY(launch_k(ep_combine_kernel, grid, dim3(128), 0, (cudaStream_t)stream, false,
                       static_cast<const __nv_bfloat16*>(ret), src_slot, weights, weights_f32, T,
                       topk, H, accumulate ? 1 : 0, static_cast<__nv_bfloat16*>(out),
                       reinterpret_cast<const long long*>(wait_flags), (int)wait_n,
                       reinterpret_cast<const long long*>(epoch), err_word, (int)code,
                       (unsigned long long)budget_ns),
              "ep_combine_kernel");
  return D3_OK;
}

int d3_ep_combine(const void* ret, const int32_t* src_slot, const void* weights,
                  int32_t weights_f32, int32_t T, int32_t topk, int32_t H, void* out,
                  int32_t accumulate, d3_stream_t stream) {
  return ep_combine(ret, src_slot, weights, weights_f32, T, topk, H, out, accumulate, nullptr, 0,
                    nullptr, nullptr, 0, 0, stream);
}

int d3_ep_combine_p2p(const void* ret, const int32_t* src_slot, const void* weights,
                      int32_t weights_f32, int32_t T, int32_t topk, int32_t H, void* out,
                      int32_t accumulate, const int64_t* flag_r, int32_t n_ranks,
                      const int64_t* epoch, int32_t* err_word, int32_t code, int64_t budget_ns,
                      d3_stream_t stream) {
  D3_CHECK_ARG(flag_r && epoch && err_word, "d3_ep_combine_p2p: null pointer");
  if (n_ranks < 1 || n_ranks > 32) return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, 32]");
  D3_CHECK_ARG(budget_ns > 0, "budget_ns must be positive");
  return ep_combine(ret, src_slot, weights, weights_f32, T, topk, H, out, accumulate, flag_r,
                    n_ranks, epoch, err_word, code, budget_ns, stream);
}

}  // extern "C"
