// Expert-parallel exchange over NVLink peer memory (no NCCL on the data path).
//
// Every rank owns one exchange buffer in its own HBM, mapped into every other
// rank's process through CUDA IPC; all ranks use the same layout:
//   recv_x   [n_ranks * cap, H] bf16   rows sent TO this rank, block per source rank
//   recv_eid [n_ranks * cap] int32    local expert id of each row (-1: unused)
//   ret      [n_ranks * cap, H] bf16   expert outputs sent back TO this rank,
//                                      block per serving rank
//   flag_d   [n_ranks] int64          dispatch epoch written by each source rank
//   flag_r   [n_ranks] int64          return epoch written by each serving rank
// (the same row layout the NCCL all-to-all path produces, so the expert call
// and d3_ep_combine are shared).
//
// Per layer, three launches on each rank:
//   d3_ep_dispatch_p2p       every pair's token row and local expert id stored
//                            straight into its destination's recv_x/recv_eid
//                            (stable per-destination order); the last CTA
//                            publishes flag_d[rank] = epoch on every
//                            destination with a system-scope release;
//   d3_moe_fp8_forward_p2p   the expert call on recv_x (moe.cu): its route
//                            launch first waits for every source's flag_d,
//                            its combine launch stores each served row into
//                            the source's ret and publishes flag_r;
//   d3_ep_combine_p2p        waits for every serving rank's flag_r, then the
//                            weighted sum of the returned rows (ep.cu).
// The epoch is a device counter the dispatch launch advances once per layer,
// so every rank agrees on it without a host round trip and the whole step
// stays graph-capturable.  (d3_ep_return_p2p and d3_ep_wait are the unfused
// steps, kept for callers that run their own expert computation.)
//
// Waits spin on system-scope acquire loads with a %globaltimer budget; on
// expiry the kernel records an error code and returns.  Plain peer stores
// only: no multicast objects, no TMA on peer memory.
//
// No counterpart in the reference (it has no multi-GPU code).
#include "d3_common.cuh"

#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

namespace d3 {

// Pairs one dispatch call takes (the decode batches of the expert-parallel
// configuration route 64-512 pairs per rank).
constexpr int kP2pDispatchMaxPairs = 4096;

struct P2pDispatchParams {
  const int32_t* ids;
  int T, topk, n_ranks, rank, epr, cap;
  int32_t* recv_eid[kP2pMaxRanks];      // each destination's recv_eid
  __nv_bfloat16* recv_x[kP2pMaxRanks];  // each destination's recv_x
  long long* flag_d[kP2pMaxRanks];      // each destination's flag_d
  int32_t* src_slot;                    // [T * topk] local
  int32_t* overflow;
  long long* epoch;                     // local device epoch
  unsigned int* counter;                // local, zero between launches
  const __nv_bfloat16* x;               // [T, H]
  int H;
};

// One CTA per pair (and at least one per destination).  Every CTA counts the
// pairs per destination and, for its own pair, the pairs before it with the
// same destination (its stable rank there: pair order, as a sequential walk
// would give), then stores the pair's token row and local expert id straight
// into the destination's receive buffer.  CTA d < n_ranks also marks the
// unused rows of this source's block on destination d (-1).  The last CTA to
// finish advances the epoch and publishes it in every destination's flag_d
// with a system-scope release, after a system fence that orders every CTA's
// peer stores first (each CTA fences once, after its barrier, before its
// arrival).
__global__ void __launch_bounds__(128) p2p_dispatch_kernel(P2pDispatchParams p) {
  __shared__ int s_cnt[kP2pMaxRanks];
  __shared__ int s_before;
  __shared__ bool s_last;
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x, tid = threadIdx.x;
  const int P = p.T * p.topk, nexp = p.n_ranks * p.epr;
  if (tid < kP2pMaxRanks) s_cnt[tid] = 0;
  if (tid == 0) s_before = 0;
  __syncthreads();
  const int ei = i < P ? p.ids[i] : -1;
  const int di = (ei >= 0 && ei < nexp) ? ei / p.epr : -1;
  int before = 0;
  for (int j = tid; j < P; j += blockDim.x) {
    const int e = p.ids[j];
    const int d = (e >= 0 && e < nexp) ? e / p.epr : -1;
    if (d >= 0) {
      atomicAdd(&s_cnt[d], 1);
      before += (j < i && d == di);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
  if ((tid & 31) == 0 && before) atomicAdd(&s_before, before);
  __syncthreads();
  const long long epoch = *p.epoch + 1;  // the epoch this layer publishes
  if (i < P) {
    int slot = -1;
    if (di >= 0) {
      const int j = s_before;
      if (j < p.cap) {
        slot = di * p.cap + j;
        const uint4* src = reinterpret_cast<const uint4*>(p.x + (size_t)(i / p.topk) * p.H);
        uint4* dst = reinterpret_cast<uint4*>(p.recv_x[di] + (size_t)(p.rank * p.cap + j) * p.H);
        for (int v = tid; v < p.H / 8; v += blockDim.x) dst[v] = src[v];
        if (tid == 0) p.recv_eid[di][p.rank * p.cap + j] = ei - di * p.epr;
      } else if (tid == 0) {
        atomicAdd(p.overflow, 1);
      }
    }
    if (tid == 0) p.src_slot[i] = slot;
  }
  if (i < p.n_ranks)
    for (int j = min(s_cnt[i], p.cap) + tid; j < p.cap; j += blockDim.x)
      p.recv_eid[i][p.rank * p.cap + j] = -1;
  // one system-scope fence per CTA, after the barrier: cumulative over every
  // peer store this CTA made
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (tid == 0) __threadfence_system();
  __syncthreads();
  if (tid < p.n_ranks) st_release_sys(p.flag_d[tid] + p.rank, epoch);
  if (tid == 0) { *p.epoch = epoch; *p.counter = 0; }
}

struct P2pReturnParams {
  const __nv_bfloat16* y;               // [n_ranks * cap, H] local expert outputs
  const int32_t* recv_eid;              // local
  int n_ranks, rank, cap, H;
  __nv_bfloat16* ret[kP2pMaxRanks];     // each source's ret
  long long* flag_r[kP2pMaxRanks];      // each source's flag_r
  const long long* epoch;
  unsigned int* counter;
};

// One CTA per received row: served rows back to their source rank.
__global__ void __launch_bounds__(128) p2p_return_kernel(P2pReturnParams p) {
  __shared__ bool s_last;
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  if (p.recv_eid[row] >= 0) {
    const int s = row / p.cap, j = row - s * p.cap;
    const uint4* src = reinterpret_cast<const uint4*>(p.y + (size_t)row * p.H);
    uint4* dst = reinterpret_cast<uint4*>(p.ret[s] + (size_t)(p.rank * p.cap + j) * p.H);
    for (int v = threadIdx.x; v < p.H / 8; v += blockDim.x) dst[v] = src[v];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.n_ranks) st_release_sys(p.flag_r[threadIdx.x] + p.rank, *p.epoch);
  if (threadIdx.x == 0) *p.counter = 0;
}

// One warp: waits (bounded) until flags[r] >= *epoch for every rank r.
__global__ void p2p_wait_kernel(const long long* flags, int n_ranks, const long long* epoch,
                                int* err, int code, unsigned long long budget_ns) {
  pdl_wait();
  const bool ok = warp_wait_epochs(flags, n_ranks, *epoch, budget_ns);
  if (!ok && threadIdx.x == 0) atomicCAS(err, 0, code);
  __syncwarp();
  pdl_trigger();
}

// ---- IPC: the owning allocation of a device pointer, shared across processes

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(f);
  });
  return fn;
}

}  // namespace d3

using namespace d3;

extern "C" {

int d3_ipc_get(const void* ptr, void* handle, uint64_t* offset) {
  D3_CHECK_ARG(ptr && handle && offset, "d3_ipc_get: null pointer");
  GetAddressRangeFn fn = address_range_fn();
  if (!fn) return fail(D3_ERR_CUDA, "cuMemGetAddressRange unavailable from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(D3_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  D3_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uint64_t>(ptr) - (uint64_t)base;
  return D3_OK;
}

int d3_ipc_open(const void* handle, void** base) {
  D3_CHECK_ARG(handle && base, "d3_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  D3_CUDA_TRY(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess),
              "cudaIpcOpenMemHandle");
  return D3_OK;
}

int d3_ipc_close(void* base) {
  D3_CHECK_ARG(base, "d3_ipc_close: null pointer");
  D3_CUDA_TRY(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
  return D3_OK;
}

int d3_ep_dispatch_p2p(const void* x, const int32_t* ids, int32_t T, int32_t topk, int32_t H,
                       int32_t n_ranks, int32_t rank, int32_t experts_per_rank, int32_t cap,
                       void* const* peer_recv_x, int32_t* const* peer_recv_eid,
                       int64_t* const* peer_flag_d, int32_t* src_slot, int32_t* overflow,
                       int64_t* epoch, uint32_t* counter, d3_stream_t stream) {
  D3_CHECK_ARG(x && ids && peer_recv_x && peer_recv_eid && peer_flag_d && src_slot && overflow &&
                   epoch && counter,
               "d3_ep_dispatch_p2p: null pointer");
  D3_CHECK_ARG(T >= 1 && topk >= 1 && topk <= 64, "T, topk out of range");
  // every CTA scans all pairs for its stable rank (P^2 id loads): fine for
  // decode batches, so larger batches are refused rather than run slowly
  if ((long)T * topk > kP2pDispatchMaxPairs)
    return fail(D3_ERR_TOO_LARGE,
                "d3_ep_dispatch_p2p: T*topk = %ld exceeds %d (use d3_ep_dispatch_pack and an "
                "all-to-all for larger batches)",
                (long)T * topk, kP2pDispatchMaxPairs);
  D3_CHECK_ARG(H >= 8 && H % 8 == 0, "H must be a positive multiple of 8");
  if (n_ranks < 1 || n_ranks > kP2pMaxRanks)
    return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, %d]", kP2pMaxRanks);
  D3_CHECK_ARG(rank >= 0 && rank < n_ranks && experts_per_rank >= 1 && cap >= 1,
               "rank, experts_per_rank, cap out of range");
  if (!aligned16(x)) return fail(D3_ERR_MISALIGNED, "x must be 16-byte aligned");
  P2pDispatchParams p{};
  p.ids = ids; p.T = T; p.topk = topk; p.n_ranks = n_ranks; p.rank = rank;
  p.epr = experts_per_rank; p.cap = cap; p.src_slot = src_slot; p.overflow = overflow;
  p.epoch = reinterpret_cast<long long*>(epoch); p.counter = counter;
  p.x = static_cast<const __nv_bfloat16*>(x); p.H = H;
  for (int d = 0; d < n_ranks; ++d) {
    D3_CHECK_ARG(peer_recv_x[d] && peer_recv_eid[d] && peer_flag_d[d],
                 "d3_ep_dispatch_p2p: null peer pointer");
    if (!aligned16(peer_recv_x[d]))
      return fail(D3_ERR_MISALIGNED, "peer recv_x must be 16-byte aligned");
    p.recv_x[d] = static_cast<__nv_bfloat16*>(peer_recv_x[d]);
    p.recv_eid[d] = peer_recv_eid[d];
    p.flag_d[d] = reinterpret_cast<long long*>(peer_flag_d[d]);
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int grid = T * topk > n_ranks ? T * topk : n_ranks;
  D3_CUDA_TRY(launch_k(p2p_dispatch_kernel, dim3((unsigned)grid), dim3(128), 0, st, false, p),
              "p2p_dispatch_kernel");
  return D3_OK;
}

int d3_ep_return_p2p(const void* y, const int32_t* recv_eid, int32_t n_ranks, int32_t rank,
                     int32_t cap, int32_t H, void* const* peer_ret, int64_t* const* peer_flag_r,
                     const int64_t* epoch, uint32_t* counter, d3_stream_t stream) {
  D3_CHECK_ARG(y && recv_eid && peer_ret && peer_flag_r && epoch && counter,
               "d3_ep_return_p2p: null pointer");
  D3_CHECK_ARG(H >= 8 && H % 8 == 0 && cap >= 1, "bad shape");
  if (n_ranks < 1 || n_ranks > kP2pMaxRanks)
    return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, %d]", kP2pMaxRanks);
  D3_CHECK_ARG(rank >= 0 && rank < n_ranks, "rank out of range");
  if (!aligned16(y)) return fail(D3_ERR_MISALIGNED, "y must be 16-byte aligned");
  P2pReturnParams p{};
  p.y = static_cast<const __nv_bfloat16*>(y); p.recv_eid = recv_eid;
  p.n_ranks = n_ranks; p.rank = rank; p.cap = cap; p.H = H;
  p.epoch = reinterpret_cast<const long long*>(epoch); p.counter = counter;
  for (int s = 0; s < n_ranks; ++s) {
    D3_CHECK_ARG(peer_ret[s] && peer_flag_r[s], "d3_ep_return_p2p: null peer pointer");
    if (!aligned16(peer_ret[s])) return fail(D3_ERR_MISALIGNED, "peer ret must be 16-byte aligned");
    p.ret[s] = static_cast<__nv_bfloat16*>(peer_ret[s]);
    p.flag_r[s] = reinterpret_cast<long long*>(peer_flag_r[s]);
  }
  D3_CUDA_TRY(launch_k(p2p_return_kernel, dim3((unsigned)(n_ranks * cap)), dim3(128), 0,
                       (cudaStream_t)stream, false, p),
              "p2p_return_kernel");
  return D3_OK;
}

int d3_ep_wait(const int64_t* flags, int32_t n_ranks, const int64_t* epoch, int32_t* err_word,
               int32_t code, int64_t budget_ns, d3_stream_t stream) {
  D3_CHECK_ARG(flags && epoch && err_word, "d3_ep_wait: null pointer");
  if (n_ranks < 1 || n_ranks > 32) return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, 32]");
  D3_CHECK_ARG(budget_ns > 0, "budget_ns must be positive");
  D3_CUDA_TRY(launch_k(p2p_wait_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, false,
                       reinterpret_cast<const long long*>(flags), (int)n_ranks,
                       reinterpret_cast<const long long*>(epoch), err_word, (int)code,
                       (unsigned long long)budget_ns),
              "p2p_wait_kernel");
  return D3_OK;
}

}  // extern "C"
