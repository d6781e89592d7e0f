// MoE router: logits = x @ gate_w^T, softmax, top-k, renormalisation.
//
// Semantics of the upstream fish-speech router the reference calls into
// (gate Linear -> softmax -> top-8 -> norm_topk_prob renorm; quoted at
// notes/01-static-findings.md:133-138): logits are bf16, the softmax runs in
// fp32, ties in the top-k go to the lower expert index.  Expert ids must be
// bit-exact, so every logit is the EXACTLY ROUNDED bf16 of the dot product:
// the bf16 x bf16 products are exact in fp64 and accumulate in fp64 (error
// ~1e-16 relative, far below a bf16 ulp), then round to fp32 and to bf16,
// both round-to-nearest-even.  Any other accumulation order only changes the
// fp64 sum's last bits, so every correct implementation agrees on the ids.
//
// Two kernels share the arithmetic and the selection:
// * T <= 2 (decode): one thread-block cluster of 16 CTAs; each CTA computes
//   E/16 experts' logits and stores them into the leader CTA's shared memory
//   over distributed shared memory; after one cluster barrier the leader
//   selects.  No global scratch.
// * T > 2: grid (E / 8 experts, ceil(T / 8) token tiles), 8 warps, one expert
//   per warp over a tile of 8 tokens staged in shared memory (each gate row is
//   read once per token tile); up to 16 tokens each expert is split over 4
//   warps (2 experts per CTA, 4x the CTAs), the partial sums added in order.  The last CTA of a token tile to finish (a
//   global arrival counter, reset by that CTA for the next launch or graph
//   replay) selects the top-k of its tokens from the workspace logits.
// Selection: one warp per token, logits 32-strided over the lanes, k rounds of
// a single warp max-reduction over (order-preserving value code, inverted
// index) keys, so ties go to the lower index.
#include "d3_common.cuh"

#include <cuda_bf16.h>

#include <mutex>

namespace d3 {

constexpr int kRouterExpertsPerCta = 8;   // one per warp
constexpr int kRouterTokensPerCta = 8;
constexpr int kRouterMaxH = 8192;
constexpr int kRouterMaxE = 1024;
constexpr int kRouterMaxT = 65536;
// Workspace layout: the per-token-tile arrival counters live at a FIXED offset
// 0 (room for kRouterMaxT tokens), the logits after them, so a workspace
// reused across calls with different T never finds stale logits where a
// counter should be zero.
constexpr size_t kRouterCounterBytes =
    ((size_t)(kRouterMaxT / kRouterTokensPerCta) * sizeof(unsigned) + 255) & ~(size_t)255;

struct RouterParams {
  const __nv_bfloat16* x;     // [T, H]
  const __nv_bfloat16* w;     // [E, H]
  int32_t T, H, E, topk, renorm;
  float* logits;              // workspace [T, E] (bf16 values held in fp32)
  unsigned int* arrivals;     // workspace [ceil(T/8)], zero between launches
  int32_t* ids_out;           // [T, topk]
  float* weights_out;         // [T, topk] or null
  __nv_bfloat16* weights_bf16_out;  // [T, topk] or null
};

__device__ __forceinline__ float exact_bf16_of(double s) {
  return __bfloat162float(__float2bfloat16_rn(__double2float_rn(s)));
}

// Selection key of a logit (a bf16 value held in fp32): the order-preserving
// 16-bit code of the value above the inverted expert index, so the unsigned
// maximum is the largest logit, ties to the lower index.  -0 is folded into
// +0 (they compare equal); 0 is below every real key and marks "taken".
__device__ __forceinline__ unsigned topk_key(float v, int i) {
  const unsigned b = __float_as_uint(v + 0.0f) >> 16;
  const unsigned code = (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
  return (code << 16) | (0xffffu - (unsigned)i);
}

__device__ __forceinline__ float topk_key_value(unsigned key) {
  const unsigned code = key >> 16;
  const unsigned b = (code & 0x8000u) ? (code & 0x7fffu) : (~code & 0xffffu);
  return __uint_as_float(b << 16);
}

// Top-k of token t's logits, held by one warp 32-strided (v[j] = logit
// j*32 + lane, -inf past E; per = ceil(E/32)): fp32 softmax (max, then the
// per-lane sums in j order combined by a butterfly), k rounds of one warp
// max-reduction over the selection keys (a tree over the lane's KPER keys,
// then one redux; lane r keeps round r's winner), then the k probabilities
// in parallel, their sum in round order and the optional renormalisation.
template <int KPER>
__device__ __forceinline__ void topk_select(const float (&v)[KPER], int per, int t,
                                            const RouterParams& p) {
  static_assert((KPER & (KPER - 1)) == 0, "KPER must be a power of two");
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < KPER; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  float denom = 0.f;
  unsigned key[KPER];
#pragma unroll
  for (int j = 0; j < KPER; ++j) {
    const int i = j * 32 + lane;
    const bool live = j < per && i < p.E;
    if (live) denom += expf(v[j] - mx);
    key[j] = live ? topk_key(v[j], i) : 0u;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, off);
  unsigned my_win = 0u;
  for (int r = 0; r < p.topk; ++r) {
    unsigned m[KPER];
#pragma unroll
    for (int j = 0; j < KPER; ++j) m[j] = key[j];
#pragma unroll
    for (int w = KPER / 2; w >= 1; w >>= 1)
#pragma unroll
      for (int j = 0; j < w; ++j) m[j] = max(m[j], m[j + w]);
    const unsigned win = __reduce_max_sync(0xffffffffu, m[0]);
    if (lane == r) my_win = win;
#pragma unroll
    for (int j = 0; j < KPER; ++j)
      if (key[j] == win) key[j] = 0u;
  }
  int sel_id = -1;
  float sel_w = 0.f;
  if (lane < p.topk) {
    sel_id = 0xffff - (int)(my_win & 0xffffu);
    sel_w = expf(topk_key_value(my_win) - mx) / denom;
  }
  float sel_sum = 0.f;
  for (int r = 0; r < p.topk; ++r) sel_sum += __shfl_sync(0xffffffffu, sel_w, r);
  if (lane < p.topk) {
    const float wgt = p.renorm ? sel_w / sel_sum : sel_w;
    p.ids_out[(size_t)t * p.topk + lane] = sel_id;
    if (p.weights_out) p.weights_out[(size_t)t * p.topk + lane] = wgt;
    if (p.weights_bf16_out) p.weights_bf16_out[(size_t)t * p.topk + lane] = __float2bfloat16_rn(wgt);
  }
}

// bf16 bit pattern (low 16 bits of b, or the high half of a packed pair
// with hi = true) -> the same value as a double: the bits placed in the upper
// half of an fp32 word ARE that value as an fp32 (same exponent range), and
// fp32 -> fp64 is exact; one logic op and one conversion per value.
// (Measured on B200 inside the decode router: the fp64 dot products of a
// 16-SM cluster took 1.9 us this way against 3.8 us when the double was
// assembled from the bits by ~12 integer operations.)
__device__ __forceinline__ double bf16_bits_to_f64(uint32_t b, bool hi = false) {
  return (double)__uint_as_float(hi ? (b & 0xffff0000u) : (b << 16));
}

// ---- decode batches (T <= 2): one cluster of 16 CTAs, no global scratch
//
// A decode step routes one token: the 1 MiB gate matrix is split over the 16
// CTAs of a thread-block cluster (E/16 experts each, one per warp), every
// logit goes straight into the leader CTA's shared memory over the cluster's
// distributed shared memory, and after one cluster barrier the leader's warps
// (one per token) select the top-k.  Compared with the general kernel below
// this removes the global logit round trip, the fence and the arrival atomic
// from the critical path.  The token rows are converted to fp64 once per CTA
// (shared memory, 8-double chunks padded to 10 so the lanes' 16-byte reads
// hit distinct banks); each gate row's loads are issued before that staging.
constexpr int kRouterClusterCtas = 16;       // non-portable cluster size (B200 allows 16)
constexpr int kRouterClusterThreads = 512;
// The cluster covers the gate matrix with 16 SMs only, so its work per SM
// grows with the token count; it is used for 1-2 tokens, where it beats the
// general kernel (measured on B200).
constexpr int kRouterClusterMaxT = 2;
// Up to this many tokens the general kernel splits each expert over 4 warps
// (measured on B200: 9.4 / 10.8 us at 8 / 16 tokens against 15.0 / 15.0 us
// unsplit; at 64 tokens the 4x CTA count costs more than it gains: 28.7 vs
// 20.0 us).
constexpr int kRouterKSplitMaxT = 16;
constexpr int kRouterXChunk = 10;            // doubles per padded 8-element chunk

__device__ __forceinline__ unsigned cluster_ctarank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(const float* local, unsigned rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

__host__ __device__ constexpr size_t router_cluster_logit_bytes(int E) {
  return ((size_t)kRouterClusterMaxT * E * sizeof(float) + 15) & ~(size_t)15;
}

template <int KPER>
__global__ void __launch_bounds__(kRouterClusterThreads, 1) router_cluster_kernel(RouterParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* s_logits = reinterpret_cast<float*>(smem_raw);  // [T][E], used in the leader
  double* xd = reinterpret_cast<double*>(smem_raw + router_cluster_logit_bytes(p.E));
  cluster_arrive_relaxed();  // "this CTA has started" (phase 1)
  const unsigned rank = cluster_ctarank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = p.T;        // <= kRouterClusterMaxT
  const int nwarps = kRouterClusterThreads / 32;
  const int epc = (p.E + kRouterClusterCtas - 1) / kRouterClusterCtas;
  const int ebase = (int)rank * epc, eend = min(p.E, ebase + epc);
  const int vec = p.H / 8;   // 8-element chunks per row
  // programmatic launch: the next launch may start its prologue now; nothing
  // of global memory is read before the preceding grid has completed
  pdl_trigger();
  pdl_wait();
  // this warp's first gate row is in flight before the token rows are staged
  const int e0 = ebase + warp;
  uint4 w[8];
  if (e0 < eend) {
    const uint4* r = reinterpret_cast<const uint4*>(p.w + (size_t)e0 * p.H);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = lane + 32 * u;
      w[u] = c < vec ? __ldg(r + c) : make_uint4(0, 0, 0, 0);
    }
  }
  // the token rows, staged as fp64: one 16-B load of 8 values per thread
  // (every load in flight at once), or element loads for an unaligned row
  if ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) {
    const uint4* xv = reinterpret_cast<const uint4*>(p.x);
    for (int c = threadIdx.x; c < nt * vec; c += blockDim.x) {
      const uint4 q = xv[c];
      const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
      double* dst = xd + (size_t)c * kRouterXChunk;   // chunk c of token c / vec
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dst[2 * j] = bf16_bits_to_f64(qq[j]);
        dst[2 * j + 1] = bf16_bits_to_f64(qq[j], true);
      }
    }
  } else {
    const uint16_t* xb = reinterpret_cast<const uint16_t*>(p.x);
    for (int i = threadIdx.x; i < nt * p.H; i += blockDim.x) {
      const int t = i / p.H, k = i - t * p.H;
      xd[((size_t)t * vec + (k >> 3)) * kRouterXChunk + (k & 7)] = bf16_bits_to_f64(xb[i]);
    }
  }
  __syncthreads();
  cluster_wait();  // every CTA of the cluster runs: its shared memory may be written
  for (int e = e0; e < eend; e += nwarps) {
    const uint4* r = reinterpret_cast<const uint4*>(p.w + (size_t)e * p.H);
    double acc[kRouterClusterMaxT] = {0.0, 0.0};
    for (int c0 = lane; c0 < vec; c0 += 32 * 8) {
      if (e != e0 || c0 != lane) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + 32 * u;
          w[u] = c < vec ? __ldg(r + c) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + 32 * u;
        if (c >= vec) break;
        const uint32_t wr[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
        double wd[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          wd[2 * q] = bf16_bits_to_f64(wr[q]);
          wd[2 * q + 1] = bf16_bits_to_f64(wr[q], true);
        }
#pragma unroll
        for (int t = 0; t < kRouterClusterMaxT; ++t) {
          if (t < nt) {
            const double2* xc =
                reinterpret_cast<const double2*>(xd + ((size_t)t * vec + c) * kRouterXChunk);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const double2 xv = xc[q];
              acc[t] = fma(xv.x, wd[2 * q], acc[t]);
              acc[t] = fma(xv.y, wd[2 * q + 1], acc[t]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kRouterClusterMaxT; ++t) {
      if (t < nt) {
        double a = acc[t];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        if (lane == 0) st_cluster_f32(s_logits + t * p.E + e, 0, exact_bf16_of(a));
      }
    }
  }
  cluster_arrive_release();  // phase 2: this CTA's logits are in the leader
  cluster_wait();
  if (rank != 0 || warp >= nt) return;
  const int per = (p.E + 31) / 32;
  float v[KPER];
#pragma unroll
  for (int j = 0; j < KPER; ++j) {
    const int i = j * 32 + lane;
    v[j] = (j < per && i < p.E) ? s_logits[warp * p.E + i] : -INFINITY;
  }
  topk_select<KPER>(v, per, warp, p);
}

// KS warps share one expert's dot products (a quarter of H each for KS = 4):
// the same fp64 work spread over KS times more SMs for mid-sized batches,
// the partial sums combined in a fixed order in shared memory.
template <int KPER, int KS>
__global__ void __launch_bounds__(256) router_kernel(RouterParams p) {
  constexpr int EPC = kRouterExpertsPerCta / KS;   // experts per CTA
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [8][H]
  __shared__ bool s_last;
  __shared__ double s_part[KS][EPC][kRouterTokensPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * kRouterTokensPerCta;
  const int nt = min(kRouterTokensPerCta, p.T - t0);
  pdl_trigger();
  pdl_wait();
  // stage the token tile (16-byte vectors; H % 8 == 0 is checked on the host)
  const int vec_per_row = p.H / 8;
  for (int i = threadIdx.x; i < nt * vec_per_row; i += blockDim.x) {
    const int r = i / vec_per_row, c = i - r * vec_per_row;
    reinterpret_cast<uint4*>(xs)[r * vec_per_row + c] =
        reinterpret_cast<const uint4*>(p.x + (size_t)(t0 + r) * p.H)[c];
  }
  __syncthreads();
  const int el = warp / KS, kq = warp - (warp / KS) * KS;
  const int e = blockIdx.x * EPC + el;
  const int cbeg = kq * (vec_per_row / KS), cend = cbeg + vec_per_row / KS;
  double acc[kRouterTokensPerCta];
#pragma unroll
  for (int t = 0; t < kRouterTokensPerCta; ++t) acc[t] = 0.0;
  if (e < p.E) {
    const uint4* wrow = reinterpret_cast<const uint4*>(p.w + (size_t)e * p.H);
    // issue all of a lane's gate-row loads before any arithmetic, so the
    // row streams in one memory latency
    constexpr int kU = 8;
    for (int c0 = cbeg + lane; c0 < cend; c0 += 32 * kU) {
      uint4 wv[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = c0 + 32 * u;
        wv[u] = c < cend ? __ldg(wrow + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int c = c0 + 32 * u;
        if (c >= cend) break;
        const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv[u]);
        double wd[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) wd[q] = (double)__bfloat162float(wb[q]);
#pragma unroll
        for (int t = 0; t < kRouterTokensPerCta; ++t) {
          if (t < nt) {
            const uint4 xv = reinterpret_cast<const uint4*>(xs + t * p.H)[c];
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              acc[t] = fma((double)__bfloat162float(xb[q]), wd[q], acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kRouterTokensPerCta; ++t) {
    if (t < nt) {
      double v = acc[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) s_part[kq][el][t] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < EPC * nt) {
    const int ee = threadIdx.x / nt, t = threadIdx.x - ee * nt;
    const int eg = blockIdx.x * EPC + ee;
    if (eg < p.E) {
      double v = s_part[0][ee][t];
#pragma unroll
      for (int k = 1; k < KS; ++k) v += s_part[k][ee][t];
      p.logits[(size_t)(t0 + t) * p.E + eg] = exact_bf16_of(v);
    }
    __threadfence();  // the logit stores before this CTA's arrival
  }
  // last CTA of this token tile does the selection
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(p.arrivals + blockIdx.y, 1u);
    s_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (warp < nt) {
    const int t = t0 + warp;
    const float* lg = p.logits + (size_t)t * p.E;
    const int per = (p.E + 31) / 32;
    float v[KPER];
#pragma unroll
    for (int j = 0; j < KPER; ++j) {
      const int i = j * 32 + lane;
      v[j] = (j < per && i < p.E) ? __ldcg(lg + i) : -INFINITY;
    }
    topk_select<KPER>(v, per, t, p);
  }
  if (threadIdx.x == 0) p.arrivals[blockIdx.y] = 0;  // ready for the next launch / replay
}

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Launch the router for p (p.arrivals / p.logits already point into the
// scratch for the general kernel).  T <= kRouterClusterMaxT runs the cluster
// kernel, which needs no scratch; larger batches the general kernel.
static int launch_router(const RouterParams& p, cudaStream_t st, const char* what) {
  const bool small_e = p.E <= 8 * 32;
  if (p.T <= kRouterClusterMaxT) {
    const size_t smem = router_cluster_logit_bytes(p.E) +
                        (size_t)kRouterClusterMaxT * (p.H / 8) * kRouterXChunk * sizeof(double);
    void (*k)(RouterParams) = small_e ? router_cluster_kernel<8> : router_cluster_kernel<32>;
    D3_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                "router cluster-size attribute");
    if (smem > 48 * 1024)
      D3_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                  "router smem attribute");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kRouterClusterCtas, 1);
    cfg.blockDim = dim3(kRouterClusterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kRouterClusterCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    D3_CUDA_TRY(cudaLaunchKernelEx(&cfg, k, p), what);
    return D3_OK;
  }
  // mid-sized batches split each expert's dot products over 4 warps (4x the
  // CTAs); large batches already fill the GPU with token tiles
  const bool ksplit = p.T <= kRouterKSplitMaxT && p.H % 32 == 0;
  const int epc = ksplit ? kRouterExpertsPerCta / 4 : kRouterExpertsPerCta;
  const dim3 grid((unsigned)((p.E + epc - 1) / epc),
                  (unsigned)((p.T + kRouterTokensPerCta - 1) / kRouterTokensPerCta));
  const size_t smem = (size_t)kRouterTokensPerCta * p.H * sizeof(__nv_bfloat16);
  void (*k)(RouterParams) = ksplit ? (small_e ? router_kernel<8, 4> : router_kernel<32, 4>)
                                   : (small_e ? router_kernel<8, 1> : router_kernel<32, 1>);
  if (smem > 48 * 1024)
    D3_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "router smem attribute");
  D3_CUDA_TRY(launch_k(k, grid, dim3(256), smem, st, pdl_enabled(), p), what);
  return D3_OK;
}

}  // namespace d3

using namespace d3;

extern "C" {

size_t d3_router_workspace_size(int32_t T, int32_t E) {
  if (T <= 0 || E <= 0) return 0;
  if (T > kRouterMaxT) return 0;
  return kRouterCounterBytes + align256((size_t)T * E * sizeof(float));
}

int d3_router_topk(const void* x, const void* gate_w, int32_t T, int32_t H, int32_t E,
                   int32_t topk, int32_t renorm, int32_t* ids_out, float* weights_out,
                   void* weights_bf16_out, void* workspace, size_t workspace_bytes,
                   d3_stream_t stream) {
  D3_CHECK_ARG(x && gate_w && ids_out, "d3_router_topk: null pointer");
  if (T < 1 || T > kRouterMaxT) return fail(D3_ERR_TOO_LARGE, "T must be in [1, %d]", kRouterMaxT);
  D3_CHECK_ARG(H >= 8 && H % 8 == 0 && H <= kRouterMaxH, "H must be a multiple of 8 in [8, %d]",
               kRouterMaxH);
  D3_CHECK_ARG(E >= 1 && E <= kRouterMaxE, "E must be in [1, %d]", kRouterMaxE);
  D3_CHECK_ARG(topk >= 1 && topk <= 32 && topk <= E, "topk must be in [1, min(32, E)]");
  if (!aligned16(x) || !aligned16(gate_w))
    return fail(D3_ERR_MISALIGNED, "x and gate_w must be 16-byte aligned");
  const size_t need = d3_router_workspace_size(T, E);
  if (!workspace || workspace_bytes < need)
    return fail(D3_ERR_WORKSPACE, "router workspace needs %zu bytes (got %zu)", need,
                workspace_bytes);
  // The arrival counters start at zero (the caller zero-fills the workspace
  // once) and every launch leaves them at zero again.
  RouterParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.w = static_cast<const __nv_bfloat16*>(gate_w);
  p.T = T; p.H = H; p.E = E; p.topk = topk; p.renorm = renorm;
  p.arrivals = static_cast<unsigned*>(workspace);
  p.logits = reinterpret_cast<float*>(static_cast<char*>(workspace) + kRouterCounterBytes);
  p.ids_out = ids_out;
  p.weights_out = weights_out;
  p.weights_bf16_out = static_cast<__nv_bfloat16*>(weights_bf16_out);
  return launch_router(p, (cudaStream_t)stream, "router_kernel launch");
}

}  // extern "C"

// ------------------------------------------------------------ no-allocation router
//
// d3_router_topk_noalloc serves callers that cannot hand the router a device
// workspace: a host runtime that binds only this C ABI and has no device
// allocator of its own, a serving loop that must not take an allocator lock
// or risk an out-of-memory error mid-decode, or a process that already gave
// every free byte of device memory to the expert cache (the reference sizes
// its cache to all free VRAM, bin/offload.py:611-661).  Its scratch -- the
// per-token-tile arrival counters and the logits -- lives in the file-scope
// array below, reserved once per GPU when the library's device code is loaded
// and kept until the process exits.  The first call on a device does a
// one-time set-up (looks the array's device address up, zeroes its counters
// with a synchronous memset), so it belongs before any stream capture on that
// device.  Every call shares the one array: calls that overlap on the GPU
// (two streams, concurrent graph replays) race and must be serialised.

namespace d3 {

constexpr int kNoAllocMaxT = 2048;                  // tokens per call
constexpr size_t kNoAllocMaxLogits = 65536;         // T * E per call (256 KiB of fp32)
constexpr size_t kNoAllocCounterBytes = 1024;       // 256 tiles of 8 tokens
constexpr size_t kNoAllocScratchBytes = kNoAllocCounterBytes + kNoAllocMaxLogits * sizeof(float);

static __device__ __align__(256) unsigned char g_router_scratch[kNoAllocScratchBytes];

// Device address of g_router_scratch on the current device.  The name is only
// a host-side stand-in in host code, so the address is looked up once per
// device (with that device current) and cached.  The same one-time set-up
// zeroes the arrival counters (a synchronous memset, before any call on that
// device can have used them); from then on every launch of the general
// kernel leaves the counters of the tiles it used at zero again, exactly as
// with a caller workspace, so no call clears them.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  D3_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(D3_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_router_scratch)");
    e = cudaMemset(p, 0, kNoAllocCounterBytes);
    if (e != cudaSuccess) return cuda_fail(e, "clear the router scratch counters");
    addr[dev] = p;
  }
  *out = addr[dev];
  return D3_OK;
}

}  // namespace d3

extern "C" {

int d3_router_topk_noalloc(const void* x, const void* gate_w, int32_t T, int32_t H, int32_t E,
                           int32_t topk, int32_t renorm, int32_t* ids_out, float* weights_out,
                           void* weights_bf16_out, d3_stream_t stream) {
  D3_CHECK_ARG(x && gate_w && ids_out, "d3_router_topk_noalloc: null pointer");
  if (T < 1 || T > kNoAllocMaxT)
    return fail(D3_ERR_TOO_LARGE, "d3_router_topk_noalloc: T must be in [1, %d] (got %d)",
                kNoAllocMaxT, T);
  D3_CHECK_ARG(H >= 8 && H % 8 == 0 && H <= kRouterMaxH, "H must be a multiple of 8 in [8, %d]",
               kRouterMaxH);
  D3_CHECK_ARG(E >= 1 && E <= kRouterMaxE, "E must be in [1, %d]", kRouterMaxE);
  if ((size_t)T * (size_t)E > kNoAllocMaxLogits)
    return fail(D3_ERR_TOO_LARGE,
                "d3_router_topk_noalloc: T*E = %zu exceeds the built-in scratch (%zu logits); "
                "use d3_router_topk with a workspace",
                (size_t)T * (size_t)E, kNoAllocMaxLogits);
  D3_CHECK_ARG(topk >= 1 && topk <= 32 && topk <= E, "topk must be in [1, min(32, E)]");
  if (!aligned16(x) || !aligned16(gate_w))
    return fail(D3_ERR_MISALIGNED, "x and gate_w must be 16-byte aligned");
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // The arrival counters are zero here: the set-up cleared them and every
  // launch returns the ones it used to zero (the cluster kernel, T <= 2,
  // uses no scratch at all).
  RouterParams p{};
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.w = static_cast<const __nv_bfloat16*>(gate_w);
  p.T = T; p.H = H; p.E = E; p.topk = topk; p.renorm = renorm;
  p.arrivals = static_cast<unsigned*>(scratch);
  p.logits = reinterpret_cast<float*>(static_cast<char*>(scratch) + kNoAllocCounterBytes);
  p.ids_out = ids_out;
  p.weights_out = weights_out;
  p.weights_bf16_out = static_cast<__nv_bfloat16*>(weights_bf16_out);
  return launch_router(p, st, "router_kernel launch (no-alloc)");
}

}  // extern "C"
