// Routed-MoE expert computation with block-scaled FP8 weights on sm_100a.
//
// Computes what the reference hands to upstream fp8_moe_forward(x, ids, w,
// w13, s13, w2, s2) (call sites bin/devcache.py:275-277, bin/offload.py:177,
// :239, :340, :388, :449): for every routed (token t, slot k) pair with expert
// e = ids[t,k],
//     h   = silu(x_t W_gate[e]^T) * (x_t W_up[e]^T)         (W13 rows [0,I) / [I,2I))
//     out_t += w[t,k] * (h W_down[e]^T)
// where W = e4m3 bytes x fp32 scale per 128x128 block.
//
// Pipeline (all launches static-shaped, sync-free, graph-capturable):
//   1. route   G CTAs, each computing the same stable counting sort of the
//              pairs by expert; together they write the tile lists for both
//              GEMMs (expert, 128-row M tile, N tile of pairs, K-split) and
//              quantise the activations of every sorted pair into two e4m3
//              planes hi/lo per 128-wide K block with one fp32 scale:
//              x ~= s*(hi + lo), hi = e4m3(x/s), lo = e4m3(x/s - hi).  Two
//              fp8 planes carry ~8 significant bits, i.e. bf16-class
//              activations on the fp8 tensor path.  (Above 4096 pairs the
//              quantisation is its own launch.)
//   2. gemm1   tcgen05 kind::f8f6f4: D[128 weight rows, BN pairs] per K block
//              = W.hi + W.lo accumulated in TMEM, TMA-staged operands (128B
//              swizzle); the epilogue warps promote each K block with
//              s_w[kb] * s_x[n,kb] into fp32 registers (per-block scales, the
//              DeepSeek-style promotion), then store the K-split partials.
//   3. act     sum the K-split partials, SwiGLU, quantise h into hi/lo planes.
//   4. gemm2   same kernel over W2 (K = I).
//   5. combine out[t] = bf16(sum_k w[t,k] * y[pair(t,k)]) in a fixed order.
// Swap-AB: weight rows are the MMA M dimension (128), routed tokens the N
// dimension (16 for decode-sized batches, 64 otherwise), so one decode token
// still runs full-height MMAs.  The GEMMs stream each weight byte from HBM
// once per N tile; K-splits spread a small batch's few experts over all SMs.
#include "d3_common.cuh"
#include "gemm_sm100.cuh"
#include "fetch_flat.cuh"
#include "moe_epilogue.cuh"
#include "moe_gemv.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <mutex>

namespace d3 {

// ---------------------------------------------------------------- tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D byte matrix [rows, cols] (row pitch = pitch bytes), box [box_rows, 128 B],
// 128-byte swizzle.  Rows past `rows` read as zero.
static int make_tmap_u8(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                        uint64_t pitch, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(D3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if (!aligned16(base) || pitch % 16)
    return fail(D3_ERR_MISALIGNED, "tensor map base/pitch not 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(D3_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return D3_OK;
}

// ---------------------------------------------------------------- layout

constexpr int kMaxExperts = 8192;
constexpr int kMaxPairs = 65536;
constexpr int kFusedQuantMaxPairs = 4096;  // route quantises in-launch up to this many pairs
constexpr int kRouteSmemBudget = 160 * 1024;  // route launch: shared memory for the sort
constexpr int kRouteKeep = 4;                  // 32-pair batches per warp whose ids stay in registers

struct Plan {
  int P;        // routed pairs = T * topk
  int Ppad;     // P rounded up to a whole N tile (rows of the operand planes)
  int n;        // experts in the weight arrays
  int H, I;
  int BN;       // pairs per N tile
  // K-split bounds: the route launch picks the split from the real tile
  // count (a sparse batch -- most rows empty, or few pairs per expert -- gets
  // more K-splits); the workspace holds partials for split*_max splits
  int split1_min, split1_max;   // gemm1 (K = H)
  int split2_min, split2_max;   // gemm2 (K = I)
  int maxt1, maxt2;    // tile list capacities
  // workspace offsets (bytes)
  size_t o_cnt, o_off, o_sorted, o_inv, o_tiles1, o_tiles2, o_ntiles, o_xq, o_xs, o_ws1, o_hq,
      o_hs, o_ws2, total;
};

static size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

static void make_plan(Plan& p, int T, int topk, int n, int H, int I, int sms) {
  p.P = T * topk; p.n = n; p.H = H; p.I = I;
  const int distinct = p.P < n ? p.P : n;     // upper bound on experts hit
  const double per_expert = (double)p.P / distinct;
  p.BN = per_expert > 24.0 ? 64 : 16;
  p.Ppad = (p.P + p.BN - 1) / p.BN * p.BN;
  const int nt_bound = p.P / p.BN + distinct;  // sum_e ceil(c_e / BN)
  // a tile spans at most kGemmMaxTileKb K-blocks (its scales fit shared
  // memory); up to 8 splits while the partials stay within ~4096 rows x split
  auto bounds = [&](int nkb, int& lo, int& hi) {
    lo = (nkb + kGemmMaxTileKb - 1) / kGemmMaxTileKb;
    int cap = 4096 / (p.P > 0 ? p.P : 1);
    if (cap > 8) cap = 8;
    if (cap > nkb) cap = nkb;
    hi = cap > lo ? cap : lo;
  };
  bounds(H / 128, p.split1_min, p.split1_max);
  bounds(I / 128, p.split2_min, p.split2_max);
  (void)sms;
  p.maxt1 = nt_bound * (2 * I / 128) * p.split1_max;
  p.maxt2 = nt_bound * (H / 128) * p.split2_max;
  // bytes [0, 256): the one-launch path's grid counter, at the same offset
  // for every shape so no other data of a reused workspace ever lands there
  size_t o = 256;
  p.o_cnt = o;     o += al(sizeof(int) * (size_t)n);
  p.o_off = o;     o += al(sizeof(int) * (size_t)n);
  p.o_sorted = o;  o += al(sizeof(int) * (size_t)p.P);
  p.o_inv = o;     o += al(sizeof(int) * (size_t)p.P);
  p.o_tiles1 = o;  o += al(sizeof(int4) * (size_t)p.maxt1);
  p.o_tiles2 = o;  o += al(sizeof(int4) * (size_t)p.maxt2);
  p.o_ntiles = o;  o += al(sizeof(int) * 8);
  p.o_xq = o;      o += al((size_t)p.Ppad * 2 * H);
  p.o_xs = o;      o += al(sizeof(float) * (size_t)p.Ppad * (H / 128));
  p.o_ws1 = o;     o += al(sizeof(float) * (size_t)p.split1_max * p.P * 2 * I);
  p.o_hq = o;      o += al((size_t)p.Ppad * 2 * I);
  p.o_hs = o;      o += al(sizeof(float) * (size_t)p.Ppad * (I / 128));
  p.o_ws2 = o;     o += al(sizeof(float) * (size_t)p.split2_max * p.P * H);
  p.total = o;
}

// ---------------------------------------------------------------- 1. route

struct RouteParams {
  const void* ids; int ids_bytes; int P; int n;
  int* cnt; int* off; int* sorted; int* inv;
  int4* tiles1; int4* tiles2; int* ntiles;
  int BN;
  int mt1, nkb1, split1_min, split1_max;
  int mt2, nkb2, split2_min, split2_max;
  int sms;
  int nw;  // warps (chunks) of the stable sort
  // expert-parallel NVLink link: wait for every source's dispatch epoch first
  const long long* wait_flags; const long long* wait_epoch; int wait_n;
  int* wait_err; int wait_code; unsigned long long wait_budget;
  // activation quantisation folded into this launch
  int fuse_quant;
  const __nv_bfloat16* x; int topk, H;
  uint8_t* xq; float* xs;
};

__device__ __forceinline__ void load_x_block(const __nv_bfloat16* __restrict__ x, int pair,
                                             int topk, int H, int kb, float (&v)[4]);
__device__ __forceinline__ void store_x_block(const float (&v)[4], int H, int row, int kb,
                                              uint8_t* __restrict__ xq, float* __restrict__ xs);

__device__ __forceinline__ int load_pair_id(const void* ids, int bytes, int i, int n) {
  long long v = bytes == 8 ? static_cast<const long long*>(ids)[i]
                           : (long long)static_cast<const int*>(ids)[i];
  return (v >= 0 && v < n) ? (int)v : -1;
}

// Tile: expert, M tile | K-split index << 16, first sorted row,
// ncount | kb0 << 8 | kb1 << 20.
__device__ __forceinline__ int4 pack_tile(int e, int m, int split, int row0, int ncount, int kb0,
                                          int kb1) {
  return make_int4(e, m | (split << 16), row0, ncount | (kb0 << 8) | (kb1 << 20));
}

// K-split for `tiles` output tiles of a K range of nkb blocks: enough tiles
// for ~2 per SM, within [lo, hi]; returns the blocks per split in *kbps.
__device__ __forceinline__ int pick_split(int tiles, int nkb, int lo, int hi, int sms, int* kbps) {
  int want = tiles > 0 ? (2 * sms + tiles - 1) / tiles : 1;
  want = max(lo, min(hi, want));
  const int per = (nkb + want - 1) / want;
  *kbps = per;
  return (nkb + per - 1) / per;
}

// Grid of G CTAs (512 threads for the route launch).  Every CTA computes the same stable
// counting sort of the pairs by expert in its own shared memory (no
// cross-CTA communication; identical inputs give identical results), then
// the CTAs share the writing: the tile lists (one entry per thread,
// grid-strided), the fused activation quantisation (one warp per sorted row
// x K block, grid-strided) and, from CTA 0 only, the per-pair tables.
//
// The stable sort runs NW warps over NW consecutive chunks of the pairs:
// pass 1 counts each expert per chunk (hist[w][e]), a column scan over the
// chunks turns the counts into chunk-local bases, and pass 2 places every
// pair at off[e] + base[w][e] + (rank among the equal ids of its 32-pair
// batch) -- exactly the order of a sequential walk.
// Dynamic shared memory (ints): cnt[n], off[n], tile prefix[n], hist[NW][n],
// then the sorted row -> pair map [P] when the quantisation is fused.
__device__ __forceinline__ int route_chunk(int P, int nw) {
  const int batches = (P + 31) / 32;
  return (batches + nw - 1) / nw * 32;
}

// The body, shared by the route launch and the first phase of the fused
// expert kernel: `sm` is its dynamic shared memory (layout above).
__device__ __forceinline__ void route_body(const RouteParams& p, int* sm) {
  const int n = p.n, NW = p.nw;
  int* s_cnt = sm;                // [n]
  int* s_off = sm + n;            // [n]
  int* s_tp = sm + 2 * n;         // [n] exclusive prefix of N tiles per expert
  int* hist = sm + 3 * n;         // [NW][n]
  int* s_sorted = hist + (size_t)NW * n;  // [P] sorted row -> pair (fused quantisation only)
  __shared__ int warp_tot[32], wt2[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool lead = blockIdx.x == 0;
  pdl_trigger();
  pdl_wait();
  if (p.wait_flags) {
    // the rows and ids come from the other ranks: every thread reads them
    // only after this acquire (CTA barrier)
    if (warp == 0 &&
        !warp_wait_epochs(p.wait_flags, p.wait_n, *p.wait_epoch, p.wait_budget) && lane == 0)
      atomicCAS(p.wait_err, 0, p.wait_code);
    __syncthreads();
  }
  for (int i = tid; i < NW * n; i += blockDim.x) hist[i] = 0;
  const int nkb = p.H / 128;
  const int gwarp = blockIdx.x * (blockDim.x >> 5) + warp;
  const int gwarps = gridDim.x * (blockDim.x >> 5);
  __syncthreads();
  const int C = route_chunk(p.P, NW);
  // ---- pass 1: per-chunk counts (leaders of a batch hold distinct ids);
  // the first kRouteKeep batches' ids stay in registers for pass 2
  int keep[kRouteKeep];
  if (warp < NW) {
    int* h = hist + (size_t)warp * n;
    const int end = min(p.P, (warp + 1) * C);
    int bi = 0;
    for (int b0 = warp * C; b0 < end; b0 += 32, ++bi) {
      const int i = b0 + lane;
      const int e = i < end ? load_pair_id(p.ids, p.ids_bytes, i, n) : -1;
#pragma unroll
      for (int q = 0; q < kRouteKeep; ++q)
        if (bi == q) keep[q] = e;
      const unsigned m = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && lane == __ffs(m) - 1) h[e] += __popc(m);
      __syncwarp();
    }
  }
  __syncthreads();
  // ---- column scan: chunk-local bases, totals per expert
  for (int e = tid; e < n; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < NW; ++w) {
      const int c = hist[(size_t)w * n + e];
      hist[(size_t)w * n + e] = run;
      run += c;
    }
    s_cnt[e] = run;
  }
  __syncthreads();
  // ---- exclusive scans of counts (-> offsets) and of N tiles per expert
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = tid * per, hi = min(n, lo + per);
  int s_c = 0, s_t = 0;
  for (int e = lo; e < hi; ++e) {
    const int c = s_cnt[e];
    s_c += c;
    s_t += (c + p.BN - 1) / p.BN;
  }
  int v = s_c, w = s_t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, v, o), b = __shfl_up_sync(0xffffffffu, w, o);
    if (lane >= o) { v += a; w += b; }
  }
  if (lane == 31) { warp_tot[warp] = v; wt2[warp] = w; }
  __syncthreads();
  // (the CTA may have fewer than 32 warps: entries past the last warp are
  // not written, and count as zero)
  const int nwarps = (int)(blockDim.x >> 5);
  if (warp == 0) {
    int a = lane < nwarps ? warp_tot[lane] : 0, b = lane < nwarps ? wt2[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
      if (lane >= o) { a += x; b += y; }
    }
    warp_tot[lane] = a; wt2[lane] = b;
  }
  __syncthreads();
  {
    int base_c = (v - s_c) + (warp > 0 ? warp_tot[warp - 1] : 0);
    int base_t = (w - s_t) + (warp > 0 ? wt2[warp - 1] : 0);
    for (int e = lo; e < hi; ++e) {
      const int c = s_cnt[e];
      s_off[e] = base_c;
      s_tp[e] = base_t;
      if (lead) { p.cnt[e] = c; p.off[e] = base_c; }
      base_c += c;
      base_t += (c + p.BN - 1) / p.BN;
    }
  }
  const int nvalid = warp_tot[31], total_ntiles = wt2[31];
  __syncthreads();
  // ---- pass 2: stable placement
  if (warp < NW) {
    int* h = hist + (size_t)warp * n;
    const int end = min(p.P, (warp + 1) * C);
    int bi = 0;
    for (int b0 = warp * C; b0 < end; b0 += 32, ++bi) {
      const int i = b0 + lane;
      int e = -1;
      if (bi < kRouteKeep) {
#pragma unroll
        for (int q = 0; q < kRouteKeep; ++q)
          if (bi == q) e = keep[q];
      } else if (i < end) {
        e = load_pair_id(p.ids, p.ids_bytes, i, n);
      }
      const unsigned m = __match_any_sync(0xffffffffu, e);
      const int leader = __ffs(m) - 1;
      int base = 0;
      if (e >= 0 && lane == leader) {
        base = h[e];
        h[e] = base + __popc(m);
      }
      base = __shfl_sync(0xffffffffu, base, leader);
      if (i < end) {
        int pos = -1;
        if (e >= 0) {
          pos = s_off[e] + base + __popc(m & ((1u << lane) - 1));
          if (lead) p.sorted[pos] = i;
        }
        if (p.fuse_quant && pos >= 0) s_sorted[pos] = i;
        if (lead) p.inv[i] = pos;
      }
      __syncwarp();
    }
  }
  // sorted positions past the valid pairs (skipped ids) hold -1
  if (lead)
    for (int i = nvalid + tid; i < p.P; i += blockDim.x) p.sorted[i] = -1;
  __syncthreads();
  const int gthreads = gridDim.x * blockDim.x;
  const int gtid = blockIdx.x * blockDim.x + tid;
  // ---- the quantisation units (valid sorted row, K block): hi/lo planes +
  // scale of each valid pair's token row at its sorted position, four units
  // per warp in flight (the GEMM never reads a row past an expert's pair
  // count, so skipped pairs get none)
  // (32-bit unit arithmetic: fused quantisation runs up to 4096 pairs x 128
  // K blocks; each unit's row and block are decoded once)
  const int qunits = p.fuse_quant ? nvalid * nkb : 0;
  for (int u0 = gwarp * 4; u0 < qunits; u0 += gwarps * 4) {
    float v[4][4];
    int qrow[4], qkb[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int u = u0 + q;
      qrow[q] = u / nkb;
      qkb[q] = u - qrow[q] * nkb;
      if (u < qunits) load_x_block(p.x, s_sorted[qrow[q]], p.topk, p.H, qkb[q], v[q]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (u0 + q < qunits) store_x_block(v[q], p.H, qrow[q], qkb[q], p.xq, p.xs);
  }
  // ---- tile lists: entry (N tile nt, split s, M tile m) at nt*per + s*mt + m;
  // the K split from the real number of N tiles
  int kbps1, kbps2;
  const int split1 = pick_split(total_ntiles * p.mt1, p.nkb1, p.split1_min, p.split1_max, p.sms,
                                &kbps1);
  const int split2 = pick_split(total_ntiles * p.mt2, p.nkb2, p.split2_min, p.split2_max, p.sms,
                                &kbps2);
  const int per_nt1 = p.mt1 * split1, per_nt2 = p.mt2 * split2;
  const int tot1 = total_ntiles * per_nt1, tot2 = total_ntiles * per_nt2;
  for (int t = gtid; t < tot1 + tot2; t += gthreads) {
    const bool first = t < tot1;
    const int tt = first ? t : t - tot1;
    const int pn = first ? per_nt1 : per_nt2, mt = first ? p.mt1 : p.mt2;
    const int nt = tt / pn, r = tt - nt * pn;
    const int sp = r / mt, m = r - sp * mt;
    // expert: the last e with s_tp[e] <= nt (experts without tiles share the
    // next one's prefix, so the last such e has tiles)
    int a = 0, b = n - 1;
    while (a < b) {
      const int mid = (a + b + 1) >> 1;
      if (s_tp[mid] <= nt) a = mid; else b = mid - 1;
    }
    const int e = a, j = nt - s_tp[e];
    const int row0 = s_off[e] + j * p.BN;
    const int nc = min(p.BN, s_cnt[e] - j * p.BN);
    if (first)
      p.tiles1[tt] = pack_tile(e, m, sp, row0, nc, sp * kbps1, min(p.nkb1, (sp + 1) * kbps1));
    else
      p.tiles2[tt] = pack_tile(e, m, sp, row0, nc, sp * kbps2, min(p.nkb2, (sp + 1) * kbps2));
  }
  if (lead && tid == 0) {
    p.ntiles[0] = tot1;
    p.ntiles[1] = tot2;
    p.ntiles[2] = nvalid;  // valid (in-range) pairs
    p.ntiles[3] = split1;  // K splits the partial sums come in
    p.ntiles[4] = split2;
  }
}

__global__ void __launch_bounds__(1024) route_kernel(RouteParams p) {
  extern __shared__ int sm[];
  route_body(p, sm);
}

// ---------------------------------------------------------------- 2/4. quantise

// One warp, one 128-wide K block of a pair's token row: 4 values per lane.
__device__ __forceinline__ void load_x_block(const __nv_bfloat16* __restrict__ x, int pair,
                                             int topk, int H, int kb, float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const int t = pair / topk;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)t * H + kb * 128 + lane * 4);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int q = 0; q < 4; ++q) v[q] = __bfloat162float(b[q]);
}

// ... -> the hi/lo planes and the block scale of sorted row `row`.
__device__ __forceinline__ void store_x_block(const float (&v)[4], int H, int row, int kb,
                                              uint8_t* __restrict__ xq, float* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  uint32_t hi4, lo4;
  const float s = quant_block(v, hi4, lo4);
  uint8_t* qrow = xq + (size_t)row * 2 * H;
  *reinterpret_cast<uint32_t*>(qrow + kb * 128 + lane * 4) = hi4;
  *reinterpret_cast<uint32_t*>(qrow + H + kb * 128 + lane * 4) = lo4;
  if (lane == 0) xs[(size_t)row * (H / 128) + kb] = s;
}

// One warp per (sorted row, K block) of the valid rows.  Rows past the valid
// pair count are never read as an in-range column by the GEMM, so they are
// left unwritten.
// (Pointers to data an overlapping launch writes carry no __restrict__, so no
// read of them takes the non-coherent read-only path; the same in the
// kernels below.)
__global__ void quant_x_kernel(const __nv_bfloat16* x, const int* sorted, const int* nvalid_ptr,
                               int topk, int H, uint8_t* __restrict__ xq,
                               float* __restrict__ xs) {
  pdl_trigger();
  pdl_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nkb = H / 128;
  if (gw >= *nvalid_ptr * nkb) return;
  const int row = gw / nkb, kb = gw - row * nkb;
  float v[4];
  load_x_block(x, sorted[row], topk, H, kb, v);
  store_x_block(v, H, row, kb, xq, xs);
}

// One warp per (sorted row, K block of I) of the valid rows: sum splits,
// SwiGLU, quantise.
__global__ void act_kernel(const float* ws1, const int* split_ptr, int P, const int* nvalid_ptr,
                           int I, uint8_t* __restrict__ hq, float* __restrict__ hs) {
  pdl_trigger();
  pdl_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nkb = I / 128;
  if (gw >= *nvalid_ptr * nkb) return;
  const int row = gw / nkb, kb = gw - row * nkb;
  act_unit(ws1, *split_ptr, P, row, kb, I, hq, hs, lane);
}

// out[t, j] = bf16( [out[t,j] +] sum_k w[t,k] * sum_s ws2[s][inv[t,k]][j] ), k in order;
// one warp per (token, 128 columns).
__global__ void combine_kernel(const float* ws2, const int* split_ptr, int P, int H,
                               const int* inv, const void* weights, int weights_f32, int T,
                               int topk, int accumulate, __nv_bfloat16* out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.y;
  const int j0 = (blockIdx.x * blockDim.x + (threadIdx.x & ~31)) * 4;
  if (t >= T || j0 >= H) return;
  combine_unit(ws2, *split_ptr, P, H, inv, weights, weights_f32, t, topk, accumulate,
               out + (size_t)t * H, j0, threadIdx.x & 31);
}

// Expert-parallel NVLink return: warp units (received row t = source s * cap
// + j, 128 output columns) over a fixed grid; the combined row goes straight
// into row (rank * cap + j) of source s's return buffer.  With one routed
// pair per received row (topk == 1, the expert-parallel layout) only the
// valid rows -- sorted rows [0, nvalid) -- are visited; rows without a valid
// pair are never read at the source and are skipped.  After its CTA barrier
// one thread per CTA fences at system scope (cumulative over the CTA's peer
// stores) and arrives; the last CTA fences once more and releases the epoch
// in every source's flag_r, one thread per source.
__global__ void __launch_bounds__(256) combine_return_kernel(const float* ws2,
                                                             const int* split_ptr, int P, int H,
                                                             const int* inv, const int* sorted,
                                                             const int* nvalid_ptr,
                                                             const void* weights,
                                                             int weights_f32, int T, int topk,
                                                             P2pLink link) {
  __shared__ bool s_last;
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long gw = (long)blockIdx.x * (blockDim.x >> 5) + warp;
  const long nw = (long)gridDim.x * (blockDim.x >> 5);
  const int split = __ldcg(split_ptr);
  const int nj = H / 128;
  auto row_of = [&](int t) {
    const int s = t / link.cap, j = t - s * link.cap;
    return link.ret[s] + (size_t)(link.rank * link.cap + j) * H;
  };
  if (topk == 1) {
    const int nv = __ldcg(nvalid_ptr);
    for (long u = gw; u < (long)nv * nj; u += nw) {
      const int r = (int)(u / nj), j0 = (int)(u - (long)r * nj) * 128;
      const int t = __ldcg(sorted + r);
      combine_unit(ws2, split, P, H, inv, weights, weights_f32, t, 1, 0, row_of(t), j0, lane);
    }
  } else {
    for (long u = gw; u < (long)T * nj; u += nw) {
      const int t = (int)(u / nj), j0 = (int)(u - (long)t * nj) * 128;
      bool valid = false;
      for (int k = 0; k < topk; ++k) valid |= __ldcg(inv + t * topk + k) >= 0;
      if (valid)
        combine_unit(ws2, split, P, H, inv, weights, weights_f32, t, topk, 0, row_of(t), j0,
                     lane);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(link.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < link.n_ranks) st_release_sys(link.flag_r[threadIdx.x] + link.rank, *link.epoch);
  if (threadIdx.x == 0) *link.counter = 0;
}

// ---------------------------------------------------------------- 3/5. GEMM
// (tile engine in gemm_sm100.cuh)

// ---------------------------------------------------------------- one-launch expert call
//
// For batches up to kFusedQuantMaxPairs pairs the whole expert call -- route,
// gate/up GEMM, SwiGLU, down GEMM, combine (or, with the NVLink link, the
// combine stored into the source ranks plus the return epoch) -- runs as ONE
// cooperative launch of one CTA per SM, the phases separated by grid-wide
// barriers on a counter at workspace offset 0:
//
//   all threads   route (the stable sort, the tile lists, the quantised
//                 activations; the stage ring's shared memory is its scratch)
//   -- barrier 1 (every CTA) --
//   warp 0        TMA producer: the gate/up tiles, then the down tiles, whose
//                 weight tiles it issues at once and whose activation tiles
//                 wait for barrier 3 (the down weights stream into the
//                 shared-memory ring while SwiGLU runs)
//   warp 1        MMA issuer: both tile lists through the same rings
//   epilogue      gate/up tiles -- barrier 2 -- SwiGLU + quantisation units of
//                 the grid -- barrier 3 -- down tiles -- barrier 4 -- combine
//                 units -- final arrival (the last CTA publishes the return
//                 epoch on every source with the NVLink link, and zeroes the
//                 counter for the next launch)
//
// The work and every summation order are those of the separate launches, so
// the outputs are bit-identical.  No launch boundary separates the phases, so
// no per-launch ramp and drain sits between them; every wait is bounded
// (error code 5 for a phase barrier).
constexpr int kFusedBarrierCode = 5;

struct FusedParams {
  RouteParams rp;
  GemmParams g1, g2;
  int I, H, P, T, topk, weights_f32, accumulate;
  const float* ws1;
  uint8_t* hq;
  float* hs;
  const float* ws2;
  const int* inv;
  const void* weights;
  __nv_bfloat16* out;
  unsigned* gbar;          // workspace offset 0, zero between launches
  int* err;
  int has_link;
  P2pLink link;
};

// The epilogue warps of every CTA meet: named barrier, then one thread
// arrives on the grid counter and waits (bounded) for `target` arrivals.
__device__ __forceinline__ void epi_grid_sync(unsigned* gbar, unsigned target, int nepi,
                                              bool leader, int* err) {
  epi_bar_sync(nepi);
  if (leader) {
    __threadfence();
    atomicAdd(gbar, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu_u32(gbar) < target) {
      if (globaltimer_ns() - t0 > kGemmWaitBudgetNs) { gemm_error(err, kFusedBarrierCode); break; }
      __nanosleep(32);
    }
    __threadfence();
  }
  epi_bar_sync(nepi);
}

template <int BN, int KPS>
__global__ void __launch_bounds__(GemmCfg<BN, KPS>::THREADS, 1)
    moe_fused_kernel(const __grid_constant__ CUtensorMap tw1,
                     const __grid_constant__ CUtensorMap tx1,
                     const __grid_constant__ CUtensorMap tw2,
                     const __grid_constant__ CUtensorMap tx2, const __grid_constant__ FusedParams f) {
  using Cfg = GemmCfg<BN, KPS>;
  constexpr int NEPI = 32 * Cfg::EPI;
  extern __shared__ uint8_t smem_raw[];
  const GemmSmem<BN, KPS> sm = GemmSmem<BN, KPS>::carve(smem_raw);
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_tile_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned G = gridDim.x;
  if (threadIdx.x == 0) {
    sm.init();
    s_abort = 0;
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tw1);
    tma_prefetch_desc(&tx1);
    tma_prefetch_desc(&tw2);
    tma_prefetch_desc(&tx2);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  // ---- phase 0: route, in the stage ring's memory (no TMA has run yet)
  route_body(f.rp, reinterpret_cast<int*>(sm.stage_base));
  fence_proxy_async_global();   // the quantised rows are read by TMA in other CTAs
  fence_proxy_async_smem();     // the ring's bytes are next written by TMA
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(f.gbar, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu_u32(f.gbar) < G) {
      if (globaltimer_ns() - t0 > kGemmWaitBudgetNs) { gemm_error(f.err, kFusedBarrierCode); break; }
      __nanosleep(32);
    }
    __threadfence();
  }
  __syncthreads();
  const int n1 = __ldcg(f.g1.ntiles), n2 = __ldcg(f.g2.ntiles);
  PipePos ps;
  if (warp == 0) {
    if (lane == 0) {
      fence_proxy_async_global();
      gemm_produce<BN, KPS>(sm, &tw1, &tx1, f.g1, n1, ps, &s_abort, nullptr);
      const OperandGate gate{f.gbar, 3 * G, f.err, kFusedBarrierCode};
      gemm_produce<BN, KPS>(sm, &tw2, &tx2, f.g2, n2, ps, &s_abort, &gate);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      gemm_mma<BN, KPS>(sm, tmem, f.g1, n1, ps, &s_abort);
      gemm_mma<BN, KPS>(sm, tmem, f.g2, n2, ps, &s_abort);
      gemm_mma_drain<BN, KPS>(sm, ps, f.err);
    }
  } else {
    const int ep = threadIdx.x - 64;
    const bool leader = ep == 0;
    const long ew = (long)blockIdx.x * Cfg::EPI + (warp - 2), nw = (long)G * Cfg::EPI;
    gemm_epilogue<BN, KPS>(sm, tmem, f.g1, n1, ps, &s_abort, &s_tile_abort);
    epi_grid_sync(f.gbar, 2 * G, NEPI, leader, f.err);
    // ---- SwiGLU + quantisation of h: one warp per (valid sorted row, I block)
    {
      const int nvalid = __ldcg(f.rp.ntiles + 2), split1 = __ldcg(f.rp.ntiles + 3);
      const int nkb = f.I / 128;
      for (long u = ew; u < (long)nvalid * nkb; u += nw) {
        const int row = (int)(u / nkb), kb = (int)(u - (long)row * nkb);
        act_unit(f.ws1, split1, f.P, row, kb, f.I, f.hq, f.hs, lane);
      }
      fence_proxy_async_global();   // h is read by TMA in other CTAs
    }
    epi_grid_sync(f.gbar, 3 * G, NEPI, leader, f.err);
    gemm_epilogue<BN, KPS>(sm, tmem, f.g2, n2, ps, &s_abort, &s_tile_abort);
    epi_grid_sync(f.gbar, 4 * G, NEPI, leader, f.err);
  }
  // ---- combine, on every warp of the CTA (the producer and MMA lanes are
  // done: their last operands were consumed before the down tiles drained):
  // one warp per (token or received row, 128 output columns)
  __syncthreads();
  {
    const int nwc = Cfg::THREADS / 32;
    const long cw = (long)blockIdx.x * nwc + warp, ncw = (long)G * nwc;
    const int split2 = __ldcg(f.rp.ntiles + 4);
    const int nj = f.H / 128;
    if (f.has_link && f.topk == 1) {
      // received rows: only the valid ones (sorted rows [0, nvalid)), each
      // stored into its source rank's return rows
      const int nvalid = __ldcg(f.rp.ntiles + 2);
      for (long u = cw; u < (long)nvalid * nj; u += ncw) {
        const int r = (int)(u / nj), j0 = (int)(u - (long)r * nj) * 128;
        const int t = __ldcg(f.rp.sorted + r);
        const int src = t / f.link.cap, j = t - src * f.link.cap;
        __nv_bfloat16* row = f.link.ret[src] + (size_t)(f.link.rank * f.link.cap + j) * f.H;
        combine_unit(f.ws2, split2, f.P, f.H, f.inv, f.weights, f.weights_f32, t, 1, 0, row, j0,
                     lane);
      }
    } else if (f.has_link) {
      for (long u = cw; u < (long)f.T * nj; u += ncw) {
        const int t = (int)(u / nj), j0 = (int)(u - (long)t * nj) * 128;
        bool valid = false;
        for (int k = 0; k < f.topk; ++k) valid |= __ldcg(f.inv + t * f.topk + k) >= 0;
        if (!valid) continue;
        const int src = t / f.link.cap, j = t - src * f.link.cap;
        __nv_bfloat16* row = f.link.ret[src] + (size_t)(f.link.rank * f.link.cap + j) * f.H;
        combine_unit(f.ws2, split2, f.P, f.H, f.inv, f.weights, f.weights_f32, t, f.topk, 0,
                     row, j0, lane);
      }
    } else {
      for (long u = cw; u < (long)f.T * nj; u += ncw) {
        const int t = (int)(u / nj), j0 = (int)(u - (long)t * nj) * 128;
        combine_unit(f.ws2, split2, f.P, f.H, f.inv, f.weights, f.weights_f32, t, f.topk,
                     f.accumulate, f.out + (size_t)t * f.H, j0, lane);
      }
    }
  }
  // ---- final arrival: the last CTA publishes (NVLink) and zeroes the counter
  // (thread 0's system fence after the CTA barrier covers every peer store
  // the CTA made)
  __syncthreads();
  if (threadIdx.x == 0) {
    if (f.has_link) __threadfence_system();
    else __threadfence();
    s_tile_abort = atomicAdd(f.gbar, 1u) == 5 * G - 1;   // (reused as "last CTA")
    if (s_tile_abort && f.has_link) __threadfence_system();
  }
  __syncthreads();
  if (s_tile_abort) {
    if (f.has_link && (int)threadIdx.x < f.link.n_ranks)
      st_release_sys(f.link.flag_r[threadIdx.x] + f.link.rank, *f.link.epoch);
    if (threadIdx.x == 0) atomicExch(f.gbar, 0u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}


// ---------------------------------------------------------------- small batch
// (GEMV kernels in moe_gemv.cuh)

// measured on B200 (8 distinct experts per token, weights from HBM): the GEMV
// path takes 13.9 / 23.8 / 40.0 us at 8 / 16 / 32 pairs against 30.4 / 42.2 /
// 60.6 us for the tensor-core path
constexpr int kGemvMaxPairsDefault = 32;

// Pairs up to which the CUDA-core GEMV path runs (D3_GEMV_MAX_PAIRS
// overrides; 0 sends every batch to the tensor-core path).
static int gemv_max_pairs() {
  const char* s = getenv("D3_GEMV_MAX_PAIRS");
  return s ? atoi(s) : kGemvMaxPairsDefault;
}

static size_t gemv2_smem(int topk, int I) { return (size_t)topk * (I / 16) * 20 * sizeof(float); }

static bool gemv_shapes_ok(int topk, int H, int I) {
  const int c1 = H / 512, c2 = I / 512;
  return H % 512 == 0 && I % 512 == 0 && (c1 == 1 || c1 == 2 || c1 == 4 || c1 == 8) &&
         (c2 == 1 || c2 == 2 || c2 == 4) && gemv2_smem(topk + 1, I) <= 96 * 1024;
}

static bool gemv_supported(int P, int topk, int H, int I) {
  return P <= gemv_max_pairs() && gemv_shapes_ok(topk, H, I);
}

template <int C1>
static cudaError_t launch_gemv13(const GemvParams& gp, int ctas, cudaStream_t st) {
  return launch_k(moe_gemv13_kernel<C1>, dim3((unsigned)ctas), dim3(kGemvThreads), 0, st, false,
                  gp);
}

template <int C2>
static cudaError_t launch_gemv2(const GemvParams& gp, dim3 grid, int rpw, size_t smem,
                                cudaStream_t st, bool pdl) {
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(
        moe_gemv2_kernel<C2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(moe_gemv2_kernel<C2>, grid, dim3(kGemvThreads), smem, st, pdl, gp, rpw);
}

static int run_gemv2(const GemvParams& gp, cudaStream_t st, bool pdl);

static int run_gemv(const GemvParams& gp, cudaStream_t st) {
  const int sms = num_sms();
  const long units1 = (long)gp.T * gp.topk * gp.I;  // one warp each
  long ctas1 = (units1 + kGemvRowsPerCta - 1) / kGemvRowsPerCta;
  if (ctas1 > 2L * sms) ctas1 = 2L * sms;  // one resident wave (2 CTAs per SM)
  cudaError_t e;
  switch (gp.H / 512) {
    case 1: e = launch_gemv13<1>(gp, (int)ctas1, st); break;
    case 2: e = launch_gemv13<2>(gp, (int)ctas1, st); break;
    case 4: e = launch_gemv13<4>(gp, (int)ctas1, st); break;
    default: e = launch_gemv13<8>(gp, (int)ctas1, st); break;
  }
  D3_CUDA_TRY(e, "moe_gemv13_kernel launch");
  return run_gemv2(gp, st, pdl_enabled());
}

static int run_gemv2(const GemvParams& gp, cudaStream_t st, bool pdl) {
  const int sms = num_sms();
  cudaError_t e;
  int rpw = 1;  // output rows per warp: more once the grid would exceed ~4 CTAs per SM
  while (rpw < 4 && (long)gp.T * gp.H / (kGemvRowsPerCta * rpw) > 4L * sms) rpw *= 2;
  const dim3 grid2((unsigned)(gp.H / (kGemvRowsPerCta * rpw)), (unsigned)gp.T);
  const size_t smem = gemv2_smem(gp.topk + (gp.sw13 ? 1 : 0), gp.I);
  switch (gp.I / 512) {
    case 1: e = launch_gemv2<1>(gp, grid2, rpw, smem, st, pdl); break;
    case 2: e = launch_gemv2<2>(gp, grid2, rpw, smem, st, pdl); break;
    default: e = launch_gemv2<4>(gp, grid2, rpw, smem, st, pdl); break;
  }
  D3_CUDA_TRY(e, "moe_gemv2_kernel launch");
  return D3_OK;
}

// ---------------------------------------------------------------- fetch + gate/up overlap
//
// Decode with offloaded experts: ONE launch both fetches the layer's missed
// experts from pinned host memory and runs the gate/up units.  CTAs
// [0, fetch_ctas) fetch -- first the W13 and S13 bytes of every job (job
// after job), then the rest (W2, S2) -- and count, per job, the W13/S13
// vectors that have landed (one fence + atomic per job per CTA, when the CTA
// leaves that job's range).  The other CTAs run the gate/up units of the
// resident experts and of the shared expert at once, then the units of each
// fetched expert after a bounded wait until its job's count is complete: a
// per-slot in-flight state (queued -> landed) instead of a launch boundary.
// The down projection (gemv2) follows as its own launch and reads W2 only
// after griddepcontrol.wait (this launch writes W2).
struct FetchOverlapParams {
  unsigned long long* done;   // [64] W13+S13 vectors landed per job (zeroed by the resolve launch)
  int fetch_ctas;
  uint32_t early_mask;        // buffers the gate/up units read (W13, S13)
  int64_t vecA;               // vectors per job in those buffers
  int* err;
  int err_code;
  unsigned long long budget_ns;
  // optional: up to kMaxWarmWindows ranges of static bytes to warm into L2
  // (the next layer's weights), as 128-byte lines; warm_end[w] = lines of
  // windows 0..w together
  const char* warm[4];
  unsigned long long warm_end[4];
  int n_warm;
};

__device__ __forceinline__ void overlap_vec(const FetchParams& f, uint32_t mask, bool early,
                                            int64_t r, int64_t e, int64_t s, const uint4** src,
                                            uint4** dst) {
  for (int b = 0; b < f.nbuf; ++b) {
    if ((((mask >> b) & 1u) != 0u) != early) continue;
    if (r < f.vecs[b]) {
      *src = f.host[b] + e * f.vecs[b] + r;
      *dst = f.cache[b] + s * f.vecs[b] + r;
      return;
    }
    r -= f.vecs[b];
  }
}

__device__ void overlap_fetch(const FetchParams& f, const FetchOverlapParams& o, int nm) {
  const int64_t vecA = o.vecA, vecB = f.vec_total - vecA;
  const int64_t totA = (int64_t)nm * vecA, total = (int64_t)nm * f.vec_total;
  constexpr int64_t kChunk = (int64_t)kFetchThreads * kFetchUnroll;
  const int64_t stride = (int64_t)o.fetch_ctas * kChunk;
  int pj = -1;                 // job whose landed vectors this CTA still has to publish
  unsigned long long pc = 0;
  // (uniform over the CTA: every thread runs the same chunk sequence)
  auto flush = [&]() {
    __syncthreads();           // every thread's stores of the counted chunks are issued
    if (threadIdx.x == 0) {
      __threadfence();         // ... and visible GPU-wide before the count moves
      atomicAdd(o.done + pj, pc);
    }
    pj = -1;
    pc = 0;
  };
  for (int64_t base = (int64_t)blockIdx.x * kChunk; base < total; base += stride) {
    uint4 v[kFetchUnroll];
    uint4* dptr[kFetchUnroll];
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u) {
      const int64_t g = base + (int64_t)u * kFetchThreads + threadIdx.x;
      dptr[u] = nullptr;
      if (g < total) {
        const bool early = g < totA;
        const int64_t gg = early ? g : g - totA, per = early ? vecA : vecB;
        const int64_t j = gg / per, r = gg - j * per;
        const uint4* src = nullptr;
        uint4* dst = nullptr;
        overlap_vec(f, o.early_mask, early, r, __ldcg(f.fetch_expert + j),
                    __ldcg(f.fetch_slot + j), &src, &dst);
        v[u] = ld_stream_u4(src);
        dptr[u] = dst;
      }
    }
#pragma unroll
    for (int u = 0; u < kFetchUnroll; ++u)
      if (dptr[u]) *dptr[u] = v[u];
    if (base < totA) {
      const int64_t hi = base + kChunk < totA ? base + kChunk : totA;
      const int j0 = (int)(base / vecA), j1 = (int)((hi - 1) / vecA);
      for (int j = j0; j <= j1; ++j) {
        const int64_t lo_j = base > (int64_t)j * vecA ? base : (int64_t)j * vecA;
        const int64_t hi_j = hi < (int64_t)(j + 1) * vecA ? hi : (int64_t)(j + 1) * vecA;
        if (pj != j) {
          if (pj >= 0) flush();
          pj = j;
        }
        pc += (unsigned long long)(hi_j - lo_j);
        if (j < j1) flush();   // this CTA's later chunks all lie past job j
      }
      const int64_t next = base + stride;
      if (pj >= 0 && (next >= totA || next >= (int64_t)(pj + 1) * vecA)) flush();
    }
  }
  if (pj >= 0) flush();
}

template <int CPL>
__global__ void __launch_bounds__(kGemvThreads) fetch_gemv13_kernel(FetchParams f, GemvParams p,
                                                                    FetchOverlapParams o) {
  __shared__ int s_job[64];
  pdl_wait();     // the allocator's job table (and cleared counters) are complete
  pdl_trigger();  // gemv2 reads nothing this launch writes before its own wait
  const int nm = *f.nmiss;
  if ((int)blockIdx.x < o.fetch_ctas) {
    if (nm > 0) overlap_fetch(f, o, nm);
    return;
  }
  const int P = p.T * p.topk;  // <= 64
  if ((int)threadIdx.x < P) {
    const int s = gemv_pair_id(p.ids, p.ids_bytes, threadIdx.x, p.n);
    int job = -1;
    for (int j = 0; j < nm; ++j)
      if (s >= 0 && __ldcg(f.fetch_slot + j) == s) job = j;
    s_job[threadIdx.x] = job;
  }
  __syncthreads();
  const GemvOverlap ov{s_job, o.done, (unsigned long long)o.vecA, o.err, o.err_code, o.budget_ns};
  const long gw = ((long)(blockIdx.x - o.fetch_ctas) * blockDim.x + threadIdx.x) >> 5;
  const long nw = ((long)(gridDim.x - o.fetch_ctas) * blockDim.x) >> 5;
  gemv13_units<CPL>(p, gw, nw, &ov);
  // With a warm window: once its units are done, each gate/up thread hints
  // its share of the window's lines into L2 (a hint, nothing waits on it),
  // while the fetch CTAs still hold the host link.  The window is static
  // weights the next launches read (the next layer's dense weights), so HBM,
  // idle during the host-bound fetch, serves them ahead of time.
  if (o.n_warm > 0) {
    const unsigned long long t =
        (unsigned long long)(blockIdx.x - o.fetch_ctas) * blockDim.x + threadIdx.x;
    const unsigned long long nt = (unsigned long long)(gridDim.x - o.fetch_ctas) * blockDim.x;
    const unsigned long long total = o.warm_end[o.n_warm - 1];
    int w = 0;
    for (unsigned long long i = t; i < total; i += nt) {
      while (i >= o.warm_end[w]) ++w;   // i < total = warm_end[n_warm - 1]: w stays in range
      const unsigned long long first = w ? o.warm_end[w - 1] : 0ull;
      prefetch_l2(o.warm[w] + ((i - first) << 7));
    }
  }
}

constexpr uint64_t kOverlapWaitBudgetNs = 2000000000ull;
constexpr int kMaxWarmWindows = 4;
constexpr int kOverlapFetchCtas = 64;   // measured: 16 -> 80, 32 -> 102, 64 / 148 -> 103.7 tok/s

static size_t overlap_workspace(int k, int I) {
  return al(64 * sizeof(unsigned long long)) + al(sizeof(float) * ((size_t)k * I + I + 1));
}

// The one-launch path is taken with D3_MOE_FUSED=1 (read per call); by
// default every call takes the separate launches, which measured faster so
// far (45.3 against 59.5 us at the 8-GPU expert-parallel rank shape).
static bool fused_enabled() {
  const char* s = getenv("D3_MOE_FUSED");
  return s && s[0] == '1';
}

constexpr int kFusedDeclined = 1;   // not an error: take the separate launches

// Launches moe_fused_kernel for the call planned in pl / rp; returns
// kFusedDeclined when the shape does not fit it (route scratch beyond the
// stage ring, or fewer resident CTAs than SMs).
template <int BN, int KPS>
static int launch_fused(const Plan& pl, RouteParams rp, char* ws, const void* x,
                        const void* weights, int weights_f32, int T, int topk, const void* w13,
                        const float* s13, const void* w2, const float* s2, int n_experts, int H,
                        int I, void* out, int accumulate, int* err_word, const P2pLink* link,
                        cudaStream_t st) {
  using Cfg = GemmCfg<BN, KPS>;
  const int sms = num_sms();
  const int P = pl.P;
  // route scratch in the stage ring: cnt, off, tile prefix [n] + pair map [P]
  // + one histogram of n per sorting warp (<= the CTA's warps)
  const size_t ring = (size_t)Cfg::STAGES * Cfg::STAGE_BYTES;
  const size_t rbase = sizeof(int) * (3 * (size_t)n_experts + (size_t)P);
  if (rbase + sizeof(int) * (size_t)n_experts > ring) return kFusedDeclined;
  long nw = (long)(ring - rbase) / (long)(sizeof(int) * (size_t)n_experts);
  const long warps = Cfg::THREADS / 32;
  nw = nw > warps ? warps : nw;
  if (nw > (P + 31) / 32) nw = (P + 31) / 32;
  if (nw < 1) nw = 1;
  rp.nw = (int)nw;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return kFusedDeclined;
  if (!attr_set[dev]) {
    D3_CUDA_TRY(cudaFuncSetAttribute(moe_fused_kernel<BN, KPS>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM),
                "fused smem attribute");
    int per_sm = 0;
    D3_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_fused_kernel<BN, KPS>,
                                                              Cfg::THREADS, Cfg::SMEM),
                "fused occupancy");
    if (per_sm < 1) return kFusedDeclined;
    attr_set[dev] = true;
  }
  int rc = D3_OK;
  CUtensorMap tw1, tx1, tw2, tx2;
  uint8_t* xq = (uint8_t*)(ws + pl.o_xq);
  uint8_t* hq = (uint8_t*)(ws + pl.o_hq);
  if ((rc = make_tmap_u8(&tw1, w13, H, (uint64_t)n_experts * 2 * I, H, 128))) return rc;
  if ((rc = make_tmap_u8(&tx1, xq, 2 * H, pl.Ppad, 2 * H, BN))) return rc;
  if ((rc = make_tmap_u8(&tw2, w2, I, (uint64_t)n_experts * H, I, 128))) return rc;
  if ((rc = make_tmap_u8(&tx2, hq, 2 * I, pl.Ppad, 2 * I, BN))) return rc;
  FusedParams f{};
  f.rp = rp;
  f.g1.tiles = rp.tiles1; f.g1.ntiles = rp.ntiles; f.g1.wscale = s13;
  f.g1.rows_per_expert = 2 * I; f.g1.mblocks = 2 * I / 128; f.g1.kblocks = H / 128;
  f.g1.xscale = (const float*)(ws + pl.o_xs); f.g1.K = H; f.g1.out = (float*)(ws + pl.o_ws1);
  f.g1.P = P; f.g1.Mtot = 2 * I; f.g1.err = err_word;
  f.g2.tiles = rp.tiles2; f.g2.ntiles = rp.ntiles + 1; f.g2.wscale = s2;
  f.g2.rows_per_expert = H; f.g2.mblocks = H / 128; f.g2.kblocks = I / 128;
  f.g2.xscale = (const float*)(ws + pl.o_hs); f.g2.K = I; f.g2.out = (float*)(ws + pl.o_ws2);
  f.g2.P = P; f.g2.Mtot = H; f.g2.err = err_word;
  f.I = I; f.H = H; f.P = P; f.T = T; f.topk = topk;
  f.weights_f32 = weights_f32 ? 1 : 0; f.accumulate = accumulate ? 1 : 0;
  f.ws1 = (const float*)(ws + pl.o_ws1);
  f.hq = hq;
  f.hs = (float*)(ws + pl.o_hs);
  f.ws2 = (const float*)(ws + pl.o_ws2);
  f.inv = rp.inv;
  f.weights = weights;
  f.out = static_cast<__nv_bfloat16*>(out);
  f.gbar = reinterpret_cast<unsigned*>(ws);
  f.err = err_word;
  f.has_link = link ? 1 : 0;
  if (link) f.link = *link;
  (void)x;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  D3_CUDA_TRY(cudaLaunchKernelEx(&cfg, moe_fused_kernel<BN, KPS>, tw1, tx1, tw2, tx2, f),
              "moe_fused_kernel launch");
  return D3_OK;
}

}  // namespace d3

using namespace d3;

extern "C" {

size_t d3_moe_workspace_size(int32_t T, int32_t topk, int32_t n_experts, int32_t H, int32_t I) {
  if (T < 1 || topk < 1 || n_experts < 1 || H < 128 || I < 128 || H % 128 || I % 128) return 0;
  if ((long)T * topk > kMaxPairs) return 0;
  Plan p;
  make_plan(p, T, topk, n_experts, H, I, num_sms());
  return p.total;
}

}  // extern "C"

// The routed experts, and optionally the shared expert (decode batches only).
static int moe_forward(const void* x, const void* ids, int32_t ids_bytes, const void* weights,
                       int32_t weights_f32, int32_t T, int32_t topk, const void* w13,
                       const float* s13, const void* w2, const float* s2, int32_t n_experts,
                       int32_t H, int32_t I, void* out, int32_t accumulate, int32_t* err_word,
                       void* workspace, size_t workspace_bytes, d3_stream_t stream,
                       const void* sw13, const void* sw2, const void* sgate,
                       const P2pLink* link = nullptr) {
  D3_CHECK_ARG(x && ids && weights && w13 && s13 && w2 && s2 && out && err_word,
               "d3_moe_fp8_forward: null pointer");
  D3_CHECK_ARG(ids_bytes == 4 || ids_bytes == 8, "ids_bytes must be 4 or 8");
  D3_CHECK_ARG(T >= 1 && topk >= 1 && topk <= 64, "T >= 1 and 1 <= topk <= 64 required");
  if ((long)T * topk > kMaxPairs)
    return fail(D3_ERR_TOO_LARGE, "T*topk = %ld exceeds %d", (long)T * topk, kMaxPairs);
  if (n_experts < 1 || n_experts > kMaxExperts)
    return fail(D3_ERR_TOO_LARGE, "n_experts must be in [1, %d]", kMaxExperts);
  if (H % 128 || I % 128 || H < 128 || I < 128 || H > 16384 || I > 16384)
    return fail(D3_ERR_UNSUPPORTED, "H and I must be multiples of 128 in [128, 16384]");
  if (!aligned16(x) || !aligned16(out) || !aligned16(w13) || !aligned16(w2))
    return fail(D3_ERR_MISALIGNED, "x, out, w13 and w2 must be 16-byte aligned");
  Plan pl;
  make_plan(pl, T, topk, n_experts, H, I, num_sms());
  if (!workspace || workspace_bytes < pl.total)
    return fail(D3_ERR_WORKSPACE, "moe workspace needs %zu bytes (got %zu)", pl.total,
                workspace_bytes);
  if (!aligned16(workspace)) return fail(D3_ERR_MISALIGNED, "workspace must be 16-byte aligned");
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  const int P = pl.P;

  if (sw13) {
    D3_CHECK_ARG(sw2 != nullptr, "shared expert: down weights missing");
    if (!aligned16(sw13) || !aligned16(sw2) || (sgate && !aligned16(sgate)))
      return fail(D3_ERR_MISALIGNED, "shared expert weights must be 16-byte aligned");
    if (P > kGemvMaxPairsDefault || !gemv_shapes_ok(topk, H, I))
      return fail(D3_ERR_UNSUPPORTED,
                  "the fused shared expert runs on the decode path only (T*topk <= %d, H and I "
                  "multiples of 512); run it separately for larger batches",
                  kGemvMaxPairsDefault);
  }
  if (sw13 || (!link && gemv_supported(P, topk, H, I))) {
    // decode-sized batch: two CUDA-core launches; h (and the shared expert's
    // h and gate) live where gemm1's partials would (split1_max * P * 2I
    // floats >= P * I + T * I + T)
    GemvParams gp{};
    gp.x = static_cast<const __nv_bfloat16*>(x);
    gp.ids = ids; gp.ids_bytes = ids_bytes;
    gp.weights = weights; gp.weights_f32 = weights_f32 ? 1 : 0;
    gp.T = T; gp.topk = topk; gp.n = n_experts; gp.H = H; gp.I = I;
    gp.accumulate = accumulate ? 1 : 0;
    gp.w13 = static_cast<const uint8_t*>(w13); gp.s13 = s13;
    gp.w2 = static_cast<const uint8_t*>(w2); gp.s2 = s2;
    gp.h = (__nv_bfloat16*)(ws + pl.o_ws1);
    gp.out = static_cast<__nv_bfloat16*>(out);
    gp.sw13 = static_cast<const __nv_bfloat16*>(sw13);
    gp.sw2 = static_cast<const __nv_bfloat16*>(sw2);
    gp.sgate = static_cast<const __nv_bfloat16*>(sgate);
    gp.hs = gp.h + (size_t)P * I;
    gp.gs = reinterpret_cast<float*>(gp.hs + (size_t)T * I);
    gp.w2_early = 1;
    return run_gemv(gp, st);
  }

  RouteParams rp{};
  rp.ids = ids; rp.ids_bytes = ids_bytes; rp.P = P; rp.n = n_experts;
  rp.cnt = (int*)(ws + pl.o_cnt); rp.off = (int*)(ws + pl.o_off);
  rp.sorted = (int*)(ws + pl.o_sorted); rp.inv = (int*)(ws + pl.o_inv);
  rp.tiles1 = (int4*)(ws + pl.o_tiles1); rp.tiles2 = (int4*)(ws + pl.o_tiles2);
  rp.ntiles = (int*)(ws + pl.o_ntiles);
  rp.BN = pl.BN;
  rp.mt1 = 2 * I / 128; rp.nkb1 = H / 128;
  rp.split1_min = pl.split1_min; rp.split1_max = pl.split1_max;
  rp.mt2 = H / 128; rp.nkb2 = I / 128;
  rp.split2_min = pl.split2_min; rp.split2_max = pl.split2_max;
  rp.sms = num_sms();
  uint8_t* xq = (uint8_t*)(ws + pl.o_xq);
  float* xs = (float*)(ws + pl.o_xs);
  // the route launch quantises the activations itself up to
  // kFusedQuantMaxPairs pairs (its CTAs share the rows)
  rp.fuse_quant = P <= kFusedQuantMaxPairs ? 1 : 0;
  rp.x = static_cast<const __nv_bfloat16*>(x);
  rp.topk = topk; rp.H = H; rp.xq = xq; rp.xs = xs;
  if (link) {
    rp.wait_flags = link->wait_flags; rp.wait_epoch = link->epoch; rp.wait_n = link->n_ranks;
    rp.wait_err = link->err; rp.wait_code = link->wait_code; rp.wait_budget = link->budget_ns;
  }
  if (rp.fuse_quant && fused_enabled()) {
    const int rc = pl.BN == 16 ? launch_fused<16, 2>(pl, rp, ws, x, weights, weights_f32, T, topk,
                                                     w13, s13, w2, s2, n_experts, H, I, out,
                                                     accumulate, err_word, link, st)
                               : launch_fused<64, 2>(pl, rp, ws, x, weights, weights_f32, T, topk,
                                                     w13, s13, w2, s2, n_experts, H, I, out,
                                                     accumulate, err_word, link, st);
    if (rc != kFusedDeclined) return rc;
  }
  const bool pdl = pdl_enabled();
  // shared memory: cnt, off, tile prefix [n] + sorted [P] (fused) + NW chunk
  // histograms of n ints, as many chunks (<= 32, <= the 32-pair batches) as
  // the budget holds
  const size_t rbase = sizeof(int) * (3 * (size_t)n_experts + (rp.fuse_quant ? (size_t)P : 0));
  long nw = ((long)kRouteSmemBudget - (long)rbase) / (long)(sizeof(int) * (size_t)n_experts);
  // 512 threads per route CTA: with its registers (< 64 per thread) a CTA of
  // the following GEMM (programmatic launch) fits beside it on the same SM
  // and runs its prologue while the route finishes
  constexpr int kRouteThreads = 512;
  nw = nw < 1 ? 1 : (nw > kRouteThreads / 32 ? kRouteThreads / 32 : nw);
  if (nw > (P + 31) / 32) nw = (P + 31) / 32;
  rp.nw = (int)nw;
  const size_t rsmem = rbase + sizeof(int) * (size_t)nw * n_experts;
  if (rsmem > 48 * 1024)
    D3_CUDA_TRY(cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)rsmem),
                "route smem attribute");
  // CTAs: enough for the tile lists (one entry per thread per sweep); with the
  // quantisation folded in, one per SM (the units are instruction-bound: a
  // CTA on every SM spreads their issue over the whole GPU, and every CTA's
  // sort of the pairs is cheap)
  long rgrid = (long)(pl.maxt1 + pl.maxt2 + 4095) / 4096;
  if (rp.fuse_quant) rgrid = num_sms();
  rgrid = rgrid < 1 ? 1 : (rgrid > num_sms() ? num_sms() : rgrid);
  // The first launch of a call is an ordinary stream dependent: whatever the
  // caller queued before it (copies, foreign kernels) must complete first;
  // only the launches inside this call are chained programmatically.
  D3_CUDA_TRY(launch_k(route_kernel, dim3((unsigned)rgrid), dim3(kRouteThreads), rsmem, st, false,
                       rp),
              "route_kernel launch");
  int rc = D3_OK;
  if (!rp.fuse_quant) {
    const long warps = (long)pl.Ppad * (H / 128);
    D3_CUDA_TRY(launch_k(quant_x_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0,
                         st, pdl, static_cast<const __nv_bfloat16*>(x), (const int*)rp.sorted,
                         (const int*)(rp.ntiles + 2), topk, H, xq, xs),
                "quant_x_kernel launch");
  }
  CUtensorMap tw1, tx1, tw2, tx2;
  if ((rc = make_tmap_u8(&tw1, w13, H, (uint64_t)n_experts * 2 * I, H, 128))) return rc;
  if ((rc = make_tmap_u8(&tx1, xq, 2 * H, pl.Ppad, 2 * H, pl.BN))) return rc;
  float* ws1 = (float*)(ws + pl.o_ws1);
  GemmParams g1{};
  g1.tiles = rp.tiles1; g1.ntiles = rp.ntiles; g1.wscale = s13;
  g1.rows_per_expert = 2 * I; g1.mblocks = 2 * I / 128; g1.kblocks = H / 128;
  g1.xscale = xs; g1.K = H; g1.out = ws1; g1.P = P; g1.Mtot = 2 * I;
  g1.err = err_word;
  rc = pl.BN == 16 ? launch_gemm<16, 2>(tw1, tx1, g1, pl.maxt1, st)
                   : launch_gemm<64, 2>(tw1, tx1, g1, pl.maxt1, st);
  if (rc) return rc;

  uint8_t* hq = (uint8_t*)(ws + pl.o_hq);
  float* hs = (float*)(ws + pl.o_hs);
  {
    const long warps = (long)pl.Ppad * (I / 128);
    D3_CUDA_TRY(launch_k(act_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st,
                         pdl, (const float*)ws1, (const int*)(rp.ntiles + 3), P,
                         (const int*)(rp.ntiles + 2), I, hq, hs),
                "act_kernel launch");
  }
  if ((rc = make_tmap_u8(&tw2, w2, I, (uint64_t)n_experts * H, I, 128))) return rc;
  if ((rc = make_tmap_u8(&tx2, hq, 2 * I, pl.Ppad, 2 * I, pl.BN))) return rc;
  float* ws2 = (float*)(ws + pl.o_ws2);
  GemmParams g2{};
  g2.tiles = rp.tiles2; g2.ntiles = rp.ntiles + 1; g2.wscale = s2;
  g2.rows_per_expert = H; g2.mblocks = H / 128; g2.kblocks = I / 128;
  g2.xscale = hs; g2.K = I; g2.out = ws2; g2.P = P; g2.Mtot = H;
  g2.err = err_word;
  rc = pl.BN == 16 ? launch_gemm<16, 2>(tw2, tx2, g2, pl.maxt2, st)
                   : launch_gemm<64, 2>(tw2, tx2, g2, pl.maxt2, st);
  if (rc) return rc;
  if (link) {
    // up to one CTA per received row (8 warps each: a row's 128-column
    // blocks in one sweep); CTAs past the valid rows only arrive
    const int cgrid = T < 16 * num_sms() ? T : 16 * num_sms();
    D3_CUDA_TRY(launch_k(combine_return_kernel, dim3((unsigned)cgrid), dim3(256), 0, st, pdl,
                         (const float*)ws2, (const int*)(rp.ntiles + 4), P, H, (const int*)rp.inv,
                         (const int*)rp.sorted, (const int*)(rp.ntiles + 2), weights, weights_f32,
                         T, topk, *link),
                "combine_return_kernel launch");
  } else {
    const dim3 grid((unsigned)((H / 4 + 127) / 128), (unsigned)T);
    D3_CUDA_TRY(launch_k(combine_kernel, grid, dim3(128), 0, st, pdl, (const float*)ws2,
                         (const int*)(rp.ntiles + 4), P, H, (const int*)rp.inv, weights,
                         weights_f32, T, topk,
                         accumulate ? 1 : 0, static_cast<__nv_bfloat16*>(out)),
                "combine_kernel launch");
  }
  return D3_OK;
}

extern "C" {

int d3_moe_fp8_forward(const void* x, const void* ids, int32_t ids_bytes, const void* weights,
                       int32_t weights_f32, int32_t T, int32_t topk, const void* w13,
                       const float* s13, const void* w2, const float* s2, int32_t n_experts,
                       int32_t H, int32_t I, void* out, int32_t accumulate, int32_t* err_word,
                       void* workspace, size_t workspace_bytes, d3_stream_t stream) {
  return moe_forward(x, ids, ids_bytes, weights, weights_f32, T, topk, w13, s13, w2, s2,
                     n_experts, H, I, out, accumulate, err_word, workspace, workspace_bytes,
                     stream, nullptr, nullptr, nullptr);
}

int d3_moe_fp8_forward_shared(const void* x, const void* ids, int32_t ids_bytes,
                              const void* weights, int32_t weights_f32, int32_t T, int32_t topk,
                              const void* w13, const float* s13, const void* w2, const float* s2,
                              int32_t n_experts, int32_t H, int32_t I, const void* shared_w13,
                              const void* shared_w2, const void* shared_gate, void* out,
                              int32_t accumulate, int32_t* err_word, void* workspace,
                              size_t workspace_bytes, d3_stream_t stream) {
  D3_CHECK_ARG(shared_w13 && shared_w2, "d3_moe_fp8_forward_shared: null shared expert");
  return moe_forward(x, ids, ids_bytes, weights, weights_f32, T, topk, w13, s13, w2, s2,
                     n_experts, H, I, out, accumulate, err_word, workspace, workspace_bytes,
                     stream, shared_w13, shared_w2, shared_gate);
}

size_t d3_resolve_fetch_moe_workspace_size(int32_t k, int32_t H, int32_t I) {
  if (k < 1 || k > 64 || H < 512 || I < 512) return 0;
  return overlap_workspace(k, I);
}

static int resolve_fetch_moe(const d3_layer_cache* L, const void* ids, int32_t ids_bytes,
                             int32_t k, const void* x, const void* weights, int32_t weights_f32,
                             int32_t H, int32_t I, const void* shared_w13, const void* shared_w2,
                             const void* shared_gate, void* out, int32_t accumulate,
                             int32_t* err_word, void* workspace, size_t workspace_bytes,
                             int32_t fetch_ctas, int32_t stages, const void* const* l2_warm,
                             const size_t* l2_warm_bytes, int32_t n_windows,
                             d3_stream_t stream) {
  D3_CHECK_ARG(L && ids && x && weights && out && err_word, "d3_resolve_fetch_moe: null pointer");
  D3_CHECK_ARG(n_windows >= 0 && n_windows <= kMaxWarmWindows,
               "d3_resolve_fetch_moe_l2warm: n_windows must be in [0, %d]", kMaxWarmWindows);
  D3_CHECK_ARG(n_windows == 0 || (l2_warm && l2_warm_bytes),
               "d3_resolve_fetch_moe_l2warm: null window arrays");
  for (int w = 0; w < n_windows; ++w)
    D3_CHECK_ARG(l2_warm[w] || !l2_warm_bytes[w], "d3_resolve_fetch_moe_l2warm: null window");
  D3_CHECK_ARG(stages >= 1 && stages <= 7, "stages must be a non-empty mask of 1, 2, 4");
  D3_CHECK_ARG(k >= 1 && k <= 64, "k must be in [1, 64] (got %d)", k);
  if (!gemv_shapes_ok(k, H, I))
    return fail(D3_ERR_UNSUPPORTED, "H and I must be 512 x {1,2,4,8} / {1,2,4}");
  D3_CHECK_ARG(L->nbuf == 4, "the layer cache must hold the 4 buffers w13, w2, s13, s2");
  const int64_t b13 = 2LL * I * H, b2 = (int64_t)H * I;
  const int64_t bs13 = (2LL * I / 128) * (H / 128) * 4, bs2 = ((int64_t)H / 128) * (I / 128) * 4;
  if (L->bytes[0] != b13 || L->bytes[1] != b2 || L->bytes[2] != bs13 || L->bytes[3] != bs2)
    return fail(D3_ERR_INVALID_ARG, "buffer sizes do not match H=%d I=%d", H, I);
  if (L->capacity < k)
    return fail(D3_ERR_UNSUPPORTED, "capacity %d < k %d (a slot could be filled twice)",
                L->capacity, k);
  D3_CHECK_ARG(fetch_ctas >= 0 && fetch_ctas <= 1024, "fetch_ctas out of range");
  if (shared_w13 || shared_w2) D3_CHECK_ARG(shared_w13 && shared_w2, "shared expert incomplete");
  if (!aligned16(x) || !aligned16(out) ||
      (shared_w13 && (!aligned16(shared_w13) || !aligned16(shared_w2))) ||
      (shared_gate && !aligned16(shared_gate)))
    return fail(D3_ERR_MISALIGNED, "x, out and the shared expert weights must be 16-byte aligned");
  if (!workspace || workspace_bytes < overlap_workspace(k, I))
    return fail(D3_ERR_WORKSPACE, "workspace needs %zu bytes (got %zu)", overlap_workspace(k, I),
                workspace_bytes);
  if (!aligned16(workspace)) return fail(D3_ERR_MISALIGNED, "workspace must be 16-byte aligned");
  char* ws = static_cast<char*>(workspace);
  auto* done = reinterpret_cast<unsigned long long*>(ws);
  cudaStream_t st = (cudaStream_t)stream;
  GemvParams gp{};
  gp.x = static_cast<const __nv_bfloat16*>(x);
  gp.ids = L->out_slot; gp.ids_bytes = 4;
  gp.weights = weights; gp.weights_f32 = weights_f32 ? 1 : 0;
  gp.T = 1; gp.topk = k; gp.n = L->capacity; gp.H = H; gp.I = I;
  gp.accumulate = accumulate ? 1 : 0;
  gp.w13 = static_cast<const uint8_t*>(L->cache[0]);
  gp.w2 = static_cast<const uint8_t*>(L->cache[1]);
  gp.s13 = static_cast<const float*>(L->cache[2]);
  gp.s2 = static_cast<const float*>(L->cache[3]);
  gp.h = reinterpret_cast<__nv_bfloat16*>(ws + al(64 * sizeof(unsigned long long)));
  gp.hs = gp.h + (size_t)k * I;
  gp.gs = reinterpret_cast<float*>(gp.hs + I);
  gp.out = static_cast<__nv_bfloat16*>(out);
  gp.sw13 = static_cast<const __nv_bfloat16*>(shared_w13);
  gp.sw2 = static_cast<const __nv_bfloat16*>(shared_w2);
  gp.sgate = static_cast<const __nv_bfloat16*>(shared_gate);
  gp.w2_early = 0;
  gp.fetch_slot = L->fetch_slot;   // the down launch loads every other slot's W2 early
  gp.nmiss = L->nmiss;
  // stages: 1 allocator, 2 fetch + gate/up, 4 down projection; a call's
  // first launch is an ordinary stream dependent (no programmatic launch)
  if (!(stages & 3)) return run_gemv2(gp, st, false);
  FetchParams fp{};
  int64_t expert_bytes = 0;
  int rc = resolve_for_fetch(L, ids, ids_bytes, k, reinterpret_cast<int64_t*>(done), 64, st, &fp,
                             &expert_bytes, (stages & 1) != 0);
  if (rc) return rc;
  if (!(stages & 2)) return (stages & 4) ? run_gemv2(gp, st, false) : D3_OK;
  FetchOverlapParams o{};
  o.done = done;
  // fetch CTAs, then the rest of one resident wave (2 CTAs per SM) runs the
  // gate/up units
  o.fetch_ctas = fetch_ctas > 0 ? fetch_ctas : kOverlapFetchCtas;
  if (o.fetch_ctas > num_sms()) o.fetch_ctas = num_sms();
  o.early_mask = (1u << 0) | (1u << 2);
  o.vecA = (b13 + bs13) / 16;
  o.err = err_word; o.err_code = 41; o.budget_ns = kOverlapWaitBudgetNs;
  {
    unsigned long long end = 0;
    for (int w = 0; w < n_windows; ++w) {
      const unsigned long long lines = (unsigned long long)(l2_warm_bytes[w] >> 7);
      if (!lines) continue;
      end += lines;
      o.warm[o.n_warm] = static_cast<const char*>(l2_warm[w]);
      o.warm_end[o.n_warm] = end;
      ++o.n_warm;
    }
  }
  const int grid = 2 * num_sms();
  cudaError_t e;
  const bool pdl = pdl_enabled() && (stages & 1);
  switch (H / 512) {
    case 1: e = launch_k(fetch_gemv13_kernel<1>, dim3(grid), dim3(kGemvThreads), 0, st, pdl, fp, gp, o); break;
    case 2: e = launch_k(fetch_gemv13_kernel<2>, dim3(grid), dim3(kGemvThreads), 0, st, pdl, fp, gp, o); break;
    case 4: e = launch_k(fetch_gemv13_kernel<4>, dim3(grid), dim3(kGemvThreads), 0, st, pdl, fp, gp, o); break;
    default: e = launch_k(fetch_gemv13_kernel<8>, dim3(grid), dim3(kGemvThreads), 0, st, pdl, fp, gp, o); break;
  }
  D3_CUDA_TRY(e, "fetch_gemv13_kernel launch");
  return (stages & 4) ? run_gemv2(gp, st, pdl_enabled()) : D3_OK;
}

int d3_resolve_fetch_moe(const d3_layer_cache* L, const void* ids, int32_t ids_bytes, int32_t k,
                         const void* x, const void* weights, int32_t weights_f32, int32_t H,
                         int32_t I, const void* shared_w13, const void* shared_w2,
                         const void* shared_gate, void* out, int32_t accumulate,
                         int32_t* err_word, void* workspace, size_t workspace_bytes,
                         int32_t fetch_ctas, int32_t stages, d3_stream_t stream) {
  return resolve_fetch_moe(L, ids, ids_bytes, k, x, weights, weights_f32, H, I, shared_w13,
                           shared_w2, shared_gate, out, accumulate, err_word, workspace,
                           workspace_bytes, fetch_ctas, stages, nullptr, nullptr, 0, stream);
}

int d3_resolve_fetch_moe_l2warm(const d3_layer_cache* L, const void* ids, int32_t ids_bytes,
                                int32_t k, const void* x, const void* weights,
                                int32_t weights_f32, int32_t H, int32_t I,
                                const void* shared_w13, const void* shared_w2,
                                const void* shared_gate, void* out, int32_t accumulate,
                                int32_t* err_word, void* workspace, size_t workspace_bytes,
                                int32_t fetch_ctas, int32_t stages,
                                const void* const* l2_warm, const size_t* l2_warm_bytes,
                                int32_t n_windows, d3_stream_t stream) {
  return resolve_fetch_moe(L, ids, ids_bytes, k, x, weights, weights_f32, H, I, shared_w13,
                           shared_w2, shared_gate, out, accumulate, err_word, workspace,
                           workspace_bytes, fetch_ctas, stages, l2_warm, l2_warm_bytes, n_windows,
                           stream);
}

int d3_moe_fp8_forward_p2p(const void* x, const void* ids, int32_t ids_bytes,
                           const void* weights, int32_t weights_f32, int32_t T, int32_t topk,
                           const void* w13, const float* s13, const void* w2, const float* s2,
                           int32_t n_experts, int32_t H, int32_t I, int32_t* err_word,
                           void* workspace, size_t workspace_bytes, const int64_t* wait_flags,
                           const int64_t* epoch, int32_t n_ranks, int32_t rank, int32_t cap,
                           void* const* peer_ret, int64_t* const* peer_flag_r, uint32_t* counter,
                           int32_t wait_code, int64_t budget_ns, d3_stream_t stream) {
  D3_CHECK_ARG(wait_flags && epoch && peer_ret && peer_flag_r && counter && err_word,
               "d3_moe_fp8_forward_p2p: null pointer");
  if (n_ranks < 1 || n_ranks > kP2pMaxRanks)
    return fail(D3_ERR_TOO_LARGE, "n_ranks must be in [1, %d]", kP2pMaxRanks);
  D3_CHECK_ARG(rank >= 0 && rank < n_ranks && cap >= 1 && (long)n_ranks * cap == T,
               "rank out of range or T != n_ranks * cap");
  D3_CHECK_ARG(budget_ns > 0, "budget_ns must be positive");
  P2pLink link{};
  link.wait_flags = reinterpret_cast<const long long*>(wait_flags);
  link.epoch = reinterpret_cast<const long long*>(epoch);
  link.n_ranks = n_ranks; link.rank = rank; link.cap = cap;
  link.err = err_word; link.wait_code = wait_code; link.budget_ns = (unsigned long long)budget_ns;
  link.counter = counter;
  for (int s = 0; s < n_ranks; ++s) {
    D3_CHECK_ARG(peer_ret[s] && peer_flag_r[s], "d3_moe_fp8_forward_p2p: null peer pointer");
    if (!aligned16(peer_ret[s])) return fail(D3_ERR_MISALIGNED, "peer ret must be 16-byte aligned");
    link.ret[s] = static_cast<__nv_bfloat16*>(peer_ret[s]);
    link.flag_r[s] = reinterpret_cast<long long*>(peer_flag_r[s]);
  }
  return moe_forward(x, ids, ids_bytes, weights, weights_f32, T, topk, w13, s13, w2, s2,
                     n_experts, H, I, peer_ret[0], 0, err_word, workspace, workspace_bytes, stream,
                     nullptr, nullptr, nullptr, &link);
}

}  // extern "C"
