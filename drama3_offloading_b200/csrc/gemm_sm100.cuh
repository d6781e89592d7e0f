// Block-scaled FP8 grouped GEMM tile engine for sm_100a (tcgen05 + TMEM + TMA).
//
// One persistent CTA per SM walks a device-built tile list.  A tile is
// (expert e, 128-row M block m of the expert's weight, N block of BN routed
// pairs starting at sorted row row0, K-block range [kb0, kb1)).  Swap-AB: the
// weight rows are the MMA's M (128) and the pairs its N, so a single decode
// token still drives full-height MMAs.
//
// Warp roles (THREADS = 64 + 32*EPI):
//   warp 0     TMA producer (one elected lane): per pipeline stage KPS
//              consecutive K-blocks of the weight tile (KPS x 128x128 B, 128 B
//              swizzle) and of the activation hi/lo planes (2 x KPS x BNx128 B).
//              Loading K-block pairs back to back asks DRAM for 256 contiguous
//              bytes of every weight row at once instead of two 128-B halves
//              a stage apart.
//   warp 1     MMA issuer (one lane): per K-block, 4 MMAs (K = 32 each) against
//              hi and 4 against lo into one TMEM accumulator (so D = W.(hi+lo)),
//              accumulators double-buffered, tcgen05.commit -> mbarriers.
//   warps 2..  epilogue: each thread owns one accumulator row (TMEM lane) and
//              CPT columns; per K-block it reads the accumulator and adds
//              scale[kb][n] * D into fp32 registers (per-block promotion, the
//              128x128 weight scale times the activation block scale); the
//              per-tile scales are staged once in shared memory, weight scale
//              folded in.  At tile end the fp32 partial sums are stored to the
//              split-K workspace (coalesced across the 32 rows of a warp).
// Every mbarrier wait is bounded by the global timer; on expiry the CTA
// records an error word, unwinds, waits for its own MMAs and frees TMEM.
#pragma once

#include "d3_common.cuh"

#include <cuda.h>

namespace d3 {

constexpr uint64_t kGemmWaitBudgetNs = 2000000000ull;  // 2 s per wait, then abort
constexpr int kGemmMaxTileKb = 32;                     // K-blocks one tile may span

struct GemmParams {
  const int4* tiles;
  const int* ntiles;          // device count of valid tiles
  const float* wscale;        // [n][mblocks][kblocks]
  int rows_per_expert;        // weight rows per expert (2I or H)
  int mblocks, kblocks;       // per expert, 128-granular
  const float* xscale;        // [rows][kblocks] activation block scales
  int K;                      // bytes per weight row = K elements
  float* out;                 // [split][P][Mtot]
  int P, Mtot;
  int* err;                   // device error word (first failure wins)
};

template <int BN, int KPS>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int KB_BYTES = A_BYTES + 2 * B_BYTES;   // one K-block
  static constexpr int STAGE_BYTES = KPS * KB_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;
  // accumulator buffers in TMEM (one per K-block in flight) and the number of
  // K-blocks the epilogue promotes per round: the MMA runs up to NB K-blocks
  // ahead of the epilogue, which loads G accumulators back to back and waits
  // once, so the per-K-block TMEM round trip no longer paces the MMA.
  static constexpr int NB = BN >= 64 ? 4 : 8;
  static constexpr int G = BN >= 64 ? 2 : 4;
  static constexpr int TMEM_COLS = NB * BN;
  static constexpr int EPI = BN >= 64 ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI;
  static constexpr int CPT = BN * 4 / EPI;
  // per-tile promotion scales, double-buffered: a tile's scales are loaded
  // while the previous tile is promoted
  static constexpr int SCALE_FLOATS = kGemmMaxTileKb * BN;
  static constexpr int SCALE_BYTES = 2 * SCALE_FLOATS * 4;
  static constexpr int SPT = (SCALE_FLOATS + 32 * EPI - 1) / (32 * EPI);  // entries per thread
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + SCALE_BYTES + 256;
  static_assert(STAGES >= 2, "pipeline needs at least two stages");
};

__device__ __forceinline__ void gemm_error(int* err, int code) { atomicCAS(err, 0, code); }

__device__ __forceinline__ void epi_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Generic-proxy global writes (st.global by other CTAs of the same launch)
// made visible to this thread's later async-proxy (TMA) reads, and this
// thread's own generic writes to later async-proxy reads by others.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Shared-memory carve-up of the tile engine (dynamic smem, 1024-aligned).
template <int BN, int KPS>
struct GemmSmem {
  uint8_t* stage_base;   // [STAGES][STAGE_BYTES]
  float* s_scale;        // [2][kGemmMaxTileKb][BN]
  uint64_t* full;        // [STAGES]
  uint64_t* empty;       // [STAGES]
  uint64_t* accf;        // [NB] accumulator ready
  uint64_t* acce;        // [NB] accumulator drained
  uint64_t* done;        // [1]  all MMAs of the CTA retired
  __device__ __forceinline__ static GemmSmem carve(uint8_t* smem_raw) {
    using Cfg = GemmCfg<BN, KPS>;
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
    GemmSmem g;
    g.stage_base = smem;
    g.s_scale = reinterpret_cast<float*>(smem + (size_t)Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)Cfg::STAGES * Cfg::STAGE_BYTES +
                                                 Cfg::SCALE_BYTES);
    g.full = bars;
    g.empty = bars + Cfg::STAGES;
    g.accf = bars + 2 * Cfg::STAGES;
    g.acce = bars + 2 * Cfg::STAGES + Cfg::NB;
    g.done = bars + 2 * Cfg::STAGES + 2 * Cfg::NB;
    return g;
  }
  // one thread: barrier init (visible to the async proxy after the fence)
  __device__ __forceinline__ void init() const {
    using Cfg = GemmCfg<BN, KPS>;
    for (int i = 0; i < Cfg::STAGES; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
    for (int i = 0; i < Cfg::NB; ++i) { mbar_init(accf + i, 1); mbar_init(acce + i, 32 * Cfg::EPI); }
    mbar_init(done, 1);
    fence_barrier_init();
  }
};

// Pipeline positions a role carries from one tile list to the next (a
// persistent kernel runs several lists through the same rings).
struct PipePos {
  int stage = 0;
  uint32_t phase = 0;
  uint32_t it = 0;      // accumulator uses (one per K-block)
};

// Optional gate on the activation operand: the producer issues each stage's
// weight tile at once but its activation tiles only after *count >= target
// (acquire, bounded), so the weights of a list whose activations another
// phase of the same launch is still writing stream in early.
struct OperandGate {
  const unsigned* count;
  unsigned target;
  int* err;
  int code;
};

// ---- warp 0, one lane: TMA producer over the tile list of p
template <int BN, int KPS>
__device__ void gemm_produce(const GemmSmem<BN, KPS>& sm, const CUtensorMap* tm_w,
                             const CUtensorMap* tm_x, const GemmParams& p, int ntiles, PipePos& ps,
                             volatile int* s_abort, const OperandGate* gate) {
  using Cfg = GemmCfg<BN, KPS>;
  constexpr int S = Cfg::STAGES;
  struct Pend { int stage, kb, nk, row0; };
  Pend pend[S];
  int npend = 0;
  bool open = gate == nullptr;
  auto issue_b = [&](int stage, int kb, int nk, int row0) {
    uint8_t* st = sm.stage_base + (size_t)stage * Cfg::STAGE_BYTES;
    for (int q = 0; q < nk; ++q) {
      uint8_t* bh = st + q * Cfg::KB_BYTES + Cfg::A_BYTES;
      tma_load_2d(bh, tm_x, sm.full + stage, (kb + q) * 128, row0);
      tma_load_2d(bh + Cfg::B_BYTES, tm_x, sm.full + stage, p.K + (kb + q) * 128, row0);
    }
  };
  auto open_gate = [&]() {
    if (open) return;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu_u32(gate->count) < gate->target) {
      if (globaltimer_ns() - t0 > kGemmWaitBudgetNs) { gemm_error(gate->err, gate->code); break; }
      __nanosleep(64);
    }
    fence_proxy_async_global();
    open = true;
    for (int i = 0; i < npend; ++i) issue_b(pend[i].stage, pend[i].kb, pend[i].nk, pend[i].row0);
    npend = 0;
  };
  for (int t = blockIdx.x; t < ntiles && !*s_abort; t += gridDim.x) {
    const int4 tl = __ldcg(p.tiles + t);
    const int e = tl.x, m = tl.y & 0xffff, row0 = tl.z;
    const int kb0 = (tl.w >> 8) & 0xFFF, kb1 = (tl.w >> 20) & 0xFFF;
    const int wrow = e * p.rows_per_expert + m * 128;
    for (int kb = kb0; kb < kb1; kb += KPS) {
      // every stage holds a weight tile whose activations wait on the gate:
      // nothing can free the next one before the gate opens
      if (npend == S) open_gate();
      if (!mbar_wait(sm.empty + ps.stage, ps.phase ^ 1, kGemmWaitBudgetNs)) {
        gemm_error(p.err, 1); *s_abort = 1; break;
      }
      const int nk = min(KPS, kb1 - kb);
      uint8_t* st = sm.stage_base + (size_t)ps.stage * Cfg::STAGE_BYTES;
      mbar_arrive_expect_tx(sm.full + ps.stage, nk * Cfg::KB_BYTES);
      for (int q = 0; q < nk; ++q)
        tma_load_2d(st + q * Cfg::KB_BYTES, tm_w, sm.full + ps.stage, (kb + q) * 128, wrow);
      if (open) issue_b(ps.stage, kb, nk, row0);
      else pend[npend++] = Pend{ps.stage, kb, nk, row0};
      if (++ps.stage == S) { ps.stage = 0; ps.phase ^= 1; }
    }
  }
  open_gate();
}

// ---- warp 1, one lane: MMA issuer over the tile list of p
template <int BN, int KPS>
__device__ void gemm_mma(const GemmSmem<BN, KPS>& sm, uint32_t tmem, const GemmParams& p,
                         int ntiles, PipePos& ps, volatile int* s_abort) {
  using Cfg = GemmCfg<BN, KPS>;
  constexpr int S = Cfg::STAGES;
  constexpr int NB = Cfg::NB;
  constexpr uint32_t idesc = idesc_e4m3_f32(128, BN);
  for (int t = blockIdx.x; t < ntiles && !*s_abort; t += gridDim.x) {
    const int4 tl = __ldcg(p.tiles + t);
    const int kb0 = (tl.w >> 8) & 0xFFF, kb1 = (tl.w >> 20) & 0xFFF;
    bool ok = true;
    for (int kb = kb0; kb < kb1 && ok; kb += KPS) {
      if (!mbar_wait(sm.full + ps.stage, ps.phase, kGemmWaitBudgetNs)) {
        gemm_error(p.err, 2); *s_abort = 1; break;
      }
      const int nk = min(KPS, kb1 - kb);
      const uint32_t st = smem_u32(sm.stage_base + (size_t)ps.stage * Cfg::STAGE_BYTES);
      for (int q = 0; q < nk; ++q, ++ps.it) {
        const uint32_t ab = ps.it % NB, aph = (ps.it / NB) & 1;
        if (!mbar_wait(sm.acce + ab, aph ^ 1, kGemmWaitBudgetNs)) {
          gemm_error(p.err, 2); *s_abort = 1; ok = false; break;
        }
        tc_fence_after();
        const uint32_t a = st + q * Cfg::KB_BYTES;
        const uint32_t bh = a + Cfg::A_BYTES, bl = bh + Cfg::B_BYTES;
        const uint32_t d = tmem + ab * BN;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8f6f4(d, smem_desc_k128(a + kk * 32), smem_desc_k128(bh + kk * 32), idesc,
                     kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8f6f4(d, smem_desc_k128(a + kk * 32), smem_desc_k128(bl + kk * 32), idesc, 1u);
        mma_commit(sm.accf + ab);
      }
      if (!ok) break;
      mma_commit(sm.empty + ps.stage);
      if (++ps.stage == S) { ps.stage = 0; ps.phase ^= 1; }
    }
  }
}

// ---- MMA lane, at the end: every issued MMA has retired before TMEM is freed
template <int BN, int KPS>
__device__ void gemm_mma_drain(const GemmSmem<BN, KPS>& sm, const PipePos& ps, int* err) {
  if (ps.it > 0) {
    mma_commit(sm.done);
    if (!mbar_wait(sm.done, 0, kGemmWaitBudgetNs)) gemm_error(err, 3);
  }
}

// ---- epilogue warps (ep = thread index among them): promotion and the
// split-K partial store of every tile of p
template <int BN, int KPS>
__device__ void gemm_epilogue(const GemmSmem<BN, KPS>& sm, uint32_t tmem, const GemmParams& p,
                              int ntiles, PipePos& ps, volatile int* s_abort,
                              volatile int* s_tile_abort) {
  using Cfg = GemmCfg<BN, KPS>;
  constexpr int NB = Cfg::NB;
  constexpr int CPT = Cfg::CPT;
  constexpr int NEPI = 32 * Cfg::EPI;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ep = threadIdx.x - 64;                // 0 .. NEPI-1
  const int q = warp & 3;
  const int col0 = ((warp - 2) >> 2) * CPT;
  const int row = q * 32 + lane;                 // weight row within the M tile
  const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + col0;
  constexpr int SPT = Cfg::SPT;
  // Promotion scales of a tile: scale[j][n] = s_w[kb0+j] * s_x[row0+n][kb0+j],
  // thread ep owns entries ep + k*NEPI.  They are loaded one tile ahead (the
  // tile descriptors two ahead) into registers, so the loads are long done
  // when the tile starts and its staging costs no memory round trip.
  // Coherent (L2) loads, never the non-coherent read-only path: under
  // programmatic launch this kernel's lifetime overlaps the kernels that
  // write the activation scales (for a reused workspace, a line cached by an
  // earlier call could otherwise be served stale).
  float pw[SPT], px[SPT];
  auto load_scales = [&](const int4 tl) {
    const int e = tl.x, m = tl.y & 0xffff, row0 = tl.z;
    const int ncount = tl.w & 0xFF;
    const int kb0 = (tl.w >> 8) & 0xFFF, kb1 = (tl.w >> 20) & 0xFFF;
    const float* ws = p.wscale + ((size_t)e * p.mblocks + m) * p.kblocks;
#pragma unroll
    for (int k = 0; k < SPT; ++k) {
      const int i = ep + k * NEPI;
      const int j = i / BN, n = i - j * BN;
      const bool live = j < kb1 - kb0 && n < ncount;
      pw[k] = live ? __ldcg(ws + kb0 + j) : 0.f;
      px[k] = live ? __ldcg(p.xscale + (size_t)(row0 + n) * p.kblocks + kb0 + j) : 0.f;
    }
  };
  int t = blockIdx.x;
  int4 tl_cur = make_int4(0, 0, 0, 0), tl_nxt = make_int4(0, 0, 0, 0);
  if (t < ntiles) {
    tl_cur = __ldcg(p.tiles + t);
    load_scales(tl_cur);
    if (t + (int)gridDim.x < ntiles) tl_nxt = __ldcg(p.tiles + t + gridDim.x);
  }
  int buf = 0;
  for (; t < ntiles; t += gridDim.x) {
    const int4 tl = tl_cur;
    const int e = tl.x, m = tl.y & 0xffff, row0 = tl.z;
    const int ncount = tl.w & 0xFF;
    const int kb0 = (tl.w >> 8) & 0xFFF, kb1 = (tl.w >> 20) & 0xFFF;
    const int nkb = kb1 - kb0;
    (void)e;
    // this tile's scales into buffer `buf` (last read two tiles ago: every
    // thread has passed the previous tile's barrier since)
    float* s_scale = sm.s_scale + buf * Cfg::SCALE_FLOATS;
#pragma unroll
    for (int k = 0; k < SPT; ++k) {
      const int i = ep + k * NEPI;
      if (i < Cfg::SCALE_FLOATS) s_scale[i] = pw[k] * px[k];
    }
    if (ep == 0) *s_tile_abort = *s_abort;
    epi_bar_sync(NEPI);
    // the next tile's scales and the descriptor after it, in flight while
    // this tile is promoted
    const bool has_next = t + (int)gridDim.x < ntiles;
    int4 tl_after = tl_nxt;
    if (has_next) {
      load_scales(tl_nxt);
      if (t + 2 * (int)gridDim.x < ntiles) tl_after = __ldcg(p.tiles + t + 2 * gridDim.x);
    }
    // the abort decision is taken once per tile from one shared word, so all
    // epilogue threads leave together (none is left waiting at a barrier)
    if (*s_tile_abort) break;
    float r[CPT];
#pragma unroll
    for (int n = 0; n < CPT; ++n) r[n] = 0.f;
    bool ok = true;
    constexpr int G = Cfg::G;
    for (int j0 = 0; j0 < nkb; j0 += G) {
      const int g = min(G, nkb - j0);
      if (ok) {
        for (int jj = 0; jj < g; ++jj) {
          const uint32_t b = (ps.it + jj) % NB, ph = ((ps.it + jj) / NB) & 1;
          if (!mbar_wait(sm.accf + b, ph, kGemmWaitBudgetNs)) {
            gemm_error(p.err, 4); *s_abort = 1; ok = false; break;
          }
        }
      }
      if (ok) {
        tc_fence_after();
        uint32_t v[G][CPT];
#pragma unroll
        for (int jj = 0; jj < G; ++jj) {
          if (jj < g) {
            const uint32_t b = (ps.it + jj) % NB;
#pragma unroll
            for (int c16 = 0; c16 < CPT / 16; ++c16) {
              uint32_t (&vv)[16] = *reinterpret_cast<uint32_t(*)[16]>(&v[jj][c16 * 16]);
              tmem_ld16(lane_base + b * BN + c16 * 16, vv);
            }
          }
        }
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < G; ++jj) {
          if (jj < g) {
            const float4* sc = reinterpret_cast<const float4*>(s_scale + (j0 + jj) * BN + col0);
#pragma unroll
            for (int c4 = 0; c4 < CPT / 4; ++c4) {
              const float4 s4 = sc[c4];
              r[4 * c4 + 0] = fmaf(s4.x, __uint_as_float(v[jj][4 * c4 + 0]), r[4 * c4 + 0]);
              r[4 * c4 + 1] = fmaf(s4.y, __uint_as_float(v[jj][4 * c4 + 1]), r[4 * c4 + 1]);
              r[4 * c4 + 2] = fmaf(s4.z, __uint_as_float(v[jj][4 * c4 + 2]), r[4 * c4 + 2]);
              r[4 * c4 + 3] = fmaf(s4.w, __uint_as_float(v[jj][4 * c4 + 3]), r[4 * c4 + 3]);
            }
          }
        }
        tc_fence_before();
        for (int jj = 0; jj < g; ++jj) mbar_arrive(sm.acce + (ps.it + jj) % NB);
      }
      ps.it += g;
    }
    tl_cur = tl_nxt;
    tl_nxt = tl_after;
    buf ^= 1;
    if (!ok) continue;  // leaves at the next tile's shared abort decision
    const int split = tl.y >> 16;  // K-split index of this tile
    float* o = p.out + ((size_t)split * p.P + row0 + col0) * p.Mtot + m * 128 + row;
#pragma unroll
    for (int n = 0; n < CPT; ++n)
      if (col0 + n < ncount) o[(size_t)n * p.Mtot] = r[n];
  }
}

template <int BN, int KPS>
__global__ void __launch_bounds__(GemmCfg<BN, KPS>::THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_x, GemmParams p) {
  using Cfg = GemmCfg<BN, KPS>;
  extern __shared__ uint8_t smem_raw[];
  const GemmSmem<BN, KPS> sm = GemmSmem<BN, KPS>::carve(smem_raw);
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_tile_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm.init();
    s_abort = 0;
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // everything above is CTA-local set-up that overlaps the previous launch;
  // the tile list and operands are produced upstream
  pdl_trigger();
  pdl_wait();
  const int ntiles = __ldcg(p.ntiles);
  PipePos ps;
  if (warp == 0) {
    if (lane == 0) gemm_produce<BN, KPS>(sm, &tm_w, &tm_x, p, ntiles, ps, &s_abort, nullptr);
  } else if (warp == 1) {
    if (lane == 0) {
      gemm_mma<BN, KPS>(sm, tmem, p, ntiles, ps, &s_abort);
      gemm_mma_drain<BN, KPS>(sm, ps, p.err);
    }
  } else {
    gemm_epilogue<BN, KPS>(sm, tmem, p, ntiles, ps, &s_abort, &s_tile_abort);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

template <int BN, int KPS>
static int launch_gemm(const CUtensorMap& tw, const CUtensorMap& tx, const GemmParams& gp,
                       int max_tiles, cudaStream_t st) {
  using Cfg = GemmCfg<BN, KPS>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    D3_CUDA_TRY(cudaFuncSetAttribute(moe_gemm_kernel<BN, KPS>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM),
                "gemm smem attribute");
    attr_set[dev] = true;
  }
  int grid = num_sms();
  if (max_tiles < grid) grid = max_tiles;
  if (grid < 1) grid = 1;
  D3_CUDA_TRY(launch_k(moe_gemm_kernel<BN, KPS>, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM, st,
                       pdl_enabled(), tw, tx, gp),
              "moe_gemm_kernel launch");
  return D3_OK;
}

}  // namespace d3
