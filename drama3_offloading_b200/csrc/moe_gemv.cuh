// Small-batch routed-MoE path: the expert GEMMs as matrix-vector products on
// the CUDA cores, two launches per call.
//
// At a decode batch (one token, eight routed pairs) every expert weight byte
// meets exactly one activation row, so the work is a GEMV over 8 x 3 MiB of
// fp8 weights: HBM-bound with ~2 FLOP per byte.  The tensor-core path pays a
// fixed cost that dominates at this size (pair sort, activation planes, TMEM
// allocation, pipeline fill, split-K partials, a combine pass); this path
// streams the weights with 16-byte loads and keeps everything else on chip:
//
//   gemv13   one warp per (pair, intermediate row j): the gate row j and the
//            up row I + j of the pair's expert against the token row (held in
//            registers as fp32), per-128 K-block scales applied to the fp32
//            partial sums, then h[pair, j] = silu(g) * u  (workspace, rounded
//            to bf16 -- the precision the reference's bf16 path holds it in --
//            which halves the bytes every gemv2 CTA stages).
//   gemv2    one CTA per (token, 8 output rows): the token's pair rows of h
//            staged in shared memory; one warp per output row j sums
//            w[t,k] * s2 * (W2[e_k][j, :] . h[pair_k]) over the token's pairs
//            and writes out[t, j] (bf16, optionally added to out).  Its first
//            W2 rows are loaded BEFORE griddepcontrol.wait: they do not depend
//            on gemv13, so with programmatic launch the down-projection weights
//            stream in while the gate/up products finish.
//
// Optional shared expert (Drama-3's per-layer bf16 SwiGLU expert that every
// token runs, gated by sigmoid(x . shared_expert_gate)): gemv13 also runs its
// (token, row) units and one gate unit per token; gemv2 adds
// sigmoid(x . g) * (W2s[j] . hs[t]) to the same output in the same warp, so
// the whole MoE block is the same two launches.
//
// Activations stay bf16 (no activation quantisation): the token row as given,
// h rounded once to bf16 (~8 significant bits, as the tensor-core path's
// hi/lo e4m3 planes carry); the products are summed in fp32.
// Ids outside [0, n) skip their pair, as everywhere in this library.
#pragma once

#include "d3_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace d3 {

constexpr int kGemvThreads = 256;                 // 8 warps
constexpr int kGemvRowsPerCta = kGemvThreads / 32;
constexpr int kGemvMaxKbI = 16;                   // I / 128 for I <= 2048 (CPL <= 4)

struct GemvParams {
  const __nv_bfloat16* x;   // [T, H]
  const void* ids;          // [T, topk] int32 or int64
  int ids_bytes;
  const void* weights;      // [T, topk] fp32 or bf16
  int weights_f32;
  int T, topk, n, H, I, accumulate;
  const uint8_t* w13;       // [n, 2I, H] e4m3
  const float* s13;         // [n, 2I/128, H/128]
  const uint8_t* w2;        // [n, H, I] e4m3
  const float* s2;          // [n, H/128, I/128]
  __nv_bfloat16* h;         // [T*topk, I] workspace (bf16, as the reference's bf16 path)
  __nv_bfloat16* out;       // [T, H]
  // optional shared expert (every token, bf16, intermediate I): null sw13 =
  // none; null sgate = ungated
  const __nv_bfloat16* sw13;   // [2I, H] (gate rows [0, I), up rows [I, 2I))
  const __nv_bfloat16* sw2;    // [H, I]
  const __nv_bfloat16* sgate;  // [H]
  __nv_bfloat16* hs;           // [T, I] workspace
  float* gs;                   // [T] workspace: sigmoid(x . sgate)
  // gemv2 loads its first W2 rows before griddepcontrol.wait (1), or only
  // after it (0: the preceding launch may still be writing W2, as the fetch +
  // gate/up overlap launch does)
  int w2_early;
  // with w2_early == 0: the job table of that preceding fetch (the slots
  // whose W2/S2 bytes it writes; written by the allocator launch before it,
  // so readable before the wait) -- every other pair's W2 rows and scales
  // are loaded early; null = none early
  const int32_t* fetch_slot;
  const int32_t* nmiss;
};

// Fetch + gate/up overlap: which queued fetch job (if any) fills each pair's
// slot, and how the gate/up units learn that a job's W13/S13 bytes landed.
struct GemvOverlap {
  const int* s_job;                  // [pairs] in shared memory: job or -1 (resident)
  const unsigned long long* done;    // [jobs] W13+S13 vectors landed
  unsigned long long need;           // vectors per job in those buffers
  int* err;
  int err_code;
  unsigned long long budget_ns;
};

__device__ __forceinline__ int gemv_pair_id(const void* ids, int bytes, int i, int n) {
  const long long v = bytes == 8 ? static_cast<const long long*>(ids)[i]
                                 : (long long)static_cast<const int*>(ids)[i];
  return (v >= 0 && v < n) ? (int)v : -1;
}

// sum_q w[q] * v[q] over one 16-byte chunk of e4m3 weights, two partial sums.
__device__ __forceinline__ float dot16_e4m3(const uint4 w, const float (&v)[16]) {
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(wr[q] & 0xffffu), __NV_E4M3);
    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(wr[q] >> 16), __NV_E4M3);
    const float2 a = __half22float2(__half2(lo));
    const float2 b = __half22float2(__half2(hi));
    s0 = fmaf(a.x, v[4 * q + 0], s0);
    s1 = fmaf(a.y, v[4 * q + 1], s1);
    s0 = fmaf(b.x, v[4 * q + 2], s0);
    s1 = fmaf(b.y, v[4 * q + 3], s1);
  }
  return s0 + s1;
}

// sum_q w[q] * v[q] over 16 bf16 weights (two 16-byte words), two partial sums.
__device__ __forceinline__ float dot16_bf16(const uint4 a, const uint4 b, const float (&v)[16]) {
  const uint32_t wr[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    s0 = fmaf(__uint_as_float(wr[q] << 16), v[2 * q], s0);
    s1 = fmaf(__uint_as_float(wr[q] & 0xffff0000u), v[2 * q + 1], s1);
  }
  return s0 + s1;
}

__device__ __forceinline__ void unpack_bf16x8(const uint4 r, float* v) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[2 * q] = __uint_as_float(w[q] << 16);
    v[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The gate/up units of warp gw of nw: routed (pair, row) units, then the
// shared expert's (token, row) units, then one gate unit per token.  With an
// overlap context, pass 0 runs the units whose expert is resident (and the
// shared expert's) and pass 1 the units of fetched experts, each after a
// bounded wait until its job's W13/S13 bytes have landed.
template <int CPL>
__device__ __forceinline__ void gemv13_units(const GemvParams& p, long gw, long nw,
                                             const GemvOverlap* ov) {
  const int lane = threadIdx.x & 31;
  const int I = p.I, H = p.H, nkb = H / 128;
  const long routed = (long)p.T * p.topk * I;
  const long units = routed + (p.sw13 ? (long)p.T * I + (p.sgate ? p.T : 0) : 0);
  float xv[CPL][16];
  int cur_t = -1;
  unsigned long long ready = 0;  // jobs this warp has seen complete
  const int npass = ov ? 2 : 1;
  for (int pass = 0; pass < npass; ++pass) {
    for (long u = gw; u < units; u += nw) {
      if (u >= routed) {  // shared expert (warp-uniform branch)
        if (pass == 1) continue;
        const long v = u - routed;
        const bool gate_unit = v >= (long)p.T * I;
        const int t = gate_unit ? (int)(v - (long)p.T * I) : (int)(v / I);
        const int j = gate_unit ? 0 : (int)(v - (long)t * I);
        if (t != cur_t) {
          cur_t = t;
          const uint4* xr = reinterpret_cast<const uint4*>(p.x + (size_t)t * H);
#pragma unroll
          for (int c = 0; c < CPL; ++c) {
            const int q = lane + 32 * c;
            unpack_bf16x8(xr[2 * q], xv[c]);
            unpack_bf16x8(xr[2 * q + 1], xv[c] + 8);
          }
        }
        const uint4* rg = reinterpret_cast<const uint4*>(gate_unit ? p.sgate
                                                                   : p.sw13 + (size_t)j * H);
        float ag = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int q = lane + 32 * c;
          ag += dot16_bf16(__ldcg(rg + 2 * q), __ldcg(rg + 2 * q + 1), xv[c]);
        }
        ag = warp_sum(ag);
        if (gate_unit) {
          if (lane == 0) p.gs[t] = 1.f / (1.f + expf(-ag));
          continue;
        }
        const uint4* ru = reinterpret_cast<const uint4*>(p.sw13 + (size_t)(I + j) * H);
        float au = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int q = lane + 32 * c;
          au += dot16_bf16(__ldcg(ru + 2 * q), __ldcg(ru + 2 * q + 1), xv[c]);
        }
        au = warp_sum(au);
        if (lane == 0) p.hs[(size_t)t * I + j] = __float2bfloat16_rn(ag / (1.f + expf(-ag)) * au);
        continue;
      }
      const int pair = (int)(u / I), j = (int)(u - (long)pair * I);
      const int e = gemv_pair_id(p.ids, p.ids_bytes, pair, p.n);
      if (e < 0) continue;  // warp-uniform: the whole warp works on one unit
      if (ov) {
        const int job = ov->s_job[pair];
        if ((job >= 0) != (pass == 1)) continue;
        if (job >= 0 && !((ready >> job) & 1ull)) {
          bool ok = true;
          if (lane == 0) {
            const unsigned long long t0 = globaltimer_ns();
            while (ld_acquire_gpu_u64(ov->done + job) < ov->need) {
              if (globaltimer_ns() - t0 > ov->budget_ns) { ok = false; break; }
              __nanosleep(128);
            }
            if (!ok) atomicCAS(ov->err, 0, ov->err_code);
          }
          __syncwarp();  // the other lanes read the slot after lane 0's acquire
          ready |= 1ull << job;
        }
      }
      const uint4* wg = reinterpret_cast<const uint4*>(p.w13 + ((size_t)e * 2 * I + j) * H);
      const uint4* wu = reinterpret_cast<const uint4*>(p.w13 + ((size_t)e * 2 * I + I + j) * H);
      uint4 g[CPL], v[CPL];
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        g[c] = __ldcg(wg + lane + 32 * c);
        v[c] = __ldcg(wu + lane + 32 * c);
      }
      const int t = pair / p.topk;
      if (t != cur_t) {
        cur_t = t;
        const uint4* xr = reinterpret_cast<const uint4*>(p.x + (size_t)t * H);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int q = lane + 32 * c;  // K elements [16q, 16q + 16)
          unpack_bf16x8(xr[2 * q], xv[c]);
          unpack_bf16x8(xr[2 * q + 1], xv[c] + 8);
        }
      }
      const float* sg = p.s13 + ((size_t)e * (2 * I / 128) + j / 128) * nkb;
      const float* su = p.s13 + ((size_t)e * (2 * I / 128) + (I + j) / 128) * nkb;
      float ag = 0.f, au = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int kb = (lane + 32 * c) >> 3;
        ag = fmaf(__ldcg(sg + kb), dot16_e4m3(g[c], xv[c]), ag);
        au = fmaf(__ldcg(su + kb), dot16_e4m3(v[c], xv[c]), au);
      }
      ag = warp_sum(ag);
      au = warp_sum(au);
      if (lane == 0) p.h[u] = __float2bfloat16_rn(ag / (1.f + expf(-ag)) * au);
    }
  }
}

// CPL = 16-byte chunks per lane of a W13 row = H / 512.
template <int CPL>
__global__ void __launch_bounds__(kGemvThreads) moe_gemv13_kernel(GemvParams p) {
  pdl_wait();
  pdl_trigger();
  const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long nw = ((long)gridDim.x * blockDim.x) >> 5;
  gemv13_units<CPL>(p, gw, nw, nullptr);
}

// CPL = 16-byte chunks per lane of a W2 row = I / 512.  Grid (H / 8 / rpw, T);
// dynamic shared memory: topk rows of h (+ the shared expert's row), each
// 16-float chunk padded to 20 floats (conflict-free 16-byte reads: lane l's
// chunk starts at bank 20 l).
template <int CPL>
__global__ void __launch_bounds__(kGemvThreads, 2) moe_gemv2_kernel(GemvParams p, int rpw) {
  constexpr int kGemvPairGroup = 8 / CPL;  // W2 rows (of pairs) a warp keeps in flight
  extern __shared__ __align__(16) float s_h[];   // [topk][I / 16][20]
  __shared__ float s_w[64];
  __shared__ int s_e[64];
  __shared__ unsigned char s_early[64];
  // the W2 block scales of this CTA's rows (all in one 128-row block) per pair
  __shared__ float s_sc[64][kGemvMaxKbI];
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int I = p.I, H = p.H, topk = p.topk, nkbI = I / 128;
  const int t = blockIdx.y;
  const int row_stride = I / 16 * 20;
  const int j_first = (blockIdx.x * rpw) * kGemvRowsPerCta + warp;
  // ids (and the overlap path's job table) were written before the gate/up
  // launch started: safe to read early.  A pair is "early" when nothing in
  // flight writes its slot's W2/S2 bytes: its first W2 row and scales are
  // loaded before griddepcontrol.wait, so they stream in while the gate/up
  // products finish.
  // Every pair's expert and early flag, once per CTA into shared memory
  // before the wait (the scale staging and the sums below read them there,
  // so nothing after the wait repeats the ids or the job table).
  if (threadIdx.x < topk) {
    const int e = gemv_pair_id(p.ids, p.ids_bytes, t * topk + threadIdx.x, p.n);
    bool ea = p.w2_early != 0;
    if (!ea && e >= 0 && p.fetch_slot) {
      const int nm = __ldcg(p.nmiss);
      bool fetched = false;
      for (int jj = 0; jj < nm; ++jj) fetched |= __ldcg(p.fetch_slot + jj) == e;
      ea = !fetched;
    }
    s_e[threadIdx.x] = e;
    s_early[threadIdx.x] = ea ? 1 : 0;
    // the combine weights come from the router, which completed before the
    // allocator did, like the ids
    const int i = t * topk + threadIdx.x;
    s_w[threadIdx.x] = p.weights_f32 ? static_cast<const float*>(p.weights)[i]
                                     : __bfloat162float(
                                           static_cast<const __nv_bfloat16*>(p.weights)[i]);
  }
  __syncthreads();
  uint4 w0[kGemvPairGroup][CPL];
#pragma unroll
  for (int q = 0; q < kGemvPairGroup; ++q) {
    const int e = q < topk ? s_e[q] : -1;
    if (q < topk && s_early[q] && e >= 0 && j_first < H) {
      const uint4* wr = reinterpret_cast<const uint4*>(p.w2 + ((size_t)e * H + j_first) * I);
#pragma unroll
      for (int c = 0; c < CPL; ++c) w0[q][c] = __ldcg(wr + lane + 32 * c);
    }
  }
  // scales: entry (k, kb) of s_sc = s2[e_k][row block][kb] (this CTA's rows
  // all lie in one 128-row block), loaded early for early pairs
  const int rb = (blockIdx.x * rpw * kGemvRowsPerCta) / 128;
  auto stage_scales = [&](bool want_early) {
    for (int i = threadIdx.x; i < topk * nkbI; i += blockDim.x) {
      const int k = i / nkbI, kb = i - k * nkbI;
      const int e = s_e[k];
      if (e < 0) continue;
      if ((s_early[k] != 0) == want_early)
        s_sc[k][kb] = __ldcg(p.s2 + ((size_t)e * (H / 128) + rb) * nkbI + kb);
    }
  };
  stage_scales(true);
  // the residual this warp's first output row adds to (not written by this
  // call's earlier launches)
  float res0 = 0.f;
  if (p.accumulate && lane == 0 && j_first < H)
    res0 = __bfloat162float(p.out[(size_t)t * H + j_first]);
  // the shared expert's first down row too (bf16: two 16-byte words per chunk)
  uint4 sw0[CPL][2];
  if (p.sw13 && j_first < H) {
    const uint4* wr = reinterpret_cast<const uint4*>(p.sw2 + (size_t)j_first * I);
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      sw0[c][0] = __ldcg(wr + 2 * (lane + 32 * c));
      sw0[c][1] = __ldcg(wr + 2 * (lane + 32 * c) + 1);
    }
  }
  // L2 prefetch hints for what is read right after the wait -- this token's
  // h rows (and the shared expert's), and the first W2 row of every pair
  // whose slot the preceding launch fills.  A hint returns no data and L2 is
  // the point of coherence, so the loads after the wait still see that
  // launch's writes; the hints only take the DRAM and address-translation
  // latency out of the tail of the layer.
  {
    const int nrows = topk + (p.sw13 ? 1 : 0);
    const int hl = I * (int)sizeof(*p.h) / 128;   // 128-B lines per h row
    for (int i = threadIdx.x; i < nrows * hl; i += blockDim.x) {
      const int k = i / hl, l = i - k * hl;
      const char* src = reinterpret_cast<const char*>(
          k < topk ? p.h + (size_t)(t * topk + k) * I : p.hs + (size_t)t * I);
      prefetch_l2(src + (size_t)l * 128);
    }
    if (j_first < H) {   // this warp's output row, for every fetched pair
      const int wl = I / 128;
      for (int i = lane; i < topk * wl; i += 32) {
        const int k = i / wl, l = i - k * wl;
        if (!s_early[k] && s_e[k] >= 0)
          prefetch_l2(p.w2 + ((size_t)s_e[k] * H + j_first) * I + (size_t)l * 128);
      }
    }
  }
  pdl_wait();
  // the first group's remaining W2 rows and scales (slots the preceding launch
  // wrote), issued before the h staging so both latencies overlap
#pragma unroll
  for (int q = 0; q < kGemvPairGroup; ++q) {
    const int e = q < topk ? s_e[q] : -1;
    if (q < topk && !s_early[q] && e >= 0 && j_first < H) {
      const uint4* wr = reinterpret_cast<const uint4*>(p.w2 + ((size_t)e * H + j_first) * I);
#pragma unroll
      for (int c = 0; c < CPL; ++c) w0[q][c] = __ldcg(wr + lane + 32 * c);
    }
  }
  stage_scales(false);
  // stage the token's pair rows of h (written by the gate/up launch), and the
  // shared expert's row as row topk
  // (kHB loads per thread issued before the first store: one round trip for
  // a decode token's 8 pair rows + the shared expert's row)
  const int nrows = topk + (p.sw13 ? 1 : 0);
  const int n8 = nrows * (I / 8);   // 16-byte groups of 8 bf16
  constexpr int kHB = CPL == 1 ? 8 : 4;
  for (int base = 0; base < n8; base += kHB * kGemvThreads) {
    uint4 hv8[kHB];
#pragma unroll
    for (int u = 0; u < kHB; ++u) {
      const int i = base + u * kGemvThreads + (int)threadIdx.x;
      if (i < n8) {
        const int k = i / (I / 8), g8 = i - k * (I / 8);
        const __nv_bfloat16* src = k < topk ? p.h + (size_t)(t * topk + k) * I : p.hs + (size_t)t * I;
        hv8[u] = __ldcg(reinterpret_cast<const uint4*>(src) + g8);
      }
    }
#pragma unroll
    for (int u = 0; u < kHB; ++u) {
      const int i = base + u * kGemvThreads + (int)threadIdx.x;
      if (i < n8) {
        const int k = i / (I / 8), g8 = i - k * (I / 8);
        const uint32_t w4[4] = {hv8[u].x, hv8[u].y, hv8[u].z, hv8[u].w};
        float f[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          f[2 * q] = __uint_as_float(w4[q] << 16);
          f[2 * q + 1] = __uint_as_float(w4[q] & 0xffff0000u);
        }
        float* dst = s_h + k * row_stride + (g8 >> 1) * 20 + (g8 & 1) * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(f[4], f[5], f[6], f[7]);
      }
    }
  }
  const float sgate = (p.sw13 && p.sgate) ? __ldcg(p.gs + t) : 1.f;
  __syncthreads();
  // acc += w[t,k] * s2 * (W2[e_k][j] . h_k) over one group of pairs, k in order
  auto group = [&](const uint4 (&w)[kGemvPairGroup][CPL], int k0, float acc) {
#pragma unroll
    for (int q = 0; q < kGemvPairGroup; ++q) {
      const int k = k0 + q;
      const int e = k < topk ? s_e[k] : -1;
      if (e < 0) continue;
      float part = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int ch = lane + 32 * c;
        const float* hp = s_h + k * row_stride + ch * 20;
        float hv[16];
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float4 a = *reinterpret_cast<const float4*>(hp + 4 * f);
          hv[4 * f] = a.x; hv[4 * f + 1] = a.y; hv[4 * f + 2] = a.z; hv[4 * f + 3] = a.w;
        }
        part = fmaf(s_sc[k][ch >> 3], dot16_e4m3(w[q][c], hv), part);
      }
      acc = fmaf(s_w[k], part, acc);
    }
    return acc;
  };
  for (int r = 0; r < rpw; ++r) {
    const int j = j_first + r * kGemvRowsPerCta;
    if (j >= H) break;
    float acc = 0.f;
    for (int k0 = 0; k0 < topk; k0 += kGemvPairGroup) {
      if (r > 0 || k0 > 0) {  // the first group's rows are in w0 already
#pragma unroll
        for (int q = 0; q < kGemvPairGroup; ++q) {
          const int k = k0 + q;
          const int e = k < topk ? s_e[k] : -1;
          if (e >= 0) {
            const uint4* wr = reinterpret_cast<const uint4*>(p.w2 + ((size_t)e * H + j) * I);
#pragma unroll
            for (int c = 0; c < CPL; ++c) w0[q][c] = __ldcg(wr + lane + 32 * c);
          }
        }
      }
      acc = group(w0, k0, acc);
    }
    if (p.sw13) {  // shared expert: acc += sigmoid gate * (W2s[j] . hs[t])
      uint4 sw[CPL][2];
      if (r == 0) {
#pragma unroll
        for (int c = 0; c < CPL; ++c) { sw[c][0] = sw0[c][0]; sw[c][1] = sw0[c][1]; }
      } else {
        const uint4* wr = reinterpret_cast<const uint4*>(p.sw2 + (size_t)j * I);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          sw[c][0] = __ldcg(wr + 2 * (lane + 32 * c));
          sw[c][1] = __ldcg(wr + 2 * (lane + 32 * c) + 1);
        }
      }
      float part = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const float* hp = s_h + topk * row_stride + (lane + 32 * c) * 20;
        float hv[16];
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float4 a = *reinterpret_cast<const float4*>(hp + 4 * f);
          hv[4 * f] = a.x; hv[4 * f + 1] = a.y; hv[4 * f + 2] = a.z; hv[4 * f + 3] = a.w;
        }
        part += dot16_bf16(sw[c][0], sw[c][1], hv);
      }
      acc = fmaf(sgate, part, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      __nv_bfloat16* o = p.out + (size_t)t * H + j;
      if (p.accumulate) acc += r == 0 ? res0 : __bfloat162float(*o);
      *o = __float2bfloat16_rn(acc);
    }
  }
}

}  // namespace d3
