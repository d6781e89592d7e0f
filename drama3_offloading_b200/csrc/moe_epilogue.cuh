// Warp units of the work between and after the expert GEMMs, shared by the
// act and combine launches (moe.cu) and the activation quantisation:
//
//   quant_block    one 128-element block held 4 values per lane -> hi/lo
//                  e4m3 planes + one fp32 scale (x ~= s * (hi + lo)).
//   act unit       (sorted row, 128-wide block of I): sum the gate and up
//                  partials over the K splits in split order, SwiGLU,
//                  quantise h.
//   combine unit   (token, 128 output columns): out = bf16([out +] sum over
//                  the token's pairs k, in k order, of w[t,k] * (sum over the
//                  splits, in split order, of the down partials)).
// Fixed summation orders: results are bit-reproducible.  Partials are read
// through L2 (ld.global.cg): under programmatic launch the reading kernel's
// lifetime overlaps the GEMM that writes them.
#pragma once

#include "d3_common.cuh"

#include <cuda_bf16.h>
#include <cuda_fp8.h>

namespace d3 {

// hi/lo e4m3 planes of one 128-element block held 4 per lane: returns scale.
__device__ __forceinline__ float quant_block(const float (&v)[4], uint32_t& hi4, uint32_t& lo4) {
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? 448.f / amax : 0.f;
  hi4 = 0; lo4 = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float y = v[q] * inv;
    const __nv_fp8_storage_t h = __nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
    const float hf = __half2float(__nv_cvt_fp8_to_halfraw(h, __NV_E4M3));
    const __nv_fp8_storage_t l = __nv_cvt_float_to_fp8(y - hf, __NV_SATFINITE, __NV_E4M3);
    hi4 |= (uint32_t)h << (8 * q);
    lo4 |= (uint32_t)l << (8 * q);
  }
  return amax > 0.f ? amax / 448.f : 0.f;
}

// ws1: [split][P][2I] fp32 partials (gate columns [0, I), up [I, 2I)).
__device__ __forceinline__ void act_unit(const float* ws1, int split, int P, int row, int kb,
                                         int I, uint8_t* hq, float* hs, int lane) {
  float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < split; ++s) {
    const float* r = ws1 + ((size_t)s * P + row) * 2 * I + kb * 128 + lane * 4;
    const float4 a = __ldcg(reinterpret_cast<const float4*>(r));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(r + I));
    g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w;
    u[0] += b.x; u[1] += b.y; u[2] += b.z; u[3] += b.w;
  }
  float h[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) h[q] = g[q] / (1.f + expf(-g[q])) * u[q];
  uint32_t hi4, lo4;
  const float s = quant_block(h, hi4, lo4);
  uint8_t* qrow = hq + (size_t)row * 2 * I;
  *reinterpret_cast<uint32_t*>(qrow + kb * 128 + lane * 4) = hi4;
  *reinterpret_cast<uint32_t*>(qrow + I + kb * 128 + lane * 4) = lo4;
  if (lane == 0) hs[(size_t)row * (I / 128) + kb] = s;
}

// ws2: [split][P][H] fp32 partials; inv[t*topk+k] = sorted row of pair (t,k)
// or -1; columns [j0, j0 + 128) of token t into out_row (token t's output row,
// local or a peer's).
__device__ __forceinline__ void combine_unit(const float* ws2, int split, int P, int H,
                                             const int* inv, const void* weights, int weights_f32,
                                             int t, int topk, int accumulate,
                                             __nv_bfloat16* out_row, int j0, int lane) {
  const int j = j0 + lane * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (accumulate) {
    const uint2 raw = *reinterpret_cast<const uint2*>(out_row + j);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = __bfloat162float(b[q]);
  }
  for (int k = 0; k < topk; ++k) {
    const int pos = __ldcg(inv + t * topk + k);
    if (pos < 0) continue;
    const float wk = weights_f32 ? static_cast<const float*>(weights)[t * topk + k]
                                 : __bfloat162float(
                                       static_cast<const __nv_bfloat16*>(weights)[t * topk + k]);
    float y[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < split; ++s) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(ws2 + ((size_t)s * P + pos) * H + j));
      y[0] += a.x; y[1] += a.y; y[2] += a.z; y[3] += a.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = fmaf(wk, y[q], acc[q]);
  }
  __nv_bfloat16 o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = __float2bfloat16_rn(acc[q]);
  *reinterpret_cast<uint2*>(out_row + j) = *reinterpret_cast<uint2*>(o);
}

}  // namespace d3
