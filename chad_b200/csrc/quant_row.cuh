// Affine quantization of one cache row by one warp (MLX's affine quantize, as mlx-lm's
// QuantizedKVCache applies it before the reference's attention, tests/test_mlx_qsdpa.py:45-49):
// the 64-value groups reduce min/max with warp shuffles and every lane packs its own codes.
// The arithmetic is float32 IEEE (no fast-math): max/min, (max-min)/(2^bits-1) clamped to
// 1e-7, sign and edge from the larger-magnitude end, q0 = rint(edge/scale), then
// scale = edge/q0 and bias = edge unless q0 == 0, codes = clamp(rint((x-bias)/scale)).
// Shared by the append kernel and the decode kernel's fused append, so both write the same
// bits.
#pragma once
#include "qkv_common.cuh"

namespace qkv {

template <typename TIn>
__device__ __forceinline__ float load_as_f32(const TIn* p);
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half* p) { return __half2float(*p); }

// One warp: src_row (D values) -> codes wrow (D*BITS/32 words), srow/brow (D/64 each).
template <typename TIn, typename TS, int BITS, int D>
__device__ __forceinline__ void quantize_row_warp(const TIn* __restrict__ src_row,
                                                  uint32_t* __restrict__ wrow,
                                                  TS* __restrict__ srow, TS* __restrict__ brow,
                                                  int lane) {
  constexpr int E = D / 32;
  constexpr int LPG = 64 / E;  // lanes per group
  float v[E];
  const TIn* src = src_row + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = load_as_f32<TIn>(src + e);

  float mx = v[0], mn = v[0];
#pragma unroll
  for (int e = 1; e < E; ++e) {
    mx = fmaxf(mx, v[e]);
    mn = fminf(mn, v[e]);
  }
#pragma unroll
  for (int o = 1; o < LPG; o <<= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  const float n_bins = float((1 << BITS) - 1);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), n_bins), 1e-7f);
  const bool side = fabsf(mn) > fabsf(mx);
  scale = side ? scale : -scale;
  const float edge = side ? mn : mx;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }

  // pack this lane's E codes at bit offset (lane*E*BITS) % 32 of word (lane*E*BITS)/32
  uint32_t part[(E * BITS + 31) / 32];
#pragma unroll
  for (int i = 0; i < (E * BITS + 31) / 32; ++i) part[i] = 0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float c = rintf(__fdiv_rn(__fsub_rn(v[e], bias), scale));
    c = fminf(fmaxf(c, 0.0f), n_bins);
    const int bit = e * BITS;
    part[bit / 32] |= uint32_t(c) << (bit % 32);
  }
  if constexpr (E * BITS >= 32) {
#pragma unroll
    for (int i = 0; i < E * BITS / 32; ++i) wrow[lane * (E * BITS / 32) + i] = part[i];
  } else {
    // several lanes share one word: OR their disjoint bit fields together
    constexpr int LPW = 32 / (E * BITS);
    uint32_t word = part[0] << ((lane % LPW) * E * BITS);
#pragma unroll
    for (int o = 1; o < LPW; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
    if (lane % LPW == 0) wrow[lane / LPW] = word;
  }
  if (lane % LPG == 0) {
    const int grp = lane / LPG;
    srow[grp] = Elem<TS>::from_f32(scale);
    brow[grp] = Elem<TS>::from_f32(bias);
  }
}

}  // namespace qkv
