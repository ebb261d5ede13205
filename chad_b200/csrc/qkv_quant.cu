// Affine quantize-on-append and dequantize for the MLX-layout KV cache (sm_100a).
//
// quantize: one warp per row of D values; the 64-value groups reduce min/max with warp
// shuffles and every lane packs its own codes, so a row is read once and written once.
// The arithmetic is float32 IEEE (no fast-math): max/min, (max-min)/(2^bits-1) clamped to
// 1e-7, sign and edge from the larger-magnitude end, q0 = rint(edge/scale), then
// scale = edge/q0 and bias = edge unless q0 == 0, codes = clamp(rint((x-bias)/scale)).
// This is MLX's affine quantization as mlx-lm's QuantizedKVCache applies it before the
// reference's attention (tests/test_mlx_qsdpa.py:45-49).
#include "qkv_common.cuh"
#include "qkv_internal.h"
#include "quant_row.cuh"

namespace qkv {

// One tensor to quantize-append: rows of x into (w, scales, biases).
template <typename TIn, typename TS>
struct QuantJob {
  const TIn* x;
  uint32_t* w;
  TS* scales;
  TS* biases;
};

// E = D/32 values per lane (2, 4 or 8); group of 64 = 64/E lanes. blockIdx.y picks the job
// (K and V of one append share a launch).
template <typename TIn, typename TS, int BITS, int D>
__global__ void __launch_bounds__(128) quantize_rows_kernel(QuantJob<TIn, TS> j0,
                                                            QuantJob<TIn, TS> j1, int H, int S,
                                                            int NP, int offset, long long n_rows) {
  // Programmatic dependent launch: the attention kernel that follows may start streaming
  // the older cache positions while this one runs; x is read only after the kernel that
  // produced it is done.
  asm volatile("griddepcontrol.launch_dependents;");
  constexpr int WPR = D * BITS / 32;
  const QuantJob<TIn, TS>& job = blockIdx.y ? j1 : j0;
  const TIn* __restrict__ x = job.x;
  uint32_t* __restrict__ w = job.w;
  TS* __restrict__ scales = job.scales;
  TS* __restrict__ biases = job.biases;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (row >= n_rows) return;
  // row = ((b*H + h)*S + s); destination position offset + s of the (b,h) slab
  const long long bh = row / S;
  const int s = (int)(row - bh * S);
  const long long drow = bh * NP + offset + s;

  quantize_row_warp<TIn, TS, BITS, D>(x + row * D, w + drow * WPR, scales + drow * (D / 64),
                                      biases + drow * (D / 64), lane);
}

// One thread per packed word: 32/BITS outputs.
template <typename TS, int BITS>
__global__ void dequantize_kernel(const uint32_t* __restrict__ w, const TS* __restrict__ scales,
                                  const TS* __restrict__ biases, TS* __restrict__ out,
                                  long long n_words, int words_per_row, int groups_per_row,
                                  int round_mode) {
  constexpr int PER = 32 / BITS;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  const long long row = i / words_per_row;
  const int wi = (int)(i - row * words_per_row);
  const int grp = wi * PER / 64;
  const float s = Elem<TS>::to_f32(scales[row * groups_per_row + grp]);
  const float b = Elem<TS>::to_f32(biases[row * groups_per_row + grp]);
  const uint32_t word = w[i];
  TS vals[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const float c = float((word >> (e * BITS)) & ((1u << BITS) - 1));
    if (round_mode == 0) {
      vals[e] = Elem<TS>::from_f32(__fmaf_rn(s, c, b));
    } else {
      const float m = Elem<TS>::to_f32(Elem<TS>::from_f32(__fmul_rn(s, c)));
      vals[e] = Elem<TS>::from_f32(__fadd_rn(m, b));
    }
  }
  TS* dst = out + i * PER;
#pragma unroll
  for (int e = 0; e < PER; ++e) dst[e] = vals[e];
}

template <typename TIn, typename TS, int BITS>
static int launch_quantize_d(const void* const* x, void* const* w, void* const* sc,
                             void* const* bi, int jobs, int B, int H, int S, int D, int NP,
                             int offset, cudaStream_t st) {
  const long long rows = (long long)B * H * S;
  const int warps = 4;
  QuantJob<TIn, TS> j[2];
  for (int i = 0; i < 2; ++i) {
    const int k = i < jobs ? i : 0;
    j[i] = QuantJob<TIn, TS>{(const TIn*)x[k], (uint32_t*)w[k], (TS*)sc[k], (TS*)bi[k]};
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rows + warps - 1) / warps), (unsigned)jobs, 1);
  cfg.blockDim = dim3(warps * 32, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  switch (D) {
    case 64:
      e = cudaLaunchKernelEx(&cfg, quantize_rows_kernel<TIn, TS, BITS, 64>, j[0], j[1], H, S, NP, offset, rows);
      break;
    case 128:
      e = cudaLaunchKernelEx(&cfg, quantize_rows_kernel<TIn, TS, BITS, 128>, j[0], j[1], H, S, NP, offset, rows);
      break;
    case 256:
      e = cudaLaunchKernelEx(&cfg, quantize_rows_kernel<TIn, TS, BITS, 256>, j[0], j[1], H, S, NP, offset, rows);
      break;
    default:
      return QKV_EUNSUPPORTED;
  }
  return e == cudaSuccess ? QKV_OK : QKV_ECUDA;
}

template <typename TIn, typename TS>
static int launch_quantize_b(const void* const* x, void* const* w, void* const* sc,
                             void* const* bi, int jobs, int B, int H, int S, int D, int NP,
                             int offset, int bits, cudaStream_t st) {
  if (bits == 4)
    return launch_quantize_d<TIn, TS, 4>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, st);
  return launch_quantize_d<TIn, TS, 8>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, st);
}

int launch_quantize_jobs(const void* const* x, int x_dtype, void* const* w, void* const* sc,
                         void* const* bi, int jobs, int B, int H, int S, int D, int NP,
                         int offset, int bits, int scale_dtype, cudaStream_t st) {
  if (B * (long long)H * S == 0) return QKV_OK;
  if (jobs < 1 || jobs > 2) return QKV_EINVAL;
  if (scale_dtype == QKV_BF16) {
    if (x_dtype == QKV_BF16)
      return launch_quantize_b<__nv_bfloat16, __nv_bfloat16>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
    if (x_dtype == QKV_F16)
      return launch_quantize_b<__half, __nv_bfloat16>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
    return launch_quantize_b<float, __nv_bfloat16>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
  }
  if (x_dtype == QKV_BF16)
    return launch_quantize_b<__nv_bfloat16, __half>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
  if (x_dtype == QKV_F16)
    return launch_quantize_b<__half, __half>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
  return launch_quantize_b<float, __half>(x, w, sc, bi, jobs, B, H, S, D, NP, offset, bits, st);
}

int launch_quantize(const void* x, int x_dtype, void* w, void* sc, void* bi, int B, int H,
                    int S, int D, int NP, int offset, int bits, int scale_dtype,
                    cudaStream_t st) {
  return launch_quantize_jobs(&x, x_dtype, &w, &sc, &bi, 1, B, H, S, D, NP, offset, bits,
                              scale_dtype, st);
}

int launch_dequantize(const void* w, const void* sc, const void* bi, void* out, long long rows,
                      int D, int bits, int dtype, int round_mode, cudaStream_t st) {
  const int wpr = D * bits / 32;
  const long long n_words = rows * wpr;
  if (n_words == 0) return QKV_OK;
  const int threads = 256;
  const unsigned grid = (unsigned)((n_words + threads - 1) / threads);
  if (dtype == QKV_BF16) {
    if (bits == 4)
      dequantize_kernel<__nv_bfloat16, 4><<<grid, threads, 0, st>>>(
          (const uint32_t*)w, (const __nv_bfloat16*)sc, (const __nv_bfloat16*)bi,
          (__nv_bfloat16*)out, n_words, wpr, D / 64, round_mode);
    else
      dequantize_kernel<__nv_bfloat16, 8><<<grid, threads, 0, st>>>(
          (const uint32_t*)w, (const __nv_bfloat16*)sc, (const __nv_bfloat16*)bi,
          (__nv_bfloat16*)out, n_words, wpr, D / 64, round_mode);
  } else {
    if (bits == 4)
      dequantize_kernel<__half, 4><<<grid, threads, 0, st>>>(
          (const uint32_t*)w, (const __half*)sc, (const __half*)bi, (__half*)out, n_words, wpr,
          D / 64, round_mode);
    else
      dequantize_kernel<__half, 8><<<grid, threads, 0, st>>>(
          (const uint32_t*)w, (const __half*)sc, (const __half*)bi, (__half*)out, n_words, wpr,
          D / 64, round_mode);
  }
  return QKV_OK;
}

}  // namespace qkv
