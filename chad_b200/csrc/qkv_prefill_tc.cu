// Tensor-core attention for many query tokens over the affine-quantized KV cache (sm_100a).
//
// Semantics follow the reference's multi-token branch (src/chad/mlx_qsdpa.py:751-766): the
// cache is dequantized to the query dtype (mx.dequantize) and attended with a causal or no
// mask (mx.fast.scaled_dot_product_attention). Here the dequantization happens tile by tile
// in shared memory and never reaches HBM:
//
//   * CTA = up to two 128-row MMA tiles of query rows of ONE kv head: row r of a tile is
//     (q head r / TT of the GQA group, token r % TT), TT = 128 / GQA; every row of the CTA
//     shares each dequantized K/V tile.
//   * Warp roles (14 warps): 0 TMA producer (packed codes, scales, biases), 1 tensor-memory
//     owner and single-thread MMA issuer, 2-3 and 12-13 dequantizers (codes -> 16-bit K/V
//     tiles in the 128-byte-swizzled operand layout), 4-7 / 8-11 softmax of tile 0 / 1.
//   * Per 64-key tile j: S_m = Q_m K^T (tcgen05, K-major operands) into tensor memory;
//     softmax threads own one S row each (no cross-thread reductions), write P (16-bit)
//     back over S and the MMA warp accumulates O_m += P_m V with P read from tensor memory
//     and V as an MN-major operand. S is double-buffered so QK(j+1) overlaps softmax(j).
//   * The running max is only raised when it grows by more than 2^8 (log2 units), so the
//     O rescale in tensor memory is rare; P values stay <= 256.
//
// Dequantized K/V values are round(code * scale + bias) in the 16-bit type with a single
// rounding (fused multiply-add), the value mx.dequantize returns up to the rare case where
// rounding the fp32 fma first lands on a 16-bit tie.
// For 4-bit codes each group of 8 head dims is stored in the order (0,4,1,5,2,6,3,7); Q is
// permuted the same way when it is staged and O is un-permuted when it is stored.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "../../include/qkv.h"
#include "qkv_common.cuh"
#include "qkv_internal.h"
#include "tc_common.cuh"

namespace qkv {

namespace {

constexpr int kD = 128;
constexpr int kKT = 64;          // keys per tile (MMA N of Q K^T)
constexpr int kWarpsTc = 14;
constexpr int kThreadsTc = kWarpsTc * 32;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kPolyEvery = 0;  // > 0: one exp2 in kPolyEvery on the FMA pipe, not the MUFU
#define kNegInfTc (-__int_as_float(0x7f800000))

template <int BITS>
struct TcGeo {
  static constexpr int RB = kD * BITS / 8;       // code bytes per key
  static constexpr int CODE = kKT * RB;          // one code tile
  static constexpr int SC = kKT * 2 * 2;         // one scale / bias array (2 groups, 16-bit)
  static constexpr int STAGE = 2 * CODE + 4 * SC;  // multiple of 1024
  static constexpr int NST = BITS == 4 ? 4 : 3;
};

constexpr int kKvBufs = 3;  // dequantized K/V tile buffers: dequant runs up to 2 tiles ahead

template <int BITS, int MT>
struct TcSmem {
  static constexpr int Q = 0;                       // MT x (2 halves x 128 rows x 128 B)
  static constexpr int KD = MT * 32768;             // kKvBufs x (2 halves x 64 keys x 128 B)
  static constexpr int VD = KD + kKvBufs * 16384;   // same layout (MN-major V)
  static constexpr int RING = VD + kKvBufs * 16384;
  static constexpr int BYTES = RING + TcGeo<BITS>::NST * TcGeo<BITS>::STAGE;
};

struct TcParams {
  AttnArgs a;
  CUtensorMap tmk, tmv;
  int TT;        // tokens per 128-row tile
  int chunk;     // keys per split
  float* parts;  // [splits][B*HQ*S][D+4] or nullptr (direct normalized output)
};

template <typename T>
struct Pack16;
template <>
struct Pack16<__nv_bfloat16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // 128.0 in both halves
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
  }
  static __device__ __forceinline__ float lo(uint32_t v) { return __uint_as_float(v << 16); }
  static __device__ __forceinline__ float hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
};
template <>
struct Pack16<__half> {
  static constexpr uint32_t kMagic = 0x64006400u;  // 1024.0 in both halves
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
  }
  static __device__ __forceinline__ float lo(uint32_t v) {
    return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu)));
  }
  static __device__ __forceinline__ float hi(uint32_t v) {
    return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
  }
};

// 2^t on the FMA/ALU pipes: t = n + f with n = rint(t), |f| <= 1/2; 2^f from a degree-3
// polynomial fitted here to relative error 8e-5 over [-1/2, 1/2] (far below the 16-bit P it
// feeds), 2^n added to the exponent bits. t is clamped at -126: 2^-126 stands in for 0.
__device__ __forceinline__ float exp2_poly(float t) {
  t = fmaxf(t, -126.0f);
  const float j = t + 12582912.0f;        // 1.5 * 2^23: low mantissa bits hold rint(t)
  const float f = t - (j - 12582912.0f);
  const float p = fmaf(fmaf(fmaf(0.05518098f, f, 0.24263459f), f, 0.69326133f), f, 0.99992621f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
}

// code (exact, in T) pair -> round(code * s + b), one rounding, both halves
template <typename T>
__device__ __forceinline__ uint32_t deq_pair(uint32_t c, uint32_t s2, uint32_t b2) {
  return Pack16<T>::fma(c, s2, b2);
}

// Dequantizes the 128 codes of one key row (words = its packed code words) and writes each
// 16-byte chunk of 8 head dims to its slot in the swizzled operand tile `dst`.
template <typename T, int BITS>
__device__ __forceinline__ void dequant_row(const uint32_t* words, uint32_t s0, uint32_t s1,
                                            uint32_t b0, uint32_t b1, uint8_t* dst, int row) {
  using P = Pack16<T>;
  if constexpr (BITS == 4) {
    const uint32_t magic = P::kMagic;
#pragma unroll
    for (int i = 0; i < 16; ++i) {  // word i = head dims 8i .. 8i+7
      const uint32_t w = words[i];
      const uint32_t s2 = i < 8 ? s0 : s1, b2 = i < 8 ? b0 : b1;
      uint4 o;
      o.x = deq_pair<T>(P::sub(and_or(w, 0x000F000Fu, magic), magic), s2, b2);        // (0,4)
      o.y = deq_pair<T>(P::sub(and_or(w >> 4, 0x000F000Fu, magic), magic), s2, b2);   // (1,5)
      o.z = deq_pair<T>(P::sub(and_or(w >> 8, 0x000F000Fu, magic), magic), s2, b2);   // (2,6)
      o.w = deq_pair<T>(P::sub(and_or(w >> 12, 0x000F000Fu, magic), magic), s2, b2);  // (3,7)
      const int h = i >> 3, c = (i & 7) ^ (row & 7);
      *reinterpret_cast<uint4*>(dst + h * 8192 + row * 128 + c * 16) = o;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {  // words 2i, 2i+1 = head dims 8i .. 8i+7
      const uint32_t s2 = i < 8 ? s0 : s1, b2 = i < 8 ? b0 : b1;
      uint32_t c[4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t w = words[2 * i + u];
        if constexpr (std::is_same<T, __half>::value) {
          c[2 * u] = P::sub(prmt(w, 0x64646464u, 0x4140), P::kMagic);
          c[2 * u + 1] = P::sub(prmt(w, 0x64646464u, 0x4342), P::kMagic);
        } else {
          // bf16 holds 0..255 exactly; build it through fp32 (2^23 + code) - 2^23
          const float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7540)) - 8388608.0f;
          const float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7541)) - 8388608.0f;
          const float f2 = __uint_as_float(prmt(w, 0x4B000000u, 0x7542)) - 8388608.0f;
          const float f3 = __uint_as_float(prmt(w, 0x4B000000u, 0x7543)) - 8388608.0f;
          c[2 * u] = prmt(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
          c[2 * u + 1] = prmt(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
        }
      }
      uint4 o;
      o.x = deq_pair<T>(c[0], s2, b2);
      o.y = deq_pair<T>(c[1], s2, b2);
      o.z = deq_pair<T>(c[2], s2, b2);
      o.w = deq_pair<T>(c[3], s2, b2);
      const int h = i >> 3, cc = (i & 7) ^ (row & 7);
      *reinterpret_cast<uint4*>(dst + h * 8192 + row * 128 + cc * 16) = o;
    }
  }
}

__device__ __forceinline__ void tma_load_3d_tc(void* dst, const CUtensorMap* map, int x, int y,
                                               int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

template <typename T, int BITS, int MT>
__global__ void __launch_bounds__(kThreadsTc, 1) prefill_tc_kernel(const __grid_constant__ TcParams P) {
  using GE = TcGeo<BITS>;
  using SM = TcSmem<BITS, MT>;
  using PK = Pack16<T>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t code_full[GE::NST], code_empty[GE::NST];
  __shared__ uint64_t kv_full[kKvBufs], kv_empty[kKvBufs];
  __shared__ uint64_t s_full[MT][2], p_full[MT][2], o_done[MT];
  __shared__ uint64_t mma_fin;
  __shared__ uint32_t tmem_sh;

  const AttnArgs& a = P.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TT = P.TT;
  const int gqa = a.HQ / a.HKV;
  const int bh = blockIdx.y;  // b * HKV + hkv
  const int b = bh / a.HKV, hkv = bh % a.HKV;
  const int t0 = blockIdx.x * (MT * TT);
  const int split = blockIdx.z;
  const int n = min(max(a.n, 0), a.NP);
  const bool causal = a.mask_kind == QKV_MASK_CAUSAL;
  // key range of this CTA: [k_begin, k_stop); every row sees at most keys < k_stop
  const int k_begin = split * P.chunk;
  const int t_last = min(t0 + MT * TT, a.S) - 1;
  const int lim_hi = causal ? n - a.S + t_last : n - 1;  // last key any row may see
  const int k_stop = min(min(k_begin + P.chunk, n), lim_hi + 1);
  const int ntiles = k_stop > k_begin ? (k_stop - k_begin + kKT - 1) / kKT : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GE::NST; ++s) {
      mbar_init(&code_full[s], 1);
      mbar_init(&code_empty[s], 4);
    }
    for (int s = 0; s < kKvBufs; ++s) {
      mbar_init(&kv_full[s], 4);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      for (int m = 0; m < MT; ++m) {
        mbar_init(&s_full[m][s], 1);
        mbar_init(&p_full[m][s], 4);
      }
    }
    for (int m = 0; m < MT; ++m) mbar_init(&o_done[m], 1);
    mbar_init(&mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&tmem_sh, 512);
    tc::tmem_relinquish();
  }
  // ---- stage Q (all threads): MT tiles x 128 rows x 16 chunks of 8 head dims -------------
  {
    const T* q = reinterpret_cast<const T*>(a.q);
    for (int i = threadIdx.x; i < MT * 128 * 16; i += kThreadsTc) {
      const int m = i / (128 * 16), r = (i / 16) % 128, c = i % 16;
      const int hl = r / TT, t = t0 + m * TT + (r % TT);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (hl < gqa && t < a.S) {
        const long long row = ((long long)b * a.HQ + hkv * gqa + hl) * a.S + t;
        v = *reinterpret_cast<const uint4*>(q + row * kD + c * 8);
        if constexpr (BITS == 4) {  // (0,1)(2,3)(4,5)(6,7) -> (0,4)(1,5)(2,6)(3,7)
          const uint4 u = v;
          v.x = prmt(u.x, u.z, 0x5410);
          v.y = prmt(u.x, u.z, 0x7632);
          v.z = prmt(u.y, u.w, 0x5410);
          v.w = prmt(u.y, u.w, 0x7632);
        }
      }
      const int h = c >> 3, cc = (c & 7) ^ (r & 7);
      *reinterpret_cast<uint4*>(smem + SM::Q + m * 32768 + h * 16384 + r * 128 + cc * 16) = v;
    }
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_sh;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j % GE::NST;
        if (j >= GE::NST) ok = mbar_wait(&code_empty[st], ((j / GE::NST) + 1) & 1, a.status, 40);
        if (!ok) break;
        const int p0 = k_begin + j * kKT;
        const int rows = min(kKT, a.NP - p0);
        const uint32_t sb = rows * 2 * 2;
        uint8_t* sp = smem + SM::RING + st * GE::STAGE;
        mbar_arrive_expect_tx(&code_full[st], 2 * GE::CODE + 4 * sb);
        tma_load_3d_tc(sp, &P.tmk, 0, p0, bh, &code_full[st]);
        tma_load_3d_tc(sp + GE::CODE, &P.tmv, 0, p0, bh, &code_full[st]);
        const long long so = ((long long)bh * a.NP + p0) * 2 * 2;
        bulk_g2s(sp + 2 * GE::CODE, (const uint8_t*)a.ks + so, sb, &code_full[st]);
        bulk_g2s(sp + 2 * GE::CODE + GE::SC, (const uint8_t*)a.kb + so, sb, &code_full[st]);
        bulk_g2s(sp + 2 * GE::CODE + 2 * GE::SC, (const uint8_t*)a.vs + so, sb, &code_full[st]);
        bulk_g2s(sp + 2 * GE::CODE + 3 * GE::SC, (const uint8_t*)a.vb + so, sb, &code_full[st]);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_f16(kBf16, 128, kKT, false, false);
      constexpr uint32_t id_o = tc::idesc_f16(kBf16, 128, kD, false, true);
      const uint32_t q_base = smem_u32(smem + SM::Q);
      const uint32_t kd_base = smem_u32(smem + SM::KD);
      const uint32_t vd_base = smem_u32(smem + SM::VD);
      auto issue_pv = [&](int jj) {
        const int pb = jj & 1;            // S / P buffer
        const int vb = jj % kKvBufs;      // V buffer
        for (int m = 0; m < MT && ok; ++m) {
          ok = mbar_wait(&p_full[m][pb], (jj >> 1) & 1, a.status, 41);
          if (!ok) break;
          tc::fence_after_sync();
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint64_t bd = tc::sdesc_sw128(vd_base + vb * 16384 + s * 2048, 8192, 1024);
            tc::mma_ts(tmem + 256 + m * 128, tmem + m * 128 + pb * 64 + s * 8, bd, id_o,
                       (jj > 0 || s > 0) ? 1u : 0u);
          }
          tc::mma_commit(&o_done[m]);
        }
        tc::mma_commit(&kv_empty[vb]);
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int buf = j % kKvBufs, sb = j & 1;
        ok = mbar_wait(&kv_full[buf], (j / kKvBufs) & 1, a.status, 42);
        if (!ok) break;
        tc::fence_after_sync();
        for (int m = 0; m < MT; ++m) {
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const uint64_t ad =
                tc::sdesc_sw128(q_base + m * 32768 + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
            const uint64_t bd =
                tc::sdesc_sw128(kd_base + buf * 16384 + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024);
            tc::mma_ss(tmem + m * 128 + sb * 64, ad, bd, id_s, s > 0 ? 1u : 0u);
          }
          tc::mma_commit(&s_full[m][sb]);
        }
        if (j > 0) issue_pv(j - 1);
      }
      if (ok && ntiles > 0) issue_pv(ntiles - 1);
      tc::mma_commit(&mma_fin);
      mbar_wait(&mma_fin, 0, a.status, 43);
    }
  } else if (warp >= 4 && warp < 4 + 4 * MT) {
    // ---------------------------------------------------------------- softmax
    const int m = (warp - 4) >> 2;
    const int r = (warp & 3) * 32 + lane;  // tensor-memory lane = row of tile m
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int hl = r / TT, t = t0 + m * TT + (r % TT);
    const bool row_ok = hl < gqa && t < a.S;
    int lim = causal ? n - a.S + t : n - 1;
    lim = min(lim, k_stop - 1);
    const float c = a.scale * 1.4426950408889634f;
    float m_run = kNegInfTc, l_run = 0.f;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      ok = mbar_wait(&s_full[m][sb], (j >> 1) & 1, a.status, 44);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::fence_after_sync();
      const uint32_t ts = tmem + lane_off + m * 128 + sb * 64;
      uint32_t x[32], y[32];
      tc::ld32(ts, x);
      tc::ld32(ts + 32, y);
      tc::wait_ld();
      const int kbase = k_begin + j * kKT;
      if (kbase + kKT - 1 > lim) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (kbase + i > lim) x[i] = __float_as_uint(kNegInfTc);
          if (kbase + 32 + i > lim) y[i] = __float_as_uint(kNegInfTc);
        }
      }
      // row max: eight independent chains, then a tree
      float mxa[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxa[i] = fmaxf(__uint_as_float(x[i]), __uint_as_float(y[i]));
#pragma unroll
      for (int i = 8; i < 32; ++i)
        mxa[i & 7] = fmaxf(mxa[i & 7], fmaxf(__uint_as_float(x[i]), __uint_as_float(y[i])));
      const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                             fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
      const float m_cand = mx * c;
      float alpha = 1.f;
      const bool resc = m_cand > m_run + kRescaleLog2;  // false while the tile is all masked
      if (resc) {
        alpha = ex2(m_run - m_cand);
        m_run = m_cand;
      }
      const float mu = m_run == kNegInfTc ? 0.f : m_run;
      // p = 2^(s*c - mu) on the MUFU (or, with kPolyEvery > 0, partly by the polynomial)
      float sa[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint32_t* src = i < 16 ? x : y;
        const int e = (i & 15) * 2;
        const float t0 = fmaf(__uint_as_float(src[e]), c, -mu);
        const float t1 = fmaf(__uint_as_float(src[e + 1]), c, -mu);
        const float p0 = (kPolyEvery > 0 && (2 * i) % kPolyEvery == kPolyEvery - 1) ? exp2_poly(t0) : ex2(t0);
        const float p1 = (kPolyEvery > 0 && (2 * i + 1) % kPolyEvery == kPolyEvery - 1) ? exp2_poly(t1) : ex2(t1);
        sa[(2 * i) & 3] += p0;
        sa[(2 * i + 1) & 3] += p1;
        pk[i] = PK::pack(p0, p1);
      }
      const float sum = (sa[0] + sa[1]) + (sa[2] + sa[3]);
      l_run = fmaf(l_run, alpha, sum);
      tc::st32(ts, pk);  // P (16-bit pairs) over the first 32 columns of S
      tc::wait_st();
      if (j > 0) {
        // Wait for PV(j-1) on every tile: a parity wait only tells phases apart while the
        // barrier is at most one phase ahead of this thread's view of it, and a rescale
        // needs O out of flight anyway. PV(j-1) normally finished during this softmax.
        ok = mbar_wait(&o_done[m], (j - 1) & 1, a.status, 45);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        // scale this row of O in place (PV(j) is not issued before p_full below)
        tc::fence_after_sync();
        const uint32_t to = tmem + lane_off + 256 + m * 128;
#pragma unroll 1
        for (int qd = 0; qd < 4; ++qd) {
          tc::ld32(to + qd * 32, x);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = __float_as_uint(__uint_as_float(x[i]) * alpha);
          tc::st32(to + qd * 32, x);
        }
        tc::wait_st();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[m][sb]);
    }
    // ---- epilogue: O row -> output (normalized) or partial row ---------------------------
    if (ok && ntiles > 0) {
      ok = mbar_wait(&o_done[m], (ntiles - 1) & 1, a.status, 46);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc::fence_after_sync();
      const uint32_t to = tmem + lane_off + 256 + m * 128;
      const long long row = ((long long)b * a.HQ + hkv * gqa + hl) * a.S + t;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
      for (int qd = 0; qd < 4; ++qd) {
        uint32_t x[32];
        if (ntiles > 0) {
          tc::ld32(to + qd * 32, x);
          tc::wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = 0u;
        }
        // column position p of 8-dim group holds dim perm[p] (4-bit) or p (8-bit)
        float o[32];
#pragma unroll
        for (int g = 0; g < 4; ++g)
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int d = BITS == 4 ? ((p & 1) ? 4 + (p >> 1) : (p >> 1)) : p;
            o[g * 8 + d] = __uint_as_float(x[g * 8 + p]);
          }
        if (row_ok) {
          if (P.parts) {
            float* dst = P.parts + ((long long)split * a.B * a.HQ * a.S + row) * (kD + 4) + qd * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
          } else {
            uint32_t* dst = reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(a.out) + row * kD + qd * 32);
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(dst + i / 2) =
                  make_uint4(PK::pack(o[i] * inv, o[i + 1] * inv), PK::pack(o[i + 2] * inv, o[i + 3] * inv),
                             PK::pack(o[i + 4] * inv, o[i + 5] * inv), PK::pack(o[i + 6] * inv, o[i + 7] * inv));
          }
        }
      }
      if (row_ok && P.parts) {
        float* dst = P.parts + ((long long)split * a.B * a.HQ * a.S + row) * (kD + 4) + kD;
        *reinterpret_cast<float4*>(dst) = make_float4(m_run, l_run, 0.f, 0.f);
      }
    }
  } else if (warp == 2 || warp == 3 || warp == 12 || warp == 13) {
    // ---------------------------------------------------------------- dequantizers
    const int dq = (warp < 4 ? warp - 2 : warp - 10) * 32 + lane;  // 0..127
    const bool is_v = dq >= 64;
    const int row = dq & 63;
    uint8_t* dst_base = smem + (is_v ? SM::VD : SM::KD);
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % GE::NST, buf = j % kKvBufs;
      ok = mbar_wait(&code_full[st], (j / GE::NST) & 1, a.status, 47);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint8_t* sp = smem + SM::RING + st * GE::STAGE;
      const uint8_t* cp = sp + (is_v ? GE::CODE : 0);
      uint32_t words[GE::RB / 4];
#pragma unroll
      for (int ch = 0; ch < GE::RB / 16; ++ch) {
        const int sw = BITS == 4 ? ((ch ^ ((row >> 1) & 3)) & 3) : (ch ^ (row & 7));
        const uint4 v = *reinterpret_cast<const uint4*>(cp + row * GE::RB + sw * 16);
        words[4 * ch] = v.x;
        words[4 * ch + 1] = v.y;
        words[4 * ch + 2] = v.z;
        words[4 * ch + 3] = v.w;
      }
      const uint32_t sc = *reinterpret_cast<const uint32_t*>(sp + 2 * GE::CODE + (is_v ? 2 : 0) * GE::SC + row * 4);
      const uint32_t bi = *reinterpret_cast<const uint32_t*>(sp + 2 * GE::CODE + (is_v ? 3 : 1) * GE::SC + row * 4);
      __syncwarp();
      if (lane == 0) mbar_arrive(&code_empty[st]);
      const uint32_t s0 = prmt(sc, 0u, 0x1010), s1 = prmt(sc, 0u, 0x3232);
      const uint32_t b0 = prmt(bi, 0u, 0x1010), b1 = prmt(bi, 0u, 0x3232);
      if (j >= kKvBufs) {  // PV(j - kKvBufs) released this buffer
        ok = mbar_wait(&kv_empty[buf], ((j / kKvBufs) + 1) & 1, a.status, 48);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      uint8_t* dst = dst_base + buf * 16384;
      const int key = k_begin + j * kKT + row;
      if (key < n) {
        dequant_row<T, BITS>(words, s0, s1, b0, b1, dst, row);
      } else {  // past the cache's valid length: zeros, so that P = 0 meets finite V
#pragma unroll
        for (int i = 0; i < 16; ++i)
          *reinterpret_cast<uint4*>(dst + (i >> 3) * 8192 + row * 128 + (((i & 7) ^ (row & 7)) * 16)) =
              make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_full[buf]);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

template <typename T, int BITS, int MT>
int launch_tc(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  using SM = TcSmem<BITS, MT>;
  TcParams prm;
  prm.a = a;
  prm.TT = p.tokens_per_tile;
  prm.chunk = p.chunk;
  const bool direct = combine && p.splits == 1 && a.out_kind == QKV_OUT_NORMALIZED;
  prm.parts = direct ? nullptr : reinterpret_cast<float*>(a.workspace);
  constexpr int RB = kD * BITS / 8;
  if (!make_code_map_bytes(&prm.tmk, a.kw, RB, a.NP, (long long)a.B * a.HKV, RB, kKT) ||
      !make_code_map_bytes(&prm.tmv, a.vw, RB, a.NP, (long long)a.B * a.HKV, RB, kKT))
    return QKV_ECUDA;
  const size_t smem = (size_t)SM::BYTES + 1024;
  auto kern = prefill_tc_kernel<T, BITS, MT>;
  static unsigned attr_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done & (1u << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return QKV_ECUDA;
    attr_done |= 1u << (dev & 31);
  }
  dim3 grid(p.tblocks, a.B * a.HKV, p.splits);
  kern<<<grid, kThreadsTc, smem, st>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return QKV_ECUDA;
  if (direct || !combine) return QKV_OK;
  const long long rows = (long long)a.B * a.HQ * a.S;
  return launch_combine(prm.parts, p.splits, rows, rows, kD, a.out, a.dtype, a.out_kind, st);
}

template <typename T, int BITS>
int launch_tc_mt(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  return p.tiles == 2 ? launch_tc<T, BITS, 2>(a, p, combine, st)
                      : launch_tc<T, BITS, 1>(a, p, combine, st);
}

}  // namespace

bool prefill_tc_eligible(int B, int HQ, int HKV, int S, int D, const int* lens,
                         const int* pos_base, const int* total_lens, int mask_kind) {
  if (D != kD || HKV <= 0 || HQ % HKV || lens || pos_base || total_lens) return false;
  if (mask_kind != QKV_MASK_NONE && mask_kind != QKV_MASK_CAUSAL) return false;
  const int gqa = HQ / HKV;
  if (gqa > 128 || 128 % gqa) return false;
  (void)B;
  return gqa * S >= 128;  // at least one full MMA tile of query rows
}

TcPlan prefill_tc_plan(int B, int HQ, int HKV, int S, int n_max, int want_splits) {
  TcPlan p;
  const int gqa = HQ / HKV;
  p.tokens_per_tile = 128 / gqa;
  p.tiles = S > p.tokens_per_tile ? 2 : 1;
  p.tblocks = (S + p.tiles * p.tokens_per_tile - 1) / (p.tiles * p.tokens_per_tile);
  const int units = std::max(1, p.tblocks * B * HKV);
  const int sms = num_sms();
  const int n = std::max(n_max, 1);
  int best = 1;
  if (want_splits > 0) {
    best = want_splits;
  } else {
    // fewest splits that fill the waves to >= 90 %, keeping >= 512 keys per split
    double best_eff = 0.0;
    for (int s = 1; s <= 16; ++s) {
      if (s > 1 && (n + s - 1) / s < 512) break;
      const long long ctas = (long long)units * s;
      const long long waves = (ctas + sms - 1) / sms;
      const double eff = (double)ctas / (double)(waves * sms);
      if (eff > best_eff + 1e-9) {
        best_eff = eff;
        best = s;
      }
      if (eff >= 0.9) break;
    }
  }
  p.chunk = ((n + best - 1) / best + kKT - 1) / kKT * kKT;
  p.splits = (n + p.chunk - 1) / p.chunk;
  return p;
}

size_t prefill_tc_workspace_bytes(int B, int HQ, int S, int D, const TcPlan& p, bool direct) {
  if (direct && p.splits == 1) return 0;
  return (size_t)p.splits * B * HQ * S * (D + 4) * sizeof(float);
}

int launch_prefill_tc(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  if (a.dtype == QKV_BF16)
    return a.bits == 4 ? launch_tc_mt<__nv_bfloat16, 4>(a, p, combine, st)
                       : launch_tc_mt<__nv_bfloat16, 8>(a, p, combine, st);
  return a.bits == 4 ? launch_tc_mt<__half, 4>(a, p, combine, st)
                     : launch_tc_mt<__half, 8>(a, p, combine, st);
}

}  // namespace qkv
