// Tensor-core attention for many query tokens over the affine-quantized KV cache (sm_100a).
//
// Semantics follow the reference's multi-token branch (src/chad/mlx_qsdpa.py:751-766): the
// cache is dequantized to the query dtype (mx.dequantize) and attended with a causal or no
// mask (mx.fast.scaled_dot_product_attention). Here the dequantization happens tile by tile
// in shared memory and never reaches HBM:
//
//   * CTA = up to two 128-row MMA tiles of query rows of ONE kv head: row r of a tile is
//     (q head r / TT of the GQA group, token r % TT), TT = 128 / GQA; every row of the CTA
//     shares each dequantized K/V tile of 128 keys.
//   * Warp roles (13 warps): 0 tensor-memory owner and single-thread MMA issuer; 1-3 and 12
//     dequantizers (packed codes read from global memory, one key row of K and of V per
//     thread, written as 16-bit tiles in the 128-byte-swizzled operand layout); 4-7 / 8-11
//     softmax of tile 0 / 1 (one S row per thread, no cross-thread reductions).
//   * Tensor memory: S_0, S_1 (128 columns each, P written back over them as 16-bit pairs),
//     O_0, O_1 (128 columns each). Per key tile i the MMA thread issues, for each tile m,
//     O_m += P_m V(i) as soon as softmax_m(i) is done and then S_m = Q_m K(i+1)^T, so one
//     tile's softmax overlaps the other tile's MMAs (ping-pong). MMAs are M=128, N=128, K=16
//     (N=64 runs at two thirds of the tensor pipe's rate on B200).
//   * The running max is only raised when it grows by more than 2^12, so the O rescale in
//     tensor memory and the two-pass softmax are rare even on key-outlier data; P values stay
//     <= 4096 (inside f16 as well as bf16).
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
constexpr int kKT = 128;         // keys per tile (MMA N of Q K^T)
constexpr int kWarpsTc = 13;
constexpr int kThreadsTc = kWarpsTc * 32;
constexpr float kRescaleLog2 = 12.0f;  // P <= 2^12: exact range in bf16 and f16
// One value pair in kPolyPairs takes exp2_poly2 (FMA pipe) instead of the MUFU: 1 in 8 for
// prefill tiles, 1 in 4 for a verify block's key-split tiles (measured: prefill over a 30K
// prefix 1215 us per layer at 1 in 8, 1235 at 1 in 4, 1233 with none; the 8-token verify
// 16.25 us at 1 in 4, 16.50 at 1 in 8).
template <bool SK>
constexpr int kPolyPairs = SK ? 4 : 8;
constexpr int kHalf = kKT * 128;       // bytes of one 64-dim half of a K or V tile
constexpr int kTileBytes = 2 * kHalf;  // one dequantized K or V tile
#define kNegInfTc (-__int_as_float(0x7f800000))

template <int MT>
struct TcSmem {
  static constexpr int Q = 0;                     // MT x (2 halves x 128 rows x 128 B)
  static constexpr int KD = MT * 32768;           // 2 buffers of K (K-major operand)
  static constexpr int VD = KD + 2 * kTileBytes;  // 2 buffers of V (MN-major operand)
  static constexpr int BYTES = VD + 2 * kTileBytes;
};

struct TcParams {
  AttnArgs a;
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

// Packed fp32 pair arithmetic (sm_100): two lanes of work per issued instruction.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                     float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^t for a pair of values on the FMA/ALU pipes instead of the MUFU: t = n + f with
// n = rint(t), |f| <= 1/2; 2^f from a degree-3 polynomial fitted here to relative error 8e-5
// over [-1/2, 1/2] (far below the 16-bit P it feeds); 2^n enters the exponent bits through
// one integer multiply-add per value. t is clamped at -126: 2^-126 stands in for 0.
__device__ __forceinline__ void exp2_poly2(float& p0, float& p1, float t0, float t1) {
  t0 = fmaxf(t0, -126.0f);
  t1 = fmaxf(t1, -126.0f);
  float j0, j1, n0, n1, f0, f1, q0, q1;
  add2(j0, j1, t0, t1, 12582912.0f, 12582912.0f);  // 1.5 * 2^23: low mantissa bits = rint(t)
  add2(n0, n1, j0, j1, -12582912.0f, -12582912.0f);
  fma2(f0, f1, n0, n1, -1.0f, -1.0f, t0, t1);
  fma2(q0, q1, 0.05518098f, 0.05518098f, f0, f1, 0.24263459f, 0.24263459f);
  fma2(q0, q1, q0, q1, f0, f1, 0.69326133f, 0.69326133f);
  fma2(q0, q1, q0, q1, f0, f1, 0.99992621f, 0.99992621f);
  p0 = __uint_as_float(__float_as_uint(j0) * 8388608u + __float_as_uint(q0));
  p1 = __uint_as_float(__float_as_uint(j1) * 8388608u + __float_as_uint(q1));
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
      *reinterpret_cast<uint4*>(dst + h * kHalf + row * 128 + c * 16) = o;
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
      *reinterpret_cast<uint4*>(dst + h * kHalf + row * 128 + cc * 16) = o;
    }
  }
}

// 16-byte read-only global load (codes and scales are immutable during the kernel)
__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// SK ("key-split tiles", MT == 2): the CTA's query rows fit one 128-row tile; both
// tensor-memory tiles hold those rows and take alternate key tiles (tile m: keys tiles
// m, m+2, ...), so one tile's softmax still overlaps the other's MMAs. The epilogue folds
// tile 1 into tile 0: one partial row per query row and split.
template <typename T, int BITS, int MT, bool SK>
__global__ void __launch_bounds__(kThreadsTc, 1) prefill_tc_kernel(const __grid_constant__ TcParams P) {
  static_assert(!SK || MT == 2, "key-split tiles need both tensor-memory tiles");
  constexpr int QT = SK ? 1 : MT;  // query tiles staged
  using SM = TcSmem<MT>;
  using PK = Pack16<T>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int RB = kD * BITS / 8;  // code bytes per key
  constexpr int RW = RB / 4;         // code words per key
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t k_full[2], k_free[2], v_full[2], v_free[2];
  __shared__ uint64_t s_full[MT], p_full[MT], o_done[MT];
  __shared__ uint64_t mma_fin;
  __shared__ uint32_t tmem_sh;
  __shared__ float sk_m[SK ? 128 : 1], sk_l[SK ? 128 : 1];  // tile 1's row state (SK)

  const AttnArgs& a = P.a;
  // Programmatic dependent launch: the next kernel may be scheduled once every CTA of this
  // one has started; this one touches no global memory before griddepcontrol.wait below.
  asm volatile("griddepcontrol.launch_dependents;");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int TT = P.TT;
  const int gqa = a.HQ / a.HKV;
  const int bh = blockIdx.y;  // b * HKV + hkv
  const int b = bh / a.HKV, hkv = bh % a.HKV;
  const int t0 = blockIdx.x * (QT * TT);
  const int split = blockIdx.z;
  const int n = min(max(a.n, 0), a.NP);
  const bool causal = a.mask_kind == QKV_MASK_CAUSAL;
  // key range of this CTA: [k_begin, k_stop); every row sees at most keys < k_stop
  const int k_begin = split * P.chunk;
  const int t_last = min(t0 + QT * TT, a.S) - 1;
  const int lim_hi = causal ? n - a.S + t_last : n - 1;  // last key any row may see
  const int k_stop = min(min(k_begin + P.chunk, n), lim_hi + 1);
  const int ntiles = k_stop > k_begin ? (k_stop - k_begin + kKT - 1) / kKT : 0;
  // softmax warps of a tile that hold query rows: a verify block packs its GQA x S rows into
  // the first lanes (TT = S), and the warps past them sit the loop out
  const int n_act = SK ? min(4, (gqa * TT + 31) / 32) : 4;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 4);
      mbar_init(&v_full[s], 4);
      mbar_init(&k_free[s], 1);
      mbar_init(&v_free[s], 1);
    }
    for (int m = 0; m < MT; ++m) {
      mbar_init(&s_full[m], 1);
      mbar_init(&p_full[m], n_act);
      mbar_init(&o_done[m], 1);
    }
    mbar_init(&mma_fin, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, 512);
    tc::tmem_relinquish();
  }
  // ---- dequantizer state; the first tile's codes are requested before Q is staged --------
  const bool is_dq = warp == 1 || warp == 2 || warp == 3 || warp == 12;
  const int dq_row = (warp == 12 ? 3 : warp - 1) * 32 + lane;  // key row of each tile, 0..127
  const uint8_t* kw_base = reinterpret_cast<const uint8_t*>(a.kw) + (long long)bh * a.NP * RB;
  const uint8_t* vw_base = reinterpret_cast<const uint8_t*>(a.vw) + (long long)bh * a.NP * RB;
  const long long sc0 = (long long)bh * a.NP * 4;  // 2 groups x 16 bit per key
  uint32_t kc[RW], vc[RW], ksc = 0, kbi = 0, vsc = 0, vbi = 0;
  auto load = [&](int i) {  // codes and scales of key row dq_row of tile i
    const int key = k_begin + i * kKT + dq_row;
    if (key < n) {
#pragma unroll
      for (int u = 0; u < RW / 4; ++u) {
        const uint4 kv = ldg16(kw_base + (long long)key * RB + u * 16);
        const uint4 vv = ldg16(vw_base + (long long)key * RB + u * 16);
        kc[4 * u] = kv.x; kc[4 * u + 1] = kv.y; kc[4 * u + 2] = kv.z; kc[4 * u + 3] = kv.w;
        vc[4 * u] = vv.x; vc[4 * u + 1] = vv.y; vc[4 * u + 2] = vv.z; vc[4 * u + 3] = vv.w;
      }
      ksc = ldg4((const uint8_t*)a.ks + sc0 + (long long)key * 4);
      kbi = ldg4((const uint8_t*)a.kb + sc0 + (long long)key * 4);
      vsc = ldg4((const uint8_t*)a.vs + sc0 + (long long)key * 4);
      vbi = ldg4((const uint8_t*)a.vb + sc0 + (long long)key * 4);
    }
  };
  // Before the dependency wait: warm L2 with the first key tiles of this CTA's range that
  // lie below a.prefetch_limit (cache positions the kernel just before does not write) and
  // with its query rows. Only hints: L2 is the point of coherence, so anything the
  // predecessor writes afterwards is still read correctly below.
  if (warp == 4 && lane == 0) {
    const int kend = min(min(k_stop, k_begin + 4 * kKT), a.prefetch_limit);
    if (kend > k_begin) {
      const uint32_t nk = (uint32_t)(kend - k_begin);
      prefetch_l2(kw_base + (long long)k_begin * RB, nk * RB);
      prefetch_l2(vw_base + (long long)k_begin * RB, nk * RB);
      const uint32_t sb = (nk * 4u) & ~15u;  // whole 16-byte pieces inside the range
      if (sb) {
        prefetch_l2((const uint8_t*)a.ks + sc0 + (long long)k_begin * 4, sb);
        prefetch_l2((const uint8_t*)a.kb + sc0 + (long long)k_begin * 4, sb);
        prefetch_l2((const uint8_t*)a.vs + sc0 + (long long)k_begin * 4, sb);
        prefetch_l2((const uint8_t*)a.vb + sc0 + (long long)k_begin * 4, sb);
      }
    }
  }
  // barriers and tensor memory are set up; q, the cache (its newest positions may come from
  // the kernel just before) and the outputs are only touched after the predecessor is done
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (is_dq && ntiles > 0) load(0);
  // ---- stage Q (all threads): MT tiles x 128 rows x 16 chunks of 8 head dims; every load of
  // a thread is issued before its first store -----------------------------------------------
  {
    const T* q = reinterpret_cast<const T*>(a.q);
    constexpr int kChunks = QT * 128 * 16;
    constexpr int kPer = (kChunks + kThreadsTc - 1) / kThreadsTc;
    uint4 qv[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * kThreadsTc;
      qv[k] = make_uint4(0, 0, 0, 0);
      if (i < kChunks) {
        const int m = i / (128 * 16), r = (i / 16) % 128, c = i % 16;
        const int hl = r / TT, t = t0 + m * TT + (r % TT);
        if (hl < gqa && t < a.S) {
          const long long row = ((long long)b * a.HQ + hkv * gqa + hl) * a.S + t;
          qv[k] = *reinterpret_cast<const uint4*>(q + row * kD + c * 8);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * kThreadsTc;
      if (i < kChunks) {
        const int m = i / (128 * 16), r = (i / 16) % 128, c = i % 16;
        uint4 v = qv[k];
        if constexpr (BITS == 4) {  // (0,1)(2,3)(4,5)(6,7) -> (0,4)(1,5)(2,6)(3,7)
          const uint4 u = v;
          v.x = prmt(u.x, u.z, 0x5410);
          v.y = prmt(u.x, u.z, 0x7632);
          v.z = prmt(u.y, u.w, 0x5410);
          v.w = prmt(u.y, u.w, 0x7632);
        }
        const int h = c >> 3, cc = (c & 7) ^ (r & 7);
        *reinterpret_cast<uint4*>(smem + SM::Q + m * 32768 + h * 16384 + r * 128 + cc * 16) = v;
      }
    }
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_sh;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_f16(kBf16, 128, kKT, false, false);
      constexpr uint32_t id_o = tc::idesc_f16(kBf16, 128, kD, false, true);
      const uint32_t q_base = smem_u32(smem + SM::Q);
      const uint32_t kd_base = smem_u32(smem + SM::KD);
      const uint32_t vd_base = smem_u32(smem + SM::VD);
      auto qk = [&](int m, int i) {  // S_m = Q_m K(i)^T
        const uint32_t kb = kd_base + (i & 1) * kTileBytes;
        const uint32_t qb = q_base + (SK ? 0 : m) * 32768;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint64_t ad = tc::sdesc_sw128(qb + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
          const uint64_t bd = tc::sdesc_sw128(kb + (s >> 2) * kHalf + (s & 3) * 32, 16, 1024);
          tc::mma_ss(tmem + m * 128, ad, bd, id_s, s > 0 ? 1u : 0u);
        }
        tc::mma_commit(&s_full[m]);
      };
      auto pv = [&](int m, int i) {  // O_m (+)= P_m V(i), P_m in tensor memory over S_m
        const uint32_t vb = vd_base + (i & 1) * kTileBytes;
#pragma unroll
        for (int s = 0; s < kKT / 16; ++s) {
          const uint64_t bd = tc::sdesc_sw128(vb + s * 2048, kHalf, 1024);
          tc::mma_ts(tmem + 256 + m * 128, tmem + m * 128 + s * 8, bd, id_o,
                     (i > (SK ? m : 0) || s > 0) ? 1u : 0u);
        }
        tc::mma_commit(&o_done[m]);
      };
      if constexpr (SK) {
        // tile m takes key tiles m, m+2, ...: each QK / PV touches one tile's buffers
        for (int m = 0; m < 2 && ok; ++m) {
          if (m < ntiles) {
            ok = mbar_wait(&k_full[m], 0, a.status, 40);
            if (!ok) break;
            tc::fence_after_sync();
            qk(m, m);
            tc::mma_commit(&k_free[m]);
          }
        }
        for (int j = 0; 2 * j < ntiles && ok; ++j) {
          for (int m = 0; m < 2 && ok; ++m) {
            const int i = 2 * j + m;
            if (i >= ntiles) break;
            ok = mbar_wait(&v_full[i & 1], (i >> 1) & 1, a.status, 41);
            if (ok) ok = mbar_wait(&p_full[m], j & 1, a.status, 42);
            if (!ok) break;
            tc::fence_after_sync();
            pv(m, i);
            tc::mma_commit(&v_free[i & 1]);
            if (i + 2 < ntiles) {
              ok = mbar_wait(&k_full[i & 1], ((i + 2) >> 1) & 1, a.status, 43);
              if (!ok) break;
              tc::fence_after_sync();
              qk(m, i + 2);  // S_m is free: P_m(i) is read by the PV issued just before
              tc::mma_commit(&k_free[i & 1]);
            }
          }
        }
      } else {
      if (ntiles > 0) {
        ok = mbar_wait(&k_full[0], 0, a.status, 40);
        if (ok) {
          tc::fence_after_sync();
          for (int m = 0; m < MT; ++m) qk(m, 0);
          tc::mma_commit(&k_free[0]);
        }
      }
      for (int i = 0; i < ntiles && ok; ++i) {
        const bool more = i + 1 < ntiles;
        ok = mbar_wait(&v_full[i & 1], (i >> 1) & 1, a.status, 41);
        for (int m = 0; m < MT && ok; ++m) {
          ok = mbar_wait(&p_full[m], i & 1, a.status, 42);
          if (!ok) break;
          tc::fence_after_sync();
          pv(m, i);
          if (more) {
            if (m == 0) {
              ok = mbar_wait(&k_full[(i + 1) & 1], ((i + 1) >> 1) & 1, a.status, 43);
              if (!ok) break;
              tc::fence_after_sync();
            }
            qk(m, i + 1);  // S_m is free: P_m(i) is read by the PV issued just before
          }
        }
        if (!ok) break;
        tc::mma_commit(&v_free[i & 1]);
        if (more) tc::mma_commit(&k_free[(i + 1) & 1]);
      }
      }
      tc::mma_commit(&mma_fin);
      mbar_wait(&mma_fin, 0, a.status, 44);
    }
  } else if (warp >= 4 && warp < 4 + 4 * MT) {
    // ---------------------------------------------------------------- softmax
    const int m = (warp - 4) >> 2;
    const int r = (warp & 3) * 32 + lane;  // tensor-memory lane = row of tile m
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int hl = r / TT, t = t0 + (SK ? 0 : m) * TT + (r % TT);
    const bool row_ok = hl < gqa && t < a.S;
    // this tile's key tiles: all (SK = false) or m, m+2, ... (SK)
    const bool idle = SK && (warp & 3) >= n_act;
    const int my_tiles = idle ? 0 : SK ? (ntiles > m ? (ntiles - m + 1) / 2 : 0) : ntiles;
    int lim = causal ? n - a.S + t : n - 1;
    lim = min(lim, k_stop - 1);
    const float c = a.scale * 1.4426950408889634f;
    const uint32_t ts = tmem + lane_off + m * 128;
    const uint32_t to = tmem + lane_off + 256 + m * 128;
    float m_run = kNegInfTc, l_run = 0.f;
    uint32_t x[32];
    for (int i = 0; i < my_tiles; ++i) {
      ok = mbar_wait(&s_full[m], i & 1, a.status, 45);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::fence_after_sync();
      const int kbase = k_begin + (SK ? 2 * i + m : i) * kKT;
      const bool msk = kbase + kKT - 1 > lim;
      // Fast path: one pass against the running max. Every chunk's max must stay within 2^12
      // of it (one vote per chunk); P stays in registers until all chunks passed, so S is
      // still intact for the two-pass path, which handles the first tile and a new maximum.
      float sa[4] = {0.f, 0.f, 0.f, 0.f};
      float alpha = 1.f;
      bool resc = false;
      bool fast = __all_sync(0xffffffffu, m_run != kNegInfTc);
      if (fast) {
        const float mu = m_run;
        const float s_hi = (m_run + kRescaleLog2) / c;  // largest raw score the pass accepts
        uint32_t pf[64];
#pragma unroll
        for (int ch = 0; ch < kKT / 32; ++ch) {
          tc::ld32(ts + ch * 32, x);
          tc::wait_ld();
          if (msk) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kbase + ch * 32 + e > lim) x[e] = __float_as_uint(kNegInfTc);
          }
          float cm[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) cm[e] = fmaxf(__uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
#pragma unroll
          for (int e = 4; e < 16; ++e)
            cm[e & 3] = max3(cm[e & 3], __uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
          if (__any_sync(0xffffffffu, fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3])) > s_hi)) {
            fast = false;
            break;
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float u0, u1, p0, p1;
            fma2(u0, u1, __uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]), c, c, -mu, -mu);
            if (kPolyPairs<SK> > 0 && e % kPolyPairs<SK> == kPolyPairs<SK> - 1) {
              exp2_poly2(p0, p1, u0, u1);
            } else {
              p0 = ex2(u0);
              p1 = ex2(u1);
            }
            add2(sa[2 * (e & 1)], sa[2 * (e & 1) + 1], sa[2 * (e & 1)], sa[2 * (e & 1) + 1], p0, p1);
            pf[ch * 16 + e] = PK::pack(p0, p1);
          }
        }
        if (fast) {
          uint32_t h0[32], h1[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            h0[e] = pf[e];
            h1[e] = pf[32 + e];
          }
          tc::st32(ts, h0);
          tc::st32(ts + 32, h1);
        } else {
          sa[0] = sa[1] = sa[2] = sa[3] = 0.f;
        }
      }
      if (!fast) {
        // pass 1: row max, eight independent chains
        float mxa[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mxa[e] = kNegInfTc;
#pragma unroll 1
        for (int ch = 0; ch < kKT / 32; ++ch) {
          tc::ld32(ts + ch * 32, x);
          tc::wait_ld();
          if (msk) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kbase + ch * 32 + e > lim) x[e] = __float_as_uint(kNegInfTc);
          }
#pragma unroll
          for (int e = 0; e < 16; ++e)
            mxa[e & 7] = max3(mxa[e & 7], __uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]));
        }
        const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                               fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
        const float m_cand = mx * c;
        resc = m_cand > m_run + kRescaleLog2;  // false while the tile is all masked
        if (resc) {
          alpha = ex2(m_run - m_cand);
          m_run = m_cand;
        }
        const float mu = m_run == kNegInfTc ? 0.f : m_run;
        // pass 2: p = 2^(s*c - mu) (MUFU; one pair in kPolyPairs<SK> by the FMA-pipe polynomial),
        // P over S.
        // P chunk ch lands in columns [16ch, 16ch+16), all read already by chunks <= ch.
#pragma unroll 1
        for (int ch = 0; ch < kKT / 32; ++ch) {
          tc::ld32(ts + ch * 32, x);
          tc::wait_ld();
          if (msk) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kbase + ch * 32 + e > lim) x[e] = __float_as_uint(kNegInfTc);
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float u0, u1, p0, p1;
            fma2(u0, u1, __uint_as_float(x[2 * e]), __uint_as_float(x[2 * e + 1]), c, c, -mu, -mu);
            if (kPolyPairs<SK> > 0 && e % kPolyPairs<SK> == kPolyPairs<SK> - 1) {
              exp2_poly2(p0, p1, u0, u1);
            } else {
              p0 = ex2(u0);
              p1 = ex2(u1);
            }
            add2(sa[2 * (e & 1)], sa[2 * (e & 1) + 1], sa[2 * (e & 1)], sa[2 * (e & 1) + 1], p0, p1);
            pk[e] = PK::pack(p0, p1);
          }
          tc::st16(ts + ch * 16, pk);
        }
      }
      tc::wait_st();
      l_run = fmaf(l_run, alpha, (sa[0] + sa[1]) + (sa[2] + sa[3]));
      if (i > 0) {
        // Wait for PV(i-1) on every tile: a parity wait only tells phases apart while the
        // barrier is at most one phase ahead of this thread's view of it, and a rescale
        // needs O out of flight anyway.
        ok = mbar_wait(&o_done[m], (i - 1) & 1, a.status, 46);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      if (i > 0 && __any_sync(0xffffffffu, resc)) {
        // scale this row of O in place (PV(i) is not issued before p_full below)
        tc::fence_after_sync();
#pragma unroll 1
        for (int qd = 0; qd < 4; ++qd) {
          tc::ld32(to + qd * 32, x);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = __float_as_uint(__uint_as_float(x[e]) * alpha);
          tc::st32(to + qd * 32, x);
        }
        tc::wait_st();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[m]);
    }
    // ---- epilogue: O row -> output (normalized) or partial row ---------------------------
    if (ok && my_tiles > 0) {
      ok = mbar_wait(&o_done[m], (my_tiles - 1) & 1, a.status, 47);
      ok = __all_sync(0xffffffffu, ok);
    }
    // SK: both tensor-memory tiles hold the same query rows over alternate key tiles. Tile 1
    // hands its (max, sum) over through shared memory and tile 0 folds tile 1's O into its
    // own (the warps 4 + j and 8 + j share tensor-memory lanes), so the CTA writes one
    // partial row per query row, or the normalized output when it is the only split.
    float f0 = 1.f, f1 = 0.f;
    bool has1 = false;
    if constexpr (SK) {
      if (m == 1) {
        sk_m[r] = m_run;
        sk_l[r] = l_run;
      }
      named_bar_sync(1, 256);  // the eight softmax warps
      has1 = ntiles > 1;
      if (m == 0 && has1) {
        const float m1 = sk_m[r], mx = fmaxf(m_run, m1);
        const float mu = mx == kNegInfTc ? 0.f : mx;
        f0 = ex2(m_run - mu);
        f1 = ex2(m1 - mu);
        l_run = fmaf(f0, l_run, f1 * sk_l[r]);
        m_run = mx;
      }
    }
    if (ok && !(SK && m == 1) && !idle) {
      tc::fence_after_sync();
      const long long row = ((long long)b * a.HQ + hkv * gqa + hl) * a.S + t;
      const int part = split;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
      for (int qd = 0; qd < 4; ++qd) {
        if (my_tiles > 0) {
          tc::ld32(to + qd * 32, x);
          tc::wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = 0u;
        }
        if (SK && has1) {
          uint32_t y[32];
          tc::ld32(to + 128 + qd * 32, y);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            x[e] = __float_as_uint(fmaf(f0, __uint_as_float(x[e]), f1 * __uint_as_float(y[e])));
        }
        // column position p of an 8-dim group holds dim perm[p] (4-bit) or p (8-bit)
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
            float* dst = P.parts + ((long long)part * a.B * a.HQ * a.S + row) * (kD + 4) + qd * 32;
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(dst + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
          } else {
            uint32_t* dst =
                reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(a.out) + row * kD + qd * 32);
#pragma unroll
            for (int e = 0; e < 32; e += 8)
              *reinterpret_cast<uint4*>(dst + e / 2) =
                  make_uint4(PK::pack(o[e] * inv, o[e + 1] * inv), PK::pack(o[e + 2] * inv, o[e + 3] * inv),
                             PK::pack(o[e + 4] * inv, o[e + 5] * inv), PK::pack(o[e + 6] * inv, o[e + 7] * inv));
          }
        }
      }
      if (row_ok && P.parts) {
        float* dst = P.parts + ((long long)part * a.B * a.HQ * a.S + row) * (kD + 4) + kD;
        *reinterpret_cast<float4*>(dst) = make_float4(m_run, l_run, 0.f, 0.f);
      }
    }
  } else if (is_dq) {
    // ---------------------------------------------------------------- dequantizers
    const int row = dq_row;
    auto store = [&](const uint32_t* codes, uint32_t sc, uint32_t bi, bool valid, uint8_t* dst) {
      if (valid) {
        dequant_row<T, BITS>(codes, prmt(sc, 0u, 0x1010), prmt(sc, 0u, 0x3232),
                             prmt(bi, 0u, 0x1010), prmt(bi, 0u, 0x3232), dst, row);
      } else {  // past the cache's valid length: zeros, so that P = 0 meets finite V
#pragma unroll
        for (int e = 0; e < 16; ++e)
          *reinterpret_cast<uint4*>(dst + (e >> 3) * kHalf + row * 128 + (((e & 7) ^ (row & 7)) * 16)) =
              make_uint4(0, 0, 0, 0);
      }
    };
    for (int i = 0; i < ntiles; ++i) {
      const int buf = i & 1;
      const bool valid = k_begin + i * kKT + row < n;
      if (i >= 2) {  // QK(i-2) released this K buffer
        ok = mbar_wait(&k_free[buf], ((i >> 1) + 1) & 1, a.status, 48);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      store(kc, ksc, kbi, valid, smem + SM::KD + buf * kTileBytes);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&k_full[buf]);
      if (i >= 2) {  // PV(i-2) released this V buffer
        ok = mbar_wait(&v_free[buf], ((i >> 1) + 1) & 1, a.status, 49);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      store(vc, vsc, vbi, valid, smem + SM::VD + buf * kTileBytes);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&v_full[buf]);
      if (i + 1 < ntiles) load(i + 1);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

template <typename T, int BITS, int MT, bool SK>
int launch_tc(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  using SM = TcSmem<MT>;
  TcParams prm;
  prm.a = a;
  prm.TT = p.tiles == 1 ? std::min(p.tokens_per_tile, a.S) : p.tokens_per_tile;
  prm.chunk = p.chunk;
  const bool direct = combine && p.parts == 1 && a.out_kind == QKV_OUT_NORMALIZED;
  prm.parts = direct ? nullptr : reinterpret_cast<float*>(a.workspace);
  const size_t smem = (size_t)SM::BYTES + 1024;
  auto kern = prefill_tc_kernel<T, BITS, MT, SK>;
  static unsigned attr_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done & (1u << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return QKV_ECUDA;
    attr_done |= 1u << (dev & 31);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.tblocks, a.B * a.HKV, p.splits);
  cfg.blockDim = dim3(kThreadsTc, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, prm) != cudaSuccess) return QKV_ECUDA;
  if (direct || !combine) return QKV_OK;
  const long long rows = (long long)a.B * a.HQ * a.S;
  // the partials sit in the attention workspace: the combine clears what it reads
  return launch_combine(prm.parts, p.parts, rows, rows, kD, a.out, a.dtype, a.out_kind, st,
                        true);
}

template <typename T, int BITS>
int launch_tc_mt(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  // one query tile: both tensor-memory tiles split its keys (see prefill_tc_kernel)
  return p.tiles == 2 ? launch_tc<T, BITS, 2, false>(a, p, combine, st)
                      : launch_tc<T, BITS, 2, true>(a, p, combine, st);
}

}  // namespace

bool prefill_tc_eligible(int B, int HQ, int HKV, int S, int D, const int* lens,
                         const int* pos_base, const int* total_lens, int mask_kind) {
  if (D != kD || HKV <= 0 || HQ % HKV || lens || pos_base || total_lens) return false;
  if (mask_kind != QKV_MASK_NONE && mask_kind != QKV_MASK_CAUSAL) return false;
  const int gqa = HQ / HKV;
  if (gqa > 128 || 128 % gqa) return false;
  (void)B;
  return gqa * S >= 64;  // at least half a 128-row MMA tile of query rows
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
  } else if (units >= sms) {
    best = 1;  // a full wave without splitting: split partials would only add traffic
  } else {
    // fewest splits that fill the waves to >= 90 %, keeping >= 256 keys per split
    double best_eff = 0.0;
    for (int s = 1; s <= 64; ++s) {
      if (s > 1 && (n + s - 1) / s < 256) break;
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
  p.parts = p.splits;
  p.parts_bound = best;
  return p;
}

size_t prefill_tc_workspace_bytes(int B, int HQ, int S, int D, const TcPlan& p, bool direct) {
  if (direct && p.parts == 1) return 0;
  return (size_t)p.parts * B * HQ * S * (D + 4) * sizeof(float);
}

int launch_prefill_tc(const AttnArgs& a, const TcPlan& p, bool combine, cudaStream_t st) {
  if (a.dtype == QKV_BF16)
    return a.bits == 4 ? launch_tc_mt<__nv_bfloat16, 4>(a, p, combine, st)
                       : launch_tc_mt<__nv_bfloat16, 8>(a, p, combine, st);
  return a.bits == 4 ? launch_tc_mt<__half, 4>(a, p, combine, st)
                     : launch_tc_mt<__half, 8>(a, p, combine, st);
}

}  // namespace qkv
