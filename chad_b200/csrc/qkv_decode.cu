// Split-KV attention over the MLX-layout quantized KV cache, sm_100a.
//
// Replaces the reference's pass 1 (`_P1_SRC`, src/chad/mlx_qsdpa.py:73-209, and its
// simdgroup-matrix retile `_P1_SGM_SRC`, :303-473) and pass 2 (`_P2_SRC`, :213-265).
//
// Shape of the work. One CTA = one (batch b, kv head, query-row group, key split). Its
// query rows are the GQA heads x query tokens that share the kv head (at most 16, stored
// contiguously in q). A producer warp streams the split's keys through a 4-deep ring of
// shared-memory stages with 1-D bulk async copies (TMA): per stage 64 keys of packed K and
// V codes plus their scales and biases. Four consumer warps take 16 keys each per stage.
//
// The tensor-core mapping is the reference's retile insight (keys share one dequantized
// tile across the whole GQA group) turned around for mma.sync m16n8k16: the 16 KEYS are
// the MMA's M rows and the query rows are its N columns, so GQA 8 fills an N=8 tile with
// no padding.
//   scores^T (16 keys x 8 rows)  = K (16 x D) . (q*scale*log2e)^T      D/16 MMAs
//   out^T    (D x 8 rows)       += V^T (D x 16 keys) . P^T (16 x 8)    D/16 MMAs
// K and V^T fragments are built straight from packed codes in registers: a code c becomes
// the f16 value 1024+c by OR-ing it into the exponent pattern 0x6400 (exact), then
// (x - 1024) * scale + bias with f16x2 FMAs. The score accumulator is turned into the
// P^T operand with one movmatrix.trans per 8x8 block, so no shared-memory round trip is
// needed between the two products.
//
// Online softmax runs in base 2 per query row (the row's 8 lanes reduce with three xor
// shuffles) and the four warps' (max, sum, out) triples are merged through shared memory
// at the end, so each CTA writes one partial per row: [out(D), max, sum, 0, 0] in fp32.
// A combine kernel (the reference's pass 2) folds the splits.
#include <algorithm>

#include "qkv_common.cuh"
#include "qkv_internal.h"

namespace qkv {

namespace {

constexpr int kWarps = 4;                  // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + producer warp
constexpr int kTP = kDecodeStagePos;        // keys per stage (16 per consumer warp)
#define kNegInf (-__int_as_float(0x7f800000))

template <int BITS>
__device__ __forceinline__ int key_perm(int k) {
  // Order in which the 16 keys of a warp tile occupy the MMA rows. For 4-bit codes
  // (64-byte rows) the order 0,3,1,2,4,7,5,6 (+8) makes the rows that one lane quarter
  // reads together alternate between the two 64-byte halves of a bank cycle.
  if constexpr (BITS == 4) {
    const int lo = k & 3;
    return (k & 12) | (lo == 0 ? 0 : lo == 1 ? 3 : lo - 1);
  } else {
    return k;
  }
}

template <typename T, int BITS, int D>
struct Cfg {
  static constexpr int RB = D * BITS / 8;       // code bytes per key row
  static constexpr int G = D / 64;              // scale groups per row
  static constexpr int KCHUNK = RB / 4;         // K bytes per lane (its quarter of D)
  static constexpr int VCHUNK = RB / 8;         // V bytes per lane (its eighth of D)
  static constexpr int KS = D / 16;             // MMA k-steps of QK / m-tiles of PV
  static constexpr int CODES_BYTES = kTP * RB;
  static constexpr int SC_BYTES = kTP * G * 2;
  static constexpr int OFF_KC = 0;
  static constexpr int OFF_VC = CODES_BYTES;
  static constexpr int OFF_KS = 2 * CODES_BYTES;
  static constexpr int OFF_KB = OFF_KS + SC_BYTES;
  static constexpr int OFF_VS = OFF_KB + SC_BYTES;
  static constexpr int OFF_VB = OFF_VS + SC_BYTES;
  static constexpr int STAGE_BYTES = ((OFF_VB + SC_BYTES) + 127) / 128 * 128;
  static constexpr int STAGES = STAGE_BYTES * 4 <= 96 * 1024 ? 4 : 3;
};

__device__ __forceinline__ uint32_t u32_load_sh(const uint8_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// Load `N` bytes (8, 16, 32 or 64) of shared memory into words.
template <int N>
__device__ __forceinline__ void lds_bytes(uint32_t* dst, const uint8_t* src) {
  if constexpr (N == 4) {
    dst[0] = *reinterpret_cast<const uint32_t*>(src);
  } else if constexpr (N == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    dst[0] = v.x;
    dst[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < N / 16; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      dst[4 * i + 0] = v.x;
      dst[4 * i + 1] = v.y;
      dst[4 * i + 2] = v.z;
      dst[4 * i + 3] = v.w;
    }
  }
}

template <typename T>
__device__ __forceinline__ float sc_to_f32(const uint8_t* p) {
  return Elem<T>::bits_to_f32(*reinterpret_cast<const uint16_t*>(p));
}

constexpr uint32_t kMagic = 0x64006400u;  // f16x2 {1024, 1024}

__device__ __forceinline__ uint32_t deq2(uint32_t biased, uint32_t s2, uint32_t b2) {
  const __half2 x = __hsub2(u32_as_h2(biased), u32_as_h2(kMagic));
  return h2_as_u32(__hfma2(x, u32_as_h2(s2), u32_as_h2(b2)));
}

template <typename T, int BITS, int D, int NT>
__global__ void __launch_bounds__(kThreads, 2) decode_split_kernel(AttnArgs a) {
  using C = Cfg<T, BITS, D>;
  constexpr int RG = 8 * NT;  // query rows per CTA
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t full_bar[4], empty_bar[4];

  const int split = blockIdx.x;
  const int hkv = blockIdx.y % a.HKV;
  const int rg = blockIdx.y / a.HKV;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;  // MMA group id
  const int tq = lane & 3;   // thread in group

  const int gqa = a.HQ / a.HKV;
  const int R = gqa * a.S;  // query rows sharing this kv head
  int len = a.lens ? a.lens[b] : a.n;
  len = min(max(len, 0), a.NP);
  const int p_begin = split * a.chunk;
  const int p_end = min(p_begin + a.chunk, len);
  const int n_iters = p_end > p_begin ? (p_end - p_begin + kTP - 1) / kTP : 0;
  const long long bh = (long long)b * a.HKV + hkv;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kWarps) {
    // ------------------------------ producer -------------------------------------------
    if (lane == 0) {
      const uint8_t* kw = (const uint8_t*)a.kw + bh * a.NP * C::RB;
      const uint8_t* vw = (const uint8_t*)a.vw + bh * a.NP * C::RB;
      const uint8_t* ks = (const uint8_t*)a.ks + bh * a.NP * C::G * 2;
      const uint8_t* kb = (const uint8_t*)a.kb + bh * a.NP * C::G * 2;
      const uint8_t* vs = (const uint8_t*)a.vs + bh * a.NP * C::G * 2;
      const uint8_t* vb = (const uint8_t*)a.vb + bh * a.NP * C::G * 2;
      bool ok = true;
      for (int it = 0; it < n_iters && ok; ++it) {
        const int slot = it % C::STAGES;
        if (it >= C::STAGES) ok = mbar_wait(&empty_bar[slot], ((it / C::STAGES) - 1) & 1, a.status, 1);
        if (!ok) break;
        const int p0 = p_begin + it * kTP;
        const int rows = min(kTP, a.NP - p0);
        const uint32_t cb = rows * C::RB, sb = rows * C::G * 2;
        uint8_t* st = smem + slot * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full_bar[slot], 2 * cb + 4 * sb);
        bulk_g2s(st + C::OFF_KC, kw + (size_t)p0 * C::RB, cb, &full_bar[slot]);
        bulk_g2s(st + C::OFF_VC, vw + (size_t)p0 * C::RB, cb, &full_bar[slot]);
        bulk_g2s(st + C::OFF_KS, ks + (size_t)p0 * C::G * 2, sb, &full_bar[slot]);
        bulk_g2s(st + C::OFF_KB, kb + (size_t)p0 * C::G * 2, sb, &full_bar[slot]);
        bulk_g2s(st + C::OFF_VS, vs + (size_t)p0 * C::G * 2, sb, &full_bar[slot]);
        bulk_g2s(st + C::OFF_VB, vb + (size_t)p0 * C::G * 2, sb, &full_bar[slot]);
      }
      // drain: every issued stage must land before the CTA may exit
      const int issued = n_iters;
      for (int it = max(0, issued - C::STAGES); it < issued; ++it)
        mbar_wait(&full_bar[it % C::STAGES], (it / C::STAGES) & 1, a.status, 2);
    }
    return;
  }

  // -------------------------------- consumers -------------------------------------------
  const T* qg = (const T*)a.q;
  const float qmul = a.scale * 1.4426950408889634f;  // softmax in base 2
  const long long row0 = ((long long)b * a.HQ + (long long)hkv * gqa) * a.S;  // first q row
  const int rbase = rg * RG;

  // Q as the B operand of QK (k = head_dim pairs in this lane's K-code order, n = row).
  uint32_t qf[NT][C::KS][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int r = rbase + nt * 8 + gq;
    const bool rv = r < R;
    const T* qr = qg + (row0 + (rv ? r : 0)) * D + tq * (D / 4);
#pragma unroll
    for (int k = 0; k < C::KS; ++k) {
      int d0, d1, d2, d3;  // lo pair (d0,d1), hi pair (d2,d3), relative to this lane's quarter
      if constexpr (BITS == 4) {
        const int w = k >> 1, h = k & 1;
        d0 = 8 * w + 2 * h;
        d1 = d0 + 4;
        d2 = d0 + 1;
        d3 = d0 + 5;
      } else {
        d0 = 4 * k;
        d1 = d0 + 2;
        d2 = d0 + 1;
        d3 = d0 + 3;
      }
      const float v0 = rv ? Elem<T>::to_f32(qr[d0]) * qmul : 0.f;
      const float v1 = rv ? Elem<T>::to_f32(qr[d1]) * qmul : 0.f;
      const float v2 = rv ? Elem<T>::to_f32(qr[d2]) * qmul : 0.f;
      const float v3 = rv ? Elem<T>::to_f32(qr[d3]) * qmul : 0.f;
      qf[nt][k][0] = pack_f16x2(v0, v1);
      qf[nt][k][1] = pack_f16x2(v2, v3);
    }
  }

  float o[NT][C::KS][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < C::KS; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[nt][j][i] = 0.f;
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = kNegInf;
    l_run[nt][0] = l_run[nt][1] = 0.f;
  }

  const int kg = tq * D / 256;  // scale group of this lane's K quarter
  const int vg = gq * D / 512;  // scale group of this lane's V eighth
  const int kr0 = key_perm<BITS>(gq), kr1 = key_perm<BITS>(gq + 8);
  const int vr0 = key_perm<BITS>(2 * tq), vr1 = key_perm<BITS>(2 * tq + 1);
  const int vr2 = key_perm<BITS>(2 * tq + 8), vr3 = key_perm<BITS>(2 * tq + 9);
  const bool any_mask = a.mask_kind != QKV_MASK_NONE;
  const int pb = a.pos_base ? a.pos_base[b] : 0;
  const int tot = a.total_lens ? a.total_lens[b] : len;

  bool ok = true;
  for (int it = 0; it < n_iters; ++it) {
    const int slot = it % C::STAGES;
    ok = mbar_wait(&full_bar[slot], (it / C::STAGES) & 1, a.status, 3);
    if (!ok) break;
    const uint8_t* st = smem + slot * C::STAGE_BYTES;
    const int tile0 = warp * 16;  // this warp's first key row in the stage
    const int p0 = p_begin + it * kTP + tile0;
    if (p0 < p_end) {
      // ---- scores^T = K . Q^T ----------------------------------------------------------
      float s[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      {
        uint32_t kc0[C::KCHUNK / 4], kc1[C::KCHUNK / 4];
        lds_bytes<C::KCHUNK>(kc0, st + C::OFF_KC + (tile0 + kr0) * C::RB + tq * C::KCHUNK);
        lds_bytes<C::KCHUNK>(kc1, st + C::OFF_KC + (tile0 + kr1) * C::RB + tq * C::KCHUNK);
        const float s0 = sc_to_f32<T>(st + C::OFF_KS + ((tile0 + kr0) * C::G + kg) * 2);
        const float s1 = sc_to_f32<T>(st + C::OFF_KS + ((tile0 + kr1) * C::G + kg) * 2);
        const float b0 = sc_to_f32<T>(st + C::OFF_KB + ((tile0 + kr0) * C::G + kg) * 2);
        const float b1 = sc_to_f32<T>(st + C::OFF_KB + ((tile0 + kr1) * C::G + kg) * 2);
        const uint32_t s20 = pack_f16x2(s0, s0), s21 = pack_f16x2(s1, s1);
        const uint32_t b20 = pack_f16x2(b0, b0), b21 = pack_f16x2(b1, b1);
        if constexpr (BITS == 4) {
          const uint32_t t20 = pack_f16x2(s0 * 0.0625f, s0 * 0.0625f);
          const uint32_t t21 = pack_f16x2(s1 * 0.0625f, s1 * 0.0625f);
#pragma unroll
          for (int w = 0; w < C::KCHUNK / 4; ++w) {
            const uint32_t x0 = kc0[w], x1 = kc1[w];
            const uint32_t y0 = x0 >> 8, y1 = x1 >> 8;
            uint32_t af[4];
            af[0] = deq2(and_or(x0, 0x000F000Fu, kMagic), s20, b20);
            af[1] = deq2(and_or(x1, 0x000F000Fu, kMagic), s21, b21);
            af[2] = deq2(and_or(x0, 0x00F000F0u, kMagic), t20, b20);
            af[3] = deq2(and_or(x1, 0x00F000F0u, kMagic), t21, b21);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(s[nt], af, qf[nt][2 * w][0], qf[nt][2 * w][1]);
            af[0] = deq2(and_or(y0, 0x000F000Fu, kMagic), s20, b20);
            af[1] = deq2(and_or(y1, 0x000F000Fu, kMagic), s21, b21);
            af[2] = deq2(and_or(y0, 0x00F000F0u, kMagic), t20, b20);
            af[3] = deq2(and_or(y1, 0x00F000F0u, kMagic), t21, b21);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              mma16816(s[nt], af, qf[nt][2 * w + 1][0], qf[nt][2 * w + 1][1]);
          }
        } else {
#pragma unroll
          for (int w = 0; w < C::KCHUNK / 4; ++w) {
            const uint32_t x0 = kc0[w], x1 = kc1[w];
            uint32_t af[4];
            af[0] = deq2(prmt(x0, kMagic, 0x5250), s20, b20);
            af[1] = deq2(prmt(x1, kMagic, 0x5250), s21, b21);
            af[2] = deq2(prmt(x0, kMagic, 0x5351), s20, b20);
            af[3] = deq2(prmt(x1, kMagic, 0x5351), s21, b21);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(s[nt], af, qf[nt][w][0], qf[nt][w][1]);
          }
        }
      }

      // ---- masking (only tiles that need it) -------------------------------------------
      if (p0 + 16 > p_end || any_mask) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int key = p0 + ((i < 2) ? kr0 : kr1);
            const int r = rbase + nt * 8 + 2 * tq + (i & 1);
            bool keep = key < p_end;
            float add = 0.f;
            if (keep && any_mask && r < R) {
              const int sq = r % a.S;
              if (a.mask_kind == QKV_MASK_CAUSAL) {
                keep = pb + key <= tot - a.S + sq;
              } else {
                const int hq = hkv * gqa + r / a.S;
                const long long off = (long long)b * a.mask_sb + (long long)hq * a.mask_sh +
                                      (long long)sq * a.mask_sq + key;
                if (key >= a.mask_nk) {
                  keep = false;
                } else if (a.mask_kind == QKV_MASK_BOOL) {
                  keep = ((const uint8_t*)a.mask)[off] != 0;
                } else {
                  add = Elem<T>::to_f32(((const T*)a.mask)[off]) * 1.4426950408889634f;
                }
              }
            }
            s[nt][i] = keep ? s[nt][i] + add : kNegInf;
          }
      }

      // ---- online softmax (base 2) -----------------------------------------------------
      uint32_t pf[NT][2];
      bool rescale = false;
      float fac[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float p[4];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float mt = fmaxf(s[nt][c], s[nt][2 + c]);
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
          const float m_new = fmaxf(m_run[nt][c], mt);
          const float m_use = m_new == kNegInf ? 0.f : m_new;
          fac[nt][c] = ex2(m_run[nt][c] - m_use);
          rescale |= m_new != m_run[nt][c];
          p[c] = ex2(s[nt][c] - m_use);
          p[2 + c] = ex2(s[nt][2 + c] - m_use);
          l_run[nt][c] = l_run[nt][c] * fac[nt][c] + (p[c] + p[2 + c]);
          m_run[nt][c] = m_new;
        }
        pf[nt][0] = movmatrix_trans(pack_f16x2(p[0], p[1]));
        pf[nt][1] = movmatrix_trans(pack_f16x2(p[2], p[3]));
      }
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < C::KS; ++j) {
            o[nt][j][0] *= fac[nt][0];
            o[nt][j][1] *= fac[nt][1];
            o[nt][j][2] *= fac[nt][0];
            o[nt][j][3] *= fac[nt][1];
          }
      }

      // ---- out^T += V^T . P^T ------------------------------------------------------------
      {
        uint32_t v0[C::VCHUNK / 4], v1[C::VCHUNK / 4], v2[C::VCHUNK / 4], v3[C::VCHUNK / 4];
        const uint8_t* vc = st + C::OFF_VC + gq * C::VCHUNK;
        lds_bytes<C::VCHUNK>(v0, vc + (tile0 + vr0) * C::RB);
        lds_bytes<C::VCHUNK>(v1, vc + (tile0 + vr1) * C::RB);
        lds_bytes<C::VCHUNK>(v2, vc + (tile0 + vr2) * C::RB);
        lds_bytes<C::VCHUNK>(v3, vc + (tile0 + vr3) * C::RB);
        const uint8_t* vsp = st + C::OFF_VS + vg * 2;
        const uint8_t* vbp = st + C::OFF_VB + vg * 2;
        float sv[4], bv[4];
        sv[0] = sc_to_f32<T>(vsp + (tile0 + vr0) * C::G * 2);
        sv[1] = sc_to_f32<T>(vsp + (tile0 + vr1) * C::G * 2);
        sv[2] = sc_to_f32<T>(vsp + (tile0 + vr2) * C::G * 2);
        sv[3] = sc_to_f32<T>(vsp + (tile0 + vr3) * C::G * 2);
        bv[0] = sc_to_f32<T>(vbp + (tile0 + vr0) * C::G * 2);
        bv[1] = sc_to_f32<T>(vbp + (tile0 + vr1) * C::G * 2);
        bv[2] = sc_to_f32<T>(vbp + (tile0 + vr2) * C::G * 2);
        bv[3] = sc_to_f32<T>(vbp + (tile0 + vr3) * C::G * 2);
        if (p0 + 16 > p_end) {
          // keys past the valid range carry weight 0 but their codes/scales may be
          // anything (padded tail); force finite values so 0 * V stays 0
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int kk = (i == 0) ? vr0 : (i == 1) ? vr1 : (i == 2) ? vr2 : vr3;
            if (p0 + kk >= p_end) sv[i] = bv[i] = 0.f;
          }
        }
        const uint32_t s01 = pack_f16x2(sv[0], sv[1]), s23 = pack_f16x2(sv[2], sv[3]);
        const uint32_t b01 = pack_f16x2(bv[0], bv[1]), b23 = pack_f16x2(bv[2], bv[3]);
        if constexpr (BITS == 4) {
          const uint32_t t01 = pack_f16x2(sv[0] * 0.0625f, sv[1] * 0.0625f);
          const uint32_t t23 = pack_f16x2(sv[2] * 0.0625f, sv[3] * 0.0625f);
#pragma unroll
          for (int u = 0; u < C::VCHUNK / 4; ++u) {
            const uint32_t xa = prmt(v0[u], v1[u], 0x5410), ya = prmt(v0[u], v1[u], 0x7632);
            const uint32_t xb = prmt(v2[u], v3[u], 0x5410), yb = prmt(v2[u], v3[u], 0x7632);
            const uint32_t srcA[4] = {xa, xa >> 8, ya, ya >> 8};
            const uint32_t srcB[4] = {xb, xb >> 8, yb, yb >> 8};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t af[4];
              af[0] = deq2(and_or(srcA[i], 0x000F000Fu, kMagic), s01, b01);
              af[1] = deq2(and_or(srcA[i], 0x00F000F0u, kMagic), t01, b01);
              af[2] = deq2(and_or(srcB[i], 0x000F000Fu, kMagic), s23, b23);
              af[3] = deq2(and_or(srcB[i], 0x00F000F0u, kMagic), t23, b23);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma16816(o[nt][4 * u + i], af, pf[nt][0], pf[nt][1]);
            }
          }
        } else {
#pragma unroll
          for (int u = 0; u < C::VCHUNK / 4; ++u) {
            const uint32_t xa = prmt(v0[u], v1[u], 0x5140), ya = prmt(v0[u], v1[u], 0x7362);
            const uint32_t xb = prmt(v2[u], v3[u], 0x5140), yb = prmt(v2[u], v3[u], 0x7362);
            uint32_t af[4];
            af[0] = deq2(prmt(xa, kMagic, 0x5150), s01, b01);
            af[1] = deq2(prmt(xa, kMagic, 0x5352), s01, b01);
            af[2] = deq2(prmt(xb, kMagic, 0x5150), s23, b23);
            af[3] = deq2(prmt(xb, kMagic, 0x5352), s23, b23);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(o[nt][2 * u], af, pf[nt][0], pf[nt][1]);
            af[0] = deq2(prmt(ya, kMagic, 0x5150), s01, b01);
            af[1] = deq2(prmt(ya, kMagic, 0x5352), s01, b01);
            af[2] = deq2(prmt(yb, kMagic, 0x5150), s23, b23);
            af[3] = deq2(prmt(yb, kMagic, 0x5352), s23, b23);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(o[nt][2 * u + 1], af, pf[nt][0], pf[nt][1]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
  }

  // ---- merge the four warps' partials and write this CTA's partial -------------------
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float l = l_run[nt][c];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      l_run[nt][c] = l;
    }
  named_bar_sync(1, kWarps * 32);  // every consumer is done with the stage ring
  float* mw = reinterpret_cast<float*>(smem);      // [kWarps][RG]
  float* lw = mw + kWarps * RG;                    // [kWarps][RG]
  float* ow = lw + kWarps * RG;                    // [kWarps][RG][D]
  if (gq == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        mw[warp * RG + nt * 8 + 2 * tq + c] = m_run[nt][c];
        lw[warp * RG + nt * 8 + 2 * tq + c] = l_run[nt][c];
      }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < C::KS; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = nt * 8 + 2 * tq + (i & 1);
        const int d = gq * (D / 8) + 2 * j + (i >> 1);
        ow[(warp * RG + r) * D + d] = o[nt][j][i];
      }
  named_bar_sync(1, kWarps * 32);

  const int rows_here = min(RG, R - rbase);
  float* part = (float*)a.workspace + ((size_t)split * a.B * a.HQ * a.S + row0 + rbase) * (D + 4);
  for (int idx = threadIdx.x; idx < rows_here * (D + 4); idx += kWarps * 32) {
    const int r = idx / (D + 4), d = idx - r * (D + 4);
    float mx = kNegInf;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, mw[w * RG + r]);
    const float mu = mx == kNegInf ? 0.f : mx;
    float acc = 0.f;
    if (d < D) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) acc += ex2(mw[w * RG + r] - mu) * ow[(w * RG + r) * D + d];
    } else if (d == D) {
      acc = mx;
    } else if (d == D + 1) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) acc += ex2(mw[w * RG + r] - mu) * lw[w * RG + r];
    }
    part[(size_t)r * (D + 4) + d] = acc;
  }
}

// One CTA (8 warps) per output row. The split maxima are reduced by all threads at once;
// then warp w folds splits w, w+8, ... with its lanes owning D/32 columns, and the eight
// warp sums meet in shared memory. Independent loads keep many L2 requests in flight.
constexpr int kCombineWarps = 8;

template <typename TO, int D>
__global__ void __launch_bounds__(kCombineWarps * 32)
    combine_kernel(const float* __restrict__ parts, int n_parts, long long part_stride_rows,
                   long long rows, TO* __restrict__ out, float* __restrict__ out_part) {
  constexpr int E = D / 32;
  __shared__ float red[kCombineWarps][D];
  __shared__ float wmax[kCombineWarps], wsum[kCombineWarps];
  const long long row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = parts + row * (D + 4);
  const size_t pstride = (size_t)part_stride_rows * (D + 4);

  float mx = kNegInf;
  for (int p = threadIdx.x; p < n_parts; p += blockDim.x) mx = fmaxf(mx, base[p * pstride + D]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) wmax[warp] = mx;
  __syncthreads();
  mx = wmax[0];
#pragma unroll
  for (int w = 1; w < kCombineWarps; ++w) mx = fmaxf(mx, wmax[w]);
  const float mu = mx == kNegInf ? 0.f : mx;

  float l = 0.f;
  for (int p = threadIdx.x; p < n_parts; p += blockDim.x) {
    const float* pr = base + p * pstride;
    l += ex2(pr[D] - mu) * pr[D + 1];
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) wsum[warp] = l;

  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
#pragma unroll 4
  for (int p = warp; p < n_parts; p += kCombineWarps) {
    const float* pr = base + p * pstride;
    const float f = ex2(pr[D] - mu);
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] += f * pr[lane * E + e];
  }
#pragma unroll
  for (int e = 0; e < E; ++e) red[warp][lane * E + e] = acc[e];
  __syncthreads();
  l = 0.f;
#pragma unroll
  for (int w = 0; w < kCombineWarps; ++w) l += wsum[w];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) v += red[w][d];
    if (out_part) {
      out_part[row * (D + 4) + d] = v;
    } else {
      out[row * D + d] = Elem<TO>::from_f32(l == 0.f ? v : v / l);
    }
  }
  if (out_part && threadIdx.x == 0) {
    float* dst = out_part + row * (D + 4);
    dst[D] = mx;
    dst[D + 1] = l;
    dst[D + 2] = 0.f;
    dst[D + 3] = 0.f;
  }
}

template <typename T, int BITS, int D, int NT>
int launch_split(const AttnArgs& a, cudaStream_t st) {
  using C = Cfg<T, BITS, D>;
  const int R = (a.HQ / a.HKV) * a.S;
  const int RG = 8 * NT;
  const int row_groups = (R + RG - 1) / RG;
  const size_t ring = (size_t)C::STAGES * C::STAGE_BYTES;
  const size_t merge = (size_t)kWarps * RG * (D + 2) * 4;
  const size_t smem = std::max(ring, merge);
  auto kern = decode_split_kernel<T, BITS, D, NT>;
  static unsigned attr_done = 0;  // one bit per device, per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done & (1u << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return QKV_ECUDA;
    attr_done |= 1u << (dev & 31);
  }
  dim3 grid(a.splits, a.HKV * row_groups, a.B);
  kern<<<grid, kThreads, smem, st>>>(a);
  return QKV_OK;
}

template <typename T, int BITS, int NT>
int launch_split_d(const AttnArgs& a, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_split<T, BITS, 64, NT>(a, st);
    case 128: return launch_split<T, BITS, 128, NT>(a, st);
    case 256: return launch_split<T, BITS, 256, NT>(a, st);
    default: return QKV_EUNSUPPORTED;
  }
}

template <typename T, int NT>
int launch_split_b(const AttnArgs& a, cudaStream_t st) {
  return a.bits == 4 ? launch_split_d<T, 4, NT>(a, st) : launch_split_d<T, 8, NT>(a, st);
}

}  // namespace

int decode_rows_per_group(int R) { return R <= 8 ? 8 : 16; }

void decode_pick_split(int B, int HKV, int row_groups, int n_max, int* splits, int* chunk) {
  const int units = std::max(1, B * HKV * row_groups);
  const int target = 2 * num_sms();  // two resident CTAs per SM, one wave
  int sp = std::max(1, (target + units - 1) / units);
  const int max_sp = std::max(1, (n_max + kTP - 1) / kTP);
  sp = std::min(sp, max_sp);
  int ch = (n_max + sp - 1) / sp;
  ch = std::max(kTP, (ch + kTP - 1) / kTP * kTP);
  *chunk = ch;
  *splits = std::max(1, (n_max + ch - 1) / ch);
}

size_t decode_workspace_bytes(int B, int HQ, int HKV, int S, int D, int splits) {
  (void)HKV;
  return (size_t)splits * B * HQ * S * (D + 4) * sizeof(float);
}

int launch_split_only(const AttnArgs& a, cudaStream_t st) {
  const int R = (a.HQ / a.HKV) * a.S;
  if (a.dtype == QKV_BF16)
    return R <= 8 ? launch_split_b<__nv_bfloat16, 1>(a, st) : launch_split_b<__nv_bfloat16, 2>(a, st);
  return R <= 8 ? launch_split_b<__half, 1>(a, st) : launch_split_b<__half, 2>(a, st);
}

int launch_decode(const AttnArgs& a, cudaStream_t st) {
  const int rc = launch_split_only(a, st);
  if (rc != QKV_OK) return rc;
  const long long rows = (long long)a.B * a.HQ * a.S;
  return launch_combine((const float*)a.workspace, a.splits, rows, rows, a.D, a.out, a.dtype,
                        a.out_kind, st);
}

int launch_combine(const float* parts, int n_parts, long long part_stride_rows, long long rows,
                   int D, void* out, int out_dtype, int out_kind, cudaStream_t st) {
  if (rows == 0) return QKV_OK;
  const int warps = kCombineWarps;
  const unsigned grid = (unsigned)rows;
  float* op = out_kind == QKV_OUT_PARTIAL ? (float*)out : nullptr;
#define QKV_C_CASE(DD)                                                                       \
  case DD:                                                                                   \
    if (out_dtype == QKV_BF16)                                                               \
      combine_kernel<__nv_bfloat16, DD><<<grid, warps * 32, 0, st>>>(                        \
          parts, n_parts, part_stride_rows, rows, (__nv_bfloat16*)out, op);                  \
    else                                                                                     \
      combine_kernel<__half, DD><<<grid, warps * 32, 0, st>>>(parts, n_parts,                \
                                                              part_stride_rows, rows,        \
                                                              (__half*)out, op);             \
    break;
  switch (D) {
    QKV_C_CASE(64)
    QKV_C_CASE(128)
    QKV_C_CASE(256)
    default:
      return QKV_EUNSUPPORTED;
  }
#undef QKV_C_CASE
  return QKV_OK;
}

}  // namespace qkv
