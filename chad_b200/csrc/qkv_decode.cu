// Split-KV attention over the MLX-layout quantized KV cache, sm_100a.
//
// Replaces the reference's pass 1 (`_P1_SRC`, src/chad/mlx_qsdpa.py:73-209, and its
// simdgroup-matrix retile `_P1_SGM_SRC`, :303-473) and pass 2 (`_P2_SRC`, :213-265).
//
// Work split. One CTA = one (batch b, kv head, query-row group, key split); its query rows
// are the GQA heads x query tokens that share the kv head (8 or 16, contiguous in q). With
// per-batch lengths and an in-kernel merge, the CTAs of a (kv head, row group) are shared
// by the batches in proportion to their key counts instead (balanced mode).
//
// Memory path. A producer warp streams stages of 64 or 128 keys into a shared-memory ring:
// K and V code tiles with 3-D TMA tensor copies (swizzled so that every consumer read below
// is free of bank conflicts) and the four scale/bias arrays with 1-D bulk copies, all
// completing on mbarriers. No multicast.
//
// Math. Four consumer warps take 16 (or 2 x 16) keys each per stage and run mma.sync
// m16n8k16 with the 16 KEYS as the M rows and the query rows as the N columns (GQA 8 fills
// N=8 exactly). The packed codes are fed to the tensor cores as they are: AND-ing a 4-bit
// code into the low bits of an f16 (or placing an 8-bit code there with PRMT) gives the
// subnormal f16 value code * 2^-24 exactly, and B200's f16 MMA is exact on subnormal
// inputs. Because every k-step of QK (and every m-tile of PV) stays inside one 64-wide
// scale group, the affine parameters factor out of the products:
//   score(key, row)  = sum_g s[key,g] * 2^24 * (codes_g . q_g)  +  sum_g b[key,g] * sum(q_g)
//   out(dim g, row) += 2^24 * sum_key (p * s[key,g]) * code  +  sum_key p * b[key,g]
// so no per-element dequantisation arithmetic is left: per code the kernel spends one
// LOP3/PRMT (4-bit: one per two codes) and the tensor cores do the rest. P^T is built from
// the score accumulator with movmatrix.trans (no shared-memory round trip).
//
// Reduction. Online softmax in base 2; the four warps merge through shared memory into one
// CTA partial (out, max, sum), which the CTA stores to the workspace as self-validating
// words (see store_part). The last splits of each row group then merge every split's
// partial inside the same kernel, one (row, 32-dim slice) unit per merging CTA, and write
// the output: the reference's pass 2 without a second launch. qkv_partials stops after the
// stores (plain floats) and leaves the merge to combine_kernel, which also serves the
// cross-GPU merge and grids too large to be resident in one wave.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "qkv_common.cuh"
#include "qkv_internal.h"
#include "quant_row.cuh"

namespace qkv {

namespace {

constexpr int kWarps = 4;                    // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + producer warp
constexpr int kBoxRows = 64;                 // key rows per TMA box
constexpr float kLazyLog2 = 4.0f;  // softmax max is only raised when exceeded by 2^4
// Stages a CTA requests before the dependency wait. One: the CTAs of the next layer start
// while this layer's merge is still polling L2, and a deeper early request floods the
// memory system right then (measured on the 32K decode, 8-bit: 13.66 us per layer with the
// whole ring requested early, 13.04 with two stages, 12.62 with one, 13.83 with none).
constexpr int kPreStages = 1;
constexpr int kMergeCols = 8;                     // float4 columns of one merge unit (32 dims)
constexpr int kMergeSlots = kThreads / kMergeCols;  // partial subsets merged side by side
constexpr int kMaxSplits = 256;              // bounds the merge's loads per thread
#define kNegInf (-__int_as_float(0x7f800000))

// Order in which the 16 keys of a warp tile occupy the MMA rows. The tables make the rows
// that one shared-memory wavefront reads land in distinct bank windows of the swizzled tile
// (64-byte rows / 64B swizzle for 4-bit D128, 128-byte rows / 128B swizzle for 8-bit).
template <int BITS>
__device__ __forceinline__ int key_perm(int k) {
  const int lo = k & 7;
  const int p = BITS == 4 ? (0x76234510 >> (4 * lo)) & 7   // 0,1,5,4,3,2,6,7
                          : (0x37156240 >> (4 * lo)) & 7;  // 0,4,2,6,5,1,7,3
  return (k & 8) | p;
}

// Per-instantiation shape of the decode kernel.
//   SUB   16-key sub-tiles per consumer warp per stage: two where registers allow, so a
//         warp runs two independent MMA chains and shares one softmax reduction.
//   CTAS  CTAs resident per SM (register cap through __launch_bounds__).
//   RING  shared-memory budget of the stage ring, so that CTAS CTAs fit in the SM's
//         228 KB with their static arrays, the alignment slack and 1 KB reserved each.
template <int BITS, int D, int NT>
struct DecodeCfg {
  static constexpr bool kNarrow = NT == 1 && D <= 128;
  static constexpr int SUB = kNarrow && BITS == 4 ? 2 : 1;
  static constexpr int CTAS = kNarrow && BITS == 8 ? 3 : 2;
  static constexpr int TP = 64 * SUB;  // keys per stage
  static constexpr int RING = CTAS == 3 ? 64 * 1024 : 104 * 1024;
};

template <int BITS, int D, int TP, int RING = 72 * 1024>
struct Geo {
  static constexpr int G = D / 64;                   // scale groups per row
  static constexpr int RB = D * BITS / 8;            // code bytes per key
  static constexpr int RBOX = RB < 128 ? RB : 128;   // TMA box inner bytes (swizzle span)
  static constexpr int NBOX = RB / RBOX;             // boxes per code row
  static constexpr int SWZ = RBOX == 128 ? 7 : RBOX == 64 ? 3 : 1;
  static constexpr int GB = 64 * BITS / 8;           // code bytes of one scale group
  static constexpr int KLB = 16 * BITS / 8;          // K bytes per lane per group per key
  static constexpr int VLB = 8 * BITS / 8;           // V bytes per lane per group per key
  static constexpr int KW = KLB / 4, VW = VLB / 4;   // words
  static constexpr int CODE_BYTES = TP * RB;
  static constexpr int SC_BYTES = TP * G * 2;
  static constexpr int OFF_KC = 0;
  static constexpr int OFF_VC = CODE_BYTES;
  static constexpr int OFF_KS = 2 * CODE_BYTES;
  static constexpr int OFF_KB = OFF_KS + SC_BYTES;
  static constexpr int OFF_VS = OFF_KB + SC_BYTES;
  static constexpr int OFF_VB = OFF_VS + SC_BYTES;
  static constexpr int STAGE_BYTES = ((OFF_VB + SC_BYTES) + 1023) / 1024 * 1024;
  static constexpr int STAGES = STAGE_BYTES * 4 <= RING ? 4 : STAGE_BYTES * 3 <= RING ? 3 : 2;
};

// Byte offset of (key row, code byte) inside a swizzled code tile.
template <int BITS, int D, int TP, int RING>
__device__ __forceinline__ int code_off(int key, int byte) {
  using g = Geo<BITS, D, TP, RING>;
  const int sub = byte / g::RBOX;
  const int lin = key * g::RBOX + (byte % g::RBOX);
  return sub * (TP * g::RBOX) + (lin ^ (((lin >> 7) & g::SWZ) << 4));
}

template <int N>
__device__ __forceinline__ void lds_words(uint32_t* dst, const uint8_t* src) {
  if constexpr (N == 1) {
    dst[0] = *reinterpret_cast<const uint32_t*>(src);
  } else if constexpr (N == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    dst[0] = v.x;
    dst[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      dst[4 * i + 0] = v.x;
      dst[4 * i + 1] = v.y;
      dst[4 * i + 2] = v.z;
      dst[4 * i + 3] = v.w;
    }
  }
}

// G consecutive scale-dtype values of one key row -> float.
template <typename T, int G>
__device__ __forceinline__ void lds_scales(float* dst, const uint8_t* src) {
  const uint16_t* p = reinterpret_cast<const uint16_t*>(src);
  if constexpr (G == 1) {
    dst[0] = Elem<T>::bits_to_f32(p[0]);
  } else if constexpr (G == 2) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(src);
    dst[0] = Elem<T>::bits_to_f32((uint16_t)(w & 0xffffu));
    dst[1] = Elem<T>::bits_to_f32((uint16_t)(w >> 16));
  } else {
    const uint2 w = *reinterpret_cast<const uint2*>(src);
    dst[0] = Elem<T>::bits_to_f32((uint16_t)(w.x & 0xffffu));
    dst[1] = Elem<T>::bits_to_f32((uint16_t)(w.x >> 16));
    dst[2] = Elem<T>::bits_to_f32((uint16_t)(w.y & 0xffffu));
    dst[3] = Elem<T>::bits_to_f32((uint16_t)(w.y >> 16));
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Partial rows of the in-kernel merge are stored as (float bits) ^ kPartKey, so that a word
// reads 0 until its value has landed: kPartKey is a signalling-NaN pattern, and arithmetic
// only ever produces quiet NaNs, so no stored value encodes to 0. The merger that reads a
// word writes 0 back; the workspace is zero before the first call and after every call.
constexpr unsigned kPartKey = 0x7FBADBADu;

// Two consecutive floats of a partial row: encoded (merge mode, workspace) or plain
// (partials handed to the caller).
__device__ __forceinline__ void store_part(float* dst, float x, float y, int encoded) {
  if (encoded)
    __stcg(reinterpret_cast<uint2*>(dst),
           make_uint2(__float_as_uint(x) ^ kPartKey, __float_as_uint(y) ^ kPartKey));
  else
    *reinterpret_cast<float2*>(dst) = make_float2(x, y);
}

struct DecodeParams {
  AttnArgs a;
  CUtensorMap tmk;  // K codes: (RB bytes, NP, B*HKV)
  CUtensorMap tmv;  // V codes
  float* gpart;     // per-CTA partial rows [splits][B*HQ*S][D+4], or [..][D+2*D/32] encoded
  int merge;        // 1: the row group's last splits merge the partials into a.out
  int phantom;      // test hook: partial sets the mergers wait for that no CTA writes
  unsigned long long spin_ns;  // bound on the merge's polling (kSpinNanos unless a test
                               // hook shortens it)
};

template <typename T, int BITS, int D, int NT>
__global__ void __launch_bounds__(kThreads, DecodeCfg<BITS, D, NT>::CTAS) decode_kernel(const __grid_constant__ DecodeParams P) {
  using CF = DecodeCfg<BITS, D, NT>;
  constexpr int kSub = CF::SUB;
  constexpr int kTP = CF::TP;  // keys per stage
  using GG = Geo<BITS, D, kTP, CF::RING>;
  constexpr int G = GG::G;
  constexpr int RG = 8 * NT;  // query rows per CTA
  constexpr int KS = 4;       // k-steps (and m-tiles) per scale group
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // swizzled TMA tiles need 1024-byte aligned stage buffers: align by hand
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full_bar[4], empty_bar[4];

  const AttnArgs& a = P.a;
  // Programmatic dependent launch: the next kernel in the stream may be scheduled as soon as
  // every CTA of this one has started. Reads of anything a predecessor may still be writing
  // wait for griddepcontrol.wait below; only the producer's first stages of cache positions
  // below a.prefetch_limit (older than the tokens appended by the predecessor) go earlier.
  asm volatile("griddepcontrol.launch_dependents;");
  int split = blockIdx.x;  // (balanced mode: batch and split follow from the lengths below)
  const int hkv = blockIdx.y % a.HKV;
  const int rg = blockIdx.y / a.HKV;
  int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = lane >> 2;  // MMA group id
  const int tq = lane & 3;   // thread in group

  const int gqa = a.HQ / a.HKV;
  const int R = gqa * a.S;  // query rows sharing this kv head
  int chunk = a.chunk;
  int p_begin = split * chunk;
  long long bh = (long long)b * a.HKV + hkv;
  long long row0 = ((long long)b * a.HQ + (long long)hkv * gqa) * a.S;  // first q row
  const int rbase = rg * RG;
  const int rows_here = min(RG, R - rbase);

  if (threadIdx.x == 0) {
    for (int s = 0; s < GG::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // stage issue (producer lane 0); returns false if a bounded wait ran out
  auto issue_stage = [&](int it) {
    const int slot = it % GG::STAGES;
    const int p0 = p_begin + it * kTP;
    const int rows = min(kTP, a.NP - p0);
    const uint32_t sb = rows * G * 2;
    uint8_t* st = smem + slot * GG::STAGE_BYTES;
    const uint8_t* ks = (const uint8_t*)a.ks + (bh * a.NP + p0) * G * 2;
    const uint8_t* kb = (const uint8_t*)a.kb + (bh * a.NP + p0) * G * 2;
    const uint8_t* vs = (const uint8_t*)a.vs + (bh * a.NP + p0) * G * 2;
    const uint8_t* vb = (const uint8_t*)a.vb + (bh * a.NP + p0) * G * 2;
    // boxes of kBoxRows keys; boxes that start past the cache's end are not issued
    const int boxes = (rows + kBoxRows - 1) / kBoxRows;
    mbar_arrive_expect_tx(&full_bar[slot], 2 * GG::NBOX * boxes * kBoxRows * GG::RBOX + 4 * sb);
#pragma unroll
    for (int bx = 0; bx < GG::NBOX; ++bx) {
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        if (j < boxes) {
          const int off = bx * kTP * GG::RBOX + j * kBoxRows * GG::RBOX;
          tma_load_3d(st + GG::OFF_KC + off, &P.tmk, bx * GG::RBOX, p0 + j * kBoxRows, (int)bh,
                      &full_bar[slot]);
          tma_load_3d(st + GG::OFF_VC + off, &P.tmv, bx * GG::RBOX, p0 + j * kBoxRows, (int)bh,
                      &full_bar[slot]);
        }
      }
    }
    bulk_g2s(st + GG::OFF_KS, ks, sb, &full_bar[slot]);
    bulk_g2s(st + GG::OFF_KB, kb, sb, &full_bar[slot]);
    bulk_g2s(st + GG::OFF_VS, vs, sb, &full_bar[slot]);
    bulk_g2s(st + GG::OFF_VB, vb, sb, &full_bar[slot]);
  };
  int pre = 0;  // stages issued before the dependency wait
  if (warp == kWarps && lane == 1 && !a.balanced) {
    // Warm L2 with this CTA's query rows: the loads after the dependency wait then hit L2
    // instead of queueing in HBM behind the KV stream. L2 is the point of coherence, so a
    // predecessor that writes q after this hint still has its values read below.
    prefetch_l2((const uint8_t*)a.q + (row0 + rbase) * D * 2, (uint32_t)(rows_here * D * 2));
  }
  if (warp == kWarps && lane == 0 && !a.lens) {
    const int len0 = min(max(a.n, 0), a.NP);
    const int end0 = min(p_begin + a.chunk, len0);
    const int it0 = end0 > p_begin ? (end0 - p_begin + kTP - 1) / kTP : 0;
    while (pre < kPreStages && pre < GG::STAGES && pre < it0 &&
           p_begin + (pre + 1) * kTP <= a.prefetch_limit)
      issue_stage(pre++);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int nsplit = gridDim.x;  // splits of this CTA's batch
  int pset = 0;            // partial set of the batch's split 0
  if (a.balanced) {
    // Ragged lengths: the gridDim.x CTAs of a (kv head, row group) are shared by all batches
    // in proportion to their key counts. chunk = total keys / a.balanced, rounded up to whole
    // stages; batch b takes max(1, ceil(len_b / chunk)) consecutive CTAs, which sum to at
    // most a.balanced + B = gridDim.x. Lengths are read only after the dependency wait.
    long long total = 0;
    for (int bb = 0; bb < a.B; ++bb) total += min(max(a.lens[bb], 0), a.NP);
    const long long per = (total + a.balanced - 1) / a.balanced;
    chunk = (int)max((long long)kTP, (per + kTP - 1) / kTP * kTP);
    int first_cta = 0;
    b = -1;
    for (int bb = 0; bb < a.B; ++bb) {
      const int lb = min(max(a.lens[bb], 0), a.NP);
      const int cb = max(1, (lb + chunk - 1) / chunk);
      if (b < 0 && (int)blockIdx.x < first_cta + cb) {
        b = bb;
        split = blockIdx.x - first_cta;
        nsplit = cb;
        pset = first_cta;
      }
      first_cta += cb;
    }
    if (b < 0) return;  // a spare CTA: every batch is covered (uniform across the CTA)
    p_begin = split * chunk;
    bh = (long long)b * a.HKV + hkv;
    row0 = ((long long)b * a.HQ + (long long)hkv * gqa) * a.S;
  }
  int len = a.lens ? a.lens[b] : a.n;
  len = min(max(len, 0), a.NP);
  const int p_end = min(p_begin + chunk, len);
  const int n_iters = p_end > p_begin ? (p_end - p_begin + kTP - 1) / kTP : 0;
  // Partial rows: [set][rows][PW] floats, see store_part for the merge mode's encoding. A
  // set is one split of all batches (rows = B*HQ*S), or in balanced mode one CTA of one
  // batch (rows = HQ*S, the batch's splits are sets pset .. pset + nsplit - 1).
  constexpr int kSlices = D / (4 * kMergeCols);
  const int PW = P.merge ? D + 2 * kSlices : D + 4;
  const size_t prows = a.balanced ? (size_t)a.HQ * a.S : (size_t)a.B * a.HQ * a.S;
  const long long prow0 = a.balanced ? (long long)hkv * gqa * a.S : row0;  // row0 within a set

  // merge area (reuses the stage ring once the main loop is over)
  float* mw = reinterpret_cast<float*>(smem);  // [kWarps][RG] running max per warp
  float* lw = mw + kWarps * RG;                // [kWarps][RG] sums
  float* ow = lw + kWarps * RG;                // [kWarps][RG*D] outputs, fragment order
  float* xm = ow + kWarps * RG * D;            // merge: [kMergeSlots][kMergeCols] running max
  float* xl = xm + kMergeSlots * kMergeCols;   // merge: [kMergeSlots][kMergeCols] sums
  float* xo = xl + kMergeSlots * kMergeCols;   // merge: [kMergeSlots][kMergeCols][4] outputs

  if (warp == kWarps) {
    // ------------------------------ producer -------------------------------------------
    if (a.k_new) {
      // Fused append (one query-row group per kv head, so one CTA per key range): this CTA
      // quantizes the new tokens that fall in its key range into the cache, with the same
      // arithmetic as qkv_quantize_append, before its TMA reads them. The stages issued
      // before the dependency wait stop short of these positions.
      const int lo = max(a.new_pos, p_begin), hi = min(a.new_pos + a.S, p_end);
      for (int pos = lo; pos < hi; ++pos) {
        const long long src = (bh * a.S + (pos - a.new_pos)) * D;
        const long long dst = bh * a.NP + pos;
        quantize_row_warp<T, T, BITS, D>(
            (const T*)a.k_new + src, (uint32_t*)a.kw + dst * (D * BITS / 32),
            (T*)a.ks + dst * (D / 64), (T*)a.kb + dst * (D / 64), lane);
        quantize_row_warp<T, T, BITS, D>(
            (const T*)a.v_new + src, (uint32_t*)a.vw + dst * (D * BITS / 32),
            (T*)a.vs + dst * (D / 64), (T*)a.vb + dst * (D / 64), lane);
      }
      // the rows written through the generic proxy are read below by TMA (async proxy)
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
    }
    if (lane == 0) {
      bool ok = true;
      for (int it = pre; it < n_iters && ok; ++it) {
        const int slot = it % GG::STAGES;
        if (it >= GG::STAGES)
          ok = mbar_wait(&empty_bar[slot], ((it / GG::STAGES) - 1) & 1, a.status, 11);
        if (!ok) break;
        issue_stage(it);
      }
      // every issued stage lands before the ring is reused for the merge
      for (int it = max(0, n_iters - GG::STAGES); it < n_iters; ++it)
        mbar_wait(&full_bar[it % GG::STAGES], (it / GG::STAGES) & 1, a.status, 12);
    }
    __syncwarp();
  } else {
    // -------------------------------- consumers -----------------------------------------
    const T* qg = (const T*)a.q;
    const float qmul = a.scale * 1.4426950408889634f;  // softmax in base 2
    // Q as the B operand of QK, per scale group: k = head_dim pairs in this lane's code
    // order (the 4-bit "x16" slots pre-divided by 16), n = query row. A lane's fragments of
    // one group are the 16 consecutive head dims 64g + 16tq .. +15 of row gq: two 16-byte
    // loads straight from global memory, all issued before any is used. The group sums of
    // the same f16 values feed the bias term.
    uint32_t qf[NT][G][KS][2];
    float qsum_mine[NT][G];
    uint4 raw[NT][G][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int r = rbase + nt * 8 + gq;
      const bool rv = r < R;
      const T* qr = qg + (row0 + (rv ? r : 0)) * D;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint4* src = reinterpret_cast<const uint4*>(qr + 64 * g + 16 * tq);
        raw[nt][g][0] = rv ? src[0] : make_uint4(0u, 0u, 0u, 0u);
        raw[nt][g][1] = rv ? src[1] : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    // The f16 MMA operands hold q * scale * log2(e). A query whose products reach 2^14 (far
    // beyond any activation a model produces, but possible in bf16) would leave f16's range:
    // then, and only then, the CTA scales them by a power of two 2^-qsh that brings the
    // largest magnitude of its rows into [2^13, 2^14), and folds 2^qsh back into the score's
    // scale factor (kmul) and the bias sums. Every warp loads the same rows, so the decision
    // and qsh are the same in all of them.
    float lmax = 0.f;          // this lane's largest |q * scale * log2(e) * 2^-qsh|
    float kmul = 16777216.0f;  // 2^(24+qsh)
    float bmul = 1.f;          // 2^qsh
    auto convert = [&](float qmul_n) {
  #pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
  #pragma unroll
        for (int g = 0; g < G; ++g) {
          const uint32_t w[8] = {raw[nt][g][0].x, raw[nt][g][0].y, raw[nt][g][0].z,
                                 raw[nt][g][0].w, raw[nt][g][1].x, raw[nt][g][1].y,
                                 raw[nt][g][1].z, raw[nt][g][1].w};
          auto qv = [&](int d) {  // dim d of the 16-dim slice, scaled, rounded to f16
            const uint32_t bitsv = (d & 1) ? (w[d >> 1] >> 16) : (w[d >> 1] & 0xffffu);
            const float x = Elem<T>::bits_to_f32((uint16_t)bitsv) * qmul_n;
            lmax = fmaxf(lmax, fabsf(x));
            return __half2float(__float2half_rn(x));
          };
          float acc = 0.f;
  #pragma unroll
          for (int k = 0; k < KS; ++k) {
            int d0, d1, d2, d3;
            if constexpr (BITS == 4) {
              const int u = k >> 1, h = k & 1;
              d0 = 8 * u + 2 * h;
              d1 = d0 + 4;
              d2 = d0 + 1;
              d3 = d0 + 5;
            } else {
              d0 = 4 * k;
              d1 = d0 + 2;
              d2 = d0 + 1;
              d3 = d0 + 3;
            }
            const float v0 = qv(d0), v1 = qv(d1), v2 = qv(d2), v3 = qv(d3);
            acc += (v0 + v1) + (v2 + v3);
            const float hs = BITS == 4 ? 0.0625f : 1.f;
            qf[nt][g][k][0] = pack_f16x2(v0, v1);
            qf[nt][g][k][1] = pack_f16x2(v2 * hs, v3 * hs);
          }
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          acc += __shfl_xor_sync(0xffffffffu, acc, 2);
          qsum_mine[nt][g] = acc * bmul;  // for row nt*8 + gq, in true (unshifted) units
        }
      }
    };
    convert(qmul);
    if (__any_sync(0xffffffffu, lmax >= 16384.f)) {
      float qmax = lmax;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, off));
      const int qsh = min(max((int)((__float_as_uint(qmax) >> 23) & 0xffu) - 127 - 13, 0), 100);
      kmul = __uint_as_float((uint32_t)(127 + 24 + qsh) << 23);
      bmul = __uint_as_float((uint32_t)(127 + qsh) << 23);
      convert(qmul * __uint_as_float((uint32_t)(127 - qsh) << 23));
    }
    // this lane's score columns are rows 2*tq, 2*tq+1 of each n-tile
    float qsum[NT][2][G];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        qsum[nt][0][g] = __shfl_sync(0xffffffffu, qsum_mine[nt][g], 8 * tq);
        qsum[nt][1][g] = __shfl_sync(0xffffffffu, qsum_mine[nt][g], 8 * tq + 4);
      }

    float o[NT][G * KS][4];
    float obias[NT][2][G];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < G * KS; ++j) o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int g = 0; g < G; ++g) obias[nt][c][g] = 0.f;
    }
    float m_run[NT][2], l_run[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = kNegInf;
      l_run[nt][0] = l_run[nt][1] = 0.f;
    }

    // P * (V group scale) is an f16 MMA operand, with P <= 2^kLazyLog2: group scales above
    // 2^11 would overflow it. This warp then scales its V operands by 2^-vsh (a power of
    // two, raised as larger scales appear, with the accumulators rescaled to match) and
    // multiplies the output back by 2^vsh. Ordinary data never takes that branch.
    float vmul = 1.f;  // 2^-vsh

    const int kA = key_perm<BITS>(gq), kB = key_perm<BITS>(gq + 8);
    const int v0k = key_perm<BITS>(2 * tq), v1k = key_perm<BITS>(2 * tq + 1);
    const int v2k = key_perm<BITS>(2 * tq + 8), v3k = key_perm<BITS>(2 * tq + 9);
    const bool any_mask = a.mask_kind != QKV_MASK_NONE;
    const bool causal = a.mask_kind == QKV_MASK_CAUSAL;
    const bool array_mask = any_mask && !causal;
    const int pb = a.pos_base ? a.pos_base[b] : 0;
    const int tot = a.total_lens ? a.total_lens[b] : len;

    // Each warp owns 2 x 16 consecutive keys of every stage. The two sub-tiles run their
    // products as independent MMA chains and share one softmax max-reduction.
    for (int it = 0; it < n_iters; ++it) {
      const int slot = it % GG::STAGES;
      if (!mbar_wait(&full_bar[slot], (it / GG::STAGES) & 1, a.status, 13)) break;
      const uint8_t* st = smem + slot * GG::STAGE_BYTES;
      const int t0 = warp * (16 * kSub);  // this warp's first key row in the stage
      const int p0 = p_begin + it * kTP + t0;
      if (p0 < p_end) {
        const bool tail = p0 + 16 * kSub > p_end;
        // ---- scores^T = codes(K) . Q^T per scale group, both sub-tiles ------------------
        float acc[kSub][NT][G][4];
#pragma unroll
        for (int h = 0; h < kSub; ++h)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int g = 0; g < G; ++g)
              acc[h][nt][g][0] = acc[h][nt][g][1] = acc[h][nt][g][2] = acc[h][nt][g][3] = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int h = 0; h < kSub; ++h) {
            uint32_t wa[GG::KW], wb[GG::KW];
            lds_words<GG::KW>(wa, st + GG::OFF_KC + code_off<BITS, D, kTP, CF::RING>(t0 + 16 * h + kA, g * GG::GB + tq * GG::KLB));
            lds_words<GG::KW>(wb, st + GG::OFF_KC + code_off<BITS, D, kTP, CF::RING>(t0 + 16 * h + kB, g * GG::GB + tq * GG::KLB));
            if constexpr (BITS == 4) {
#pragma unroll
              for (int u = 0; u < GG::KW; ++u) {
                const uint32_t ya = wa[u] >> 8, yb = wb[u] >> 8;
                uint32_t af[4];
                af[0] = wa[u] & 0x000F000Fu;
                af[1] = wb[u] & 0x000F000Fu;
                af[2] = wa[u] & 0x00F000F0u;
                af[3] = wb[u] & 0x00F000F0u;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(acc[h][nt][g], af, qf[nt][g][2 * u][0], qf[nt][g][2 * u][1]);
                af[0] = ya & 0x000F000Fu;
                af[1] = yb & 0x000F000Fu;
                af[2] = ya & 0x00F000F0u;
                af[3] = yb & 0x00F000F0u;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(acc[h][nt][g], af, qf[nt][g][2 * u + 1][0], qf[nt][g][2 * u + 1][1]);
              }
            } else {
#pragma unroll
              for (int u = 0; u < GG::KW; ++u) {
                uint32_t af[4];
                af[0] = prmt(wa[u], 0u, 0x4240);
                af[1] = prmt(wb[u], 0u, 0x4240);
                af[2] = prmt(wa[u], 0u, 0x4341);
                af[3] = prmt(wb[u], 0u, 0x4341);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma16816(acc[h][nt][g], af, qf[nt][g][u][0], qf[nt][g][u][1]);
              }
            }
          }
        }
        float s[kSub][NT][4];
#pragma unroll
        for (int h = 0; h < kSub; ++h) {
          float ksA[G], kbA[G], ksB[G], kbB[G];
          lds_scales<T, G>(ksA, st + GG::OFF_KS + (t0 + 16 * h + kA) * G * 2);
          lds_scales<T, G>(ksB, st + GG::OFF_KS + (t0 + 16 * h + kB) * G * 2);
          lds_scales<T, G>(kbA, st + GG::OFF_KB + (t0 + 16 * h + kA) * G * 2);
          lds_scales<T, G>(kbB, st + GG::OFF_KB + (t0 + 16 * h + kB) * G * 2);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float v = 0.f;
#pragma unroll
              for (int g = 0; g < G; ++g) {
                const float sc = (i < 2 ? ksA[g] : ksB[g]) * kmul;
                const float bi = i < 2 ? kbA[g] : kbB[g];
                v = fmaf(sc, acc[h][nt][g][i], fmaf(bi, qsum[nt][i & 1][g], v));
              }
              s[h][nt][i] = v;
            }
        }

        // ---- masking (only tiles that need it: a causal mask hides nothing before the
        // first query row's position) ----------------------------------------------------
        if (tail || array_mask || (causal && pb + p0 + 16 * kSub - 1 > tot - a.S)) {
#pragma unroll
          for (int h = 0; h < kSub; ++h)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int key = p0 + 16 * h + ((i < 2) ? kA : kB);
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
                s[h][nt][i] = keep ? s[h][nt][i] + add : kNegInf;
              }
        }

        // ---- online softmax (base 2), one max-reduction for both sub-tiles ---------------
        float vsA[kSub][G], vbA[kSub][G], vsB[kSub][G], vbB[kSub][G];
#pragma unroll
        for (int h = 0; h < kSub; ++h) {
          lds_scales<T, G>(vsA[h], st + GG::OFF_VS + (t0 + 16 * h + kA) * G * 2);
          lds_scales<T, G>(vsB[h], st + GG::OFF_VS + (t0 + 16 * h + kB) * G * 2);
          lds_scales<T, G>(vbA[h], st + GG::OFF_VB + (t0 + 16 * h + kA) * G * 2);
          lds_scales<T, G>(vbB[h], st + GG::OFF_VB + (t0 + 16 * h + kB) * G * 2);
          if (tail) {
            // keys past the valid range carry weight 0; their scales may be anything
            // (padded tail), so zero them to keep 0 * V finite
            if (p0 + 16 * h + kA >= p_end) {
#pragma unroll
              for (int g = 0; g < G; ++g) vsA[h][g] = vbA[h][g] = 0.f;
            }
            if (p0 + 16 * h + kB >= p_end) {
#pragma unroll
              for (int g = 0; g < G; ++g) vsB[h][g] = vbB[h][g] = 0.f;
            }
          }
        }
        {
          float vabs = 0.f;
#pragma unroll
          for (int h = 0; h < kSub; ++h)
#pragma unroll
            for (int g = 0; g < G; ++g) vabs = fmaxf(vabs, fmaxf(fabsf(vsA[h][g]), fabsf(vsB[h][g])));
          if (__any_sync(0xffffffffu, vabs * vmul > 2048.f)) {
#pragma unroll
            for (int off = 1; off < 32; off <<= 1)
              vabs = fmaxf(vabs, __shfl_xor_sync(0xffffffffu, vabs, off));
            const int vsh = 127 - (int)(__float_as_uint(vmul) >> 23);
            const int e = (int)((__float_as_uint(vabs) >> 23) & 0xffu) - 127;  // floor(log2)
            const int ns = min(max(vsh, e - 10), 126);  // vabs * 2^-ns < 2^11
            if (ns > vsh) {
              const float r = __uint_as_float((uint32_t)(127 - (ns - vsh)) << 23);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < G * KS; ++j) {
                  o[nt][j][0] *= r;
                  o[nt][j][1] *= r;
                  o[nt][j][2] *= r;
                  o[nt][j][3] *= r;
                }
              vmul = __uint_as_float((uint32_t)(127 - ns) << 23);
            }
          }
          if (vmul != 1.f) {
#pragma unroll
            for (int h = 0; h < kSub; ++h)
#pragma unroll
              for (int g = 0; g < G; ++g) {
                vsA[h][g] *= vmul;
                vsB[h][g] *= vmul;
              }
          }
        }
        uint32_t pf[kSub][NT][G][2];
        bool rescale = false;
        float fac[NT][2];
        // Lazy running max: the cross-lane reduction (and the rescale) only runs when some
        // lane's score exceeds the running max by more than 2^kLazyLog2; otherwise the stale
        // max stands and p stays <= 2^kLazyLog2 (P*scale remains well inside f16).
        float mloc[NT][2];
        bool need = false;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float mt = fmaxf(s[0][nt][c], s[0][nt][2 + c]);
#pragma unroll
            for (int h = 1; h < kSub; ++h) mt = fmaxf(mt, fmaxf(s[h][nt][c], s[h][nt][2 + c]));
            mloc[nt][c] = mt;
            need |= mt > m_run[nt][c] + kLazyLog2;
          }
        const bool full = __any_sync(0xffffffffu, need);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float p[kSub][4];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float m_new = m_run[nt][c];
            if (full) {
              float mt = mloc[nt][c];
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
              mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
              m_new = fmaxf(m_new, mt);
            }
            const float m_use = m_new == kNegInf ? 0.f : m_new;
            fac[nt][c] = full ? ex2(m_run[nt][c] - m_use) : 1.f;
            rescale |= m_new != m_run[nt][c];
            float lsum = 0.f;
            float ob[G];
#pragma unroll
            for (int g = 0; g < G; ++g) ob[g] = obias[nt][c][g] * fac[nt][c];
#pragma unroll
            for (int h = 0; h < kSub; ++h) {
              p[h][c] = ex2(s[h][nt][c] - m_use);
              p[h][2 + c] = ex2(s[h][nt][2 + c] - m_use);
              lsum += p[h][c] + p[h][2 + c];
#pragma unroll
              for (int g = 0; g < G; ++g) ob[g] = fmaf(p[h][c], vbA[h][g], fmaf(p[h][2 + c], vbB[h][g], ob[g]));
            }
#pragma unroll
            for (int g = 0; g < G; ++g) obias[nt][c][g] = ob[g];
            l_run[nt][c] = fmaf(l_run[nt][c], fac[nt][c], lsum);
            m_run[nt][c] = m_new;
          }
#pragma unroll
          for (int h = 0; h < kSub; ++h)
#pragma unroll
            for (int g = 0; g < G; ++g) {
              pf[h][nt][g][0] = movmatrix_trans(pack_f16x2(p[h][0] * vsA[h][g], p[h][1] * vsA[h][g]));
              pf[h][nt][g][1] = movmatrix_trans(pack_f16x2(p[h][2] * vsB[h][g], p[h][3] * vsB[h][g]));
            }
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < G * KS; ++j) {
              o[nt][j][0] *= fac[nt][0];
              o[nt][j][1] *= fac[nt][1];
              o[nt][j][2] *= fac[nt][0];
              o[nt][j][3] *= fac[nt][1];
            }
        }

        // ---- out^T += codes(V)^T . (P*scale)^T per scale group, both sub-tiles -----------
#pragma unroll
        for (int h = 0; h < kSub; ++h) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            uint32_t w0[GG::VW], w1[GG::VW], w2[GG::VW], w3[GG::VW];
            const int vb0 = g * GG::GB + gq * GG::VLB;
            const int tr = t0 + 16 * h;
            lds_words<GG::VW>(w0, st + GG::OFF_VC + code_off<BITS, D, kTP, CF::RING>(tr + v0k, vb0));
            lds_words<GG::VW>(w1, st + GG::OFF_VC + code_off<BITS, D, kTP, CF::RING>(tr + v1k, vb0));
            lds_words<GG::VW>(w2, st + GG::OFF_VC + code_off<BITS, D, kTP, CF::RING>(tr + v2k, vb0));
            lds_words<GG::VW>(w3, st + GG::OFF_VC + code_off<BITS, D, kTP, CF::RING>(tr + v3k, vb0));
            if constexpr (BITS == 4) {
              const uint32_t xa = prmt(w0[0], w1[0], 0x5410), ya = prmt(w0[0], w1[0], 0x7632);
              const uint32_t xb = prmt(w2[0], w3[0], 0x5410), yb = prmt(w2[0], w3[0], 0x7632);
              const uint32_t srcA[4] = {xa, xa >> 8, ya, ya >> 8};
              const uint32_t srcB[4] = {xb, xb >> 8, yb, yb >> 8};
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) {
                uint32_t af[4];
                af[0] = srcA[jj] & 0x000F000Fu;
                af[1] = srcA[jj] & 0x00F000F0u;
                af[2] = srcB[jj] & 0x000F000Fu;
                af[3] = srcB[jj] & 0x00F000F0u;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(o[nt][g * KS + jj], af, pf[h][nt][g][0], pf[h][nt][g][1]);
              }
            } else {
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const uint32_t xa = prmt(w0[u], w1[u], 0x5140), ya = prmt(w0[u], w1[u], 0x7362);
                const uint32_t xb = prmt(w2[u], w3[u], 0x5140), yb = prmt(w2[u], w3[u], 0x7362);
                uint32_t af[4];
                af[0] = prmt(xa, 0u, 0x4140);
                af[1] = prmt(xa, 0u, 0x4342);
                af[2] = prmt(xb, 0u, 0x4140);
                af[3] = prmt(xb, 0u, 0x4342);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(o[nt][g * KS + 2 * u], af, pf[h][nt][g][0], pf[h][nt][g][1]);
                af[0] = prmt(ya, 0u, 0x4140);
                af[1] = prmt(ya, 0u, 0x4342);
                af[2] = prmt(yb, 0u, 0x4140);
                af[3] = prmt(yb, 0u, 0x4342);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                  mma16816(o[nt][g * KS + 2 * u + 1], af, pf[h][nt][g][0], pf[h][nt][g][1]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[slot]);
    }

    // ---- per-warp finalisation: reduce l and the bias sums over the key lanes -----------
    float l_fin[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float l = l_run[nt][c];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_fin[nt][c] = l;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float v = obias[nt][c][g];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          obias[nt][c][g] = v;
        }
      }
    named_bar_sync(1, kWarps * 32);  // every consumer is done with the stage ring
    if (gq == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) mw[warp * RG + nt * 8 + 2 * tq + c] = m_run[nt][c];
    }
    named_bar_sync(1, kWarps * 32);
    // rescale this warp's rows to the CTA-wide max, then publish the rows in MMA fragment
    // order (one 16-byte store per lane per m-tile: conflict-free)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float f[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int r = nt * 8 + 2 * tq + c;
        float mx = mw[r];
#pragma unroll
        for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, mw[w * RG + r]);
        f[c] = ex2(m_run[nt][c] - (mx == kNegInf ? 0.f : mx));
        if (gq == 0) lw[warp * RG + r] = l_fin[nt][c] * f[c];
      }
      // out = f * (2^vsh * 2^24 * o + obias) (2^20 for the x16 rows), one FMA per value
      const float vpow = __uint_as_float((uint32_t)(254u - (__float_as_uint(vmul) >> 23)) << 23);  // 2^vsh
      const float shi = BITS == 4 ? 1048576.0f : 16777216.0f;
      const float ka0 = 16777216.0f * vpow * f[0], ka1 = 16777216.0f * vpow * f[1];
      const float kb0 = shi * vpow * f[0], kb1 = shi * vpow * f[1];
      float ob0[G], ob1[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        ob0[g] = obias[nt][0][g] * f[0];
        ob1[g] = obias[nt][1][g] * f[1];
      }
#pragma unroll
      for (int j = 0; j < G * KS; ++j) {
        const int g = j / KS;
        float4 v;
        v.x = fmaf(o[nt][j][0], ka0, ob0[g]);
        v.y = fmaf(o[nt][j][1], ka1, ob1[g]);
        v.z = fmaf(o[nt][j][2], kb0, ob0[g]);
        v.w = fmaf(o[nt][j][3], kb1, ob1[g]);
        reinterpret_cast<float4*>(ow + warp * RG * D)[(nt * G * KS + j) * 32 + lane] = v;
      }
    }
    named_bar_sync(1, kWarps * 32);
    // CTA sum of the warps' rows, stored straight into this CTA's partial rows. Fragment
    // float4 k holds head dims (d0, d0 + 1) of query rows r0 (x, z) and r0 + 1 (y, w).
    float* gp = P.gpart + ((size_t)(pset + split) * prows + prow0 + rbase) * PW;
    for (int k = threadIdx.x; k < RG * D / 4; k += kWarps * 32) {
      float4 acc4 = reinterpret_cast<const float4*>(ow)[k];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) {
        const float4 x = reinterpret_cast<const float4*>(ow + w * RG * D)[k];
        acc4.x += x.x;
        acc4.y += x.y;
        acc4.z += x.z;
        acc4.w += x.w;
      }
      const int ln = k & 31, t = k >> 5, j = t % (G * KS), nt = t / (G * KS);
      const int r0 = nt * 8 + 2 * (ln & 3);
      const int d0 = 64 * (j / KS) + 8 * (ln >> 2) + 2 * (j % KS);
      if (r0 < rows_here) store_part(gp + (size_t)r0 * PW + d0, acc4.x, acc4.z, P.merge);
      if (r0 + 1 < rows_here) store_part(gp + (size_t)(r0 + 1) * PW + d0, acc4.y, acc4.w, P.merge);
    }
    if (threadIdx.x < rows_here) {
      const int r = threadIdx.x;
      float mx = mw[r], l = lw[r];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) {
        mx = fmaxf(mx, mw[w * RG + r]);
        l += lw[w * RG + r];
      }
      if (P.merge) {
#pragma unroll
        for (int s = 0; s < kSlices; ++s) store_part(gp + (size_t)r * PW + D + 2 * s, mx, l, 1);
      } else {
        store_part(gp + (size_t)r * PW + D, mx, l, 0);
      }
    }
  }
  // ---- the row group's last `nm` splits merge the partials, one (row, 32-dim slice) unit
  // each. Every other CTA is done once its stores are issued. A merger polls the words it
  // needs until none reads as "not written" (0), then zeroes them for the next call. Those
  // splits are dispatched after the rest of their row group, so nothing they wait for
  // still needs a slot.
  if (!P.merge) return;
  const int units = kSlices * rows_here;
  const int nm = min(nsplit, units);
  const int first = nsplit - nm;
  if (split < first) return;
  const int nwait = nsplit + P.phantom;  // partial sets to merge (phantom: a test hook)
  // the merge scratch reuses the stage ring: no thread (the producer warp's lanes included,
  // which may have nothing to poll) writes it before every consumer is done with the ring
  __syncthreads();
  const int q4 = threadIdx.x % kMergeCols, slot = threadIdx.x / kMergeCols;  // columns x slots
  static_assert(kThreads % kMergeCols == 0 && D % (4 * kMergeCols) == 0, "merge layout");
  static_assert(kMergeCols == 8 && 32 % kMergeCols == 0, "a slot's threads share one warp");
  for (int u = split - first; u < units; u += nm) {
    const int r = u / kSlices, sl = u - r * kSlices;
    const size_t rowi = row0 + rbase + r;   // output row
    const size_t prowi = prow0 + rbase + r;  // row within a partial set
    float mt = kNegInf, lt = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    {
      // this thread's partials: p = slot, slot + kMergeSlots, ... in batches of 8 (online).
      // Every thread runs every batch (a slot past the last split just has nothing to
      // load), so the warp votes in the poll below always see all 32 lanes.
      for (int b0 = 0; b0 < nwait; b0 += 8 * kMergeSlots) {
        const int p0 = b0 + slot;
        float pm[8], pl[8];
        float4 po[8];
        unsigned need = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          pm[k] = kNegInf;
          pl[k] = 0.f;
          po[k] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (p0 + k * kMergeSlots < nwait) need |= 1u << k;
        }
        const unsigned want = need;
        unsigned long long t0 = 0;
        for (;;) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (need & (1u << k)) {
              const float* src =
                  P.gpart + ((size_t)(pset + p0 + k * kMergeSlots) * prows + prowi) * PW;
              const uint2 ml = __ldcg(reinterpret_cast<const uint2*>(src + D + 2 * sl));
              const uint4 o4 = __ldcg(reinterpret_cast<const uint4*>(src + sl * 4 * kMergeCols) + q4);
              if (ml.x && ml.y && o4.x && o4.y && o4.z && o4.w) {
                need &= ~(1u << k);
                pm[k] = __uint_as_float(ml.x ^ kPartKey);
                pl[k] = __uint_as_float(ml.y ^ kPartKey);
                po[k] = make_float4(__uint_as_float(o4.x ^ kPartKey), __uint_as_float(o4.y ^ kPartKey),
                                    __uint_as_float(o4.z ^ kPartKey), __uint_as_float(o4.w ^ kPartKey));
              }
            }
          }
          if (!__any_sync(0xffffffffu, need)) break;
          const unsigned long long now = global_ns();
          if (t0 == 0) t0 = now;
          if (__any_sync(0xffffffffu, now - t0 > P.spin_ns)) {  // (one verdict per warp)
            flag_device_error(a.status, 14);
            break;
          }
          __nanosleep(32);
        }
        // every lane of the slot holds its words: hand them back as "not written"
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (want & (1u << k)) {
            float* src = P.gpart + ((size_t)(pset + p0 + k * kMergeSlots) * prows + prowi) * PW;
            __stcg(reinterpret_cast<uint4*>(src + sl * 4 * kMergeCols) + q4, make_uint4(0u, 0u, 0u, 0u));
            if (q4 == 0) __stcg(reinterpret_cast<uint2*>(src + D + 2 * sl), make_uint2(0u, 0u));
          }
        }
        float mx = mt;
#pragma unroll
        for (int k = 0; k < 8; ++k) mx = fmaxf(mx, pm[k]);
        const float mu = mx == kNegInf ? 0.f : mx;
        const float fr = ex2(mt - mu);
        lt *= fr;
        acc.x *= fr; acc.y *= fr; acc.z *= fr; acc.w *= fr;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float f = ex2(pm[k] - mu);
          lt = fmaf(f, pl[k], lt);
          acc.x = fmaf(f, po[k].x, acc.x);
          acc.y = fmaf(f, po[k].y, acc.y);
          acc.z = fmaf(f, po[k].z, acc.z);
          acc.w = fmaf(f, po[k].w, acc.w);
        }
        mt = mx;
      }
      // the warp's four slots of each column fold through shuffles (lanes 8 and 16 apart)
#pragma unroll
      for (int sh = 8; sh <= 16; sh *= 2) {
        const float m2 = __shfl_xor_sync(0xffffffffu, mt, sh);
        const float l2 = __shfl_xor_sync(0xffffffffu, lt, sh);
        float4 a2;
        a2.x = __shfl_xor_sync(0xffffffffu, acc.x, sh);
        a2.y = __shfl_xor_sync(0xffffffffu, acc.y, sh);
        a2.z = __shfl_xor_sync(0xffffffffu, acc.z, sh);
        a2.w = __shfl_xor_sync(0xffffffffu, acc.w, sh);
        const float mx = fmaxf(mt, m2);
        const float mu = mx == kNegInf ? 0.f : mx;
        const float f1 = ex2(mt - mu), f2 = ex2(m2 - mu);
        lt = fmaf(f1, lt, f2 * l2);
        acc.x = fmaf(f1, acc.x, f2 * a2.x);
        acc.y = fmaf(f1, acc.y, f2 * a2.y);
        acc.z = fmaf(f1, acc.z, f2 * a2.z);
        acc.w = fmaf(f1, acc.w, f2 * a2.w);
        mt = mx;
      }
      if ((threadIdx.x & 31) < kMergeCols) {
        const int w = threadIdx.x >> 5;
        xm[w * kMergeCols + q4] = mt;
        xl[w * kMergeCols + q4] = lt;
        reinterpret_cast<float4*>(xo)[w * kMergeCols + q4] = acc;
      }
    }
    __syncthreads();
    if (slot == 0) {
      constexpr int kWarpsAll = kThreads / 32;
      float mx = kNegInf;
#pragma unroll
      for (int k = 0; k < kWarpsAll; ++k) mx = fmaxf(mx, xm[k * kMergeCols + q4]);
      const float mu = mx == kNegInf ? 0.f : mx;
      float l = 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < kWarpsAll; ++k) {
        const float f = ex2(xm[k * kMergeCols + q4] - mu);
        const float4 v = reinterpret_cast<const float4*>(xo)[k * kMergeCols + q4];
        l = fmaf(f, xl[k * kMergeCols + q4], l);
        o.x = fmaf(f, v.x, o.x);
        o.y = fmaf(f, v.y, o.y);
        o.z = fmaf(f, v.z, o.z);
        o.w = fmaf(f, v.w, o.w);
      }
      const int d0 = sl * 4 * kMergeCols + 4 * q4;
      if (a.out_kind == QKV_OUT_PARTIAL) {
        float* dst = reinterpret_cast<float*>(a.out) + rowi * (D + 4);
        *reinterpret_cast<float4*>(dst + d0) = o;
        if (sl == 0 && q4 == 0) *reinterpret_cast<float4*>(dst + D) = make_float4(mx, l, 0.f, 0.f);
      } else {
        const float inv = l == 0.f ? 1.f : 1.f / l;
        T* dst = reinterpret_cast<T*>(a.out) + rowi * D + d0;
        dst[0] = Elem<T>::from_f32(o.x * inv);
        dst[1] = Elem<T>::from_f32(o.y * inv);
        dst[2] = Elem<T>::from_f32(o.z * inv);
        dst[3] = Elem<T>::from_f32(o.w * inv);
      }
    }
    __syncthreads();
  }

}

// One CTA (8 warps) per output row. Warp w owns partials w, w+8, ... (up to kCombineBatch
// per warp per pass): their (max, sum) and this lane's D/32 columns load in one round of
// independent requests, then the CTA agrees on the max through shared memory and folds.
// Rows with more than 8 * kCombineBatch partials take several passes merged online.
constexpr int kCombineWarps = 8;
constexpr int kCombineBatch = 10;  // 80 partials per pass: a verify block's key splits in one

// E consecutive floats at p (16-byte aligned when VEC): vector loads keep the LSU queue short
template <int E, bool VEC>
__device__ __forceinline__ void load_cols(const float* p, float* o) {
  if constexpr (VEC && E % 4 == 0) {
#pragma unroll
    for (int i = 0; i < E / 4; ++i) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(p) + i);
      o[4 * i] = v.x;
      o[4 * i + 1] = v.y;
      o[4 * i + 2] = v.z;
      o[4 * i + 3] = v.w;
    }
  } else if constexpr (VEC && E == 2) {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(p));
    o[0] = v.x;
    o[1] = v.y;
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = __ldcg(p + e);
  }
}

template <int E, bool VEC>
__device__ __forceinline__ void zero_cols(float* p) {
  if constexpr (VEC && E % 4 == 0) {
#pragma unroll
    for (int i = 0; i < E / 4; ++i) reinterpret_cast<float4*>(p)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  } else if constexpr (VEC && E == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(0.f, 0.f);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) p[e] = 0.f;
  }
}

template <typename TO, int D, bool VEC>
__global__ void __launch_bounds__(kCombineWarps * 32)
    combine_kernel(const float* parts, int n_parts, long long part_stride_rows, long long rows,
                   TO* __restrict__ out, float* __restrict__ out_part, float* clear) {
  constexpr int E = D / 32;
  __shared__ float red[kCombineWarps][D];
  __shared__ float wmax[kCombineWarps], wsum[kCombineWarps];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the partials come from the kernel before
  const long long row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = parts + row * (D + 4);
  const size_t pstride = (size_t)part_stride_rows * (D + 4);

  float run_m = kNegInf, run_l = 0.f;  // CTA-wide running state (identical in all threads)
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int p0 = 0; p0 < n_parts; p0 += kCombineWarps * kCombineBatch) {
    float pm[kCombineBatch], pl[kCombineBatch], po[kCombineBatch][E];
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
      const int p = p0 + warp + k * kCombineWarps;
      if (p < n_parts) {
        const float* pr = base + p * pstride;
        if constexpr (VEC) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(pr + D));
          pm[k] = ml.x;
          pl[k] = ml.y;
        } else {
          pm[k] = __ldcg(pr + D);
          pl[k] = __ldcg(pr + D + 1);
        }
        load_cols<E, VEC>(pr + lane * E, po[k]);
      } else {
        pm[k] = kNegInf;
        pl[k] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) po[k][e] = 0.f;
      }
    }
    if (clear) {  // partials in an attention workspace: leave the words read as zero
      __syncwarp();
#pragma unroll
      for (int k = 0; k < kCombineBatch; ++k) {
        const int p = p0 + warp + k * kCombineWarps;
        if (p < n_parts) {
          float* pr = clear + row * (D + 4) + p * pstride;
          zero_cols<E, VEC>(pr + lane * E);
          if (lane == 0) *reinterpret_cast<float2*>(pr + D) = make_float2(0.f, 0.f);
        }
      }
    }
    float mx = pm[0];
#pragma unroll
    for (int k = 1; k < kCombineBatch; ++k) mx = fmaxf(mx, pm[k]);
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    float bm = run_m;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) bm = fmaxf(bm, wmax[w]);
    const float mu = bm == kNegInf ? 0.f : bm;
    const float fr = ex2(run_m - mu);  // rescale what earlier passes accumulated
    float l = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] *= fr;
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
      const float f = ex2(pm[k] - mu);
      l = fmaf(f, pl[k], l);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(f, po[k][e], acc[e]);
    }
    if (lane == 0) wsum[warp] = l;
    __syncthreads();
    float tl = run_l * fr;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) tl += wsum[w];
    run_l = tl;
    run_m = bm;
    __syncthreads();  // wmax/wsum are rewritten by the next pass
  }
#pragma unroll
  for (int e = 0; e < E; ++e) red[warp][lane * E + e] = acc[e];
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) v += red[w][d];
    if (out_part) {
      out_part[row * (D + 4) + d] = v;
    } else {
      out[row * D + d] = Elem<TO>::from_f32(run_l == 0.f ? v : v / run_l);
    }
  }
  if (out_part && threadIdx.x == 0) {
    float* dst = out_part + row * (D + 4);
    dst[D] = run_m;
    dst[D + 1] = run_l;
    dst[D + 2] = 0.f;
    dst[D + 3] = 0.f;
  }
}

// ---------------------------------------------------------------------------------------
// host side: tensor maps, launch
// ---------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// K or V code tensor viewed as bytes (RB, NP, B*H); box (RBOX, 64 keys, 1), swizzled.
template <int BITS, int D>
bool make_code_map(CUtensorMap* m, const void* base, int NP, long long bhs) {
  using GG = Geo<BITS, D, kBoxRows>;
  return make_code_map_bytes(m, base, GG::RB, NP, bhs, GG::RBOX, kBoxRows);
}

// Shared memory the epilogue needs (the stage ring is reused): per-warp rows, the CTA's
// rows and the merge's per-slot running (max, sum, 4 outputs) of 16 float4 columns.
template <int D, int NT>
constexpr size_t merge_bytes() {
  constexpr int RG = 8 * NT;
  return ((size_t)kWarps * RG * 2 + (size_t)kWarps * RG * D + (size_t)kMergeSlots * kMergeCols * 6) *
         4;
}

template <typename T, int BITS, int D, int NT>
int launch_split(const AttnArgs& a, bool merge, cudaStream_t st) {
  using CF = DecodeCfg<BITS, D, NT>;
  using GG = Geo<BITS, D, CF::TP, CF::RING>;
  constexpr int RG = 8 * NT;
  const int R = (a.HQ / a.HKV) * a.S;
  const int row_groups = (R + RG - 1) / RG;
  const size_t ring = (size_t)GG::STAGES * GG::STAGE_BYTES;
  const size_t smem = std::max(ring, merge_bytes<D, NT>()) + 1024;  // + alignment slack
  DecodeParams p;
  p.a = a;
  p.merge = merge ? 1 : 0;
  p.gpart = reinterpret_cast<float*>(a.workspace);
  p.phantom = merge ? a.phantom : 0;
  p.spin_ns = a.spin_ns ? a.spin_ns : kSpinNanos;
  if (!make_code_map<BITS, D>(&p.tmk, a.kw, a.NP, (long long)a.B * a.HKV) ||
      !make_code_map<BITS, D>(&p.tmv, a.vw, a.NP, (long long)a.B * a.HKV))
    return QKV_ECUDA;
  auto kern = decode_kernel<T, BITS, D, NT>;
  static unsigned attr_done = 0;  // one bit per device, per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done & (1u << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return QKV_ECUDA;
    attr_done |= 1u << (dev & 31);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.HKV * row_groups, a.balanced ? 1 : a.B);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? QKV_OK : QKV_ECUDA;
}

template <typename T, int BITS, int NT>
int launch_split_d(const AttnArgs& a, bool merge, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_split<T, BITS, 64, NT>(a, merge, st);
    case 128: return launch_split<T, BITS, 128, NT>(a, merge, st);
    case 256:
      if constexpr (NT == 1) return launch_split<T, BITS, 256, NT>(a, merge, st);
      return QKV_EUNSUPPORTED;
    default: return QKV_EUNSUPPORTED;
  }
}

template <typename T, int NT>
int launch_split_b(const AttnArgs& a, bool merge, cudaStream_t st) {
  return a.bits == 4 ? launch_split_d<T, 4, NT>(a, merge, st) : launch_split_d<T, 8, NT>(a, merge, st);
}

int launch_split_any(const AttnArgs& a, bool merge, cudaStream_t st) {
  const bool nt1 = decode_rows_per_group((a.HQ / a.HKV) * a.S, a.D) == 8;
  if (a.dtype == QKV_BF16)
    return nt1 ? launch_split_b<__nv_bfloat16, 1>(a, merge, st) : launch_split_b<__nv_bfloat16, 2>(a, merge, st);
  return nt1 ? launch_split_b<__half, 1>(a, merge, st) : launch_split_b<__half, 2>(a, merge, st);
}

}  // namespace

// 16-row groups (two MMA n-tiles) only where the accumulators fit in registers.
int decode_rows_per_group(int R, int D) { return (R <= 8 || D > 128) ? 8 : 16; }

namespace {

// Co-resident CTAs of one decode instantiation on the current device (cached); 0 when the
// query is unavailable (e.g. no device).
template <int BITS, int D, int NT>
int max_ctas() {
  using CF = DecodeCfg<BITS, D, NT>;
  using GG = Geo<BITS, D, CF::TP, CF::RING>;
  static int cache[64];
  static bool init[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 0;
  }
  if (init[dev]) return cache[dev];
  const size_t ring = (size_t)GG::STAGES * GG::STAGE_BYTES;
  const size_t smem = std::max(ring, merge_bytes<D, NT>()) + 1024;
  auto kern = decode_kernel<__nv_bfloat16, BITS, D, NT>;
  int per_sm = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess)
    per_sm = 0;
  cudaGetLastError();
  cache[dev] = per_sm * num_sms();
  init[dev] = true;
  return cache[dev];
}

int max_ctas_any(int bits, int D, int R) {
  const bool nt1 = decode_rows_per_group(R, D) == 8;
#define QKV_MC(BB, DD) \
  if (bits == BB && D == DD) return nt1 ? max_ctas<BB, DD, 1>() : max_ctas<BB, DD, 2>();
  QKV_MC(4, 64) QKV_MC(4, 128) QKV_MC(8, 64) QKV_MC(8, 128)
  if (D == 256) return bits == 4 ? max_ctas<4, 256, 1>() : max_ctas<8, 256, 1>();
#undef QKV_MC
  return 0;
}

int round_chunk(int n_max, int sp) {
  int ch = (std::max(n_max, 1) + sp - 1) / sp;
  return std::max(16, (ch + 15) / 16 * 16);  // whole 16-key warp tiles
}

}  // namespace

// Split plan: as many co-resident CTAs as the GPU holds in one wave (the in-kernel merge's
// last arrivals wait for the rest of their row group), at least 16 keys per split.
void decode_plan(int B, int HQ, int HKV, int S, int D, int bits, int n_max, int want,
                 int* splits, int* chunk) {
  const int R = (HQ / HKV) * S;
  const int rgs = (R + decode_rows_per_group(R, D) - 1) / decode_rows_per_group(R, D);
  const int units = std::max(1, B * HKV * rgs);
  const int max_sp = std::max(1, (std::max(n_max, 1) + 15) / 16);
  int sp;
  if (want > 0) {
    sp = want;
  } else {
    int slots = max_ctas_any(bits, D, R);
    if (slots <= 0) slots = decode_ctas_per_sm(R, D, bits) * num_sms();  // no device to ask
    sp = std::max(1, slots / units);
  }
  sp = std::min(std::min(sp, max_sp), kMaxSplits);
  *splits = sp;
  *chunk = round_chunk(n_max, sp);
}

int decode_plan_balanced(int B, int HQ, int HKV, int S, int D, int bits) {
  const int R = (HQ / HKV) * S;
  const int rgs = (R + decode_rows_per_group(R, D) - 1) / decode_rows_per_group(R, D);
  const int cols = std::max(1, HKV * rgs);
  int slots = max_ctas_any(bits, D, R);
  if (slots <= 0) slots = decode_ctas_per_sm(R, D, bits) * num_sms();
  // one wave: balanced + B CTAs per column; a batch's split count stays below kMaxSplits
  return std::max(1, std::min(slots / cols - B, kMaxSplits - 1));
}

size_t decode_balanced_bytes(int B, int HQ, int S, int D, int balanced) {
  return (size_t)(balanced + B) * HQ * S * (D + 2 * (D / 32)) * sizeof(float);
}

size_t decode_workspace_bytes(int B, int HQ, int S, int D, int splits) {
  // encoded partial rows: D values and one (max, sum) pair per 32-dim merge slice
  return (size_t)splits * B * HQ * S * (D + 2 * (D / 32)) * sizeof(float);
}

int launch_split_only(const AttnArgs& a, cudaStream_t st) { return launch_split_any(a, false, st); }

size_t decode_fallback_bytes(int B, int HQ, int S, int D, int splits) {
  return (size_t)splits * B * HQ * S * (D + 4) * sizeof(float);
}

bool decode_merges_in_kernel(const AttnArgs& a) {
  // The merging splits wait for the other CTAs of their row group, so every CTA of the
  // grid must be able to hold an SM slot at once: the split plan keeps automatic grids to
  // one wave, and balanced grids are one wave by construction. A forced split count past
  // that takes the two-launch route instead (plain partial rows, then combine_kernel).
  if (a.balanced) return true;
  const int R = (a.HQ / a.HKV) * a.S;
  const int rg = (R + decode_rows_per_group(R, a.D) - 1) / decode_rows_per_group(R, a.D);
  const long long ctas = (long long)a.splits * a.HKV * rg * a.B;
  int cap = max_ctas_any(a.bits, a.D, R);
  if (cap <= 0) cap = decode_ctas_per_sm(R, a.D, a.bits) * num_sms();
  return ctas <= cap;
}

int launch_decode(const AttnArgs& a, cudaStream_t st) {
  if (decode_merges_in_kernel(a)) return launch_split_any(a, true, st);
  int rc = launch_split_any(a, false, st);
  if (rc) return rc;
  const long long rows = (long long)a.B * a.HQ * a.S;
  // combine clears every word it reads: the workspace is left zero for the next call
  return launch_combine(reinterpret_cast<const float*>(a.workspace), a.splits, rows, rows, a.D,
                        a.out, a.dtype, a.out_kind, st, true);
}

int launch_combine(const float* parts, int n_parts, long long part_stride_rows, long long rows,
                   int D, void* out, int out_dtype, int out_kind, cudaStream_t st, bool clear) {
  if (rows == 0) return QKV_OK;
  const int warps = kCombineWarps;
  const unsigned grid = (unsigned)rows;
  float* op = out_kind == QKV_OUT_PARTIAL ? (float*)out : nullptr;
  float* cl = clear ? const_cast<float*>(parts) : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(warps * 32, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  // rows of D+4 floats keep a 16-byte aligned base aligned: vector loads then
  const bool vec = (reinterpret_cast<uintptr_t>(parts) & 15u) == 0;
#define QKV_C_LAUNCH(TO, DD, V)                                                             \
  e = cudaLaunchKernelEx(&cfg, combine_kernel<TO, DD, V>, parts, n_parts, part_stride_rows, \
                         rows, (TO*)out, op, cl);
#define QKV_C_CASE(DD)                                                                       \
  case DD:                                                                                   \
    if (out_dtype == QKV_BF16) {                                                             \
      if (vec) { QKV_C_LAUNCH(__nv_bfloat16, DD, true) }                                     \
      else { QKV_C_LAUNCH(__nv_bfloat16, DD, false) }                                        \
    } else {                                                                                 \
      if (vec) { QKV_C_LAUNCH(__half, DD, true) }                                            \
      else { QKV_C_LAUNCH(__half, DD, false) }                                               \
    }                                                                                        \
    break;
  switch (D) {
    QKV_C_CASE(64)
    QKV_C_CASE(128)
    QKV_C_CASE(256)
    default:
      return QKV_EUNSUPPORTED;
  }
#undef QKV_C_CASE
#undef QKV_C_LAUNCH
  return e == cudaSuccess ? QKV_OK : QKV_ECUDA;
}

// Byte-typed tiled tensor map over (RB, NP, bhs) codes, box (box_inner bytes, box_rows
// keys, 1), swizzled by the box's inner span (32, 64 or 128 bytes).
bool make_code_map_bytes(CUtensorMap* m, const void* base, int RB, int NP, long long bhs,
                         int box_inner, int box_rows) {
  // A decode step encodes the same few maps (K and V of each layer's cache) every call: keep
  // the last encodings per host thread, keyed by every argument.
  struct Entry {
    const void* base;
    long long bhs;
    int RB, NP, box_inner, box_rows;
    CUtensorMap map;
  };
  constexpr int kEntries = 256;
  thread_local Entry cache[kEntries];
  thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i) {
    const Entry& e = cache[i];
    if (e.base == base && e.bhs == bhs && e.RB == RB && e.NP == NP && e.box_inner == box_inner &&
        e.box_rows == box_rows) {
      *m = e.map;
      return true;
    }
  }
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)RB, (cuuint64_t)NP, (cuuint64_t)bhs};
  const cuuint64_t strides[2] = {(cuuint64_t)RB, (cuuint64_t)RB * (cuuint64_t)NP};
  const cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = box_inner == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : box_inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  if (fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  Entry& e = cache[next];
  e = Entry{base, bhs, RB, NP, box_inner, box_rows, *m};
  next = (next + 1) % kEntries;
  used = used < kEntries ? used + 1 : kEntries;
  return true;
}

}  // namespace qkv
