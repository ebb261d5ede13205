// Cross-GPU merge of sequence shards over peer memory (NVLink): qkv_gather_combine.
//
// Each rank of a sequence-sharded decode holds one partial row (out, max, sum) per query
// row for its key range. Instead of an all_gather collective followed by a combine launch,
// one kernel per rank pushes its rows straight into every rank's receive buffer (peer
// pointers: the buffers are mapped into every process), then reads every rank's rows of
// this call from its own buffer as they land and merges them with the log-sum-exp rule of
// the reference's pass 2 (src/chad/mlx_qsdpa.py:233-258).
//
// Every pushed float travels with the call's flag in the same 64-bit word (flag << 32 |
// float bits; a naturally aligned 64-bit store lands whole), so a reader knows a value is
// this call's from the word alone: no fence, no counter, no second round trip over NVLink.
// Receive buffer of one rank (zero before the first call, see qkv_gather_buffer_size):
//   data  u64 [2][world][rows][D+4]   words of call parity 0 / 1, by source rank
//   seen  u32 [rows]                  calls this rank has merged, per row
// The flag of a call is seen + 1 (never 0, the zeroed buffer's value), so the kernel needs
// no host-side epoch and replays in a CUDA graph. Two parities suffice: a rank cannot push
// call k+2 before every rank has merged call k (its own call k+1 waits for every rank's push
// of k+1, which each rank issues only after its call k finished reading: the kernel's
// dependency wait orders it after the kernels before it on the stream).
// A wait that gives up sets the status word and the call still counts, so words that land
// late carry a flag the next calls do not accept; outputs since the give-up are not to be
// trusted, and a rank that fell a call behind needs every rank's buffer zeroed again.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>

#include "../../include/qkv.h"
#include "qkv_common.cuh"
#include "qkv_internal.h"

namespace qkv {

namespace {

constexpr int kGatherThreads = 128;
#define kNegInfG (-__int_as_float(0x7f800000))

__device__ __forceinline__ void st_words2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ uint64_t word(uint32_t flag, float v) {
  return ((uint64_t)flag << 32) | __float_as_uint(v);
}

__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float((uint32_t)w); }

struct GatherLayout {
  long long rows;
  int D;
  int world;
  __host__ __device__ size_t data_words() const { return (size_t)2 * world * rows * (D + 4); }
  __host__ __device__ uint32_t* seen(void* base) const {
    return reinterpret_cast<uint32_t*>(reinterpret_cast<uint64_t*>(base) + data_words());
  }
  __host__ __device__ size_t bytes() const {
    return data_words() * sizeof(uint64_t) + (size_t)rows * sizeof(uint32_t);
  }
};

// Reads the word pair at p until both carry `flag` or the deadline passes (then sets the
// status word and returns false; the values are then whatever was read).
__device__ __forceinline__ bool wait_words2(const uint64_t* p, uint32_t flag,
                                            unsigned long long deadline, float& a, float& b,
                                            int* status) {
  uint64_t w0, w1;
  ld_words2(p, w0, w1);
  while ((uint32_t)(w0 >> 32) != flag || (uint32_t)(w1 >> 32) != flag) {
    if (global_ns() > deadline) {
      flag_device_error(status, 60);
      a = word_value(w0);
      b = word_value(w1);
      return false;
    }
    __nanosleep(32);
    ld_words2(p, w0, w1);
  }
  a = word_value(w0);
  b = word_value(w1);
  return true;
}

// A grid that is resident in one wave (the host caps it at the occupancy limit), each CTA
// over rows blockIdx.x, blockIdx.x + gridDim.x, ...: first every row of the CTA is pushed to
// every rank, then the CTA reads and merges its rows one by one. No CTA waits before all of
// its own pushes are out, and every CTA of the grid becomes resident, so every rank's
// pushes are issued whatever order the ranks' CTAs run in.
template <typename TO, int D>
__global__ void __launch_bounds__(kGatherThreads)
    gather_combine_kernel(const float* __restrict__ parts, GatherLayout L, void* const* peers,
                          void* mine, int rank, TO* __restrict__ out, float* __restrict__ out_part,
                          int* status, unsigned long long spin_ns) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the rows come from the kernel before
  const int world = L.world;
  constexpr int Q = (D + 4) / 2;  // word pairs per row
  const size_t rstride = (size_t)L.rows * (D + 4);  // words between source ranks
  uint32_t* seen_base = L.seen(mine);
  // ---- push: this CTA's rows to every rank's buffer, slot (parity, this rank) ------------
  for (long long row = blockIdx.x; row < L.rows; row += gridDim.x) {
    const uint32_t seen = seen_base[row];  // (only this CTA of this rank touches the word)
    const uint32_t flag = seen + 1;
    const float2* src = reinterpret_cast<const float2*>(parts + row * (D + 4));
    const size_t off = ((size_t)(seen & 1) * world + rank) * rstride + row * (D + 4);
    for (int i = threadIdx.x; i < world * Q; i += kGatherThreads) {
      const int p = i / Q, e = i - p * Q;
      const float2 v = __ldcg(src + e);
      st_words2(reinterpret_cast<uint64_t*>(peers[p]) + off + 2 * e, word(flag, v.x),
                word(flag, v.y));
    }
  }
  // ---- per row: read every rank's words of this call as they land, merge -----------------
  __shared__ float s_m[kGatherThreads], s_l[kGatherThreads];
  const unsigned long long deadline = global_ns() + spin_ns;
  bool ok = true;  // after one give-up this thread waits no more
  for (long long row = blockIdx.x; row < L.rows; row += gridDim.x) {
    const uint32_t seen = seen_base[row];
    const uint32_t flag = seen + 1;
    const uint64_t* base =
        reinterpret_cast<const uint64_t*>(mine) + (size_t)(seen & 1) * world * rstride +
        row * (D + 4);
    if (threadIdx.x < world) {
      float m, l;
      const uint64_t* w = base + threadIdx.x * rstride + D;
      if (ok) {
        ok = wait_words2(w, flag, deadline, m, l, status);
      } else {
        uint64_t w0, w1;
        ld_words2(w, w0, w1);
        m = word_value(w0);
        l = word_value(w1);
      }
      s_m[threadIdx.x] = m;
      s_l[threadIdx.x] = l;
    }
    __syncthreads();
    float mx = kNegInfG;
    for (int p = 0; p < world; ++p) mx = fmaxf(mx, s_m[p]);
    const float mu = mx == kNegInfG ? 0.f : mx;
    float l = 0.f;
    for (int p = 0; p < world; ++p) l = fmaf(ex2(s_m[p] - mu), s_l[p], l);
    for (int t = threadIdx.x; t < D / 2; t += kGatherThreads) {
      float v0 = 0.f, v1 = 0.f;
      for (int p = 0; p < world; ++p) {
        float a, b;
        const uint64_t* w = base + p * rstride + 2 * t;
        if (ok) {
          ok = wait_words2(w, flag, deadline, a, b, status);
        } else {
          uint64_t w0, w1;
          ld_words2(w, w0, w1);
          a = word_value(w0);
          b = word_value(w1);
        }
        const float f = ex2(s_m[p] - mu);
        v0 = fmaf(f, a, v0);
        v1 = fmaf(f, b, v1);
      }
      if (out_part) {
        *reinterpret_cast<float2*>(out_part + row * (D + 4) + 2 * t) = make_float2(v0, v1);
      } else {
        out[row * D + 2 * t] = Elem<TO>::from_f32(l == 0.f ? v0 : v0 / l);
        out[row * D + 2 * t + 1] = Elem<TO>::from_f32(l == 0.f ? v1 : v1 / l);
      }
    }
    if (threadIdx.x == 0) {
      if (out_part)
        *reinterpret_cast<float4*>(out_part + row * (D + 4) + D) = make_float4(mx, l, 0.f, 0.f);
      seen_base[row] = flag;  // the call counts even after a give-up (see the header)
    }
    __syncthreads();  // s_m / s_l are rewritten for the next row
  }
}

// Resident CTAs of one instantiation on the current device (cached per device; threads
// that race here compute the same value).
template <typename TO, int D>
int gather_grid_cap() {
  static std::atomic<int> cap[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  int c = cap[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    int per_sm = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gather_combine_kernel<TO, D>,
                                                      kGatherThreads, 0) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 0;
    c = per_sm * sms;
    cap[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

}  // namespace

}  // namespace qkv

using namespace qkv;

extern "C" size_t qkv_gather_buffer_size(long long rows, int D, int world) {
  if (rows <= 0 || world <= 0 || (D != 64 && D != 128 && D != 256)) return 0;
  return GatherLayout{rows, D, world}.bytes();
}

extern "C" int qkv_gather_combine(const float* parts, long long rows, int D,
                                  void* const* peer_bufs, void* my_buf, int world, int rank,
                                  void* out, int out_dtype, int out_kind, void* stream) {
  if (!parts || !peer_bufs || !my_buf || !out)
    return set_last_error(QKV_EINVAL, "qkv_gather_combine: null pointer");
  if (rows <= 0 || world <= 0 || world > kGatherThreads || rank < 0 || rank >= world)
    return set_last_error(QKV_EINVAL, "qkv_gather_combine: bad sizes (rows %lld, world %d, rank %d)",
                          rows, world, rank);
  if (D != 64 && D != 128 && D != 256)
    return set_last_error(QKV_EUNSUPPORTED, "qkv_gather_combine: head_dim %d", D);
  if (out_dtype != QKV_BF16 && out_dtype != QKV_F16)
    return set_last_error(QKV_EINVAL, "qkv_gather_combine: bad dtype %d", out_dtype);
  if (out_kind != QKV_OUT_NORMALIZED && out_kind != QKV_OUT_PARTIAL)
    return set_last_error(QKV_EINVAL, "qkv_gather_combine: bad out_kind %d", out_kind);
  if ((reinterpret_cast<uintptr_t>(parts) | reinterpret_cast<uintptr_t>(my_buf)) & 15u)
    return set_last_error(QKV_EALIGN, "qkv_gather_combine: pointers must be 16-byte aligned");
  int* status = device_status_word();
  const TestHooks h = test_hooks();
  const unsigned long long spin = h.spin_ns ? (unsigned long long)h.spin_ns : kSpinNanos;
  const GatherLayout L{rows, D, world};
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGatherThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  float* op = out_kind == QKV_OUT_PARTIAL ? static_cast<float*>(out) : nullptr;
  cudaError_t e = cudaSuccess;
  int cap = 0;
#define QKV_G_LAUNCH(TO, DD)                                                               \
  cap = gather_grid_cap<TO, DD>();                                                         \
  if (cap <= 0) return set_last_error(QKV_ECUDA, "qkv_gather_combine: occupancy query failed"); \
  cfg.gridDim = dim3((unsigned)std::min<long long>(rows, cap), 1, 1);                      \
  e = cudaLaunchKernelEx(&cfg, gather_combine_kernel<TO, DD>, parts, L, peer_bufs, my_buf, \
                         rank, (TO*)out, op, status, spin);
#define QKV_G_CASE(DD)                    \
  case DD:                                \
    if (out_dtype == QKV_BF16) {          \
      QKV_G_LAUNCH(__nv_bfloat16, DD)     \
    } else {                              \
      QKV_G_LAUNCH(__half, DD)            \
    }                                     \
    break;
  switch (D) {
    QKV_G_CASE(64)
    QKV_G_CASE(128)
    QKV_G_CASE(256)
  }
#undef QKV_G_CASE
#undef QKV_G_LAUNCH
  if (e != cudaSuccess)
    return set_last_error(QKV_ECUDA, "qkv_gather_combine: %s", cudaGetErrorString(e));
  return QKV_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == QKV_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int qkv_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || bytes == 0) return set_last_error(QKV_EINVAL, "qkv_peer_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zero before any stream touches it
  if (e == cudaSuccess && ipc_handle)
    e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return set_last_error(QKV_ECUDA, "qkv_peer_alloc: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return QKV_OK;
}

extern "C" int qkv_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return set_last_error(QKV_EINVAL, "qkv_peer_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return set_last_error(QKV_ECUDA, "qkv_peer_open: %s", cudaGetErrorString(e));
  return QKV_OK;
}

extern "C" int qkv_peer_free(void* ptr, int opened) {
  if (!ptr) return QKV_OK;
  const cudaError_t e = opened ? cudaIpcCloseMemHandle(ptr) : cudaFree(ptr);
  if (e != cudaSuccess)
    return set_last_error(QKV_ECUDA, "qkv_peer_free: %s", cudaGetErrorString(e));
  return QKV_OK;
}
