// qkv_attention_noalloc: qkv_attention for callers that cannot allocate device memory.
//
// Some hosts of this library cannot hand it a workspace: a C or FFI caller (Go, Java,
// Rust bindings) that has no CUDA allocator of its own, or an engine whose device memory is
// reserved up front by a fixed-budget pool, where an extra cudaMalloc would fail, break the
// pool's accounting, or stall the device while it runs. For them this entry point keeps the
// split-KV partials in a scratch array that lives in the library itself: a file-scope
// __device__ array of kNoAllocScratchBytes (4 MiB). Every GPU that loads libqkv.so holds that
// array until the process exits. Nothing here calls cudaMalloc, cudaFree or any allocating
// library routine.
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; host code never passes the
// array's name to a kernel, since in host code that name is only a stand-in, not a device
// address. Make that first call on a device before any stream capture begins.
//
// Sharing: every call on a device uses the same array. The attention kernel's merge reads a
// partial-row word as "not yet written" while it is zero and zeroes every word it reads, so
// the array starts at zero (static storage is zero-initialized) and every call returns it to
// zero. Two calls whose kernels overlap on the GPU (for example on two streams at once) race
// on the array: serialize them. A merge that gave up on a bounded wait (reported later by
// qkv_device_status as QKV_EDEVICE) can leave words behind; qkv_device_status(stream, 1)
// synchronizes the stream and zeroes the array again (a memset, not an allocation).
//
// The address looked up at set-up stays cached for the life of the process: after a
// cudaDeviceReset, restart the process before calling this entry point again.
#include <algorithm>

#include "../../include/qkv.h"
#include "qkv_internal.h"

namespace qkv {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_ptrs[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
// Returns a QKV status; *out receives the address.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_last_error(QKV_ECUDA, "qkv_attention_noalloc: cudaGetDevice failed: %s",
                          cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_last_error(QKV_EUNSUPPORTED,
                          "qkv_attention_noalloc: device ordinal %d is beyond the %d devices "
                          "this library tracks",
                          dev, kMaxDevices);
  if (!g_scratch_ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_last_error(QKV_ECUDA,
                            "qkv_attention_noalloc: cannot resolve the static scratch on "
                            "device %d: %s",
                            dev, cudaGetErrorString(e));
    }
    g_scratch_ptrs[dev] = p;
  }
  *out = g_scratch_ptrs[dev];
  return QKV_OK;
}

}  // namespace

cudaError_t noalloc_scratch_clear(cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return cudaSuccess;  // nothing of ours can be on such a device
  }
  if (!g_scratch_ptrs[dev]) return cudaSuccess;  // never used here: still zero
  return cudaMemsetAsync(g_scratch_ptrs[dev], 0, kNoAllocScratchBytes, st);
}

}  // namespace qkv

extern "C" int qkv_attention_noalloc(const void* q, const void* kw, const void* ks,
                                     const void* kb, const void* vw, const void* vs,
                                     const void* vb, void* out, int B, int HQ, int HKV, int S,
                                     int D, int NP, int n, const int* lens, const int* pos_base,
                                     const int* total_lens, int bits, int group_size, int dtype,
                                     float scale, int mask_kind, const void* mask, int mask_nk,
                                     long long mask_sb, long long mask_sh, long long mask_sq,
                                     int out_kind, int splits, void* stream) {
  using namespace qkv;
  void* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  // The plan (and so the scratch it needs) is the one qkv_attention makes for these
  // arguments; a call that needs more than the static scratch is refused by its own check.
  rc = qkv_attention(q, kw, ks, kb, vw, vs, vb, out, B, HQ, HKV, S, D, NP, n, lens, pos_base,
                     total_lens, bits, group_size, dtype, scale, mask_kind, mask, mask_nk,
                     mask_sb, mask_sh, mask_sq, out_kind, splits, ws, kNoAllocScratchBytes,
                     stream);
  if (rc == QKV_EWORKSPACE)
    return set_last_error(QKV_EWORKSPACE,
                          "qkv_attention_noalloc: this call needs %zu bytes of scratch, more "
                          "than the %zu-byte static scratch; use qkv_attention with a "
                          "caller-owned workspace",
                          last_workspace_need(), kNoAllocScratchBytes);
  return rc;
}
