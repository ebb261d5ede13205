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
// on the array: serialize them.
#include <algorithm>

#include "../../include/qkv.h"
#include "qkv_internal.h"

namespace qkv {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device (looked up once per device).
void* noalloc_scratch(int* err) {
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *err = (int)e;
    return nullptr;
  }
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *err = (int)e;
      cudaGetLastError();
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace

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
  // Scratch the call needs, computed the way qkv_attention sizes its split; argument errors
  // are left to qkv_attention's own validation.
  if (B > 0 && HQ > 0 && HKV > 0 && S > 0 && HQ % HKV == 0 && n >= 0 && splits >= 0 &&
      (D == 64 || D == 128 || D == 256)) {
    const int n_max = std::max(lens ? std::min(n, std::max(NP, 0)) : n, 1);
    size_t need;
    if (splits == 0) {
      need = qkv_workspace_size(B, HQ, HKV, S, D, n_max, bits, group_size);
    } else {
      int sp = 1, ch = 16, cl = 1;
      decode_plan(B, HQ, HKV, S, D, bits, n_max, splits, &sp, &ch, &cl);
      need = decode_workspace_bytes(B, HQ, HKV, S, D, sp, cl);
    }
    if (need > kNoAllocScratchBytes)
      return set_last_error(QKV_EWORKSPACE,
                            "qkv_attention_noalloc: this call needs %zu bytes of scratch, more "
                            "than the %zu-byte static scratch; use qkv_attention with a "
                            "caller-owned workspace",
                            need, kNoAllocScratchBytes);
  }
  int err = 0;
  void* ws = noalloc_scratch(&err);
  if (!ws)
    return set_last_error(QKV_ECUDA,
                          "qkv_attention_noalloc: cannot resolve the static scratch on this "
                          "device (cuda error %d)",
                          err);
  return qkv_attention(q, kw, ks, kb, vw, vs, vb, out, B, HQ, HKV, S, D, NP, n, lens, pos_base,
                       total_lens, bits, group_size, dtype, scale, mask_kind, mask, mask_nk,
                       mask_sb, mask_sh, mask_sq, out_kind, splits, ws, kNoAllocScratchBytes,
                       stream);
}
